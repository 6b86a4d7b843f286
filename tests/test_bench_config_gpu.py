"""Parity at the benchmark's own configuration: the 28-layer resident decode.

The graphs are built exactly as the default benchmark builds them: one
context with the library's default options, 28 layers of 12 q / 2 KV heads
at t_max 4096 (seeded device-filled caches), eight input slots each captured
in its own graph of the 28 layer calls with the device position advanced at
the end, positions 3840..4095 and the window wrapping back to 3840.  All 258
steps run; at steps 0, 1, 255 (position 4095), 256 (the wrap, position 3840
again, over rows the window already appended) and 257, the caches of layers
0, 13 and 27 are copied right before the step and that step's outputs and
appended rows are checked against the oracle on those copies.

Tolerance (the fp32 decode bar): max |gpu - oracle| / RMS(oracle) <= 1e-4;
appended V rows exact, appended K rows within 1e-5 absolute.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4
LAYERS, T_MAX, POS_LO, POS_HI, SLOTS = 28, 4096, 3840, 4096, 8
QKV_W, OUT_W = 2048, 1536
CHECK_STEPS = (0, 1, 255, 256, 257)
CHECK_LAYERS = (0, 13, 27)


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def test_resident28_graph_window_matches_oracle(pkg, orc, cuda):
    torch = cuda
    with pkg.Context(t_max=T_MAX) as ctx:
        caches = torch.empty((LAYERS, 2, 2, T_MAX, 128), device="cuda")
        ctx.fill_normal(caches, caches.numel(), 4242, pkg.seeded.K_CACHE)
        kvs = [pkg.kv_of(caches[l, 0], caches[l, 1]) for l in range(LAYERS)]
        qkv_slots = torch.empty((SLOTS, LAYERS, QKV_W), device="cuda")
        ctx.fill_normal(qkv_slots, qkv_slots.numel(), 4242, pkg.seeded.QKV)
        out = torch.empty((LAYERS, OUT_W), device="cuda")
        d_pos = torch.tensor([POS_LO], dtype=torch.int32, device="cuda")
        ctx.reserve(1, T_MAX)
        graphs = [ctx.graph_create_layers(kvs, qkv_slots[s], QKV_W, out, OUT_W, d_pos,
                                          advance=True, wrap_lo=POS_LO, wrap_hi=POS_HI)
                  for s in range(SLOTS)]
        stream = torch.cuda.current_stream()
        h_slots = qkv_slots.cpu().numpy()
        try:
            for step in range(max(CHECK_STEPS) + 1):
                pos = POS_LO + step % (POS_HI - POS_LO)
                check = step in CHECK_STEPS
                if check:
                    torch.cuda.synchronize()
                    assert int(d_pos.item()) == pos
                    before = {l: caches[l].cpu().numpy() for l in CHECK_LAYERS}
                graphs[step % SLOTS].launch(stream)
                if not check:
                    continue
                torch.cuda.synchronize()
                got = out.cpu().numpy()
                for l in CHECK_LAYERS:
                    rq = h_slots[step % SLOTS, l].copy()
                    rk, rv = before[l][0].copy(), before[l][1].copy()
                    orc.layer_attention(rq, rk, rv, pos, pos + 1)
                    assert nerr(got[l], rq[:OUT_W]) <= TOL, (step, l)
                    k_row = caches[l, 0, :, pos].cpu().numpy()
                    v_row = caches[l, 1, :, pos].cpu().numpy()
                    assert np.abs(k_row - rk[:, pos]).max() <= 1e-5, (step, l)
                    assert np.array_equal(v_row, rv[:, pos]), (step, l)
            assert ctx.device_status() == 0
        finally:
            for g in graphs:
                g.destroy()
