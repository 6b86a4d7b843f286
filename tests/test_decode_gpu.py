"""GPU parity of the fp32 decode path against the oracle, through the C ABI.

Tolerance (the workload's stated bar for fp32 decode): max |gpu - oracle|
divided by the RMS of the oracle output <= 1e-4.  Appended V rows are copies
and must match exactly; appended K rows go through RoPE (sincosf on the
device vs libm on the host) and must match to 1e-5 absolute.
"""
import hashlib
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "decode_golden.npz")


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


@pytest.fixture(scope="module")
def ctx4096(pkg, cuda):
    c = pkg.Context(t_max=4096)
    yield c
    c.close()


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_smoke_entry(cuda):
    import __graft_entry__
    __graft_entry__.smoke()


@pytest.mark.parametrize("i", range(17))
def test_layer_attention_matches_reference_golden(pkg, orc, cuda, ctx4096, i):
    torch = cuda
    g = np.load(GOLDEN)
    pos, seq_len = int(g["pos"][i]), int(g["seq_len"][i])
    qkv, kc, vc = pkg.seeded.decode_inputs(int(g["seed"][i]), 4096, dist=str(g["dist"][i]))
    h = hashlib.sha256()
    for a in (qkv, kc, vc):
        h.update(a.tobytes())
    assert h.hexdigest() == str(g["digest"][i])
    d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
    ctx4096.layer_attention(pkg.kv_of(d_k, d_v), d_qkv, pos, seq_len)
    torch.cuda.synchronize()
    assert ctx4096.device_status() == 0
    out = d_qkv.cpu().numpy()
    assert nerr(out[:1536], g["attn_out"][i]) <= TOL, str(g["name"][i])
    assert np.array_equal(out[1536:], qkv[1536:]), "k/v slice of qkv must be left unchanged"
    assert np.abs(d_k[:, pos].cpu().numpy() - g["k_rows"][i]).max() <= 1e-5
    assert np.array_equal(d_v[:, pos].cpu().numpy(), g["v_rows"][i])
    # rows other than pos untouched
    kk = d_k.cpu().numpy()
    kk[:, pos] = kc[:, pos]
    assert np.array_equal(kk, kc)


@pytest.mark.parametrize("t_max,pos,seq_len", [
    (512, 511, 512),            # single-step workload shape
    (33, 32, 33), (64, 0, 1), (64, 63, 64), (300, 150, 151),
    (8192, 8191, 8192), (32768, 20000, 20001), (32768, 32767, 32768),
])
def test_layer_attention_matches_oracle(pkg, orc, cuda, t_max, pos, seq_len):
    torch = cuda
    qkv, kc, vc = pkg.seeded.decode_inputs(31 + pos, t_max)
    rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
    orc.layer_attention(rq, rk, rv, pos, seq_len)
    with pkg.Context(t_max=t_max) as ctx:
        d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
        out = torch.empty(1536, device="cuda")
        ctx.layer_attention_out(pkg.kv_of(d_k, d_v), d_qkv, pos, seq_len, out)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(out.cpu().numpy(), rq[:1536]) <= TOL
        assert np.array_equal(d_qkv.cpu().numpy(), qkv), "out-of-place call must not touch qkv"
        assert np.abs(d_k[:, pos].cpu().numpy() - rk[:, pos]).max() <= 1e-5


@pytest.mark.parametrize("target", [1, 7, 148, 600])
def test_split_counts_do_not_change_results(pkg, orc, cuda, target):
    torch = cuda
    t_max, pos = 4096, 3000
    qkv, kc, vc = pkg.seeded.decode_inputs(99, t_max)
    rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
    orc.layer_attention(rq, rk, rv, pos, pos + 1)
    with pkg.Context(t_max=t_max) as ctx:
        ctx.set_option(pkg.gqa.GQA_OPT_TARGET_CTAS, target)
        d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
        ctx.layer_attention(pkg.kv_of(d_k, d_v), d_qkv, pos, pos + 1)
        torch.cuda.synchronize()
        assert nerr(d_qkv[:1536].cpu().numpy(), rq[:1536]) <= TOL


def test_rope_append_then_unfused_decode(pkg, orc, cuda, ctx4096):
    torch = cuda
    pos = 1234
    qkv, kc, vc = pkg.seeded.decode_inputs(5, 4096)
    rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
    orc.rope_kv_append(rq[:1536], rq[1536:1792], rq[1792:], rk, rv, pos)
    ref = orc.attention(rq[:1536], rk, rv, pos + 1)
    d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
    kv = pkg.kv_of(d_k, d_v)
    base = d_qkv.data_ptr()
    ctx4096.rope_kv_append(kv, base, base + 1536 * 4, base + 1792 * 4, pos)
    out = torch.empty(1536, device="cuda")
    ctx4096.decode(kv, d_qkv, pos + 1, out)
    torch.cuda.synchronize()
    assert np.abs(d_qkv[:1536].cpu().numpy() - rq[:1536]).max() <= 1e-5
    assert np.abs(d_k.cpu().numpy() - rk).max() <= 1e-5
    assert np.array_equal(d_v.cpu().numpy(), rv)
    assert nerr(out.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("t_begin,t_end", [(0, 1), (0, 4096), (17, 2500), (1000, 1033),
                                           (4000, 4096), (5, 5)])
def test_split_partial_matches_oracle(pkg, orc, cuda, ctx4096, t_begin, t_end):
    torch = cuda
    qkv, kc, vc = pkg.seeded.decode_inputs(11, 4096)
    q = qkv[:1536].copy()
    m, l, o = orc.attention_partial(q, kc, vc, t_begin, t_end)
    d_k, d_v = to_dev(torch, kc), to_dev(torch, vc)
    dm = torch.empty(12, device="cuda")
    dl = torch.empty(12, device="cuda")
    do = torch.empty(12 * 128, device="cuda")
    ctx4096.decode_split_partial(pkg.kv_of(d_k, d_v), to_dev(torch, q), t_begin, t_end, dm, dl, do)
    torch.cuda.synchronize()
    gm, gl, go = dm.cpu().numpy(), dl.cpu().numpy(), do.cpu().numpy()
    if t_end == t_begin:
        assert np.all(np.isneginf(gm)) and np.all(gl == 0) and np.all(go == 0)
        return
    # A partial (m, l, o) is defined up to a common factor: (m', l e^(m-m'), o e^(m-m'))
    # is the same partial.  The kernel's m is a running reference that trails the
    # true maximum by at most 8 log2 units (its lazy rescale threshold).
    assert np.all(gm <= m + 1e-5) and np.all(gm >= m - 8 * np.log(2) - 1e-5)
    scale = np.exp((gm - m).astype(np.float64))
    assert np.abs(gl * scale - l).max() / l.max() < 1e-4
    assert nerr((go.reshape(12, 128) / (gl[:, None])).reshape(-1),
                (o.reshape(12, 128) / l[:, None]).reshape(-1)) <= TOL


def test_lse_combine_matches_oracle(pkg, orc, cuda, ctx4096):
    torch = cuda
    qkv, kc, vc = pkg.seeded.decode_inputs(12, 4096)
    q = qkv[:1536].copy()
    cuts = [0, 700, 700, 2049, 4096]
    parts = [orc.attention_partial(q, kc, vc, a, b) for a, b in zip(cuts[:-1], cuts[1:])]
    m = np.stack([p[0] for p in parts]).astype(np.float32)
    l = np.stack([p[1] for p in parts]).astype(np.float32)
    o = np.stack([p[2] for p in parts]).astype(np.float32)
    ref = orc.lse_combine(m, l, o.reshape(len(parts), 12, 128)).reshape(-1)
    out = torch.empty(12 * 128, device="cuda")
    ctx4096.lse_combine(len(parts), 12, to_dev(torch, m), to_dev(torch, l), to_dev(torch, o), out)
    torch.cuda.synchronize()
    assert nerr(out.cpu().numpy(), ref) <= TOL
    full = orc.attention(q, kc, vc, 4096)
    assert nerr(out.cpu().numpy(), full) <= TOL


def _batched_case(pkg, torch, lens, t_max, seed):
    n = len(lens)
    qkv = np.stack([pkg.seeded.normal(seed + s, pkg.seeded.QKV, 2048) for s in range(n)])
    kc = np.stack([pkg.seeded.normal(seed + s, pkg.seeded.K_CACHE, 2 * t_max * 128)
                   .reshape(2, t_max, 128) for s in range(n)])
    vc = np.stack([pkg.seeded.normal(seed + s, pkg.seeded.V_CACHE, 2 * t_max * 128)
                   .reshape(2, t_max, 128) for s in range(n)])
    return qkv, kc, vc


@pytest.mark.parametrize("lens,t_max", [([1, 2, 33, 256, 257, 1000, 2048, 17], 2048),
                                        ([4096] * 3 + [1], 4096)])
def test_batched_matches_oracle(pkg, orc, cuda, lens, t_max):
    torch = cuda
    n = len(lens)
    qkv, kc, vc = _batched_case(pkg, torch, lens, t_max, 500)
    ref_q = [qkv[s].copy() for s in range(n)]
    ref_k = [kc[s].copy() for s in range(n)]
    ref_v = [vc[s].copy() for s in range(n)]
    ref = orc.decode_batched(ref_q, ref_k, ref_v, lens)
    with pkg.Context(t_max=t_max) as ctx:
        d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
        stride = 2 * t_max * 128 * 4
        kp = torch.tensor([d_k.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        vp = torch.tensor([d_v.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        ctx.decode_batched(n, kp, vp, d_qkv, 2048, dl, max(lens), d_qkv, 2048)  # in place
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        got = d_qkv.cpu().numpy()
        for s in range(n):
            assert nerr(got[s, :1536], ref[s]) <= TOL, f"sequence {s} (len {lens[s]})"
            assert np.array_equal(got[s, 1536:], qkv[s, 1536:])
            p = lens[s] - 1
            assert np.abs(d_k[s, :, p].cpu().numpy() - ref_k[s][:, p]).max() <= 1e-5
            assert np.array_equal(d_v[s, :, p].cpu().numpy(), ref_v[s][:, p])


@pytest.mark.parametrize("lens", [[1, 40, 300, 1500, 2000], [1, 7, 100, 200]])
def test_batched_advance_matches_oracle(pkg, orc, cuda, lens):
    """GQA_OPT_BATCH_ADVANCE with PDL on: two steps in a row, the device
    lengths advanced by the library after each (by the combine, or by its own
    small kernel when the plan has one split); each step equals the oracle's
    step at those lengths, with the rows the first step appended in place."""
    torch = cuda
    t_max = 2048
    n = len(lens)
    qkv1, kc, vc = _batched_case(pkg, torch, lens, t_max, 2100)
    qkv2 = np.stack([pkg.seeded.normal(2300 + s, pkg.seeded.QKV, 2048) for s in range(n)])
    ref_k = [kc[s].copy() for s in range(n)]
    ref_v = [vc[s].copy() for s in range(n)]
    ref1 = orc.decode_batched([qkv1[s].copy() for s in range(n)], ref_k, ref_v, lens)
    ref2 = orc.decode_batched([qkv2[s].copy() for s in range(n)], ref_k, ref_v,
                              [L + 1 for L in lens])
    with pkg.Context(t_max=t_max) as ctx:
        ctx.set_option(pkg.gqa.GQA_OPT_PDL, 1)
        ctx.set_option(pkg.gqa.GQA_OPT_BATCH_ADVANCE, 1)
        d_k, d_v = to_dev(torch, kc), to_dev(torch, vc)
        d1, d2 = to_dev(torch, qkv1), to_dev(torch, qkv2)
        stride = 2 * t_max * 128 * 4
        kp = torch.tensor([d_k.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        vp = torch.tensor([d_v.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        out1 = torch.empty((n, 1536), device="cuda")
        out2 = torch.empty((n, 1536), device="cuda")
        ctx.decode_batched(n, kp, vp, d1, 2048, dl, max(lens) + 1, out1, 1536)
        ctx.decode_batched(n, kp, vp, d2, 2048, dl, max(lens) + 1, out2, 1536)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert dl.cpu().tolist() == [L + 2 for L in lens]
        for s in range(n):
            assert nerr(out1[s].cpu().numpy(), ref1[s]) <= TOL, (s, 1)
            assert nerr(out2[s].cpu().numpy(), ref2[s]) <= TOL, (s, 2)
        got_k = d_k.cpu().numpy()
        for s in range(n):
            for p in (lens[s] - 1, lens[s]):
                assert np.abs(got_k[s, :, p] - ref_k[s][:, p]).max() <= 1e-5


def test_batched_host_buffers_match_oracle(pkg, orc, cuda):
    """gqa_decode_batched_host: page-locked host qkv in, the batched step on a
    device buffer, packed host outputs back -- the same outputs as the oracle
    (and the appended rows in the device caches), on a non-blocking stream,
    two steps in a row, output written in place over the device qkv."""
    torch = cuda
    lens, t_max = [1, 40, 300, 1500, 2048], 2048
    n = len(lens)
    qkv, kc, vc = _batched_case(pkg, torch, lens, t_max, 1700)
    ref_q = [qkv[s].copy() for s in range(n)]
    ref_k = [kc[s].copy() for s in range(n)]
    ref_v = [vc[s].copy() for s in range(n)]
    ref = orc.decode_batched(ref_q, ref_k, ref_v, lens)
    st = torch.cuda.Stream()
    with pkg.Context(t_max=t_max) as ctx:
        d_k, d_v = to_dev(torch, kc), to_dev(torch, vc)
        d_qkv = torch.empty((n, 2048), device="cuda")
        stride = 2 * t_max * 128 * 4
        kp = torch.tensor([d_k.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        vp = torch.tensor([d_v.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        h_qkv = torch.from_numpy(qkv.astype(np.float32)).pin_memory()
        h_out = torch.full((n, 1536), float("nan")).pin_memory()
        torch.cuda.synchronize()
        for _ in range(2):  # the second step appends the same row at the same position
            ctx.decode_batched_host(n, kp, vp, h_qkv, d_qkv, 2048, dl, max(lens), d_qkv, 2048,
                                    h_out, st)
        st.synchronize()
        assert ctx.device_status() == 0
        got = h_out.numpy()
        for s in range(n):
            assert nerr(got[s], ref[s]) <= TOL, f"sequence {s} (len {lens[s]})"
            p = lens[s] - 1
            assert np.abs(d_k[s, :, p].cpu().numpy() - ref_k[s][:, p]).max() <= 1e-5
            assert np.array_equal(d_v[s, :, p].cpu().numpy(), ref_v[s][:, p])
        with pytest.raises(pkg.gqa.GqaError):
            ctx.decode_batched_host(n, kp, vp, None, d_qkv, 2048, dl, max(lens), d_qkv, 2048,
                                    h_out, st)


def test_batched_full_size_workload_sampled(pkg, orc, cuda):
    """The batched workload at full size (64 sequences, lengths uniform in
    [256, 8192], fp32 caches filled on the device); 6 sequences are checked
    against the oracle after one step, the rest for finiteness."""
    torch = cuda
    n, t_max, seed = 64, 8192, 20260
    lens = [int(x) for x in pkg.seeded.uniform_int(seed, pkg.seeded.LENGTHS, n, 256, 8192)]
    with pkg.Context(t_max=t_max) as ctx:
        k = torch.empty((n, 2, t_max, 128), device="cuda")
        v = torch.empty((n, 2, t_max, 128), device="cuda")
        qkv = torch.empty((n, 2048), device="cuda")
        ctx.fill_normal(k, k.numel(), seed, pkg.seeded.K_CACHE)
        ctx.fill_normal(v, v.numel(), seed, pkg.seeded.V_CACHE)
        ctx.fill_normal(qkv, qkv.numel(), seed, pkg.seeded.QKV)
        torch.cuda.synchronize()
        check = [0, 1, 17, 31, 50, 63]
        host = {s: (qkv[s].cpu().numpy().copy(), k[s].cpu().numpy().copy(),
                    v[s].cpu().numpy().copy()) for s in check}
        stride = 2 * t_max * 128 * 4
        kp = torch.tensor([k.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        vp = torch.tensor([v.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                          device="cuda")
        dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        out = torch.empty((n, 1536), device="cuda")
        ctx.decode_batched(n, kp, vp, qkv, 2048, dl, max(lens), out, 1536)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got))
        ref = orc.decode_batched([host[s][0] for s in check], [host[s][1] for s in check],
                                 [host[s][2] for s in check], [lens[s] for s in check])
        for s, r in zip(check, ref):
            assert nerr(got[s], r) <= TOL, f"sequence {s} (len {lens[s]})"


def test_decode_layers_and_graph_replay_match_oracle(pkg, orc, cuda):
    """The per-token layer loop with pos on the device, as direct launches and
    as a replayed CUDA graph, over several autoregressive steps."""
    torch = cuda
    n_layers, t_max, pos0, steps = 3, 1024, 900, 4
    caches = [pkg.seeded.decode_inputs(700 + l, t_max) for l in range(n_layers)]
    step_qkv = [np.stack([pkg.seeded.normal(800 + 10 * s + l, pkg.seeded.QKV, 2048)
                          for l in range(n_layers)]) for s in range(steps)]
    rk = [c[1].copy() for c in caches]
    rv = [c[2].copy() for c in caches]
    ref_out = []
    for s in range(steps):
        outs = []
        for l in range(n_layers):
            q = step_qkv[s][l].copy()
            orc.layer_attention(q, rk[l], rv[l], pos0 + s, pos0 + s + 1)
            outs.append(q[:1536])
        ref_out.append(np.stack(outs))
    with pkg.Context(t_max=t_max) as ctx:
        for mode in ("direct", "graph"):
            ks = [to_dev(torch, c[1]) for c in caches]
            vs = [to_dev(torch, c[2]) for c in caches]
            kvs = [pkg.kv_of(k, v) for k, v in zip(ks, vs)]
            d_qkv = torch.empty((n_layers, 2048), device="cuda")
            d_out = torch.empty((n_layers, 1536), device="cuda")
            d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
            graph = None
            if mode == "graph":
                graph = ctx.graph_create_layers(kvs, d_qkv, 2048, d_out, 1536, d_pos, advance=True)
            for s in range(steps):
                d_qkv.copy_(torch.from_numpy(step_qkv[s]))
                if graph:
                    graph.launch()
                else:
                    ctx.decode_layers(kvs, d_qkv, 2048, d_out, 1536, d_pos, advance=True)
                torch.cuda.synchronize()
                assert nerr(d_out.cpu().numpy().reshape(-1), ref_out[s].reshape(-1)) <= TOL, \
                    (mode, s)
            assert int(d_pos.item()) == pos0 + steps
            for l in range(n_layers):
                assert np.abs(ks[l].cpu().numpy() - rk[l]).max() <= 1e-5
                assert np.array_equal(vs[l].cpu().numpy(), rv[l])
            if graph:
                graph.destroy()
        assert ctx.device_status() == 0


def test_graph_step_host_buffers(pkg, orc, cuda):
    torch = cuda
    n_layers, t_max, pos0 = 2, 512, 100
    caches = [pkg.seeded.decode_inputs(40 + l, t_max) for l in range(n_layers)]
    qkv = np.stack([pkg.seeded.normal(50 + l, pkg.seeded.QKV, 2048) for l in range(n_layers)])
    ref = []
    for l in range(n_layers):
        q = qkv[l].copy()
        orc.layer_attention(q, caches[l][1].copy(), caches[l][2].copy(), pos0, pos0 + 1)
        ref.append(q[:1536])
    with pkg.Context(t_max=t_max) as ctx:
        tensors = [(to_dev(torch, c[1]), to_dev(torch, c[2])) for c in caches]
        kvs = [pkg.kv_of(k, v) for k, v in tensors]
        d_qkv = torch.empty((n_layers, 2048), device="cuda")
        d_out = torch.empty((n_layers, 1536), device="cuda")
        d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
        g = ctx.graph_create_layers(kvs, d_qkv, 2048, d_out, 1536, d_pos, advance=False)
        h_qkv = torch.from_numpy(qkv).pin_memory()
        h_out = torch.empty((n_layers, 1536)).pin_memory()
        g.step_host(h_qkv, h_out)
        torch.cuda.synchronize()
        assert nerr(h_out.numpy().reshape(-1), np.stack(ref).reshape(-1)) <= TOL
        g.destroy()


def test_invalid_arguments_raise(pkg, cuda, ctx4096):
    torch = cuda
    k = torch.zeros((2, 4096, 128), device="cuda")
    v = torch.zeros((2, 4096, 128), device="cuda")
    qkv = torch.zeros(2048, device="cuda")
    kv = pkg.kv_of(k, v)
    for pos, L in [(-1, 1), (4096, 4097), (0, 0), (0, 4097)]:
        with pytest.raises(pkg.GqaError) as e:
            ctx4096.layer_attention(kv, qkv, pos, L)
        assert e.value.code == pkg.gqa.GQA_ERR_INVALID_ARG
    with pytest.raises(pkg.GqaError):
        ctx4096.layer_attention(kv, qkv.data_ptr() + 4, 0, 1)  # misaligned
    with pytest.raises(pkg.GqaError):
        ctx4096.layer_attention(pkg.kv_of(0, 0), qkv, 0, 1)
    assert ctx4096.device_status() == 0


def test_device_side_bad_position_sets_status(pkg, cuda):
    """A device-resident pos outside the cache is caught by the kernel, which
    skips all memory access and raises a status bit (no fault)."""
    torch = cuda
    with pkg.Context(t_max=256) as ctx:
        k = torch.zeros((2, 256, 128), device="cuda")
        v = torch.zeros((2, 256, 128), device="cuda")
        qkv = torch.zeros((1, 2048), device="cuda")
        out = torch.zeros((1, 1536), device="cuda")
        d_pos = torch.tensor([256], dtype=torch.int32, device="cuda")
        ctx.decode_layers([pkg.kv_of(k, v)], qkv, 2048, out, 1536, d_pos)
        torch.cuda.synchronize()
        st = ctx.device_status(clear=True)
        assert st & pkg.gqa.STATUS_BAD_LENGTH
        assert ctx.device_status() == 0
        assert float(k.abs().sum()) == 0.0


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4, 5, 6])
def test_every_kernel_variant_matches_oracle(pkg, orc, cuda, variant):
    """Each instantiated kernel shape gives the same results (fused single
    sequence at several lengths, unfused partials, and a ragged batch)."""
    torch = cuda
    t_max = 2048
    with pkg.Context(t_max=t_max) as ctx:
        ctx.set_option(pkg.gqa.GQA_OPT_KERNEL_VARIANT, variant)
        for pos, seq_len in [(0, 1), (37, 38), (700, 701), (2047, 2048), (900, 20)]:
            qkv, kc, vc = pkg.seeded.decode_inputs(3000 + pos + variant, t_max)
            rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
            orc.layer_attention(rq, rk, rv, pos, seq_len)
            d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
            ctx.layer_attention(pkg.kv_of(d_k, d_v), d_qkv, pos, seq_len)
            torch.cuda.synchronize()
            assert nerr(d_qkv[:1536].cpu().numpy(), rq[:1536]) <= TOL, (variant, pos, seq_len)
            assert np.abs(d_k[:, pos].cpu().numpy() - rk[:, pos]).max() <= 1e-5
        lens = [1, 64, 65, 1999, 300]
        qkv, kc, vc = _batched_case(pkg, torch, lens, t_max, 900 + variant)
        ref = orc.decode_batched([qkv[s].copy() for s in range(len(lens))],
                                 [kc[s].copy() for s in range(len(lens))],
                                 [vc[s].copy() for s in range(len(lens))], lens)
        d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
        stride = 2 * t_max * 128 * 4
        kp = torch.tensor([d_k.data_ptr() + s * stride for s in range(len(lens))],
                          dtype=torch.int64, device="cuda")
        vp = torch.tensor([d_v.data_ptr() + s * stride for s in range(len(lens))],
                          dtype=torch.int64, device="cuda")
        dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        out = torch.empty((len(lens), 1536), device="cuda")
        ctx.decode_batched(len(lens), kp, vp, d_qkv, 2048, dl, max(lens), out, 1536)
        torch.cuda.synchronize()
        for s in range(len(lens)):
            assert nerr(out[s].cpu().numpy(), ref[s]) <= TOL, (variant, s)
        assert ctx.device_status() == 0


@pytest.mark.parametrize("variant", [0, 3, 5])
@pytest.mark.parametrize("cluster", [0, 1])
def test_cluster_reduction_matches_oracle(pkg, orc, cuda, variant, cluster):
    """Single-sequence decode with and without the in-kernel cluster reduction
    (several lengths, repeated calls so the arrival counters are reused)."""
    torch = cuda
    t_max = 4096
    with pkg.Context(t_max=t_max) as ctx:
        ctx.set_option(pkg.gqa.GQA_OPT_KERNEL_VARIANT, variant)
        ctx.set_option(pkg.gqa.GQA_OPT_GRID_MERGE, 0)
        ctx.set_option(pkg.gqa.GQA_OPT_CLUSTER, cluster)
        for pos, seq_len in [(4095, 4096), (3000, 3001), (300, 301), (256, 257), (4000, 2000)]:
            for rep in range(2):
                qkv, kc, vc = pkg.seeded.decode_inputs(7000 + pos + rep, t_max)
                rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
                orc.layer_attention(rq, rk, rv, pos, seq_len)
                d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
                ctx.layer_attention(pkg.kv_of(d_k, d_v), d_qkv, pos, seq_len)
                torch.cuda.synchronize()
                assert nerr(d_qkv[:1536].cpu().numpy(), rq[:1536]) <= TOL, (pos, seq_len, rep)
                assert np.abs(d_k[:, pos].cpu().numpy() - rk[:, pos]).max() <= 1e-5
        assert ctx.device_status() == 0


@pytest.mark.parametrize("target_ctas", [0, 12, 40, 148])
def test_grid_merge_matches_oracle(pkg, orc, cuda, target_ctas):
    """Single-sequence decode merged inside the split kernel (grid barrier, one
    merge slice per CTA): lengths from below the 6-split minimum (which falls
    back to split + combine) to t_max, a row appended outside the attended
    range, and repeated calls so the barrier counter keeps counting."""
    torch = cuda
    t_max = 4096
    with pkg.Context(t_max=t_max) as ctx:
        if target_ctas:
            ctx.set_option(pkg.gqa.GQA_OPT_TARGET_CTAS, target_ctas)
        for pos, seq_len in [(4095, 4096), (3840, 3841), (1000, 1001), (47, 48), (40, 41),
                             (4000, 2000), (0, 1)]:
            for rep in range(2):
                qkv, kc, vc = pkg.seeded.decode_inputs(9100 + pos + rep, t_max)
                rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
                orc.layer_attention(rq, rk, rv, pos, seq_len)
                d_qkv, d_k, d_v = to_dev(torch, qkv), to_dev(torch, kc), to_dev(torch, vc)
                ctx.layer_attention(pkg.kv_of(d_k, d_v), d_qkv, pos, seq_len)
                torch.cuda.synchronize()
                assert nerr(d_qkv[:1536].cpu().numpy(), rq[:1536]) <= TOL, (pos, seq_len, rep)
                assert np.abs(d_k[:, pos].cpu().numpy() - rk[:, pos]).max() <= 1e-5
                assert np.array_equal(d_v[:, pos].cpu().numpy(), rv[:, pos])
        assert ctx.device_status() == 0
