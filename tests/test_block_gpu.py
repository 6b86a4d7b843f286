"""The attention half of the decoder layer (gqa_attention_block): RMSNorm,
Q4_0 QKV projection + bias, RoPE + KV append, attention, Q4_0 Wo projection
into the residual state -- against the reference's own decoder-layer step
(compiled, FFN weights zero)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-4


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def _device(torch, pkg, x, wq, bq, wo, gamma):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dev = [t(wq), t(bq), t(wo), t(gamma)]
    return dev, pkg.block_weights_of(*dev)


@pytest.mark.parametrize("pos", [0, 1, 255, 2048, 4095])
def test_attention_block_matches_reference(pkg, orc, cuda, pos):
    torch = cuda
    x, wq, bq, wo, gamma, kc, vc = pkg.seeded.attention_block_inputs(40 + pos)
    rk, rv = kc.copy(), vc.copy()
    want = orc.ref_attention_block(x, wq, bq, wo, gamma, rk, rv, pos, pos + 1)
    with pkg.Context(t_max=4096) as ctx:
        keep, w = _device(torch, pkg, x, wq, bq, wo, gamma)
        k, v = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
        state = torch.from_numpy(x).cuda()
        ctx.attention_block(w, pkg.kv_of(k, v), state, pos, pos + 1)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        got = state.cpu().numpy()
        # the block's own contribution (state' - state) to the fp32 bar
        assert nerr(got - x, want - x) <= TOL
        assert nerr(k[:, pos].cpu().numpy(), rk[:, pos]) <= TOL
        assert np.array_equal(v[:, pos].cpu().numpy(), rv[:, pos]) or \
            nerr(v[:, pos].cpu().numpy(), rv[:, pos]) <= TOL
        assert np.array_equal(k[:, :pos].cpu().numpy(), kc[:, :pos])  # older rows untouched


def test_attention_block_layers_graph(pkg, orc, cuda):
    """Three layers per token, position on the device, two tokens; the same
    call captured in a CUDA graph and replayed gives the same state."""
    torch = cuda
    n_layers, pos0 = 3, 3000
    layers = [pkg.seeded.attention_block_inputs(70 + l) for l in range(n_layers)]
    x0 = layers[0][0]
    # reference: token loop over layers, caches updated in place
    ref_caches = [(L[5].copy(), L[6].copy()) for L in layers]
    state = x0.copy()
    want = []
    for step in range(2):
        for l, L in enumerate(layers):
            state = orc.ref_attention_block(state, L[1], L[2], L[3], L[4], ref_caches[l][0],
                                            ref_caches[l][1], pos0 + step, pos0 + step + 1)
        want.append(state.copy())
    with pkg.Context(t_max=4096) as ctx:
        keep, ws, kvs = [], [], []
        for L in layers:
            dev, w = _device(torch, pkg, *L[:5])
            k, v = torch.from_numpy(L[5]).cuda(), torch.from_numpy(L[6]).cuda()
            keep += dev + [k, v]
            ws.append(w)
            kvs.append(pkg.kv_of(k, v))
        d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
        st = torch.from_numpy(x0).cuda()
        ctx.attention_block_layers(ws, kvs, st, d_pos, advance=True)
        torch.cuda.synchronize()
        assert nerr(st.cpu().numpy() - x0, want[0] - x0) <= TOL
        # second token from a graph replay
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                ctx.attention_block_layers(ws, kvs, st, d_pos, advance=True)
        torch.cuda.synchronize()
        assert int(d_pos.item()) == pos0 + 1  # capture launched nothing
        g.replay()
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert int(d_pos.item()) == pos0 + 2
        assert nerr(st.cpu().numpy() - want[0], want[1] - want[0]) <= TOL
        del g


def test_attention_block_rejects_bad_weights(pkg, cuda):
    torch = cuda
    with pkg.Context(t_max=1024) as ctx:
        k = torch.zeros((2, 1024, 128), device="cuda")
        state = torch.zeros(1536, device="cuda")
        with pytest.raises(pkg.GqaError):
            ctx.attention_block(pkg.BlockWeights(0, 0, 0, 0), pkg.kv_of(k, k), state, 5, 6)
        buf = torch.zeros(4096 * 48 * 18 + 16, dtype=torch.uint8, device="cuda")
        f = torch.zeros(2048 + 4, device="cuda")
        bad = pkg.BlockWeights(buf.data_ptr() + 2, f.data_ptr(), buf.data_ptr(), f.data_ptr())
        with pytest.raises(pkg.GqaError):
            ctx.attention_block(bad, pkg.kv_of(k, k), state, 5, 6)


def _ffn_device(torch, pkg, wg, wu, wd, gf):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dev = [t(wg), t(wu), t(wd), t(gf)]
    return dev, pkg.ffn_weights_of(*dev)


def test_ffn_block_matches_reference(pkg, orc, cuda):
    """The FFN half alone: the reference layer with a zero attention half
    (W_qkv = 0, b_qkv = 0, W_o = 0 add exactly 0) is x + FFN(x)."""
    torch = cuda
    x, _, _, _, gamma_a, kc, vc = pkg.seeded.attention_block_inputs(31)
    wg, wu, wd, gf = pkg.seeded.ffn_block_inputs(31)
    zq = np.zeros(2048 * 48 * 18, np.uint8)
    zo = np.zeros(1536 * 48 * 18, np.uint8)
    want = orc.ref_decoder_layer(x, (zq, np.zeros(2048, np.float32), zo, gamma_a),
                                 (wg, wu, wd, gf), kc.copy(), vc.copy(), 10, 11)
    with pkg.Context(t_max=4096) as ctx:
        keep, w = _ffn_device(torch, pkg, wg, wu, wd, gf)
        state = torch.from_numpy(x).cuda()
        ctx.ffn_block(w, state)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(state.cpu().numpy() - x, want - x) <= TOL


def test_decoder_layers_match_reference(pkg, orc, cuda):
    """Two whole layers per token, two tokens (the second from a CUDA graph
    replay), position on the device."""
    torch = cuda
    n_layers, pos0 = 2, 1500
    attn = [pkg.seeded.attention_block_inputs(80 + l) for l in range(n_layers)]
    ffn = [pkg.seeded.ffn_block_inputs(80 + l) for l in range(n_layers)]
    x0 = attn[0][0]
    caches = [(A[5].copy(), A[6].copy()) for A in attn]
    state, want = x0.copy(), []
    for step in range(2):
        for l in range(n_layers):
            A = attn[l]
            state = orc.ref_decoder_layer(state, (A[1], A[2], A[3], A[4]), ffn[l], caches[l][0],
                                          caches[l][1], pos0 + step, pos0 + step + 1)
        want.append(state.copy())
    with pkg.Context(t_max=4096) as ctx:
        keep, aw, fw, kvs = [], [], [], []
        for l in range(n_layers):
            d1, w1 = _device(torch, pkg, *attn[l][:5])
            d2, w2 = _ffn_device(torch, pkg, *ffn[l])
            k, v = torch.from_numpy(attn[l][5]).cuda(), torch.from_numpy(attn[l][6]).cuda()
            keep += d1 + d2 + [k, v]
            aw.append(w1)
            fw.append(w2)
            kvs.append(pkg.kv_of(k, v))
        d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
        st = torch.from_numpy(x0).cuda()
        ctx.decoder_layers(aw, fw, kvs, st, d_pos, advance=True)
        torch.cuda.synchronize()
        assert nerr(st.cpu().numpy() - x0, want[0] - x0) <= TOL
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                ctx.decoder_layers(aw, fw, kvs, st, d_pos, advance=True)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(st.cpu().numpy() - want[0], want[1] - want[0]) <= TOL
        del g
