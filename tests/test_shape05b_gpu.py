"""The Qwen2.5-0.5B attention shape (head_dim 64, 14 q / 2 KV heads, 7 per
KV head; generate_stream_05b.c:19-31) on the shape-generic kernels, through
the same layer call, against the C restatement of the reference's attention
at that shape (its loops are shape-generic; at the 1.5B shape they equal the
compiled reference bit for bit)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
NQ, NKV, D, T_MAX = 14, 2, 64, 4096
TOL = 1e-4


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def _inputs(pkg, seed):
    s = pkg.seeded
    qkv = s.normal(seed, s.QKV, (NQ + 2 * NKV) * D)
    kc = s.normal(seed, s.K_CACHE, NKV * T_MAX * D).reshape(NKV, T_MAX, D)
    vc = s.normal(seed, s.V_CACHE, NKV * T_MAX * D).reshape(NKV, T_MAX, D)
    return qkv, kc, vc


@pytest.mark.parametrize("pos,seq_len", [(0, 1), (1, 2), (63, 64), (64, 65), (127, 128),
                                         (128, 129), (511, 512), (2047, 2048), (4095, 4096),
                                         (100, 50), (3000, 3001)])
def test_layer_attention_05b(pkg, orc, cuda, pos, seq_len):
    torch = cuda
    qkv, kc, vc = _inputs(pkg, 7000 + pos)
    rq, rk, rv = qkv.copy(), kc.copy(), vc.copy()
    orc.layer_attention(rq, rk, rv, pos, seq_len, n_heads_q=NQ, n_heads_kv=NKV, head_dim=D)
    with pkg.Context(n_heads_q=NQ, n_heads_kv=NKV, head_dim=D, t_max=T_MAX) as ctx:
        d_qkv, k, v = (torch.from_numpy(a.copy()).cuda() for a in (qkv, kc, vc))
        ctx.layer_attention(pkg.kv_of(k, v), d_qkv, pos, seq_len)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(d_qkv[:NQ * D].cpu().numpy(), rq[:NQ * D]) <= TOL
        assert np.allclose(k[:, pos].cpu().numpy(), rk[:, pos], rtol=0, atol=1e-5)
        assert np.array_equal(v[:, pos].cpu().numpy(), rv[:, pos])
        others = [t for t in (0, pos - 1, pos + 1, T_MAX - 1) if 0 <= t < T_MAX and t != pos]
        assert np.array_equal(k[:, others].cpu().numpy(), kc[:, others])
        # the k / v part of the input row is left as given (q is rotated in scratch)
        assert np.array_equal(d_qkv[NQ * D:].cpu().numpy(), qkv[NQ * D:])


def test_token_by_token_with_pdl_05b(pkg, orc, cuda):
    """Single layer calls one token after another on one cache with
    programmatic dependent launch on: each call's split kernel requests its
    first cache rows before its dependency wait, and must still see the row
    the previous call appended (the prompt walk of generate_stream_05b.c:
    744-753, one layer)."""
    torch = cuda
    pos0, n_tok = 190, 6   # crosses the 64-row tile and split boundary at 192
    _, kc, vc = _inputs(pkg, 7300)
    rows = [pkg.seeded.normal(7301 + t, pkg.seeded.QKV, (NQ + 2 * NKV) * D) for t in range(n_tok)]
    rk, rv = kc.copy(), vc.copy()
    want = []
    for t, row in enumerate(rows):
        r = row.copy()
        orc.layer_attention(r, rk, rv, pos0 + t, pos0 + t + 1, n_heads_q=NQ, n_heads_kv=NKV,
                            head_dim=D)
        want.append(r[:NQ * D].copy())
    with pkg.Context(n_heads_q=NQ, n_heads_kv=NKV, head_dim=D, t_max=T_MAX) as ctx:
        ctx.set_option(pkg.gqa.GQA_OPT_PDL, 1)
        k, v = torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda()
        bufs = [torch.from_numpy(r.copy()).cuda() for r in rows]
        for t in range(n_tok):  # queued back to back, no host synchronisation
            ctx.layer_attention(pkg.kv_of(k, v), bufs[t], pos0 + t, pos0 + t + 1)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        for t in range(n_tok):
            assert nerr(bufs[t][:NQ * D].cpu().numpy(), want[t]) <= TOL
        assert np.array_equal(v[:, pos0:pos0 + n_tok].cpu().numpy(), rv[:, pos0:pos0 + n_tok])


def test_decode_layers_graph_05b(pkg, orc, cuda):
    """Three layers per step, position on the device, two steps; the second
    from a graph replay; the layer inputs stay unrotated between replays."""
    torch = cuda
    n_layers, pos0 = 3, 1500
    ins = [_inputs(pkg, 7100 + l) for l in range(n_layers)]
    qkv = np.stack([x[0] for x in ins])
    ref_k = [x[1].copy() for x in ins]
    ref_v = [x[2].copy() for x in ins]
    want = []
    for step in range(2):
        outs = []
        for l in range(n_layers):
            r = qkv[l].copy()
            orc.layer_attention(r, ref_k[l], ref_v[l], pos0 + step, pos0 + step + 1,
                                n_heads_q=NQ, n_heads_kv=NKV, head_dim=D)
            outs.append(r[:NQ * D])
        want.append(np.stack(outs))
    with pkg.Context(n_heads_q=NQ, n_heads_kv=NKV, head_dim=D, t_max=T_MAX) as ctx:
        kvs, keep = [], []
        for x in ins:
            k, v = torch.from_numpy(x[1].copy()).cuda(), torch.from_numpy(x[2].copy()).cuda()
            keep += [k, v]
            kvs.append(pkg.kv_of(k, v))
        d_qkv = torch.from_numpy(qkv.copy()).cuda()
        out = torch.zeros((n_layers, NQ * D), device="cuda")
        d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
        ctx.reserve(1, T_MAX)
        ctx.decode_layers(kvs, d_qkv, qkv.shape[1], out, NQ * D, d_pos, advance=True)
        torch.cuda.synchronize()
        assert nerr(out.cpu().numpy(), want[0]) <= TOL
        g = ctx.graph_create_layers(kvs, d_qkv, qkv.shape[1], out, NQ * D, d_pos, advance=True)
        g.launch()
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(out.cpu().numpy(), want[1]) <= TOL
        assert int(d_pos.item()) == pos0 + 2
        assert np.array_equal(d_qkv.cpu().numpy(), qkv)
        g.destroy()


def test_tuned_only_entry_points_refuse_05b(pkg, cuda):
    torch = cuda
    with pkg.Context(n_heads_q=NQ, n_heads_kv=NKV, head_dim=D, t_max=256) as ctx:
        kv = ctx.kv_alloc(1)[0]
        q = torch.zeros(NQ * D, device="cuda")
        out = torch.zeros(NQ * D, device="cuda")
        with pytest.raises(pkg.GqaError, match="head_dim 128"):
            ctx.decode(kv, q, 10, out)
        with pytest.raises(pkg.GqaError, match="head_dim 128"):
            ctx.prefill_bf16(1, 128, torch.zeros(128 * (NQ + 2 * NKV) * D, device="cuda"),
                             torch.zeros(128 * NQ * D, device="cuda"))
        ctx.kv_free([kv])
    with pytest.raises(pkg.GqaError, match="not built"):
        pkg.Context(n_heads_q=16, n_heads_kv=2, head_dim=64)
