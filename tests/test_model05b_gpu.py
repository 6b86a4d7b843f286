"""The Qwen2.5-0.5B token step on the GPU (generate_stream_05b.c): the Q4_0
projections at d_model 896 / d_ffn 4864 (gqa_attention_block, gqa_ffn_block,
gqa_decoder_layers on a head_dim 64, 14 / 2 context), the 28-block Q4_0
embedding, the Q8_0 LM head with the greedy pick (gqa_lm_head_q8_0), the
whole step (gqa_decode_token) and a 0.5B-shaped GGUF through the loader and
the request loop -- against the layer composed from the reference's compiled
GEMVs (pinned to its compiled layer step by the CPU tests), the shape-generic
attention restatement and the restated Q8_0 kernel."""
import numpy as np
import pytest

import gguf_writer as gw

pytestmark = pytest.mark.gpu
D, DFFN, NQ, NKV, HD = 896, 4864, 14, 2, 64
ROW8 = 952
TOL = 1e-4  # normalised by the output's RMS


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def _ctx(pkg, t_max=4096):
    return pkg.Context(n_heads_q=NQ, n_heads_kv=NKV, head_dim=HD, t_max=t_max)


def _t(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _packed(torch, ctx, pkg, w, n_rows):
    packed = torch.empty(pkg.Context.lm_head_q8_0_packed_bytes(n_rows), dtype=torch.uint8,
                         device="cuda")
    ctx.lm_head_q8_0_pack(_t(torch, w), n_rows, packed)
    return packed


def _run_head(torch, ctx, packed, n_rows, gamma, state):
    logits = torch.empty(n_rows, dtype=torch.float32, device="cuda")
    token = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    ctx.lm_head_q8_0(packed, n_rows, _t(torch, gamma.astype(np.float32)),
                     _t(torch, state.astype(np.float32)), logits, token)
    torch.cuda.synchronize()
    return logits.cpu().numpy(), int(token.item())


@pytest.fixture(scope="module")
def head_w(pkg):
    return pkg.seeded.q8_0_matrix(21, pkg.seeded.W_HEAD, 151936, D)


def test_q8_pack_layout(pkg, cuda, head_w):
    torch = cuda
    n = 1001
    with _ctx(pkg) as ctx:
        packed = _packed(torch, ctx, pkg, head_w[:n * ROW8], n)
        torch.cuda.synchronize()
        assert np.array_equal(packed.cpu().numpy(), pkg.seeded.q8_0_planes(head_w[:n * ROW8], n))


@pytest.mark.parametrize("seed", [1, 2])
def test_q8_head_full_vocab(pkg, orc, cuda, head_w, seed):
    torch = cuda
    S = pkg.seeded
    n = 151936
    state = S.normal(seed, S.STATE, D)
    gamma = (1.0 + 0.1 * S.normal(seed, S.GAMMA_OUT, D)).astype(np.float32)
    want, want_tok = orc.lm_head_q8_0(state, gamma, head_w, n)
    with _ctx(pkg) as ctx:
        packed = _packed(torch, ctx, pkg, head_w, n)
        got, tok = _run_head(torch, ctx, packed, n, gamma, state)
        assert ctx.device_status() == 0
    assert nerr(got, want) <= TOL
    assert tok == orc.greedy_pick(got)
    top = np.sort(want)[-2:]
    if top[1] - top[0] > 2 * TOL * np.sqrt(np.mean(want.astype(np.float64) ** 2)):
        assert tok == want_tok


@pytest.mark.parametrize("n_rows", [1, 3, 4, 31, 32, 33, 1001, 4737])
def test_q8_head_ragged_rows(pkg, orc, cuda, head_w, n_rows):
    torch = cuda
    S = pkg.seeded
    state = S.normal(7, S.STATE, D)
    gamma = np.ones(D, dtype=np.float32)
    w = head_w[:n_rows * ROW8]
    want, _ = orc.lm_head_q8_0(state, gamma, w, n_rows)
    with _ctx(pkg) as ctx:
        got, tok = _run_head(torch, ctx, _packed(torch, ctx, pkg, w, n_rows), n_rows, gamma,
                             state)
    assert nerr(got, want) <= TOL and tok == orc.greedy_pick(got)


def _set_d(w, row, value_f16):
    """Sets every block scale of a row (bytes 0..1 of each 34-byte block)."""
    w.reshape(-1, 28, 34)[row, :, 0:2] = np.frombuffer(np.float16(value_f16).tobytes(),
                                                      dtype=np.uint8)


def test_q8_pick_ties_nan_and_empty(pkg, orc, cuda, head_w):
    """The host loop's rules (generate_stream_05b.c:872-878) on the device:
    equal maxima -> the first row, NaN never wins, nothing above -1e30 -> 0."""
    torch = cuda
    n = 20000
    w = head_w[:n * ROW8].copy()
    wr = w.reshape(n, ROW8)
    _set_d(w, 9001, 1.0)
    wr[3001] = wr[9001]   # an odd and an even row, different CTAs
    wr[17000] = wr[9001]
    _set_d(w, 6, np.nan)
    state = pkg.seeded.normal(3, pkg.seeded.STATE, D)
    gamma = np.ones(D, dtype=np.float32)
    with _ctx(pkg) as ctx:
        packed = _packed(torch, ctx, pkg, w, n)
        got, tok = _run_head(torch, ctx, packed, n, gamma, state)
        assert np.isnan(got[6])
        assert got[3001] == got[9001] == got[17000]
        if got[9001] > 0:
            assert tok == 3001
        assert tok == orc.greedy_pick(got)
        all_nan = head_w[:64 * ROW8].copy()
        for r in range(64):
            _set_d(all_nan, r, np.nan)
        got2, tok2 = _run_head(torch, ctx, _packed(torch, ctx, pkg, all_nan, 64), 64, gamma,
                               state)
        assert np.isnan(got2).all() and tok2 == 0
        got3, tok3 = _run_head(torch, ctx, packed, n, gamma, state)
        assert tok3 == tok and np.array_equal(got3.view(np.uint32), got.view(np.uint32))


def test_head_kind_follows_shape(pkg, cuda, head_w):
    """The Q8_0 head is built for d_model 896 and the Q6_K head for 1536; the
    other pairing is refused, not misread."""
    torch = cuda
    state = torch.zeros(1536, dtype=torch.float32, device="cuda")
    gamma = torch.ones(1536, dtype=torch.float32, device="cuda")
    logits = torch.empty(64, dtype=torch.float32, device="cuda")
    with _ctx(pkg) as ctx:
        packed = _packed(torch, ctx, pkg, head_w[:64 * ROW8], 64)
        with pytest.raises(pkg.GqaError, match="Q6_K"):
            ctx.lm_head(packed, 64, gamma, state, logits)
        with pytest.raises(pkg.GqaError, match="no output"):
            ctx.lm_head_q8_0(packed, 64, gamma, state)
    with pkg.Context() as ctx:
        with pytest.raises(pkg.GqaError, match="Q8_0"):
            ctx.lm_head_q8_0(packed, 64, gamma, state, logits)


def test_token_embedding_05b(pkg, orc, cuda):
    torch = cuda
    rows = 3000
    table = pkg.seeded.q4_0_matrix(5, pkg.seeded.TOKEN_EMBD, rows, D, 1.0 / 4.6)
    with _ctx(pkg) as ctx:
        t = _t(torch, table)
        state = torch.zeros(D, dtype=torch.float32, device="cuda")
        for tok in (0, 1, 2047, rows - 1):
            ctx.token_embedding(t, rows, torch.tensor([tok], dtype=torch.int32, device="cuda"),
                                state)
            torch.cuda.synchronize()
            want = orc.token_embedding(table, tok, D)
            assert np.array_equal(state.cpu().numpy().view(np.uint32), want.view(np.uint32))
        ctx.token_embedding(t, rows, torch.tensor([rows], dtype=torch.int32, device="cuda"), state)
        torch.cuda.synchronize()
        assert ctx.device_status() == pkg.gqa.STATUS_BAD_TOKEN


def _layer(pkg, seed, t_max=4096):
    S = pkg.seeded
    x, wq, bq, wo, ga, kc, vc = S.attention_block_inputs(seed, t_max=t_max, d_model=D,
                                                         n_heads_kv=NKV, head_dim=HD)
    wg, wu, wd, gf = S.ffn_block_inputs(seed, d_model=D, d_ffn=DFFN)
    return x, (wq, bq, wo, ga), (wg, wu, wd, gf), kc, vc


@pytest.mark.parametrize("pos", [0, 1, 127, 2500, 4095])
def test_attention_and_ffn_blocks_05b(pkg, orc, cuda, pos):
    torch = cuda
    x, attn, ffn, kc, vc = _layer(pkg, 40 + pos % 7)
    # oracle: the attention half, then the FFN half, as decoder_layer_sized
    k_ref, v_ref = kc.copy(), vc.copy()
    z1 = orc.output_norm(x, attn[3])
    qkv = orc.ref_gemv_q4_0(attn[0], z1, attn[1], D + 2 * NKV * HD, D)
    orc.layer_attention(qkv, k_ref, v_ref, pos, pos + 1, NQ, NKV, head_dim=HD)
    r = (orc.ref_gemv_q4_0(attn[2], qkv[:D], None, D, D) + x).astype(np.float32)
    h = orc.ref_swiglu(ffn[0], ffn[1], orc.output_norm(r, ffn[3]), DFFN, D)
    y = (orc.ref_gemv_q4_0(ffn[2], h, None, D, DFFN) + r).astype(np.float32)
    with _ctx(pkg) as ctx:
        da, df = [_t(torch, a) for a in attn], [_t(torch, a) for a in ffn]
        k, v = _t(torch, kc), _t(torch, vc)
        state = _t(torch, x)
        ctx.attention_block(pkg.block_weights_of(*da), pkg.kv_of(k, v), state, pos, pos + 1)
        torch.cuda.synchronize()
        assert nerr(state.cpu().numpy(), r) <= TOL
        ctx.ffn_block(pkg.ffn_weights_of(*df), state)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(state.cpu().numpy(), y) <= TOL
        # the new K / V rows come from the projection (its own summation order)
        assert nerr(k.cpu().numpy()[:, pos], k_ref[:, pos]) <= TOL
        assert nerr(v.cpu().numpy()[:, pos], v_ref[:, pos]) <= TOL


def test_decoder_layers_05b(pkg, orc, cuda):
    """Three layers with the position on the device, advanced afterwards,
    then the same from a graph replay at the next position."""
    torch = cuda
    pos0 = 1800
    layers = [_layer(pkg, 60 + l) for l in range(3)]
    x = layers[0][0]
    ref_kv = [(L[3].copy(), L[4].copy()) for L in layers]
    want = []
    y = x
    for step in range(2):
        for (xx, attn, ffn, _, _), (kc, vc) in zip(layers, ref_kv):
            y = orc.decoder_layer_sized(y, attn, ffn, kc, vc, pos0 + step, pos0 + step + 1,
                                        NQ, NKV, HD, DFFN)
        want.append(y.copy())
    with _ctx(pkg) as ctx:
        keep, attn, ffn, kvs = [], [], [], []
        for (_, wa, wf, kc, vc) in layers:
            da, df = [_t(torch, a) for a in wa], [_t(torch, a) for a in wf]
            k, v = _t(torch, kc), _t(torch, vc)
            keep += da + df + [k, v]
            attn.append(pkg.block_weights_of(*da))
            ffn.append(pkg.ffn_weights_of(*df))
            kvs.append(pkg.kv_of(k, v))
        state = _t(torch, x)
        d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
        ctx.decoder_layers(attn, ffn, kvs, state, d_pos, advance=True)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0 and int(d_pos.item()) == pos0 + 1
        assert nerr(state.cpu().numpy(), want[0]) <= TOL
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                ctx.decoder_layers(attn, ffn, kvs, state, d_pos, advance=True, stream=s)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        assert ctx.device_status() == 0 and int(d_pos.item()) == pos0 + 2
        assert nerr(state.cpu().numpy(), want[1]) <= TOL
        del g


def test_decode_token_05b(pkg, orc, cuda, head_w):
    """Two layers + the Q8_0 head, three greedy steps chained on the device,
    the third from a graph replay, against the oracle step by step."""
    torch = cuda
    S = pkg.seeded
    n_layers, pos0, vocab = 2, 900, 32768
    w_head = head_w[:vocab * ROW8]
    table = S.q4_0_matrix(6, S.TOKEN_EMBD, vocab, D, 1.0 / 4.6)
    gamma_out = (1.0 + 0.1 * S.normal(6, S.GAMMA_OUT, D)).astype(np.float32)
    layers = [_layer(pkg, 300 + l) for l in range(n_layers)]
    ref_kv = [(L[3].copy(), L[4].copy()) for L in layers]
    tok = 77
    want_tokens, want_logits = [], []
    for step in range(3):
        logits, tok = orc.ref_decode_token(table, [(L[1], L[2]) for L in layers], ref_kv,
                                           gamma_out, w_head, tok, pos0 + step, model="0.5b")
        want_tokens.append(tok)
        want_logits.append(logits)
    with _ctx(pkg) as ctx:
        keep, attn, ffn, kvs = [], [], [], []
        for (_, wa, wf, kc, vc) in layers:
            da, df = [_t(torch, a) for a in wa], [_t(torch, a) for a in wf]
            k, v = _t(torch, kc), _t(torch, vc)
            keep += da + df + [k, v]
            attn.append(pkg.block_weights_of(*da))
            ffn.append(pkg.ffn_weights_of(*df))
            kvs.append(pkg.kv_of(k, v))
        packed = _packed(torch, ctx, pkg, w_head, vocab)
        model = pkg.ModelHandle(attn, ffn, kvs, _t(torch, table), _t(torch, gamma_out), packed,
                                vocab, pkg.gqa.HEAD_Q8_0)
        state = torch.zeros(D, dtype=torch.float32, device="cuda")
        logits = torch.empty(vocab, dtype=torch.float32, device="cuda")
        d_tok = torch.tensor([77], dtype=torch.int32, device="cuda")
        d_pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
        for step in range(2):
            ctx.decode_token(model, state, d_tok, d_pos, logits)
            torch.cuda.synchronize()
            assert ctx.device_status() == 0
            assert nerr(logits.cpu().numpy(), want_logits[step]) <= TOL
            assert int(d_tok.item()) == want_tokens[step]
            assert int(d_pos.item()) == pos0 + step + 1
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                ctx.decode_token(model, state, d_tok, d_pos, logits, stream=s)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert nerr(logits.cpu().numpy(), want_logits[2]) <= TOL
        assert int(d_tok.item()) == want_tokens[2]
        del g
        # the Q6_K head type is refused on this shape
        bad = pkg.ModelHandle(attn, ffn, kvs, _t(torch, table), _t(torch, gamma_out), packed,
                              vocab, pkg.gqa.HEAD_Q6_K)
        with pytest.raises(pkg.GqaError, match="Q6_K"):
            ctx.decode_token(bad, state, d_tok, d_pos)


def test_gguf_05b_load_and_query(pkg, orc, cuda, tmp_path):
    """A 0.5B-shaped GGUF (two layers, Q8_0 head) through gqa_model_load and a
    RAW_QUERY of the session, against the request loop over the 0.5B pieces."""
    vocab, n_layers = 2048, 2
    path = tmp_path / "q05.gguf"
    offsets, arrays = gw.qwen_model(path, pkg.seeded, n_layers=n_layers, vocab=vocab, seed=13,
                                    model="0.5b")
    layers = [(a, f) for a, f in arrays["layers"]]
    kv = [(np.zeros((NKV, 4096, HD), np.float32), np.zeros((NKV, 4096, HD), np.float32))
          for _ in layers]
    prompt = [5, 17, 999, 3]
    margins = []
    want = orc.ref_server_query(arrays["embd"], layers, kv, arrays["gamma_out"], arrays["head"],
                                prompt, 0, 5, margins=margins, model="0.5b")
    with _ctx(pkg) as ctx:
        with pkg.Gguf(str(path)) as g:
            model = pkg.LoadedModel(ctx, g)
        kvs = ctx.kv_alloc(n_layers)
        try:
            view = model.view(kvs)
            assert view.lm_head_type == pkg.gqa.HEAD_Q8_0 and view.vocab == vocab
            s = pkg.Session(ctx, view, 4096)
            try:
                got = s.query(prompt, 5, raw=True)
            finally:
                s.destroy()
        finally:
            ctx.kv_free(kvs)
            model.free()
    if min(margins) < 1e-3:
        pytest.skip("near-tie in the oracle's picks")
    assert got == want and len(got) == 5
