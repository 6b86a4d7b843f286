"""The model's ends on the GPU: Q6_K LM head with the output RMSNorm and the
greedy pick (gqa_lm_head), the Q4_0 token embedding (gqa_token_embedding) and
the whole-model decode step (gqa_decode_token) -- against the reference's own
CPU Q6_K GEMV (test_gemv_q6_k.c, compiled), its embedding lookup
(test_full_model_logits.c, compiled) and decoder-layer step, with the output
norm and the pick restated (test_full_model_logits.c:944-948,
qwen_server.c:998-1005)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
VOCAB = 151936
ROW = 1260
TOL = 1e-4  # normalised by the logits' RMS
# the columns the reference's own Q6_K test probes with unit vectors
# (test_gemv_q6_k.c:209): nibble, high-bit, scale and superblock boundaries
BASIS = [0, 15, 16, 31, 32, 63, 64, 95, 96, 127, 128, 255, 512, 1024, 1535]


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def rel_l2(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(np.asarray(got, dtype=np.float64) - ref) / np.linalg.norm(ref))


def cos_sim(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.fixture(scope="module")
def head_w(pkg):
    return pkg.seeded.q6_k_matrix(11, pkg.seeded.W_HEAD, VOCAB)


def _packed(torch, ctx, pkg, w, n_rows):
    raw = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    packed = torch.empty(pkg.Context.lm_head_packed_bytes(n_rows), dtype=torch.uint8,
                         device="cuda")
    ctx.lm_head_pack(raw, n_rows, packed)
    return packed


def _run_head(torch, ctx, packed, n_rows, gamma, state):
    g = torch.from_numpy(np.ascontiguousarray(gamma, dtype=np.float32)).cuda()
    s = torch.from_numpy(np.ascontiguousarray(state, dtype=np.float32)).cuda()
    logits = torch.empty(n_rows, dtype=torch.float32, device="cuda")
    token = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    ctx.lm_head(packed, n_rows, g, s, logits, token)
    torch.cuda.synchronize()
    return logits.cpu().numpy(), int(token.item())


def test_pack_layout(pkg, cuda, head_w):
    torch = cuda
    n = 4096
    w = head_w[:n * ROW]
    with pkg.Context() as ctx:
        packed = _packed(torch, ctx, pkg, w, n)
        torch.cuda.synchronize()
        assert np.array_equal(packed.cpu().numpy(), pkg.seeded.q6_k_planes(w, n))


def _gamma_for_unit(orc, i, target=32.0):
    """state = e_i and a gamma with gamma[i] tuned so that the output norm
    gives z = target * e_i exactly (a power of two keeps every product exact)."""
    state = np.zeros(1536, dtype=np.float32)
    state[i] = 1.0
    gamma = np.ones(1536, dtype=np.float32)
    z1 = orc.output_norm(state, gamma)[i]
    g = np.float32(target / z1)
    for _ in range(64):
        gamma[i] = g
        z = orc.output_norm(state, gamma)[i]
        if z == np.float32(target):
            return state, gamma
        g = np.nextafter(g, np.float32(np.inf) if z < target else np.float32(-np.inf))
    raise AssertionError("no gamma gives an exact unit")


def test_head_basis_vectors_bit_exact(pkg, orc, cuda, head_w):
    """Unit inputs at the reference test's columns: every logit is one
    dequantised weight times 32, bit for bit the reference's."""
    torch = cuda
    n = 8192
    w = head_w[:n * ROW]
    with pkg.Context() as ctx:
        packed = _packed(torch, ctx, pkg, w, n)
        for i in BASIS:
            state, gamma = _gamma_for_unit(orc, i)
            got, tok = _run_head(torch, ctx, packed, n, gamma, state)
            z = orc.output_norm(state, gamma)
            want = orc.ref_gemv_q6_k(w, z)
            assert np.array_equal(got, want), i  # exact values
            assert tok == orc.greedy_pick(got)
        assert ctx.device_status() == 0


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_head_full_vocab_matches_reference(pkg, orc, cuda, head_w, seed):
    torch = cuda
    state = pkg.seeded.normal(100 + seed, pkg.seeded.STATE, 1536) * (1 + seed)
    gamma = (1.0 + 0.1 * pkg.seeded.normal(100 + seed, pkg.seeded.GAMMA_OUT, 1536)).astype(
        np.float32)
    want, want_tok = orc.ref_lm_head(state, gamma, head_w)
    with pkg.Context() as ctx:
        packed = _packed(torch, ctx, pkg, head_w, VOCAB)
        got, tok = _run_head(torch, ctx, packed, VOCAB, gamma, state)
        assert ctx.device_status() == 0
    # the reference test's own bar (test_gemv_q6_k.c:310) and the fp32 bar
    assert rel_l2(got, want) < 1e-5
    assert cos_sim(got, want) > 0.999999
    assert nerr(got, want) <= TOL
    assert np.isfinite(got).all()
    assert tok == orc.greedy_pick(got)
    top2 = np.sort(want)[-2:]
    if top2[1] - top2[0] > 1e-3:
        assert tok == want_tok


@pytest.mark.parametrize("n_rows", [1, 7, 37, 300, 4097])
def test_head_ragged_row_counts(pkg, orc, cuda, head_w, n_rows):
    """Fewer rows than warps, and counts that are no multiple of anything."""
    torch = cuda
    w = head_w[:n_rows * ROW]
    state = pkg.seeded.normal(7, pkg.seeded.STATE, 1536)
    gamma = np.ones(1536, dtype=np.float32)
    want, _ = orc.ref_lm_head(state, gamma, w)
    with pkg.Context() as ctx:
        packed = _packed(torch, ctx, pkg, w, n_rows)
        got, tok = _run_head(torch, ctx, packed, n_rows, gamma, state)
    assert nerr(got, want) <= TOL
    assert tok == orc.greedy_pick(got)


def _set_d(w, row, value_f16):
    """Sets every superblock scale d of a row (bytes 208..209 of each block)."""
    w = w.reshape(-1, 6, 210)
    w[row, :, 208:210] = np.frombuffer(np.float16(value_f16).tobytes(), dtype=np.uint8)


def test_pick_ties_nan_and_empty(pkg, orc, cuda, head_w):
    """The host loop's rules on the device: equal maxima -> the first row,
    NaN never wins, and nothing above -1e30 -> token 0."""
    torch = cuda
    n = 20000
    w = head_w[:n * ROW].copy()
    wr = w.reshape(n, ROW)
    # rows 3000 and 17000 (different CTAs) are copies of row 9000, scaled up
    # to be the maximum; row 5 has NaN scales
    _set_d(w, 9000, 1.0)
    wr[3000] = wr[9000]
    wr[17000] = wr[9000]
    _set_d(w, 5, np.nan)
    state = pkg.seeded.normal(3, pkg.seeded.STATE, 1536)
    gamma = np.ones(1536, dtype=np.float32)
    with pkg.Context() as ctx:
        packed = _packed(torch, ctx, pkg, w, n)
        got, tok = _run_head(torch, ctx, packed, n, gamma, state)
        assert np.isnan(got[5])
        if got[9000] > 0:  # the copies are the maximum
            assert got[3000] == got[9000] == got[17000]
            assert tok == 3000
        else:  # the copies are the minimum: the pick is elsewhere
            assert tok == orc.greedy_pick(got)
        assert tok == orc.greedy_pick(got)
        # every logit NaN: no candidate, token 0
        all_nan = head_w[:512 * ROW].copy()
        for r in range(512):
            _set_d(all_nan, r, np.nan)
        packed2 = _packed(torch, ctx, pkg, all_nan, 512)
        got2, tok2 = _run_head(torch, ctx, packed2, 512, gamma, state)
        assert np.isnan(got2).all() and tok2 == 0
        # the arrival counter is back at zero: the next launch picks again
        got3, tok3 = _run_head(torch, ctx, packed, n, gamma, state)
        assert tok3 == tok and np.array_equal(got3.view(np.uint32), got.view(np.uint32))


def test_head_token_only(pkg, orc, cuda, head_w):
    torch = cuda
    n = 50000
    w = head_w[:n * ROW]
    state = pkg.seeded.normal(9, pkg.seeded.STATE, 1536)
    gamma = np.ones(1536, dtype=np.float32)
    with pkg.Context() as ctx:
        packed = _packed(torch, ctx, pkg, w, n)
        got, tok = _run_head(torch, ctx, packed, n, gamma, state)
        g = torch.from_numpy(gamma).cuda()
        s = torch.from_numpy(state).cuda()
        token = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        ctx.lm_head(packed, n, g, s, None, token)
        torch.cuda.synchronize()
        assert int(token.item()) == tok
        with pytest.raises(pkg.GqaError):
            ctx.lm_head(packed, n, g, s, None, None)


def test_token_embedding(pkg, orc, cuda):
    torch = cuda
    rows = 4096
    table = pkg.seeded.q4_0_matrix(5, pkg.seeded.TOKEN_EMBD, rows, 1536, 1.0 / 4.6)
    with pkg.Context() as ctx:
        t = torch.from_numpy(table).cuda()
        state = torch.zeros(1536, dtype=torch.float32, device="cuda")
        for tok in (0, 1, 1234, rows - 1):
            d_tok = torch.tensor([tok], dtype=torch.int32, device="cuda")
            ctx.token_embedding(t, rows, d_tok, state)
            torch.cuda.synchronize()
            want = orc.ref_token_embedding(table, tok)
            assert np.array_equal(state.cpu().numpy().view(np.uint32), want.view(np.uint32))
        assert ctx.device_status() == 0
        before = state.clone()
        for bad in (-1, rows):
            ctx.token_embedding(t, rows, torch.tensor([bad], dtype=torch.int32, device="cuda"),
                                state)
            torch.cuda.synchronize()
            assert ctx.device_status() == pkg.gqa.STATUS_BAD_TOKEN
            assert torch.equal(state, before)


def test_decode_token_steps_and_graph(pkg, orc, cuda, head_w):
    """Two decoder layers + head, three greedy steps chained on the device
    (the picked token feeds the next step's embedding), the third step from a
    graph replay; against the reference's CPU step by step."""
    torch = cuda
    n_layers, pos0, vocab = 2, 1000, 32768
    w_head = head_w[:vocab * ROW]
    table = pkg.seeded.q4_0_matrix(6, pkg.seeded.TOKEN_EMBD, vocab, 1536, 1.0 / 4.6)
    gamma_out = (1.0 + 0.1 * pkg.seeded.normal(6, pkg.seeded.GAMMA_OUT, 1536)).astype(np.float32)
    layers = []
    for l in range(n_layers):
        x, wq, bq, wo, ga, kc, vc = pkg.seeded.attention_block_inputs(300 + l)
        wg, wu, wd, gf = pkg.seeded.ffn_block_inputs(300 + l)
        layers.append(((wq, bq, wo, ga), (wg, wu, wd, gf), kc, vc))
    ref_kv = [(L[2].copy(), L[3].copy()) for L in layers]
    tok = 77
    want_tokens, want_logits = [], []
    for step in range(3):
        logits, tok = orc.ref_decode_token(table, [(L[0], L[1]) for L in layers], ref_kv,
                                           gamma_out, w_head, tok, pos0 + step)
        want_tokens.append(tok)
        want_logits.append(logits)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    with pkg.Context(t_max=4096) as ctx:
        keep, attn, ffn, kvs = [], [], [], []
        for (wa, wf, kc, vc) in layers:
            da, df = [t(a) for a in wa], [t(a) for a in wf]
            k, v = t(kc), t(vc)
            keep += da + df + [k, v]
            attn.append(pkg.block_weights_of(*da))
            ffn.append(pkg.ffn_weights_of(*df))
            kvs.append(pkg.kv_of(k, v))
        d_table, d_gamma = t(table), t(gamma_out)
        packed = _packed(torch, ctx, pkg, w_head, vocab)
        model = pkg.ModelHandle(attn, ffn, kvs, d_table, d_gamma, packed, vocab)
        state = torch.zeros(1536, dtype=torch.float32, device="cuda")
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
