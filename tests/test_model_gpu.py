"""A GGUF model end to end on the GPU: gqa_model_load from a Qwen2.5-1.5B-
shaped file (two layers, small vocabulary, seeded weights) and the server's
requests (gqa_session_*: SET_BASE, QUERY, RAW_QUERY, STATUS) against the
reference's request loop restated over its compiled pieces
(qwen_server.c:815-1049)."""
import numpy as np
import pytest

import gguf_writer as gw

pytestmark = pytest.mark.gpu
VOCAB = 2048
N_LAYERS = 2


@pytest.fixture(scope="module")
def model_file(pkg, tmp_path_factory):
    path = tmp_path_factory.mktemp("gguf") / "qwen2-test.gguf"
    offsets, arrays = gw.qwen_model(path, pkg.seeded, n_layers=N_LAYERS, vocab=VOCAB, seed=12)
    return path, arrays


def _ref_state(arrays):
    layers = [(a, f) for a, f in arrays["layers"]]
    kv = [(np.zeros((2, 4096, 128), np.float32), np.zeros((2, 4096, 128), np.float32))
          for _ in layers]
    return layers, kv


def _ref_query(orc, arrays, layers, kv, tokens, cur_pos, max_new, eog=(151643, 151645)):
    margins = []
    out = orc.ref_server_query(arrays["embd"], layers, kv, arrays["gamma_out"], arrays["head"],
                               tokens, cur_pos, max_new, eog=eog, margins=margins)
    return out, margins


def _close_call(margins):
    return min(margins) < 1e-3 if margins else False


@pytest.fixture(scope="module")
def loaded(pkg, cuda, model_file):
    path, arrays = model_file
    ctx = pkg.Context(t_max=4096)
    with pkg.Gguf(str(path)) as g:
        model = pkg.LoadedModel(ctx, g)
    kvs = ctx.kv_alloc(N_LAYERS)
    yield ctx, model, kvs, arrays
    ctx.kv_free(kvs)
    model.free()
    ctx.close()


def test_loader_layout(pkg, cuda, loaded):
    ctx, model, kvs, arrays = loaded
    assert model.n_layers == N_LAYERS and model.vocab == VOCAB
    view = model.view(kvs)
    torch = cuda
    # W_qkv on the device is attn_q | attn_k | attn_v rows, as the server stacks them
    w_qkv = arrays["layers"][1][0][0]
    from cuda.bindings import runtime as rt
    host = np.empty(w_qkv.size, dtype=np.uint8)
    (err,) = rt.cudaMemcpy(host.ctypes.data, view.attn[1].w_qkv, w_qkv.size,
                           rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    assert np.array_equal(host, w_qkv)
    torch.cuda.synchronize()


def test_raw_query_matches_reference(pkg, orc, cuda, loaded):
    ctx, model, kvs, arrays = loaded
    layers, kv = _ref_state(arrays)
    prompt = [5, 17, 999, 3]
    want, margins = _ref_query(orc, arrays, layers, kv, prompt, 0, 5)
    s = pkg.Session(ctx, model.view(kvs), 4096)
    try:
        got = s.query(prompt, 5, raw=True)
        if _close_call(margins):
            pytest.skip("near-tie in the reference's picks")
        assert got == want and len(got) == 5
        assert s.status() == {"base_pos": 0, "base_hash": 0, "base_generation": 0,
                              "ready": False}
    finally:
        s.destroy()


def test_set_base_then_queries(pkg, orc, cuda, loaded):
    ctx, model, kvs, arrays = loaded
    layers, kv = _ref_state(arrays)
    base = [3, 1, 4, 1, 5, 9, 2, 6]
    h = orc.ref_server_set_base(arrays["embd"], layers, kv, base)
    s = pkg.Session(ctx, model.view(kvs), 4096)
    try:
        with pytest.raises(pkg.GqaError, match="ERR_NOT_READY"):
            s.query([1, 2], 3)
        s.set_base(base)
        st = s.status()
        assert st == {"base_pos": len(base), "base_hash": h, "base_generation": 1, "ready": True}
        for prompt, max_new in (([7, 7, 100], 4), ([1500], 3)):
            want, margins = _ref_query(orc, arrays, layers, kv, prompt, len(base), max_new)
            got = s.query(prompt, max_new)
            assert _close_call(margins) or got == want
        with pytest.raises(pkg.GqaError, match="ERR_RAW_NOT_ALLOWED_WHEN_BASE_ACTIVE"):
            s.query([1], 2, raw=True)
        with pytest.raises(pkg.GqaError, match="ERR_INVALID_TOKEN"):
            s.query([VOCAB], 2)
        with pytest.raises(pkg.GqaError, match="ERR_INVALID_TOKEN"):
            s.query([1], 0)
        with pytest.raises(pkg.GqaError, match="ERR_CONTEXT_FULL"):
            s.query([1], 4096 - len(base) - 1)
        with pytest.raises(pkg.GqaError, match="ERR_BAD_REQUEST"):
            s.set_base([])
        with pytest.raises(pkg.GqaError, match="ERR_CONTEXT_FULL"):
            s.set_base([1] * 4095)
        assert s.status()["base_generation"] == 1  # rejected requests change nothing
    finally:
        s.destroy()


def test_end_of_generation_stop(pkg, orc, cuda, loaded):
    """With the third generated id declared end-of-generation, the query stops
    before emitting it (the server's EOG check, qwen_server.c:1007-1010)."""
    ctx, model, kvs, arrays = loaded
    layers, kv = _ref_state(arrays)
    prompt = [11, 22, 33]
    free_run, margins = _ref_query(orc, arrays, layers, kv, prompt, 0, 4)
    if _close_call(margins):
        pytest.skip("near-tie in the reference's picks")
    eog = free_run[2]
    expect = free_run[:free_run.index(eog)]
    s = pkg.Session(ctx, model.view(kvs), 4096, eog=[eog])
    try:
        assert s.query(prompt, 4, raw=True) == expect
    finally:
        s.destroy()


def test_loader_rejects_wrong_types(pkg, cuda, tmp_path):
    """A projection stored in another quantisation is an error, not a misread."""
    d = 1536
    path = tmp_path / "wrong.gguf"
    rng = np.random.default_rng(1)
    tensors = [("token_embd.weight", gw.T_Q4_0, [d, 64], rng.integers(0, 256, 64 * 864, np.uint8)),
               ("output_norm.weight", gw.T_F32, [d], np.ones(d, np.float32)),
               ("output.weight", gw.T_Q8_0, [d, 64], rng.integers(0, 256, 64 * 48 * 34, np.uint8))]
    gw.write(path, [("qwen2.block_count", gw.U32, 1)], tensors)
    with pkg.Context() as ctx, pkg.Gguf(str(path)) as g:
        with pytest.raises(pkg.GqaError, match="output.weight"):
            pkg.LoadedModel(ctx, g)
