"""ctypes access to the oracle -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and the cpu_baseline leg of
bench.py, as the checker (never as the thing measured or shipped).

* ``liboracle.so``      -- gqa_oracle.c, the C restatement of the reference's
                           fp32 attention with run-time shapes (any t_max).
* ``_ref/libgqa_ref_bench.so`` / ``_ref/libgqa_ref_layer.so`` /
  ``_ref/libgqa_ref_head.so`` / ``_ref/libgqa_ref_model.so`` -- the
  reference's own cpu_attention_gqa_pipeline (attention_gqa_benchmark.c:
  109-216), cpu_decoder_layer_step (test_28_layers_real.c:192-318), Q6_K
  LM-head GEMV cpu_gemv_q6_k_ref (test_gemv_q6_k.c:46-94), token embedding
  lookup get_token_embedding (test_full_model_logits.c:584-597) and the
  server's GGUF reading parse_gguf_tensors / load_tokenizer_tokens
  (qwen_server.c:113-266, ``_ref/libgqa_ref_server.so``), compiled unmodified
  from its sources by oracle/Makefile.  They exist only where the
  reference sources were present at build time; REF_T_MAX = 4096 is their
  compile-time cache stride.  The layer library also exports the reference's
  size-generic cpu_gemv_q4_0_bias / cpu_swiglu_fused (test_28_layers_real.c:
  90-131), from which decoder_layer_sized() composes the Qwen2.5-0.5B layer
  (pinned bit for bit to cpu_decoder_layer_step at the 1.5B sizes).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_BENCH_SO = os.path.join(HERE, "_ref", "libgqa_ref_bench.so")
REF_LAYER_SO = os.path.join(HERE, "_ref", "libgqa_ref_layer.so")
REF_HEAD_SO = os.path.join(HERE, "_ref", "libgqa_ref_head.so")
REF_MODEL_SO = os.path.join(HERE, "_ref", "libgqa_ref_model.so")
REF_SERVER_SO = os.path.join(HERE, "_ref", "libgqa_ref_server.so")
REF_Q8_SO = os.path.join(HERE, "_ref", "libgqa_ref_q8.so")
REF_T_MAX = 4096

_f = ctypes.c_float
_i = ctypes.c_int
_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)
_fpp = ctypes.POINTER(_fp)

_libs: dict[str, ctypes.CDLL] = {}


def build() -> None:
    """make -C oracle (restatement always; the reference only if its sources exist)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load(path: str) -> ctypes.CDLL:
    if path not in _libs:
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run make -C oracle)")
        _libs[path] = ctypes.CDLL(path)
    return _libs[path]


def have_reference() -> bool:
    return all(os.path.exists(p) for p in (REF_BENCH_SO, REF_LAYER_SO, REF_HEAD_SO, REF_MODEL_SO,
                                           REF_SERVER_SO))


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _lib():
    lib = _load(ORACLE_SO)
    if not getattr(lib, "_typed", False):
        lib.oracle_inv_freq.argtypes = [_f, _i, _fp]
        lib.oracle_rope_kv_append.argtypes = [_fp, _fp, _fp, _fp, _fp, _i, _i, _i, _i, _i, _f]
        lib.oracle_attention.argtypes = [_fp, _fp, _fp, _i, _i, _i, _i, _i, _fp]
        lib.oracle_layer_attention.argtypes = [_fp, _fp, _fp, _i, _i, _i, _i, _i, _i, _f]
        lib.oracle_decode_batched.argtypes = [_i, _fpp, _fpp, _fpp, _ip, _i, _i, _i, _i, _f, _fpp,
                                              _i]
        lib.oracle_attention_batched.argtypes = [_i, _fpp, _fpp, _fpp, _ip, _i, _i, _i, _i, _fpp,
                                                 _i]
        lib.oracle_attention_partial.argtypes = [_fp, _fp, _fp, _i, _i, _i, _i, _i, _i, _fp, _fp,
                                                 _fp]
        lib.oracle_lse_combine.argtypes = [_i, _fp, _fp, _fp, _i, _i, _fp]
        lib.oracle_prefill_rows.argtypes = [_fp, _fp, _fp, _i, _i, _i, _i, _i, _f, _fp, _fp, _ip,
                                            _i, _fp, _i]
        for fn in (lib.oracle_inv_freq, lib.oracle_rope_kv_append, lib.oracle_attention,
                   lib.oracle_layer_attention, lib.oracle_decode_batched,
                   lib.oracle_attention_batched, lib.oracle_attention_partial,
                   lib.oracle_lse_combine, lib.oracle_prefill_rows):
            fn.restype = None
        lib._typed = True
    return lib


def inv_freq(rope_base: float = 1e6, head_dim: int = 128) -> np.ndarray:
    out = np.zeros(head_dim // 2, dtype=np.float32)
    _lib().oracle_inv_freq(rope_base, head_dim, _fptr(out))
    return out


def layer_attention(qkv: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, pos: int,
                    seq_len: int, n_heads_q: int = 12, n_heads_kv: int = 2,
                    rope_base: float = 1e6, head_dim: int = 128) -> None:
    """In place: caches [n_kv][t_max][head_dim] get row pos, qkv[:n_q*head_dim]
    becomes attn_out.  The restatement's loops take any head_dim; at 128 it is
    pinned to the compiled reference bit for bit."""
    t_max = k_cache.shape[1]
    _lib().oracle_layer_attention(_fptr(qkv), _fptr(k_cache), _fptr(v_cache), pos, seq_len, t_max,
                                  n_heads_q, n_heads_kv, head_dim, rope_base)


def rope_kv_append(q, k, v, k_cache, v_cache, pos, n_heads_q=12, n_heads_kv=2, rope_base=1e6):
    t_max = k_cache.shape[1]
    _lib().oracle_rope_kv_append(_fptr(q), _fptr(k), _fptr(v), _fptr(k_cache), _fptr(v_cache),
                                 pos, t_max, n_heads_q, n_heads_kv, 128, rope_base)


def attention(q, k_cache, v_cache, seq_len, n_heads_q=12, n_heads_kv=2) -> np.ndarray:
    out = np.zeros(n_heads_q * 128, dtype=np.float32)
    _lib().oracle_attention(_fptr(q), _fptr(k_cache), _fptr(v_cache), seq_len, k_cache.shape[1],
                            n_heads_q, n_heads_kv, 128, _fptr(out))
    return out


def _ptr_array(arrs):
    return (_fp * len(arrs))(*[_fptr(a) for a in arrs])


def decode_batched(qkv: list, k_caches: list, v_caches: list, seq_lens, n_heads_q=12,
                   n_heads_kv=2, rope_base=1e6, n_threads=None, head_dim=128) -> list:
    """One new token per sequence; caches appended in place; returns attn_out per sequence."""
    n = len(qkv)
    outs = [np.zeros(n_heads_q * head_dim, dtype=np.float32) for _ in range(n)]
    lens = (ctypes.c_int * n)(*[int(x) for x in seq_lens])
    _lib().oracle_decode_batched(n, _ptr_array(qkv), _ptr_array(k_caches), _ptr_array(v_caches),
                                 lens, k_caches[0].shape[1], n_heads_q, n_heads_kv, head_dim,
                                 rope_base, _ptr_array(outs), n_threads or os.cpu_count())
    return outs


def attention_batched(q: list, k_caches: list, v_caches: list, seq_lens, n_heads_q=12,
                      n_heads_kv=2, n_threads=None) -> list:
    n = len(q)
    outs = [np.zeros(n_heads_q * 128, dtype=np.float32) for _ in range(n)]
    lens = (ctypes.c_int * n)(*[int(x) for x in seq_lens])
    _lib().oracle_attention_batched(n, _ptr_array(q), _ptr_array(k_caches), _ptr_array(v_caches),
                                    lens, k_caches[0].shape[1], n_heads_q, n_heads_kv, 128,
                                    _ptr_array(outs), n_threads or os.cpu_count())
    return outs


def attention_partial(q, k_cache, v_cache, t_begin, t_end, n_heads_q=12, n_heads_kv=2):
    m = np.zeros(n_heads_q, dtype=np.float32)
    l = np.zeros(n_heads_q, dtype=np.float32)
    o = np.zeros(n_heads_q * 128, dtype=np.float32)
    _lib().oracle_attention_partial(_fptr(q), _fptr(k_cache), _fptr(v_cache), t_begin, t_end,
                                    k_cache.shape[1], n_heads_q, n_heads_kv, 128, _fptr(m),
                                    _fptr(l), _fptr(o))
    return m, l, o


def lse_combine(m: np.ndarray, l: np.ndarray, o: np.ndarray) -> np.ndarray:
    """m, l: [parts][rows]; o: [parts][rows][128] -> [rows][128]."""
    n_parts, n_rows = m.shape
    out = np.zeros((n_rows, 128), dtype=np.float32)
    _lib().oracle_lse_combine(n_parts, _fptr(np.ascontiguousarray(m)),
                              _fptr(np.ascontiguousarray(l)), _fptr(np.ascontiguousarray(o)),
                              n_rows, 128, _fptr(out))
    return out


def prefill_rows(q, k, v, rows, n_heads_q=12, n_heads_kv=2, rope_base=1e6, n_threads=None):
    """Causal attention rows of one sequence (q/k/v [S][heads*128], pre-RoPE)."""
    S = q.shape[0]
    kc = np.zeros((n_heads_kv, S, 128), dtype=np.float32)
    vc = np.zeros((n_heads_kv, S, 128), dtype=np.float32)
    rows_c = (ctypes.c_int * len(rows))(*[int(r) for r in rows])
    out = np.zeros((len(rows), n_heads_q * 128), dtype=np.float32)
    _lib().oracle_prefill_rows(_fptr(q), _fptr(k), _fptr(v), S, S, n_heads_q, n_heads_kv, 128,
                               rope_base, _fptr(kc), _fptr(vc), rows_c, len(rows), _fptr(out),
                               n_threads or os.cpu_count())
    return out, kc, vc


# ---- the reference itself (compiled from its sources) ----------------------

def _ref_lib(path, prefix):
    lib = _load(path)
    fn = getattr(lib, prefix + "_attention")
    if fn.argtypes is None:
        fn.argtypes = [_fp, _fp, _fp, _i, _i, _fp]
        fn.restype = _i
    return lib


def ref_bench_attention(qkv: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, pos: int,
                        seq_len: int) -> np.ndarray:
    """cpu_attention_gqa_pipeline with q/k/v injected; caches [2][4096][128] updated in place."""
    assert k_cache.shape == (2, REF_T_MAX, 128) and v_cache.shape == (2, REF_T_MAX, 128)
    out = np.zeros(1536, dtype=np.float32)
    rc = _ref_lib(REF_BENCH_SO, "ref_bench").ref_bench_attention(
        _fptr(qkv), _fptr(k_cache), _fptr(v_cache), pos, seq_len, _fptr(out))
    if rc != 0:
        raise ValueError("reference rejected pos/seq_len")
    return out


def ref_bench_attention_many(qkv: list, k_caches: list, v_caches: list, pos: list,
                             seq_len: list, n_threads: int) -> list:
    lib = _load(REF_BENCH_SO)
    fn = lib.ref_bench_attention_many
    if fn.argtypes is None:
        fn.argtypes = [_i, _fpp, _fpp, _fpp, _ip, _ip, _fpp, _i]
        fn.restype = _i
    n = len(qkv)
    outs = [np.zeros(1536, dtype=np.float32) for _ in range(n)]
    rc = fn(n, _ptr_array(qkv), _ptr_array(k_caches), _ptr_array(v_caches),
            (ctypes.c_int * n)(*pos), (ctypes.c_int * n)(*seq_len), _ptr_array(outs), n_threads)
    if rc != 0:
        raise ValueError("reference rejected pos/seq_len")
    return outs


def ref_layer_attention(qkv, k_cache, v_cache, pos, seq_len) -> np.ndarray:
    """cpu_decoder_layer_step's attention slice (weights chosen so y_out == attn_out)."""
    assert k_cache.shape == (2, REF_T_MAX, 128)
    out = np.zeros(1536, dtype=np.float32)
    rc = _ref_lib(REF_LAYER_SO, "ref_layer").ref_layer_attention(
        _fptr(qkv), _fptr(k_cache), _fptr(v_cache), pos, seq_len, _fptr(out))
    if rc != 0:
        raise ValueError("reference rejected pos/seq_len")
    return out


def ref_attention_block(x_in, w_qkv, b_qkv, w_o, gamma, k_cache, v_cache, pos, seq_len) -> np.ndarray:
    """The reference's cpu_decoder_layer_step with zero FFN weights: x_in +
    W_o * attn(RoPE(W_qkv * rmsnorm(x_in, gamma) + b_qkv)).  w_qkv / w_o are
    Q4_0 byte arrays ([2048][48] and [1536][48] blocks of 18 bytes); caches
    [2][4096][128] are updated in place at row pos."""
    assert k_cache.shape == (2, REF_T_MAX, 128) and v_cache.shape == (2, REF_T_MAX, 128)
    w_qkv = np.ascontiguousarray(w_qkv, dtype=np.uint8)
    w_o = np.ascontiguousarray(w_o, dtype=np.uint8)
    assert w_qkv.size == 2048 * 48 * 18 and w_o.size == 1536 * 48 * 18
    lib = _load(REF_LAYER_SO)
    fn = lib.ref_attention_block
    if fn.argtypes is None:
        _vp = ctypes.c_void_p
        fn.argtypes = [_fp, _vp, _fp, _vp, _fp, _fp, _fp, _i, _i, _fp]
        fn.restype = _i
    out = np.zeros(1536, dtype=np.float32)
    rc = fn(_fptr(np.ascontiguousarray(x_in, dtype=np.float32)), w_qkv.ctypes.data,
            _fptr(np.ascontiguousarray(b_qkv, dtype=np.float32)), w_o.ctypes.data,
            _fptr(np.ascontiguousarray(gamma, dtype=np.float32)), _fptr(k_cache), _fptr(v_cache),
            pos, seq_len, _fptr(out))
    if rc != 0:
        raise ValueError("reference rejected pos/seq_len")
    return out


def ref_decoder_layer(x_in, attn, ffn, k_cache, v_cache, pos, seq_len) -> np.ndarray:
    """The reference's cpu_decoder_layer_step with all weights given:
    attn = (w_qkv, b_qkv, w_o, gamma_attn), ffn = (w_gate, w_up, w_down,
    gamma_ffn) as Q4_0 byte arrays / float arrays; caches [2][4096][128]
    updated in place at row pos."""
    assert k_cache.shape == (2, REF_T_MAX, 128) and v_cache.shape == (2, REF_T_MAX, 128)
    w_qkv, b_qkv, w_o, g_a = attn
    w_gate, w_up, w_down, g_f = ffn
    arrs = [np.ascontiguousarray(a, dtype=np.uint8) for a in (w_qkv, w_o, w_gate, w_up, w_down)]
    assert arrs[2].size == 8960 * 48 * 18 and arrs[4].size == 1536 * 280 * 18
    lib = _load(REF_LAYER_SO)
    fn = lib.ref_decoder_layer
    if fn.argtypes is None:
        _vp = ctypes.c_void_p
        fn.argtypes = [_fp, _vp, _fp, _vp, _fp, _vp, _vp, _vp, _fp, _fp, _fp, _i, _i, _fp]
        fn.restype = _i
    f32 = lambda a: _fptr(np.ascontiguousarray(a, dtype=np.float32))
    out = np.zeros(1536, dtype=np.float32)
    rc = fn(f32(x_in), arrs[0].ctypes.data, f32(b_qkv), arrs[1].ctypes.data, f32(g_a),
            arrs[2].ctypes.data, arrs[3].ctypes.data, arrs[4].ctypes.data, f32(g_f),
            _fptr(k_cache), _fptr(v_cache), pos, seq_len, _fptr(out))
    if rc != 0:
        raise ValueError("reference rejected pos/seq_len")
    return out


def ref_gemv_q4_0(w, x, bias, M: int, K: int) -> np.ndarray:
    """The reference's own cpu_gemv_q4_0_bias (test_28_layers_real.c:90-108) at
    any size: y = W x (+ bias), W Q4_0 bytes [M][K / 32 blocks]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size == M * (K // 32) * 18
    fn = _load(REF_LAYER_SO).ref_gemv_q4_0_bias
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_void_p, _fp, _fp, _fp, _i, _i]
        fn.restype = None
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.zeros(M, dtype=np.float32)
    fn(w.ctypes.data, _fptr(x), None if b is None else _fptr(b), _fptr(y), M, K)
    return y


def ref_swiglu(w_gate, w_up, x, M: int, K: int) -> np.ndarray:
    """The reference's own cpu_swiglu_fused (test_28_layers_real.c:110-131):
    h = silu(W_gate x) * (W_up x) with its stable SiLU."""
    wg = np.ascontiguousarray(w_gate, dtype=np.uint8)
    wu = np.ascontiguousarray(w_up, dtype=np.uint8)
    assert wg.size == wu.size == M * (K // 32) * 18
    fn = _load(REF_LAYER_SO).ref_swiglu_fused
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _fp, _fp, _i, _i]
        fn.restype = None
    x = np.ascontiguousarray(x, dtype=np.float32)
    h = np.zeros(M, dtype=np.float32)
    fn(wg.ctypes.data, wu.ctypes.data, _fptr(x), _fptr(h), M, K)
    return h


def decoder_layer_sized(x_in, attn, ffn, k_cache, v_cache, pos: int, seq_len: int,
                        n_heads_q: int, n_heads_kv: int, head_dim: int, d_ffn: int) -> np.ndarray:
    """One decoder layer at any size, in the order of cpu_decoder_layer_step
    (test_28_layers_real.c:192-318) and of the 0.5B generator's layer step
    (generate_stream_05b.c:364-476): RMSNorm, the reference's compiled Q4_0
    GEMV + bias, RoPE + append + attention (the shape-generic restatement),
    W_o GEMV + residual, RMSNorm, the reference's compiled fused SwiGLU GEMV,
    down GEMV + residual.  At the 1.5B sizes it equals the compiled
    cpu_decoder_layer_step (checked by the CPU tests).  Caches are updated in
    place at row pos."""
    w_qkv, b_qkv, w_o, g_a = attn
    w_gate, w_up, w_down, g_f = ffn
    d_model = n_heads_q * head_dim
    d_qkv = d_model + 2 * n_heads_kv * head_dim
    x = np.ascontiguousarray(x_in, dtype=np.float32)
    z1 = output_norm(x, g_a)
    qkv = ref_gemv_q4_0(w_qkv, z1, b_qkv, d_qkv, d_model)
    layer_attention(qkv, k_cache, v_cache, pos, seq_len, n_heads_q, n_heads_kv,
                    head_dim=head_dim)
    r = ref_gemv_q4_0(w_o, qkv[:d_model], None, d_model, d_model)
    r = (r + x).astype(np.float32)
    z2 = output_norm(r, g_f)
    h = ref_swiglu(w_gate, w_up, z2, d_ffn, d_model)
    y = ref_gemv_q4_0(w_down, h, None, d_model, d_ffn)
    return (y + r).astype(np.float32)


# ---- around the decoder layers: embedding, output norm, LM head, pick -------

Q6_K_ROW_BYTES = 1260  # 6 superblocks of 210 bytes per 1536-wide row
D05B_MODEL, D05B_FFN = 896, 4864  # Qwen2.5-0.5B (generate_stream_05b.c:22-26)


def token_embedding(table: np.ndarray, token: int, d_model: int = 1536) -> np.ndarray:
    """get_token_embedding (qwen_server.c:188-201), restated in gqa_oracle.c."""
    table = np.ascontiguousarray(table, dtype=np.uint8)
    assert 0 <= token and (token + 1) * (d_model // 32) * 18 <= table.size
    fn = _lib().oracle_token_embedding
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_void_p, _i, _i, _fp]
        fn.restype = None
    out = np.zeros(d_model, dtype=np.float32)
    fn(table.ctypes.data, d_model, token, _fptr(out))
    return out


def output_norm(x: np.ndarray, gamma: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """The output RMSNorm of test_full_model_logits.c:944-948 (restated)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32)
    fn = _lib().oracle_output_norm
    if fn.argtypes is None:
        fn.argtypes = [_fp, _fp, _i, _f, _fp]
        fn.restype = None
    out = np.zeros_like(x)
    fn(_fptr(x), _fptr(gamma), x.size, eps, _fptr(out))
    return out


def greedy_pick(logits: np.ndarray) -> int:
    """The server's host argmax (qwen_server.c:998-1005, restated)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    fn = _lib().oracle_greedy_pick
    if fn.argtypes is None:
        fn.argtypes = [_fp, _i]
        fn.restype = _i
    return int(fn(_fptr(logits), logits.size))


def gemv_q8_0(w: np.ndarray, x: np.ndarray, n_rows: int, k: int = 896) -> np.ndarray:
    """The 0.5B model's Q8_0 LM head GEMV (kernel_q8_0.cl:10-61), restated in
    gqa_oracle.c with the kernel's lane sums and reduction tree."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size >= n_rows * (k // 32) * 34
    fn = _lib().oracle_gemv_q8_0
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_void_p, _fp, _i, _i, _fp]
        fn.restype = None
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(n_rows, dtype=np.float32)
    fn(w.ctypes.data, _fptr(x), n_rows, k, _fptr(y))
    return y


def have_reference_q8() -> bool:
    return os.path.exists(REF_Q8_SO)


def ref_gemv_q8_0(w: np.ndarray, x: np.ndarray, n_rows: int, k: int = 896) -> np.ndarray:
    """The reference's own gemv_q8_0 (kernel_q8_0.cl:10-61): its OpenCL C
    compiled as C, every 128-work-item group run by a coroutine scheduler
    (oracle/ref_q8_harness.c).  Slow (one context switch per work-item per
    barrier): for a few thousand rows at most."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size >= n_rows * (k // 32) * 34 and k == 896
    lib = _load(REF_Q8_SO)
    fn = lib.ref_gemv_q8_0
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_void_p, _fp, _fp, _i, _i]
        fn.restype = _i
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(n_rows, dtype=np.float32)
    if fn(w.ctypes.data, _fptr(x), _fptr(y), n_rows, k) != 0:
        raise RuntimeError("ref_gemv_q8_0: coroutine set-up failed")
    return y


def lm_head_q8_0(state, gamma, w, n_rows: int):
    """(logits, pick) of the 0.5B generator's step end (generate_stream_05b.c:
    845-878): output RMSNorm, the Q8_0 GEMV, the host argmax."""
    z = output_norm(state, gamma)
    logits = gemv_q8_0(w, z, n_rows, z.size)
    return logits, greedy_pick(logits)


def ref_token_embedding(table: np.ndarray, token: int) -> np.ndarray:
    """The reference's own get_token_embedding on a Q4_0 table."""
    table = np.ascontiguousarray(table, dtype=np.uint8).reshape(-1)
    lib = _load(REF_MODEL_SO)
    fn = lib.ref_token_embedding
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, _i, _fp]
        fn.restype = _i
    out = np.zeros(1536, dtype=np.float32)
    rc = fn(table.ctypes.data, table.size, token, _fptr(out))
    if rc != 0:
        raise ValueError(f"reference embedding lookup failed ({rc})")
    return out


def _head_lib():
    lib = _load(REF_HEAD_SO)
    if lib.ref_gemv_q6_k.argtypes is None:
        lib.ref_gemv_q6_k.argtypes = [ctypes.c_void_p, _fp, _fp, _i]
        lib.ref_gemv_q6_k.restype = None
        lib.ref_dequant_q6_k.argtypes = [ctypes.c_void_p, _fp]
        lib.ref_dequant_q6_k.restype = None
    return lib


def ref_gemv_q6_k(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """The reference's cpu_gemv_q6_k_ref: y[r] = dequant(row r) . x in fp32,
    rows of 1260 bytes (GGUF order)."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    assert w.size % Q6_K_ROW_BYTES == 0
    m = w.size // Q6_K_ROW_BYTES
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.size == 1536
    y = np.zeros(m, dtype=np.float32)
    _head_lib().ref_gemv_q6_k(w.ctypes.data, _fptr(x), _fptr(y), m)
    return y


def ref_dequant_q6_k(row: np.ndarray) -> np.ndarray:
    """dequantize_row_q6_k_ref of one 1260-byte row (1536 floats)."""
    row = np.ascontiguousarray(row, dtype=np.uint8).reshape(-1)
    assert row.size == Q6_K_ROW_BYTES
    y = np.zeros(1536, dtype=np.float32)
    _head_lib().ref_dequant_q6_k(row.ctypes.data, _fptr(y))
    return y


def ref_lm_head(state: np.ndarray, gamma: np.ndarray, w: np.ndarray):
    """Output norm + the reference's Q6_K GEMV + greedy pick: (logits, token)."""
    logits = ref_gemv_q6_k(w, output_norm(state, gamma))
    return logits, greedy_pick(logits)


def ref_decode_token(table, layers, kv, gamma_out, w_head, token: int, pos: int,
                     model: str = "1.5b"):
    """One greedy step of the whole model on the CPU: embedding of `token`,
    the decoder layer for every layer (layers[l] = (attn, ffn), kv[l] =
    (k_cache, v_cache) updated in place at row pos), output norm, head, pick.
    model "1.5b": the compiled cpu_decoder_layer_step and Q6_K GEMV; "0.5b":
    decoder_layer_sized at the Qwen2.5-0.5B sizes and the Q8_0 head
    (generate_stream_05b.c:836-878).  Returns (logits, next token)."""
    if model == "0.5b":
        x = token_embedding(table, token, D05B_MODEL)
        for (attn, ffn), (kc, vc) in zip(layers, kv):
            x = decoder_layer_sized(x, attn, ffn, kc, vc, pos, pos + 1, 14, 2, 64, D05B_FFN)
        return lm_head_q8_0(x, gamma_out, w_head, len(w_head) // (D05B_MODEL // 32 * 34))
    x = token_embedding(table, token)
    for (attn, ffn), (kc, vc) in zip(layers, kv):
        x = ref_decoder_layer(x, attn, ffn, kc, vc, pos, pos + 1)
    return ref_lm_head(x, gamma_out, w_head)


# ---- the server: GGUF reading (compiled) and its request loop (restated) -----

def ref_gguf_parse(path: str, max_tensors: int = 4096):
    """The reference's parse_gguf_tensors on a file: (tensors, data_start) with
    tensors = [{"name", "n_dims", "ne", "type", "offset"}] (absolute offsets)."""
    lib = _load(REF_SERVER_SO)
    fn = lib.ref_gguf_parse
    if fn.argtypes is None:
        _u32p = ctypes.POINTER(ctypes.c_uint32)
        _u64p = ctypes.POINTER(ctypes.c_uint64)
        fn.argtypes = [ctypes.c_char_p, _i, ctypes.c_char_p, _u32p, _u64p, _u32p, _u64p, _u64p]
        fn.restype = _i
    names = ctypes.create_string_buffer(64 * max_tensors)
    n_dims = (ctypes.c_uint32 * max_tensors)()
    ne = (ctypes.c_uint64 * (4 * max_tensors))()
    types = (ctypes.c_uint32 * max_tensors)()
    offs = (ctypes.c_uint64 * max_tensors)()
    start = ctypes.c_uint64()
    n = fn(str(path).encode(), max_tensors, names, n_dims, ne, types, offs, ctypes.byref(start))
    if n < 0:
        raise ValueError(f"reference parser failed ({n})")
    out = []
    for i in range(n):
        raw = names.raw[64 * i:64 * i + 64]
        out.append({"name": raw.split(b"\0", 1)[0].decode(), "n_dims": n_dims[i],
                    "ne": [ne[4 * i + d] for d in range(n_dims[i])], "type": types[i],
                    "offset": offs[i]})
    return out, start.value


def ref_gguf_token(path: str, token: int) -> bytes:
    """The reference's load_tokenizer_tokens, one entry."""
    lib = _load(REF_SERVER_SO)
    fn = lib.ref_gguf_token
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_char_p, _i, ctypes.c_char_p, _i]
        fn.restype = _i
    buf = ctypes.create_string_buffer(1024)
    rc = fn(str(path).encode(), token, buf, len(buf))
    if rc < 0:
        raise ValueError(f"reference tokenizer read failed ({rc})")
    return buf.value


def ref_server_query(table, layers, kv, gamma_out, w_head, tokens, cur_pos: int, max_new: int,
                     eog=(151643, 151645), t_max: int = REF_T_MAX, margins=None,
                     model: str = "1.5b"):
    """The server's QUERY loop (qwen_server.c:957-1049), restated over the
    compiled pieces: every prompt token through the layers at cur_pos + p (the
    head only after the last), then greedy picks -- stop before an
    end-of-generation id, emit, stop at max_new or t_max, else run the pick
    through the layers and the head.  kv[l] = (k_cache, v_cache) updated in
    place.  Returns the emitted ids; `margins`, when a list, receives the gap
    between the two largest logits of every pick.  model "0.5b" runs the same
    loop over the Qwen2.5-0.5B pieces (ref_decode_token)."""
    logits = None
    for p, tok in enumerate(tokens):
        if p == len(tokens) - 1:
            logits, _ = ref_decode_token(table, layers, kv, gamma_out, w_head, tok, cur_pos + p,
                                         model)
        elif model == "0.5b":
            x = token_embedding(table, tok, D05B_MODEL)
            for (attn, ffn), (kc, vc) in zip(layers, kv):
                x = decoder_layer_sized(x, attn, ffn, kc, vc, cur_pos + p, cur_pos + p + 1, 14, 2,
                                        64, D05B_FFN)
        else:
            x = token_embedding(table, tok)
            for (attn, ffn), (kc, vc) in zip(layers, kv):
                x = ref_decoder_layer(x, attn, ffn, kc, vc, cur_pos + p, cur_pos + p + 1)
    out = []
    next_pos = cur_pos + len(tokens)
    for gen in range(max_new):
        best = greedy_pick(logits)
        if margins is not None:  # gap between the two largest logits of each pick
            top = np.sort(logits)[-2:]
            margins.append(float(top[1] - top[0]))
        if best in eog:
            break
        out.append(best)
        if gen + 1 >= max_new or next_pos >= t_max:
            break
        logits, _ = ref_decode_token(table, layers, kv, gamma_out, w_head, best, next_pos, model)
        next_pos += 1
    return out


def ref_server_set_base(table, layers, kv, tokens):
    """SET_BASE (qwen_server.c:815-860): the tokens through the layers at
    positions 0 .. n-1; returns the FNV-1a hash of the ids."""
    h = 14695981039346656037
    for p, tok in enumerate(tokens):
        h ^= tok
        h = (h * 1099511628211) & ((1 << 64) - 1)
        x = token_embedding(table, tok)
        for (attn, ffn), (kc, vc) in zip(layers, kv):
            x = ref_decoder_layer(x, attn, ffn, kc, vc, p, p + 1)
    return h
