"""Seeded synthetic inputs shared by the tests, the fixtures and the bench.

Every tensor is drawn from a named stream of one 64-bit seed: element ``e`` of
stream ``(seed, stream_id)`` is one half of the Box-Muller pair ``e // 2``
whose two uniforms are the splitmix64 outputs number ``e - e % 2`` and
``e - e % 2 + 1`` of the stream key (splitmix64: Steele, Lea, Flood, "Fast
splittable pseudorandom number generators", OOPSLA 2014; Box-Muller in double
precision, then rounded to fp32).  Being counter-based, any slice can be
generated on its own; ``gqa_fill_normal`` in the library produces the same
streams on the device.

The reference seeds glibc ``rand()`` with 42 and draws uniform values
(compute/attention-gqa-resident/attention_gqa_benchmark.c:350-369); the
workloads here ask for N(0, 1) q/k/v and caches instead, so the generator is
our own.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_STREAM_MUL = 0xD1B54A32D192ED03
_MASK = (1 << 64) - 1

# Stream ids used across tests and the bench, so that the same seed names the
# same tensor everywhere.
QKV, K_CACHE, V_CACHE, LENGTHS, PREFILL_Q, PREFILL_K, PREFILL_V = 1, 2, 3, 4, 5, 6, 7
W_QKV, B_QKV, W_O, GAMMA, STATE = 8, 9, 10, 11, 12
W_GATE, W_UP, W_DOWN, GAMMA_FFN = 13, 14, 15, 16
W_HEAD, GAMMA_OUT, TOKEN_EMBD, HEAD_X = 17, 18, 19, 20

Q4_0_BLOCK_BYTES = 18
Q6_K_BLOCK_BYTES = 210
Q8_0_BLOCK_BYTES = 34


def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _mix_int(z: int) -> int:
    z &= _MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK
    return z ^ (z >> 31)


def stream_key(seed: int, stream_id: int) -> int:
    """Key of stream ``stream_id`` of ``seed`` (same formula as gqa_fill_normal)."""
    return _mix_int((seed & _MASK) ^ ((stream_id * _STREAM_MUL) & _MASK))


def uniform_u64(seed: int, stream_id: int, n: int, offset: int = 0) -> np.ndarray:
    """splitmix64 outputs number offset .. offset+n-1 of the stream."""
    key = np.uint64(stream_key(seed, stream_id))
    idx = np.arange(offset, offset + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix(key + (idx + np.uint64(1)) * _GOLDEN)


def normal(seed: int, stream_id: int, n: int, offset: int = 0) -> np.ndarray:
    """fp32 N(0, 1) values number offset .. offset+n-1 of the stream."""
    if n <= 0:
        return np.zeros(0, dtype=np.float32)
    first_pair = offset // 2
    last_pair = (offset + n - 1) // 2
    n_pairs = last_pair - first_pair + 1
    r = uniform_u64(seed, stream_id, 2 * n_pairs, 2 * first_pair)
    r1 = r[0::2]
    r2 = r[1::2]
    u1 = ((r1 >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u2 = (r2 >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    rad = np.sqrt(-2.0 * np.log(u1))
    ang = 6.283185307179586 * u2
    out = np.empty(2 * n_pairs, dtype=np.float64)
    out[0::2] = rad * np.cos(ang)
    out[1::2] = rad * np.sin(ang)
    start = offset - 2 * first_pair
    return out[start:start + n].astype(np.float32)


def uniform_int(seed: int, stream_id: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive), by 128-bit multiply-shift."""
    r = uniform_u64(seed, stream_id, n)
    span = hi - lo + 1
    return np.array([lo + ((int(x) * span) >> 64) for x in r], dtype=np.int64)


def grid_uniform(seed: int, stream_id: int, n: int) -> np.ndarray:
    """Values on the grid {-1.00, -0.99, ..., 0.99}: the distribution of the
    reference benchmark's cache contents (attention_gqa_benchmark.c:366-369),
    drawn from our own generator instead of glibc rand()."""
    r = uniform_u64(seed, stream_id, n)
    return ((r % np.uint64(200)).astype(np.int64) - 100).astype(np.float32) * np.float32(0.01)


def decode_inputs(seed: int, t_max: int = 4096, n_heads_q: int = 12, n_heads_kv: int = 2,
                  dist: str = "normal"):
    """(qkv [n_q*128 + 2*n_kv*128], k_cache, v_cache [n_kv][t_max][128]) for one
    layer of one sequence.  dist "normal": everything N(0,1); "grid": q/k/v
    N(0,1) and the caches on the reference benchmark's uniform grid."""
    n_qkv = (n_heads_q + 2 * n_heads_kv) * 128
    qkv = normal(seed, QKV, n_qkv)
    n = n_heads_kv * t_max * 128
    if dist == "normal":
        kc = normal(seed, K_CACHE, n)
        vc = normal(seed, V_CACHE, n)
    elif dist == "grid":
        kc = grid_uniform(seed, K_CACHE, n)
        vc = grid_uniform(seed, V_CACHE, n)
    else:
        raise ValueError(dist)
    return qkv, kc.reshape(n_heads_kv, t_max, 128), vc.reshape(n_heads_kv, t_max, 128)


def q4_0_matrix(seed: int, stream_id: int, rows: int, cols: int, scale: float) -> np.ndarray:
    """A Q4_0 matrix [rows][cols / 32 blocks] as bytes (the reference's
    block_q4_0: little-endian fp16 scale, then 16 bytes of 4-bit codes).
    Block b takes splitmix64 outputs 3b .. 3b+2 of the stream: the first sets
    d = scale * (0.5 + u), u uniform in [0, 1), the other two are the codes."""
    nb = rows * (cols // 32)
    u = uniform_u64(seed, stream_id, 3 * nb)
    frac = (u[0::3] >> np.uint64(11)).astype(np.float64) / float(1 << 53)
    d = (scale * (0.5 + frac)).astype(np.float16)
    out = np.empty((nb, Q4_0_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = np.stack([u[1::3], u[2::3]], axis=1).astype("<u8").view(np.uint8).reshape(nb, 16)
    return out.reshape(-1)


def q4_0_dequant(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Dense float32 [rows][cols] of a Q4_0 byte matrix (w = d * (code - 8))."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(rows * (cols // 32), Q4_0_BLOCK_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].astype(np.int32)
    w = np.concatenate([(q & 15) - 8, (q >> 4) - 8], axis=1).astype(np.float32) * d
    return w.reshape(rows, cols)


def q6_k_matrix(seed: int, stream_id: int, rows: int, cols: int = 1536,
                scale: float = 2.0 ** -12) -> np.ndarray:
    """A Q6_K matrix [rows][cols / 256 superblocks] as bytes (the reference's
    block_q6_K: ql[128], qh[64], int8 scales[16], little-endian fp16 d).
    Superblock s takes splitmix64 outputs 27s .. 27s+26: the first 26 give
    bytes 0..207 (codes and scales, uniform), the last d = scale * (0.5 + u),
    u uniform in [0, 1).  With the default scale, d stays a normal fp16 and
    rows dotted with a unit-RMS input give logits of about 13 RMS."""
    nb = rows * (cols // 256)
    u = uniform_u64(seed, stream_id, 27 * nb).reshape(nb, 27)
    out = np.empty((nb, Q6_K_BLOCK_BYTES), dtype=np.uint8)
    out[:, :208] = np.ascontiguousarray(u[:, :26]).astype("<u8").view(np.uint8).reshape(nb, 208)
    frac = (u[:, 26] >> np.uint64(11)).astype(np.float64) / float(1 << 53)
    d = (scale * (0.5 + frac)).astype(np.float16)
    out[:, 208:] = d.view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def q6_k_dequant(blocks: np.ndarray, rows: int, cols: int = 1536) -> np.ndarray:
    """Dense float32 [rows][cols] of a Q6_K byte matrix, in the reference's
    arithmetic: weight (n, c, l) of a superblock = (d * scales[8n + 2c + l/16])
    * (code - 32), code = ((ql[64n + 32(c & 1) + l] >> 4(c >> 1)) & 15)
    | ((qh[32n + l] >> 2c) & 3) << 4 (test_gemv_q6_k.c:46-74)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(rows * (cols // 256), Q6_K_BLOCK_BYTES)
    ql = b[:, :128].astype(np.int32)
    qh = b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
    y = np.empty((b.shape[0], 256), dtype=np.float32)
    l = np.arange(32)
    for n in range(2):
        for c in range(4):
            lo = (ql[:, 64 * n + 32 * (c & 1) + l] >> (4 * (c >> 1))) & 15
            hi = (qh[:, 32 * n + l] >> (2 * c)) & 3
            code = (lo | (hi << 4)) - 32
            ds = d[:, None] * sc[:, 8 * n + 2 * c + l // 16]
            y[:, 128 * n + 32 * c + l] = ds * code.astype(np.float32)
    return y.reshape(rows, cols)


def q6_k_planes(blocks: np.ndarray, rows: int) -> np.ndarray:
    """The byte layout gqa_lm_head_pack writes, over the rows rounded up to a
    multiple of 4 (padding rows zero): ql [Np][768], qh [Np][384], scales
    [Np][96], d [Np][12], each row the concatenation of its six superblocks'
    bytes of that kind in their own order, except that row r's ql and qh rows
    are rotated right by 16 * (r % 8) bytes (byte i of the row is stored at
    (i + 16 (r % 8)) mod the row length), so that eight consecutive rows read
    at one offset fall on different shared-memory banks."""
    np_rows = (rows + 3) // 4 * 4
    b = np.zeros((np_rows, 6, Q6_K_BLOCK_BYTES), dtype=np.uint8)
    b[:rows] = np.asarray(blocks, dtype=np.uint8).reshape(rows, 6, Q6_K_BLOCK_BYTES)
    ql = np.ascontiguousarray(b[:, :, :128]).reshape(np_rows, 768)
    qh = np.ascontiguousarray(b[:, :, 128:192]).reshape(np_rows, 384)
    for r in range(min(np_rows, 8)):
        sel = np.arange(r, np_rows, 8)
        ql[sel] = np.roll(ql[sel], 16 * r, axis=1)
        qh[sel] = np.roll(qh[sel], 16 * r, axis=1)
    sc = np.ascontiguousarray(b[:, :, 192:208]).reshape(np_rows, 96)
    dd = np.ascontiguousarray(b[:, :, 208:]).reshape(np_rows, 12)
    return np.concatenate([ql.reshape(-1), qh.reshape(-1), sc.reshape(-1), dd.reshape(-1)])


def q8_0_matrix(seed: int, stream_id: int, rows: int, cols: int = 896,
                scale: float = 2.0 ** -8) -> np.ndarray:
    """A Q8_0 matrix [rows][cols / 32 blocks] as bytes (the reference's
    block_q8_0, generate_stream_05b.c:42-45: little-endian fp16 d, then 32
    int8 codes).  Block b takes splitmix64 outputs 5b .. 5b+4 of the stream:
    the first sets d = scale * (0.5 + u), u uniform in [0, 1), the other four
    are the codes.  With the default scale, rows dotted with a unit-RMS input
    give logits of about 8 RMS."""
    nb = rows * (cols // 32)
    u = uniform_u64(seed, stream_id, 5 * nb).reshape(nb, 5)
    frac = (u[:, 0] >> np.uint64(11)).astype(np.float64) / float(1 << 53)
    d = (scale * (0.5 + frac)).astype(np.float16)
    out = np.empty((nb, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = np.ascontiguousarray(u[:, 1:]).astype("<u8").view(np.uint8).reshape(nb, 32)
    return out.reshape(-1)


def q8_0_dequant(blocks: np.ndarray, rows: int, cols: int = 896) -> np.ndarray:
    """Dense float32 [rows][cols] of a Q8_0 byte matrix (w = d * q)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(rows * (cols // 32), Q8_0_BLOCK_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, cols)


def q8_0_planes(blocks: np.ndarray, rows: int) -> np.ndarray:
    """The byte layout gqa_lm_head_q8_0_pack writes for 896-wide rows, over the
    rows rounded up to a multiple of 4: codes [Np][896] then scales [Np][28]
    (fp16).  In a row, the int8 codes of block b = li + 14 s (li < 14, s < 2),
    16 at a time (half mq < 2), sit at byte 16 ((2s + mq) 14 + li); padding rows
    hold code 0 and scale 0."""
    np_rows = (rows + 3) // 4 * 4
    b = np.zeros((np_rows, 28, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    b[:rows] = np.asarray(blocks, dtype=np.uint8).reshape(rows, 28, Q8_0_BLOCK_BYTES)
    q = b[:, :, 2:]                                            # [row][b][32]
    q = q.reshape(np_rows, 2, 14, 2, 16).transpose(0, 1, 3, 2, 4)  # [row][s][mq][li][16]
    return np.concatenate([np.ascontiguousarray(q).reshape(-1), b[:, :, 0:2].reshape(-1)])


def head_inputs(seed: int, vocab: int = 151936, d_model: int = 1536):
    """(w_head Q6_K bytes, gamma_out, token_embd Q4_0 bytes) of the model's
    ends: gamma_out ~ 1 + N(0, 0.1^2); embedding rows of unit RMS."""
    w_head = q6_k_matrix(seed, W_HEAD, vocab, d_model)
    gamma = (1.0 + 0.1 * normal(seed, GAMMA_OUT, d_model)).astype(np.float32)
    embd = q4_0_matrix(seed, TOKEN_EMBD, vocab, d_model, 1.0 / 4.6)
    return w_head, gamma, embd


def head_q8_inputs(seed: int, vocab: int = 151936, d_model: int = 896):
    """(w_head Q8_0 bytes, gamma_out, token_embd Q4_0 bytes) of the 0.5B
    model's ends, drawn from the same streams as head_inputs."""
    w_head = q8_0_matrix(seed, W_HEAD, vocab, d_model)
    gamma = (1.0 + 0.1 * normal(seed, GAMMA_OUT, d_model)).astype(np.float32)
    embd = q4_0_matrix(seed, TOKEN_EMBD, vocab, d_model, 1.0 / 4.6)
    return w_head, gamma, embd


def attention_block_inputs(seed: int, t_max: int = 4096, d_model: int = 1536, n_heads_kv: int = 2,
                           head_dim: int = 128):
    """(state, w_qkv, b_qkv, w_o, gamma, k_cache, v_cache) of one layer's
    attention block: state, caches N(0, 1); Q4_0 weights scaled so each
    projection has unit-RMS rows; b_qkv ~ N(0, 0.1^2); gamma ~ 1 + N(0, 0.1^2)."""
    n_qkv = d_model + 2 * n_heads_kv * head_dim
    scale = 1.0 / (4.6 * np.sqrt(d_model))  # RMS of (code - 8) is ~4.6
    state = normal(seed, STATE, d_model)
    w_qkv = q4_0_matrix(seed, W_QKV, n_qkv, d_model, scale)
    b_qkv = (0.1 * normal(seed, B_QKV, n_qkv)).astype(np.float32)
    w_o = q4_0_matrix(seed, W_O, d_model, d_model, scale)
    gamma = (1.0 + 0.1 * normal(seed, GAMMA, d_model)).astype(np.float32)
    n = n_heads_kv * t_max * head_dim
    kc = normal(seed, K_CACHE, n).reshape(n_heads_kv, t_max, head_dim)
    vc = normal(seed, V_CACHE, n).reshape(n_heads_kv, t_max, head_dim)
    return state, w_qkv, b_qkv, w_o, gamma, kc, vc


def ffn_block_inputs(seed: int, d_model: int = 1536, d_ffn: int = 8960):
    """(w_gate, w_up, w_down, gamma_ffn) of one layer's FFN: Q4_0 weights
    scaled for unit-RMS projection rows; gamma ~ 1 + N(0, 0.1^2)."""
    s_in = 1.0 / (4.6 * np.sqrt(d_model))
    s_down = 1.0 / (4.6 * np.sqrt(d_ffn))
    w_gate = q4_0_matrix(seed, W_GATE, d_ffn, d_model, s_in)
    w_up = q4_0_matrix(seed, W_UP, d_ffn, d_model, s_in)
    w_down = q4_0_matrix(seed, W_DOWN, d_model, d_ffn, s_down)
    gamma = (1.0 + 0.1 * normal(seed, GAMMA_FFN, d_model)).astype(np.float32)
    return w_gate, w_up, w_down, gamma
