"""Writes GGUF files for the tests (test infrastructure).

The GGUF layout as the reference reads it (qwen_server.c:113-178,
:203-266): magic "GGUF", version, tensor count, key-value count; each key a
length-prefixed string, a value type and the value (scalars, strings,
arrays); each tensor info its name, dimension count, dimensions (innermost
first), type and data offset; the data section starts at the next multiple
of the alignment (general.alignment, 32 by default) and every tensor's data
at a multiple of it too.
"""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}
T_F32, T_F16, T_Q4_0, T_Q8_0, T_Q6_K = 0, 1, 2, 8, 14


def _s(b: bytes | str) -> bytes:
    if isinstance(b, str):
        b = b.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vt: int, v) -> bytes:
    if vt in _SCALAR:
        return struct.pack(_SCALAR[vt], v)
    if vt == STR:
        return _s(v)
    if vt == ARR:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_value(et, x) for x in items)
    raise ValueError(vt)


def write(path, metadata, tensors, alignment: int = 32, version: int = 3,
          honour_alignment_key: bool = True) -> dict:
    """metadata: [(key, value_type, value)]; tensors: [(name, type, ne, bytes)].
    Returns {name: absolute data offset}.  With honour_alignment_key False, a
    general.alignment entry is written but the data is laid out on 32."""
    align = alignment if honour_alignment_key else 32
    tensors = [(n, t, ne, np.ascontiguousarray(d).tobytes() if isinstance(d, np.ndarray)
                else bytes(d)) for n, t, ne, d in tensors]
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata))
    for key, vt, v in metadata:
        head += _s(key) + struct.pack("<I", vt) + _value(vt, v)
    rel, offsets = 0, []
    for name, tt, ne, data in tensors:
        offsets.append(rel)
        rel += len(data)
        rel = (rel + align - 1) // align * align
    for (name, tt, ne, data), off in zip(tensors, offsets):
        head += _s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", n) for n in ne)
        head += struct.pack("<IQ", tt, off)
    start = (len(head) + align - 1) // align * align
    with open(path, "wb") as f:
        f.write(head + b"\0" * (start - len(head)))
        for (name, tt, ne, data), off in zip(tensors, offsets):
            f.seek(start + off)
            f.write(data)
        f.truncate(start + rel)
    return {name: start + off for (name, _, _, _), off in zip(tensors, offsets)}


def qwen_model(path, seeded, n_layers: int, vocab: int, seed: int, tokens=None,
               model: str = "1.5b"):
    """A Qwen2.5-1.5B-shaped GGUF (Q4_0 projections and embedding, Q6_K head,
    F32 norms and biases) with seeded weights, and the same weights as arrays:
    (offsets, {"embd", "head", "gamma_out", "layers": [((w_qkv, b_qkv, w_o, g_attn),
    (w_gate, w_up, w_down, g_ffn))]}).  model "0.5b": the Qwen2.5-0.5B sizes
    (d_model 896, 14 / 2 heads of 64, d_ffn 4864) with a Q8_0 head, the tensors
    generate_stream_05b.c:553-615 reads."""
    small = model == "0.5b"
    d, dkv, dffn = (896, 128, 4864) if small else (1536, 256, 8960)
    s_in = 1.0 / (4.6 * np.sqrt(d))
    s_down = 1.0 / (4.6 * np.sqrt(dffn))
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32).tobytes()
    embd = seeded.q4_0_matrix(seed, seeded.TOKEN_EMBD, vocab, d, 1.0 / 4.6)
    head = (seeded.q8_0_matrix(seed, seeded.W_HEAD, vocab, d) if small
            else seeded.q6_k_matrix(seed, seeded.W_HEAD, vocab, d))
    gamma_out = (1.0 + 0.1 * seeded.normal(seed, seeded.GAMMA_OUT, d)).astype(np.float32)
    tensors = [("token_embd.weight", T_Q4_0, [d, vocab], embd),
               ("output_norm.weight", T_F32, [d], f32(gamma_out)),
               ("output.weight", T_Q8_0 if small else T_Q6_K, [d, vocab], head)]
    layers = []
    for l in range(n_layers):
        ls = seed * 100 + l
        w_qkv = seeded.q4_0_matrix(ls, seeded.W_QKV, d + 2 * dkv, d, s_in)
        b_qkv = (0.1 * seeded.normal(ls, seeded.B_QKV, d + 2 * dkv)).astype(np.float32)
        w_o = seeded.q4_0_matrix(ls, seeded.W_O, d, d, s_in)
        g_attn = (1.0 + 0.1 * seeded.normal(ls, seeded.GAMMA, d)).astype(np.float32)
        w_gate = seeded.q4_0_matrix(ls, seeded.W_GATE, dffn, d, s_in)
        w_up = seeded.q4_0_matrix(ls, seeded.W_UP, dffn, d, s_in)
        w_down = seeded.q4_0_matrix(ls, seeded.W_DOWN, d, dffn, s_down)
        g_ffn = (1.0 + 0.1 * seeded.normal(ls, seeded.GAMMA_FFN, d)).astype(np.float32)
        row = (d // 32) * 18
        b = f"blk.{l}."
        tensors += [(b + "attn_norm.weight", T_F32, [d], f32(g_attn)),
                    (b + "attn_q.weight", T_Q4_0, [d, d], w_qkv[:d * row]),
                    (b + "attn_k.weight", T_Q4_0, [d, dkv], w_qkv[d * row:(d + dkv) * row]),
                    (b + "attn_v.weight", T_Q4_0, [d, dkv], w_qkv[(d + dkv) * row:]),
                    (b + "attn_q.bias", T_F32, [d], f32(b_qkv[:d])),
                    (b + "attn_k.bias", T_F32, [dkv], f32(b_qkv[d:d + dkv])),
                    (b + "attn_v.bias", T_F32, [dkv], f32(b_qkv[d + dkv:])),
                    (b + "attn_output.weight", T_Q4_0, [d, d], w_o),
                    (b + "ffn_norm.weight", T_F32, [d], f32(g_ffn)),
                    (b + "ffn_gate.weight", T_Q4_0, [d, dffn], w_gate),
                    (b + "ffn_up.weight", T_Q4_0, [d, dffn], w_up),
                    (b + "ffn_down.weight", T_Q4_0, [dffn, d], w_down)]
        layers.append(((w_qkv, b_qkv, w_o, g_attn), (w_gate, w_up, w_down, g_ffn)))
    meta = [("general.architecture", STR, "qwen2"), ("qwen2.block_count", U32, n_layers),
            ("qwen2.embedding_length", U32, d),
            ("qwen2.attention.head_count", U32, 14 if small else 12),
            ("qwen2.attention.head_count_kv", U32, 2), ("qwen2.rope.freq_base", F32, 1e6),
            ("tokenizer.ggml.tokens", ARR,
             (STR, tokens if tokens is not None else [f"t{i}" for i in range(vocab)]))]
    offsets = write(path, meta, tensors)
    return offsets, {"embd": embd, "head": head, "gamma_out": gamma_out, "layers": layers}
