"""ctypes binding of the C ABI declared in include/gqa.h.

This is the host-side mirror of the reference's layer-call API for the
attention slice: ``Context.layer_attention(kv, qkv, pos, seq_len)`` has the
argument meaning of gpu_decoder_layer_step (qwen_server.c:344-455, attention
launches :446-450) -- q/k/v of the new token in, KV cache appended at ``pos``,
attention over ``seq_len`` rows, ``attn_out`` written over ``qkv[0:1536]``.
Where the reference exits on a failed OpenCL call (CHECK_CL, qwen_server.c:53-58),
every call here raises :class:`GqaError` carrying the library's status code
and message; the process keeps running.

Device memory, streams and pinned host buffers are plain pointers; torch
tensors are accepted wherever a pointer is expected (their ``data_ptr()``) and
torch's current stream is used when no stream is given.  There is no CPU
fallback: if the CUDA library is not built, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# GQA_LIB selects another build of the library (e.g. the phase-trace build).
LIB_PATH = os.environ.get("GQA_LIB") or os.path.join(_HERE, "libgqa_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "gqa.h")

GQA_OK = 0
GQA_ERR_INVALID_ARG = -1
GQA_ERR_CUDA = -2
GQA_ERR_UNSUPPORTED = -3
GQA_ERR_DEVICE = -4
GQA_ERR_NO_MEMORY = -5
GQA_ERR_TIMEOUT = -6

GQA_OPT_PDL = 1
GQA_OPT_TARGET_CTAS = 2
GQA_OPT_BATCH_CHUNK = 3
GQA_OPT_KERNEL_VARIANT = 4
GQA_OPT_LAYERS_PDL = 5   # tuning knobs (internal): PDL inside the layer loop,
GQA_OPT_CLUSTER = 6      # the cluster reduction,
GQA_OPT_GRID_MERGE = 7   # the grid-merged single-sequence decode (default on)
GQA_OPT_BATCH_ADVANCE = 8  # batched steps advance seq_lens on the device after use
# rows per split quantum of each decode kernel variant (csrc/gqa_decode.cu)
VARIANT_QUANT = {0: 32, 1: 32, 2: 32, 3: 64, 4: 32, 5: 64, 6: 32}

STATUS_BAD_LENGTH = 1
STATUS_WAIT_TIMEOUT = 2
STATUS_BAD_TOKEN = 8

HEAD_Q6_K = 0   # gqa_model.lm_head_type: gqa_lm_head_pack layout (Qwen2.5-1.5B)
HEAD_Q8_0 = 1   # gqa_lm_head_q8_0_pack layout (Qwen2.5-0.5B)


class GqaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"gqa error {code}: {message}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [("n_heads_q", ctypes.c_int), ("n_heads_kv", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("t_max", ctypes.c_int),
                ("rope_theta", ctypes.c_float)]


class BlockWeights(ctypes.Structure):
    _fields_ = [("w_qkv", ctypes.c_void_p), ("b_qkv", ctypes.c_void_p),
                ("w_o", ctypes.c_void_p), ("gamma", ctypes.c_void_p)]


class FfnWeights(ctypes.Structure):
    _fields_ = [("w_gate", ctypes.c_void_p), ("w_up", ctypes.c_void_p),
                ("w_down", ctypes.c_void_p), ("gamma", ctypes.c_void_p)]


class LayerKV(ctypes.Structure):
    """One layer's cache: the reference's LayerKVDevice {k_cache, v_cache}."""
    _fields_ = [("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p)]


class GgufTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("n_dims", ctypes.c_int),
                ("ne", ctypes.c_longlong * 4), ("type", ctypes.c_int),
                ("offset", ctypes.c_ulonglong), ("bytes", ctypes.c_ulonglong)]


class Model(ctypes.Structure):
    """gqa_model: everything one whole-model decode step reads."""
    _fields_ = [("n_layers", ctypes.c_int), ("attn", ctypes.POINTER(BlockWeights)),
                ("ffn", ctypes.POINTER(FfnWeights)), ("kv", ctypes.POINTER(LayerKV)),
                ("token_embd", ctypes.c_void_p), ("gamma_output", ctypes.c_void_p),
                ("lm_head", ctypes.c_void_p), ("vocab", ctypes.c_int),
                ("lm_head_type", ctypes.c_int)]


_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_ull = ctypes.c_ulonglong

# name -> argtypes (restype is int unless listed in _RESTYPES)
_SIGNATURES = {
    "gqa_create": [ctypes.POINTER(Config), _i, ctypes.POINTER(_vp)],
    "gqa_destroy": [_vp],
    "gqa_last_error_string": [],
    "gqa_set_option": [_vp, _i, _ll],
    "gqa_reserve": [_vp, _i, _i],
    "gqa_device_status": [_vp, ctypes.POINTER(_i), _i],
    "gqa_kv_alloc": [_vp, _i, ctypes.POINTER(LayerKV)],
    "gqa_kv_free": [_vp, _i, ctypes.POINTER(LayerKV)],
    "gqa_layer_attention": [_vp, _vp, ctypes.POINTER(LayerKV), _vp, _i, _i],
    "gqa_layer_attention_out": [_vp, _vp, ctypes.POINTER(LayerKV), _vp, _i, _i, _vp],
    "gqa_decode_layers": [_vp, _vp, _i, ctypes.POINTER(LayerKV), _vp, _ll, _vp, _ll, _vp, _i,
                          _i, _i],
    "gqa_graph_create_layers": [_vp, _i, ctypes.POINTER(LayerKV), _vp, _ll, _vp, _ll, _vp, _i,
                                _i, _i, ctypes.POINTER(_vp)],
    "gqa_graph_launch": [_vp, _vp],
    "gqa_graph_step_host": [_vp, _vp, _vp, _vp],
    "gqa_graph_destroy": [_vp],
    "gqa_rope_kv_append": [_vp, _vp, ctypes.POINTER(LayerKV), _vp, _vp, _vp, _i],
    "gqa_decode": [_vp, _vp, ctypes.POINTER(LayerKV), _vp, _i, _vp],
    "gqa_decode_batched": [_vp, _vp, _i, _vp, _vp, _vp, _ll, _vp, _i, _vp, _ll],
    "gqa_decode_batched_host": [_vp, _vp, _i, _vp, _vp, _vp, _vp, _ll, _vp, _i, _vp, _ll, _vp],
    "gqa_decode_split_partial": [_vp, _vp, ctypes.POINTER(LayerKV), _vp, _i, _i, _vp, _vp, _vp],
    "gqa_lse_combine": [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp],
    "gqa_decode_kv_shard": [_vp, _vp, ctypes.POINTER(LayerKV), _vp, _i, _i, _i, _vp, _vp, _vp],
    "gqa_lse_combine_packed": [_vp, _vp, _i, _i, _vp, _ll, _vp],
    "gqa_attention_block": [_vp, _vp, ctypes.POINTER(BlockWeights), ctypes.POINTER(LayerKV), _vp,
                            _i, _i],
    "gqa_attention_block_layers": [_vp, _vp, _i, ctypes.POINTER(BlockWeights),
                                   ctypes.POINTER(LayerKV), _vp, _vp, _i, _i, _i],
    "gqa_ffn_block": [_vp, _vp, ctypes.POINTER(FfnWeights), _vp],
    "gqa_decoder_layers": [_vp, _vp, _i, ctypes.POINTER(BlockWeights), ctypes.POINTER(FfnWeights),
                           ctypes.POINTER(LayerKV), _vp, _vp, _i, _i, _i],
    "gqa_exchange_create": [_vp, _i, _i, ctypes.POINTER(_vp), _vp],
    "gqa_exchange_open": [_vp, _vp],
    "gqa_exchange_destroy": [_vp],
    "gqa_decode_kv_shard_exchange": [_vp, _vp, _vp, ctypes.POINTER(LayerKV), _vp, _i, _i, _i,
                                     _vp],
    "gqa_lm_head_packed_bytes": [_i],
    "gqa_lm_head_pack": [_vp, _vp, _vp, _i, _vp],
    "gqa_lm_head": [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp],
    "gqa_lm_head_q8_0_packed_bytes": [_i],
    "gqa_lm_head_q8_0_pack": [_vp, _vp, _vp, _i, _vp],
    "gqa_lm_head_q8_0": [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp],
    "gqa_token_embedding": [_vp, _vp, _vp, _i, _vp, _vp],
    "gqa_decode_token": [_vp, _vp, ctypes.POINTER(Model), _vp, _vp, _vp, _vp, _i, _i],
    "gqa_gguf_open": [ctypes.c_char_p, ctypes.POINTER(_vp)],
    "gqa_gguf_close": [_vp],
    "gqa_gguf_tensor_count": [_vp],
    "gqa_gguf_tensor_at": [_vp, _i, ctypes.POINTER(GgufTensor)],
    "gqa_gguf_find": [_vp, ctypes.c_char_p, ctypes.POINTER(GgufTensor)],
    "gqa_gguf_read": [_vp, ctypes.POINTER(GgufTensor), _vp],
    "gqa_gguf_meta_int": [_vp, ctypes.c_char_p, ctypes.POINTER(_ll)],
    "gqa_gguf_vocab_size": [_vp],
    "gqa_gguf_token_string": [_vp, _i, ctypes.c_char_p, _i],
    "gqa_model_load": [_vp, _vp, _i, ctypes.POINTER(_vp)],
    "gqa_model_view": [_vp, _vp, ctypes.POINTER(Model)],
    "gqa_model_free": [_vp],
    "gqa_session_create": [_vp, ctypes.POINTER(Model), _i, _vp, _i, ctypes.POINTER(_vp)],
    "gqa_session_destroy": [_vp],
    "gqa_session_set_base": [_vp, _vp, _i],
    "gqa_session_query": [_vp, _vp, _i, _i, _i, _vp, ctypes.POINTER(_i)],
    "gqa_session_status": [_vp, ctypes.POINTER(_i), ctypes.POINTER(_ull), ctypes.POINTER(_i),
                           ctypes.POINTER(_i)],
    "gqa_prefill_bf16": [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp],
    "gqa_fill_normal": [_vp, _vp, _vp, _ll, _ull, _ull, _ll],
    "gqa_inv_freq": [_vp, ctypes.POINTER(ctypes.c_float)],
    "gqa_version": [],
    "gqa_layer_attention_static": [ctypes.POINTER(Config), _vp, ctypes.POINTER(LayerKV), _vp, _i,
                                   _i],
    "gqa_static_status": [_i, ctypes.POINTER(_i), _i],
    "gqa_phase_trace_read": [_vp, _i, _i, ctypes.POINTER(_i)],
}
_RESTYPES = {"gqa_last_error_string": ctypes.c_char_p, "gqa_version": ctypes.c_char_p,
             "gqa_lm_head_packed_bytes": ctypes.c_longlong,
             "gqa_lm_head_q8_0_packed_bytes": ctypes.c_longlong}

_lib = None


def header_functions(path: str = HEADER_PATH) -> list[str]:
    """Names of the functions declared in include/gqa.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gqa_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """The loaded CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GqaError(GQA_ERR_UNSUPPORTED,
                           f"CUDA library {LIB_PATH} is not built; run __graft_entry__.build()")
        h = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGNATURES.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = h
    return _lib


def last_error() -> str:
    # (a message can quote a name from a damaged file: never fail on its bytes)
    return (lib().gqa_last_error_string() or b"").decode("utf-8", "replace")


def _check(rc: int) -> None:
    if rc != GQA_OK:
        raise GqaError(rc, last_error())


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take a device pointer of {type(x)}")


def _stream(s) -> int | None:
    if s is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(s, int):
        return s
    return s.cuda_stream


def kv_of(k_cache, v_cache) -> LayerKV:
    return LayerKV(_ptr(k_cache), _ptr(v_cache))


def block_weights_of(w_qkv, b_qkv, w_o, gamma) -> BlockWeights:
    """BlockWeights of device tensors (Q4_0 byte tensors and float tensors)."""
    return BlockWeights(_ptr(w_qkv), _ptr(b_qkv), _ptr(w_o), _ptr(gamma))


def ffn_weights_of(w_gate, w_up, w_down, gamma) -> FfnWeights:
    """FfnWeights of device tensors (Q4_0 byte tensors and a float tensor)."""
    return FfnWeights(_ptr(w_gate), _ptr(w_up), _ptr(w_down), _ptr(gamma))


def _kv_array(kvs) -> ctypes.Array:
    if isinstance(kvs, LayerKV):
        kvs = [kvs]
    arr = (LayerKV * len(kvs))()
    for i, kv in enumerate(kvs):
        arr[i] = kv
    return arr


class Graph:
    """A captured multi-layer decode step (gqa_graph_create_layers)."""

    def __init__(self, handle: int, keep: tuple):
        self._h = handle
        self._keep = keep  # keeps the ctypes arrays alive

    def launch(self, stream=None) -> None:
        _check(lib().gqa_graph_launch(self._h, _stream(stream)))

    def step_host(self, h_qkv, h_out, stream=None) -> None:
        _check(lib().gqa_graph_step_host(self._h, _stream(stream), _ptr(h_qkv), _ptr(h_out)))

    def destroy(self) -> None:
        if self._h:
            lib().gqa_graph_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


IPC_HANDLE_BYTES = 64


class Exchange:
    """This GPU's member of a group that decodes one sequence with its KV
    rows split across GPUs and merges the partials through peer memory
    (gqa_exchange_create / _open / gqa_decode_kv_shard_exchange).

    `handle` (bytes) is this GPU's inbox handle; gather every rank's handle
    in rank order and pass the list to open()."""

    def __init__(self, ctx: "Context", rank: int, world: int):
        h = _vp()
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _check(lib().gqa_exchange_create(ctx._h, rank, world, ctypes.byref(h), buf))
        self._h = h.value
        self.ctx, self.rank, self.world = ctx, rank, world
        self.handle = buf.raw

    def open(self, handles) -> None:
        blob = b"".join(bytes(x) for x in handles)
        if len(blob) != self.world * IPC_HANDLE_BYTES:
            raise ValueError("need one handle of IPC_HANDLE_BYTES per rank")
        _check(lib().gqa_exchange_open(self._h, blob))

    def step(self, kv, qkv, pos: int, shard_begin: int, shard_rows: int, out,
             stream=None) -> None:
        _check(lib().gqa_decode_kv_shard_exchange(self.ctx._h, self._h, _stream(stream),
                                                  ctypes.byref(kv), _ptr(qkv), pos, shard_begin,
                                                  shard_rows, _ptr(out)))

    def destroy(self) -> None:
        if getattr(self, "_h", None):
            lib().gqa_exchange_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class Gguf:
    """A GGUF file opened by the library's reader (host only, no GPU needed)."""

    def __init__(self, path: str):
        h = _vp()
        _check(lib().gqa_gguf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h.value

    def close(self) -> None:
        if self._h:
            lib().gqa_gguf_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _info(t: GgufTensor) -> dict:
        # names are bytes in the file (the reference reads them as char arrays):
        # undecodable bytes survive as surrogates and round-trip into find()
        return {"name": t.name.decode("utf-8", "surrogateescape"), "n_dims": t.n_dims,
                "ne": list(t.ne)[:t.n_dims],
                "type": t.type, "offset": t.offset, "bytes": t.bytes}

    def tensors(self) -> list[dict]:
        out = []
        for i in range(lib().gqa_gguf_tensor_count(self._h)):
            t = GgufTensor()
            _check(lib().gqa_gguf_tensor_at(self._h, i, ctypes.byref(t)))
            out.append(self._info(t))
        return out

    def find(self, name: str) -> dict:
        t = GgufTensor()
        _check(lib().gqa_gguf_find(self._h, name.encode("utf-8", "surrogateescape"),
                                   ctypes.byref(t)))
        return self._info(t)

    def read(self, name: str) -> np.ndarray:
        t = GgufTensor()
        _check(lib().gqa_gguf_find(self._h, name.encode("utf-8", "surrogateescape"),
                                   ctypes.byref(t)))
        out = np.empty(t.bytes, dtype=np.uint8)
        _check(lib().gqa_gguf_read(self._h, ctypes.byref(t), out.ctypes.data))
        return out

    def meta_int(self, key: str) -> int:
        v = _ll()
        _check(lib().gqa_gguf_meta_int(self._h, key.encode("utf-8", "surrogateescape"),
                                       ctypes.byref(v)))
        return v.value

    def vocab_size(self) -> int:
        return lib().gqa_gguf_vocab_size(self._h)

    def token(self, i: int) -> bytes:
        buf = ctypes.create_string_buffer(1024)
        n = lib().gqa_gguf_token_string(self._h, i, buf, len(buf))
        if n < 0:
            _check(n)
        return buf.raw[:min(n, len(buf) - 1)]


class LoadedModel:
    """gqa_model_load's device weights; view(kvs) gives the gqa_model."""

    def __init__(self, ctx: "Context", gguf: Gguf, n_layers: int = 0):
        h = _vp()
        _check(lib().gqa_model_load(ctx._h, gguf._h, n_layers, ctypes.byref(h)))
        self._h = h.value
        m = Model()
        _check(lib().gqa_model_view(self._h, None, ctypes.byref(m)))
        self.n_layers, self.vocab = m.n_layers, m.vocab

    def view(self, kvs) -> Model:
        n = len(kvs)
        assert n == self.n_layers
        self._kv = (LayerKV * n)(*kvs)
        m = Model()
        _check(lib().gqa_model_view(self._h, self._kv, ctypes.byref(m)))
        return m

    def free(self) -> None:
        if self._h:
            lib().gqa_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Session:
    """The server's SET_BASE / QUERY / RAW_QUERY / STATUS over a model."""

    def __init__(self, ctx: "Context", model: Model, t_max: int, eog=None):
        h = _vp()
        self._keep = (ctx, model)
        eog_arr = (ctypes.c_int * len(eog))(*eog) if eog is not None else None
        _check(lib().gqa_session_create(ctx._h, ctypes.byref(model), t_max, eog_arr,
                                        len(eog) if eog is not None else 0, ctypes.byref(h)))
        self._h = h.value

    def set_base(self, tokens) -> None:
        arr = (ctypes.c_int * len(tokens))(*tokens)
        _check(lib().gqa_session_set_base(self._h, arr, len(tokens)))

    def query(self, tokens, max_new: int, raw: bool = False) -> list[int]:
        arr = (ctypes.c_int * max(len(tokens), 1))(*tokens)
        out = (ctypes.c_int * max(max_new, 1))()
        n = _i()
        _check(lib().gqa_session_query(self._h, arr, len(tokens), max_new, int(raw), out,
                                       ctypes.byref(n)))
        return list(out[:n.value])

    def status(self) -> dict:
        bp, gen, ready = _i(), _i(), _i()
        hsh = _ull()
        _check(lib().gqa_session_status(self._h, ctypes.byref(bp), ctypes.byref(hsh),
                                        ctypes.byref(gen), ctypes.byref(ready)))
        return {"base_pos": bp.value, "base_hash": hsh.value, "base_generation": gen.value,
                "ready": bool(ready.value)}

    def destroy(self) -> None:
        if self._h:
            lib().gqa_session_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class ModelHandle:
    """A gqa_model together with the ctypes arrays it points into."""

    def __init__(self, attn, ffn, kvs, token_embd, gamma_output, lm_head_packed, vocab: int,
                 lm_head_type: int = 0):
        n = len(attn)
        assert len(ffn) == n and len(kvs) == n
        self._attn = (BlockWeights * n)(*attn)
        self._ffn = (FfnWeights * n)(*ffn)
        self._kv = (LayerKV * n)(*kvs)
        self._keep = (token_embd, gamma_output, lm_head_packed)
        self.struct = Model(n, self._attn, self._ffn, self._kv, _ptr(token_embd),
                            _ptr(gamma_output), _ptr(lm_head_packed), vocab, lm_head_type)


class Context:
    """One gqa_ctx on one device (see include/gqa.h for every call)."""

    def __init__(self, n_heads_q: int = 12, n_heads_kv: int = 2, head_dim: int = 128,
                 t_max: int = 4096, rope_theta: float = 1e6, device: int = 0):
        self.cfg = Config(n_heads_q, n_heads_kv, head_dim, t_max, rope_theta)
        h = _vp()
        _check(lib().gqa_create(ctypes.byref(self.cfg), device, ctypes.byref(h)))
        self._h = h.value
        self.device = device
        self.n_heads_q, self.n_heads_kv, self.head_dim, self.t_max = (
            n_heads_q, n_heads_kv, head_dim, t_max)

    # -- lifetime / options -------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().gqa_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_option(self, option: int, value: int) -> None:
        _check(lib().gqa_set_option(self._h, option, value))

    def reserve(self, n_seq: int, max_len: int) -> None:
        _check(lib().gqa_reserve(self._h, n_seq, max_len))

    def device_status(self, clear: bool = True) -> int:
        st = _i(0)
        _check(lib().gqa_device_status(self._h, ctypes.byref(st), 1 if clear else 0))
        return st.value

    def inv_freq(self) -> np.ndarray:
        buf = (ctypes.c_float * (self.head_dim // 2))()
        _check(lib().gqa_inv_freq(self._h, buf))
        return np.frombuffer(buf, dtype=np.float32).copy()

    # -- KV cache -----------------------------------------------------------
    def kv_alloc(self, n_layers: int) -> list[LayerKV]:
        arr = (LayerKV * n_layers)()
        _check(lib().gqa_kv_alloc(self._h, n_layers, arr))
        return [arr[i] for i in range(n_layers)]

    def kv_free(self, kvs) -> None:
        arr = _kv_array(kvs)
        _check(lib().gqa_kv_free(self._h, len(arr), arr))

    # -- layer call ---------------------------------------------------------
    def layer_attention(self, kv: LayerKV, qkv, pos: int, seq_len: int, stream=None) -> None:
        _check(lib().gqa_layer_attention(self._h, _stream(stream), ctypes.byref(kv), _ptr(qkv),
                                         pos, seq_len))

    def layer_attention_out(self, kv: LayerKV, qkv, pos: int, seq_len: int, out,
                            stream=None) -> None:
        _check(lib().gqa_layer_attention_out(self._h, _stream(stream), ctypes.byref(kv),
                                             _ptr(qkv), pos, seq_len, _ptr(out)))

    def decode_layers(self, kvs, qkv, qkv_stride: int, out, out_stride: int, d_pos,
                      advance: bool = False, wrap_lo: int = 0, wrap_hi: int = 0,
                      stream=None) -> None:
        arr = _kv_array(kvs)
        _check(lib().gqa_decode_layers(self._h, _stream(stream), len(arr), arr, _ptr(qkv),
                                       qkv_stride, _ptr(out), out_stride, _ptr(d_pos),
                                       1 if advance else 0, wrap_lo, wrap_hi))

    def graph_create_layers(self, kvs, qkv, qkv_stride: int, out, out_stride: int, d_pos,
                            advance: bool = True, wrap_lo: int = 0, wrap_hi: int = 0) -> Graph:
        arr = _kv_array(kvs)
        h = _vp()
        _check(lib().gqa_graph_create_layers(self._h, len(arr), arr, _ptr(qkv), qkv_stride,
                                             _ptr(out), out_stride, _ptr(d_pos),
                                             1 if advance else 0, wrap_lo, wrap_hi,
                                             ctypes.byref(h)))
        return Graph(h.value, (arr,))

    # -- kernel-level operations ---------------------------------------------
    def rope_kv_append(self, kv: LayerKV, q, k, v, pos: int, stream=None) -> None:
        _check(lib().gqa_rope_kv_append(self._h, _stream(stream), ctypes.byref(kv), _ptr(q),
                                        _ptr(k), _ptr(v), pos))

    def decode(self, kv: LayerKV, q_rot, seq_len: int, out, stream=None) -> None:
        _check(lib().gqa_decode(self._h, _stream(stream), ctypes.byref(kv), _ptr(q_rot), seq_len,
                                _ptr(out)))

    def decode_batched(self, n_seq: int, k_ptrs, v_ptrs, qkv, qkv_stride: int, seq_lens,
                       max_len: int, out, out_stride: int, stream=None) -> None:
        _check(lib().gqa_decode_batched(self._h, _stream(stream), n_seq, _ptr(k_ptrs),
                                        _ptr(v_ptrs), _ptr(qkv), qkv_stride, _ptr(seq_lens),
                                        max_len, _ptr(out), out_stride))

    def decode_batched_host(self, n_seq: int, k_ptrs, v_ptrs, h_qkv, d_qkv, qkv_stride: int,
                            seq_lens, max_len: int, d_out, out_stride: int, h_out,
                            stream=None) -> None:
        """gqa_decode_batched with host input and output: h_qkv / h_out are
        host buffers (page-locked tensors or arrays), d_qkv / d_out the device
        buffers the step runs on; h_out receives n_seq packed output rows."""
        _check(lib().gqa_decode_batched_host(self._h, _stream(stream), n_seq, _ptr(k_ptrs),
                                             _ptr(v_ptrs), _ptr(h_qkv), _ptr(d_qkv), qkv_stride,
                                             _ptr(seq_lens), max_len, _ptr(d_out), out_stride,
                                             _ptr(h_out)))

    def decode_split_partial(self, kv: LayerKV, q_rot, t_begin: int, t_end: int, m, l, o,
                             stream=None) -> None:
        _check(lib().gqa_decode_split_partial(self._h, _stream(stream), ctypes.byref(kv),
                                              _ptr(q_rot), t_begin, t_end, _ptr(m), _ptr(l),
                                              _ptr(o)))

    def decode_kv_shard(self, kv: LayerKV, qkv, pos: int, shard_begin: int, shard_rows: int,
                        m, l, o, stream=None) -> None:
        _check(lib().gqa_decode_kv_shard(self._h, _stream(stream), ctypes.byref(kv), _ptr(qkv),
                                         pos, shard_begin, shard_rows, _ptr(m), _ptr(l), _ptr(o)))

    def lse_combine(self, n_parts: int, n_rows: int, m, l, o, out, stream=None) -> None:
        _check(lib().gqa_lse_combine(self._h, _stream(stream), n_parts, n_rows, _ptr(m), _ptr(l),
                                     _ptr(o), _ptr(out)))

    def attention_block(self, w: "BlockWeights", kv: LayerKV, state, pos: int, seq_len: int,
                        stream=None) -> None:
        _check(lib().gqa_attention_block(self._h, _stream(stream), ctypes.byref(w),
                                         ctypes.byref(kv), _ptr(state), pos, seq_len))

    def attention_block_layers(self, weights, kvs, state, d_pos, advance: bool = False,
                               wrap_lo: int = 0, wrap_hi: int = 0, stream=None) -> None:
        n = len(weights)
        warr = (BlockWeights * n)(*weights)
        karr = (LayerKV * n)(*kvs)
        _check(lib().gqa_attention_block_layers(self._h, _stream(stream), n, warr, karr,
                                                _ptr(state), _ptr(d_pos), int(advance), wrap_lo,
                                                wrap_hi))

    def ffn_block(self, w: "FfnWeights", state, stream=None) -> None:
        _check(lib().gqa_ffn_block(self._h, _stream(stream), ctypes.byref(w), _ptr(state)))

    def decoder_layers(self, attn, ffn, kvs, state, d_pos, advance: bool = False,
                       wrap_lo: int = 0, wrap_hi: int = 0, stream=None) -> None:
        n = len(attn)
        _check(lib().gqa_decoder_layers(self._h, _stream(stream), n, (BlockWeights * n)(*attn),
                                        (FfnWeights * n)(*ffn), (LayerKV * n)(*kvs), _ptr(state),
                                        _ptr(d_pos), int(advance), wrap_lo, wrap_hi))

    # ---- the model's ends and the whole decode step ----

    @staticmethod
    def lm_head_packed_bytes(n_rows: int) -> int:
        return int(lib().gqa_lm_head_packed_bytes(n_rows))

    def lm_head_pack(self, q6k, n_rows: int, packed, stream=None) -> None:
        _check(lib().gqa_lm_head_pack(self._h, _stream(stream), _ptr(q6k), n_rows, _ptr(packed)))

    def lm_head(self, packed, n_rows: int, gamma, state, logits=None, token=None,
                stream=None) -> None:
        _check(lib().gqa_lm_head(self._h, _stream(stream), _ptr(packed), n_rows, _ptr(gamma),
                                 _ptr(state), _ptr(logits), _ptr(token)))

    @staticmethod
    def lm_head_q8_0_packed_bytes(n_rows: int) -> int:
        return int(lib().gqa_lm_head_q8_0_packed_bytes(n_rows))

    def lm_head_q8_0_pack(self, q8, n_rows: int, packed, stream=None) -> None:
        _check(lib().gqa_lm_head_q8_0_pack(self._h, _stream(stream), _ptr(q8), n_rows,
                                           _ptr(packed)))

    def lm_head_q8_0(self, packed, n_rows: int, gamma, state, logits=None, token=None,
                     stream=None) -> None:
        _check(lib().gqa_lm_head_q8_0(self._h, _stream(stream), _ptr(packed), n_rows, _ptr(gamma),
                                      _ptr(state), _ptr(logits), _ptr(token)))

    def token_embedding(self, table, n_rows: int, d_token, state, stream=None) -> None:
        _check(lib().gqa_token_embedding(self._h, _stream(stream), _ptr(table), n_rows,
                                         _ptr(d_token), _ptr(state)))

    def decode_token(self, model: "ModelHandle", state, d_token, d_pos, logits=None,
                     wrap_lo: int = 0, wrap_hi: int = 0, stream=None) -> None:
        _check(lib().gqa_decode_token(self._h, _stream(stream), ctypes.byref(model.struct),
                                      _ptr(state), _ptr(d_token), _ptr(d_pos), _ptr(logits),
                                      wrap_lo, wrap_hi))

    def lse_combine_packed(self, n_parts: int, n_rows: int, packed, part_stride: int, out,
                           stream=None) -> None:
        _check(lib().gqa_lse_combine_packed(self._h, _stream(stream), n_parts, n_rows,
                                            _ptr(packed), part_stride, _ptr(out)))

    def prefill_bf16(self, n_seq: int, seq_len: int, qkv, out, k_ptrs=None, v_ptrs=None,
                     stream=None) -> None:
        _check(lib().gqa_prefill_bf16(self._h, _stream(stream), n_seq, seq_len, _ptr(qkv),
                                      _ptr(out), _ptr(k_ptrs), _ptr(v_ptrs)))

    def fill_normal(self, dst, n: int, seed: int, stream_id: int, offset: int = 0,
                    stream=None) -> None:
        _check(lib().gqa_fill_normal(self._h, _stream(stream), _ptr(dst), n, seed, stream_id,
                                     offset))
