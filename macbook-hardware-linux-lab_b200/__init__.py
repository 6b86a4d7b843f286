"""B200 (sm_100a) grouped-query-attention decode path.

A from-scratch CUDA build of the GQA attention hot path of
fbetancourt-dev/macbook-hardware-linux-lab (compute/attention-gqa-resident, as
used by gguf-real-weights-loader/qwen_server.c): RoPE on q/k, KV-cache append,
QK^T for 6 query heads per KV head, stable softmax and PV, plus split-KV with a
log-sum-exp combine.  The product is the C-ABI library libgqa_b200.so
(include/gqa.h); this package holds its sources (csrc/), the build script, a
ctypes binding and the host-side helpers for sharding across GPUs.

The directory name contains hyphens, so it is loaded by path (see
``__graft_entry__.load_package``) under the module name ``gqa_b200``.
"""
from . import seeded, shard  # noqa: F401
from .gqa import (BlockWeights, Context, Exchange, FfnWeights, Gguf, GqaError,  # noqa: F401
                  Graph, LayerKV, LoadedModel, Model, ModelHandle, Session, block_weights_of,
                  ffn_weights_of, header_functions, kv_of, last_error, lib)
