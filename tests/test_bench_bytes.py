"""The algorithmic byte counts behind bench.py's GB/s and roofline figures,
recomputed from the sizes of the arrays the workloads are generated from (no
GPU): KV rows, Q4_0 projection and FFN weights, biases and norms, and the two
LM heads at both model sizes."""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _nbytes(*arrays):
    return sum(np.asarray(a).nbytes for a in arrays)


def test_kv_row_bytes():
    # K and V of one attended position, both KV heads, fp32
    assert bench.ROW_BYTES == 2 * 2 * 128 * 4 == 2048
    assert bench.ROW05 == 2 * 2 * 64 * 4 == 1024


def test_layer_weight_bytes_15b(pkg):
    s = pkg.seeded
    _, w_qkv, b_qkv, w_o, gamma, _, _ = s.attention_block_inputs(1, t_max=8)
    assert bench.BLOCK_WEIGHT_BYTES == _nbytes(w_qkv, b_qkv, w_o, gamma)
    assert bench.FFN_WEIGHT_BYTES == _nbytes(*s.ffn_block_inputs(1))


def test_layer_weight_bytes_05b(pkg):
    s = pkg.seeded
    _, w_qkv, b_qkv, w_o, gamma, _, _ = s.attention_block_inputs(1, t_max=8, d_model=896,
                                                                 n_heads_kv=2, head_dim=64)
    assert bench.BLOCK05_BYTES == _nbytes(w_qkv, b_qkv, w_o, gamma)
    assert bench.FFN05_BYTES == _nbytes(*s.ffn_block_inputs(1, d_model=896, d_ffn=4864))
    assert bench.Q4_ROW05 == 896 // 32 * 18


def test_head_bytes(pkg):
    s = pkg.seeded
    rows = 64
    # per vocabulary row, as generated; plus gamma_output and the state
    q6 = s.q6_k_matrix(1, s.W_HEAD, rows, 1536).nbytes // rows
    q8 = s.q8_0_matrix(1, s.W_HEAD, rows, 896).nbytes // rows
    assert bench.HEAD_BYTES == bench.VOCAB * q6 + 1536 * 4 * 2
    assert bench.HEAD05_BYTES == bench.VOCAB * q8 + 896 * 4 * 2
    # the packed layouts hold exactly the tensor's bytes for the full vocabulary
    assert pkg.Context.lm_head_packed_bytes(bench.VOCAB) == bench.VOCAB * q6
    assert pkg.Context.lm_head_q8_0_packed_bytes(bench.VOCAB) == bench.VOCAB * q8


def test_packed_sizes_edges(pkg):
    """Rows are rounded up to a multiple of 4; no rows, no bytes."""
    C = pkg.Context
    for n in (-1, 0):
        assert C.lm_head_packed_bytes(n) == 0 and C.lm_head_q8_0_packed_bytes(n) == 0
    for n, padded in ((1, 4), (3, 4), (4, 4), (5, 8), (151936, 151936)):
        assert C.lm_head_packed_bytes(n) == padded * 1260
        assert C.lm_head_q8_0_packed_bytes(n) == padded * 952


def test_batched_traffic_reference_bytes(pkg):
    """The batched traffic file's algorithmic bytes: the 64 seeded lengths'
    cache rows (one GPU holding them all) x 2048 B, a few steps into the window."""
    lens = [int(x) for x in pkg.seeded.uniform_int(777, pkg.seeded.LENGTHS, 64, 256, 8192)]
    vals = {}
    for line in open(os.path.join(bench.REPO, "profiles", "traffic_batched.txt")):
        if "=" in line and not line.startswith("#"):
            k, v = line.split("=", 1)
            vals[k.strip()] = float(v)
    first = bench.ROW_BYTES * sum(lens)
    alg = vals["algorithmic_bytes_per_launch"]
    assert first <= alg <= first + 8 * 64 * bench.ROW_BYTES


def test_traffic_scaled_to_a_share():
    """A GPU's share of a sharded workload gets the one-GPU capture's traffic
    scaled by its own algorithmic bytes (batched) or by the sequence share
    (prefill); unsharded workloads keep the captured figure."""
    full = bench.profile_traffic("batched")
    alg = 542771200
    assert bench.profile_traffic("batched", alg) == round(full)
    assert bench.profile_traffic("batched", alg / 4) == round(full / 4)
    pre = bench.profile_traffic("prefill")
    assert bench.profile_traffic("prefill", scale=1 / 8) == round(pre / 8)
    res = bench.profile_traffic("resident28")
    assert bench.profile_traffic("resident28", 7.9e6) == res
    assert bench.profile_traffic("no_such_workload", 1e6) is None
