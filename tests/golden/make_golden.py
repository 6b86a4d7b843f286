"""Regenerates tests/golden/decode_golden.npz from the reference itself.

Runs the reference's own CPU attention -- cpu_attention_gqa_pipeline
(compute/attention-gqa-resident/attention_gqa_benchmark.c:109-216), compiled
unmodified into oracle/_ref/libgqa_ref_bench.so by oracle/Makefile -- on
seeded inputs and stores its outputs: attn_out and the K/V rows it appended.
Inputs are not stored; they are regenerated from the seed by the package's
seeded.decode_inputs() and pinned by a SHA-256 of their bytes.

Needs the reference sources at build time (oracle/_ref); run from the repo
root:  python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)
import __graft_entry__  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_golden.npz")

# (name, pos, seq_len, dist).  The reference sweep (attention_gqa_benchmark.c:424,
# pos = seq_len - 1 at :437), then edge cases around the 32-row split quantum and
# the reference's 256-row PV segment, a row appended outside the attended range,
# and two cases with the reference benchmark's own cache distribution.
CASES = [(f"sweep_T{T}", T - 1, T, "normal") for T in (1, 32, 128, 512, 1024, 2048, 4096)] + [
    ("edge_T2", 1, 2, "normal"),
    ("edge_T31", 30, 31, "normal"),
    ("edge_T33", 32, 33, "normal"),
    ("edge_T255", 254, 255, "normal"),
    ("edge_T257", 256, 257, "normal"),
    ("edge_T4095", 4094, 4095, "normal"),
    ("pos_outside_T50", 100, 50, "normal"),
    ("pos0_T5", 0, 5, "normal"),
    ("grid_T512", 511, 512, "grid"),
    ("grid_T4096", 4095, 4096, "grid"),
]


def input_digest(qkv, kc, vc) -> str:
    h = hashlib.sha256()
    for a in (qkv, kc, vc):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    assert orc.have_reference(), "oracle/_ref not built (needs the reference sources)"
    rec = {k: [] for k in ("name", "pos", "seq_len", "seed", "dist", "digest", "attn_out",
                           "k_rows", "v_rows")}
    for i, (name, pos, seq_len, dist) in enumerate(CASES):
        seed = 424200 + i
        qkv, kc, vc = g.seeded.decode_inputs(seed, orc.REF_T_MAX, dist=dist)
        digest = input_digest(qkv, kc, vc)
        k1, v1 = kc.copy(), vc.copy()
        out = orc.ref_bench_attention(qkv.copy(), k1, v1, pos, seq_len)
        for key, val in (("name", name), ("pos", pos), ("seq_len", seq_len), ("seed", seed),
                         ("dist", dist), ("digest", digest), ("attn_out", out),
                         ("k_rows", k1[:, pos].copy()), ("v_rows", v1[:, pos].copy())):
            rec[key].append(val)
    np.savez_compressed(OUT, **{k: np.array(v) for k, v in rec.items()})
    print(f"wrote {OUT} ({len(CASES)} cases)")


if __name__ == "__main__":
    main()
