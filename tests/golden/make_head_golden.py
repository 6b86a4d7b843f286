"""Regenerates tests/golden/head_golden.npz from the reference itself.

Runs the reference's own CPU Q6_K LM-head GEMV -- cpu_gemv_q6_k_ref
(compute/gguf-real-weights-loader/test_gemv_q6_k.c:77-94), compiled
unmodified into oracle/_ref/libgqa_ref_head.so -- on a seeded Q6_K matrix
with the unit vectors its own test uses (:209) and two dense inputs, and its
token embedding lookup get_token_embedding (test_full_model_logits.c:584-597,
oracle/_ref/libgqa_ref_model.so) on a seeded Q4_0 table.  Inputs are not
stored: they regenerate from the seed through the package's seeded module and
are pinned by a SHA-256.

Needs the reference sources at build time (oracle/_ref); run from the repo
root:  python tests/golden/make_head_golden.py
"""
import hashlib
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)
import __graft_entry__  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "head_golden.npz")
SEED, ROWS, EMBD_ROWS = 5150, 256, 64
BASIS = [0, 15, 16, 31, 32, 63, 64, 95, 96, 127, 128, 255, 512, 1024, 1535]


def main():
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    assert orc.have_reference(), "oracle/_ref not built (needs the reference sources)"
    s = g.seeded
    w = s.q6_k_matrix(SEED, s.W_HEAD, ROWS)
    xs = []
    for i in BASIS:
        x = np.zeros(1536, dtype=np.float32)
        x[i] = 1.0
        xs.append(x)
    xs.append(s.normal(SEED, s.HEAD_X, 1536))
    xs.append((s.normal(SEED + 1, s.HEAD_X, 1536) * 40).astype(np.float32))
    ys = [orc.ref_gemv_q6_k(w, x) for x in xs]
    table = s.q4_0_matrix(SEED, s.TOKEN_EMBD, EMBD_ROWS, 1536, 1.0 / 4.6)
    toks = [0, 1, 31, EMBD_ROWS - 1]
    embd = [orc.ref_token_embedding(table, t) for t in toks]
    np.savez_compressed(OUT, seed=SEED, rows=ROWS, digest=hashlib.sha256(w.tobytes()).hexdigest(),
                        x=np.array(xs), y=np.array(ys), embd_rows=EMBD_ROWS,
                        embd_tokens=np.array(toks), embd=np.array(embd))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
