"""Pins the oracle (CPU, no GPU needed).

1. The C restatement (oracle/gqa_oracle.c) reproduces the reference's own
   compiled cpu_attention_gqa_pipeline (attention_gqa_benchmark.c:109-216) bit
   for bit: attention output and the appended cache rows.
2. The reference's two CPU attention variants agree (the benchmark's and the
   decoder layer's, test_28_layers_real.c:250-289).
3. The restatement reproduces the committed golden vectors (made from the
   reference by tests/golden/make_golden.py), which also pins it where the
   reference sources are absent.
"""
import hashlib
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "decode_golden.npz")


def _digest(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_inv_freq_matches_reference_expression(orc):
    got = orc.inv_freq(1e6, 128)
    i = np.arange(64, dtype=np.float32)
    expect = np.power(np.float64(1e6), (np.float32(-2.0) * i / np.float32(128.0)).astype(np.float64))
    # fp32 powf vs fp64 pow rounded: within 1 ulp
    assert np.allclose(got, expect.astype(np.float32), rtol=2e-7, atol=0)


@pytest.mark.parametrize("i", range(17))
def test_restatement_matches_golden(golden, pkg, orc, i):
    pos, seq_len = int(golden["pos"][i]), int(golden["seq_len"][i])
    qkv, kc, vc = pkg.seeded.decode_inputs(int(golden["seed"][i]), orc.REF_T_MAX,
                                           dist=str(golden["dist"][i]))
    assert _digest(qkv, kc, vc) == str(golden["digest"][i]), "seeded inputs changed"
    q = qkv.copy()
    orc.layer_attention(q, kc, vc, pos, seq_len)
    assert np.array_equal(q[:1536], golden["attn_out"][i])
    assert np.array_equal(kc[:, pos], golden["k_rows"][i])
    assert np.array_equal(vc[:, pos], golden["v_rows"][i])
    assert np.array_equal(q[1536:], qkv[1536:])


@pytest.mark.parametrize("pos,seq_len", [(0, 1), (1, 2), (2, 3), (6, 7), (63, 64), (100, 50),
                                         (511, 512), (999, 1000), (4095, 4096), (0, 4096)])
def test_restatement_bit_exact_vs_compiled_reference(pkg, orc, pos, seq_len):
    if not orc.have_reference():
        pytest.skip("oracle/_ref not built (reference sources absent at build time)")
    qkv, kc, vc = pkg.seeded.decode_inputs(9000 + pos, orc.REF_T_MAX)
    k1, v1, k2, v2 = kc.copy(), vc.copy(), kc.copy(), vc.copy()
    ref = orc.ref_bench_attention(qkv.copy(), k1, v1, pos, seq_len)
    q = qkv.copy()
    orc.layer_attention(q, k2, v2, pos, seq_len)
    assert np.array_equal(ref, q[:1536])
    assert np.array_equal(k1, k2) and np.array_equal(v1, v2)


@pytest.mark.parametrize("pos,seq_len", [(0, 1), (5, 6), (511, 512), (3000, 3001)])
def test_reference_variants_agree(pkg, orc, pos, seq_len):
    if not orc.have_reference():
        pytest.skip("oracle/_ref not built")
    qkv, kc, vc = pkg.seeded.decode_inputs(77 + pos, orc.REF_T_MAX)
    a = orc.ref_bench_attention(qkv.copy(), kc.copy(), vc.copy(), pos, seq_len)
    b = orc.ref_layer_attention(qkv.copy(), kc.copy(), vc.copy(), pos, seq_len)
    assert np.array_equal(a, b)


def test_partial_and_combine_equal_full_attention(pkg, orc):
    qkv, kc, vc = pkg.seeded.decode_inputs(5, 1024)
    q = qkv[:1536].copy()
    full = orc.attention(q, kc, vc, 1000)
    cuts = [0, 1, 300, 301, 777, 1000]
    parts = [orc.attention_partial(q, kc, vc, a, b) for a, b in zip(cuts[:-1], cuts[1:])]
    m = np.stack([p[0] for p in parts])
    l = np.stack([p[1] for p in parts])
    o = np.stack([p[2].reshape(12, 128) for p in parts])
    got = orc.lse_combine(m, l, o).reshape(-1)
    assert np.abs(got - full).max() / np.sqrt(np.mean(full ** 2)) < 1e-5
    # an empty part carries no weight
    m0, l0, o0 = orc.attention_partial(q, kc, vc, 10, 10)
    assert np.all(np.isneginf(m0)) and np.all(l0 == 0)


def test_batched_oracle_equals_single(pkg, orc):
    lens = [1, 7, 64, 300]
    qkvs, ks, vs, singles = [], [], [], []
    for i, L in enumerate(lens):
        qkv, kc, vc = pkg.seeded.decode_inputs(60 + i, 512)
        qkvs.append(qkv.copy()); ks.append(kc.copy()); vs.append(vc.copy())
        q = qkv.copy(); k2 = kc.copy(); v2 = vc.copy()
        orc.layer_attention(q, k2, v2, L - 1, L)
        singles.append(q[:1536])
    outs = orc.decode_batched(qkvs, ks, vs, lens, n_threads=4)
    for a, b in zip(outs, singles):
        assert np.array_equal(a, b)
