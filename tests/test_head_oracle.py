"""The oracle of the model's ends, pinned on the CPU: the Q6_K dequantisation
and GEMV (the reference's own test_gemv_q6_k.c, compiled), its restatement in
numpy, the golden vectors made from the reference, and the restated
embedding lookup, output norm and greedy pick."""
import os

import numpy as np
import pytest

ROW = 1260
BASIS = [0, 15, 16, 31, 32, 63, 64, 95, 96, 127, 128, 255, 512, 1024, 1535]
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "head_golden.npz")


@pytest.fixture(scope="module")
def need_ref(orc):
    if not orc.have_reference():
        pytest.skip("oracle/_ref not built (reference sources absent)")


def _edge_rows(pkg):
    """Seeded rows plus rows of extreme bytes: all codes 0 / 63, scales -128 / 127."""
    w = pkg.seeded.q6_k_matrix(21, pkg.seeded.W_HEAD, 8).reshape(8, 6, 210)
    w[0, :, :192] = 0x00
    w[1, :, :192] = 0xFF
    w[2, :, 192:208] = 0x80  # int8 -128
    w[3, :, 192:208] = 0x7F
    return w.reshape(-1)


def test_dequant_restatement_matches_reference(pkg, orc, need_ref):
    w = np.concatenate([pkg.seeded.q6_k_matrix(20, pkg.seeded.W_HEAD, 64), _edge_rows(pkg)])
    n = w.size // ROW
    deq = pkg.seeded.q6_k_dequant(w, n)
    for r in range(n):
        ref = orc.ref_dequant_q6_k(w[r * ROW:(r + 1) * ROW])
        assert np.array_equal(ref.view(np.uint32), deq[r].view(np.uint32)), r


def test_reference_gemv_unit_columns(pkg, orc, need_ref):
    """The reference's GEMV on a unit vector returns that column of the
    dequantised matrix exactly -- the property its own basis test checks."""
    w = np.concatenate([pkg.seeded.q6_k_matrix(22, pkg.seeded.W_HEAD, 200), _edge_rows(pkg)])
    n = w.size // ROW
    deq = pkg.seeded.q6_k_dequant(w, n)
    for i in BASIS:
        x = np.zeros(1536, dtype=np.float32)
        x[i] = 1.0
        assert np.array_equal(orc.ref_gemv_q6_k(w, x), deq[:, i])


def test_golden_vectors(pkg, orc):
    """head_golden.npz (made by tests/golden/make_head_golden.py from the
    compiled reference): the inputs regenerate from the seed, and the oracle
    reproduces the stored outputs -- exactly with the reference built, else
    through the numpy restatement in float64."""
    z = np.load(GOLDEN)
    rows, seed = int(z["rows"]), int(z["seed"])
    w = pkg.seeded.q6_k_matrix(seed, pkg.seeded.W_HEAD, rows)
    import hashlib
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(z["digest"])
    xs, ys = z["x"], z["y"]
    deq = pkg.seeded.q6_k_dequant(w, rows).astype(np.float64)
    for x, y in zip(xs, ys):
        approx = deq @ x.astype(np.float64)
        assert np.abs(approx - y).max() <= 1e-5 * max(np.sqrt(np.mean(approx ** 2)), 1e-30)
        if orc.have_reference():
            assert np.array_equal(orc.ref_gemv_q6_k(w, x).view(np.uint32), y.view(np.uint32))
    table = pkg.seeded.q4_0_matrix(seed, pkg.seeded.TOKEN_EMBD, int(z["embd_rows"]), 1536,
                                   1.0 / 4.6)
    for tok, e in zip(z["embd_tokens"], z["embd"]):
        assert np.array_equal(orc.token_embedding(table, int(tok)).view(np.uint32),
                              e.view(np.uint32))


def test_embedding_restatement_matches_reference(pkg, orc, need_ref):
    rows = 300
    table = pkg.seeded.q4_0_matrix(23, pkg.seeded.TOKEN_EMBD, rows, 1536, 0.3)
    for tok in (0, 1, 150, rows - 1):
        a = orc.token_embedding(table, tok)
        b = orc.ref_token_embedding(table, tok)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    with pytest.raises(ValueError):
        orc.ref_token_embedding(table, rows)


def test_output_norm_restatement(pkg, orc):
    x = pkg.seeded.normal(24, pkg.seeded.STATE, 1536) * 3
    g = (1.0 + 0.1 * pkg.seeded.normal(24, pkg.seeded.GAMMA_OUT, 1536)).astype(np.float32)
    z = orc.output_norm(x, g)
    x64 = x.astype(np.float64)
    want = x64 / np.sqrt(np.mean(x64 ** 2) + 1e-6) * g
    assert np.abs(z - want).max() <= 1e-5 * np.sqrt(np.mean(want ** 2))


def test_greedy_pick_rules(orc):
    a = np.array([1.0, 5.0, 5.0, 2.0], dtype=np.float32)
    assert orc.greedy_pick(a) == 1  # first maximum
    a = np.array([np.nan, 3.0, np.nan, 3.5], dtype=np.float32)
    assert orc.greedy_pick(a) == 3  # NaN never wins
    assert orc.greedy_pick(np.full(9, np.nan, dtype=np.float32)) == 0
    assert orc.greedy_pick(np.full(9, -1e30, dtype=np.float32)) == 0  # not above -1e30
    a = np.array([-2e30, -1e30, -9.9e29], dtype=np.float32)
    assert orc.greedy_pick(a) == 2
    a = np.array([0.0, np.inf, np.inf], dtype=np.float32)
    assert orc.greedy_pick(a) == 1


def test_planes_layout(pkg):
    """Planes over 12 rows (11 real + 1 zero padding row): each row's ql and
    qh bytes in superblock order, rotated right by 16 * (row % 8) bytes;
    scales and d in superblock order."""
    rows = 11
    w = pkg.seeded.q6_k_matrix(25, pkg.seeded.W_HEAD, rows)
    p = pkg.seeded.q6_k_planes(w, rows)
    n = 12
    assert p.size == n * ROW
    b = w.reshape(rows, 6, 210)
    for r in range(rows):
        ql = p[768 * r:768 * (r + 1)]
        qh = p[n * 768 + 384 * r:n * 768 + 384 * (r + 1)]
        rot = 16 * (r % 8)
        for i in (0, 1, 127, 128, 500, 767):
            assert ql[(i + rot) % 768] == b[r, i // 128, i % 128], (r, i)
        for i in (0, 63, 64, 200, 383):
            assert qh[(i + rot) % 384] == b[r, i // 64, 128 + i % 64], (r, i)
        assert np.array_equal(p[n * 1152 + 96 * r:n * 1152 + 96 * (r + 1)],
                              b[r, :, 192:208].reshape(-1))
        assert np.array_equal(p[n * 1248 + 12 * r:n * 1248 + 12 * (r + 1)],
                              b[r, :, 208:].reshape(-1))
    for base, width in ((0, 768), (n * 768, 384), (n * 1152, 96), (n * 1248, 12)):
        assert not p[base + width * rows:base + width * n].any()             # padding row
