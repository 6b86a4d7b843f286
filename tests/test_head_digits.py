"""The integer arithmetic of the two LM heads, restated in numpy from the
packed planes (no GPU): the inputs split into three signed 8-bit digits, the
exact integer dot products, and the bounds the kernels rely on -- every digit
inside its range; the Q6_K head's per-superblock sums inside int32, the Q8_0
head's digit sums below 2^22 in magnitude, where the 2^23 + 2^22 magic
conversion to float is exact -- on worst-case weights and inputs; with unit
inputs z = 32 e_i the Q6_K logits equal the reference's compiled GEMV bit for
bit (the property tests/test_head_gpu.py checks on the device)."""
import numpy as np
import pytest

F32 = np.float32
MAGIC = F32(12582912.0)  # 1.5 * 2^23: adding it rounds to an integer
LIMIT = 1 << 22


def _round(x):
    t = (x + MAGIC).astype(F32)
    return (t - MAGIC).astype(F32)


def q6_digits(z):
    """lm_head_kernel's split: one power-of-two scale s >= max|z| / 63 for the
    whole input vector, then three digits in base 126, each in [-63, 63]."""
    z = np.asarray(z, F32)
    mx = F32(np.abs(z).max())
    mb = int(np.array([mx / F32(63)], F32).view(np.uint32)[0])
    sb = (mb & 0x7F800000) + 0x00800000 if mb & 0x007FFFFF else mb
    s = np.array([sb], np.uint32).view(F32)[0] if mx > 0 else F32(1)
    x = (z * (F32(1) / s)).astype(F32)
    d1 = _round(x)
    r1 = ((x - d1).astype(F32) * F32(126)).astype(F32)
    d2 = _round(r1)
    d3 = _round(((r1 - d2).astype(F32) * F32(126)).astype(F32))
    return F32(s), np.stack([d1, d2, d3]).astype(np.int64)


def q8_digits(z_blocks):
    """lm_head_q8_kernel's split: per 32-input block s = max|z| / 127, digits
    in base 254."""
    mx = np.abs(z_blocks).max(axis=1).astype(F32)
    inv = np.where(mx > 0, F32(127) / np.where(mx > 0, mx, F32(1)), F32(0)).astype(F32)
    x = (z_blocks * inv[:, None]).astype(F32)
    d1 = _round(x)
    r1 = ((x - d1).astype(F32) * F32(254)).astype(F32)
    d2 = _round(r1)
    d3 = _round(((r1 - d2).astype(F32) * F32(254)).astype(F32))
    return (mx / F32(127)).astype(F32), np.stack([d1, d2, d3], axis=1).astype(np.int64)


def _fma(a, b, c):
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) +
            np.asarray(c, np.float64)).astype(F32)


def q6_logits(planes, n_rows, z):
    """The kernel's row arithmetic from the gqa_lm_head_pack planes: the ql and
    qh rows un-rotated, 6-bit codes assembled, per superblock and digit the
    exact integer K_k = sum_g scale_g * sum_i (code - 32) e_k over its 16
    groups of 16 weights (the tensor-core products, code - 32 by the
    accumulator's offset), the superblock's term (d s)(K1 + K2/126 +
    K3/126^2), the terms summed in pairs of superblocks (0+1, 2+3, 4+5, one
    warp each) and the pairs in order.  Returns (logits, max |K|)."""
    np_rows = (n_rows + 3) // 4 * 4
    ql = np.ascontiguousarray(planes[:np_rows * 768]).reshape(np_rows, 768)[:n_rows].copy()
    qh = np.ascontiguousarray(planes[np_rows * 768:np_rows * 1152]).reshape(np_rows, 384)[:n_rows].copy()
    sc = np.ascontiguousarray(planes[np_rows * 1152:np_rows * 1248]).view(np.int8).reshape(np_rows, 96)
    dd = np.ascontiguousarray(planes[np_rows * 1248:]).view(np.float16).reshape(np_rows, 6).astype(F32)
    for r in range(min(n_rows, 8)):
        sel = np.arange(r, n_rows, 8)
        ql[sel] = np.roll(ql[sel], -16 * r, axis=1)
        qh[sel] = np.roll(qh[sel], -16 * r, axis=1)
    s, e = q6_digits(z)
    assert np.abs(e).max() <= 63
    j = np.arange(256)
    n, rr = j // 128, j % 128
    c, l = rr // 32, rr % 32
    kmax = 0
    terms = []
    for sb in range(6):
        lo = ql[:, sb * 128 + 64 * n + 32 * (c & 1) + l].astype(np.int64)
        hi = qh[:, sb * 64 + 32 * n + l].astype(np.int64)
        code = ((lo >> (4 * (c >> 1))) & 15) | (((hi >> (2 * c)) & 3) << 4)   # [rows][256]
        scale = sc[:n_rows, sb * 16:sb * 16 + 16].astype(np.int64)            # [rows][16]
        k = np.zeros((n_rows, 3), np.int64)
        for kk in range(3):
            prod = (code - 32) * e[kk, sb * 256:sb * 256 + 256][None, :]
            k[:, kk] = (scale * prod.reshape(n_rows, 16, 16).sum(2)).sum(1)
        kmax = max(kmax, int(np.abs(k).max()))
        f = _fma(k[:, 2].astype(F32), F32(1 / 15876), _fma(k[:, 1].astype(F32), F32(1 / 126),
                                                          k[:, 0].astype(F32)))
        terms.append((f * (dd[:n_rows, sb] * s).astype(F32)).astype(F32))
    pairs = [(terms[2 * p] + terms[2 * p + 1]).astype(F32) for p in range(3)]
    return ((pairs[0] + pairs[1]).astype(F32) + pairs[2]).astype(F32), kmax


def _worst_q6(pkg, n):
    """Rows whose codes are all 0 or all 63 with scales -128 / 127, so every
    |code - 32| * |scale| is as large as the format allows."""
    w = pkg.seeded.q6_k_matrix(41, pkg.seeded.W_HEAD, n).reshape(n, 6, 210)
    for r in range(n):
        code_lo = 0x00 if r % 2 == 0 else 0xFF   # ql nibbles 0 or 15
        w[r, :, :128] = code_lo
        w[r, :, 128:192] = 0x00 if r % 2 == 0 else 0xFF  # qh: high bits 0 or 3
        w[r, :, 192:208] = 0x80 if r % 4 < 2 else 0x7F  # scales -128 or 127
    return w.reshape(-1)


def test_q6_digits_and_bounds(pkg, orc):
    S = pkg.seeded
    n = 64
    rng = np.random.default_rng(3)
    for w in (S.q6_k_matrix(31, S.W_HEAD, n), _worst_q6(pkg, n)):
        planes = S.q6_k_planes(w, n)
        dense = S.q6_k_dequant(w, n).astype(np.float64)
        for z in (S.normal(2, S.STATE, 1536),
                  np.full(1536, 63.0, F32),                       # at the digit range's edge
                  (np.sign(rng.standard_normal(1536)) * 63 * 2.0 ** rng.integers(-20, 20, 1536)
                   ).astype(F32),                                 # mixed powers of two
                  (rng.standard_normal(1536) * 1e-30).astype(F32)):  # tiny inputs
            got, kmax = q6_logits(planes, n, z)
            assert kmax < 2 ** 31 - 1
            want = dense @ z.astype(np.float64)
            err = np.abs(got - want).max() / max(np.sqrt(np.mean(want ** 2)), 1e-300)
            assert err <= 1e-5, err


def test_q6_unit_columns_bit_exact(pkg, orc):
    if not orc.have_reference():
        pytest.skip("oracle/_ref not built")
    S = pkg.seeded
    n = 48
    w = S.q6_k_matrix(11, S.W_HEAD, n)
    planes = S.q6_k_planes(w, n)
    for col in (0, 15, 16, 31, 32, 63, 64, 95, 96, 127, 128, 255, 512, 1024, 1535):
        z = np.zeros(1536, F32)
        z[col] = 32.0
        got, _ = q6_logits(planes, n, z)
        want = orc.ref_gemv_q6_k(w, z)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), col


def test_q8_digits_and_bounds(pkg):
    """The Q8_0 head: |I_k| = |sum_j q_j e_kj| <= 32 * 128 * 127 < 2^22 for
    any codes, and the three digits rebuild each input to about 1e-7 of its
    block's maximum."""
    rng = np.random.default_rng(5)
    assert 32 * 128 * 127 < LIMIT
    for z in (rng.standard_normal((28, 32)).astype(F32),
              np.full((28, 32), -3.5, F32),
              (rng.standard_normal((28, 32)) * 10.0 ** rng.integers(-6, 6, (28, 1))).astype(F32)):
        s, e = q8_digits(z)
        assert np.abs(e).max() <= 127
        rebuilt = s[:, None].astype(np.float64) * (e[:, 0] + e[:, 1] / 254.0 + e[:, 2] / 64516.0)
        assert np.all(np.abs(rebuilt - z) <= 2e-7 * np.abs(z).max(axis=1, keepdims=True))
        codes = np.where(rng.random((28, 32)) < 0.5, -128, 127)
        sums = (codes[:, None, :] * e).sum(axis=2)
        assert np.abs(sums).max() < LIMIT
