"""The attention-block oracle (the reference's decoder-layer step with zero
FFN weights) and the seeded Q4_0 weights, on the CPU."""
import numpy as np
import pytest


def q4_blocks(d, codes):
    """One Q4_0 row of blocks: d (fp16 scales) and codes [n_blocks][32] in 0..15."""
    codes = np.asarray(codes, dtype=np.uint8)
    nb = codes.shape[0]
    out = np.empty((nb, 18), dtype=np.uint8)
    out[:, 0:2] = np.asarray(d, dtype=np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = (codes[:, :16] & 15) | ((codes[:, 16:] & 15) << 4)
    return out.reshape(-1)


def test_q4_0_dequant_formula(pkg):
    codes = np.arange(32) % 16
    blk = q4_blocks([0.5], codes[None, :])
    w = pkg.seeded.q4_0_dequant(blk, 1, 32)
    assert np.array_equal(w[0], 0.5 * (codes - 8).astype(np.float32))


def test_q4_0_matrix_is_seeded(pkg):
    a = pkg.seeded.q4_0_matrix(3, pkg.seeded.W_O, 64, 1536, 0.01)
    b = pkg.seeded.q4_0_matrix(3, pkg.seeded.W_O, 64, 1536, 0.01)
    c = pkg.seeded.q4_0_matrix(4, pkg.seeded.W_O, 64, 1536, 0.01)
    assert a.shape == (64 * 48 * 18,) and np.array_equal(a, b) and not np.array_equal(a, c)
    d = a.reshape(-1, 18)[:, :2].copy().view(np.float16).astype(np.float32)
    assert np.all((d >= 0.005) & (d <= 0.015))


def _identity_q4(n):
    """W = I as Q4_0: code 9 (weight 1) on the diagonal, 8 (weight 0) elsewhere, d = 1."""
    codes = np.full((n, n // 32, 32), 8, dtype=np.uint8)
    for r in range(n):
        codes[r, r // 32, r % 32] = 9
    return q4_blocks(np.ones(n * (n // 32)), codes.reshape(-1, 32))


def test_block_oracle_reduces_to_the_pinned_attention(pkg, orc):
    """x_in = 0, gamma = 1, W_qkv = 0, b_qkv = qkv, W_o = I: the block is the
    attention slice, which must equal ref_layer_attention bit for bit."""
    if not orc.have_reference():
        pytest.skip("reference not compiled")
    qkv, kc, vc = pkg.seeded.decode_inputs(11, 4096)
    zero = q4_blocks(np.ones(2048 * 48), np.full((2048 * 48, 32), 8))
    k1, v1, k2, v2 = kc.copy(), vc.copy(), kc.copy(), vc.copy()
    y = orc.ref_attention_block(np.zeros(1536, np.float32), zero, qkv, _identity_q4(1536),
                                np.ones(1536, np.float32), k1, v1, 900, 901)
    want = orc.ref_layer_attention(qkv, k2, v2, 900, 901)
    assert np.array_equal(y, want)
    assert np.array_equal(k1, k2) and np.array_equal(v1, v2)


def test_block_oracle_matches_dense_restatement(pkg, orc):
    """The reference block against a float64 restatement with dense dequantised
    weights and the oracle's attention: RMSNorm, QKV + bias, RoPE/append,
    attention, Wo + residual."""
    if not orc.have_reference():
        pytest.skip("reference not compiled")
    x, wq, bq, wo, gamma, kc, vc = pkg.seeded.attention_block_inputs(12)
    pos = 2500
    k1, v1 = kc.copy(), vc.copy()
    y = orc.ref_attention_block(x, wq, bq, wo, gamma, k1, v1, pos, pos + 1)
    z = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6) * gamma
    qkv = (pkg.seeded.q4_0_dequant(wq, 2048, 1536).astype(np.float64) @ z + bq).astype(np.float32)
    k2, v2 = kc.copy(), vc.copy()
    orc.layer_attention(qkv, k2, v2, pos, pos + 1)
    want = x + (pkg.seeded.q4_0_dequant(wo, 1536, 1536).astype(np.float64) @ qkv[:1536])
    delta, wdelta = y - x, want - x
    assert np.abs(delta - wdelta).max() / np.sqrt(np.mean(wdelta ** 2)) <= 1e-4


def _silu(x):
    return np.where(x >= 0, x / (1 + np.exp(-np.abs(x))), x * np.exp(-np.abs(x)) / (1 + np.exp(-np.abs(x))))


def test_layer_oracle_ffn_matches_dense_restatement(pkg, orc):
    """With W_qkv = 0, b_qkv = 0, W_o = 0 the attention half adds exactly 0, so
    the reference layer is x + FFN(x); against a float64 restatement."""
    if not orc.have_reference():
        pytest.skip("reference not compiled")
    x, _, _, _, gamma_a, kc, vc = pkg.seeded.attention_block_inputs(21)
    zq = np.zeros(2048 * 48 * 18, np.uint8)
    zo = np.zeros(1536 * 48 * 18, np.uint8)
    wg, wu, wd, gf = pkg.seeded.ffn_block_inputs(21)
    y = orc.ref_decoder_layer(x, (zq, np.zeros(2048, np.float32), zo, gamma_a), (wg, wu, wd, gf),
                              kc.copy(), vc.copy(), 100, 101)
    z = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6) * gf
    g = pkg.seeded.q4_0_dequant(wg, 8960, 1536).astype(np.float64) @ z
    u = pkg.seeded.q4_0_dequant(wu, 8960, 1536).astype(np.float64) @ z
    want = x + pkg.seeded.q4_0_dequant(wd, 1536, 8960).astype(np.float64) @ (_silu(g) * u)
    assert np.abs((y - x) - (want - x)).max() / np.sqrt(np.mean((want - x) ** 2)) <= 1e-4


def test_layer_oracle_without_ffn_is_the_block_oracle(pkg, orc):
    if not orc.have_reference():
        pytest.skip("reference not compiled")
    x, wq, bq, wo, gamma, kc, vc = pkg.seeded.attention_block_inputs(22)
    zg = np.zeros(8960 * 48 * 18, np.uint8)
    zd = np.zeros(1536 * 280 * 18, np.uint8)
    y1 = orc.ref_decoder_layer(x, (wq, bq, wo, gamma), (zg, zg, zd, np.ones(1536, np.float32)),
                               kc.copy(), vc.copy(), 700, 701)
    y2 = orc.ref_attention_block(x, wq, bq, wo, gamma, kc.copy(), vc.copy(), 700, 701)
    assert np.array_equal(y1, y2)
