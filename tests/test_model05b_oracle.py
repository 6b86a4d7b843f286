"""The CPU side of the Qwen2.5-0.5B token step (no GPU): the layer oracle
composed from the reference's compiled size-generic GEMVs is pinned to the
compiled cpu_decoder_layer_step at the 1.5B sizes; the Q8_0 head restatement
(kernel_q8_0.cl:10-61) pinned bit for bit to the reference's own kernel source
run on the CPU, and against a float64 product; the byte layout that
gqa_lm_head_q8_0_pack writes; and a 0.5B-shaped GGUF file through the reader."""
import numpy as np
import pytest

import gguf_writer as gw


def _need_ref(orc):
    if not orc.have_reference():
        pytest.skip("oracle/_ref not built")


def test_composed_layer_equals_reference_layer(pkg, orc):
    """decoder_layer_sized at the 1.5B sizes == cpu_decoder_layer_step, bit for
    bit (output and both caches), at two positions."""
    _need_ref(orc)
    S = pkg.seeded
    state, w_qkv, b_qkv, w_o, g_a, kc, vc = S.attention_block_inputs(5)
    w_gate, w_up, w_down, g_f = S.ffn_block_inputs(5)
    attn, ffn = (w_qkv, b_qkv, w_o, g_a), (w_gate, w_up, w_down, g_f)
    for pos in (0, 700):
        k1, v1, k2, v2 = kc.copy(), vc.copy(), kc.copy(), vc.copy()
        want = orc.ref_decoder_layer(state, attn, ffn, k1, v1, pos, pos + 1)
        got = orc.decoder_layer_sized(state, attn, ffn, k2, v2, pos, pos + 1, 12, 2, 128, 8960)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert np.array_equal(k1, k2) and np.array_equal(v1, v2)


def test_reference_gemvs_at_05b_sizes(pkg, orc):
    """The compiled reference GEMVs at d_model 896 / d_ffn 4864 against a
    float64 product of the dequantised weights."""
    _need_ref(orc)
    S = pkg.seeded
    x = S.normal(4, S.STATE, 896)
    w = S.q4_0_matrix(4, S.W_QKV, 1152, 896, 1.0 / (4.6 * np.sqrt(896)))
    b = (0.1 * S.normal(4, S.B_QKV, 1152)).astype(np.float32)
    got = orc.ref_gemv_q4_0(w, x, b, 1152, 896)
    want = S.q4_0_dequant(w, 1152, 896).astype(np.float64) @ x + b
    assert np.abs(got - want).max() <= 1e-5 * np.sqrt(np.mean(want ** 2))
    wd = S.q4_0_matrix(4, S.W_DOWN, 896, 4864, 1.0 / (4.6 * np.sqrt(4864)))
    h = S.normal(4, S.HEAD_X, 4864)
    got = orc.ref_gemv_q4_0(wd, h, None, 896, 4864)
    want = S.q4_0_dequant(wd, 896, 4864).astype(np.float64) @ h
    assert np.abs(got - want).max() <= 1e-5 * np.sqrt(np.mean(want ** 2))


@pytest.mark.parametrize("seed", [3, 11])
def test_q8_0_restatement_equals_reference_kernel(pkg, orc, seed):
    """The restated Q8_0 GEMV == the reference's gemv_q8_0 (kernel_q8_0.cl,
    its OpenCL C compiled as C, each work-group's 128 work-items run to every
    barrier in turn), bit for bit: seeded weights and inputs, a row count that
    leaves a partial last work-group, extreme fp16 scales (subnormal, large,
    negative zero) and all-zero / saturated code blocks."""
    if not orc.have_reference_q8():
        pytest.skip("oracle/_ref not built")
    S = pkg.seeded
    n = 203  # 50 full groups of 4 rows and one of 3
    w = S.q8_0_matrix(seed, S.W_HEAD, n, 896).reshape(n, 28, 34).copy()
    x = S.normal(seed, S.HEAD_X, 896)
    w[1, 3, 0:2] = np.frombuffer(np.float16(6.0e-8).tobytes(), np.uint8)   # subnormal d
    w[2, 5, 0:2] = np.frombuffer(np.float16(-0.0).tobytes(), np.uint8)     # -0 d
    w[3, 7, 0:2] = np.frombuffer(np.float16(3.0e4).tobytes(), np.uint8)    # large d
    w[4, 9, 2:] = 0                                                         # zero codes
    w[5, 11, 2:] = 0x80                                                     # -128 codes
    w[6, 13, 2:] = 0x7F                                                     # 127 codes
    w = w.reshape(-1)
    got = orc.gemv_q8_0(w, x, n)
    want = orc.ref_gemv_q8_0(w, x, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q8_0_head_restatement(pkg, orc):
    S = pkg.seeded
    n = 3000
    w = S.q8_0_matrix(3, S.W_HEAD, n, 896)
    x = S.normal(3, S.HEAD_X, 896)
    got = orc.gemv_q8_0(w, x, n)
    want = S.q8_0_dequant(w, n).astype(np.float64) @ x.astype(np.float64)
    assert np.abs(got - want).max() <= 1e-6 * np.sqrt(np.mean(want ** 2))
    # with the output norm and the pick
    gamma = (1.0 + 0.1 * S.normal(3, S.GAMMA_OUT, 896)).astype(np.float32)
    logits, tok = orc.lm_head_q8_0(x, gamma, w, n)
    assert np.array_equal(logits, orc.gemv_q8_0(w, orc.output_norm(x, gamma), n))
    assert tok == int(np.argmax(logits))


def test_q8_0_planes_layout(pkg):
    """Reading the planes the way the head kernel addresses them gives back
    the dequantised matrix; padding rows are code 0 with scale 0."""
    S = pkg.seeded
    n = 1001
    w = S.q8_0_matrix(8, S.W_HEAD, n, 896)
    planes = S.q8_0_planes(w, n)
    np_rows = 1004
    assert planes.size == np_rows * 952
    qs = planes[:np_rows * 896].reshape(np_rows, 896)
    d = planes[np_rows * 896:].reshape(np_rows, 28, 2).copy().view(np.float16)[:, :, 0]
    dense = np.zeros((np_rows, 896), np.float32)
    for b in range(28):
        s, li = divmod(b, 14)
        for mq in range(2):
            at = 16 * ((2 * s + mq) * 14 + li)
            dense[:, 32 * b + 16 * mq:32 * b + 16 * mq + 16] = \
                qs[:, at:at + 16].view(np.int8).astype(np.float32) * d[:, b:b + 1].astype(np.float32)
    assert np.array_equal(dense[:n], S.q8_0_dequant(w, n))
    assert (qs[n:] == 0).all() and (d[n:] == 0).all()


def test_gguf_05b_file(pkg, orc, tmp_path):
    """A 0.5B-shaped file (Q8_0 head, 896-wide rows) reads back through the
    library's reader with the shapes the loader checks; the reference's
    parser agrees on the table."""
    path = tmp_path / "q05.gguf"
    offsets, arrays = gw.qwen_model(path, pkg.seeded, n_layers=2, vocab=300, seed=4,
                                    model="0.5b")
    with pkg.Gguf(str(path)) as g:
        t = g.find("output.weight")
        assert t["type"] == gw.T_Q8_0 and t["ne"] == [896, 300] and t["bytes"] == 300 * 952
        assert np.array_equal(g.read("output.weight"), arrays["head"])
        t = g.find("blk.1.ffn_down.weight")
        assert t["ne"] == [4864, 896] and t["bytes"] == 896 * 152 * 18
        assert g.find("blk.0.attn_k.weight")["ne"] == [896, 128]
        if orc.have_reference():
            ref, _ = orc.ref_gguf_parse(str(path))
            assert [(r["name"], r["offset"]) for r in ref] == \
                   [(x["name"], x["offset"]) for x in g.tensors()]
