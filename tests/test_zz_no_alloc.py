"""The layer call that allocates nothing (gqa_layer_attention_static).

It exists for callers that cannot allocate device memory while they run the
layer call (host callbacks, plugins whose framework owns all device memory).
It must give the same result as the context-based gqa_layer_attention; it is
checked here through the C ABI on two calls in a row, since the static scratch
keeps the previous call's contents.  This file sorts last so that a failure
here never hides the other tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # normalised max error, as for every fp32 decode test


def nerr(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(np.asarray(got, dtype=np.float64) - ref).max() /
                 max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def test_static_scratch_call_matches_context_call_twice(pkg, orc, cuda):
    torch = cuda
    lib = pkg.lib()
    t_max = 4096
    cfg = pkg.gqa.Config(12, 2, 128, t_max, 1e6)
    stream = torch.cuda.current_stream().cuda_stream
    with pkg.Context(t_max=t_max) as ctx:
        for seed, pos, seq_len in [(51, 4095, 4096), (52, 700, 701)]:
            qkv, kc, vc = pkg.seeded.decode_inputs(seed, t_max)
            # existing entry point
            a_qkv = torch.from_numpy(qkv.copy()).cuda()
            a_k, a_v = torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda()
            ctx.layer_attention(pkg.kv_of(a_k, a_v), a_qkv, pos, seq_len)
            # the allocation-free entry point, through the C ABI
            b_qkv = torch.from_numpy(qkv.copy()).cuda()
            b_k, b_v = torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda()
            kv = pkg.kv_of(b_k, b_v)
            rc = lib.gqa_layer_attention_static(ctypes.byref(cfg), stream, ctypes.byref(kv),
                                                b_qkv.data_ptr(), pos, seq_len)
            assert rc == 0, pkg.last_error()
            torch.cuda.synchronize()
            a, b = a_qkv[:1536].cpu().numpy(), b_qkv[:1536].cpu().numpy()
            assert nerr(b, a) <= TOL, (seed, pos)
            assert np.array_equal(b_qkv[1536:].cpu().numpy(), qkv[1536:])
            assert np.abs(b_k.cpu().numpy() - a_k.cpu().numpy()).max() <= 1e-5
            assert np.array_equal(b_v.cpu().numpy(), a_v.cpu().numpy())
            # and both match the oracle
            rq = qkv.copy()
            orc.layer_attention(rq, kc.copy(), vc.copy(), pos, seq_len)
            assert nerr(b, rq[:1536]) <= TOL


def test_static_scratch_call_rejects_bad_arguments(pkg, cuda):
    torch = cuda
    lib = pkg.lib()
    cfg = pkg.gqa.Config(12, 2, 128, 256, 1e6)
    k = torch.zeros((2, 256, 128), device="cuda")
    v = torch.zeros((2, 256, 128), device="cuda")
    qkv = torch.zeros(2048, device="cuda")
    kv = pkg.kv_of(k, v)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.gqa_layer_attention_static(ctypes.byref(cfg), stream, ctypes.byref(kv),
                                          qkv.data_ptr(), 256, 257) == pkg.gqa.GQA_ERR_INVALID_ARG
    bad = pkg.gqa.Config(12, 2, 64, 256, 1e6)
    assert lib.gqa_layer_attention_static(ctypes.byref(bad), stream, ctypes.byref(kv),
                                          qkv.data_ptr(), 0, 1) == pkg.gqa.GQA_ERR_UNSUPPORTED


def test_static_scratch_theta_changes_are_stream_ordered(pkg, orc, cuda):
    """Calls queued back to back on one non-blocking stream, alternating two
    rope_theta values, with no synchronisation between them: each call must
    use its own RoPE table (the table is rewritten on the caller's stream)."""
    torch = cuda
    lib = pkg.lib()
    t_max = 1024
    cases = [(61, 1e6, 1000), (62, 1e4, 700), (63, 1e6, 1023), (64, 1e4, 300)]
    stream = torch.cuda.Stream()
    bufs = []
    for seed, theta, pos in cases:
        qkv, kc, vc = pkg.seeded.decode_inputs(seed, t_max)
        d = (torch.from_numpy(qkv.copy()).cuda(), torch.from_numpy(kc.copy()).cuda(),
             torch.from_numpy(vc.copy()).cuda())
        bufs.append((qkv, kc, vc, d))
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for (seed, theta, pos), (_, _, _, d) in zip(cases, bufs):
            cfg = pkg.gqa.Config(12, 2, 128, t_max, theta)
            kv = pkg.kv_of(d[1], d[2])
            rc = lib.gqa_layer_attention_static(ctypes.byref(cfg), stream.cuda_stream,
                                                ctypes.byref(kv), d[0].data_ptr(), pos, pos + 1)
            assert rc == 0, pkg.last_error()
    stream.synchronize()
    for (seed, theta, pos), (qkv, kc, vc, d) in zip(cases, bufs):
        rq = qkv.copy()
        orc.layer_attention(rq, kc.copy(), vc.copy(), pos, pos + 1, rope_base=theta)
        assert nerr(d[0][:1536].cpu().numpy(), rq[:1536]) <= TOL, (seed, theta)
    st = ctypes.c_int(-1)
    assert lib.gqa_static_status(torch.cuda.current_device(), ctypes.byref(st), 1) == 0
    assert st.value == 0


def test_static_status_arguments(pkg, cuda):
    lib = pkg.lib()
    st = ctypes.c_int(-1)
    assert lib.gqa_static_status(0, None, 0) == pkg.gqa.GQA_ERR_INVALID_ARG
    assert lib.gqa_static_status(-1, ctypes.byref(st), 0) == pkg.gqa.GQA_ERR_INVALID_ARG
    assert lib.gqa_static_status(0, ctypes.byref(st), 0) == 0 and st.value == 0
