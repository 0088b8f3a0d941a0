"""cwen_cuda_gemvb_static: the verify GEMV that allocates nothing.

Some callers cannot call cudaMalloc while they run -- a framework whose
caching allocator already holds the device memory, or a latency-critical
loop where an allocation would synchronize the device.  This entry point
runs the GEMV on scratch that is a fixed array of device memory inside the
library.  It takes the same kernel path as the regular entry point
(cwen_cuda_gemvb), so on the same weights and inputs its output must be
bit-identical to it, on consecutive calls that reuse the shared scratch; and
both must match the CPU oracle within test_gemv.py's tolerance: max abs <=
1e-4 (scaled by the output magnitude) and relative L2 <= 1e-5.

This file is collected last on purpose, so a first-failure run has already
run every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import gen_normal, gen_q, rel_l2, vp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, 64, 16), "init")
    yield L
    L.cwen_cuda_shutdown()


def _close(got, ref):
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max() / 10), np.abs(got - ref).max()
    assert rel_l2(got, ref) <= 1e-5, rel_l2(got, ref)


@pytest.mark.parametrize("typ,K,M", [(2, 5120, 17408), (8, 17408, 5120), (2, 1024, 48)])
def test_static_scratch_matches_gemvb(eng, orc, typ, K, M):
    import torch

    import cwen_b200
    L = eng
    W = gen_q(orc, 21, f"na_w{K}x{M}", typ, K, M)
    wid = C.c_int(-1)
    cwen_b200.check(L.cwen_cuda_weight_upload(typ, W.ctypes.data_as(C.c_void_p), K, M, C.byref(wid)), "upload")
    dev = torch.device("cuda", 0)
    stream = C.c_void_p(L.cwen_cuda_stream())
    # two calls in a row with different inputs and batch sizes: the second
    # reuses the scratch the first one left behind
    for call, B in enumerate((8, 13)):
        Xh = gen_normal(orc, 22 + call, f"na_x{K}", B * K).reshape(B, K)
        X = torch.from_numpy(Xh).to(dev)
        Y_ref = torch.full((B, M), float("nan"), device=dev)
        Y = torch.full((B, M), float("nan"), device=dev)
        torch.cuda.synchronize()  # the fills ran on torch's stream, the GEMVs run on the engine's
        cwen_b200.check(L.cwen_cuda_gemvb(wid.value, C.c_void_p(X.data_ptr()), K, C.c_void_p(Y_ref.data_ptr()), M, B,
                                          stream), "gemvb")
        cwen_b200.check(L.cwen_cuda_gemvb_static(wid.value, C.c_void_p(X.data_ptr()), K, C.c_void_p(Y.data_ptr()), M,
                                                 B, stream), "gemvb_static")
        cwen_b200.check(L.cwen_cuda_gemvb_static_status(stream), "gemvb_static_status")
        torch.cuda.synchronize()
        got, reg = Y.cpu().numpy(), Y_ref.cpu().numpy()
        assert np.array_equal(got, reg), "static-scratch GEMV differs from cwen_cuda_gemvb"
        ref = np.zeros((B, M), np.float32)
        orc.or_gemvb(typ, vp(W), K, M, vp(np.ascontiguousarray(Xh)), K, vp(ref), M, B)
        _close(got, ref)


def test_static_scratch_rejects_oversize(eng, orc):
    import torch

    import cwen_b200
    L = eng
    # 1,048,832 rows: accepted by the engine, beyond the static scratch's 1,048,576
    K, M = 64, 4097 * 256
    W = gen_q(orc, 23, "na_big", 2, K, M)
    wid = C.c_int(-1)
    cwen_b200.check(L.cwen_cuda_weight_upload(2, W.ctypes.data_as(C.c_void_p), K, M, C.byref(wid)), "upload")
    X = torch.zeros((17, K), device="cuda")
    Y = torch.zeros((17, M), device="cuda")
    torch.cuda.synchronize()  # the zero fills ran on torch's stream
    rc = L.cwen_cuda_gemvb_static(wid.value, C.c_void_p(X.data_ptr()), K, C.c_void_p(Y.data_ptr()), M, 1, None)
    assert rc == -1 and b"static scratch" in L.cwen_cuda_last_error()
    rc = L.cwen_cuda_gemvb_static(wid.value, C.c_void_p(X.data_ptr()), K, C.c_void_p(Y.data_ptr()), M, 17, None)
    assert rc == -1
    # the regular entry point still handles the shape
    cwen_b200.check(L.cwen_cuda_gemvb(wid.value, C.c_void_p(X.data_ptr()), K, C.c_void_p(Y.data_ptr()), M, 1, None))
    torch.cuda.synchronize()
    assert L.cwen_cuda_gemvb_static_status(None) == 0
