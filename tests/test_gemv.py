"""Verify GEMV (a): CUDA path vs the CPU oracle and the reference goldens,
through the C ABI (include/cwen_cuda.h), plus batch invariance -- for every
kernel an engine can run (the warp-level mma.sync kernel, the default; qmv
with CWEN_GEMV=qmv and the tcgen05 kernel with CWEN_GEMV=tcgen05, selected at
cwen_cuda_init).

Tolerance: the reference's gemv acceptance, max_abs <= 1e-4 (run.c:4352),
and relative L2 <= 1e-5 (the kernel computes X as f16 hi+lo, ~2^-22
relative, with fp32 accumulation).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import gen_normal, gen_q, oracle_gemvb, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["mma", "qmv", "tcgen05"])
def eng(request):
    import os

    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    old = os.environ.get("CWEN_GEMV")
    os.environ["CWEN_GEMV"] = request.param
    try:
        cwen_b200.check(L.cwen_cuda_init(0, 64, 16), "init")
    finally:
        if old is None:
            os.environ.pop("CWEN_GEMV")
        else:
            os.environ["CWEN_GEMV"] = old
    yield L
    L.cwen_cuda_shutdown()


def _upload(L, typ, W, K, M):
    import cwen_b200
    wid = C.c_int(-1)
    cwen_b200.check(L.cwen_cuda_weight_upload(typ, W.ctypes.data_as(C.c_void_p), K, M, C.byref(wid)), "upload")
    return wid.value


def _gemv(L, wid, X, M):
    import cwen_b200
    B, K = X.shape
    X = np.ascontiguousarray(X, np.float32)
    Y = np.full((B, M), np.nan, np.float32)
    cwen_b200.check(L.cwen_cuda_gemvb_host(wid, X.ctypes.data_as(C.c_void_p), K, Y.ctypes.data_as(C.c_void_p), M, B),
                    "gemvb")
    return Y


# Work-split paths the shapes reach (one CTA per SM, 148 SMs):
#   (2, 512, 96), (2, 1024, 48): one tile split 2 / 4 ways -> cluster reduction, local X
#   (2, 5120, 34816): 68 tiles x 2 (gate_up) -> cluster reduction, prepared X (40 k-pairs per CTA)
#   (2, 5120, 16480): 33 tiles x 4 (GDN in_proj) -> cluster reduction, local X
#   (2, 17408, 5120), (2, 6144, 5120), (2, 5120, 17408): 10 / 10 / 34 tiles -> global reduction, local X
#   (2, 512, 102400): 200 tiles > CTAs -> stream-K, prepared X
#   (2, 256, 10240): 20 tiles, one CTA each -> no split, local X
#   (8, ...): Q8_0 -> prepared X
SHAPES = [(2, 512, 96), (2, 1024, 48), (8, 512, 64), (2, 5120, 64), (2, 5120, 1040), (8, 10240, 5120),
          (2, 17408, 5120), (2, 5120, 17408), (2, 6144, 5120), (2, 5120, 34816), (2, 5120, 16480),
          (2, 512, 102400), (2, 256, 10240)]


@pytest.mark.parametrize("typ,K,M", SHAPES)
def test_gemv_vs_oracle(eng, orc, typ, K, M):
    W = gen_q(orc, 3, f"w{K}x{M}", typ, K, M)
    X = gen_normal(orc, 4, f"x{K}", 16 * K).reshape(16, K)
    wid = _upload(eng, typ, W, K, M)
    for B in (1, 3, 8, 9, 16):
        got = _gemv(eng, wid, X[:B], M)
        ref = oracle_gemvb(orc, typ, W, K, M, X[:B])
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max() / 10), (B, np.abs(got - ref).max())
        assert rel_l2(got, ref) <= 1e-5, (B, rel_l2(got, ref))


def test_gemv_vs_reference_goldens(eng, orc, golden):
    for ti in range(4):
        typ, K, M, wseed, xseed = golden[f"gemv{ti}_meta"].tolist()
        W = gen_q(orc, wseed, f"gw{ti}", typ, K, M)
        X = gen_normal(orc, xseed, f"gx{ti}", 16 * K).reshape(16, K)
        wid = _upload(eng, typ, W, K, M)
        for B in (1, 2, 8, 9, 16):
            got = _gemv(eng, wid, X[:B], M)
            ref = golden[f"gemv{ti}_B{B}"]
            assert np.abs(got - ref).max() <= 1e-4, (ti, B)
            assert rel_l2(got, ref) <= 1e-5, (ti, B)


@pytest.mark.parametrize("typ,K,M", [(2, 5120, 17408), (8, 512, 64), (2, 17408, 5120), (2, 5120, 34816),
                                     (2, 5120, 16480)])
def test_gemv_batch_invariant(eng, orc, typ, K, M):
    """Column b of a B-row call is bit-identical to a 1-row call on row b."""
    W = gen_q(orc, 5, "binv", typ, K, M)
    X = gen_normal(orc, 6, "binvx", 16 * K).reshape(16, K) * 3.0
    wid = _upload(eng, typ, W, K, M)
    singles = [_gemv(eng, wid, X[b:b + 1], M)[0] for b in range(16)]
    for B in (2, 7, 8, 9, 16):
        Y = _gemv(eng, wid, X[:B], M)
        for b in range(B):
            assert np.array_equal(Y[b].view(np.uint32), singles[b].view(np.uint32)), (B, b)


def test_gemv_extreme_magnitudes(eng, orc):
    """Per-column power-of-two scaling keeps f16 hi/lo exact across ranges."""
    K, M = 1024, 64
    W = gen_q(orc, 8, "ext", 2, K, M)
    X = gen_normal(orc, 9, "extx", 4 * K).reshape(4, K)
    X[0] *= 1e4
    X[1] *= 1e-6
    X[2, ::7] = 0.0
    X[3] = 0.0
    wid = _upload(eng, 2, W, K, M)
    got = _gemv(eng, wid, X, M)
    ref = oracle_gemvb(orc, 2, W, K, M, X)
    for b in range(3):
        assert rel_l2(got[b], ref[b]) <= 1e-5, b
    assert np.all(got[3] == 0)
