"""The fused argmax + greedy-walk kernel (one launch) on caller device logits,
through cwen_cuda_accept_logits, against the reference's own argmax_of
(run.c:2647-2669, compiled into oracle/_ref) and its walk (run.c:4954-4959).

argmax_of scans with a strict `>` from bv = lg[0]: ties go to the lowest
index, -0.0 and +0.0 compare equal, a NaN never replaces the running
maximum, and a NaN at index 0 is never replaced.  Every row is built to hit
one of those cases; the walk compares row j's argmax with blk[j+1].
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import vp

pytestmark = pytest.mark.gpu

V = 248320  # the reference's argmax_of scans its compiled-in vocabulary


@pytest.fixture(scope="module")
def eng():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, 64, 16), "init")
    yield L
    L.cwen_cuda_shutdown()


def _ref():
    import bench
    path, _ = bench.ref_lib_path()
    if not path.exists():
        pytest.skip("oracle/_ref reference build missing")
    ref = C.CDLL(str(path))
    ref.cwref_argmax.argtypes = [C.c_void_p]
    ref.cwref_argmax.restype = C.c_int
    return ref


def _rows(rng, B):
    lg = rng.standard_normal((B, V)).astype(np.float32)
    special = []
    # 0: plain random
    # 1: the maximum planted at three indices -> the lowest
    lg[1, [9000, 77, 200000]] = 50.0
    # 2: all negative except -0.0 at 3 and +0.0 at 7 -> 3 (they compare equal)
    lg[2] = -np.abs(lg[2]) - 1.0
    lg[2, 3] = -0.0
    lg[2, 7] = 0.0
    # 3: +0.0 first, -0.0 later -> the +0.0
    lg[3] = -np.abs(lg[3]) - 1.0
    lg[3, 11] = 0.0
    lg[3, 12] = -0.0
    # 4: NaNs inside, one above the true maximum's position
    lg[4, [5, 1000, 123456]] = np.nan
    lg[4, 1001] = 40.0
    # 5: NaN at index 0 -> 0
    lg[5, 0] = np.nan
    lg[5, 17] = 99.0
    # 6: all -inf -> 0
    lg[6] = -np.inf
    # 7: +inf at two places -> the first
    lg[7, [4321, 22]] = np.inf
    # 8: the maximum in the last element
    lg[8, V - 1] = 60.0
    return lg, special


def test_fused_accept_matches_reference_argmax(eng):
    import torch

    import cwen_b200
    L = eng
    ref = _ref()
    rng = np.random.default_rng(42)
    B = 9
    lg, _ = _rows(rng, B)
    want = [ref.cwref_argmax(vp(np.ascontiguousarray(lg[b]))) for b in range(B)]
    assert want[1] == 77 and want[2] == 3 and want[3] == 11 and want[4] == 1001
    assert want[5] == 0 and want[6] == 0 and want[7] == 22 and want[8] == V - 1
    dlg = torch.from_numpy(lg).cuda()
    torch.cuda.synchronize()
    res = np.zeros(2 + B, np.int32)
    # walk: drafts agree with rows 0..4, disagree at row 5
    for k_want in (0, 3, 5, B - 1):
        blk = np.zeros(B, np.int32)
        blk[0] = 1234
        for j in range(B - 1):
            blk[j + 1] = want[j] if j < k_want else (want[j] + 1) % V
        cwen_b200.check(L.cwen_cuda_accept_logits(C.c_void_p(dlg.data_ptr()), V, V, B, vp(blk), B - 1, vp(res), None),
                        "accept_logits")
        assert list(res[2:]) == want
        assert res[0] == k_want and res[1] == want[k_want], (k_want, res[:2])
    # no drafts: ustar is row 0's argmax
    cwen_b200.check(L.cwen_cuda_accept_logits(C.c_void_p(dlg.data_ptr()), V, V, 1, None, 0, vp(res), None))
    assert res[0] == 0 and res[1] == want[0] and res[2] == want[0]
    # strided rows (ldl > n): a prefix of each row
    n = 100000
    cwen_b200.check(L.cwen_cuda_accept_logits(C.c_void_p(dlg.data_ptr()), n, V, B, None, 0, vp(res), None))
    for b in range(B):
        row = lg[b, :n]
        bi, bv = 0, row[0]
        for i in np.flatnonzero(row > bv):  # numpy restatement of the strict scan (prefix maxima)
            if row[i] > bv:
                bi, bv = int(i), row[i]
        assert res[2 + b] == bi, (b, res[2 + b], bi)


def test_fused_accept_rejects_bad_arguments(eng):
    L = eng
    res = np.zeros(20, np.int32)
    assert L.cwen_cuda_accept_logits(None, 10, 10, 1, None, 0, vp(res), None) == -1
    x = np.zeros(1, np.int32)
    assert L.cwen_cuda_accept_logits(C.c_void_p(16), 10, 10, 2, None, 1, vp(res), None) == -1  # E > 0 needs blk
    assert L.cwen_cuda_accept_logits(C.c_void_p(16), 10, 10, 17, vp(x), 0, vp(res), None) == -1
    assert L.cwen_cuda_accept_logits(C.c_void_p(16), 10, 10, 2, vp(x), 2, vp(res), None) == -1  # E < B
