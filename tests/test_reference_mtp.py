"""MTP drafter at the full 27B geometry (blk.64 Q8_0) against the reference
itself (maci0/cwen run.c compiled into oracle/_ref: its mtp_commit /
mtp_draft, run.c:3147-3187) and the CPU oracle's restatement of them.

The same seeded weights and prompt go through the three implementations;
each folds every prompt slot into the nextn stream and drafts 3 tokens after
it.  Where the oracle and the reference agree (fp32 reassociation can flip a
near-tied argmax in a random-init model), the engine must draft the same
tokens; the oracle must agree with the reference on at least the first
draft, which pins its MTP restatement.
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import CwDims, load_oracle, vp

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 21
CTX = 64
NTOK = 3
ND = 3


def test_mtp_full_geometry_matches_reference():
    import bench
    import cwen_b200
    from cwen_b200 import build
    path, _ = bench.ref_lib_path()
    if not path.exists():
        pytest.skip("oracle/_ref reference build missing (oracle/build_ref.sh)")
    build.build()
    toks = np.random.default_rng(31).integers(0, 248320, size=NTOK).astype(np.int32)

    ref = C.CDLL(str(path))
    ref.cwref_mtp_commit.argtypes = [C.c_int, C.c_int, C.c_void_p]
    ref.cwref_mtp_draft.argtypes = [C.c_int, C.c_void_p, C.c_int]
    assert ref.cwref_load_synth(C.c_uint64(SEED), 1, 0) == 0
    ref.cwref_alloc_state(CTX, 1, 1)
    ref.cwref_reset_state()
    H, V = 5120, 248320
    xr = np.zeros(H, np.float32)
    lg = np.zeros(V, np.float32)
    for p, t in enumerate(toks):
        ref.cwref_set_pos(p)
        ref.cwref_forward_ex(int(t), 1)
        ref.cwref_get_x(vp(xr))
        ref.cwref_mtp_commit(p, int(t), vp(xr))
    ref.cwref_get_logits(vp(lg))
    rpend = int(np.argmax(lg))
    rdraft = np.zeros(16, np.int32)
    assert ref.cwref_mtp_draft(rpend, vp(rdraft), ND) == ND

    orc = load_oracle()
    orc.or_mtp_commit.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    orc.or_mtp_draft.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
    orc.or_mtp_draft.restype = C.c_int
    od = CwDims()
    orc.cw_dims_full(C.byref(od))
    od.has_mtp = 1
    om = orc.or_model_synth(C.byref(od), SEED, CTX, 0)
    assert om
    try:
        for p, t in enumerate(toks):
            orc.or_forward(om, int(t), p, 1)
            orc.or_mtp_commit(om, p, int(t), orc.or_hidden(om))
        opend = int(np.argmax(np.ctypeslib.as_array(orc.or_logits(om), shape=(V,))))
        odraft = np.zeros(16, np.int32)
        assert orc.or_mtp_draft(om, NTOK - 1, opend, vp(odraft), ND) == ND
    finally:
        orc.or_model_free(om)

    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, CTX, 16), "init")
    try:
        d = cwen_b200.dims("reference")
        d.has_mtp = 1
        cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 0), "load_synth")
        assert L.cwen_cuda_mtp_ready() == 1
        cwen_b200.check(L.cwen_cuda_reset())
        for p, t in enumerate(toks):
            am = C.c_int(-1)
            cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, C.byref(am)), "forward_serial")
            cwen_b200.check(L.cwen_cuda_mtp_commit(p, int(t), 0), "mtp_commit")
        epend = am.value
        edraft = np.zeros(16, np.int32)
        assert L.cwen_cuda_mtp_draft(epend, vp(edraft), ND) == ND
    finally:
        L.cwen_cuda_shutdown()

    print(f"pend ref {rpend} oracle {opend} engine {epend}; drafts ref {list(rdraft[:ND])} "
          f"oracle {list(odraft[:ND])} engine {list(edraft[:ND])}")
    assert opend == rpend and odraft[0] == rdraft[0]
    agree = 0
    while agree < ND and odraft[agree] == rdraft[agree]:
        agree += 1
    assert epend == rpend
    assert list(edraft[:agree]) == list(rdraft[:agree])
