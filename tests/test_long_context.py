"""Attention at a long context on the small seeded geometry, through the C ABI:
a verify block whose rows straddle slot 4096, where a row's KV splits grow
from 64 to 128 slots (rows 4088..4095 use 64-slot splits, rows 4096..4103
128-slot ones, in one launch), against the CPU oracle's serial forward at
the same slots: per-row logits rel L2 <= 1e-3 (the
softmax sums over ~4,100 slots in a different order).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import CwDims, rel_l2, vp

pytestmark = pytest.mark.gpu

SEED = 7
CTX = 4352
PROMPT = 4088


@pytest.fixture(scope="module")
def eng_long():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, CTX, 16), "init")
    d = cwen_b200.dims("small")
    cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 0), "load_synth")
    yield L, d
    L.cwen_cuda_shutdown()


def test_block_across_split_growth_matches_oracle(eng_long, orc):
    import cwen_b200
    L, d = eng_long
    od = CwDims()
    orc.cw_dims_tiny(C.byref(od))
    om = orc.or_model_synth(C.byref(od), SEED, CTX, 0)
    assert om
    try:
        ids = np.random.default_rng(11).integers(0, d.n_vocab, size=PROMPT + 16).astype(np.int32)
        cwen_b200.check(L.cwen_cuda_reset())
        for a in range(0, PROMPT, 16):  # prefill: blocks of up to 16 rows, every row kept
            n = min(16, PROMPT - a)
            blk = np.ascontiguousarray(ids[a:a + n])
            cwen_b200.check(L.cwen_cuda_forward_block(vp(blk), n, 0), "forward_block")
            cwen_b200.check(L.cwen_cuda_commit(n - 1), "commit")
        blk = np.ascontiguousarray(ids[PROMPT:PROMPT + 16])
        cwen_b200.check(L.cwen_cuda_forward_block(vp(blk), 16, 16), "verify block")
        orc.or_reset(om)
        for p in range(PROMPT):
            orc.or_forward(om, int(ids[p]), p, 0)
        lg = np.zeros(d.n_vocab, np.float32)
        for j in range(16):
            orc.or_forward(om, int(ids[PROMPT + j]), PROMPT + j, 1)
            ref = np.ctypeslib.as_array(orc.or_logits(om), shape=(d.n_vocab,)).copy()
            cwen_b200.check(L.cwen_cuda_logits(j, vp(lg)), "logits")
            assert rel_l2(lg, ref) <= 1e-3, (PROMPT + j, rel_l2(lg, ref))
    finally:
        orc.or_model_free(om)
