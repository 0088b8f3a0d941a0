"""MTP (nextn) drafter on the device vs the CPU oracle, small seeded model
with the MTP block (blk.<n_layer>, Q8_0 matrices), through the C ABI.

- after a prompt folded into the nextn stream, the device drafts the same
  tokens as the oracle's mtp_draft (run.c:3166-3187) and the last draft
  step's logits agree to rel L2 <= 1e-4 (fp32 math, X split f16 hi+lo);
- speculative generation with the MTP drafter emits exactly the serial
  stream (drafts only decide what is verified, never what is emitted).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import CwDims, rel_l2, vp

pytestmark = pytest.mark.gpu

SEED = 5
CTX = 256


@pytest.fixture(scope="module")
def mtp_model():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, CTX, 16), "init")
    d = cwen_b200.dims("small")
    d.has_mtp = 1
    cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 0), "load_synth")
    yield L, d
    L.cwen_cuda_shutdown()


def _oracle(orc):
    orc.or_mtp_commit.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    orc.or_mtp_draft.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
    orc.or_mtp_draft.restype = C.c_int
    orc.or_mtp_logits.argtypes = [C.c_void_p]
    orc.or_mtp_logits.restype = C.POINTER(C.c_float)
    d = CwDims()
    orc.cw_dims_tiny(C.byref(d))
    d.has_mtp = 1
    m = orc.or_model_synth(C.byref(d), SEED, CTX, 0)
    assert m
    return d, m


def test_mtp_ready(mtp_model):
    L, _ = mtp_model
    assert L.cwen_cuda_mtp_ready() == 1


def test_mtp_draft_matches_oracle(mtp_model, orc):
    import cwen_b200
    L, d = mtp_model
    od, om = _oracle(orc)
    try:
        toks = np.random.default_rng(3).integers(0, d.n_vocab, size=10).astype(np.int32)
        # engine: prefill as one verify block, fold every slot into the nextn stream
        cwen_b200.check(L.cwen_cuda_reset())
        cwen_b200.check(L.cwen_cuda_forward_block(vp(toks), len(toks), -1), "forward_block")
        pend = C.c_int(-1)
        cwen_b200.check(L.cwen_cuda_accept(None, C.byref(pend), None), "accept")
        cwen_b200.check(L.cwen_cuda_commit(len(toks) - 1), "commit")
        for p, t in enumerate(toks):
            cwen_b200.check(L.cwen_cuda_mtp_commit(p, int(t), p), "mtp_commit")
        # oracle: serial forward + mtp_commit per slot
        orc.or_reset(om)
        for p, t in enumerate(toks):
            orc.or_forward(om, int(t), p, 1)
            orc.or_mtp_commit(om, p, int(t), orc.or_hidden(om))
        opend = int(np.argmax(np.ctypeslib.as_array(orc.or_logits(om), shape=(d.n_vocab,))))
        assert pend.value == opend
        for nd in (1, 4):
            out = np.zeros(16, np.int32)
            n = L.cwen_cuda_mtp_draft(pend.value, vp(out), nd)
            assert n == nd, cwen_b200.lib().cwen_cuda_last_error()
            oout = np.zeros(16, np.int32)
            on = orc.or_mtp_draft(om, len(toks) - 1, opend, vp(oout), nd)
            assert on == nd
            assert list(out[:n]) == list(oout[:on])
            lg = np.zeros(d.n_vocab, np.float32)
            cwen_b200.check(L.cwen_cuda_logits(0, vp(lg)), "logits")
            olg = np.ctypeslib.as_array(orc.or_mtp_logits(om), shape=(d.n_vocab,))
            assert rel_l2(lg, olg) <= 1e-4, rel_l2(lg, olg)
    finally:
        orc.or_model_free(om)


def test_mtp_spec_equals_serial(mtp_model):
    import cwen_b200
    L, d = mtp_model
    prompt = np.random.default_rng(9).integers(0, d.n_vocab, size=24).astype(np.int32)
    serial, _ = cwen_b200.generate(prompt, 48, cwen_b200.spec_cfg(spec=0))
    for md in (3, 8):
        spec, st = cwen_b200.generate(prompt, 48, cwen_b200.spec_cfg(spec=1, use_mtp=1, max_draft=md))
        assert np.array_equal(serial, spec), md
        assert st.drafted > 0


def _fold_and_draft(L, toks, cuts, blockwise, nd=4):
    """Prefill `toks` as verify blocks split at `cuts`, folding each block
    into the nextn stream row by row or in one block commit; return the
    draft tokens and the last draft step's logits."""
    import cwen_b200
    cwen_b200.check(L.cwen_cuda_reset())
    pend = C.c_int(-1)
    edges = [0] + list(cuts) + [len(toks)]
    for a, b in zip(edges[:-1], edges[1:]):
        blk = np.ascontiguousarray(toks[a:b])
        cwen_b200.check(L.cwen_cuda_forward_block(vp(blk), b - a, -1), "forward_block")
        cwen_b200.check(L.cwen_cuda_accept(None, C.byref(pend), None), "accept")
        cwen_b200.check(L.cwen_cuda_commit(b - a - 1), "commit")
        if blockwise:
            cwen_b200.check(L.cwen_cuda_mtp_commit_block(a, vp(blk), b - a), "mtp_commit_block")
        else:
            for j in range(b - a):
                cwen_b200.check(L.cwen_cuda_mtp_commit(a + j, int(blk[j]), j), "mtp_commit")
    out = np.zeros(16, np.int32)
    n = L.cwen_cuda_mtp_draft(pend.value, vp(out), nd)
    assert n == nd, L.cwen_cuda_last_error()
    return out[:n].copy(), pend.value


def test_mtp_commit_block_equals_rows(mtp_model):
    """One block commit gives the bits of n row commits in order: the nextn
    steps are batch-invariant and attend causally over the nextn cache."""
    import cwen_b200
    L, d = mtp_model
    toks = np.random.default_rng(11).integers(0, d.n_vocab, size=16).astype(np.int32)
    for cuts in ((), (9,), (1, 5, 12)):
        res = []
        for blockwise in (False, True):
            dr, pend = _fold_and_draft(L, toks, cuts, blockwise)
            lg = np.zeros(d.n_vocab, np.float32)
            cwen_b200.check(L.cwen_cuda_logits(0, vp(lg)), "logits")
            res.append((dr, pend, lg))
        (d0, p0, l0), (d1, p1, l1) = res
        assert p0 == p1 and list(d0) == list(d1), cuts
        assert np.array_equal(l0.view(np.uint32), l1.view(np.uint32)), cuts


def test_mtp_step_export_matches_oracle(mtp_model, orc):
    """cwen_cuda_mtp_step (mtp_step, run.c:3099-3131) from the parked hidden,
    then chained from its own output slot, against the oracle's mtp_step on
    the same stream: the output hiddens agree to rel L2 <= 1e-4."""
    import cwen_b200
    L, d = mtp_model
    od, om = _oracle(orc)
    orc.or_mtp_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    orc.or_mtp_hprev.argtypes = [C.c_void_p]
    orc.or_mtp_hprev.restype = C.POINTER(C.c_float)
    H = d.n_embd
    try:
        toks = np.random.default_rng(21).integers(0, d.n_vocab, size=7).astype(np.int32)
        cwen_b200.check(L.cwen_cuda_reset())
        cwen_b200.check(L.cwen_cuda_forward_block(vp(toks), len(toks), -1), "forward_block")
        cwen_b200.check(L.cwen_cuda_accept(None, None, None), "accept")
        cwen_b200.check(L.cwen_cuda_commit(len(toks) - 1), "commit")
        cwen_b200.check(L.cwen_cuda_mtp_commit_block(0, vp(toks), len(toks)), "mtp_commit_block")
        orc.or_reset(om)
        for p, t in enumerate(toks):
            orc.or_forward(om, int(t), p, 1)
            orc.or_mtp_commit(om, p, int(t), orc.or_hidden(om))
        park = np.zeros(H, np.float32)
        cwen_b200.check(L.cwen_cuda_mtp_read(0, vp(park)), "mtp_read")
        opark = np.ctypeslib.as_array(orc.or_mtp_hprev(om), shape=(H,)).copy()
        assert rel_l2(park, opark) <= 1e-4
        pos = len(toks)
        h1, oh1, oh2 = np.zeros(H, np.float32), np.zeros(H, np.float32), np.zeros(H, np.float32)
        cwen_b200.check(L.cwen_cuda_mtp_step(101, pos, 0, 1), "mtp_step")
        cwen_b200.check(L.cwen_cuda_mtp_read(1, vp(h1)), "mtp_read")
        orc.or_mtp_step(om, 101, pos, vp(opark), vp(oh1))
        assert rel_l2(h1, oh1) <= 1e-4, rel_l2(h1, oh1)
        h2 = np.zeros(H, np.float32)
        cwen_b200.check(L.cwen_cuda_mtp_step(202, pos + 1, 1, 2), "mtp_step")
        cwen_b200.check(L.cwen_cuda_mtp_read(2, vp(h2)), "mtp_read")
        orc.or_mtp_step(om, 202, pos + 1, vp(oh1), vp(oh2))
        assert rel_l2(h2, oh2) <= 1e-4, rel_l2(h2, oh2)
        # range checks: slot 0 is not an output slot, pos 0 has no attendable slot
        assert L.cwen_cuda_mtp_step(1, pos + 2, 1, 0) == -1
        assert L.cwen_cuda_mtp_step(1, 0, 0, 1) == -1
        assert L.cwen_cuda_mtp_step(d.n_vocab, pos + 2, 0, 1) == -5
    finally:
        orc.or_model_free(om)
