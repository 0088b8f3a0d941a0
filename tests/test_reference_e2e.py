"""Full 27B geometry on seeded random weights: the engine against the
reference itself (maci0/cwen run.c compiled into oracle/_ref), the residual
stream after every layer that its CWEN_DUMP writes (run.c:2601-2629) taken
in memory through the harness's cwref_forward_layers -- the reference fixes
its dump choice at its first forward in a process, which another test may
already have run -- at the first slots of a sequence (the 27B model past
slot 512 is test_reference_chain.py).

Bar (north star): per-layer hidden states and logits within 1e-3 relative L2
of the reference's CPU path.  The random-init model is chaotic at some
positions (position 0 of this seed): there, CPU restatements of the
reference's own algorithm that round differently drift apart by far more
than 1e-3 in the deep layers.  Two such restatements run beside the engine:
the fp32 oracle (the reference's scalar summation order; the reference runs
AVX-512 orders) and the same oracle with every GEMV's X rounded to the
engine's operand precision (f16 hi + lo after a power-of-two column scale,
22 significant bits; or_set_xround).  The spread at a layer is the larger of
their two distances from the reference.  A position whose spread stays
within 1e-3 everywhere holds every layer and the logits to 1e-3.  At a
chaotic position the layers up to the onset (the first layer whose spread
passes 1e-3) are held to max(1e-3, 3 x the largest spread so far); past the
onset the two restatements, which differ only in operand rounding, already
disagree with the reference by more than the bar, so no rounding-level bar
exists there: those checks are printed with their spread, not asserted.
The per-layer bar past slot 512 on several seeds is in
test_reference_chain.py.  Token ids must agree wherever the oracle and the
reference agree and the reference's top-2 margin exceeds 1e-4.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import CwDims, load_oracle, rel_l2, vp

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

ROOT = Path(__file__).resolve().parents[1]
SEED = 11
CTX = 64
NPOS = 4


def _ref_lib():
    import bench
    path, _ = bench.ref_lib_path()
    if not path.exists():
        pytest.skip("oracle/_ref reference build missing (oracle/build_ref.sh)")
    return path


def test_full_geometry_matches_reference():
    import cwen_b200
    from cwen_b200 import build
    path = _ref_lib()
    build.build()
    ref = C.CDLL(str(path))
    ref.cwref_forward_layers.argtypes = [C.c_int, C.c_void_p, C.c_void_p]
    assert ref.cwref_load_synth(C.c_uint64(SEED), 0, 0) == 0
    ref.cwref_alloc_state(CTX, 0, 0)
    ref.cwref_reset_state()
    orc = load_oracle()
    od = CwDims()
    orc.cw_dims_full(C.byref(od))
    om = orc.or_model_synth(C.byref(od), SEED, CTX, 0)
    om22 = orc.or_model_synth(C.byref(od), SEED, CTX, 0)  # run with the engine's operand rounding
    assert om and om22

    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, CTX, 16), "init")
    try:
        d = cwen_b200.dims("reference")
        cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 0), "load_synth")
        toks = np.random.default_rng(12).integers(0, d.n_vocab, size=NPOS).astype(np.int32)
        cwen_b200.check(L.cwen_cuda_reset())
        cwen_b200.check(L.cwen_cuda_dump_layers(1))
        H, V = d.n_embd, d.n_vocab
        hid = np.zeros(H, np.float32)
        rlay = np.zeros((d.n_layer, H), np.float32)
        rl = np.zeros(V, np.float32)
        n_chaotic = n_wide = 0
        past = []
        for p, t in enumerate(toks):
            ref.cwref_set_pos(p)
            ref.cwref_forward_layers(int(t), vp(rlay), vp(rl))
            orc.or_forward(om, int(t), p, 1)
            orc.or_set_xround(1)
            try:
                orc.or_forward(om22, int(t), p, 1)
            finally:
                orc.or_set_xround(0)
            am = C.c_int(-1)
            cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, C.byref(am)))
            eng, spread = [], []
            for layer in range(d.n_layer):
                r = rlay[layer]
                cwen_b200.check(L.cwen_cuda_dump_read(layer, 0, vp(hid)))
                o = np.ctypeslib.as_array(orc.or_layer_out(om, layer), shape=(H,))
                o22 = np.ctypeslib.as_array(orc.or_layer_out(om22, layer), shape=(H,))
                eng.append(rel_l2(hid, r))
                spread.append(max(rel_l2(o, r), rel_l2(o22, r)))
            gl = np.zeros(V, np.float32)
            cwen_b200.check(L.cwen_cuda_logits(0, vp(gl)))
            ol = np.ctypeslib.as_array(orc.or_logits(om), shape=(V,))
            ol22 = np.ctypeslib.as_array(orc.or_logits(om22), shape=(V,))
            eng.append(rel_l2(gl, rl))
            spread.append(max(rel_l2(ol, rl), rel_l2(ol22, rl)))
            print(f"pos {p}: engine-vs-ref per layer max {max(eng[:-1]):.2e} (spread max {max(spread[:-1]):.2e}); "
                  f"logits {eng[-1]:.2e} (spread {spread[-1]:.2e})")
            chaotic = max(spread) > 1e-3
            n_chaotic += chaotic
            run = 0.0
            for i in range(len(eng)):  # the layers in order, then the logits
                run = max(run, spread[i])
                if run > 1e-3:
                    # past the chaotic onset: the restatements themselves
                    # disagree by more than the bar; reported, not asserted
                    past.append((p, i, eng[i], spread[i]))
                    continue
                bar = max(1e-3, 3.0 * run)
                n_wide += bar > 1e-3
                assert eng[i] <= bar, (p, i, eng[i], spread[i], run)
            ref_am, orc_am = int(np.argmax(rl)), int(np.argmax(ol))
            top2 = np.sort(rl)[-2:]
            if ref_am == orc_am and top2[1] - top2[0] > 1e-4:
                assert am.value == ref_am, p
        cwen_b200.check(L.cwen_cuda_dump_layers(0))
        print(f"chaotic positions (spread above 1e-3): {n_chaotic} of {NPOS}; checks with a bar above 1e-3 "
              f"(3 x the spread): {n_wide}; checks past a chaotic onset (not asserted): {len(past)} "
              f"of {NPOS * (d.n_layer + 1)}")
        for p, i, e, sp in past:
            print(f"  pos {p} {'logits' if i == d.n_layer else f'layer {i}'}: engine {e:.2e}, spread {sp:.2e}")
        assert len(past) <= (d.n_layer + 1) * NPOS // 4, "most checks past a chaotic onset: pick another seed"
    finally:
        L.cwen_cuda_shutdown()
        orc.or_model_free(om)
        orc.or_model_free(om22)
