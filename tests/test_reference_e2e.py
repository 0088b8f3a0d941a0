"""Full 27B geometry on seeded random weights: the engine against the
reference itself (maci0/cwen run.c compiled into oracle/_ref, running its own
forward_ex with its CWEN_DUMP per-layer dumps, run.c:2601-2629), at the
first slots of a sequence (the 27B model past slot 512 is
test_reference_chain.py).

Bar (north star): per-layer hidden states and logits within 1e-3 relative L2
of the reference's CPU path.  The random-init model is chaotic at some
positions (position 0 of this seed): there, two fp32 CPU implementations of
the reference's own algorithm (the oracle's scalar summation order and the
reference's AVX-512 order) drift apart by far more than 1e-3 in the deep
layers, and any other summation order lands a random distance of that order
away.  So every layer and the logits are held to max(1e-3, 3 x spread),
spread = the oracle-vs-reference relative L2 at that layer and position; the
test prints how many checks needed more than 1e-3.  Token ids must agree
wherever the oracle and the reference agree and the reference's top-2 margin
exceeds 1e-4.
"""
import ctypes as C
import os
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


def test_full_geometry_matches_reference(tmp_path):
    import cwen_b200
    from cwen_b200 import build
    path = _ref_lib()
    build.build()
    dump = tmp_path / "dump"
    dump.mkdir()
    os.environ["CWEN_DUMP"] = str(dump)
    os.environ.pop("CWEN_DUMP_LAYERS", None)
    ref = C.CDLL(str(path))
    assert ref.cwref_load_synth(C.c_uint64(SEED), 0, 0) == 0
    ref.cwref_alloc_state(CTX, 0, 0)
    ref.cwref_reset_state()
    orc = load_oracle()
    od = CwDims()
    orc.cw_dims_full(C.byref(od))
    om = orc.or_model_synth(C.byref(od), SEED, CTX, 0)
    assert om

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
        loose = checks = 0
        for p, t in enumerate(toks):
            ref.cwref_set_pos(p)
            ref.cwref_forward_ex(int(t), 1)
            orc.or_forward(om, int(t), p, 1)
            am = C.c_int(-1)
            cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, C.byref(am)))
            eng, flo = [], []
            for layer in range(d.n_layer):
                r = np.fromfile(dump / f"layer{layer:02d}_pos{p:02d}.bin", np.float32)
                cwen_b200.check(L.cwen_cuda_dump_read(layer, 0, vp(hid)))
                o = np.ctypeslib.as_array(orc.or_layer_out(om, layer), shape=(H,))
                eng.append(rel_l2(hid, r))
                flo.append(rel_l2(o, r))
            rl = np.zeros(V, np.float32)
            ref.cwref_get_logits(vp(rl))
            gl = np.zeros(V, np.float32)
            cwen_b200.check(L.cwen_cuda_logits(0, vp(gl)))
            ol = np.ctypeslib.as_array(orc.or_logits(om), shape=(V,))
            e_lg, f_lg = rel_l2(gl, rl), rel_l2(ol, rl)
            print(f"pos {p}: engine-vs-ref per layer max {max(eng):.2e} (floor max {max(flo):.2e}); "
                  f"logits {e_lg:.2e} (floor {f_lg:.2e})")
            for layer in range(d.n_layer):
                bar = max(1e-3, 3.0 * flo[layer])
                loose += bar > 1e-3
                checks += 1
                assert eng[layer] <= bar, (p, layer, eng[layer], flo[layer])
            bar = max(1e-3, 3.0 * f_lg)
            loose += bar > 1e-3
            checks += 1
            assert e_lg <= bar, (p, e_lg, f_lg)
            ref_am, orc_am = int(np.argmax(rl)), int(np.argmax(ol))
            top2 = np.sort(rl)[-2:]
            if ref_am == orc_am and top2[1] - top2[0] > 1e-4:
                assert am.value == ref_am, p
        cwen_b200.check(L.cwen_cuda_dump_layers(0))
        print(f"bar above 1e-3 (3 x the oracle-vs-reference spread) at {loose} of {checks} checks")
    finally:
        L.cwen_cuda_shutdown()
        orc.or_model_free(om)
        os.environ.pop("CWEN_DUMP", None)
