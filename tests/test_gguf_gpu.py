"""A GGUF file written by cwen_write_synth_gguf and read by cwen_load_gguf
gives the engine exactly the model cwen_load_synth uploads: the same logits
bit for bit, the same serial stream, and the same MTP-drafted speculation
(the nextn block comes from the file too).  The CPU side of the loader and
writer is covered by test_gguf.py.
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import vp

pytestmark = pytest.mark.gpu

SEED = 7


def _run(L, load):
    import cwen_b200
    cwen_b200.check(L.cwen_cuda_init(0, 256, 16), "init")
    try:
        d = cwen_b200.dims("small")
        d.has_mtp = 1
        cwen_b200.check(load(d), "load")
        prompt = np.random.default_rng(3).integers(0, d.n_vocab, size=12).astype(np.int32)
        serial, _ = cwen_b200.generate(prompt, 16, cwen_b200.spec_cfg(spec=0))
        spec, st = cwen_b200.generate(prompt, 16, cwen_b200.spec_cfg(spec=1, use_mtp=1, max_draft=4))
        lg = np.zeros(d.n_vocab, np.float32)
        cwen_b200.check(L.cwen_cuda_logits(0, vp(lg)), "logits")
        return serial, spec, (st.cycles, st.drafted, st.kept), lg
    finally:
        L.cwen_cuda_shutdown()


def test_gguf_load_equals_synth(tmp_path):
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    path = str(tmp_path / "small.gguf").encode()
    d = cwen_b200.dims("small")
    d.has_mtp = 1
    cwen_b200.check(L.cwen_write_synth_gguf(path, C.byref(d), SEED, 0), "write")
    a = _run(L, lambda d: L.cwen_load_gguf(path))
    b = _run(L, lambda d: L.cwen_load_synth(SEED, C.byref(d), 0))
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[1], a[0])
    assert a[2] == b[2]
    assert np.array_equal(a[3], b[3])
