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


def test_cwenr_sidecar_supplies_the_q4_weights(tmp_path, monkeypatch):
    """A CWENR sidecar beside the GGUF (load_cwenr, run.c:3486-3643) supplies
    the Q4_0 weights the engine runs: GGUF A with a v4 sidecar that holds the
    Q4_0 tensors of another seed's model gives, bit for bit, the logits and
    serial stream of GGUF A with those tensors written into the file itself
    (and not A's own).  A v3 sidecar of A's own tensors changes nothing."""
    import cwen_b200
    from cwen_b200 import build
    from cwenr_util import GGUF_Q4_0, read_gguf_table, write_cwenr
    build.build()
    monkeypatch.delenv("CWEN_REPACK", raising=False)
    L = cwen_b200.lib()
    d = cwen_b200.dims("small")
    d.has_mtp = 1
    a_path, b_path = tmp_path / "a.gguf", tmp_path / "b.gguf"
    cwen_b200.check(L.cwen_write_synth_gguf(str(a_path).encode(), C.byref(d), SEED, 0), "write a")
    cwen_b200.check(L.cwen_write_synth_gguf(str(b_path).encode(), C.byref(d), SEED + 1, 0), "write b")
    a, b = a_path.read_bytes(), b_path.read_bytes()
    ta, tb = read_gguf_table(a), {n: (o, nb) for n, t, _, _, o, nb in read_gguf_table(b)}
    blobs = {n: b[tb[n][0]:tb[n][0] + tb[n][1]] for n, t, _, _, _, _ in ta if t == GGUF_Q4_0}
    assert blobs
    c = bytearray(a)  # A with B's Q4_0 tensors in the file
    for n, t, _, _, o, nb in ta:
        if t == GGUF_Q4_0:
            c[o:o + nb] = blobs[n]
    c_path = tmp_path / "c.gguf"
    c_path.write_bytes(bytes(c))
    ref_c = _run(L, lambda d: L.cwen_load_gguf(str(c_path).encode()))
    ref_a = _run(L, lambda d: L.cwen_load_gguf(str(a_path).encode()))
    (tmp_path / "a.cwenr").write_bytes(write_cwenr(a, 4, blobs=blobs))
    got = _run(L, lambda d: L.cwen_load_gguf(str(a_path).encode()))
    assert np.array_equal(got[3], ref_c[3]) and np.array_equal(got[0], ref_c[0])
    assert not np.array_equal(got[3], ref_a[3])
    (tmp_path / "a.cwenr").write_bytes(write_cwenr(a, 3))
    same = _run(L, lambda d: L.cwen_load_gguf(str(a_path).encode()))
    assert np.array_equal(same[3], ref_a[3]) and np.array_equal(same[0], ref_a[0])
