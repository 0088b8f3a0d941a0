"""n-gram drafters of the C host against the reference's own (no GPU).

The prompt-lookup scan (cwen_ngram_draft vs ngram_draft, run.c:4533) and the
counted-map proposal of a speculative cycle (cwen_ngram_map_* vs the map of
run.c:4552-4654 driven as generate_tokens_spec drives it, run.c:4903-4930)
must propose the same ids for the same history: drafts do not change the
emitted tokens (verification is lossless) but they decide the acceptance
statistics the benchmarks report.  The reference runs from oracle/_ref
(compiled from run.c); the tests skip when it is not built.
"""
import ctypes as C

import numpy as np
import pytest

I32P = C.POINTER(C.c_int32)


@pytest.fixture(scope="module")
def libs():
    import bench
    import cwen_b200
    from cwen_b200 import build
    build.build()
    path, _ = bench.ref_lib_path()
    if not path.exists():
        pytest.skip("reference library (oracle/_ref) not built")
    ref = C.CDLL(str(path))
    ref.cwref_ngram_draft.argtypes = [I32P, C.c_int, I32P, C.c_int, C.c_int]
    ref.cwref_ngmap_init.argtypes = [C.c_int]
    ref.cwref_ng_update_range.argtypes = [I32P, C.c_int, C.c_int]
    ref.cwref_ng_propose.argtypes = [I32P, C.c_int, I32P, C.c_int]
    L = cwen_b200.lib()
    L.cwen_ngram_draft.argtypes = [I32P, C.c_int, I32P, C.c_int, C.c_int]
    L.cwen_ngram_map_new.argtypes = [C.c_int]
    L.cwen_ngram_map_new.restype = C.c_void_p
    L.cwen_ngram_map_free.argtypes = [C.c_void_p]
    L.cwen_ngram_map_free.restype = None
    L.cwen_ngram_map_update.argtypes = [C.c_void_p, I32P, C.c_int, C.c_int]
    L.cwen_ngram_map_update.restype = None
    L.cwen_ngram_map_draft.argtypes = [C.c_void_p, I32P, C.c_int, I32P, C.c_int]
    return L, ref


def _p(a):
    return a.ctypes.data_as(I32P)


def _history(rng, n, vocab, motif_len, sub):
    """Motif repeats with substitutions: the shape of the config-3 prompt."""
    motif = rng.integers(0, vocab, size=motif_len)
    h = np.resize(motif, n).astype(np.int32)
    s = rng.random(n) < sub
    h[s] = rng.integers(0, vocab, size=int(s.sum()))
    return h


@pytest.mark.parametrize("n_key,vocab,motif,sub", [(2, 50, 7, 0.1), (4, 1000, 37, 0.05), (16, 248320, 37, 0.05)])
def test_scan_matches_reference(libs, n_key, vocab, motif, sub):
    L, ref = libs
    rng = np.random.default_rng(n_key)
    h = _history(rng, 1500, vocab, motif, sub)
    a, b = np.zeros(300, np.int32), np.zeros(300, np.int32)
    proposed = 0
    for hn in list(range(0, 80)) + list(range(80, 1500, 37)):
        for max_d in (0, 1, 3, 8, 15, 300):
            na = L.cwen_ngram_draft(_p(h), hn, _p(a), n_key, max_d)
            nb = ref.cwref_ngram_draft(_p(h), hn, _p(b), n_key, max_d)
            assert na == nb, (hn, max_d)
            assert np.array_equal(a[:na], b[:nb]), (hn, max_d)
            proposed += na > 0
    assert proposed > 20  # the histories do repeat


@pytest.mark.parametrize("n_key,vocab,motif,sub", [(2, 30, 5, 0.2), (16, 248320, 37, 0.05)])
def test_map_proposals_match_reference(libs, n_key, vocab, motif, sub):
    """Grow a history the way the driver does (fold new positions, propose,
    append accepted ids) and compare every proposal."""
    L, ref = libs
    rng = np.random.default_rng(100 + n_key)
    h = _history(rng, 3000, vocab, motif, sub)
    m = L.cwen_ngram_map_new(n_key)
    assert m
    try:
        assert ref.cwref_ngmap_init(n_key) == 0
        a, b = np.zeros(16, np.int32), np.zeros(16, np.int32)
        upd, hn, proposed = 0, 64, 0
        while hn < len(h):
            L.cwen_ngram_map_update(m, _p(h), upd, hn)
            ref.cwref_ng_update_range(_p(h), upd, hn)
            upd = hn
            cap = int(rng.integers(1, 16))
            na = L.cwen_ngram_map_draft(m, _p(h), hn, _p(a), cap)
            nb = ref.cwref_ng_propose(_p(h), hn, _p(b), cap)
            assert na == nb and np.array_equal(a[:na], b[:nb]), hn
            proposed += na > 0
            hn += int(rng.integers(1, 10))
        assert proposed > 50
    finally:
        L.cwen_ngram_map_free(m)


def test_map_eviction_matches_reference(libs):
    """More distinct keys than the map's 2^18 slots: least-hit eviction with
    the rotating hand and backward-shift deletion keeps both maps equal."""
    L, ref = libs
    n_key = 2
    rng = np.random.default_rng(7)
    n = (1 << 18) + 1200
    h = rng.integers(0, 1 << 30, size=n, dtype=np.int64).astype(np.int32)
    h[-400:] = h[5000:5400]  # a tail whose keys were seen early (some evicted, some kept)
    m = L.cwen_ngram_map_new(n_key)
    assert m
    try:
        assert ref.cwref_ngmap_init(n_key) == 0
        L.cwen_ngram_map_update(m, _p(h), 0, n - 400)
        ref.cwref_ng_update_range(_p(h), 0, n - 400)
        a, b = np.zeros(16, np.int32), np.zeros(16, np.int32)
        proposed = 0
        for hn in range(n - 400, n, 7):
            L.cwen_ngram_map_update(m, _p(h), hn - 7 if hn - 7 >= n - 400 else n - 400, hn)
            ref.cwref_ng_update_range(_p(h), hn - 7 if hn - 7 >= n - 400 else n - 400, hn)
            na = L.cwen_ngram_map_draft(m, _p(h), hn, _p(a), 15)
            nb = ref.cwref_ng_propose(_p(h), hn, _p(b), 15)
            assert na == nb and np.array_equal(a[:na], b[:nb]), hn
            proposed += na > 0
        assert proposed > 10
    finally:
        L.cwen_ngram_map_free(m)


def test_map_argument_errors(libs):
    L, _ = libs
    assert not L.cwen_ngram_map_new(1)
    assert b"n_key" in L.cwen_cuda_last_error()
    assert not L.cwen_ngram_map_new(257)
    out = np.zeros(4, np.int32)
    assert L.cwen_ngram_map_draft(None, _p(out), 4, _p(out), 4) == -1
