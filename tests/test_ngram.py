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


# ---- NGC2 persistence (ng_save / ng_load, run.c:4656-4716) ----
V_REF = 248320  # the reference's compiled-in vocabulary, which its files carry


def _ngc2_libs(libs):
    L, ref = libs
    ref.cwref_ng_save.argtypes = [C.c_char_p]
    ref.cwref_ng_load.argtypes = [C.c_char_p]
    ref.cwref_ng_used.restype = C.c_longlong
    L.cwen_ngram_map_save.argtypes = [C.c_void_p, C.c_char_p, C.c_int]
    L.cwen_ngram_map_load.argtypes = [C.c_void_p, C.c_char_p, C.c_int]
    return L, ref


def _both_from(L, ref, h, n_key, upto):
    m = L.cwen_ngram_map_new(n_key)
    assert m and ref.cwref_ngmap_init(n_key) == 0
    L.cwen_ngram_map_update(m, _p(h), 0, upto)
    ref.cwref_ng_update_range(_p(h), 0, upto)
    return m


def _proposals(L, ref, m, h, n_key, points):
    a, b = np.zeros(16, np.int32), np.zeros(16, np.int32)
    for hn in points:
        na = L.cwen_ngram_map_draft(m, _p(h), hn, _p(a), 15)
        nb = ref.cwref_ng_propose(_p(h), hn, _p(b), 15)
        assert na == nb and np.array_equal(a[:na], b[:nb]), hn


def test_ngc2_file_equals_reference(libs, tmp_path):
    L, ref = _ngc2_libs(libs)
    n_key = 4
    h = _history(np.random.default_rng(21), 4000, V_REF, 37, 0.05)
    m = _both_from(L, ref, h, n_key, 3000)
    try:
        ours, theirs = tmp_path / "ours.ngc", tmp_path / "ref.ngc"
        assert L.cwen_ngram_map_save(m, str(ours).encode(), V_REF) == 0
        ref.cwref_ng_save(str(theirs).encode())
        assert ours.read_bytes() == theirs.read_bytes()
        assert not (tmp_path / "ours.ngc.tmp").exists()
        hdr = np.frombuffer(ours.read_bytes()[:16], np.uint32)
        assert hdr[0] == 0x3243474E and hdr[1] == n_key and hdr[2] == V_REF
        assert hdr[3] == ref.cwref_ng_used() and len(ours.read_bytes()) == 16 + hdr[3] * (n_key + 2) * 4
    finally:
        L.cwen_ngram_map_free(m)


def test_ngc2_load_merge_matches_reference(libs, tmp_path):
    """Each side loads the other's file into a fresh map, twice (the counts
    merge); both maps then save the same bytes and propose the same ids."""
    L, ref = _ngc2_libs(libs)
    n_key = 4
    h = _history(np.random.default_rng(22), 4000, V_REF, 37, 0.05)
    m = _both_from(L, ref, h, n_key, 2500)
    src = tmp_path / "src.ngc"
    try:
        assert L.cwen_ngram_map_save(m, str(src).encode(), V_REF) == 0
    finally:
        L.cwen_ngram_map_free(m)
    m = L.cwen_ngram_map_new(n_key)
    try:
        assert ref.cwref_ngmap_init(n_key) == 0
        n1 = L.cwen_ngram_map_load(m, str(src).encode(), V_REF)
        ref.cwref_ng_load(str(src).encode())
        assert n1 > 0 and n1 == ref.cwref_ng_used()
        assert L.cwen_ngram_map_load(m, str(src).encode(), V_REF) == n1  # same keys: counts add
        ref.cwref_ng_load(str(src).encode())
        a, b = tmp_path / "a.ngc", tmp_path / "b.ngc"
        assert L.cwen_ngram_map_save(m, str(a).encode(), V_REF) == 0
        ref.cwref_ng_save(str(b).encode())
        assert a.read_bytes() == b.read_bytes()
        # the reloaded maps draft alike on the rest of the history
        L.cwen_ngram_map_update(m, _p(h), 2500, 3500)
        ref.cwref_ng_update_range(_p(h), 2500, 3500)
        _proposals(L, ref, m, h, n_key, range(2500, 3500, 11))
    finally:
        L.cwen_ngram_map_free(m)


def test_ngc2_damaged_files_match_reference(libs, tmp_path):
    """Foreign or damaged files: each side merges exactly the same records."""
    L, ref = _ngc2_libs(libs)
    n_key = 4
    h = _history(np.random.default_rng(23), 3000, V_REF, 37, 0.05)
    m = _both_from(L, ref, h, n_key, 2000)
    good = tmp_path / "good.ngc"
    try:
        assert L.cwen_ngram_map_save(m, str(good).encode(), V_REF) == 0
    finally:
        L.cwen_ngram_map_free(m)
    blob = bytearray(good.read_bytes())
    rec = (n_key + 2) * 4
    bad_tok = bytearray(blob)
    bad_tok[16 + n_key * 4:16 + n_key * 4 + 4] = np.int32(V_REF).tobytes()       # first record: tok = V
    bad_cnt = bytearray(blob)
    bad_cnt[16 + rec + (n_key + 1) * 4:16 + 2 * rec] = np.int32(0).tobytes()      # second record: cnt = 0
    cases = {
        "short": bytes(blob[:10]),
        "magic": b"NGC1" + bytes(blob[4:]),
        "n_key": bytes(blob[:4]) + np.uint32(5).tobytes() + bytes(blob[8:]),
        "vocab": bytes(blob[:8]) + np.uint32(1000).tobytes() + bytes(blob[12:]),
        "truncated": bytes(blob[:16 + 7 * rec + 5]),
        "bad_tok": bytes(bad_tok),
        "bad_cnt": bytes(bad_cnt),
        "count_beyond": bytes(blob[:12]) + np.uint32(1 << 30).tobytes() + bytes(blob[16:]),
    }
    for name, data in cases.items():
        f = tmp_path / f"{name}.ngc"
        f.write_bytes(data)
        m = L.cwen_ngram_map_new(n_key)
        try:
            assert ref.cwref_ngmap_init(n_key) == 0
            got = L.cwen_ngram_map_load(m, str(f).encode(), V_REF)
            ref.cwref_ng_load(str(f).encode())
            assert got == ref.cwref_ng_used(), name
            a, b = tmp_path / "a.ngc", tmp_path / "b.ngc"
            assert L.cwen_ngram_map_save(m, str(a).encode(), V_REF) == 0
            ref.cwref_ng_save(str(b).encode())
            assert a.read_bytes() == b.read_bytes(), name
        finally:
            L.cwen_ngram_map_free(m)
    m = L.cwen_ngram_map_new(n_key)
    try:
        assert L.cwen_ngram_map_load(m, str(tmp_path / "missing.ngc").encode(), V_REF) == 0
        assert L.cwen_ngram_map_load(m, None, V_REF) == -1
        assert L.cwen_ngram_map_save(m, str(tmp_path / "no" / "dir.ngc").encode(), V_REF) == -1
    finally:
        L.cwen_ngram_map_free(m)


def test_ngc2_mutated_files_never_crash(libs, tmp_path):
    """Random flips and cuts of an NGC2 file: a load merges what it can and
    never crashes (the reference's cache fuzz hook, cw_fuzz_ngcache)."""
    L, ref = _ngc2_libs(libs)
    n_key = 4
    h = _history(np.random.default_rng(31), 2000, V_REF, 37, 0.05)
    m = _both_from(L, ref, h, n_key, 1500)
    src = tmp_path / "src.ngc"
    try:
        assert L.cwen_ngram_map_save(m, str(src).encode(), V_REF) == 0
    finally:
        L.cwen_ngram_map_free(m)
    base = bytearray(src.read_bytes())
    rng = np.random.default_rng(5)
    f = tmp_path / "fz.ngc"
    for it in range(150):
        b = bytearray(base)
        if it % 2:
            for _ in range(int(rng.integers(1, 8))):
                b[int(rng.integers(0, len(b)))] ^= int(rng.integers(1, 256))
        else:
            b = b[:int(rng.integers(0, len(b)))]
        f.write_bytes(bytes(b))
        m = L.cwen_ngram_map_new(n_key)
        try:
            got = L.cwen_ngram_map_load(m, str(f).encode(), V_REF)
            assert got >= 0
            out = np.zeros(16, np.int32)
            assert L.cwen_ngram_map_draft(m, _p(h), 1500, _p(out), 15) >= 0
        finally:
            L.cwen_ngram_map_free(m)
