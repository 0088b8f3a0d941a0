"""Forward pass of the engine on the small seeded geometry, through the C ABI.

- per-layer residual streams and logits vs the CPU oracle (the reference's
  algorithm restated): relative L2 <= 1e-4 (fp32 math throughout; the GEMV
  input is split f16 hi+lo to ~2^-22);
- the verify block is bit-identical to serial decode (batch invariance), and
  a short-walk commit restores exactly the serial state;
- speculative generation emits exactly the serial token stream.
Every test runs under each verify-GEMV kernel an engine can use (mma.sync,
the default; qmv with CWEN_GEMV=qmv; tcgen05 with CWEN_GEMV=tcgen05).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import CwDims, load_oracle, rel_l2, vp

pytestmark = pytest.mark.gpu

SEED = 7
CTX = 512


@pytest.fixture(scope="module", params=["mma", "qmv", "tcgen05"])
def small(request):
    import os

    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    old = os.environ.get("CWEN_GEMV")
    os.environ["CWEN_GEMV"] = request.param
    try:
        cwen_b200.check(L.cwen_cuda_init(0, CTX, 16), "init")
    finally:
        if old is None:
            os.environ.pop("CWEN_GEMV")
        else:
            os.environ["CWEN_GEMV"] = old
    d = cwen_b200.dims("small")
    cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 0), "load_synth")
    yield L, d
    L.cwen_cuda_shutdown()


def _oracle_model(orc):
    d = CwDims()
    orc.cw_dims_tiny(C.byref(d))
    m = orc.or_model_synth(C.byref(d), SEED, CTX, 0)
    assert m
    return d, m


def _ids(n, V, seed):
    return np.random.default_rng(seed).integers(0, V, size=n).astype(np.int32)


def _logits(L, d, row=0):
    import cwen_b200
    lg = np.zeros(d.n_vocab, np.float32)
    cwen_b200.check(L.cwen_cuda_logits(row, vp(lg)), "logits")
    return lg


def test_forward_matches_oracle(small, orc):
    import cwen_b200
    L, d = small
    od, om = _oracle_model(orc)
    try:
        toks = _ids(12, d.n_vocab, 1)
        cwen_b200.check(L.cwen_cuda_reset())
        orc.or_reset(om)
        cwen_b200.check(L.cwen_cuda_dump_layers(1))
        hid = np.zeros(d.n_embd, np.float32)
        for p, t in enumerate(toks):
            am = C.c_int(-1)
            cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, C.byref(am)), "forward_serial")
            orc.or_forward(om, int(t), p, 1)
            for layer in range(d.n_layer):
                cwen_b200.check(L.cwen_cuda_dump_read(layer, 0, vp(hid)))
                ref = np.ctypeslib.as_array(orc.or_layer_out(om, layer), shape=(d.n_embd,))
                assert rel_l2(hid, ref) <= 1e-4, (p, layer, rel_l2(hid, ref))
            ref_lg = np.ctypeslib.as_array(orc.or_logits(om), shape=(d.n_vocab,))
            lg = _logits(L, d)
            assert rel_l2(lg, ref_lg) <= 1e-4, (p, rel_l2(lg, ref_lg))
            assert am.value == int(np.argmax(lg))
        cwen_b200.check(L.cwen_cuda_dump_layers(0))
    finally:
        orc.or_model_free(om)


def _prefill(L, toks):
    import cwen_b200
    cwen_b200.check(L.cwen_cuda_reset())
    i = 0
    while i < len(toks):
        B = min(16, len(toks) - i)
        cwen_b200.check(L.cwen_cuda_forward_block(vp(np.ascontiguousarray(toks[i:i + B])), B, 0))
        cwen_b200.check(L.cwen_cuda_commit(B - 1))
        i += B


def test_block_bitwise_equals_serial(small):
    import cwen_b200
    L, d = small
    prompt = _ids(21, d.n_vocab, 2)
    blk = _ids(9, d.n_vocab, 3)
    # serial: one token at a time
    _prefill(L, prompt)
    serial = []
    for t in blk:
        cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, None))
        serial.append(_logits(L, d))
    # block: all 9 rows in one verify pass
    _prefill(L, prompt)
    cwen_b200.check(L.cwen_cuda_forward_block(vp(blk), len(blk), len(blk)))
    for b in range(len(blk)):
        assert np.array_equal(_logits(L, d, b).view(np.uint32), serial[b].view(np.uint32)), b
    cwen_b200.check(L.cwen_cuda_commit(len(blk) - 1))


@pytest.mark.parametrize("k", [0, 3, 7])
def test_short_walk_commit_restores_serial_state(small, k):
    """commit(k) after a block must leave exactly the state of k+1 serial steps."""
    import cwen_b200
    L, d = small
    prompt = _ids(13, d.n_vocab, 4)
    blk = _ids(9, d.n_vocab, 5)
    nxt = int(_ids(1, d.n_vocab, 6)[0])
    _prefill(L, prompt)
    for t in blk[:k + 1]:
        cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 0, None))
    cwen_b200.check(L.cwen_cuda_forward_serial(nxt, 1, None))
    want = _logits(L, d)
    QKV = (2 * d.ssm_n_kh + d.ssm_n_vh) * 128
    S_ser = np.zeros(d.ssm_n_vh * 128 * 128, np.float32)
    c_ser = np.zeros(QKV * 3, np.float32)
    cwen_b200.check(L.cwen_cuda_gdn_state(0, vp(S_ser), vp(c_ser)))

    _prefill(L, prompt)
    cwen_b200.check(L.cwen_cuda_forward_block(vp(blk), len(blk), len(blk)))
    cwen_b200.check(L.cwen_cuda_commit(k))
    assert L.cwen_cuda_n_past() == len(prompt) + k + 1
    cwen_b200.check(L.cwen_cuda_forward_serial(nxt, 1, None))
    got = _logits(L, d)
    S_blk = np.zeros_like(S_ser)
    c_blk = np.zeros_like(c_ser)
    cwen_b200.check(L.cwen_cuda_gdn_state(0, vp(S_blk), vp(c_blk)))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(S_blk.view(np.uint32), S_ser.view(np.uint32))
    assert np.array_equal(c_blk.view(np.uint32), c_ser.view(np.uint32))


def _motif_prompt(n, V, seed):
    rng = np.random.default_rng(seed)
    motif = rng.integers(0, V, size=37)
    p = np.resize(motif, n).astype(np.int32)
    sub = rng.random(n) < 0.05
    p[sub] = rng.integers(0, V, size=int(sub.sum()))
    return p


@pytest.mark.parametrize("max_draft", [3, 8, 15])
def test_spec_stream_equals_serial(small, max_draft):
    import cwen_b200
    L, d = small
    prompt = _motif_prompt(200, d.n_vocab, 8)
    ser, _ = cwen_b200.generate(prompt, 64, cwen_b200.spec_cfg(spec=0))
    spec, st = cwen_b200.generate(prompt, 64, cwen_b200.spec_cfg(spec=1, max_draft=max_draft, n_key=4, min_draft=1))
    assert np.array_equal(ser, spec)
    assert st.cycles > 0


def test_ngram_cache_knob(small, tmp_path, monkeypatch):
    """CWEN_NGRAM_CACHE (run.c:5198-5205): a speculative run saves its n-gram
    map as an NGC2 file; the next run merges it before the prompt and still
    emits the serial stream."""
    import cwen_b200
    L, d = small
    path = tmp_path / "map.ngc"
    prompt = _motif_prompt(200, d.n_vocab, 9)
    ser, _ = cwen_b200.generate(prompt, 48, cwen_b200.spec_cfg(spec=0))
    monkeypatch.setenv("CWEN_NGRAM_CACHE", str(path))
    cfg = cwen_b200.spec_cfg(spec=1, use_mtp=0, max_draft=8, n_key=4, min_draft=1)
    a, _ = cwen_b200.generate(prompt, 48, cfg)
    hdr = np.frombuffer(path.read_bytes()[:16], np.uint32)
    assert hdr[0] == 0x3243474E and hdr[1] == 4 and hdr[2] == d.n_vocab and hdr[3] > 0
    b, _ = cwen_b200.generate(prompt, 48, cfg)
    assert np.array_equal(a, ser) and np.array_equal(b, ser)


def test_forced_rejections_keep_stream(small):
    """Short key + min_draft 1 forces short walks (run through rollback)."""
    import cwen_b200
    L, d = small
    prompt = _ids(64, d.n_vocab, 9)
    prompt = np.concatenate([prompt, prompt[:40], prompt[:40]]).astype(np.int32)
    ser, _ = cwen_b200.generate(prompt, 48, cwen_b200.spec_cfg(spec=0))
    spec, st = cwen_b200.generate(prompt, 48, cwen_b200.spec_cfg(spec=1, max_draft=8, n_key=2, min_draft=1,
                                                                  cooldown=0))
    assert np.array_equal(ser, spec)
    assert st.drafted > 0


def test_bad_token_is_an_error_not_an_exit(small):
    import cwen_b200
    L, d = small
    cwen_b200.check(L.cwen_cuda_reset())
    bad = np.array([d.n_vocab], np.int32)
    assert L.cwen_cuda_forward_block(vp(bad), 1, 1) == -5  # CWEN_ERANGE
    assert L.cwen_cuda_n_past() == 0


def test_context_cap(small):
    import cwen_b200
    L, d = small
    prompt = _ids(CTX - 3, d.n_vocab, 10)
    out, _ = cwen_b200.generate(prompt, 10, cwen_b200.spec_cfg(spec=0))
    assert len(out) == 3  # emits only while a slot is left, like the reference
