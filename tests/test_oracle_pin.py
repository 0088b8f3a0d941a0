"""Pin the CPU oracle (oracle/cwen_oracle.c) against outputs of the reference
itself (maci0/cwen run.c, compiled into oracle/_ref) stored in
tests/golden/ref_kernels.npz by tests/golden/make_golden.py.

The reference's SIMD kernels reassociate fp32 sums, so agreement is to fp32
rounding: the reference's own gemv acceptance (max_abs <= 1e-4, run.c:4352)
and relative L2 <= 1e-5 elsewhere.
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import CwDims, gen_normal, gen_q, oracle_gemvb, rel_l2, vp


def test_gemv_matches_reference(orc, golden):
    for ti in range(4):
        typ, K, M, wseed, xseed = golden[f"gemv{ti}_meta"].tolist()
        W = gen_q(orc, wseed, f"gw{ti}", typ, K, M)
        X = gen_normal(orc, xseed, f"gx{ti}", 16 * K).reshape(16, K)
        for B in (1, 2, 8, 9, 16):
            ref = golden[f"gemv{ti}_B{B}"]
            got = oracle_gemvb(orc, typ, W, K, M, X[:B])
            assert np.abs(got - ref).max() <= 1e-4, (ti, B)
            assert rel_l2(got, ref) <= 1e-5, (ti, B)


def test_rmsnorm_rope_match_reference(orc, golden):
    x = gen_normal(orc, 11, "rx", 5120) * 3.0
    w = gen_normal(orc, 12, "rw", 5120) * 0.1 + 1.0
    o = np.zeros(5120, np.float32)
    orc.or_rmsnorm(vp(o), vp(x), vp(w), 5120)
    assert rel_l2(o, golden["rmsnorm"]) <= 1e-6
    q = gen_normal(orc, 13, "rq", 24 * 256)
    orc.or_rope(vp(q), 24, 256, 777)
    assert rel_l2(q, golden["rope_p777"]) <= 1e-6


def _full():
    d = CwDims()
    from oracle_lib import load_oracle
    load_oracle().cw_dims_full(C.byref(d))
    return d


def test_attention_matches_reference(orc, golden):
    d = _full()
    T, NKV, HD, NH = 38, 4, 256, 24
    Kb = gen_normal(orc, 14, "ak", T * NKV * HD)
    Vb = gen_normal(orc, 15, "av", T * NKV * HD)
    qa = gen_normal(orc, 16, "aq", NH * HD)
    ga = gen_normal(orc, 17, "ag", NH * HD)
    y = np.zeros(NH * HD, np.float32)
    for t0, key in ((0, "attn_t0_p37"), (1, "attn_t1_p37")):
        orc.or_attention(C.byref(d), vp(Kb), vp(Vb), t0, T - 1, vp(qa), vp(ga), vp(y))
        assert rel_l2(y, golden[key]) <= 1e-5, key


def test_gdn_matches_reference(orc, golden):
    d = _full()
    LVH, LSD, QKV = 48, 128, 10240
    S = gen_normal(orc, 18, "gs", LVH * LSD * LSD) * 0.1
    cs = gen_normal(orc, 19, "gc", QKV * 3)
    cw = gen_normal(orc, 20, "gcw", QKV * 4) * 0.1
    nw = np.ones(LSD, np.float32)
    for p in range(3):
        qkv = gen_normal(orc, 30 + p, "gq", QKV)
        z = gen_normal(orc, 40 + p, "gz", LVH * LSD)
        a = gen_normal(orc, 50 + p, "ga", LVH)
        b = gen_normal(orc, 60 + p, "gb", LVH)
        # decay/beta transform with A=-1, dt=0 (run.c:2339-2344)
        a = (-np.log1p(np.exp(a.astype(np.float64)))).astype(np.float32)
        b = (1.0 / (1.0 + np.exp(-b.astype(np.float64)))).astype(np.float32)
        orc.or_conv1d_update(vp(qkv), vp(cs), vp(cw), QKV)
        o = np.zeros(LVH * LSD, np.float32)
        orc.or_gdn_step(C.byref(d), vp(S), vp(qkv), vp(z), vp(a), vp(b), vp(nw), vp(o))
        assert rel_l2(o, golden[f"gdn_out_p{p}"]) <= 1e-5, p
    assert rel_l2(S.reshape(-1)[::97], golden["gdn_S_sub"]) <= 1e-5
    assert rel_l2(cs, golden["gdn_conv"]) <= 1e-6


def _xround_np(x):
    """numpy restatement of the oracle's test-only operand rounding: the
    column scaled by 2^sh (largest |x| in [2^14, 2^15)), split into f16 hi + lo."""
    mx = float(np.abs(x).max())
    sh = 15 - int(np.frexp(np.float32(mx))[1])
    xs = np.ldexp(x.astype(np.float32), sh).astype(np.float32)
    hi = xs.astype(np.float16).astype(np.float32)
    lo = (xs - hi).astype(np.float16).astype(np.float32)
    return np.ldexp(hi + lo, -sh).astype(np.float32)


def test_xround_switch(orc):
    """or_set_xround(1) rounds each X column to 22 significant bits before the
    dots and changes nothing else; off again, the oracle is the plain fp32 one."""
    K, M, B = 1024, 96, 3
    W = gen_q(orc, 5, "xr_w", 2, K, M)
    X = gen_normal(orc, 6, "xr_x", B * K).reshape(B, K) * np.float32(3.0)
    X[1] *= np.float32(1e-3)
    Xr = np.stack([_xround_np(X[b]) for b in range(B)])
    err = np.abs(Xr - X) / np.maximum(np.abs(X), 1e-30)
    assert err.max() <= 2.0 ** -22 and (Xr != X).any()
    plain = oracle_gemvb(orc, 2, W, K, M, X)
    orc.or_set_xround(1)
    try:
        rounded = oracle_gemvb(orc, 2, W, K, M, X)
    finally:
        orc.or_set_xround(0)
    assert np.array_equal(rounded, oracle_gemvb(orc, 2, W, K, M, Xr))
    assert np.array_equal(plain, oracle_gemvb(orc, 2, W, K, M, X))
    assert not np.array_equal(rounded, plain)
