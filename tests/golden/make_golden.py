"""Generate the golden fixtures in tests/golden/ by running the REFERENCE.

Runs maci0/cwen's own C kernels (run.c compiled where it lies into
oracle/_ref/ by oracle/build_ref.sh) on seeded inputs and stores inputs'
seeds plus the reference outputs as small .npz files.  Inputs are
regenerated at test time from the same seeds with the synth generator
(cwen_b200/host/synth.c), so only outputs need storing.

Run where the reference sources are available (oracle/build_ref.sh takes
their directory as its argument or CWEN_REFERENCE_DIR):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "tests"))
from oracle_lib import gen_normal, gen_q, load_oracle  # noqa: E402

REF_DIR = ROOT / "oracle" / "_ref"


def vp(a):
    return a.ctypes.data_as(C.c_void_p)


def load_ref():
    so = REF_DIR / "libcwref_avx512.so"
    if not so.exists():
        subprocess.check_call([str(ROOT / "oracle" / "build_ref.sh")])
    return C.CDLL(str(so))


def gemv_cases(ref, orc):
    out = {}
    for ti, (typ, K, M) in enumerate([(2, 512, 96), (2, 1024, 48), (8, 512, 64), (2, 5120, 64)]):
        W = gen_q(orc, 7 + ti, f"gw{ti}", typ, K, M)
        X = gen_normal(orc, 100 + ti, f"gx{ti}", 16 * K).reshape(16, K)
        Y = np.zeros((16, M), np.float32)
        for B in (1, 2, 8, 9, 16):
            ref.cwref_gemvb(typ, vp(W), K, M, vp(X), K, vp(Y), M, B)
            out[f"gemv{ti}_B{B}"] = Y[:B].copy()
        out[f"gemv{ti}_meta"] = np.array([typ, K, M, 7 + ti, 100 + ti], np.int64)
    return out


def kernel_cases(ref, orc):
    out = {}
    # rmsnorm
    x = gen_normal(orc, 11, "rx", 5120) * 3.0
    w = gen_normal(orc, 12, "rw", 5120) * 0.1 + 1.0
    o = np.zeros(5120, np.float32)
    ref.cwref_rmsnorm(vp(o), vp(x), vp(w), 5120)
    out["rmsnorm"] = o
    # rope on 24 heads x 256 at pos 777
    q = gen_normal(orc, 13, "rq", 24 * 256)
    qq = q.copy()
    ref.cwref_rope(vp(qq), 24, 777)
    out["rope_p777"] = qq
    # attention: KV over 38 slots, query at pos 37, full geometry
    T, NKV, HD, NH = 38, 4, 256, 24
    Kb = gen_normal(orc, 14, "ak", T * NKV * HD)
    Vb = gen_normal(orc, 15, "av", T * NKV * HD)
    qa = gen_normal(orc, 16, "aq", NH * HD)
    ga = gen_normal(orc, 17, "ag", NH * HD)
    y = np.zeros(NH * HD, np.float32)
    ref.cwref_attention(vp(Kb), vp(Vb), 0, T - 1, vp(qa), vp(ga), vp(y))
    out["attn_t0_p37"] = y.copy()
    ref.cwref_attention(vp(Kb), vp(Vb), 1, T - 1, vp(qa), vp(ga), vp(y))
    out["attn_t1_p37"] = y.copy()
    # GDN: conv + gdn_step, 3 consecutive positions from a seeded state
    LVH, LSD, QKV = 48, 128, 10240
    S = gen_normal(orc, 18, "gs", LVH * LSD * LSD) * 0.1
    cs = gen_normal(orc, 19, "gc", QKV * 3)
    cw = gen_normal(orc, 20, "gcw", QKV * 4) * 0.1
    nw = np.ones(LSD, np.float32)
    A = -np.ones(LVH, np.float32)
    dt = np.zeros(LVH, np.float32)
    for p in range(3):
        qkv = gen_normal(orc, 30 + p, "gq", QKV)
        z = gen_normal(orc, 40 + p, "gz", LVH * LSD)
        a = gen_normal(orc, 50 + p, "ga", LVH)
        b = gen_normal(orc, 60 + p, "gb", LVH)
        ref.cwref_decay_beta(vp(A), vp(dt), vp(a), vp(b), LVH)
        o = np.zeros(LVH * LSD, np.float32)
        ref.cwref_gdn_step(vp(S), vp(cs), vp(cw), vp(nw), vp(qkv), vp(z), vp(a), vp(b), vp(o))
        out[f"gdn_out_p{p}"] = o.copy()
    out["gdn_S_sub"] = S.reshape(-1)[::97].copy()
    out["gdn_S_norm"] = np.array([np.linalg.norm(S.astype(np.float64))])
    out["gdn_conv"] = cs.copy()
    return out


def main():
    ref = load_ref()
    orc = load_oracle()
    fx = {}
    fx.update(gemv_cases(ref, orc))
    fx.update(kernel_cases(ref, orc))
    np.savez_compressed(HERE / "ref_kernels.npz", **fx)
    print("wrote", HERE / "ref_kernels.npz", sum(v.nbytes for v in fx.values()), "bytes raw")


if __name__ == "__main__":
    main()
