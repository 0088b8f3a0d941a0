"""GatedDeltaNet verify step with rollback (b), stand-alone through the C ABI
(cwen_cuda_gdn_verify): conv1d_update + decay/beta + gdn_step with its gated
norm over the rows of a verify block, then the committed state advanced by
the kept rows only.

Checked against the reference's own outputs (the golden fixture of three
consecutive gdn_step positions, run.c:2014-2200), against the CPU oracle at
the benchmark geometry (48 value / 16 key heads, B = 8, every
rejection index 0..8), and through the rollback property: keeping k rows of
a B-row block leaves the state bit-identical to a k-row block.

Tolerance: relative L2 <= 1e-5 against the oracle and the reference (fp32
throughout; the kernel sums S^T k and S^T q in four partial sums of 32).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import CwDims, gen_normal, rel_l2, vp

pytestmark = pytest.mark.gpu

NKH, NVH, D = 16, 48, 128
QKV, Z = (2 * NKH + NVH) * D, NVH * D
PS = QKV + Z + 2 * NVH
EINVAL = -1  # CWEN_EINVAL (include/cwen_cuda.h)


@pytest.fixture(scope="module")
def eng():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, 64, 16), "init")
    yield L
    L.cwen_cuda_shutdown()


def _dims(nkh, nvh):
    d = CwDims()
    d.ssm_n_kh, d.ssm_n_vh, d.ssm_d = nkh, nvh, D
    return d


def _proj(orc, seed, B, nkh=NKH, nvh=NVH):
    qkv = (2 * nkh + nvh) * D
    ps = qkv + nvh * D + 2 * nvh
    return gen_normal(orc, seed, "gdnv.proj", B * ps).reshape(B, ps)


def _params(orc, seed, nkh=NKH, nvh=NVH):
    qkv = (2 * nkh + nvh) * D
    return {"convw": gen_normal(orc, seed, "gdnv.cw", qkv * 4) * 0.1,
            "A": -np.ones(nvh, np.float32), "dt": np.zeros(nvh, np.float32),
            "wn": np.ones(D, np.float32),
            "S": gen_normal(orc, seed + 1, "gdnv.S", nvh * D * D) * 0.1,
            "conv": gen_normal(orc, seed + 2, "gdnv.conv", qkv * 3)}


def _gpu_verify(L, proj, p, keep, nkh=NKH, nvh=NVH):
    """Run cwen_cuda_gdn_verify on copies of the state; returns (out, S, conv)."""
    import torch

    import cwen_b200
    dev = torch.device("cuda", 0)
    B, ps = proj.shape
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in p.items()}
    dproj = torch.from_numpy(np.ascontiguousarray(proj)).to(dev)
    out = torch.full((B, nvh * D), float("nan"), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    P = lambda x: C.c_void_p(x.data_ptr())
    cwen_b200.check(L.cwen_cuda_gdn_verify(nkh, nvh, B, P(dproj), ps, P(t["convw"]), P(t["A"]), P(t["dt"]),
                                           P(t["wn"]), P(t["S"]), P(t["conv"]), keep, P(out), None), "gdn_verify")
    torch.cuda.synchronize()
    return out.cpu().numpy(), t["S"].cpu().numpy(), t["conv"].cpu().numpy()


def _oracle_rows(orc, proj, p, rows, nkh=NKH, nvh=NVH):
    """The oracle's layer_linear GDN part (run.c:2339-2346) over block rows
    0..rows-1 from the committed state; returns (outs, S, conv)."""
    d = _dims(nkh, nvh)
    qkv_n, z_n = (2 * nkh + nvh) * D, nvh * D
    S, cs = p["S"].copy(), p["conv"].copy()
    outs = np.zeros((rows, z_n), np.float32)
    for b in range(rows):
        qkv = proj[b, :qkv_n].copy()
        z = proj[b, qkv_n:qkv_n + z_n].copy()
        al = proj[b, qkv_n + z_n:qkv_n + z_n + nvh].astype(np.float64) + p["dt"]
        be = proj[b, qkv_n + z_n + nvh:qkv_n + z_n + 2 * nvh].astype(np.float64)
        a = (p["A"] * np.where(al > 20, al, np.log1p(np.exp(al)))).astype(np.float32)
        bt = (1.0 / (1.0 + np.exp(-be))).astype(np.float32)
        orc.or_conv1d_update(vp(qkv), vp(cs), vp(p["convw"]), qkv_n)
        orc.or_gdn_step(C.byref(d), vp(S), vp(qkv), vp(z), vp(a), vp(bt), vp(p["wn"]), vp(outs[b]))
    return outs, S, cs


def test_gdn_verify_vs_reference_goldens(eng, orc, golden):
    """The reference's three consecutive gdn_step positions (the golden
    fixture's seeds and streams) as one 3-row block, all rows kept."""
    S = gen_normal(orc, 18, "gs", NVH * D * D) * 0.1
    cs = gen_normal(orc, 19, "gc", QKV * 3)
    cw = gen_normal(orc, 20, "gcw", QKV * 4) * 0.1
    proj = np.zeros((3, PS), np.float32)
    for r in range(3):
        proj[r, :QKV] = gen_normal(orc, 30 + r, "gq", QKV)
        proj[r, QKV:QKV + Z] = gen_normal(orc, 40 + r, "gz", Z)
        proj[r, QKV + Z:QKV + Z + NVH] = gen_normal(orc, 50 + r, "ga", NVH)
        proj[r, QKV + Z + NVH:] = gen_normal(orc, 60 + r, "gb", NVH)
    p = {"convw": cw, "A": -np.ones(NVH, np.float32), "dt": np.zeros(NVH, np.float32),
         "wn": np.ones(D, np.float32), "S": S, "conv": cs}
    out, S1, c1 = _gpu_verify(eng, proj, p, 3)
    for r in range(3):
        assert rel_l2(out[r], golden[f"gdn_out_p{r}"]) <= 1e-5, (r, rel_l2(out[r], golden[f"gdn_out_p{r}"]))
    assert rel_l2(S1.reshape(-1)[::97], golden["gdn_S_sub"]) <= 1e-5
    assert abs(np.linalg.norm(S1.astype(np.float64)) / golden["gdn_S_norm"][0] - 1) <= 1e-5
    assert np.array_equal(c1, golden["gdn_conv"])  # the raw inputs shift through unchanged


@pytest.mark.parametrize("keep", [0, 1, 3, 7, 8])
def test_gdn_verify_config1_vs_oracle(eng, orc, keep):
    """Config 1: B = 8 drafted rows, rejection index `keep` (0..8)."""
    B = 8
    proj = _proj(orc, 100, B)
    p = _params(orc, 200)
    out, S1, c1 = _gpu_verify(eng, proj, p, keep)
    ref_out, _, _ = _oracle_rows(orc, proj, p, B)
    _, S_k, c_k = _oracle_rows(orc, proj, p, keep)
    assert np.isfinite(out).all()
    assert rel_l2(out, ref_out) <= 1e-5, rel_l2(out, ref_out)
    if keep == 0:
        assert np.array_equal(S1, p["S"]) and np.array_equal(c1, p["conv"])
    else:
        assert rel_l2(S1, S_k) <= 1e-5, rel_l2(S1, S_k)
        assert np.array_equal(c1, c_k)


def test_gdn_verify_rollback_bitwise(eng, orc):
    """Keeping k rows of a 16-row block == a k-row block, bit for bit (state,
    conv state and the kept rows' outputs)."""
    B = 16
    proj = _proj(orc, 300, B)
    p = _params(orc, 400)
    full_out, _, _ = _gpu_verify(eng, proj, p, B)
    for k in (1, 2, 5, 9, 15, 16):
        out_k, S_k, c_k = _gpu_verify(eng, proj[:k], p, k)
        out_b, S_b, c_b = _gpu_verify(eng, proj, p, k)
        assert np.array_equal(S_b, S_k), k
        assert np.array_equal(c_b, c_k), k
        assert np.array_equal(out_b, full_out)
        assert np.array_equal(out_k, full_out[:k]), k


def test_gdn_verify_small_heads(eng, orc):
    """Another head geometry (4 key heads, 12 value heads; value head h reads
    key head h % 4), B = 5, 2 rows kept."""
    nkh, nvh = 4, 12
    proj = _proj(orc, 500, 5, nkh, nvh)
    p = _params(orc, 600, nkh, nvh)
    out, S1, c1 = _gpu_verify(eng, proj, p, 2, nkh, nvh)
    ref_out, _, _ = _oracle_rows(orc, proj, p, 5, nkh, nvh)
    _, S_k, c_k = _oracle_rows(orc, proj, p, 2, nkh, nvh)
    assert rel_l2(out, ref_out) <= 1e-5, rel_l2(out, ref_out)
    assert rel_l2(S1, S_k) <= 1e-5
    assert np.array_equal(c1, c_k)


def test_gdn_verify_range_errors(eng):
    L = eng
    nul = C.c_void_p(0)
    one = C.c_void_p(16)  # never dereferenced: every call below fails its argument check
    assert L.cwen_cuda_gdn_verify(NKH, NVH, 17, one, PS, one, one, one, one, one, one, 0, one, nul) == EINVAL
    assert L.cwen_cuda_gdn_verify(NKH, NVH, 8, one, PS, one, one, one, one, one, one, 9, one, nul) == EINVAL
    assert L.cwen_cuda_gdn_verify(NKH, NVH, 8, one, PS - 1, one, one, one, one, one, one, 0, one, nul) == EINVAL
    assert L.cwen_cuda_gdn_verify(NKH, NVH, 8, nul, PS, one, one, one, one, one, one, 0, one, nul) == EINVAL
    assert L.cwen_cuda_gdn_verify(0, NVH, 8, one, PS, one, one, one, one, one, one, 0, one, nul) == EINVAL
