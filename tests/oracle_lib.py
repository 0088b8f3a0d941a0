"""Test-side access to the CPU oracle (oracle/liboracle.so) and the seeded
input generator it shares with the engine (cwen_b200/host/synth.c).

Test infrastructure only: the oracle is the checker, never the thing measured.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_SO = ROOT / "oracle" / "liboracle.so"
_orc = None


def vp(a):
    return a.ctypes.data_as(C.c_void_p)


class CwDims(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "n_embd", "n_ff", "n_vocab", "n_layer", "n_head", "n_head_kv", "head_dim", "n_rot",
        "ssm_n_kh", "ssm_n_vh", "ssm_d", "conv_k", "full_interval", "has_mtp")]


def load_oracle():
    global _orc
    if _orc is None:
        srcs = [ROOT / "oracle" / "cwen_oracle.c", ROOT / "cwen_b200" / "host" / "synth.c"]
        if not ORACLE_SO.exists() or any(s.stat().st_mtime > ORACLE_SO.stat().st_mtime for s in srcs):
            subprocess.check_call([str(ROOT / "oracle" / "build_oracle.sh")])
        L = C.CDLL(str(ORACLE_SO))
        L.cw_synth_q4_0.argtypes = [C.c_uint64, C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
        L.cw_synth_q8_0.argtypes = [C.c_uint64, C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
        L.cw_synth_normal.argtypes = [C.c_uint64, C.c_char_p, C.c_float, C.c_float, C.c_void_p, C.c_size_t]
        L.cw_synth_ids.argtypes = [C.c_uint64, C.c_char_p, C.c_int, C.c_void_p, C.c_size_t]
        L.or_gemvb.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]
        L.or_set_xround.argtypes = [C.c_int]
        L.or_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.or_rope.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.or_attention.argtypes = [C.POINTER(CwDims), C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                   C.c_void_p, C.c_void_p]
        L.or_gdn_step.argtypes = [C.POINTER(CwDims), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p]
        L.or_conv1d_update.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.or_argmax.argtypes = [C.c_void_p, C.c_int]
        L.or_argmax.restype = C.c_int
        L.cw_dims_full.argtypes = [C.POINTER(CwDims)]
        L.cw_dims_tiny.argtypes = [C.POINTER(CwDims)]
        L.or_model_synth.argtypes = [C.POINTER(CwDims), C.c_uint64, C.c_int, C.c_int]
        L.or_model_synth.restype = C.c_void_p
        L.or_model_free.argtypes = [C.c_void_p]
        L.or_reset.argtypes = [C.c_void_p]
        L.or_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.or_logits.argtypes = [C.c_void_p]
        L.or_logits.restype = C.POINTER(C.c_float)
        L.or_hidden.argtypes = [C.c_void_p]
        L.or_hidden.restype = C.POINTER(C.c_float)
        L.or_layer_out.argtypes = [C.c_void_p, C.c_int]
        L.or_layer_out.restype = C.POINTER(C.c_float)
        L.or_gdn_state.argtypes = [C.c_void_p, C.c_int]
        L.or_gdn_state.restype = C.POINTER(C.c_float)
        L.or_generate.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.or_generate.restype = C.c_int
        _orc = L
    return _orc


def gen_q(orc, seed: int, stream: str, typ: int, K: int, M: int) -> np.ndarray:
    """Seeded GGUF Q4_0 (typ 2) or Q8_0 (typ 8) matrix, K per row, M rows."""
    nbytes = (K // 32) * (18 if typ == 2 else 34) * M
    W = np.zeros(nbytes, np.uint8)
    fn = orc.cw_synth_q4_0 if typ == 2 else orc.cw_synth_q8_0
    fn(seed, stream.encode(), K, M, vp(W), 0)
    return W


def gen_normal(orc, seed: int, stream: str, n: int) -> np.ndarray:
    v = np.zeros(n, np.float32)
    orc.cw_synth_normal(seed, stream.encode(), 0.0, 1.0, vp(v), n)
    return v


def oracle_gemvb(orc, typ, W, K, M, X):
    B = X.shape[0]
    Y = np.zeros((B, M), np.float32)
    orc.or_gemvb(typ, vp(W), K, M, vp(np.ascontiguousarray(X, np.float32)), K, vp(Y), M, B)
    return Y


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
