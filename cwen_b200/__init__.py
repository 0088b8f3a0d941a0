"""ctypes binding of the cwen B200 engine (include/cwen_cuda.h).

The engine is native: CUDA kernels for sm_100a and a C host side, all in
cwen_b200/libcwen_cuda.so.  This module only loads that library and declares
its C ABI for tests and bench.py; there is no Python or CPU fallback, and
`lib()` raises if the library is missing.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libcwen_cuda.so"

CWEN_T_F32, CWEN_T_Q4_0, CWEN_T_Q8_0 = 0, 2, 8


class Dims(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "n_embd", "n_ff", "n_vocab", "n_layer", "n_head", "n_head_kv", "head_dim", "n_rot",
        "ssm_n_kh", "ssm_n_vh", "ssm_d", "conv_k", "full_interval", "has_mtp")]


class SpecCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("spec", "use_mtp", "max_draft", "min_draft", "n_key", "cooldown", "debug")]


class SpecStats(C.Structure):
    _fields_ = [(n, C.c_longlong) for n in ("cycles", "drafted", "full", "shortw", "kept", "plain_steps")]


class CwenError(RuntimeError):
    pass


_lib = None

# name -> (restype, argtypes)
_SIGS = {
    "cwen_cuda_last_error": (C.c_char_p, []),
    "cwen_cuda_init": (C.c_int, [C.c_int, C.c_int, C.c_int]),
    "cwen_cuda_shutdown": (None, []),
    "cwen_cuda_weight_upload": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "cwen_cuda_gemvb": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "cwen_cuda_gemvb_static": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "cwen_cuda_gemvb_static_status": (C.c_int, [C.c_void_p]),
    "cwen_cuda_accept_logits": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                          C.c_void_p]),
    "cwen_cuda_mtp_step": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "cwen_cuda_mtp_read": (C.c_int, [C.c_int, C.c_void_p]),
    "cwen_cuda_shard_config": (C.c_int, [C.c_int, C.c_int]),
    "cwen_cuda_shard_handle": (C.c_int, [C.c_void_p, C.c_int]),
    "cwen_cuda_shard_open": (C.c_int, [C.c_void_p, C.c_int]),
    "cwen_shard_rows": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "cwen_cuda_shard_rows_for": (C.c_int, [C.c_char_p, C.c_int, C.c_void_p, C.c_void_p]),
    "cwen_cuda_gemvb_host": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]),
    "cwen_cuda_gdn_verify": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                       C.c_void_p]),
    "cwen_cuda_model_config": (C.c_int, [C.POINTER(Dims)]),
    "cwen_cuda_upload": (C.c_int, [C.c_char_p, C.c_int, C.c_void_p, C.c_int, C.c_int]),
    "cwen_cuda_model_finalize": (C.c_int, []),
    "cwen_cuda_reset": (C.c_int, []),
    "cwen_cuda_n_past": (C.c_int, []),
    "cwen_cuda_forward_block": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "cwen_cuda_accept": (C.c_int, [C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_void_p]),
    "cwen_cuda_commit": (C.c_int, [C.c_int]),
    "cwen_cuda_forward_serial": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "cwen_cuda_logits": (C.c_int, [C.c_int, C.c_void_p]),
    "cwen_cuda_hidden": (C.c_int, [C.c_int, C.c_void_p]),
    "cwen_cuda_dump_layers": (C.c_int, [C.c_int]),
    "cwen_cuda_dump_read": (C.c_int, [C.c_int, C.c_int, C.c_void_p]),
    "cwen_cuda_mtp_ready": (C.c_int, []),
    "cwen_cuda_mtp_commit": (C.c_int, [C.c_int, C.c_int, C.c_int]),
    "cwen_cuda_mtp_commit_block": (C.c_int, [C.c_int, C.c_void_p, C.c_int]),
    "cwen_cuda_mtp_draft": (C.c_int, [C.c_int, C.c_void_p, C.c_int]),
    "cwen_cuda_gdn_state": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p]),
    "cwen_cuda_ctx": (C.c_int, []),
    "cwen_cuda_stream": (C.c_void_p, []),
    "cwen_load_gguf": (C.c_int, [C.c_char_p]),
    "cwen_gguf_dims": (C.c_int, [C.c_char_p, C.POINTER(Dims)]),
    "cwen_gguf_tensor_bytes": (C.c_int, [C.c_char_p, C.c_char_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]),
    "cwen_write_synth_gguf": (C.c_int, [C.c_char_p, C.POINTER(Dims), C.c_uint64, C.c_int]),
    "cw_model_tensor_count": (C.c_int, [C.POINTER(Dims)]),
    "cwen_load_synth": (C.c_int, [C.c_uint64, C.POINTER(Dims), C.c_int]),
    "cwen_dims_reference": (None, [C.POINTER(Dims)]),
    "cwen_dims_small": (None, [C.POINTER(Dims)]),
    "cwen_spec_defaults": (None, [C.POINTER(SpecCfg)]),
    "cwen_spec_from_env": (C.c_int, [C.POINTER(SpecCfg)]),
    "cwen_generate": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.POINTER(SpecCfg),
                                C.POINTER(SpecStats)]),
    "cwen_ngram_draft": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]),
    "cwen_ngram_map_new": (C.c_void_p, [C.c_int]),
    "cwen_ngram_map_free": (None, [C.c_void_p]),
    "cwen_ngram_map_update": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "cwen_ngram_map_draft": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]),
    "cwen_ngram_map_save": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "cwen_ngram_map_load": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "cwen_cuda_model_dims": (C.c_int, [C.POINTER(Dims)]),
    "cwen_serve": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "cw_synth_q4_0": (None, [C.c_uint64, C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_int]),
    "cw_synth_q8_0": (None, [C.c_uint64, C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_int]),
    "cw_synth_normal": (None, [C.c_uint64, C.c_char_p, C.c_float, C.c_float, C.c_void_p, C.c_size_t]),
    "cw_synth_ids": (None, [C.c_uint64, C.c_char_p, C.c_int, C.c_void_p, C.c_size_t]),
    "cwen_cuda_profile": (C.c_int, [C.c_int]),
    "cwen_cuda_profile_read": (C.c_int, [C.POINTER(C.c_double), C.POINTER(C.c_double),
                                         C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
}


def lib() -> C.CDLL:
    """Load libcwen_cuda.so (build it with `python cwen_b200/build.py`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise CwenError(f"{LIB_PATH} is missing: the engine is CUDA-only, build it first")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str = "cwen") -> None:
    if rc != 0:
        raise CwenError(f"{what}: rc={rc}: {lib().cwen_cuda_last_error().decode()}")


def ptr(a) -> C.c_void_p:
    """Address of a numpy array's data (or a torch tensor's device data)."""
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)


def dims(kind: str = "reference") -> Dims:
    d = Dims()
    (lib().cwen_dims_small if kind == "small" else lib().cwen_dims_reference)(C.byref(d))
    return d


def spec_cfg(**kw) -> SpecCfg:
    c = SpecCfg()
    lib().cwen_spec_defaults(C.byref(c))
    for k, v in kw.items():
        setattr(c, k, int(v))
    return c


def generate(tokens, n_gen: int, cfg: SpecCfg | None = None):
    """Prefill `tokens` and greedily generate n_gen ids through the C host
    driver (serial, or speculative when cfg.spec)."""
    import numpy as np
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.zeros(max(n_gen, 1), dtype=np.int32)
    st = SpecStats()
    n = lib().cwen_generate(ptr(t), len(t), n_gen, ptr(out), C.byref(cfg) if cfg else None, C.byref(st))
    if n < 0:
        check(n, "cwen_generate")
    return out[:n], st


# ---- seeded synthetic inputs (host/synth.c, the generator behind cwen_load_synth) ----
def synth_q(seed: int, stream: str, typ: int, K: int, M: int):
    """Seeded GGUF Q4_0 (typ 2) or Q8_0 (typ 8) matrix of M rows x K: scales
    |N(0, 0.01)| as f16, nibbles / int8 uniform."""
    import numpy as np
    W = np.zeros((K // 32) * (18 if typ == CWEN_T_Q4_0 else 34) * M, np.uint8)
    fn = lib().cw_synth_q4_0 if typ == CWEN_T_Q4_0 else lib().cw_synth_q8_0
    fn(seed, stream.encode(), K, M, ptr(W), 0)
    return W


def synth_normal(seed: int, stream: str, n: int, mean: float = 0.0, std: float = 1.0):
    import numpy as np
    v = np.zeros(n, np.float32)
    lib().cw_synth_normal(seed, stream.encode(), mean, std, ptr(v), n)
    return v


def synth_ids(seed: int, stream: str, V: int, n: int):
    import numpy as np
    v = np.zeros(n, np.int32)
    lib().cw_synth_ids(seed, stream.encode(), V, ptr(v), n)
    return v
