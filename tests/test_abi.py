"""The C ABI library loads without a GPU and exports every function that
include/*.h declares (no compute calls here)."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(cwen_[a-z0-9_]+)\s*\(", txt):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def built():
    from cwen_b200 import build
    return build.build()


def test_library_loads(built):
    import cwen_b200
    L = cwen_b200.lib()
    assert L.cwen_cuda_last_error()


def test_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", str(built)], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    missing = sorted(_declared() - exported)
    assert not missing, missing
    assert len(_declared()) >= 6


def test_calls_before_init_fail_cleanly(built):
    import ctypes as C
    import cwen_b200
    L = cwen_b200.lib()
    wid = C.c_int(-1)
    rc = L.cwen_cuda_weight_upload(2, None, 64, 16, C.byref(wid))
    assert rc < 0


def test_every_entry_point_before_init_fails_cleanly(built):
    """Without an engine every call returns an error code (or the documented
    neutral value) -- no crash, no exit -- whatever its pointer arguments."""
    import ctypes as C

    import cwen_b200
    L = cwen_b200.lib()
    L.cwen_cuda_shutdown()  # idempotent when no engine is live
    assert L.cwen_cuda_ctx() == 0
    assert L.cwen_cuda_stream() is None
    skip = {"cwen_cuda_last_error", "cwen_cuda_init", "cwen_cuda_shutdown", "cwen_cuda_ctx", "cwen_cuda_stream",
            "cwen_cuda_n_past", "cwen_cuda_mtp_ready", "cwen_dims_reference", "cwen_dims_small",
            "cwen_spec_defaults", "cwen_spec_from_env", "cwen_ngram_draft", "cwen_ngram_map_new",
            "cwen_ngram_map_free", "cwen_ngram_map_update", "cwen_write_synth_gguf", "cwen_gguf_dims",
            "cwen_serve", "cwen_ngram_map_save", "cwen_ngram_map_load", "cwen_ngram_map_draft"}
    called = 0
    for name, (res, args) in cwen_b200._SIGS.items():
        if not name.startswith("cwen_") or name in skip or res is not C.c_int:
            continue
        vals = []
        for a in args:
            vals.append(None if a in (C.c_void_p, C.c_char_p) or issubclass(a, C._Pointer) else 0)
        rc = getattr(L, name)(*vals)
        assert rc < 0, (name, rc)
        assert L.cwen_cuda_last_error(), name
        called += 1
    assert called >= 20


def test_python_binding_declares_every_entry_point(built):
    """cwen_b200._SIGS gives every C-ABI function of include/*.h its ctypes
    signature, so Python callers never pass arguments unchecked."""
    import cwen_b200
    assert not sorted(_declared() - set(cwen_b200._SIGS))
