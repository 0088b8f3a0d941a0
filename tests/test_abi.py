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
