"""Generate the CWENR fixtures in tests/golden/ with the REFERENCE's own tool.

Writes a tiny GGUF v3 file (cwenr_tiny.gguf) whose Q4_0 tensors cover every
kind of sidecar entry -- an ffn_gate/ffn_up pair and an attn_k/attn_v pair
(interleaved in v4), a solo Q4_0 matrix, plus an f32 vector and a Q8_0
matrix that a sidecar never holds -- and runs maci0/cwen's
tools/repack_q4.py on it for sidecar versions 2, 3 and 4
(cwenr_tiny.v2.cwenr ...).  The tests read the committed files; only this
script needs the reference sources.

Run where they are (first argument, else CWEN_REFERENCE_DIR, else a
checkout named "reference" beside this repository):
    python tests/golden/make_cwenr.py [REFERENCE_DIR]
"""
from __future__ import annotations

import os
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]

GGUF_F32, GGUF_Q4_0, GGUF_Q8_0 = 0, 2, 8

# (name, type, ne0, rows)
TENSORS = [
    ("blk.0.attn_norm.weight", GGUF_F32, 64, 1),
    ("blk.0.attn_k.weight", GGUF_Q4_0, 64, 3),
    ("blk.0.attn_v.weight", GGUF_Q4_0, 64, 3),
    ("blk.0.ffn_gate.weight", GGUF_Q4_0, 96, 5),
    ("blk.0.ffn_up.weight", GGUF_Q4_0, 96, 5),
    ("blk.0.ssm_out.weight", GGUF_Q4_0, 128, 4),
    ("output.weight", GGUF_Q8_0, 64, 2),
]


def tensor_bytes(rng, typ, ne0, rows):
    if typ == GGUF_F32:
        return rng.standard_normal(ne0 * rows).astype("<f4").tobytes()
    nb = ne0 // 32 * rows
    d = np.abs(rng.standard_normal(nb) * 0.01).astype("<f2")
    blk = np.zeros((nb, 18 if typ == GGUF_Q4_0 else 34), np.uint8)
    blk[:, :2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = rng.integers(0, 256, (nb, blk.shape[1] - 2), dtype=np.uint8)
    return blk.tobytes()


def gguf_string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: Path, seed: int = 11) -> None:
    """GGUF v3: one string kv, the tensor table, 32-byte aligned data."""
    rng = np.random.default_rng(seed)
    blobs = [tensor_bytes(rng, t, ne0, rows) for _, t, ne0, rows in TENSORS]
    head = b"GGUF" + struct.pack("<IQQ", 3, len(TENSORS), 1)
    head += gguf_string("general.architecture") + struct.pack("<I", 8) + gguf_string("cwen-test")
    off = 0
    table = b""
    offs = []
    for (name, typ, ne0, rows), blob in zip(TENSORS, blobs):
        off = (off + 31) & ~31
        offs.append(off)
        dims = [ne0] if rows == 1 else [ne0, rows]
        table += gguf_string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", x) for x in dims)
        table += struct.pack("<IQ", typ, off)
        off += len(blob)
    out = bytearray(head + table)
    out += b"\0" * (((len(out) + 31) & ~31) - len(out))
    base = len(out)
    out += b"\0" * off
    for o, blob in zip(offs, blobs):
        out[base + o: base + o + len(blob)] = blob
    path.write_bytes(bytes(out))


def main() -> int:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CWEN_REFERENCE_DIR", ROOT.parent / "reference"))
    tool = ref / "tools" / "repack_q4.py"
    if not tool.is_file():
        print(f"make_cwenr: no reference tool at {tool}", file=sys.stderr)
        return 1
    gguf = HERE / "cwenr_tiny.gguf"
    write_gguf(gguf)
    for ver in (2, 3, 4):
        out = HERE / f"cwenr_tiny.v{ver}.cwenr"
        subprocess.check_call([sys.executable, str(tool), str(gguf), "-o", str(out), "--sidecar-version", str(ver)],
                              cwd=str(ref / "tools"), env=dict(os.environ, PYTHONPATH=str(ref / "tools")),
                              stdout=subprocess.DEVNULL)
        print(f"{out.name}: {out.stat().st_size} bytes")
    print(f"{gguf.name}: {gguf.stat().st_size} bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
