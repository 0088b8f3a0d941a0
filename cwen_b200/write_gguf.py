"""Write the seeded random-init model as a GGUF file.

    python -m cwen_b200.write_gguf OUT.gguf [--seed N] [--small] [--mtp]

The file carries the reference's tensor names, shapes and types (Q4_0
matrices with f16 scales |N(0, 0.01)|, F32 norms = 1, ssm_a = -1,
ssm_dt.bias = 0, conv weights ~N(0, 0.1); --mtp adds the blk.<n_layer>
nextn block in Q8_0) with 32-byte aligned data, so the reference's own CLI
and this engine's `cwen` load it to the same weights `cwen_load_synth`
generates in memory.  The full geometry is a 15 GB file.
"""
from __future__ import annotations

import argparse
import ctypes as C
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m cwen_b200.write_gguf", description=__doc__.splitlines()[0])
    ap.add_argument("out")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--small", action="store_true", help="the small test geometry instead of the 27B one")
    ap.add_argument("--mtp", action="store_true", help="add the blk.<n_layer> nextn (MTP) block")
    ap.add_argument("--threads", type=int, default=0, help="host threads (0: all cores)")
    a = ap.parse_args(argv)
    import cwen_b200
    d = cwen_b200.dims("small" if a.small else "reference")
    d.has_mtp = 1 if a.mtp else 0
    L = cwen_b200.lib()
    rc = L.cwen_write_synth_gguf(a.out.encode(), C.byref(d), a.seed, a.threads)
    if rc:
        print(f"write_gguf: {L.cwen_cuda_last_error().decode()}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
