"""Test helpers for CWENR sidecars (test infrastructure, not the product).

read_gguf_table: an independent GGUF v2/v3 table reader (name, type, ne0,
rows, absolute data offset, byte count).  write_cwenr: a restatement of the
sidecar layout maci0/cwen's tools/repack_q4.py writes (its module docstring
and main(), lines 1-30 and 195-300): Q4_0 tensors in name order, v4 pairing
ffn_gate+ffn_up and attn_k+attn_v, every stream 64-byte aligned from a data
base that is itself 64-byte aligned past the directory, and the
{"CWEN", source pages} stamp.  test_cwenr.py checks it byte for byte
against sidecars the reference tool wrote (tests/golden/cwenr_tiny.*), so
the GPU test can build sidecars for models it writes at run time.
"""
from __future__ import annotations

import struct

import numpy as np

GGUF_F32, GGUF_Q4_0, GGUF_Q8_0 = 0, 2, 8
PAIRS = (("ffn_gate.weight", "ffn_up.weight"), ("attn_k.weight", "attn_v.weight"))


def _nbytes(typ, ne0, rows):
    return {GGUF_F32: ne0 * 4, GGUF_Q4_0: ne0 // 32 * 18, GGUF_Q8_0: ne0 // 32 * 34}[typ] * rows


def read_gguf_table(buf: bytes):
    """[(name, type, ne0, rows, abs_off, nbytes)] of a GGUF v2/v3 file."""
    p = 0

    def take(n):
        nonlocal p
        v = buf[p:p + n]
        p += n
        return v

    def u32():
        return struct.unpack("<I", take(4))[0]

    def u64():
        return struct.unpack("<Q", take(8))[0]

    def string():
        return take(u64()).decode()

    def skip(t):
        if t in (0, 1, 7):
            take(1)
        elif t in (2, 3):
            take(2)
        elif t in (4, 5, 6):
            take(4)
        elif t in (10, 11, 12):
            take(8)
        elif t == 8:
            string()
        elif t == 9:
            at, n = u32(), u64()
            for _ in range(n):
                skip(at)
        else:
            raise ValueError(f"kv type {t}")

    assert take(4) == b"GGUF"
    assert u32() in (2, 3)
    n_t, n_kv = u64(), u64()
    align = 32
    for _ in range(n_kv):
        key, t = string(), u32()
        if key == "general.alignment" and t in (4, 5):
            align = u32()
        else:
            skip(t)
    rows_ = []
    for _ in range(n_t):
        name = string()
        nd = u32()
        ne = [u64() for _ in range(nd)]
        typ, off = u32(), u64()
        rows = int(np.prod(ne[1:])) if nd > 1 else 1
        rows_.append((name, typ, ne[0], rows, off))
    base = (p + align - 1) // align * align
    return [(n, t, ne0, r, base + o, _nbytes(t, ne0, r)) for n, t, ne0, r, o in rows_]


def _align(n, a=64):
    return (n + a - 1) // a * a


def write_cwenr(gguf: bytes, ver: int, stamp_pages: int | None = None, blobs: dict | None = None) -> bytes:
    """The sidecar of a GGUF's Q4_0 tensors.  blobs: name -> replacement
    Q4_0 bytes (GGUF block form) to store instead of the GGUF's.
    stamp_pages None stamps the GGUF's own page count; 0 writes no stamp."""
    tab = {n: (t, ne0, r, o, nb) for n, t, ne0, r, o, nb in read_gguf_table(gguf)}
    q4 = sorted(n for n, v in tab.items() if v[0] == GGUF_Q4_0)

    def raw(n):
        if blobs and n in blobs:
            return np.frombuffer(blobs[n], np.uint8)
        _, ne0, r, o, nb = tab[n]
        return np.frombuffer(gguf[o:o + nb], np.uint8)

    plans, used = [], set()
    for n in q4:
        if n in used:
            continue
        partner = None
        if ver == 4:
            for a, b in PAIRS:
                if n.endswith(a) and n[:-len(a)] + b in tab and tab[n[:-len(a)] + b][0] == GGUF_Q4_0:
                    pn = n[:-len(a)] + b
                    if tab[pn][1:3] == tab[n][1:3]:
                        partner = pn
                    break
        plans.append((n, partner))
        used.add(n)
        if partner:
            used.add(partner)
    entries, payload, off = [], [], 0
    for n, partner in plans:
        _, ne0, r, _, _ = tab[n]
        nblk = ne0 // 32 * r
        src = raw(n).reshape(nblk, 18)
        if ver == 2:
            off = _align(off)
            d = src[:, :2].copy().view("<f2").astype("<f4").reshape(nblk, 1)
            blk = np.concatenate([src[:, 2:], d.view(np.uint8).reshape(nblk, 4)], axis=1)
            entries.append((n, ne0, r, off, nblk * 20, 0))
            payload.append((off, blk.tobytes()))
            off += nblk * 20
            continue
        if partner:
            srcb = raw(partner).reshape(nblk, 18)
            qs = np.stack([src[:, 2:], srcb[:, 2:]], axis=1).tobytes()
            sc = np.stack([src[:, :2], srcb[:, :2]], axis=1).tobytes()
        else:
            qs, sc = np.ascontiguousarray(src[:, 2:]).tobytes(), np.ascontiguousarray(src[:, :2]).tobytes()
        off = _align(off)
        qs_off = off
        off = _align(off + len(qs))
        sc_off = off
        off += len(sc)
        payload += [(qs_off, qs), (sc_off, sc)]
        if partner:
            entries.append((n, ne0, r, qs_off, sc_off, 1))
            entries.append((partner, ne0, r, qs_off, sc_off, 2))
        else:
            entries.append((n, ne0, r, qs_off, sc_off, 0))
    base = _align(32 + 128 * len(entries))
    pages = (len(gguf) + 4095) // 4096 if stamp_pages is None else stamp_pages
    out = bytearray(b"CWENR001" + struct.pack("<IIQ", ver, len(entries), base))
    out += struct.pack("<II", 0x4E455743 if pages else 0, pages)
    for n, ne0, r, a, b, flags in entries:
        rec = bytearray(128)
        rec[:len(n)] = n.encode()
        struct.pack_into("<iiQQII", rec, 96, ne0, r, a, b, flags if ver > 2 else 0, 0)
        out += rec
    out += b"\0" * (base - len(out))
    for o, blob in payload:
        out += b"\0" * (base + o - len(out))
        out += blob
    return bytes(out)
