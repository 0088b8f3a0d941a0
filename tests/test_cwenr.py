"""CWENR sidecars on the C host (no GPU).

The reference binds Q4_0 tensors of a GGUF to an offline sidecar written by
its repack tool (load_cwenr, run.c:3305-3643).  cwen_load_gguf does the same
and uploads the sidecar's bytes; cwen_gguf_tensor_bytes returns exactly the
bytes it would upload, so the binding rules are checked here without a GPU:

- fixtures: a tiny GGUF and its v2/v3/v4 sidecars written by the reference's
  own tools/repack_q4.py (tests/golden/make_cwenr.py); every Q4_0 tensor is
  bound and reads back as the GGUF's bytes, the f32 and Q8_0 tensors come
  from the GGUF;
- the bytes come from the sidecar: a changed qs byte or scale in the sidecar
  (each side of a v4 pair separately) shows up in that tensor only;
- whole-file rejections (short file, bad magic, stale stamp, bad version,
  too many entries, data base or directory outside the file, nothing bound)
  and per-entry skips (unknown name, non-Q4_0 tensor, shape, streams out of
  the file, v2 byte count) fall back to the GGUF like the reference;
- the sidecar path rule (CWEN_REPACK, MODEL.gguf -> MODEL.cwenr, else
  MODEL + ".cwenr") and an unstamped sidecar;
- the test writer (cwenr_util.write_cwenr, used by the GPU test) reproduces
  the reference tool's files byte for byte.
"""
import ctypes as C
import shutil
import struct
from pathlib import Path

import pytest

from cwenr_util import GGUF_Q4_0, read_gguf_table, write_cwenr

GOLD = Path(__file__).resolve().parent / "golden"
GGUF = GOLD / "cwenr_tiny.gguf"


@pytest.fixture(scope="module")
def L():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    return cwen_b200.lib()


@pytest.fixture(autouse=True)
def _no_env(monkeypatch):
    monkeypatch.delenv("CWEN_REPACK", raising=False)


def _read(L, path, name):
    side = C.c_int(-1)
    n = L.cwen_gguf_tensor_bytes(str(path).encode(), name.encode(), None, 0, C.byref(side))
    assert n > 0, n
    buf = C.create_string_buffer(n)
    assert L.cwen_gguf_tensor_bytes(str(path).encode(), name.encode(), buf, n, C.byref(side)) == n
    return buf.raw, side.value


def _setup(tmp_path, sidecar: bytes, name="m.cwenr"):
    g = tmp_path / "m.gguf"
    shutil.copy(GGUF, g)
    (tmp_path / name).write_bytes(sidecar)
    return g


def _table():
    return read_gguf_table(GGUF.read_bytes())


def _expect_all(L, g, bound):
    """Every tensor reads back as the GGUF's bytes; Q4_0 ones from the sidecar iff bound."""
    raw = GGUF.read_bytes()
    for n, t, ne0, r, o, nb in _table():
        b, side = _read(L, g, n)
        assert b == raw[o:o + nb], n
        assert side == (1 if bound and t == GGUF_Q4_0 else 0), n


@pytest.mark.parametrize("ver", [2, 3, 4])
def test_reference_sidecar_binds_every_q4_tensor(L, tmp_path, ver):
    g = _setup(tmp_path, (GOLD / f"cwenr_tiny.v{ver}.cwenr").read_bytes())
    _expect_all(L, g, True)


@pytest.mark.parametrize("ver", [2, 3, 4])
def test_writer_matches_reference_tool(ver):
    assert write_cwenr(GGUF.read_bytes(), ver) == (GOLD / f"cwenr_tiny.v{ver}.cwenr").read_bytes()


def _entries(sc):
    ver, n, base = struct.unpack_from("<IIQ", sc, 8)
    out = {}
    for i in range(n):
        e = 32 + 128 * i
        name = sc[e:e + 96].split(b"\0")[0].decode()
        ne0, ne1, a, b, flags = struct.unpack_from("<iiQQI", sc, e + 96)
        out[name] = (i, ne0, ne1, a, b, flags)
    return ver, base, out


@pytest.mark.parametrize("ver", [2, 3, 4])
def test_bytes_come_from_the_sidecar(L, tmp_path, ver):
    sc = bytearray((GOLD / f"cwenr_tiny.v{ver}.cwenr").read_bytes())
    _, base, ents = _entries(sc)
    raw = GGUF.read_bytes()
    tab = {n: (o, nb) for n, t, ne0, r, o, nb in _table()}
    # change block 1's first qs byte and its scale in the sidecar, per tensor
    for name in ("blk.0.ffn_gate.weight", "blk.0.ffn_up.weight", "blk.0.ssm_out.weight"):
        _, ne0, ne1, a, b, flags = ents[name]
        side = {1: 0, 2: 1}.get(flags, -1) if ver == 4 else -1
        if ver == 2:
            sc[base + a + 20 + 0] ^= 0x5A
            d = struct.unpack_from("<f", sc, base + a + 20 + 16)[0]
            struct.pack_into("<f", sc, base + a + 20 + 16, d * 2.0)
        elif side >= 0:
            sc[base + a + 32 + 16 * side] ^= 0x5A
            sc[base + b + 4 + 2 * side + 1] ^= 0x04  # exponent bit of dA / dB
        else:
            sc[base + a + 16] ^= 0x5A
            sc[base + b + 2 + 1] ^= 0x04
    g = _setup(tmp_path, bytes(sc))
    for name in ("blk.0.ffn_gate.weight", "blk.0.ffn_up.weight", "blk.0.ssm_out.weight"):
        o, nb = tab[name]
        want = bytearray(raw[o:o + nb])
        want[18 + 2] ^= 0x5A  # block 1: qs[0]
        if ver == 2:
            import numpy as np
            d = np.frombuffer(bytes(want[18:20]), "<f2").astype(np.float32)[0] * 2.0
            want[18:20] = np.float16(d).tobytes()
        else:
            want[18 + 1] ^= 0x04
        b, side = _read(L, g, name)
        assert side == 1 and b == bytes(want), name
    for name in ("blk.0.attn_k.weight", "blk.0.attn_v.weight"):  # untouched
        o, nb = tab[name]
        assert _read(L, g, name) == (raw[o:o + nb], 1)


def _patched(ver, fn):
    sc = bytearray((GOLD / f"cwenr_tiny.v{ver}.cwenr").read_bytes())
    fn(sc)
    return bytes(sc)


@pytest.mark.parametrize("case", ["short", "magic", "stale", "version", "count", "base", "directory", "none"])
def test_unusable_sidecar_is_ignored(L, tmp_path, case):
    def f(sc):
        if case == "magic":
            sc[0:8] = b"CWENR002"
        elif case == "stale":
            struct.pack_into("<I", sc, 28, struct.unpack_from("<I", sc, 28)[0] + 1)
        elif case == "version":
            struct.pack_into("<I", sc, 8, 5)
        elif case == "count":
            struct.pack_into("<I", sc, 12, 1025)
        elif case == "base":
            struct.pack_into("<Q", sc, 16, len(sc))
        elif case == "directory":
            struct.pack_into("<I", sc, 12, (len(sc) - 32) // 128 + 1)
        elif case == "none":  # every entry names a tensor the GGUF lacks
            n = struct.unpack_from("<I", sc, 12)[0]
            for i in range(n):
                sc[32 + 128 * i] = ord("X")
    sc = b"CWENR001" + bytes(8) if case == "short" else _patched(3, f)
    _expect_all(L, _setup(tmp_path, sc), False)


@pytest.mark.parametrize("case", ["unknown", "q8", "shape", "oob_qs", "oob_sc", "v2_size"])
def test_bad_entry_is_skipped(L, tmp_path, case):
    ver = 2 if case == "v2_size" else 3
    sc = bytearray((GOLD / f"cwenr_tiny.v{ver}.cwenr").read_bytes())
    _, base, ents = _entries(sc)
    victim = "blk.0.ssm_out.weight"
    i, ne0, ne1, a, b, flags = ents[victim]
    e = 32 + 128 * i
    if case == "unknown":
        sc[e:e + 96] = b"blk.9.nothing.weight".ljust(96, b"\0")
    elif case == "q8":
        sc[e:e + 96] = b"output.weight".ljust(96, b"\0")
        struct.pack_into("<ii", sc, e + 96, 64, 2)
    elif case == "shape":
        struct.pack_into("<i", sc, e + 100, ne1 + 1)
    elif case == "oob_qs":
        struct.pack_into("<Q", sc, e + 104, len(sc) - base - 8)
    elif case == "oob_sc":
        struct.pack_into("<Q", sc, e + 112, (1 << 64) - 8)  # would wrap as an end offset
    elif case == "v2_size":
        struct.pack_into("<Q", sc, e + 112, b - 20)
    g = _setup(tmp_path, bytes(sc))
    raw = GGUF.read_bytes()
    for n, t, ne0_, r, o, nb in _table():
        data, side = _read(L, g, n)
        assert data == raw[o:o + nb]
        assert side == (1 if t == GGUF_Q4_0 and n != victim else 0), n


def test_sidecar_path_rules(L, tmp_path, monkeypatch):
    sc = (GOLD / "cwenr_tiny.v4.cwenr").read_bytes()
    # MODEL.gguf -> MODEL.cwenr
    g = _setup(tmp_path, sc)
    assert _read(L, g, "blk.0.ffn_up.weight")[1] == 1
    # a path without .gguf: MODEL + ".cwenr"
    d2 = tmp_path / "b"
    d2.mkdir()
    g2 = d2 / "model.bin"
    shutil.copy(GGUF, g2)
    (d2 / "model.bin.cwenr").write_bytes(sc)
    assert _read(L, g2, "blk.0.ffn_up.weight")[1] == 1
    # CWEN_REPACK names the sidecar (and the default one is then not used)
    d3 = tmp_path / "c"
    d3.mkdir()
    g3 = d3 / "m.gguf"
    shutil.copy(GGUF, g3)
    assert _read(L, g3, "blk.0.ffn_up.weight")[1] == 0
    (d3 / "elsewhere.bin").write_bytes(sc)
    monkeypatch.setenv("CWEN_REPACK", str(d3 / "elsewhere.bin"))
    assert _read(L, g3, "blk.0.ffn_up.weight")[1] == 1
    monkeypatch.setenv("CWEN_REPACK", str(d3 / "missing.cwenr"))
    assert _read(L, g, "blk.0.ffn_up.weight")[1] == 0


def test_unstamped_sidecar_is_trusted(L, tmp_path):
    # a legacy sidecar (zero stamp) binds even when the GGUF's size differs
    sc = write_cwenr(GGUF.read_bytes(), 3, stamp_pages=0)
    g = _setup(tmp_path, sc)
    with open(g, "ab") as f:
        f.write(bytes(8192))
    raw = GGUF.read_bytes()
    for n, t, ne0, r, o, nb in _table():
        assert _read(L, g, n) == (raw[o:o + nb], 1 if t == GGUF_Q4_0 else 0)


def test_stamp_follows_the_gguf_size(L, tmp_path):
    g = _setup(tmp_path, (GOLD / "cwenr_tiny.v3.cwenr").read_bytes())
    with open(g, "ab") as f:  # same page count: still fresh
        f.write(bytes(4096 - GGUF.stat().st_size % 4096 - 1))
    assert _read(L, g, "blk.0.ssm_out.weight")[1] == 1
    with open(g, "ab") as f:  # one page more: stale
        f.write(bytes(2))
    assert _read(L, g, "blk.0.ssm_out.weight")[1] == 0


def test_v2_scale_rounds_to_nearest_even(L, tmp_path):
    """A v2 sidecar stores f32 scales; the loader rounds them to f16 the way
    the reference's runtime split does (f32_to_f16, run.c:3623: IEEE
    round-to-nearest-even, as F16C's vcvtps2ph), including ties, the
    subnormal range and overflow to infinity."""
    import numpy as np
    sc = bytearray((GOLD / "cwenr_tiny.v2.cwenr").read_bytes())
    _, base, ents = _entries(sc)
    _, ne0, ne1, a, b, _ = ents["blk.0.ssm_out.weight"]
    nblk = ne0 // 32 * ne1
    one = np.float32(1.0)
    tie = np.float32(1.0 + 2.0 ** -11)       # halfway between two f16 values: rounds to even (1.0)
    tie_up = np.float32(1.0 + 3 * 2.0 ** -11)  # halfway, rounds up to the even neighbour
    vals = [np.float32(0.0123456), tie, tie_up, np.float32(3e-6), np.float32(-7.5e-8), np.float32(7e4),
            np.float32(-0.0), one]
    vals = (vals * ((nblk + len(vals) - 1) // len(vals)))[:nblk]
    for k, v in enumerate(vals):
        struct.pack_into("<f", sc, base + a + 20 * k + 16, float(v))
    g = _setup(tmp_path, bytes(sc))
    data, side = _read(L, g, "blk.0.ssm_out.weight")
    assert side == 1
    got = np.frombuffer(data, np.uint8).reshape(nblk, 18)[:, :2].copy().view("<u2").ravel()
    with np.errstate(over="ignore"):  # 7e4 is past the f16 range: +inf, as in the reference
        want = np.array(vals, np.float32).astype(np.float16).view("<u2")
    assert np.array_equal(got, want), (got[:8], want[:8])
