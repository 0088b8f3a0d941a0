"""GGUF loading and writing on the C host (no GPU).

The loader keeps the reference's checks (load_gguf, run.c:3230-3303): magic,
version 2/3, at most 4 dims, no zero or int-truncating dims, every tensor's
offset and extent inside the file.  cwen_gguf_dims runs the same parse and
geometry derivation as cwen_load_gguf without the engine, so every rejection
and the derived geometry are checked here; the GPU test (test_gguf_gpu.py)
loads the file into the engine.

The writer (cwen_write_synth_gguf) is checked against an independent reader
written here with `struct`: header, tensor table in the seeded model's
order, 32-byte aligned data, and every tensor's bytes equal to the seeded
generator's.
"""
import ctypes as C
import struct

import numpy as np
import pytest

EINVAL, ESTATE = -1, -4
GGUF_F32, GGUF_Q4_0, GGUF_Q8_0 = 0, 2, 8


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char * 96), ("type", C.c_int), ("ne0", C.c_int), ("ne1", C.c_int), ("kind", C.c_int)]


@pytest.fixture(scope="module")
def L():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    lib = cwen_b200.lib()
    lib.cw_model_tensor_desc.argtypes = [C.POINTER(cwen_b200.Dims), C.c_int, C.POINTER(TensorDesc)]
    lib.cw_tensor_nbytes.argtypes = [C.c_int, C.c_int, C.c_int]
    lib.cw_tensor_nbytes.restype = C.c_size_t
    lib.cw_synth_tensor.argtypes = [C.c_uint64, C.POINTER(TensorDesc), C.c_void_p, C.c_int]
    return lib


def _small(has_mtp=0):
    import cwen_b200
    d = cwen_b200.dims("small")
    d.has_mtp = has_mtp
    return d


def _dims_tuple(d):
    return tuple(getattr(d, f) for f, _ in d._fields_)


def _write(L, path, d, seed=7):
    import cwen_b200
    cwen_b200.check(L.cwen_write_synth_gguf(str(path).encode(), C.byref(d), seed, 2), "write_synth_gguf")
    return path.read_bytes()


def _read_gguf(buf):
    """Independent GGUF v3 reader: (version, kv dict, tensors [(name, dims, type, off)], data offset)."""
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from("<" + fmt, buf, pos)
        pos += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string():
        nonlocal pos
        n = take("Q")
        s = buf[pos:pos + n].decode()
        pos += n
        return s

    assert buf[:4] == b"GGUF"
    pos = 4
    ver = take("I")
    n_t, n_kv = take("Q"), take("Q")
    kv = {}
    for _ in range(n_kv):
        k = string()
        t = take("I")
        assert t == 8, "the writer stores string values only"
        kv[k] = string()
    tensors = []
    for _ in range(n_t):
        name = string()
        nd = take("I")
        dims = [take("Q") for _ in range(nd)]
        typ = take("I")
        off = take("Q")
        tensors.append((name, dims, typ, off))
    data = (pos + 31) // 32 * 32
    return ver, kv, tensors, data


@pytest.mark.parametrize("has_mtp", [0, 1])
def test_writer_matches_seeded_generator(L, tmp_path, has_mtp):
    import cwen_b200
    d = _small(has_mtp)
    buf = _write(L, tmp_path / "m.gguf", d)
    ver, kv, tensors, data = _read_gguf(buf)
    assert ver == 3 and kv == {"general.architecture": "qwen35"}
    assert len(tensors) == L.cw_model_tensor_count(C.byref(d))
    for i, (name, dims, typ, off) in enumerate(tensors):
        td = TensorDesc()
        assert L.cw_model_tensor_desc(C.byref(d), i, C.byref(td)) == 0
        assert name == td.name.decode() and typ == td.type
        assert dims == ([td.ne0, td.ne1] if td.ne1 > 1 else [td.ne0])
        assert off % 32 == 0 and (data + off) % 32 == 0
        nb = L.cw_tensor_nbytes(td.type, td.ne0, td.ne1)
        want = np.zeros(nb, np.uint8)
        L.cw_synth_tensor(7, C.byref(td), want.ctypes.data_as(C.c_void_p), 2)
        assert buf[data + off:data + off + nb] == want.tobytes(), name
    assert (has_mtp == 1) == any(t[0].startswith(f"blk.{d.n_layer}.nextn.") for t in tensors)
    # the engine's own parse derives the geometry the file was written from
    got = cwen_b200.Dims()
    cwen_b200.check(L.cwen_gguf_dims(str(tmp_path / "m.gguf").encode(), C.byref(got)), "gguf_dims")
    assert _dims_tuple(got) == _dims_tuple(d)


def test_load_without_engine_fails_after_the_parse(L, tmp_path):
    """A valid file parses; the load then stops at the engine (not initialised)."""
    _write(L, tmp_path / "m.gguf", _small())
    assert L.cwen_load_gguf(str(tmp_path / "m.gguf").encode()) == ESTATE
    assert b"model_config" in L.cwen_cuda_last_error() or b"init" in L.cwen_cuda_last_error()


# ---- malformed files: a minimal GGUF builder ----
def _gguf(tensors, kvs=(), version=3, magic=b"GGUF", n_tensors=None, data=b"", pad=True):
    """tensors: [(name, dims, type, off)]; kvs: [(key, type, payload bytes)]."""
    out = bytearray(magic + struct.pack("<I", version))
    out += struct.pack("<QQ", len(tensors) if n_tensors is None else n_tensors, len(kvs))
    for k, t, payload in kvs:
        out += struct.pack("<Q", len(k)) + k.encode() + struct.pack("<I", t) + payload
    for name, dims, typ, off in tensors:
        out += struct.pack("<Q", len(name)) + name.encode() + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", x) for x in dims) + struct.pack("<IQ", typ, off)
    if pad:
        out += b"\0" * ((-len(out)) % 32)
    return bytes(out + data)


def _vec(name, n):
    return (name, [n], GGUF_F32, 0)


def _expect_einval(L, tmp_path, blob, why):
    import cwen_b200
    p = tmp_path / "bad.gguf"
    p.write_bytes(blob)
    d = cwen_b200.Dims()
    assert L.cwen_gguf_dims(str(p).encode(), C.byref(d)) == EINVAL, why
    msg = L.cwen_cuda_last_error().decode()
    assert why in msg, msg


def test_rejections(L, tmp_path):
    ok = [_vec("output_norm.weight", 64)]
    data = b"\0" * 256
    # header
    _expect_einval(L, tmp_path, b"GGUF" + b"\0" * 10, "not a gguf file")
    _expect_einval(L, tmp_path, _gguf(ok, magic=b"GGUG", data=data), "bad magic")
    _expect_einval(L, tmp_path, _gguf(ok, version=1, data=data), "unsupported gguf version")
    _expect_einval(L, tmp_path, _gguf(ok, version=4, data=data), "unsupported gguf version")
    _expect_einval(L, tmp_path, _gguf(ok, n_tensors=5000, data=data), "too many tensors")
    # key/values
    _expect_einval(L, tmp_path, _gguf(ok, kvs=[("x", 13, b"")], data=data), "unknown kv type")
    _expect_einval(L, tmp_path, _gguf(ok, kvs=[("general.alignment", 4, struct.pack("<I", 3))], data=data),
                   "bad general.alignment")
    _expect_einval(L, tmp_path, _gguf(ok, kvs=[("s", 8, struct.pack("<Q", 1 << 40))], data=data), "truncated")
    _expect_einval(L, tmp_path, _gguf([("a" * 200, [64], GGUF_F32, 0)], data=data), "string too long")
    # tensor table
    _expect_einval(L, tmp_path, _gguf([("t", [1, 1, 1, 1, 1], GGUF_F32, 0)], data=data), "n_dims outside 1..4")
    _expect_einval(L, tmp_path, _gguf([("t", [0], GGUF_F32, 0)], data=data), "dim zero or beyond INT_MAX")
    _expect_einval(L, tmp_path, _gguf([("t", [1 << 31], GGUF_F32, 0)], data=data), "dim zero or beyond INT_MAX")
    _expect_einval(L, tmp_path, _gguf([("t", [32, 65536, 65536], GGUF_F32, 0)], data=data),
                   "tensor rows beyond INT_MAX")
    _expect_einval(L, tmp_path, _gguf([("t", [48, 2], GGUF_Q4_0, 0)], data=data),
                   "quantized row length not a multiple of 32")
    # data extents
    _expect_einval(L, tmp_path, _gguf([("t", [64], GGUF_F32, 256)], data=data), "tensor offset out of file")
    _expect_einval(L, tmp_path, _gguf([("t", [65], GGUF_F32, 0)], data=data), "extent beyond file")
    _expect_einval(L, tmp_path, _gguf([("t", [64, 4], GGUF_Q4_0, 200)], data=data), "extent beyond file")
    # geometry
    _expect_einval(L, tmp_path, _gguf(ok, data=data), "missing token_embd.weight")
    # paths
    import cwen_b200
    d = cwen_b200.Dims()
    assert L.cwen_gguf_dims(str(tmp_path / "nope.gguf").encode(), C.byref(d)) == EINVAL
    assert L.cwen_gguf_dims(str(tmp_path).encode(), C.byref(d)) == EINVAL


def test_truncations_of_a_valid_file(L, tmp_path):
    """Every cut of the header and tensor table, and a cut inside the last
    tensor's data, is an error (never a read past the end)."""
    import cwen_b200
    buf = _write(L, tmp_path / "m.gguf", _small())
    _, _, tensors, data = _read_gguf(buf)
    cuts = sorted(set(list(range(0, data, max(1, data // 97))) + [data - 1, len(buf) - 1]))
    d = cwen_b200.Dims()
    p = tmp_path / "cut.gguf"
    for n in cuts:
        p.write_bytes(buf[:n])
        assert L.cwen_gguf_dims(str(p).encode(), C.byref(d)) == EINVAL, n


def test_write_gguf_tool(L, tmp_path):
    """python -m cwen_b200.write_gguf: the maintained writer of the seeded model."""
    import subprocess
    import sys

    import cwen_b200
    out = tmp_path / "tool.gguf"
    r = subprocess.run([sys.executable, "-m", "cwen_b200.write_gguf", str(out), "--small", "--mtp", "--seed", "7"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert out.read_bytes() == _write(L, tmp_path / "lib.gguf", _small(1))
    got = cwen_b200.Dims()
    cwen_b200.check(L.cwen_gguf_dims(str(out).encode(), C.byref(got)), "gguf_dims")
    assert _dims_tuple(got) == _dims_tuple(_small(1))
    r = subprocess.run([sys.executable, "-m", "cwen_b200.write_gguf", str(tmp_path / "no" / "x.gguf"), "--small"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "cannot write" in r.stderr


def test_mutated_files_never_crash(L, tmp_path):
    """Fuzz in the spirit of the reference's loader fuzzer (run.c:3811-3926):
    random flips, overwrites and cuts of a valid file are accepted or
    rejected -- never a crash, never a read outside the mapping (a fault here
    would end the test process)."""
    import cwen_b200
    base = bytearray(_write(L, tmp_path / "m.gguf", _small(1)))
    _, _, tensors, data = _read_gguf(bytes(base))
    rng = np.random.default_rng(1234)
    p = tmp_path / "fz.gguf"
    d = cwen_b200.Dims()
    outcomes = set()
    for it in range(400):
        b = bytearray(base)
        kind = it % 4
        if kind == 0:  # flip bytes in the header and tensor table
            for _ in range(int(rng.integers(1, 6))):
                b[int(rng.integers(0, data))] ^= int(rng.integers(1, 256))
        elif kind == 1:  # a random u64 over a count, dim or offset field
            pos = int(rng.integers(4, data - 8))
            b[pos:pos + 8] = int(rng.integers(0, 1 << 63)).to_bytes(8, "little")
        elif kind == 2:  # cut anywhere
            b = b[:int(rng.integers(0, len(b)))]
        else:  # a huge or tiny value in a tensor's dims
            pos = int(rng.integers(24, data - 8))
            b[pos:pos + 8] = int(rng.choice([0, 1, 31, 0x7FFFFFFF, 0x80000000, 1 << 40])).to_bytes(8, "little")
        p.write_bytes(bytes(b))
        rc = L.cwen_gguf_dims(str(p).encode(), C.byref(d))
        assert rc in (0, EINVAL, -3), rc
        outcomes.add(rc)
    assert EINVAL in outcomes
