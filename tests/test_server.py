"""Binary-frame server (CWEN_SERVER=1; server_loop run.c:5063-5078 and
server_read_frame run.c:4216-4235) without a GPU: cwen_serve runs over a pair
of pipes with a Python function standing in for generation, so every framing
decision is checked -- valid requests, rejected counts with their payload
consumed, out-of-range ids, end of input between and inside frames, and a
generation error ending the loop.  The GPU test at the end drives the real
CLI on the small seeded model.
"""
import ctypes as C
import os
import struct
import subprocess
import threading

import numpy as np
import pytest

GEN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.POINTER(C.c_int32))
CTX, VOCAB = 64, 1000


def _frame(ids, n_gen, n_prompt=None):
    ids = list(ids)
    return struct.pack("<II", len(ids) if n_prompt is None else n_prompt, n_gen) + struct.pack(f"<{len(ids)}i", *ids)


def _serve(L, data, gen_py):
    calls = []

    @GEN
    def gen(user, toks, n_tok, n_gen, out):
        t = [toks[i] for i in range(n_tok)]
        calls.append((t, n_gen))
        r = gen_py(t, n_gen)
        if isinstance(r, int):
            return r
        for i, v in enumerate(r):
            out[i] = v
        return len(r)

    ri, wi = os.pipe()
    ro, wo = os.pipe()
    feeder = threading.Thread(target=lambda: (os.write(wi, data), os.close(wi)))
    chunks = []

    def read_all():
        for b in iter(lambda: os.read(ro, 1 << 20), b""):
            chunks.append(b)

    reader = threading.Thread(target=read_all)
    feeder.start()
    reader.start()
    rc = L.cwen_serve(ri, wo, CTX, VOCAB, gen, None)
    os.close(ri)
    os.close(wo)
    feeder.join()
    reader.join()
    os.close(ro)
    return rc, b"".join(chunks), calls


def _replies(buf):
    out, p = [], 0
    while p < len(buf):
        (n,) = struct.unpack_from("<I", buf, p)
        p += 4
        out.append(list(struct.unpack_from(f"<{n}i", buf, p)))
        p += 4 * n
    return out


@pytest.fixture(scope="module")
def L():
    import cwen_b200
    from cwen_b200 import build
    build.build()
    lib = cwen_b200.lib()
    lib.cwen_serve.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, GEN, C.c_void_p]
    return lib


def echo(t, n):
    return [(t[-1] + 1 + i) % VOCAB for i in range(n)]


def test_valid_and_rejected_frames(L):
    data = (_frame([5, 6, 7], 4)                      # valid
            + _frame([], 3)                           # n_prompt 0
            + _frame([1, 2], 0)                       # n_gen 0: payload consumed
            + _frame(list(range(CTX + 1)), 2)         # n_prompt > ctx: payload consumed
            + _frame([1, 2], CTX + 1)                 # n_gen > ctx
            + _frame([3, VOCAB], 2)                   # id out of range
            + _frame([-1], 2)                         # negative id
            + _frame([9], CTX))                       # valid again: the stream stayed aligned
    rc, out, calls = _serve(L, data, echo)
    assert rc == 0
    assert _replies(out) == [echo([5, 6, 7], 4), [], [], [], [], [], [], echo([9], CTX)]
    assert calls == [([5, 6, 7], 4), ([9], CTX)]


def test_end_of_input(L):
    # between frames, inside a header, inside a payload: a clean stop, no reply for the cut frame
    for tail in (b"", b"\x03\x00", _frame([1, 2, 3], 2)[:-4]):
        rc, out, calls = _serve(L, _frame([4], 1) + tail, echo)
        assert rc == 0 and _replies(out) == [echo([4], 1)] and len(calls) == 1
    # a count of 0xffffffff reads as end of input (the reference's sentinel)
    rc, out, _ = _serve(L, struct.pack("<II", 0xFFFFFFFF, 1) + _frame([4], 1), echo)
    assert rc == 0 and out == b""


def test_generation_error_ends_the_loop(L):
    rc, out, calls = _serve(L, _frame([1], 1) + _frame([2], 1) + _frame([3], 1),
                            lambda t, n: -5 if t == [2] else echo(t, n))
    assert rc == -5 and _replies(out) == [echo([1], 1)] and len(calls) == 2


def test_short_generation_is_replied_as_is(L):
    rc, out, _ = _serve(L, _frame([1], 10), lambda t, n: [7, 8])  # e.g. the context window filled
    assert rc == 0 and _replies(out) == [[7, 8]]


def test_bad_arguments(L):
    assert L.cwen_serve(-1, 1, CTX, VOCAB, GEN(echo), None) == -1


def test_cli_server_knob():
    from cwen_b200 import build
    r = subprocess.run([str(build.CLI), "synth:1:small"], env={**os.environ, "CWEN_SERVER": "yes"},
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "CWEN_SERVER must be 0 or 1" in r.stderr


@pytest.mark.gpu
def test_cli_server_on_gpu():
    """The CLI as a server on the small seeded model: replies equal the
    in-process serial generation of the same requests."""
    import cwen_b200
    from cwen_b200 import build
    build.build()
    d = cwen_b200.dims("small")
    reqs = [(np.random.default_rng(s).integers(0, d.n_vocab, size=n).astype(np.int32), g)
            for s, n, g in ((1, 12, 8), (2, 5, 3), (3, 30, 16))]
    data = b"".join(_frame(ids.tolist(), g) for ids, g in reqs) + _frame([d.n_vocab], 2)
    r = subprocess.run([str(build.CLI), "synth:7:small"], input=data, capture_output=True, timeout=300,
                       env={**{k: v for k, v in os.environ.items() if not k.startswith("CWEN_")},
                            "CWEN_SERVER": "1", "CWEN_CTX": "256"})
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    got = _replies(r.stdout)
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, 256, 16), "init")
    try:
        cwen_b200.check(L.cwen_load_synth(7, C.byref(d), 0), "load_synth")
        want = [cwen_b200.generate(ids, g, cwen_b200.spec_cfg(spec=0))[0].tolist() for ids, g in reqs]
    finally:
        L.cwen_cuda_shutdown()
    assert got == want + [[]]


def test_random_byte_streams_never_crash(L):
    """Random request streams (the reference fuzzes its frame decoder,
    run.c:3873-3891): every complete frame gets exactly one reply, nothing
    crashes, and the loop ends at end of input."""
    rng = np.random.default_rng(99)
    for it in range(60):
        parts = []
        for _ in range(int(rng.integers(1, 6))):
            n = int(rng.integers(0, 8))
            ids = rng.integers(-3, VOCAB + 3, size=n).tolist()
            parts.append(_frame(ids, int(rng.integers(0, CTX + 3)), n_prompt=int(rng.choice([n, n, 0, CTX + 1]))))
        data = b"".join(parts)
        if it % 3 == 0:
            data = data[:int(rng.integers(0, len(data) + 1))]
        rc, out, _ = _serve(L, data, echo)
        assert rc == 0
        _replies(out)  # well-formed: a count and that many ids, frame after frame
