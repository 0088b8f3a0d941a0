"""The cwen CLI's command line and knobs (no GPU): the reference's argument
rules (main, run.c:5128-5160; spec_config_init, run.c:4021-4053) -- help
exits 0, a bad argument exits 2 naming it, a bad knob exits 1 naming it --
and a clean failure when no GPU is present.
"""
import os
import subprocess

import pytest

CLI = None


@pytest.fixture(scope="module", autouse=True)
def cli():
    global CLI
    from cwen_b200 import build
    build.build()
    CLI = str(build.CLI)


def _run(*args, env=None):
    e = {k: v for k, v in os.environ.items() if not k.startswith("CWEN_")}
    e.update(env or {})
    return subprocess.run([CLI, *args], capture_output=True, text=True, env=e, timeout=120)


def test_help():
    r = _run("--help")
    assert r.returncode == 0 and r.stdout.startswith("usage: cwen")
    assert _run("-h").returncode == 0


@pytest.mark.parametrize("args,msg", [
    (["--bogus"], "unknown option '--bogus'"),
    (["-d"], "-d requires a value"),
    (["-d", "16"], "-d must be an integer in [1,15]"),
    (["-d", "0"], "-d must be an integer in [1,15]"),
    (["--draft-tokens", "x"], "--draft-tokens must be an integer in [1,15]"),
    (["m.gguf", "ids", "5", "extra"], "too many arguments"),
    (["m.gguf", "ids", "five"], "N_PREDICT must be an integer"),
])
def test_bad_arguments_exit_2(args, msg):
    r = _run(*args)
    assert r.returncode == 2, r.stderr
    assert msg in r.stderr, r.stderr


@pytest.mark.parametrize("env,msg", [
    ({"CWEN_SPEC": "2"}, "CWEN_SPEC must be 0 or 1"),
    ({"CWEN_SPEC": "yes"}, "CWEN_SPEC=yes is not an integer"),
    ({"CWEN_SPEC_NGRAM_N": "1"}, "CWEN_SPEC_NGRAM_N must be in [2,256]"),
    ({"CWEN_SPEC_MAX_DRAFT": "16"}, "CWEN_SPEC_MAX_DRAFT must be in [1,15]"),
    ({"CWEN_SPEC_MIN_DRAFT": "9"}, "CWEN_SPEC_MIN_DRAFT must be in [1,8]"),
    ({"CWEN_SPEC_COOLDOWN": "-1"}, "CWEN_SPEC_COOLDOWN must be in [0,100000]"),
    ({"CWEN_SPEC_DEBUG": "2"}, "CWEN_SPEC_DEBUG must be 0 or 1"),
    ({"CWEN_MTP": "on"}, "CWEN_MTP must be 0 or 1"),
])
def test_bad_knobs_exit_1(env, msg):
    r = _run("synth:1:small", env=env)
    assert r.returncode == 1, r.stderr
    assert msg in r.stderr, r.stderr


def test_context_knob_range():
    r = _run("synth:1:small", env={"CWEN_CTX": "63"})
    assert r.returncode == 2 and "CWEN_CTX must be an integer in [64,32768]" in r.stderr


def test_knob_defaults_and_parse_through_the_library():
    """cwen_spec_from_env: the reference's defaults (run.c:194-199) and the
    same messages through cwen_cuda_last_error for library callers."""
    import ctypes as C

    import cwen_b200
    L = cwen_b200.lib()
    c = cwen_b200.SpecCfg()
    L.cwen_spec_defaults(C.byref(c))
    assert (c.spec, c.use_mtp, c.max_draft, c.min_draft, c.n_key, c.cooldown, c.debug) == (0, 1, 8, 2, 16, 8, 0)
    old = {k: os.environ.get(k) for k in ("CWEN_SPEC", "CWEN_SPEC_MAX_DRAFT", "CWEN_SPEC_MIN_DRAFT", "CWEN_MTP")}
    try:
        os.environ.update(CWEN_SPEC="1", CWEN_SPEC_MAX_DRAFT="15", CWEN_SPEC_MIN_DRAFT="3", CWEN_MTP="0")
        assert L.cwen_spec_from_env(C.byref(c)) == 0
        assert (c.spec, c.max_draft, c.min_draft, c.use_mtp) == (1, 15, 3, 0)
        os.environ["CWEN_SPEC_MAX_DRAFT"] = "0"
        assert L.cwen_spec_from_env(C.byref(c)) == -1
        assert b"CWEN_SPEC_MAX_DRAFT must be in [1,15]" in L.cwen_cuda_last_error()
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def test_no_gpu_is_a_clean_error():
    """Without a usable GPU the CLI reports the CUDA error and exits 1."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _run("synth:1:small", "/nonexistent.ids", "2")
    assert r.returncode == 1, r.stderr
    assert r.stderr.strip().splitlines()[-1].startswith("cwen: "), r.stderr


def test_generate_rejects_knobs_outside_the_reference_ranges():
    """A caller-built cwen_spec_cfg is range-checked like the knobs (the
    driver's block buffers hold 1 + max_draft rows); the check comes before
    any engine call, so it runs without a GPU."""
    import ctypes as C

    import numpy as np

    import cwen_b200
    L = cwen_b200.lib()
    toks = np.arange(4, dtype=np.int32)
    out = np.zeros(4, np.int32)
    for kw in ({"max_draft": 16}, {"max_draft": 0}, {"min_draft": 0}, {"n_key": 1}, {"n_key": 257},
               {"cooldown": -1}):
        c = cwen_b200.spec_cfg(spec=1, **kw)
        rc = L.cwen_generate(cwen_b200.ptr(toks), 4, 4, cwen_b200.ptr(out), C.byref(c), None)
        assert rc == -1, kw
        assert b"spec knobs out of range" in L.cwen_cuda_last_error(), kw
    assert L.cwen_generate(None, 4, 4, cwen_b200.ptr(out), None, None) == -1
    c = cwen_b200.spec_cfg(spec=1)
    assert L.cwen_generate(cwen_b200.ptr(toks), 4, 4, cwen_b200.ptr(out), C.byref(c), None) == -4  # no engine
