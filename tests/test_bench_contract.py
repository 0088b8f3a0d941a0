"""bench.py's JSON line keeps its contract (no GPU): the engine-facing
measurement functions are replaced by stand-ins returning fixed numbers, and
the line the default (decode) and GEMV workloads print is checked for every
key the harness reads -- metric/value/unit, the timing fields, `roofline`,
`e2e` with its copy bytes, `cpu_baseline`, `gpu_launches`, `clocks` -- and for
the arithmetic that turns the stand-in timings into the reported values.
A failing side measurement is reported inside the line, never instead of it.
"""
import argparse
import json

import pytest

import bench

CLK = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 10}


def _args(**kw):
    a = argparse.Namespace(gpus=1, steps=8, warmup=3, impl="ours", workload="decode", no_cpu_baseline=False,
                           no_side_workloads=False)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def _check_common(rec):
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "gpu_launches", "clocks", "roofline", "e2e"):
        assert k in rec, k
    assert rec["config"]["workload"]
    r = rec["roofline"]
    for k in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert k in r, k
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    e = rec["e2e"]
    for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"):
        assert k in e, k
    assert rec["clocks"] == CLK


def test_decode_line(monkeypatch, capsys):
    kern = {"gemv_ms_per_token": 3.0, "gemv_bytes_per_token": 14.4e9,
            "gemv_calls_per_token": 258.0, "launches_per_token": 470.0,
            "verify_ceiling": {"8": {"block_ms": 8.0, "serial_ms": 54.0, "x": 6.75, "pass": True}}}
    spec = {"workload": "config3", "tok_s": 600.0, "mtp_d8": {"workload": "mtp", "tok_s": 130.0}}
    monkeypatch.setattr(bench, "run_decode_ours", lambda a, ws, r, l: (6.8, kern, 145.0, CLK, spec, 30.0, [1, 2, 3]))
    monkeypatch.setattr(bench, "cpu_decode_baseline", lambda: (3.0, {"kind": "reference", "cores": 16,
                                                                     "variant": "avx512", "sample": "s"}, [1, 2, 3]))
    monkeypatch.setattr(bench, "gemv_ours_line", lambda *a, **k: ({"metric": "g", "value": 1.0, "unit": "GB/s",
                                                                    "roofline": {}, "e2e": {}}, None, None))

    def boom(*a, **k):
        raise RuntimeError("no engine here")

    monkeypatch.setattr(bench, "gdn_ours_line", boom)
    monkeypatch.setattr(bench, "run_mtp_ours", lambda ws, l: {
        "tps": 90.0, "clocks": CLK, "prefill": {"tokens": 32495, "seconds": 70.0, "tok_s": 464.2},
        "identical_to_serial": True, "mtp": {"cycles": 255}})
    monkeypatch.setattr(bench, "peaks", lambda: (6541.1, 1590.0, "measured"))
    import cwen_b200
    monkeypatch.setattr(cwen_b200, "lib", lambda: type("L", (), {"cwen_cuda_shutdown": staticmethod(lambda: None)}))
    assert bench.main_decode(_args(), 1, 0, 0) == 0
    rec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    _check_common(rec)
    assert rec["unit"] == "tok/s" and abs(rec["value"] - 1000.0 / 6.8) < 1e-2
    assert rec["gpu_launches"] == 470 * 8
    assert rec["cpu_baseline"]["kind"] == "reference" and rec["cpu_baseline"]["value"] == 3.0
    assert rec["cpu_baseline"]["same_prompt"] is True
    assert rec["spec_d8"]["tok_s"] == 600.0 and rec["mtp_d8"]["tok_s"] == 130.0
    assert rec["verify_ceiling"]["8"]["pass"] is True
    assert rec["gemv_config0"]["value"] == 1.0
    assert "no engine here" in rec["gdn_config1"]["error"]
    assert rec["mtp_config4"]["tok_s"] == 90.0 and rec["mtp_config4"]["identical_to_serial"] is True
    assert rec["mtp_config4"]["prefill_tok_s"] == 464.2
    assert rec["roofline"]["bound"] == "hbm" and rec["roofline"]["peak"] == 6541.1
    assert abs(rec["roofline"]["achieved"] - 14.4e9 / 3.0e-3 / 1e9) < 0.1  # bytes per token / GEMV time per token


def test_gemv_line(monkeypatch):
    kern = {"ms": 0.030, "bytes": float(bench.GEMV_BYTES), "launches": 32}
    monkeypatch.setattr(bench, "run_gemv_ours", lambda a, ws, r, l: (0.031, kern, 1e-4, CLK, None, None))
    monkeypatch.setattr(bench, "peaks", lambda: (6541.1, 1590.0, "measured"))
    line, _, _ = bench.gemv_ours_line(_args(workload="gemv", steps=32), 1, 0, 0, bench.gemv_config(1))
    _check_common(line)
    assert abs(line["value"] - bench.GEMV_BYTES / 0.031e-3 / 1e9) < 0.1
    # the roofline reads the timed loop (one launch per step), not the serialised event pass
    assert abs(line["roofline"]["achieved"] - bench.GEMV_BYTES / 0.031e-3 / 1e9) < 0.1
    assert line["roofline"]["serialised_kernel_ms"] == 0.030
    assert line["roofline"]["traffic"] == bench.GEMV_NCU_TRAFFIC
    assert line["e2e"]["h2d_bytes_per_step"] == bench.GEMV_B * bench.GEMV_K * 4


def test_gdn_minimum_bytes():
    """Config 1's roofline bytes: inputs, state and conv weights once, outputs
    once, the committed state once when rows are kept."""
    nokeep, keep = bench.gdn_min_bytes(0), bench.gdn_min_bytes(3)
    assert keep - nokeep == (bench.GDN_S + bench.GDN_QKV * 3) * 4
    assert nokeep > bench.GDN_S * 4 and keep == bench.gdn_min_bytes(8)
    ks = bench.gdn_keeps(9000)
    assert ks.min() == 0 and ks.max() == bench.GDN_B and abs(ks.mean() - 4.0) < 0.15


@pytest.mark.parametrize("ws,local_ws,cores", [(1, 1, 16), (8, 8, 16), (2, 2, 3)])
def test_synth_threads_share_the_node(monkeypatch, ws, local_ws, cores):
    monkeypatch.setenv("LOCAL_WORLD_SIZE", str(local_ws))
    monkeypatch.setattr(bench, "host_cores", lambda: cores)
    assert bench.synth_threads(ws) == max(1, cores // local_ws)


def test_reference_arm_loads_no_engine(tmp_path):
    """The reference arm runs the reference build alone: its inputs come from
    the synth code linked into oracle/_ref, and the engine's library is never
    loaded into the process."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(bench.__file__).resolve().parent
    if not bench.ref_lib_path()[0].exists():
        pytest.skip("reference build (oracle/_ref) missing")
    code = ("import sys, argparse, bench\n"
            "a = argparse.Namespace(gpus=1, steps=1, warmup=3, impl='reference', workload='gdn', "
            "no_cpu_baseline=False, no_side_workloads=True)\n"
            "rc = bench.main_gdn(a, 1, 0, 0)\n"
            "maps = open('/proc/self/maps').read()\n"
            "print('ENGINE_LOADED' if 'libcwen_cuda' in maps else 'ENGINE_NOT_LOADED')\n"
            "print('REF_LOADED' if 'libcwref_' in maps else 'REF_NOT_LOADED')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = r.stdout
    assert "ENGINE_NOT_LOADED" in out and "REF_LOADED" in out, out[-2000:]
    rec = json.loads([ln for ln in out.splitlines() if ln.startswith("{")][-1])
    assert rec["impl"] == "reference" and rec["cpu_baseline"]["kind"] == "reference"
