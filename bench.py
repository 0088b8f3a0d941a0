"""Benchmark of the cwen B200 verify-decode engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|gemv|mtp|gdn]

Workload `decode` (default; serial decode and n-gram speculation): the random-init 27B
hybrid (64 layers, Q4_0 weights with scales |N(0,0.01)|, norms 1, seeded),
greedy decode of one sequence after a 512-id random prompt.  A step is one
decoded token: the forward pass of the previous token at the next slot plus
its argmax back on the host (cwen_cuda_forward_serial).  value = tok/s over
K timed steps (CUDA events on the engine stream).  The same run also times
config 3: n-gram speculative decode, draft depth 8, 2048-id motif prompt,
512 new tokens, checked token-for-token against serial decode.

On one GPU the decode line also carries `gemv_config0` and `gdn_config1`:
the config-0 and config-1 measurements below (200 steps each, no CPU leg).

Workload `gemv` (the verify-GEMV microkernel): the B=8 Q4_0 verify GEMV, W 17408x5120,
X fp32 8x5120 ~N(0,1), scales |N(0,0.01)|, nibbles uniform.  A step is one
call over a weight copy from a ring of 8 distinct copies (400 MB > 126 MB L2),
so every step streams W from HBM.  value = algorithmic bytes / device time.

Workload `gdn` (GDN verify step with rollback): one GatedDeltaNet layer's verify block
(B=8 rows) and the rollback to a rejection index uniform in 0..8, through
cwen_cuda_gdn_verify, over a ring of 64 layers' states (253 MB > L2).
value = us per step (CUDA events around the K steps captured in one CUDA
graph; the stream-launched loop is reported beside it).

Workload `mtp` (MTP speculation at 32k context): the hybrid plus the blk.64 MTP block,
a 32767-id prefill, 256 new tokens drafted by the MTP head and verified;
MTP spec tok/s, prefill rate, stream checked against serial decode.

Multi-GPU: one process per GPU (torchrun); the GEMV has no exchange, each
rank runs the same per-GPU work ("scaling": "weak"), the barrier-bracketed
device time is max-reduced over ranks.

The CPU baseline (rank 0, N=1) and `--impl reference` run the reference's own
C code (maci0/cwen run.c compiled into oracle/_ref) on the same bytes.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

DEC_SEED = 1
PROMPT_LEN, N_GEN = 512, 256          # config 2
SPEC_PROMPT, SPEC_GEN = 2048, 512     # config 3
MTP_GEN = 128
DEC_CTX = 4096
GEMV_K, GEMV_M, GEMV_B = 5120, 17408, 8
GEMV_BYTES = (GEMV_K // 32) * 18 * GEMV_M + GEMV_B * GEMV_K * 4 + GEMV_B * GEMV_M * 4  # 50,855,936
RING = 8
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) that ncu measured for
# one config-0 GEMV launch of the current kernel; scaled by algorithmic bytes for
# the decode-step launches (traffic grows in proportion with the weight bytes).
GEMV_NCU_TRAFFIC = 51_597_312
GEMV_NCU_SOURCE = ("constant: dram__bytes_read.sum + dram__bytes_write.sum of one config-0 launch in the ncu "
                   "capture summarised in profiles/qgemv_q4_0_b8_config0.md")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        def run():
            while not self._stop.is_set():
                try:
                    out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                         timeout=5).stdout.strip()
                    if out:
                        self.rows.append([s.strip() for s in out.split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def _backend() -> str:
    # NCCL on the GPU box; gloo lets the multi-rank plumbing run on CPU (tests)
    return os.environ.get("CWEN_DIST_BACKEND", "nccl")


def dist_init(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist
        if _backend() == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(_backend(), timeout=datetime.timedelta(seconds=120))
    return ws, rank, local


def barrier_max(ws, value: float) -> float:
    """Max over ranks (every multi-GPU time is the slowest rank's)."""
    if ws == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda" if _backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------- reference (CPU) ----------------
def ref_lib_path():
    flags = ""
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except Exception:
        pass
    need = ["avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512_vnni"]
    v = "avx512" if all(f in flags for f in need) else "avx2"
    return ROOT / "oracle" / "_ref" / f"libcwref_{v}.so", v


def synth_threads(ws):
    """Host threads for generating the seeded model: the cores shared by the
    ranks of this node, so that N ranks do not each start one per core."""
    per_node = int(os.environ.get("LOCAL_WORLD_SIZE", ws))
    return max(1, host_cores() // max(1, per_node))


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_gemv_baseline(W, X, budget_s: float = 12.0):
    """Reference gemvb (run.c:1577) on the GGUF Q4_0 layout and on its split
    T_Q4_0RS layout (dot_q4_bcol, run.c:1544), best of the two; bounded by
    a time budget.  Returns (GB/s of the config-0 algorithmic bytes, info)."""
    ref, variant = ref_lib()
    if ref is None:
        return None
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    K, M, B = GEMV_K, GEMV_M, GEMV_B
    Y = np.zeros((B, M), np.float32)
    nb = K // 32
    qs = np.zeros(nb * M * 16 + 64, np.uint8)
    off = (-qs.ctypes.data) % 64
    qs = qs[off:off + nb * M * 16]
    sc = np.zeros(nb * M, np.uint16)
    ref.cwref_split_q4_0(vp(W), K, M, vp(qs), vp(sc))
    best = None
    for name, fn in (("gguf_q4_0", lambda: ref.cwref_gemvb(2, vp(W), K, M, vp(X), K, vp(Y), M, B)),
                     ("split_q4_0rs", lambda: ref.cwref_gemvb_split(vp(qs), vp(sc), K, M, vp(X), K, vp(Y), M, B))):
        fn()
        n, t0 = 0, time.perf_counter()
        while True:
            fn()
            n += 1
            el = time.perf_counter() - t0
            if el > budget_s / 2 or n >= 200:
                break
        gbs = GEMV_BYTES * n / el / 1e9
        if best is None or gbs > best[0]:
            best = (gbs, name, n, el)
    gbs, name, n, el = best
    return gbs, {"kind": "reference", "cores": int(ref.cwref_threads()), "variant": f"{variant}/{name}",
                 "sample": f"{n} B=8 gemvb calls on W 17408x5120 Q4_0 ({el:.1f} s)"}


# ---------------- our engine ----------------
def make_gemv_inputs(seed=1, synth=None):
    synth = synth or Synth()
    W = synth.q(seed, "bench.gemv.w", 2, GEMV_K, GEMV_M)
    X = synth.normal(seed + 1, "bench.gemv.x", GEMV_B * GEMV_K).reshape(GEMV_B, GEMV_K)
    return W, X


def run_gemv_ours(args, ws, rank, local):
    import torch

    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(local, 64, 16), "init")
    W, X = make_gemv_inputs()
    wids = []
    for _ in range(RING):
        wid = C.c_int(-1)
        cwen_b200.check(L.cwen_cuda_weight_upload(2, W.ctypes.data_as(C.c_void_p), GEMV_K, GEMV_M, C.byref(wid)))
        wids.append(wid.value)
    dev = torch.device("cuda", local)
    dX = torch.from_numpy(X).to(dev)
    dY = torch.zeros((GEMV_B, GEMV_M), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(stream.cuda_stream)

    def step(i):
        cwen_b200.check(L.cwen_cuda_gemvb(wids[i % RING], C.c_void_p(dX.data_ptr()), GEMV_K,
                                          C.c_void_p(dY.data_ptr()), GEMV_M, GEMV_B, sp))

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("bench_timed")
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    clk = clocks.stop()
    # kernel roofline pass: CUDA events around every GEMV launch (serialises
    # the launches; not in the headline number)
    cwen_b200.check(L.cwen_cuda_profile(1), "profile")
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            step(i)
    torch.cuda.synchronize()
    gm, gb, gc, nl = C.c_double(), C.c_double(), C.c_longlong(), C.c_longlong()
    cwen_b200.check(L.cwen_cuda_profile_read(C.byref(gm), C.byref(gb), C.byref(gc), C.byref(nl)), "profile_read")
    cwen_b200.check(L.cwen_cuda_profile(0), "profile")
    kern = {"ms": gm.value / max(gc.value, 1), "bytes": gb.value / max(gc.value, 1), "launches": nl.value}
    ms = barrier_max(ws, ms)

    # end to end through the host-buffer entry point (copies in the timed
    # region), X in and Y out in pinned host memory
    hX = torch.from_numpy(np.ascontiguousarray(X)).pin_memory()
    hY = torch.zeros((GEMV_B, GEMV_M), dtype=torch.float32).pin_memory()
    hxp, hyp = C.c_void_p(hX.data_ptr()), C.c_void_p(hY.data_ptr())
    for i in range(3):
        cwen_b200.check(L.cwen_cuda_gemvb_host(wids[i % RING], hxp, GEMV_K, hyp, GEMV_M, GEMV_B))
    t0 = time.perf_counter()
    for i in range(args.steps):
        cwen_b200.check(L.cwen_cuda_gemvb_host(wids[i % RING], hxp, GEMV_K, hyp, GEMV_M, GEMV_B))
    e2e_s = (time.perf_counter() - t0) / args.steps
    e2e_s = barrier_max(ws, e2e_s)
    L.cwen_cuda_shutdown()
    return ms, kern, e2e_s, clk, W, X


def gemv_config(ws):
    return {"workload": "config0: Q4_0 verify GEMV W[17408x5120], X fp32[8x5120], Y[8x17408]",
            "B": GEMV_B, "K": GEMV_K, "M": GEMV_M,
            "l2": "weight ring of 8 copies (400 MB > 126 MB L2), new copy every step",
            "parallelism": f"replicas{ws}" if ws > 1 else "single"}


def gemv_ours_line(args, ws, rank, local, config):
    """Config 0 through our engine: the JSON line without the CPU baseline."""
    hbm, _, peak_kind = peaks()
    ms, kern, e2e_s, clk, W, X = run_gemv_ours(args, ws, rank, local)
    gbs = GEMV_BYTES / (ms * 1e-3) / 1e9
    total = gbs * ws
    line = {"metric": "verify-GEMV GB/s (B=8 Q4_0, config 0)", "value": round(total, 2), "unit": "GB/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "numerics": "q4_0 weights x f32 X -> f32 Y (f16 hi+lo tensor-core operands, f32 accumulate)",
            "data": "synthetic (seeded)", "config": config, "gpu_launches": kern["launches"], "clocks": clk}
    # achieved bandwidth from the timed loop (one kernel launch per step,
    # back to back on the launching stream); the per-launch event pass
    # (launches serialised by the events) is reported beside it
    ach = GEMV_BYTES / (ms * 1e-3) / 1e9
    line["roofline"] = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(ach / hbm, 4), "peak_kind": peak_kind, "traffic": GEMV_NCU_TRAFFIC,
                        "traffic_source": GEMV_NCU_SOURCE,
                        "kernel": "qgemv_kernel<Q4_0, two n-tiles of 4 columns (f16 hi | lo), local X>",
                        "kernel_ms": round(ms, 5), "serialised_kernel_ms": round(kern["ms"], 5)}
    e2e_gbs = GEMV_BYTES / e2e_s / 1e9
    line["e2e"] = {"value": round(e2e_gbs * ws, 2), "unit": "GB/s", "h2d_bytes_per_step": GEMV_B * GEMV_K * 4,
                   "d2h_bytes_per_step": GEMV_B * GEMV_M * 4,
                   "note": "cwen_cuda_gemvb_host: pinned host X in, pinned host Y out, synchronous"}
    return line, W, X


# ---------------- decode (configs 2 / 3) ----------------
def synth_ids(n, seed, stream, V, synth=None):
    return (synth or Synth()).ids(seed, stream, V, n)


def motif_prompt(n, V, seed=3):
    """2048 ids: a seed-random 37-token motif repeated, 5% uniform substitutions."""
    rng = np.random.default_rng(seed)
    motif = rng.integers(0, V, size=37)
    p = np.resize(motif, n).astype(np.int32)
    sub = rng.random(n) < 0.05
    p[sub] = rng.integers(0, V, size=int(sub.sum()))
    return p


def verify_ceiling(L, prompt, reps=4):
    """The reference's verify-ceiling gate (bench_spec, run.c:4455-4495): one
    verify block of B rows against B serial steps from the same context, min
    of `reps` alternating repetitions; batching must not lose (block <= 1.05 x
    serial).  Wall clock around calls that end in a host read (accept, the
    serial argmax), as the reference times them."""
    import cwen_b200
    toks = np.ascontiguousarray(prompt[:16], np.int32)
    k, u = C.c_int(), C.c_int()
    nxt = C.c_int()
    res = {}
    for B in (2, 4, 8, 16):
        blk_ms = ser_ms = float("inf")
        for _ in range(reps):
            t0 = time.perf_counter()
            cwen_b200.check(L.cwen_cuda_forward_block(cwen_b200.ptr(toks), B, B), "forward_block")
            cwen_b200.check(L.cwen_cuda_accept(C.byref(k), C.byref(u), None), "accept")
            cwen_b200.check(L.cwen_cuda_commit(B - 1), "commit")
            blk_ms = min(blk_ms, (time.perf_counter() - t0) * 1e3)
            t0 = time.perf_counter()
            for i in range(B):
                cwen_b200.check(L.cwen_cuda_forward_serial(int(toks[i]), 1, C.byref(nxt)), "forward_serial")
            ser_ms = min(ser_ms, (time.perf_counter() - t0) * 1e3)
        res[str(B)] = {"block_ms": round(blk_ms, 3), "serial_ms": round(ser_ms, 3),
                       "x": round(ser_ms / blk_ms, 2), "pass": blk_ms <= 1.05 * ser_ms}
    return res


def run_decode_ours(args, ws, rank, local):
    import torch

    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(local, DEC_CTX, 16), "init")
    d = cwen_b200.dims("reference")
    d.has_mtp = 1  # blk.64 nextn block (Q8_0), used only by the MTP-drafted run below
    t0 = time.perf_counter()
    cwen_b200.check(L.cwen_load_synth(DEC_SEED, C.byref(d), synth_threads(ws)), "load_synth")
    load_s = time.perf_counter() - t0
    V = d.n_vocab
    prompt = synth_ids(PROMPT_LEN, DEC_SEED, "bench.prompt", V)
    serial = cwen_b200.spec_cfg(spec=0)
    first, _ = cwen_b200.generate(prompt, 1, serial)
    tok = int(first[0])
    nxt = C.c_int(0)
    stream = torch.cuda.ExternalStream(L.cwen_cuda_stream(), device=torch.device("cuda", local))

    def steps(n, tok):
        for _ in range(n):
            cwen_b200.check(L.cwen_cuda_forward_serial(tok, 1, C.byref(nxt)), "forward_serial")
            tok = nxt.value
        return tok

    tok = steps(args.warmup, tok)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("bench_timed")  # ncu --nvtx-include bench_timed/ selects the timed steps
    ev0.record(stream)
    tok = steps(args.steps, tok)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = barrier_max(ws, ms)
    # GEMV roofline pass: per-launch CUDA events around every GEMV (not in the headline number)
    kp = max(4, min(args.steps, 16))
    cwen_b200.check(L.cwen_cuda_profile(1), "profile")
    tok = steps(kp, tok)
    gm, gb, gc, nl = C.c_double(), C.c_double(), C.c_longlong(), C.c_longlong()
    cwen_b200.check(L.cwen_cuda_profile_read(C.byref(gm), C.byref(gb), C.byref(gc), C.byref(nl)), "profile_read")
    cwen_b200.check(L.cwen_cuda_profile(0), "profile")
    kern = {"gemv_ms_per_token": gm.value / kp, "gemv_bytes_per_token": gb.value / kp,
            "gemv_calls_per_token": gc.value / kp, "launches_per_token": nl.value / kp}
    try:
        kern["verify_ceiling"] = verify_ceiling(L, prompt)
    except Exception as e:  # noqa: BLE001 -- reported beside the headline, never in place of it
        kern["verify_ceiling"] = {"error": f"{type(e).__name__}: {e}"}
    # end to end through the public host API (bench_toks method): (t(n) - t(1)) / (n - 1)
    t0 = time.perf_counter()
    cwen_b200.generate(prompt, 1, serial)
    t1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    out_ser, _ = cwen_b200.generate(prompt, N_GEN, serial)
    tn = time.perf_counter() - t0
    e2e_tps = (N_GEN - 1) / (tn - t1)
    # config 3: n-gram speculation, depth 8, motif prompt; stream must equal serial
    mp = motif_prompt(SPEC_PROMPT, V)
    t0 = time.perf_counter()
    cwen_b200.generate(mp, 1, serial)
    s1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    ref_stream, _ = cwen_b200.generate(mp, SPEC_GEN, serial)
    sn = time.perf_counter() - t0
    spec_cfg = cwen_b200.spec_cfg(spec=1, use_mtp=0, max_draft=8)
    t0 = time.perf_counter()
    spec_stream, st = cwen_b200.generate(mp, SPEC_GEN, spec_cfg)
    pn = time.perf_counter() - t0
    spec = {"workload": "config3: n-gram spec d=8, 2048-id motif prompt, 512 new",
            "tok_s": round((SPEC_GEN - 1) / (pn - s1), 2), "serial_tok_s": round((SPEC_GEN - 1) / (sn - s1), 2),
            "identical_to_serial": bool(np.array_equal(ref_stream, spec_stream)),
            "cycles": st.cycles, "drafted": st.drafted, "full_accept": st.full, "short": st.shortw,
            "avg_kept": round(st.kept / st.drafted, 3) if st.drafted else 0.0}
    # MTP-drafted speculation, depth 8, on the config-2 prompt (a 512-slot
    # context, not config 4's 32k prefill); stream checked against serial
    mtp_cfg = cwen_b200.spec_cfg(spec=1, use_mtp=1, max_draft=8)
    t0 = time.perf_counter()
    cwen_b200.generate(prompt, 1, mtp_cfg)
    m1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    mtp_stream, mst = cwen_b200.generate(prompt, MTP_GEN, mtp_cfg)
    mn = time.perf_counter() - t0
    mtp = {"workload": f"MTP (blk.64 nextn, Q8_0) drafter, depth 8, config-2 prompt, {MTP_GEN} new",
           "tok_s": round((MTP_GEN - 1) / (mn - m1), 2),
           "identical_to_serial": bool(np.array_equal(out_ser[:MTP_GEN], mtp_stream)),
           "cycles": mst.cycles, "drafted": mst.drafted, "full_accept": mst.full, "short": mst.shortw,
           "avg_kept": round(mst.kept / mst.drafted, 3) if mst.drafted else 0.0,
           "note": "random-init weights: the nextn head is not trained on the target, so few drafts are kept"}
    spec["mtp_d8"] = mtp
    L.cwen_cuda_shutdown()
    return ms, kern, e2e_tps, clk, spec, load_s, prompt


def ref_lib():
    """The reference build (oracle/_ref, run.c compiled unmodified) with all
    host cores; None when it is missing.  Nothing of the engine is loaded."""
    path, variant = ref_lib_path()
    if not path.exists():
        return None, variant
    os.environ.setdefault("OMP_NUM_THREADS", str(host_cores()))
    os.environ.setdefault("OMP_PROC_BIND", "close")
    os.environ.setdefault("OMP_PLACES", "cores")
    ref = C.CDLL(str(path))
    ref.cwref_threads.restype = C.c_int
    ref.cwref_decode_step.restype = C.c_int
    return ref, variant


class Synth:
    """Seeded synthetic inputs (cwen_b200/host/synth.c) through whichever
    library is loaded: the engine's, or the reference build, which links the
    same synth.c -- so the reference arm makes the same bytes without loading
    the engine."""

    def __init__(self, lib=None):
        if lib is None:
            import cwen_b200
            lib = cwen_b200.lib()
        self.L = lib
        u64, vp, cp = C.c_uint64, C.c_void_p, C.c_char_p
        lib.cw_synth_q4_0.argtypes = [u64, cp, C.c_int, C.c_int, vp, C.c_int]
        lib.cw_synth_q8_0.argtypes = [u64, cp, C.c_int, C.c_int, vp, C.c_int]
        lib.cw_synth_normal.argtypes = [u64, cp, C.c_float, C.c_float, vp, C.c_size_t]
        lib.cw_synth_ids.argtypes = [u64, cp, C.c_int, vp, C.c_size_t]
        for f in ("cw_synth_q4_0", "cw_synth_q8_0", "cw_synth_normal", "cw_synth_ids"):
            getattr(lib, f).restype = None

    def q(self, seed, stream, typ, K, M):
        W = np.zeros((K // 32) * (18 if typ == 2 else 34) * M, np.uint8)
        (self.L.cw_synth_q4_0 if typ == 2 else self.L.cw_synth_q8_0)(seed, stream.encode(), K, M,
                                                                     W.ctypes.data_as(C.c_void_p), 0)
        return W

    def normal(self, seed, stream, n, mean=0.0, std=1.0):
        v = np.zeros(n, np.float32)
        self.L.cw_synth_normal(seed, stream.encode(), mean, std, v.ctypes.data_as(C.c_void_p), n)
        return v

    def ids(self, seed, stream, V, n):
        v = np.zeros(n, np.int32)
        self.L.cw_synth_ids(seed, stream.encode(), V, v.ctypes.data_as(C.c_void_p), n)
        return v


SHARD_HANDLE = 256  # CWEN_SHARD_HANDLE_BYTES


def shard_exchange(blob: bytes, ws: int) -> bytes:
    """Every rank's exchange-buffer handles, in rank order (one all-gather of
    small host objects over the process group: plumbing, not the data path)."""
    import torch.distributed as dist
    out = [None] * ws
    dist.all_gather_object(out, blob)
    assert all(isinstance(b, bytes) and len(b) == len(blob) for b in out)
    return b"".join(out)


def run_decode_sharded(args, ws, rank, local):
    """The same serial greedy decode with the FFN and lm_head row-sharded
    over the ws GPUs (cwen_cuda_shard_*): one sequence, every GPU works on
    every token.  Returns the per-token device time (max over ranks), the
    end-to-end rate through cwen_generate, and an n-gram speculative run
    checked token for token against the group's own serial stream."""
    import torch

    import cwen_b200
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(local, DEC_CTX, 16), "init")
    try:
        cwen_b200.check(L.cwen_cuda_shard_config(rank, ws), "shard_config")
        d = cwen_b200.dims("reference")
        t0 = time.perf_counter()
        cwen_b200.check(L.cwen_load_synth(DEC_SEED, C.byref(d), synth_threads(ws)), "load_synth")
        load_s = time.perf_counter() - t0
        blob = (C.c_uint8 * SHARD_HANDLE)()
        cwen_b200.check(L.cwen_cuda_shard_handle(blob, SHARD_HANDLE), "shard_handle")
        allb = shard_exchange(bytes(blob), ws)
        cwen_b200.check(L.cwen_cuda_shard_open(allb, ws), "shard_open")
        V = d.n_vocab
        prompt = synth_ids(PROMPT_LEN, DEC_SEED, "bench.prompt", V)
        serial = cwen_b200.spec_cfg(spec=0)
        first, _ = cwen_b200.generate(prompt, 1, serial)
        nxt = C.c_int(0)
        stream = torch.cuda.ExternalStream(L.cwen_cuda_stream(), device=torch.device("cuda", local))

        def steps(n, tok):
            for _ in range(n):
                cwen_b200.check(L.cwen_cuda_forward_serial(tok, 1, C.byref(nxt)), "forward_serial")
                tok = nxt.value
            return tok

        tok = steps(args.warmup, int(first[0]))
        torch.cuda.synchronize()
        barrier(ws)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        tok = steps(args.steps, tok)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = barrier_max(ws, ev0.elapsed_time(ev1) / args.steps)
        n_e2e = 64
        t0 = time.perf_counter()
        cwen_b200.generate(prompt, 1, serial)
        t1 = time.perf_counter() - t0
        t0 = time.perf_counter()
        cwen_b200.generate(prompt, n_e2e, serial)
        tn = time.perf_counter() - t0
        e2e = 1.0 / barrier_max(ws, (tn - t1) / (n_e2e - 1))
        mp = motif_prompt(SPEC_PROMPT, V)
        n_spec = 128
        ser_stream, _ = cwen_b200.generate(mp, n_spec, serial)
        t0 = time.perf_counter()
        cwen_b200.generate(mp, 1, serial)
        s1 = time.perf_counter() - t0
        t0 = time.perf_counter()
        spec_stream, st = cwen_b200.generate(mp, n_spec, cwen_b200.spec_cfg(spec=1, use_mtp=0, max_draft=8))
        sn = time.perf_counter() - t0
        spec_tps = 1.0 / barrier_max(ws, (sn - s1) / (n_spec - 1))
        return {"workload": f"serial greedy decode of one sequence, FFN + lm_head row-sharded over {ws} GPUs "
                            f"(NVLink stores + cross-GPU barrier, replicated GDN/attention)",
                "tok_s": round(1000.0 / ms, 3), "ms_per_token": round(ms, 4),
                "e2e_tok_s": round(e2e, 3), "model_load_s": round(load_s, 1),
                "spec_d8_tok_s": round(spec_tps, 2),
                "spec_identical_to_serial": bool(np.array_equal(ser_stream, spec_stream)),
                "spec_avg_kept": round(st.kept / st.drafted, 3) if st.drafted else 0.0}
    finally:
        L.cwen_cuda_shutdown()


def cpu_decode_baseline(steps: int = 24, warmup: int = 2):
    """The reference's own greedy decode on the seeded model in host memory,
    all host cores, on the same workload as the engine: generate_tokens
    (run.c:5027) prefills the same 512-id prompt and emits the first token,
    then `warmup` untimed and `steps` timed iterations of its decode loop
    (run.c:5033-5041: next slot, forward_ex, argmax of the logits).
    Returns (tok/s, info, prompt)."""
    ref, variant = ref_lib()
    if ref is None:
        return None
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    t0 = time.perf_counter()
    if ref.cwref_load_synth(C.c_uint64(DEC_SEED), 0, 0):
        return None
    load_s = time.perf_counter() - t0
    ref.cwref_alloc_state(DEC_CTX, 0, 0)
    prompt = Synth(ref).ids(DEC_SEED, "bench.prompt", 248320, PROMPT_LEN)
    out = np.zeros(4, np.int32)
    t0 = time.perf_counter()
    ref.cwref_generate(vp(prompt), PROMPT_LEN, 1, vp(out))
    pf_s = time.perf_counter() - t0
    tok = int(out[0])
    for _ in range(warmup):
        tok = ref.cwref_decode_step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = ref.cwref_decode_step(tok)
    el = time.perf_counter() - t0
    tps = steps / max(el, 1e-9)
    return tps, {"kind": "reference", "cores": int(ref.cwref_threads()), "variant": variant,
                 "sample": f"reference generate_tokens on the same seeded 27B model and 512-id prompt "
                           f"(prefill {pf_s:.1f} s), then {steps} timed decode steps at slots "
                           f"{PROMPT_LEN + warmup}..{PROMPT_LEN + warmup + steps - 1} ({el:.1f} s; "
                           f"model synth {load_s:.0f} s)"}, prompt


def main_decode(args, ws, rank, local):
    hbm, bf16, peak_kind = peaks()
    config = {"workload": "config2: serial greedy decode, random-init 27B hybrid (64 layers, GDN:attention 3:1, "
                          "Q4_0, scales |N(0,0.01)|, seeded synthetic weights), prompt 512 random ids",
              "prompt": PROMPT_LEN, "ctx": DEC_CTX, "batch": 1,
              "l2": "every step streams 14.4 GB of weights (>> 126 MB L2)",
              "parallelism": f"replicas{ws} (independent sequence per GPU)" if ws > 1 else "single"}
    metric = "decode tok/s (serial greedy, config 2)"
    if args.impl == "reference":
        if rank != 0:
            return 0
        res = cpu_decode_baseline(steps=max(4, min(64, args.steps)), warmup=min(args.warmup, 8))
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref reference build missing"}))
            return 0
        tps, info, _ = res
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(tps, 4), "unit": "tok/s",
                          "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": round(1000.0 / tps, 3), "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "numerics": "q4_0 weights, f32 activations", "data": "synthetic (seeded)",
                          "config": config, "cpu_baseline": {**info, "value": round(tps, 4), "unit": "tok/s"},
                          "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0
    ms, kern, e2e_tps, clk, spec, load_s, prompt = run_decode_ours(args, ws, rank, local)
    tps = 1000.0 / ms
    gemv_ms = kern["gemv_ms_per_token"] / max(kern["gemv_calls_per_token"], 1)
    gemv_bytes = kern["gemv_bytes_per_token"] / max(kern["gemv_calls_per_token"], 1)
    ach = kern["gemv_bytes_per_token"] / (kern["gemv_ms_per_token"] * 1e-3) / 1e9
    line = {"metric": metric, "value": round(tps * ws, 3), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "numerics": "q4_0 weights, f32 activations (f16 hi+lo tensor-core operands, f32 accumulate)",
            "data": "synthetic (seeded random-init weights, random prompt ids)", "config": config,
            "gpu_launches": int(round(kern["launches_per_token"] * args.steps)), "clocks": clk,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4), "peak_kind": peak_kind,
                         "traffic": round(GEMV_NCU_TRAFFIC / GEMV_BYTES * gemv_bytes),
                         "traffic_note": "ncu DRAM bytes of a config-0 launch, scaled to the average decode launch",
                         "traffic_source": GEMV_NCU_SOURCE,
                         "kernel": "qgemv_kernel (all verify-GEMV launches of a decode step)",
                         "launches_per_token": round(kern["gemv_calls_per_token"], 1),
                         "avg_launch_ms": round(gemv_ms, 5), "avg_launch_bytes": round(gemv_bytes),
                         "gemv_share_of_step": round(kern["gemv_ms_per_token"] / ms, 3)},
            "e2e": {"value": round(e2e_tps * ws, 3), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 12, "method": "cwen_generate (C host driver): (t(256)-t(1))/255"},
            "spec_d8": spec, "mtp_d8": spec.pop("mtp_d8", None), "model_load_s": round(load_s, 1),
            "verify_ceiling": kern.get("verify_ceiling")}
    if ws > 1:
        # the latency-oriented alternative to the replicas: one sequence over
        # all ws GPUs; a failure is reported in the line, never in place of it
        try:
            line["sharded"] = run_decode_sharded(args, ws, rank, local)
        except Exception as e:  # noqa: BLE001 -- recorded, not raised
            line["sharded"] = {"error": f"{type(e).__name__}: {e}"}
    if ws == 1 and not args.no_side_workloads:
        # configs 0 and 1 beside the headline (their own workloads give the
        # full lines, CPU baselines included); a failure here is reported in
        # the line and never costs the headline
        sub = argparse.Namespace(**{**vars(args), "steps": 200, "warmup": 5})
        for key, fn in (("gemv_config0", lambda: gemv_ours_line(sub, ws, rank, local, gemv_config(ws))[0]),
                        ("gdn_config1", lambda: gdn_ours_line(sub, ws, rank, local, gdn_config(ws), GDN_METRIC))):
            try:
                r = fn()
                line[key] = {k: r[k] for k in ("metric", "value", "unit", "steps", "ms_per_step", "gpu_launches",
                                               "clocks", "roofline", "e2e", "timing", "stream_launched_us")
                             if k in r}
            except Exception as e:  # noqa: BLE001 -- recorded, not raised
                line[key] = {"error": f"{type(e).__name__}: {e}"}
                import cwen_b200
                cwen_b200.lib().cwen_cuda_shutdown()  # no-op when the engine is not live
        # config 4 (32k prefill, MTP spec d=8, 256 new) in compact form
        try:
            r = run_mtp_ours(ws, local)
            line["mtp_config4"] = {"workload": f"config4: {MTP_PROMPT}-id prefill in a {MTP_CTX} context, MTP spec "
                                               f"d=8, {MTP_NEW} new through cwen_generate",
                                   "tok_s": round(r["tps"], 2), "identical_to_serial": r["identical_to_serial"],
                                   "prefill_s": r["prefill"]["seconds"], "prefill_tok_s": r["prefill"]["tok_s"],
                                   "clocks": r["clocks"], "mtp": r["mtp"]}
        except Exception as e:  # noqa: BLE001 -- recorded, not raised
            line["mtp_config4"] = {"error": f"{type(e).__name__}: {e}"}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        res = cpu_decode_baseline()
        if res:
            line["cpu_baseline"] = {**res[1], "value": round(res[0], 4), "unit": "tok/s",
                                    "same_prompt": bool(np.array_equal(res[2], prompt))}
    if rank == 0:
        print(json.dumps(line))
    return 0


# ---------------- config 4: MTP speculation after a 32k prefill ----------------
# The context window is the reference's maximum (CWEN_CTX <= 32768); the prompt
# leaves room for the 256 new tokens and a full verify block after them.
MTP_CTX, MTP_NEW = 32768, 256
MTP_PROMPT = MTP_CTX - MTP_NEW - 17


def cpu_mtp_baseline(n_gen=16, prompt_len=64):
    """The reference's MTP-drafted speculation (generate_tokens_spec with the
    nextn drafter, depth 8) on the same seeded model with blk.64, all host
    cores, on a bounded sample: a 64-id prompt instead of the 32k prefill
    (which takes the reference about an hour), (t(1 + n) - t(1)) / n."""
    ref, variant = ref_lib()
    if ref is None:
        return None
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    t0 = time.perf_counter()
    if ref.cwref_load_synth(C.c_uint64(DEC_SEED), 1, 0):
        return None
    load_s = time.perf_counter() - t0
    ref.cwref_alloc_state(4096, 1, 1)
    ref.cwref_spec_config(8, 2, 16, 8)
    prompt = np.ascontiguousarray(Synth(ref).ids(DEC_SEED, "bench.mtp.prompt", 248320, prompt_len), np.int32)
    out = np.zeros(n_gen + 32, np.int32)
    t0 = time.perf_counter()
    ref.cwref_generate(vp(prompt), prompt_len, 1, vp(out))
    t1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    n = ref.cwref_generate(vp(prompt), prompt_len, 1 + n_gen, vp(out))
    tn = time.perf_counter() - t0
    return n_gen / max(tn - t1, 1e-9), {
        "kind": "reference", "cores": int(ref.cwref_threads()), "variant": variant, "n_gen": n_gen,
        "sample": f"reference MTP spec d=8 (generate_tokens_spec, nextn drafter) on the seeded model with blk.64: "
                  f"{prompt_len}-id prompt instead of the 32k prefill, (t({1 + n_gen}) - t(1))/{n_gen} "
                  f"({tn:.1f} s; {n} ids; model synth {load_s:.0f} s)"}


def run_mtp_ours(ws, local):
    """Config 4 on this GPU through cwen_generate: engine at a 32k context,
    the hybrid plus blk.64 (MTP, Q8_0), the 32k prompt pre-filled, 256 new
    tokens drafted by the MTP head at depth 8 and verified, then the same 256
    by serial decode for the identical-stream check.  tok/s = 255 / (t(256) -
    t(1)).  The engine is shut down on return."""
    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(local, MTP_CTX, 16), "init")
    try:
        d = cwen_b200.dims("reference")
        d.has_mtp = 1
        cwen_b200.check(L.cwen_load_synth(DEC_SEED, C.byref(d), synth_threads(ws)), "load_synth")
        prompt = synth_ids(MTP_PROMPT, DEC_SEED, "bench.mtp.prompt", d.n_vocab)
        mtp_cfg = cwen_b200.spec_cfg(spec=1, use_mtp=1, max_draft=8)
        barrier(ws)
        clocks = ClockSampler(local)
        clocks.start()
        t0 = time.perf_counter()
        cwen_b200.generate(prompt, 1, mtp_cfg)
        t1 = time.perf_counter() - t0
        t0 = time.perf_counter()
        spec_stream, st = cwen_b200.generate(prompt, MTP_NEW, mtp_cfg)
        tn = time.perf_counter() - t0
        clk = clocks.stop()
        serial, _ = cwen_b200.generate(prompt, MTP_NEW, cwen_b200.spec_cfg(spec=0))
    finally:
        L.cwen_cuda_shutdown()
    return {"tps": (MTP_NEW - 1) / max(tn - t1, 1e-9), "clocks": clk,
            "prefill": {"tokens": MTP_PROMPT, "seconds": round(t1, 2), "tok_s": round(MTP_PROMPT / t1, 1),
                        "note": "blocks of 16 verify rows, each folded into the nextn stream in one 16-row MTP pass; "
                                "includes the first token"},
            "identical_to_serial": bool(np.array_equal(serial, spec_stream)),
            "mtp": {"cycles": st.cycles, "drafted": st.drafted, "full_accept": st.full, "short": st.shortw,
                    "avg_kept": round(st.kept / st.drafted, 3) if st.drafted else 0.0,
                    "note": "random-init weights: the nextn head is not trained on the target"}}


def main_mtp(args, ws, rank, local):
    """MTP speculation at 32k context: the hybrid plus the blk.64 MTP block (Q8_0), a 32k
    context pre-filled with random ids, 256 new tokens drafted by the MTP head
    (depth 8) and verified; the stream must equal serial decode.  value =
    (t(256) - t(1)) / 255 through cwen_generate; the prefill rate (blocks of
    16 verify rows plus the nextn fold of every slot) is reported beside it."""
    metric = "MTP spec decode tok/s (config 4: 32k prefill, depth 8)"
    config = {"workload": f"config4: random-init 27B hybrid + blk.64 MTP (Q8_0), {MTP_PROMPT}-id random prompt "
                          f"in a {MTP_CTX} context, {MTP_NEW} new",
              "ctx": MTP_CTX, "parallelism": f"replicas{ws}" if ws > 1 else "single"}
    if args.impl == "reference":
        if rank != 0:
            return 0
        res = cpu_mtp_baseline(n_gen=max(4, min(32, args.steps)))
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref reference build missing"}))
            return 0
        tps, info = res
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(tps, 4), "unit": "tok/s",
                          "n_gpus": 0, "steps": info["n_gen"], "warmup": 1, "ms_per_step": round(1000.0 / tps, 3),
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "f32", "numerics": "q4_0 / q8_0 weights, f32 activations", "data": "synthetic (seeded)",
                          "config": config, "cpu_baseline": {**info, "value": round(tps, 4), "unit": "tok/s"},
                          "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0
    r = run_mtp_ours(ws, local)
    tps = 1.0 / barrier_max(ws, 1.0 / r["tps"])
    if rank == 0:
        line = {
            "metric": metric, "value": round(tps * ws, 3), "unit": "tok/s", "n_gpus": ws, "steps": MTP_NEW,
            "warmup": 1, "ms_per_step": round(1000.0 / tps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "numerics": "q4_0 / q8_0 weights, f32 activations", "data": "synthetic (seeded)",
            "config": config, "clocks": r["clocks"], "prefill": r["prefill"],
            "identical_to_serial": r["identical_to_serial"], "mtp": r["mtp"],
            "e2e": {"value": round(tps * ws, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 12,
                    "method": "cwen_generate (C host driver): (t(256)-t(1))/255"}}
        if ws == 1 and not args.no_cpu_baseline:
            res = cpu_mtp_baseline(n_gen=8)
            if res:
                line["cpu_baseline"] = {**res[1], "value": round(res[0], 4), "unit": "tok/s"}
        print(json.dumps(line))
    return 0



# ---------------- config 1: GatedDeltaNet verify step with rollback ----------------
GDN_NKH, GDN_NVH, GDN_D, GDN_B = 16, 48, 128, 8
GDN_QKV = (2 * GDN_NKH + GDN_NVH) * GDN_D        # 10240 conv channels
GDN_Z = GDN_NVH * GDN_D                          # 6144
GDN_PS = GDN_QKV + GDN_Z + 2 * GDN_NVH           # proj row: q|k|v|z|alpha|beta
GDN_S = GDN_NVH * GDN_D * GDN_D                  # 786,432 floats = 3,145,728 B
GDN_RING = 64                                    # distinct layers: 64 x 3.96 MB = 253 MB > 126 MB L2
GDN_SEED = 11
# dram__bytes_read.sum + dram__bytes_write.sum of one gdn_fused_kernel launch
GDN_NCU_TRAFFIC = 4_031_488
GDN_NCU_SOURCE = ("constant: DRAM bytes of one launch in the ncu capture summarised in "
                  "profiles/gdn_fused_config1.md (the state written back stays in L2 past the launch)")


def gdn_min_bytes(keep: int) -> int:
    """Bytes a verify step must move at least: the block's input rows, the
    committed state and the conv weights read once, the head outputs written
    once, and the committed state written once when rows are kept."""
    rd = GDN_B * GDN_PS * 4 + GDN_S * 4 + GDN_QKV * 3 * 4 + GDN_QKV * 4 * 4 + (2 * GDN_NVH + GDN_D) * 4
    wr = GDN_B * GDN_Z * 4 + ((GDN_S + GDN_QKV * 3) * 4 if keep > 0 else 0)
    return rd + wr


def gdn_keeps(n: int) -> np.ndarray:
    """Rejection indices uniform in 0..8 (rows kept of the 8-row block)."""
    return np.random.default_rng(GDN_SEED).integers(0, GDN_B + 1, size=n)


def make_gdn_layer(i: int, synth=None):
    """One layer's seeded inputs (config 1): state ~N(0, 0.1), conv state and
    block rows ~N(0, 1) (q, k, v, z, alpha, beta; the kernel L2-normalises q
    and k after the conv and applies decay = exp(-softplus(alpha)), beta =
    sigmoid(beta): A = -1, dt = 0), conv weights ~N(0, 0.1), norm 1."""
    synth = synth or Synth()
    sd = GDN_SEED * 1000 + i
    return {"proj": synth.normal(sd, "bench.gdn.proj", GDN_B * GDN_PS).reshape(GDN_B, GDN_PS),
            "convw": synth.normal(sd, "bench.gdn.convw", GDN_QKV * 4, 0.0, 0.1),
            "S": synth.normal(sd, "bench.gdn.S", GDN_S, 0.0, 0.1),
            "conv": synth.normal(sd, "bench.gdn.conv", GDN_QKV * 3)}


def cpu_gdn_baseline(budget_s: float = 12.0):
    """The reference's own kernels on the same step: for each of the 8 rows
    decay/beta (run.c:2339-2344), conv1d_update + gdn_step (run.c:2183-2200,
    2014-2180) and a snapshot of the state (the snap_save copy, run.c:2787),
    then the state restored from the snapshot at the rejection index
    (snap_load, run.c:2802).  Bounded by a time budget; all host cores."""
    ref, variant = ref_lib()
    if ref is None:
        return None
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    lay = make_gdn_layer(0, Synth(ref))
    S, cs = lay["S"].copy(), lay["conv"].copy()
    cw, nw = lay["convw"], np.ones(GDN_D, np.float32)
    A, dt = -np.ones(GDN_NVH, np.float32), np.zeros(GDN_NVH, np.float32)
    snapS = np.zeros((GDN_B + 1, GDN_S), np.float32)
    snapC = np.zeros((GDN_B + 1, GDN_QKV * 3), np.float32)
    out = np.zeros((GDN_B, GDN_Z), np.float32)
    keeps = gdn_keeps(100000)

    def step(keep):
        snapS[0] = S
        snapC[0] = cs
        for b in range(GDN_B):
            row = lay["proj"][b]
            qkv = row[:GDN_QKV].copy()
            z = row[GDN_QKV:GDN_QKV + GDN_Z].copy()
            a = row[GDN_QKV + GDN_Z:GDN_QKV + GDN_Z + GDN_NVH].copy()
            bt = row[GDN_QKV + GDN_Z + GDN_NVH:].copy()
            ref.cwref_decay_beta(vp(A), vp(dt), vp(a), vp(bt), GDN_NVH)
            ref.cwref_gdn_step(vp(S), vp(cs), vp(cw), vp(nw), vp(qkv), vp(z), vp(a), vp(bt), vp(out[b]))
            snapS[b + 1] = S
            snapC[b + 1] = cs
        S[:] = snapS[keep]
        cs[:] = snapC[keep]

    step(int(keeps[0]))
    n, t0 = 0, time.perf_counter()
    while True:
        step(int(keeps[n % len(keeps)]))
        n += 1
        el = time.perf_counter() - t0
        if el > budget_s or n >= 20000:
            break
    us = el / n * 1e6
    return us, {"kind": "reference", "cores": int(ref.cwref_threads()), "variant": variant,
                "sample": f"{n} config-1 verify steps (8 rows of conv1d_update + gdn_step, 9 state snapshots, "
                          f"restore at the rejection index) in {el:.1f} s"}


def main_gdn(args, ws, rank, local):
    """The GDN verify step with rollback.  A step is one layer's verify block (B = 8 rows:
    conv + decay/beta + recurrence with the gated norm) followed by the
    rollback to a rejection index uniform in 0..8, through
    cwen_cuda_gdn_verify on device buffers, over a ring of 64 layers' states
    (253 MB > 126 MB L2) so every step reads its state from HBM."""
    metric = GDN_METRIC
    config = gdn_config(ws)
    if args.impl == "reference":
        if rank != 0:
            return 0
        res = cpu_gdn_baseline(budget_s=max(4.0, min(60.0, 1.0 * args.steps)))
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref reference build missing"}))
            return 0
        us, info = res
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(us, 3), "unit": "us",
                          "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": round(us / 1000.0, 5), "higher_is_better": False, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "config": config,
                          "cpu_baseline": {**info, "value": round(us, 3), "unit": "us"},
                          "e2e": {"value": round(us, 3), "unit": "us", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0
    line = gdn_ours_line(args, ws, rank, local, config, metric)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        res = cpu_gdn_baseline()
        if res:
            line["cpu_baseline"] = {**res[1], "value": round(res[0], 3), "unit": "us"}
    if rank == 0:
        print(json.dumps(line))
    return 0


def gdn_config(ws):
    return {"workload": "config1: GatedDeltaNet verify step, 48 value / 16 key heads x 128, B=8, "
                        "state ~N(0,0.1), rejection index uniform 0..8",
            "B": GDN_B, "heads": [GDN_NVH, GDN_NKH], "head_dim": GDN_D, "conv_channels": GDN_QKV,
            "l2": "ring of 64 layers' states and inputs (253 MB > 126 MB L2), next layer every step",
            "parallelism": f"replicas{ws}" if ws > 1 else "single"}


GDN_METRIC = "GDN verify step with rollback, us per step (config 1)"


def gdn_ours_line(args, ws, rank, local, config, metric):
    """Config 1 through our engine: the JSON line without the CPU baseline."""
    import torch

    import cwen_b200
    from cwen_b200 import build
    build.build()
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(local, 64, 16), "init")
    hbm, _, peak_kind = peaks()
    dev = torch.device("cuda", local)
    layers = []
    for i in range(GDN_RING):
        lay = make_gdn_layer(i)
        layers.append({k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in lay.items()})
    A = torch.full((GDN_NVH,), -1.0, dtype=torch.float32, device=dev)
    dt = torch.zeros(GDN_NVH, dtype=torch.float32, device=dev)
    wn = torch.ones(GDN_D, dtype=torch.float32, device=dev)
    out = torch.zeros((GDN_B, GDN_Z), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(stream.cuda_stream)
    P = lambda x: C.c_void_p(x.data_ptr())
    n_all = args.warmup + 2 * args.steps
    keeps = gdn_keeps(n_all)

    def step(i, proj=None):
        lay = layers[i % GDN_RING]
        cwen_b200.check(L.cwen_cuda_gdn_verify(GDN_NKH, GDN_NVH, GDN_B, P(lay["proj"] if proj is None else proj),
                                               GDN_PS, P(lay["convw"]), P(A), P(dt), P(wn), P(lay["S"]),
                                               P(lay["conv"]), int(keeps[i]), P(out), sp), "gdn_verify")

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    idx = range(args.warmup, args.warmup + args.steps)
    torch.cuda.nvtx.range_push("bench_timed")
    ev0.record(stream)
    for i in idx:
        step(i)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk = clocks.stop()
    stream_ms = ev0.elapsed_time(ev1) / args.steps
    # the same K steps captured once into a CUDA graph and replayed: the
    # device time of a step without the host's per-launch cost, which bounds
    # the stream-launched loop above at this step size
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in idx:
            step(i)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(local)
    clocks.start()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    del graph
    ms = barrier_max(ws, ms)
    stream_ms = barrier_max(ws, stream_ms)
    kk = [int(keeps[i]) for i in idx]
    launches = len(kk)  # one fused launch per step (conv, recurrence, gated norm, rollback)
    min_bytes = sum(gdn_min_bytes(k) for k in kk) / args.steps
    ach = min_bytes / (ms * 1e-3) / 1e9

    # end to end: the block's rows from pinned host memory in, the head
    # outputs back to host memory, every step (the state stays resident)
    hproj = [torch.from_numpy(make_gdn_layer(i)["proj"]).pin_memory() for i in range(4)]
    hout = torch.zeros((GDN_B, GDN_Z), dtype=torch.float32).pin_memory()
    dproj = torch.empty((GDN_B, GDN_PS), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    e0 = args.warmup + args.steps
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for j, i in enumerate(range(e0, e0 + args.steps)):
            dproj.copy_(hproj[j % 4], non_blocking=True)
            step(i, dproj)
            hout.copy_(out, non_blocking=True)
            stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / args.steps
    e2e_s = barrier_max(ws, e2e_s)
    L.cwen_cuda_shutdown()
    line = {"metric": metric, "value": round(ms * 1000.0, 3), "unit": "us", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "config": config,
            "gpu_launches": launches, "clocks": clk,
            "timing": "K steps captured in one CUDA graph, replayed between CUDA events",
            "stream_launched_us": round(stream_ms * 1000.0, 3),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4), "peak_kind": peak_kind, "traffic": GDN_NCU_TRAFFIC,
                         "traffic_source": GDN_NCU_SOURCE,
                         "kernel": "gdn_fused_kernel (conv, SiLU, l2norm, decay/beta, recurrence, gated norm and "
                                   "rollback in one launch per step)",
                         "bytes_per_step": round(min_bytes),
                         "bytes_note": "minimum bytes of the step (inputs, state and conv weights read once, "
                                       "outputs written once, committed state written once when rows are kept); "
                                       "the reference's per-position snapshots would add 8 state copies"},
            "e2e": {"value": round(e2e_s * 1e6, 3), "unit": "us", "h2d_bytes_per_step": GDN_B * GDN_PS * 4,
                    "d2h_bytes_per_step": GDN_B * GDN_Z * 4,
                    "note": "pinned host rows in, head outputs out, stream synchronized every step"}}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "gemv", "mtp", "gdn"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-side-workloads", action="store_true",
                    help="decode: skip the config-0 GEMV and config-1 GDN lines reported beside the headline")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_init(args)
    if args.workload in ("decode", "mtp", "gdn"):
        rc = {"decode": main_decode, "mtp": main_mtp, "gdn": main_gdn}[args.workload](args, ws, rank, local)
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return rc
    config = gemv_config(ws)
    if args.impl == "reference":
        if rank != 0:
            return 0
        ref, _ = ref_lib()
        if ref is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref reference build missing"}))
            return 0
        W, X = make_gemv_inputs(synth=Synth(ref))
        res = cpu_gemv_baseline(W, X, budget_s=max(4.0, min(60.0, 2.0 * args.steps)))
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref reference build missing"}))
            return 0
        gbs, info = res
        line = {"impl": "reference", "metric": "verify-GEMV GB/s (B=8 Q4_0, config 0)", "value": round(gbs, 2),
                "unit": "GB/s", "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(GEMV_BYTES / gbs / 1e6, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "numerics": "q4_0 weights x f32 X -> f32 Y (f16 hi+lo tensor-core operands, f32 accumulate)", "data": "synthetic (seeded)",
                "config": config, "cpu_baseline": {**info, "value": round(gbs, 2), "unit": "GB/s"},
                "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    line, W, X = gemv_ours_line(args, ws, rank, local, config)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        res = cpu_gemv_baseline(W, X)
        if res:
            line["cpu_baseline"] = {**res[1], "value": round(res[0], 2), "unit": "GB/s"}
    if rank == 0:
        print(json.dumps(line))
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
