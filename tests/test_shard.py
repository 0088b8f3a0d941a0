"""Row-sharded decode over 2 GPUs of one node (cwen_cuda_shard_*), small
seeded geometry, one process per GPU.  Needs >= 2 GPUs (skipped otherwise).

- every GPU of the group computes the same logits (bit-identical: the
  replicated layers run the same kernels on the same inputs, the sharded
  rows are exchanged);
- the group's logits match a single-GPU engine within relative L2 1e-5 and
  the CPU oracle within 1e-4, over several decode positions (the sharded
  GEMVs sum in another fp32 order than one GPU's, K is never split);
- speculative decode in the group emits exactly the group's serial stream.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 7
CTX = 256
N_POS = 12


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, ws, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(ws),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import torch.distributed as dist

    import bench
    import cwen_b200
    from oracle_lib import vp
    try:
        bench.dist_init(None)
        L = cwen_b200.lib()
        cwen_b200.check(L.cwen_cuda_init(rank, CTX, 16), "init")
        cwen_b200.check(L.cwen_cuda_shard_config(rank, ws), "shard_config")
        d = cwen_b200.dims("small")
        cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 2), "load_synth")
        blob = (C.c_uint8 * bench.SHARD_HANDLE)()
        cwen_b200.check(L.cwen_cuda_shard_handle(blob, bench.SHARD_HANDLE), "shard_handle")
        cwen_b200.check(L.cwen_cuda_shard_open(bench.shard_exchange(bytes(blob), ws), ws), "shard_open")
        toks = np.random.default_rng(3).integers(0, d.n_vocab, size=N_POS).astype(np.int32)
        lgs = np.zeros((N_POS, d.n_vocab), np.float32)
        cwen_b200.check(L.cwen_cuda_reset())
        for p, t in enumerate(toks):
            am = C.c_int(-1)
            cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, C.byref(am)), "forward_serial")
            cwen_b200.check(L.cwen_cuda_logits(0, vp(lgs[p])), "logits")
        prompt = np.random.default_rng(9).integers(0, d.n_vocab, size=24).astype(np.int32)
        serial, _ = cwen_b200.generate(prompt, 40, cwen_b200.spec_cfg(spec=0))
        spec, st = cwen_b200.generate(prompt, 40, cwen_b200.spec_cfg(spec=1, use_mtp=0, max_draft=8))
        L.cwen_cuda_shutdown()
        q.put((rank, lgs, serial, spec))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        q.put((rank, repr(e), None, None))


def test_sharded_decode_two_gpus(orc):
    if _gpus() < 2:
        pytest.skip("row-sharded decode needs 2 GPUs")
    import torch.multiprocessing as mp

    import cwen_b200
    from oracle_lib import CwDims, rel_l2
    ws = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = dict((r, (lg, se, sp)) for r, lg, se, sp in (q.get(timeout=600) for _ in range(ws)))
    for p in procs:
        p.join(timeout=120)
    for r in range(ws):
        assert not isinstance(res[r][0], str), res[r][0]
    lg0, ser0, spec0 = res[0]
    lg1, ser1, spec1 = res[1]
    assert np.array_equal(lg0.view(np.uint32), lg1.view(np.uint32)), "GPUs of the group disagree"
    assert np.array_equal(ser0, ser1) and np.array_equal(spec0, ser0), "spec differs from the group's serial stream"
    # one GPU, same model and ids
    L = cwen_b200.lib()
    cwen_b200.check(L.cwen_cuda_init(0, CTX, 16), "init")
    od = CwDims()
    orc.cw_dims_tiny(C.byref(od))
    om = orc.or_model_synth(C.byref(od), SEED, CTX, 0)
    try:
        d = cwen_b200.dims("small")
        cwen_b200.check(L.cwen_load_synth(SEED, C.byref(d), 0), "load_synth")
        toks = np.random.default_rng(3).integers(0, d.n_vocab, size=N_POS).astype(np.int32)
        cwen_b200.check(L.cwen_cuda_reset())
        orc.or_reset(om)
        lg = np.zeros(d.n_vocab, np.float32)
        for p, t in enumerate(toks):
            am = C.c_int(-1)
            cwen_b200.check(L.cwen_cuda_forward_serial(int(t), 1, C.byref(am)), "forward_serial")
            cwen_b200.check(L.cwen_cuda_logits(0, lg.ctypes.data_as(C.c_void_p)), "logits")
            orc.or_forward(om, int(t), p, 1)
            olg = np.ctypeslib.as_array(orc.or_logits(om), shape=(d.n_vocab,))
            assert rel_l2(lg0[p], lg) <= 1e-5, (p, rel_l2(lg0[p], lg))
            assert rel_l2(lg0[p], olg) <= 1e-4, (p, rel_l2(lg0[p], olg))
    finally:
        L.cwen_cuda_shutdown()
        orc.or_model_free(om)
