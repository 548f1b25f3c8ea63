"""Multi-GPU sharding logic, run as world-size-2 ``gloo`` process groups on CPU.

Each rank takes its shard of one seeded decode step (by batch rows or by KV
heads, rotatek_b200.sharding), computes its outputs with the float64 oracle in
place of the GPU kernel, and gathers them; rank 0 checks the gathered output
against the oracle run on the full, unsharded inputs.  This covers the shard
arithmetic (GQA group of each KV head, per-head R / delta_mu / K / V slices,
mask rows) and the gather layout, which are host logic; the kernel on each
shard is the single-GPU path the GPU tests cover.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import decode as odec
from rotatek_b200 import sharding, synthetic as syn

B, HQ, HKV, SV, SF = 4, 8, 4, 70, 33


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    d = syn.make_decode(B, HQ, HKV, SV, SF, keep=32, seed=5, dtype=torch.float32)
    kw = d.as_kwargs()
    mask = torch.ones(B, SF, dtype=torch.uint8)
    mask[1, ::3] = 0
    kw["mask_full"] = mask
    return kw


def _worker(rank, world, port, mode, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kw = _inputs()
        p = sharding.plan(rank, world, B, HKV, HQ // HKV, mode=mode)
        local = sharding.shard_inputs(p, kw["q_full"], kw["R_partial"], kw["delta_mu"], kw["k_full"],
                                      kw["v_full"], kw["mask_full"], kw["k_sparse"], kw["v_sparse"])
        out_local = torch.from_numpy(odec.rotatek_decode(**local)).float()
        assert out_local.shape == (p.local_batch, 1, p.local_q_heads, 128)
        full = sharding.gather_output(p, out_local)
        if rank == 0:
            want = odec.rotatek_decode(**kw)
            result["err"] = float(np.abs(full.numpy() - want).max())
            result["shape"] = tuple(full.shape)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "batch"])
def test_sharded_decode_matches_unsharded(mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, result)) for r in range(2)]
        for pr in procs:
            pr.start()
        for pr in procs:
            pr.join(timeout=240)
        codes = [pr.exitcode for pr in procs]
        for pr in procs:
            if pr.is_alive():
                pr.kill()
        assert codes == [0, 0], codes
        assert result["shape"] == (B, 1, HQ, 128)
        assert result["err"] < 1e-6, result["err"]


def test_plan_rules():
    p = sharding.plan(3, 8, 64, 8, 8)
    assert p.mode == "heads" and (p.h0, p.h1, p.b0, p.b1) == (3, 4, 0, 64) and p.needs_gather
    p = sharding.plan(1, 4, 64, 8, 8)
    assert p.mode == "batch" and (p.b0, p.b1, p.h0, p.h1) == (16, 32, 0, 8) and not p.needs_gather
    assert sharding.plan(0, 1, 64, 8, 8).mode == "batch"
    with pytest.raises(ValueError):
        sharding.plan(0, 3, 64, 8, 8)
    with pytest.raises(ValueError):
        sharding.plan(0, 3, 64, 8, 8, mode="heads")
