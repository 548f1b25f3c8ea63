#!/usr/bin/env python
"""Decode-step benchmark of the RotateK hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark config 2, the headline metric): one attention layer's
single-token decode at the Qwen2.5-VL-7B attention shape -- bf16, B=32,
28 query / 4 KV heads (G=7), head_dim 128, D_keep=32 (channel_ratio 0.75),
64 prompt + 15 360 visual + 576 text tokens.  A step is one call of
``rotatek_b200.kernels.rotatek_decode`` over that batch (one kernel launch).
Inputs are seeded synthetic tensors (low-rank-plus-noise Keys rotated into a
top-32 basis, N(0,1) Values and queries); their 672.6 MB exceed the 126 MB
L2, so no flush is needed between steps.

With --gpus N (launched under torchrun) every rank runs its own batch of 32
(batch-sharded replicas, weak scaling, no data-path collective); the timed
region is bracketed by barriers and the max over ranks is reported.

`value` is the whole-job time per batch-32 decode step in microseconds
(timed region / (steps * ranks)), lower is better.

--impl reference times the reference's own math on the host CPU: the eager
PyTorch restatement of rotatek/kernels/fused_decode.py (the reference has no
CPU decode of its own; its kernels are Triton-only), on the full batch.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "fused decode-attn us/step & HBM GB/s %peak, bs32 16k ctx, 25% K channels kept"
UNIT = "us/step"
CFG = dict(batch=32, q_heads=28, kv_heads=4, head_dim=128, keep=32, prompt=64, vision=15360,
           text=576)
WORKLOAD = ("config2: Qwen2.5-VL-7B attention decode, bf16, B=32, H_q=28, H_kv=4 (G=7), "
            "D=128, D_keep=32, S = 64 prompt + 15360 visual + 576 text")
DATA = "synthetic: seeded low-rank+noise Keys rotated to a top-32 basis; N(0,1) Values/queries"
FALLBACK_HBM_GBS = 6650.0


def algorithmic_bytes(d) -> int:
    """Every input read once + output written once (mask excluded: all ones)."""
    return d.nbytes()


def load_peak_hbm():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic_per_launch(name="decode_tc_config2.txt", key="dram_bytes_per_launch"):
    """dram bytes per launch of a kernel from its committed ncu summary."""
    path = os.path.join(REPO, "profiles", name)
    try:
        for line in open(path):
            if line.startswith(key + " ") or line.startswith(key + "="):
                return int(float(line.split("=")[1].split()[0]))
    except OSError:
        pass
    return None


_SAMPLER_CHILD = r"""
import json, select, sys, time
import pynvml as nv
REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
           0x4: "sw_power_cap", 0x1: "gpu_idle", 0x80: "hw_power_brake_slowdown"}
nv.nvmlInit()
uuid, index = sys.argv[1], int(sys.argv[2])
try:
    h = nv.nvmlDeviceGetHandleByUUID(uuid)
except Exception:
    h = nv.nvmlDeviceGetHandleByIndex(index)
out = {"max": nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM), "mhz": [], "reasons": []}
print("ready", flush=True)
seen = set()
while True:
    out["mhz"].append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
    mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
    seen.update(name for bit, name in REASONS.items() if mask & bit)
    if select.select([sys.stdin], [], [], 0.001)[0]:
        break
out["reasons"] = sorted(seen)
print(json.dumps(out), flush=True)
"""


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, polled through NVML (what
    nvidia-smi reads) by a child process for as long as the context is open, so
    that sampling neither waits for nor delays the launching thread.  Reads only;
    changes no GPU setting."""

    def __init__(self, device: int):
        import subprocess
        self.proc, self.result = None, None
        try:
            props = torch.cuda.get_device_properties(device)
            uuid = "GPU-" + str(props.uuid)
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_CHILD, uuid, str(device)],
                                         stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            if self.proc.stdout.readline().strip() != "ready":
                self._close()
        except Exception:
            self._close()

    def _close(self):
        if self.proc is not None:
            try:
                self.proc.kill()
                self.proc.wait(timeout=10)
            except Exception:
                pass
        self.proc = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return
        try:
            out, _ = self.proc.communicate("stop\n", timeout=30)
            self.result = json.loads(out.strip().splitlines()[-1])
        except Exception:
            self._close()

    def summary(self):
        r = self.result
        if not r or not r["mhz"]:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(r["mhz"]), "sm_max_mhz": r["max"],
                "sm_min_mhz": min(r["mhz"]),
                "reasons": [x for x in r["reasons"] if x != "gpu_idle"], "samples": len(r["mhz"])}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def ramp_clocks(fn, min_s: float = 0.3) -> int:
    """Untimed calls of ``fn`` until ``min_s`` seconds of device work have run:
    an idle GPU needs some hundreds of milliseconds of load to reach its
    working SM and memory clocks, more than a few warm-up steps of a 0.1 ms
    kernel give it.  Returns the number of calls."""
    n, t0 = 0, time.perf_counter()
    while True:
        for _ in range(20):
            fn()
        n += 20
        torch.cuda.synchronize()
        if time.perf_counter() - t0 >= min_s:
            return n


def lead_in(cycles: int = 2_000_000) -> None:
    """Queue ~1 ms of device idling before a timed region's start event, so that
    the host has already queued the first timed launches when the GPU reaches
    them: the first step then measures the kernel, not the host's launch
    latency after an idle, synchronised stream."""
    torch.cuda._sleep(cycles)


def step_stats(per_step_ms) -> dict:
    """Percentiles of per-step device times (us) and the first five steps."""
    xs = sorted(per_step_ms)
    pick = lambda q: xs[min(len(xs) - 1, int(q * (len(xs) - 1) + 0.5))] * 1e3  # noqa: E731
    return {"p10_us": pick(0.1), "p50_us": pick(0.5), "p90_us": pick(0.9), "min_us": xs[0] * 1e3,
            "max_us": xs[-1] * 1e3, "first5_us": [x * 1e3 for x in per_step_ms[:5]]}


def make_inputs(device, dtype=torch.bfloat16, seed=0, batch=None):
    from rotatek_b200 import synthetic as syn
    b = CFG["batch"] if batch is None else batch
    return syn.make_decode(b, CFG["q_heads"], CFG["kv_heads"], CFG["vision"],
                           CFG["prompt"] + CFG["text"], head_dim=CFG["head_dim"],
                           keep=CFG["keep"], seed=seed, device=device, dtype=dtype)


def use_all_host_threads() -> int:
    """The CPU arms use every host thread this process may run on (torchrun sets
    OMP_NUM_THREADS=1 for its ranks; only rank 0 does CPU work here)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_baseline_sample(target_s: float = 12.0):
    """The reference's math, eager PyTorch on the host CPU (all threads), on a
    batch sample; returns (us per full batch-32 step, sample description, threads)."""
    from oracle.eager_torch import rotatek_decode_eager
    threads = use_all_host_threads()
    d = make_inputs("cpu", seed=1)
    kw = d.as_kwargs()
    rotatek_decode_eager(**kw)                       # warm-up
    t0 = time.perf_counter()
    rotatek_decode_eager(**kw)
    one = time.perf_counter() - t0
    reps = max(1, int(target_s / max(one, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        rotatek_decode_eager(**kw)
    us_full = (time.perf_counter() - t0) / reps * 1e6
    sample = (f"the full batch-32 step (bf16 inputs, fp32 math), {reps} reps, eager torch "
              f"restatement of fused_decode.py")
    return us_full, sample, threads


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from oracle.eager_torch import rotatek_decode_eager
    threads = use_all_host_threads()
    d = make_inputs("cpu", seed=1)
    kw = d.as_kwargs()
    for _ in range(args.warmup):
        rotatek_decode_eager(**kw)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        rotatek_decode_eager(**kw)
        times.append(time.perf_counter() - t0)
    per_full_us = statistics.mean(times) * 1e6
    sample = ("the full batch-32 step per step (bf16 inputs, fp32 math), eager torch restatement "
              "of fused_decode.py")
    line = {
        "impl": "reference", "metric": METRIC, "value": per_full_us, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_full_us / 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": {"workload": WORKLOAD, "global_batch": CFG["batch"], "seq_len": 16000,
                   "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": per_full_us, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": per_full_us, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist
    from rotatek_b200 import _lib
    from rotatek_b200.kernels import rotatek_decode

    d = make_inputs(dev, seed=1000 + rank, batch=args.batch)
    kw = d.as_kwargs()
    nbytes = algorithmic_bytes(d)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if pg is not None:
            pg.barrier()

    for _ in range(max(args.warmup, 3)):
        rotatek_decode(**kw)
    torch.cuda.synchronize()
    ramp_calls = ramp_clocks(lambda: rotatek_decode(**kw))

    # ---- device-timed region: inputs resident in HBM.  Two events around the K
    # steps (an event between every pair of launches costs ~1.4 us per step);
    # the per-step times for `step_stats` come from a second, separate pass.
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        lead_in()
        e_start.record(stream)
        for i in range(args.steps):
            rotatek_decode(**kw)
        e_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = e_start.elapsed_time(e_end)
    n_stats = min(args.steps, 200)
    events = [torch.cuda.Event(enable_timing=True) for _ in range(n_stats + 1)]
    lead_in()
    events[0].record(stream)
    for i in range(n_stats):
        rotatek_decode(**kw)
        events[i + 1].record(stream)
    torch.cuda.synchronize()
    per_step_ms = [events[i].elapsed_time(events[i + 1]) for i in range(n_stats)]
    mine_ms = total_ms
    if pg is not None:
        t = torch.tensor([total_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms = float(t.item())
    status = _lib.read_status(dev)
    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"kernel_only": True, "batch": args.batch or CFG["batch"],
                              "us_per_step": total_ms * 1e3 / args.steps,
                              "device_status": status}), flush=True)
        if pg is not None:
            pg.destroy_process_group()
        return 0

    # ---- end-to-end through the public API with host buffers
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    host = {k: (v.cpu().pin_memory() if torch.is_tensor(v) else v) for k, v in kw.items()}
    dev_in = {k: (torch.empty_like(v) if torch.is_tensor(v) else v) for k, v in kw.items()}
    h2d = sum(v.numel() * v.element_size() for v in host.values() if torch.is_tensor(v))
    out_host = torch.empty((CFG["batch"], 1, CFG["q_heads"], CFG["head_dim"]),
                           dtype=torch.bfloat16).pin_memory()
    d2h = out_host.numel() * out_host.element_size()

    def e2e_step():
        for k, v in host.items():
            if torch.is_tensor(v):
                dev_in[k].copy_(v, non_blocking=True)
        out, _, _ = rotatek_decode(**dev_in)
        out_host.copy_(out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    barrier()
    clocks = sampler.summary()
    if pg is not None:
        per_rank = [None] * world
        pg.all_gather_object(per_rank, clocks)
        mhz = [c["sm_mhz"] for c in per_rank if c["sm_mhz"] is not None]
        clocks = {"sm_mhz": statistics.median(mhz) if mhz else None,
                  "sm_max_mhz": per_rank[0]["sm_max_mhz"],
                  "reasons": sorted({x for c in per_rank for x in c["reasons"]}),
                  "samples": sum(c["samples"] for c in per_rank), "per_rank": per_rank}

    if rank == 0:
        peak, peak_kind = load_peak_hbm()
        avg_launch_s = mine_ms / args.steps / 1e3
        achieved = nbytes / avg_launch_s / 1e9
        us_per_step = total_ms * 1e3 / (args.steps * world)
        line = {
            "metric": METRIC, "value": us_per_step, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": total_ms / args.steps, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": DATA,
            "config": {"workload": WORKLOAD, "global_batch": CFG["batch"] * world,
                       "seq_len": CFG["prompt"] + CFG["vision"] + CFG["text"],
                       "parallelism": f"batch-sharded replicas x{world} (no collective)",
                       "l2": "inputs 672.6 MB per step > 126 MB L2; no flush"},
            "hbm_gbs": achieved, "hbm_frac": achieved / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": nbytes,
                         "traffic": ncu_traffic_per_launch()},
            "e2e": {"value": e2e_ms * 1e3 / (e2e_steps * world), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    # every step copies its inputs from pinned host memory, so the
                    # end-to-end time is set by the host link, not by the kernel
                    "bound": "host link (pinned H2D copy of the step's inputs)",
                    "host_link_gbs": (h2d + d2h) / (e2e_ms / e2e_steps / 1e3) / 1e9 if e2e_ms > 0 else None},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "device_status": status,
            "step_stats": dict(step_stats(per_step_ms), steps=n_stats,
                               note="a second pass with an event after every step (they add ~1.4 us each); "
                                    "value and roofline come from the K steps between two events"),
            "warmup_calls": {"steps": max(args.warmup, 3), "clock_ramp": ramp_calls,
                             "why": "untimed calls until 0.3 s of device work, so that an idle GPU's "
                                    "clocks have ramped before the timed steps"},
        }
        if world == 1:
            dense_us, dense_bytes = dense_same_context(d, max(50, args.steps // 4))
            line["dense_same_context"] = {
                "value": dense_us, "unit": UNIT, "speedup": dense_us / us_per_step,
                "algorithmic_bytes_per_launch": dense_bytes,
                "hbm_frac": dense_bytes / dense_us / 1e3 / peak,
                "what": "full_channel_decode over the same 16000-token context with full-width visual Keys"}
        if world == 1 and not args.no_extras:
            ours_out, _, _ = rotatek_decode(**kw)
            line["reference_gpu_same_box"] = reference_gpu_decode(d, us_per_step, ours_out, 50)
        if world == 1 and not args.no_cpu_baseline:
            us_cpu, sample, threads = cpu_baseline_sample()
            line["cpu_baseline"] = {"value": us_cpu, "unit": UNIT, "cores": threads,
                                    "kind": "port", "sample": sample}
    # ---- the other benchmark configurations, measured in the same run
    if not args.no_extras:
        del d, kw, host, dev_in
        torch.cuda.empty_cache()
        extras = {}
        if world == 1:
            extras["build_config4"] = build_summary(dev, steps=10, warmup=3)
            extras.update(fp8_spark_extras(dev))
        else:
            extras["strong_config2"] = strong_config2(dev, pg, rank, world, steps=200)
        # measured: at 2 GPUs the all_gather hides behind a 0.4 ms layer decode with no
        # reserve; at 8 GPUs (0.1 ms per layer) leaving it 8 SMs is fastest
        extras["config5"] = config5_step(dev, pg, rank, world, steps=5, warmup=2,
                                         sm_reserve=0 if world <= 2 else 8)
        if rank == 0:
            line.update(extras)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


REF_DIR = os.path.join(REPO, "baseline", "_ref")


def reference_gpu_decode(d, ours_us: float, ours_out: torch.Tensor, steps: int) -> dict:
    """The reference's own Triton decode kernels on this GPU at the same inputs:
    ``rotatek_decode_fused_triton`` (ROTATEK_KERNEL=paper, fused_decode.py:303-420)
    and ``rotatek_decode_gqa`` (gqa_decode.py:280-321), imported unmodified from
    baseline/_ref.  CUDA events over ``steps`` back-to-back calls after warm-up;
    each output is compared with ours (max abs difference).  A comparison
    outside the product path, reported beside the headline."""
    pkg = os.path.join(REF_DIR, "rotatek")
    if not os.path.isdir(pkg):
        return {"unavailable": "baseline/_ref/rotatek is absent (the reference is not pip-installable; "
                               "its rotatek/ package is copied there unmodified)"}
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    res = {}
    try:
        import triton
        from rotatek.kernels.fused_decode import rotatek_decode_fused_triton
        from rotatek.kernels.gqa_decode import rotatek_decode_gqa
        res["triton"] = triton.__version__
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"import failed: {type(exc).__name__}: {exc}"[:300]}
    kw = d.as_kwargs()
    for name, fn in (("paper", rotatek_decode_fused_triton), ("gqa", rotatek_decode_gqa)):
        try:
            for _ in range(3):
                out = fn(**kw)[0]
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            lead_in()
            e0.record()
            for _ in range(steps):
                fn(**kw)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / steps
            out = fn(**kw)[0].float()
            res[name] = {"us_per_step": us, "speedup_of_ours": us / ours_us,
                         "max_abs_diff_vs_ours": float((out.reshape(d.q_full.shape) -
                                                        ours_out.float().reshape(d.q_full.shape)).abs().max())}
        except Exception as exc:  # noqa: BLE001
            res[name] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    return res



def dense_same_context(d, steps):
    """Config 2's comparison: a full-channel flash-decode of the same context
    (prompt/text Keys plus the visual Keys at full width, rotated back as K~ R^T)
    through ``full_channel_decode``; CUDA events over ``steps`` back-to-back calls.
    Returns (us per call, algorithmic bytes per call)."""
    from rotatek_b200.kernels import full_channel_decode
    G = CFG["q_heads"] // CFG["kv_heads"]
    k_vis = torch.matmul(d.k_sparse, d.R_partial.transpose(-1, -2))
    keys = torch.cat([d.k_full, k_vis], dim=2)
    values = torch.cat([d.v_full, d.v_sparse], dim=2)
    del k_vis
    e = lambda t: t.numel() * t.element_size()  # noqa: E731
    nbytes = e(keys) + e(values) + 2 * e(d.q_full)
    for _ in range(5):
        full_channel_decode(d.q_full, keys, values, num_kv_groups=G)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lead_in()
    e0.record()
    for _ in range(steps):
        full_channel_decode(d.q_full, keys, values, num_kv_groups=G)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / steps, nbytes


# ---------------------------------------------------------------- config 4: the rotation build
BUILD_METRIC = "config4 prefill rotation build us/step (28 layers x B=8 x 4 KV heads, S_v=15360, bf16)"
CFG4 = dict(layers=28, batch=8, q_heads=28, kv_heads=4, head_dim=128, keep=32, vision=15360, window=32)
BUILD_WORKLOAD = ("config4: Qwen2.5-VL-7B prefill rotation build for all 28 layers, bf16, B=8, "
                  "H_kv=4 (G=7), D=128, keep 32, 15360 visual Keys per head (896 128x128 solves)")


def build_inputs(device, seed=0, layers=None, batch=None):
    from rotatek_b200 import synthetic as syn
    nb = (CFG4["layers"] if layers is None else layers) * (CFG4["batch"] if batch is None else batch)
    keys = syn.lowrank_keys(nb, CFG4["kv_heads"], CFG4["vision"], seed=seed, device=device,
                            dtype=torch.bfloat16)
    queries = syn.normal((nb, CFG4["q_heads"], CFG4["window"], CFG4["head_dim"]), seed + 1, device,
                         torch.bfloat16)
    return keys, queries


# Minimum HBM traffic of one config-4 build step: the visual Keys read twice
# (covariance pass, rotation pass) and the rotated-truncated Keys written once.
def build_min_bytes(keys, keep) -> int:
    kbytes = keys.numel() * keys.element_size()
    return 2 * kbytes + kbytes * keep // keys.shape[-1]


def build_summary(dev, steps: int, warmup: int, seed: int = 100) -> dict:
    """The config-4 build measured on its own (CUDA events): the whole step, its
    HBM fraction on the minimum bytes, each kernel's time and share, the
    eigensolver's time per 128x128 solve and the one-layer (32-matrix) build."""
    from rotatek_b200 import rotation as rot
    G = CFG4["q_heads"] // CFG4["kv_heads"]
    keep = CFG4["keep"]
    keys, queries = build_inputs(dev, seed=seed)
    nmat = keys.shape[0] * keys.shape[1]
    stream = torch.cuda.current_stream(dev)

    def timed(fn, reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
        lead_in()
        ev[0].record(stream)
        for i in range(reps):
            fn()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
        return [ev[i].elapsed_time(ev[i + 1]) for i in range(reps)]

    step = lambda: rot.build_rotation(keys, queries, keep, G)  # noqa: E731
    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    step_ms = statistics.mean(timed(step, steps))
    kept, R, dm, _ = step()
    cov_ms = statistics.mean(timed(lambda: rot.key_covariance(keys), 3))
    rot_ms = statistics.mean(timed(lambda: rot.rotate_keys(keys, R), 3))
    layer = lambda: rot.build_rotation(keys[:CFG4["batch"]], queries[:CFG4["batch"]], keep, G)  # noqa: E731
    layer()
    layer_ms = statistics.mean(timed(layer, 5))
    eig_ms = max(step_ms - cov_ms - rot_ms, 0.0)
    peak, peak_kind = load_peak_hbm()
    nbytes = build_min_bytes(keys, keep)
    out = {"what": BUILD_WORKLOAD, "us_per_step": step_ms * 1e3, "steps": steps,
           "hbm": {"achieved": nbytes / step_ms / 1e6, "peak": peak, "unit": "GB/s",
                   "frac": nbytes / step_ms / 1e6 / peak, "min_bytes": nbytes, "peak_source": peak_kind},
           "phases_us": {"covariance": cov_ms * 1e3, "eigensolver": eig_ms * 1e3, "rotate": rot_ms * 1e3},
           "share": {"covariance": cov_ms / step_ms, "eigensolver": eig_ms / step_ms, "rotate": rot_ms / step_ms},
           "eigensolver_us_per_128x128_solve": eig_ms * 1e3 / nmat,
           "one_layer_build_us": layer_ms * 1e3,
           "device_status": rot.read_build_status(dev)}
    del keys, queries, kept, R, dm
    torch.cuda.empty_cache()
    return out


def run_build(args):
    """Config 4: one step builds all 28 layers' rotations in one batched call
    (the 28 x 8 (layer, batch) problems stacked on the batch axis)."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist
    from rotatek_b200 import rotation as rot
    G = CFG4["q_heads"] // CFG4["kv_heads"]
    keep = CFG4["keep"]
    keys, queries = build_inputs(dev, seed=100 + rank, layers=args.layers)
    nmat = keys.shape[0] * keys.shape[1]
    stream = torch.cuda.current_stream(dev)

    def step():
        return rot.build_rotation(keys, queries, keep, G)

    def barrier():
        if pg is not None:
            pg.barrier()

    def timed(fn, reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
        lead_in()
        ev[0].record(stream)
        for i in range(reps):
            fn()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
        return [ev[i].elapsed_time(ev[i + 1]) for i in range(reps)]

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        per_step = timed(step, args.steps)
    barrier()
    total_ms = sum(per_step)
    if pg is not None:
        t = torch.tensor([total_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms = float(t.item())
    status = rot.read_build_status(dev)

    # the build's kernels one at a time, on the same inputs (CUDA events)
    kept, R, dm, _ = step()
    cov_ms = statistics.mean(timed(lambda: rot.key_covariance(keys), 3))
    rot_ms = statistics.mean(timed(lambda: rot.rotate_keys(keys, R), 3))
    layer = lambda: rot.build_rotation(keys[:CFG4["batch"]], queries[:CFG4["batch"]], keep, G)  # noqa: E731
    layer()
    layer_ms = statistics.mean(timed(layer, 3))
    step_ms = statistics.mean(per_step)
    jac_ms = max(step_ms - cov_ms - rot_ms, 0.0)

    # end to end through the public API: Keys and queries from pinned host memory,
    # kept / R / delta_mu back to pinned host memory, every step
    e2e_steps = max(1, min(args.steps, 2))
    hk, hq = keys.cpu().pin_memory(), queries.cpu().pin_memory()
    dk, dq = torch.empty_like(keys), torch.empty_like(queries)
    ok, oR, od = (torch.empty(kept.shape, dtype=kept.dtype).pin_memory(),
                  torch.empty(R.shape, dtype=R.dtype).pin_memory(),
                  torch.empty(dm.shape, dtype=dm.dtype).pin_memory())

    def e2e():
        dk.copy_(hk, non_blocking=True)
        dq.copy_(hq, non_blocking=True)
        k2, r2, d2, _ = rot.build_rotation(dk, dq, keep, G)
        ok.copy_(k2, non_blocking=True)
        oR.copy_(r2, non_blocking=True)
        od.copy_(d2, non_blocking=True)

    e2e()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = sum(timed(e2e, e2e_steps))
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    clocks = sampler.summary()
    if pg is not None:
        per_rank = [None] * world
        pg.all_gather_object(per_rank, clocks)
        mhz = [c["sm_mhz"] for c in per_rank if c["sm_mhz"] is not None]
        clocks = {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": per_rank[0]["sm_max_mhz"],
                  "reasons": sorted({x for c in per_rank for x in c["reasons"]}),
                  "samples": sum(c["samples"] for c in per_rank), "per_rank": per_rank}

    if rank == 0:
        peak, peak_kind = load_peak_hbm()
        kbytes = keys.numel() * keys.element_size()
        cov_bytes = kbytes + nmat * (128 * 128 + 128) * 4
        rot_bytes = kbytes + kept.numel() * kept.element_size() + R.numel() * R.element_size()
        us_per_step = total_ms * 1e3 / (args.steps * world)
        h2d = (hk.numel() + hq.numel()) * 2
        d2h = ok.numel() * 2 + oR.numel() * 2 + od.numel() * 2
        line = {
            "metric": BUILD_METRIC, "value": us_per_step, "unit": "us/step", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded low-rank+noise Keys (the benchmark generator), N(0,1) queries",
            "config": {"workload": BUILD_WORKLOAD, "layers": keys.shape[0] // CFG4["batch"],
                       "global_batch": CFG4["batch"] * world,
                       "seq_len": CFG4["vision"], "parallelism": f"replicas x{world} (no collective)",
                       "l2": f"Keys {kbytes / 1e9:.2f} GB per step > 126 MB L2; no flush"},
            "phases_us": {"covariance": cov_ms * 1e3, "rotate": rot_ms * 1e3,
                          "eigensolve_and_rest": jac_ms * 1e3,
                          "eigensolve_us_per_128x128_solve": jac_ms * 1e3 / nmat,
                          "one_layer_build": layer_ms * 1e3,
                          "per_layer_sequential_28": layer_ms * 1e3 * CFG4["layers"]},
            "roofline": {"bound": "hbm", "kernel": "whole build step (covariance + eigensolver + rotate)",
                         "achieved": build_min_bytes(keys, keep) / (total_ms / args.steps * 1e-3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": build_min_bytes(keys, keep) / (total_ms / args.steps * 1e-3) / 1e9 / peak,
                         "min_bytes": build_min_bytes(keys, keep), "traffic": None,
                         "note": "the eigensolver (eigh_kernel) moves ~0.07 MB per matrix and is bound by "
                                 "its sequential steps; reported as time per solve"},
            "hbm_kernels": {
                "covariance": {"bound": "hbm", "achieved": cov_bytes / cov_ms / 1e6, "peak": peak,
                               "unit": "GB/s", "frac": cov_bytes / cov_ms / 1e6 / peak,
                               "algorithmic_bytes": cov_bytes, "peak_source": peak_kind},
                "rotate": {"bound": "hbm", "achieved": rot_bytes / rot_ms / 1e6, "peak": peak,
                           "unit": "GB/s", "frac": rot_bytes / rot_ms / 1e6 / peak,
                           "algorithmic_bytes": rot_bytes, "peak_source": peak_kind}},
            "e2e": {"value": e2e_ms * 1e3 / (e2e_steps * world), "unit": "us/step",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "gpu_launches": 3 * args.steps, "clocks": clocks, "device_status": status,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = build_cpu_baseline()
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def build_cpu_baseline(target_s: float = 12.0):
    """The reference's update_rotatek (eigh solver) in eager torch on the host:
    one layer at batch 1 (4 KV heads), scaled x8 x28 to the config-4 step."""
    from oracle.eager_torch import update_rotatek_eager
    threads = use_all_host_threads()
    keys, queries = build_inputs("cpu", seed=7, layers=1, batch=1)
    G = CFG4["q_heads"] // CFG4["kv_heads"]
    update_rotatek_eager(keys, queries, CFG4["keep"], G)
    t0 = time.perf_counter()
    update_rotatek_eager(keys, queries, CFG4["keep"], G)
    one = time.perf_counter() - t0
    reps = max(1, int(target_s / max(one, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        update_rotatek_eager(keys, queries, CFG4["keep"], G)
    per = (time.perf_counter() - t0) / reps
    scale = CFG4["layers"] * CFG4["batch"]
    return {"value": per * 1e6 * scale, "unit": "us/step", "cores": threads, "kind": "port",
            "sample": f"1 layer at batch 1 (4 KV heads, full S_v), {reps} reps, eager torch "
                      f"update_rotatek (eigh), scaled x{scale}"}


def run_build_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from oracle.eager_torch import update_rotatek_eager
    threads = use_all_host_threads()
    keys, queries = build_inputs("cpu", seed=7, layers=1, batch=1)
    G = CFG4["q_heads"] // CFG4["kv_heads"]
    for _ in range(args.warmup):
        update_rotatek_eager(keys, queries, CFG4["keep"], G)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        update_rotatek_eager(keys, queries, CFG4["keep"], G)
        times.append(time.perf_counter() - t0)
    scale = CFG4["layers"] * CFG4["batch"]
    v = statistics.mean(times) * 1e6 * scale
    line = {"impl": "reference", "metric": BUILD_METRIC, "value": v, "unit": "us/step", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v / 1e3, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded low-rank+noise Keys, N(0,1) queries",
            "config": {"workload": BUILD_WORKLOAD, "global_batch": CFG4["batch"], "seq_len": CFG4["vision"],
                       "parallelism": "host CPU, rank 0 only"},
            "cpu_baseline": {"value": v, "unit": "us/step", "cores": threads, "kind": "port",
                             "sample": f"1 layer at batch 1 per step, eager torch update_rotatek (eigh), "
                                       f"scaled x{scale}"},
            "e2e": {"value": v, "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- config 2 with cache maintenance
STEP_METRIC = "decode step incl. KV-cache append us/step, config 2 shape (bs32 16k ctx, 25% K channels kept)"


def run_decode_step(args):
    """One decode step of one layer as a model runs it: append the new token's
    K/V to the cache, then the fused decode.  ``SpanKVCache`` appends in place and
    hands the decode views; the reference's cache and adapter instead copy the
    whole V cache (torch.cat, cache_utils.py:52-53) and build k_full / v_full /
    mask with torch.cat and torch.ones (llama_visionzip.py:203-214) every step --
    timed here as ``adapter_path`` with the same decode kernel."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from rotatek_b200 import synthetic as syn
    from rotatek_b200.cache import SpanKVCache
    from rotatek_b200.kernels import rotatek_decode
    G = CFG["q_heads"] // CFG["kv_heads"]
    sp, st, sv = CFG["prompt"], CFG["text"], CFG["vision"]
    d = make_inputs(dev, seed=3)
    kw = d.as_kwargs()
    b, h = CFG["batch"], CFG["kv_heads"]
    # prefill-order tensors: V = [prompt | visual | text]
    k_prompt, k_text = kw["k_full"][:, :, :sp].contiguous(), kw["k_full"][:, :, sp:].contiguous()
    values = torch.cat([kw["v_full"][:, :, :sp], kw["v_sparse"], kw["v_full"][:, :, sp:]], dim=-2)
    n_steps = max(args.warmup, 3) + args.steps
    cache = SpanKVCache(max_new_tokens=n_steps)
    cache.store_pruned(kw["k_sparse"], k_prompt, k_text, values, kw["R_partial"], kw["delta_mu"], 0)
    new_k = syn.normal((n_steps, b, h, 1, 128), 41, dev, torch.bfloat16)
    new_v = syn.normal((n_steps, b, h, 1, 128), 42, dev, torch.bfloat16)
    qs = syn.normal((n_steps, b, CFG["q_heads"], 128), 43, dev, torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def cache_step(i):
        cache.update(new_k[i], new_v[i], 0)
        rotatek_decode(q_full=qs[i], num_kv_groups=G, **cache.decode_args(0))

    state = {"k_text": k_text, "values": values}

    def adapter_step(i):
        state["k_text"] = torch.cat([state["k_text"], new_k[i]], dim=-2)
        state["values"] = torch.cat([state["values"], new_v[i]], dim=-2)
        vals = state["values"]
        rotatek_decode(q_full=qs[i], R_partial=kw["R_partial"], delta_mu=kw["delta_mu"],
                       k_full=torch.cat([k_prompt, state["k_text"]], dim=-2),
                       v_full=torch.cat([vals[:, :, :sp], vals[:, :, sp + sv:]], dim=-2),
                       mask_full=torch.ones(b, sp + state["k_text"].shape[2], device=dev, dtype=torch.uint8),
                       k_sparse=kw["k_sparse"], v_sparse=vals[:, :, sp:sp + sv], num_kv_groups=G)

    def timed(fn):
        w = max(args.warmup, 3)
        for i in range(w):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(w, w + args.steps):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / args.steps

    sampler = ClockSampler(0)
    with sampler:
        ours = timed(cache_step)
    adapter = timed(adapter_step)
    line = {"metric": STEP_METRIC, "value": ours, "unit": "us/step", "n_gpus": 1, "steps": args.steps,
            "warmup": max(args.warmup, 3), "higher_is_better": False, "dtype": "bf16",
            "data": DATA, "config": {"workload": WORKLOAD + "; one token appended per step"},
            "adapter_path_us": adapter, "speedup_vs_adapter_path": adapter / ours,
            "gpu_launches": 3 * args.steps, "clocks": sampler.summary()}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- ThinK baseline at config 2
THINK_METRIC = "ThinK decode step us/step, config 2 shape (bs32 16k ctx, 32 of 128 K channels kept per head)"


def run_think(args):
    """ThinK's decode at the config-2 shape: ``think_decode`` (the kept channels
    through the fused kernel) against the adapters' path -- zero-filled
    recovery of the visual Keys, concatenation and the dense decode
    (llama_visionzip.py:217-240) -- both on this GPU."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from rotatek_b200 import synthetic as syn
    from rotatek_b200.kernels import full_channel_decode, think_decode
    b, hkv, G, sp, sv, st = CFG["batch"], CFG["kv_heads"], CFG["q_heads"] // CFG["kv_heads"], CFG["prompt"], \
        CFG["vision"], CFG["text"]
    keep = CFG["keep"]
    k_all = syn.lowrank_keys(b, hkv, sp + sv + st, seed=5, device=dev, dtype=torch.bfloat16)
    values = syn.normal((b, hkv, sp + sv + st, 128), 6, dev, torch.bfloat16)
    q = syn.normal((b, CFG["q_heads"], 128), 7, dev, torch.bfloat16)
    score = torch.rand(b, hkv, 128, device=dev)
    think_mask = torch.zeros(b, hkv, 128, dtype=torch.bool, device=dev)
    think_mask.scatter_(2, score.topk(keep, dim=-1).indices, True)
    k_vis = k_all[:, :, sp:sp + sv]
    sel = think_mask.unsqueeze(2).expand(-1, -1, sv, -1)
    key_pruned = k_vis[sel].view(b, hkv, sv, keep)
    k_prompt, k_text = k_all[:, :, :sp].contiguous(), k_all[:, :, sp + sv:].contiguous()
    k_full = torch.cat([k_prompt, k_text], dim=-2)
    v_full = torch.cat([values[:, :, :sp], values[:, :, sp + sv:]], dim=-2)
    v_vis = values[:, :, sp:sp + sv]

    from rotatek_b200.kernels import think_selection
    selection = think_selection(think_mask, keep, q.dtype)   # once per layer, after prefill

    def fused():
        think_decode(q, think_mask, key_pruned, k_full, v_full, None, v_vis, G, selection=selection)

    def adapter():
        recovered = torch.zeros(b, hkv, sv, 128, dtype=key_pruned.dtype, device=dev)
        recovered[sel] = key_pruned.reshape(-1)
        keys = torch.cat([k_prompt, recovered, k_text], dim=-2)
        full_channel_decode(q, keys, values, num_kv_groups=G)

    def timed(fn, n):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    sampler = ClockSampler(0)
    with sampler:
        ours = timed(fused, args.steps)
    theirs = timed(adapter, max(10, args.steps // 10))
    nbytes = (key_pruned.numel() + v_vis.numel() + k_full.numel() + v_full.numel() + 2 * q.numel()) * 2
    peak, peak_kind = load_peak_hbm()
    print(json.dumps({"metric": THINK_METRIC, "value": ours, "unit": "us/step", "n_gpus": 1, "steps": args.steps,
                      "higher_is_better": False, "dtype": "bf16", "data": DATA,
                      "config": {"workload": WORKLOAD + "; ThinK channel selection instead of a rotation"},
                      "adapter_path_us": theirs, "speedup_vs_adapter_path": theirs / ours,
                      "roofline": {"bound": "hbm", "achieved": nbytes / ours / 1e3, "peak": peak, "unit": "GB/s",
                                   "frac": nbytes / ours / 1e3 / peak, "peak_source": peak_kind,
                                   "algorithmic_bytes_per_launch": nbytes},
                      "clocks": sampler.summary()}), flush=True)
    return 0


# ---------------------------------------------------------------- fp8 visual span (config 2 shape)
FP8_METRIC = "fp8 visual-span decode us/step & HBM GB/s %peak, config 2 shape (bs32 16k ctx, 25% K channels kept)"


def fp8_spark_extras(dev, steps=300):
    """The two decode variants of this build at the config-2 shape, measured in
    the default run: the visual span in e4m3 (``rotatek_decode_fp8``) and SparK
    (``spark_decode``).  CUDA events over ``steps`` back-to-back calls after
    warm-up; each against the measured HBM peak on its own algorithmic bytes
    (every input read once, inputs larger than L2).  Their own workloads
    (``--workload decode_fp8`` / ``spark``) add the comparisons."""
    from rotatek_b200 import synthetic as syn
    from rotatek_b200.kernels import pack_spark_indices, quantize_visual_fp8, rotatek_decode_fp8, spark_decode
    e = lambda t: t.numel() * t.element_size()  # noqa: E731
    peak, peak_kind = load_peak_hbm()

    def timed(fn, n):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    def summary(us, nbytes, what):
        return {"value": us, "unit": "us/step", "algorithmic_bytes_per_launch": nbytes,
                "hbm_frac": nbytes / us / 1e3 / peak, "peak_source": peak_kind, "steps": steps, "what": what}

    out = {}
    d = make_inputs(dev, seed=0)
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    args8 = (d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full, k8, ksc, v8, vsc, d.num_kv_groups)
    nbytes = (e(k8) + e(ksc) + e(v8) + e(vsc) + e(d.k_full) + e(d.v_full) + e(d.R_partial) + e(d.delta_mu)
              + 2 * e(d.q_full))
    out["decode_fp8"] = summary(timed(lambda: rotatek_decode_fp8(*args8), steps), nbytes,
                                "config 2 with the visual K~ and V in e4m3 (quantize_visual_fp8 once)")
    del d, k8, ksc, v8, vsc, args8
    torch.cuda.empty_cache()
    b, hkv, sp, sv, st = CFG["batch"], CFG["kv_heads"], CFG["prompt"], CFG["vision"], CFG["text"]
    g = CFG["q_heads"] // hkv
    d = syn.make_spark(b, CFG["q_heads"], hkv, sv, sp + st, keep=CFG["keep"], seed=0, device=dev,
                       dtype=torch.bfloat16)
    idx = pack_spark_indices(d.keep_mask, CFG["keep"])
    nbytes = (e(d.k_kept) + e(idx) + e(d.pruned_mean) + e(d.v_sparse) + e(d.k_full) + e(d.v_full)
              + 2 * e(d.q_full))
    out["spark"] = summary(timed(lambda: spark_decode(d.q_full, d.k_full, d.v_full, None, d.k_kept, idx,
                                                      d.pruned_mean, d.v_sparse, g), steps), nbytes,
                           "config 2 with SparK's per-token channel pruning (kept values + indices)")
    del d, idx
    torch.cuda.empty_cache()
    return out


def run_decode_fp8(args):
    """The config-2 decode step with the visual span stored in e4m3
    (``quantize_visual_fp8`` once after prefill, then ``rotatek_decode_fp8``);
    the 16-bit decode of the same inputs timed beside it."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from rotatek_b200.kernels import quantize_visual_fp8, rotatek_decode, rotatek_decode_fp8
    d = make_inputs(dev, seed=0, batch=args.batch)
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    fp8_args = (d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full, k8, ksc, v8, vsc,
                d.num_kv_groups)

    def timed(fn, n):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    sampler = ClockSampler(0)
    with sampler:
        ours = timed(lambda: rotatek_decode_fp8(*fp8_args), args.steps)
    bf16 = timed(lambda: rotatek_decode(**d.as_kwargs()), max(10, args.steps // 4))
    out8, _, _ = rotatek_decode_fp8(*fp8_args)
    ref, _, _ = rotatek_decode(**d.as_kwargs())
    rel = float((out8.float() - ref.float()).norm() / ref.float().norm())
    e = lambda t: t.numel() * t.element_size()  # noqa: E731
    nbytes = (e(k8) + e(ksc) + e(v8) + e(vsc) + e(d.k_full) + e(d.v_full) + e(d.R_partial) + e(d.delta_mu)
              + 2 * e(d.q_full))
    peak, peak_kind = load_peak_hbm()
    if args.kernel_only:
        return 0
    print(json.dumps({"metric": FP8_METRIC, "value": ours, "unit": "us/step", "n_gpus": 1, "steps": args.steps,
                      "warmup": max(args.warmup, 3), "higher_is_better": False,
                      "dtype": "e4m3 visual span (K~ per-channel, V per-token scales), bf16 prompt/text",
                      "data": DATA, "config": {"workload": WORKLOAD + "; visual K~ and V stored in e4m3",
                                               "l2": f"{nbytes / 1e6:.0f} MB per step > 126 MB L2; no flush"},
                      "bf16_decode_us": bf16, "speedup_vs_bf16_decode": bf16 / ours,
                      "rel_error_vs_bf16_decode": rel,
                      "roofline": {"bound": "hbm", "achieved": nbytes / ours / 1e3, "peak": peak, "unit": "GB/s",
                                   "frac": nbytes / ours / 1e3 / peak, "peak_source": peak_kind,
                                   "algorithmic_bytes_per_launch": nbytes},
                      "gpu_launches": args.steps, "clocks": sampler.summary()}), flush=True)
    return 0


# ---------------------------------------------------------------- SparK baseline at config 2
SPARK_METRIC = "SparK decode step us/step, config 2 shape (bs32 16k ctx, 32 of 128 K channels kept per token)"


def run_spark(args):
    """SparK's decode at the config-2 shape: ``spark_decode`` (kept values,
    kept-channel indices and the pruned mean; Keys rebuilt block by block in
    shared memory) against the adapters' path on the same GPU -- recovery of the
    full-width visual Keys, concatenation and the dense decode
    (llama_visionzip.py:226-242) -- and against the dense decode alone over Keys
    recovered beforehand."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from rotatek_b200 import synthetic as syn
    from rotatek_b200.kernels import full_channel_decode, pack_spark_indices, spark_decode
    b, hkv, G, sp, sv, st = CFG["batch"], CFG["kv_heads"], CFG["q_heads"] // CFG["kv_heads"], CFG["prompt"], \
        CFG["vision"], CFG["text"]
    if args.batch:                   # profiling cases only
        b = args.batch
    keep = CFG["keep"]
    d = syn.make_spark(b, CFG["q_heads"], hkv, sv, sp + st, keep=keep, seed=0, device=dev, dtype=torch.bfloat16)
    idx = pack_spark_indices(d.keep_mask, keep)          # once per layer, after prefill
    k_prompt, k_text = d.k_full[:, :, :sp], d.k_full[:, :, sp:]
    values = torch.cat([d.v_full[:, :, :sp], d.v_sparse, d.v_full[:, :, sp:]], dim=-2)

    def fused():
        spark_decode(d.q_full, d.k_full, d.v_full, None, d.k_kept, idx, d.pruned_mean, d.v_sparse, G)

    def adapter():
        rec = d.pruned_mean.expand(b, hkv, sv, 128).contiguous()
        rec[d.keep_mask] = d.k_kept.reshape(-1)
        keys = torch.cat([k_prompt, rec, k_text], dim=-2)
        full_channel_decode(d.q_full, keys, values, num_kv_groups=G)

    keys_rec = torch.cat([k_prompt, d.recovered(), k_text], dim=-2)

    def dense_only():
        full_channel_decode(d.q_full, keys_rec, values, num_kv_groups=G)

    def timed(fn, n):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    sampler = ClockSampler(0)
    with sampler:
        ours = timed(fused, args.steps)
    if args.kernel_only:
        return 0
    dense = timed(dense_only, max(10, args.steps // 4))
    theirs = timed(adapter, max(10, args.steps // 20))
    e = lambda t: t.numel() * t.element_size()  # noqa: E731
    nbytes = (e(d.k_kept) + e(idx) + e(d.pruned_mean) + e(d.v_sparse) + e(d.k_full) + e(d.v_full)
              + 2 * e(d.q_full))
    peak, peak_kind = load_peak_hbm()
    print(json.dumps({"metric": SPARK_METRIC, "value": ours, "unit": "us/step", "n_gpus": 1, "steps": args.steps,
                      "warmup": max(args.warmup, 3), "higher_is_better": False, "dtype": "bf16",
                      "data": "synthetic: seeded low-rank+noise Keys pruned per token (SparK scoring against a "
                              "N(0,1) query window); N(0,1) Values/queries",
                      "config": {"workload": WORKLOAD + "; SparK per-token channel pruning instead of a rotation",
                                 "l2": f"{nbytes / 1e6:.0f} MB per step > 126 MB L2; no flush"},
                      "adapter_path_us": theirs, "speedup_vs_adapter_path": theirs / ours,
                      "dense_decode_of_recovered_keys_us": dense, "speedup_vs_dense_decode": dense / ours,
                      "roofline": {"bound": "hbm", "achieved": nbytes / ours / 1e3, "peak": peak, "unit": "GB/s",
                                   "frac": nbytes / ours / 1e3 / peak, "peak_source": peak_kind,
                                   "algorithmic_bytes_per_launch": nbytes},
                      "gpu_launches": args.steps, "clocks": sampler.summary()}), flush=True)
    return 0


# ---------------------------------------------------------------- fused Key projection (config 4 layer)
KPROJ_METRIC = ("config4 layer prefill Key path + rotation build us/layer (Qwen2.5-VL-7B shape: B=8, "
                "S=64+15360+576, hidden 3584, 4 KV heads, bf16)")
KPROJ = dict(batch=8, prompt=64, vision=15360, text=576, hidden=3584)


def run_kproj(args):
    """One layer's prefill Key path as the adapters run it -- k_proj, RoPE,
    then the rotation build of the visual span (llama_visionzip.py:144-165) --
    from the layer's hidden states.  Ours: ``build_rotation_projected``
    (projection + bias + RoPE in one tensor-core kernel, the visual span's sums
    from the Keys it wrote, eigensolver, rotate).  Beside it on the same GPU:
    cuBLAS k_proj + torch RoPE + ``build_rotation`` (the adapter path with this
    build's builder)."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from rotatek_b200 import rotation as rot
    from rotatek_b200 import synthetic as syn
    b, sp, sv, st, hid = KPROJ["batch"], KPROJ["prompt"], KPROJ["vision"], KPROJ["text"], KPROJ["hidden"]
    if args.batch:                   # profiling cases only
        b = args.batch
    if args.kproj_vision:
        sv = args.kproj_vision
    hkv, G, keep = CFG4["kv_heads"], CFG4["q_heads"] // CFG4["kv_heads"], CFG4["keep"]
    s = sp + sv + st
    dt = torch.bfloat16
    x = syn.normal((b, s, hid), 21, dev, dt)
    w = (syn.normal((hkv * 128, hid), 22, dev, torch.float32) * hid ** -0.5).to(dt)
    bias = (syn.normal((hkv * 128,), 23, dev, torch.float32) * 0.1).to(dt)
    inv = 1.0 / 1e6 ** (torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128)
    ang = torch.arange(s, device=dev, dtype=torch.float32)[:, None] * inv[None]
    ang = torch.cat([ang, ang], dim=-1)
    cos = ang.cos().to(dt)[None].expand(b, -1, -1).contiguous()
    sin = ang.sin().to(dt)[None].expand(b, -1, -1).contiguous()
    q = syn.normal((b, CFG4["q_heads"], CFG4["window"], 128), 24, dev, dt)

    def fused():
        return rot.build_rotation_projected(x, w, bias, cos, sin, sp, sv, q, keep, G)

    def projection():
        return rot.key_projection(x, w, bias, cos, sin, sp, sv)

    def adapter():
        k = torch.nn.functional.linear(x, w, bias).view(b, s, hkv, 128).transpose(1, 2)
        k = k * cos[:, None] + torch.cat([-k[..., 64:], k[..., :64]], dim=-1) * sin[:, None]
        return rot.build_rotation(k[:, :, sp:sp + sv], q, keep, G)

    def cublas():
        return torch.nn.functional.linear(x, w, bias)

    def timed(fn, n):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    sampler = ClockSampler(0)
    with sampler:
        ours = timed(fused, args.steps)
        proj = timed(projection, args.steps)
    status = rot.read_build_status(dev)
    theirs = timed(adapter, max(3, args.steps // 4))
    lin = timed(cublas, max(3, args.steps // 4))
    flops = 2 * b * s * hid * hkv * 128 + 2 * b * hkv * sv * 128 * 128   # projection + K^T K
    peak = None
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
        peak_kind = "measured (bf16 burst, MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        peak, peak_kind = 1590.0, "fallback 1.59 PFLOP/s"
    achieved = flops / proj / 1e6
    print(json.dumps({
        "metric": KPROJ_METRIC, "value": ours, "unit": "us/layer", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "higher_is_better": False, "dtype": "bf16",
        "data": "synthetic: N(0,1) hidden states, scaled N(0,1) k_proj weight and bias, RoPE theta 1e6",
        "config": {"workload": f"config4 layer: hidden states -> post-RoPE Keys (all {s} tokens) + rotation "
                               f"build of the {sv} visual tokens, B={b}, H_kv=4 (G=7), keep 32",
                   "l2": f"hidden states {x.numel() * 2 / 1e9:.2f} GB > 126 MB L2; no flush"},
        "phases_us": {"key_projection_fused": proj, "cublas_k_proj_alone": lin},
        "adapter_path_us": theirs, "speedup_vs_adapter_path": theirs / ours,
        "roofline": {"bound": "tensor", "kernel": "kproj_pair_kernel + cov_tc_kernel (visual-span sums)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "algorithmic_flops_per_launch": flops,
                     "traffic": ncu_traffic_per_launch("kproj_pair_small_case.txt", "dram_bytes_per_launch_config4"),
                     "algorithmic_bytes_per_launch": (x.numel() + w.numel() + bias.numel() + b * hkv * s * 128
                                                      + 2 * cos.numel()) * 2 + b * hkv * (128 * 128 + 128) * 4,
                     "cublas_k_proj_tflops": 2 * b * s * hid * hkv * 128 / lin / 1e6},
        "gpu_launches": 4 * args.steps, "clocks": sampler.summary(), "device_status": status}), flush=True)
    return 0


# ---------------------------------------------------------------- config 3: end-to-end decode
E2E_METRIC = "config3 e2e greedy decode tokens/s (LLaVA-NeXT-7B-shaped, fp16, 16384 visual tokens, 128 steps)"


def run_e2e(args):
    """Config 3: a random-init LLaVA-NeXT-7B-shaped decoder (32 layers, 32 MHA
    heads, hidden 4096, FFN 11008, vocab 32000, fp16), visual span of 16384
    synthetic tokens; prefill with the per-layer rotation build, then 128 greedy
    steps, each one CUDA-graph replay of the whole 32-layer step."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from rotatek_b200.kernels import rotatek_decode
    from rotatek_b200.llama_e2e import DecoderConfig, RandomLlamaDecoder
    cfg = DecoderConfig(max_new_tokens=args.e2e_tokens)
    model = RandomLlamaDecoder(cfg, dev, seed=0)
    batches = [args.batch] if args.batch else [1, 4, 8]
    peak, peak_kind = load_peak_hbm()
    # one untimed prefill first: the process's first calls load kernels and
    # cuBLAS heuristics, which would otherwise land in the first batch's time
    x = model.prompt_embeddings(1, seed=0)
    model.prefill(x)
    del x
    torch.cuda.synchronize()
    for b in batches:
        x = model.prompt_embeddings(b, seed=b)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        logits = model.prefill(x)
        e1.record()
        torch.cuda.synchronize()
        prefill_ms = e0.elapsed_time(e1)
        del x
        model.init_decode(logits.argmax(-1))
        model.decode_step()                      # warm-up (workspaces); token 1
        g = model.capture_decode_graph()
        steps = cfg.max_new_tokens - 1
        sampler = ClockSampler(0)
        with sampler:
            e0.record()
            for _ in range(steps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
        decode_ms = e0.elapsed_time(e1)
        # one layer's decode attention on its own (same static arguments)
        q = torch.randn(b, cfg.heads, cfg.head_dim, device=dev, dtype=cfg.dtype)
        la = model.cache.static_decode_args(cfg.layers - 1, model.mask)
        for _ in range(5):
            rotatek_decode(q_full=q, num_kv_groups=1, **la)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(50):
            rotatek_decode(q_full=q, num_kv_groups=1, **la)
        e1.record()
        torch.cuda.synchronize()
        attn_us = e0.elapsed_time(e1) * 1e3 / 50
        attn_bytes = model.attention_bytes_per_step() // cfg.layers
        line = {
            "metric": E2E_METRIC, "value": b * steps / (decode_ms * 1e-3), "unit": "tokens/s",
            "n_gpus": 1, "steps": steps, "warmup": 1, "higher_is_better": True, "dtype": "fp16",
            "data": "random-init weights, synthetic visual-span embeddings, random prompt tokens",
            "config": {"workload": "config3: LLaVA-NeXT-7B-shaped decoder (Vicuna: 32 layers, 32 MHA heads, "
                                   "hidden 4096, FFN 11008, vocab 32000), 32 prompt + 16384 visual + 32 text "
                                   "tokens, channel_ratio 0.75", "batch": b},
            "decode_ms_per_step": decode_ms / steps, "prefill_ms_incl_rotation_build": prefill_ms,
            "decode_attention_us_per_layer": attn_us,
            "decode_attention_hbm": {"achieved": attn_bytes / (attn_us * 1e-6) / 1e9, "peak": peak,
                                     "unit": "GB/s", "frac": attn_bytes / (attn_us * 1e-6) / 1e9 / peak,
                                     "algorithmic_bytes_per_layer": attn_bytes, "peak_source": peak_kind},
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
        del g, logits
        model.cache = None
        torch.cuda.empty_cache()
    return 0


# ---------------------------------------------------------------- config 5: multi-GPU decode
DEC72_METRIC = "config5 decode step us/step (80 layers, B=64, 64/8 heads, 32k ctx, 25% K channels kept)"
CFG5 = dict(layers=80, batch=64, q_heads=64, kv_heads=8, head_dim=128, keep=32, prompt=64, vision=31744,
            text=960)
DEC72_WORKLOAD = ("config5: 72B-class GQA decode attention, bf16, 80 layers, B=64, H_q=64, H_kv=8 (G=8), "
                  "D=128, D_keep=32, S = 64 prompt + 31744 visual + 960 text")


def config5_step(dev, pg, rank: int, world: int, steps: int, warmup: int, pool: int = 2,
                 mode: str = "heads", sm_reserve: int = 0) -> dict:
    """One config-5 decode step (all 80 layers, one new token for the batch of
    64) on this rank's share.  N = 1: the whole step on one GPU.  N > 1: KV heads
    sharded (8 / N per rank, their query groups for the whole batch); every
    layer's decode writes its heads head-major straight into that layer's
    all_gather send buffer, and one NCCL all_gather (issued asynchronously, so
    it runs beside the next layer's decode) leaves every rank with all 64
    heads.  Device time per step (CUDA events, max over ranks), also without
    the gathers, to show what the collective costs."""
    from rotatek_b200 import _lib, sharding, synthetic as syn
    from rotatek_b200.kernels import rotatek_decode
    G = CFG5["q_heads"] // CFG5["kv_heads"]
    p = sharding.plan(rank, world, CFG5["batch"], CFG5["kv_heads"], G, mode=mode if world > 1 else "batch")
    gather = world > 1 and p.mode == "heads"
    full_len = CFG5["prompt"] + CFG5["text"]
    layers = []
    for j in range(pool):
        d = syn.make_decode(p.local_batch, p.local_q_heads, p.local_kv_heads, CFG5["vision"], full_len,
                            keep=CFG5["keep"], seed=500 + 10 * j + rank, device=dev, dtype=torch.bfloat16)
        kw = d.as_kwargs()
        kw.pop("q_full")
        layers.append(kw)
        layer_bytes = d.nbytes()
        del d
    B, Hl, D = p.local_batch, p.local_q_heads, CFG5["head_dim"]
    qs = [syn.normal((B, Hl, D), 900 + l, dev, torch.bfloat16) for l in range(CFG5["layers"])]
    # send [H_loc, B, D] per layer (the decode's output, head-major); recv [H_q, B, D]
    send = [torch.empty((Hl, B, D), dtype=torch.bfloat16, device=dev) for _ in range(CFG5["layers"])]
    outs = [t.permute(1, 0, 2).unsqueeze(1) for t in send]          # [B, 1, H_loc, D] views
    recv = [torch.empty((world * Hl, B, D), dtype=torch.bfloat16, device=dev) for _ in range(CFG5["layers"])]
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()

    def step(with_gather: bool):
        works = []
        for l in range(CFG5["layers"]):
            rotatek_decode(q_full=qs[l], **layers[l % pool], out=outs[l])
            if with_gather:
                works.append(pg.all_gather_into_tensor(recv[l], send[l], async_op=True))
        for w in works:
            w.wait()

    def timed(gather: bool) -> float:
        for _ in range(max(warmup, 3)):
            step(gather)
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        lead_in()
        e0.record(stream)
        for _ in range(steps):
            step(gather)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        if pg is not None:
            t = torch.tensor([ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    _lib.set_decode_sm_reserve(sm_reserve if gather else 0)
    decode_only = timed(False)
    with_gather = timed(True) if gather else decode_only
    _lib.set_decode_sm_reserve(0)
    ok = True
    if gather:
        # the gathered heads are every rank's own outputs, in rank order
        mine = recv[-1][rank * Hl:(rank + 1) * Hl]
        ok = bool(torch.equal(mine, send[-1]))
    if world > 1:
        t = torch.tensor([float(ok)], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MIN)
        ok = bool(t.item() > 0)
    peak, peak_kind = load_peak_hbm()
    rank_bytes = layer_bytes * CFG5["layers"]
    plan = ("whole batch on one GPU" if world == 1 else
            f"KV heads {p.h0}..{p.h1 - 1} per rank, NCCL all_gather of the outputs per layer" if gather else
            f"batch rows {p.b0}..{p.b1 - 1} per rank (no collective)")
    out = {"what": DEC72_WORKLOAD, "plan": plan, "decode_sm_reserve": sm_reserve if gather else 0,
           "ms_per_step": with_gather, "decode_only_ms_per_step": decode_only,
           "tokens_per_s": CFG5["batch"] / (with_gather * 1e-3), "steps": steps, "layers_resident": pool,
           "hbm_rank": {"achieved": rank_bytes / (with_gather * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": rank_bytes / (with_gather * 1e-3) / 1e9 / peak, "bytes_per_rank_step": rank_bytes,
                        "peak_source": peak_kind},
           "gather_ok": ok}
    del layers, qs, send, outs, recv
    torch.cuda.empty_cache()
    return out


def strong_config2(dev, pg, rank: int, world: int, steps: int) -> dict:
    """Config 2's global batch of 32 split over the ranks (32 / N rows each, no
    collective): device time per global step, max over ranks.  Each rank cycles
    over enough input copies that a step's inputs are not left in L2 by the
    previous steps (>= 3 x 126 MB per rank)."""
    from rotatek_b200.kernels import rotatek_decode
    if CFG["batch"] % world:
        return {"unavailable": f"batch {CFG['batch']} does not split over {world} ranks"}
    b = CFG["batch"] // world
    d1 = make_inputs(dev, seed=2000 + rank, batch=b)
    per_rank = algorithmic_bytes(d1)
    del d1
    sets = max(1, math.ceil(3 * 126e6 / per_rank))
    d = make_inputs(dev, seed=2000 + rank, batch=b * sets)
    kw = d.as_kwargs()
    views = [{k: (v[i * b:(i + 1) * b] if torch.is_tensor(v) else v) for k, v in kw.items()} for i in range(sets)]
    for _ in range(5):
        for v in views:
            rotatek_decode(**v)
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lead_in()
    e0.record(stream)
    for i in range(steps):
        rotatek_decode(**views[i % sets])
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    mine = us
    if pg is not None:
        t = torch.tensor([us], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        us = float(t.item())
    peak, _ = load_peak_hbm()
    del d, kw, views
    torch.cuda.empty_cache()
    return {"what": f"config 2, global batch {CFG['batch']} split {b} rows per rank (strong scaling, no collective)",
            "us_per_step": us, "rows_per_rank": b, "input_sets_cycled": sets, "steps": steps,
            "hbm_frac_rank0": per_rank / (mine * 1e-6) / 1e9 / peak}


def run_decode72b(args):
    """Config 5 on its own line: one step = the decode attention of all 80 layers
    for one new token of the whole batch (strong scaling: the batch is fixed,
    ranks split it), KV heads sharded (``--shard heads``, NCCL all_gather of the
    outputs per layer) or batch rows (``--shard batch``, no collective)."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist
    mode = args.shard if args.shard != "auto" else "heads"
    sampler = ClockSampler(local)
    with sampler:
        r = config5_step(dev, pg, rank, world, args.steps, args.warmup, pool=args.pool, mode=mode,
                         sm_reserve=args.sm_reserve)
    clocks = sampler.summary()
    from rotatek_b200 import _lib
    status = _lib.read_status(dev)
    if rank == 0:
        line = {"metric": DEC72_METRIC, "value": r["ms_per_step"] * 1e3, "unit": "us/step", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": r["ms_per_step"],
                "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic: seeded low-rank+noise Keys rotated to a top-32 basis; N(0,1) Values/queries",
                "config": {"workload": DEC72_WORKLOAD, "global_batch": CFG5["batch"],
                           "seq_len": CFG5["prompt"] + CFG5["vision"] + CFG5["text"], "parallelism": r["plan"],
                           "layers_resident": r["layers_resident"],
                           "l2": "each layer's K/V per rank > 126 MB L2; no flush"},
                "detail": r, "clocks": clocks, "device_status": status,
                "gpu_launches": CFG5["layers"] * args.steps * (2 if world > 1 and mode == "heads" else 1)}
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 2000 decode steps, 20 build steps)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode workload: skip the same-box reference kernels, config 4 build, config-2 strong "
                         "scaling and config 5 measurements that ride along the headline line")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the batch (profiling cases only; the bench line uses 32)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="decode launches only: no e2e, no CPU baseline, no JSON bench line")
    ap.add_argument("--workload", choices=["decode", "build", "decode72b", "decode_step", "e2e", "think", "kproj",
                                           "decode_fp8", "spark"],
                    default="decode",
                    help="decode: benchmark config 2 (the headline); build: config 4 rotation build; "
                         "decode72b: config 5 multi-GPU decode; decode_step: config 2 with cache appends; "
                         "e2e: config 3 LLaVA-NeXT-7B-shaped end-to-end decode; think: ThinK at config 2; "
                         "kproj: one config-4 layer from hidden states (fused Key projection + build); "
                         "decode_fp8: config 2 with the visual span in e4m3; spark: SparK at config 2")
    ap.add_argument("--shard", choices=["auto", "heads", "batch"], default="auto",
                    help="decode72b: KV-head or batch sharding (auto: heads when N = 8)")
    ap.add_argument("--pool", type=int, default=2, help="decode72b: resident layers cycled over the 80")
    ap.add_argument("--sm-reserve", type=int, default=8,
                    help="config 5 with heads sharded: SMs the decode leaves to the concurrent all_gather")
    ap.add_argument("--e2e-tokens", type=int, default=128, help="e2e: greedy tokens per sequence")
    ap.add_argument("--kproj-vision", type=int, default=None,
                    help="kproj workload: visual tokens (profiling cases only; the bench line uses 15360)")
    ap.add_argument("--layers", type=int, default=None,
                    help="build workload: layers per step (profiling cases only; the bench line uses 28)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"build": 20, "decode72b": 10, "decode_step": 200, "think": 200,
                      "kproj": 20, "decode_fp8": 1000, "spark": 1000}.get(args.workload, 2000)
    if args.workload == "decode_step":
        return run_decode_step(args)
    if args.workload == "e2e":
        return run_e2e(args)
    if args.workload == "think":
        return run_think(args)
    if args.workload == "decode_fp8":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "metric": FP8_METRIC,
                              "unavailable": "fp8 storage is this build's extension; the reference keeps the "
                                             "visual span in the model dtype"}), flush=True)
            return 0
        return run_decode_fp8(args)
    if args.workload == "spark":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "metric": SPARK_METRIC,
                              "unavailable": "measured for this build only; its line carries the adapter "
                                             "path (recovery + concatenation + dense decode) timed beside it"}),
                  flush=True)
            return 0
        return run_spark(args)
    if args.workload == "kproj":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "metric": KPROJ_METRIC,
                              "unavailable": "measured for this build only; its line carries the adapter "
                                             "path (cuBLAS k_proj + torch RoPE + build) timed beside it"}),
                  flush=True)
            return 0
        return run_kproj(args)
    if args.workload == "decode72b":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "metric": DEC72_METRIC,
                              "unavailable": "config 5 is measured for this build only; the reference "
                                             "CPU arm covers configs 2 and 4"}), flush=True)
            return 0
        return run_decode72b(args)
    if args.workload == "build":
        return run_build_reference(args) if args.impl == "reference" else run_build(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
