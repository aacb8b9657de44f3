"""Benchmark of the AVQ-attention forward on B200.

Headline workload (the driver's line): the prefill configuration -- B=4,
Tq=S=8192, 32 heads x d=128 (E=4096), 512 parents x 4 children, budget 32,
single pass, bf16, Gaussian-mixture keys (512 centres, sigma 0.3), q/v ~
N(0,1), seed 1; codebook initialised from the keys with the fixed key-based
recipe (``avqa_b200.codebook.codebook_from_keys``).  Inputs are synthetic.

A step is one ``AVQAttention.forward`` of that batch through the public API:
quantize all S keys of every (b,h), parent attention, global budget routing,
child correction, fp32 output.  The inputs (0.8 GB) exceed the 126 MB L2,
so no flush is needed between steps.  After the timed region one (b,h)
slice of the last output is checked against the oracle.

Multi-GPU (torchrun, one rank per GPU): weak scaling -- every rank processes
its own batch of 4 (its shard of one global batch: the same key mixture,
independent samples); the ranks form one global batch, so the routing budget
min(P, min over all (b,h) of non-empty parents) is an all-reduce(MIN) over
NCCL each step (on a side stream, overlapping parent attention), exactly as
one reference call over the concatenated batch would compute it.

The other configurations are measured in the same run and reported under
``configs`` (each with its own step time, tokens/s, roofline and kernel
shares): the README fp32 example (latency), decode over a paged KV cache,
multi-pass refinement with the HVAQ temperature (fp16), and the long-context
chunked attention -- the last three head-sharded over the ranks with one
NCCL all-gather of the output (strong scaling) -- and, under ``fx``, the
rows beside the hot path at the headline's shapes with one batch entry: a
causal forward, a BCAR codebook update, the dense attention path and a
streaming-VQ token stream.

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/, numpy with all host threads) on a bounded sample (one (b,h) slice
of the headline workload per step) and reports the same metric.
"""
from __future__ import annotations

import argparse
import contextlib
import gc
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "query tokens/s/GPU at 1/2/4/8 B200; % of HBM/tensor roofline per kernel"
UNIT = "query tokens/s"
SUB_DEFAULT = "c1,c3,c4,c5,fx"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2")
    ap.add_argument("--configs", default=SUB_DEFAULT,
                    help="comma-separated sub-records measured after the headline ('none' for none)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the oracle check of one output slice")
    ap.add_argument("--cpu-slices", type=int, default=1,
                    help="(b,h) slices in the CPU-baseline sample; 0 skips the baseline (profiling runs)")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the per-GPU batch B (smaller cases for profiler captures)")
    ap.add_argument("--sub-batch", type=int, default=0,
                    help="override the batch of the c3 / c4 records (smaller cases for profiler captures)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class _NvmlPoller(threading.Thread):
    """Read-only NVML reads of the SM clock, its maximum, power and the clock
    event reasons every 5 ms, so that a timed region shorter than the
    nvidia-smi interval still holds samples.  Rows have the nvidia-smi
    sampler's shape; without NVML (no driver) it records nothing."""

    REASONS = ("nvmlClocksEventReasonHwSlowdown", "nvmlClocksEventReasonHwThermalSlowdown",
               "nvmlClocksEventReasonSwThermalSlowdown", "nvmlClocksEventReasonSwPowerCap")

    def __init__(self, gpu_uuid: str, period: float = 0.005):
        super().__init__(daemon=True)
        self.gpu, self.period, self.rows = gpu_uuid, period, []
        self.stop_evt = threading.Event()

    def run(self) -> None:
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self.gpu)
            sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            masks = [getattr(pynvml, n) for n in self.REASONS]
        except Exception:
            return
        try:
            while not self.stop_evt.is_set():
                try:
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    flags = ["Active" if rs & m else "Not Active" for m in masks]
                    self.rows.append((time.time(), sm, sm_max, pw, flags))
                except Exception:
                    return
                self.stop_evt.wait(self.period)
        finally:
            try:
                pynvml.nvmlShutdown()
            except Exception:
                pass


def gpu_uuid(dev) -> str | None:
    """NVML/nvidia-smi id (``GPU-<uuid>``) of the torch device ``dev``.

    NVML and nvidia-smi number GPUs physically and ignore
    CUDA_VISIBLE_DEVICES, so the sampler addresses the GPU by its UUID."""
    try:
        import torch
        u = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return None
    return u if u.startswith("GPU-") else f"GPU-{u}"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 50 ms with host
    timestamps, joined by NVML reads every 5 ms, both for the GPU with the
    given UUID.  ``summary(t0, t1)`` uses the samples inside a window, and
    widens to the whole sampling span before it only when the window held
    fewer than three samples."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, uuid: str | None):
        self.gpu = uuid
        self.proc = None
        self.path = None
        self.t_open = None
        self.nvml = _NvmlPoller(uuid) if uuid else None

    def __enter__(self):
        if self.gpu is None:
            return self
        self.nvml.start()
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        try:
            with os.fdopen(fd, "w") as f:
                self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                              "--format=csv,noheader,nounits", "-lms", "50"], stdout=f,
                                             stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        deadline = time.time() + 10.0  # wait for the first sample so the window is covered
        while time.time() < deadline and self.proc.poll() is None and os.path.getsize(self.path) == 0:
            time.sleep(0.02)
        self.t_open = time.time()
        return self

    def __exit__(self, *exc):
        if self.nvml is not None:
            self.nvml.stop_evt.set()
            self.nvml.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def _rows(self) -> list:
        from datetime import datetime
        rows = list(self.nvml.rows) if self.nvml is not None else []
        if self.path and os.path.exists(self.path):
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    rows.append((ts, float(parts[2]), float(parts[3]), float(parts[4]), parts[6:10]))
                except ValueError:
                    continue
        return rows

    def summary(self, t0: float, t1: float) -> dict:
        rows = self._rows()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "gpu": self.gpu, "reasons": ["no clock samples"]}
        window = "timed"
        sel = [r for r in rows if t0 <= r[0] <= t1]
        if len(sel) < 3:
            window = "warmup+timed"
            sel = [r for r in rows if (self.t_open or 0) <= r[0] <= t1]
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "gpu": self.gpu, "reasons": ["no samples"]}
        reasons = sorted({self.NAMES[i] for *_, flags in sel for i, f in enumerate(flags) if f.lower() == "active"})
        load = sorted(r[1] for r in sel)
        return {"sm_mhz": load[len(load) // 2], "sm_max_mhz": sel[0][2], "power_w_max": max(r[3] for r in sel),
                "samples": len(sel), "window": window, "gpu": self.gpu, "reasons": reasons}

    def close(self) -> None:
        if self.path and os.path.exists(self.path):
            os.unlink(self.path)


# ---------------------------------------------------------------------------
# roofline bookkeeping (algorithmic work per launch)
# ---------------------------------------------------------------------------
def algorithmic_work(w, B: int, T: int | None = None, decode: bool = False, sel_total: int | None = None) -> dict:
    """FLOPs (tensor-bound kernels) or bytes (memory-bound kernels) per launch.

    ``T`` overrides the queries per (b,h) of one launch; ``sel_total`` is the
    sum of the refinement passes' budgets (default P).  Decode steps (T=1) are
    bound by HBM: their kernels count the bytes each must move once."""
    T = w.T if T is None else T
    G, S, D, M0, C, P = B * w.H, w.S, w.D, w.M0, w.C, w.P
    es = 2 if w.dtype in ("bf16", "f16") else 4
    nsel = P if sel_total is None else sel_total
    if decode:
        pagg = G * M0 * D * es + G * M0 * 4                    # parent sums + counts
        sel = G * nsel * (1 + C) * D * es + G * nsel * C * 4   # selected parent / child sums + child counts
        return {
            "parent_attn_tc": ("hbm", pagg), "parent_attn": ("hbm", pagg), "parent_attn_exact": ("hbm", pagg),
            # every parent-sum row, the selected rows, the exponentials (fp32) and the output
            "decode_value": ("hbm", pagg + sel + G * M0 * 4 + G * T * D * 4),
            # the logits read, the exponentials and the importance written, the counts
            "decode_route": ("hbm", G * M0 * (es + 4 + 4)),
            "decode_logits": ("tensor", 2.0 * G * T * M0 * D),
            "append_assign": ("tensor", 2.0 * G * T * M0 * D),
            "correct_tc": ("hbm", sel), "correct": ("hbm", sel), "correct_exact": ("hbm", sel),
            # new token k/v read, the fp32 sums of its parent and child rows
            # (read + write) and their dtype copies written, the page slots
            "append": ("hbm", G * T * (2 * D * es + 2 * 2 * D * 4 + 2 * D * es + 2 * D * es)),
            "route": ("hbm", G * M0 * 8),
        }
    return {
        "parent_attn": ("tensor", 4.0 * G * T * M0 * D),          # q.P^T and e @ V (mma.sync kernel)
        "parent_attn_tc": ("tensor", 4.0 * G * T * M0 * D),       # the same on tcgen05
        "parent_attn_hvaq": ("tensor", 4.0 * G * T * M0 * D),     # HVAQ rescaled pass
        "parent_attn_exact": ("tensor", 4.0 * G * T * M0 * D),
        "assign": ("tensor", 2.0 * G * S * M0 * D + 2.0 * G * S * C * D),
        "assign_exact": ("tensor", 2.0 * G * S * M0 * D + 2.0 * G * S * C * D),  # fp32 path
        "assign_tc": ("tensor", 2.0 * G * S * M0 * D),            # the parent pass; children in "child"
        # child stage in parent order: each key row, its order / parent /
        # cassign words, every parent's child rows and norms once
        "child": ("hbm", G * S * D * es + G * S * 16 + G * M0 * C * (D * es + 4)),
        "correct": ("tensor", 2.0 * G * T * nsel * D * (2 + 2 * C)),  # parent+child logits, value sums
        "correct_tc": ("tensor", 2.0 * G * T * nsel * D * (2 + 2 * C)),
        "correct_exact": ("tensor", 2.0 * G * T * nsel * D * (2 + 2 * C)),
        "aggregate": ("hbm", G * S * D * es + G * S * 8 + G * M0 * (1 + C) * D * es + G * M0 * (1 + C) * 4),
        "bucket_sort": ("hbm", G * S * 4 * 4),
        "route": ("hbm", G * M0 * 8),
    }


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic() -> dict:
    p = ROOT / "profiles" / "dram_traffic_per_launch.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except json.JSONDecodeError:
            return {}
    return {}


def kernel_table(prof: dict, work: dict, peaks: dict, peak_src: str, region_s: float) -> tuple[dict, dict | None]:
    """Per-kernel shares and roofline fractions, and the dominant kernel's
    roofline.  Tensor kernels divide by the burst bf16 peak when the timed
    region is short (under 2 s), by the sustained one otherwise."""
    sustained = region_s >= 2.0
    tpeak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) if sustained else peaks["bf16_tflops"]
    tlabel = "sustained" if sustained else "burst"
    total = sum(v[0] for v in prof.values()) or 1.0
    kernels = {}
    for name, (ms, n) in sorted(prof.items(), key=lambda x: -x[1][0]):
        entry = {"launches": n, "avg_ms": ms / n, "share": ms / total}
        if name in work:
            bound, amount = work[name]
            avg_s = ms / n / 1e3
            if bound == "tensor":
                a = amount / avg_s / 1e12
                entry.update(achieved_tflops=a, frac=a / tpeak)
            else:
                a = amount / avg_s / 1e9
                entry.update(achieved_gbs=a, frac=a / peaks["hbm_gbs"])
        kernels[name] = entry
    kern = {k: v for k, v in prof.items() if k in work}
    if not kern:
        return kernels, None
    dom = max(kern, key=lambda k: kern[k][0])
    bound, amount = work[dom]
    avg_s = kern[dom][0] / kern[dom][1] / 1e3
    if bound == "tensor":
        achieved, peak, unit = amount / avg_s / 1e12, tpeak, "TFLOP/s"
        src = f"{peak_src} bf16 tensor peak ({tlabel}: timed region {region_s:.3f} s)"
    else:
        achieved, peak, unit = amount / avg_s / 1e9, peaks["hbm_gbs"], "GB/s"
        src = f"{peak_src} HBM copy bandwidth"
    roof = {"kernel": dom, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": None, "peak_source": src, "algorithmic_per_launch": amount, "avg_launch_ms": avg_s * 1e3}
    return kernels, roof


# ---------------------------------------------------------------------------
# CPU baseline (oracle port)
# ---------------------------------------------------------------------------
def _cores() -> int:
    cores = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:
        pass
    return cores


def _all_threads() -> None:
    """All host threads for the numpy port (torchrun sets OMP_NUM_THREADS=1)."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(os.cpu_count())
    except Exception:
        pass


def cpu_baseline(w, slices: int = 1) -> dict:
    """Time the numpy restatement of the reference on ``slices`` (b,h) slices."""
    import torch

    from avqa_b200.codebook import codebook_from_keys
    from avqa_b200.workloads import make_inputs
    from oracle import avq_oracle as O
    _all_threads()
    q, k, v = make_inputs(w, B=1)
    H, D = w.H, w.D
    total = 0.0
    for hh in range(slices):
        sl = lambda x, n: O.rnd(x.view(1, n, H, D)[:, :, hh].reshape(1, n, D).numpy(), w.dtype)
        qn, kn, vn = sl(q, w.T), sl(k, w.S), sl(v, w.S)
        cb = codebook_from_keys(torch.from_numpy(kn), w.M0, w.C, w.seed)
        pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), w.dtype)
        cfg = O.ForwardConfig(1, w.M0, w.C, w.P, w.dtype, w.passes, w.pass_decay, w.hvaq)
        t0 = time.perf_counter()
        O.forward_heads(qn, kn, vn, pd, cd, cfg)
        total += time.perf_counter() - t0
    # one slice serves T queries of one head: 1/H of T query tokens
    tokens = slices * w.T / H
    return {"value": tokens / total, "unit": "query tokens/s", "cores": _cores(), "kind": "port",
            "seconds": total,
            "sample": f"{slices} (b,h) slice(s) of the workload (T=S={w.T}, M0={w.M0}, C={w.C}, P={w.P}, "
                      f"{w.dtype}), oracle/avq_oracle.py numpy restatement, {total:.2f} s; a slice is 1/{H} of "
                      f"{w.T} query tokens, so the whole-batch figure is extrapolated from the sample"}


# ---------------------------------------------------------------------------
def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args) -> None:
    """The CPU implementation of the path on the host cores: each step is one
    (b,h) slice of the headline workload through the oracle port (the
    reference is pure Python and cannot run on the GPU box), all threads."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    _all_threads()
    from avqa_b200.workloads import WORKLOADS
    w = WORKLOADS[args.workload]
    times = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(w, slices=args.cpu_slices)
        if i >= args.warmup:
            times.append(cb)
    secs = [c["seconds"] for c in times]
    value = sum(c["value"] for c in times) / len(times)
    sample_ms = 1e3 * sum(secs) / len(secs)
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "query tokens/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": sample_ms,
           "ms_per_step_note": f"one step = {args.cpu_slices} (b,h) slice(s) of the workload, the bounded sample; "
                               f"a whole-batch step ({w.B * w.H} slices) extrapolates to "
                               f"{sample_ms * w.B * w.H / args.cpu_slices / 1e3:.1f} s",
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
           "config": workload_config(w, world),
           "cpu_baseline": {k: times[-1][k] for k in ("kind", "cores", "sample")} | {"value": value,
                                                                                     "unit": "query tokens/s"},
           "e2e": {"value": value, "unit": "query tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def workload_config(w, world: int) -> dict:
    return {"workload": f"{w.name}: prefill B={w.B}/GPU Tq=S={w.T} H={w.H} D={w.D} M0={w.M0} C={w.C} P={w.P} "
                        f"{w.dtype} {w.keys} keys",
            "global_batch": w.B * world, "seq_len": w.T, "parallelism": f"batch-sharded x{world}, global budget "
                                                                        f"all-reduce(MIN)",
            "l2": "inputs (0.8 GB/GPU) exceed L2; no flush"}


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
class Ctx:
    """Per-process benchmark context (device, ranks, peaks)."""

    def __init__(self, world: int, rank: int, dev):
        import torch
        import torch.distributed as dist
        self.world, self.rank, self.dev = world, rank, dev
        self.sub_batch = 0  # batch override of the c3 / c4 records
        self.stream = torch.cuda.current_stream(dev)
        self.group = dist.group.WORLD if world > 1 else None
        self.peaks, self.peak_src = load_peaks()

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], device=self.dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, fn, steps: int, start: int = 0) -> tuple[float, list[float]]:
        """Run ``fn(i)`` for i in [start, start + steps) between CUDA events on
        the launching stream, with a barrier and a synchronize on both sides;
        returns (max over ranks of the total ms, this rank's per-step ms)."""
        import torch
        self.barrier()
        torch.cuda.synchronize(self.dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        with no_gc():
            ev[0].record(self.stream)
            for i in range(steps):
                fn(start + i)
                ev[i + 1].record(self.stream)
            torch.cuda.synchronize(self.dev)
        self.barrier()
        per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
        return self.max_over_ranks(ev[0].elapsed_time(ev[-1])), per


@contextlib.contextmanager
def no_gc():
    """Python's cyclic collector paused over a timed region (as ``timeit``
    does): a full collection stalls the host for tens of milliseconds, which
    a host-bound loop of short steps would count as device idle time."""
    gc.collect()
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()


def _median(xs: list[float]) -> float:
    s = sorted(xs)
    return s[len(s) // 2] if s else 0.0


def measure(ctx: Ctx, fn, warmup: int, steps: int, work: dict, tokens_per_step: float, clk=None,
            start: int = 0) -> dict:
    """Warm up, time ``steps`` steps with the library's per-kernel timing on,
    and summarise: ms/step (mean and median), tokens/s, kernels, roofline."""
    from avqa_b200 import _lib
    for i in range(warmup):
        fn(start + i)
    _lib.profile_begin()
    t0 = time.time()
    total_ms, per = ctx.timed(fn, steps, start + warmup)
    t1 = time.time()
    prof = _lib.profile_end()
    kernels, roof = kernel_table(prof, work, ctx.peaks, ctx.peak_src, total_ms / 1e3)
    rec = {"steps": steps, "warmup": warmup, "ms_per_step": total_ms / steps, "ms_per_step_median": _median(per),
           "ms_per_step_max": max(per) if per else 0.0, "value": tokens_per_step * steps / (total_ms / 1e3),
           # the same throughput from the median step: steady against a lone slow step of a
           # host-bound loop (the mean above keeps it)
           "value_median": tokens_per_step / (_median(per) / 1e3) if per and _median(per) > 0 else None,
           "unit": UNIT, "roofline": roof, "kernels": kernels,
           "gpu_launches": sum(n * (3 if k == "bucket_sort" else 1) for k, (_, n) in prof.items())}
    if clk is not None:
        rec["clocks"] = clk.summary(t0, t1)
    return rec


# ---------------------------------------------------------------------------
# oracle checks of one output slice (rank 0, after the timed region)
# ---------------------------------------------------------------------------
def check_slice(w, qg, kg, vg, out_g, parents32, children32, budget_floor: int, hh: int) -> dict:
    """Compare one (b,h) slice of a CUDA output with the oracle on the same
    inputs and codebook head; ``*_g`` are ``[1, n, D]`` CPU fp32 tensors
    holding dtype values, ``budget_floor`` the global minimum of non-empty
    parents the GPU used."""
    import numpy as np

    from oracle import avq_oracle as O
    _all_threads()
    pd, cd = O.cast_codebook(parents32[hh:hh + 1].numpy(), children32[hh:hh + 1].numpy(), w.dtype)
    cfg = O.ForwardConfig(1, w.M0, w.C, w.P, w.dtype, w.passes, w.pass_decay, w.hvaq)
    t0 = time.perf_counter()
    res = O.forward_heads(qg.numpy(), kg.numpy(), vg.numpy(), pd, cd, cfg, budget_floor=budget_floor)
    dt = time.perf_counter() - t0
    ref, got = res["out"].astype(np.float64), out_g.numpy().astype(np.float64)
    # the reference's own non-finite outputs (fp16 overflow) must sit in the same places
    bad_g, bad_r = ~np.isfinite(got), ~np.isfinite(ref)
    same_nonfinite = bool(np.array_equal(bad_g, bad_r))
    keep = ~(bad_g | bad_r)
    err = float(np.linalg.norm(got[keep] - ref[keep]) / max(np.linalg.norm(ref[keep]), 1e-30))
    tol = 2e-5 if w.dtype == "f32" else 1e-2
    return {"slice": f"b=0 h={hh}", "normwise_error": err, "tolerance": tol,
            "nonfinite_rows": int(bad_r.any(-1).sum()), "ok": bool(err <= tol and same_nonfinite),
            "oracle_s": round(dt, 2)}


# ---------------------------------------------------------------------------
# headline: c2 prefill, batch-sharded
# ---------------------------------------------------------------------------
def run_headline(args, ctx: Ctx, clk) -> dict:
    import torch

    from avqa_b200 import AVQAttention, AVQConfig
    from avqa_b200.codebook import codebook_from_keys
    from avqa_b200.config import AttentionShapeConfig, CodebookConfig, RefinementConfig, RoutingConfig
    from avqa_b200.workloads import TORCH_DTYPE, WORKLOADS, Workload, make_inputs

    dev, world, rank = ctx.dev, ctx.world, ctx.rank
    w: Workload = WORKLOADS[args.workload]
    if args.batch:
        w = Workload(**{**w.__dict__, "B": args.batch})
    dt = TORCH_DTYPE[w.dtype]
    H, D = w.H, w.D
    # codebook from batch 0 of the global batch (rank 0's seed), identical on every rank
    _, k0, _ = make_inputs(w, device=dev, B=1, T=1)
    cb = codebook_from_keys(k0.to(dt).view(1, w.S, H, D).transpose(1, 2)[0].float(), w.M0, w.C, w.seed)
    del k0
    # rank r holds batch shard r of one global batch: the same key mixture, its own samples
    q, k, v = make_inputs(w, device=dev, part=rank)
    q, k, v = q.to(dt), k.to(dt), v.to(dt)
    cfg = AVQConfig(attention=AttentionShapeConfig(embed_dim=w.E, num_heads=H),
                    codebook=CodebookConfig(num_codewords=w.M0, children_per_codeword=w.C),
                    routing=RoutingConfig(refinement_budget=w.P),
                    refinement=RefinementConfig(passes=w.passes, pass_decay=w.pass_decay))
    mod = AVQAttention(cfg, in_proj=False, out_proj=False)
    mod.codebook.parents, mod.codebook.children = cb.parents.to(dev), cb.children.to(dev)
    if world > 1:
        mod.process_group = ctx.group
    work = algorithmic_work(w, w.B)
    last = {}

    def step(i):
        last["out"] = mod(q, k, v)

    with torch.no_grad():
        rec = measure(ctx, step, args.warmup, args.steps, work, world * w.B * w.T, clk)
        traffic = load_traffic()
        if rec["roofline"]:
            rec["roofline"]["traffic"] = traffic.get(f"{args.workload}:{rec['roofline']['kernel']}")
        check = None
        if not args.no_check:
            # the budget floor the forward used: min over every (b,h) of every rank
            from avqa_b200 import ops
            from avqa_b200.attention_module import AVQAttention as M
            from avqa_b200.attention_module import global_min_valid
            cbp = mod.backend.prepared_codebook(mod.codebook.parents, mod.codebook.children, dt, dev)
            qs = ops.quantize(M.split_heads(k, H), M.split_heads(v, H), cbp)
            floor_t, _ = global_min_valid(qs, ctx.group)
            floor = int(floor_t.item())
            del qs, floor_t
            if rank == 0:
                hh = 1 % H
                sl = lambda x: x[:1, :, hh * D:(hh + 1) * D].float().cpu()
                check = check_slice(w, sl(q), sl(k), sl(v), sl(last["out"]), cb.parents.cpu(), cb.children.cpu(),
                                    floor, hh)
                check["budget_floor"] = floor
        e2e = None
        if not args.no_e2e:
            e2e = run_e2e(ctx, mod, q, k, v, w, args.steps)
    rec["check"] = check
    rec["e2e"] = e2e
    rec["w"] = w
    del q, k, v, mod, last
    torch.cuda.empty_cache()
    return rec


def run_e2e(ctx: Ctx, mod, q, k, v, w, steps: int) -> dict:
    """Through the public API with the copies inside the timed region: every
    step copies its q/k/v from pinned host memory and reads the fp32 output
    back.  Copies run on their own streams with two device buffer sets, so
    step i+1's H2D and step i-1's D2H overlap step i."""
    import torch
    dev, stream = ctx.dev, ctx.stream
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = [torch.empty(w.B, w.T, w.E, dtype=torch.float32).pin_memory() for _ in range(2)]
    dbuf = [[torch.empty(x.shape, dtype=x.dtype, device=dev) for x in (hq, hk, hv)] for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in, ev_comp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def e2e_step(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_comp[j])  # step i-2 no longer reads slot j
            for d, hx in zip(dbuf[j], (hq, hk, hv)):
                d.copy_(hx, non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        o = mod(*dbuf[j])
        ev_comp[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[j])
            if i >= 2:
                s_out.wait_event(ev_out[j])
            hout[j].copy_(o, non_blocking=True)
            ev_out[j].record(s_out)
        o.record_stream(s_out)

    def e2e_timed(n):
        ctx.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with no_gc():
            e0.record(stream)
            s_in.wait_event(e0)
            for i in range(n):
                e2e_step(i)
            stream.wait_stream(s_out)
            stream.wait_stream(s_in)
            e1.record(stream)
            torch.cuda.synchronize(dev)
        ctx.barrier()
        return ctx.max_over_ranks(e0.elapsed_time(e1))

    def copies_only(n):
        """The same copies with no compute: the host link's floor for a step."""
        ctx.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        o = torch.empty(hout[0].shape, dtype=hout[0].dtype, device=dev)
        with no_gc():
            e0.record(stream)
            s_in.wait_event(e0)
            s_out.wait_event(e0)
            for i in range(n):
                with torch.cuda.stream(s_in):
                    for d, hx in zip(dbuf[i % 2], (hq, hk, hv)):
                        d.copy_(hx, non_blocking=True)
                with torch.cuda.stream(s_out):
                    hout[i % 2].copy_(o, non_blocking=True)
            stream.wait_stream(s_out)
            stream.wait_stream(s_in)
            e1.record(stream)
            torch.cuda.synchronize(dev)
        ctx.barrier()
        return ctx.max_over_ranks(e0.elapsed_time(e1))

    e2e_timed(2)
    # steady state of a serving loop: enough steps that filling and draining
    # the three-stream pipeline (the first upload, the last download) weigh
    # little, about 0.3 s at the c2 shapes
    nb = max(16, steps)
    ms = e2e_timed(nb)
    link_ms = copies_only(nb)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
    d2h = hout[0].numel() * hout[0].element_size()
    return {"value": ctx.world * w.B * w.T * nb / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms / nb, "steps": nb,
            "host_copy_gbs_per_gpu": (h2d + d2h) / (ms / nb / 1e3) / 1e9,
            "copies_only_ms_per_step": link_ms / nb,
            "frac_of_copy_bound": link_ms / ms,
            "overlap": "H2D, compute and D2H on separate streams, two device buffer sets"}


# ---------------------------------------------------------------------------
# sub-records
# ---------------------------------------------------------------------------
def _sharded(ctx: Ctx, w, cb, dt):
    from avqa_b200.config import (AttentionShapeConfig, AVQConfig, BackendConfig, CodebookConfig, HopfieldConfig,
                                  RefinementConfig, RoutingConfig)
    from avqa_b200.parallel import ShardedAVQAttention
    cfg = AVQConfig(attention=AttentionShapeConfig(embed_dim=w.E, num_heads=w.H),
                    codebook=CodebookConfig(num_codewords=w.M0, children_per_codeword=w.C),
                    routing=RoutingConfig(refinement_budget=w.P),
                    refinement=RefinementConfig(passes=w.passes, pass_decay=w.pass_decay),
                    backend=BackendConfig(hopfield=w.hvaq),
                    hopfield=HopfieldConfig(enabled=w.hvaq, adaptive="entropy" if w.hvaq else "none"))
    return ShardedAVQAttention(cfg, cb.parents.to(ctx.dev), cb.children.to(ctx.dev), group=ctx.group,
                               device=ctx.dev, dtype=dt)


def _codebook(w, k_b0, dt):
    """Key-based codebook from batch 0's keys ``[1, S, E]`` (any device)."""
    from avqa_b200.codebook import codebook_from_keys
    H, D = w.H, w.D
    return codebook_from_keys(k_b0.to(dt).view(1, -1, H, D).transpose(1, 2)[0].float(), w.M0, w.C, w.seed)


def sub_c1(ctx: Ctx, clk) -> dict:
    """README fp32 example: latency of one forward (replicated on each rank)."""
    import torch

    from avqa_b200 import AVQAttention, AVQConfig
    from avqa_b200.config import AttentionShapeConfig, CodebookConfig, RoutingConfig
    from avqa_b200.workloads import WORKLOADS, make_inputs
    from oracle import avq_oracle as O
    w = WORKLOADS["c1"]
    q, k, v = make_inputs(w)  # torch.manual_seed(0) draws, README order
    cb = _codebook(w, k[:1], torch.float32)
    cfg = AVQConfig(attention=AttentionShapeConfig(embed_dim=w.E, num_heads=w.H),
                    codebook=CodebookConfig(num_codewords=w.M0, children_per_codeword=w.C),
                    routing=RoutingConfig(strategy="budget", refinement_budget=w.P))
    mod = AVQAttention(cfg, in_proj=False, out_proj=False)
    mod.codebook.parents, mod.codebook.children = cb.parents.to(ctx.dev), cb.children.to(ctx.dev)
    qd, kd, vd = (x.to(ctx.dev) for x in (q, k, v))
    last = {}

    def step(i):
        last["o"] = mod(qd, kd, vd)

    with torch.no_grad():
        rec = measure(ctx, step, 20, 100, algorithmic_work(w, w.B), w.B * w.T, clk)
    rec["value_scope"] = "one GPU's rate (every GPU runs its own replica)"
    pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), "f32")
    _all_threads()
    t0 = time.perf_counter()
    res = O.forward(q.numpy(), k.numpy(), v.numpy(), pd, cd, O.ForwardConfig(w.H, w.M0, w.C, w.P, "f32"))
    cpu_s = time.perf_counter() - t0
    import numpy as np
    got = last["o"].cpu().numpy()
    err = float(np.linalg.norm(got - res["out_bte"]) / np.linalg.norm(res["out_bte"]))
    rec.update(workload="c1: README example B=2 Tq=64 S=128 E=512 H=8 D=64 M0=64 C=4 P=8 fp32",
               parallelism="replicated (one forward per GPU)", latency_ms=rec["ms_per_step_median"],
               check={"normwise_error": err, "tolerance": 2e-5, "ok": bool(err <= 2e-5)},
               cpu_baseline={"value": w.B * w.T / cpu_s, "unit": "query tokens/s", "cores": _cores(), "kind": "port",
                             "sample": f"the whole forward, oracle/avq_oracle.py, {cpu_s * 1e3:.1f} ms"})
    return rec


def sub_c4(ctx: Ctx, clk) -> dict:
    """Multi-pass refinement (3 passes, budgets 48/24/12) + HVAQ entropy, fp16,
    head-sharded over the ranks."""
    import torch

    from avqa_b200.workloads import TORCH_DTYPE, WORKLOADS, Workload, make_inputs
    w = WORKLOADS["c4"]
    if ctx.sub_batch:
        w = Workload(**{**w.__dict__, "B": ctx.sub_batch})
    dt = TORCH_DTYPE[w.dtype]
    q, k, v = make_inputs(w, device=ctx.dev)
    cb = _codebook(w, k[:1], dt)
    q, k, v = q.to(dt), k.to(dt), v.to(dt)
    mod = _sharded(ctx, w, cb, dt)
    hloc = mod.h1 - mod.h0
    from types import SimpleNamespace
    wl = SimpleNamespace(**{**w.__dict__, "H": hloc})
    work = algorithmic_work(wl, w.B, sel_total=48 + 24 + 12)
    last = {}

    def step(i):
        last["o"] = mod(q, k, v)

    with torch.no_grad():
        rec = measure(ctx, step, 3, 10, work, w.B * w.T, clk)
    rec.update(workload=f"c4: B={w.B} Tq=S=16384 H=16 D=64 M0=256 C=4 fp16, 3 passes (48/24/12), HVAQ entropy, "
                        "Student-t keys", parallelism=f"head-sharded x{ctx.world} ({hloc} heads/GPU), output "
                                                      f"all-gather")
    if ctx.rank == 0:
        if ctx.world == 1:  # one slice of the output against the oracle, with the floor of all 16 heads
            from avqa_b200 import ops
            from avqa_b200.attention_module import AVQAttention as M
            st = ops.quantize(M.split_heads(k, w.H), M.split_heads(v, w.H), mod.compute.cb)
            floor = int(st.gmin.item())
            del st
            sl = lambda x: x[:1, :, 0:w.D].float().cpu()
            rec["check"] = check_slice(w, sl(q), sl(k), sl(v), sl(last["o"]), cb.parents.cpu(), cb.children.cpu(),
                                       floor, 0)
        rec["cpu_baseline"] = cpu_baseline(w, 1)
    del q, k, v, mod, last
    torch.cuda.empty_cache()
    return rec


def sub_c5(ctx: Ctx, clk) -> dict:
    """Long context: S=131072 keys quantized once, 2048 queries in eight
    256-query chunks (each routed on its own), 64 heads sharded over the
    ranks, one output all-gather per step."""
    import torch

    from avqa_b200.workloads import TORCH_DTYPE, WORKLOADS, make_inputs
    w = WORKLOADS["c5"]
    dt = TORCH_DTYPE[w.dtype]
    q, k, v = make_inputs(w, device=ctx.dev)
    q, k, v = q.to(dt), k.to(dt), v.to(dt)
    cb = _codebook(w, k[:1], dt)
    mod = _sharded(ctx, w, cb, dt)
    hloc = mod.h1 - mod.h0
    from types import SimpleNamespace
    wl = SimpleNamespace(**{**w.__dict__, "H": hloc})
    work = algorithmic_work(wl, 8, T=w.q_chunk)  # one forward launch carries the eight chunks as a batch
    work.update({k2: v2 for k2, v2 in algorithmic_work(wl, 1).items() if k2 in ("assign", "assign_tc", "aggregate",
                                                                               "bucket_sort")})
    last = {}

    def step(i):
        last["o"] = mod(q, k, v, chunk_size=w.q_chunk)

    with torch.no_grad():
        rec = measure(ctx, step, 3, 5, work, w.T, clk)
    rec.update(workload="c5: B=1 S=131072 Tq=2048 in 256-query chunks, H=64 D=128 M0=4096 C=8 P=128 bf16, "
                        "RoPE mixture keys; a step quantizes the keys once and attends all eight chunks",
               parallelism=f"head-sharded x{ctx.world} ({hloc} heads/GPU), output all-gather")
    rec["check_note"] = "the oracle check of a c5 slice runs in the -m gpu parity tests (the port's " \
                        "quantization of 131072 keys is ~70 GFLOP of float64)"
    rec["cpu_baseline"] = None
    del q, k, v, mod, last
    torch.cuda.empty_cache()
    return rec


def sub_c3(ctx: Ctx, clk) -> dict:
    """Decode over a paged KV cache: a 32768-token prior in 256-token pages,
    then 128 steps that each append one token per (b,h) and attend to the
    whole cache.  Heads are sharded over the ranks (B=64 on every rank)."""
    import torch

    from avqa_b200 import PagedKVCache
    from avqa_b200.workloads import TORCH_DTYPE, WORKLOADS, Workload, make_decode_tokens, make_inputs
    w = WORKLOADS["c3"]
    if ctx.sub_batch:
        w = Workload(**{**w.__dict__, "B": ctx.sub_batch})
    dt = TORCH_DTYPE[w.dtype]
    dev = ctx.dev
    # the prior, batch by batch (the same cluster centres, each batch its own samples)
    kp = torch.empty(w.B, w.S, w.E, dtype=dt, device=dev)
    vp = torch.empty(w.B, w.S, w.E, dtype=dt, device=dev)
    for b in range(w.B):
        _, kb, vb = make_inputs(w, device=dev, B=1, T=1, part=b)
        kp[b].copy_(kb[0])
        vp[b].copy_(vb[0])
        del kb, vb
    cb = _codebook(w, kp[:1], dt)
    mod = _sharded(ctx, w, cb, dt)
    hloc = mod.h1 - mod.h0
    cache = PagedKVCache(page_size=w.page_size, num_heads=hloc, head_dim_k=w.D, head_dim_v=w.D, device=dev, dtype=dt)
    toks = [tuple(x.to(dev, dt) for x in t) for t in make_decode_tokens(w, w.decode_steps)]
    with torch.no_grad():
        # prefill: the prior enters the cache and is quantized once (its query is discarded)
        mod(toks[0][0], kp, vp, kv_cache=cache)
        del kp, vp
        torch.cuda.empty_cache()
        from types import SimpleNamespace
        wl = SimpleNamespace(**{**w.__dict__, "H": hloc})
        work = algorithmic_work(wl, w.B, T=1, decode=True)

        def step(i):
            qt, kt, vt = toks[i]
            mod(qt, kt, vt, kv_cache=cache)

        warm = 3
        rec = measure(ctx, step, warm, w.decode_steps - warm, work, w.B, clk)
    rec.update(workload=f"c3: decode B={w.B} H=32 D=128 bf16, prior S=32768 in 256-token pages, M0=1024 C=8 P=64; "
                        f"{w.decode_steps} steps of one token per (b,h): {warm} warm-up, "
                        f"{w.decode_steps - warm} timed", parallelism=f"head-sharded x{ctx.world} ({hloc} heads/GPU), "
                                                                      f"output all-gather",
               cache_tokens_after=cache.size)
    rec["cpu_baseline"] = None
    del cache, mod, toks
    torch.cuda.empty_cache()
    return rec


def sub_fx(ctx: Ctx, clk) -> dict:
    """The rows beside the hot path at the c2 shapes (B=1 per GPU, replicated):
    a causal forward (mask bits + the masked kernel variants), one BCAR
    codebook update after a quantization, the dense attention path, and a
    streaming-VQ token stream (one key per extend call)."""
    import torch

    from avqa_b200 import AVQAttention, AVQConfig, StreamingVQBuffer, ops
    from avqa_b200.backend import CUDABackend
    from avqa_b200.config import AttentionShapeConfig, CodebookConfig, RoutingConfig
    from avqa_b200.workloads import TORCH_DTYPE, WORKLOADS, Workload, make_inputs
    w = Workload(**{**WORKLOADS["c2"].__dict__, "B": 1})
    dt, dev = TORCH_DTYPE[w.dtype], ctx.dev
    G, H, T, S, D, M0, C = w.H, w.H, w.T, w.S, w.D, w.M0, w.C
    es = 2
    q, k, v = (x.to(dt) for x in make_inputs(w, device=dev))
    cb = _codebook(w, k, dt)
    heads = lambda x: x.view(1, -1, H, D).transpose(1, 2)
    out = {}
    # causal forward
    cfg = AVQConfig(causal=True, attention=AttentionShapeConfig(embed_dim=w.E, num_heads=H),
                    codebook=CodebookConfig(num_codewords=M0, children_per_codeword=C),
                    routing=RoutingConfig(refinement_budget=w.P))
    mod = AVQAttention(cfg, in_proj=False, out_proj=False)
    mod.codebook.parents, mod.codebook.children = cb.parents.to(dev), cb.children.to(dev)
    work = algorithmic_work(w, 1) | {"presence": ("hbm", G * S * 4 + G * T * ((M0 + 31) // 32) * 4)}
    with torch.no_grad():
        rec = measure(ctx, lambda i: mod(q, k, v), 3, 10, work, T, clk)
    rec.update(workload=f"causal forward, c2 shapes B=1: Tq=S={T} H={H} D={D} M0={M0} C={C} P={w.P} bf16",
               parallelism="replicated (one forward per GPU)")
    rec["value_scope"] = "one GPU's rate (every GPU runs its own replica)"
    out["causal"] = rec
    # BCAR: one EMA step of the codebook toward this call's keys
    pc = cb.parents.to(dev, dt).contiguous()
    cc = cb.children.to(dev, dt).contiguous()
    pcb = ops.prepare_codebook(cb.parents, cb.children, dt, dev)
    kh = heads(k)
    st = ops.quantize(kh, heads(v), pcb)
    work = {"bcar": ("hbm", G * S * (D * es + 8) + 2 * H * M0 * C * D * es + H * M0 * D * es)}
    rec = measure(ctx, lambda i: ops.bcar_update(kh, st, pc, cc, 0.99), 3, 20, work, S, clk)
    rec.update(unit="keys/s", workload=f"BCAR update after quantizing S={S} keys, H={H} M0={M0} C={C} D={D} bf16",
               parallelism="replicated")
    rec["value_scope"] = "one GPU's rate (every GPU runs its own replica)"
    out["bcar"] = rec
    # dense path (execution.mode = "reference" / refinement off)
    be = CUDABackend()
    qh, vh = heads(q), heads(v)
    work = {"dense_attn": ("tensor", 4.0 * G * T * S * D)}
    with torch.no_grad():
        rec = measure(ctx, lambda i: be.naive_attention(qh, kh, vh), 2, 5, work, T, clk)
    rec.update(workload=f"dense attention Tq=S={T} H={H} D={D} bf16 (tcgen05 kernel)", parallelism="replicated")
    rec["value_scope"] = "one GPU's rate (every GPU runs its own replica)"
    out["dense"] = rec
    # streaming VQ: one key per extend, shared by every head
    buf = StreamingVQBuffer(H, M0, C, D, device=dev, dtype=dt)
    keys1 = kh[0, 0]  # [S, D] head 0's keys as the stream
    work = {"stream_parent": ("hbm", H * M0 * D * es), "stream_child": ("hbm", H * C * D * es),
            "stream_aggregate": ("hbm", 2 * H * (2 * D * es + 16))}
    rec = measure(ctx, lambda i: buf.extend(keys1[i % S:i % S + 1], pc, cc), 20, 200, work, 1, clk)
    rec.update(unit="keys/s", workload=f"StreamingVQBuffer.extend of one key, H={H} M0={M0} C={C} D={D} bf16 "
                                       "(timed through the Python API: host launch overhead included)",
               parallelism="replicated")
    rec["value_scope"] = "one GPU's rate (every GPU runs its own replica)"
    out["stream"] = rec
    # the same stream fed 256 keys per extend call (a prefill chunk)
    nb = 256
    work = {"stream_parent": ("hbm", H * M0 * D * es + nb * D * es), "stream_child": ("hbm", nb * H * C * D * es),
            "stream_aggregate": ("hbm", 2 * nb * H * (2 * D * es + 16))}
    buf = StreamingVQBuffer(H, M0, C, D, device=dev, dtype=dt)
    rec = measure(ctx, lambda i: buf.extend(keys1[(i * nb) % (S - nb):(i * nb) % (S - nb) + nb], pc, cc), 5, 50,
                  work, nb, clk)
    rec.update(unit="keys/s", workload=f"StreamingVQBuffer.extend of {nb} keys per call, H={H} M0={M0} C={C} D={D} "
                                       "bf16", parallelism="replicated")
    rec["value_scope"] = "one GPU's rate (every GPU runs its own replica)"
    out["stream_b256"] = rec
    return out


SUBS = {"c1": sub_c1, "c3": sub_c3, "c4": sub_c4, "c5": sub_c5, "fx": sub_fx}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = Ctx(world, rank, dev)
    ctx.sub_batch = args.sub_batch
    subs = [s for s in args.configs.split(",") if s and s != "none"]
    with ClockSampler(gpu_uuid(dev)) as clk:
        head = run_headline(args, ctx, clk)
        configs = {}
        for name in subs:
            try:
                configs[name] = SUBS[name](ctx, clk)
            except Exception as exc:  # every rank raises alike; report, keep the headline
                configs[name] = {"error": f"{type(exc).__name__}: {exc}"}
                torch.cuda.empty_cache()
    clk.close()
    if rank == 0:
        w = head.pop("w")
        try:
            cpu = cpu_baseline(w, slices=args.cpu_slices) if args.cpu_slices > 0 else None
        except Exception as exc:  # the baseline must never hide the GPU number
            cpu = {"value": None, "unit": "query tokens/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {exc}"}
        out = {"metric": METRIC, "value": head["value"], "value_scope": "whole job: the sum over all GPUs",
               "value_per_gpu": head["value"] / world, "unit": UNIT,
               "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
               "ms_per_step_median": head["ms_per_step_median"],
               "timing": "ms_per_step = timed-region CUDA-event time / steps (mean, max over ranks); the median "
                         "of the per-step event times is given beside it",
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype,
               "data": "synthetic (seeded Gaussian-mixture keys, N(0,1) q/v)", "config": workload_config(w, world),
               "clocks": head.get("clocks"), "e2e": head["e2e"], "gpu_launches": head["gpu_launches"],
               "roofline": head["roofline"], "kernels": head["kernels"], "check": head["check"],
               "cpu_baseline": cpu, "configs": configs}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
