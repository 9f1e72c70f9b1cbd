"""Benchmark of the DSA sparse-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|indexer_prefill|sparse_prefill]

Default workload (BASELINE config 2 at 128k context): sparse MLA decode, batch
64, 64 heads, q 576-d bf16, fp8_ds_mla paged latent cache (64-token blocks,
random block permutation), seq_len 131,072, top-k 2,048 sorted uniform
positions per row, bf16 output. A step is one decode call over the batch.
`value` = query rows/s (tok/s) for the whole job, timed on the device with
CUDA events over K CUDA-graph replays (the per-step idx sets rotate over 8
sets, so consecutive steps read different cache rows: inputs larger than L2).
`e2e` times the same call through the public op with the step's q and idx
copied from pinned host memory and o / lse copied back, every step.

--impl reference times the reference's own CPU torch path (a port of
TritonMLAImpl._forward_mqa_torch, oracle/ref_port.py) on the host cores.
Multi-GPU (torchrun): each rank decodes its own batch of independent rows
(no data-path collective; weak scaling); timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROW_BYTES = 656
ROOFLINE_NOTE = "of measured"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes recorded in profiles/<name>.md ('traffic_bytes_per_launch: N')."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """NVML sampling of SM clock and throttle reasons during the timed region."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index, period_s=0.01):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                r = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self.REASONS.items():
                    if r & bit and k != "gpu_idle":
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() and args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------- workloads
class DecodeWorkload:
    metric = "sparse MLA decode tok/s/GPU @128k ctx (HBM % peak)"
    unit = "tok/s"
    B, H, S, PAGE, TOPK, NSETS = 64, 64, 131072, 64, 2048, 8
    scale = 1.0 / (192 ** 0.5)
    bytes_per_row = TOPK * ROW_BYTES + TOPK * 4 + H * 576 * 2 + H * 512 * 2 + H * 4  # 1,491,200

    def config(self):
        return {"workload": "sparse_mla_decode", "batch": self.B, "heads": self.H, "ctx": self.S, "topk": self.TOPK,
                "page": self.PAGE, "kv_cache": "fp8_ds_mla", "q_dtype": "bf16", "o_dtype": "bf16",
                "l2": f"inputs larger than L2: idx rotates over {self.NSETS} sets of {self.B}x{self.TOPK} rows "
                      f"of a {self.B * self.S * ROW_BYTES / 1e9:.1f} GB cache"}

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = self.B * (self.S // self.PAGE)
        kv = torch.randint(0, 256, (nb, self.PAGE, ROW_BYTES), dtype=torch.uint8, device=dev, generator=g)
        codes = kv[..., :512]
        codes[(codes & 0x7F) == 0x7F] = 0x7E
        sc = (torch.rand(nb, self.PAGE, 4, device=dev, generator=g) + 0.5) / 448.0
        kv[..., 512:528] = sc.view(torch.uint8).view(nb, self.PAGE, 16)
        kv[..., 528:656] = torch.randn(nb, self.PAGE, 64, device=dev, generator=g).to(torch.float16).view(
            torch.uint8).view(nb, self.PAGE, 128)
        self.kv = kv
        self.bt = torch.randperm(nb, device=dev, generator=g).view(self.B, -1).to(torch.int32)
        self.seq = torch.full((self.B,), self.S, dtype=torch.int32, device=dev)
        self.q = [torch.randn(self.B, self.H, 576, device=dev, generator=g).to(torch.bfloat16)
                  for _ in range(self.NSETS)]
        self.idx = [torch.sort(torch.rand(self.B, self.S, device=dev, generator=g).topk(self.TOPK, dim=1).indices,
                               dim=1).values.to(torch.int32) for _ in range(self.NSETS)]
        self.o = torch.empty(self.B, self.H, 512, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(self.B, self.H, dtype=torch.float32, device=dev)

    def units_per_step(self):
        return self.B

    def step(self, dsa, i):
        dsa.sm70_sparse_mla_decode(self.o, self.lse, self.q[i % self.NSETS], self.kv, self.idx[i % self.NSETS],
                                   self.bt, self.seq, self.scale)

    def launches_per_step(self, dsa):
        ws = dsa._lib.lib().dsa_sparse_mla_decode_workspace_bytes(self.B, self.H, self.TOPK)
        return 2 if ws else 1

    def algorithmic(self):
        return self.B * self.bytes_per_row, "GB/s", "hbm"

    def e2e_setup(self, dev):
        self.h_q = [t.cpu().pin_memory() for t in self.q]
        self.h_idx = [t.cpu().pin_memory() for t in self.idx]
        self.h_o = torch.empty(self.o.shape, dtype=self.o.dtype).pin_memory()
        self.h_lse = torch.empty(self.lse.shape, dtype=self.lse.dtype).pin_memory()
        self.d_q = torch.empty_like(self.q[0])
        self.d_idx = torch.empty_like(self.idx[0])
        h2d = self.h_q[0].numel() * 2 + self.h_idx[0].numel() * 4
        d2h = self.h_o.numel() * 2 + self.h_lse.numel() * 4
        return h2d, d2h

    def e2e_step(self, dsa, i):
        k = i % self.NSETS
        self.d_q.copy_(self.h_q[k], non_blocking=True)
        self.d_idx.copy_(self.h_idx[k], non_blocking=True)
        dsa.sm70_sparse_mla_decode(self.o, self.lse, self.d_q, self.kv, self.d_idx, self.bt, self.seq, self.scale)
        self.h_o.copy_(self.o, non_blocking=True)
        self.h_lse.copy_(self.lse, non_blocking=True)

    # ---- CPU legs (reference torch path port)
    def cpu_setup(self, rows):
        g = torch.Generator().manual_seed(7)
        self.cpu_rows = rows
        nb = rows * (self.S // self.PAGE)  # the sampled rows' own blocks
        self.c_kv = torch.randint(0, 256, (nb * self.PAGE, ROW_BYTES), dtype=torch.uint8, generator=g)
        codes = self.c_kv[:, :512]
        codes[(codes & 0x7F) == 0x7F] = 0x7E
        self.c_kv[:, 512:528] = ((torch.rand(nb * self.PAGE, 4, generator=g) + 0.5) / 448.0).view(torch.uint8)
        self.c_kv[:, 528:656] = torch.randn(nb * self.PAGE, 64, generator=g).to(torch.float16).view(torch.uint8)
        self.c_bt = torch.randperm(nb, generator=g).view(rows, -1).to(torch.int32)
        self.c_seq = torch.full((rows,), self.S, dtype=torch.int32)
        self.c_q = torch.randn(rows, self.H, 576, generator=g).to(torch.bfloat16)
        self.c_idx = torch.sort(torch.rand(rows, self.S, generator=g).topk(self.TOPK, dim=1).indices,
                                dim=1).values.to(torch.int32)

    def cpu_step(self):
        from oracle.ref_port import sparse_decode_cpu

        sparse_decode_cpu(self.c_q, self.c_kv, self.c_idx, self.c_bt, self.c_seq, self.PAGE, self.scale)


def run_ours(args, world, rank, local):
    dsa = importlib.import_module("glm5-on-v100_b200")
    dev = torch.device("cuda", local)
    wl = DecodeWorkload()
    wl.setup(dev, seed=1234 + rank)
    hbm_peak, tf_peak, peak_kind = load_peaks()

    stream = torch.cuda.Stream(dev)
    graphs = []
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            wl.step(dsa, i)
        stream.synchronize()
        for k in range(wl.NSETS):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                wl.step(dsa, k)
            graphs.append(g)
        for i in range(max(3, args.warmup)):
            graphs[i % wl.NSETS].replay()
    torch.cuda.synchronize()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler, torch.cuda.stream(stream):
        start.record(stream)
        for i in range(args.steps):
            graphs[i % wl.NSETS].replay()
        stop.record(stream)
        stop.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world)
    ms_per_step = ms / args.steps
    units = wl.units_per_step() * args.steps * world
    value = units / (ms / 1e3)

    # end to end through the public op with host buffers
    e2e = None
    if not args.no_e2e:
        h2d, d2h = wl.e2e_setup(dev)
        for i in range(3):
            wl.e2e_step(dsa, i)
        torch.cuda.synchronize()
        barrier(world)
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record()
        for i in range(args.steps):
            wl.e2e_step(dsa, i)
        e_stop.record()
        e_stop.synchronize()
        barrier(world)
        e_ms = max_over_ranks(e_start.elapsed_time(e_stop), world)
        e2e = {"value": wl.units_per_step() * args.steps * world / (e_ms / 1e3), "unit": wl.unit,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    alg, unit, bound = wl.algorithmic()
    achieved = alg / (ms_per_step / 1e3) / 1e9
    traffic = profile_traffic("sparse_mla_decode_b64_ctx128k")
    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random fp8_ds_mla cache, N(0,1) q)",
        "config": dict(wl.config(), parallelism=f"dp{world} (independent rows per rank)"),
        "e2e": e2e,
        "gpu_launches": args.steps * wl.launches_per_step(dsa),
        "roofline": {"bound": bound, "achieved": achieved, "peak": hbm_peak, "unit": unit,
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "note": f"peak {peak_kind} HBM copy; achieved = {wl.bytes_per_row} B/row x {wl.B} rows "
                             f"per launch / CUDA-event time of the op (decode kernel + merge)"},
        "clocks": sampler.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, args)
    if rank == 0:
        print(json.dumps(line), flush=True)
    graphs.clear()


def cpu_baseline(wl, args, steps=None, rows=None):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = rows or args.cpu_rows
    wl.cpu_setup(rows)
    wl.cpu_step()  # warm-up
    steps = steps or args.cpu_steps
    t0 = time.perf_counter()
    for _ in range(steps):
        wl.cpu_step()
    dt = time.perf_counter() - t0
    return {"value": rows * steps / dt, "unit": wl.unit, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{steps} steps x {rows} rows of the same workload through the reference torch decode path "
                      f"(oracle/ref_port.py, fp8 rows dequantised on the host)"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    wl = DecodeWorkload()
    steps, rows = args.steps, args.cpu_rows
    cb = cpu_baseline(wl, args, steps=steps, rows=rows)
    ms_per_step = 1e3 * rows / cb["value"]
    line = {
        "metric": wl.metric, "value": cb["value"], "unit": wl.unit, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (host)", "data": "synthetic", "impl": "reference",
        "config": dict(wl.config(), parallelism="host cores"),
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-rows", type=int, default=8, help="rows per CPU-baseline step")
    ap.add_argument("--cpu-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--ctx", type=int, default=DecodeWorkload.S,
                    help="context length (smaller values make the ncu profiling case)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    DecodeWorkload.S = args.ctx
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
