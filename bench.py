"""Benchmark of the DSA sparse-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|indexer_prefill|sparse_prefill]

Default workload: the DSA decode layer at 180k context, batch 8 (indexer
logits + top-2048 + sparse MLA decode; on N GPUs the keys of every row are
split N ways with a P2P top-k merge and the 64 heads N ways); at N = 1 the
line also carries named sub-records for the rest of the headline metric.
Sub-record "sparse_mla_decode_b64_ctx128k": sparse MLA decode, batch
64, 64 heads, q 576-d bf16, fp8_ds_mla paged latent cache (64-token blocks,
random block permutation), seq_len 131,072, top-k 2,048 sorted uniform
positions per row, bf16 output. A step is one decode call over the batch.
`value` = query rows/s (tok/s) for the whole job, timed on the device with
CUDA events over K CUDA-graph replays (the per-step idx sets rotate over 8
sets, so consecutive steps read different cache rows: inputs larger than L2).
`e2e` times the same call through the public op with the step's q and idx
copied from pinned host memory and o / lse copied back, every step.

Other workloads (same JSON contract, value in
TFLOP/s of the algorithmic FLOPs):
  indexer_prefill  one causal chunk of 65,536 queries x 65,536 keys, 32
                   indexer heads x 128, bf16 q and keys, logits then top-2048
                   per row, in sub-blocks of 4,096 rows.
  sparse_prefill   16,384 query tokens x 64 heads at the end of a 180,224-token
                   fp8_ds_mla cache, top-2048 causal positions per token, plus
                   the indexer-K scatter of the 16,384 new keys.

--impl reference times the reference's own CPU torch path (a port of
TritonMLAImpl._forward_mqa_torch and of the indexer math, oracle/ref_port.py)
on the host cores. Multi-GPU (torchrun, one rank per GPU): the default
dsa_layer workload splits the fixed batch-8 layer across the ranks (strong
scaling: keys and heads sharded, P2P exchange of the local top-k lists);
the other workloads run a copy per rank (weak scaling). Timing is the max
over ranks.
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

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROW_BYTES = 656


def load_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, kind)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def scaled(x, f):
    return None if x is None else x * f


def profile_traffic(name):
    """Per-launch DRAM bytes recorded in profiles/<name>.md ('traffic_bytes_per_launch: N')."""
    if name is None:
        return None
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


def causal_topk_positions(n_rows, lens, K, dev, g, chunk=512):
    """[n_rows, K] int32: K distinct uniform-random positions < lens[r], sorted."""
    out = torch.empty(n_rows, K, dtype=torch.int32, device=dev)
    S = int(lens.max())
    pos = torch.arange(S, device=dev)
    for r0 in range(0, n_rows, chunk):
        r1 = min(n_rows, r0 + chunk)
        u = torch.rand(r1 - r0, S, device=dev, generator=g)
        u.masked_fill_(pos.view(1, S) >= lens[r0:r1].view(-1, 1), -1.0)
        out[r0:r1] = torch.sort(u.topk(K, dim=1).indices, dim=1).values.to(torch.int32)
        del u
    return out


def random_dsmla_cache(nb, page, dev, g):
    kv = torch.randint(0, 256, (nb, page, ROW_BYTES), dtype=torch.uint8, device=dev, generator=g)
    codes = kv[..., :512]
    codes[(codes & 0x7F) == 0x7F] = 0x7E
    sc = (torch.rand(nb, page, 4, device=dev, generator=g) + 0.5) / 448.0
    kv[..., 512:528] = sc.view(torch.uint8).view(nb, page, 16)
    kv[..., 528:656] = torch.randn(nb, page, 64, device=dev, generator=g).to(torch.float16).view(
        torch.uint8).view(nb, page, 128)
    return kv


# --------------------------------------------------------------- workloads
class Workload:
    """One benchmark configuration. `units_per_step` is in the numerator of
    `unit` (rows for tok/s, TFLOP for TFLOP/s)."""

    nsets = 1
    data = "synthetic (seeded)"
    traffic_profile = None
    graph = True  # steps replayed from CUDA graphs; False: launched eagerly (host-side sequencing)
    scaling = "weak"  # "weak": per-GPU work fixed as N grows; "strong": total work fixed
    cpu_rows_default = 8
    cpu_steps_default = None  # None: --cpu-steps

    def after_timing(self, dsa, dev):
        """Checks that the timed work ran as claimed (raises otherwise)."""

    def traffic_scale(self):
        """Units of this run's dominant launch per unit of the profiled one
        (the profile's DRAM bytes scale with it)."""
        return 1.0

    def roofline_part(self):
        """None, or (graph-capturable callable, its algorithmic amount) for the
        dominant kernel when the step holds more than that kernel."""
        return None


class DecodeWorkload(Workload):
    metric = "sparse MLA decode tok/s/GPU @128k ctx (HBM % peak)"
    unit = "tok/s"
    data = "synthetic (seeded random fp8_ds_mla cache, N(0,1) q)"
    traffic_profile = "sparse_mla_decode_b64_ctx128k"
    B, H, S, PAGE, TOPK, NSETS = 64, 64, 131072, 64, 2048, 8
    nsets = NSETS
    scale = 1.0 / (192 ** 0.5)
    bytes_per_row = TOPK * ROW_BYTES + TOPK * 4 + H * 576 * 2 + H * 512 * 2 + H * 4  # 1,491,200

    def config(self):
        return {"workload": "sparse_mla_decode", "batch": self.B, "heads": self.H, "ctx": self.S, "topk": self.TOPK,
                "page": self.PAGE, "kv_cache": "fp8_ds_mla", "q_dtype": "bf16", "o_dtype": "bf16",
                "l2": (f"inputs larger than L2: idx rotates over {self.NSETS} sets of {self.B}x{self.TOPK} rows "
                       f"of a {self.B * self.S * ROW_BYTES / 1e9:.1f} GB cache")
                if self.B * self.S * ROW_BYTES > 126e6 else
                f"the whole {self.B * self.S * ROW_BYTES / 1e6:.0f} MB cache fits in L2 at this size"}

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = self.B * (self.S // self.PAGE)
        self.kv = random_dsmla_cache(nb, self.PAGE, dev, g)
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
        return dsa.ops.decode_plan(self.B, self.H, self.TOPK, dsa._lib.DSA_FP8_DS_MLA)["launches"]

    def algorithmic(self):
        return self.B * self.bytes_per_row, "GB/s", "hbm"

    def roofline_note(self, kind):
        return (f"peak {kind} HBM copy; achieved = {self.bytes_per_row} B/row x {self.B} rows per launch / "
                f"CUDA-event time of the op (one kernel: slices merge inside a cluster)")

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

    def cpu_units(self):
        return self.cpu_rows

    def cpu_sample(self, steps):
        return (f"{steps} steps x {self.cpu_rows} rows of the same workload through the reference torch decode path "
                f"(oracle/ref_port.py, fp8 rows dequantised on the host)")


class IndexerPrefillWorkload(Workload):
    """Indexer prefill: one causal chunk of 65,536 queries, logits then top-K per row."""

    metric = "indexer prefill TFLOPS (causal QK FLOPs, logits + top-2048)"
    unit = "TFLOP/s"
    data = "synthetic (seeded N(0,1) bf16 q and keys, w ~ N(0, 1/32))"
    traffic_profile = "indexer_prefill_n65536"
    N, HI, HD, PAGE, TOPK, SUB = 65536, 32, 128, 64, 2048, 4096

    def flops(self, rows_lens):
        return 2.0 * self.HD * self.HI * float(rows_lens)

    def config(self):
        return {"workload": "indexer_prefill", "queries": self.N, "keys": self.N, "indexer_heads": self.HI,
                "head_dim": self.HD, "topk": self.TOPK, "page": self.PAGE, "q_dtype": "bf16", "k_cache": "bf16",
                "w_dtype": "fp16", "sub_block_rows": self.SUB, "causal": True,
                "flop_convention": "2*128*32*N(N+1)/2 causal pairs (QK only)",
                "l2": "inputs larger than L2 (q 512 MB, scores 1 GB per sub-block)"}

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = self.N // self.PAGE
        self.k_cache = torch.randn(nb, self.PAGE, self.HD, device=dev, generator=g).to(torch.bfloat16)
        bt_row = torch.randperm(nb, device=dev, generator=g).to(torch.int32)
        self.bt = bt_row.view(1, nb).expand(self.SUB, nb).contiguous()
        self.q = torch.randn(self.N, self.HI, self.HD, device=dev, generator=g).to(torch.bfloat16)
        self.w = (torch.randn(self.N, self.HI, device=dev, generator=g) / (self.HI ** 0.5)).to(torch.float16)
        self.lens = torch.arange(1, self.N + 1, dtype=torch.int32, device=dev)
        self.score = torch.empty(self.SUB, self.N, dtype=torch.float32, device=dev)
        self.idx = torch.empty(self.N, self.TOPK, dtype=torch.int32, device=dev)
        self.ws = torch.empty(1, dtype=torch.uint8, device=dev)
        self._bt_row = bt_row

    def _logits(self, dsa, q, w, r0, r1):
        dsa.sm70_indexer_logits(self.score[: r1 - r0, :r1], q[r0:r1], self.k_cache, w[r0:r1],
                                self.bt[: r1 - r0], self.lens[r0:r1], None)

    def step_on(self, dsa, q, w, idx):
        for r0 in range(0, self.N, self.SUB):
            r1 = min(self.N, r0 + self.SUB)
            self._logits(dsa, q, w, r0, r1)
            dsa.persistent_topk(self.score[: r1 - r0, :r1], self.lens[r0:r1], idx[r0:r1], self.ws, self.TOPK, r1)

    def step(self, dsa, i):
        self.step_on(dsa, self.q, self.w, self.idx)

    def units_per_step(self):
        return self.flops(self.N * (self.N + 1) // 2) / 1e12

    def launches_per_step(self, dsa):
        return 2 * ((self.N + self.SUB - 1) // self.SUB)

    def algorithmic(self):
        return self.flops(self.N * (self.N + 1) // 2), "TFLOP/s", "tensor"

    def roofline_part(self):
        def logits_only(dsa):
            for r0 in range(0, self.N, self.SUB):
                self._logits(dsa, self.q, self.w, r0, min(self.N, r0 + self.SUB))

        return logits_only, self.flops(self.N * (self.N + 1) // 2)

    def roofline_note(self, kind):
        return (f"peak {kind} bf16 dense (sustained); achieved = causal QK FLOPs / CUDA-event time of the "
                f"{(self.N + self.SUB - 1) // self.SUB} logits launches alone (top-k excluded)")

    def e2e_setup(self, dev):
        self.h_q = self.q.cpu().pin_memory()
        self.h_w = self.w.cpu().pin_memory()
        self.h_idx = torch.empty(self.idx.shape, dtype=torch.int32).pin_memory()
        self.d_q = torch.empty_like(self.q)
        self.d_w = torch.empty_like(self.w)
        return self.h_q.numel() * 2 + self.h_w.numel() * 2, self.h_idx.numel() * 4

    def e2e_step(self, dsa, i):
        self.d_q.copy_(self.h_q, non_blocking=True)
        self.d_w.copy_(self.h_w, non_blocking=True)
        self.step_on(dsa, self.d_q, self.d_w, self.idx)
        self.h_idx.copy_(self.idx, non_blocking=True)

    def cpu_setup(self, rows):
        g = torch.Generator().manual_seed(7)
        # rows spread over the chunk, so the sample has the chunk's mean causal length
        self.c_rows = torch.linspace(self.N // (2 * rows), self.N - 1 - self.N // (2 * rows), rows).long()
        self.c_k = torch.randn(self.N, self.HD, generator=g).to(torch.bfloat16)
        self.c_q = torch.randn(rows, self.HI, self.HD, generator=g).to(torch.bfloat16)
        self.c_w = (torch.randn(rows, self.HI, generator=g) / (self.HI ** 0.5)).to(torch.float16)
        self.c_lens = self.c_rows + 1

    def cpu_step(self):
        from oracle.ref_port import indexer_prefill_cpu

        indexer_prefill_cpu(self.c_q, self.c_k, self.c_w, self.c_lens, self.TOPK)

    def cpu_units(self):
        return self.flops(int(self.c_lens.sum())) / 1e12

    def cpu_sample(self, steps):
        return (f"{steps} steps x {len(self.c_rows)} query rows spread over the chunk (logits over their causal "
                f"keys + torch.topk, oracle/ref_port.py)")


class SparsePrefillWorkload(Workload):
    """Sparse prefill attention (16,384 tokens over a 180k cache) + indexer-K scatter."""

    metric = "sparse prefill attention TFLOPS (top-2048, 64 heads)"
    unit = "TFLOP/s"
    data = "synthetic (seeded random fp8_ds_mla cache, N(0,1) bf16 q and k)"
    traffic_profile = "sparse_prefill_t16384_ctx180k"
    T, H, S, PAGE, TOPK = 16384, 64, 180224, 64, 2048
    scale = 1.0 / (192 ** 0.5)

    def flops(self, rows):
        return 2.0 * rows * self.H * self.TOPK * (576 + 512)

    def config(self):
        return {"workload": "sparse_prefill", "queries": self.T, "heads": self.H, "ctx": self.S, "topk": self.TOPK,
                "page": self.PAGE, "kv_cache": "fp8_ds_mla", "q_dtype": "bf16", "o_dtype": "bf16",
                "k_store": f"{self.T} x 128 bf16 rows into random slots of a bf16 indexer-K cache",
                "l2": "inputs larger than L2 (q 1.2 GB, o 1 GB); the 118 MB latent cache itself stays L2-resident "
                      "as in the real layer"}

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = self.S // self.PAGE
        self.kv = random_dsmla_cache(nb, self.PAGE, dev, g)
        bt_row = torch.randperm(nb, device=dev, generator=g).to(torch.int32)
        self.bt = bt_row.view(1, nb).expand(self.T, nb).contiguous()
        self.seq = torch.arange(self.S - self.T + 1, self.S + 1, dtype=torch.int32, device=dev)
        self.idx = causal_topk_positions(self.T, self.seq, self.TOPK, dev, g)
        self.q = torch.randn(self.T, self.H, 576, device=dev, generator=g).to(torch.bfloat16)
        self.o = torch.empty(self.T, self.H, 512, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(self.T, self.H, dtype=torch.float32, device=dev)
        self.k_cache = torch.zeros(nb, self.PAGE, 128, dtype=torch.bfloat16, device=dev)
        self.k_new = torch.randn(self.T, 128, device=dev, generator=g).to(torch.bfloat16)
        self.slots = torch.randperm(self.S, device=dev, generator=g)[: self.T].to(torch.int32)

    def _attention(self, dsa, q, idx):
        dsa.sm70_sparse_mla_decode(self.o, self.lse, q, self.kv, idx, self.bt, self.seq, self.scale)

    def step_on(self, dsa, q, idx, k_new):
        dsa.sm70_indexer_k_store(self.k_cache, k_new, self.slots)
        self._attention(dsa, q, idx)

    def step(self, dsa, i):
        self.step_on(dsa, self.q, self.idx, self.k_new)

    def units_per_step(self):
        return self.flops(self.T) / 1e12

    def launches_per_step(self, dsa):
        return 1 + dsa.ops.decode_plan(self.T, self.H, self.TOPK, dsa._lib.DSA_FP8_DS_MLA)["launches"]

    def algorithmic(self):
        return self.flops(self.T), "TFLOP/s", "tensor"

    def roofline_part(self):
        return (lambda dsa: self._attention(dsa, self.q, self.idx)), self.flops(self.T)

    def roofline_note(self, kind):
        return (f"peak {kind} bf16 dense (sustained); achieved = 2*T*H*K*(576+512) FLOPs / CUDA-event time of "
                f"the attention launch alone (K scatter excluded)")

    def e2e_setup(self, dev):
        self.h_q = self.q.cpu().pin_memory()
        self.h_idx = self.idx.cpu().pin_memory()
        self.h_k = self.k_new.cpu().pin_memory()
        self.h_o = torch.empty(self.o.shape, dtype=self.o.dtype).pin_memory()
        self.h_lse = torch.empty(self.lse.shape, dtype=self.lse.dtype).pin_memory()
        self.d_q, self.d_idx, self.d_k = (torch.empty_like(self.q), torch.empty_like(self.idx),
                                          torch.empty_like(self.k_new))
        h2d = self.h_q.numel() * 2 + self.h_idx.numel() * 4 + self.h_k.numel() * 2
        return h2d, self.h_o.numel() * 2 + self.h_lse.numel() * 4

    def e2e_step(self, dsa, i):
        self.d_q.copy_(self.h_q, non_blocking=True)
        self.d_idx.copy_(self.h_idx, non_blocking=True)
        self.d_k.copy_(self.h_k, non_blocking=True)
        self.step_on(dsa, self.d_q, self.d_idx, self.d_k)
        self.h_o.copy_(self.o, non_blocking=True)
        self.h_lse.copy_(self.lse, non_blocking=True)

    def cpu_setup(self, rows):
        g = torch.Generator().manual_seed(7)
        self.cpu_rows = rows
        # the sampled rows read from a cache of their own, the full context long
        nb = self.S // self.PAGE
        self.c_kv = torch.randint(0, 256, (nb * self.PAGE, ROW_BYTES), dtype=torch.uint8, generator=g)
        codes = self.c_kv[:, :512]
        codes[(codes & 0x7F) == 0x7F] = 0x7E
        self.c_kv[:, 512:528] = ((torch.rand(nb * self.PAGE, 4, generator=g) + 0.5) / 448.0).view(torch.uint8)
        self.c_kv[:, 528:656] = torch.randn(nb * self.PAGE, 64, generator=g).to(torch.float16).view(torch.uint8)
        self.c_bt = torch.randperm(nb, generator=g).to(torch.int32).view(1, nb).expand(rows, nb).contiguous()
        self.c_seq = torch.arange(self.S - rows + 1, self.S + 1, dtype=torch.int32)
        self.c_q = torch.randn(rows, self.H, 576, generator=g).to(torch.bfloat16)
        self.c_idx = torch.sort(torch.rand(rows, self.S - rows, generator=g).topk(self.TOPK, dim=1).indices,
                                dim=1).values.to(torch.int32)

    def cpu_step(self):
        from oracle.ref_port import sparse_decode_cpu

        sparse_decode_cpu(self.c_q, self.c_kv, self.c_idx, self.c_bt, self.c_seq, self.PAGE, self.scale)

    def cpu_units(self):
        return self.flops(self.cpu_rows) / 1e12

    def cpu_sample(self, steps):
        return (f"{steps} steps x {self.cpu_rows} query rows through the reference torch decode path "
                f"(oracle/ref_port.py, fp8 rows dequantised on the host; K scatter not included)")


class IndexerDecodeWorkload(Workload):
    cpu_rows_default = 1
    """The indexer half of a batch-64 decode step: per row, logits
    with the fused level-1 histogram over its 128k keys in the fp8 indexer-K
    cache, then the exact top-2048 from that histogram."""

    metric = "decode indexer tok/s @128k ctx (logits + fused histogram + top-2048)"
    unit = "tok/s"
    data = "synthetic (seeded random fp8 indexer-K cache, N(0,1) bf16 q, w ~ N(0, 1/32))"
    traffic_profile = "indexer_decode_b64_ctx128k"
    B, HI, HD, PAGE, TOPK, NSETS = 64, 32, 128, 64, 2048, 4
    S = 131072
    nsets = NSETS

    def bytes_per_row(self):
        # keys (fp8 + scale), scores written and read back, q, w, histogram,
        # indices, block table
        return (self.S * (132 + 4 + 4) + self.HI * self.HD * 2 + self.HI * 4 + 4096 * 4 * 2 + self.TOPK * 4
                + (self.S // self.PAGE) * 4)

    def config(self):
        return {"workload": "indexer_decode", "batch": self.B, "indexer_heads": self.HI, "head_dim": self.HD,
                "ctx": self.S, "topk": self.TOPK, "page": self.PAGE, "k_cache": "fp8 (128 e4m3 + f32 scale)",
                "q_dtype": "bf16", "w_dtype": "f32",
                "l2": f"inputs larger than L2: a {self.B * self.S * 132 / 1e9:.1f} GB key cache"}

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = self.B * (self.S // self.PAGE)
        kc = torch.randint(0, 256, (nb, self.PAGE, 132), dtype=torch.uint8, device=dev, generator=g)
        codes = kc[..., :128]
        codes[(codes & 0x7F) == 0x7F] = 0x7E  # no NaN codes
        sc = (torch.rand(nb, self.PAGE, 1, device=dev, generator=g) + 0.5) / 448.0
        kc[..., 128:132] = sc.view(torch.uint8).view(nb, self.PAGE, 4)
        self.k_cache = kc
        self.bt = torch.randperm(nb, device=dev, generator=g).view(self.B, -1).to(torch.int32)
        self.seq = torch.full((self.B,), self.S, dtype=torch.int32, device=dev)
        self.q = [torch.randn(self.B, self.HI, self.HD, device=dev, generator=g).to(torch.bfloat16)
                  for _ in range(self.NSETS)]
        self.w = torch.randn(self.B, self.HI, device=dev, generator=g) / (self.HI ** 0.5)
        self.score = torch.empty(self.B, self.S, dtype=torch.float32, device=dev)
        self.hist = torch.zeros(self.B, 4096, dtype=torch.int32, device=dev)
        self.idx = torch.empty(self.B, self.TOPK, dtype=torch.int32, device=dev)

    def step_on(self, dsa, q, w):
        self.hist.zero_()
        dsa.sm70_indexer_logits(self.score, q, self.k_cache, w, self.bt, self.seq, self.hist)
        dsa.sm70_decode_topk(self.idx, self.score, self.seq, self.hist, self.TOPK)

    def step(self, dsa, i):
        self.step_on(dsa, self.q[i % self.NSETS], self.w)

    def units_per_step(self):
        return self.B

    def launches_per_step(self, dsa):
        return 2  # logits, top-k (the histogram memset is torch's)

    def algorithmic(self):
        return self.B * self.bytes_per_row(), "GB/s", "hbm"

    def roofline_note(self, kind):
        return (f"peak {kind} HBM copy; achieved = {self.bytes_per_row()} B/row x {self.B} rows / CUDA-event time "
                f"of the whole step (logits + top-k)")

    def e2e_setup(self, dev):
        self.h_q = [t.cpu().pin_memory() for t in self.q]
        self.h_w = self.w.cpu().pin_memory()
        self.h_idx = torch.empty(self.idx.shape, dtype=torch.int32).pin_memory()
        self.d_q = torch.empty_like(self.q[0])
        self.d_w = torch.empty_like(self.w)
        return self.h_q[0].numel() * 2 + self.h_w.numel() * 4, self.h_idx.numel() * 4

    def e2e_step(self, dsa, i):
        self.d_q.copy_(self.h_q[i % self.NSETS], non_blocking=True)
        self.d_w.copy_(self.h_w, non_blocking=True)
        self.step_on(dsa, self.d_q, self.d_w)
        self.h_idx.copy_(self.idx, non_blocking=True)

    def cpu_setup(self, rows):
        g = torch.Generator().manual_seed(7)
        self.cpu_rows = rows
        self.c_k = [torch.randn(self.S, self.HD, generator=g).to(torch.bfloat16) for _ in range(rows)]
        self.c_q = torch.randn(rows, self.HI, self.HD, generator=g).to(torch.bfloat16)
        self.c_w = torch.randn(rows, self.HI, generator=g) / (self.HI ** 0.5)

    def cpu_step(self):
        from oracle.ref_port import indexer_prefill_cpu

        lens = torch.tensor([self.S])
        for r in range(self.cpu_rows):  # each decode row has keys of its own
            indexer_prefill_cpu(self.c_q[r:r + 1], self.c_k[r], self.c_w[r:r + 1], lens, self.TOPK)

    def cpu_units(self):
        return self.cpu_rows

    def cpu_sample(self, steps):
        return (f"{steps} steps x {self.cpu_rows} rows, each over 131,072 keys of its own (logits + torch.topk, "
                f"oracle/ref_port.py; keys already decoded to bf16)")


class ShardMergeWorkload(Workload):
    cpu_rows_default = 512
    """The exact merge of the key-sharded indexer (the 8-way key split's
    8-way key split) on one GPU: for each of R query rows, the global top-2048
    of 8 shards' local top-2048 (value, position) lists, lowest position first
    on ties, positions ascending."""

    metric = "indexer shard merge rows/s (8 shards x top-2048)"
    unit = "rows/s"
    data = "synthetic (seeded N(0,1) candidate values, distinct positions per shard)"
    traffic_profile = "shard_merge_r4096_tp8"
    TP, R, TOPK, S = 8, 4096, 2048, 184320
    nsets = 2
    sorted_runs = True  # False: shuffled lists (the merge sorts the selected positions itself)

    def bytes_per_row(self):
        return self.TP * 2 * self.TOPK * 4 + self.TOPK * 4

    def config(self):
        return {"workload": "shard_merge", "shards": self.TP, "rows": self.R, "topk": self.TOPK,
                "keys": self.S, "runs": "ascending per shard" if self.sorted_runs else "shuffled",
                "l2": f"inputs larger than L2: {self.nsets} candidate sets of "
                f"{self.TP * self.R * 2 * self.TOPK * 4 / 1e6:.0f} MB"}

    def _candidates(self, dev, g, R):
        span = self.S // self.TP
        vals = torch.randn(self.TP, R, self.TOPK, device=dev, generator=g)
        base = torch.arange(self.TP, device=dev).view(self.TP, 1, 1) * span
        off = torch.randint(0, span, (self.TP, R, 1), device=dev, generator=g)
        pos = (base + (torch.arange(self.TOPK, device=dev).view(1, 1, -1) * 89 + off) % span).to(torch.int32)
        if self.sorted_runs:  # each shard's list ascending, as the top-k kernels of this build emit it
            pos = torch.sort(pos, dim=2).values
        return torch.cat([vals, pos.view(torch.float32)], dim=2).contiguous()

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        self.allf = [self._candidates(dev, g, self.R) for _ in range(self.nsets)]
        self.out = torch.empty(self.R, self.TOPK, dtype=torch.int32, device=dev)
        self.rows = torch.empty(0, dtype=torch.int32, device=dev)

    def step_on(self, dsa, allf):
        dsa.sm70_indexer_shard_merge(self.out, allf, self.rows, 0, self.TOPK)

    def step(self, dsa, i):
        self.step_on(dsa, self.allf[i % self.nsets])

    def units_per_step(self):
        return self.R

    def launches_per_step(self, dsa):
        return 1

    def algorithmic(self):
        return self.R * self.bytes_per_row(), "GB/s", "hbm"

    def roofline_note(self, kind):
        return (f"peak {kind} HBM copy; achieved = {self.bytes_per_row()} B/row (8 x 2048 candidates in, 2048 "
                f"positions out) x {self.R} rows / CUDA-event time of the merge launch")

    def e2e_setup(self, dev):
        self.h_allf = [t.cpu().pin_memory() for t in self.allf]
        self.h_out = torch.empty(self.out.shape, dtype=torch.int32).pin_memory()
        self.d_allf = torch.empty_like(self.allf[0])
        return self.h_allf[0].numel() * 4, self.h_out.numel() * 4

    def e2e_step(self, dsa, i):
        self.d_allf.copy_(self.h_allf[i % self.nsets], non_blocking=True)
        self.step_on(dsa, self.d_allf)
        self.h_out.copy_(self.out, non_blocking=True)

    def cpu_setup(self, rows):
        g = torch.Generator().manual_seed(7)
        self.cpu_rows = rows
        self.c_allf = self._candidates(torch.device("cpu"), g, rows).numpy()

    def cpu_step(self):
        from oracle.dsa_oracle import shard_merge_torch_epilogue

        shard_merge_torch_epilogue(self.c_allf, self.TOPK)

    def cpu_units(self):
        return self.cpu_rows

    def cpu_sample(self, steps):
        return (f"{steps} steps x {self.cpu_rows} rows through the reference's torch merge epilogue "
                f"(torch.topk over the 8 x 2048 candidates, oracle/dsa_oracle.py)")


class DecodeLayerWorkload(Workload):
    cpu_rows_default = 1
    """One DSA decode layer step per row: the indexer (logits with the fused
    histogram over the row's keys in the fp8 indexer-K cache, exact top-2048)
    and sparse MLA decode attention over the selected rows of the
    fp8_ds_mla latent cache; both caches share the block table, as the
    reference's layer does. At B = 8 and 180k keys this is the sharded layer's
    layer on one GPU."""

    metric = "DSA decode layer tok/s @128k ctx (indexer + top-2048 + sparse MLA)"
    unit = "tok/s"
    data = "synthetic (seeded random fp8 indexer-K and fp8_ds_mla caches, N(0,1) q)"
    B, H, HI, S, PAGE, TOPK, NSETS = 64, 64, 32, 131072, 64, 2048, 4
    nsets = NSETS
    scale = 1.0 / (192 ** 0.5)

    def bytes_per_row(self):
        idx = (self.S * (132 + 4 + 4) + self.HI * 128 * 2 + self.HI * 4 + 4096 * 4 * 2 + self.TOPK * 4
               + (self.S // self.PAGE) * 4)
        return idx + DecodeWorkload.bytes_per_row

    def config(self):
        return {"workload": "decode_layer", "batch": self.B, "heads": self.H, "indexer_heads": self.HI,
                "ctx": self.S, "topk": self.TOPK, "page": self.PAGE, "kv_cache": "fp8_ds_mla",
                "k_cache": "fp8 (128 e4m3 + f32 scale)", "q_dtype": "bf16", "o_dtype": "bf16",
                "l2": f"inputs larger than L2: {self.B * self.S * (ROW_BYTES + 132) / 1e9:.1f} GB of caches"}

    def setup(self, dev, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = self.B * (self.S // self.PAGE)
        self.kv = random_dsmla_cache(nb, self.PAGE, dev, g)
        kc = torch.randint(0, 256, (nb, self.PAGE, 132), dtype=torch.uint8, device=dev, generator=g)
        codes = kc[..., :128]
        codes[(codes & 0x7F) == 0x7F] = 0x7E
        sc = (torch.rand(nb, self.PAGE, 1, device=dev, generator=g) + 0.5) / 448.0
        kc[..., 128:132] = sc.view(torch.uint8).view(nb, self.PAGE, 4)
        self.k_cache = kc
        self.bt = torch.randperm(nb, device=dev, generator=g).view(self.B, -1).to(torch.int32)
        self.seq = torch.full((self.B,), self.S, dtype=torch.int32, device=dev)
        self.q = [torch.randn(self.B, self.H, 576, device=dev, generator=g).to(torch.bfloat16)
                  for _ in range(self.NSETS)]
        self.qi = [torch.randn(self.B, self.HI, 128, device=dev, generator=g).to(torch.bfloat16)
                   for _ in range(self.NSETS)]
        self.w = torch.randn(self.B, self.HI, device=dev, generator=g) / (self.HI ** 0.5)
        self.score = torch.empty(self.B, self.S, dtype=torch.float32, device=dev)
        self.hist = torch.zeros(self.B, 4096, dtype=torch.int32, device=dev)
        self.idx = torch.empty(self.B, self.TOPK, dtype=torch.int32, device=dev)
        self.o = torch.empty(self.B, self.H, 512, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(self.B, self.H, dtype=torch.float32, device=dev)

    def step_on(self, dsa, q, qi, w):
        self.hist.zero_()
        dsa.sm70_indexer_logits(self.score, qi, self.k_cache, w, self.bt, self.seq, self.hist)
        dsa.sm70_decode_topk(self.idx, self.score, self.seq, self.hist, self.TOPK)
        dsa.sm70_sparse_mla_decode(self.o, self.lse, q, self.kv, self.idx, self.bt, self.seq, self.scale)

    def step(self, dsa, i):
        self.step_on(dsa, self.q[i % self.NSETS], self.qi[i % self.NSETS], self.w)

    def units_per_step(self):
        return self.B

    def launches_per_step(self, dsa):
        return 2 + dsa.ops.decode_plan(self.B, self.H, self.TOPK, dsa._lib.DSA_FP8_DS_MLA)["launches"]

    def algorithmic(self):
        return self.B * self.bytes_per_row(), "GB/s", "hbm"

    def roofline_note(self, kind):
        return (f"peak {kind} HBM copy; achieved = {self.bytes_per_row()} B/row (indexer + attention) x {self.B} "
                f"rows / CUDA-event time of the whole layer step")

    def e2e_setup(self, dev):
        self.h_q = [t.cpu().pin_memory() for t in self.q]
        self.h_qi = [t.cpu().pin_memory() for t in self.qi]
        self.h_w = self.w.cpu().pin_memory()
        self.h_o = torch.empty(self.o.shape, dtype=self.o.dtype).pin_memory()
        self.h_lse = torch.empty(self.lse.shape, dtype=self.lse.dtype).pin_memory()
        self.d_q, self.d_qi, self.d_w = (torch.empty_like(self.q[0]), torch.empty_like(self.qi[0]),
                                         torch.empty_like(self.w))
        h2d = self.h_q[0].numel() * 2 + self.h_qi[0].numel() * 2 + self.h_w.numel() * 4
        return h2d, self.h_o.numel() * 2 + self.h_lse.numel() * 4

    def e2e_step(self, dsa, i):
        k = i % self.NSETS
        self.d_q.copy_(self.h_q[k], non_blocking=True)
        self.d_qi.copy_(self.h_qi[k], non_blocking=True)
        self.d_w.copy_(self.h_w, non_blocking=True)
        self.step_on(dsa, self.d_q, self.d_qi, self.d_w)
        self.h_o.copy_(self.o, non_blocking=True)
        self.h_lse.copy_(self.lse, non_blocking=True)

    # CPU legs: the two reference CPU paths in sequence on a bounded sample
    def cpu_setup(self, rows):
        self._ci = IndexerDecodeWorkload()
        self._ci.S, self._ci.TOPK = self.S, self.TOPK
        self._ci.cpu_setup(rows)
        self._cd = DecodeWorkload()
        self._cd.S, self._cd.TOPK = self.S, self.TOPK
        self._cd.cpu_setup(rows)
        self.cpu_rows = rows

    def cpu_step(self):
        self._ci.cpu_step()
        self._cd.cpu_step()

    def cpu_units(self):
        return self.cpu_rows

    def cpu_sample(self, steps):
        return (f"{steps} steps x {self.cpu_rows} rows: logits over 131,072 keys + torch.topk, then the reference "
                f"torch decode path over 2048 rows (oracle/ref_port.py)")


class ShardMergeP2PWorkload(ShardMergeWorkload):
    """The key-sharded indexer's merge over peer memory (one rank per GPU under
    torchrun): every rank stages its local top-2048 (value, position) lists
    of R rows in a CUDA IPC slot and merges all ranks' slots with plain peer
    loads after bounded waits on the peers' staged flags, so each rank ends
    with the global top-2048 of every row. Launched eagerly: the exchange's
    sequence numbers live on the host."""

    metric = "indexer P2P shard merge rows/s (tp shards x top-2048, per-rank output)"
    data = "synthetic (seeded N(0,1) candidate values, distinct positions per shard)"
    traffic_profile = None
    graph = False
    R = 1024  # the P2P slot capacity (the reference's max_num_batched_tokens)

    def config(self):
        return {"workload": "shard_merge_p2p", "shards": getattr(self, "tp", None), "rows": self.R,
                "topk": self.TOPK,
                "keys": self.S, "merge": "p2p (CUDA IPC slots, plain peer loads)",
                "l2": "each rank's slot is written once per step and read by every rank"}

    def setup(self, dev, seed):
        import importlib as _il

        import torch.distributed as dist

        if not dist.is_initialized() or dist.get_world_size() < 2:
            raise SystemExit("shard_merge_p2p needs torchrun with 2 or more ranks (one per GPU)")
        self.tp = dist.get_world_size()
        self.rank = dist.get_rank()
        self.TP = self.tp
        sai = _il.import_module("glm5-on-v100_b200.sparse_attn_indexer")
        cpu = dist.new_group(backend="gloo")
        self.shard = sai.ShardConfig(tp=self.tp, rank=self.rank, cpu_group=cpu, merge="p2p", rows_cap=self.R)
        self._merge = sai.merge_shards
        g = torch.Generator(device=dev).manual_seed(seed)
        span = self.S // max(self.tp, 1)
        self.vals = [torch.randn(self.R, self.TOPK, device=dev, generator=g) for _ in range(self.nsets)]
        off = torch.randint(0, span, (self.R, 1), device=dev, generator=g)
        pos = (self.rank * span + (torch.arange(self.TOPK, device=dev).view(1, -1) * 89 + off) % span).to(torch.int32)
        self.pos = torch.sort(pos, dim=1).values.contiguous()  # ascending, as this build's top-k emits its lists
        self.out = torch.empty(self.R, self.TOPK, dtype=torch.int32, device=dev)

    def bytes_per_row(self):
        return self.tp * 2 * self.TOPK * 4 + self.TOPK * 4

    def after_timing(self, dsa, dev):
        if self.shard.p2p_failed:
            raise RuntimeError("the P2P merge fell back to the all-gather path during the run: the figure would not "
                               "be a P2P one")

    def step_on(self, dsa, vals):
        self._merge([(0, self.R, vals, self.pos)], self.out, self.TOPK, self.shard)

    def step(self, dsa, i):
        self.step_on(dsa, self.vals[i % self.nsets])

    def units_per_step(self):
        return self.R

    def launches_per_step(self, dsa):
        return 4  # staged and merged flags, slot-reuse wait, merge kernel

    def roofline_note(self, kind):
        return (f"peak {kind} HBM copy; achieved = {self.bytes_per_row()} B/row ({self.tp} slots of 2 x 2048 x 4 B "
                f"read, {self.tp - 1} of them over NVLink, 2048 positions written) x {self.R} rows / CUDA-event time "
                f"of the eager step")

    def e2e_setup(self, dev):
        self.h_vals = [t.cpu().pin_memory() for t in self.vals]
        self.h_out = torch.empty(self.out.shape, dtype=torch.int32).pin_memory()
        self.d_vals = torch.empty_like(self.vals[0])
        return self.h_vals[0].numel() * 4, self.h_out.numel() * 4

    def e2e_step(self, dsa, i):
        self.d_vals.copy_(self.h_vals[i % self.nsets], non_blocking=True)
        self.step_on(dsa, self.d_vals)
        self.h_out.copy_(self.out, non_blocking=True)

    def cpu_setup(self, rows):
        self.TP = getattr(self, "tp", 2)
        super().cpu_setup(rows)


class ShardedLayerWorkload(DecodeLayerWorkload):
    """A DSA decode layer step at 180k context, batch 8, on N GPUs (one rank
    per GPU). Every rank holds the replicated fp8 indexer-K and fp8_ds_mla
    caches; rank r scores the contiguous key span r of every row (S / N keys,
    logits + fused histogram), writes its local top-2048 straight into its
    P2P exchange slot, and the exact merge over all ranks' slots (plain peer
    loads, device-side sequence numbers) gives every rank the global top-2048;
    sparse MLA decode then runs on the rank's 64 / N heads. At N = 1 the same
    layer runs unsharded (logits + top-2048 + decode over all 64 heads). One
    CUDA graph replay per step; total work is fixed as N grows (strong
    scaling)."""

    metric = "DSA decode layer tok/s @180k ctx, batch 8 (key-sharded indexer + P2P top-2048 merge + head-split sparse MLA)"
    data = "synthetic (seeded random fp8 indexer-K and fp8_ds_mla caches, replicated on every rank; N(0,1) q)"
    scaling = "strong"
    B, H, HI, S, PAGE, TOPK, NSETS = 8, 64, 32, 180224, 64, 2048, 4
    nsets = NSETS
    traffic_profile = "indexer_decode_tc_b8_ctx180k"  # the logits launch over 8 rows x 180,224 keys

    def config(self):
        tp = getattr(self, "tp", 1)
        return {"workload": "dsa_decode_layer", "batch": self.B, "heads": self.H, "heads_per_gpu": self.H // tp,
                "indexer_heads": self.HI, "ctx": self.S, "keys_per_gpu": self.span if tp > 1 else self.S,
                "topk": self.TOPK, "page": self.PAGE, "kv_cache": "fp8_ds_mla", "k_cache": "fp8 (128 e4m3 + f32)",
                "q_dtype": "bf16", "o_dtype": "bf16",
                "merge": "p2p exchange (IPC slots, plain peer loads, device sequence)" if tp > 1 else "none (1 GPU)",
                "l2": f"inputs larger than L2: {self.B * self.S * (ROW_BYTES + 132) / 1e9:.2f} GB of caches, "
                      f"{self.NSETS} rotating q sets"}

    def setup(self, dev, seed):
        import importlib as _il

        import torch.distributed as dist

        self.tp = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        super().setup(dev, 1234)  # identical caches and queries on every rank
        h0, h1 = self.rank * self.H // self.tp, (self.rank + 1) * self.H // self.tp
        self.q = [t[:, h0:h1].contiguous() for t in self.q]
        self.o = torch.empty(self.B, h1 - h0, 512, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(self.B, h1 - h0, dtype=torch.float32, device=dev)
        self.span = self.S
        if self.tp > 1:
            sai = _il.import_module("glm5-on-v100_b200.sparse_attn_indexer")
            self._sai = sai
            cpu = dist.new_group(backend="gloo")
            self.shard = sai.ShardConfig(tp=self.tp, rank=self.rank, cpu_group=cpu, merge="p2p", decode=True,
                                         rows_cap=self.B)
            self.bufs = {}
            _, self.span, _, _ = sai.decode_span(self.bt.shape[1] * self.PAGE, self.shard, self.PAGE)
            del self.score

    def step_on(self, dsa, q, qi, w):
        if self.tp == 1:
            super().step_on(dsa, q, qi, w)
            return
        self._sai.decode_indexer_sharded(qi, self.k_cache, w, self.bt, self.seq, self.TOPK, self.idx, self.shard,
                                         self.bufs)
        dsa.sm70_sparse_mla_decode(self.o, self.lse, q, self.kv, self.idx, self.bt, self.seq, self.scale)

    def units_per_step(self):
        return self.B / self.tp  # every rank finishes the same B rows (its heads): B rows per step for the job

    def launches_per_step(self, dsa):
        heads = self.H // getattr(self, "tp", 1)
        attn = dsa.ops.decode_plan(self.B, heads, self.TOPK, dsa._lib.DSA_FP8_DS_MLA)["launches"]
        return 2 + attn if getattr(self, "tp", 1) == 1 else 3 + attn

    def indexer_bytes(self):
        return self.B * (self.span * (132 + 4) + self.HI * 128 * 2 + self.HI * 4)

    def traffic_scale(self):
        return self.B * self.span / (8 * 180224)  # keys this rank's logits launch reads vs the profiled launch

    def roofline_part(self):
        """The indexer logits with the fused histogram over this rank's key
        span (the O(S) scan), the kernel the layer step launches."""
        hist = torch.zeros(self.B, 4096, dtype=torch.int32, device=self.bt.device)
        if self.tp == 1:
            def fn(dsa):
                dsa.sm70_indexer_logits(self.score, self.qi[0], self.k_cache, self.w, self.bt, self.seq, hist)
        else:
            off, span, lo, hi = self._sai.decode_span(self.bt.shape[1] * self.PAGE, self.shard, self.PAGE)
            score = torch.empty(self.B, span, dtype=torch.float32, device=self.bt.device)
            seg = self.bt[:, lo:hi]
            sl = (self.seq - off).clamp(0, span)

            def fn(dsa):
                dsa.sm70_indexer_logits(score, self.qi[0], self.k_cache, self.w, seg, sl, hist)
        return fn, self.indexer_bytes()

    def roofline_note(self, kind):
        return (f"peak {kind} HBM copy; dominant kernel = the indexer logits over this rank's {self.span} keys per "
                f"row, timed alone: achieved = {self.B} rows x {self.span} keys x (132 B key + 4 B score) + q/w "
                f"/ its CUDA-event time")

    def after_timing(self, dsa, dev):
        if self.tp > 1 and dsa.ops.p2p_failed(dev):
            raise RuntimeError("a bounded P2P exchange wait expired during the run: the measurement is invalid")

    def cpu_setup(self, rows):
        super().cpu_setup(rows)

    def cpu_sample(self, steps):
        return (f"{steps} steps x {self.cpu_rows} row: indexer logits over {self.S} keys + torch.topk(2048), then "
                f"the reference torch decode path over the 2048 selected rows, 64 heads (oracle/ref_port.py)")


WORKLOADS = {"decode": DecodeWorkload, "indexer_prefill": IndexerPrefillWorkload,
             "sparse_prefill": SparsePrefillWorkload, "indexer_decode": IndexerDecodeWorkload,
             "shard_merge": ShardMergeWorkload, "decode_layer": DecodeLayerWorkload,
             "shard_merge_p2p": ShardMergeP2PWorkload, "dsa_layer": ShardedLayerWorkload}


def capture(fn, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def time_graphs(graphs, steps, stream):
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for i in range(steps):
            graphs[i % len(graphs)].replay()
        stop.record(stream)
        stop.synchronize()
    return start.elapsed_time(stop)


def measure(wl, dsa, args, world, rank, dev, steps, warmup, e2e_steps, cpu):
    """Time one workload: W eager warm-up steps, then K steps (CUDA-graph
    replays unless the workload sequences on the host) between CUDA events on
    the launching stream, barrier + synchronize on both sides, max over ranks;
    the dominant kernel alone for the roofline; the end-to-end leg through the
    public op with pinned host buffers; the CPU baseline on rank 0 at N = 1."""
    wl.setup(dev, seed=1234 + rank)
    torch.cuda.synchronize()  # inputs are made on the default stream; the steps run on their own stream
    hbm_peak, tf_burst, tf_sustained, peak_kind = load_peaks()
    stream = torch.cuda.Stream(dev)
    graphs = []
    with torch.cuda.stream(stream):
        for i in range(warmup):
            wl.step(dsa, i)
        stream.synchronize()
        if wl.graph:
            graphs = [capture(lambda k=k: wl.step(dsa, k), stream) for k in range(wl.nsets)]
            for i in range(max(3, warmup)):
                graphs[i % wl.nsets].replay()
    torch.cuda.synchronize()

    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler:
        if wl.graph:
            ms = time_graphs(graphs, steps, stream)
        else:
            with torch.cuda.stream(stream):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for i in range(steps):
                    wl.step(dsa, i)
                e1.record(stream)
                e1.synchronize()
                ms = e0.elapsed_time(e1)
    torch.cuda.synchronize()
    barrier(world)
    wl.after_timing(dsa, dev)
    ms = max_over_ranks(ms, world)
    ms_per_step = ms / steps
    value = wl.units_per_step() * steps * world / (ms / 1e3)

    # the dominant kernel alone, where the step holds more than it
    part = wl.roofline_part()
    alg, unit, bound = wl.algorithmic()
    if part is not None:
        fn, alg = part
        torch.cuda.synchronize()  # the part's buffers are made on the default stream
        with torch.cuda.stream(stream):
            pg = [capture(lambda: fn(dsa), stream)]
            pg[0].replay()
        torch.cuda.synchronize()
        part_steps = max(3, min(steps, 20))
        part_ms = max_over_ranks(time_graphs(pg, part_steps, stream), world) / part_steps
        pg.clear()
    else:
        part_ms = ms_per_step
    if unit == "GB/s":
        achieved, peak = alg / (part_ms / 1e3) / 1e9, hbm_peak
    else:
        achieved, peak = alg / (part_ms / 1e3) / 1e12, tf_sustained

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
        for i in range(e2e_steps):
            wl.e2e_step(dsa, i)
        e_stop.record()
        e_stop.synchronize()
        barrier(world)
        wl.after_timing(dsa, dev)
        e_ms = max_over_ranks(e_start.elapsed_time(e_stop), world)
        e2e = {"value": wl.units_per_step() * e2e_steps * world / (e_ms / 1e3), "unit": wl.unit,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    rec = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "steps": steps, "warmup": warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": wl.scaling, "data": wl.data,
        "config": wl.config(), "e2e": e2e, "gpu_launches": int(steps * wl.launches_per_step(dsa)),
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                     "traffic": scaled(profile_traffic(wl.traffic_profile), wl.traffic_scale()),
                     "note": wl.roofline_note(peak_kind)},
        "clocks": sampler.summary(),
    }
    if cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_baseline(wl, args, steps=wl.cpu_steps_default, rows=wl.cpu_rows_default)
    graphs.clear()
    return rec


# Named sub-records of the default line (N = 1): the rest of the reference's
# headline metric on its own configurations, each timed alone.
SUB_RECORDS = [
    ("sparse_mla_decode_b64_ctx128k", "decode", {"B": 64, "S": 131072}, 200),
    ("sparse_mla_decode_b16_ctx128k", "decode", {"B": 16, "S": 131072}, 200),
    ("sparse_mla_decode_b4_ctx128k", "decode", {"B": 4, "S": 131072}, 200),
    ("indexer_prefill_n65536", "indexer_prefill", {}, 5),
    ("sparse_prefill_t16384_ctx180k", "sparse_prefill", {}, 5),
]


def run_ours(args, world, rank, local):
    dsa = importlib.import_module("glm5-on-v100_b200")
    dev = torch.device("cuda", local)
    wl = WORKLOADS[args.workload]()
    e2e_steps = args.steps if args.workload in ("decode", "dsa_layer") else max(3, min(args.steps, 10))
    rec = measure(wl, dsa, args, world, rank, dev, args.steps, args.warmup, e2e_steps, cpu=True)
    par = (f"tp{world}: keys split {world} ways, heads {wl.H // world} per GPU, P2P top-k merge"
           if getattr(wl, "scaling", "weak") == "strong" and world > 1 else
           ("1 GPU" if world == 1 else f"dp{world} (independent work per rank)"))
    line = {"metric": rec["metric"], "value": rec["value"], "unit": rec["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
            "scaling": rec["scaling"], "vs_baseline": None, "dtype": "bf16", "data": rec["data"],
            "config": dict(rec["config"], parallelism=par), "e2e": rec["e2e"], "gpu_launches": rec["gpu_launches"],
            "roofline": rec["roofline"], "clocks": rec["clocks"]}
    if "cpu_baseline" in rec:
        line["cpu_baseline"] = rec["cpu_baseline"]
    del wl
    if world == 1 and args.workload == "dsa_layer" and not args.no_sub_records:
        subs = {}
        for name, kind, attrs, steps in SUB_RECORDS:
            torch.cuda.empty_cache()
            sw = WORKLOADS[kind]()
            for k, v in attrs.items():
                setattr(sw, k, v)
            sw.cpu_steps_default = 2
            r = measure(sw, dsa, args, world, rank, dev, steps, args.warmup,
                        steps if kind == "decode" else 3, cpu=True)
            r["n_gpus"] = 1
            subs[name] = r
            del sw
        line["sub_records"] = subs
        line["gpu_launches"] = rec["gpu_launches"] + sum(r["gpu_launches"] for r in subs.values())
    if rank == 0:
        print(json.dumps(line), flush=True)


def cpu_baseline(wl, args, steps=None, rows=None):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = rows or args.cpu_rows or wl.cpu_rows_default
    wl.cpu_setup(rows)
    wl.cpu_step()  # warm-up
    steps = steps or args.cpu_steps
    t0 = time.perf_counter()
    for _ in range(steps):
        wl.cpu_step()
    dt = time.perf_counter() - t0
    return {"value": wl.cpu_units() * steps / dt, "unit": wl.unit, "cores": torch.get_num_threads(), "kind": "port",
            "sample": wl.cpu_sample(steps)}


def run_reference(args, world, rank):
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]()
    steps, rows = args.steps, args.cpu_rows
    cb = cpu_baseline(wl, args, steps=steps, rows=rows)
    ms_per_step = 1e3 * wl.cpu_units() / cb["value"]
    line = {
        "metric": wl.metric, "value": cb["value"], "unit": wl.unit, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": wl.scaling,
        "vs_baseline": None, "dtype": "f32 (host)", "data": "synthetic", "impl": "reference",
        "config": dict(wl.config(), parallelism="host cores"),
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="dsa_layer")
    ap.add_argument("--cpu-rows", type=int, default=None, help="rows per CPU-baseline step")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-sub-records", action="store_true", help="default line without the per-config records")
    ap.add_argument("--batch", type=int, default=None, help="decode / decode-indexer rows per step")
    ap.add_argument("--ctx", type=int, default=None,
                    help="decode / decode-indexer / layer context length (smaller values make the ncu profiling case)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    for cls in (DecodeWorkload, IndexerDecodeWorkload, DecodeLayerWorkload, ShardedLayerWorkload):
        if args.ctx is not None:
            cls.S = args.ctx
        if args.batch is not None:
            cls.B = args.batch
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
