#!/usr/bin/env python
"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Headline step (configs[3] of the baseline): Llama-3-8B-shape causal prefill,
B=4, S=8192, Hq=32, Hkv=8, d=128, RoPE theta 5e5 on Q and K, bf16. At N GPUs the
8 kv-head groups are split N ways (each rank holds only its heads' Q/K/V) and the
output is all-gathered over NVLink (NCCL), overlapped with compute in batch
chunks. value = whole-job algorithmic causal TFLOP/s = 4*B*Hq*d*S(S+1)/2 / max
over ranks of the step time.

Secondary figures in the same line (``workloads``): configs[1] prefill d=64,
configs[2] paged decode and configs[4] speculative verify (HBM GB/s of
algorithmic K/V bytes), each with its roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

``--impl reference`` times the reference's own CPU path (its torch
``kernels.ref`` RoPE + fp32 attention, imported unmodified from the installed
reference, all host threads) on bounded samples of the headline workload and
prints the same line with "impl": "reference". ``cpu_baseline`` (and one per
secondary workload) times the same code, plus the reference's
``PagedKVCache.gather`` for the paged workloads, at 1 thread and at all cores.
Without an installed reference both fall back to the numpy restatement in
oracle/ and say so ("kind": "port").
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "custom-inference-engine_b200"
REF_ENV = "CIE_REFERENCE_ENGINE"


def reference_root() -> Path | None:
    """The installed reference (its ``kernels`` and ``engine`` packages), or None."""
    cands = [Path(os.environ[REF_ENV])] if os.environ.get(REF_ENV) else []
    cands.append(REPO / "baseline" / "_ref")
    for c in cands:
        if (c / "kernels" / "ref" / "rope_apply_ref.py").is_file() and \
                (c / "engine" / "cache" / "kv_cache.py").is_file():
            return c
    return None


def _path_product():
    """This repo's package (kernels, engine) on sys.path."""
    for p in (str(REPO), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)


def _path_reference(root: Path | None):
    """The reference's own packages (not this repo's) on sys.path; the oracle
    (under REPO) stays importable for the fallback."""
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    if root is not None and str(root) not in sys.path:
        sys.path.insert(0, str(root))

BASELINE = json.loads((REPO / "BASELINE.json").read_text())
METRIC = BASELINE["metric"]
THETA = 500000.0

HEADLINE = dict(name="cfg4_prefill_llama3_8b", B=4, Hq=32, Hkv=8, S=8192, d=128)
HEADLINE_FLOPS = 4.0 * 4 * 32 * 128 * 8192 * 8193 / 2
CFG2 = dict(name="cfg2_prefill_llama32_1b", B=8, Hq=32, Hkv=8, S=2048, d=64)
CFG3 = dict(name="cfg3_paged_decode", B=64, Hq=32, Hkv=8, M=1, d=64, lo=256, hi=8192, bs=16)
CFG5 = dict(name="cfg5_spec_verify", B=32, Hq=32, Hkv=8, M=5, d=128, lo=1024, hi=32768, bs=16)


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def _traffic(kind: str):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary."""
    p = REPO / "profiles" / "traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(kind)


def prefill_flops(B, Hq, S, d, M=None, N=None):
    M = S if M is None else M
    N = S if N is None else N
    # causal, bottom-right aligned: row i sees N - M + i + 1 keys
    vis = sum(min(N, N - M + i + 1) for i in range(M)) if M != N else S * (S + 1) // 2
    return 4.0 * B * Hq * d * vis


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU, sampled through NVML
    every 5 ms by a background thread while the timed region runs (a timed region
    of tens of ms gets several samples). Falls back to nvidia-smi at 200 ms when
    NVML is unavailable. Reads only; changes no setting."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None
        self.thread = None
        self.samples = []

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        prop = torch.cuda.get_device_properties(torch.cuda.current_device())
        bus = f"{prop.pci_domain_id:08X}:{prop.pci_bus_id:02X}:{prop.pci_device_id:02X}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def start(self):
        import threading

        try:
            nv, h = self._nvml_handle()
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - fall back to the nvidia-smi sampler
            return self._start_smi()
        self.stop_evt = threading.Event()
        names = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}

        def run():
            while not self.stop_evt.is_set():
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, [n for n, b in names.items() if bits & b]))
                except Exception:  # noqa: BLE001
                    pass
                self.stop_evt.wait(0.005)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def _start_smi(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=2)
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                        "source": "nvml"}
            reasons = sorted({r for _, rs in self.samples for r in rs})
            return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                    "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml, every 5 ms"}
        return self._stop_smi()

    def _stop_smi(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(idx=int(parts[0]), sm=float(parts[1]), smax=float(parts[2]),
                                 util=float(parts[4]), hw=parts[5], hwt=parts[6], swt=parts[7],
                                 pcap=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        loaded = [r for r in rows if r["util"] > 0] or rows
        if not loaded:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["smax"] for r in loaded), "reasons": sorted(reasons),
                "samples": len(loaded), "source": "nvidia-smi, every 200 ms"}


# ---------------------------------------------------------------- distributed
def init_dist():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    import torch

    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def l2_flush_buffer():
    import torch

    return torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")


# ---------------------------------------------------------------- prefill
class PrefillWorkload:
    """One rank's slice of a causal RoPE prefill (kv-head group sharding)."""

    def __init__(self, cfg, world, rank, seed=0, chunks=1, gather="peers"):
        import torch

        from engine.head_shard import local_heads, shard_heads
        from kernels import build_rope_cache

        self.cfg, self.world, self.rank = cfg, world, rank
        B, S, d = cfg["B"], cfg["S"], cfg["d"]
        self.shard = shard_heads(cfg["Hq"], cfg["Hkv"], world, rank)
        self.seed = seed
        q, k, v = self.full_inputs()
        # this rank's heads only (the full tensors are drawn identically on every
        # rank so that the gathered output can be checked against one GPU's)
        self.q = local_heads(q, self.shard, kv=False).contiguous()
        self.k = local_heads(k, self.shard, kv=True).contiguous()
        self.v = local_heads(v, self.shard, kv=True).contiguous()
        del q, k, v
        self.cos, self.sin = build_rope_cache(S, d, theta=THETA, device="cuda")
        self.scale = 1.0 / math.sqrt(d)
        self.out = torch.empty_like(self.q)
        self.chunks = chunks if world > 1 else 1
        if self.chunks < 1 or B % self.chunks:
            raise ValueError(f"--chunks {self.chunks} must divide the batch ({B})")
        # N > 1: the fused kernel writes every output tile into every rank's full
        # output over NVLink (symmetric memory); NCCL all-gather if that cannot be set up
        self.peer, self.gather = None, "none (1 GPU)"
        if world > 1:
            self.gather = "nccl all_gather_into_tensor, batch chunks"
            if gather == "peers":
                from engine.head_shard import PeerOutput

                try:
                    self.peer = PeerOutput((B, cfg["Hq"], S, d), torch.bfloat16, "cuda")
                    self.gather = "fused: output tiles stored to peers inside the kernel + peer barrier"
                except Exception as e:  # noqa: BLE001 - reported in the JSON line
                    self.gather = f"nccl (symmetric memory unavailable: {type(e).__name__}: {e})"
        self.flops_total = prefill_flops(B, cfg["Hq"], S, d)
        self.launches_per_step = 2  # rope(K) + attention
        self.kernel_ms = []

    def full_inputs(self):
        """All heads' Q, K, V (bf16, seeded, the same on every rank)."""
        import torch

        c = self.cfg
        g = torch.Generator(device="cuda").manual_seed(self.seed * 1000 + 17)
        shape_q = (c["B"], c["Hq"], c["S"], c["d"])
        shape_kv = (c["B"], c["Hkv"], c["S"], c["d"])
        return (torch.randn(shape_q, device="cuda", generator=g).to(torch.bfloat16),
                torch.randn(shape_kv, device="cuda", generator=g).to(torch.bfloat16),
                torch.randn(shape_kv, device="cuda", generator=g).to(torch.bfloat16))

    def assemble(self, outs):
        """The step's output in global head order, (B, Hq, S, d)."""
        import torch

        if self.world == 1:
            return torch.cat(outs, 0)
        if self.peer is not None:
            return outs[0]                         # already (B, Hq, S, d) on every rank
        g = torch.cat(outs, 1)                     # (W, B, hq, S, d), rank-major
        W, B, hq, S, d = g.shape
        return g.permute(1, 0, 2, 3, 4).reshape(B, W * hq, S, d)

    def check_against_one_gpu(self):
        """N > 1: the gathered output of one step must equal, bit for bit, the
        output of the whole problem on one GPU (every head runs the same kernel
        on the same inputs). Every rank takes the step; rank 0 compares."""
        import torch

        from kernels.flash_attention import apply_rotary, flash_attention

        got = self.assemble(self.step())
        torch.cuda.synchronize()
        res = None
        if self.rank == 0:
            q, k, v = self.full_inputs()
            want = flash_attention(q, apply_rotary(k, self.cos, self.sin), v, True, self.scale,
                                   rope=(self.cos, self.sin), rope_k=False)
            diff = (got.float() - want.float()).abs()
            res = {"bit_exact": bool(torch.equal(got, want)),
                   "max_abs_diff": float(diff.nan_to_num(nan=float("inf")).max()),
                   "what": "gathered (B, Hq, S, d) output of one step vs the same problem on "
                           "one GPU"}
            del q, k, v, want, diff
        del got
        torch.cuda.empty_cache()
        return res

    def step(self, events=None):
        """RoPE(K) -> attention (RoPE(Q) in-kernel) -> all-gather (N > 1)."""
        from engine.head_shard import gather_output
        from kernels.flash_attention import apply_rotary, flash_attention

        k_rot = apply_rotary(self.k, self.cos, self.sin)
        if events is not None:
            events[0].record()
        if self.peer is not None:
            full = self.peer.attention(self.q, k_rot, self.v, self.shard, True, self.scale,
                                       rope=(self.cos, self.sin), rope_k=False,
                                       on_kernel_done=(events[1].record if events is not None
                                                       else None))
            return [full]
        B = self.cfg["B"]
        per = B // self.chunks
        works, outs = [], []
        for c in range(self.chunks):
            sl = slice(c * per, (c + 1) * per)
            o = flash_attention(self.q[sl], k_rot[sl], self.v[sl], True, self.scale,
                                rope=(self.cos, self.sin), rope_k=False)
            if self.world > 1:
                g, w = gather_output(o, async_op=True)
                outs.append(g)
                works.append(w)
            else:
                outs.append(o)
        if events is not None:
            events[1].record()
        for w in works:
            w.wait()
        return outs


# ---------------------------------------------------------------- paged
class PagedWorkload:
    """paged decode / verify over random block tables.

    A decode step on one GPU's slice is short (~15 us at N = 8), shorter than the
    Python wrapper takes to launch it, so the step's paged_attention call is
    captured once in a CUDA graph and every step replays it, as a serving loop
    would; the events time the GPU work. The output gather (N > 1) stays eager.
    """

    def __init__(self, cfg, world, rank, seed=0, split_tokens=0, slice_of=0):
        import numpy as np
        import torch

        from engine.head_shard import shard_heads
        from kernels import build_rope_cache

        self.cfg, self.world, self.rank = cfg, world, rank
        B, M, d, bs = cfg["B"], cfg["M"], cfg["d"], cfg["bs"]
        # slice_of > 1 (one GPU, no collectives): rank 0's head slice of a slice_of-way job
        self.shard = shard_heads(cfg["Hq"], cfg["Hkv"], slice_of or world, rank)
        rng = np.random.default_rng(seed)
        ctx = rng.integers(cfg["lo"], cfg["hi"] + 1, size=B)
        lens = ctx + M
        nblk = (lens + bs - 1) // bs
        pool = int(nblk.sum())
        perm = rng.permutation(pool).astype(np.int32)
        tables = np.zeros((B, int(nblk.max())), np.int32)
        o = 0
        for i in range(B):
            tables[i, : nblk[i]] = perm[o: o + nblk[i]]
            o += nblk[i]
        g = torch.Generator(device="cuda").manual_seed(seed * 1000 + rank)
        hkv = self.shard.hkv
        self.k_pool = torch.randn(pool, bs, hkv, d, device="cuda", generator=g).to(torch.bfloat16)
        self.v_pool = torch.randn(pool, bs, hkv, d, device="cuda", generator=g).to(torch.bfloat16)
        self.q = torch.randn(B, self.shard.hq, M, d, device="cuda", generator=g).to(torch.bfloat16)
        self.tables = torch.from_numpy(tables).cuda()
        self.kv_lens = torch.from_numpy(lens.astype(np.int32)).cuda()
        self.cos, self.sin = build_rope_cache(int(lens.max()) + 1, d, theta=THETA, device="cuda")
        self.lens = lens
        H_all = cfg["Hkv"] // (slice_of or 1)
        self.bytes_total = (float(lens.sum()) * H_all * d * 2 * 2 +
                            2 * B * cfg["Hq"] // (slice_of or 1) * M * d * 2 +
                            tables.size * 4 * world + B * 4 * world)
        self.flops_total = float(sum(4.0 * cfg["Hq"] * d * sum(L - M + i + 1 for i in range(M))
                                     for L in lens))
        from kernels import _lib

        lib = _lib.load()
        ws = lib.cie_paged_attn_workspace(B, self.shard.hq, hkv, M, d, bs, tables.shape[1], 0)
        self.launches_per_step = 2 if ws > 0 else 1
        from kernels.flash_attention import paged_attention

        def call():
            return paged_attention(self.q, self.k_pool, self.v_pool, self.tables, self.kv_lens,
                                   True, rope=(self.cos, self.sin), split_tokens=split_tokens)

        call()  # first call outside the capture (kernel attributes, tensor maps)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = call()
        torch.cuda.synchronize()

    def step(self, events=None):
        from engine.head_shard import gather_output

        if events is not None:
            events[0].record()
        self.graph.replay()
        o = self.out
        if events is not None:
            events[1].record()
        if self.world > 1:
            return gather_output(o)
        return o


class Int8Workload:
    """Weight-only INT8 GEMMs of the engine's QKV projection (Llama-3-8B: K=4096,
    N=(32+2*8)*128=6144) for a decode batch of 64 tokens, int8 weights with
    per-channel scales, bf16 activations (kernels/int8_matmul.py), one call per
    layer for `layers` layers with their own weights (200 MB at 8 layers, more
    than L2, so every call streams its weights from HBM).

    A decode call takes ~15 us on the GPU, less than the Python wrapper needs to
    launch it, so the step's calls are captured once in a CUDA graph and each
    step replays it, as a decode loop would: the events time the GPU work."""

    M, N, K = 64, 6144, 4096

    def __init__(self, seed=0, layers=8):
        import torch

        from kernels.int8_matmul import int8_matmul

        g = torch.Generator(device="cuda").manual_seed(seed)
        self.layers = layers
        self.x = torch.randn(self.M, self.K, device="cuda", generator=g).to(torch.bfloat16)
        self.w = [torch.randint(-128, 128, (self.N, self.K), device="cuda", generator=g,
                                dtype=torch.int8) for _ in range(layers)]
        self.s = [torch.rand(self.N, device="cuda", generator=g) * 0.01 for _ in range(layers)]
        per_call = (self.N * self.K + self.M * self.K * 2 + self.M * self.N * 2 + self.N * 4)
        self.bytes_total = float(per_call * layers)
        self.flops_total = 2.0 * self.M * self.N * self.K * layers
        self.launches_per_step = 2 * layers
        for w, s in zip(self.w, self.s):
            int8_matmul(self.x, w, s)  # first calls outside capture (kernel attributes)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y = [int8_matmul(self.x, w, s) for w, s in zip(self.w, self.s)]
        torch.cuda.synchronize()

    def step(self, events=None):
        if events is not None:
            events[0].record()
        self.graph.replay()
        if events is not None:
            events[1].record()
        return self.y


def time_steps(wl, steps, warmup, world, flush=None):
    """W untimed steps, then exactly K timed steps between barriers; returns
    (max-over-ranks total ms, mean per-launch kernel ms from events)."""
    import torch

    for _ in range(warmup):
        wl.step()
    barrier(world)
    kernel_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                     for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if flush is None:
        start.record()
        for i in range(steps):
            wl.step(kernel_events[i])
        end.record()
        torch.cuda.synchronize()
        total = start.elapsed_time(end)
    else:
        # inputs smaller than L2: flush it between iterations, time each one
        total = 0.0
        for i in range(steps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            wl.step(kernel_events[i])
            e.record()
            torch.cuda.synchronize()
            total += s.elapsed_time(e)
    barrier(world)
    kms = sum(a.elapsed_time(b) for a, b in kernel_events) / steps
    return max_over_ranks(total, world), max_over_ranks(kms, world)


# ---------------------------------------------------------------- e2e
def e2e_prefill(cfg, world, rank, steps, warmup):
    """Through the public API with host buffers, every step: pinned H2D of this
    rank's Q/K/V, flash_attention (fused RoPE), the all-gather of the outputs
    (N > 1) and a D2H read of the whole result (each gathered batch element is
    read back by one rank, b % N).

    The step is pipelined per batch element the way a serving loop would run it:
    H2D copies on one stream, attention and the all-gather on the compute stream,
    D2H copies on a third, so the two PCIe directions and the tensor cores work
    at the same time (events keep each buffer from being overwritten before its
    consumer is done with it, across steps too).
    """
    import torch

    from engine.head_shard import gather_output, shard_heads
    from kernels import build_rope_cache
    from kernels.flash_attention import flash_attention

    B, S, d = cfg["B"], cfg["S"], cfg["d"]
    sh = shard_heads(cfg["Hq"], cfg["Hkv"], world, rank)
    g = torch.Generator().manual_seed(7 + rank)
    hq = torch.randn(B, sh.hq, S, d, generator=g).to(torch.bfloat16).pin_memory()
    hk = torch.randn(B, sh.hkv, S, d, generator=g).to(torch.bfloat16).pin_memory()
    hv = torch.randn(B, sh.hkv, S, d, generator=g).to(torch.bfloat16).pin_memory()
    hout = torch.empty(B, world, sh.hq, S, d, dtype=torch.bfloat16).pin_memory()
    dq, dk, dv = (torch.empty_like(t, device="cuda") for t in (hq, hk, hv))
    cos, sin = build_rope_cache(S, d, theta=THETA, device="cuda")
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    mine = [b for b in range(B) if b % world == rank]

    def ev():
        return torch.cuda.Event()

    in_ready = [ev() for _ in range(B)]     # H2D of element b landed
    in_free = [ev() for _ in range(B)]      # attention of element b no longer reads dq/dk/dv[b]
    out_ready = [ev() for _ in range(B)]    # gathered output of element b complete
    out_done = [ev() for _ in range(B)]     # D2H of element b finished
    for e in in_free + out_done:
        e.record(comp)
    keep = [None] * B

    def step():
        for b in range(B):
            with torch.cuda.stream(s_in):
                s_in.wait_event(in_free[b])
                dq[b].copy_(hq[b], non_blocking=True)
                dk[b].copy_(hk[b], non_blocking=True)
                dv[b].copy_(hv[b], non_blocking=True)
                in_ready[b].record(s_in)
            comp.wait_event(in_ready[b])
            o = flash_attention(dq[b:b + 1], dk[b:b + 1], dv[b:b + 1], True, 1.0 / math.sqrt(d),
                                rope=(cos, sin))
            in_free[b].record(comp)
            full = gather_output(o) if world > 1 else o.unsqueeze(0)  # (W, 1, hq, S, d)
            out_ready[b].record(comp)
            if b in mine:
                with torch.cuda.stream(s_out):
                    s_out.wait_event(out_ready[b])
                    hout[b].copy_(full[:, 0], non_blocking=True)
                    out_done[b].record(s_out)
                full.record_stream(s_out)
            keep[b] = full

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(comp)
    s_in.wait_stream(comp)  # no copy of the timed steps starts before the start event
    for _ in range(steps):
        step()
    for b in mine:
        comp.wait_event(out_done[b])
    e.record(comp)
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / steps, world)
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2 * world
    d2h = B * world * sh.hq * S * d * 2  # the whole output, read back once
    return prefill_flops(B, cfg["Hq"], S, d) / (ms * 1e-3) / 1e12, h2d, d2h


def time_all_gather(nbytes_per_rank, world, reps=10):
    """ms of one NCCL all_gather_into_tensor of nbytes_per_rank from every rank
    (CUDA events, max over ranks), with nothing else running."""
    import torch
    import torch.distributed as dist

    src = torch.empty(nbytes_per_rank, dtype=torch.uint8, device="cuda")
    dst = torch.empty(nbytes_per_rank * world, dtype=torch.uint8, device="cuda")
    dist.all_gather_into_tensor(dst, src)
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        dist.all_gather_into_tensor(dst, src)
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / reps, world)
    del src, dst
    return ms


def measure_pcie(world, mib=256, reps=5):
    """Pinned host<->device copy bandwidth of this rank while every rank copies at
    the same time (the condition the e2e leg runs in): GB/s H2D and D2H, max time
    over ranks. It bounds e2e: a step moves h2d + d2h bytes over these links."""
    import torch

    n = mib * 1024 * 1024
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    dev = torch.empty(n, dtype=torch.uint8, device="cuda")
    out = {}
    for name, fn in (("h2d", lambda: dev.copy_(host, non_blocking=True)),
                     ("d2h", lambda: host.copy_(dev, non_blocking=True))):
        fn()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(s.elapsed_time(e) / reps, world)
        out[f"{name}_gbs_per_rank"] = n / (ms * 1e-3) / 1e9
        out[f"{name}_gbs_all_ranks"] = world * n / (ms * 1e-3) / 1e9
    del host, dev
    return out


# ---------------------------------------------------------------- CPU baseline
def _host_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def _paged_lens(cfg, seed=0):
    """The paged workloads' history lengths (same draw as PagedWorkload)."""
    import numpy as np

    rng = np.random.default_rng(seed)
    ctx = rng.integers(cfg["lo"], cfg["hi"] + 1, size=cfg["B"])
    return (ctx + cfg["M"]).tolist()


class _CpuPath:
    """The reference's CPU path for one workload sample, on the host.

    ``backend == "reference"``: the reference's own torch code, imported from its
    installed copy (kernels/ref/rope_apply_ref.py:6-53 build_rope_cache +
    apply_rotary_ref, kernels/ref/flash_attention_ref.py:8-56 in fp32, and for
    the paged workloads engine/cache/kv_cache.py:141-165 PagedKVCache.gather on a
    CPU cache). ``backend == "port"``: the numpy restatement in oracle/.
    """

    def __init__(self, backend: str):
        self.backend = backend

    def prefill(self, cfg, rows=None):
        """One (batch element, query head) of a prefill config: RoPE(q, k) and
        causal fp32 attention over the last ``rows`` query rows (default all)."""
        S, d = cfg["S"], cfg["d"]
        rows = S if rows is None else rows
        scale = 1.0 / math.sqrt(d)
        if self.backend == "reference":
            import torch
            from kernels.ref import apply_rotary_ref, build_rope_cache, flash_attention_ref

            g = torch.Generator().manual_seed(0)
            q = torch.randn(1, 1, rows, d, generator=g).bfloat16().float()
            k = torch.randn(1, 1, S, d, generator=g).bfloat16().float()
            v = torch.randn(1, 1, S, d, generator=g).bfloat16().float()
            cos, sin = build_rope_cache(S, d, theta=THETA)
            qpos = torch.arange(S - rows, S)

            def step():
                qr = apply_rotary_ref(q, cos, sin, positions=qpos)
                kr = apply_rotary_ref(k, cos, sin)
                flash_attention_ref(qr, kr, v, causal=True, scale=scale)
        else:
            import numpy as np

            import oracle

            rng = np.random.default_rng(0)
            c, s_ = oracle.build_rope_cache(S, d, THETA)
            q = oracle.bf16_round(rng.standard_normal((1, 1, rows, d), dtype=np.float32))
            k = oracle.bf16_round(rng.standard_normal((1, 1, S, d), dtype=np.float32))
            v = oracle.bf16_round(rng.standard_normal((1, 1, S, d), dtype=np.float32))

            def step():
                qr = oracle.apply_rotary(q, c, s_, np.arange(S - rows, S))
                kr = oracle.apply_rotary(k, c, s_)
                oracle.attention(qr, kr, v, causal=True, scale=scale)
        work = prefill_flops(1, 1, S, d, M=rows, N=S) / 1e12
        what = (f"{'all' if rows == S else f'last {rows}'} query rows of one (batch, head) of "
                f"{cfg['name']}")
        return step, work, "TFLOP/s", what

    def paged(self, cfg, n_seq):
        """``n_seq`` sequences of a paged config: gather each history from a paged
        cache, RoPE(q) at its positions, causal fp32 attention of all Hq heads."""
        lens = _paged_lens(cfg)[:n_seq]
        Hq, Hkv, M, d, bs = cfg["Hq"], cfg["Hkv"], cfg["M"], cfg["d"], cfg["bs"]
        scale = 1.0 / math.sqrt(d)
        if self.backend == "reference":
            import torch
            from engine.cache.kv_cache import KVCacheConfig, PagedKVCache
            from kernels.ref import apply_rotary_ref, build_rope_cache, flash_attention_ref

            nblk = sum((L + bs - 1) // bs for L in lens)
            cache = PagedKVCache(KVCacheConfig(num_layers=1, num_kv_heads=Hkv, head_dim=d,
                                               num_blocks=nblk, block_size=bs,
                                               dtype=torch.bfloat16, device="cpu"))
            g = torch.Generator().manual_seed(0)
            tables = []
            for L in lens:
                t = cache.new_sequence()
                cache.append(0, t, torch.randn(L, Hkv, d, generator=g).bfloat16(),
                             torch.randn(L, Hkv, d, generator=g).bfloat16())
                tables.append(t)
            qs = [torch.randn(1, Hq, M, d, generator=g).bfloat16().float() for _ in lens]
            cos, sin = build_rope_cache(max(lens) + 1, d, theta=THETA)

            def step():
                for t, q, L in zip(tables, qs, lens):
                    k, v = cache.gather(0, t)
                    k = k.float().transpose(0, 1).unsqueeze(0)
                    v = v.float().transpose(0, 1).unsqueeze(0)
                    qr = apply_rotary_ref(q, cos, sin, positions=torch.arange(L - M, L))
                    flash_attention_ref(qr, k, v, causal=True, scale=scale)
        else:
            import numpy as np

            import oracle

            rng = np.random.default_rng(0)
            c, s_ = oracle.build_rope_cache(max(lens) + 1, d, THETA)
            hist = [(oracle.bf16_round(rng.standard_normal((1, Hkv, L, d), dtype=np.float32)),
                     oracle.bf16_round(rng.standard_normal((1, Hkv, L, d), dtype=np.float32)))
                    for L in lens]
            qs = [oracle.bf16_round(rng.standard_normal((1, Hq, M, d), dtype=np.float32))
                  for _ in lens]

            def step():
                for (k, v), q, L in zip(hist, qs, lens):
                    qr = oracle.apply_rotary(q, c, s_, np.arange(L - M, L))
                    oracle.attention(qr, k.copy(), v.copy(), causal=True, scale=scale)
        work = sum(lens) * Hkv * d * 2 * 2 / 1e9
        return step, work, "GB/s", f"{n_seq} of the {cfg['B']} sequences of {cfg['name']}"


def _time_step(step, seconds: float, max_reps: int = 50):
    step()  # warm-up (allocations, thread pool)
    reps, t0 = 0, time.perf_counter()
    while True:
        step()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= max_reps:
            return el / reps


CPU_SAMPLES = {"cfg2": ("prefill", CFG2, None), "cfg4": ("prefill", HEADLINE, None),
               "cfg3": ("paged", CFG3, 8), "cfg5": ("paged", CFG5, 4)}


def cpu_worker(names, seconds: float):
    """Run in a child process whose sys.path holds the reference, not this repo's
    package: every named CPU sample at 1 thread and at all host cores."""
    root = reference_root()
    _path_reference(root)
    import torch

    path = _CpuPath("reference" if root is not None else "port")
    cores = _host_cores()
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:
        threadpool_limits = None
    out = {}
    for name in names:
        kind, cfg, n = CPU_SAMPLES[name]
        step, work, unit, what = path.prefill(cfg) if kind == "prefill" else path.paged(cfg, n)
        vals = {}
        for threads in sorted({1, cores}):
            torch.set_num_threads(threads)
            if threadpool_limits is not None:
                threadpool_limits(threads)
            vals[threads] = work / _time_step(step, seconds)
        out[name] = {"unit": unit, "values": vals, "sample": what, "kind": path.backend,
                     "cores": cores}
    print(json.dumps(out), flush=True)


def cpu_baselines(names, seconds: float = 1.0) -> dict:
    """The CPU samples, measured in a child process (the reference's packages and
    this repo's share top-level names, so they cannot share one interpreter)."""
    env = {k: v for k, v in os.environ.items()
           if k not in ("OMP_NUM_THREADS", "MKL_NUM_THREADS", "CUDA_VISIBLE_DEVICES")}
    env["CUDA_VISIBLE_DEVICES"] = ""
    res = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--cpu-worker",
                          ",".join(names), "--cpu-seconds", str(seconds)],
                         capture_output=True, text=True, env=env, timeout=600)
    if res.returncode != 0:
        raise RuntimeError(f"CPU baseline worker failed:\n{res.stderr[-2000:]}")
    raw = json.loads(res.stdout.strip().splitlines()[-1])
    out = {}
    for name, r in raw.items():
        vals = {int(k): v for k, v in r["values"].items()}
        cores = r["cores"]
        out[name] = {"value": vals[cores], "unit": r["unit"], "cores": cores,
                     "value_1_thread": vals[1], "kind": r["kind"],
                     "sample": r["sample"] + (" (the reference's torch kernels.ref"
                                              + (" + PagedKVCache.gather" if "paged" in
                                                 CPU_SAMPLES[name][0] else "")
                                              + ", installed copy)" if r["kind"] == "reference"
                                              else " (numpy restatement in oracle/)")
                     + f"; value at {cores} threads, value_1_thread at 1"}
    return out


def run_reference(args, world, rank):
    """--impl reference: the reference's own CPU path on rank 0, all host threads.

    Each step is one (batch element, query head) of the headline workload, the
    unit the per-step sample scales with: RoPE of q and k and the causal fp32
    attention, through the reference's kernels.ref (numpy port if the reference
    is not installed)."""
    if rank != 0:
        return
    root = reference_root()
    _path_reference(root)
    import torch

    cores = _host_cores()
    torch.set_num_threads(cores)
    path = _CpuPath("reference" if root is not None else "port")
    step, work, unit, what = path.prefill(HEADLINE)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    val = work * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": HEADLINE["name"] + " (bounded CPU sample per step)",
                   "B": HEADLINE["B"], "S": HEADLINE["S"], "Hq": HEADLINE["Hq"],
                   "Hkv": HEADLINE["Hkv"], "d": HEADLINE["d"]},
        "cpu_baseline": {"value": val, "unit": unit, "cores": cores, "kind": path.backend,
                         "sample": f"per step: {what}"
                                   + (" (the reference's torch kernels.ref, installed copy)"
                                      if path.backend == "reference" else
                                      " (numpy restatement in oracle/)")},
        "e2e": {"value": val, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_only(args, world, rank):
    """One workload, no extras: the command line the ncu captures profile."""
    cfg = {"cfg2": CFG2, "cfg3": CFG3, "cfg4": HEADLINE, "cfg5": CFG5}.get(args.only, {})
    cfg = dict(cfg)
    if args.batch:
        cfg["B"] = args.batch
    if args.only == "int8":
        wl = Int8Workload()
        unit, work = "GB/s", wl.bytes_total / 1e9
        cfg = {"name": "f4_int8_qkv_decode", "B": wl.M}
    elif args.only in ("cfg2", "cfg4"):
        wl = PrefillWorkload(cfg, world, rank)
        unit, work = "TFLOP/s", wl.flops_total / 1e12
    else:
        wl = PagedWorkload(cfg, world, rank, split_tokens=args.split, slice_of=args.slice_of)
        unit, work = "GB/s", wl.bytes_total / 1e9
    total, kms = time_steps(wl, args.steps, args.warmup, world)
    if rank == 0:
        print(json.dumps({"workload": cfg["name"], "B": cfg["B"], "unit": unit,
                          "value": work / (total / args.steps * 1e-3),
                          "kernel_value": work / world / (kms * 1e-3), "kernel_ms": kms,
                          "ms_per_step": total / args.steps}), flush=True)


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--only", choices=["cfg2", "cfg3", "cfg4", "cfg5", "int8"],
                    help="time one workload only (used for ncu captures)")
    ap.add_argument("--chunks", type=int, default=0,
                    help="N > 1: batch chunks whose all-gather overlaps the next chunk's "
                         "attention (0: the measured default)")
    ap.add_argument("--gather", choices=["peers", "nccl"], default="peers",
                    help="N > 1: output all-gather fused into the kernel over peer memory "
                         "(default) or NCCL all_gather_into_tensor")
    ap.add_argument("--batch", type=int, default=0,
                    help="with --only: override the batch size (smaller ncu captures)")
    ap.add_argument("--split", type=int, default=0,
                    help="with --only cfg3/cfg5: split-KV partition size (0: automatic)")
    ap.add_argument("--slice-of", type=int, default=0,
                    help="with --only cfg3/cfg5 on one GPU: time rank 0's head slice of an "
                         "N-way job")
    ap.add_argument("--cpu-worker", default="", help=argparse.SUPPRESS)
    ap.add_argument("--cpu-seconds", type=float, default=1.0, help=argparse.SUPPRESS)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.cpu_worker:
        cpu_worker(args.cpu_worker.split(","), args.cpu_seconds)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return

    _path_product()
    import torch

    world, rank, _ = init_dist()
    peaks = _peaks()
    from kernels import _lib

    _lib.device_status(clear=True)
    if args.only:
        run_only(args, world, rank)
        return

    # ---------------- headline
    # measured: 4 chunks best at N <= 4 (the gather hides behind later chunks), 1 at N = 8
    # (the gather dominates and smaller launches only lose waves)
    wl = PrefillWorkload(HEADLINE, world, rank, chunks=args.chunks or (4 if world <= 4 else 1),
                         gather=args.gather)
    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
    total_ms, kern_ms = time_steps(wl, args.steps, args.warmup, world)
    clk = clocks.stop() if rank == 0 else None
    ms_step = total_ms / args.steps
    value = wl.flops_total / (ms_step * 1e-3) / 1e12
    # the dominant kernel: attention launches of one step (all chunks), per rank
    flops_rank = wl.flops_total / world
    achieved = flops_rank / (kern_ms * 1e-3) / 1e12
    traffic = _traffic("prefill_cfg4")
    roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16"],
            "frac_of_sustained": achieved / peaks["bf16_sustained"],
            "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
            "traffic": traffic if world == 1 else None,
            "kernel": "prefill_attn_kernel<128,bf16> (tcgen05)", "kernel_ms": kern_ms}
    launches = args.steps * ((3 if wl.peer is not None else 1 + wl.chunks) if world > 1 else 2)
    gather_mode = wl.gather
    check = wl.check_against_one_gpu() if world > 1 else None
    # scaling, split: the attention launches alone (with their in-kernel peer copies
    # on the fused path) and, at N > 1, an NCCL all-gather of this rank's output
    # timed alone (the collective the fused path replaces)
    split = {"kernel_only_value": wl.flops_total / (kern_ms * 1e-3) / 1e12,
             "kernel_ms": kern_ms, "step_ms": ms_step}
    if world > 1:
        split["nccl_all_gather_alone_ms"] = time_all_gather(wl.q.numel() * 2, world)
        split["note"] = ("kernel_only_value: whole-job TFLOP/s if a step were only the "
                         "attention launches (max over ranks); on the fused path they include "
                         "the NVLink copies of the output")
    del wl
    torch.cuda.empty_cache()

    # ---------------- secondary workloads
    workloads = {}
    if not args.no_secondary:
        flush = l2_flush_buffer()
        w2 = PrefillWorkload(CFG2, world, rank)
        t2, k2 = time_steps(w2, max(20, args.steps // 4), args.warmup, world, flush=flush)
        n2 = max(20, args.steps // 4)
        a2 = w2.flops_total / world / (k2 * 1e-3) / 1e12
        workloads[CFG2["name"]] = {
            "value": w2.flops_total / (t2 / n2 * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": t2 / n2, "l2": "flushed between iterations (inputs < L2)",
            "roofline": {"bound": "tensor", "achieved": a2, "peak": peaks["bf16"],
                         "frac": a2 / peaks["bf16"], "traffic": _traffic("prefill_cfg2")}}
        del w2, flush
        torch.cuda.empty_cache()
        for cfg in (CFG3, CFG5):
            w = PagedWorkload(cfg, world, rank)
            n = max(50, args.steps)
            t, kms = time_steps(w, n, args.warmup, world)
            gbs = w.bytes_total / (t / n * 1e-3) / 1e9
            ach = w.bytes_total / world / (kms * 1e-3) / 1e9
            workloads[cfg["name"]] = {
                "value": gbs, "unit": "GB/s", "ms_per_step": t / n,
                "tflops": w.flops_total / (t / n * 1e-3) / 1e12,
                "kv_bytes": w.bytes_total, "l2": "inputs larger than L2",
                "timing": "CUDA graph replay of the step's paged_attention call"
                          + ("; NCCL gather of the outputs eager" if world > 1 else ""),
                "roofline": {"bound": "hbm", "achieved": ach, "peak": peaks["hbm"],
                             "frac": ach / peaks["hbm"], "unit": "GB/s",
                             "traffic": _traffic(cfg["name"]) if world == 1 else None,
                             "kernel_ms": kms}}
            del w
            torch.cuda.empty_cache()

        if world == 1:
            w8 = Int8Workload()
            n8 = max(20, args.steps // 4)
            t8, k8 = time_steps(w8, n8, args.warmup, world)
            workloads["f4_int8_qkv_decode"] = {
                "value": w8.bytes_total / (t8 / n8 * 1e-3) / 1e9, "unit": "GB/s",
                "ms_per_step": t8 / n8, "tflops": w8.flops_total / (t8 / n8 * 1e-3) / 1e12,
                "shape": {"M": w8.M, "N": w8.N, "K": w8.K, "layers": w8.layers},
                "l2": "inputs larger than L2 (one weight matrix per layer, 200 MB per step)",
                "timing": "one CUDA graph replay of the step's int8_matmul calls",
                "roofline": {"bound": "hbm", "achieved": w8.bytes_total / (k8 * 1e-3) / 1e9,
                             "peak": peaks["hbm"],
                             "frac": w8.bytes_total / (k8 * 1e-3) / 1e9 / peaks["hbm"],
                             "unit": "GB/s", "kernel_ms": k8,
                             "kernel": "int8_gemv_kernel<bf16,64> (tcgen05, A in TMEM) + "
                                       "split-K reduce, per layer",
                             "traffic_per_call": _traffic("f4_int8_qkv_decode")}}
            del w8
            torch.cuda.empty_cache()

    # ---------------- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        n = max(5, min(args.steps, 20))
        ev, h2d, d2h = e2e_prefill(HEADLINE, world, rank, n, 2)
        pcie = measure_pcie(world)
        # the copies alone, at the bandwidth every rank gets while all copy at once,
        # bound the e2e step from below (H2D and D2H overlap each other and the math)
        t_copy = max(h2d / (pcie["h2d_gbs_all_ranks"] * 1e9), d2h / (pcie["d2h_gbs_all_ranks"] * 1e9))
        e2e = {"value": ev, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": n, "pcie": pcie,
               "copy_bound_value": HEADLINE_FLOPS / t_copy / 1e12}

    status = _lib.device_status(clear=True)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        names = ["cfg4"] + ([] if args.no_secondary else ["cfg2", "cfg3", "cfg5"])
        cpus = cpu_baselines(names)
        cpu = cpus.pop("cfg4")
        for name, c in cpus.items():
            key = {"cfg2": CFG2, "cfg3": CFG3, "cfg5": CFG5}[name]["name"]
            if key in workloads:
                workloads[key]["cpu_baseline"] = c

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) rounded to bf16; RoPE theta 5e5; "
                    "seeded random-permutation block tables",
            "config": {"workload": HEADLINE["name"] + ": causal GQA prefill + fused RoPE",
                       "B": HEADLINE["B"], "S": HEADLINE["S"], "Hq": HEADLINE["Hq"],
                       "Hkv": HEADLINE["Hkv"], "d": HEADLINE["d"],
                       "parallelism": f"kv-head groups / {world}; output gather: {gather_mode}"
                       if world > 1 else "1 GPU",
                       "l2": "inputs larger than L2 (402 MB per step)"},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": launches, "device_status": status, "workloads": workloads,
        }
        line["scaling_split"] = split
        if check is not None:
            line["multi_gpu_check"] = check
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
