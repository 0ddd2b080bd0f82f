#!/usr/bin/env python
"""Benchmark of PaceServe's per-layer op chain on B200 (the headline workload).

One step = one pass of the Llama-3-8B 32-layer op sequence over one Sarathi
mixed batch of T=512 tokens (a 448-token prefill chunk at positions 0..447 plus
64 decode tokens at positions uniform in 1..8191), bf16 activations, fp32
cos/sin cache:
    per layer: rms_norm (layer 0) or fused_add_rms_norm (input norm),
               rotary_embedding (neox, 32 q / 8 kv heads x 128 on the q/k views
               of a fused qkv tensor), fused_add_rms_norm (post-attention),
               silu_and_mul (intermediate 14336).
Every layer owns distinct buffers (2.1 GB per step), far more than the 126 MB
L2, so no L2 flush is needed between steps.  The step is captured once as a
CUDA graph; `value` times graph replays with inputs resident in HBM.  `e2e`
drives the same chain eagerly through the public ops (the engine's call path)
with a host->device copy of the step's inputs (positions, initial hidden
states) and a device->host read of its output, every step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (under torchrun): N independent replicas, one per GPU (the op chain
does not shard), value = aggregate tokens/s over max-over-ranks time; with N
>= 2 the LP->HP KV promotion is also measured on rank pairs (0->1, 2->3, ...).
--impl reference: the reference's CPU formulas (the oracle port) on the host
cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Layer-op chain tokens/s & % HBM peak; LP→HP KV-promotion GB/s vs NVLink"
UNIT = "tokens/s"
T_PREFILL, T_DECODE = 448, 64
T = T_PREFILL + T_DECODE
H, I, NQ, NKV, HD, L = 4096, 14336, 32, 8, 128, 32
MAX_POS, THETA, EPS = 8192, 500000.0, 1e-5
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
NOMINAL_HBM_GBS = 7700.0  # B200 HGX HBM3e figure; the roofline uses the measured copy peak

# Algorithmic bytes (bf16 activations, fp32 cos/sin cache), per launch at T tokens
B_RMS = 4 * H * T + 2 * H
B_FUSED = 8 * H * T + 2 * H
B_ROPE = 4 * (NQ + NKV) * HD * T + T * HD * 4 + 8 * T
B_SILU = 6 * I * T
B_STEP = B_RMS + B_ROPE + B_FUSED + B_SILU + (L - 1) * (B_FUSED + B_ROPE + B_FUSED + B_SILU)
LAUNCHES_PER_STEP = 4 * L
TIMED_BLOCKS = 5  # timed blocks of K steps each; the line reports the median block

WORKLOAD = (
    "Llama-3-8B 32-layer op chain (rms_norm/fused_add_rms_norm, neox rope 32/8x128 fp32 cache, "
    "fused_add_rms_norm, silu_and_mul I=14336), Sarathi mixed batch T=512 "
    "(448 prefill @0..447 + 64 decode @U[1,8191]), bf16"
)


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
                "source": "fallback"}


def ncu_traffic(kernel_key: str):
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/ncu_traffic.txt:
    lines `<kernel_key> <bytes_per_launch>`), or None."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == kernel_key:
                return int(float(parts[1]))
    except OSError:
        pass
    return None


# --------------------------------------------------------------- clocks --
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.period = period_s
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nvml = pynvml
            try:  # match the CUDA device to its NVML handle by PCI bus id
                bus = torch.cuda.get_device_properties(device_index).pci_bus_id
                dom = torch.cuda.get_device_properties(device_index).pci_domain_id
                dev = torch.cuda.get_device_properties(device_index).pci_device_id
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0")
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
                self.reasons |= int(n.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        names = [k for k, bit in self.REASONS.items() if self.reasons & bit and k != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# --------------------------------------------------------------- chain --
def make_positions(gen, device):
    import torch

    pre = torch.arange(T_PREFILL, dtype=torch.int64)
    dec = torch.randint(1, MAX_POS, (T_DECODE,), generator=gen, dtype=torch.int64)
    return torch.cat([pre, dec]).to(device)


def rope_cache(device, max_pos: int = MAX_POS):
    """cos/sin cache [max_pos, HD] in fp32: [cos | sin] of pos * theta^(-2i/HD)."""
    import torch

    inv = 1.0 / (THETA ** (torch.arange(0, HD, 2, dtype=torch.float64) / HD))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], -1).float().to(device)


def build_chain(device, seed=0, tokens=None):
    """The 32 layers' buffers.  tokens=None: the Sarathi batch (448 prefill + 64
    decode tokens); otherwise a pure decode batch of `tokens` tokens at
    positions uniform in [1, MAX_POS)."""
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    cpu_gen = torch.Generator().manual_seed(seed)
    T = tokens or globals()["T"]

    def rn(*shape, mean=0.0, std=1.0):
        return (torch.randn(*shape, generator=gen, device=device) * std + mean).to(torch.bfloat16)

    layers = []
    for l in range(L):
        b = {
            "hidden": rn(T, H),
            "w_in": rn(H, mean=1.0, std=0.02),
            "qkv": rn(T, (NQ + 2 * NKV) * HD),
            "attn": rn(T, H),
            "residual2": rn(T, H),
            "w_post": rn(H, mean=1.0, std=0.02),
            "gate_up": rn(T, 2 * I),
            "act": torch.empty(T, I, dtype=torch.bfloat16, device=device),
        }
        if l == 0:
            b["normed"] = torch.empty(T, H, dtype=torch.bfloat16, device=device)
        else:
            b["residual"] = rn(T, H)
        b["q"] = b["qkv"][:, : NQ * HD]
        b["k"] = b["qkv"][:, NQ * HD: (NQ + NKV) * HD]
        layers.append(b)
    if tokens:
        pos = torch.randint(1, MAX_POS, (T,), generator=cpu_gen, dtype=torch.int64).to(device)
    else:
        pos = make_positions(cpu_gen, device)
    return {"layers": layers, "positions": pos, "cache": rope_cache(device), "tokens": T}


def run_chain(ch, ops) -> None:
    ln, pe, act = ops
    pos, cache = ch["positions"], ch["cache"]
    for l, b in enumerate(ch["layers"]):
        if l == 0:
            ln.rms_norm(b["normed"], b["hidden"], b["w_in"], EPS)
        else:
            ln.fused_add_rms_norm(b["hidden"], b["residual"], b["w_in"], EPS)
        pe.rotary_embedding(pos, b["q"], b["k"], HD, cache, True)
        ln.fused_add_rms_norm(b["attn"], b["residual2"], b["w_post"], EPS)
        act.silu_and_mul(b["act"], b["gate_up"])


def capture(fn):
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_replays(g, steps, warmup, sampler=None) -> float:
    """Milliseconds for `steps` replays (after `warmup`), CUDA events on the replay stream."""
    import torch

    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        e1.synchronize()
    return e0.elapsed_time(e1)


def time_blocks(g, steps, warmup, blocks, sampler=None, ws=1):
    """Milliseconds of each of `blocks` timed blocks of exactly `steps` graph
    replays, after `warmup` replays.  Each block is bracketed by a barrier (N > 1)
    and a device synchronisation, timed with CUDA events on the replay stream,
    and reduced to the max over ranks."""
    import torch

    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    ctx = sampler if sampler is not None else _Null()
    out = []
    with ctx:
        for _ in range(blocks):
            if ws > 1:
                import torch.distributed as dist

                dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                g.replay()
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            if ws > 1:
                t = torch.tensor([ms], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = t.item()
            out.append(ms)
    return out


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def per_op_times(ch, ops, reps=20):
    """Each op alone: a graph of its 32 launches over the 32 layers' buffers."""
    ln, pe, act = ops
    pos, cache = ch["positions"], ch["cache"]
    lay = ch["layers"]
    fns = {
        "rms_norm": (lambda: [ln.rms_norm(b["act"][:, :H], b["hidden"], b["w_in"], EPS) for b in lay],
                     B_RMS),
        "fused_add_rms_norm": (lambda: [ln.fused_add_rms_norm(b["attn"], b["residual2"], b["w_post"], EPS)
                                        for b in lay], B_FUSED),
        "rotary_embedding": (lambda: [pe.rotary_embedding(pos, b["q"], b["k"], HD, cache, True)
                                      for b in lay], B_ROPE),
        "silu_and_mul": (lambda: [act.silu_and_mul(b["act"], b["gate_up"]) for b in lay], B_SILU),
    }
    out = {}
    for name, (fn, nbytes) in fns.items():
        g = capture(fn)
        ms = time_replays(g, reps, 3)
        us = ms * 1e3 / (reps * L)
        out[name] = {"us_per_launch": round(us, 3), "bytes_per_launch": nbytes,
                     "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
        del g
    return out


def e2e_chain(chs, ops, steps, warmup, ws=1):
    """Public-API path, pipelined the way a serving engine runs it: step i uses chain
    state i % 2 (`chs` holds two); its inputs go host -> device on an H2D stream
    from page-locked memory, the ops run eagerly (pybind -> C ABI) on the compute
    stream, and its result -- the last layer's residual stream [T, H], what a layer
    hands to the next -- goes device -> host on a D2H stream, so the copies of
    one step overlap the ops of the next.  Events order every reuse of a buffer.
    Every step's copies lie inside the timed region.  With ws > 1 every rank runs
    it between barriers; the time is the max over ranks and the value the whole
    job's tokens/s."""
    import torch

    dev = chs[0]["positions"].device
    comp = torch.cuda.current_stream()
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()
    h_pos = [c["positions"].cpu().pin_memory() for c in chs]
    h_hidden = [c["layers"][0]["hidden"].cpu().pin_memory() for c in chs]
    h_out = [torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True) for _ in chs]
    comp_done = [torch.cuda.Event() for _ in chs]
    d2h_done = [torch.cuda.Event() for _ in chs]
    for e in comp_done + d2h_done:
        e.record(comp)

    def step(i):
        k = i % len(chs)
        ch = chs[k]
        h2d_done = torch.cuda.Event()
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(comp_done[k])  # the previous step on this state read its inputs
            ch["positions"].copy_(h_pos[k], non_blocking=True)
            ch["layers"][0]["hidden"].copy_(h_hidden[k], non_blocking=True)
            h2d_done.record(h2d_s)
        comp.wait_event(h2d_done)
        comp.wait_event(d2h_done[k])  # ... and its output has been copied out
        run_chain(ch, ops)
        comp_done[k].record(comp)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(comp_done[k])
            h_out[k].copy_(ch["layers"][-1]["residual2"], non_blocking=True)
            d2h_done[k].record(d2h_s)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()
        torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    h2d_s.wait_event(e0)
    d2h_s.wait_event(e0)
    for i in range(steps):
        step(i)
    for e in d2h_done:
        comp.wait_event(e)
    e1.record(comp)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return {"value": round(ws * T / (ms * 1e-3), 1), "unit": UNIT,
            "h2d_bytes_per_step": h_pos[0].numel() * 8 + h_hidden[0].numel() * 2,
            "d2h_bytes_per_step": h_out[0].numel() * 2, "ms_per_step": round(ms, 4),
            "steps": steps,
            "path": "eager calls of paceserve_b200 ops (pybind -> C ABI); inputs in and the "
                    "last layer's residual stream out every step, on copy streams "
                    "overlapping the next step's ops"}


def e2e_breakdown(chs, ops, steps, warmup, ws=1):
    """What limits the e2e number: the same eager chain with no host copies
    (launch_only: the host's pybind -> C-ABI calls and the GPU work), and the
    host copies alone with no ops (copies_only: the same H2D/D2H bytes per step
    on the copy streams).  Each timed like e2e (events, max over ranks)."""
    import torch

    dev = chs[0]["positions"].device
    comp = torch.cuda.current_stream()
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()
    h_pos = [c["positions"].cpu().pin_memory() for c in chs]
    h_hidden = [c["layers"][0]["hidden"].cpu().pin_memory() for c in chs]
    h_out = [torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True) for _ in chs]

    def timed(step):
        for i in range(warmup):
            step(i)
        torch.cuda.synchronize(dev)
        if ws > 1:
            import torch.distributed as dist

            dist.barrier()
            torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record(comp)
        h2d_s.wait_event(e0)
        d2h_s.wait_event(e0)
        for i in range(steps):
            step(i)
        host_ms = (time.perf_counter() - t0) * 1e3 / steps
        comp.wait_stream(h2d_s)
        comp.wait_stream(d2h_s)
        e1.record(comp)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        if ws > 1:
            t = torch.tensor([ms, host_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, host_ms = t[0].item(), t[1].item()
        return ms, host_ms

    def launches(i):
        run_chain(chs[i % len(chs)], ops)

    def copies(i):
        k = i % len(chs)
        with torch.cuda.stream(h2d_s):
            chs[k]["positions"].copy_(h_pos[k], non_blocking=True)
            chs[k]["layers"][0]["hidden"].copy_(h_hidden[k], non_blocking=True)
        with torch.cuda.stream(d2h_s):
            h_out[k].copy_(chs[k]["layers"][-1]["residual2"], non_blocking=True)

    ms_l, host_l = timed(launches)
    ms_c, _ = timed(copies)
    nbytes = h_pos[0].numel() * 8 + h_hidden[0].numel() * 2 + h_out[0].numel() * 2
    return {"launch_only": {"ms_per_step": round(ms_l, 4), "value": round(ws * T / (ms_l * 1e-3), 1),
                            "host_ms_per_step": round(host_l, 4),
                            "host_us_per_call": round(host_l * 1e3 / LAUNCHES_PER_STEP, 3)},
            "copies_only": {"ms_per_step": round(ms_c, 4), "bytes_per_step": nbytes,
                            "gbs_per_gpu": round(nbytes / (ms_c * 1e-3) / 1e9, 1)},
            "steps": steps}


# ------------------------------------------------------------ CPU oracle --
def cpu_chain_run(steps: int, warmup: int, budget_s: float):
    """The reference's formulas (the oracle port) on the host cores, `steps` timed
    steps after `warmup`: a step is one pass of the 32-layer op chain at T=512
    bf16 (layer 0: rms_norm; layers 1..31: fused_add_rms_norm, rope,
    fused_add_rms_norm, silu_and_mul), all host threads.  When `steps` full
    chains would take longer than `budget_s`, each step is a bounded sample of
    the first layers of the chain, scaled to 32 layers (stated in `sample`)."""
    import torch

    from oracle import ops_ref

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)

    def rn(*shape, mean=0.0, std=1.0):
        return (torch.randn(*shape, generator=g) * std + mean).bfloat16()

    bufs = {"hidden": rn(T, H), "residual": rn(T, H), "w_in": rn(H, mean=1, std=0.02),
            "qkv": rn(T, (NQ + 2 * NKV) * HD), "attn": rn(T, H), "residual2": rn(T, H),
            "w_post": rn(H, mean=1, std=0.02), "gate_up": rn(T, 2 * I)}
    pos = make_positions(g, "cpu")
    cache = rope_cache("cpu")

    def chain(layers: int):
        for layer in range(layers):
            ops_ref.chain_layer(0 if layer == 0 else 1, bufs, cache, pos, EPS, NQ, NKV, HD)

    t0 = time.perf_counter()
    chain(L)  # the first full chain also sizes the steps
    t_full = time.perf_counter() - t0
    layers = L
    if (steps + max(0, warmup - 1)) * t_full > budget_s:
        layers = max(1, int(L * budget_s / ((steps + max(0, warmup - 1)) * t_full)))
    for _ in range(max(0, warmup - 1)):
        chain(layers)
    t0 = time.perf_counter()
    for _ in range(steps):
        chain(layers)
    dt = (time.perf_counter() - t0) / steps * (L / layers)
    what = "the full 32-layer chain" if layers == L else f"the first {layers} of 32 layers, scaled to 32"
    return {"value": round(T / dt, 1), "unit": UNIT, "cores": cores, "kind": "port",
            "ms_per_step": round(dt * 1e3, 3), "steps_timed": steps,
            "sample": f"T=512 bf16 op chain on the host CPU (torch, {cores} threads), {steps} timed "
                      f"steps after {warmup} warm-up, each step {what}"}


def cpu_config1_sample(budget_s: float = 3.0):
    """The CPU-runnable workload on the host cores: one Llama-3-8B layer's ops in fp32 at
    T=64 (fused_add_rms_norm -> neox rope -> silu_and_mul), the oracle's torch
    formulas; wall time per chain and fp32 algorithmic bytes per second."""
    import torch

    from oracle import ops_ref

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    inp = ops_ref.config1_inputs(seed=0)
    ops_ref.config1_chain(inp)
    n, t_sum = 0, 0.0
    while n < 3 or t_sum < budget_s:
        t0 = time.perf_counter()
        ops_ref.config1_chain(inp)
        t_sum += time.perf_counter() - t0
        n += 1
    ms = t_sum / n * 1e3
    nbytes = ops_ref.CONFIG1["T"] * ops_ref.CONFIG1_BYTES_PER_TOKEN
    return {"workload": "one Llama-3-8B layer, fp32, T=64 (fused_add_rms_norm, neox "
                        "rope q[64,32,128] k[64,8,128], silu_and_mul [64,28672])",
            "ms_per_chain": round(ms, 3), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 2),
            "tokens_per_s": round(ops_ref.CONFIG1["T"] / (ms * 1e-3), 1), "cores": cores,
            "passes": n}


# ------------------------------------------------------------ KV promotion --
KV_NB, KV_L, KV_SLAB = 8192, 32, (2, 16, 8, 128)
KV_BLOCK_BYTES = 2 * 16 * 8 * 128 * 2
KV_METHODS = {1: "simt", 2: "bulk"}


def kv_requests(seed: int):
    """The promotion workload: 8 promoted requests, prompt lengths
    min(8192, round(lognormal(6.9, 0.7))) -> ceil(len/16) blocks each, taken from
    random occupied blocks of an 80 %-full LP cache and scattered into random free
    blocks of an HP cache that is 80 % full with other requests."""
    import numpy as np

    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(rng.lognormal(6.9, 0.7, 8)), 1, 8192).astype(np.int64)
    blocks = int(((lens + 15) // 16).sum())
    occupied = rng.permutation(KV_NB)[: int(0.8 * KV_NB)]
    free = rng.permutation(KV_NB)[int(0.8 * KV_NB):]
    blocks = min(blocks, len(free))
    src = rng.choice(occupied, blocks, replace=False)
    dst = rng.choice(free, blocks, replace=False)
    return lens, src, dst


def _kv_caches(dev, fill_seed=None):
    """The 32 per-layer caches [KV_NB, 2, 16, 8, 128] bf16 as views of one
    allocation (layer stride KV_NB blocks), so the copy-engine path can move a
    run of blocks of every layer with one 2-D copy; the kernels see the same
    per-layer tensors either way."""
    import torch

    whole = torch.zeros(KV_L, KV_NB, *KV_SLAB, dtype=torch.bfloat16, device=dev)
    if fill_seed is not None:
        g = torch.Generator(device=dev).manual_seed(fill_seed)
        for layer in whole.unbind(0):
            layer.copy_(torch.randn(KV_NB, *KV_SLAB, generator=g, device=dev))
    return list(whole.unbind(0))


def _time_copy(fn, steps, warmup):
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def kv_cpu_copy(src, dst, layers: int = 2):
    """The block move done on the host cores: per layer, torch's fancy-index copy
    dst[dst_ids] = src[src_ids] between host caches of the same shape, all
    threads; a bounded sample of `layers` layers, scaled to GB/s."""
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(3)
    # 2-byte elements as int16: the move is a byte copy, and integer equality
    # has no NaN patterns
    sc = [torch.randint(-30000, 30000, (KV_NB, *KV_SLAB), generator=g, dtype=torch.int16)
          for _ in range(layers)]
    dc = [torch.zeros(KV_NB, *KV_SLAB, dtype=torch.int16) for _ in range(layers)]
    s_ids = torch.as_tensor(src, dtype=torch.long)
    d_ids = torch.as_tensor(dst, dtype=torch.long)
    dc[0][d_ids] = sc[0][s_ids]  # warm-up (first touch of the pages)
    t0 = time.perf_counter()
    for s_, d_ in zip(sc, dc):
        d_[d_ids] = s_[s_ids]
    dt = time.perf_counter() - t0
    nbytes = layers * len(src) * KV_BLOCK_BYTES
    ok = all(torch.equal(d_[d_ids], s_[s_ids]) for s_, d_ in zip(sc, dc))
    return {"value": round(nbytes / dt / 1e9, 2), "unit": "GB/s", "cores": cores, "kind": "port",
            "byte_exact": bool(ok),
            "sample": f"{layers} of {KV_L} layers' block moves ({nbytes / 1e6:.0f} MB) as a host "
                      f"fancy-index copy with {cores} threads"}


def kv_reference_path(src_caches, dst_caches, src, dst, dev):
    """The reference mechanism (KVhelper GPU->CPU gather, CPU->GPU index-put), one pass."""
    import torch

    from oracle import kv_ref

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    host = kv_ref.get_kv_cache(src_caches, src.tolist())
    t1 = time.perf_counter()
    kv_ref.insert_kv_cache(dst_caches, host, dst.tolist(), dev)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1


def kv_host_path(sc, dc, sids, dids, steps, warmup):
    """The KVhelper host round trip (DRAM swap-out of a preempted request and
    swap-in, decode_llm_engine.py:31-40 / base_worker.py `_get_kv_cache_nofree`,
    and the Ray-path get_kv_cache / insert_kv_cache): one gather kernel writing
    every layer's blocks into page-locked host memory, one scatter kernel back."""
    import torch

    from paceserve_b200 import kv_transfer_ops as kvo

    host = torch.empty(KV_L, sids.numel(), *KV_SLAB, dtype=torch.bfloat16, pin_memory=True)
    nbytes = host.numel() * 2
    ms_g = _time_copy(lambda: kvo.gather_blocks(list(sc), sids, host), steps, warmup)
    for c in dc:
        c.zero_()
    ms_s = _time_copy(lambda: kvo.scatter_blocks(host, list(dc), dids), steps, warmup)
    ok = all(torch.equal(dc[l][dids.long()], sc[l][sids.long()]) for l in range(KV_L))
    return {"bytes": nbytes, "byte_exact": bool(ok),
            "gather_to_host": {"ms": round(ms_g, 3), "gbs": round(nbytes / (ms_g * 1e-3) / 1e9, 1)},
            "scatter_from_host": {"ms": round(ms_s, 3), "gbs": round(nbytes / (ms_s * 1e-3) / 1e9, 1)},
            "round_trip_gbs": round(nbytes / ((ms_g + ms_s) * 1e-3) / 1e9, 2)}


def _overlap_one(g, chain_ms, copy, nbytes, reps, threaded=False):
    """The chain graph `g` on the current stream and `copy` on a side stream,
    launched interleaved so both run for about the same time.  threaded: the
    copies are issued by a second host thread (the copy-engine path spends
    milliseconds of host time per call, which must not delay the chain's
    launches)."""
    import torch

    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        copy_ms = _time_copy(copy, 10 if not threaded else 3, 3 if not threaded else 1)
    n_copy = max(1, round(reps * chain_ms / copy_ms))
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record(main)
    ev[2].record(side)
    if threaded:
        def issue():
            with torch.cuda.stream(side):
                for _ in range(n_copy):
                    copy()
        th = threading.Thread(target=issue)
        th.start()
        for _ in range(reps):
            g.replay()
        th.join()
    else:
        for i in range(max(reps, n_copy)):
            if i < reps:
                g.replay()
            if i < n_copy:
                with torch.cuda.stream(side):
                    copy()
    ev[1].record(main)
    ev[3].record(side)
    torch.cuda.synchronize()
    c_ms = ev[0].elapsed_time(ev[1]) / reps
    k_ms = ev[2].elapsed_time(ev[3]) / n_copy
    return {"copy_gbs_alone": round(nbytes / (copy_ms * 1e-3) / 1e9, 1),
            "chain_ms_concurrent": round(c_ms, 4),
            "chain_slowdown": round(c_ms / chain_ms - 1, 4),
            "copy_gbs_concurrent": round(nbytes / (k_ms * 1e-3) / 1e9, 1)}


def _overlap_chain(dev, copies, nbytes, reps):
    """Chain alone, then beside each copy in `copies` ({name: callable})."""
    import paceserve_b200 as pb

    ops = (pb.layernorm_ops, pb.pos_encoding_ops, pb.activation_ops)
    ch = build_chain(dev, seed=5)
    g = capture(lambda: run_chain(ch, ops))
    chain_ms = time_replays(g, reps, 5) / reps
    out = {"chain_ms_alone": round(chain_ms, 4), "copy_bytes": nbytes}
    for name, copy in copies.items():
        out[name] = _overlap_one(g, chain_ms, copy, nbytes, reps, threaded="copy_engine" in name)
    del g
    return out


# Promotion paths measured beside the serving chain: (side, method, max_ctas).
# "pull" runs on the HP (serving) GPU, "push" on the LP GPU; method 3 is the
# copy engines (no SM); max_ctas caps the kernel's CTAs.
KV_PATHS = {
    "pull_simt": ("pull", 1, 0),
    "pull_simt_16ctas": ("pull", 1, 16),
    "pull_bulk": ("pull", 2, 0),
    "pull_copy_engine": ("pull", 3, 0),
    "push_simt": ("push", 1, 0),
    "push_copy_engine": ("push", 3, 0),
}


def kv_overlap(dev, reps: int = 100):
    """Promotion while serving, on one GPU: the 32-layer chain (a CUDA graph) on
    the main stream and the promotion copy (1.1 GB, HBM -> HBM) on a side
    stream at the same time.  Per copy path: the chain's ms per step and the
    copy's GB/s, alone and concurrent; each path's copy checked byte-exact."""
    import torch

    from paceserve_b200 import kv_transfer as kvt

    _, src, dst = kv_requests(7)
    sc = _kv_caches(dev, fill_seed=100)
    dc = _kv_caches(dev)
    sids = torch.tensor(src, dtype=torch.int32, device=dev)
    dids = torch.tensor(dst, dtype=torch.int32, device=dev)
    sids_h, dids_h = sids.cpu(), dids.cpu()
    nbytes = len(src) * KV_L * KV_BLOCK_BYTES
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    copies, exact = {}, {}
    for name, (_side, m, ctas) in KV_PATHS.items():
        if name.startswith("push"):
            continue  # one GPU: push and pull are the same copy
        ids = (sids_h, dids_h) if m == 3 else (sids, dids)
        fn = (lambda m=m, ctas=ctas, ids=ids: kvt.promote(sc, dc, ids[0], ids[1], method=m,
                                                        bad_pairs=bad, max_ctas=ctas))
        for c in dc:
            c[dids.long()] = 0
        fn()
        torch.cuda.synchronize()
        exact[name] = bool(all(torch.equal(dc[l][dids.long()], sc[l][sids.long()])
                               for l in range(KV_L))) and bad.item() == 0
        copies[name] = fn
    out = _overlap_chain(dev, copies, nbytes, reps)
    for name in copies:
        out[name]["byte_exact"] = exact[name]
    return out


def _pair_overlap(role, pair_lp, pair_hp, imported, caches, peer_caches, sids, dids, nbytes,
                  g_ref, dev, reps=60):
    """Promotion while serving across a pair: the HP GPU replays the 32-layer
    chain while the promotion runs by each path of KV_PATHS (pull on the HP GPU
    or push from the LP GPU, by SM kernel or copy engine).  Every rank takes the
    same collective steps.  Returns {path: result} on HP ranks, None elsewhere."""
    import torch
    import torch.distributed as dist

    import paceserve_b200 as pb
    from paceserve_b200 import kv_transfer as kvt

    ops = (pb.layernorm_ops, pb.pos_encoding_ops, pb.activation_ops)
    g = chain_ms = None
    if role == "hp":
        ch = build_chain(dev, seed=5)
        g = capture(lambda: run_chain(ch, ops))
        chain_ms = time_replays(g, reps, 5) / reps
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    sids_h = sids.cpu() if sids is not None else None
    dids_h = dids.cpu() if dids is not None else None
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    results = {}
    for name, (where, m, ctas) in KV_PATHS.items():
        mine = role == ("hp" if where == "pull" else "lp")
        fn = None
        if mine:
            ids = (sids_h, dids_h) if m == 3 else (sids, dids)
            if where == "pull":
                fn = (lambda m=m, ctas=ctas, ids=ids: kvt.promote(
                    imported, caches, ids[0], ids[1], method=m, bad_pairs=bad, max_ctas=ctas))
            else:
                fn = (lambda m=m, ctas=ctas, ids=ids: kvt.push(
                    caches, peer_caches, ids[0], ids[1], method=m, bad_pairs=bad, max_ctas=ctas))
        # 1. byte-exactness of this path: clear the targets, copy once, compare
        if role == "hp":
            for c in caches:
                c[dids.long()] = 0
            torch.cuda.synchronize()
        dist.barrier()
        bad.zero_()
        if fn is not None:
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ok = None
        if role == "hp":
            ok = bool(torch.equal(torch.stack([c[dids.long()] for c in caches]), g_ref))
        # 2. the copy alone
        copy_ms = 0.0
        if fn is not None:
            with torch.cuda.stream(side):
                copy_ms = _time_copy(fn, 5, 2)
        info = [None] * dist.get_world_size()
        dist.all_gather_object(info, (role, copy_ms, int(bad.item()), chain_ms or 0.0))
        # 3. both at once: the chain on HP, as many copies on the side that runs
        # them as fill the chain's time
        n_copy = 0
        if fn is not None and copy_ms > 0:
            hp_chain = chain_ms if role == "hp" else info[pair_hp][3]
            n_copy = max(1, round(reps * hp_chain / copy_ms))
        dist.barrier()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(main)
        ev[2].record(side)
        if role == "hp" and fn is not None and m == 3:
            # copy-engine copies take milliseconds of host time per call: issue
            # them from a second thread so the chain's launches are not delayed
            def issue(fn=fn, n=n_copy):
                with torch.cuda.stream(side):
                    for _ in range(n):
                        fn()
            th = threading.Thread(target=issue)
            th.start()
            for _ in range(reps):
                g.replay()
            th.join()
        else:
            for i in range(max(reps if role == "hp" else 0, n_copy if fn is not None else 0)):
                if role == "hp" and i < reps:
                    g.replay()
                if fn is not None and i < n_copy:
                    with torch.cuda.stream(side):
                        fn()
        ev[1].record(main)
        ev[3].record(side)
        torch.cuda.synchronize()
        c_ms = ev[0].elapsed_time(ev[1]) / reps if role == "hp" else 0.0
        k_ms = ev[2].elapsed_time(ev[3]) / n_copy if (fn is not None and n_copy) else 0.0
        res = [None] * dist.get_world_size()
        dist.all_gather_object(res, (role, c_ms, k_ms, ok, int(bad.item())))
        if role == "hp":
            copy_ms_pair = copy_ms if mine else info[pair_lp][1]
            peer_k = k_ms if mine else res[pair_lp][2]
            peer_bad = int(bad.item()) if mine else res[pair_lp][4]
            results[name] = {
                "runs_on": "HP GPU" if where == "pull" else "LP GPU",
                "engine": "copy engines" if m == 3 else ("SM kernel, %s" % (
                    f"{ctas} CTAs" if ctas else "all SMs")),
                "byte_exact": bool(ok) and peer_bad == 0,
                "copy_gbs_alone": round(nbytes / (copy_ms_pair * 1e-3) / 1e9, 1),
                "chain_ms_concurrent": round(c_ms, 4),
                "chain_slowdown": round(c_ms / chain_ms - 1, 4),
                "copy_gbs_concurrent": round(nbytes / (peer_k * 1e-3) / 1e9, 1) if peer_k else None}
    if g is not None:
        del g
    return ({"chain_ms_alone": round(chain_ms, 4), "copy_bytes": nbytes, "paths": results}
            if role == "hp" else None)


def kv_promotion(ws, rank, local, steps, warmup, baseline=True, overlap=False):
    """LP->HP promotion on rank pairs (0->1, 2->3, ...): the HP rank pulls the
    request blocks from the LP rank's caches (CUDA IPC) with one kernel per
    method.  With one GPU, LP and HP caches both live on it (an HBM-to-HBM copy).
    overlap=True adds, on every pair, the chain's slowdown while a promotion runs
    by each path of KV_PATHS.  Returns the result dict on every rank
    (collectives are taken by all ranks in the same order)."""
    import torch

    from paceserve_b200 import kv_transfer as kvt

    dev = torch.device(f"cuda:{local}")
    out = {"workload": f"LP->HP KV promotion, Llama-3-8B paged cache [{KV_NB}, 2, 16, 8, 128] bf16 x "
                       "32 layers, 8 requests lognormal(6.9, 0.7) capped 8192, 80 % occupied"}
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    if ws == 1:
        lens, src, dst = kv_requests(7)
        sc = _kv_caches(dev, fill_seed=100)
        dc = _kv_caches(dev)
        sids = torch.tensor(src, dtype=torch.int32, device=dev)
        dids = torch.tensor(dst, dtype=torch.int32, device=dev)
        nbytes = len(src) * KV_L * KV_BLOCK_BYTES
        res = {}
        for m, name in KV_METHODS.items():
            ms = _time_copy(lambda: kvt.promote(sc, dc, sids, dids, method=m, bad_pairs=bad), steps,
                            warmup)
            res[name] = {"ms": round(ms, 4), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                         "hbm_gbs": round(2 * nbytes / (ms * 1e-3) / 1e9, 1)}
        ok = all(torch.equal(dc[l][dids.long()], sc[l][sids.long()]) for l in range(KV_L))
        out.update({"mode": "one GPU: HBM -> HBM", "blocks": int(len(src)), "bytes": nbytes,
                    "byte_exact": bool(ok) and bad.item() == 0, "methods": res})
        out["host_path"] = kv_host_path(sc, dc, sids, dids, max(2, steps // 4), 2)
        if baseline:
            d2h, h2d = kv_reference_path(sc, dc, src, dst, dev)
            out["reference_path"] = {"gbs": round(nbytes / (d2h + h2d) / 1e9, 2),
                                     "d2h_s": round(d2h, 4), "h2d_s": round(h2d, 4),
                                     "kind": "port", "sample": "KVhelper get_kv_cache/insert_kv_cache "
                                     "restated (per-layer fancy-index gather to host, index-put back), "
                                     "one pass, without the Ray object-store hop"}
            out["cpu_baseline"] = kv_cpu_copy(src, dst)
        return out

    import torch.distributed as dist

    pairs = kvt.pair_ranks(ws)
    mine = next(((i, lp, hp) for i, (lp, hp) in enumerate(pairs) if rank in (lp, hp)), None)
    role = None if mine is None else ("lp" if rank == mine[1] else "hp")
    caches = None
    if role == "lp":
        caches = _kv_caches(dev, fill_seed=100 + mine[0])
    elif role == "hp":
        caches = _kv_caches(dev)
    # both sides export: the HP rank pulls from the LP caches, the LP rank pushes
    # into the HP caches
    exports = kvt.exchange_exports(kvt.export_caches(caches) if role is not None else None)
    times = {m: 0.0 for m in KV_METHODS}
    nbytes, nblocks, imported = 0, 0, None
    sids = dids = None
    if mine is not None:
        lens, src, dst = kv_requests(7)  # the same promotion on every pair
        nblocks = len(src)
        nbytes = nblocks * KV_L * KV_BLOCK_BYTES
        sids = torch.tensor(src, dtype=torch.int32, device=dev)
        dids = torch.tensor(dst, dtype=torch.int32, device=dev)
        imported = kvt.ImportedCaches(exports[mine[2] if role == "lp" else mine[1]], local)
    dist.barrier()
    if role == "hp":
        for m in KV_METHODS:
            times[m] = _time_copy(lambda: kvt.promote(imported, caches, sids, dids, method=m,
                                                      bad_pairs=bad), steps, warmup)
    t = torch.tensor([times[m] for m in KV_METHODS], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ok = True
    g_ref = None
    if role == "lp":
        g = torch.stack([c[sids.long()] for c in caches])
        dist.send(g, dst=mine[2])
        del g
    elif role == "hp":
        g_ref = torch.empty(KV_L, nblocks, *KV_SLAB, dtype=torch.bfloat16, device=dev)
        dist.recv(g_ref, src=mine[1])
        ok = bool(torch.equal(torch.stack([c[dids.long()] for c in caches]), g_ref)) and \
            bad.item() == 0
    ov = None
    if overlap:
        # Promotion while serving: the HP GPU runs the chain while the promotion
        # runs by each path.
        ov = _pair_overlap(role, mine[1] if mine else None, mine[2] if mine else None, imported,
                           caches, imported, sids, dids, nbytes, g_ref, dev)
    torch.cuda.synchronize()
    dist.barrier()
    if imported is not None:
        imported.close()
    del g_ref
    info = [None] * ws
    dist.all_gather_object(info, (role, ok, nbytes, [times[m] for m in KV_METHODS], ov))
    dist.barrier()
    hps = [x for x in info if x[0] == "hp"]
    total = sum(x[2] for x in hps)
    res = {}
    for i, (m, name) in enumerate(KV_METHODS.items()):
        ms = t[i].item()
        own = [x[2] / (x[3][i] * 1e-3) / 1e9 for x in hps]  # each pair: its bytes / its time
        res[name] = {"ms_max_over_pairs": round(ms, 4),
                     "gbs_per_pair": round(total / len(pairs) / (ms * 1e-3) / 1e9, 1),
                     "gbs_per_pair_min_max": [round(min(own), 1), round(max(own), 1)],
                     "aggregate_gbs": round(total / (ms * 1e-3) / 1e9, 1)}
    best = max(res.values(), key=lambda r: r["gbs_per_pair"])
    out.update({"mode": f"{len(pairs)} LP->HP pairs over NVLink (pull on the HP GPU, CUDA IPC)",
                "pairs": len(pairs), "bytes_per_pair_avg": total // max(1, len(pairs)),
                "byte_exact": all(x[1] for x in info), "methods": res,
                "nvlink_frac": round(best["gbs_per_pair"] / NVLINK_GBS, 4),
                "nvlink_peak_gbs": NVLINK_GBS, "nvlink_peak_source": "measured peer copy on this pool"})
    if overlap:
        out["promotion_while_serving"] = {
            "what": "per pair: the HP GPU replays the 32-layer chain while the promotion runs by "
                    "each path (pull = on the HP GPU, push = from the LP GPU)",
            "per_pair": [x[4] for x in hps]}
    return out


def append_metadata(seed: int = 11, page_size: int = 16, num_pages: int = 4096):
    """begin_forward's append metadata (flashinfer_attention_wrapper.py:75-209) for the
    Sarathi batch: one 448-token prefill chunk starting at position 0, then 64
    decode requests with contexts uniform in [1, 1024]; distinct random pages."""
    import numpy as np
    import torch

    rng = np.random.default_rng(seed)
    free = list(rng.permutation(num_pages))
    ai, kp, ki, kl = [0], [0], [], []
    lens = [T_PREFILL] + [int(x) for x in rng.integers(1, 1025, T_DECODE)]
    chunks = [T_PREFILL] + [1] * T_DECODE
    for n_new, total in zip(chunks, lens):
        pages = (total + page_size - 1) // page_size
        ki += [int(free.pop()) for _ in range(pages)]
        ai.append(ai[-1] + n_new)
        kp.append(kp[-1] + pages)
        kl.append(total % page_size or page_size)
    t = lambda x: torch.tensor(x, dtype=torch.int32)  # noqa: E731
    return t(ai), t(kp), t(ki), t(kl)


def append_bench(dev, reps: int = 20):
    """Paged-KV append of one step's 512 new K/V tokens into each of the 32
    layers' caches (graph of 32 launches, distinct caches and qkv buffers)."""
    import torch

    import paceserve_b200 as pb

    num_pages = 4096
    layers = L if KV_NB >= 8192 else 4  # the small --kv-blocks case (for ncu) keeps 1 GiB
    ai, kp, ki, kl = (x.to(dev) for x in append_metadata(num_pages=num_pages))
    g = torch.Generator(device=dev).manual_seed(5)
    caches = [torch.zeros(num_pages, 2, 16, NKV, HD, dtype=torch.bfloat16, device=dev)
              for _ in range(layers)]
    qkvs = [torch.randn(T, (NQ + 2 * NKV) * HD, generator=g, device=dev).bfloat16()
            for _ in range(layers)]
    kv = pb.kv_transfer_ops

    def fn():
        for c, q in zip(caches, qkvs):
            kv.append_paged_kv_cache_by_indptr(q[:, NQ * HD:(NQ + NKV) * HD], q[:, (NQ + NKV) * HD:],
                                               ai, c, ki, kp, kl)
    gr = capture(fn)
    us = time_replays(gr, reps, 3) * 1e3 / (reps * layers)
    nbytes = 2 * 2 * T * NKV * HD * 2  # read K and V rows, write them into the pages
    return {"us_per_layer": round(us, 3), "bytes_per_layer": nbytes,
            "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
            "workload": "append_paged_kv_cache_by_indptr, 448 prefill + 64 decode tokens, "
                        "8 kv heads x 128, page 16, per layer"}


NVLINK_GBS = 770.0  # measured peer copy per direction on this pool (900 nominal)


# ------------------------------------------------------------ sweep / MoE --
def sweep(dev, reps=10):
    """Token sweep: per-op GB/s for T in {1..16384}, Llama-3-8B and -70B shapes,
    bf16 and fp16.  Each op is timed as a CUDA graph over enough distinct buffers
    that every launch reads cold data (working set >= 512 MB per cycle)."""
    import torch

    import paceserve_b200 as pb

    shapes = {"llama3-8b": (4096, 14336, 32, 8), "llama3-70b": (8192, 28672, 64, 8)}
    out = []
    for sname, (h, inter, nq, nkv) in shapes.items():
        for dtype in (torch.bfloat16, torch.float16):
            for t in (1, 16, 128, 512, 2048, 8192, 16384):
                per = {"rms_norm": 4 * h * t + 2 * h, "fused_add_rms_norm": 8 * h * t + 2 * h,
                       "rotary_embedding": 4 * (nq + nkv) * HD * t + t * HD * 4 + 8 * t,
                       "silu_and_mul": 6 * inter * t}
                row = {"shape": sname, "dtype": str(dtype).split(".")[1], "T": t}
                for op, nbytes in per.items():
                    nbuf = int(min(32, max(2, -(-512 * 2**20 // nbytes))))
                    g_ = torch.Generator(device=dev).manual_seed(t)
                    rn = lambda *sh: torch.randn(*sh, generator=g_, device=dev).to(dtype)  # noqa: E731
                    if op == "rms_norm":
                        bufs = [(rn(t, h), torch.empty(t, h, dtype=dtype, device=dev), rn(h)) for _ in range(nbuf)]
                        fn = lambda: [pb.layernorm_ops.rms_norm(o, x, w, EPS) for x, o, w in bufs]  # noqa: E731
                    elif op == "fused_add_rms_norm":
                        bufs = [(rn(t, h), rn(t, h), rn(h)) for _ in range(nbuf)]
                        fn = lambda: [pb.layernorm_ops.fused_add_rms_norm(x, r, w, EPS) for x, r, w in bufs]  # noqa: E731
                    elif op == "rotary_embedding":
                        cache = rope_cache(dev, max(MAX_POS, t))  # every position in range
                        pos = torch.randint(0, t, (t,), device=dev)
                        bufs = [rn(t, (nq + 2 * nkv) * HD) for _ in range(nbuf)]
                        fn = lambda: [pb.pos_encoding_ops.rotary_embedding(  # noqa: E731
                            pos, q[:, : nq * HD], q[:, nq * HD: (nq + nkv) * HD], HD, cache, True) for q in bufs]
                    else:
                        bufs = [(rn(t, 2 * inter), torch.empty(t, inter, dtype=dtype, device=dev)) for _ in range(nbuf)]
                        fn = lambda: [pb.activation_ops.silu_and_mul(o, x) for x, o in bufs]  # noqa: E731
                    g = capture(fn)
                    us = time_replays(g, reps, 3) * 1e3 / (reps * nbuf)
                    row[op] = {"us": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
                    del g, bufs
                out.append(row)
                torch.cuda.empty_cache()
    return out


def moe_routing(dev, reps=50):
    """Mixtral-8x7B routing: topk_softmax (E=8, top-2, renormalised) then
    moe_align_block_size (block 64) on N(0,1) fp32 gating logits."""
    import numpy as np
    import torch

    import paceserve_b200 as pb
    from oracle import moe_ref

    out = []
    for t in (64, 512, 4096, 16384):
        E, k, bs = 8, 2, 64
        gating = torch.randn(t, E, generator=torch.Generator().manual_seed(t)).to(dev)
        w = torch.empty(t, k, device=dev)
        ids = torch.empty(t, k, dtype=torch.int32, device=dev)
        tei = torch.empty(t, k, dtype=torch.int32, device=dev)
        cap = t * k + E * (bs - 1)
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
        expert_ids = torch.empty((cap + bs - 1) // bs, dtype=torch.int32, device=dev)
        total = torch.empty(1, dtype=torch.int32, device=dev)
        topk = lambda: pb.moe_ops.topk_softmax(w, ids, tei, gating, True)  # noqa: E731
        align = lambda: pb.moe_ops.moe_align_block_size(ids, E, bs, sorted_ids, expert_ids, total, True)  # noqa: E731
        res = {"T": t}
        for name, fn, nbytes in (("topk_softmax", topk, t * (4 * E + 12 * k)),
                                 ("moe_align_block_size", align,
                                  4 * t * k + 4 * cap + 4 * ((cap + bs - 1) // bs) + 4)):
            g = capture(lambda: [fn() for _ in range(reps)])
            us = time_replays(g, 5, 3) * 1e3 / (5 * reps)
            res[name] = {"us": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 2)}
            del g
        topk()
        align()
        torch.cuda.synchronize()
        ow, oi, ot = moe_ref.topk_softmax(gating.cpu().numpy(), k, renormalize=True)
        os_, oe, otot = moe_ref.moe_align_block_size(oi, E, bs)
        n = int(total.item())
        res["bit_exact"] = bool(np.array_equal(ids.cpu().numpy(), oi) and n == otot
                                and np.array_equal(sorted_ids.cpu().numpy(), os_)
                                and np.array_equal(expert_ids.cpu().numpy()[: n // bs], oe))
        out.append(res)
    return out


def gemm_workspace(dev, t):
    """One zeroed workspace for every fused GEMM of a Llama-3-8B layer at t
    tokens (stream-ordered calls may share it), or None when none needs one.
    Passed explicitly, so no CUDA-graph capture records the shim allocating and
    zero-filling its own."""
    import torch

    from paceserve_b200 import cabi

    lib = cabi.load()
    d = torch.device(dev).index or 0
    need = max(lib.pace_qkv_proj_rope_workspace_size(t, H, NQ, NKV, d),
               lib.pace_linear_residual_workspace_size(t, H, H, d),
               lib.pace_linear_residual_workspace_size(t, H, I, d),
               lib.pace_gate_up_silu_workspace_size(t, H, I, d))
    return torch.zeros(need, dtype=torch.uint8, device=dev) if need else None


def qkv_rope_bench(dev, tokens=(1, 2, 128, 512, 2048), reps=10):
    """The fused qkv projection + rotary embedding (tcgen05 GEMM, rope in the
    epilogue; at most 2 tokens, the weight-streaming CUDA-core kernel) against
    the path it replaces: cuBLAS (torch.matmul) for the
    projection, then the rotary_embedding op on the q/k views.  Llama-3-8B
    (hidden 4096 -> 6144 = 32 q + 8 k + 8 v heads of 128), bf16, fp32 cache,
    positions as the Sarathi batch draws them.  Each variant is a CUDA graph
    over 4 distinct weight matrices (4 x 50 MB > L2); the fused output is
    checked against the unfused one within the bf16 rule."""
    import torch

    import paceserve_b200 as pb

    nq, nkv = NQ, NKV
    n = (nq + 2 * nkv) * HD
    nbuf = 4
    g_ = torch.Generator(device=dev).manual_seed(77)
    weights = [(torch.randn(n, H, generator=g_, device=dev) / H ** 0.5).bfloat16()
               for _ in range(nbuf)]
    cache = rope_cache(dev)
    peak = peaks()
    rows = []
    for t in tokens:
        xs = [torch.randn(t, H, generator=g_, device=dev).bfloat16() for _ in range(nbuf)]
        pos = torch.randint(0, MAX_POS, (t,), generator=g_, device=dev)
        outs = [torch.empty(t, n, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        refs = [torch.empty(t, n, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        ws = gemm_workspace(dev, t)

        def fused():
            for x, w, o in zip(xs, weights, outs):
                pb.pos_encoding_ops.qkv_proj_rotary_embedding(o, x, w, pos, HD, nq, nkv, cache,
                                                              True, None, ws)

        def gemm():
            for x, w, o in zip(xs, weights, refs):
                torch.matmul(x, w.t(), out=o)

        def unfused():
            for x, w, o in zip(xs, weights, refs):
                torch.matmul(x, w.t(), out=o)
                pb.pos_encoding_ops.rotary_embedding(pos, o[:, : nq * HD],
                                                     o[:, nq * HD: (nq + nkv) * HD], HD, cache,
                                                     True)

        res = {"T": t}
        for name, fn in (("fused_us", fused), ("cublas_gemm_us", gemm),
                         ("cublas_gemm_plus_rope_us", unfused)):
            fn()  # eager once
            gr = capture(fn)
            res[name] = round(time_replays(gr, reps, 3) * 1e3 / (reps * nbuf), 3)
            del gr
        torch.cuda.synchronize()
        ref = refs[-1].float()
        err = ((outs[-1].float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()
        flops = 2.0 * t * n * H
        res["tflops"] = round(flops / (res["fused_us"] * 1e-6) / 1e12, 1)
        res["frac_of_bf16_peak"] = round(res["tflops"] / peak["bf16_tflops"], 4)
        res["speedup_vs_unfused"] = round(res["cublas_gemm_plus_rope_us"] / res["fused_us"], 3)
        # roofline: the larger of tensor time and the time to move the weight,
        # the hidden rows and the output once
        nbytes = 2.0 * (n * H + t * H + t * n)
        t_roof_us = max(flops / (peak["bf16_tflops"] * 1e12), nbytes / (peak["hbm_gbs"] * 1e9)) * 1e6
        res["roofline_us"] = round(t_roof_us, 2)
        res["frac_of_roofline"] = round(t_roof_us / res["fused_us"], 4)
        res["rel_err_vs_unfused"] = round(err, 5)
        rows.append(res)
        del xs, outs, refs
        torch.cuda.empty_cache()
    return rows


def norm_gemm_bench(dev, tokens=(512, 2048), reps=10):
    """The layer boundary o_proj -> residual add -> input RMSNorm -> qkv_proj
    -> rope (Llama-3-8B, bf16) fused into two tensor-core GEMMs
    (linear_residual with the residual add and the norm's sum-of-squares
    partials in its epilogue; qkv_proj_rmsnorm_rotary_embedding with the norm
    factor and rope in its epilogue) against the unfused path: cuBLAS o_proj,
    this package's fused_add_rms_norm, cuBLAS qkv_proj and rotary_embedding.
    CUDA graphs over 3 weight sets (> L2); outputs compared within the bf16
    rule."""
    import torch

    import paceserve_b200 as pb

    nbuf = 3
    n = (NQ + 2 * NKV) * HD
    g_ = torch.Generator(device=dev).manual_seed(21)
    w_o = [(torch.randn(H, H, generator=g_, device=dev) / H ** 0.5).bfloat16() for _ in range(nbuf)]
    w_qkv = [(torch.randn(n, H, generator=g_, device=dev) / H ** 0.5).bfloat16() for _ in range(nbuf)]
    w_norm = [(torch.randn(H, generator=g_, device=dev) * 0.02 + 1).bfloat16() for _ in range(nbuf)]
    folded = [pb.fold_rmsnorm_weight(w, nw) for w, nw in zip(w_qkv, w_norm)]
    cache = rope_cache(dev)
    rows = []
    for t in tokens:
        attn = [torch.randn(t, H, generator=g_, device=dev).bfloat16() for _ in range(nbuf)]
        res0 = [torch.randn(t, H, generator=g_, device=dev).bfloat16() for _ in range(nbuf)]
        pos = torch.randint(0, MAX_POS, (t,), generator=g_, device=dev)
        res_f = [r.clone() for r in res0]
        res_u = [r.clone() for r in res0]
        ss = [torch.empty(t, H // 32, device=dev) for _ in range(nbuf)]
        qkv_f = [torch.empty(t, n, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        qkv_u = [torch.empty(t, n, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        xo = [torch.empty(t, H, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]

        ws = gemm_workspace(dev, t)

        def fused():
            for i in range(nbuf):
                pb.layernorm_ops.linear_residual(res_f[i], attn[i], w_o[i], ss[i], workspace=ws)
                pb.pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding(
                    qkv_f[i], res_f[i], folded[i], ss[i], EPS, pos, HD, NQ, NKV, cache, True,
                    workspace=ws)

        def unfused():
            for i in range(nbuf):
                torch.matmul(attn[i], w_o[i].t(), out=xo[i])
                pb.layernorm_ops.fused_add_rms_norm(xo[i], res_u[i], w_norm[i], EPS)
                torch.matmul(xo[i], w_qkv[i].t(), out=qkv_u[i])
                q = qkv_u[i]
                pb.pos_encoding_ops.rotary_embedding(pos, q[:, : NQ * HD],
                                                     q[:, NQ * HD: (NQ + NKV) * HD], HD, cache,
                                                     True)

        res = {"T": t}
        for name, fn, resets in (("fused_us", fused, res_f), ("unfused_us", unfused, res_u)):
            fn()  # eager once
            gr = capture(fn)
            res[name] = round(time_replays(gr, reps, 3) * 1e3 / (reps * nbuf), 3)
            del gr
            for r_, r0 in zip(resets, res0):  # the residual accumulated over replays
                r_.copy_(r0)
        fused()
        unfused()
        torch.cuda.synchronize()
        qf, qu = qkv_f[0].float(), qkv_u[0].float()
        res["speedup_vs_unfused"] = round(res["unfused_us"] / res["fused_us"], 3)
        res["rel_err_qkv"] = round(((qf - qu).abs().max() / qu.abs().max()).item(), 5)
        rows.append(res)
        del attn, res0, res_f, res_u, ss, qkv_f, qkv_u, xo
        torch.cuda.empty_cache()
    return rows


def layer_gemms_bench(dev, tokens=(1, 512, 2048, 8192), reps=5):
    """Everything in a Llama-3-8B decoder layer but attention, bf16: o_proj ->
    residual add -> post-attention RMSNorm -> gate_up_proj -> SiLU-and-mul ->
    down_proj -> residual add -> next input RMSNorm -> qkv_proj -> rope.
    Fused: four tensor-core GEMMs (linear_residual, gate_up_silu with the norm
    factor, linear_residual, qkv_proj_rmsnorm_rotary_embedding); the norms'
    sums of squares come out of the residual GEMMs' epilogues.  Unfused: four
    cuBLAS GEMMs with this package's fused_add_rms_norm (twice), silu_and_mul
    and rotary_embedding between them.  Graphs over 2 weight sets (868 MB);
    the final residual and qkv of the two paths compared within the bf16 rule.
    Reported FLOP rate: the four GEMMs' 2 T (H H + 2 I H + I H + 6144 H)."""
    import torch

    import paceserve_b200 as pb

    nbuf = 2
    n = (NQ + 2 * NKV) * HD
    g_ = torch.Generator(device=dev).manual_seed(23)

    def w(rows, cols):
        return (torch.randn(rows, cols, generator=g_, device=dev) / cols ** 0.5).bfloat16()

    def nw():
        return (torch.randn(H, generator=g_, device=dev) * 0.02 + 1).bfloat16()

    sets = []
    for _ in range(nbuf):
        s_ = {"o": w(H, H), "gu": w(2 * I, H), "down": w(H, I), "qkv": w(n, H), "n2": nw(),
              "n1": nw()}
        s_["gu_f"] = pb.fold_rmsnorm_weight(s_["gu"], s_["n2"])
        s_["qkv_f"] = pb.fold_rmsnorm_weight(s_["qkv"], s_["n1"])
        sets.append(s_)
    cache = rope_cache(dev)
    flops_per_token = 2 * H * (H + 2 * I + I + n)
    rows = []
    for t in tokens:
        attn = [torch.randn(t, H, generator=g_, device=dev).bfloat16() for _ in range(nbuf)]
        res0 = [torch.randn(t, H, generator=g_, device=dev).bfloat16() for _ in range(nbuf)]
        pos = torch.randint(0, MAX_POS, (t,), generator=g_, device=dev)
        res_f = [r.clone() for r in res0]
        res_u = [r.clone() for r in res0]
        ss1 = [torch.empty(t, H // 32, device=dev) for _ in range(nbuf)]
        ss2 = [torch.empty(t, H // 32, device=dev) for _ in range(nbuf)]
        act = [torch.empty(t, I, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        gu = [torch.empty(t, 2 * I, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        xh = [torch.empty(t, H, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        qkv_f = [torch.empty(t, n, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        qkv_u = [torch.empty(t, n, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
        ws = gemm_workspace(dev, t)

        def fused():
            for i, s_ in enumerate(sets):
                pb.layernorm_ops.linear_residual(res_f[i], attn[i], s_["o"], ss1[i], workspace=ws)
                pb.activation_ops.gate_up_silu(act[i], res_f[i], s_["gu_f"], ss1[i], EPS,
                                               workspace=ws)
                pb.layernorm_ops.linear_residual(res_f[i], act[i], s_["down"], ss2[i],
                                                 workspace=ws)
                pb.pos_encoding_ops.qkv_proj_rmsnorm_rotary_embedding(
                    qkv_f[i], res_f[i], s_["qkv_f"], ss2[i], EPS, pos, HD, NQ, NKV, cache, True,
                    workspace=ws)

        def unfused():
            for i, s_ in enumerate(sets):
                torch.matmul(attn[i], s_["o"].t(), out=xh[i])
                pb.layernorm_ops.fused_add_rms_norm(xh[i], res_u[i], s_["n2"], EPS)
                torch.matmul(xh[i], s_["gu"].t(), out=gu[i])
                pb.activation_ops.silu_and_mul(act[i], gu[i])
                torch.matmul(act[i], s_["down"].t(), out=xh[i])
                pb.layernorm_ops.fused_add_rms_norm(xh[i], res_u[i], s_["n1"], EPS)
                torch.matmul(xh[i], s_["qkv"].t(), out=qkv_u[i])
                q = qkv_u[i]
                pb.pos_encoding_ops.rotary_embedding(pos, q[:, : NQ * HD],
                                                     q[:, NQ * HD: (NQ + NKV) * HD], HD, cache,
                                                     True)

        res = {"T": t}
        for name, fn, resets in (("fused_us", fused, res_f), ("unfused_us", unfused, res_u)):
            fn()  # eager once
            gr = capture(fn)
            res[name] = round(time_replays(gr, reps, 3) * 1e3 / (reps * nbuf), 3)
            del gr
            for r_, r0 in zip(resets, res0):  # the residual accumulated over replays
                r_.copy_(r0)
        fused()
        unfused()
        torch.cuda.synchronize()
        res["fused_tflops"] = round(flops_per_token * t / res["fused_us"] / 1e6, 1)
        res["unfused_tflops"] = round(flops_per_token * t / res["unfused_us"] / 1e6, 1)
        res["speedup_vs_unfused"] = round(res["unfused_us"] / res["fused_us"], 3)
        for key, a, b in (("rel_err_residual", res_f[0], res_u[0]),
                          ("rel_err_qkv", qkv_f[0], qkv_u[0])):
            a, b = a.float(), b.float()
            res[key] = round(((a - b).abs().max() / b.abs().max()).item(), 5)
        rows.append(res)
        del attn, res0, res_f, res_u, ss1, ss2, act, gu, xh, qkv_f, qkv_u
        torch.cuda.empty_cache()
    return rows


def _vllm_fused_experts():
    """vLLM's fused_experts (the library version of the reference's Triton
    fused MoE) as a baseline, or the reason it cannot run."""
    try:
        from vllm.model_executor.layers.fused_moe.fused_moe import fused_experts

        return fused_experts
    except Exception as exc:  # reported in the line, never fatal
        return f"{type(exc).__name__}: {exc}"[:200]


def moe_experts_bench(dev, tokens=(64, 512, 4096), reps=5):
    """Mixtral-8x7B expert layer (hidden 4096, intermediate 14336, 8 experts,
    top-2): the fused_experts drop-in (moe_align block 128, row gather, tcgen05
    gate/up GEMM with SiLU-and-mul in the epilogue, tcgen05 down GEMM with the
    routing weight, top-k sum) against the same computation done per expert
    with cuBLAS (torch.matmul on the gathered rows, this package's silu_and_mul,
    index_add_).  bf16, random routing from N(0,1) gating; checked against
    each other within the bf16 rule."""
    import torch

    import paceserve_b200 as pb
    from paceserve_b200 import fused_moe as pb_moe

    E, k, inter = 8, 2, 14336
    g_ = torch.Generator(device=dev).manual_seed(5)
    w1 = (torch.randn(E, 2 * inter, H, generator=g_, device=dev) / H ** 0.5).bfloat16()
    w2 = (torch.randn(E, H, inter, generator=g_, device=dev) / inter ** 0.5).bfloat16()
    peak = peaks()
    rows = []
    for t in tokens:
        x = torch.randn(t, H, generator=g_, device=dev).bfloat16()
        gating = torch.randn(t, E, generator=g_, device=dev)
        tw = torch.empty(t, k, device=dev)
        ids = torch.empty(t, k, dtype=torch.int32, device=dev)
        tei = torch.empty(t, k, dtype=torch.int32, device=dev)
        pb.moe_ops.topk_softmax(tw, ids, tei, gating, True)

        def ours():
            return pb_moe.fused_experts(x, w1, w2, tw, ids)

        def per_expert():
            out = torch.zeros(t, H, dtype=torch.float32, device=dev)
            flat = ids.view(-1).long()
            for e in range(E):
                sel = (flat == e).nonzero(as_tuple=True)[0]
                if sel.numel() == 0:
                    continue
                tok = sel // k
                gu = x[tok] @ w1[e].t()
                act = torch.empty(sel.numel(), inter, dtype=torch.bfloat16, device=dev)
                pb.activation_ops.silu_and_mul(act, gu)
                y = (act @ w2[e].t()).float() * tw.view(-1)[sel][:, None]
                out.index_add_(0, tok, y)
            return out.bfloat16()

        variants = [("fused_experts_us", ours), ("cublas_per_expert_us", per_expert)]
        vllm_fn = _vllm_fused_experts()
        if callable(vllm_fn):
            variants.append(("vllm_fused_experts_us", lambda: vllm_fn(x, w1, w2, tw, ids)))
        res = {"T": t}
        if not callable(vllm_fn):
            res["vllm_fused_experts_us"] = None
            res["vllm_unavailable"] = vllm_fn
        for name, fn in variants:
            try:
                fn()
                torch.cuda.synchronize()
            except Exception as exc:  # only the baseline can fail here
                if name == "fused_experts_us":
                    raise
                res[name] = None
                res["vllm_unavailable"] = f"{type(exc).__name__}: {exc}"[:200]
                continue
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            e1.synchronize()
            res[name] = round(e0.elapsed_time(e1) * 1e3 / reps, 1)
        a, b = ours().float(), per_expert().float()
        torch.cuda.synchronize()
        flops = 2.0 * t * k * (H * 2 * inter + inter * H)
        res["tflops"] = round(flops / (res["fused_experts_us"] * 1e-6) / 1e12, 1)
        res["frac_of_bf16_peak"] = round(res["tflops"] / peak["bf16_tflops"], 4)
        res["speedup_vs_per_expert"] = round(res["cublas_per_expert_us"] / res["fused_experts_us"], 3)
        if res.get("vllm_fused_experts_us"):
            res["speedup_vs_vllm"] = round(res["vllm_fused_experts_us"] / res["fused_experts_us"], 3)
        # roofline: the larger of tensor time and the time to read the experts'
        # weights once (the layer is weight-bound at small T)
        wbytes = 2.0 * (w1.numel() + w2.numel())
        t_roof_us = max(flops / (peak["bf16_tflops"] * 1e12), wbytes / (peak["hbm_gbs"] * 1e9)) * 1e6
        res["roofline_us"] = round(t_roof_us, 1)
        res["frac_of_roofline"] = round(t_roof_us / res["fused_experts_us"], 4)
        res["rel_err_vs_per_expert"] = round(((a - b).abs().max() / b.abs().max()).item(), 5)
        rows.append(res)
    return rows


def tc_calls(dev, tokens: int, calls: int):
    """`calls` eager calls each of the fused qkv projection + rope (Llama-3-8B,
    4096 -> 6144) and of fused_moe (Mixtral-8x7B, E=8, top-2) at `tokens`
    tokens: the launches an ncu capture of the tensor-core kernels selects
    from.  Returns the calls' mean wall time (not a bench figure)."""
    import torch

    import paceserve_b200 as pb
    from paceserve_b200 import fused_moe as pb_moe

    g_ = torch.Generator(device=dev).manual_seed(3)
    n = (NQ + 2 * NKV) * HD
    w = (torch.randn(n, H, generator=g_, device=dev) / H ** 0.5).bfloat16()
    x = torch.randn(tokens, H, generator=g_, device=dev).bfloat16()
    pos = torch.randint(0, MAX_POS, (tokens,), generator=g_, device=dev)
    cache = rope_cache(dev)
    qkv = torch.empty(tokens, n, dtype=torch.bfloat16, device=dev)
    E, k, inter = 8, 2, 14336
    w1 = (torch.randn(E, 2 * inter, H, generator=g_, device=dev) / H ** 0.5).bfloat16()
    w2 = (torch.randn(E, H, inter, generator=g_, device=dev) / inter ** 0.5).bfloat16()
    gating = torch.randn(tokens, E, generator=g_, device=dev)
    t0 = time.perf_counter()
    for _ in range(calls):
        pb.pos_encoding_ops.qkv_proj_rotary_embedding(qkv, x, w, pos, HD, NQ, NKV, cache, True)
        out = pb_moe.fused_moe(x, w1, w2, gating, k, True)
    torch.cuda.synchronize()
    return {"tokens": tokens, "calls": calls,
            "wall_ms_per_call_pair": round((time.perf_counter() - t0) * 1e3 / calls, 3),
            "checksum": round(float(out.float().abs().mean()), 5)}


# ------------------------------------------------------------------ main --
def init_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    return ws, rank, local


def run_reference(args, rank):
    """Reference arm: the reference's own formulas for the path (the oracle port;
    the reference has no CPU implementation of these ops) on the host cores, one
    process with every host thread, rank 0 only.  A step is one pass of the
    32-layer op chain at T=512 (bounded as cpu_chain_run says).  Under torchrun
    the other ranks exit without work: the value is the whole host CPU's rate,
    the same at every N, comparable to the whole job's rate of the GPU arm."""
    if rank != 0:
        return
    base = cpu_chain_run(args.steps, args.warmup, budget_s=90.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens_per_step": T, "layers": L,
                   "scope": "whole host CPU: one process, all cores, independent of N"},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_config1": cpu_config1_sample(),
    }
    print(json.dumps(line), flush=True)


def run_side_workload(args, ws, rank, local):
    import torch

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if args.workload == "kv":
        res = kv_promotion(ws, rank, local, steps=min(args.steps, 50), warmup=args.warmup,
                           baseline=not args.no_cpu_baseline, overlap=ws > 1)
        line = {"metric": "LP->HP KV-promotion GB/s", "n_gpus": ws, "kv_promotion": res}
        if rank == 0:
            torch.cuda.empty_cache()
            line["kv_append"] = append_bench(dev)
            if ws == 1:
                torch.cuda.empty_cache()
                line["kv_overlap"] = kv_overlap(dev)
    elif args.workload == "opgraph":
        # For a graph-level ncu capture of one op's launches (ncu --graph-profiling
        # graph): DRAM bytes counted over the whole graph include the write-backs
        # of each launch's output, which a per-launch capture misses (they leave
        # L2 after the launch ends).  No eager launch precedes the graph.
        import paceserve_b200 as pb

        ch = build_chain(dev, seed=1)
        layers = ch["layers"][: args.layers]
        ln, pe, act = pb.layernorm_ops, pb.pos_encoding_ops, pb.activation_ops
        pos, cache = ch["positions"], ch["cache"]
        one = {
            "silu_and_mul": (lambda b: act.silu_and_mul(b["act"], b["gate_up"]), B_SILU),
            "fused_add_rms_norm": (lambda b: ln.fused_add_rms_norm(b["attn"], b["residual2"],
                                                                   b["w_post"], EPS), B_FUSED),
            "rotary_embedding": (lambda b: pe.rotary_embedding(pos, b["q"], b["k"], HD, cache,
                                                               True), B_ROPE),
            "rms_norm": (lambda b: ln.rms_norm(b["act"][:, :H], b["hidden"], b["w_in"], EPS),
                         B_RMS),
        }[args.op]
        s_ = torch.cuda.Stream()
        s_.wait_stream(torch.cuda.current_stream())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s_):
            for b in layers:
                one[0](b)
        # the replays sit in an NVTX range, so a graph-level ncu capture can
        # select them (ncu --graph-profiling graph --nvtx --nvtx-include opgraph_replays/)
        torch.cuda.nvtx.range_push("opgraph_replays")
        for _ in range(args.steps):
            gr.replay()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        line = {"metric": f"{args.op} graph replays (T=512 Sarathi batch, Llama-3-8B shapes) "
                          "for ncu captures",
                "launches_per_replay": len(layers), "replays": args.steps,
                "algorithmic_bytes_per_launch": one[1]}
    elif args.workload == "sweep":
        line = {"metric": "per-op HBM GB/s, token sweep", "sweep": sweep(dev) if rank == 0 else None,
                "peak_gbs": peaks()["hbm_gbs"]}
    elif args.workload == "tc":
        line = {"metric": "tensor-core ops: fused qkv projection + rope and the MoE expert "
                          "layer, eager calls (for ncu captures)",
                "tc": tc_calls(dev, args.tokens, args.steps)}
    else:
        line = {"metric": "MoE routing us/op", "moe": moe_routing(dev) if rank == 0 else None}
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    global KV_NB
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the config-3 sweep and config-4 MoE keys of the N=1 line")
    ap.add_argument("--kv-blocks", type=int, default=8192,
                    help="blocks per layer of the kv workload's caches (a smaller case for ncu)")
    ap.add_argument("--workload", choices=["chain", "kv", "sweep", "moe", "opgraph", "tc"],
                    default="chain",
                    help="chain: the headline op chain (the driver's line); kv: LP->HP "
                         "promotion; sweep: per-op token sweep; moe: Mixtral-8x7B routing; "
                         "opgraph: one op's launches over distinct layer buffers, as a CUDA "
                         "graph (for ncu captures); tc: --steps eager calls of the fused qkv "
                         "projection + rope (Llama-3-8B) and of fused_moe (Mixtral-8x7B) at "
                         "--tokens tokens (for ncu captures)")
    ap.add_argument("--tokens", type=int, default=512, help="tc: tokens per call")
    ap.add_argument("--layers", type=int, default=32,
                    help="opgraph: launches (layers) per graph")
    ap.add_argument("--op", default="silu_and_mul",
                    choices=["silu_and_mul", "fused_add_rms_norm", "rotary_embedding", "rms_norm"],
                    help="opgraph: the op whose launches the graph holds")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    KV_NB = args.kv_blocks
    if args.impl == "reference":
        # host-CPU arm: no process group, no GPU
        run_reference(args, int(os.environ.get("RANK", "0")))
        return
    ws, rank, local = init_dist()
    if args.workload != "chain":
        run_side_workload(args, ws, rank, local)
        return

    import torch

    import paceserve_b200 as pb

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    ops = (pb.layernorm_ops, pb.pos_encoding_ops, pb.activation_ops)
    ch = build_chain(dev, seed=1234 + rank)
    g = capture(lambda: run_chain(ch, ops))
    sampler = ClockSampler(local)
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()
    blocks = time_blocks(g, args.steps, args.warmup, TIMED_BLOCKS, sampler, ws)
    ms_total = statistics.median(blocks)
    del g
    ms_step = ms_total / args.steps
    value = ws * T * args.steps / (ms_total * 1e-3)
    pk = peaks()
    chain_gbs = B_STEP / (ms_step * 1e-3) / 1e9

    ops_t = per_op_times(ch, ops)
    silu = ops_t["silu_and_mul"]
    roof = {"kernel": "silu_and_mul (act_vec_kernel)", "bound": "hbm",
            "achieved": silu["gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(silu["gbs"] / pk["hbm_gbs"], 4), "peak_source": pk["source"],
            "frac_of_nominal": round(silu["gbs"] / NOMINAL_HBM_GBS, 4),
            "traffic": ncu_traffic("silu_and_mul_T512"),
            "traffic_source": "DRAM read + write per launch from an ncu capture of the whole "
                              "32-launch graph (write-backs included), profiles/ncu_traffic.txt",
            "algorithmic_bytes": B_SILU}
    chs = [ch, build_chain(dev, seed=4321 + rank)]
    e2e = e2e_chain(chs, ops, steps=min(args.steps, 50), warmup=3, ws=ws)
    e2e_parts = e2e_breakdown(chs, ops, steps=min(args.steps, 50), warmup=3, ws=ws)
    del chs
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens_per_step": T, "layers": L,
                   "parallelism": f"{ws} independent replicas" if ws > 1 else "single GPU",
                   "l2": "distinct per-layer buffers, 2.1 GB per step > 126 MB L2 (no flush)",
                   "graph": "one CUDA graph per step, PDL between kernels"},
        "timing": {"blocks": TIMED_BLOCKS, "steps_per_block": args.steps,
                   "ms_per_block": [round(b, 4) for b in blocks],
                   "reported": "median block (each block: barrier + sync, CUDA events, max over ranks)"},
        "chain_hbm": {"bytes_per_step": B_STEP, "achieved_gbs": round(chain_gbs, 1),
                      "frac": round(chain_gbs / pk["hbm_gbs"], 4),
                      "frac_of_nominal": round(chain_gbs / NOMINAL_HBM_GBS, 4)},
        "roofline": roof,
        "ops": ops_t,
        "e2e": e2e,
        "e2e_breakdown": e2e_parts,
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": sampler.summary(),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_chain_run(min(args.steps, 20), 1, budget_s=12.0)
        line["cpu_baseline"]["config1"] = cpu_config1_sample()
    if ws == 1 and not args.no_sweep:
        del ch
        torch.cuda.empty_cache()
        line["sweep"] = {"what": "BASELINE config 3: per-op GB/s, T in {1..16384}, Llama-3-8B and "
                                 "-70B shapes, bf16 and fp16, 32-launch graphs over distinct "
                                 "buffers (>= 512 MB per cycle)",
                         "peak_gbs": pk["hbm_gbs"], "rows": sweep(dev, reps=5)}
        torch.cuda.empty_cache()
        line["moe"] = {"what": "BASELINE config 4: Mixtral-8x7B routing, topk_softmax (E=8, top-2, "
                               "renormalised) + moe_align_block_size (block 64); latency bound",
                       "rows": moe_routing(dev, reps=50)}
        torch.cuda.empty_cache()
        line["qkv_rope"] = {"what": "fused qkv projection + rotary embedding (tcgen05 GEMM, rope in "
                                    "the epilogue; at most 2 tokens: a weight-streaming kernel on "
                                    "CUDA cores) vs cuBLAS GEMM then the rope op; Llama-3-8B "
                                    "4096 -> 6144, bf16, 4 weight buffers per graph (> L2)",
                            "peak_tflops": pk["bf16_tflops"], "rows": qkv_rope_bench(dev)}
        torch.cuda.empty_cache()
        line["norm_gemm"] = {"what": "o_proj + residual add + input RMSNorm + qkv_proj + rope "
                                     "(Llama-3-8B, bf16) as two tensor-core GEMMs with the add, "
                                     "the norm and rope in their epilogues, vs cuBLAS + this "
                                     "package's fused_add_rms_norm and rope",
                             "rows": norm_gemm_bench(dev)}
        torch.cuda.empty_cache()
        line["layer_gemms"] = {"what": "a Llama-3-8B layer minus attention (o_proj, residual, "
                                       "RMSNorm, gate_up, SiLU-and-mul, down, residual, RMSNorm, "
                                       "qkv, rope; bf16) as four GEMMs with the rest in their "
                                       "epilogues (tensor cores; at one token the CUDA-core "
                                       "weight stream, plus row_sumsq twice), vs cuBLAS + this "
                                       "package's ops",
                               "peak_tflops": pk["bf16_tflops"], "rows": layer_gemms_bench(dev)}
        torch.cuda.empty_cache()
        line["moe_experts"] = {"what": "Mixtral-8x7B expert layer (E=8, top-2, 4096 -> 14336 -> "
                                       "4096, bf16): fused_experts on tcgen05 grouped GEMMs vs "
                                       "cuBLAS per expert; eager calls, times include routing "
                                       "alignment, gather and the top-k sum",
                               "peak_tflops": pk["bf16_tflops"], "rows": moe_experts_bench(dev)}
    if ws > 1:
        del ch
        torch.cuda.empty_cache()
        try:
            line["kv_promotion"] = kv_promotion(ws, rank, local, steps=min(args.steps, 20), warmup=3,
                                                overlap=True)
        except Exception as exc:  # reported, never fatal for the chain line
            line["kv_promotion"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
