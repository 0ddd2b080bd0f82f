#!/usr/bin/env python
"""Benchmark of PaceServe's per-layer op chain on B200.

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

# Algorithmic bytes (bf16 activations, fp32 cos/sin cache), per launch at T tokens
B_RMS = 4 * H * T + 2 * H
B_FUSED = 8 * H * T + 2 * H
B_ROPE = 4 * (NQ + NKV) * HD * T + T * HD * 4 + 8 * T
B_SILU = 6 * I * T
B_STEP = B_RMS + B_ROPE + B_FUSED + B_SILU + (L - 1) * (B_FUSED + B_ROPE + B_FUSED + B_SILU)
LAUNCHES_PER_STEP = 4 * L

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
        return {"hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback"}


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


def rope_cache(device):
    """cos/sin cache [MAX_POS, HD] in fp32: [cos | sin] of pos * theta^(-2i/HD)."""
    import torch

    inv = 1.0 / (THETA ** (torch.arange(0, HD, 2, dtype=torch.float64) / HD))
    t = torch.arange(MAX_POS, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], -1).float().to(device)


def build_chain(device, seed=0):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    cpu_gen = torch.Generator().manual_seed(seed)

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
    return {"layers": layers, "positions": make_positions(cpu_gen, device), "cache": rope_cache(device)}


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


def e2e_chain(ch, ops, steps, warmup):
    """Public-API path: pinned host inputs -> device, eager op calls, device -> host output."""
    import torch

    dev = ch["positions"].device
    h_pos = ch["positions"].cpu().pin_memory()
    h_hidden = ch["layers"][0]["hidden"].cpu().pin_memory()
    h_out = torch.empty(T, I, dtype=torch.bfloat16, pin_memory=True)
    out_dev = ch["layers"][-1]["act"]

    def step():
        ch["positions"].copy_(h_pos, non_blocking=True)
        ch["layers"][0]["hidden"].copy_(h_hidden, non_blocking=True)
        run_chain(ch, ops)
        h_out.copy_(out_dev, non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"value": round(T / (ms * 1e-3), 1), "unit": UNIT,
            "h2d_bytes_per_step": h_pos.numel() * 8 + h_hidden.numel() * 2,
            "d2h_bytes_per_step": h_out.numel() * 2, "ms_per_step": round(ms, 4),
            "steps": steps, "path": "eager calls of paceserve_b200 ops (pybind -> C ABI)"}


# ------------------------------------------------------------ CPU oracle --
def cpu_chain_sample(budget_s: float = 8.0, max_passes: int = 1 << 30, warmup: int = 1):
    """The reference formulas (oracle port) on the host cores: time one input-norm
    layer-0 pass and repeated layer>=1 passes at T=512 bf16 (at most `max_passes`,
    stopping after `budget_s` seconds), scale to 32 layers."""
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
    for _ in range(max(1, warmup)):
        ops_ref.chain_layer(1, dict(bufs), cache, pos, EPS, NQ, NKV, HD)
    t0 = time.perf_counter()
    ops_ref.chain_layer(0, dict(bufs), cache, pos, EPS, NQ, NKV, HD)
    t_l0 = time.perf_counter() - t0
    n, t_sum = 0, 0.0
    while n < 2 or (t_sum < budget_s and n < max_passes):
        t0 = time.perf_counter()
        ops_ref.chain_layer(1, bufs, cache, pos, EPS, NQ, NKV, HD)
        t_sum += time.perf_counter() - t0
        n += 1
    t_l = t_sum / n
    step_s = t_l0 + (L - 1) * t_l
    return {"value": round(T / step_s, 1), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"T=512 bf16 op chain on CPU (torch, {cores} threads): 1 layer-0 pass + "
                      f"{n} layer>=1 passes ({t_sum:.1f} s), scaled to 32 layers"}


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


def run_reference(args, ws, rank):
    """Reference arm: each step is one decoder layer of the chain computed by the
    reference's formulas on the host CPU (bounded sample), scaled to 32 layers."""
    if rank != 0:
        return
    base = cpu_chain_sample(budget_s=30.0, max_passes=args.steps, warmup=args.warmup)
    ms = T / base["value"] * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens_per_step": T, "layers": L},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    ws, rank, local = init_dist()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
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
    ms_total = time_replays(g, args.steps, args.warmup, sampler)
    if ws > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = t.item()
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
            "traffic": ncu_traffic("silu_and_mul_T512"),
            "algorithmic_bytes": B_SILU}
    e2e = e2e_chain(ch, ops, steps=min(args.steps, 50), warmup=3)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens_per_step": T, "layers": L,
                   "parallelism": f"{ws} independent replicas" if ws > 1 else "single GPU",
                   "l2": "distinct per-layer buffers, 2.1 GB per step > 126 MB L2 (no flush)",
                   "graph": "one CUDA graph per step, PDL between kernels"},
        "chain_hbm": {"bytes_per_step": B_STEP, "achieved_gbs": round(chain_gbs, 1),
                      "frac": round(chain_gbs / pk["hbm_gbs"], 4)},
        "roofline": roof,
        "ops": ops_t,
        "e2e": e2e,
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": sampler.summary(),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_chain_sample()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
