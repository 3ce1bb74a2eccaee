"""Benchmark of the B200 attention path (BASELINE.json metric).

Default workload: 1B-class decode attention, 16 layers,
32 query heads, 8 KV heads, head_dim 64, fp16 KV cache with 4096 cached
tokens + 1 new token per sequence, batch 64, RoPE theta 5e5. One step = one
decode token for every sequence through all 16 layers (append + attention).
Inputs are synthetic (seeded N(0,1), fp16) and larger than L2 (8.6 GB of
cache per step), so no L2 flush is needed between steps.

Multi-GPU (torchrun): every rank runs the full workload on its own GPU
(batch sharding: each rank owns 64 sequences), no collective on the data
path; `value` is the aggregate over ranks divided by the slowest rank's time.

--impl reference: the reference's attention (the CPU oracle restating
packages/three-llm/src/runtime/math.ts causalAttention) on the host cores,
all threads, on a bounded sample of the same workload.
"""
import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "decode attn GB/s (%HBM) + tok/s @1/2/4/8 B200; prefill attn TFLOP/s"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------- workload definitions
DECODE_1B = dict(name="decode_1b", Hq=32, Hk=8, D=64, T=4096, layers=16, theta=500000.0)


def decode_bytes_per_seq_layer(w):
    """Algorithmic HBM bytes of one sequence's decode in one layer: the K and V of
    T+1 tokens read, Q read and O written, the new K/V read and appended."""
    T1 = w["T"] + 1
    return 2 * T1 * w["Hk"] * w["D"] * 2 + 2 * w["Hq"] * w["D"] * 2 + 2 * w["Hk"] * w["D"] * 2


def decode_flops_per_seq_layer(w):
    return 4 * (w["T"] + 1) * w["D"] * w["Hq"]


PREFILL_05B = dict(name="prefill_05b", Hq=14, Hk=2, D=64, S=2048, B=4, T=4096, theta=1e6)


def prefill_causal_flops(w):
    """Causal FLOPs of one prefill call: 4*D*S(S+1)/2 per (sequence, query head)."""
    return 4 * w["D"] * w["S"] * (w["S"] + 1) // 2 * w["B"] * w["Hq"]


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            names = {
                "hw_slowdown": getattr(pynvml, "nvmlClocksThrottleReasonHwSlowdown", 0x8),
                "hw_thermal_slowdown": getattr(pynvml, "nvmlClocksThrottleReasonHwThermalSlowdown", 0x40),
                "sw_thermal_slowdown": getattr(pynvml, "nvmlClocksThrottleReasonSwThermalSlowdown", 0x20),
                "sw_power_cap": getattr(pynvml, "nvmlClocksThrottleReasonSwPowerCap", 0x4),
            }

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        r = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                        for k, bit in names.items():
                            if r & bit:
                                self.reasons.add(k)
                    except Exception:
                        pass
                    time.sleep(0.01)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- our arm
def fill_cache_random(pkg, layer, gen, torch):
    """Fill a layer's whole fp16 cache with N(0,1) values (stand-in for post-RoPE keys / values)."""
    v = layer.cache_view()
    n = layer.maxBatch * layer.kvHeadCount * layer.maxTokens * layer.headDim

    class _Arr:
        def __init__(self, ptr):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f2", "data": (ptr, False), "version": 3}

    for ptr in (v.key, v.value):
        t = torch.as_tensor(_Arr(ptr), device=layer.device)
        t.normal_(generator=gen)


def run_decode(args, torch, rank, world, device):
    import __graft_entry__ as ge

    pkg = ge.load_package()
    w = dict(DECODE_1B)
    B, L, T = args.batch, w["layers"], w["T"]
    Hq, Hk, D = w["Hq"], w["Hk"], w["D"]
    row = (Hq + 2 * Hk) * D
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + rank)
    layers = []
    for _ in range(L):
        layer = pkg.CUDAAttention(None, Hq * D, Hq, T + 1, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": w["theta"],
                                                            "maxBatch": B, "dtype": torch.float16})
        fill_cache_random(pkg, layer, gen, torch)
        layers.append(layer)
    qkv = torch.randn(L, B, row, generator=gen, device=device).half()
    positions = torch.full((B,), T, dtype=torch.int32, device=device)
    outs = torch.empty(L, B, Hq * D, dtype=torch.float16, device=device)
    stream = torch.cuda.current_stream()

    def step():
        for i in range(L):
            layers[i].decode(qkv[i], positions, out=outs[i])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    # per-launch events on the launching stream give the kernel's average duration
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps * L)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        k = 0
        for _ in range(args.steps):
            for i in range(L):
                ev[k][0].record(stream)
                layers[i].decode(qkv[i], positions, out=outs[i])
                ev[k][1].record(stream)
                k += 1
        stop.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(stop)
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    err = layers[0].context.error()
    if err != 0:
        raise RuntimeError(f"device reported status {err}")

    # end to end through the public API: host (pinned) qkv in, outputs back to the host
    qkv_host = qkv.cpu().pin_memory()
    out_host = torch.empty(L, B, Hq * D, dtype=torch.float16).pin_memory()
    pos_host = positions.cpu().pin_memory()
    qkv_dev = torch.empty_like(qkv)
    pos_dev = torch.empty_like(positions)

    def e2e_step():
        qkv_dev.copy_(qkv_host, non_blocking=True)
        pos_dev.copy_(pos_host, non_blocking=True)
        for i in range(L):
            layers[i].decode(qkv_dev[i], pos_dev, out=outs[i])
        out_host.copy_(outs, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    bytes_per_launch = B * decode_bytes_per_seq_layer(w)
    res = dict(elapsed_ms=elapsed_ms, e2e_ms=e2e_ms, launch_ms=float(np.mean(launch_ms)),
               bytes_per_step=bytes_per_launch * L, bytes_per_launch=bytes_per_launch,
               flops_per_step=B * L * decode_flops_per_seq_layer(w), tokens_per_step=B,
               h2d=qkv.numel() * 2 + positions.numel() * 4, d2h=outs.numel() * 2, launches=args.steps * L,
               clocks=clk.summary())
    for layer in layers:
        layer.close()
    return res


def run_prefill(args, torch, device):
    """causal prefill of 4 x 2048 tokens, 14 q / 2 kv heads, d64,
    RoPE theta 1e6 applied in-kernel, K/V written into a 4096-slot cache. The
    working set fits in L2, so a 256 MiB buffer is rewritten before every timed call."""
    import __graft_entry__ as ge

    pkg = ge.load_package()
    w = PREFILL_05B
    B, S, Hq, Hk, D = w["B"], w["S"], w["Hq"], w["Hk"], w["D"]
    row = (Hq + 2 * Hk) * D
    gen = torch.Generator(device=device)
    gen.manual_seed(99)
    layer = pkg.CUDAAttention(None, Hq * D, Hq, w["T"], {"headDim": D, "kvHeadCount": Hk, "ropeTheta": w["theta"],
                                                         "maxBatch": B, "dtype": torch.float16})
    qkv = torch.randn(B, S, row, generator=gen, device=device).half()
    start = torch.zeros(B, dtype=torch.int32, device=device)
    out = torch.empty(B, S, Hq * D, dtype=torch.float16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        layer.prefill(qkv, start, out=out)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.nvtx.range_push("timed_prefill")
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        layer.prefill(qkv, start, out=out)
        b.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    err = layer.context.error()
    if err != 0:
        raise RuntimeError(f"device reported status {err}")
    flops = prefill_causal_flops(w)
    layer.close()
    return dict(ms=ms, flops=flops, tflops=flops / (ms * 1e-3) / 1e12, launches=2 * args.steps)


# ---------------------------------------------------------------- CPU legs (oracle)
def cpu_decode_sample(threads, layers_in_sample=1, batch=None, heads=None):
    """Time the reference's causalAttention attention loops (the oracle) on a bounded
    sample of the decode workload: `batch` sequences x `heads` query heads of one
    layer at 4096 cached tokens. Returns (GB/s of algorithmic bytes, seconds, description)."""
    from oracle import oracle

    w = DECODE_1B
    Hq, Hk, D, T = w["Hq"], w["Hk"], w["D"], w["T"]
    B = batch or 1
    heads = heads or Hq
    rng = np.random.default_rng(0)
    kc = rng.standard_normal((B, T + 1, Hk * D), dtype=np.float32)
    vc = rng.standard_normal((B, T + 1, Hk * D), dtype=np.float32)
    q = rng.standard_normal((B, Hq * D), dtype=np.float32)
    pos = np.full(B, T, np.int32)
    opts = dict(head_count=Hq, kv_head_count=Hk, head_dim=D)
    oracle.attend_heads(q, pos, kc, vc, 0, min(heads, 2), threads=threads, **opts)  # warm
    t0 = time.perf_counter()
    for _ in range(layers_in_sample):
        oracle.attend_heads(q, pos, kc, vc, 0, heads, threads=threads, **opts)
    dt = time.perf_counter() - t0
    frac = heads / Hq
    nbytes = layers_in_sample * B * decode_bytes_per_seq_layer(w) * frac
    desc = f"{B} seq x {heads}/{Hq} q heads x {layers_in_sample} layer(s) at 4096 cached tokens, fp32 (oracle)"
    return nbytes / dt / 1e9, dt, desc


def run_reference(args):
    from oracle import oracle

    threads = oracle.cpu_count()
    vals = []
    for _ in range(args.warmup):
        cpu_decode_sample(threads, batch=args.ref_batch)
    for _ in range(args.steps):
        gbs, dt, desc = cpu_decode_sample(threads, batch=args.ref_batch)
        vals.append((gbs, dt))
    gbs = statistics.median(v[0] for v in vals)
    dt = statistics.median(v[1] for v in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode_1b: 16 layers x 32q/8kv heads x d64, 4096 cached + 1, batch 64, theta 5e5",
                   "sample": desc},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ref-batch", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if rank == 0:
            if args.steps > 3:
                args.steps = 3  # each reference step is a multi-second CPU sample
            run_reference(args)
        return

    import torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    res = run_decode(args, torch, rank, world, device)
    pre = None if args.no_prefill else run_prefill(args, torch, device)
    t = torch.tensor([res["elapsed_ms"], res["e2e_ms"]], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    elapsed_ms, e2e_ms = float(t[0]), float(t[1])
    hbm, tc, src = peaks()
    if rank == 0:
        ms = elapsed_ms / args.steps
        total_bytes = res["bytes_per_step"] * args.steps * world
        gbs = total_bytes / (elapsed_ms * 1e-3) / 1e9
        e2e_gbs = total_bytes / (e2e_ms * 1e-3) / 1e9
        achieved = res["bytes_per_launch"] / (res["launch_ms"] * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic (seeded N(0,1) fp16 cache and qkv)",
            "config": {"workload": "decode_1b: 16 layers x 32q/8kv heads x d64, fp16 KV, 4096 cached + 1 new, "
                                   "theta 5e5", "batch_per_gpu": args.batch, "global_batch": args.batch * world,
                       "parallelism": f"batch-sharded x{world}",
                       "l2": "inputs (8.6 GB cache per step per GPU) larger than L2; no flush"},
            "tok_s": round(args.batch * world / (ms * 1e-3), 1),
            "hbm_frac": round(gbs / world / hbm, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": None,
                         "kernel": "decode_fast_kernel<64,half>", "peak_source": src,
                         "launch_ms": round(res["launch_ms"], 5)},
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": res["h2d"],
                    "d2h_bytes_per_step": res["d2h"], "ms_per_step": round(e2e_ms / args.steps, 4)},
            "gpu_launches": res["launches"] + (pre["launches"] if pre else 0),
            "clocks": res["clocks"],
        }
        if pre:
            line["prefill"] = {"workload": "prefill_05b: 4 x 2048 tokens, 14q/2kv heads, d64, causal, RoPE theta 1e6 "
                                           "in-kernel, K/V appended to a 4096-slot cache; L2 flushed per call",
                               "tflops": round(pre["tflops"], 2), "ms": round(pre["ms"], 5),
                               "causal_gflop": round(pre["flops"] / 1e9, 3),
                               "frac": round(pre["tflops"] / tc, 4), "peak_tflops": tc, "peak_source": src,
                               "kernels": "rope_append_kernel + prefill_tc_kernel<64,half>"}
        if not args.no_cpu_baseline:
            gb, dt, desc = cpu_decode_sample(1, batch=4, heads=32)
            line["cpu_baseline"] = {"value": round(gb, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                                    "sample": desc + f" ({dt:.2f} s)"}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
