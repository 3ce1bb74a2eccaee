"""Benchmark of the B200 attention path (BASELINE.json metric).

One JSON line on rank 0. The headline is BASELINE config 2 (decode_1b):
16 layers, 32 q / 8 kv heads, d64, fp16 KV, 4096 cached + 1 new token, batch
64 per GPU, RoPE theta 5e5; one step = one decode token for every sequence
through every layer. Multi-GPU: every rank owns its own 64 sequences (batch
sharding, weak scaling, no collective).

The same line carries sub-records for the other configurations, measured the
same way (whole job, device time, max over ranks) at the same GPU count:

  decode_1b_batch  config 2 at batch 1, 8 and 32 per GPU.
  ragged_8b        config 4: 32 layers, 32/8 heads, d128, batch 64 with
                   context lengths U[512, 8192] (seed 0); KV-head groups split
                   across the GPUs (strong scaling, no collective).
  long_ctx_heads   config 5: 32 layers, one sequence of 131072 cached tokens,
                   KV-head groups split across the GPUs (no exchange).
  long_ctx_seq     config 5 split by contiguous token blocks: per layer each
                   GPU decodes its block and the (m, l, o) triples meet in the
                   fused NVLink exchange kernel (one GPU: a plain decode).
  prefill          config 3: causal prefill of 4 x 2048 tokens, 14/2 heads,
                   d64, RoPE theta 1e6 in-kernel, K/V appended to a 4096-slot
                   cache; (sequence, KV-head group) units split across GPUs.

Every record is timed as >= 5 blocks of exactly --steps steps (>= 1 s of
timed work in total for the headline), each block between a barrier and a
device synchronisation, with CUDA events on the launching stream; a block's
time is the maximum over ranks; value / ms_per_step come from the median
block, with p10 / p90 beside it. Decode inputs exceed L2 (no flush); the
prefill working set fits in L2, so a 256 MiB buffer is rewritten before each
timed prefill call (outside its events). Each record with a `parity` entry
checked one layer of the sharded output on rank 0 against the oracle after
its timing (head subsets of the full problem).

--impl reference: the reference's attention (the CPU oracle restating
packages/three-llm/src/runtime/math.ts causalAttention) on all host threads,
each step a bounded sample of the chosen workload.
"""
import argparse
import datetime
import json
import math
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

DECODE_1B = dict(Hq=32, Hk=8, D=64, T=4096, layers=16, theta=500000.0, batch=64)
RAGGED_8B = dict(Hq=32, Hk=8, D=128, layers=32, theta=500000.0, batch=64, lo=512, hi=8192)
LONG_CTX = dict(Hq=32, Hk=8, D=128, T=131072, layers=32, theta=500000.0, batch=1)
PREFILL_05B = dict(Hq=14, Hk=2, D=64, S=2048, B=4, T=4096, theta=1e6)
WORKLOAD_LABELS = {
    "decode_1b": "decode_1b (config 2): 16 layers x 32q/8kv heads x d64, fp16 KV, 4096 cached + 1 new, theta 5e5",
    "ragged_8b": "ragged_8b (config 4): 32 layers x 32q/8kv heads x d128, fp16 KV, batch 64, context U[512, 8192] "
                 "(seed 0), theta 5e5",
    "long_ctx": "long_ctx (config 5): 32 layers x 32q/8kv heads x d128, one sequence, 131072 cached tokens + 1 new, "
                "fp16 KV, theta 5e5",
    "prefill_05b": "prefill_05b (config 3): 4 x 2048 tokens, 14q/2kv heads, d64, causal, RoPE theta 1e6 in-kernel, "
                   "K/V appended to a 4096-slot cache",
}
ATOL, RTOL = 2e-3, 1e-2  # north-star parity bound |a - e| <= ATOL + RTOL |e|
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu
# --set full capture of each kernel (the commands are in profiles/). The decode
# capture is config 2 at batch 16 (134.47 + 3.78 MB for 16 sequences); the
# traffic grows with the sequences a launch covers, so a launch of B sequences
# is B times the per-sequence figure. The prefill capture is the full config-3
# call (18.93 MB read, nothing written back to DRAM).
NCU_DECODE_1B_BYTES_PER_SEQ = (134.466816e6 + 3.778304e6) / 16
NCU_PREFILL_05B_BYTES = 18.933504e6  # read; 0 bytes written


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def decode_seq_bytes(T1, Hq, Hk, D):
    """Algorithmic HBM bytes of one sequence's decode in one layer: K and V of the
    T1 attended tokens read, Q read and O written, the new K/V read and appended."""
    return 2 * T1 * Hk * D * 2 + 2 * Hq * D * 2 + 2 * Hk * D * 2


def ragged_lengths(w):
    return np.random.default_rng(0).integers(w["lo"], w["hi"] + 1, size=w["batch"])


def prefill_causal_flops(D, S, B, Hq):
    """Causal FLOPs of a prefill call: 4*D*S(S+1)/2 per (sequence, query head)."""
    return 4 * D * S * (S + 1) // 2 * B * Hq


def stats(times_ms, steps):
    """Per-step ms of timed blocks: median, p10, p90."""
    a = np.asarray(times_ms, np.float64) / steps
    return {"median": float(np.median(a)), "p10": float(np.percentile(a, 10)), "p90": float(np.percentile(a, 90)),
            "blocks": len(a), "steps_per_block": steps}


def rnd(d, n=4):
    return {k: (round(v, n) if isinstance(v, float) else v) for k, v in d.items()}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML (read-only) while the timed region runs."""

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
            names = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
                     "sw_power_cap": 0x4}

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


# ---------------------------------------------------------------- cache helpers
def cache_tensors(torch, layer):
    """The layer's fp16 K and V caches as torch views [max_batch, Hk, max_tokens, D]."""
    v = layer.cache_view()
    shape = (layer.maxBatch, layer.kvHeadCount, layer.maxTokens, layer.headDim)

    class _Arr:
        def __init__(self, ptr):
            self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (ptr, False), "version": 3}

    return torch.as_tensor(_Arr(v.key), device=layer.device), torch.as_tensor(_Arr(v.value), device=layer.device)


def fill_cache_random(layer, gen, torch):
    """Fill a layer's whole fp16 cache with N(0,1) values (stand-in for post-RoPE keys / values)."""
    for t in cache_tensors(torch, layer):
        t.normal_(generator=gen)


def close_enough(got, exp):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    err = np.abs(got - exp)
    return float(err.max()), bool(np.all(np.isfinite(got)) and np.all(err <= ATOL + RTOL * np.abs(exp)))


# ---------------------------------------------------------------- decode workloads (our arm)
class Decode1B:
    """Config 2. step() launches one step (all layers) on the current stream;
    e2e_step() does the same through pinned host buffers."""

    name = "decode_1b"

    def __init__(self, pkg, torch, device, rank, world, args, batch=None):
        w = DECODE_1B
        self.torch = torch
        B = batch or args.batch
        L, T, Hq, Hk, D = w["layers"], w["T"], w["Hq"], w["Hk"], w["D"]
        gen = torch.Generator(device=device)
        gen.manual_seed(1234 + rank)
        self.layers = []
        for _ in range(L):
            layer = pkg.CUDAAttention(None, Hq * D, Hq, T + 1, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": w["theta"],
                                                                "maxBatch": B, "dtype": torch.float16})
            fill_cache_random(layer, gen, torch)
            self.layers.append(layer)
        self.qkv = torch.randn(L, B, (Hq + 2 * Hk) * D, generator=gen, device=device).half()
        self.pos = torch.full((B,), T, dtype=torch.int32, device=device)
        self.outs = torch.empty(L, B, Hq * D, dtype=torch.float16, device=device)
        self.bytes_per_step = L * B * decode_seq_bytes(T + 1, Hq, Hk, D)
        self.bytes_per_launch = B * decode_seq_bytes(T + 1, Hq, Hk, D)
        self.traffic_per_launch = B * NCU_DECODE_1B_BYTES_PER_SEQ
        self.tokens_per_step = B
        self.launches_per_step = L
        self.kernel = "decode_fast_kernel<64,half>"
        self.config = {"workload": WORKLOAD_LABELS["decode_1b"], "batch_per_gpu": B, "global_batch": B * world,
                       "parallelism": f"batch-sharded x{world}",
                       "l2": f"inputs ({self.bytes_per_step / 1e9:.2f} GB of cache per step per GPU, "
                             f"{self.bytes_per_launch / 1e6:.0f} MB per layer) larger than L2; no flush",
                       "launch": "step captured as one CUDA graph and replayed",
                       "e2e": "eager CUDAAttention.decode calls; per-layer qkv H2D and output D2H on a copy stream, "
                              "overlapping the neighbouring layers' kernels"}
        self.scaling = "weak"
        self.shape = (Hq, Hk, D, w["theta"])

    def step(self, record=None):
        for i, layer in enumerate(self.layers):
            if record:
                record[0]()
            layer.decode(self.qkv[i], self.pos, out=self.outs[i])
            if record:
                record[1]()

    def e2e_setup(self):
        t = self.torch
        self.qkv_host = self.qkv.cpu().pin_memory()
        self.pos_host = self.pos.cpu().pin_memory()
        self.out_host = t.empty(self.outs.shape, dtype=t.float16).pin_memory()
        self.qkv_dev = t.empty_like(self.qkv)
        self.pos_dev = t.empty_like(self.pos)
        self.h2d = self.qkv.numel() * 2 + self.pos.numel() * 4
        self.d2h = self.outs.numel() * 2
        self.copy_stream = t.cuda.Stream()
        self.in_ready = [t.cuda.Event() for _ in self.layers]
        self.out_ready = [t.cuda.Event() for _ in self.layers]

    def e2e_step(self):
        """One step through CUDAAttention.decode from pinned host buffers: each
        layer's qkv is copied in and its output copied out on a copy stream, so
        the transfers of one layer overlap the kernels of its neighbours; the
        step ends when the last output has reached the host."""
        t, main, cs = self.torch, self.torch.cuda.current_stream(), self.copy_stream
        cs.wait_stream(main)  # the previous step's kernels are done with the device buffers
        with t.cuda.stream(cs):
            self.pos_dev.copy_(self.pos_host, non_blocking=True)
            for i in range(len(self.layers)):
                self.qkv_dev[i].copy_(self.qkv_host[i], non_blocking=True)
                self.in_ready[i].record(cs)
        for i, layer in enumerate(self.layers):
            main.wait_event(self.in_ready[i])
            layer.decode(self.qkv_dev[i], self.pos_dev, out=self.outs[i])
            self.out_ready[i].record(main)
        with t.cuda.stream(cs):
            for i in range(len(self.layers)):
                cs.wait_event(self.out_ready[i])
                self.out_host[i].copy_(self.outs[i], non_blocking=True)
        main.wait_stream(cs)

    def check_heads(self):
        """(sequences, query heads of the shard's first KV head) checked against the oracle."""
        return min(4, self.qkv.shape[1])

    def parity(self, world, rank):
        """Layer 0 of this rank, first KV head's query group of a few sequences,
        against the oracle over the same cache rows (run after the timing)."""
        from oracle import oracle

        t = self.torch
        layer = self.layers[0]
        Hq, Hk, D, G = layer.headCount, layer.kvHeadCount, layer.headDim, layer.headCount // layer.kvHeadCount
        nseq = self.check_heads()
        pos = self.pos.cpu().numpy()
        kc, vc = cache_tensors(t, layer)
        T = int(pos[:nseq].max()) + 1
        k_host = kc[:nseq, 0, :T].float().cpu().numpy().copy()  # [n, T, D]: kv head 0
        v_host = vc[:nseq, 0, :T].float().cpu().numpy().copy()
        out = layer.decode(self.qkv[0], self.pos).float().cpu().numpy()
        x = self.qkv[0, :nseq].float().cpu().numpy().reshape(nseq, Hq + 2 * Hk, D)
        sub = np.concatenate([x[:, :G], x[:, Hq:Hq + 1], x[:, Hq + Hk:Hq + Hk + 1]], axis=1).reshape(nseq, -1)
        Hq_, Hk_, D_, theta = self.shape
        exp = oracle.decode_batch(sub, pos[:nseq], k_host, v_host, threads=oracle.cpu_count(), head_count=G,
                                  kv_head_count=1, head_dim=D, rope_theta=theta)
        err, ok = close_enough(out[:nseq, :G * D], exp)
        return {"max_abs_err": err, "ok": ok,
                "checked": f"rank 0, layer 0: {nseq} sequences x query heads 0..{G - 1} (kv head 0) vs oracle"}

    def close(self):
        for layer in self.layers:
            layer.close()


class Ragged8B(Decode1B):
    """Config 4, sharded by KV-head group (each rank: its kv heads of every sequence)."""

    name = "ragged_8b"

    def __init__(self, pkg, torch, device, rank, world, args):
        from three_llm_b200 import sharding

        w = RAGGED_8B
        self.torch = torch
        B, L, Hq, Hk, D = w["batch"], w["layers"], w["Hq"], w["Hk"], w["D"]
        sh = sharding.head_shard(Hq, Hk, world, rank)
        hq, hk = sh.q_count, sh.kv_count
        lens = ragged_lengths(w)
        T = int(lens.max()) + 1
        gen = torch.Generator(device=device)
        gen.manual_seed(77 + rank)
        self.layers = []
        for _ in range(L):
            layer = pkg.CUDAAttention(None, hq * D, hq, T, {"headDim": D, "kvHeadCount": hk, "ropeTheta": w["theta"],
                                                            "maxBatch": B, "dtype": torch.float16})
            fill_cache_random(layer, gen, torch)
            self.layers.append(layer)
        self.qkv = torch.randn(L, B, (hq + 2 * hk) * D, generator=gen, device=device).half()
        self.pos = torch.from_numpy(lens.astype(np.int32)).to(device)
        self.outs = torch.empty(L, B, hq * D, dtype=torch.float16, device=device)
        per_layer = sum(decode_seq_bytes(int(t) + 1, hq, hk, D) for t in lens)
        self.bytes_per_step = L * per_layer
        self.bytes_per_launch = per_layer
        self.traffic_per_launch = None
        self.tokens_per_step = B / world  # a rank computes its heads of every sequence
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        deferred = 2 * sms > 4 * B * hk  # split pairs merged by their own kernel (grid > 4 CTAs per pair)
        self.launches_per_step = L * (2 if deferred else 1)
        self.kernel = "decode_fast_kernel<128,half>" + (" + decode_merge_kernel" if deferred else "")
        self.config = {"workload": WORKLOAD_LABELS["ragged_8b"], "global_batch": B,
                       "parallelism": f"kv-head groups x{world} ({hk} kv / {hq} q heads per GPU)",
                       "l2": "inputs larger than L2; no flush", "launch": "32-layer step as one CUDA graph"}
        self.scaling = "strong"
        self.shape = (Hq, Hk, D, w["theta"])

    def check_heads(self):
        return 8


class LongCtxHeads(Decode1B):
    """Config 5 sharded by KV-head group: rank r holds kv heads [r Hk/N, (r+1) Hk/N)
    of the one 131072-token sequence and their query groups, so its layer is a
    smaller layer, there is no exchange, and the output stays head-sharded for
    a tensor-parallel output projection (as config 4)."""

    name = "long_ctx_heads"

    def __init__(self, pkg, torch, device, rank, world, args):
        from three_llm_b200 import sharding

        w = LONG_CTX
        self.torch = torch
        L, T, Hq, Hk, D = w["layers"], w["T"], w["Hq"], w["Hk"], w["D"]
        sh = sharding.head_shard(Hq, Hk, world, rank)
        hq, hk = sh.q_count, sh.kv_count
        gen = torch.Generator(device=device)
        gen.manual_seed(5 + rank)
        self.layers = []
        for _ in range(L):
            layer = pkg.CUDAAttention(None, hq * D, hq, T + 1, {"headDim": D, "kvHeadCount": hk,
                                                                "ropeTheta": w["theta"], "dtype": torch.float16})
            fill_cache_random(layer, gen, torch)
            self.layers.append(layer)
        self.qkv = torch.randn(L, 1, (hq + 2 * hk) * D, generator=gen, device=device).half()
        self.pos = torch.full((1,), T, dtype=torch.int32, device=device)
        self.outs = torch.empty(L, 1, hq * D, dtype=torch.float16, device=device)
        self.bytes_per_step = L * decode_seq_bytes(T + 1, hq, hk, D)
        self.bytes_per_launch = decode_seq_bytes(T + 1, hq, hk, D)
        self.traffic_per_launch = None
        self.tokens_per_step = 1 / world  # the ranks together produce the sequence's next token
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        deferred = 2 * sms > 4 * hk
        self.launches_per_step = L * (2 if deferred else 1)
        self.kernel = "decode_fast_kernel<128,half>" + (" + decode_merge_kernel" if deferred else "")
        self.config = {"workload": WORKLOAD_LABELS["long_ctx"], "global_batch": 1,
                       "parallelism": f"kv-head groups x{world} ({hk} kv / {hq} q heads per GPU, no exchange)",
                       "l2": "inputs larger than L2; no flush", "launch": "32-layer step as one CUDA graph"}
        self.scaling = "strong"
        self.shape = (Hq, Hk, D, w["theta"])

    def check_heads(self):
        return 1


class LongCtxSeq:
    """Config 5 sharded by token blocks: each rank decodes its block and the
    per-head (m, l, o) triples meet in the fused peer exchange (or an NCCL
    all-gather with --exchange nccl)."""

    name = "long_ctx_seq"

    def __init__(self, pkg, torch, device, rank, world, args):
        from three_llm_b200 import sharding

        w = LONG_CTX
        self.torch = torch
        L, T, Hq, Hk, D = w["layers"], w["T"], w["Hq"], w["Hk"], w["D"]
        gen = torch.Generator(device=device)
        gen.manual_seed(5 + rank)
        self.shards = []
        self.exchange = None
        mode = getattr(args, "exchange", "p2p")
        if world > 1 and mode == "p2p":  # one peer exchange serves all layers
            self.exchange = sharding.PeerExchange(rank, world, Hq * (D + 2) * 4, device)
        for _ in range(L):
            s = sharding.SequenceShardedDecode(Hq, Hk, D, T, rank, world, {"ropeTheta": w["theta"]},
                                               exchange=mode, peer_exchange=self.exchange)
            fill_cache_random(s.layer, gen, torch)
            self.shards.append(s)
        self.layers = [s.layer for s in self.shards]
        g0 = torch.Generator(device=device)
        g0.manual_seed(5)  # identical queries on every rank
        self.qkv = torch.randn(L, 1, (Hq + 2 * Hk) * D, generator=g0, device=device).half()
        self.pos = torch.full((1,), T, dtype=torch.int32, device=device)
        local = self.shards[0].shard.tokens + (1 if self.shards[0].shard.owns_next else 0)
        self.bytes_per_step = L * decode_seq_bytes(T + 1, Hq, Hk, D) / world  # this rank's share
        self.bytes_per_launch = decode_seq_bytes(local, Hq, Hk, D)
        self.traffic_per_launch = None
        self.tokens_per_step = 1 / world
        # one GPU: decode + merge; p2p: decode + fused merge/exchange; nccl: decode + merge + combine
        self.launches_per_step = (2 if world == 1 or mode == "p2p" else 3) * L
        if world == 1:
            self.kernel = "decode_fast_kernel<128,half> + decode_merge_kernel (one shard: plain decode)"
            xname = "none"
        elif mode == "p2p":
            self.kernel = ("decode_fast_kernel<128,half> partial + decode_exchange_kernel "
                           "(segment merge, NVLink exchange, LSE merge)")
            xname = "fused segment merge + peer-memory exchange (NVLink stores, epoch-word wait) + LSE merge"
        else:
            self.kernel = "decode_fast_kernel<128,half> partial + NCCL all-gather + combine_lse_kernel"
            xname = "NCCL all-gather of (m,l,o) + LSE merge"
        self.config = {"workload": WORKLOAD_LABELS["long_ctx"], "global_batch": 1,
                       "parallelism": f"sequence blocks x{world}, {xname} per layer",
                       "l2": "inputs larger than L2; no flush",
                       "launch": "32-layer step as one CUDA graph (partial kernel, exchange, merge)"}
        self.scaling = "strong"
        self.outs = torch.empty(L, 1, Hq * D, dtype=torch.float16, device=device)
        self.world, self.rank = world, rank
        self.shape = (Hq, Hk, D, w["theta"])

    def step(self, record=None):
        for i, s in enumerate(self.shards):
            if record:
                record[0]()
            self.outs[i].copy_(s.step(self.qkv[i], self.pos))
            if record:
                record[1]()

    def parity(self, world, rank):
        """Layer 0's merged output, query heads of kv head 0, against the oracle over
        the whole sequence: every rank's block of kv head 0 is gathered to rank 0."""
        from oracle import oracle

        t = self.torch
        s0 = self.shards[0]
        Hq, Hk, D, theta = self.shape
        G = Hq // Hk
        kc, vc = cache_tensors(t, s0.layer)
        n = s0.shard.tokens
        k_loc = kc[0, 0, :n].contiguous()
        v_loc = vc[0, 0, :n].contiguous()
        if world > 1:
            ks = [t.empty_like(k_loc) for _ in range(world)]
            vs = [t.empty_like(v_loc) for _ in range(world)]
            t.distributed.all_gather(ks, k_loc)
            t.distributed.all_gather(vs, v_loc)
        else:
            ks, vs = [k_loc], [v_loc]
        out = s0.step(self.qkv[0], self.pos).float().cpu().numpy()
        t.cuda.synchronize()
        if rank != 0:
            return None
        k_host = t.cat(ks).float().cpu().numpy()[None].copy()  # [1, T, D]
        v_host = t.cat(vs).float().cpu().numpy()[None].copy()
        T = k_host.shape[1]
        k_host = np.concatenate([k_host, np.zeros((1, 1, D), np.float32)], axis=1)
        v_host = np.concatenate([v_host, np.zeros((1, 1, D), np.float32)], axis=1)
        x = self.qkv[0, :1].float().cpu().numpy().reshape(1, Hq + 2 * Hk, D)
        sub = np.concatenate([x[:, :G], x[:, Hq:Hq + 1], x[:, Hq + Hk:Hq + Hk + 1]], axis=1).reshape(1, -1)
        exp = oracle.decode_batch(sub, [T], k_host, v_host, threads=oracle.cpu_count(), head_count=G,
                                  kv_head_count=1, head_dim=D, rope_theta=theta)
        err, ok = close_enough(out[:1, :G * D], exp)
        return {"max_abs_err": err, "ok": ok,
                "checked": f"rank 0, layer 0: merged output of query heads 0..{G - 1} over all {world} token blocks "
                           f"({T} tokens, gathered) vs oracle"}

    def close(self):
        for s in self.shards:
            s.close()
        if self.exchange is not None:
            self.exchange.close()


# ---------------------------------------------------------------- timing
def timed_blocks(torch, run, steps, repeats, world, per_call=None):
    """`repeats` blocks of exactly `steps` calls of run(), each between a barrier and
    a synchronize, timed with CUDA events on the current stream; per_call (a
    callable run before each call, outside the events) switches to per-call
    events. Returns per-block ms, max over ranks."""
    stream = torch.cuda.current_stream()
    out = []
    for _ in range(repeats):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        if per_call is None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(steps):
                run()
            b.record(stream)
            torch.cuda.synchronize()
            out.append(a.elapsed_time(b))
        else:
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for a, b in ev:
                per_call()
                a.record(stream)
                run()
                b.record(stream)
            torch.cuda.synchronize()
            out.append(sum(a.elapsed_time(b) for a, b in ev))
    t = torch.tensor(out, dtype=torch.float64, device=torch.cuda.current_device())
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(x) for x in t.cpu().tolist()]


def agree_repeats(torch, est_ms, min_seconds, world, lo=5, hi=4000):
    """Blocks so that the timed work is >= min_seconds, the same on every rank."""
    t = torch.tensor([est_ms], dtype=torch.float64, device=torch.cuda.current_device())
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    est = max(float(t.item()), 1e-3)
    return int(min(hi, max(lo, math.ceil(min_seconds * 1e3 / est))))


def measure_decode(torch, wl, args, world, device, min_seconds, clocks=False, eager_launches=False):
    """Warm-up, optional eager per-launch events, CUDA-graph capture of one step,
    then repeated blocks of exactly --steps replays. Returns (stats, extras)."""
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    extras = {}
    if eager_launches:  # kernel-only launch times, eager (PDL prologues not overlapped)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(len(wl.layers))]
        k = [0]

        def rec_start():
            ev[k[0]][0].record(stream)

        def rec_stop():
            ev[k[0]][1].record(stream)
            k[0] += 1

        wl.step((rec_start, rec_stop))
        torch.cuda.synchronize()
        extras["eager_launch_ms"] = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        wl.step()
    stream.wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        wl.step()
    graph.replay()
    torch.cuda.synchronize()
    est = timed_blocks(torch, graph.replay, args.steps, 1, world)[0]
    repeats = agree_repeats(torch, est, min_seconds, world)
    sampler = ClockSampler(device.index) if clocks else None
    if sampler:
        sampler.__enter__()
    try:
        times = timed_blocks(torch, graph.replay, args.steps, repeats, world)
    finally:
        if sampler:
            sampler.__exit__()
    del graph  # may hold NCCL work: release before the process group goes away
    torch.cuda.synchronize()
    err = wl.layers[0].context.error()
    if err != 0:
        raise RuntimeError(f"device reported status {err}")
    if sampler:
        extras["clocks"] = sampler.summary()
    extras["timed_s"] = sum(times) / 1e3
    return stats(times, args.steps), extras


def measure_e2e(torch, wl, args, world):
    wl.e2e_setup()
    for _ in range(max(1, args.warmup)):
        wl.e2e_step()
    torch.cuda.synchronize()
    return timed_blocks(torch, wl.e2e_step, args.steps, 1, world)[0] / args.steps


def decode_record(wl, st, world, hbm):
    ms = st["median"]
    gbs = wl.bytes_per_step * world / (ms * 1e-3) / 1e9
    return {"ms_per_step": round(ms, 5), "ms_p10": round(st["p10"], 5), "ms_p90": round(st["p90"], 5),
            "blocks": st["blocks"], "gbs": round(gbs, 2), "frac": round(gbs / world / hbm, 4),
            "tok_s": round(wl.tokens_per_step * world / (ms * 1e-3), 1), "scaling": wl.scaling,
            "kernel": wl.kernel, "gpu_launches": int(st["blocks"] * st["steps_per_block"] * wl.launches_per_step)}


# ---------------------------------------------------------------- prefill (config 3)
class Prefill05B:
    """Config 3; on N GPUs each rank holds (sequence, KV-head group) units
    (sharding.batch_head_shard): a smaller layer over its own sequences."""

    def __init__(self, pkg, torch, device, rank, world):
        from three_llm_b200 import sharding

        w = PREFILL_05B
        self.torch = torch
        B, S, Hq, Hk, D = w["B"], w["S"], w["Hq"], w["Hk"], w["D"]
        sh = sharding.batch_head_shard(B, Hq, Hk, world, rank)
        self.sh = sh
        self.b, self.hq, self.hk = sh.seq_count, sh.q_count, sh.kv_count
        g = torch.Generator(device=device)
        g.manual_seed(99)  # the full problem on every rank, then this rank's slice
        full = torch.randn(B, S, (Hq + 2 * Hk) * D, generator=g, device=device).half()
        rows = full[sh.seq_begin:sh.seq_begin + sh.seq_count].reshape(-1, (Hq + 2 * Hk) * D)
        self.qkv = sharding.slice_qkv_for_heads(rows, sh, Hq, Hk, D).view(self.b, S, -1)
        del full
        self.layer = pkg.CUDAAttention(None, self.hq * D, self.hq, w["T"],
                                       {"headDim": D, "kvHeadCount": self.hk, "ropeTheta": w["theta"],
                                        "maxBatch": self.b, "dtype": torch.float16})
        self.start = torch.zeros(self.b, dtype=torch.int32, device=device)
        self.out = torch.empty(self.b, S, self.hq * D, dtype=torch.float16, device=device)
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.flops = prefill_causal_flops(D, S, B, Hq)  # whole job
        self.S, self.D = S, D

    def call(self):
        self.layer.prefill(self.qkv, self.start, out=self.out)

    def e2e_setup(self):
        t = self.torch
        self.qkv_host = self.qkv.cpu().pin_memory()
        self.start_host = self.start.cpu().pin_memory()
        self.out_host = t.empty(self.out.shape, dtype=t.float16).pin_memory()
        self.qkv_dev = t.empty_like(self.qkv)
        self.start_dev = t.empty_like(self.start)
        self.h2d = self.qkv.numel() * 2 + self.start.numel() * 4
        self.d2h = self.out.numel() * 2

    def e2e_call(self):
        self.qkv_dev.copy_(self.qkv_host, non_blocking=True)
        self.start_dev.copy_(self.start_host, non_blocking=True)
        self.layer.prefill(self.qkv_dev, self.start_dev, out=self.out)
        self.out_host.copy_(self.out, non_blocking=True)

    def parity(self, rank, tokens=512):
        """The first `tokens` positions of this rank's first sequence, query heads
        of its first KV head, against the oracle's token-by-token replay (position
        p depends only on positions <= p)."""
        from oracle import oracle

        G = self.hq // self.hk
        x = self.qkv[0, :tokens].float().cpu().numpy().reshape(tokens, self.hq + 2 * self.hk, self.D)
        sub = np.concatenate([x[:, :G], x[:, self.hq:self.hq + 1], x[:, self.hq + self.hk:self.hq + self.hk + 1]],
                             axis=1).reshape(1, tokens, -1)
        kc = np.zeros((1, tokens, self.D), np.float32)
        vc = np.zeros_like(kc)
        exp = oracle.prefill(sub, [0], kc, vc, threads=oracle.cpu_count(), head_count=G, kv_head_count=1,
                             head_dim=self.D, rope_theta=PREFILL_05B["theta"])
        got = self.out[0, :tokens].float().cpu().numpy()[:, :G * self.D]
        err, ok = close_enough(got, exp[0])
        return {"max_abs_err": err, "ok": ok,
                "checked": f"rank {rank}: sequence {self.sh.seq_begin}, query heads {self.sh.q_begin}.."
                           f"{self.sh.q_begin + G - 1}, positions 0..{tokens - 1} vs oracle replay"}

    def close(self):
        self.layer.close()


def run_prefill(pkg, torch, device, rank, world, args, tc, src, cpu=True):
    pf = Prefill05B(pkg, torch, device, rank, world)
    for _ in range(max(3, args.warmup)):
        pf.call()
    torch.cuda.synchronize()
    steps = args.steps
    est = timed_blocks(torch, pf.call, steps, 1, world, per_call=pf.flush.zero_)[0]
    repeats = agree_repeats(torch, est, min(0.05, args.sub_seconds), world, lo=5, hi=200)
    times = timed_blocks(torch, pf.call, steps, repeats, world, per_call=pf.flush.zero_)
    st = stats(times, steps)
    err = pf.layer.context.error()
    if err != 0:
        raise RuntimeError(f"device reported status {err}")
    pf.e2e_setup()
    for _ in range(2):
        pf.e2e_call()
    torch.cuda.synchronize()
    e2e_ms = timed_blocks(torch, pf.e2e_call, steps, 1, world, per_call=pf.flush.zero_)[0] / steps
    pf.call()
    parity = pf.parity(rank) if rank == 0 else None
    ms = st["median"]
    tflops = pf.flops / (ms * 1e-3) / 1e12
    rec = {"workload": WORKLOAD_LABELS["prefill_05b"] + "; L2 flushed before each call (outside its events)",
           "parallelism": f"(sequence, kv-head group) units x{world} ({pf.b} seq x {pf.hk} kv / {pf.hq} q heads "
                          "per GPU)",
           "tflops": round(tflops, 2), "ms": round(ms, 5), "ms_p10": round(st["p10"], 5),
           "ms_p90": round(st["p90"], 5), "calls": st["blocks"] * steps, "causal_gflop": round(pf.flops / 1e9, 3),
           "frac": round(tflops / world / tc, 4), "peak_tflops": tc, "peak_source": src,
           "kernels": "rope_rows_kernel<64> + prefill_pp_kernel<half> (persistent, two query tiles per CTA)",
           "gpu_launches": int(2 * st["blocks"] * steps), "scaling": "strong",
           "e2e": {"tflops": round(pf.flops / (e2e_ms * 1e-3) / 1e12, 2), "ms": round(e2e_ms, 5),
                   "h2d_bytes_per_call": pf.h2d, "d2h_bytes_per_call": pf.d2h,
                   "how": "pinned-host qkv H2D, CUDAAttention.prefill, output D2H, per call"}}
    if parity is not None:
        rec["parity"] = parity
    if cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_prefill_sample(1, min_seconds=5.0)
    pf.close()
    return rec


# ---------------------------------------------------------------- projections around the attention
HIDDEN_1B, HIDDEN_05B, HIDDEN_8B = 2048, 896, 4096


class QkvDecode1B(Decode1B):
    """Config 2 with the QKV projection in front (Llama-3.2-1B shapes: hidden
    2048): every layer is one tla_qkv_decode, the tcgen05 projection whose
    epilogue does QK-norm / RoPE / append, then the decode kernel."""

    name = "qkv_decode_1b"

    def __init__(self, pkg, torch, device, rank, world, args):
        super().__init__(pkg, torch, device, rank, world, args)
        Hq, Hk, D = DECODE_1B["Hq"], DECODE_1B["Hk"], DECODE_1B["D"]
        L, B, H = len(self.layers), self.qkv.shape[1], HIDDEN_1B
        N = (Hq + 2 * Hk) * D
        g = torch.Generator(device=device)
        g.manual_seed(31 + rank)
        self.x = torch.randn(L, B, H, generator=g, device=device).half()
        self.w = (torch.randn(L, H, N, generator=g, device=device) / math.sqrt(H)).half()
        self.b = torch.randn(L, N, generator=g, device=device) * 0.1
        self.lib = pkg.lib()
        self.bytes_per_step += L * (H * N * 2 + B * H * 2)
        self.bytes_per_launch = self.bytes_per_step / L
        self.launches_per_step = 2 * L
        self.kernel = "proj_tc_kernel<64> (QKV + QK-norm/RoPE/append epilogue) + decode_fast_kernel<64,half>"
        self.config = dict(self.config, parallelism=f"batch-sharded x{world}",
                           projection=f"x [{B}, {H}] @ W [{H}, {N}] fp16 + bias per layer")

    def step(self, record=None):
        import ctypes

        s = ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)
        for i, layer in enumerate(self.layers):
            if record:
                record[0]()
            rc = self.lib.tla_qkv_decode(layer.handle, ctypes.c_void_p(self.x[i].data_ptr()),
                                         ctypes.c_void_p(self.w[i].data_ptr()), ctypes.c_void_p(self.b[i].data_ptr()),
                                         HIDDEN_1B, ctypes.c_void_p(self.pos.data_ptr()), None,
                                         ctypes.c_void_p(self.outs[i].data_ptr()), self.x.shape[1], s)
            if rc:
                raise RuntimeError(f"tla_qkv_decode: {rc}")
            if record:
                record[1]()

    def e2e_setup(self):
        super().e2e_setup()
        self.h2d = self.x.numel() * 2 + self.pos.numel() * 4
        self.x_host = self.x.cpu().pin_memory()

    def e2e_step(self):
        self.x.copy_(self.x_host, non_blocking=True)
        self.step()
        self.out_host.copy_(self.outs, non_blocking=True)

    def parity(self, world, rank):
        from oracle import oracle

        t = self.torch
        layer = self.layers[0]
        Hq, Hk, D = layer.headCount, layer.kvHeadCount, layer.headDim
        G, n = Hq // Hk, 4
        pos = self.pos.cpu().numpy()
        kc, vc = cache_tensors(t, layer)
        T = int(pos[:n].max()) + 1
        k_host = kc[:n, 0, :T].float().cpu().numpy().copy()
        v_host = vc[:n, 0, :T].float().cpu().numpy().copy()
        self.step()
        out = self.outs[0, :n].float().cpu().numpy()
        cols = np.r_[0:G * D, Hq * D:(Hq + 1) * D, (Hq + Hk) * D:(Hq + Hk + 1) * D]
        x = self.x[0, :n].float().cpu().numpy()
        w = self.w[0].float().cpu().numpy()[:, cols]
        b = self.b[0].float().cpu().numpy()[cols]
        qkv = oracle.linear(x, w, b, threads=oracle.cpu_count())
        exp = oracle.decode_batch(qkv, pos[:n], k_host, v_host, threads=oracle.cpu_count(), head_count=G,
                                  kv_head_count=1, head_dim=D, rope_theta=DECODE_1B["theta"])
        err, ok = close_enough(out[:, :G * D], exp)
        return {"max_abs_err": err, "ok": ok,
                "checked": f"rank 0, layer 0: {n} sequences x query heads 0..{G - 1}: oracle linear + attention"}


def run_qkv_prefill(pkg, torch, device, rank, world, args, tc):
    """Config 3 from the hidden states (Qwen2-0.5B shapes, hidden 896): the fused
    projection (tcgen05, QK-norm / RoPE / append epilogue) then the causal
    tensor-core attention; the FLOPs counted are the projection's plus the
    causal attention's."""
    import ctypes

    from three_llm_b200 import sharding

    w_ = PREFILL_05B
    B, S, Hq, Hk, D, H = w_["B"], w_["S"], w_["Hq"], w_["Hk"], w_["D"], HIDDEN_05B
    sh = sharding.batch_head_shard(B, Hq, Hk, world, rank)
    g = torch.Generator(device=device)
    g.manual_seed(98)
    N = (Hq + 2 * Hk) * D
    x_full = torch.randn(B, S, H, generator=g, device=device).half()
    w_full = (torch.randn(H, N, generator=g, device=device) / math.sqrt(H)).half()
    b_full = torch.randn(N, generator=g, device=device) * 0.1
    heads = list(range(sh.q_begin, sh.q_begin + sh.q_count)) + \
        [Hq + k for k in range(sh.kv_begin, sh.kv_begin + sh.kv_count)] + \
        [Hq + Hk + k for k in range(sh.kv_begin, sh.kv_begin + sh.kv_count)]
    cols = torch.cat([torch.arange(h * D, (h + 1) * D, device=device) for h in heads])
    x = x_full[sh.seq_begin:sh.seq_begin + sh.seq_count].contiguous()
    w = w_full[:, cols].contiguous()
    b = b_full[cols].contiguous()
    layer = pkg.CUDAAttention(None, sh.q_count * D, sh.q_count, w_["T"],
                              {"headDim": D, "kvHeadCount": sh.kv_count, "ropeTheta": w_["theta"],
                               "maxBatch": sh.seq_count, "dtype": torch.float16})
    start = torch.zeros(sh.seq_count, dtype=torch.int32, device=device)
    out = torch.empty(sh.seq_count, S, sh.q_count * D, dtype=torch.float16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    lib = pkg.lib()

    def call():
        rc = lib.tla_qkv_prefill(layer.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                 ctypes.c_void_p(b.data_ptr()), H, ctypes.c_void_p(start.data_ptr()), None, S,
                                 ctypes.c_void_p(out.data_ptr()), sh.seq_count,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if rc:
            raise RuntimeError(f"tla_qkv_prefill: {rc}")

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    est = timed_blocks(torch, call, args.steps, 1, world, per_call=flush.zero_)[0]
    repeats = agree_repeats(torch, est, min(0.05, args.sub_seconds), world, lo=5, hi=200)
    st = stats(timed_blocks(torch, call, args.steps, repeats, world, per_call=flush.zero_), args.steps)
    if layer.context.error() != 0:
        raise RuntimeError("device reported an error")
    flops = prefill_causal_flops(D, S, B, Hq) + 2 * B * S * H * N
    ms = st["median"]
    rec = {"workload": "config 3 from hidden states: x [4, 2048, 896] @ W_qkv [896, 1152] + bias, QK-norm-free "
                       "RoPE theta 1e6 + append in the GEMM epilogue, then causal attention; L2 flushed per call",
           "parallelism": f"(sequence, kv-head group) units x{world}",
           "tflops": round(flops / (ms * 1e-3) / 1e12, 2), "ms": round(ms, 5), "ms_p10": round(st["p10"], 5),
           "ms_p90": round(st["p90"], 5), "gflop": round(flops / 1e9, 3),
           "frac": round(flops / (ms * 1e-3) / 1e12 / world / tc, 4),
           "kernels": "proj_tc_kernel<64> (QKV + RoPE/append epilogue) + prefill_pp_kernel<half>",
           "gpu_launches": int(2 * st["blocks"] * args.steps)}
    if rank == 0:  # first 256 positions of the rank's first sequence, first kv head's query group
        from oracle import oracle

        n, G = 256, sh.q_count // sh.kv_count
        sub_heads = list(range(G)) + [sh.q_count, sh.q_count + sh.kv_count]
        sc = torch.cat([torch.arange(h * D, (h + 1) * D, device=device) for h in sub_heads])
        qkv = oracle.linear(x[0, :n].float().cpu().numpy(), w[:, sc].float().cpu().numpy(),
                            b[sc].float().cpu().numpy(), threads=oracle.cpu_count())[None]
        kc = np.zeros((1, n, D), np.float32)
        vc = np.zeros_like(kc)
        exp = oracle.prefill(qkv, [0], kc, vc, threads=oracle.cpu_count(), head_count=G, kv_head_count=1, head_dim=D,
                             rope_theta=w_["theta"])
        err, ok = close_enough(out[0, :n, :G * D].float().cpu().numpy(), exp[0])
        rec["parity"] = {"max_abs_err": err, "ok": ok, "checked": f"rank 0: positions 0..{n - 1}, query heads of its "
                                                                  "first kv head: oracle linear + replay"}
    layer.close()
    return rec


def run_out_proj(pkg, torch, device, rank, world, args, hbm):
    """The attention output projection + residual of config 4 (8B shapes: 32
    query heads x d128 = 4096 inputs, hidden 4096), batch 64, 32 layers per
    step. One GPU: tla_out_proj. N GPUs: the query heads are sharded, each rank
    multiplies its 4096/N input columns by its rows of W and
    tla_out_proj_allreduce sums the partials over NVLink (GEMM epilogue stores
    into the owner's buffer, then one finishing kernel); beside it the same
    partials summed by an NCCL all-reduce."""
    from three_llm_b200 import sharding

    rows, fin, H, L = 64, 32 * 128, HIDDEN_8B, 32
    per = fin // world
    g = torch.Generator(device=device)
    g.manual_seed(61)  # the full problem on every rank
    attn = torch.randn(L, rows, fin, generator=g, device=device).half()
    w = (torch.randn(L, fin, H, generator=g, device=device) / math.sqrt(fin)).half()
    bias = torch.randn(L, H, generator=g, device=device) * 0.1
    res = torch.randn(L, rows, H, generator=g, device=device).half()
    a_r = attn[:, :, rank * per:(rank + 1) * per].contiguous()
    w_r = w[:, rank * per:(rank + 1) * per].contiguous()
    del attn, w
    y = torch.empty(L, rows, H, dtype=torch.float16, device=device)
    ctx = pkg.Context.default(device.index or 0)
    op = sharding.HeadShardedOutProj(rows, H, rank, world, device, context=ctx) if world > 1 else None
    import ctypes

    lib = pkg.lib()

    def step():
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for i in range(L):
            if op is not None:
                op(a_r[i], w_r[i], bias[i], res[i], out=y[i])
            else:
                rc = lib.tla_out_proj(ctx.handle, ctypes.c_void_p(a_r[i].data_ptr()),
                                      ctypes.c_void_p(w_r[i].data_ptr()), ctypes.c_void_p(bias[i].data_ptr()),
                                      ctypes.c_void_p(res[i].data_ptr()), ctypes.c_void_p(y[i].data_ptr()), rows,
                                      per, H, 0, s)
                if rc:
                    raise RuntimeError(f"tla_out_proj: {rc}")

    def measure(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()  # the 32-layer step replayed as one graph
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        torch.cuda.synchronize()
        est = timed_blocks(torch, graph.replay, args.steps, 1, world)[0]
        out = stats(timed_blocks(torch, graph.replay, args.steps, agree_repeats(torch, est, args.sub_seconds, world),
                                 world), args.steps)
        del graph  # may hold NCCL work: released before the process group goes away
        torch.cuda.synchronize()
        return out

    st = measure(step)
    if ctx.error() != 0:
        raise RuntimeError("device reported an error")
    ms = st["median"]
    wbytes = L * per * H * 2 * world
    rec = {"workload": "output projection + residual, 8B shapes: attn [64, 4096] @ W_o [4096, 4096] + bias + "
                       "residual, 32 layers per step",
           "parallelism": (f"query heads x{world}: partial GEMM per rank, NVLink reduce-scatter from the GEMM "
                           "epilogue + all-gather kernel" if world > 1 else "one GPU"),
           "ms_per_step": round(ms, 5), "ms_p10": round(st["p10"], 5), "ms_p90": round(st["p90"], 5),
           "us_per_layer": round(ms * 1e3 / L, 2), "weight_gbs": round(wbytes / (ms * 1e-3) / 1e9, 1),
           "frac": round(wbytes / world / (ms * 1e-3) / 1e9 / hbm, 4),
           "gpu_launches": int(st["blocks"] * args.steps * L * (2 if world > 1 else 1))}
    if world > 1:  # the same partial products summed by NCCL, for comparison
        part = torch.empty(L, rows, H, dtype=torch.float32, device=device)

        def nccl_step():
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for i in range(L):
                lib.tla_out_proj(ctx.handle, ctypes.c_void_p(a_r[i].data_ptr()), ctypes.c_void_p(w_r[i].data_ptr()),
                                 None, None, ctypes.c_void_p(part[i].data_ptr()), rows, per, H, 4, s)
                torch.distributed.all_reduce(part[i])
                y[i].copy_(part[i] + bias[i] + res[i])

        rec["nccl_allreduce_ms_per_step"] = round(measure(nccl_step)["median"], 5)
    step()
    torch.cuda.synchronize()
    if rank == 0:  # 8 rows of layer 0 against the oracle's full (unsharded) product
        from oracle import oracle

        g2 = torch.Generator(device=device)
        g2.manual_seed(61)
        attn0 = torch.randn(L, rows, fin, generator=g2, device=device).half()[0, :8].float().cpu().numpy()
        w0 = (torch.randn(L, fin, H, generator=g2, device=device) / math.sqrt(fin)).half()[0].float().cpu().numpy()
        exp = oracle.linear(attn0, w0, bias[0].cpu().numpy(), threads=oracle.cpu_count()) + \
            res[0, :8].float().cpu().numpy()
        err, ok = close_enough(y[0, :8].float().cpu().numpy(), exp)
        rec["parity"] = {"max_abs_err": err, "ok": ok, "checked": "rank 0, layer 0, rows 0..7 vs oracle linear + "
                                                                  "residual over all 4096 inputs"}
    if op is not None:
        op.close()
    return rec


# ---------------------------------------------------------------- CPU legs (oracle, torch eager)
def cpu_decode_sample(threads, workload="decode_1b", batch=4, heads=None, min_seconds=0.0):
    """Time the oracle's attention loops (the reference's causalAttention restated) on a
    bounded sample of a decode workload, repeated until at least min_seconds have
    passed (at most 64 passes). Returns (GB/s of algorithmic bytes, seconds, description)."""
    from oracle import oracle

    if workload == "ragged_8b":
        w = RAGGED_8B
        T = int(np.mean(ragged_lengths(w)))
    elif workload == "long_ctx":
        w = LONG_CTX
        T = 16384  # a bounded slice of the 131072-token context
    else:
        w = DECODE_1B
        T = w["T"]
    Hq, Hk, D = w["Hq"], w["Hk"], w["D"]
    heads = heads or Hq
    rng = np.random.default_rng(0)
    kc = rng.standard_normal((batch, T + 1, Hk * D), dtype=np.float32)
    vc = rng.standard_normal((batch, T + 1, Hk * D), dtype=np.float32)
    q = rng.standard_normal((batch, Hq * D), dtype=np.float32)
    pos = np.full(batch, T, np.int32)
    opts = dict(head_count=Hq, kv_head_count=Hk, head_dim=D)
    oracle.attend_heads(q, pos, kc, vc, 0, min(heads, 2), threads=threads, **opts)  # warm
    passes = 0
    t0 = time.perf_counter()
    while True:
        oracle.attend_heads(q, pos, kc, vc, 0, heads, threads=threads, **opts)
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds or passes >= 64:
            break
    nbytes = passes * batch * decode_seq_bytes(T + 1, Hq, Hk, D) * heads / Hq
    desc = (f"{batch} seq x {heads}/{Hq} q heads x 1 layer at {T} cached tokens, fp32 (oracle)"
            + (f", {passes} passes" if passes > 1 else ""))
    return nbytes / dt / 1e9, dt, desc


def cpu_prefill_sample(threads, tokens=768, min_seconds=5.0):
    """The oracle's token-by-token prefill replay (the reference's prefill,
    DecoderTSLRunner.ts:504-530) on one sequence's first `tokens` positions of
    one KV-head group of config 3 (7 query heads), repeated until min_seconds."""
    from oracle import oracle

    w = PREFILL_05B
    G, D = w["Hq"] // w["Hk"], w["D"]
    rng = np.random.default_rng(1)
    qkv = rng.standard_normal((1, tokens, (G + 2) * D)).astype(np.float16).astype(np.float32)
    passes, t0 = 0, time.perf_counter()
    while True:
        kc = np.zeros((1, tokens, D), np.float32)
        vc = np.zeros_like(kc)
        oracle.prefill(qkv, [0], kc, vc, threads=threads, head_count=G, kv_head_count=1, head_dim=D,
                       rope_theta=w["theta"])
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds or passes >= 64:
            break
    flops = passes * prefill_causal_flops(D, tokens, 1, G)
    return {"value": round(flops / dt / 1e12, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"1 sequence x {G} q heads (one kv head) x positions 0..{tokens - 1}, fp32 oracle replay, "
                      f"{passes} passes ({dt:.2f} s)"}


def torch_cpu_eager_sample(batch=16, min_seconds=3.0):
    """BASELINE's second CPU baseline: float32 RoPE + matmul / softmax / matmul
    in PyTorch on all host threads, on the config-2 decode sample."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = DECODE_1B
    Hq, Hk, D, T = w["Hq"], w["Hk"], w["D"], w["T"]
    g = torch.Generator().manual_seed(0)
    k = torch.randn(batch, Hk, T + 1, D, generator=g)
    v = torch.randn(batch, Hk, T + 1, D, generator=g)
    q = torch.randn(batch, Hq, 1, D, generator=g)
    inv = 1.0 / (w["theta"] ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = (T * inv).float()
    cos, sin = torch.cos(ang), torch.sin(ang)

    def once():
        q1, q2 = q[..., :D // 2], q[..., D // 2:]
        qr = torch.cat([q1 * cos - q2 * sin, q2 * cos + q1 * sin], dim=-1)
        kk = k.repeat_interleave(Hq // Hk, dim=1)
        vv = v.repeat_interleave(Hq // Hk, dim=1)
        s = (qr @ kk.transpose(-1, -2)) / math.sqrt(D)
        return torch.softmax(s, dim=-1) @ vv

    once()
    passes, t0 = 0, time.perf_counter()
    while True:
        once()
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds or passes >= 200:
            break
    nbytes = passes * batch * decode_seq_bytes(T + 1, Hq, Hk, D)
    return {"value": round(nbytes / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "torch_cpu_eager",
            "sample": f"{batch} seq x {Hq} q heads x 1 layer at {T} cached tokens, float32, {passes} passes "
                      f"({dt:.2f} s)"}


def run_reference(args):
    from oracle import oracle

    threads = oracle.cpu_count()
    workload = "long_ctx" if args.workload == "long_ctx_heads" else args.workload
    if workload == "prefill_05b":
        workload = "decode_1b"
    batch = args.ref_batch if workload == "decode_1b" else (8 if workload == "ragged_8b" else 1)
    cpu_decode_sample(threads, workload, batch=min(batch, 2))  # warm
    vals = [cpu_decode_sample(threads, workload, batch=batch) for _ in range(max(1, args.steps))]
    gbs = statistics.median(v[0] for v in vals)
    dt = statistics.median(v[1] for v in vals)
    desc = vals[0][2] + " per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if workload == "decode_1b" else "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD_LABELS[workload], "sample": desc},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if workload == "decode_1b" and not args.ref_no_prefill:
        line["prefill"] = cpu_prefill_sample(threads, tokens=512, min_seconds=0.5)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- main
def guarded(fn, *a, **kw):
    """A sub-record that fails is reported in the line instead of losing it."""
    try:
        return fn(*a, **kw)
    except Exception as e:  # noqa: BLE001
        import traceback

        traceback.print_exc()
        return {"error": f"{type(e).__name__}: {e}"}


def sub_decode(name, cls, pkg, torch, device, rank, world, args, hbm, parity=True, **kw):
    wl = cls(pkg, torch, device, rank, world, args, **kw)
    try:
        st, _ = measure_decode(torch, wl, args, world, device, args.sub_seconds)
        rec = decode_record(wl, st, world, hbm)
        rec["parallelism"] = wl.config["parallelism"]
        if parity:
            p = wl.parity(world, rank)
            if p is not None and rank == 0:
                rec["parity"] = p
    finally:
        wl.close()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode_1b",
                    choices=["decode_1b", "ragged_8b", "long_ctx", "long_ctx_heads", "prefill_05b", "out_proj",
                             "prefill_qkv", "qkv_decode_1b"],
                    help="headline workload (long_ctx: token blocks; the default line carries all as sub-records)")
    ap.add_argument("--batch", type=int, default=DECODE_1B["batch"], help="decode_1b sequences per GPU")
    ap.add_argument("--ref-batch", type=int, default=64)
    ap.add_argument("--ref-no-prefill", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", "--no-prefill", dest="headline_only", action="store_true",
                    help="skip the sub-records")
    ap.add_argument("--min-seconds", type=float, default=1.0, help="timed work of the headline record")
    ap.add_argument("--sub-seconds", type=float, default=0.3, help="timed work of each decode sub-record")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="long_ctx_seq: merge of the sequence shards across GPUs")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return

    import torch

    import __graft_entry__ as ge

    pkg = ge.load_package()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    hbm, tc, src = peaks()
    single = {"ragged_8b": Ragged8B, "long_ctx": LongCtxSeq, "long_ctx_heads": LongCtxHeads,
              "qkv_decode_1b": QkvDecode1B}
    if args.workload in ("out_proj", "prefill_qkv"):  # one sub-record alone (profiling)
        rec = (run_out_proj(pkg, torch, device, rank, world, args, hbm) if args.workload == "out_proj"
               else run_qkv_prefill(pkg, torch, device, rank, world, args, tc))
        if rank == 0:
            print(json.dumps({"metric": METRIC, "workload": args.workload, args.workload: rec}), flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    if args.workload == "prefill_05b":
        rec = run_prefill(pkg, torch, device, rank, world, args, tc, src)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": rec["tflops"], "unit": "TFLOP/s", "n_gpus": world,
                              "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms"],
                              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
                              "data": "synthetic", "config": {"workload": rec["workload"]}, "prefill": rec}),
                  flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return

    # ---- headline
    if args.workload == "decode_1b":
        wl = Decode1B(pkg, torch, device, rank, world, args)
    else:
        wl = single[args.workload](pkg, torch, device, rank, world, args)
    st, extras = measure_decode(torch, wl, args, world, device, args.min_seconds, clocks=True, eager_launches=True)
    e2e_ms = measure_e2e(torch, wl, args, world) if hasattr(wl, "e2e_setup") else None
    head_parity = wl.parity(world, rank)
    ms = st["median"]
    total_bytes = wl.bytes_per_step * world
    gbs = total_bytes / (ms * 1e-3) / 1e9
    # roofline of the dominant kernel from the same graph replay: per-GPU bytes of
    # one layer's launch over the replayed per-layer time
    layer_ms = ms / len(wl.layers)
    achieved = wl.bytes_per_launch / (layer_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": wl.scaling,
        "vs_baseline": None, "dtype": "fp16", "data": "synthetic (seeded N(0,1) fp16 cache and qkv)",
        "config": dict(wl.config, timing=f"median of {st['blocks']} blocks of exactly {args.steps} graph-replayed "
                                         f"steps ({extras['timed_s']:.2f} s timed), max over ranks"),
        "repeats": rnd({"ms_median": ms, "ms_p10": st["p10"], "ms_p90": st["p90"], "blocks": st["blocks"]}, 5),
        "tok_s": round(wl.tokens_per_step * world / (ms * 1e-3), 1), "hbm_frac": round(gbs / world / hbm, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4),
                     "traffic": (round(wl.traffic_per_launch) if getattr(wl, "traffic_per_launch", None) else None),
                     "traffic_unit": "DRAM bytes per launch (ncu, scaled by sequences)", "kernel": wl.kernel,
                     "peak_source": src, "layer_ms": round(layer_ms, 5),
                     "how": "per-launch algorithmic bytes / (graph-replayed ms_per_step / layers)",
                     "eager_launch_ms": round(extras["eager_launch_ms"], 5)},
        "gpu_launches": int(st["blocks"] * args.steps * wl.launches_per_step),
        "clocks": extras.get("clocks"),
    }
    if e2e_ms is not None:
        line["e2e"] = {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                       "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h, "ms_per_step": round(e2e_ms, 5)}
    if head_parity is not None and rank == 0:
        line["parity"] = head_parity
    wl.close()
    del wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    # ---- sub-records (every rank runs the same ones in the same order)
    if args.workload == "decode_1b" and not args.headline_only:
        sweep = {}
        for b in (1, 8, 32):
            sweep[str(b)] = guarded(sub_decode, "decode_1b", Decode1B, pkg, torch, device, rank, world, args, hbm,
                                    parity=False, batch=b)
        line["decode_1b_batch"] = sweep
        line["ragged_8b"] = guarded(sub_decode, "ragged_8b", Ragged8B, pkg, torch, device, rank, world, args, hbm)
        line["long_ctx_heads"] = guarded(sub_decode, "long_ctx_heads", LongCtxHeads, pkg, torch, device, rank, world,
                                         args, hbm)
        if world > 1:
            line["long_ctx_seq"] = guarded(sub_decode, "long_ctx_seq", LongCtxSeq, pkg, torch, device, rank, world,
                                           args, hbm)
        else:
            line["long_ctx_seq"] = dict(line["long_ctx_heads"], note="one GPU holds every token block: the plain "
                                                                     "decode of long_ctx_heads")
        line["prefill"] = guarded(run_prefill, pkg, torch, device, rank, world, args, tc, src)
        line["qkv_decode_1b"] = guarded(sub_decode, "qkv_decode_1b", QkvDecode1B, pkg, torch, device, rank, world,
                                        args, hbm)
        line["prefill_qkv"] = guarded(run_qkv_prefill, pkg, torch, device, rank, world, args, tc)
        line["out_proj"] = guarded(run_out_proj, pkg, torch, device, rank, world, args, hbm)
        for key in ("ragged_8b", "long_ctx_heads", "long_ctx_seq"):
            line[key].setdefault("workload", WORKLOAD_LABELS["long_ctx" if key.startswith("long") else key])
    if rank == 0:
        checks = [line.get("parity")] + [line.get(k, {}).get("parity") for k in
                                         ("ragged_8b", "long_ctx_heads", "long_ctx_seq", "prefill", "qkv_decode_1b",
                                          "prefill_qkv", "out_proj")]
        checks = [c for c in checks if c]
        line["parity_ok"] = bool(checks) and all(c["ok"] for c in checks)
        line["parity_max_err"] = max(c["max_abs_err"] for c in checks) if checks else None
        if world == 1 and not args.no_cpu_baseline:
            gb, dt, desc = cpu_decode_sample(1, args.workload, batch=16 if args.workload == "decode_1b" else 1,
                                             min_seconds=10.0)
            line["cpu_baseline"] = {"value": round(gb, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                                    "sample": desc + f" ({dt:.2f} s)"}
            if args.workload == "decode_1b":
                line["cpu_baseline_torch_eager"] = torch_cpu_eager_sample()
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
