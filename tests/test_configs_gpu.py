"""Full-size BASELINE configurations against the oracle, one layer each.

The oracle restates causalAttention (packages/three-llm/src/runtime/math.ts:
179-276) in double arithmetic; here it sees the same fp16 cache contents and
fp16 inputs as the GPU, on all host threads. Config 3 (prefill) is in
test_prefill_gpu.py. Tolerance
|a - e| <= 2e-3 + 1e-2 |e|.

Also at full size on one GPU: the KV-head shard of config 4 that one of eight
GPUs holds, and config 5 split into token blocks whose partial triples are
merged with the log-sum-exp combine, the two multi-GPU partitions.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_decode_gpu import assert_close

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8


def cache_tensors(layer):
    """The layer's fp16 K and V caches as torch views [max_batch, Hk, max_tokens, D]."""
    v = layer.cache_view()
    shape = (layer.maxBatch, layer.kvHeadCount, layer.maxTokens, layer.headDim)

    class Arr:
        def __init__(self, ptr):
            self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (ptr, False), "version": 3}

    return torch.as_tensor(Arr(v.key), device=layer.device), torch.as_tensor(Arr(v.value), device=layer.device)


def fill_random(layer, seed):
    """N(0,1) fp16 cache contents; returns the oracle's token-major float32 copies [B, T, Hk*D]."""
    g = torch.Generator(device=layer.device)
    g.manual_seed(seed)
    kc, vc = cache_tensors(layer)
    kc.normal_(generator=g)
    vc.normal_(generator=g)
    B, Hk, T, D = kc.shape

    def host(t):
        return t.permute(0, 2, 1, 3).reshape(B, T, Hk * D).float().cpu().numpy()

    return host(kc), host(vc)


def decode_vs_oracle(pkg, cuda, Hq, Hk, D, lengths, theta, seed, what):
    B = len(lengths)
    T = int(max(lengths)) + 1
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": theta,
                                                    "maxBatch": B, "dtype": torch.float16})
    kc, vc = fill_random(layer, seed)
    g = torch.Generator(device=cuda)
    g.manual_seed(seed + 1)
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, generator=g, device=cuda).half()
    pos = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    out = layer.decode(qkv, pos).float().cpu().numpy()
    assert layer.context.error() == 0
    exp = oracle.decode_batch(qkv.float().cpu().numpy(), np.asarray(lengths, np.int32), kc, vc, threads=THREADS,
                              head_count=Hq, kv_head_count=Hk, head_dim=D, rope_theta=theta)
    assert_close(out, exp, what=what)
    for b in (0, B - 1):  # the appended rows
        k, v = layer.read_cache(b, int(lengths[b]), 1)
        assert_close(k[0], kc[b, lengths[b]], 2e-3, 2e-3, f"{what}: appended key")
        assert_close(v[0], vc[b, lengths[b]], 2e-3, 2e-3, f"{what}: appended value")
    layer.close()


def test_config2_one_layer_batch64_vs_oracle(pkg, cuda):
    """Config 2: 32/8 heads, d64, 4096 cached + 1 new, batch 64, theta 5e5."""
    decode_vs_oracle(pkg, cuda, 32, 8, 64, [4096] * 64, 5e5, 21, "config 2")


@pytest.mark.parametrize("batch", [1, 8])
def test_config2_batch_sweep_vs_oracle(pkg, cuda, batch):
    decode_vs_oracle(pkg, cuda, 32, 8, 64, [4096] * batch, 5e5, 22 + batch, f"config 2 batch {batch}")


def test_config4_ragged_batch64_d128_vs_oracle(pkg, cuda):
    """Config 4: batch 64, lengths U[512, 8192] (seed 0), 32/8 heads, d128, theta 5e5."""
    lengths = [int(x) for x in np.random.default_rng(0).integers(512, 8193, size=64)]
    decode_vs_oracle(pkg, cuda, 32, 8, 128, lengths, 5e5, 41, "config 4")


def test_config5_131072_tokens_vs_oracle(pkg, cuda):
    """Config 5 on one GPU: one sequence of 131072 cached tokens, 32/8 heads, d128;
    every CTA of the persistent grid takes a segment of the 8 (sequence, kv head)
    pairs, merged by the deferred segment-merge kernel."""
    decode_vs_oracle(pkg, cuda, 32, 8, 128, [131072], 5e5, 51, "config 5")


def test_config4_kv_head_shard_of_eight_vs_oracle(pkg, cuda):
    """One rank's share of config 4 at eight GPUs (sharding.head_shard): kv head 3
    and its four query heads of every sequence, against the oracle's full layer."""
    from three_llm_b200 import sharding

    Hq, Hk, D, theta = 32, 8, 128, 5e5
    lengths = [int(x) for x in np.random.default_rng(0).integers(512, 8193, size=64)]
    B, T = len(lengths), max(lengths) + 1
    sh = sharding.head_shard(Hq, Hk, 8, 3)
    full = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": theta,
                                                   "maxBatch": B, "dtype": torch.float16})
    kc, vc = fill_random(full, 43)
    part = pkg.CUDAAttention(None, sh.q_count * D, sh.q_count, T,
                             {"headDim": D, "kvHeadCount": sh.kv_count, "ropeTheta": theta, "maxBatch": B,
                              "dtype": torch.float16})
    fk, fv = cache_tensors(full)
    pk, pv = cache_tensors(part)
    pk.copy_(fk[:, sh.kv_begin:sh.kv_begin + sh.kv_count])
    pv.copy_(fv[:, sh.kv_begin:sh.kv_begin + sh.kv_count])
    full.close()
    g = torch.Generator(device=cuda)
    g.manual_seed(44)
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, generator=g, device=cuda).half()
    pos = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    out = part.decode(sharding.slice_qkv_for_heads(qkv, sh, Hq, Hk, D), pos).float().cpu().numpy()
    assert part.context.error() == 0
    exp = oracle.decode_batch(qkv.float().cpu().numpy(), np.asarray(lengths, np.int32), kc, vc, threads=THREADS,
                              head_count=Hq, kv_head_count=Hk, head_dim=D, rope_theta=theta)
    exp = exp.reshape(B, Hq, D)[:, sh.q_begin:sh.q_begin + sh.q_count].reshape(B, -1)
    assert_close(out, exp, what="config 4 kv-head shard")


@pytest.mark.parametrize("ranks", [2, 8])
def test_config5_token_blocks_lse_merge_vs_oracle(pkg, cuda, ranks):
    """Config 5 split into `ranks` contiguous token blocks (sharding.sequence_shard),
    each decoded to partial (m, l, o) triples on this GPU and merged with the
    log-sum-exp combine: the protocol each GPU runs, against the oracle."""
    from three_llm_b200 import sharding

    Hq, Hk, D, T, theta = 32, 8, 128, 131072, 5e5
    whole = pkg.CUDAAttention(None, Hq * D, Hq, T + 1, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": theta,
                                                        "dtype": torch.float16})
    kc, vc = fill_random(whole, 57)
    wk, wv = cache_tensors(whole)
    g = torch.Generator(device=cuda)
    g.manual_seed(58)
    qkv = torch.randn(1, (Hq + 2 * Hk) * D, generator=g, device=cuda).half()
    pos = torch.tensor([T], dtype=torch.int32, device=cuda)
    parts = []
    for r in range(ranks):
        s = sharding.sequence_shard(T, ranks, r)
        local = s.tokens + (1 if s.owns_next else 0)
        layer = pkg.CUDAAttention(None, Hq * D, Hq, local, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": theta,
                                                            "dtype": torch.float16})
        lk, lv = cache_tensors(layer)
        lk[:, :, :s.tokens].copy_(wk[:, :, s.slot_offset:s.slot_offset + s.tokens])
        lv[:, :, :s.tokens].copy_(wv[:, :, s.slot_offset:s.slot_offset + s.tokens])
        parts.append(layer.decode_partial(qkv, pos, s.slot_offset, local, s.owns_next))
        assert layer.context.error() == 0
        layer.close()
    whole.close()
    out = pkg.combine_lse(torch.stack(parts)).float().cpu().numpy()
    exp = oracle.decode_batch(qkv.float().cpu().numpy(), [T], kc, vc, threads=THREADS, head_count=Hq,
                              kv_head_count=Hk, head_dim=D, rope_theta=theta)
    assert_close(out, exp, what=f"config 5 in {ranks} token blocks")
