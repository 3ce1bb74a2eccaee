"""GPU parity of causal prefill (tla_prefill) against the reference's prefill,
which replays the one-token step at positions start..start+S-1
(packages/three-llm/src/decoder/DecoderTSLRunner.ts:504-530). Outputs for
every position and the cache contents must agree with the oracle."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_decode_gpu import assert_close, f16

pytestmark = pytest.mark.gpu


def prefill_case(pkg, cuda, Hq, Hk, D, S, starts, max_tokens, dtype=torch.float16, layer_kw=None, oracle_kw=None,
                 seed=0, cache_dtype="float16", gate=False):
    rng = np.random.default_rng(seed)
    B = len(starts)
    row = (Hq + 2 * Hk) * D
    pre = f16(rng.standard_normal((B, max_tokens, Hk * D)))  # existing cache contents before the prefill
    kc, vc = pre.copy(), f16(rng.standard_normal((B, max_tokens, Hk * D)))
    vpre = vc.copy()
    qkv = f16(rng.standard_normal((B, S, row)))
    g = f16(rng.standard_normal((B, S, Hq * D)) * 2) if gate else None
    opts = {"headDim": D, "kvHeadCount": Hk, "maxBatch": B, "dtype": dtype, "cacheDtype": cache_dtype}
    opts.update(layer_kw or {})
    layer = pkg.CUDAAttention(None, Hq * D, Hq, max_tokens, opts)
    for b in range(B):
        layer.write_cache(b, 0, pre[b], vpre[b])
    sp = torch.tensor(starts, dtype=torch.int32, device=cuda)
    out = layer.prefill(torch.from_numpy(qkv).to(cuda, dtype), sp,
                        gate=None if g is None else torch.from_numpy(g).to(cuda, dtype)).float().cpu().numpy()
    exp = oracle.prefill(qkv, starts, kc, vc, gate=g, threads=os.cpu_count(), head_count=Hq, kv_head_count=Hk,
                         head_dim=D, **(oracle_kw or {}))
    assert layer.context.error() == 0
    assert_close(out, exp, what="prefill outputs")
    for b in range(B):
        k, v = layer.read_cache(b, starts[b], S)
        assert_close(k, kc[b, starts[b]:starts[b] + S], 2e-3, 2e-3, "prefill key cache")
        assert_close(v, vc[b, starts[b]:starts[b] + S], 2e-3, 2e-3, "prefill value cache")
    return layer


@pytest.mark.parametrize("D,dtype", [(64, torch.float16), (128, torch.float16), (64, torch.float32)])
def test_prefill_output_gate(pkg, cuda, D, dtype):
    # Qwen3.5 full-attention layers gate every prompt position's output
    # (qwen/QwenTSLRunner.ts:172-186; the replayed decode graph applies
    # gateNode, TSLAttention.ts:418-423): the fused sigmoid epilogue of the
    # tensor-core kernel, 200 tokens leave a partial last query tile
    qn = np.random.default_rng(4).standard_normal(D).astype(np.float32) * 0.1
    prefill_case(pkg, cuda, 16, 4, D, 200, [0, 45], 512, dtype=dtype, gate=True,
                 layer_kw={"ropeTheta": 1e6, "qNormWeight": qn, "kNormWeight": qn, "offsetRMSNorm": True},
                 oracle_kw={"rope_theta": 1e6, "q_norm_weight": qn, "k_norm_weight": qn, "offset_rms_norm": True})


def test_prefill_output_gate_generic_path(pkg, cuda):
    prefill_case(pkg, cuda, 4, 2, 8, 19, [0, 3], 32, dtype=torch.float32, gate=True,
                 layer_kw={"ropeTheta": 10000.0}, oracle_kw={"rope_theta": 10000.0}, cache_dtype="float32")


def test_prefill_small_generic_shapes(pkg, cuda):
    prefill_case(pkg, cuda, 4, 2, 8, 19, [0, 3], 32, dtype=torch.float32, layer_kw={"ropeTheta": 10000.0},
                 oracle_kw={"rope_theta": 10000.0}, cache_dtype="float32")


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_chunk_after_cached_prefix(pkg, cuda, D):
    # a second prefill chunk on top of cached tokens (chunked prefill, DecoderTSLRunner.ts:504-530)
    prefill_case(pkg, cuda, 14, 2, D, 200, [0, 37, 129], 512, layer_kw={"ropeTheta": 1e6},
                 oracle_kw={"rope_theta": 1e6})


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_fp32_io_tensor_core_path(pkg, cuda, D):
    # float32 qkv and outputs over the fp16 cache: the tensor-core kernel with
    # 32-bit output rows (at head_dim 64 they leave through the shared-memory
    # stage as 256-byte rows); 200 tokens leave partial last query tiles
    prefill_case(pkg, cuda, 8, 2, D, 200, [0, 37], 512, dtype=torch.float32, layer_kw={"ropeTheta": 5e5},
                 oracle_kw={"rope_theta": 5e5})


def test_prefill_sliding_window_and_qk_norm(pkg, cuda):
    rng = np.random.default_rng(2)
    qn = rng.standard_normal(64).astype(np.float32) * 0.1
    kn = rng.standard_normal(64).astype(np.float32) * 0.1
    prefill_case(pkg, cuda, 8, 2, 64, 150, [0, 10], 256,
                 layer_kw={"ropeTheta": 10000.0, "slidingWindow": 48, "qNormWeight": qn, "kNormWeight": kn},
                 oracle_kw={"rope_theta": 10000.0, "sliding_window": 48, "q_norm_weight": qn, "k_norm_weight": kn})


@pytest.mark.parametrize("dtype,window", [(torch.float16, 0), (torch.float32, 0), (torch.float16, 300)])
def test_prefill_kv_range_pieces(pkg, cuda, dtype, window):
    # One sequence, one kv head of 7 query heads, 1000 tokens after a 37-token
    # prefix: 28 tile pairs for the SMs, so the head_dim-64 kernel cuts each
    # pair's KV steps into pieces and merges their partial rows (with the gate)
    kw = {"ropeTheta": 1e6}
    okw = {"rope_theta": 1e6}
    if window:
        kw["slidingWindow"] = window
        okw["sliding_window"] = window
    prefill_case(pkg, cuda, 7, 1, 64, 1000, [37], 1100, dtype=dtype, gate=True, layer_kw=kw, oracle_kw=okw,
                 seed=11)


def test_prefill_config3_share_of_eight_gpus_vs_oracle(pkg, cuda):
    # one rank's share of config 3 on eight GPUs: one sequence, one kv head and
    # its 7 query heads, 2048 tokens (KV-range pieces)
    prefill_case(pkg, cuda, 7, 1, 64, 2048, [0], 4096, layer_kw={"ropeTheta": 1e6}, oracle_kw={"rope_theta": 1e6},
                 seed=12)


def test_prefill_then_decode_continues(pkg, cuda):
    """Prefill S tokens, then decode the next one: same as S+1 reference steps."""
    rng = np.random.default_rng(9)
    Hq, Hk, D, S, T = 32, 8, 64, 300, 512
    row = (Hq + 2 * Hk) * D
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                    "dtype": torch.float16})
    qkv = f16(rng.standard_normal((1, S + 1, row)))
    kc = np.zeros((1, T, Hk * D), np.float32)
    vc = np.zeros_like(kc)
    exp = oracle.prefill(qkv, [0], kc, vc, threads=8, head_count=Hq, kv_head_count=Hk, head_dim=D, rope_theta=5e5)
    layer.prefill(torch.from_numpy(qkv[:, :S]).to(cuda, torch.float16), torch.tensor([0], dtype=torch.int32,
                                                                                      device=cuda))
    out = layer.decode(torch.from_numpy(qkv[:, S]).to(cuda, torch.float16),
                       torch.tensor([S], dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert layer.context.error() == 0
    assert_close(out, exp[:, S], what="decode after prefill")


@pytest.mark.parametrize("rotary", [18, 32])
def test_prefill_partial_rotary_yarn_vnorm(pkg, cuda, rotary):
    # rotary 18 takes the block-per-token RoPE kernel, rotary 32 the warp-per-token one
    yarn = {"type": "yarn", "factor": 4.0, "original_context_length": 128.0, "beta_fast": 32.0, "beta_slow": 1.0}
    prefill_case(pkg, cuda, 8, 2, 64, 160, [0, 20], 256,
                 layer_kw={"ropeTheta": 10000.0, "rotaryDim": rotary, "ropeScaling": yarn, "vNorm": True},
                 oracle_kw={"rope_theta": 10000.0, "rotary_dim": rotary, "rope_scaling": yarn, "v_norm": True})


def test_prefill_config3_full_size_vs_oracle(pkg, cuda):
    """BASELINE config 3 at full size (4 x 2048 tokens, 14/2 heads, d64, theta 1e6,
    K/V into a 4096-slot cache) against the oracle's token-by-token replay."""
    B, S, Hq, Hk, D, T = 4, 2048, 14, 2, 64, 4096
    rng = np.random.default_rng(3)
    qkv = f16(rng.standard_normal((B, S, (Hq + 2 * Hk) * D)))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 1e6, "maxBatch": B,
                                                    "dtype": torch.float16})
    out = layer.prefill(torch.from_numpy(qkv).to(cuda, torch.float16),
                        torch.zeros(B, dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert layer.context.error() == 0
    kc = np.zeros((B, T, Hk * D), np.float32)
    vc = np.zeros_like(kc)
    exp = oracle.prefill(qkv, [0] * B, kc, vc, threads=os.cpu_count(), head_count=Hq, kv_head_count=Hk, head_dim=D,
                         rope_theta=1e6)
    assert_close(out, exp, what="config 3 prefill")
    for b in (0, B - 1):
        k, v = layer.read_cache(b, 0, S)
        assert_close(k, kc[b, :S], 2e-3, 2e-3, "config 3 key cache")
        assert_close(v, vc[b, :S], 2e-3, 2e-3, "config 3 value cache")
