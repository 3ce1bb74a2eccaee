"""GPU parity of causal prefill (tla_prefill) against the reference's prefill,
which replays the one-token step at positions start..start+S-1
(packages/three-llm/src/decoder/DecoderTSLRunner.ts:504-530). Outputs for
every position and the cache contents must agree with the oracle."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_decode_gpu import assert_close, f16

pytestmark = pytest.mark.gpu


def prefill_case(pkg, cuda, Hq, Hk, D, S, starts, max_tokens, dtype=torch.float16, layer_kw=None, oracle_kw=None,
                 seed=0, cache_dtype="float16"):
    rng = np.random.default_rng(seed)
    B = len(starts)
    row = (Hq + 2 * Hk) * D
    pre = f16(rng.standard_normal((B, max_tokens, Hk * D)))  # existing cache contents before the prefill
    kc, vc = pre.copy(), f16(rng.standard_normal((B, max_tokens, Hk * D)))
    vpre = vc.copy()
    qkv = f16(rng.standard_normal((B, S, row)))
    opts = {"headDim": D, "kvHeadCount": Hk, "maxBatch": B, "dtype": dtype, "cacheDtype": cache_dtype}
    opts.update(layer_kw or {})
    layer = pkg.CUDAAttention(None, Hq * D, Hq, max_tokens, opts)
    for b in range(B):
        layer.write_cache(b, 0, pre[b], vpre[b])
    sp = torch.tensor(starts, dtype=torch.int32, device=cuda)
    out = layer.prefill(torch.from_numpy(qkv).to(cuda, dtype), sp).float().cpu().numpy()
    exp = oracle.prefill(qkv, starts, kc, vc, threads=8, head_count=Hq, kv_head_count=Hk, head_dim=D,
                         **(oracle_kw or {}))
    assert layer.context.error() == 0
    assert_close(out, exp, what="prefill outputs")
    for b in range(B):
        k, v = layer.read_cache(b, starts[b], S)
        assert_close(k, kc[b, starts[b]:starts[b] + S], 2e-3, 2e-3, "prefill key cache")
        assert_close(v, vc[b, starts[b]:starts[b] + S], 2e-3, 2e-3, "prefill value cache")
    return layer


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


def torch_rope(x, pos, inv_freq, rotary, attn_factor=1.0):
    """float32 rotate-half RoPE with float64 angles (x [..., T, D], pos [T])."""
    ang = pos.double()[:, None] * inv_freq.double()[None, :]
    c, s = torch.cos(ang).float(), torch.sin(ang).float()
    half = rotary // 2
    x1, x2, rest = x[..., :half], x[..., half:rotary], x[..., rotary:]
    return torch.cat([(x1 * c - x2 * s) * attn_factor, (x2 * c + x1 * s) * attn_factor, rest], dim=-1)


def test_prefill_config3_full_size_vs_torch_fp32(pkg, cuda):
    """BASELINE config 3 at full size (4 x 2048 tokens, 14/2 heads, d64, theta 1e6)
    against a float32 PyTorch restatement of the same causal attention."""
    from three_llm_b200.attention import rope_parameters

    torch.backends.cuda.matmul.allow_tf32 = False
    B, S, Hq, Hk, D, T = 4, 2048, 14, 2, 64, 4096
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    qkv = torch.randn(B, S, (Hq + 2 * Hk) * D, generator=g, device=cuda).half()
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 1e6, "maxBatch": B,
                                                    "dtype": torch.float16})
    out = layer.prefill(qkv, torch.zeros(B, dtype=torch.int32, device=cuda)).float()
    assert layer.context.error() == 0
    inv, _ = rope_parameters(D, 1e6)
    inv = torch.from_numpy(inv).to(cuda)
    x = qkv.float().view(B, S, Hq + 2 * Hk, D).transpose(1, 2)  # [B, H, S, D]
    pos = torch.arange(S, device=cuda)
    q = torch_rope(x[:, :Hq], pos, inv, D)
    k = torch_rope(x[:, Hq:Hq + Hk], pos, inv, D).repeat_interleave(Hq // Hk, dim=1)
    v = x[:, Hq + Hk:].repeat_interleave(Hq // Hk, dim=1)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(D)
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device=cuda), 1), float("-inf"))
    ref = (torch.softmax(s, dim=-1) @ v).transpose(1, 2).reshape(B, S, Hq * D)
    err = (out - ref).abs()
    assert bool(torch.all(err <= 2e-3 + 1e-2 * ref.abs())), f"max abs err {err.max().item():.3e}"
