"""The projections around the attention, on the tensor cores, against the oracle.

QKV projection fused with the attention's front end (tla_qkv_decode /
tla_qkv_prefill): the reference computes qkv = linear(norm1, attnQKVWeight,
attnQKVBias) (runtime/math.ts:6-25; TSLLinear.ts:56-75 on the GPU) and feeds
it to the attention (decoder/DecoderTSLRunner.ts:293-297). The oracle does
exactly that, in double arithmetic, on the same fp16-rounded x and W; the GPU
result (outputs and appended cache rows) must match within the north-star
bound. Output projection + residual (tla_out_proj): y = residual +
linear(attn, attnProjWeight, attnProjBias) (DecoderTSLRunner.ts:299-309).
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_decode_gpu import assert_close, f16

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def weights(rng, hidden, n, scale=None):
    w = f16(rng.standard_normal((hidden, n)) * (scale or 1 / np.sqrt(hidden)))
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    return w, b


@pytest.mark.parametrize("D,Hq,Hk,hidden", [(64, 16, 4, 1024), (128, 8, 2, 512), (64, 32, 8, 2048)])
def test_qkv_decode_fused_vs_oracle(pkg, cuda, D, Hq, Hk, hidden):
    """Ragged batch, bias, offset QK-norm, vNorm and the output gate."""
    rng = np.random.default_rng(D + Hq + hidden)
    B, T = 12, 700
    N = (Hq + 2 * Hk) * D
    w, bias = weights(rng, hidden, N)
    x = f16(rng.standard_normal((B, hidden)))
    g = f16(rng.standard_normal((B, Hq * D)))
    qn = (rng.standard_normal(D) * 0.1).astype(np.float32)
    kn = (rng.standard_normal(D) * 0.1).astype(np.float32)
    lengths = [int(v) for v in rng.integers(0, T - 1, size=B)]
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5, "maxBatch": B,
                                                    "dtype": torch.float16, "qNormWeight": qn, "kNormWeight": kn,
                                                    "offsetRMSNorm": True, "vNorm": True})
    for b in range(B):
        layer.write_cache(b, 0, kc[b], vc[b])
    xd, wd = torch.from_numpy(x).to(cuda, torch.float16), torch.from_numpy(w).to(cuda, torch.float16)
    bd, gd = torch.from_numpy(bias).to(cuda), torch.from_numpy(g).to(cuda, torch.float16)
    pos = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    out = torch.full((B, Hq * D), float("nan"), dtype=torch.float16, device=cuda)
    rc = pkg.lib().tla_qkv_decode(layer.handle, P(xd), P(wd), P(bd), hidden, P(pos), P(gd), P(out), B, stream())
    assert rc == 0, pkg.lib().tla_status_string(rc).decode()
    got = out.float().cpu().numpy()
    assert layer.context.error() == 0
    qkv = oracle.linear(x, w, bias, threads=THREADS)
    exp = oracle.decode_batch(qkv, lengths, kc, vc, gate=g, threads=THREADS, head_count=Hq, kv_head_count=Hk,
                              head_dim=D, rope_theta=5e5, q_norm_weight=qn, k_norm_weight=kn, offset_rms_norm=True,
                              v_norm=True)
    assert_close(got, exp, what="fused QKV projection + decode")
    for b in (0, B - 1):
        k, v = layer.read_cache(b, lengths[b], 1)
        assert_close(k[0], kc[b, lengths[b]], 2e-3, 2e-3, "appended key")
        assert_close(v[0], vc[b, lengths[b]], 2e-3, 2e-3, "appended value")


@pytest.mark.parametrize("D,gate", [(64, False), (64, True), (128, False)])
def test_qkv_prefill_fused_vs_oracle(pkg, cuda, D, gate):
    """A chunk after a cached prefix through the fused projection + tensor-core
    prefill, against the oracle's token-by-token replay of linear + attention."""
    rng = np.random.default_rng(5 + D)
    Hq, Hk, hidden, S, T = 8, 2, 512, 200, 512
    starts = [0, 37]
    B = len(starts)
    N = (Hq + 2 * Hk) * D
    w, bias = weights(rng, hidden, N)
    x = f16(rng.standard_normal((B, S, hidden)))
    g = f16(rng.standard_normal((B, S, Hq * D))) if gate else None
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 1e6, "maxBatch": B,
                                                    "dtype": torch.float16})
    for b in range(B):
        layer.write_cache(b, 0, kc[b], vc[b])
    xd, wd = torch.from_numpy(x).to(cuda, torch.float16), torch.from_numpy(w).to(cuda, torch.float16)
    bd = torch.from_numpy(bias).to(cuda)
    gd = None if g is None else torch.from_numpy(g).to(cuda, torch.float16)
    sp = torch.tensor(starts, dtype=torch.int32, device=cuda)
    out = torch.full((B, S, Hq * D), float("nan"), dtype=torch.float16, device=cuda)
    rc = pkg.lib().tla_qkv_prefill(layer.handle, P(xd), P(wd), P(bd), hidden, P(sp), P(gd), S, P(out), B, stream())
    assert rc == 0, pkg.lib().tla_status_string(rc).decode()
    got = out.float().cpu().numpy()
    assert layer.context.error() == 0
    qkv = oracle.linear(x, w, bias, threads=THREADS)
    exp = oracle.prefill(qkv, starts, kc, vc, gate=g, threads=THREADS, head_count=Hq, kv_head_count=Hk, head_dim=D,
                         rope_theta=1e6)
    assert_close(got, exp, what="fused QKV projection + prefill")
    for b in range(B):
        k, v = layer.read_cache(b, starts[b], S)
        assert_close(k, kc[b, starts[b]:starts[b] + S], 2e-3, 2e-3, "prefill key cache")
        assert_close(v, vc[b, starts[b]:starts[b] + S], 2e-3, 2e-3, "prefill value cache")


def test_qkv_decode_position_error_skips_row(pkg, cuda):
    rng = np.random.default_rng(3)
    Hq, Hk, D, hidden, T = 8, 2, 64, 256, 64
    w, _ = weights(rng, hidden, (Hq + 2 * Hk) * D)
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "maxBatch": 2,
                                                    "dtype": torch.float16})
    x = torch.from_numpy(f16(rng.standard_normal((2, hidden)))).to(cuda, torch.float16)
    out = torch.zeros(2, Hq * D, dtype=torch.float16, device=cuda)
    pos = torch.tensor([3, T], dtype=torch.int32, device=cuda)
    wd = torch.from_numpy(w).to(cuda, torch.float16)
    assert pkg.lib().tla_qkv_decode(layer.handle, P(x), P(wd), None, hidden, P(pos), None, P(out), 2, stream()) == 0
    assert layer.context.error() == -12  # TLA_ERR_POSITION
    assert pkg.lib().tla_qkv_decode(layer.handle, P(x), P(wd), None, 12, P(pos), None, P(out), 2, stream()) == -1


@pytest.mark.parametrize("rows,fin,hidden,f32", [(64, 2048, 2048, False), (8192, 896, 896, False),
                                                 (37, 512, 768, True)])
def test_out_proj_residual_vs_oracle(pkg, cuda, rows, fin, hidden, f32):
    """y = residual + linear(attn, W_o, b): decode rows (1B), prefill rows
    (0.5B), and a ragged row count with float32 residual / output."""
    rng = np.random.default_rng(rows)
    attn = f16(rng.standard_normal((rows, fin)))
    w, bias = weights(rng, fin, hidden)
    res = rng.standard_normal((rows, hidden)).astype(np.float32)
    if not f32:
        res = f16(res)
    dt = torch.float32 if f32 else torch.float16
    ad, wd = torch.from_numpy(attn).to(cuda, torch.float16), torch.from_numpy(w).to(cuda, torch.float16)
    bd, rd = torch.from_numpy(bias).to(cuda), torch.from_numpy(res).to(cuda, dt)
    y = torch.full((rows, hidden), float("nan"), dtype=dt, device=cuda)
    ctx = pkg.Context.default(0)
    rc = pkg.lib().tla_out_proj(ctx.handle, P(ad), P(wd), P(bd), P(rd), P(y), rows, fin, hidden, 4 if f32 else 0,
                                stream())
    assert rc == 0, pkg.lib().tla_status_string(rc).decode()
    torch.cuda.synchronize()
    assert ctx.error() == 0
    exp = oracle.linear(attn, w, bias, threads=THREADS) + res
    assert_close(y.float().cpu().numpy(), exp, what="output projection + residual")


def test_out_proj_allreduce_one_rank_vs_oracle(pkg, cuda):
    """The head-sharded path with a single rank: the GEMM's partial tiles go
    through the exchange buffer (epoch words) and the finishing kernel adds
    bias and residual; three calls in a row cover both buffer parities."""
    from three_llm_b200 import sharding

    rng = np.random.default_rng(17)
    rows, fin, hidden = 64, 1024, 2048
    w, bias = weights(rng, fin, hidden)
    wd, bd = torch.from_numpy(w).to(cuda, torch.float16), torch.from_numpy(bias).to(cuda)
    op = sharding.HeadShardedOutProj(rows, hidden, 0, 1, cuda.index or 0, group=False)
    try:
        op.exchange.connect_buffers([op.exchange.buffer()])
        for call in range(3):
            attn = f16(rng.standard_normal((rows, fin)))
            res = f16(rng.standard_normal((rows, hidden)))
            y = op(torch.from_numpy(attn).to(cuda, torch.float16), wd, bd,
                   torch.from_numpy(res).to(cuda, torch.float16))
            torch.cuda.synchronize()
            assert op.exchange.context.error() == 0
            exp = oracle.linear(attn, w, bias, threads=THREADS) + res
            assert_close(y.float().cpu().numpy(), exp, what=f"all-reduce output projection, call {call}")
    finally:
        op.close()

