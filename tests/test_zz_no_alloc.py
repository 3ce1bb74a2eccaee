"""The allocation-free decode entry point, tla_decode_noalloc.

Some hosts cannot call cudaMalloc: their device memory is all owned by their
own pool or a fixed budget, or their serving loop must not take cudaMalloc's
implicit device-wide synchronisation. For them the library offers one decode
entry point that allocates nothing: its scratch is a fixed static device array
inside libtla.so, and the caller passes every other buffer.

These checks call it through the C ABI and compare it with the allocating
entry point, tla_decode, on the same cache and inputs, twice in a row (the
static array keeps the previous call's contents, so the second call shows
that nothing stale leaks into it), and with the oracle. The file is named to
be collected last. (The grid clamp to what the 8 MiB array holds does not
trigger on a B200: even GQA group 16 at head_dim 128 needs 500 CTAs of scratch
slots, above the persistent grid of 2 x 148.)
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.test_decode_gpu import assert_close, f16

pytestmark = pytest.mark.gpu


def config_struct(pkg, Hq, Hk, D, max_tokens, max_batch, theta, scaling=None, flags=0):
    from three_llm_b200 import _abi

    c = _abi.AttnConfig()
    c.head_count, c.kv_head_count, c.head_dim = Hq, Hk, D
    c.max_tokens, c.max_batch = max_tokens, max_batch
    c.rotary_dim, c.rope_freq_dim, c.rope_pair_count = -1, 0, -1
    c.rope_theta = theta
    c.rope_scaling = _abi.make_scaling(scaling)
    c.has_attn_scale = 0
    c.rms_epsilon = 0.0
    c.flags = flags
    return c


def noalloc_decode(pkg, cfg, view, qkv, positions, out, status, gate=None, qn=None, kn=None):
    lib = pkg.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def p(t):
        return None if t is None else ctypes.c_void_p(t.data_ptr())

    return lib.tla_decode_noalloc(ctypes.byref(cfg), ctypes.c_void_p(view.key), ctypes.c_void_p(view.value), p(qn),
                                  p(kn), p(qkv), p(positions), p(gate), p(out), p(status), qkv.shape[0], stream)


YARN = {"type": "yarn", "factor": 4.0, "original_context_length": 512.0, "beta_fast": 32.0, "beta_slow": 1.0}


@pytest.mark.parametrize("D,Hq,Hk", [(64, 32, 8), (128, 32, 8), (64, 32, 2), (128, 16, 1)])
def test_noalloc_decode_matches_tla_decode_twice(pkg, cuda, D, Hq, Hk):
    """Two calls in a row through the C ABI, each against tla_decode on a twin
    layer with the same cache contents and, for the first call, against the
    oracle. GQA groups 4 and 16, head_dim 64 and 128, with the output gate,
    offset QK-norm and YaRN scaling switched on."""
    from oracle import oracle
    from three_llm_b200 import _abi

    rng = np.random.default_rng(21 + D + Hk)
    T, B = 1536, 6
    qn = (rng.standard_normal(D) * 0.1).astype(np.float32)
    kn = (rng.standard_normal(D) * 0.1).astype(np.float32)
    opts = {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5, "maxBatch": B, "dtype": torch.float16,
            "ropeScaling": YARN, "qNormWeight": qn, "kNormWeight": kn, "offsetRMSNorm": True}
    twin = pkg.CUDAAttention(None, Hq * D, Hq, T, opts)   # tla_decode, allocating path
    own = pkg.CUDAAttention(None, Hq * D, Hq, T, opts)    # only its cache is used, by tla_decode_noalloc
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    for b in range(B):
        twin.write_cache(b, 0, kc[b], vc[b])
        own.write_cache(b, 0, kc[b], vc[b])
    cfg = config_struct(pkg, Hq, Hk, D, T, B, 5e5, YARN, _abi.FLAG_OFFSET_RMS_NORM)
    view = own.cache_view()
    qn_d = torch.from_numpy(qn).to(cuda)
    kn_d = torch.from_numpy(kn).to(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call, lengths in enumerate([[5, 64, 700, 1024, 1300, 1535], [6, 129, 640, 1000, 1200, 1400]]):
        qkv_h = f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))
        gate_h = f16(rng.standard_normal((B, Hq * D)))
        qkv = torch.from_numpy(qkv_h).to(cuda, torch.float16)
        gate = torch.from_numpy(gate_h).to(cuda, torch.float16)
        pos = torch.tensor(lengths, dtype=torch.int32, device=cuda)
        expected = twin.decode(qkv, pos, gate=gate).float().cpu().numpy()
        out = torch.full((B, Hq * D), float("nan"), dtype=torch.float16, device=cuda)
        rc = noalloc_decode(pkg, cfg, view, qkv, pos, out, status, gate, qn_d, kn_d)
        assert rc == 0, pkg.lib().tla_status_string(rc).decode()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert twin.context.error() == 0
        got = out.float().cpu().numpy()
        assert_close(got, expected, what=f"noalloc call {call} vs tla_decode")
        if call == 0:
            exp = oracle.decode_batch(qkv_h, lengths, kc.copy(), vc.copy(), gate=gate_h, threads=8, head_count=Hq,
                                      kv_head_count=Hk, head_dim=D, rope_theta=5e5, rope_scaling=YARN,
                                      q_norm_weight=qn, k_norm_weight=kn, offset_rms_norm=True)
            assert_close(got, exp, what="noalloc vs oracle")
        k_new, v_new = own.read_cache(B - 1, lengths[-1], 1)
        k_twin, v_twin = twin.read_cache(B - 1, lengths[-1], 1)
        np.testing.assert_array_equal(k_new, k_twin)  # the same appended row
        np.testing.assert_array_equal(v_new, v_twin)
    twin.close()
    own.close()


def test_noalloc_with_smaller_batch_leaves_larger_layers_working(pkg, cuda):
    """The decode kernel's shared-memory limit is shared with the allocating
    layers: an allocation-free call with a small max_batch must not lower it
    below what a layer created earlier with a larger max_batch needs."""
    from oracle import oracle

    rng = np.random.default_rng(31)
    Hq, Hk, D, T, B = 32, 8, 64, 512, 64
    big = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                  "maxBatch": B, "dtype": torch.float16})
    small = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                    "maxBatch": 4, "dtype": torch.float16})
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    qkv4 = torch.from_numpy(f16(rng.standard_normal((4, (Hq + 2 * Hk) * D)))).to(cuda, torch.float16)
    out4 = torch.empty(4, Hq * D, dtype=torch.float16, device=cuda)
    rc = noalloc_decode(pkg, config_struct(pkg, Hq, Hk, D, T, 4, 5e5), small.cache_view(), qkv4,
                        torch.tensor([1, 2, 3, 4], dtype=torch.int32, device=cuda), out4, status)
    assert rc == 0
    lengths = [int(x) for x in rng.integers(1, T - 1, size=B)]
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    for b in range(B):
        big.write_cache(b, 0, kc[b], vc[b])
    qkv = f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))
    out = big.decode(torch.from_numpy(qkv).to(cuda, torch.float16),
                     torch.tensor(lengths, dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert big.context.error() == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    exp = oracle.decode_batch(qkv, lengths, kc, vc, threads=8, head_count=Hq, kv_head_count=Hk, head_dim=D,
                              rope_theta=5e5)
    assert_close(out, exp, what="batch-64 decode after a batch-4 allocation-free call")
    small.close()
    big.close()


def test_noalloc_rejects_requests_beyond_its_scratch(pkg, cuda):
    """Every case below is rejected on the host before any device memory is touched."""
    Hq, D = 32, 64
    view_stub = type("V", (), {"key": 1 << 20, "value": 1 << 20})()  # never dereferenced
    row = 3 * Hq * D
    qkv = torch.zeros(1024, row, dtype=torch.float16, device=cuda)
    pos = torch.zeros(1024, dtype=torch.int32, device=cuda)
    out = torch.zeros(1, dtype=torch.float16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    cfg = config_struct(pkg, Hq, Hq, D, 64, 1024, 5e5)                         # 1024 x 32 kv heads > 16384
    assert noalloc_decode(pkg, cfg, view_stub, qkv, pos, out, status) == -16    # TLA_ERR_SCRATCH_LIMIT
    cfg = config_struct(pkg, Hq, 8, D, 64, 2048, 5e5)
    assert noalloc_decode(pkg, cfg, view_stub, qkv[:8], pos[:8], out, status) == -9   # max_batch > 1024
    cfg = config_struct(pkg, Hq, 8, D, 64, 4, 5e5)
    assert noalloc_decode(pkg, cfg, view_stub, qkv[:8], pos[:8], out, status) == -1   # batch > max_batch
