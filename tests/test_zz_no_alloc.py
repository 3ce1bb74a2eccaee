"""The allocation-free decode entry point, tla_decode_noalloc.

Some hosts cannot call cudaMalloc: their device memory is all owned by their
own pool or a fixed budget, or their serving loop must not take cudaMalloc's
implicit device-wide synchronisation. For them the library offers one decode
entry point that allocates nothing: its scratch is a fixed static device array
inside libtla.so, and the caller passes every other buffer.

These checks call it through the C ABI and compare it with the allocating
entry point, tla_decode, on the same cache and inputs, twice in a row (the
static array keeps the previous call's contents, so the second call shows
that nothing stale leaks into it). The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.test_decode_gpu import assert_close, f16

pytestmark = pytest.mark.gpu


def config_struct(pkg, Hq, Hk, D, max_tokens, max_batch, theta):
    from three_llm_b200 import _abi

    c = _abi.AttnConfig()
    c.head_count, c.kv_head_count, c.head_dim = Hq, Hk, D
    c.max_tokens, c.max_batch = max_tokens, max_batch
    c.rotary_dim, c.rope_freq_dim, c.rope_pair_count = -1, 0, -1
    c.rope_theta = theta
    c.has_attn_scale = 0
    c.rms_epsilon = 0.0
    c.flags = 0
    return c


def noalloc_decode(pkg, cfg, view, qkv, positions, out, status):
    lib = pkg.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.tla_decode_noalloc(ctypes.byref(cfg), ctypes.c_void_p(view.key), ctypes.c_void_p(view.value), None,
                                  None, ctypes.c_void_p(qkv.data_ptr()), ctypes.c_void_p(positions.data_ptr()), None,
                                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                                  qkv.shape[0], stream)


def test_noalloc_decode_matches_tla_decode_twice(pkg, cuda):
    rng = np.random.default_rng(21)
    Hq, Hk, D, T, B = 32, 8, 64, 1536, 6
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                    "maxBatch": B, "dtype": torch.float16})
    for b in range(B):
        layer.write_cache(b, 0, f16(rng.standard_normal((T, Hk * D))), f16(rng.standard_normal((T, Hk * D))))
    cfg = config_struct(pkg, Hq, Hk, D, T, B, 5e5)
    view = layer.cache_view()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call, lengths in enumerate([[5, 64, 700, 1024, 1300, 1535], [1, 129, 640, 1000, 1200, 1400]]):
        qkv = torch.from_numpy(f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))).to(cuda, torch.float16)
        pos = torch.tensor(lengths, dtype=torch.int32, device=cuda)
        expected = layer.decode(qkv, pos).float().cpu().numpy()  # appends the new token
        out = torch.full((B, Hq * D), float("nan"), dtype=torch.float16, device=cuda)
        rc = noalloc_decode(pkg, cfg, view, qkv, pos, out, status)  # appends the same values again
        assert rc == 0, pkg.lib().tla_status_string(rc).decode()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert layer.context.error() == 0
        assert_close(out.float().cpu().numpy(), expected, what=f"noalloc call {call}")


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
