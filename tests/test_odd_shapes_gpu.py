"""Odd shapes against the oracle, and the same shapes under the bounds-check
build (libtla_check.so, -DTLA_BOUNDS_CHECK: every guarded index is checked
against its buffer and a bad one is reported as TLA_ERR_BOUNDS, which these
tests would see as a non-zero device status).

The shapes are the edges of the kernels' tiling: a single cached token (T=1),
context lengths that are not a multiple of the 64-token decode tile or the
128-token prefill step, a GQA ratio of 7 (14 query / 2 kv heads), one-token
and 77-token prefill chunks, at head_dim 64 and 128.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_decode_gpu import assert_close, f16

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("lengths", [[0], [1, 77, 130, 191], [63, 64, 65, 127, 129]])
def test_odd_decode_lengths_gqa7(pkg, cuda, D, lengths):
    rng = np.random.default_rng(len(lengths) + D)
    Hq, Hk, T = 14, 2, 256
    B = len(lengths)
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    qkv = f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 1e6,
                                                    "maxBatch": B, "dtype": torch.float16})
    for b in range(B):
        layer.write_cache(b, 0, kc[b], vc[b])
    out = layer.decode(torch.from_numpy(qkv).to(cuda, torch.float16),
                       torch.tensor(lengths, dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert layer.context.error() == 0
    exp = oracle.decode_batch(qkv, lengths, kc, vc, threads=8, head_count=Hq, kv_head_count=Hk, head_dim=D,
                              rope_theta=1e6)
    assert_close(out, exp, what=f"decode lengths {lengths}")


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S,starts", [(1, [0, 5]), (77, [0, 51]), (130, [3, 0])])
def test_odd_prefill_chunks_gqa7(pkg, cuda, D, S, starts):
    rng = np.random.default_rng(S + D)
    Hq, Hk, T = 14, 2, 256
    B = len(starts)
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    pre_k, pre_v = kc.copy(), vc.copy()
    qkv = f16(rng.standard_normal((B, S, (Hq + 2 * Hk) * D)))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 1e6,
                                                    "maxBatch": B, "dtype": torch.float16})
    for b in range(B):
        layer.write_cache(b, 0, pre_k[b], pre_v[b])
    out = layer.prefill(torch.from_numpy(qkv).to(cuda, torch.float16),
                        torch.tensor(starts, dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert layer.context.error() == 0
    exp = oracle.prefill(qkv, starts, kc, vc, threads=8, head_count=Hq, kv_head_count=Hk, head_dim=D,
                         rope_theta=1e6)
    assert_close(out, exp, what=f"prefill S={S} starts {starts}")


def test_odd_shapes_under_bounds_check_build(pkg):
    """The odd-shape tests above, the exchange and the projections, in a fresh
    process that loads libtla_check.so: no guarded index may leave its buffer."""
    subprocess.run(["make", "-s", "-j8", "-C", str(ROOT / "three-llm_b200" / "csrc"), "check"], check=True)
    lib = ROOT / "three-llm_b200" / "libtla_check.so"
    env = dict(os.environ, TLA_LIBRARY=str(lib))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "gpu",
                        "tests/test_odd_shapes_gpu.py", "-k", "not bounds_check",
                        "tests/test_proj_gpu.py", "tests/test_zz_no_alloc.py",
                        "tests/test_decode_gpu.py::test_sequence_shards_combine_equals_full_decode",
                        "tests/test_decode_gpu.py::test_qk_norm_vnorm_gate_partial_rope_yarn",
                        "tests/test_prefill_gpu.py::test_prefill_output_gate",
                        "tests/test_prefill_gpu.py::test_prefill_small_generic_shapes"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
