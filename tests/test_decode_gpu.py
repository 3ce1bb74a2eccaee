"""GPU parity of the decode path (tla_decode through the C ABI) against the oracle.

Shapes and options follow the reference's own attention tests
(packages/three-llm/src/test/tsl.browser.test.ts:201-394, harness
test/gpu.ts:138-242: every step's output against the CPU reference with the
cache written in lockstep) and the BASELINE configs. Tolerance: the
north-star bound |a - e| <= 2e-3 + 1e-2 |e| for the fp16 cache (inputs are
fp16-representable, so the oracle sees the same values); 1e-4 absolute, the
reference's own bound, for the float32 cache.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def assert_close(got, exp, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    assert got.shape == exp.shape, (got.shape, exp.shape)
    assert np.all(np.isfinite(got)), what
    err = np.abs(got - exp)
    bad = err > atol + rtol * np.abs(exp)
    assert not bad.any(), f"{what}: max abs err {err.max():.3e}, {bad.sum()} elements out of tolerance"


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def oracle_opts(Hq, Hk, D, **kw):
    o = dict(head_count=Hq, kv_head_count=Hk, head_dim=D)
    o.update(kw)
    return o


def layer_options(Hk, D, **kw):
    o = {"headDim": D, "kvHeadCount": Hk}
    o.update(kw)
    return o


def run_sequence(pkg, cuda, Hq, Hk, D, steps, max_tokens, options=None, oopts=None, dtype=torch.float32,
                 cache_dtype="float16", atol=ATOL, rtol=RTOL, gates=None):
    """Decode `steps` tokens one at a time through CUDAAttention.compute (the
    reference's operator call) and check every step against causalAttention."""
    row = (Hq + 2 * Hk) * D
    qkv_node = torch.zeros(row, dtype=dtype, device=cuda)
    opts = layer_options(Hk, D, cacheDtype=cache_dtype, **(options or {}))
    gate_node = None
    if gates is not None:
        gate_node = torch.zeros(Hq * D, dtype=dtype, device=cuda)
        opts["gateNode"] = gate_node
    layer = pkg.CUDAAttention(qkv_node, Hq * D, Hq, max_tokens, opts)
    kc = np.zeros((max_tokens, Hk * D), np.float32)
    vc = np.zeros_like(kc)
    for pos, x in enumerate(steps):
        x = np.asarray(x, np.float32)
        if dtype == torch.float16:
            x = f16(x)
        qkv_node.copy_(torch.from_numpy(x))
        g = None
        if gates is not None:
            g = np.asarray(gates[pos], np.float32)
            if dtype == torch.float16:
                g = f16(g)
            gate_node.copy_(torch.from_numpy(g))
        out = layer.compute(None, pos).float().cpu().numpy()
        exp = oracle.causal_attention(x, pos, kc, vc, gate=g, **(oopts or {}))
        assert_close(out, exp, atol, rtol, f"step {pos}")
    assert layer.context.error() == 0
    return layer, kc, vc


def fill_sin(n, seed):
    return oracle.fill_sin(n, seed)


# ---------------------------------------------------------------- reference test shapes
def test_mha_one_and_two_tokens(pkg, cuda):
    # tsl.browser.test.ts:201-215 (hidden 4, 2 heads, head_dim 2)
    steps = [[1, 0, 0, 1, 1, 0, 0, 1, 2, 3, 4, 5], [0, 1, 1, 0, 0, 1, 1, 0, 1, 1, 1, 1]]
    for cache in ("float32", "float16"):
        tol = (1e-4, 0) if cache == "float32" else (ATOL, RTOL)
        run_sequence(pkg, cuda, 2, 2, 2, steps, 4, options={"ropeTheta": 0}, oopts=oracle_opts(2, 2, 2),
                     cache_dtype=cache, atol=tol[0], rtol=tol[1])


def test_longer_cached_sequence(pkg, cuda):
    # tsl.browser.test.ts:217-233
    steps = [[1, 0, 0, 1, 1, 0, 0, 1, 2, 3, 4, 5], [0, 1, 1, 0, 0, 1, 1, 0, 1, 1, 1, 1],
             [0.5, -1, 2, 0, 0.25, 0.5, -0.5, 1, 0, 2, -1, 3], [-2, 1, 0.5, 0.5, 1, -1, 0, 0.25, 4, 0, 1, -2]]
    run_sequence(pkg, cuda, 2, 2, 2, steps, 8, oopts=oracle_opts(2, 2, 2), cache_dtype="float32", atol=1e-4, rtol=0)


@pytest.mark.parametrize("cache", ["float32", "float16"])
def test_gpt2_sized_heads(pkg, cuda, cache):
    # tsl.browser.test.ts:235-248: hidden 128, 2 heads (head_dim 64), 4 sin-filled steps
    steps = []
    for p in range(4):
        i = np.arange(128 * 3)
        steps.append((np.sin(p * 19.1 + i * 0.17) * 0.35).astype(np.float32))
    tol = (2e-4, 0) if cache == "float32" else (ATOL, RTOL)
    run_sequence(pkg, cuda, 2, 2, 64, steps, 8, oopts=oracle_opts(2, 2, 64), cache_dtype=cache,
                 atol=tol[0], rtol=tol[1])


CAUSAL_CASES = {
    # tsl.browser.test.ts:318-394 (assertCausalSequence)
    "gqa_no_rope": (4, 2, 2, 4, [0.3, 1.1], {}),
    "rope_mha": (2, 2, 2, 8, [0.2, 0.8, 1.4], {"rope_theta": 10000.0}),
    "gqa_rope": (4, 2, 2, 4, [0.5, 1.5], {"rope_theta": 10000.0, "rotary_dim": 2}),
    "partial_rope_scale": (2, 2, 4, 4, [0.6, 1.6], {"rope_theta": 10000.0, "rotary_dim": 2, "attn_scale": 0.25}),
    "sliding_window_gqa": (4, 2, 2, 8, [0.4, 1.4, 2.4], {"sliding_window": 2}),
    "qk_norm_rope": (2, 1, 4, 4, [0.7, 1.7], {"rope_theta": 10000.0,
                                              "q_norm_weight": [0.5, -0.25, 0.1, 0],
                                              "k_norm_weight": [0.2, 0.3, -0.1, 0.4],
                                              "offset_rms_norm": True, "rms_epsilon": 1e-6}),
}


def to_layer_options(kw):
    m = {"rope_theta": "ropeTheta", "rotary_dim": "rotaryDim", "attn_scale": "attnScale",
         "sliding_window": "slidingWindow", "q_norm_weight": "qNormWeight", "k_norm_weight": "kNormWeight",
         "offset_rms_norm": "offsetRMSNorm", "rms_epsilon": "rmsEpsilon", "v_norm": "vNorm",
         "rope_scaling": "ropeScaling", "rope_pair_count": "ropePairCount"}
    return {m[k]: v for k, v in kw.items()}


@pytest.mark.parametrize("name", list(CAUSAL_CASES))
@pytest.mark.parametrize("cache", ["float32", "float16"])
def test_reference_causal_cases(pkg, cuda, name, cache):
    Hq, Hk, D, T, seeds, kw = CAUSAL_CASES[name]
    n = (Hq + 2 * Hk) * D
    steps = [fill_sin(n, s) for s in seeds]
    tol = (1e-4, 0) if cache == "float32" else (ATOL, RTOL)
    run_sequence(pkg, cuda, Hq, Hk, D, steps, T, options=to_layer_options(kw), oopts=oracle_opts(Hq, Hk, D, **kw),
                 cache_dtype=cache, atol=tol[0], rtol=tol[1])


# ---------------------------------------------------------------- BASELINE config 1
@pytest.mark.parametrize("io", [torch.float32, torch.float16])
def test_config1_tiny_gqa_decode_every_step(pkg, cuda, io):
    """8 q heads, 2 kv heads, head_dim 64, positions 0..128 (128 cached + 1 new), theta 1e4, scale 1/8."""
    rng = np.random.default_rng(0)
    Hq, Hk, D, T = 8, 2, 64, 129
    steps = rng.standard_normal((T, (Hq + 2 * Hk) * D)).astype(np.float32)
    if io == torch.float16:
        steps = f16(steps)
    layer, kc, vc = run_sequence(pkg, cuda, Hq, Hk, D, steps, T, options={"ropeTheta": 10000.0},
                                 oopts=oracle_opts(Hq, Hk, D, rope_theta=10000.0), dtype=io)
    k, v = layer.read_cache(0, 0, T)
    assert_close(k, kc, 2e-3, 2e-3, "post-RoPE key cache")   # fp16 storage of the oracle's values
    assert_close(v, vc, 2e-3, 2e-3, "value cache")


# ---------------------------------------------------------------- batched / long / options
def batched_case(pkg, cuda, Hq, Hk, D, lengths, max_tokens, seed=0, dtype=torch.float16, layer_kw=None,
                 oracle_kw=None, gate=False, threads=8):
    """Random cached K/V (already post-RoPE, fp16 values) at ragged lengths, then one decode step
    per sequence at position = length; checks outputs and the appended cache rows."""
    rng = np.random.default_rng(seed)
    B = len(lengths)
    kc = f16(rng.standard_normal((B, max_tokens, Hk * D)))
    vc = f16(rng.standard_normal((B, max_tokens, Hk * D)))
    qkv = f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))
    g = f16(rng.standard_normal((B, Hq * D))) if gate else None
    opts = layer_options(Hk, D, maxBatch=B, **(layer_kw or {}))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, max_tokens, dict(opts, dtype=dtype))
    for b in range(B):
        layer.write_cache(b, 0, kc[b], vc[b])
    pos = np.asarray(lengths, np.int32)
    out = layer.decode(torch.from_numpy(qkv).to(cuda, dtype), torch.from_numpy(pos).to(cuda),
                       gate=None if g is None else torch.from_numpy(g).to(cuda, dtype))
    got = out.float().cpu().numpy()
    exp = oracle.decode_batch(qkv, pos, kc, vc, gate=g, threads=threads, **oracle_opts(Hq, Hk, D, **(oracle_kw or {})))
    assert layer.context.error() == 0
    assert_close(got, exp, what="batched decode")
    for b in range(B):
        k, v = layer.read_cache(b, int(pos[b]), 1)
        assert_close(k[0], kc[b, pos[b]], 2e-3, 2e-3, "appended key")
        assert_close(v[0], vc[b, pos[b]], 2e-3, 2e-3, "appended value")
    return layer


@pytest.mark.parametrize("D", [64, 128])
def test_batched_ragged_decode(pkg, cuda, D):
    batched_case(pkg, cuda, 32, 8, D, [0, 1, 63, 64, 65, 300, 511, 1000], 1024,
                 layer_kw={"ropeTheta": 500000.0}, oracle_kw={"rope_theta": 500000.0})


def test_many_sequences_span_cta_segments(pkg, cuda):
    # total tiles >> persistent CTAs: CTAs cover several (sequence, kv head) pairs
    rng = np.random.default_rng(3)
    lengths = rng.integers(100, 2048, size=24)
    batched_case(pkg, cuda, 32, 8, 64, list(lengths), 2048, layer_kw={"ropeTheta": 500000.0},
                 oracle_kw={"rope_theta": 500000.0})


@pytest.mark.parametrize("Hq,Hk", [(32, 2), (16, 16), (14, 2), (12, 1)])
def test_gqa_ratios(pkg, cuda, Hq, Hk):
    batched_case(pkg, cuda, Hq, Hk, 64, [5, 130, 700], 768, layer_kw={"ropeTheta": 1e6},
                 oracle_kw={"rope_theta": 1e6})


def test_fp32_io_d128(pkg, cuda):
    batched_case(pkg, cuda, 32, 8, 128, [17, 900], 1024, dtype=torch.float32, layer_kw={"ropeTheta": 500000.0},
                 oracle_kw={"rope_theta": 500000.0})


def test_sliding_window_fast_path(pkg, cuda):
    batched_case(pkg, cuda, 8, 2, 64, [3, 200, 513], 640, layer_kw={"ropeTheta": 10000.0, "slidingWindow": 128},
                 oracle_kw={"rope_theta": 10000.0, "sliding_window": 128})


def test_qk_norm_vnorm_gate_partial_rope_yarn(pkg, cuda):
    rng = np.random.default_rng(7)
    qn = rng.standard_normal(64).astype(np.float32) * 0.1
    kn = rng.standard_normal(64).astype(np.float32) * 0.1
    yarn = {"type": "yarn", "factor": 4.0, "original_context_length": 256.0, "beta_fast": 32.0, "beta_slow": 1.0}
    batched_case(pkg, cuda, 16, 4, 64, [10, 333, 900], 1024, gate=True,
                 layer_kw={"ropeTheta": 10000.0, "rotaryDim": 32, "qNormWeight": qn, "kNormWeight": kn,
                           "offsetRMSNorm": True, "vNorm": True, "ropeScaling": yarn, "rmsEpsilon": 1e-6},
                 oracle_kw={"rope_theta": 10000.0, "rotary_dim": 32, "q_norm_weight": qn, "k_norm_weight": kn,
                            "offset_rms_norm": True, "v_norm": True, "rope_scaling": yarn, "rms_epsilon": 1e-6})


def test_large_positions_rope_accuracy(pkg, cuda):
    # positions near 131072: the angle reduction must keep float32 accuracy
    batched_case(pkg, cuda, 8, 2, 128, [131000], 131072, layer_kw={"ropeTheta": 500000.0},
                 oracle_kw={"rope_theta": 500000.0})


# ---------------------------------------------------------------- error channel / sharing / reset
def test_position_outside_cache_reports_status(pkg, cuda):
    layer = pkg.CUDAAttention(None, 8 * 64, 8, 64, {"headDim": 64, "kvHeadCount": 2, "dtype": torch.float16})
    qkv = torch.zeros(1, 12 * 64, dtype=torch.float16, device=cuda)
    layer.decode(qkv, torch.tensor([64], dtype=torch.int32, device=cuda))
    assert layer.context.error() == -12  # TLA_ERR_POSITION, kernel skipped the work
    layer.decode(qkv, torch.tensor([63], dtype=torch.int32, device=cuda))
    assert layer.context.error() == 0


def test_shared_attention_reads_owner_cache(pkg, cuda):
    rng = np.random.default_rng(11)
    Hq, Hk, D, T = 8, 2, 64, 256
    owner = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "dtype": torch.float16,
                                                    "ropeTheta": 10000.0})
    kc = f16(rng.standard_normal((T, Hk * D)))
    vc = f16(rng.standard_normal((T, Hk * D)))
    owner.write_cache(0, 0, kc, vc)
    borrower = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "dtype": torch.float16,
                                                       "ropeTheta": 10000.0, "sharedAttention": owner})
    qkv = f16(rng.standard_normal((1, (Hq + 2 * Hk) * D)))
    out = borrower.decode(torch.from_numpy(qkv).to(cuda, torch.float16),
                          torch.tensor([200], dtype=torch.int32, device=cuda)).float().cpu().numpy()
    exp = oracle.decode_batch(qkv, [200], kc[None].copy(), vc[None].copy(),
                              **oracle_opts(Hq, Hk, D, rope_theta=10000.0, write_cache=False))
    assert_close(out, exp, what="sharedAttention")
    k, _ = owner.read_cache(0, 200, 1)
    np.testing.assert_array_equal(k[0], kc[200])  # the borrower did not append
    borrower.reset()  # no-op for a borrower (TSLAttention.ts:435)
    k, _ = owner.read_cache(0, 200, 1)
    np.testing.assert_array_equal(k[0], kc[200])
    owner.reset()
    k, _ = owner.read_cache(0, 0, T)
    assert not k.any()


# ---------------------------------------------------------------- sequence shards + LSE combine
@pytest.mark.parametrize("D", [64, 128])
def test_sequence_shards_combine_equals_full_decode(pkg, cuda, D):
    rng = np.random.default_rng(5)
    Hq, Hk, T, R = 32, 8, 3000, 4
    kc = f16(rng.standard_normal((1, T + 1, Hk * D)))
    vc = f16(rng.standard_normal((1, T + 1, Hk * D)))
    qkv = f16(rng.standard_normal((1, (Hq + 2 * Hk) * D)))
    bounds = [0, 700, 1600, 1601, T + 1]  # one rank with a single token, last rank owns the new token
    parts = []
    for r in range(R):
        lo, hi = bounds[r], bounds[r + 1]
        layer = pkg.CUDAAttention(None, Hq * D, Hq, hi - lo, {"headDim": D, "kvHeadCount": Hk,
                                                              "dtype": torch.float16, "ropeTheta": 500000.0})
        owns = r == R - 1
        n_fill = (hi - lo) - (1 if owns else 0)
        if n_fill > 0:
            layer.write_cache(0, 0, kc[0, lo:lo + n_fill], vc[0, lo:lo + n_fill])
        parts.append(layer.decode_partial(torch.from_numpy(qkv).to(cuda, torch.float16),
                                          torch.tensor([T], dtype=torch.int32, device=cuda), lo, hi - lo, owns))
        assert layer.context.error() == 0
    out = pkg.combine_lse(torch.stack(parts)).float().cpu().numpy()
    exp = oracle.decode_batch(qkv, [T], kc, vc, threads=8, **oracle_opts(Hq, Hk, D, rope_theta=500000.0))
    assert_close(out, exp, what="LSE combine of sequence shards")


# ---------------------------------------------------------------- recovery and shared launch limits
def test_counters_recover_after_error_launch(pkg, cuda):
    """A launch whose positions are partly invalid (TLA_ERR_POSITION: those
    sequences are skipped) over many CTA-spanning sequences, then a correct
    launch on the same context: the second launch's split-KV tickets start
    from clean counters and its output matches the oracle."""
    rng = np.random.default_rng(12)
    Hq, Hk, D, T, B = 32, 8, 64, 2048, 24
    lengths = [int(x) for x in rng.integers(300, T - 1, size=B)]
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    layer = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                    "maxBatch": B, "dtype": torch.float16})
    for b in range(B):
        layer.write_cache(b, 0, kc[b], vc[b])
    qkv = f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))
    qkv_d = torch.from_numpy(qkv).to(cuda, torch.float16)
    bad = list(lengths)
    bad[3], bad[17] = T + 5, -1
    layer.decode(qkv_d, torch.tensor(bad, dtype=torch.int32, device=cuda))
    assert layer.context.error() == -12  # TLA_ERR_POSITION; the reset also clears the counters
    for b in range(B):  # undo the first launch's appends of the valid sequences
        layer.write_cache(b, 0, kc[b], vc[b])
    out = layer.decode(qkv_d, torch.tensor(lengths, dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert layer.context.error() == 0
    exp = oracle.decode_batch(qkv, lengths, kc, vc, threads=8, **oracle_opts(Hq, Hk, D, rope_theta=5e5))
    assert_close(out, exp, what="decode after an error launch")


def test_dynamic_smem_limit_is_never_lowered(pkg, cuda):
    """Every layer of one kernel instance shares its dynamic shared-memory
    limit: a layer created later with a smaller batch must not lower it below
    what an earlier layer's full-batch launch needs."""
    rng = np.random.default_rng(13)
    Hq, Hk, D, T = 32, 8, 64, 512
    big = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                  "maxBatch": 256, "dtype": torch.float16})
    small = pkg.CUDAAttention(None, Hq * D, Hq, T, {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5,
                                                    "maxBatch": 1, "dtype": torch.float16})
    B = 256
    lengths = [int(x) for x in rng.integers(1, T - 1, size=B)]
    kc = f16(rng.standard_normal((B, T, Hk * D)))
    vc = f16(rng.standard_normal((B, T, Hk * D)))
    for b in range(B):
        big.write_cache(b, 0, kc[b], vc[b])
    qkv = f16(rng.standard_normal((B, (Hq + 2 * Hk) * D)))
    out = big.decode(torch.from_numpy(qkv).to(cuda, torch.float16),
                     torch.tensor(lengths, dtype=torch.int32, device=cuda)).float().cpu().numpy()
    assert big.context.error() == 0
    exp = oracle.decode_batch(qkv, lengths, kc, vc, threads=8, **oracle_opts(Hq, Hk, D, rope_theta=5e5))
    assert_close(out, exp, what="full-batch launch after a smaller layer")
    small.close()
    big.close()


# ---------------------------------------------------------------- queryAttribute / scoreAttribute
ROPE_FIXTURE = None


def rope_fixture():
    global ROPE_FIXTURE
    if ROPE_FIXTURE is None:
        import json
        from pathlib import Path

        ROPE_FIXTURE = json.loads((Path(__file__).resolve().parent / "golden" / "rope_cases.json").read_text())
    return ROPE_FIXTURE["cases"]


@pytest.mark.parametrize("case", range(5))
def test_query_attribute_matches_pinned_rotated_q(pkg, cuda, case):
    """reference.browser.test.ts:41-67: one head of dim 8, theta 1e4 and the
    case's RoPE scaling; after each compute() the rotated query
    (queryAttribute) and the cached key equal the pinned Transformers values,
    at the reference's tolerance (expectClose, test/reference.ts:39-47)."""
    c = rope_fixture()[case]
    node = torch.zeros(24, dtype=torch.float32, device=cuda)
    layer = pkg.CUDAAttention(node, 8, 1, 64, {"ropeTheta": c["theta"], "ropeScaling": c["scaling"],
                                               "cacheDtype": "float32"})
    for i, pos in enumerate(c["positions"]):
        x = np.zeros(24, np.float32)
        x[:8] = c["query"][i]
        x[8:16] = c["key"][i]
        node.copy_(torch.from_numpy(x))
        layer.compute(None, pos)
        assert_close(layer.queryAttribute, c["rotated_query"][i], 2e-5, 2e-4, f"{c['name']} query @ {pos}")
        assert_close(layer.keyCacheAttribute[pos * 8:(pos + 1) * 8], c["rotated_key"][i], 2e-5, 2e-4,
                     f"{c['name']} key @ {pos}")
    assert layer.context.error() == 0


def expected_scores(x, pos, kc, Hq, Hk, D, opts):
    """attnScale * <Q'_h, K_t> over the window (test/gpu.ts cpuAttentionScores), from
    the oracle's rotated query and its cache after the step."""
    q = np.asarray(x[:Hq * D], np.float32).copy()
    if opts.get("q_norm_weight") is not None:
        for h in range(Hq):
            q[h * D:(h + 1) * D] = oracle.rms_norm(q[h * D:(h + 1) * D], opts["q_norm_weight"],
                                                   opts.get("rms_epsilon", 1e-6), opts.get("offset_rms_norm", False))
    if opts.get("rope_theta"):
        for h in range(Hq):
            q = oracle.apply_rope(q, h * D, opts.get("rotary_dim", D), pos, opts["rope_theta"])
    scale = opts.get("attn_scale", 1 / np.sqrt(D))
    first = max(0, pos - opts["sliding_window"] + 1) if opts.get("sliding_window") else 0
    s = {}
    for h in range(Hq):
        kvh = h * Hk // Hq
        for t in range(first, pos + 1):
            s[(h, t)] = scale * float(np.dot(q[h * D:(h + 1) * D].astype(np.float64),
                                             kc[t, kvh * D:(kvh + 1) * D].astype(np.float64)))
    return s


@pytest.mark.parametrize("name,cache", [("mha", "float32"), ("gqa_rope", "float32"),
                                        ("sliding_window_gqa", "float32"), ("qk_norm_rope", "float32"),
                                        ("d64_gqa", "float16")])
def test_score_attribute_matches_reference_scores(pkg, cuda, name, cache):
    """test/gpu.ts:138-171 (assertAttentionSequence): after every step the score
    buffer holds attnScale * <Q', K_t> for the window's tokens."""
    if name == "mha":
        Hq, Hk, D, T, kw, steps = 2, 2, 2, 4, {}, [[1, 0, 0, 1, 1, 0, 0, 1, 2, 3, 4, 5],
                                                  [0, 1, 1, 0, 0, 1, 1, 0, 1, 1, 1, 1]]
    elif name == "d64_gqa":
        rng = np.random.default_rng(8)
        Hq, Hk, D, T, kw = 8, 2, 64, 40, {"rope_theta": 10000.0}
        steps = list(f16(rng.standard_normal((6, (Hq + 2 * Hk) * D))))
    else:
        Hq, Hk, D, T, seeds, kw = CAUSAL_CASES[name]
        steps = [fill_sin((Hq + 2 * Hk) * D, s) for s in seeds]
    layer, kc, vc = None, None, None
    node = torch.zeros((Hq + 2 * Hk) * D, dtype=torch.float32, device=cuda)
    layer = pkg.CUDAAttention(node, Hq * D, Hq, T, layer_options(Hk, D, cacheDtype=cache, **to_layer_options(kw)))
    kc = np.zeros((T, Hk * D), np.float32)
    vc = np.zeros_like(kc)
    tol = (1e-4, 0) if cache == "float32" else (ATOL, RTOL)
    for pos, x in enumerate(steps):
        x = np.asarray(x, np.float32)
        node.copy_(torch.from_numpy(x))
        layer.compute(None, pos)
        oracle.causal_attention(x, pos, kc, vc, **oracle_opts(Hq, Hk, D, **kw))
        got = layer.scoreAttribute.reshape(Hq, T)
        exp = expected_scores(x, pos, kc, Hq, Hk, D, kw)
        keys = sorted(exp)
        assert_close([got[h, t] for h, t in keys], [exp[k] for k in keys], tol[0], tol[1], f"{name} scores @ {pos}")
    assert layer.context.error() == 0
