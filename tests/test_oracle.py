"""Pins the CPU oracle to the reference's own golden vectors and known answers.

Mirrors packages/three-llm/src/runtime/rope.test.ts:8-47 (RoPE tables,
rotated Q/K and tiny-Llama logits against pinned Transformers output) and
packages/three-llm/src/engine.test.ts:506-551 (closed-form softmax, RMSNorm
and RoPE checks).
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
ROPE = json.loads((GOLDEN / "rope_cases.json").read_text())
CASES = ROPE["cases"]


def expect_close(actual, expected, atol=2e-5, rtol=2e-4):
    """expectClose of packages/three-llm/src/test/reference.ts:39-47."""
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    assert a.shape == e.shape
    assert np.all(np.isfinite(a))
    bad = np.abs(a - e) > atol + rtol * np.abs(e)
    assert not bad.any(), f"max err {np.max(np.abs(a - e))} at {np.argmax(bad)}"


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_rope_tables_and_rotation_match_pinned_transformers(case):
    inv, af = oracle.rope_parameters(8, case["theta"], case["scaling"])
    expect_close(inv, case["inv_freq"], 1e-8, 1e-6)
    assert af == pytest.approx(case["attention_factor"], abs=5e-7)
    for i, pos in enumerate(case["positions"]):
        for src, dst in (("query", "rotated_query"), ("key", "rotated_key")):
            got = oracle.apply_rope(case[src][i], 0, 8, pos, case["theta"], scaling=case["scaling"])
            expect_close(got, case[dst][i])


def test_rope_rejections():
    with pytest.raises(oracle.OracleError, match="even integer"):
        oracle.rope_parameters(3, 10000)
    with pytest.raises(oracle.OracleError, match="theta"):
        oracle.rope_parameters(8, 1.0)
    with pytest.raises(oracle.OracleError, match="factor"):
        oracle.rope_parameters(8, 10000, {"type": "linear", "factor": 0.5})
    with pytest.raises(oracle.OracleError, match="factor"):
        oracle.rope_parameters(8, 10000, {"type": "yarn", "factor": float("nan")})
    with pytest.raises(oracle.OracleError, match="YaRN"):
        oracle.rope_parameters(8, 10000, {"type": "yarn", "factor": 4, "original_context_length": 16,
                                          "beta_fast": 1, "beta_slow": 2})
    with pytest.raises(oracle.OracleError, match="Llama 3"):
        oracle.rope_parameters(8, 10000, {"type": "llama3", "factor": 4})
    # rotary dim 0 is the identity (rope.test.ts:42-43)
    v = np.array([1, 2, 3, 4], dtype=np.float32)
    np.testing.assert_array_equal(oracle.apply_rope(v, 0, 0, 8, 10000), v)


def test_closed_form_kats():
    # engine.test.ts:506-509
    expect_close(oracle.softmax([1, 2, 3]), [0.09003057, 0.24472848, 0.66524094], 1e-6, 0)
    expect_close(oracle.softmax([1, 1, 1]), [1 / 3] * 3, 1e-6, 0)
    expect_close(oracle.softmax([100, 101, 102]), oracle.softmax([0, 1, 2]), 1e-6, 0)
    assert float(np.sum(oracle.softmax([-5, 0, 2.5]).astype(np.float64))) == pytest.approx(1, abs=1e-6)
    # engine.test.ts:532-539
    inv_rms = 1 / math.sqrt(14 / 3 + 1e-5)
    expect_close(oracle.rms_norm([1, 2, 3], [1, 1, 1], 1e-5), [inv_rms, 2 * inv_rms, 3 * inv_rms], 1e-5, 0)
    expect_close(oracle.rms_norm([1, 2, 3], [0.5, 0, -0.25], 1e-5, True),
                 [inv_rms * 1.5, 2 * inv_rms, 3 * inv_rms * 0.75], 1e-5, 0)
    # engine.test.ts:550-551
    rope = oracle.apply_rope([1, 0, 0, 1], 0, 4, 1, 10000)
    assert abs(rope[0] - math.cos(1)) < 1e-5


def _linear(x, w_out_in):
    return (w_out_in.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)


def _tiny_llama_logits(case):
    """DecoderCPURunner.forwardToken (decoder/DecoderCPURunner.ts:47-138, pre-norm
    Llama branch) with the oracle's causalAttention for the attention step."""
    z = np.load(GOLDEN / "tiny_llama.npz")
    cfg = ROPE["meta"]["configs"][case["name"]]
    w = lambda n: z["w:" + n]
    H, Hq, Hk = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    D = H // Hq
    eps = cfg["rms_norm_eps"]
    L = cfg["num_hidden_layers"]
    T = 64
    caches = [(np.zeros((T, Hk * D), np.float32), np.zeros((T, Hk * D), np.float32)) for _ in range(L)]
    out = []
    for pos, tok in enumerate(ROPE["meta"]["input_ids"]):
        x = w("model.embed_tokens.weight")[tok].copy()
        for i in range(L):
            p = f"model.layers.{i}."
            n1 = oracle.rms_norm(x, w(p + "input_layernorm.weight"), eps)
            wqkv = np.concatenate([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                                   w(p + "self_attn.v_proj.weight")])
            qkv = _linear(n1, wqkv)
            kc, vc = caches[i]
            attn = oracle.causal_attention(qkv, pos, kc, vc, head_count=Hq, kv_head_count=Hk, head_dim=D,
                                           rope_theta=cfg["rope_theta"], rope_scaling=case["scaling"],
                                           rms_epsilon=eps)
            x = (x + _linear(attn, w(p + "self_attn.o_proj.weight"))).astype(np.float32)
            n2 = oracle.rms_norm(x, w(p + "post_attention_layernorm.weight"), eps)
            g = _linear(n2, w(p + "mlp.gate_proj.weight")).astype(np.float64)
            u = _linear(n2, w(p + "mlp.up_proj.weight")).astype(np.float64)
            hdn = (g / (1 + np.exp(-g)) * u).astype(np.float32)
            x = (x + _linear(hdn, w(p + "mlp.down_proj.weight"))).astype(np.float32)
        xn = oracle.rms_norm(x, w("model.norm.weight"), eps)
        out.append(_linear(xn, w("lm_head.weight")))
    return np.stack(out), z["logits:" + case["name"]]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_tiny_llama_logits_match_pinned_transformers(case):
    got, expected = _tiny_llama_logits(case)
    expect_close(got, expected)


def test_decode_batch_and_prefill_equal_single_steps():
    rng = np.random.default_rng(1)
    Hq, Hk, D, T, B, S = 4, 2, 8, 16, 3, 5
    opts = dict(head_count=Hq, kv_head_count=Hk, head_dim=D, rope_theta=10000.0)
    row = (Hq + 2 * Hk) * D
    qkv = rng.standard_normal((B, S, row)).astype(np.float32)
    kc = np.zeros((B, T, Hk * D), np.float32)
    vc = np.zeros_like(kc)
    ref = np.stack([np.stack([oracle.causal_attention(qkv[b, t], 2 + t, kc[b], vc[b], **opts) for t in range(S)])
                    for b in range(B)])
    kc2 = np.zeros_like(kc)
    vc2 = np.zeros_like(kc)
    got = oracle.prefill(qkv, [2] * B, kc2, vc2, threads=4, **opts)
    np.testing.assert_array_equal(got, ref)
    np.testing.assert_array_equal(kc2, kc)
    kc3 = np.zeros_like(kc)
    vc3 = np.zeros_like(kc)
    steps = [oracle.decode_batch(qkv[:, t], [2 + t] * B, kc3, vc3, threads=3, **opts) for t in range(S)]
    np.testing.assert_array_equal(np.stack(steps, 1), ref)
