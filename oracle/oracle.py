"""ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY. Imported by tests/, by the smoke check and by the
CPU-baseline legs of bench.py, always as the checker or the timed reference
CPU implementation; the product path never imports it.

The option names mirror the reference's CausalAttentionOptions
(packages/three-llm/src/types.ts:314-331) in snake_case; `rope_scaling`
takes the recipe-level scaling object of types.ts:245-256 as a dict:
{"type": "linear"|"yarn"|"llama3", "factor": ..., ...}.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

ROPE_TYPES = {"default": 0, "none": 0, "linear": 1, "yarn": 2, "llama3": 3}


class OracleError(ValueError):
    pass


class RopeScaling(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("factor", ctypes.c_double),
        ("original_context_length", ctypes.c_double),
        ("beta_fast", ctypes.c_double),
        ("beta_slow", ctypes.c_double),
        ("has_attention_factor", ctypes.c_int32),
        ("attention_factor", ctypes.c_double),
        ("low_freq_factor", ctypes.c_double),
        ("high_freq_factor", ctypes.c_double),
    ]


class AttnOptions(ctypes.Structure):
    _fields_ = [
        ("head_count", ctypes.c_int32),
        ("kv_head_count", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("rotary_dim", ctypes.c_int32),
        ("rope_freq_dim", ctypes.c_int32),
        ("rope_pair_count", ctypes.c_int32),
        ("rope_theta", ctypes.c_double),
        ("scaling", RopeScaling),
        ("sliding_window", ctypes.c_int32),
        ("has_attn_scale", ctypes.c_int32),
        ("attn_scale", ctypes.c_double),
        ("q_norm_weight", ctypes.c_void_p),
        ("k_norm_weight", ctypes.c_void_p),
        ("rms_epsilon", ctypes.c_double),
        ("offset_rms_norm", ctypes.c_int32),
        ("query_only", ctypes.c_int32),
        ("write_cache", ctypes.c_int32),
        ("v_norm", ctypes.c_int32),
    ]


def build():
    """Compile liboracle.so with the Makefile next to this file."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        i32, f64 = ctypes.c_int32, ctypes.c_double
        L.orc_error_string.restype = ctypes.c_char_p
        L.orc_error_string.argtypes = [ctypes.c_int]
        L.orc_rope_parameters.argtypes = [i32, f64, P, P, P]
        L.orc_apply_rope.argtypes = [P, i32, i32, i32, f64, i32, i32, P]
        L.orc_softmax.argtypes = [P, i32, P]
        L.orc_softmax.restype = None
        L.orc_rms_norm.argtypes = [P, i32, P, f64, i32, P]
        L.orc_rms_norm.restype = None
        L.orc_rms_norm_packed_heads.argtypes = [P, i32, i32, P, f64, i32]
        L.orc_rms_norm_packed_heads.restype = None
        L.orc_causal_attention.argtypes = [P, i32, P, P, P, P, P]
        L.orc_decode_batch.argtypes = [P, P, i32, i32, P, P, P, P, P, i32]
        L.orc_prefill.argtypes = [P, P, P, i32, i32, i32, P, P, P, P, i32]
        L.orc_attend_heads.argtypes = [P, P, i32, i32, P, P, P, i32, i32, P, i32]
        L.orc_linear.argtypes = [P, i32, P, P, i32, i32, P, i32]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _check(rc):
    if rc != 0:
        raise OracleError(lib().orc_error_string(rc).decode())


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def make_scaling(spec):
    s = RopeScaling()
    if not spec:
        return s
    s.type = ROPE_TYPES[spec.get("type", "yarn")]
    s.factor = float(spec.get("factor", 1.0))
    s.original_context_length = float(spec.get("original_context_length", float("nan")))
    s.beta_fast = float(spec.get("beta_fast", float("nan")))
    s.beta_slow = float(spec.get("beta_slow", float("nan")))
    if spec.get("attention_factor") is not None:
        s.has_attention_factor = 1
        s.attention_factor = float(spec["attention_factor"])
    s.low_freq_factor = float(spec.get("low_freq_factor", float("nan")))
    s.high_freq_factor = float(spec.get("high_freq_factor", float("nan")))
    return s


def rope_parameters(dim, theta, scaling=None):
    """ropeParameters (rope.ts:4-52) -> (inv_freq float32[dim/2], attention_factor)."""
    inv = np.zeros(max(dim // 2, 1), dtype=np.float32)
    af = ctypes.c_double(0)
    s = make_scaling(scaling)
    _check(lib().orc_rope_parameters(int(dim), float(theta), ctypes.byref(s), _ptr(inv), ctypes.byref(af)))
    return inv[: dim // 2], af.value


def apply_rope(vector, head_offset, rotary_dim, position, theta, rope_freq_dim=0, rope_pair_count=-1, scaling=None):
    """applyRoPE (math.ts:118-152); returns a rotated float32 copy."""
    v = _f32(vector).copy()
    s = make_scaling(scaling)
    _check(lib().orc_apply_rope(_ptr(v), int(head_offset), int(rotary_dim), int(position), float(theta),
                                int(rope_freq_dim), int(rope_pair_count), ctypes.byref(s)))
    return v


def softmax(values):
    v = _f32(values)
    out = np.empty_like(v)
    lib().orc_softmax(_ptr(v), v.size, _ptr(out))
    return out


def rms_norm(values, weight=None, epsilon=1e-5, offset=False):
    v = _f32(values)
    w = None if weight is None else _f32(weight)
    out = np.empty_like(v)
    lib().orc_rms_norm(_ptr(v), v.size, _ptr(w), float(epsilon), int(bool(offset)), _ptr(out))
    return out


def make_options(head_count, head_dim, kv_head_count=None, rope_theta=0.0, rotary_dim=None, rope_freq_dim=0,
                 rope_pair_count=None, rope_scaling=None, sliding_window=0, attn_scale=None, q_norm_weight=None,
                 k_norm_weight=None, rms_epsilon=1e-6, offset_rms_norm=False, query_only=False, write_cache=True,
                 v_norm=False):
    """Options with causalAttention's defaults (math.ts:180-203). Returns (struct, keepalive)."""
    o = AttnOptions()
    o.head_count = head_count
    o.kv_head_count = kv_head_count or head_count
    o.head_dim = head_dim
    o.rotary_dim = head_dim if rotary_dim is None else rotary_dim
    o.rope_freq_dim = rope_freq_dim or 0
    o.rope_pair_count = -1 if rope_pair_count is None else rope_pair_count
    o.rope_theta = rope_theta or 0.0
    o.scaling = make_scaling(rope_scaling)
    o.sliding_window = sliding_window or 0
    if attn_scale is not None:
        o.has_attn_scale = 1
        o.attn_scale = attn_scale
    keep = []
    if q_norm_weight is not None:
        qn = _f32(q_norm_weight)
        keep.append(qn)
        o.q_norm_weight = qn.ctypes.data
    if k_norm_weight is not None:
        kn = _f32(k_norm_weight)
        keep.append(kn)
        o.k_norm_weight = kn.ctypes.data
    o.rms_epsilon = rms_epsilon
    o.offset_rms_norm = int(bool(offset_rms_norm))
    o.query_only = int(bool(query_only))
    o.write_cache = int(bool(write_cache))
    o.v_norm = int(bool(v_norm))
    return o, keep


def causal_attention(qkv, position, key_cache, value_cache, gate=None, **opts):
    """causalAttention (math.ts:179-276). key_cache/value_cache: float32 [max_tokens, Hk*D], updated in place."""
    o, keep = make_options(**opts)
    q = _f32(qkv)
    g = None if gate is None else _f32(gate)
    assert key_cache.dtype == np.float32 and key_cache.flags.c_contiguous
    assert value_cache.dtype == np.float32 and value_cache.flags.c_contiguous
    out = np.zeros(o.head_count * o.head_dim, dtype=np.float32)
    _check(lib().orc_causal_attention(_ptr(q), int(position), _ptr(key_cache), _ptr(value_cache), ctypes.byref(o),
                                      _ptr(g), _ptr(out)))
    return out


def decode_batch(qkv, positions, key_cache, value_cache, gate=None, threads=1, **opts):
    """One decode step for B sequences. qkv [B, (Hq+2Hk)*D]; caches [B, max_tokens, Hk*D] float32 (in place)."""
    o, keep = make_options(**opts)
    q = _f32(qkv)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    g = None if gate is None else _f32(gate)
    B, T = key_cache.shape[0], key_cache.shape[1]
    out = np.zeros((B, o.head_count * o.head_dim), dtype=np.float32)
    _check(lib().orc_decode_batch(_ptr(q), _ptr(pos), B, T, _ptr(key_cache), _ptr(value_cache), ctypes.byref(o),
                                  _ptr(g), _ptr(out), int(threads)))
    return out


def prefill(qkv, start_pos, key_cache, value_cache, gate=None, threads=1, **opts):
    """Prefill as the reference's token-by-token replay. qkv [B, S, (Hq+2Hk)*D];
    gate None or [B, S, Hq*D]; caches [B, max_tokens, Hk*D] float32 (in place)."""
    o, keep = make_options(**opts)
    q = _f32(qkv)
    B, S = q.shape[0], q.shape[1]
    sp = np.ascontiguousarray(start_pos, dtype=np.int32)
    g = None if gate is None else _f32(gate)
    assert key_cache.dtype == np.float32 and key_cache.flags.c_contiguous
    assert value_cache.dtype == np.float32 and value_cache.flags.c_contiguous
    out = np.zeros((B, S, o.head_count * o.head_dim), dtype=np.float32)
    _check(lib().orc_prefill(_ptr(q), _ptr(sp), _ptr(g), B, S, key_cache.shape[1], _ptr(key_cache),
                             _ptr(value_cache), ctypes.byref(o), _ptr(out), int(threads)))
    return out


def attend_heads(q_rot, positions, key_cache, value_cache, head_begin, head_end, threads=1, **opts):
    """Attention of query heads [head_begin, head_end) over filled caches, without appending."""
    o, keep = make_options(**opts)
    q = _f32(q_rot)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    B, T = key_cache.shape[0], key_cache.shape[1]
    out = np.zeros((B, o.head_count * o.head_dim), dtype=np.float32)
    _check(lib().orc_attend_heads(_ptr(q), _ptr(pos), B, T, _ptr(key_cache), _ptr(value_cache), ctypes.byref(o),
                                  int(head_begin), int(head_end), _ptr(out), int(threads)))
    return out


def linear(x, weight, bias=None, threads=1):
    """linear (math.ts:6-25): x [..., in] @ weight [in, out] + bias, double sums, float32 result."""
    x = _f32(x)
    w = _f32(weight)
    b = None if bias is None else _f32(bias)
    lead = x.shape[:-1]
    rows = int(np.prod(lead)) if lead else 1
    out = np.zeros((rows, w.shape[1]), dtype=np.float32)
    _check(lib().orc_linear(_ptr(x), rows, _ptr(w), _ptr(b), w.shape[0], w.shape[1], _ptr(out), int(threads)))
    return out.reshape(*lead, w.shape[1])


def fill_sin(n, seed):
    """fillSin (packages/three-llm/src/test/helpers.ts:13-16), float32."""
    i = np.arange(n, dtype=np.float64)
    return (np.sin(seed + i * 0.17) * 0.35).astype(np.float32)


def cpu_count():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
