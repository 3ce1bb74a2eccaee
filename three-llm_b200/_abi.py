"""ctypes binding of libtla.so (include/tla_api.h).

This is the same binding a three-llm host would write over the C ABI (an
N-API addon in a Node host does the same in C++). There is no CPU fallback:
loading fails loudly if the CUDA library has not been built.
"""
import ctypes
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
# TLA_LIBRARY selects another build of the same library (e.g. a tuning variant).
LIB_PATH = Path(os.environ.get("TLA_LIBRARY", HERE / "libtla.so"))

TLA_OK = 0
STATUS = {
    0: "TLA_OK", -1: "TLA_ERR_INVALID_ARG", -2: "TLA_ERR_ROPE_DIM", -3: "TLA_ERR_ROPE_THETA",
    -4: "TLA_ERR_ROPE_FACTOR", -5: "TLA_ERR_YARN_RANGE", -6: "TLA_ERR_YARN_FACTOR", -7: "TLA_ERR_LLAMA3_RANGE",
    -8: "TLA_ERR_ROTARY_DIM", -9: "TLA_ERR_UNSUPPORTED", -10: "TLA_ERR_CUDA", -11: "TLA_ERR_OUT_OF_MEMORY",
    -12: "TLA_ERR_POSITION", -13: "TLA_ERR_TIMEOUT", -14: "TLA_ERR_NO_DEVICE", -15: "TLA_ERR_SHARED",
    -16: "TLA_ERR_SCRATCH_LIMIT", -17: "TLA_ERR_BOUNDS",
}
ROPE_TYPES = {"default": 0, "none": 0, "linear": 1, "yarn": 2, "llama3": 3}
FLAG_OFFSET_RMS_NORM = 1 << 0
FLAG_V_NORM = 1 << 1
FLAG_IO_FP32 = 1 << 2
FLAG_CACHE_FP32 = 1 << 3

EXPORTS = [
    "tla_status_string", "tla_create", "tla_destroy", "tla_get_error", "tla_rope_parameters", "tla_layer_create",
    "tla_layer_share_cache", "tla_layer_destroy", "tla_layer_cache_view", "tla_decode", "tla_prefill",
    "tla_decode_partial", "tla_combine_lse", "tla_cache_reset", "tla_cache_read", "tla_cache_write",
    "tla_decode_noalloc", "tla_exchange_create", "tla_exchange_connect", "tla_exchange_combine",
    "tla_exchange_buffer", "tla_exchange_connect_buffers", "tla_exchange_destroy", "tla_decode_exchange",
    "tla_query", "tla_scores", "tla_qkv_decode", "tla_qkv_prefill", "tla_out_proj", "tla_out_proj_allreduce",
]


class TlaError(RuntimeError):
    def __init__(self, code, what=""):
        self.code = code
        msg = lib().tla_status_string(code).decode() if _lib is not None else STATUS.get(code, str(code))
        super().__init__(f"{what}: {STATUS.get(code, code)} ({msg})" if what else f"{STATUS.get(code, code)} ({msg})")


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


class AttnConfig(ctypes.Structure):
    _fields_ = [
        ("head_count", ctypes.c_int32),
        ("kv_head_count", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("max_batch", ctypes.c_int32),
        ("rotary_dim", ctypes.c_int32),
        ("rope_freq_dim", ctypes.c_int32),
        ("rope_pair_count", ctypes.c_int32),
        ("rope_theta", ctypes.c_double),
        ("rope_scaling", RopeScaling),
        ("sliding_window", ctypes.c_int32),
        ("has_attn_scale", ctypes.c_int32),
        ("attn_scale", ctypes.c_double),
        ("rms_epsilon", ctypes.c_double),
        ("flags", ctypes.c_uint32),
    ]


class CacheView(ctypes.Structure):
    _fields_ = [
        ("key", ctypes.c_void_p),
        ("value", ctypes.c_void_p),
        ("seq_stride", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("token_stride", ctypes.c_int64),
        ("elem_bytes", ctypes.c_int32),
    ]


_lib = None


def lib():
    """Load libtla.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C three-llm_b200/csrc` "
                              "(this package has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        P, i32, u32, f64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_double
        L.tla_status_string.restype = ctypes.c_char_p
        L.tla_status_string.argtypes = [ctypes.c_int]
        L.tla_create.argtypes = [ctypes.c_int, ctypes.POINTER(P)]
        L.tla_destroy.argtypes = [P]
        L.tla_get_error.argtypes = [P, ctypes.c_int]
        L.tla_rope_parameters.argtypes = [i32, f64, P, P, P]
        L.tla_layer_create.argtypes = [P, ctypes.POINTER(AttnConfig), P, P, ctypes.POINTER(P)]
        L.tla_layer_share_cache.argtypes = [P, P]
        L.tla_layer_destroy.argtypes = [P]
        L.tla_layer_cache_view.argtypes = [P, ctypes.POINTER(CacheView)]
        L.tla_decode.argtypes = [P, P, P, P, P, i32, P]
        L.tla_prefill.argtypes = [P, P, P, P, i32, P, i32, P]
        L.tla_query.argtypes = [P, P, P, P, i32, P]
        L.tla_scores.argtypes = [P, P, P, P, i32, P]
        L.tla_qkv_decode.argtypes = [P, P, P, P, i32, P, P, P, i32, P]
        L.tla_qkv_prefill.argtypes = [P, P, P, P, i32, P, P, i32, P, i32, P]
        L.tla_out_proj.argtypes = [P, P, P, P, P, P, i32, i32, i32, u32, P]
        L.tla_out_proj_allreduce.argtypes = [P, P, P, P, P, P, i32, i32, i32, u32, P]
        L.tla_decode_partial.argtypes = [P, P, P, i32, i32, i32, P, i32, P]
        L.tla_combine_lse.argtypes = [P, i32, i32, i32, i32, P, P, u32, P]
        L.tla_cache_reset.argtypes = [P, P]
        L.tla_cache_read.argtypes = [P, i32, i32, i32, P, P]
        L.tla_cache_write.argtypes = [P, i32, i32, i32, P, P]
        L.tla_exchange_create.argtypes = [P, i32, i32, ctypes.c_size_t, ctypes.POINTER(P), P]
        L.tla_exchange_connect.argtypes = [P, P]
        L.tla_exchange_combine.argtypes = [P, P, i32, i32, i32, P, P, u32, P]
        L.tla_exchange_buffer.argtypes = [P, ctypes.POINTER(P)]
        L.tla_exchange_connect_buffers.argtypes = [P, P]
        L.tla_exchange_destroy.argtypes = [P]
        L.tla_decode_exchange.argtypes = [P, P, P, P, i32, i32, i32, P, P, P, i32, P]
        L.tla_decode_noalloc.argtypes = [ctypes.POINTER(AttnConfig), P, P, P, P, P, P, P, P, P, i32, P]
        for name in EXPORTS:
            if name != "tla_status_string":
                getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def check(rc, what=""):
    if rc != TLA_OK:
        raise TlaError(rc, what)
    return rc


def make_scaling(spec):
    s = RopeScaling()
    if not spec:
        return s
    s.type = ROPE_TYPES[spec.get("type", "yarn")]
    s.factor = float(spec.get("factor", 1.0))
    s.original_context_length = float(spec.get("original_context_length", spec.get("originalContextLength",
                                                                                   float("nan"))))
    s.beta_fast = float(spec.get("beta_fast", spec.get("betaFast", float("nan"))))
    s.beta_slow = float(spec.get("beta_slow", spec.get("betaSlow", float("nan"))))
    af = spec.get("attention_factor", spec.get("attentionFactor"))
    if af is not None:
        s.has_attention_factor = 1
        s.attention_factor = float(af)
    s.low_freq_factor = float(spec.get("low_freq_factor", spec.get("lowFreqFactor", float("nan"))))
    s.high_freq_factor = float(spec.get("high_freq_factor", spec.get("highFreqFactor", float("nan"))))
    return s
