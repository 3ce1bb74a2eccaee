"""Host-side mirror of three-llm's attention operator over the C ABI.

`CUDAAttention` keeps the constructor, options and members of the reference's
`TSLAttention` (packages/three-llm/src/tsl/TSLAttention.ts:19-448) so code
written against that operator reads the same; the four WebGPU dispatches per
step become one `tla_decode` call on the layer's CUDA stream. Device memory
comes from PyTorch tensors; the kernels live in libtla.so.
"""
import ctypes
import math

import numpy as np
import torch

from . import _abi
from ._abi import check, lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class Context:
    """One tla_ctx per device (owns the error word and split-KV scratch)."""

    _default = {}

    def __init__(self, device=0):
        self.device = int(device)
        h = ctypes.c_void_p()
        check(lib().tla_create(self.device, ctypes.byref(h)), "tla_create")
        self.handle = h

    @classmethod
    def default(cls, device=0):
        device = int(device)
        if device not in cls._default:
            cls._default[device] = Context(device)
        return cls._default[device]

    def error(self, reset=True):
        """Device-reported status since the last reset (0 = none); synchronises."""
        return lib().tla_get_error(self.handle, 1 if reset else 0)

    def close(self):
        if self.handle:
            lib().tla_destroy(self.handle)
            self.handle = None


def rope_parameters(dim, theta, scaling=None):
    """ropeParameters (packages/three-llm/src/runtime/rope.ts:4-52) through the C ABI."""
    inv = np.zeros(max(dim // 2, 1), dtype=np.float32)
    af = ctypes.c_double(0)
    s = _abi.make_scaling(scaling)
    check(lib().tla_rope_parameters(int(dim), float(theta), ctypes.byref(s),
                                    inv.ctypes.data_as(ctypes.c_void_p), ctypes.byref(af)), "ropeParameters")
    return inv[: dim // 2], af.value


class CUDAAttention:
    """Drop-in for TSLAttention: `new TSLAttention(qkvNode, hiddenSize, headCount, maxTokens, options)`.

    qkv_node: CUDA tensor holding packed [Q | K | V] for one token
    ([headCount + 2*kvHeadCount] * headDim elements, float16 or float32).
    options: the AttentionKernelOptions keys (types.ts:288-312): headDim,
    kvHeadCount, ropeTheta, rotaryDim, ropeFreqDim, ropePairCount, yarn,
    ropeScaling, slidingWindow, attnScale, rmsEpsilon, offsetRMSNorm, vNorm,
    qNormWeight, kNormWeight, positionNode, gateNode, sharedAttention; plus
    `cacheDtype` ('float16' default, or 'float32') and `maxBatch`.
    """

    def __init__(self, qkv_node, hidden_size, head_count, max_tokens, options=None, context=None):
        o = dict(options or {})
        self.qkvNode = qkv_node
        self.hiddenSize = hidden_size
        self.headCount = head_count
        self.headDim = o.get("headDim") or hidden_size // head_count          # TSLAttention.ts:74
        self.kvHeadCount = o.get("kvHeadCount") or head_count                  # :75
        self.qSize = self.headCount * self.headDim
        self.kvSize = self.kvHeadCount * self.headDim
        self.maxTokens = max_tokens
        self.maxBatch = int(o.get("maxBatch", 1))
        self.ropeTheta = o.get("ropeTheta") or 0                               # :80
        self.rotaryDim = o["rotaryDim"] if o.get("rotaryDim") is not None else self.headDim   # :81
        self.ropeFreqDim = o.get("ropeFreqDim") or self.rotaryDim              # :82
        self.ropePairCount = (o["ropePairCount"] if o.get("ropePairCount") is not None
                              else self.rotaryDim // 2)                        # :83
        self.slidingWindow = o.get("slidingWindow") or 0                       # :94
        self.attnScale = o["attnScale"] if o.get("attnScale") is not None else 1 / math.sqrt(self.headDim)
        self.rmsEpsilon = o.get("rmsEpsilon") or 1e-6                          # :96
        self.offsetRMSNorm = o.get("offsetRMSNorm") is True
        self.vNorm = o.get("vNorm") is True
        self.gateNode = o.get("gateNode")
        self.positionNode = o.get("positionNode")
        self.sharedKV = o.get("sharedAttention") is not None
        dtype = qkv_node.dtype if qkv_node is not None else o.get("dtype", torch.float16)
        if dtype not in (torch.float16, torch.float32):
            raise TypeError("qkv must be float16 or float32")
        self.dtype = dtype
        self.device = qkv_node.device if qkv_node is not None else torch.device("cuda", torch.cuda.current_device())
        self.context = context or Context.default(self.device.index or 0)
        scaling = o.get("ropeScaling") or o.get("yarn")
        if scaling is not None and o.get("ropeScaling") is None and "type" not in scaling:
            scaling = dict(scaling, type="yarn")
        cfg = _abi.AttnConfig()
        cfg.head_count = self.headCount
        cfg.kv_head_count = self.kvHeadCount
        cfg.head_dim = self.headDim
        cfg.max_tokens = max_tokens
        cfg.max_batch = self.maxBatch
        cfg.rotary_dim = self.rotaryDim
        cfg.rope_freq_dim = self.ropeFreqDim
        cfg.rope_pair_count = self.ropePairCount
        cfg.rope_theta = float(self.ropeTheta)
        cfg.rope_scaling = _abi.make_scaling(scaling)
        cfg.sliding_window = self.slidingWindow
        cfg.has_attn_scale = 1
        cfg.attn_scale = float(self.attnScale)
        cfg.rms_epsilon = float(self.rmsEpsilon)
        flags = 0
        if self.offsetRMSNorm:
            flags |= _abi.FLAG_OFFSET_RMS_NORM
        if self.vNorm:
            flags |= _abi.FLAG_V_NORM
        if dtype == torch.float32:
            flags |= _abi.FLAG_IO_FP32
        if o.get("cacheDtype", "float16") in ("float32", torch.float32):
            flags |= _abi.FLAG_CACHE_FP32
        cfg.flags = flags
        self._qn = None if o.get("qNormWeight") is None else np.ascontiguousarray(o["qNormWeight"], np.float32)
        self._kn = None if o.get("kNormWeight") is None else np.ascontiguousarray(o["kNormWeight"], np.float32)
        h = ctypes.c_void_p()
        check(lib().tla_layer_create(self.context.handle, ctypes.byref(cfg),
                                     None if self._qn is None else self._qn.ctypes.data_as(ctypes.c_void_p),
                                     None if self._kn is None else self._kn.ctypes.data_as(ctypes.c_void_p),
                                     ctypes.byref(h)), "TSLAttention constructor")
        self.handle = h
        if self.sharedKV:
            check(lib().tla_layer_share_cache(h, o["sharedAttention"].handle), "sharedAttention")
        self.qNormAttribute = self._qn
        self.kNormAttribute = self._kn
        self.outputNode = torch.empty(self.qSize, dtype=dtype, device=self.device)
        self.outputAttribute = self.outputNode
        self._position = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._last_position = None   # the position tensor of the last compute()
        self._score_buf = None       # scoreAttribute's buffer, created on first read
        self.computeNodes = [self]   # one fused launch (orderedComputeNodes keeps working)
        self.computeNode = self

    # ---- TSLAttention members
    def setPosition(self, position):
        """setPosition (TSLAttention.ts:430-432): a no-op when positionNode drives the position."""
        if self.positionNode is None:
            self._position.fill_(int(position))

    def compute(self, *args, stream=None):
        """compute(renderer, position) / compute(position) (TSLAttention.ts:443-447)."""
        position = args[-1] if args else None
        if position is not None:
            self.setPosition(position)
        pos = self.positionNode if self.positionNode is not None else self._position
        self.decode(self.qkvNode.view(1, -1), pos, gate=None if self.gateNode is None else self.gateNode.view(1, -1),
                    out=self.outputNode.view(1, -1), stream=stream)
        self._last_position = pos
        return self.outputNode

    def _step_inputs(self):
        if self._last_position is None:
            raise RuntimeError("compute() has not run yet")
        return self.qkvNode.view(1, -1), self._last_position.view(1)

    @property
    def queryAttribute(self):
        """queryAttribute (TSLAttention.ts:53): the last compute() step's rotated
        queries, float32 [Hq * headDim], formed by tla_query from the qkv node and
        position that step used (QK-norm, then RoPE, as the decode forms them)."""
        qkv, pos = self._step_inputs()
        return self.query(qkv, pos)[0].cpu().numpy()

    @property
    def scoreAttribute(self):
        """scoreAttribute (TSLAttention.ts:52): float32 [Hq * maxTokens] with the
        last compute() step's scaled scores at the slots of its window
        [start, position] of sequence 0 (tla_scores over the cache, new token
        included); other slots keep what earlier reads left (zero at first), as
        the reference's score buffer does."""
        qkv, pos = self._step_inputs()
        if self._score_buf is None:
            self._score_buf = torch.zeros(1, self.headCount, self.maxTokens, dtype=torch.float32, device=self.device)
        self.scores(self.query(qkv, pos), pos, out=self._score_buf)
        return self._score_buf.view(-1).cpu().numpy()

    def reset(self, stream=None):
        """reset() (TSLAttention.ts:434-441)."""
        check(lib().tla_cache_reset(self.handle, _stream(stream)), "reset")

    def _cache(self, which, seq=0, begin=0, count=None):
        count = self.maxTokens - begin if count is None else count
        buf = np.zeros(count * self.kvSize, dtype=np.float32)
        p = buf.ctypes.data_as(ctypes.c_void_p)
        check(lib().tla_cache_read(self.handle, seq, begin, count, p if which == 0 else None,
                                   p if which == 1 else None), "cache read")
        return buf

    @property
    def keyCacheAttribute(self):
        """Token-major float32 view [maxTokens * kvSize] of sequence 0's keys (post-RoPE)."""
        return self._cache(0)

    @property
    def valueCacheAttribute(self):
        return self._cache(1)

    def read_cache(self, seq, begin, count):
        """(keys, values) float32 [count, kvHeadCount*headDim] of one sequence."""
        k = self._cache(0, seq, begin, count).reshape(count, self.kvSize)
        v = self._cache(1, seq, begin, count).reshape(count, self.kvSize)
        return k, v

    def write_cache(self, seq, begin, keys, values):
        k = np.ascontiguousarray(keys, np.float32)
        v = np.ascontiguousarray(values, np.float32)
        count = k.shape[0]
        check(lib().tla_cache_write(self.handle, seq, begin, count, k.ctypes.data_as(ctypes.c_void_p),
                                    v.ctypes.data_as(ctypes.c_void_p)), "cache write")

    def cache_view(self):
        v = _abi.CacheView()
        check(lib().tla_layer_cache_view(self.handle, ctypes.byref(v)))
        return v

    # ---- batched entry points
    def _check_io(self, t, name):
        if t is None:
            return
        if t.dtype != self.dtype or not t.is_cuda or not t.is_contiguous():
            raise TypeError(f"{name} must be a contiguous CUDA {self.dtype} tensor")

    def decode(self, qkv, positions, gate=None, out=None, stream=None):
        """One decode step for B sequences: qkv [B, (Hq+2Hk)*D], positions int32 [B] on the device."""
        B = qkv.shape[0]
        self._check_io(qkv, "qkv")
        self._check_io(gate, "gate")
        if out is None:
            out = torch.empty(B, self.qSize, dtype=self.dtype, device=self.device)
        self._check_io(out, "out")
        if positions.dtype != torch.int32 or not positions.is_cuda:
            raise TypeError("positions must be a CUDA int32 tensor")
        check(lib().tla_decode(self.handle, _ptr(qkv), _ptr(positions), _ptr(gate), _ptr(out), B, _stream(stream)),
              "decode")
        return out

    def query(self, qkv, positions, out=None, stream=None):
        """Rotated queries of a decode step (tla_query): float32 [B, Hq*D], nothing appended."""
        B = qkv.shape[0]
        self._check_io(qkv, "qkv")
        if out is None:
            out = torch.empty(B, self.qSize, dtype=torch.float32, device=self.device)
        check(lib().tla_query(self.handle, _ptr(qkv), _ptr(positions), _ptr(out), B, _stream(stream)), "query")
        return out

    def scores(self, query, positions, out=None, stream=None):
        """Scaled scores over each sequence's window (tla_scores): float32 [B, Hq, maxTokens];
        slots outside [window start, position] keep out's previous contents (zeros if out is None)."""
        B = query.shape[0]
        if out is None:
            out = torch.zeros(B, self.headCount, self.maxTokens, dtype=torch.float32, device=self.device)
        check(lib().tla_scores(self.handle, _ptr(query.contiguous()), _ptr(positions), _ptr(out), B,
                               _stream(stream)), "scores")
        return out

    def prefill(self, qkv, start_pos, gate=None, out=None, stream=None):
        """Causal prefill: qkv [B, S, (Hq+2Hk)*D], start_pos int32 [B], gate None or
        [B, S, Hq*D] (out *= sigmoid(gate) at every position); out [B, S, Hq*D]."""
        B, S = qkv.shape[0], qkv.shape[1]
        self._check_io(qkv, "qkv")
        self._check_io(gate, "gate")
        if out is None:
            out = torch.empty(B, S, self.qSize, dtype=self.dtype, device=self.device)
        self._check_io(out, "out")
        check(lib().tla_prefill(self.handle, _ptr(qkv), _ptr(start_pos), _ptr(gate), S, _ptr(out), B,
                                _stream(stream)), "prefill")
        return out

    def decode_partial(self, qkv, positions, slot_offset, local_tokens, append, partial=None, stream=None):
        """Sequence-shard step: float32 partial triples [B, Hq, D + 2] = (m_log2, l, o)."""
        B = qkv.shape[0]
        self._check_io(qkv, "qkv")
        if partial is None:
            partial = torch.empty(B, self.headCount, self.headDim + 2, dtype=torch.float32, device=self.device)
        check(lib().tla_decode_partial(self.handle, _ptr(qkv), _ptr(positions), int(slot_offset), int(local_tokens),
                                       1 if append else 0, _ptr(partial), B, _stream(stream)), "decode_partial")
        return partial

    def close(self):
        if getattr(self, "handle", None):
            lib().tla_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def combine_lse(partials, out=None, gate=None, stream=None):
    """Merge [R, B, Hq, D+2] partial triples into [B, Hq*D] (dtype of `out`, default float16)."""
    R, B, H, D2 = partials.shape
    D = D2 - 2
    if out is None:
        out = torch.empty(B, H * D, dtype=torch.float16, device=partials.device)
    flags = _abi.FLAG_IO_FP32 if out.dtype == torch.float32 else 0
    check(lib().tla_combine_lse(_ptr(partials.contiguous()), R, B, H, D, _ptr(gate), _ptr(out), flags,
                                _stream(stream)), "combine_lse")
    return out
