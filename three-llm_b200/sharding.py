"""Multi-GPU partitioning of the attention path (one process per GPU).

The reference runs one sequence on one device (packages/three-llm/src/runtime/
generate.ts:240-298); these plans split the work only where it splits without
an exchange, plus the one place that needs one:

- head_shard: rank r owns KV heads [r*Hk/N, (r+1)*Hk/N) and their query
  groups (the contiguous GQA mapping floor(h*Hk/Hq), TSLAttention.ts:340), so
  its layer is just a smaller layer and its output stays head-sharded for a
  tensor-parallel output projection. No collective.
- batch_head_shard: (sequence, KV-head group) units for batched prefill and
  decode when there are more ranks than KV-head groups: KV-head part times
  sequence part, again without a collective.
- sequence_shard: rank r owns the contiguous token block
  [r*T/N, (r+1)*T/N); every rank emits (m, l, o) per query head with
  tla_decode_partial, and the triples meet either through one all-gather of
  the process group followed by tla_combine_lse ("nccl"), or through
  PeerExchange ("p2p"): one kernel that stores them into every peer's buffer
  over NVLink, waits for the peers' triples and merges them.
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _abi
from ._abi import check, lib
from .attention import Context, CUDAAttention, _ptr, _stream, combine_lse

IPC_HANDLE_BYTES = 64


@dataclass(frozen=True)
class HeadShard:
    q_begin: int
    q_count: int
    kv_begin: int
    kv_count: int


def head_shard(head_count, kv_head_count, world, rank):
    """KV-head-group shard of rank `rank` out of `world` (kv_head_count % world == 0)."""
    if kv_head_count % world or head_count % kv_head_count:
        raise ValueError("kv heads must divide evenly across ranks and query heads across kv heads")
    group = head_count // kv_head_count
    kv = kv_head_count // world
    return HeadShard(rank * kv * group, kv * group, rank * kv, kv)


def slice_qkv_for_heads(qkv, shard, head_count, kv_head_count, head_dim):
    """Rows [B, (Hq+2Hk)*D] -> this shard's packed [Q_r | K_r | V_r] rows (a copy)."""
    B = qkv.shape[0]
    x = qkv.view(B, head_count + 2 * kv_head_count, head_dim)
    q = x[:, shard.q_begin:shard.q_begin + shard.q_count]
    k = x[:, head_count + shard.kv_begin:head_count + shard.kv_begin + shard.kv_count]
    v = x[:, head_count + kv_head_count + shard.kv_begin:head_count + kv_head_count + shard.kv_begin + shard.kv_count]
    return torch.cat([q, k, v], dim=1).reshape(B, -1).contiguous()


@dataclass(frozen=True)
class BatchHeadShard:
    seq_begin: int
    seq_count: int
    q_begin: int
    q_count: int
    kv_begin: int
    kv_count: int


def batch_head_shard(batch, head_count, kv_head_count, world, rank):
    """Batched prefill / decode split over (sequence, KV-head group) units: the
    KV heads are split over g = gcd(world, kv_head_count) rank groups and the
    sequences over world / g, so rank r holds KV-head part r % g of sequences
    part r // g (batch must divide by world / g). No exchange: every unit is a
    smaller layer over its own sequences."""
    import math

    g = math.gcd(world, kv_head_count)
    nb = world // g
    if batch % nb or head_count % kv_head_count:
        raise ValueError("the sequences must divide evenly over world / gcd(world, kv_head_count) ranks")
    h = head_shard(head_count, kv_head_count, g, rank % g)
    per = batch // nb
    return BatchHeadShard((rank // g) * per, per, h.q_begin, h.q_count, h.kv_begin, h.kv_count)


@dataclass(frozen=True)
class SequenceShard:
    slot_offset: int   # global position of local slot 0
    tokens: int        # cached tokens held by this rank
    owns_next: bool    # whether the next decoded token is appended here


def sequence_shard(total_tokens, world, rank):
    """Contiguous token block of rank `rank` for a cache of `total_tokens` cached tokens;
    the last rank also owns the slot of the next token."""
    begin = rank * total_tokens // world
    end = (rank + 1) * total_tokens // world
    return SequenceShard(begin, end - begin, rank == world - 1)


class PeerExchange:
    """tla_exchange_*: gather + log-sum-exp merge of sequence-shard triples over peer memory.

    Every rank of `group` constructs one with the same `slot_bytes` (the
    byte size of one rank's [B, Hq, D+2] float32 triples); the IPC handles of
    the ranks' buffers travel once through the process group. combine() is one
    kernel launch per call, stream-ordered and graph-capturable; a peer that
    never arrives ends the wait after about two seconds with TLA_ERR_TIMEOUT
    on the context's error word.
    """

    def __init__(self, rank, world, slot_bytes, device=None, group=None, context=None):
        if device is None:
            device = torch.cuda.current_device()
        elif isinstance(device, torch.device):
            device = device.index or 0
        self.context = context or Context.default(device)
        self.rank, self.world = rank, world
        h = ctypes.c_void_p()
        handle = (ctypes.c_char * IPC_HANDLE_BYTES)()
        check(lib().tla_exchange_create(self.context.handle, rank, world, slot_bytes, ctypes.byref(h), handle),
              "tla_exchange_create")
        self.handle = h
        if group is not False and world > 1:
            handles = [None] * world
            torch.distributed.all_gather_object(handles, bytes(handle), group=group)
            blob = b"".join(handles)
            check(lib().tla_exchange_connect(self.handle, ctypes.c_char_p(blob)), "tla_exchange_connect")

    def buffer(self):
        p = ctypes.c_void_p()
        check(lib().tla_exchange_buffer(self.handle, ctypes.byref(p)), "tla_exchange_buffer")
        return p.value

    def connect_buffers(self, buffers):
        """Connect with device pointers of every rank's buffer (ranks that share one process)."""
        arr = (ctypes.c_void_p * len(buffers))(*buffers)
        check(lib().tla_exchange_connect_buffers(self.handle, arr), "tla_exchange_connect_buffers")

    def combine(self, partial, out, gate=None, stream=None):
        """partial [B, Hq, D+2] float32 -> out [B, Hq*D] (float16 or float32), merged over all ranks."""
        B, H, D2 = partial.shape
        flags = _abi.FLAG_IO_FP32 if out.dtype == torch.float32 else 0
        check(lib().tla_exchange_combine(self.handle, _ptr(partial), B, H, D2 - 2, _ptr(gate), _ptr(out), flags,
                                         _stream(stream)), "tla_exchange_combine")
        return out

    def close(self):
        if self.handle:
            lib().tla_exchange_destroy(self.handle)
            self.handle = None


class SequenceShardedDecode:
    """One layer of long-context decode sharded by token blocks.

    step(): exchange="nccl" runs tla_decode_partial on this rank's block,
    all-gathers the (m, l, o) triples over the process group and merges them
    with tla_combine_lse; exchange="p2p" runs tla_decode_exchange (the
    split-KV kernel, then one kernel that merges each row's segments, stores
    the row's triple into every rank's PeerExchange buffer over NVLink, waits
    for the peers' triples and merges). Every rank ends with the full output
    [B, Hq*D] (fp16). All ranks take the same steps in the same order.
    """

    def __init__(self, head_count, kv_head_count, head_dim, total_tokens, rank, world, options=None, batch=1,
                 group=None, exchange="nccl", peer_exchange=None):
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.shard = sequence_shard(total_tokens, world, rank)
        self.world, self.rank, self.group = world, rank, group
        self.capacity = self.shard.tokens + (1 if self.shard.owns_next else 0)
        opts = {"headDim": head_dim, "kvHeadCount": kv_head_count, "maxBatch": batch, "dtype": torch.float16}
        opts.update(options or {})
        self.layer = CUDAAttention(None, head_count * head_dim, head_count, max(self.capacity, 1), opts)
        self.Hq, self.D, self.B = head_count, head_dim, batch
        dev = self.layer.device
        self.partial = torch.empty(batch, head_count, head_dim + 2, dtype=torch.float32, device=dev)
        self.gathered = torch.empty(world, batch, head_count, head_dim + 2, dtype=torch.float32, device=dev)
        self.out = torch.empty(batch, head_count * head_dim, dtype=torch.float16, device=dev)
        self.exchange = None
        self.owns_exchange = False
        if exchange == "p2p" and world > 1:
            # one PeerExchange can serve every layer of a model (same triple size)
            self.exchange = peer_exchange or PeerExchange(rank, world, self.partial.numel() * 4, dev, group,
                                                          self.layer.context)
            self.owns_exchange = peer_exchange is None

    def step(self, qkv, positions, stream=None):
        """qkv [B, (Hq+2Hk)*D] fp16 (identical on every rank); positions int32 [B] (global)."""
        if self.world == 1:  # one shard holds the whole sequence: a plain decode step
            return self.layer.decode(qkv.view(self.B, -1), positions, out=self.out, stream=stream)
        s = self.shard
        local = s.tokens + (1 if s.owns_next else 0)
        if self.exchange is not None:  # split-KV decode + segment merge + NVLink exchange + merge: two kernels
            self.layer._check_io(qkv, "qkv")
            check(lib().tla_decode_exchange(self.layer.handle, self.exchange.handle, _ptr(qkv), _ptr(positions),
                                            s.slot_offset, local, 1 if s.owns_next else 0, _ptr(self.partial),
                                            None, _ptr(self.out), self.B, _stream(stream)), "tla_decode_exchange")
            return self.out
        self.layer.decode_partial(qkv, positions, s.slot_offset, local, s.owns_next, partial=self.partial,
                                  stream=stream)
        if self.world > 1:
            torch.distributed.all_gather_into_tensor(self.gathered.view(-1), self.partial.view(-1), group=self.group)
            parts = self.gathered
        else:
            parts = self.partial.unsqueeze(0)
        return combine_lse(parts, out=self.out, stream=stream)

    def close(self):
        if self.owns_exchange and self.exchange is not None:
            self.exchange.close()
        self.exchange = None
        self.layer.close()


class HeadShardedOutProj:
    """Output projection + residual after head-sharded attention
    (DecoderTSLRunner.ts:299-309: attnProj, then TSLAdd), across the ranks:
    tla_out_proj_allreduce multiplies this rank's attention columns by its rows
    of W on the tensor cores, the GEMM epilogue stores each partial tile over
    NVLink into the exchange buffer of the rank owning those hidden columns,
    and one kernel sums each owned block, adds bias + residual and sends it to
    every rank. Every rank ends with the full y [rows, hidden]."""

    def __init__(self, rows, hidden, rank, world, device=None, group=None, context=None, exchange=None):
        if hidden % (64 * world):
            raise ValueError("hidden must be a multiple of 64 * world")
        self.rows, self.hidden = rows, hidden
        slot = 2 * rows * (hidden // world) * 4
        self.owns = exchange is None
        self.exchange = exchange or PeerExchange(rank, world, slot, device, group, context)

    def __call__(self, attn, weight, bias=None, residual=None, out=None, stream=None):
        """attn [rows, in_r] fp16 (this rank's heads), weight [in_r, hidden] fp16 (its rows of W)."""
        rows, fin = attn.shape
        f32 = residual is not None and residual.dtype == torch.float32
        if out is None:
            out = torch.empty(rows, self.hidden, dtype=torch.float32 if f32 else torch.float16, device=attn.device)
        check(lib().tla_out_proj_allreduce(self.exchange.handle, _ptr(attn), _ptr(weight), _ptr(bias),
                                           _ptr(residual), _ptr(out), rows, fin, self.hidden,
                                           _abi.FLAG_IO_FP32 if out.dtype == torch.float32 else 0, _stream(stream)),
              "tla_out_proj_allreduce")
        return out

    def close(self):
        if self.owns and self.exchange is not None:
            self.exchange.close()
        self.exchange = None

