"""Multi-GPU partitioning of the attention path (one process per GPU).

The reference runs one sequence on one device (packages/three-llm/src/runtime/
generate.ts:240-298); these plans split the work only where it splits without
an exchange, plus the one place that needs one:

- head_shard: rank r owns KV heads [r*Hk/N, (r+1)*Hk/N) and their query
  groups (the contiguous GQA mapping floor(h*Hk/Hq), TSLAttention.ts:340), so
  its layer is just a smaller layer and its output stays head-sharded for a
  tensor-parallel output projection. No collective.
- sequence_shard: rank r owns the contiguous token block
  [r*T/N, (r+1)*T/N); every rank emits (m, l, o) per query head with
  tla_decode_partial and one all-gather of those triples feeds tla_combine_lse.
"""
from dataclasses import dataclass

import torch

from .attention import CUDAAttention, combine_lse


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


class SequenceShardedDecode:
    """One layer of long-context decode sharded by token blocks.

    step(): tla_decode_partial on this rank's block -> all-gather of the
    (m, l, o) triples over the process group -> tla_combine_lse. Every rank
    ends with the full output [B, Hq*D] (fp16). All ranks take the same
    collective steps in the same order.
    """

    def __init__(self, head_count, kv_head_count, head_dim, total_tokens, rank, world, options=None, batch=1,
                 group=None):
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

    def step(self, qkv, positions, stream=None):
        """qkv [B, (Hq+2Hk)*D] fp16 (identical on every rank); positions int32 [B] (global)."""
        s = self.shard
        local = s.tokens + (1 if s.owns_next else 0)
        self.layer.decode_partial(qkv, positions, s.slot_offset, local, s.owns_next, partial=self.partial,
                                  stream=stream)
        if self.world > 1:
            torch.distributed.all_gather_into_tensor(self.gathered.view(-1), self.partial.view(-1), group=self.group)
            parts = self.gathered
        else:
            parts = self.partial.unsqueeze(0)
        return combine_lse(parts, out=self.out, stream=stream)
