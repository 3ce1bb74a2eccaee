"""Host-side multi-rank logic on CPU (gloo, world size 2; no GPU).

Covers the partition plans of three_llm_b200.sharding and the
sequence-shard protocol: every rank computes the (m, l, o) triples of its
token block, the triples are all-gathered, and the log-sum-exp merge equals
the reference attention over the whole sequence (the oracle). Also checks
that a rank that dies before the exchange makes the other rank's collective
fail within the process-group timeout instead of hanging.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle


def _sharding():
    import __graft_entry__ as ge

    ge.load_package()
    from three_llm_b200 import sharding

    return sharding


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plans_cover_every_head_and_token_once(world):
    sh = _sharding()
    Hq, Hk, T = 32, 8, 131072
    q, kv, toks = [], [], []
    for r in range(world):
        s = sh.head_shard(Hq, Hk, world, r)
        q += list(range(s.q_begin, s.q_begin + s.q_count))
        kv += list(range(s.kv_begin, s.kv_begin + s.kv_count))
        # the shard's query heads map onto its own kv heads (floor(h*Hk/Hq))
        assert {h * Hk // Hq for h in range(s.q_begin, s.q_begin + s.q_count)} == set(
            range(s.kv_begin, s.kv_begin + s.kv_count))
        t = sh.sequence_shard(T, world, r)
        toks += list(range(t.slot_offset, t.slot_offset + t.tokens))
        assert t.owns_next == (r == world - 1)
    assert q == list(range(Hq)) and kv == list(range(Hk)) and toks == list(range(T))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_batch_head_plan_covers_every_unit_once(world):
    """Config 3's (sequence, KV-head group) units: 4 sequences x 2 KV heads over 1..8 ranks."""
    sh = _sharding()
    B, Hq, Hk = 4, 14, 2
    units = []
    for r in range(world):
        s = sh.batch_head_shard(B, Hq, Hk, world, r)
        assert s.q_count == s.kv_count * Hq // Hk and s.q_begin == s.kv_begin * Hq // Hk
        units += [(b, k) for b in range(s.seq_begin, s.seq_begin + s.seq_count)
                  for k in range(s.kv_begin, s.kv_begin + s.kv_count)]
    assert sorted(units) == [(b, k) for b in range(B) for k in range(Hk)]
    assert len(units) == len(set(units))


def test_slice_qkv_for_heads():
    sh = _sharding()
    Hq, Hk, D, B = 8, 4, 3, 2
    qkv = torch.arange(B * (Hq + 2 * Hk) * D, dtype=torch.float32).view(B, -1)
    s = sh.head_shard(Hq, Hk, 2, 1)
    got = sh.slice_qkv_for_heads(qkv, s, Hq, Hk, D).view(B, -1, D)
    x = qkv.view(B, Hq + 2 * Hk, D)
    exp = torch.cat([x[:, 4:8], x[:, 10:12], x[:, 14:16]], dim=1)
    assert torch.equal(got, exp)


def partial_triples(q_rot, keys, values, scale):
    """(m in log2 units, l, unnormalised o) per query head over one token block:
    the quantities tla_decode_partial emits. q_rot [Hq, D], keys/values [n, Hk, D]."""
    Hq, D = q_rot.shape
    Hk = keys.shape[1]
    out = np.zeros((Hq, D + 2), np.float64)
    for h in range(Hq):
        kvh = h * Hk // Hq
        if keys.shape[0] == 0:
            out[h, 0], out[h, 1] = -np.inf, 0.0
            continue
        s = keys[:, kvh].astype(np.float64) @ q_rot[h].astype(np.float64) * scale * np.log2(np.e)
        m = s.max()
        p = np.exp2(s - m)
        out[h, 0], out[h, 1] = m, p.sum()
        out[h, 2:] = p @ values[:, kvh].astype(np.float64)
    return out


def combine(parts):
    """The log-sum-exp merge tla_combine_lse performs, in float64."""
    m = parts[:, :, 0]
    M = m.max(axis=0)
    w = np.exp2(m - M)
    L = (parts[:, :, 1] * w).sum(axis=0)
    O = (parts[:, :, 2:] * w[:, :, None]).sum(axis=0)
    return O / L[:, None]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, mode, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        sh = _sharding()
        rng = np.random.default_rng(0)
        Hq, Hk, D, T = 8, 2, 16, 37
        keys = rng.standard_normal((T + 1, Hk, D)).astype(np.float32)
        values = rng.standard_normal((T + 1, Hk, D)).astype(np.float32)
        qkv = rng.standard_normal((Hq + 2 * Hk) * D).astype(np.float32)
        # the reference over the whole sequence: the new token (position T) is appended
        kc = keys.reshape(T + 1, Hk * D).copy()
        vc = values.reshape(T + 1, Hk * D).copy()
        full = oracle.causal_attention(qkv, T, kc, vc, head_count=Hq, kv_head_count=Hk, head_dim=D, rope_theta=1e4)
        q_rot = np.stack([oracle.apply_rope(qkv[h * D:(h + 1) * D], 0, D, T, 1e4) for h in range(Hq)])
        keys_all = kc.reshape(T + 1, Hk, D)  # post-RoPE keys as cached by the reference
        s = sh.sequence_shard(T, world, rank)
        n = s.tokens + (1 if s.owns_next else 0)
        mine = partial_triples(q_rot, keys_all[s.slot_offset:s.slot_offset + n],
                               values[s.slot_offset:s.slot_offset + n], 1 / np.sqrt(D))
        if mode == "die" and rank == 1:
            raise SystemExit(3)  # leaves before the exchange
        buf = torch.from_numpy(mine).float().contiguous()
        gathered = torch.empty(world, *buf.shape)
        try:
            dist.all_gather_into_tensor(gathered, buf)
        except Exception as e:  # the peer is gone: the collective must fail, not hang
            np.save(result_path, np.array([-1.0]))
            raise SystemExit(0) from e
        got = combine(gathered.double().numpy())
        np.save(result_path, np.array([np.max(np.abs(got.ravel() - full))]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["ok", "die"])
def test_sequence_shard_protocol_gloo(tmp_path, mode):
    world = 2
    port = _free_port()
    path = str(tmp_path / "r0.npy")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, path if r == 0 else str(tmp_path / "r1.npy")))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    res = np.load(path)
    if mode == "ok":
        assert procs[0].exitcode == 0 and procs[1].exitcode == 0
        assert res[0] < 1e-5
    else:
        assert procs[1].exitcode == 3
        assert res[0] == -1.0  # rank 0 saw an error from its collective
