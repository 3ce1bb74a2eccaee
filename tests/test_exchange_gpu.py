"""Peer-memory exchange of sequence-shard triples (tla_exchange_*).

Single GPU: the merge arithmetic with one rank against tla_combine_lse, and the
bounded wait: rank 0 of two waits for a flag that nothing sets and must come
back with TLA_ERR_TIMEOUT while the context stays usable. Two or more GPUs: one
process per GPU, a gloo group carries only the IPC handles, and the sharded
decode (p2p exchange, eager and replayed from a CUDA graph) must equal the
oracle's decode over the whole sequence.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def _partials(cuda, B, H, D, seed):
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    p = torch.randn(B, H, D + 2, generator=g, device=cuda)
    p[..., 0] = p[..., 0] * 4.0            # running max (log2 domain)
    p[..., 1] = p[..., 1].abs() * 10 + 1   # softmax denominator
    return p


def test_exchange_one_rank_matches_combine_lse(pkg, cuda):
    from three_llm_b200 import sharding

    B, H, D = 2, 32, 128
    part = _partials(cuda, B, H, D, 1)
    ex = sharding.PeerExchange(0, 1, part.numel() * 4, cuda.index or 0, group=False)
    try:
        ex.connect_buffers([ex.buffer()])
        for dtype in (torch.float16, torch.float32):
            out = torch.empty(B, H * D, dtype=dtype, device=cuda)
            for _ in range(3):  # both buffer parities
                ex.combine(part, out)
            exp = pkg.combine_lse(part.unsqueeze(0), out=torch.empty_like(out))
            torch.cuda.synchronize()
            assert ex.context.error() == 0
            torch.testing.assert_close(out, exp, rtol=1e-3, atol=1e-3)
    finally:
        ex.close()


@pytest.mark.parametrize("D,T", [(128, 20000), (64, 3000)])
def test_decode_exchange_one_rank_equals_decode(pkg, cuda, D, T):
    """tla_decode_exchange with a single rank: the split-KV kernel, the fused
    segment merge and the exchange path must reproduce the plain decode."""
    from three_llm_b200 import _abi, sharding
    from three_llm_b200._abi import check, lib
    from three_llm_b200.attention import _ptr, _stream

    Hq, Hk = 32, 8
    g = torch.Generator(device=cuda)
    g.manual_seed(9)
    opts = {"headDim": D, "kvHeadCount": Hk, "ropeTheta": 5e5, "dtype": torch.float16}
    a = pkg.CUDAAttention(None, Hq * D, Hq, T + 1, opts)
    b = pkg.CUDAAttention(None, Hq * D, Hq, T + 1, opts)
    kv = torch.randn(T + 1, Hk * D, generator=g, device=cuda).cpu().numpy()
    vv = torch.randn(T + 1, Hk * D, generator=g, device=cuda).cpu().numpy()
    for layer in (a, b):
        layer.write_cache(0, 0, kv[:T], vv[:T])
    qkv = torch.randn(1, (Hq + 2 * Hk) * D, generator=g, device=cuda).half()
    pos = torch.tensor([T], dtype=torch.int32, device=cuda)
    exp = a.decode(qkv, pos)
    ex = sharding.PeerExchange(0, 1, Hq * (D + 2) * 4, cuda.index or 0, group=False, context=b.context)
    try:
        ex.connect_buffers([ex.buffer()])
        partial = torch.empty(1, Hq, D + 2, device=cuda)
        out = torch.empty(1, Hq * D, dtype=torch.float16, device=cuda)
        for _ in range(2):  # the new token is rewritten in place: both calls see the same inputs
            check(lib().tla_decode_exchange(b.handle, ex.handle, _ptr(qkv), _ptr(pos), 0, T + 1, 1, _ptr(partial),
                                            None, _ptr(out), 1, _stream(None)), "decode_exchange")
        torch.cuda.synchronize()
        assert b.context.error() == 0
        torch.testing.assert_close(out.float(), exp.float(), rtol=1e-2, atol=2e-3)
    finally:
        ex.close()
        a.close()
        b.close()


def test_exchange_missing_peer_times_out(pkg, cuda):
    """Rank 1 never runs: rank 0's wait must end with TLA_ERR_TIMEOUT, not hang."""
    from three_llm_b200 import _abi, sharding

    B, H, D = 1, 8, 64
    part = _partials(cuda, B, H, D, 2)
    ctx = pkg.Context(cuda.index or 0)
    exs = [sharding.PeerExchange(r, 2, part.numel() * 4, group=False, context=ctx) for r in range(2)]
    try:
        bufs = [e.buffer() for e in exs]
        for e in exs:
            e.connect_buffers(bufs)
        out = torch.empty(B, H * D, dtype=torch.float16, device=cuda)
        exs[0].combine(part, out)
        torch.cuda.synchronize()
        timeout = {name: code for code, name in _abi.STATUS.items()}["TLA_ERR_TIMEOUT"]
        assert ctx.error() == timeout
        # the context stays usable: a merge on the same device still runs and is right
        got = pkg.combine_lse(part.unsqueeze(0))
        torch.cuda.synchronize()
        assert ctx.error() == 0
        assert torch.isfinite(got.float()).all()
    finally:
        for e in exs:
            e.close()
        ctx.close()


# ---------------------------------------------------------------- 2+ GPUs, one process per GPU
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    import datetime
    import sys

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    import __graft_entry__ as ge

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    errs = []
    try:
        ge.load_package()
        from three_llm_b200 import sharding

        dev = torch.device("cuda", rank)
        Hq, Hk, D, T, steps = 32, 8, 128, 5000, 3
        rng = np.random.default_rng(11)  # identical on every rank
        kc = rng.standard_normal((1, T + 1, Hk * D)).astype(np.float16).astype(np.float32)
        vc = rng.standard_normal((1, T + 1, Hk * D)).astype(np.float16).astype(np.float32)
        qkvs = rng.standard_normal((steps, 1, (Hq + 2 * Hk) * D)).astype(np.float16).astype(np.float32)
        opts = {"ropeTheta": 5e5}
        layer = sharding.SequenceShardedDecode(Hq, Hk, D, T, rank, world, opts, exchange="p2p")
        s = layer.shard
        if s.tokens:
            layer.layer.write_cache(0, 0, kc[0, s.slot_offset:s.slot_offset + s.tokens],
                                    vc[0, s.slot_offset:s.slot_offset + s.tokens])
        pos = torch.tensor([T], dtype=torch.int32, device=dev)
        qkv_dev = torch.from_numpy(qkvs).to(dev, torch.float16)
        exp = [oracle.decode_batch(qkvs[i], [T], kc, vc, threads=4, head_count=Hq, kv_head_count=Hk, head_dim=D,
                                   rope_theta=5e5) for i in range(steps)]
        dist.barrier()  # the exchange's wait is bounded (about 2 s): start together
        # eager: the same new token decoded three times with different queries
        for i in range(steps):
            out = layer.step(qkv_dev[i], pos).float().cpu().numpy()
            errs.append(float(np.max(np.abs(out - exp[i]) - (2e-3 + 1e-2 * np.abs(exp[i])))))
        # graph: capture one step and replay it on every rank the same number of times
        stream = torch.cuda.Stream()
        static_q = qkv_dev[0].clone()
        with torch.cuda.stream(stream):
            layer.step(static_q, pos)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            gout = layer.step(static_q, pos)
        dist.barrier()
        for i in range(steps):
            static_q.copy_(qkv_dev[i])
            graph.replay()
            out = gout.float().cpu().numpy()
            errs.append(float(np.max(np.abs(out - exp[i]) - (2e-3 + 1e-2 * np.abs(exp[i])))))
        torch.cuda.synchronize()
        del graph
        # the output projection of head-sharded attention (query heads split
        # over the ranks), summed over NVLink by tla_out_proj_allreduce
        rows, fin, hidden = 16, Hq * D, 1024
        attn = rng.standard_normal((rows, fin)).astype(np.float16).astype(np.float32)
        w = (rng.standard_normal((fin, hidden)) / np.sqrt(fin)).astype(np.float16).astype(np.float32)
        bias = rng.standard_normal(hidden).astype(np.float32)
        res = rng.standard_normal((rows, hidden)).astype(np.float16).astype(np.float32)
        per = fin // world
        op = sharding.HeadShardedOutProj(rows, hidden, rank, world, dev, context=layer.layer.context)
        dist.barrier()
        for _ in range(2):
            y = op(torch.from_numpy(attn[:, rank * per:(rank + 1) * per]).to(dev, torch.float16).contiguous(),
                   torch.from_numpy(w[rank * per:(rank + 1) * per]).to(dev, torch.float16).contiguous(),
                   torch.from_numpy(bias).to(dev), torch.from_numpy(res).to(dev, torch.float16))
            exp_y = oracle.linear(attn, w, bias, threads=4) + res
            got = y.float().cpu().numpy()
            errs.append(float(np.max(np.abs(got - exp_y) - (2e-3 + 1e-2 * np.abs(exp_y)))))
        torch.cuda.synchronize()
        dist.barrier()
        op.close()
        errs.append(float(layer.layer.context.error()))
        layer.close()
        dist.barrier()
    finally:
        np.save(result_path, np.array(errs if errs else [1e9]))
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_sequence_sharded_decode_multi_gpu(pkg, tmp_path):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    port = _free_port()
    ctx = mp.get_context("spawn")
    paths = [str(tmp_path / f"r{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, paths[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        res = np.load(paths[r])
        assert res[-1] == 0, f"rank {r} device error {res[-1]}"
        assert np.all(res[:-1] <= 0), f"rank {r} out of tolerance: {res[:-1]}"
