"""Expert-sharded MoeVerify and MoeDecode: the distributed host logic on CPU ``gloo`` ranks.

The per-shard computation is the oracle's shard partial (the CUDA shard kernel is covered by
``tests/test_gpu_sharded.py``); what runs here is the product's partitioning, weight slicing,
all-reduce of the fp32 partials and the final cast.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from nemotron_ops_b200.sharded import ShardedMoeDecode, ShardedMoeVerify, expert_range
from nemotron_ops_b200 import workloads as W


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_range_partitions():
    for E in (1, 7, 304):
        for world in (1, 2, 3, 4, 8):
            ranges = [expert_range(E, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == E
            for (a0, b0), (a1, b1) in zip(ranges, ranges[1:]):
                assert b0 == a1
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def _case(E, I, R, topk, iq2, seed):
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=seed, device="cpu")
    if iq2 == 1:
        ex["fc1_w"] &= 0x66
        ex["fc2_w"] &= 0x66
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int()
    w = torch.rand(R, topk, generator=g)
    z = W.moe_latent(R=R, seed=seed + 1, device="cpu")
    return z, idx, w, ex


def _worker(rank, world, port, E, I, R, topk, iq2, seed, q, op="verify"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        z, idx, w, ex = _case(E, I, R, topk, iq2, seed)

        def shard_fn(z_, idx_, w_, weights, e0, e1):
            if op == "decode":
                return O.moe_decode_partial(z_, idx_, w_, *weights, topk, e0, e1, num_experts=E)
            return O.moe_verify_partial(z_, idx_, w_, *weights, topk, iq2, e0, e1, num_experts=E)

        cast = lambda t: t.to(torch.bfloat16)  # noqa: E731
        if op == "decode":
            moe = ShardedMoeDecode(E, topk, shard_fn=shard_fn, cast_fn=cast)
        else:
            moe = ShardedMoeVerify(E, topk, iq2, shard_fn=shard_fn, cast_fn=cast)
        weights = [moe.local_slice(ex[k]) for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")]
        assert weights[0].shape[0] == moe.e_end - moe.e_begin
        out = moe(z, idx, w, weights)
        q.put((rank, out, moe.e_begin, moe.e_end))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,E,I,R,topk,iq2", [(2, 8, 256, 3, 3, 0), (2, 9, 256, 8, 4, 2), (3, 7, 128, 2, 5, 1)])
def test_sharded_verify_matches_single_gpu_op(world, E, I, R, topk, iq2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, E, I, R, topk, iq2, 11, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    z, idx, w, ex = _case(E, I, R, topk, iq2, 11)
    ref = O.moe_verify(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk=topk, iq2=iq2)[0]
    got.sort(key=lambda g: g[0])
    assert [g[2:] for g in got] == [expert_range(E, r, world) for r in range(world)]
    for _, out, _, _ in got:
        # every rank holds the same all-reduced result; fp32 reassociation of the shard sums only
        assert torch.equal(out, got[0][1])
        err = (out.float() - ref.float()).abs()
        assert bool((err <= 1e-3 + 1e-2 * ref.float().abs()).all())


@pytest.mark.parametrize("world,E,I,R,topk", [(2, 8, 256, 1, 6), (3, 10, 256, 2, 4)])
def test_sharded_decode_matches_single_gpu_op(world, E, I, R, topk):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, E, I, R, topk, 0, 5, q, "decode"))
             for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    z, idx, w, ex = _case(E, I, R, topk, 0, 5)
    ref = O.moe_decode(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk=topk)[0]
    got.sort(key=lambda g: g[0])
    assert [g[2:] for g in got] == [expert_range(E, r, world) for r in range(world)]
    for _, out, _, _ in got:
        assert torch.equal(out, got[0][1])
        err = (out.float() - ref.float()).abs()
        assert bool((err <= 1e-3 + 1e-2 * ref.float().abs()).all())
