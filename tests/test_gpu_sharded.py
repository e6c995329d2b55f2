"""GPU parity of the expert-sharded MoeVerify and MoeDecode steps (bolt_moe_verify_shard,
bolt_moe_decode_shard through the C ABI).

The shards of a G-way split run one after another on one GPU, each with only its own experts'
weights; their fp32 partials are summed and cast, as the all-reduce would do across GPUs.
"""
import pytest
import torch

import oracle as O
from nemotron_ops_b200 import ops
from nemotron_ops_b200.sharded import expert_range
from nemotron_ops_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _routing(R, E, topk, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int()
    w = torch.rand(R, topk, generator=g)
    return idx.to(DEV), w.to(DEV)


@pytest.mark.parametrize("G", [2, 4, 8])
@pytest.mark.parametrize("iq2", [0, 2])
def test_sharded_partials_sum_to_the_op(G, iq2):
    E, I, R, topk = 40, 512, 8, 8
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=G + iq2)
    z = W.moe_latent(R=R, seed=G)
    idx, w = _routing(R, E, topk, seed=G)
    total = torch.zeros(R, 1024, dtype=torch.float64, device=DEV)
    for g in range(G):
        e0, e1 = expert_range(E, g, G)
        local = [ex[k][e0:e1].contiguous() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")]
        part, _, _, meta = ops.moe_verify_shard(z, idx, w, *local, topk=topk, iq2=iq2, e_begin=e0, e_end=e1,
                                                num_experts=E)
        ref = O.moe_verify_partial(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk, iq2, e0, e1)
        # a shard's partial: tolerance of the op, scaled by the partial's own magnitude
        err = (part.double() - ref.double()).abs()
        assert bool((err <= 1e-3 + 1e-2 * ref.double().abs() + 1e-2 * ref.double().abs().max()).all())
        local_ids = idx[(idx >= e0) & (idx < e1)]
        assert int(meta[0]) == int(local_ids.unique().numel())
        total += part.double()
    out = ops.f32_to_bf16(total.float())
    ref_out = O.moe_verify(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk=topk, iq2=iq2)[0]
    rel = ((out.float() - ref_out.float()).norm() / ref_out.float().norm()).item()
    assert rel < 1e-2
    assert ops.device_status() == 0


def test_single_shard_equals_unsharded_op():
    E, I, R, topk = 24, 256, 4, 6
    ex = W.moe_experts(E=E, I=I, seed=3)
    z = W.moe_latent(R=R, seed=3)
    idx, w = _routing(R, E, topk, seed=3)
    args = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    out = ops.MoeVerify(*args, topk=topk)[0]
    part, _, _, _ = ops.moe_verify_shard(*args, topk=topk, iq2=0, e_begin=0, e_end=E)
    assert torch.equal(ops.f32_to_bf16(part), out)


@pytest.mark.parametrize("G", [2, 8])
@pytest.mark.parametrize("R,topk", [(1, 8), (3, 6)])
def test_sharded_decode_partials_sum_to_the_op(G, R, topk):
    E, I = 40, 512
    ex = W.moe_experts(E=E, I=I, seed=7 + G)
    z = W.moe_latent(R=R, seed=G + R)
    idx, w = _routing(R, E, topk, seed=G + 1)
    total = torch.zeros(R, 1024, dtype=torch.float64, device=DEV)
    for g in range(G):
        e0, e1 = expert_range(E, g, G)
        local = [ex[k][e0:e1].contiguous() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")]
        part, _, _ = ops.moe_decode_shard(z, idx, w, *local, topk=topk, e_begin=e0, e_end=e1, num_experts=E)
        ref = O.moe_decode_partial(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk, e0, e1)
        err = (part.double() - ref.double()).abs()
        assert bool((err <= 1e-3 + 1e-2 * ref.double().abs() + 1e-2 * ref.double().abs().max()).all())
        total += part.double()
    out = ops.f32_to_bf16(total.float())
    ref_out = O.moe_decode(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk=topk)[0]
    rel = ((out.float() - ref_out.float()).norm() / ref_out.float().norm()).item()
    assert rel < 1e-2
    assert ops.device_status() == 0


def test_single_shard_decode_equals_unsharded_op():
    E, I, R, topk = 24, 256, 1, 8
    ex = W.moe_experts(E=E, I=I, seed=4)
    z = W.moe_latent(R=R, seed=4)
    idx, w = _routing(R, E, topk, seed=4)
    args = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    out = ops.MoeDecode(*args, topk=topk)[0]
    part, _, _ = ops.moe_decode_shard(*args, topk=topk, e_begin=0, e_end=E)
    assert torch.equal(ops.f32_to_bf16(part), out)
