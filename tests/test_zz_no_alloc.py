"""bolt_moe_verify_noalloc through the C ABI: MoeVerify whose scratch (h, part, meta) lives in
the library's static device buffer.  Two consecutive calls must each match bolt_moe_verify with
caller buffers; a call whose scratch would not fit must fail with a message.

The file name sorts last so the entry point also runs after every other GPU test of a session.
"""
import ctypes

import pytest
import torch

from nemotron_ops_b200 import ops
from nemotron_ops_b200 import workloads as W
from nemotron_ops_b200._lib import last_error, lib, shape_arg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _routing(R, E, topk, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int()
    w = torch.rand(R, topk, generator=g)
    return idx.to(DEV), w.to(DEV)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def verify_noalloc(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, iq2=0):
    """out bf16 [R, 1024] of MoeVerify, computed without caller scratch buffers."""
    out = torch.empty(z.shape[0], 1024, dtype=torch.bfloat16, device=z.device)
    zs, _k1 = shape_arg(z.shape)
    w1s, _k2 = shape_arg(fc1_w.shape)
    rc = lib().bolt_moe_verify_noalloc(_p(z), zs, z.dim(), _p(idx), _p(w), _p(fc1_w), w1s, fc1_w.dim(), _p(fc1_s),
                                       _p(fc2_w), _p(fc2_s), int(topk), int(iq2), _p(out),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


@pytest.mark.parametrize("iq2", [0, 2])
def test_two_consecutive_calls_match_the_buffered_entry_point(iq2):
    # Both entry points run the same kernels on the same inputs, so they must agree bit for bit.
    # The second call is smaller (3 rows, topk 4) and routes to other experts than the first
    # (8 rows, topk 8), so a call that read the first call's leftover meta / h / part from the
    # shared static buffer instead of writing its own would give a different result.
    E, I = 40, 2304
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=21 + iq2)
    weights = [ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    first = [W.moe_latent(R=8, seed=5), *_routing(8, E, 8, seed=7)]
    second = [W.moe_latent(R=3, seed=6), *_routing(3, E, 4, seed=8)]
    for (z, idx, w), topk in ((first, 8), (second, 4)):
        ref = ops.MoeVerify(z, idx, w, *weights, topk=topk, iq2=iq2)[0]
        rc, out = verify_noalloc(z, idx, w, *weights, topk=topk, iq2=iq2)
        torch.cuda.synchronize()
        assert rc == 0, last_error()
        assert torch.equal(out, ref)
    assert ops.device_status() == 0


def test_oversized_scratch_is_rejected():
    R, E, I, topk = 8, 16, 8192, 16  # h alone would need 2 MiB
    ex = W.moe_experts(E=E, I=I, seed=9)
    args = [W.moe_latent(R=R, seed=9), *_routing(R, E, topk, seed=9), ex["fc1_w"], ex["fc1_s"], ex["fc2_w"],
            ex["fc2_s"]]
    rc, _ = verify_noalloc(*args, topk=topk)
    assert rc != 0
    assert "static buffer" in last_error()
