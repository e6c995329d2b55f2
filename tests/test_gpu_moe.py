"""GPU parity of MoeRoute / MoeDecode / MoeVerify (CUDA path through the C ABI) against the oracle."""
import pytest
import torch

import oracle as O
from golden_io import case_names, load, rel
from nemotron_ops_b200 import ops
from nemotron_ops_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def assert_close(y, ref, rtol=1e-2, atol=1e-3):
    y, ref = y.float().cpu(), ref.float().cpu()
    err = (y - ref).abs()
    bad = err > atol + rtol * ref.abs()
    assert not bool(bad.any()), f"{int(bad.sum())}/{bad.numel()} outside tolerance, max err {float(err.max()):.3g}"


def _dev(ts):
    return [t.to(DEV) for t in ts]


# ---------------------------------------------------------------------------------------------
# MoeRoute
# ---------------------------------------------------------------------------------------------
def _check_route(x, gw, b, topk, scale):
    idx, w, scores = ops.MoeRoute(x, gw, b, topk, scale)
    oi, ow, osc = O.moe_route(x.cpu(), gw.cpu(), b.cpu(), topk, scale)
    gap = O.route_min_gap(x.cpu(), gw.cpu(), b.cpu(), topk)
    assert_close(scores, osc, rtol=1e-5, atol=1e-6)
    if gap > 1e-5:  # selection is decided well above fp32 summation noise: bit-exact, in order
        assert torch.equal(idx.cpu(), oi)
        assert_close(w, ow, rtol=1e-5, atol=1e-6)
    return idx, w


@pytest.mark.parametrize("name", case_names("route_"))
def test_route_golden(name):
    c = load(name)
    x, gw, b = _dev(c.inputs)
    idx, w = _check_route(x, gw, b, c.attrs["topk"], c.attrs["scale"])
    R, E = c.ref.shape
    got = torch.zeros(R, E).scatter_(1, idx.cpu().long(), w.cpu())
    assert torch.equal(got != 0, c.ref != 0)
    assert rel(got, c.ref) < 1e-3


@pytest.mark.parametrize("R,E,topk", [(1, 304, 8), (4, 496, 9), (8, 304, 8), (8, 512, 32), (3, 40, 40 // 2)])
def test_route_config(R, E, topk):
    d = W.moe_route(R=R, E=E, K=4096, seed=R * 100 + E)
    _check_route(d["x"], d["gate_w"], d["bias"], topk, 5.0)


def test_route_ties_go_to_lower_index():
    x = torch.zeros(2, 256, dtype=torch.bfloat16, device=DEV)
    gw = torch.zeros(70, 256, dtype=torch.bfloat16, device=DEV)
    b = torch.zeros(70, device=DEV)
    b[[5, 33, 64, 65, 69]] = 0.25
    idx, w, s = ops.MoeRoute(x, gw, b, 4, 1.0)
    assert idx.cpu().tolist() == [[5, 33, 64, 65], [5, 33, 64, 65]]
    assert torch.allclose(w.cpu(), torch.full((2, 4), 0.25))


@pytest.mark.parametrize("E,topk", [(1, 1), (5, 8), (31, 8), (32, 32), (33, 9), (70, 4), (304, 8), (497, 32),
                                    (512, 32), (512, 1)])
def test_route_selection_bit_exact(E, topk):
    # x = 0 makes every logit 0 and every score exactly 0.5, so the bias alone orders the experts
    # and the selection can be compared bit for bit: values drawn from a small set (exact ties,
    # +0 / -0, +-inf, NaN) plus random ones exercise the tie rule, the never-chosen values and the
    # selection order; the weights (0.5 / sum in selection order * scale) must match exactly too
    g = torch.Generator().manual_seed(E * 37 + topk)
    pool = torch.tensor([0.5, 0.25, -0.0, 0.0, 1.5, -2.0, float("inf"), float("-inf"), float("nan"), 0.125])
    for trial in range(4):
        b = pool[torch.randint(0, len(pool), (E,), generator=g)]
        rnd = torch.rand(E, generator=g) < 0.3
        b[rnd] = torch.randn(int(rnd.sum()), generator=g)
        if trial == 3:
            b[:] = float("-inf")  # nothing can be chosen
        x = torch.zeros(3, 256, dtype=torch.bfloat16)
        gw = torch.randn(E, 256, generator=g).to(torch.bfloat16)
        idx, w, s = ops.MoeRoute(x.to(DEV), gw.to(DEV), b.to(DEV), topk, 3.0)
        oi, ow, osc = O.moe_route(x, gw, b, topk, 3.0)
        assert torch.equal(s.cpu(), osc)
        assert torch.equal(idx.cpu(), oi), (trial, idx.cpu()[0].tolist(), oi[0].tolist())
        assert torch.equal(w.cpu(), ow)


def test_route_topk_above_expert_count():
    d = W.moe_route(R=1, E=5, K=256, seed=1)
    idx, w, s = ops.MoeRoute(d["x"], d["gate_w"], d["bias"], 8, 1.0)
    assert idx.cpu()[0, 5:].tolist() == [-1, -1, -1]
    assert w.cpu()[0, 5:].tolist() == [0.0, 0.0, 0.0]
    assert sorted(idx.cpu()[0, :5].tolist()) == [0, 1, 2, 3, 4]


# ---------------------------------------------------------------------------------------------
# MoeDecode / MoeVerify
# ---------------------------------------------------------------------------------------------
# The MoE epilogues round twice before fc2 (a = bf16(z . W1), h = bf16(relu(a)^2)), so h may
# differ from the fp64 oracle by up to ~1.2% where either rounding flips; such a flip then
# moves fc2's partial sums by far more than 1e-3 where they cancel.  Each stage is therefore
# checked against the oracle fed with the kernel's own input of that stage, and the end-to-end
# output with the reference tests' own relative-norm criterion (tests/test_bolt_ops.py:63-65).
H_RTOL = 1.6e-2  # two bf16 roundings (2^-8 each, the first one doubled by the square)


def _check_moe(op, ins, topk, iq2=0, on_device=False):
    dev = _dev(ins)
    src = dev if on_device else ins
    if op == "MoeDecode":
        out, h, part = ops.MoeDecode(*dev, topk=topk)
        oo, oh, op_ = O.moe_decode(*src, topk=topk)
        _, _, op2 = O.moe_decode(*src, topk=topk, h_in=h.to(src[0].device))
    else:
        out, h, part, meta = ops.MoeVerify(*dev, topk=topk, iq2=iq2)
        oo, oh, op_, om = O.moe_verify(*src, topk=topk, iq2=iq2)
        _, _, op2, _ = O.moe_verify(*src, topk=topk, iq2=iq2, h_in=h.to(src[0].device))
        assert torch.equal(meta.cpu(), om)
    assert_close(h, oh, rtol=H_RTOL)                            # fc1 + relu^2
    assert_close(part, op2)                                     # fc2 from the kernel's h
    assert_close(out, O.moe_combine(part.to(src[0].device), src[2], topk))  # weighted sum
    assert rel(out, oo) < 1e-2                                  # end to end
    assert ops.device_status() == 0
    return out


@pytest.mark.parametrize("name", case_names("moe_"))
def test_moe_golden(name):
    c = load(name)
    iq2 = c.attrs.get("iq2", 0)
    out = _check_moe(c.op, c.inputs, c.attrs["topk"], iq2)
    assert rel(out, c.ref) < 1e-2


def _routed(R, E, topk, seed):
    r = W.moe_route(R=R, E=E, K=4096, seed=seed)
    idx, w, _ = ops.MoeRoute(r["x"], r["gate_w"], r["bias"], topk, 5.0)
    return idx, w


def test_moe_decode_config_r1():
    idx, w = _routed(1, 304, 8, 0)
    ex = W.moe_experts(E=304, I=2304)
    z = W.moe_latent(R=1)
    ins = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    _check_moe("MoeDecode", [t.cpu() for t in ins], 8)


@pytest.mark.parametrize("iq2", [0, 2])
def test_moe_verify_config_r8(iq2):
    idx, w = _routed(8, 304, 8, 3)
    ex = W.moe_experts(E=304, I=2304, iq2=iq2)
    z = W.moe_latent(R=8)
    # fp64 oracle run on the GPU tensors (the oracle is device-agnostic torch)
    _check_moe("MoeVerify", [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]], 8, iq2, on_device=True)


@pytest.mark.parametrize("uniq", [19, 23])
@pytest.mark.parametrize("iq2", [0, 2])
def test_moe_verify_split_fc2_tiles(uniq, iq2):
    # fc2 has 8 tiles of 128 rows per expert: 19 experts give 152 tiles for 148 SMs, so almost
    # every tile is split between two CTAs at a K-segment boundary (23: 184 tiles, other cuts)
    R, topk, E, I = 8, 3, 32, 2304
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=uniq)
    picks = list(range(uniq)) + [(5 * j) % uniq for j in range(R * topk - uniq)]
    idx = torch.tensor(picks, dtype=torch.int32).reshape(R, topk)
    w = torch.rand(R, topk, generator=torch.Generator().manual_seed(uniq))
    z = W.moe_latent(R=R, seed=uniq)
    _check_moe("MoeVerify", [z, idx.to(DEV), w.to(DEV), ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]], topk,
               iq2, on_device=True)


@pytest.mark.parametrize("R,E,I,topk", [(2, 24, 256, 3), (5, 40, 512, 4), (8, 12, 256, 6), (8, 64, 768, 8)])
@pytest.mark.parametrize("iq2", [0, 1, 2])
def test_moe_verify_small(R, E, I, topk, iq2):
    if iq2 == 2 and I % 256:
        pytest.skip("native IQ2_XXS needs I % 256")
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=R + E)
    if iq2 == 1:  # valid LUT codes only
        ex["fc1_w"] &= 0x66
        ex["fc2_w"] &= 0x66
    g = torch.Generator().manual_seed(R * E)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int()
    w = torch.rand(R, topk, generator=g)
    z = W.moe_latent(R=R, seed=E).cpu()
    _check_moe("MoeVerify", [z, idx, w] + [ex[k].cpu() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")], topk, iq2)


@pytest.mark.parametrize("R,E,I,topk", [(1, 8, 64, 3), (2, 24, 2304, 8), (3, 16, 160, 4), (1, 300, 2048, 9)])
def test_moe_decode_small(R, E, I, topk):
    ex = W.moe_experts(E=E, I=I, seed=R + E)
    g = torch.Generator().manual_seed(R * E)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int()
    w = torch.rand(R, topk, generator=g)
    z = W.moe_latent(R=R, seed=E).cpu()
    _check_moe("MoeDecode", [z, idx, w] + [ex[k].cpu() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")], topk)


def test_moe_decode_skips_out_of_range_expert():
    E, I, topk = 8, 64, 3
    ex = W.moe_experts(E=E, I=I, seed=5)
    idx = torch.tensor([[2, -1, 9]], dtype=torch.int32)
    w = torch.rand(1, topk)
    z = W.moe_latent(R=1, seed=5).cpu()
    ins = [z, idx, w] + [ex[k].cpu() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")]
    out, h, part = ops.MoeDecode(*_dev(ins), topk=topk)
    oo, oh, op_ = O.moe_decode(*ins, topk=topk)
    assert_close(h, oh, rtol=H_RTOL)
    assert rel(out, oo) < 1e-2
    assert float(h[1:].abs().max()) == 0.0 and float(part[1:].abs().max()) == 0.0


def test_moe_verify_graph_capture():
    idx, w = _routed(8, 64, 8, 7)
    ex = W.moe_experts(E=64, I=512, seed=3)
    z = W.moe_latent(R=8, seed=3)
    args = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ref = ops.MoeVerify(*args, topk=8)[0]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ops.MoeVerify(*args, topk=8)[0]
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("op,R", [("MoeDecode", 1), ("MoeVerify", 8)])
def test_route_then_moe_one_graph(op, R):
    # MoeRoute and the MoE layer captured back to back in one CUDA graph (the launches chain by
    # programmatic dependent launch); replays equal the eager sequence and the oracle
    E, I, topk = 64, 512, 8
    r = W.moe_route(R=R, E=E, K=4096, seed=11)
    ex = W.moe_experts(E=E, I=I, seed=11)
    z = W.moe_latent(R=R, seed=11)
    fn = ops.MoeDecode if op == "MoeDecode" else ops.MoeVerify

    def step():
        idx, w, _ = ops.MoeRoute(r["x"], r["gate_w"], r["bias"], topk, 5.0)
        return (idx, w) + tuple(fn(z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"], topk=topk))

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ref = [t.clone() for t in step()]
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        got = step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    idx, w = got[0], got[1]
    _check_route(r["x"], r["gate_w"], r["bias"], topk, 5.0)
    ins = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    _check_moe(op, ins, topk, on_device=True)
