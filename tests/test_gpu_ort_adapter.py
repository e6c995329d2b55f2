"""Ops run through ONNX Runtime's custom-op interface on a GPU, via the stand-in session
(oracle/ort_shim):

* the product's ORT adapter (nemotron_ops_b200/ort/bolt_ort.cc): every op of the domain, with
  outputs allocated by the kernel through GetOutput, must equal the direct C-ABI call bit for bit
  and report the reference's errors;
* the reference's own kernels (its src/bolt_ops.cu recompiled for sm_100a, oracle/_ref/libbolt_ref.so,
  built where the reference checkout exists and carried with the tree): our ops against them on
  the same inputs, on shapes from the reference's own test list (tests/test_bolt_ops.py:341-371),
  with the reference test's criteria.
"""
import os

import pytest
import torch

import oracle as O
from golden_io import rel
from nemotron_ops_b200 import ops
from nemotron_ops_b200 import workloads as W
from oracle.ort_shim import build as shim_build
from oracle.ort_shim.shim import OrtError, OrtShim

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF, F32, I32 = torch.bfloat16, torch.float32, torch.int32


@pytest.fixture(scope="module")
def shim():
    built = shim_build.build(reference=False)
    s = OrtShim(built["host"])
    s.adapter = s.load(built["adapter"])
    ref = os.path.join(shim_build.OUT, "libbolt_ref.so")
    s.reference = s.load(ref) if os.path.exists(ref) else None
    return s


def run(shim, lib, op, inputs, outs, **attrs):
    """outs: [(shape, dtype)]; returns the output tensors (shapes as the kernel set them)."""
    k = shim.kernel(lib, op, **attrs)
    bufs = [torch.empty(s, dtype=d, device=DEV) for s, d in outs]
    shapes = k.run(inputs, bufs)
    torch.cuda.synchronize()
    for b, s in zip(bufs, shapes):
        assert s == tuple(b.shape), (op, s, tuple(b.shape))
    return bufs


def _gemv_cases():
    d1 = W.nvfp4_gemv(R=1, N=512, K=2048, seed=1, device=DEV)
    d8 = W.nvfp4_gemv(R=8, N=512, K=2048, seed=2, device=DEV)
    q8 = W.q8_gemv(R=3, N=256, K=1024, seed=3, device=DEV)
    q4 = W.q4_gemv(R=1, N=256, K=1024, seed=4, device=DEV)
    q4n = W.q4_gemv(R=4, N=256, K=1024, iq2=2, seed=5, device=DEV)
    return [
        ("Nvfp4Gemv", [d1["x"], d1["w"], d1["w_scale"], d1["g"]], {}, lambda: ops.Nvfp4Gemv(d1["x"], d1["w"], d1["w_scale"], d1["g"])),
        ("Nvfp4Gemv", [d8["x"], d8["w"], d8["w_scale"], d8["g"]], {}, lambda: ops.Nvfp4Gemv(d8["x"], d8["w"], d8["w_scale"], d8["g"])),
        ("Q8Gemv", [q8["x"], q8["B"], q8["scales"]], {}, lambda: ops.Q8Gemv(q8["x"], q8["B"], q8["scales"])),
        ("Q4Gemv", [q4["x"], q4["B"], q4["scales"]], {}, lambda: ops.Q4Gemv(q4["x"], q4["B"], q4["scales"])),
        ("Q4Gemv", [q4n["x"], q4n["B"], q4n["scales"]], {"iq2": 2},
         lambda: ops.Q4Gemv(q4n["x"], q4n["B"], q4n["scales"], iq2=2)),
    ]


@pytest.mark.parametrize("case", range(5))
def test_adapter_gemv_equals_direct_call(shim, case):
    op, ins, attrs, direct = _gemv_cases()[case]
    want = direct()
    (got,) = run(shim, shim.adapter, op, ins, [(tuple(want.shape), BF)], **attrs)
    assert torch.equal(got, want)


def test_adapter_moe_route_equals_direct_call(shim):
    r = W.moe_route(R=8, E=64, K=1024, seed=6, device=DEV)
    want = ops.MoeRoute(r["x"], r["gate_w"], r["bias"], 6, 2.5)
    got = run(shim, shim.adapter, "MoeRoute", [r["x"], r["gate_w"], r["bias"]], [((8, 6), I32), ((8, 6), F32),
                                                                                ((8, 64), F32)], topk=6, scale=2.5)
    for a, b in zip(got, want):
        assert torch.equal(a, b)


@pytest.mark.parametrize("op,iq2", [("MoeDecode", 0), ("MoeVerify", 0), ("MoeVerify", 2)])
def test_adapter_moe_equals_direct_call(shim, op, iq2):
    R, E, I, topk = (1, 24, 256, 4) if op == "MoeDecode" else (8, 24, 256, 4)
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=7, device=DEV)
    g = torch.Generator().manual_seed(8)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int().to(DEV)
    w = torch.rand(R, topk, generator=g).to(DEV)
    z = W.moe_latent(R=R, seed=9, device=DEV)
    ins = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    P = R * topk
    outs = [((R, 1024), BF), ((P, I), BF), ((P, 1024), F32)]
    if op == "MoeDecode":
        want = ops.MoeDecode(*ins, topk=topk)
        got = run(shim, shim.adapter, op, ins, outs, topk=topk)
    else:
        want = ops.MoeVerify(*ins, topk=topk, iq2=iq2)
        attrs = {"topk": topk, "iq2": iq2} if iq2 else {"topk": topk}
        got = run(shim, shim.adapter, op, ins, outs + [((1 + P + 8 * P,), I32)], **attrs)
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_adapter_relu2_equals_direct_call(shim):
    x = (torch.randn(3, 1000, device=DEV) * 3).to(BF)
    (got,) = run(shim, shim.adapter, "Relu2", [x], [((3, 1000), BF)])
    assert torch.equal(got, ops.Relu2(x))


@pytest.mark.parametrize("verify", [False, True])
def test_adapter_mamba_equals_direct_call(shim, verify):
    heads, ng, R = 8, 2, 3
    g = torch.Generator().manual_seed(10)
    di, cd = heads * 64, heads * 64 + 2 * ng * 128
    rows = R if verify else 1
    ins = [(torch.randn(R, di + cd + heads, generator=g) * 0.7).bfloat16(),
           (torch.randn(rows, cd, 3, generator=g) * 0.5).bfloat16(),
           torch.randn(rows, heads, 128, 64, generator=g) * 0.1,
           (torch.randn(cd, 1, 4, generator=g) * 0.3).bfloat16(), (torch.randn(cd, generator=g) * 0.1).bfloat16(),
           torch.randn(heads, generator=g) * 0.3, -torch.rand(heads, generator=g) * 4 - 0.1,
           torch.randn(heads, generator=g), torch.rand(di, generator=g) + 0.5]
    ins = [t.to(DEV) for t in ins]
    attrs = dict(heads=heads, head_dim=64, d_state=128, n_groups=ng, epsilon=1e-5, time_step_min=0.001)
    outs = [((R, di), BF), (tuple(ins[1].shape), BF), (tuple(ins[2].shape), F32), ((R, cd), BF), ((R, di), F32)]
    if verify:
        sel = torch.tensor([1], dtype=I32, device=DEV)
        want = ops.MambaVerify(*ins, sel, **attrs)
        got = run(shim, shim.adapter, "MambaVerify", ins + [sel], outs, **attrs)
    else:
        want = ops.MambaStep(*ins, **attrs)
        got = run(shim, shim.adapter, "MambaStep", ins, outs, **attrs)
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_adapter_reports_the_reference_error(shim):
    d = W.nvfp4_gemv(R=1, N=64, K=1024, seed=11, device=DEV)
    x = torch.zeros(1, 1536, dtype=BF, device=DEV)  # K % 1024 != 0 and != 2 * w's width
    with pytest.raises(OrtError) as e:
        run(shim, shim.adapter, "Nvfp4Gemv", [x, d["w"], d["w_scale"], d["g"]], [((1, 64), BF)])
    assert e.value.code == 1 and "Nvfp4Gemv: K mismatch" in e.value.msg


# ---------------------------------------------------------------------------------------------
# the reference's own kernels on the same B200
# ---------------------------------------------------------------------------------------------
def _need_ref(shim):
    if shim.reference is None:
        pytest.skip("oracle/_ref/libbolt_ref.so is absent (built where the reference checkout exists)")


@pytest.mark.parametrize("R,N,K", [(1, 4096, 8192), (8, 4096, 8192), (5, 1024, 4096)])
def test_reference_kernels_nvfp4(shim, R, N, K):
    _need_ref(shim)
    d = W.nvfp4_gemv(R=R, N=N, K=K, seed=12 + R, device=DEV)
    ins = [d["x"], d["w"], d["w_scale"], d["g"]]
    (ref,) = run(shim, shim.reference, "Nvfp4Gemv", ins, [((R, N), BF)])
    ours = ops.Nvfp4Gemv(*ins)
    exact = O.nvfp4_gemv(*[t.cpu() for t in ins])
    assert rel(ours, ref) < 1e-2 and rel(ref, exact) < 1e-2  # the reference test's criterion (:79)
    assert rel(ours, exact) <= rel(ref, exact) + 1e-4       # ours is no less accurate than the reference


@pytest.mark.parametrize("bits,R,N,K", [(8, 1, 1024, 4096), (4, 1, 1024, 4096), (8, 3, 1024, 4096),
                                        (4, 8, 4096, 1024)])
def test_reference_kernels_qgemv(shim, bits, R, N, K):
    _need_ref(shim)
    d = (W.q8_gemv if bits == 8 else W.q4_gemv)(R=R, N=N, K=K, seed=20 + R, device=DEV)
    ins = [d["x"], d["B"], d["scales"]]
    op = "Q8Gemv" if bits == 8 else "Q4Gemv"
    (ref,) = run(shim, shim.reference, op, ins, [((R, N), BF)])
    ours = (ops.Q8Gemv if bits == 8 else ops.Q4Gemv)(*ins)
    assert rel(ours, ref) < 1e-2


def test_reference_kernels_route(shim):
    _need_ref(shim)
    r = W.moe_route(R=8, E=304, K=4096, seed=30, device=DEV)
    ins = [r["x"], r["gate_w"], r["bias"]]
    ridx, rw, rsc = run(shim, shim.reference, "MoeRoute", ins, [((8, 9), I32), ((8, 9), F32), ((8, 304), F32)],
                        topk=9, scale=5.0)
    idx, w, sc = ops.MoeRoute(*ins, 9, 5.0)
    assert rel(sc, rsc) < 1e-5
    if O.route_min_gap(*[t.cpu() for t in ins], 9) > 1e-5:
        assert torch.equal(idx, ridx)
        assert rel(w, rw) < 1e-5


@pytest.mark.parametrize("op,R,E,I,iq2", [("MoeDecode", 1, 240, 2048, 0), ("MoeVerify", 8, 304, 2304, 0),
                                          ("MoeVerify", 8, 304, 2304, 2)])
def test_reference_kernels_moe(shim, op, R, E, I, iq2):
    _need_ref(shim)
    topk = 9
    ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=31, device=DEV)
    g = torch.Generator().manual_seed(32)
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int().to(DEV)
    w = torch.rand(R, topk, generator=g).to(DEV)
    z = W.moe_latent(R=R, seed=33, device=DEV)
    ins = [z, idx, w, ex["fc1_w"], ex["fc1_s"], ex["fc2_w"], ex["fc2_s"]]
    P = R * topk
    outs = [((R, 1024), BF), ((P, I), BF), ((P, 1024), F32)]
    if op == "MoeDecode":
        ref = run(shim, shim.reference, op, ins, outs, topk=topk)
        ours = ops.MoeDecode(*ins, topk=topk)
    else:
        attrs = {"topk": topk, "iq2": iq2} if iq2 else {"topk": topk}
        ref = run(shim, shim.reference, op, ins, outs + [((1 + P + 8 * P,), I32)], **attrs)
        ours = ops.MoeVerify(*ins, topk=topk, iq2=iq2)
        # meta: U, the unique experts in first-occurrence order and the pair map (the reference leaves
        # slots U + 1 .. P of the expert list unwritten, src/bolt_ops.cu:1084-1112)
        U = int(ref[3][0])
        assert torch.equal(ours[3][:1 + U], ref[3][:1 + U])
        assert torch.equal(ours[3][1 + P:], ref[3][1 + P:])
    assert rel(ours[0], ref[0]) < 1e-2        # the reference test's criterion (:165)
    assert rel(ours[1], ref[1]) < 1e-2
