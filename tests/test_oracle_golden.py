"""Pin the CPU oracle against golden vectors produced by the reference's own test code.

Every fixture under tests/golden/ holds the inputs and the expected tensor that
tests/test_bolt_ops.py of the reference computes (see tests/golden/make_golden.py).
Two levels are checked per case:

* format decode: the oracle's exact-weight GEMV reproduces the reference's expected
  output to fp32 summation noise (any decode slip -- nibble order, zero point, scale
  layout, sign bits -- would show up orders of magnitude above that);
* op contract: the oracle's op output (with the kernel's bf16 rounding points) is within
  the reference test's own threshold of the reference's expected output.
"""
import pytest
import torch

import oracle as O
from golden_io import case_names, load, rel


def _close_to_fp32(y, ref, tol=2e-5):
    err = (y.double() - ref.double()).abs().max().item()
    scale = ref.double().abs().max().item()
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("name", case_names("nvfp4_"))
def test_nvfp4_oracle(name):
    c = load(name)
    x, w, ws, g = c.inputs
    W = O.nvfp4_dequant(w, ws) * float(g[0])
    _close_to_fp32(x.double() @ W.double().T, c.ref)
    y = O.nvfp4_gemv(x, w, ws, g)
    assert rel(y, c.ref) < 1e-2


@pytest.mark.parametrize("name", case_names("q8_") + case_names("q4_r"))
def test_qgemv_oracle(name):
    c = load(name)
    x, B, s = c.inputs
    if c.op == "Q8Gemv":
        W, y = O.q8_dequant(B, s, "exact"), O.q8_gemv(x, B, s)
    else:
        W, y = O.q4_dequant(B, s, "exact"), O.q4_gemv(x, B, s)
    _close_to_fp32(x.double() @ W.double().T, c.ref)
    assert rel(y, c.ref) < 1e-2


@pytest.mark.parametrize("name", case_names("q4_iq2lut_"))
def test_q4_iq2_lut_oracle(name):
    c = load(name)
    x, B, s = c.inputs
    N, nb = s.shape
    codes = O.unpack_nibbles(B.reshape(N, nb, 16)).long()
    W = (O.IQ2_LUT_BF16[codes] * s.float().unsqueeze(-1)).reshape(N, -1)
    _close_to_fp32(x.double() @ W.double().T, c.ref)
    assert rel(O.q4_gemv(x, B, s, iq2=1), c.ref) < 6e-3


@pytest.mark.parametrize("name", case_names("q4_iq2n_"))
def test_q4_iq2_native_oracle(name):
    c = load(name)
    x, B, D = c.inputs
    # bit-exact restatement of gguf's IQ2_XXS dequantisation (the reference test's oracle)
    g = O.iq2n_dequant_gguf_style(B, D)
    assert torch.equal(g, c.gguf_deq)
    # the kernel contract bf16(mag * bf16(db)) is within one bf16 ulp of bf16(gguf)
    kc = O.iq2n_dequant(B, D)
    gb = O.bf16_round(g)
    ulp = torch.where(gb == 0, torch.ones_like(gb), gb.abs()) * 2.0 ** -7
    assert bool(((kc - gb).abs() <= ulp).all())
    _close_to_fp32(x.double() @ gb.double().T, c.ref)
    assert rel(O.q4_gemv(x, B, D, iq2=2), c.ref) < 6e-3


@pytest.mark.parametrize("name", case_names("route_"))
def test_route_oracle(name):
    c = load(name)
    x, gw, b = c.inputs
    topk, scale = c.attrs["topk"], c.attrs["scale"]
    idx, wts, scores = O.moe_route(x, gw, b, topk, scale)
    R, E = c.ref.shape
    got = torch.zeros(R, E).scatter_(1, idx.long(), wts)
    assert torch.equal(got != 0, c.ref != 0)  # same expert sets
    _close_to_fp32(got, c.ref, 1e-5)
    # selection order: descending bias-corrected score
    val = scores + b.unsqueeze(0)
    sel = val.gather(1, idx.long())
    assert bool((sel[:, :-1] >= sel[:, 1:]).all())
    assert O.route_min_gap(x, gw, b, topk) > 0


@pytest.mark.parametrize("name", case_names("moe_decode_"))
def test_moe_decode_oracle(name):
    c = load(name)
    out, h, part = O.moe_decode(*c.inputs, topk=c.attrs["topk"])
    assert rel(out, c.ref) < 4e-3


@pytest.mark.parametrize("name", case_names("moe_verify_"))
def test_moe_verify_oracle(name):
    c = load(name)
    iq2 = c.attrs.get("iq2", 0)
    out, h, part, meta = O.moe_verify(*c.inputs, topk=c.attrs["topk"], iq2=iq2)
    assert rel(out, c.ref) < 1e-2
    P = c.inputs[1].numel()
    U = int(meta[0])
    ids = meta[1:1 + U].tolist()
    assert sorted(set(c.inputs[1].reshape(-1).tolist())) == sorted(ids)
    pm = meta[1 + P:].reshape(P, 8)
    assert int((pm >= 0).sum()) == P


def test_moe_group_meta_layout():
    idx = torch.tensor([[3, 1, 2], [1, 5, 3]], dtype=torch.int32)
    m = O.moe_group_meta(idx, 3)
    P = 6
    assert m[0] == 4 and m[1:5].tolist() == [3, 1, 2, 5] and m[5:7].tolist() == [-1, -1]
    pm = m[1 + P:].reshape(P, 8)
    assert pm[0, :2].tolist() == [0, 5] and pm[1, :2].tolist() == [1, 3]
    assert pm[2, :2].tolist() == [2, -1] and pm[3, :2].tolist() == [-1, 4]


def test_route_ties_lower_index():
    # equal bias-corrected scores: the lower expert index wins (src/bolt_ops.cu:420)
    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    gw = torch.zeros(5, 256, dtype=torch.bfloat16)
    b = torch.tensor([0.1, 0.3, 0.3, 0.2, 0.3])
    idx, w, s = O.moe_route(x, gw, b, 3, 5.0)
    assert idx.tolist() == [[1, 2, 4]]
    assert torch.allclose(w, torch.full((1, 3), 5.0 / 3))


def test_route_topk_exceeds_experts():
    x = torch.randn(1, 256).bfloat16()
    gw = torch.randn(3, 256).bfloat16()
    idx, w, s = O.moe_route(x, gw, torch.zeros(3), 5, 1.0)
    assert idx[0, 3:].tolist() == [-1, -1] and w[0, 3:].tolist() == [0.0, 0.0]


def test_relu2_oracle():
    c = load("relu2")
    (x,) = c.inputs
    assert torch.equal(O.relu2(x).float(), c.ref)  # the reference test demands equality
    # the kernel's fmaxf: NaN and -0 give +0; overflow of the fp32 square gives inf
    s = torch.tensor([float("nan"), -0.0, 0.0, -1e30, 1e30, float("inf"), -float("inf"), 1e-30, 2.5],
                     dtype=torch.bfloat16)
    assert O.relu2(s).float().tolist()[:8] == [0.0, 0.0, 0.0, 0.0, float("inf"), float("inf"), 0.0, 0.0]


@pytest.mark.parametrize("name", case_names("mamba_"))
def test_mamba_oracle(name):
    c = load(name)
    a = c.attrs
    y, cst, sst, _xbc, _ypre = O.mamba_step(*c.inputs, a["heads"], a["head_dim"], a["d_state"], a["n_groups"],
                                            a["epsilon"], a["time_step_min"])
    # the reference test's thresholds (tests/test_bolt_ops.py:305), met here to rounding noise
    assert rel(y, c.ref) < 1e-6
    assert rel(sst[-1], c.extra["ssm"]) < 1e-6
    assert rel(cst[-1].float(), c.extra["conv"]) < 1e-6
