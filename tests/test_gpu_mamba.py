"""GPU parity of MambaStep / MambaVerify (CUDA path through the C ABI): against the reference
test's own expected tensors (tests/golden/mamba_*.npz) with its thresholds
(tests/test_bolt_ops.py:305, :336-338), and against the oracle at the reference test's full size."""
import pytest
import torch

import oracle as O
from golden_io import case_names, load, rel
from nemotron_ops_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATTRS = dict(head_dim=64, d_state=128, epsilon=1e-5, time_step_min=0.001)


def _inputs(R, rows, heads, ng, seed):
    """Inputs shaped and scaled as the reference test builds them (tests/test_bolt_ops.py:265-276)."""
    g = torch.Generator().manual_seed(seed)
    di = heads * 64
    cd = di + 2 * ng * 128
    t = [(torch.randn(R, di + cd + heads, generator=g) * 0.7).bfloat16(),
         (torch.randn(rows, cd, 3, generator=g) * 0.5).bfloat16(),
         torch.randn(rows, heads, 128, 64, generator=g) * 0.1,
         (torch.randn(cd, 1, 4, generator=g) * 0.3).bfloat16(),
         (torch.randn(cd, generator=g) * 0.1).bfloat16(),
         torch.randn(heads, generator=g) * 0.3,
         -torch.rand(heads, generator=g) * 4 - 0.1,
         torch.randn(heads, generator=g),
         torch.rand(di, generator=g) + 0.5]
    return [x.to(DEV) for x in t]


def _check_against_oracle(outs, ref, R):
    y, cs_o, ss_o, xbc, ypre = outs
    oy, ocs, oss, oxbc, oypre = ref
    assert rel(y, oy) < 1e-2
    # the conv output is rounded to bf16: fp32 summation order may move it by one bf16 ulp
    d = (xbc.float() - oxbc.float()).abs()
    assert bool((d <= oxbc.float().abs() * 2.0 ** -7 + 1e-6).all())
    assert rel(ypre, oypre) < 1e-4
    return cs_o, ss_o, ocs, oss


@pytest.mark.parametrize("name", case_names("mamba_"))
def test_mamba_golden(name):
    c = load(name)
    a = c.attrs
    ins = [t.to(DEV) for t in c.inputs]
    y, cs_o, ss_o, _xbc, _ypre = ops.MambaStep(*ins, a["heads"], a["head_dim"], a["d_state"], a["n_groups"],
                                               a["epsilon"], a["time_step_min"])
    assert rel(y, c.ref) < 1e-2
    assert rel(ss_o[0], c.extra["ssm"]) < 1e-4
    assert rel(cs_o[0].float(), c.extra["conv"]) < 1e-6
    assert ops.device_status() == 0


@pytest.mark.parametrize("R", [1, 2, 8, 16])
def test_mamba_step_full_size(R):
    heads, ng = 128, 8
    ins = _inputs(R, 1, heads, ng, seed=R)
    outs = ops.MambaStep(*ins, heads=heads, n_groups=ng, **ATTRS)
    ref = O.mamba_step(*ins, heads=heads, n_groups=ng, **ATTRS)
    cs_o, ss_o, ocs, oss = _check_against_oracle(outs, ref, R)
    assert rel(ss_o[0], oss[-1]) < 1e-4
    assert torch.equal(cs_o[0], ocs[-1])
    assert ops.device_status() == 0


def test_mamba_verify_matches_steps():
    # the reference test's protocol (tests/test_bolt_ops.py:308-338): every row's state equals the
    # state of single-token steps run from row sel, and y matches those steps' outputs
    R, sel, heads, ng = 8, 3, 128, 8
    ins = _inputs(R, R, heads, ng, seed=7)
    sel_t = torch.tensor([sel], dtype=torch.int32, device=DEV)
    y_v, cs_all, ss_all, _, _ = ops.MambaVerify(*ins, sel_t, heads=heads, n_groups=ng, **ATTRS)
    st_conv, st_ssm = ins[1][sel:sel + 1].clone(), ins[2][sel:sel + 1].clone()
    ys = []
    for r in range(R):
        one = [ins[0][r:r + 1], st_conv, st_ssm] + ins[3:]
        y, st_conv, st_ssm, _, _ = ops.MambaStep(*one, heads=heads, n_groups=ng, **ATTRS)
        ys.append(y)
        assert rel(ss_all[r], st_ssm[0]) < 1e-5 and rel(cs_all[r].float(), st_conv[0].float()) < 1e-6, r
    assert rel(y_v, torch.cat(ys)) < 1e-4
    # and against the oracle from row sel
    ref = O.mamba_step(*ins, heads=heads, n_groups=ng, sel=sel, **ATTRS)
    cs_o, ss_o, ocs, oss = _check_against_oracle((y_v, cs_all, ss_all, *ops.MambaVerify(
        *ins, sel_t, heads=heads, n_groups=ng, **ATTRS)[3:]), ref, R)
    for r in range(R):
        assert rel(ss_o[r], oss[r]) < 1e-4 and torch.equal(cs_o[r], ocs[r]), r
    assert ops.device_status() == 0


def test_mamba_verify_sel_outside_the_buffer_writes_nothing():
    R, heads, ng = 2, 16, 4
    ins = _inputs(R, 2, heads, ng, seed=3)
    assert ops.device_status() == 0
    y, *_ = ops.MambaVerify(*ins, torch.tensor([5], dtype=torch.int32, device=DEV), heads=heads, n_groups=ng,
                            **ATTRS)
    assert ops.device_status() == 1 << 6
