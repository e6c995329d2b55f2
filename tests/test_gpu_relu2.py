"""GPU parity of Relu2 (CUDA path through the C ABI) against the oracle: bit-exact, as the
reference's own test demands (tests/test_bolt_ops.py:99-104)."""
import pytest
import torch

import oracle as O
from golden_io import load
from nemotron_ops_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _check(x):
    y = ops.Relu2(x)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    ref = O.relu2(x.cpu())
    assert torch.equal(y.cpu().view(torch.int16), ref.view(torch.int16))


def test_relu2_golden():
    c = load("relu2")
    y = ops.Relu2(c.inputs[0].to(DEV))
    assert torch.equal(y.cpu().float(), c.ref)


@pytest.mark.parametrize("shape", [(3, 1000), (1,), (7,), (8,), (9,), (1023,), (4097,), (2, 3, 5, 7), (),
                                   (1 << 24) + 3])
def test_relu2_shapes(shape):
    shape = shape if isinstance(shape, tuple) else (shape,)
    g = torch.Generator(device=DEV).manual_seed(sum(shape) + 1)
    _check((torch.randn(shape, generator=g, device=DEV) * 3).to(torch.bfloat16))


def test_relu2_every_bf16_value():
    # all 65536 bit patterns: NaNs, infinities, -0, subnormals, the largest finite values
    x = torch.arange(-32768, 32768, dtype=torch.int32, device=DEV).to(torch.int16).view(torch.bfloat16)
    _check(x.contiguous())


def test_relu2_unaligned_input():
    base = (torch.randn(4099, device=DEV) * 3).to(torch.bfloat16)
    _check(base[1:])  # 2-byte offset: the element-by-element path
    _check(base[8:])  # 16-byte offset: the vector path


def test_relu2_empty():
    y = ops.Relu2(torch.empty(0, 5, dtype=torch.bfloat16, device=DEV))
    assert y.shape == (0, 5)
