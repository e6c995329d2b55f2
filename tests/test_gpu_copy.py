"""bolt_memcpy_async (ops.copy_async): host <-> device copies ordered on the current stream."""
import pytest
import torch

from nemotron_ops_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 8192, 1 << 20])
def test_copy_async_round_trip(n):
    src = torch.randint(0, 255, (n,), dtype=torch.uint8).pin_memory()
    dev = torch.empty(n, dtype=torch.uint8, device="cuda")
    back = torch.zeros(n, dtype=torch.uint8).pin_memory()
    ops.copy_async(dev, src)
    dev2 = dev.clone()  # device-to-device through the same entry
    ops.copy_async(dev, torch.zeros_like(dev))
    ops.copy_async(dev, dev2)
    ops.copy_async(back, dev)
    torch.cuda.synchronize()
    assert torch.equal(back, src)


def test_copy_async_rejects_size_mismatch():
    with pytest.raises(RuntimeError):
        ops.copy_async(torch.empty(4, device="cuda"), torch.empty(5).pin_memory())
