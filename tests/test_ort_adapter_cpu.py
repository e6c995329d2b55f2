"""The ORT adapter's registration, checked on CPU through the ONNX Runtime stand-in
(oracle/ort_shim): RegisterCustomOps must register domain "bolt" with the reference's op set and
signatures (src/bolt_ops.cu:1469-1625), and kernel creation must fail the way the reference's does.
No kernel runs here (tests/test_gpu_ort_adapter.py runs them on a GPU).
"""
import os

import pytest

from oracle.ort_shim import build as shim_build
from oracle.ort_shim.shim import OrtError, OrtShim

BF, F32, U8, I32 = 16, 1, 2, 6
# (name, input types, output types) in the reference's registration order (src/bolt_ops.cu:1489-1589, :1598-1618)
REFERENCE_OPS = [
    ("MambaStep", [BF, BF, F32, BF, BF, F32, F32, F32, F32], [BF, BF, F32, BF, F32]),
    ("MambaVerify", [BF, BF, F32, BF, BF, F32, F32, F32, F32, I32], [BF, BF, F32, BF, F32]),
    ("MoeRoute", [BF, BF, F32], [I32, F32, F32]),
    ("MoeDecode", [BF, I32, F32, U8, BF, U8, BF], [BF, BF, F32]),
    ("MoeVerify", [BF, I32, F32, U8, BF, U8, BF], [BF, BF, F32, I32]),
    ("Relu2", [BF], [BF]),
    ("Nvfp4Gemv", [BF, U8, U8, F32], [BF]),
    ("Q8Gemv", [BF, U8, BF], [BF]),
    ("Q4Gemv", [BF, U8, BF], [BF]),
]


@pytest.fixture(scope="module")
def built():
    return shim_build.build(reference=False)


@pytest.fixture(scope="module")
def shim(built):
    return OrtShim(built["host"])


@pytest.fixture(scope="module")
def adapter(shim, built):
    return shim.load(built["adapter"])


def table(shim, lib):
    out = []
    for domain, name in shim.ops(lib):
        it, ic, ot, oc, ep = shim.signature(lib, name, domain)
        out.append((domain, name, it, ot, ep, set(ic) | set(oc)))
    return out


def test_registers_the_reference_op_set(shim, adapter):
    got = table(shim, adapter)
    assert [(d, n) for d, n, *_ in got] == [("bolt", n) for n, _, _ in REFERENCE_OPS]
    for (d, name, it, ot, ep, chars), (rname, rit, rot) in zip(got, REFERENCE_OPS):
        assert (it, ot) == (rit, rot), name
        assert ep == "CUDAExecutionProvider"
        assert chars == {0}  # every input and output INPUT_OUTPUT_REQUIRED


def test_registration_matches_the_reference_library(shim, adapter, built):
    ref = built.get("reference") or os.path.join(shim_build.OUT, "libbolt_ref.so")
    if not os.path.exists(ref):
        pytest.skip("the reference's library was not built here (needs its checkout)")
    assert table(shim, shim.load(ref)) == table(shim, adapter)


def test_registering_twice_is_harmless(shim, built):
    # the ops are registered once (std::call_once) and the same domain is added again
    lib = shim.load(built["adapter"])
    assert [n for _, n in shim.ops(lib)] == [n for n, _, _ in REFERENCE_OPS]


@pytest.mark.parametrize("name,attrs", [("MoeRoute", {"topk": 8}), ("MoeDecode", {}), ("MoeVerify", {}),
                                        ("MambaStep", {"heads": 4, "head_dim": 64, "d_state": 128})])
def test_missing_attribute_is_invalid_argument(shim, adapter, name, attrs):
    with pytest.raises(OrtError) as e:
        shim.kernel(adapter, name, **attrs)
    assert e.value.code == 2  # ORT_INVALID_ARGUMENT, as the reference's CreateKernelV2 (src/bolt_ops.cu:1477)


def test_unsupported_mamba_dims_are_rejected_at_creation(shim, adapter):
    with pytest.raises(OrtError) as e:
        shim.kernel(adapter, "MambaStep", heads=4, head_dim=32, d_state=128, n_groups=1, epsilon=1e-5,
                    time_step_min=0.001)
    assert e.value.code == 2
    assert "only head_dim=64, d_state=128" in e.value.msg


def test_optional_iq2_defaults_to_zero(shim, adapter):
    # Q4Gemv / MoeVerify read iq2 when present and default to 0 (src/bolt_ops.cu:1170-1176)
    shim.kernel(adapter, "Q4Gemv")
    shim.kernel(adapter, "Q4Gemv", iq2=2)
    shim.kernel(adapter, "MoeVerify", topk=8)
    shim.kernel(adapter, "Q8Gemv")
    shim.kernel(adapter, "MoeRoute", topk=8, scale=5.0)
