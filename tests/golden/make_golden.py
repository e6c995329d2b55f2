"""Generate golden fixtures by executing the reference's own torch references.

The reference's test module (``tests/test_bolt_ops.py`` of tianleiwu/nemotron_ops) builds its
expected outputs with CPU torch code and then runs one ORT node on the GPU.  ``onnx`` and
``onnxruntime`` are not installed in the build container, so this script imports the module
with inert stand-ins for those two packages, replaces ``run`` (the ORT call) with a recorder
that returns zeros, and replaces ``rel`` with a recorder of its second argument -- the
reference's expected tensor.  Everything that computes the expected values (the torch
dequantisation, ``gguf.quants.dequantize`` for IQ2_XXS, the MoE rounding loop) is the
reference's own unmodified code.

Usage (build container only; needs the reference checkout and the ``gguf`` package)::

    python tests/golden/make_golden.py --reference DIR    (or BOLT_REFERENCE_DIR=DIR)

Each case becomes ``tests/golden/<name>.npz`` holding the op name, attributes, inputs,
the reference output (``ref``) and, for native IQ2_XXS GEMVs, gguf's fp32 weights
(``gguf_deq``).  bf16 tensors are stored as their uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_stand_ins():
    onnx = types.ModuleType("onnx")

    class TensorProto:  # element-type tags read at import time (test_bolt_ops.py:16)
        FLOAT, UINT8, INT32, BFLOAT16 = 1, 2, 6, 16

    onnx.TensorProto = TensorProto
    helper = types.ModuleType("onnx.helper")
    onnx.helper = helper
    sys.modules.setdefault("onnx", onnx)
    sys.modules.setdefault("onnx.helper", helper)
    sys.modules.setdefault("onnxruntime", types.ModuleType("onnxruntime"))


def load_reference_tests(ref_dir: str):
    _install_stand_ins()
    path = os.path.join(ref_dir, "tests", "test_bolt_ops.py")
    spec = importlib.util.spec_from_file_location("reference_test_bolt_ops", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.DEV = "cpu"
    return mod


class Recorder:
    def __init__(self, mod):
        self.mod = mod
        self.calls = []
        self.refs = []
        self.deq = []
        orig_native = mod.iq2_native_dequant

        def run(op, inputs, out_types, attrs=None):
            self.calls.append((op, [(n, t.detach().clone()) for n, t in inputs], dict(attrs or {})))
            return self._fake_outputs(op, inputs, attrs or {})

        def rel(a, b):
            self.refs.append(b.detach().clone())
            return 0.0

        def native(blk):
            out = orig_native(blk)
            self.deq.append(out.detach().clone())
            return out

        mod.run, mod.rel, mod.iq2_native_dequant = run, rel, native
        # test_relu2 checks with torch.equal(y, ref) instead of rel: the module's torch is
        # replaced by a forwarder whose equal() records its second argument as well
        recorder = self

        class TorchForwarder:
            def __getattr__(self, name):
                return getattr(torch, name)

            @staticmethod
            def equal(a, b):
                recorder.refs.append(b.detach().clone())
                return True

        mod.torch = TorchForwarder()

    @staticmethod
    def _fake_outputs(op, inputs, attrs):
        x = inputs[0][1]
        if op in ("Nvfp4Gemv", "Q8Gemv", "Q4Gemv"):
            return [torch.zeros(x.shape[0], inputs[1][1].shape[0], dtype=torch.bfloat16)]
        if op == "MoeRoute":
            R, E, k = x.shape[0], inputs[1][1].shape[0], attrs["topk"]
            return [torch.zeros(R, k, dtype=torch.int32), torch.zeros(R, k), torch.zeros(R, E)]
        if op == "Relu2":
            return [torch.zeros_like(x)]
        if op == "MambaStep":
            R, heads, hd, ds, ng = x.shape[0], attrs["heads"], attrs["head_dim"], attrs["d_state"], attrs["n_groups"]
            di = heads * hd
            cd = di + 2 * ng * ds
            return [torch.zeros(R, di, dtype=torch.bfloat16), torch.zeros_like(inputs[1][1]),
                    torch.zeros_like(inputs[2][1]), torch.zeros(R, cd, dtype=torch.bfloat16), torch.zeros(R, di)]
        R = x.shape[0]
        return [torch.zeros(R, 1024, dtype=torch.bfloat16)]

    def take(self):
        c, r, d = self.calls, self.refs, self.deq
        self.calls, self.refs, self.deq = [], [], []
        return c, r, d


def _to_np(t: torch.Tensor):
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.uint16).numpy(), "bfloat16"
    return t.contiguous().numpy(), str(t.dtype).replace("torch.", "")


def save_case(name, op, inputs, attrs, ref, deq=None, meta=None, extra=None):
    arrays, dtypes, names = {}, {}, []
    for n, t in inputs:
        a, dt = _to_np(t)
        arrays["in_" + n] = a
        dtypes[n] = dt
        names.append(n)
    arrays["ref"] = ref.to(torch.float32).numpy()
    if deq is not None:
        arrays["gguf_deq"] = deq.to(torch.float32).numpy()
    for k, t in (extra or {}).items():
        arrays["ref_" + k] = t.to(torch.float32).numpy()
    info = {"op": op, "attrs": attrs, "inputs": names, "dtypes": dtypes, **(meta or {})}
    arrays["info"] = np.frombuffer(json.dumps(info).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


# (test function name, kwargs, fixture name); shapes are small versions of the reference's
# own test shapes, chosen to satisfy each op's constraints and to cover the R dispatch.
CASES = [
    ("test_nvfp4", dict(R=1, N=64, K=1024), "nvfp4_r1"),
    ("test_nvfp4", dict(R=2, N=32, K=2048), "nvfp4_r2"),
    ("test_nvfp4", dict(R=8, N=48, K=1024), "nvfp4_r8"),
    ("test_nvfp4", dict(R=1, N=32, K=1024, XSCALE=3000.0), "nvfp4_r1_massive"),
    ("test_nvfp4", dict(R=8, N=32, K=1024, XSCALE=3000.0), "nvfp4_r8_massive"),
    ("test_qgemv", dict(bits=8, R=1, N=64, K=1024), "q8_r1"),
    ("test_qgemv", dict(bits=8, R=3, N=40, K=512), "q8_r3"),
    ("test_qgemv", dict(bits=8, R=8, N=32, K=256), "q8_r8"),
    ("test_qgemv", dict(bits=8, R=5, N=24, K=96), "q8_r5_k96"),
    ("test_qgemv", dict(bits=4, R=1, N=64, K=1024), "q4_r1"),
    ("test_qgemv", dict(bits=4, R=4, N=48, K=512), "q4_r4"),
    ("test_qgemv", dict(bits=4, R=8, N=32, K=256), "q4_r8"),
    ("test_qgemv", dict(bits=4, R=6, N=24, K=160), "q4_r6_k160"),
    ("test_q4_iq2", dict(R=2, N=32, K=512), "q4_iq2lut_r2"),
    ("test_q4_iq2", dict(R=8, N=48, K=256), "q4_iq2lut_r8"),
    ("test_q4_iq2", dict(R=5, N=16, K=384), "q4_iq2lut_r5"),
    ("test_q4_iq2_native", dict(R=1, N=32, K=512), "q4_iq2n_r1"),
    ("test_q4_iq2_native", dict(R=3, N=24, K=256), "q4_iq2n_r3"),
    ("test_q4_iq2_native", dict(R=8, N=40, K=768), "q4_iq2n_r8"),
    ("test_route", dict(R=1, E=24, topk=4, K=256), "route_r1"),
    ("test_route", dict(R=4, E=40, topk=9, K=512), "route_r4"),
    ("test_route", dict(R=8, E=33, topk=6, K=256), "route_r8"),
    ("test_moe_decode", dict(R=1, E=8, I=64, topk=3), "moe_decode_r1"),
    ("test_moe_decode", dict(R=2, E=6, I=96, topk=4), "moe_decode_r2"),
    ("test_moe_decode", dict(R=3, E=8, I=64, topk=4, op="MoeVerify"), "moe_verify_r3"),
    ("test_moe_decode", dict(R=8, E=4, I=128, topk=3, op="MoeVerify"), "moe_verify_r8_shared"),
    ("test_moe_iq2", dict(R=4, E=6, I=128, topk=3), "moe_verify_iq2lut_r4"),
    ("test_moe_iq2_native", dict(R=2, E=5, I=256, topk=3), "moe_verify_iq2n_r2"),
    ("test_moe_iq2_native", dict(R=8, E=3, I=256, topk=2), "moe_verify_iq2n_r8_shared"),
    ("test_relu2", dict(), "relu2"),  # the reference's own shape (3, 1000); unseeded there: seed 0 here
    # MambaStep: 16 heads in 4 groups keep the fixtures small (the kernels' head_dim 64, d_state 128)
    ("test_mamba", dict(R=1, heads=16, ng=4), "mamba_r1"),
    ("test_mamba", dict(R=5, heads=16, ng=4), "mamba_r5"),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BOLT_REFERENCE_DIR"),
                    help="checkout of tianleiwu/nemotron_ops (or set BOLT_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("the reference checkout is required: pass --reference DIR or set BOLT_REFERENCE_DIR")
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    mod = load_reference_tests(args.reference)
    rec = Recorder(mod)
    for fn, kw, name in CASES:
        if fn == "test_relu2":
            torch.manual_seed(0)
        try:
            getattr(mod, fn)(**kw)
        except AssertionError:
            pass  # test_route compares against the recorder's zero outputs; the expected values are captured
        calls, refs, deqs = rec.take()
        assert len(calls) == 1 and refs, (name, len(calls), len(refs))
        op, inputs, attrs = calls[0]
        deq = deqs[0] if (deqs and op == "Q4Gemv") else None
        # test_mamba checks y, then the ssm state, then the conv state (tests/test_bolt_ops.py:304-305)
        extra = {"ssm": refs[1], "conv": refs[2]} if op == "MambaStep" else None
        save_case(name, op, inputs, attrs, refs[0], deq, {"test": fn, "kwargs": kw}, extra)
        print(f"{name:28s} {op:10s} ref{tuple(refs[0].shape)}")


if __name__ == "__main__":
    main()
