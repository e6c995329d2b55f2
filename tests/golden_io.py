"""Load the golden fixtures written by tests/golden/make_golden.py."""
from __future__ import annotations

import glob
import json
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

_DT = {"bfloat16": torch.bfloat16, "float32": torch.float32, "uint8": torch.uint8, "int32": torch.int32,
       "int16": torch.int16, "float16": torch.float16}


class Case:
    def __init__(self, path):
        self.name = os.path.splitext(os.path.basename(path))[0]
        z = np.load(path)
        self.info = json.loads(bytes(z["info"]).decode())
        self.op = self.info["op"]
        self.attrs = self.info["attrs"]
        self.inputs = []
        for n in self.info["inputs"]:
            a = z["in_" + n]
            dt = self.info["dtypes"][n]
            t = torch.from_numpy(a.copy())
            if dt == "bfloat16":
                t = t.view(torch.bfloat16)
            else:
                t = t.to(_DT[dt])
            self.inputs.append(t)
        self.ref = torch.from_numpy(z["ref"].copy())
        self.gguf_deq = torch.from_numpy(z["gguf_deq"].copy()) if "gguf_deq" in z.files else None
        # further expected tensors of a case (e.g. MambaStep's ssm and conv states)
        self.extra = {k[4:]: torch.from_numpy(z[k].copy()) for k in z.files if k.startswith("ref_")}

    def __repr__(self):
        return f"Case({self.name})"


def cases(prefix: str = ""):
    paths = sorted(glob.glob(os.path.join(GOLDEN_DIR, prefix + "*.npz")))
    return [Case(p) for p in paths]


def case_names(prefix: str = ""):
    return [os.path.splitext(os.path.basename(p))[0] for p in sorted(glob.glob(os.path.join(GOLDEN_DIR, prefix + "*.npz")))]


def load(name: str) -> Case:
    return Case(os.path.join(GOLDEN_DIR, name + ".npz"))


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    """Relative Frobenius error, as the reference tests use (tests/test_bolt_ops.py:63-65)."""
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
