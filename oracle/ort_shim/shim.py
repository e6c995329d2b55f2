"""ctypes front end of the ONNX Runtime stand-in (ort_host.cc) -- TEST INFRASTRUCTURE.

    shim = OrtShim()
    lib = shim.load(path)                        # dlopen + RegisterCustomOps
    shim.ops(lib)                                # [("bolt", "MoeRoute"), ...]
    k = shim.kernel(lib, "MoeRoute", topk=8, scale=5.0)   # ints -> int64, floats -> float attributes
    shapes = shim.run(k, [x, gate_w, bias], [idx, w, scores])   # CUDA tensors; outputs preallocated

Used by the tests (the product's ORT adapter and the reference's own library, both built against
the stand-in header by oracle/ort_shim/build.py) and by bench.py's reference-GPU leg.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(os.path.dirname(HERE), "_ref")

ELEM = {"float32": 1, "uint8": 2, "int32": 6, "float16": 10, "bfloat16": 16}


class OrtError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class OrtShim:
    def __init__(self, host: str = None):
        path = host or os.path.join(REF_DIR, "libort_shim_host.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run python oracle/ort_shim/build.py")
        h = ctypes.CDLL(path)
        P, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        h.ort_shim_last_error.restype = ctypes.c_char_p
        h.ort_shim_load.argtypes = [ctypes.c_char_p]
        h.ort_shim_load.restype = I
        h.ort_shim_list_ops.argtypes = [I, ctypes.c_char_p, I]
        h.ort_shim_op_signature.argtypes = [I, ctypes.c_char_p, ctypes.c_char_p] + [ctypes.POINTER(I)] * 6 + \
            [ctypes.c_char_p, I]
        h.ort_shim_create_kernel.argtypes = [I, ctypes.c_char_p, ctypes.c_char_p, I, ctypes.POINTER(ctypes.c_char_p),
                                             ctypes.POINTER(I), ctypes.POINTER(L), ctypes.POINTER(ctypes.c_float),
                                             ctypes.POINTER(I)]
        h.ort_shim_create_kernel.restype = P
        h.ort_shim_destroy_kernel.argtypes = [P]
        h.ort_shim_compute.argtypes = [P, P, I, ctypes.POINTER(P), ctypes.POINTER(L), ctypes.POINTER(I), I,
                                       ctypes.POINTER(P), ctypes.POINTER(L), ctypes.POINTER(I), ctypes.POINTER(L),
                                       ctypes.POINTER(I)]
        self.h = h

    def error(self) -> str:
        m = self.h.ort_shim_last_error()
        return m.decode() if m else ""

    def load(self, path: str) -> int:
        lib = self.h.ort_shim_load(path.encode())
        if lib < 0:
            raise OrtError(1, self.error())
        return lib

    def ops(self, lib: int):
        buf = ctypes.create_string_buffer(4096)
        n = self.h.ort_shim_list_ops(lib, buf, 4096)
        if n < 0:
            raise OrtError(1, self.error())
        return [tuple(s.split(":", 1)) for s in buf.value.decode().split(";") if s]

    def signature(self, lib: int, name: str, domain: str = "bolt"):
        """(input types, input characteristics, output types, output characteristics, EP type)"""
        n_in, n_out = ctypes.c_int(), ctypes.c_int()
        it, ic, ot, oc = [(ctypes.c_int * 16)() for _ in range(4)]
        ep = ctypes.create_string_buffer(64)
        rc = self.h.ort_shim_op_signature(lib, domain.encode(), name.encode(), ctypes.byref(n_in), it, ic,
                                          ctypes.byref(n_out), ot, oc, ep, 64)
        if rc != 0:
            raise OrtError(rc, self.error())
        return (list(it[:n_in.value]), list(ic[:n_in.value]), list(ot[:n_out.value]), list(oc[:n_out.value]),
                ep.value.decode())

    def kernel(self, lib: int, name: str, domain: str = "bolt", **attrs):
        names = (ctypes.c_char_p * max(1, len(attrs)))(*[k.encode() for k in attrs])
        kinds = (ctypes.c_int * max(1, len(attrs)))(*[1 if isinstance(v, float) else 0 for v in attrs.values()])
        ivals = (ctypes.c_int64 * max(1, len(attrs)))(*[0 if isinstance(v, float) else int(v) for v in attrs.values()])
        fvals = (ctypes.c_float * max(1, len(attrs)))(*[float(v) if isinstance(v, float) else 0.0
                                                        for v in attrs.values()])
        code = ctypes.c_int(0)
        k = self.h.ort_shim_create_kernel(lib, domain.encode(), name.encode(), len(attrs), names, kinds, ivals, fvals,
                                          ctypes.byref(code))
        if not k:
            raise OrtError(code.value, self.error())
        return Kernel(self, k)


class Kernel:
    """One created kernel; run() binds CUDA tensors (inputs, preallocated outputs) and computes
    on the current torch stream (or `stream`, a raw cudaStream_t)."""

    def __init__(self, shim: OrtShim, handle):
        self.shim, self.handle = shim, handle

    def __del__(self):
        try:
            if self.handle:
                self.shim.h.ort_shim_destroy_kernel(self.handle)
        except Exception:
            pass

    def run(self, inputs, outputs, stream=None):
        import torch
        n_in, n_out = len(inputs), len(outputs)
        P = ctypes.c_void_p
        ip = (P * n_in)(*[t.data_ptr() for t in inputs])
        ishape = (ctypes.c_int64 * (8 * n_in))()
        irank = (ctypes.c_int * n_in)()
        for i, t in enumerate(inputs):
            irank[i] = t.dim()
            for d, s in enumerate(t.shape):
                ishape[8 * i + d] = s
        op = (P * n_out)(*[t.data_ptr() for t in outputs])
        caps = (ctypes.c_int64 * n_out)(*[t.numel() * t.element_size() for t in outputs])
        otypes = (ctypes.c_int * n_out)(*[ELEM[str(t.dtype).replace("torch.", "")] for t in outputs])
        oshape = (ctypes.c_int64 * (8 * n_out))()
        orank = (ctypes.c_int * n_out)()
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream if outputs and outputs[0].is_cuda else 0
        rc = self.shim.h.ort_shim_compute(self.handle, P(stream), n_in, ip, ishape, irank, n_out, op, caps, otypes,
                                          oshape, orank)
        if rc != 0:
            raise OrtError(rc, self.shim.error())
        return [tuple(oshape[8 * i:8 * i + orank[i]]) if orank[i] >= 0 else None for i in range(n_out)]
