"""The bolt ops on torch CUDA tensors -- a host-side mirror of the reference's ORT ops.

Each function is one node of the reference's custom-op domain ``bolt`` (src/bolt_ops.cu:1469-1589):
same name, inputs in the same order, same attributes, and outputs allocated in the shapes the
reference's ``ComputeV2`` allocates.  The work runs on the current torch CUDA stream through
libbolt_b200.so; there is no CPU path.  A failing shape check raises ``RuntimeError`` with the
reference's message (the reference returns ORT_FAIL with the same text).
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import last_error, lib, shape_arg

__all__ = ["Nvfp4Gemv", "Q8Gemv", "Q4Gemv", "MoeRoute", "MoeDecode", "MoeVerify", "moe_verify_shard",
           "f32_to_bf16", "copy_async", "dequant", "set_launch_options", "device_status", "FMT_Q8", "FMT_Q4", "FMT_NVFP4",
           "FMT_IQ2_LUT", "FMT_IQ2_NATIVE"]

FMT_Q8, FMT_Q4, FMT_NVFP4, FMT_IQ2_LUT, FMT_IQ2_NATIVE = 0, 1, 2, 3, 4


def _ptr(t):
    # plain ints: ctypes converts them for c_void_p parameters without a wrapper object per call
    return t.data_ptr() if t is not None else None


def _stream(t):
    # the raw cudaStream_t of torch's current stream on t's device (as current_stream().cuda_stream)
    return torch._C._cuda_getCurrentRawStream(t.device.index)


def _need(*tensors):
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("bolt ops take CUDA tensors (there is no CPU implementation)")
        if not t.is_contiguous():
            raise RuntimeError("bolt ops take contiguous tensors")


def _check(rc):
    if rc != 0:
        raise RuntimeError(last_error())


def set_launch_options(pdl: bool = True, early_weights: bool = False, smem_budget: int = 0) -> None:
    """Process-wide launch options (see bolt_set_launch_options in include/bolt_b200.h); the
    defaults are the library's own (programmatic dependent launch on, early weights off)."""
    _check(lib().bolt_set_launch_options(int(pdl), int(early_weights), int(smem_budget)))


def device_status() -> int:
    """Read and clear the device status word of the current device (0 = no kernel gave up)."""
    v = ctypes.c_uint(0)
    _check(lib().bolt_get_device_status(ctypes.byref(v)))
    return v.value


def Nvfp4Gemv(x, w, w_scale, g):
    """y[..., N] = bf16(g * x @ (e2m1 * e4m3)^T); w u8 [N, K/2], w_scale u8 [N, K/16], g f32 [1]."""
    _need(x, w, w_scale, g)
    y = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.bfloat16, device=x.device)
    xs, _k1 = shape_arg(x.shape)
    ws, _k2 = shape_arg(w.shape)
    _check(lib().bolt_nvfp4_gemv(_ptr(x), xs, x.dim(), _ptr(w), ws, w.dim(), _ptr(w_scale), _ptr(g), _ptr(y),
                                 _stream(x)))
    return y


def Q8Gemv(x, B, scales):
    """y[..., N] = x @ W^T, W = (B - 128) * s; B u8 [N, K/32, 32], scales bf16 [N, K/32]."""
    _need(x, B, scales)
    y = torch.empty(*x.shape[:-1], B.shape[0], dtype=torch.bfloat16, device=x.device)
    xs, _k1 = shape_arg(x.shape)
    bs, _k2 = shape_arg(B.shape)
    _check(lib().bolt_q8_gemv(_ptr(x), xs, x.dim(), _ptr(B), bs, B.dim(), _ptr(scales), _ptr(y), _stream(x)))
    return y


def Q4Gemv(x, B, scales, iq2: int = 0):
    """int4 (iq2=0), IQ2_XXS LUT codes (iq2=1) or native IQ2_XXS records (iq2=2)."""
    _need(x, B, scales)
    y = torch.empty(*x.shape[:-1], B.shape[0], dtype=torch.bfloat16, device=x.device)
    xs, _k1 = shape_arg(x.shape)
    bs, _k2 = shape_arg(B.shape)
    _check(lib().bolt_q4_gemv(_ptr(x), xs, x.dim(), _ptr(B), bs, B.dim(), _ptr(scales), int(iq2), _ptr(y),
                              _stream(x)))
    return y


def MoeRoute(x, gate_w, bias, topk: int, scale: float):
    """Returns (idx i32 [R, topk], w f32 [R, topk], scores f32 [R, E])."""
    _need(x, gate_w, bias)
    R, E = x.shape[0], gate_w.shape[0]
    idx = torch.empty(R, topk, dtype=torch.int32, device=x.device)
    w = torch.empty(R, topk, dtype=torch.float32, device=x.device)
    scores = torch.empty(R, E, dtype=torch.float32, device=x.device)
    xs, _k1 = shape_arg(x.shape)
    gs, _k2 = shape_arg(gate_w.shape)
    _check(lib().bolt_moe_route(_ptr(x), xs, x.dim(), _ptr(gate_w), gs, gate_w.dim(), _ptr(bias), int(topk),
                                float(scale), _ptr(idx), _ptr(w), _ptr(scores), _stream(x)))
    return idx, w, scores


def _moe_outputs(z, fc1_w, topk):
    R = z.shape[0]
    I = fc1_w.shape[1]
    P = R * topk
    out = torch.empty(R, 1024, dtype=torch.bfloat16, device=z.device)
    h = torch.empty(P, I, dtype=torch.bfloat16, device=z.device)
    part = torch.empty(P, 1024, dtype=torch.float32, device=z.device)
    return out, h, part


def MoeDecode(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int):
    """Returns (out bf16 [R, 1024], h bf16 [R*topk, I], part f32 [R*topk, 1024])."""
    _need(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s)
    out, h, part = _moe_outputs(z, fc1_w, topk)
    zs, _k1 = shape_arg(z.shape)
    w1s, _k2 = shape_arg(fc1_w.shape)
    _check(lib().bolt_moe_decode(_ptr(z), zs, z.dim(), _ptr(idx), _ptr(w), _ptr(fc1_w), w1s, fc1_w.dim(),
                                 _ptr(fc1_s), _ptr(fc2_w), _ptr(fc2_s), int(topk), _ptr(out), _ptr(h), _ptr(part),
                                 _stream(z)))
    return out, h, part


def MoeVerify(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, iq2: int = 0):
    """Returns (out, h, part, meta i32 [1 + P + 8P])."""
    _need(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s)
    out, h, part = _moe_outputs(z, fc1_w, topk)
    P = z.shape[0] * topk
    meta = torch.empty(1 + P + 8 * P, dtype=torch.int32, device=z.device)
    zs, _k1 = shape_arg(z.shape)
    w1s, _k2 = shape_arg(fc1_w.shape)
    _check(lib().bolt_moe_verify(_ptr(z), zs, z.dim(), _ptr(idx), _ptr(w), _ptr(fc1_w), w1s, fc1_w.dim(),
                                 _ptr(fc1_s), _ptr(fc2_w), _ptr(fc2_s), int(topk), int(iq2), _ptr(out), _ptr(h),
                                 _ptr(part), _ptr(meta), _stream(z)))
    return out, h, part, meta


def _expert_ptr(t, e_begin: int):
    """Device address of expert 0 for a tensor holding experts [e_begin, ...) only (the kernels
    read experts >= e_begin exclusively, so the shifted base is never dereferenced below them)."""
    return ctypes.c_void_p(t.data_ptr() - int(e_begin) * t[0].numel() * t.element_size())


def moe_verify_shard(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, iq2: int, e_begin: int, e_end: int,
                     num_experts: int = None, out_partial=None, outputs=None):
    """MoeVerify over experts [e_begin, e_end) only; returns (out_partial f32 [R, 1024], h, part, meta).

    The weight tensors hold either all ``num_experts`` experts, or only the local experts
    [e_begin, e_end) (then ``num_experts`` gives the global count).  Rows of h / part of
    non-local pairs are left untouched.
    """
    _need(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s)
    R = z.shape[0]
    P = R * topk
    E = int(num_experts) if num_experts is not None else fc1_w.shape[0]
    local = fc1_w.shape[0] != E
    if local and fc1_w.shape[0] != e_end - e_begin:
        raise RuntimeError("moe_verify_shard: local weights must hold exactly experts [e_begin, e_end)")
    if outputs is None:
        _, h, part = _moe_outputs(z, fc1_w, topk)
        meta = torch.empty(1 + P + 8 * P, dtype=torch.int32, device=z.device)
    else:
        h, part, meta = outputs
    if out_partial is None:
        out_partial = torch.empty(R, 1024, dtype=torch.float32, device=z.device)
    zs, _k1 = shape_arg(z.shape)
    w1s, _k2 = shape_arg((E,) + tuple(fc1_w.shape[1:]))
    wp = [_expert_ptr(t, e_begin) if local else _ptr(t) for t in (fc1_w, fc1_s, fc2_w, fc2_s)]
    _check(lib().bolt_moe_verify_shard(_ptr(z), zs, z.dim(), _ptr(idx), _ptr(w), wp[0], w1s, fc1_w.dim(),
                                       wp[1], wp[2], wp[3], int(topk), int(iq2), int(e_begin), int(e_end),
                                       ctypes.c_void_p(0), _ptr(h), _ptr(part), _ptr(meta), _ptr(out_partial),
                                       _stream(z)))
    return out_partial, h, part, meta


def moe_verify_shard_allreduce(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, iq2: int, e_begin: int,
                               e_end: int, reducer, num_experts: int = None, out=None, outputs=None):
    """Expert-sharded MoeVerify whose last kernel also sums every rank's partial through peer
    memory (``reducer``: a :class:`nemotron_ops_b200.sharded.PeerReducer`); returns out bf16
    [R, 1024], identical on every rank.  Weights and ``outputs`` as for :func:`moe_verify_shard`."""
    _need(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s)
    R = z.shape[0]
    P = R * topk
    E = int(num_experts) if num_experts is not None else fc1_w.shape[0]
    local = fc1_w.shape[0] != E
    if local and fc1_w.shape[0] != e_end - e_begin:
        raise RuntimeError("moe_verify_shard_allreduce: local weights must hold exactly experts [e_begin, e_end)")
    if outputs is None:
        _, h, part = _moe_outputs(z, fc1_w, topk)
        meta = torch.empty(1 + P + 8 * P, dtype=torch.int32, device=z.device)
    else:
        h, part, meta = outputs
    if out is None:
        out = torch.empty(R, 1024, dtype=torch.bfloat16, device=z.device)
    zs, _k1 = shape_arg(z.shape)
    w1s, _k2 = shape_arg((E,) + tuple(fc1_w.shape[1:]))
    wp = [_expert_ptr(t, e_begin) if local else _ptr(t) for t in (fc1_w, fc1_s, fc2_w, fc2_s)]
    _check(lib().bolt_moe_verify_shard_allreduce(
        _ptr(z), zs, z.dim(), _ptr(idx), _ptr(w), wp[0], w1s, fc1_w.dim(), wp[1], wp[2], wp[3], int(topk), int(iq2),
        int(e_begin), int(e_end), _ptr(h), _ptr(part), _ptr(meta), ctypes.c_void_p(reducer.bufs_dev),
        _ptr(reducer.counters), int(reducer.half), int(reducer.rank), int(reducer.world), _ptr(out), _stream(z)))
    return out


def moe_decode_shard(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, e_begin: int, e_end: int,
                     num_experts: int = None, out_partial=None, outputs=None):
    """MoeDecode over experts [e_begin, e_end) only; returns (out_partial f32 [R, 1024], h, part).

    Weight tensors as for :func:`moe_verify_shard` (all experts, or only the local ones with
    ``num_experts`` giving the global count).  Requires I % 256 == 0.
    """
    _need(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s)
    R = z.shape[0]
    E = int(num_experts) if num_experts is not None else fc1_w.shape[0]
    local = fc1_w.shape[0] != E
    if local and fc1_w.shape[0] != e_end - e_begin:
        raise RuntimeError("moe_decode_shard: local weights must hold exactly experts [e_begin, e_end)")
    if outputs is None:
        _, h, part = _moe_outputs(z, fc1_w, topk)
    else:
        h, part = outputs
    if out_partial is None:
        out_partial = torch.empty(R, 1024, dtype=torch.float32, device=z.device)
    zs, _k1 = shape_arg(z.shape)
    w1s, _k2 = shape_arg((E,) + tuple(fc1_w.shape[1:]))
    wp = [_expert_ptr(t, e_begin) if local else _ptr(t) for t in (fc1_w, fc1_s, fc2_w, fc2_s)]
    _check(lib().bolt_moe_decode_shard(_ptr(z), zs, z.dim(), _ptr(idx), _ptr(w), wp[0], w1s, fc1_w.dim(),
                                       wp[1], wp[2], wp[3], int(topk), int(e_begin), int(e_end), ctypes.c_void_p(0),
                                       _ptr(h), _ptr(part), _ptr(out_partial), _stream(z)))
    return out_partial, h, part


def _mamba(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, sel, heads, head_dim,
           d_state, n_groups, epsilon, time_step_min):
    tensors = [proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w]
    _need(*tensors + ([sel] if sel is not None else []))
    R = proj.shape[0]
    di = heads * head_dim
    cd = di + 2 * n_groups * d_state
    dev = proj.device
    y = torch.empty(R, di, dtype=torch.bfloat16, device=dev)
    conv_out = torch.empty_like(conv_state)
    ssm_out = torch.empty_like(ssm_state)
    xbc = torch.empty(R, cd, dtype=torch.bfloat16, device=dev)
    ypre = torch.empty(R, di, dtype=torch.float32, device=dev)
    ps, _k1 = shape_arg(proj.shape)
    cs, _k2 = shape_arg(conv_state.shape)
    ss, _k3 = shape_arg(ssm_state.shape)
    head = [_ptr(proj), ps, proj.dim(), _ptr(conv_state), cs, conv_state.dim(), _ptr(ssm_state), ss,
            ssm_state.dim()] + [_ptr(t) for t in tensors[3:]]
    tail = [int(heads), int(head_dim), int(d_state), int(n_groups), float(epsilon), float(time_step_min), _ptr(y),
            _ptr(conv_out), _ptr(ssm_out), _ptr(xbc), _ptr(ypre), _stream(proj)]
    if sel is None:
        _check(lib().bolt_mamba_step(*head, *tail))
    else:
        _check(lib().bolt_mamba_verify(*head, _ptr(sel), *tail))
    return y, conv_out, ssm_out, xbc, ypre


def MambaStep(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, heads: int,
              head_dim: int, d_state: int, n_groups: int, epsilon: float, time_step_min: float):
    """Returns (y bf16 [R, di], conv_state_out, ssm_state_out, xbc_act bf16 [R, cd], ypre f32 [R, di])
    (src/bolt_ops.cu:299-357); the state outputs are shaped like the inputs, row 0 written."""
    return _mamba(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, None, heads, head_dim,
                  d_state, n_groups, epsilon, time_step_min)


def MambaVerify(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, sel, heads: int,
                head_dim: int, d_state: int, n_groups: int, epsilon: float, time_step_min: float):
    """As MambaStep from state row sel (i32 [1] on the device); the state after token r goes to
    row r of the state outputs (rows >= R only are left unwritten)."""
    return _mamba(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, sel, heads, head_dim,
                  d_state, n_groups, epsilon, time_step_min)


def Relu2(x):
    """Returns y bf16 of x's shape, bf16(max(x, 0)^2) (src/bolt_ops.cu:624-646)."""
    _need(x)
    if x.dtype != torch.bfloat16:
        raise RuntimeError("Relu2 takes bf16")
    y = torch.empty_like(x)
    xs, _keep = shape_arg(x.shape)
    _check(lib().bolt_relu2(_ptr(x), xs, x.dim(), _ptr(y), _stream(x)))
    return y


def f32_to_bf16(t, out=None):
    _need(t)
    if out is None:
        out = torch.empty(t.shape, dtype=torch.bfloat16, device=t.device)
    _check(lib().bolt_f32_to_bf16(_ptr(t), _ptr(out), t.numel(), _stream(t)))
    return out


def copy_async(dst, src):
    """dst <- src between host (pinned for an asynchronous copy) and device memory, ordered on
    the current stream of whichever tensor is on the GPU (one cudaMemcpyAsync)."""
    if dst.nbytes != src.nbytes or not dst.is_contiguous() or not src.is_contiguous():
        raise RuntimeError("copy_async: contiguous tensors of the same byte size")
    _check(lib().bolt_memcpy_async(_ptr(dst), _ptr(src), dst.nbytes, _stream(dst if dst.is_cuda else src)))
    return dst


def dequant(fmt: int, w, scales, N: int, K: int, exact: bool = False):
    """Weights [N, K] f32 decoded by the kernels' own decoders (contract checks)."""
    _need(w, scales)
    out = torch.empty(N, K, dtype=torch.float32, device=w.device)
    _check(lib().bolt_dequant(int(fmt), int(exact), _ptr(w), _ptr(scales), int(N), int(K), _ptr(out), _stream(w)))
    return out
