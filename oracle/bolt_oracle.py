"""CPU oracle: a torch-CPU restatement of the reference's weight-streaming decode path.

TEST INFRASTRUCTURE ONLY -- the checker for ``nemotron_ops_b200`` and the timed CPU
baseline.  Nothing in the product imports this module.

What it restates (all citations are ``path:line`` inside the reference project
tianleiwu/nemotron_ops):

* the torch references of ``tests/test_bolt_ops.py`` (the reference's own oracle):
  NVFP4 ``:68,76-78``, Q8/Q4 ``:88-95``, MoeRoute ``:115-119``, the MoE rounding
  points ``:145-150``, IQ2 LUT codes ``:157-180``, native IQ2_XXS ``:211-243``, Relu2
  ``:99-104`` and MambaStep ``:281-303``;
* the kernel rounding contract of ``src/bolt_ops.cu`` that the tests only check to a
  tolerance: ``DequantRow`` ``:860-919`` (weights of the tensor-core path are
  rounded to bf16), the exact fp32 weights of the SIMT kernels ``:480-494,1315-1326``,
  the MoE epilogues ``:519-520,549,582-585,1159-1164`` and the router
  ``:386,420,436-440``.

Two weight contracts exist in the reference and are kept apart here:

* ``exact``: the SIMT GEMVs (R=1, or any R when K % 64 != 0) and MoeDecode use the
  exact fp32 product ``(q - zp) * s`` (``src/bolt_ops.cu:1323,1381,488-490,546``).
* ``mma``: the tensor-core path (R=2..8 Q8/Q4, every ``iq2`` mode, MoeVerify) rounds
  every weight to bf16 once (``src/bolt_ops.cu:880,904,893,869``).

NVFP4 weights ``e2m1 * e4m3`` are exact in both (<= 6 significant bits).

Parity is pinned by ``tests/golden/`` fixtures produced by executing the reference's
own test functions (``tests/golden/make_golden.py``).  IQ2_XXS arithmetic follows the
third-party ``gguf`` package 0.19.0 (``gguf.quants.IQ2_XXS``), which the reference's
tests call at ``tests/test_bolt_ops.py:226-229``; its codebook is read from that
package at run time.
"""
from __future__ import annotations

import numpy as np
import torch

__all__ = [
    "FP4_VALUES", "IQ2_LUT_BF16", "iq2xxs_grid", "bf16_round", "unpack_nibbles",
    "q8_dequant", "q4_dequant", "nvfp4_dequant", "iq2_lut_dequant", "iq2n_dequant",
    "iq2n_dequant_gguf_style", "gemv_contract", "q8_gemv", "q4_gemv", "nvfp4_gemv", "relu2", "mamba_step",
    "moe_route", "route_min_gap", "moe_group_meta", "moe_decode", "moe_verify", "moe_combine", "moe_verify_partial",
    "moe_decode_partial",
    "moe_expert_weights",
]

# e2m1 code -> value, nibble low first (tests/test_bolt_ops.py:68).
FP4_VALUES = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6],
                          dtype=torch.float32)

# iq2=1 LUT codes: code = magnitude index (8, 25, 43) + 4 * negative (README.md "Exact
# IQ2_XXS", tests/test_bolt_ops.py:157).  The kernel decodes codes 0..7 through byte-plane
# tables (src/bolt_ops.cu:885-894); codes 3 and 7 decode to 0.  Codes 8..15 are outside the
# format (the reference's prmt selector would switch to sign-replicate mode) and are not
# part of the contract.
IQ2_LUT_BF16 = torch.tensor([8, 25, 43, 0, -8, -25, -43, 0], dtype=torch.float32)

_GRID = None


def iq2xxs_grid() -> torch.Tensor:
    """The 256 x 8 IQ2_XXS magnitude codebook (values 8/25/43) from gguf 0.19.0."""
    global _GRID
    if _GRID is None:
        from gguf import quants
        q = quants.IQ2_XXS
        q.init_grid()
        _GRID = torch.from_numpy(np.asarray(q.grid, dtype=np.float32).reshape(256, 8).copy())
    return _GRID


def bf16_round(t: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest-even to bf16, returned as float32.  Input must be exact in fp32."""
    return t.to(torch.float32).to(torch.bfloat16).to(torch.float32)


def unpack_nibbles(b: torch.Tensor) -> torch.Tensor:
    """u8 [..., m] -> u8 [..., 2m], low nibble first (tests/test_bolt_ops.py:93)."""
    return torch.stack([b & 15, b >> 4], -1).reshape(*b.shape[:-1], b.shape[-1] * 2)


def _scale_f32(s: torch.Tensor) -> torch.Tensor:
    return s.to(torch.float32)


# ----------------------------------------------------------------------------------------
# dequantisation contracts
# ----------------------------------------------------------------------------------------
def q8_dequant(B: torch.Tensor, scales: torch.Tensor, contract: str = "exact") -> torch.Tensor:
    """Q8 block-32, zero point 128: B u8 [N, K/32, 32], scales bf16 [N, K/32] -> fp32 [N, K].

    exact: ``(b - 128) * s`` in fp32 (src/bolt_ops.cu:1323,1380-1381).
    mma:   ``bf16((b - 128) * s)`` (src/bolt_ops.cu:880-881; the fp32 product is exact).
    """
    N = B.shape[0]
    w = (B.to(torch.float32) - 128.0) * _scale_f32(scales).unsqueeze(-1)
    w = w.reshape(N, -1)
    return bf16_round(w) if contract == "mma" else w


def q4_dequant(B: torch.Tensor, scales: torch.Tensor, contract: str = "exact") -> torch.Tensor:
    """Q4 block-32, zero point 8, low nibble first: B u8 [N, K/32, 16], scales bf16 [N, K/32].

    exact: ``(n - 8) * s`` in fp32 (src/bolt_ops.cu:488-490,1379-1381).
    mma:   ``bf16((n - 8) * bf16(s))`` (src/bolt_ops.cu:897-905).
    """
    N = B.shape[0]
    nb = scales.shape[-1]
    q = unpack_nibbles(B.reshape(N, nb, -1)).to(torch.float32) - 8.0
    w = (q * _scale_f32(scales).unsqueeze(-1)).reshape(N, -1)
    return bf16_round(w) if contract == "mma" else w


def nvfp4_dequant(w: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """NVFP4 weights without the global scale: e2m1 * e4m3 (exact in fp32 and bf16).

    w u8 [N, K/2] (two e2m1 per byte, low nibble first), w_scale u8 e4m3 bytes [N, K/16]
    (tests/test_bolt_ops.py:76-77; src/bolt_ops.cu:652-656,908-916).
    """
    v = FP4_VALUES.to(w.device)[unpack_nibbles(w).long()]
    s = w_scale.contiguous().view(torch.float8_e4m3fn).to(torch.float32).repeat_interleave(16, dim=1)
    return v * s


def iq2_lut_dequant(B: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """iq2=1: 4-bit LUT codes -> ``bf16(value * bf16(s))`` (src/bolt_ops.cu:883-895).

    B u8 [N, K/32, 16] packed low nibble first, scales bf16 [N, K/32].
    """
    N = B.shape[0]
    nb = scales.shape[-1]
    codes = unpack_nibbles(B.reshape(N, nb, -1)).long()
    v = IQ2_LUT_BF16.to(B.device)[codes & 7]
    return bf16_round(v * _scale_f32(scales).unsqueeze(-1)).reshape(N, -1)


def _iq2n_parts(B: torch.Tensor, D: torch.Tensor):
    """Split native IQ2_XXS records.  B u8 [N, K/32, 8], D = fp16 bits in a bf16 tensor [N, K/256].

    Record layout (README.md "Native IQ2_XXS", src/bolt_ops.cu:769-772,820-829): bytes 0..3
    are codebook indices of the four 8-element sub-blocks; bytes 4..7 are a little-endian
    u32 holding four 7-bit sign indices (bits 7j..7j+6) and the 4-bit scale (bits 28..31).
    """
    N, G = B.shape[0], B.shape[1]
    rec = B.reshape(N, G, 8).to(torch.int64)
    gidx = rec[..., :4]
    sg = rec[..., 4] | (rec[..., 5] << 8) | (rec[..., 6] << 16) | (rec[..., 7] << 24)
    d = D.contiguous().view(torch.int16).view(torch.float16).to(torch.float32)  # [N, K/256]
    d = d.repeat_interleave(8, dim=1)[:, :G]
    s4 = (sg >> 28).to(torch.float32)
    db = d * (0.5 + s4) * 0.25  # exact in fp32 (11 x 5 significant bits)
    signs7 = torch.stack([(sg >> (7 * j)) & 127 for j in range(4)], -1)  # [N, G, 4]
    parity = torch.zeros_like(signs7)
    for b in range(7):
        parity ^= (signs7 >> b) & 1
    pattern = signs7 | (parity << 7)  # ggml ksigns: 8th sign = parity (src/bolt_ops.cu:827)
    bits = torch.stack([(pattern >> e) & 1 for e in range(8)], -1)  # [N, G, 4, 8]
    mag = iq2xxs_grid().to(B.device)[gidx]  # [N, G, 4, 8]
    sign = 1.0 - 2.0 * bits.to(torch.float32)
    return db, mag, sign


def iq2n_dequant(B: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """iq2=2 kernel contract: ``+-bf16(mag * bf16(d * (0.5 + s4) * 0.25))``.

    (src/bolt_ops.cu:829 builds the fp32 block scale, :863 rounds it to bf16, :869-876 apply
    sign and the bf16 multiply.)  The reference's own test instead rounds gguf's fp32 weight
    ``bf16(d * (0.5 + s4) * 0.25 * mag)`` once; the two differ by <= 1 bf16 ulp.
    """
    db, mag, sign = _iq2n_parts(B, D)
    w = bf16_round(mag * bf16_round(db)[..., None, None]) * sign
    return w.reshape(B.shape[0], -1)


def iq2n_dequant_gguf_style(B: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """gguf's fp32 dequantisation of the same records (gguf.quants.IQ2_XXS.dequantize_blocks)."""
    db, mag, sign = _iq2n_parts(B, D)
    return (db[..., None, None] * mag * sign).reshape(B.shape[0], -1)


# ----------------------------------------------------------------------------------------
# GEMV ops (dispatch mirrors QGemvState / Nvfp4GemvState::ComputeV2)
# ----------------------------------------------------------------------------------------
def gemv_contract(x: torch.Tensor, W: torch.Tensor, gscale: float = 1.0, fp32: bool = False) -> torch.Tensor:
    """y = bf16(x @ W^T * g), accumulated in fp64 (or fp32 for the timed CPU baseline)."""
    K = x.shape[-1]
    xr = x.reshape(-1, K)
    if fp32:
        y = (xr.to(torch.float32) @ W.to(torch.float32).T) * gscale
    else:
        y = (xr.to(torch.float64) @ W.to(torch.float64).T) * gscale
    return y.to(torch.float32).to(torch.bfloat16).reshape(*x.shape[:-1], W.shape[0])


def _rows(x: torch.Tensor) -> int:
    return x.numel() // x.shape[-1]


def q8_gemv(x, B, scales, fp32: bool = False):
    """Q8Gemv (src/bolt_ops.cu:1429-1468): MMA contract when 2 <= R <= 8 and K % 64 == 0."""
    R, K = _rows(x), x.shape[-1]
    contract = "mma" if (2 <= R <= 8 and K % 64 == 0) else "exact"
    return gemv_contract(x, q8_dequant(B, scales, contract), fp32=fp32)


def q4_gemv(x, B, scales, iq2: int = 0, fp32: bool = False):
    """Q4Gemv (src/bolt_ops.cu:1429-1468) with its ``iq2`` modes."""
    R, K = _rows(x), x.shape[-1]
    if iq2 == 2:
        W = iq2n_dequant(B, scales)
    elif iq2 == 1:
        W = iq2_lut_dequant(B, scales)
    else:
        contract = "mma" if (2 <= R <= 8 and K % 64 == 0) else "exact"
        W = q4_dequant(B, scales, contract)
    return gemv_contract(x, W, fp32=fp32)


def nvfp4_gemv(x, w, w_scale, g, fp32: bool = False):
    """Nvfp4Gemv (src/bolt_ops.cu:1259-1306): y = bf16(g * x @ (e2m1 * e4m3)^T)."""
    gs = float(torch.as_tensor(g).reshape(-1)[0])
    return gemv_contract(x, nvfp4_dequant(w, w_scale), gscale=gs, fp32=fp32)


# ----------------------------------------------------------------------------------------
# MambaStep / MambaVerify
# ----------------------------------------------------------------------------------------
def mamba_step(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, heads: int,
               head_dim: int, d_state: int, n_groups: int, epsilon: float, time_step_min: float, sel=None):
    """One Mamba-2 step over the R rows of proj, starting from state row ``sel`` (0 when None).

    Restates the reference test's torch reference (tests/test_bolt_ops.py:281-303) with the
    kernels' rounding points (src/bolt_ops.cu:92, conv output rounded to bf16 before the SSM).
    Returns (y f32 [R, di] before the output's bf16 rounding, conv states bf16 [R, cd, 3] and
    ssm states f32 [R, heads, d_state, head_dim] after each token, xbc_act bf16 [R, cd],
    ypre f32 [R, di]).
    """
    F = torch.nn.functional
    R = proj.shape[0]
    di = heads * head_dim
    cd = di + 2 * n_groups * d_state
    row = 0 if sel is None else int(sel)
    gate, xbc, dt = proj.float().split([di, cd, heads], -1)
    inp = torch.cat([conv_state[row].float().T, xbc], 0)  # [3 + R, cd]
    cw = conv_w[:, 0, :].float().T                         # [4, cd]
    conv = torch.stack([F.silu((inp[r:r + 4] * cw).sum(0) + conv_b.float()) for r in range(R)])
    xbc_act = conv.to(torch.bfloat16)
    conv_states = torch.stack([inp[r + 1:r + 4].T for r in range(R)]).to(torch.bfloat16)
    xs, Bm, Cm = xbc_act.float().split([di, n_groups * d_state, n_groups * d_state], -1)
    hpg = heads // n_groups
    st = ssm_state[row].float().clone()
    states, ys = [], []
    for r in range(R):
        dts = torch.clamp(F.softplus(dt[r] + dt_bias.float()), min=time_step_min)
        dA = torch.exp(a_neg.float() * dts)
        xh = xs[r].reshape(heads, head_dim)
        Bh = Bm[r].reshape(n_groups, d_state).repeat_interleave(hpg, 0)
        Ch = Cm[r].reshape(n_groups, d_state).repeat_interleave(hpg, 0)
        st = st * dA[:, None, None] + (dts[:, None] * xh)[:, None, :] * Bh[:, :, None]
        states.append(st.clone())
        ys.append((st * Ch[:, :, None]).sum(1) + d_skip.float()[:, None] * xh)
    ypre = torch.stack(ys).reshape(R, di)
    g = (ypre * F.silu(gate)).reshape(R, n_groups, di // n_groups)
    g = g * torch.rsqrt(g.pow(2).mean(-1, keepdim=True) + epsilon)
    y = g.reshape(R, di) * norm_w.float()
    return y, conv_states, torch.stack(states), xbc_act, ypre


# ----------------------------------------------------------------------------------------
# Relu2
# ----------------------------------------------------------------------------------------
def relu2(x: torch.Tensor) -> torch.Tensor:
    """bf16(max(x, 0)^2), square in fp32 (Relu2Kernel, src/bolt_ops.cu:624-629; the reference
    test's expression tests/test_bolt_ops.py:102).  max follows the kernel's fmaxf: NaN -> 0."""
    xf = x.float()
    r = torch.where(xf > 0, xf, torch.zeros_like(xf))
    return (r * r).to(torch.bfloat16)


# ----------------------------------------------------------------------------------------
# MoE
# ----------------------------------------------------------------------------------------
def moe_route(x, gate_w, bias, topk: int, scale: float):
    """MoeRoute (src/bolt_ops.cu:368-441).

    scores = sigmoid(x @ gate_w^T) (fp32 output); selection = ``topk`` rounds of arg-max over
    ``score + bias`` (fp32 add), ties to the lower expert index (:420), in selection order;
    w = score / (sum of selected scores + 1e-20) * scale with the fp32 sum taken in selection
    order (:429-440).  Rounds that find nothing (topk > E) yield index -1 and score 0.
    """
    K = x.shape[-1]
    xr = x.reshape(-1, K).to(torch.float64)
    logits = xr @ gate_w.to(torch.float64).T
    scores = (1.0 / (1.0 + torch.exp(-logits))).to(torch.float32)
    R, E = scores.shape
    val = scores + bias.to(torch.float32).unsqueeze(0)
    scores, val = scores.cpu(), val.cpu()
    idx = torch.full((R, topk), -1, dtype=torch.int32)
    wts = torch.zeros((R, topk), dtype=torch.float32)
    for r in range(R):
        v = val[r].clone()
        picked = []
        total = torch.tensor(0.0, dtype=torch.float32)
        for j in range(topk):
            best = -float("inf")
            bi = -1
            for e in range(E):
                ve = float(v[e])
                if ve > best:
                    best, bi = ve, e
            if bi >= 0:
                v[bi] = -float("inf")
                s = scores[r, bi]
            else:
                s = torch.tensor(0.0, dtype=torch.float32)
            picked.append((bi, s))
            total = total + s
        denom = total + torch.tensor(1e-20, dtype=torch.float32)
        for j, (bi, s) in enumerate(picked):
            idx[r, j] = bi
            wts[r, j] = (s / denom) * torch.tensor(scale, dtype=torch.float32)
    return idx, wts, scores


def route_min_gap(x, gate_w, bias, topk: int) -> float:
    """Smallest fp64 gap between consecutive bias-corrected scores among the first topk+1.

    A gap below ~1e-6 means a GPU kernel's fp32 summation order can legitimately reorder
    the selection (the reference test compares index *sets* for this reason, :121).
    """
    K = x.shape[-1]
    logits = x.reshape(-1, K).to(torch.float64) @ gate_w.to(torch.float64).T
    val = 1.0 / (1.0 + torch.exp(-logits)) + bias.to(torch.float64)
    srt = torch.sort(val, dim=-1, descending=True).values[:, : topk + 1]
    if srt.shape[1] < 2:
        return float("inf")
    return float((srt[:, :-1] - srt[:, 1:]).min())


def moe_group_meta(idx: torch.Tensor, topk: int) -> torch.Tensor:
    """MoeGroupKernel's meta layout (src/bolt_ops.cu:1083-1112).

    [0] = U unique experts; [1..U] = their ids in first-occurrence order over the flattened
    pairs p = row * topk + k; [1+P + u*8 + row] = pair index p of row `row` for expert u,
    or -1.  The reference leaves slots [1+U, 1+P) unwritten; this contract sets them to -1.
    """
    flat = idx.reshape(-1).cpu().tolist()
    P = len(flat)
    meta = torch.full((1 + P + 8 * P,), -1, dtype=torch.int32)
    uniq = []
    for p, e in enumerate(flat):
        if e not in uniq:
            uniq.append(e)
        u = uniq.index(e)
        meta[1 + P + u * 8 + p // topk] = p
    meta[0] = len(uniq)
    for u, e in enumerate(uniq):
        meta[1 + u] = e
    return meta


def moe_expert_weights(fc_w, fc_s, e: int, n_out: int, k_in: int, fmt: str):
    """Dequantised weights [n_out, k_in] of expert e for one MoE projection."""
    if fmt == "q4_exact":
        return q4_dequant(fc_w[e].reshape(n_out, k_in // 32, 16), fc_s[e].reshape(n_out, k_in // 32), "exact")
    if fmt == "q4_mma":
        return q4_dequant(fc_w[e].reshape(n_out, k_in // 32, 16), fc_s[e].reshape(n_out, k_in // 32), "mma")
    if fmt == "iq2_lut":
        return iq2_lut_dequant(fc_w[e].reshape(n_out, k_in // 32, 16), fc_s[e].reshape(n_out, k_in // 32))
    if fmt == "iq2n":
        return iq2n_dequant(fc_w[e].reshape(n_out, k_in // 32, 8), fc_s[e].reshape(n_out, k_in // 256))
    raise ValueError(fmt)


def _moe_pairs(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, fmt, fp32=False, h_in=None):
    """h_in: stage-wise checking -- take the fc1 output h [P, I] from the caller instead of
    computing it, so the fc2 stage can be compared against a reference that shares its input
    exactly with the kernel under test."""
    R = z.shape[0]
    I = fc1_w.shape[1]
    E = fc1_w.shape[0]
    P = R * topk
    acc_t = torch.float32 if fp32 else torch.float64
    dev = z.device
    h = torch.zeros((P, I), dtype=torch.bfloat16, device=dev)
    part = torch.zeros((P, 1024), dtype=torch.float32, device=dev)
    flat = idx.reshape(-1).cpu()
    cache = {}
    for p in range(P):
        t = p // topk
        e = int(flat[p])
        if e < 0 or e >= E:
            continue  # out-of-range expert ids contribute nothing (the reference reads out of bounds)
        if e not in cache:
            if len(cache) >= 4:
                cache.pop(next(iter(cache)))
            cache[e] = (moe_expert_weights(fc1_w, fc1_s, e, I, 1024, fmt).to(acc_t),
                        moe_expert_weights(fc2_w, fc2_s, e, 1024, I, fmt).to(acc_t))
        W1, W2 = cache[e]
        if h_in is None:
            a = bf16_round((z[t].to(acc_t) @ W1.T).to(torch.float32))  # bf16(z . W1) (:519, :1159)
            r = torch.clamp(a, min=0.0)
            h[p] = (r * r).to(torch.bfloat16)  # bf16(relu^2), r*r exact in fp32 (:520, :1162)
        else:
            h[p] = h_in[p].to(device=dev, dtype=torch.bfloat16)
        part[p] = bf16_round((h[p].to(acc_t) @ W2.T).to(torch.float32))  # float(bf16(h . W2)) (:549, :1164)
    wt = w.reshape(R, topk).to(acc_t)
    pr = part.reshape(R, topk, 1024).to(acc_t)
    out = (wt.unsqueeze(-1) * pr).sum(1).to(torch.float32).to(torch.bfloat16)  # (:552-587)
    return out, h, part


def moe_decode(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, fp32: bool = False, h_in=None):
    """MoeDecode (src/bolt_ops.cu:474-619): int4 experts with the exact fp32 weight contract."""
    return _moe_pairs(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, "q4_exact", fp32, h_in=h_in)


def moe_verify(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, iq2: int = 0, fp32: bool = False, h_in=None):
    """MoeVerify (src/bolt_ops.cu:1078-1257): bf16-rounded (tensor-core) weight contract."""
    fmt = {0: "q4_mma", 1: "iq2_lut", 2: "iq2n"}[iq2]
    out, h, part = _moe_pairs(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, fmt, fp32, h_in=h_in)
    return out, h, part, moe_group_meta(idx, topk)


def moe_combine(part: torch.Tensor, w: torch.Tensor, topk: int) -> torch.Tensor:
    """out[r] = bf16(sum_k w[r, k] * part[r * topk + k]) (src/bolt_ops.cu:552-587), fp64 sum."""
    R = w.numel() // topk
    pr = part.reshape(R, topk, 1024).to(torch.float64)
    wt = w.reshape(R, topk).to(device=part.device, dtype=torch.float64)
    return (wt.unsqueeze(-1) * pr).sum(1).to(torch.float32).to(torch.bfloat16)


def moe_verify_partial(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, iq2: int, e_begin: int, e_end: int,
                       num_experts: int = None):
    """fp32 [R, 1024] = sum over the pairs whose expert is in [e_begin, e_end) of w * part
    (fp64 sum, k ascending): one shard's share of the expert-parallel MoeVerify.  The weight
    tensors hold all experts, or only experts [e_begin, e_end) when ``num_experts`` is given."""
    fmt = {0: "q4_mma", 1: "iq2_lut", 2: "iq2n"}[iq2]
    return _moe_partial(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, fmt, e_begin, e_end, num_experts)


def moe_decode_partial(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk: int, e_begin: int, e_end: int,
                       num_experts: int = None):
    """One shard's share of the expert-parallel MoeDecode (exact fp32 weight contract); as
    :func:`moe_verify_partial`."""
    return _moe_partial(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, "q4_exact", e_begin, e_end, num_experts)


def _moe_partial(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, fmt, e_begin, e_end, num_experts):
    E = fc1_w.shape[0] if num_experts is None else int(num_experts)
    R = z.shape[0]
    flat = idx.reshape(-1).to(torch.int64).cpu()
    local = (flat >= e_begin) & (flat < e_end)
    if fc1_w.shape[0] != E:  # local slices: renumber the local experts from 0
        idx_l = torch.where(local, flat - e_begin, torch.full_like(flat, -1)).reshape(idx.shape).to(torch.int32)
    else:
        idx_l = torch.where(local, flat, torch.full_like(flat, -1)).reshape(idx.shape).to(torch.int32)
    _, _, part = _moe_pairs(z, idx_l.to(z.device), w, fc1_w, fc1_s, fc2_w, fc2_s, topk, fmt)
    wt = w.reshape(R, topk).to(torch.float64) * local.reshape(R, topk).to(torch.float64).to(w.device)
    return (wt.unsqueeze(-1) * part.reshape(R, topk, 1024).to(torch.float64)).sum(1).to(torch.float32)
