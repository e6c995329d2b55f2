"""Seeded synthetic inputs in the shapes, layouts and value distributions of the benchmark configs.

No dataset or checkpoint is involved: every config of the decode path is specified by shapes
and distributions, reproduced here with torch generators.  Each function returns a dict of
tensors on `device`.

Layouts follow the reference ops (src/bolt_ops.cu:1469-1589, README.md):
  Q8:     B u8 [N, K/32, 32] = q + 128, scales bf16 [N, K/32]
  Q4:     B u8 [N, K/32, 16] int4 low nibble first (zero point 8), scales bf16 [N, K/32]
  IQ2N:   B u8 [N, K/32, 8] ggml records, scales = fp16 bits [N, K/256] in a bf16 tensor
  NVFP4:  w u8 [N, K/2], w_scale u8 e4m3 [N, K/16], g f32 [1]
  MoE:    fc1_w [E, I, 512] / fc1_s [E, I, 32]; fc2_w [E, 1024, I/2] / fc2_s [E, 1024, I/32]
          (native IQ2_XXS: fc1_w [E, I, 32, 8] / [E, I, 4]; fc2_w [E, 1024, I/32, 8] / [E, 1024, I/256])
"""
from __future__ import annotations

import torch


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _bytes(shape, g, device, lo=0, hi=256):
    return torch.randint(lo, hi, shape, generator=g, device=device, dtype=torch.int32).to(torch.uint8)


def _absn(shape, scale, g, device, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=g, device=device).abs() * scale).to(dtype)


def iq2n_records(shape_prefix, K, g, device):
    """Native IQ2_XXS records u8 [*prefix, K/32, 8]: 4 codebook indices U[0,255], then a u32 of
    four 7-bit sign indices U[0,127] and a 4-bit scale U[0,15] in bits 28..31."""
    G = K // 32
    idx = _bytes((*shape_prefix, G, 4), g, device)
    signs = torch.randint(0, 128, (*shape_prefix, G, 4), generator=g, device=device, dtype=torch.int64)
    s4 = torch.randint(0, 16, (*shape_prefix, G), generator=g, device=device, dtype=torch.int64)
    u32 = signs[..., 0] | (signs[..., 1] << 7) | (signs[..., 2] << 14) | (signs[..., 3] << 21) | (s4 << 28)
    word = torch.stack([(u32 >> (8 * i)) & 255 for i in range(4)], -1).to(torch.uint8)
    return torch.cat([idx, word], -1).contiguous()


def fp16_bits_as_bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float16).view(torch.int16).view(torch.bfloat16)


def q8_gemv(R=1, N=4096, K=4096, seed=0, device="cuda"):
    """Q8Gemv config: x ~N(0,1); codes q uniform in [-127, 127] stored as q + 128; s = |N|*0.01."""
    g = _gen(seed, device)
    x = torch.randn(R, K, generator=g, device=device).to(torch.bfloat16)
    B = (torch.randint(-127, 128, (N, K // 32, 32), generator=g, device=device, dtype=torch.int32) + 128).to(torch.uint8)
    s = _absn((N, K // 32), 0.01, g, device)
    return dict(x=x, B=B, scales=s)


def q4_gemv(R=1, N=8192, K=4096, iq2=0, seed=0, device="cuda"):
    """Q4Gemv config: int4 (iq2=0) random bytes, s = |N|*0.02; or native IQ2_XXS (iq2=2)
    records with fp16 super-block scales |N|*1e-3."""
    g = _gen(seed, device)
    x = torch.randn(R, K, generator=g, device=device).to(torch.bfloat16)
    if iq2 == 2:
        B = iq2n_records((N,), K, g, device)
        s = fp16_bits_as_bf16(_absn((N, K // 256), 1e-3, g, device, torch.float32))
    else:
        B = _bytes((N, K // 32, 16), g, device)
        s = _absn((N, K // 32), 0.02, g, device)
    return dict(x=x, B=B, scales=s, iq2=iq2)


def e4m3_uniform(shape, lo, hi, g, device):
    u = torch.rand(shape, generator=g, device=device) * (hi - lo) + lo
    return u.to(torch.float8_e4m3fn).view(torch.uint8)


def nvfp4_gemv(R=1, N=4096, K=8192, seed=0, device="cuda"):
    """Nvfp4Gemv config: w uniform bytes, w_scale = e4m3(U(0.25, 4)), g = 0.01, x ~N(0,1)."""
    g = _gen(seed, device)
    x = torch.randn(R, K, generator=g, device=device).to(torch.bfloat16)
    w = _bytes((N, K // 2), g, device)
    ws = e4m3_uniform((N, K // 16), 0.25, 4.0, g, device)
    gs = torch.tensor([0.01], device=device, dtype=torch.float32)
    return dict(x=x, w=w, w_scale=ws, g=gs)


def moe_route(R=1, E=304, K=4096, seed=0, device="cuda"):
    """MoeRoute inputs: x ~N(0,1), gate_w ~N(0, 0.02) bf16, bias ~N(0, 0.1) f32."""
    g = _gen(seed, device)
    x = torch.randn(R, K, generator=g, device=device).to(torch.bfloat16)
    gw = (torch.randn(E, K, generator=g, device=device) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, generator=g, device=device) * 0.1
    return dict(x=x, gate_w=gw, bias=b)


def moe_experts(E=304, I=2304, iq2=0, seed=1, device="cuda"):
    """Expert weights: int4 random bytes with bf16 scales |N|*0.02, or native IQ2_XXS records
    with fp16 super-block scales |N|*1e-3."""
    g = _gen(seed, device)
    if iq2 == 2:
        fc1_w = iq2n_records((E, I), 1024, g, device)
        fc1_s = fp16_bits_as_bf16(_absn((E, I, 4), 1e-3, g, device, torch.float32))
        fc2_w = iq2n_records((E, 1024), I, g, device)
        fc2_s = fp16_bits_as_bf16(_absn((E, 1024, I // 256), 1e-3, g, device, torch.float32))
    else:
        fc1_w = _bytes((E, I, 512), g, device)
        fc1_s = _absn((E, I, 32), 0.02, g, device)
        fc2_w = _bytes((E, 1024, I // 2), g, device)
        fc2_s = _absn((E, 1024, I // 32), 0.02, g, device)
    return dict(fc1_w=fc1_w, fc1_s=fc1_s, fc2_w=fc2_w, fc2_s=fc2_s)


def moe_latent(R=1, seed=2, device="cuda"):
    g = _gen(seed, device)
    return torch.randn(R, 1024, generator=g, device=device).to(torch.bfloat16)
