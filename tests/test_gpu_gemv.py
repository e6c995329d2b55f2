"""GPU parity of Nvfp4Gemv / Q8Gemv / Q4Gemv (CUDA path through the C ABI) against the oracle.

* golden fixtures (inputs + expected outputs computed by the reference's own tests);
* the kernels' weight decoders are bit-exact with the oracle's contracts on random bytes;
* the benchmark configs at full size against the oracle's contract (fp64 accumulation);
* the reference's own test shapes (N up to 131072) against an fp32 torch reference;
* edge shapes: ragged N, small N, K % 64 != 0, misaligned pointers.
Tolerance for float outputs: |y - ref| <= 1e-3 + 1e-2 |ref| elementwise, ref = bf16-rounded
contract output.
"""
import pytest
import torch

import oracle as O
from golden_io import case_names, load, rel
from nemotron_ops_b200 import ops
from nemotron_ops_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
RTOL, ATOL = 1e-2, 1e-3


def assert_contract_close(y, ref, rtol=RTOL, atol=ATOL):
    y, ref = y.float().cpu(), ref.float().cpu()
    err = (y - ref).abs()
    bad = err > atol + rtol * ref.abs()
    assert not bool(bad.any()), f"{int(bad.sum())}/{bad.numel()} outside tolerance, max err {float(err.max()):.3g}"


def _run(op, inputs, attrs):
    ins = [t.to(DEV) for t in inputs]
    if op == "Nvfp4Gemv":
        return ops.Nvfp4Gemv(*ins)
    if op == "Q8Gemv":
        return ops.Q8Gemv(*ins)
    return ops.Q4Gemv(*ins, iq2=attrs.get("iq2", 0))


def _oracle(op, inputs, attrs):
    if op == "Nvfp4Gemv":
        return O.nvfp4_gemv(*inputs)
    if op == "Q8Gemv":
        return O.q8_gemv(*inputs)
    return O.q4_gemv(*inputs, iq2=attrs.get("iq2", 0))


@pytest.mark.parametrize("name", case_names("nvfp4_") + case_names("q8_") + case_names("q4_"))
def test_gemv_golden(name):
    c = load(name)
    y = _run(c.op, c.inputs, c.attrs)
    torch.cuda.synchronize()
    assert rel(y, c.ref) < (6e-3 if "iq2" in name else 1e-2)  # the reference test's thresholds
    assert_contract_close(y, _oracle(c.op, c.inputs, c.attrs))
    assert ops.device_status() == 0


# ---------------------------------------------------------------------------------------------
# decoders
# ---------------------------------------------------------------------------------------------
def _rand_scales_bf16(shape, g):
    mag = torch.pow(10.0, torch.rand(shape, generator=g) * 4 - 3)
    sign = torch.where(torch.rand(shape, generator=g) < 0.5, -1.0, 1.0)
    return (torch.randn(shape, generator=g).abs() * mag * sign).to(torch.bfloat16)


@pytest.mark.parametrize("fmt,exact", [(0, 1), (1, 1), (0, 0), (1, 0), (2, 0), (3, 0), (4, 0)])
def test_decoder_bit_exact(fmt, exact):
    g = torch.Generator().manual_seed(100 + fmt * 2 + exact)
    N, K = 96, 2048
    if fmt == 0:
        w = torch.randint(0, 256, (N, K // 32, 32), generator=g, dtype=torch.int32).to(torch.uint8)
        s = _rand_scales_bf16((N, K // 32), g)
        ref = O.q8_dequant(w, s, "exact" if exact else "mma")
    elif fmt == 1:
        w = torch.randint(0, 256, (N, K // 32, 16), generator=g, dtype=torch.int32).to(torch.uint8)
        s = _rand_scales_bf16((N, K // 32), g)
        ref = O.q4_dequant(w, s, "exact" if exact else "mma")
    elif fmt == 2:
        w = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.int32).to(torch.uint8)
        s = torch.randint(0, 256, (N, K // 16), generator=g, dtype=torch.int32).to(torch.uint8)
        s[(s & 0x7F) == 0x7F] = 0x38  # no NaN scales
        ref = O.nvfp4_dequant(w, s)
    elif fmt == 3:
        w = (torch.randint(0, 256, (N, K // 32, 16), generator=g, dtype=torch.int32) & 0x77).to(torch.uint8)
        s = _rand_scales_bf16((N, K // 32), g)
        ref = O.iq2_lut_dequant(w, s)
    else:
        w = W.iq2n_records((N,), K, g, "cpu")
        d = torch.randn(N, K // 256, generator=g) * torch.pow(10.0, torch.rand(N, K // 256, generator=g) * 3 - 4)
        s = W.fp16_bits_as_bf16(d)
        ref = O.iq2n_dequant(w, s)
    got = ops.dequant(fmt, w.to(DEV), s.to(DEV), N, K, exact=bool(exact)).cpu()
    assert torch.equal(got, ref), f"{int((got != ref).sum())} weights differ"


def test_iq2n_decoder_all_grid_and_sign_patterns():
    # every codebook entry with every 7-bit sign index at least once, scale nibble 0..15
    N, K = 128, 256 * 32
    G = K // 32
    idx = torch.arange(N * G * 4) % 256
    signs = (torch.arange(N * G * 4) // 3) % 128
    s4 = torch.arange(N * G) % 16
    sg = signs.reshape(N * G, 4)
    u32 = sg[:, 0] | (sg[:, 1] << 7) | (sg[:, 2] << 14) | (sg[:, 3] << 21) | (s4 << 28)
    word = torch.stack([(u32 >> (8 * i)) & 255 for i in range(4)], -1)
    rec = torch.cat([idx.reshape(N * G, 4), word], -1).to(torch.uint8).reshape(N, G, 8)
    d = W.fp16_bits_as_bf16(torch.linspace(-0.05, 0.05, N * K // 256).reshape(N, K // 256))
    got = ops.dequant(4, rec.to(DEV), d.to(DEV), N, K).cpu()
    assert torch.equal(got, O.iq2n_dequant(rec, d))


# ---------------------------------------------------------------------------------------------
# benchmark configs at full size
# ---------------------------------------------------------------------------------------------
def _cpu(d):
    return {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def test_q8_r1_config():
    d = W.q8_gemv(R=1, N=4096, K=4096)
    y = ops.Q8Gemv(d["x"], d["B"], d["scales"])
    c = _cpu(d)
    assert_contract_close(y, O.q8_gemv(c["x"], c["B"], c["scales"]))


@pytest.mark.parametrize("R", [1, 8])
def test_nvfp4_config(R):
    d = W.nvfp4_gemv(R=R, N=4096, K=8192)
    y = ops.Nvfp4Gemv(d["x"], d["w"], d["w_scale"], d["g"])
    c = _cpu(d)
    assert_contract_close(y, O.nvfp4_gemv(c["x"], c["w"], c["w_scale"], c["g"]))


@pytest.mark.parametrize("R", [1, 4, 8])
@pytest.mark.parametrize("iq2", [0, 2])
def test_q4_config(R, iq2):
    d = W.q4_gemv(R=R, N=8192, K=4096, iq2=iq2)
    y = ops.Q4Gemv(d["x"], d["B"], d["scales"], iq2=iq2)
    c = _cpu(d)
    assert_contract_close(y, O.q4_gemv(c["x"], c["B"], c["scales"], iq2=iq2))


# ---------------------------------------------------------------------------------------------
# the reference's own test shapes (tests/test_bolt_ops.py:305-315) vs an fp32 torch reference
# ---------------------------------------------------------------------------------------------
def _torch_ref(x, W_):
    return (x.float() @ W_.float().T)


NVFP4_SHAPES = [(1, 18560, 4096), (2, 18560, 4096), (8, 18560, 4096), (1, 4096, 8192), (3, 4096, 8192),
                (5, 1024, 4096), (7, 18560, 4096)]


@pytest.mark.parametrize("R,N,K", NVFP4_SHAPES)
def test_nvfp4_reference_shapes(R, N, K):
    d = W.nvfp4_gemv(R=R, N=N, K=K, seed=R * 7 + N)
    y = ops.Nvfp4Gemv(d["x"], d["w"], d["w_scale"], d["g"])
    ref = _torch_ref(d["x"], O.nvfp4_dequant(d["w"], d["w_scale"])) * d["g"]
    assert_contract_close(y, ref.to(torch.bfloat16))


@pytest.mark.parametrize("xscale", [3000.0])
@pytest.mark.parametrize("R", [1, 8])
def test_nvfp4_massive_activations(R, xscale):
    d = W.nvfp4_gemv(R=R, N=18560, K=4096, seed=5)
    x = (d["x"].float() * xscale).to(torch.bfloat16)
    y = ops.Nvfp4Gemv(x, d["w"], d["w_scale"], d["g"])
    ref = _torch_ref(x, O.nvfp4_dequant(d["w"], d["w_scale"])) * d["g"]
    assert torch.isfinite(y.float()).all()
    assert_contract_close(y, ref.to(torch.bfloat16))


Q_SHAPES = [(1, 1024, 4096), (1, 4096, 1024), (4, 4096, 5376), (1, 131072, 4096), (8, 131072, 4096),
            (3, 1024, 4096), (8, 4096, 1024), (6, 4096, 5376), (5, 2688, 4096)]


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("R,N,K", Q_SHAPES)
def test_qgemv_reference_shapes(bits, R, N, K):
    g = torch.Generator(device=DEV).manual_seed(R + N + K + bits)
    nb = K // 32
    B = torch.randint(0, 256, (N, nb, 32 if bits == 8 else 16), generator=g, device=DEV, dtype=torch.int32).to(torch.uint8)
    s = (torch.rand(N, nb, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(R, K, generator=g, device=DEV).to(torch.bfloat16)
    contract = "mma" if (2 <= R <= 8 and K % 64 == 0) else "exact"
    if bits == 8:
        y = ops.Q8Gemv(x, B, s)
        Wd = O.q8_dequant(B, s, contract)
    else:
        y = ops.Q4Gemv(x, B, s)
        Wd = O.q4_dequant(B, s, contract)
    assert_contract_close(y, _torch_ref(x, Wd).to(torch.bfloat16))


@pytest.mark.parametrize("R,N,K", [(8, 5376, 4096), (2, 4096, 5376), (5, 1024, 4096), (8, 16384, 4096)])
def test_q4_iq2_lut_reference_shapes(R, N, K):
    g = torch.Generator(device=DEV).manual_seed(11 + R)
    codes = torch.randint(0, 3, (N, K), generator=g, device=DEV) + 4 * torch.randint(0, 2, (N, K), generator=g, device=DEV)
    B = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8).reshape(N, K // 32, 16)
    s = (torch.rand(N, K // 32, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(R, K, generator=g, device=DEV).to(torch.bfloat16)
    y = ops.Q4Gemv(x, B, s, iq2=1)
    assert_contract_close(y, _torch_ref(x, O.iq2_lut_dequant(B, s)).to(torch.bfloat16))


@pytest.mark.parametrize("R,N,K", [(8, 5376, 4096), (1, 4096, 5376), (3, 1024, 4096), (8, 4096, 5376)])
def test_q4_iq2_native_reference_shapes(R, N, K):
    d = W.q4_gemv(R=R, N=N, K=K, iq2=2, seed=21 + R)
    y = ops.Q4Gemv(d["x"], d["B"], d["scales"], iq2=2)
    assert_contract_close(y, _torch_ref(d["x"], O.iq2n_dequant(d["B"], d["scales"])).to(torch.bfloat16))


# ---------------------------------------------------------------------------------------------
# edges
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("N", [1, 3, 17, 149, 1000])
@pytest.mark.parametrize("R,fmt", [(1, "q4"), (1, "q8"), (5, "q4"), (1, "nvfp4"), (8, "nvfp4"), (1, "iq2n"), (3, "iq2n")])
def test_ragged_rows(N, R, fmt):
    K = 1024
    if fmt == "nvfp4":
        d = W.nvfp4_gemv(R=R, N=N, K=K, seed=N)
        y = ops.Nvfp4Gemv(d["x"], d["w"], d["w_scale"], d["g"])
        c = _cpu(d)
        ref = O.nvfp4_gemv(c["x"], c["w"], c["w_scale"], c["g"])
    elif fmt == "q8":
        d = W.q8_gemv(R=R, N=N, K=K, seed=N)
        y = ops.Q8Gemv(d["x"], d["B"], d["scales"])
        c = _cpu(d)
        ref = O.q8_gemv(c["x"], c["B"], c["scales"])
    else:
        iq2 = 2 if fmt == "iq2n" else 0
        d = W.q4_gemv(R=R, N=N, K=K, iq2=iq2, seed=N)
        y = ops.Q4Gemv(d["x"], d["B"], d["scales"], iq2=iq2)
        c = _cpu(d)
        ref = O.q4_gemv(c["x"], c["B"], c["scales"], iq2=iq2)
    assert_contract_close(y, ref)


@pytest.mark.parametrize("N,K", [(1000, 2560), (149, 512), (300, 4608), (149, 6144), (149, 8192), (77, 1056),
                                 (77, 2080)])
def test_q8_r1_staged_and_exact_paths(N, K):
    """Q8Gemv R = 1: K % 512 == 0 and K <= 4096 take the shared-memory staged kernel, the other
    shapes the exact streaming kernel (every 16-k slot count from 65 to 1024) or the generic one;
    all against the exact contract."""
    d = W.q8_gemv(R=1, N=N, K=K, seed=K)
    y = ops.Q8Gemv(d["x"], d["B"], d["scales"])
    c = _cpu(d)
    assert_contract_close(y, O.q8_gemv(c["x"], c["B"], c["scales"]))


@pytest.mark.parametrize("K", [1056, 2080, 3104])
def test_q4_r1_exact_stream_slot_counts(K):
    """Q4Gemv R = 1 with K % 256 != 0: the exact streaming kernel at 66, 130 and 194 slots."""
    d = W.q4_gemv(R=1, N=77, K=K, seed=K)
    y = ops.Q4Gemv(d["x"], d["B"], d["scales"])
    c = _cpu(d)
    assert_contract_close(y, O.q4_gemv(c["x"], c["B"], c["scales"]))


@pytest.mark.parametrize("N,K", [(1000, 2048), (149, 6144), (17, 8192)])
def test_iq2n_r1_staged_shapes(N, K):
    """IQ2_XXS R = 1 on the staged kernel at every chunk count it compiles (K / 2048 = 1, 3, 4)."""
    d = W.q4_gemv(R=1, N=N, K=K, iq2=2, seed=N + K)
    y = ops.Q4Gemv(d["x"], d["B"], d["scales"], iq2=2)
    c = _cpu(d)
    assert_contract_close(y, O.q4_gemv(c["x"], c["B"], c["scales"], iq2=2))


def test_iq2n_r1_scales_off_16_bytes_take_register_kernel():
    """Scales 2 bytes past a 16-byte boundary: the register-streaming IQ2_XXS kernel."""
    d = W.q4_gemv(R=1, N=300, K=4096, iq2=2, seed=5)
    s = d["scales"]
    buf = torch.empty(s.numel() + 1, dtype=s.dtype, device=DEV)
    s2 = buf[1:].view(s.shape)
    s2.copy_(s)
    y = ops.Q4Gemv(d["x"], d["B"], s2, iq2=2)
    c = _cpu(d)
    assert_contract_close(y, O.q4_gemv(c["x"], c["B"], c["scales"], iq2=2))


@pytest.mark.parametrize("K", [32, 96, 160, 544])
@pytest.mark.parametrize("R", [1, 4])
def test_k_not_multiple_of_64(K, R):
    d = W.q4_gemv(R=R, N=77, K=K, seed=K)
    y = ops.Q4Gemv(d["x"], d["B"], d["scales"])
    c = _cpu(d)
    assert_contract_close(y, O.q4_gemv(c["x"], c["B"], c["scales"]))


def test_three_dim_activations():
    d = W.q4_gemv(R=6, N=256, K=1024, seed=3)
    x3 = d["x"].reshape(2, 3, 1024)
    y = ops.Q4Gemv(x3, d["B"], d["scales"])
    assert y.shape == (2, 3, 256)
    c = _cpu(d)
    assert_contract_close(y.reshape(6, 256), O.q4_gemv(c["x"], c["B"], c["scales"]))


def test_unaligned_activation_r1_takes_generic_path():
    d = W.q4_gemv(R=1, N=300, K=1024, seed=9)
    buf = torch.empty(1024 + 1, dtype=torch.bfloat16, device=DEV)
    x = buf[1:].view(1, 1024)
    x.copy_(d["x"])
    y = ops.Q4Gemv(x, d["B"], d["scales"])
    c = _cpu(d)
    assert_contract_close(y, O.q4_gemv(c["x"], c["B"], c["scales"]))


def test_unaligned_activation_mma_path_is_rejected():
    d = W.q4_gemv(R=4, N=64, K=1024, seed=9)
    buf = torch.empty(4 * 1024 + 1, dtype=torch.bfloat16, device=DEV)
    x = buf[1:].view(4, 1024)
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        ops.Q4Gemv(x, d["B"], d["scales"])


@pytest.mark.parametrize("fmt", ["q4", "nvfp4"])
def test_launch_options_pdl_matches_default(fmt):
    if fmt == "q4":
        d = W.q4_gemv(R=1, N=4096, K=4096, seed=4)
        call = lambda: ops.Q4Gemv(d["x"], d["B"], d["scales"])  # noqa: E731
    else:
        d = W.nvfp4_gemv(R=1, N=4096, K=8192, seed=4)
        call = lambda: ops.Nvfp4Gemv(d["x"], d["w"], d["w_scale"], d["g"])  # noqa: E731
    y0 = call()
    ops.set_launch_options(pdl=True, early_weights=True)
    try:
        y1 = call()
        y2 = call()
    finally:
        ops.set_launch_options()
    ops.set_launch_options(pdl=False)
    try:
        y3 = call()
    finally:
        ops.set_launch_options()
    assert torch.equal(y0, y1) and torch.equal(y1, y2) and torch.equal(y0, y3)


@pytest.mark.parametrize("R", [1, 8])
def test_cuda_graph_capture_replay(R):
    d = W.nvfp4_gemv(R=R, N=2048, K=4096, seed=8)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y_eager = ops.Nvfp4Gemv(d["x"], d["w"], d["w_scale"], d["g"])
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = ops.Nvfp4Gemv(d["x"], d["w"], d["w_scale"], d["g"])
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y_eager)
