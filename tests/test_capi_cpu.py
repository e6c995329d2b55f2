"""CPU checks of the C ABI: the library loads, exports every declared symbol, and rejects bad
shapes with the reference's messages before any device work (no GPU needed)."""
import ctypes
import os
import re

import pytest

from nemotron_ops_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "bolt_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"BOLT_API\s+[\w\s\*]+?\b(bolt_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    syms = declared_symbols()
    assert len(syms) >= 13
    assert sorted(_lib.SIGNATURES) == syms


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.bolt_abi_version() == 100
    assert lib.bolt_last_error() == b""


def _sh(*dims):
    return _lib.shape_arg(dims)


NULL = ctypes.c_void_p(0)


def _call_q4(x_shape, b_shape, iq2=0):
    lib = _lib.lib()
    xs, k1 = _sh(*x_shape)
    bs, k2 = _sh(*b_shape)
    rc = lib.bolt_q4_gemv(NULL, xs, len(x_shape), NULL, bs, len(b_shape), NULL, iq2, NULL, NULL)
    return rc, _lib.last_error()


@pytest.mark.parametrize("x_shape,b_shape,iq2,msg", [
    ((1, 4096), (64, 100, 16), 0, "QGemv: K mismatch"),
    ((1, 4000), (64, 124, 16), 0, "QGemv: K mismatch"),
    ((1, 4004), (64, 125, 16), 0, "QGemv: K mismatch"),
    ((9, 4096), (64, 128, 16), 0, "QGemv: rows must be in [1,8]"),
    ((1, 4096), (64, 128, 16), 1, "Q4Gemv iq2: needs 2..8 rows and K % 128 == 0"),
    ((2, 4160), (64, 130, 16), 1, "Q4Gemv iq2: needs 2..8 rows and K % 128 == 0"),
    ((1, 4096), (64, 128, 16), 2, "Q4Gemv iq2=2: needs B [N, K/32, 8] and 1..8 rows"),
    ((9, 4096), (64, 128, 8), 2, "Q4Gemv iq2=2: needs B [N, K/32, 8] and 1..8 rows"),
    ((1, 4128), (64, 129, 8), 2, "Q4Gemv iq2=2: needs B [N, K/32, 8] and 1..8 rows"),
])
def test_q4_validation(x_shape, b_shape, iq2, msg):
    rc, err = _call_q4(x_shape, b_shape, iq2)
    assert rc == 1 and err == msg


def test_q8_validation():
    lib = _lib.lib()
    xs, k1 = _sh(1, 4096)
    bs, k2 = _sh(64, 64, 32)
    assert lib.bolt_q8_gemv(NULL, xs, 2, NULL, bs, 3, NULL, NULL, NULL) == 1
    assert _lib.last_error() == "QGemv: K mismatch"


@pytest.mark.parametrize("x_shape,w_shape,msg", [
    ((1, 4096), (64, 1024), "Nvfp4Gemv: K mismatch (K % 1024 required)"),
    ((1, 3072 + 64), (64, 1568), "Nvfp4Gemv: K mismatch (K % 1024 required)"),
    ((9, 4096), (64, 2048), "Nvfp4Gemv: rows must be in [1,8]"),
])
def test_nvfp4_validation(x_shape, w_shape, msg):
    lib = _lib.lib()
    xs, k1 = _sh(*x_shape)
    ws, k2 = _sh(*w_shape)
    assert lib.bolt_nvfp4_gemv(NULL, xs, len(x_shape), NULL, ws, len(w_shape), NULL, NULL, NULL, NULL) == 1
    assert _lib.last_error() == msg


@pytest.mark.parametrize("x_shape,gw_shape,topk", [((1, 4096), (513, 4096), 8), ((1, 4000), (304, 4000), 8),
                                                   ((1, 4096), (304, 4096), 33)])
def test_route_validation(x_shape, gw_shape, topk):
    lib = _lib.lib()
    xs, k1 = _sh(*x_shape)
    gs, k2 = _sh(*gw_shape)
    rc = lib.bolt_moe_route(NULL, xs, 2, NULL, gs, 2, NULL, topk, 5.0, NULL, NULL, NULL, NULL)
    assert rc == 1 and _lib.last_error() == "MoeRoute: unsupported shape"


def test_moe_validation():
    lib = _lib.lib()
    zs, k1 = _sh(1, 512)
    ws, k2 = _sh(304, 2304, 512)
    rc = lib.bolt_moe_decode(NULL, zs, 2, NULL, NULL, NULL, ws, 3, NULL, NULL, NULL, 8, NULL, NULL, NULL, NULL)
    assert rc == 1 and _lib.last_error() == "MoeDecode: latent size must be 1024"
    zs, k1 = _sh(1, 1024)
    ws, k2 = _sh(304, 2300, 512)
    rc = lib.bolt_moe_decode(NULL, zs, 2, NULL, NULL, NULL, ws, 3, NULL, NULL, NULL, 8, NULL, NULL, NULL, NULL)
    assert rc == 1 and _lib.last_error() == "MoeDecode: bad inter size"
    zs, k1 = _sh(9, 1024)
    ws, k2 = _sh(304, 2304, 512)
    rc = lib.bolt_moe_verify(NULL, zs, 2, NULL, NULL, NULL, ws, 3, NULL, NULL, NULL, 8, 0, NULL, NULL, NULL, NULL, NULL)
    assert rc == 1 and _lib.last_error() == "MoeVerify: rows must be in [1,8] and rows*topk <= 128"
    zs, k1 = _sh(8, 1024)
    rc = lib.bolt_moe_verify(NULL, zs, 2, NULL, NULL, NULL, ws, 3, NULL, NULL, NULL, 17, 0, NULL, NULL, NULL, NULL, NULL)
    assert rc == 1 and _lib.last_error() == "MoeVerify: rows must be in [1,8] and rows*topk <= 128"
    ws, k2 = _sh(304, 2336, 512)
    rc = lib.bolt_moe_verify(NULL, zs, 2, NULL, NULL, NULL, ws, 3, NULL, NULL, NULL, 8, 0, NULL, NULL, NULL, NULL, NULL)
    assert rc == 1 and _lib.last_error() == "MoeVerify: inter size must be a multiple of 64"


def test_dequant_validation():
    lib = _lib.lib()
    assert lib.bolt_dequant(7, 0, NULL, NULL, 4, 64, NULL, NULL) == 1
    assert _lib.last_error() == "bolt_dequant: unknown format"
    assert lib.bolt_dequant(2, 1, NULL, NULL, 4, 64, NULL, NULL) == 1


def test_relu2_validation_and_empty():
    lib = _lib.lib()
    xs, k1 = _sh(3, -1)
    assert lib.bolt_relu2(NULL, xs, 2, NULL, NULL) != 0
    assert "Relu2: negative dimension" in _lib.last_error()
    xs, k2 = _sh(0, 1000)  # nothing to do: no device work, no pointer needed
    assert lib.bolt_relu2(NULL, xs, 2, NULL, NULL) == 0


def _call_mamba(proj_shape, cs_shape, ss_shape, hd=64, ds=128, heads=16, ng=4, sel=False):
    lib = _lib.lib()
    ps, k1 = _sh(*proj_shape)
    cs, k2 = _sh(*cs_shape)
    ss, k3 = _sh(*ss_shape)
    head = [NULL, ps, len(proj_shape), NULL, cs, len(cs_shape), NULL, ss, len(ss_shape)] + [NULL] * 6
    tail = [heads, hd, ds, ng, 1e-5, 1e-3] + [NULL] * 6
    if sel:
        rc = lib.bolt_mamba_verify(*head, ctypes.c_void_p(16), *tail)
    else:
        rc = lib.bolt_mamba_step(*head, *tail)
    return rc, _lib.last_error()


@pytest.mark.parametrize("kw,msg", [
    (dict(hd=32), "MambaStep: only head_dim=64, d_state=128 are implemented"),
    (dict(proj_shape=(17, 3088)), "MambaStep: rows must be in [1,16]"),
    (dict(proj_shape=(2, 3000)), "MambaStep: bad proj width"),
    (dict(ng=3), "MambaStep: heads must be a multiple of n_groups"),
    (dict(proj_shape=(4, 3088), sel=True), "MambaVerify: state buffer needs >= R rows"),
    (dict(cs_shape=(2, 2048, 4)), "MambaStep: conv state must be [rows, conv_dim, 3]"),
    (dict(ss_shape=(2, 16, 128, 32)), "MambaStep: ssm state must be"),
])
def test_mamba_validation(kw, msg):
    args = dict(proj_shape=(2, 3088), cs_shape=(2, 2048, 3), ss_shape=(2, 16, 128, 64))
    args.update(kw)
    rc, err = _call_mamba(**args)
    assert rc != 0 and msg in err, err


def test_memcpy_async_validation():
    lib = _lib.lib()
    assert lib.bolt_memcpy_async(NULL, NULL, 0, NULL) == 0  # nothing to copy: no CUDA call
    assert lib.bolt_memcpy_async(NULL, NULL, -1, NULL) != 0
    assert b"negative size" in lib.bolt_last_error()
    assert lib.bolt_memcpy_async(NULL, NULL, 16, NULL) != 0
    assert b"null buffer" in lib.bolt_last_error()
