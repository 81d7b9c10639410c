"""GPU parity of every operator against the CPU oracle, through the C ABI.

Bars: palette expansion bit-exact; FP32 GEMM (CUDA-core fp32 fma chain)
bit-exact with the oracle; FP16 tensor-core GEMM within 2e-3 relative
Frobenius of the oracle's wide (fp32-accumulate) mode and within the FP16
package tolerance 2e-2 of the reference algorithm (f16 accumulation); FP32
package ops within 1e-4; FP16 package ops within 2e-2 (tighter where the
arithmetic allows, stated per test)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import cuda, gemm, host, vp

pytestmark = pytest.mark.gpu

FP16_TOL = 2e-2  # north_star: FP16 package relative-Frobenius tolerance
FP32_TOL = 1e-4  # north_star: FP32 package relative-Frobenius tolerance
WIDE_TOL = 2e-3  # tensor-core fp32 accumulation vs oracle fp32 accumulation (f16 output rounding)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ------------------------------------------------------------------ expansion

@pytest.mark.parametrize("precision,bits,layout,groups,inner,columns", [
    ("fp16", 5, 0, 1, 256, 256), ("fp16", 5, 1, 1, 1024, 4096), ("fp16", 6, 1, 1, 1024, 1024),
    ("fp16", 5, 1, 3, 1024, 3072), ("fp32", 5, 0, 1, 4096, 1024), ("fp32", 5, 1, 1, 1024, 2048),
    ("fp32", 6, 1, 1, 1024, 4096),
])
def test_palette_expand_bit_exact(pk, oracle, device, precision, bits, layout, groups, inner, columns):
    import torch

    rng = np.random.default_rng(inner + columns + bits)
    codes, lut = pk.synthetic.palette_matrix(rng, inner, columns, bits, groups, precision)
    dt = np.float16 if precision == "fp16" else np.float32
    out = torch.empty(inner * columns, dtype=torch.float16 if precision == "fp16" else torch.float32,
                      device="cuda")
    tc, tl = cuda(codes["data"]), cuda(lut["data"])
    L = pk._lib
    desc = L.PaletteDesc(L.FP16 if precision == "fp16" else L.FP32, bits, inner, columns, groups,
                         columns // groups, layout, vp(tc), vp(tl), vp(out))
    L.call("pk_palette_expand", device.handle, ctypes.byref(desc), None)
    ref = oracle.palette_expand(codes["data"], lut["data"], bits, inner, columns, layout=layout)
    np.testing.assert_array_equal(host(out).view(np.uint16 if dt == np.float16 else np.uint32),
                                  ref.view(np.uint16 if dt == np.float16 else np.uint32))


def test_palette_expand_rejects_row_major_palette6(pk, device):
    L = pk._lib
    dummy = cuda(np.zeros(16, np.float32))
    desc = L.PaletteDesc(L.FP16, 6, 32, 64, 1, 64, 0, vp(dummy), vp(dummy), vp(dummy))
    with pytest.raises(pk.PkError, match="no row-major palette6"):
        L.call("pk_palette_expand", device.handle, ctypes.byref(desc), None)


# ------------------------------------------------------------------ GEMM

GEMM_CASES = [
    # rows, inner, columns, bits, groups, act, bias, residual_scale
    (188, 1024, 4096, 5, 1, "silu", False, None),   # ff-expand, B1 prefix
    (376, 4096, 1024, 5, 1, "none", False, 0.5),    # ff-contract + half residual
    (188, 1024, 3072, 5, 3, "none", False, None),   # qkv, 3 palette groups
    (564, 1024, 1024, 6, 1, "none", False, 1.0),    # o_proj 6-bit + residual
    (300, 1024, 2048, 5, 1, "none", False, None),   # pw1, ragged row count
    (188, 1024, 640, 5, 1, "none", True, None),     # projector + bias
    (1000, 256, 256, 5, 1, "relu", True, None),     # subsampling pointwise
    (188, 4096, 1024, 5, 1, "none", True, None),    # flatten projection
    (1, 1024, 1024, 5, 1, "none", False, 1.0),      # single row
    (129, 1024, 1024, 6, 1, "silu", False, None),   # 6-bit, just past one 128 tile
]


def _gemm_inputs(pk, case, precision, seed):
    rows, inner, columns, bits, groups, act, bias, rs = case
    rng = np.random.default_rng(seed)
    codes, lut = pk.synthetic.palette_matrix(rng, inner, columns, bits, groups, precision)
    dt = np.float16 if precision == "fp16" else np.float32
    a = rng.standard_normal((rows, inner)).astype(dt)
    b = (0.1 * rng.standard_normal(columns)).astype(np.float32) if bias else None
    r = rng.standard_normal((rows, columns)).astype(dt) if rs is not None else None
    return a, codes["data"], lut["data"], b, r


@pytest.mark.parametrize("case", GEMM_CASES)
def test_fp16_tensor_core_gemm(pk, oracle, device, case):
    rows, inner, columns, bits, groups, act, bias, rs = case
    a, codes, lut, b, r = _gemm_inputs(pk, case, "fp16", rows + columns)
    pk.kernels.set_gemm_route("tensor")
    try:
        out = gemm(pk, device, a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
                   activation=act)
    finally:
        pk.kernels.set_gemm_route("auto")
    assert device.status() == 0
    assert np.isfinite(out).all()
    wide = oracle.palette_gemm(a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
                               activation=act, acc_mode=1)
    assert rel(out, wide) < WIDE_TOL
    ref = oracle.palette_gemm(a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
                              activation=act, acc_mode=0)
    assert rel(out, ref) < FP16_TOL


PAIR_CASES = [c for c in GEMM_CASES if c[2] % 256 == 0] + [
    (6016, 1024, 1024, 5, 1, "none", False, 1.0),  # C3 o_proj shape, 47 row tiles of 128
    (3000, 4096, 1024, 6, 1, "none", True, None),  # 6-bit, bias, K = 4096, ragged rows
    (700, 1024, 1024, 5, 1, "none", False, 0.3),   # residual scale not a power of two: single-CTA path
    (300, 1024, 2048, 5, 1, "silu", False, 0.5),   # activation before a residual: single-CTA path
]


@pytest.mark.parametrize("tile", [-256, -384, -512])
@pytest.mark.parametrize("case", PAIR_CASES)
def test_fp16_cta_pair_gemm(pk, oracle, device, case, tile):
    """The cta_group::2 kernel (256 features per CTA pair, half of a 256-,
    384- or 512-token tile per CTA, one or two MMAs per decoded weight stage)
    against the oracle's wide mode and the single-CTA kernel."""
    rows, inner, columns, bits, groups, act, bias, rs = case
    a, codes, lut, b, r = _gemm_inputs(pk, case, "fp16", 5 * rows + columns)
    kw = dict(bias=b, residual=r, residual_scale=rs or 1.0, activation=act)
    try:
        pk.kernels.set_gemm_tile(tile)
        pair = gemm(pk, device, a, codes, lut, bits, columns, **kw)
        pair2 = gemm(pk, device, a, codes, lut, bits, columns, **kw)
        pk.kernels.set_gemm_tile(0)
        pk.kernels.set_gemm_route("tensor-single")
        single = gemm(pk, device, a, codes, lut, bits, columns, **kw)
    finally:
        pk.kernels.set_gemm_tile(0)
        pk.kernels.set_gemm_route("auto")
    assert device.status() == 0
    np.testing.assert_array_equal(pair.view(np.uint16), pair2.view(np.uint16))  # deterministic
    assert rel(pair, single) < 1e-3
    if rows <= 1024:
        wide = oracle.palette_gemm(a, codes, lut, bits, columns, acc_mode=1, **kw)
        assert rel(pair, wide) < WIDE_TOL


@pytest.mark.parametrize("case", GEMM_CASES[:6])
def test_fp16_simt_gemm_matches_oracle_wide(pk, oracle, device, case):
    rows, inner, columns, bits, groups, act, bias, rs = case
    a, codes, lut, b, r = _gemm_inputs(pk, case, "fp16", rows * 3 + columns)
    pk.kernels.set_gemm_route("simt")
    try:
        out = gemm(pk, device, a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
                   activation=act)
    finally:
        pk.kernels.set_gemm_route("auto")
    wide = oracle.palette_gemm(a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
                               activation=act, acc_mode=1)
    assert rel(out, wide) < WIDE_TOL


@pytest.mark.parametrize("case", [GEMM_CASES[i] for i in (0, 1, 3, 5, 6)])
def test_fp32_gemm_bit_exact(pk, oracle, device, case):
    rows, inner, columns, bits, groups, act, bias, rs = case
    a, codes, lut, b, r = _gemm_inputs(pk, case, "fp32", rows + 7 * columns)
    out = gemm(pk, device, a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
               activation=act)
    ref = oracle.palette_gemm(a, codes, lut, bits, columns, bias=b, residual=r, residual_scale=rs or 1.0,
                              activation=act, acc_mode=0)
    if act == "none":
        np.testing.assert_array_equal(out.view(np.uint32), ref.view(np.uint32))
    assert rel(out, ref) < FP32_TOL / 100


def test_config1_fp32_single_gemm(pk, oracle, device):
    """[188x1024] f32 N(0,1) x 6-bit [1024x4096] with a sorted
    64-entry N(0, 0.02) f32 LUT, seed 0; raw product and SiLU epilogue."""
    rng = np.random.default_rng(0)
    a = rng.standard_normal((188, 1024)).astype(np.float32)
    codes, lut = pk.synthetic.palette_matrix(rng, 1024, 4096, 6, 1, "fp32")
    for act in ("none", "silu"):
        out = gemm(pk, device, a, codes["data"], lut["data"], 6, 4096, activation=act)
        ref = oracle.palette_gemm(a, codes["data"], lut["data"], 6, 4096, activation=act, acc_mode=0)
        assert rel(out, ref) < FP32_TOL


def test_tensor_core_gemm_large_vs_simt(pk, device):
    """Full-size check (C3 ff-expand shape, M = 32 x 188) of the tcgen05 kernel
    against the independent CUDA-core kernel, both fp32-accumulating."""
    import torch

    rng = np.random.default_rng(11)
    rows, inner, columns = 6016, 1024, 4096
    codes, lut = pk.synthetic.palette_matrix(rng, inner, columns, 5, 1, "fp16")
    a = rng.standard_normal((rows, inner)).astype(np.float16)
    pk.kernels.set_gemm_route("simt")
    simt = gemm(pk, device, a, codes["data"], lut["data"], 5, columns, activation="silu")
    pk.kernels.set_gemm_route("tensor")
    try:
        tc1 = gemm(pk, device, a, codes["data"], lut["data"], 5, columns, activation="silu")
        tc2 = gemm(pk, device, a, codes["data"], lut["data"], 5, columns, activation="silu")
    finally:
        pk.kernels.set_gemm_route("auto")
    assert device.status() == 0
    np.testing.assert_array_equal(tc1.view(np.uint16), tc2.view(np.uint16))  # deterministic
    assert rel(tc1, simt) < WIDE_TOL
    # Every row is independent of the others: a one-row launch reproduces row 777 bit-exactly.
    pk.kernels.set_gemm_route("tensor")
    try:
        one = gemm(pk, device, a[777:778].copy(), codes["data"], lut["data"], 5, columns, activation="silu")
    finally:
        pk.kernels.set_gemm_route("auto")
    np.testing.assert_array_equal(one[0].view(np.uint16), tc1[777].view(np.uint16))
    del torch


def test_gemm_rejects_bad_shapes(pk, device):
    L = pk._lib
    x = cuda(np.zeros(64, np.float32))
    desc = L.GemmDesc(L.FP16, 10, 100, 256, 5, 1, 256, 0, 0, 1.0, None, None, vp(x), vp(x), vp(x), vp(x))
    with pytest.raises(pk.PkError, match="PK_E_SHAPE"):
        L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), None)
    desc = L.GemmDesc(L.FP16, 10, 128, 256, 5, 1, 256, 0, 1, 1.0, vp(x), vp(x), vp(x), vp(x), vp(x), vp(x))
    with pytest.raises(pk.PkError, match="bias and residual"):
        L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), None)
    desc = L.GemmDesc(L.FP16, 10, 128, 256, 7, 1, 256, 0, 0, 1.0, None, None, vp(x), vp(x), vp(x), vp(x))
    with pytest.raises(pk.PkError, match="PK_E_LAYOUT"):
        L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), None)


def test_operator_api_gemm_dispatch_active_rows(pk, oracle, device):
    """The reference operator flow: create -> createDispatch (B40 signature) ->
    encode(shape={rows}) on an active prefix."""
    import torch

    K = pk.kernels
    rng = np.random.default_rng(21)
    codes, lut = pk.synthetic.palette_matrix(rng, 1024, 4096, 5, 1, "fp16")
    b = K.GpuTensor.from_record("ff1", codes)
    pal = K.GpuTensor.from_record("ff1.palette", lut)
    a = torch.from_numpy(rng.standard_normal((7520, 1024)).astype(np.float16)).cuda()
    out = torch.zeros((7520, 4096), dtype=torch.float16, device="cuda")
    kern = K.F16GemmKernel.create(device)
    disp = kern.create_dispatch(K.GemmDescriptor("ff1", a, b, out, 7520, 1024, 4096, b_palette=pal,
                                                 palette_group_columns=4096, activation="silu"))
    disp.encode(shape={"rows": 376})
    got = host(out)
    ref = oracle.palette_gemm(a[:376].cpu().numpy(), codes["data"], lut["data"], 5, 4096, activation="silu",
                              acc_mode=1)
    assert rel(got[:376], ref) < WIDE_TOL
    assert np.all(got[376:] == 0)  # rows past the active prefix untouched
    with pytest.raises(K.RangeError):
        disp.encode(shape={"rows": 7521})


# ------------------------------------------------------------------ LayerNorm

@pytest.mark.parametrize("precision,rows", [("fp16", 6016), ("fp16", 3), ("fp32", 376)])
def test_layernorm(pk, oracle, device, precision, rows):
    import torch

    rng = np.random.default_rng(rows)
    dt = np.float16 if precision == "fp16" else np.float32
    x = (rng.standard_normal((rows, 1024)) * 2 + 0.5).astype(dt)
    g = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    bb = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    tx, y = cuda(x), torch.empty((rows, 1024), dtype=torch.float16 if dt == np.float16 else torch.float32,
                                 device="cuda")
    pk._lib.call("pk_layernorm", device.handle, pk._lib.FP16 if dt == np.float16 else pk._lib.FP32, rows, 1024,
                 vp(tx), vp(cuda(g)), vp(cuda(bb)), 1e-5, vp(y), None)
    ref = oracle.layernorm(x, g, bb)
    assert rel(host(y), ref) < (1e-3 if dt == np.float16 else 1e-6)


# ------------------------------------------------------------------ attention

@pytest.mark.parametrize("precision,lengths", [("fp16", [188, 188]), ("fp16", [150, 1, 188]),
                                               ("fp32", [188, 97])])
def test_rel_attention(pk, oracle, device, precision, lengths):
    import torch

    batch, frames = len(lengths), 188
    rng = np.random.default_rng(sum(lengths))
    dt = np.float16 if precision == "fp16" else np.float32
    qkv = rng.standard_normal((batch * frames, 3072)).astype(dt)
    pos = (0.5 * rng.standard_normal((8, 32, 375, 4))).astype(dt)
    u = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    v = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    lens = np.array(lengths, np.uint32)
    ctx = torch.full((batch * frames, 1024), float("nan"),
                     dtype=torch.float16 if dt == np.float16 else torch.float32, device="cuda")
    pk._lib.call("pk_rel_attention", device.handle, pk._lib.FP16 if dt == np.float16 else pk._lib.FP32, batch,
                 frames, vp(cuda(qkv)), vp(cuda(pos)), vp(cuda(u)), vp(cuda(v)), vp(cuda(lens)), vp(ctx), None)
    got = host(ctx)
    ref = oracle.rel_attention(qkv, pos, u, v, lens, batch, frames)
    assert np.isfinite(got).all()
    assert rel(got, ref) < (FP16_TOL / 4 if dt == np.float16 else FP32_TOL)
    for b, L in enumerate(lengths):
        assert np.all(got.reshape(batch, frames, 1024)[b, L:] == 0)


def test_rel_attention_simt_route_matches_tensor_core(pk, oracle, device):
    """FP16: the CUDA-core kernel (f32 math throughout, like the shader) and the
    tensor-core kernel agree with the oracle and with each other."""
    import torch

    batch, frames = 2, 188
    rng = np.random.default_rng(77)
    qkv = rng.standard_normal((batch * frames, 3072)).astype(np.float16)
    pos = (0.5 * rng.standard_normal((8, 32, 375, 4))).astype(np.float16)
    u = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    v = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    lens = np.array([188, 61], np.uint32)
    outs = []
    for route in ("simt", "auto"):
        ctx = torch.full((batch * frames, 1024), float("nan"), dtype=torch.float16, device="cuda")
        pk.kernels.set_attention_route(route)
        try:
            pk._lib.call("pk_rel_attention", device.handle, pk._lib.FP16, batch, frames, vp(cuda(qkv)),
                         vp(cuda(pos)), vp(cuda(u)), vp(cuda(v)), vp(cuda(lens)), vp(ctx), None)
        finally:
            pk.kernels.set_attention_route("auto")
        outs.append(host(ctx))
    ref = oracle.rel_attention(qkv, pos, u, v, lens, batch, frames)
    assert rel(outs[0], ref) < 1e-3
    assert rel(outs[1], ref) < 5e-3
    assert rel(outs[0], outs[1]) < 5e-3


@pytest.mark.parametrize("frames,lengths", [(188, [188, 150, 1]), (192, [192, 130]), (77, [77, 40]),
                                            (129, [129, 128])])
def test_rel_attention_tcgen05(pk, oracle, device, frames, lengths):
    """FP16 tcgen05 kernel (positions row-major, as the encoder holds them)
    against the oracle and against the mma.sync kernel."""
    import torch

    batch = len(lengths)
    rng = np.random.default_rng(frames + sum(lengths))
    P = 2 * frames - 1
    qkv = rng.standard_normal((batch * frames, 3072)).astype(np.float16)
    pos = (0.5 * rng.standard_normal((8, 32, P, 4))).astype(np.float16)
    pos_rm = np.ascontiguousarray(pos.transpose(0, 2, 1, 3).reshape(8, P, 128))
    u = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    v = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    lens = np.array(lengths, np.uint32)
    outs = []
    for route, positions in (("tcgen05-rowmajor", pos_rm), ("mma", pos), ("tcgen05-rowmajor", pos_rm)):
        ctx = torch.full((batch * frames, 1024), float("nan"), dtype=torch.float16, device="cuda")
        pk.kernels.set_attention_route(route)
        try:
            pk._lib.call("pk_rel_attention", device.handle, pk._lib.FP16, batch, frames, vp(cuda(qkv)),
                         vp(cuda(positions)), vp(cuda(u)), vp(cuda(v)), vp(cuda(lens)), vp(ctx), None)
        finally:
            pk.kernels.set_attention_route("auto")
        outs.append(host(ctx))
    assert device.status() == 0
    ref = oracle.rel_attention(qkv, pos, u, v, lens, batch, frames)
    got = outs[0]
    assert np.isfinite(got).all()
    assert rel(got, ref) < FP16_TOL / 4
    assert rel(got, outs[1]) < 5e-3
    np.testing.assert_array_equal(got, outs[2])  # deterministic
    for b, L in enumerate(lengths):
        assert np.all(got.reshape(batch, frames, 1024)[b, L:] == 0)


def test_rel_attention_rejects_long_windows(pk, device):
    x = cuda(np.zeros(8, np.float32))
    with pytest.raises(pk.PkError, match="PK_E_SHAPE"):
        pk._lib.call("pk_rel_attention", device.handle, 0, 1, 193, vp(x), vp(x), vp(x), vp(x), vp(x), vp(x), None)


# ------------------------------------------------------------------ conformer conv

@pytest.mark.parametrize("precision,lengths", [("fp16", [188, 120]), ("fp32", [188, 5, 188])])
def test_conformer_conv(pk, oracle, device, precision, lengths):
    import torch

    batch, frames = len(lengths), 188
    rng = np.random.default_rng(len(lengths) * 31)
    dt = np.float16 if precision == "fp16" else np.float32
    g = rng.standard_normal((batch * frames, 2048)).astype(dt)
    dw = (0.1 * rng.standard_normal((9, 1024))).astype(dt)
    sc = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    sh = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    lens = np.array(lengths, np.uint32)
    out = torch.empty((batch * frames, 1024), dtype=torch.float16 if dt == np.float16 else torch.float32,
                      device="cuda")
    pk._lib.call("pk_conformer_conv", device.handle, pk._lib.FP16 if dt == np.float16 else pk._lib.FP32, batch,
                 frames, vp(cuda(g)), vp(cuda(dw)), vp(cuda(sc)), vp(cuda(sh)), vp(cuda(lens)), vp(out), None)
    ref = oracle.conformer_conv(g, dw, sc, sh, lens, batch, frames)
    assert rel(host(out), ref) < (1e-3 if dt == np.float16 else 1e-6)


# ------------------------------------------------------------------ subsampling

@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_subsampling_kernels(pk, oracle, device, precision):
    import torch

    rng = np.random.default_rng(5)
    dt = np.float16 if precision == "fp16" else np.float32
    tdt = torch.float16 if precision == "fp16" else torch.float32
    P = pk._lib.FP16 if precision == "fp16" else pk._lib.FP32
    lens = np.array([1501, 1500, 777], np.uint32)
    batch = len(lens)
    fb = rng.normal(-4, 2, size=(batch, 128, 1501)).astype(np.float32)
    w0 = (0.3 * rng.standard_normal((3, 3, 256))).astype(dt)
    b0 = (0.02 * rng.standard_normal(256)).astype(np.float32)
    wd = (0.1 * rng.standard_normal((3, 3, 256))).astype(dt)
    bd = (0.02 * rng.standard_normal(256)).astype(np.float32)
    tl = cuda(lens)
    s376 = torch.empty((batch, 376, 32, 256), dtype=tdt, device="cuda")
    pk._lib.call("pk_subsampling_conv0_dw2", device.handle, P, batch, vp(cuda(fb)), vp(cuda(w0)), vp(cuda(b0)),
                 vp(cuda(wd)), vp(cuda(bd)), vp(tl), vp(s376), None)
    ref376 = oracle.subsampling_conv0_dw2(fb, w0, b0, wd, bd, lens, dt)
    assert rel(host(s376), ref376) < (2e-3 if dt == np.float16 else 1e-6)
    # depthwise 5 on the oracle's stage output
    w5 = (0.1 * rng.standard_normal((3, 3, 256))).astype(dt)
    b5 = (0.02 * rng.standard_normal(256)).astype(np.float32)
    s188 = torch.empty((batch, 188, 16, 256), dtype=tdt, device="cuda")
    pk._lib.call("pk_subsampling_depthwise", device.handle, P, batch, 376, 32, 256, vp(cuda(ref376)), vp(cuda(w5)),
                 vp(cuda(b5)), vp(tl), 3, vp(s188), None)
    ref188 = oracle.subsampling_depthwise(ref376, w5, b5, lens, 3)
    assert rel(host(s188), ref188) < (1e-3 if dt == np.float16 else 1e-6)
    # time mask
    vals = rng.standard_normal((batch, 188, 16, 256)).astype(dt)
    tv = cuda(vals)
    pk._lib.call("pk_subsampling_time_mask", device.handle, P, batch, 188, 16, 256, vp(tv), vp(tl), 3, None)
    np.testing.assert_array_equal(host(tv), oracle.subsampling_time_mask(vals, lens, 3))
