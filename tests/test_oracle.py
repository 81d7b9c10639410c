"""CPU checks of the oracle itself: each restated shader against an independent
numpy formulation of the same reference semantics, and the reference's own
plan invariants (test/model/palette-expander.test.ts:147-247)."""
from __future__ import annotations

import numpy as np
import pytest


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_tile_major_vec4_contiguity(oracle, pk):
    # palette-expander.test.ts:147-176 (fp32, N128) and :178-247 (fp16, N256)
    for tile_cols, inner, columns in ((128, 64, 256), (256, 64, 3072), (256, 64, 1024)):
        for scalar in range(0, inner * columns, 4 * 7):
            s = scalar - scalar % 4
            phys = oracle.tile_major_index(s, inner, columns, tile_cols)
            assert phys % 4 == 0
            assert pk.runtime_plan.tile_major_index(s, inner, columns, tile_cols) == phys
            for c in range(1, 4):
                assert oracle.tile_major_index(s + c, inner, columns, tile_cols) == phys + c


def test_tile_major_is_a_permutation(oracle):
    inner, columns = 64, 512
    idx = {oracle.tile_major_index(s, inner, columns, 256) for s in range(inner * columns)}
    assert idx == set(range(inner * columns))


def test_palette_groups_never_straddle_codes():
    # palette-expander.test.ts:178-212: a code group never crosses a palette boundary.
    for bits, columns, group_cols in ((5, 3072, 1024), (6, 1024, 1024)):
        per = 32 if bits == 5 else 16
        for base in range(0, 64 * columns, per):
            assert len({((base + c) % columns) // group_cols for c in range(per)}) == 1


@pytest.mark.parametrize("bits,dtype,layout,groups", [
    (5, np.float16, 0, 1), (5, np.float16, 1, 3), (6, np.float16, 1, 1),
    (5, np.float32, 0, 1), (5, np.float32, 1, 1), (6, np.float32, 1, 1),
])
def test_palette_expand_matches_numpy(oracle, pk, bits, dtype, layout, groups):
    rng = np.random.default_rng(bits * 10 + layout)
    inner, columns = 64, 768
    per, words = (32, 5) if bits == 5 else (16, 3)
    packed = rng.integers(0, 1 << 32, size=(inner * columns // per, words), dtype=np.uint64).astype("<u4")
    lut = rng.standard_normal((groups, 1 << bits)).astype(dtype)
    out = oracle.palette_expand(packed, lut, bits, inner, columns, layout=layout)
    dense = pk.runtime_plan.expand(packed, lut, bits, inner, columns).reshape(-1)
    if layout == 0:
        np.testing.assert_array_equal(out, dense)
    else:
        tile = 256 if dtype == np.float16 else 128
        idx = np.array([pk.runtime_plan.tile_major_index(s, inner, columns, tile) for s in range(inner * columns)])
        np.testing.assert_array_equal(out[idx], dense)


def _dense(pk, packed, lut, bits, inner, columns):
    return pk.runtime_plan.expand(packed, lut, bits, inner, columns).astype(np.float64)


@pytest.mark.parametrize("act,bias,res_scale", [("none", False, None), ("silu", False, None),
                                                ("relu", True, None), ("none", False, 0.5), ("none", False, 1.0)])
def test_gemm_wide_matches_float64(oracle, pk, act, bias, res_scale):
    rng = np.random.default_rng(1)
    rows, inner, columns, bits = 37, 256, 256, 5
    codes, lut = pk.synthetic.palette_matrix(rng, inner, columns, bits, 1, "fp32")
    a = rng.standard_normal((rows, inner)).astype(np.float32)
    b = rng.standard_normal(columns).astype(np.float32) if bias else None
    r = rng.standard_normal((rows, columns)).astype(np.float32) if res_scale is not None else None
    out = oracle.palette_gemm(a, codes["data"], lut["data"], bits, columns, bias=b, residual=r,
                              residual_scale=res_scale or 1.0, activation=act, acc_mode=1)
    v = a.astype(np.float64) @ _dense(pk, codes["data"], lut["data"], bits, inner, columns)
    if b is not None:
        v = v + b
    if act == "silu":
        v = v / (1 + np.exp(-np.clip(v, -20, 20)))
    elif act == "relu":
        v = np.maximum(v, 0)
    if r is not None:
        v = r + res_scale * v
    assert rel(out, v) < 1e-6


def test_fp32_reference_mode_is_the_fp32_fma_chain(oracle, pk):
    # FP32 package: reference mode == wide mode (both one fp32 fma chain).
    rng = np.random.default_rng(2)
    codes, lut = pk.synthetic.palette_matrix(rng, 128, 64, 6, 1, "fp32")
    a = rng.standard_normal((9, 128)).astype(np.float32)
    r0 = oracle.palette_gemm(a, codes["data"], lut["data"], 6, 64, acc_mode=0)
    r1 = oracle.palette_gemm(a, codes["data"], lut["data"], 6, 64, acc_mode=1)
    np.testing.assert_array_equal(r0, r1)


def test_f16_accumulation_is_within_package_tolerance(oracle, pk):
    # The reference's f16-accumulating GEMM vs exact math: this is the error
    # budget the FP16 package tolerance (2e-2) has to absorb.
    rng = np.random.default_rng(3)
    rows, inner, columns = 64, 1024, 512
    codes, lut = pk.synthetic.palette_matrix(rng, inner, columns, 5, 1, "fp16")
    a = rng.standard_normal((rows, inner)).astype(np.float16)
    ref = oracle.palette_gemm(a, codes["data"], lut["data"], 5, columns, acc_mode=0)
    wide = oracle.palette_gemm(a, codes["data"], lut["data"], 5, columns, acc_mode=1)
    exact = a.astype(np.float64) @ _dense(pk, codes["data"], lut["data"], 5, inner, columns)
    assert rel(wide, exact) < 1e-3
    assert 1e-4 < rel(ref, exact) < 2e-2


def test_layernorm_matches_numpy(oracle):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((50, 1024)) * 3 + 1).astype(np.float16)
    g = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    y = oracle.layernorm(x, g, b)
    xf = x.astype(np.float64)
    m = xf.mean(1, keepdims=True)
    v = np.maximum((xf * xf).mean(1, keepdims=True) - m * m, 0)
    ref = (xf - m) / np.sqrt(v + 1e-5) * g + b
    assert rel(y, ref) < 1e-3


def _attention_numpy(qkv, pos_packed, u, v, lens, batch, frames):
    P = 2 * frames - 1
    pos = pos_packed.astype(np.float64).transpose(2, 0, 1, 3).reshape(P, 1024)  # [P, C]
    q = qkv[:, :1024].astype(np.float64).reshape(batch, frames, 8, 128)
    k = qkv[:, 1024:2048].astype(np.float64).reshape(batch, frames, 8, 128)
    vv = qkv[:, 2048:].astype(np.float64).reshape(batch, frames, 8, 128)
    out = np.zeros((batch, frames, 8, 128))
    for b in range(batch):
        L = min(int(lens[b]), frames)
        for h in range(8):
            pu = q[b, :L, h] + u[h]
            pv = q[b, :L, h] + v[h]
            ac = pu @ k[b, :L, h].T
            rel_idx = frames - 1 - np.arange(L)[:, None] + np.arange(L)[None, :]
            bd = np.einsum("id,ijd->ij", pv, pos[rel_idx][:, :, h * 128:(h + 1) * 128])
            s = (ac + bd) / np.sqrt(128)
            s = np.exp(s - s.max(1, keepdims=True))
            s /= s.sum(1, keepdims=True)
            out[b, :L, h] = s @ vv[b, :L, h]
    return out.reshape(batch * frames, 1024)


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_attention_matches_numpy(oracle, dtype):
    rng = np.random.default_rng(5)
    batch, frames = 2, 20
    qkv = rng.standard_normal((batch * frames, 3072)).astype(dtype)
    pos = (rng.standard_normal((8, 32, 2 * frames - 1, 4)) * 0.5).astype(dtype)
    u = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    v = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    lens = np.array([20, 13], np.uint32)
    out = oracle.rel_attention(qkv, pos, u, v, lens, batch, frames)
    ref = _attention_numpy(qkv, pos, u, v, lens, batch, frames)
    assert rel(out, ref) < (2e-3 if dtype == np.float16 else 1e-5)
    assert np.all(out.reshape(batch, frames, 1024)[1, 13:] == 0)


def test_conformer_conv_matches_numpy(oracle):
    rng = np.random.default_rng(6)
    batch, frames = 2, 30
    g = rng.standard_normal((batch * frames, 2048)).astype(np.float32)
    dw = (0.1 * rng.standard_normal((9, 1024))).astype(np.float32)
    sc = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    sh = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    lens = np.array([30, 11], np.uint32)
    out = oracle.conformer_conv(g, dw, sc, sh, lens, batch, frames)
    sig = lambda x: 1 / (1 + np.exp(-np.clip(x, -20, 20)))  # noqa: E731
    gg = g.astype(np.float64).reshape(batch, frames, 2048)
    ref = np.zeros((batch, frames, 1024))
    for b in range(batch):
        glu = gg[b, :, :1024] * sig(gg[b, :, 1024:])
        glu[lens[b]:] = 0
        pad = np.concatenate([np.zeros((4, 1024)), glu, np.zeros((4, 1024))])
        s = sum(pad[k:k + frames] * dw[k] for k in range(9))
        a = s * sc + sh
        ref[b] = a * sig(a)
    assert rel(out, ref.reshape(-1, 1024)) < 1e-5


def test_subsampling_shapes_and_masks(oracle):
    rng = np.random.default_rng(7)
    fb = rng.normal(-4, 2, size=(2, 128, 1501)).astype(np.float32)
    w0 = (0.3 * rng.standard_normal((3, 3, 256))).astype(np.float16)
    b0 = (0.02 * rng.standard_normal(256)).astype(np.float32)
    wd = (0.1 * rng.standard_normal((3, 3, 256))).astype(np.float16)
    bd = (0.02 * rng.standard_normal(256)).astype(np.float32)
    lens = np.array([1501, 700], np.uint32)
    s376 = oracle.subsampling_conv0_dw2(fb, w0, b0, wd, bd, lens, np.float16)
    assert s376.shape == (2, 376, 32, 256)
    assert np.all(s376[1, oracle.sub_len(700, 2):] == 0)
    assert np.any(s376[1, : oracle.sub_len(700, 2)] != 0)
    # One conv0 + depthwise output checked by hand (window 0, row 10, col 5, ch 7).
    c = 7

    def conv0(y, x):
        s = np.float32(b0[c])
        for ky in range(3):
            iy = 2 * y + ky - 1
            if not 0 <= iy < 1501:
                continue
            for kx in range(3):
                ix = 2 * x + kx - 1
                if 0 <= ix < 128:
                    s = np.float32(s + np.float32(w0[ky, kx, c]) * fb[0, ix, iy])
        return np.float32(np.float16(max(s, 0)))

    s = np.float32(bd[c])
    for ky in range(3):
        for kx in range(3):
            iy, ix = 2 * 10 + ky - 1, 2 * 5 + kx - 1
            if 0 <= iy < 751 and 0 <= ix < 64:
                s = s + conv0(iy, ix) * np.float32(wd[ky, kx, c])
    assert abs(float(s376[0, 10, 5, c]) - float(s)) < 2e-3 * max(1.0, abs(float(s)))
