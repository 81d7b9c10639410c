"""CPU oracle for the parakeet.wgsl encoder hot path (TEST INFRASTRUCTURE ONLY).

This module wraps ``oracle/_build/libpk_oracle.so`` (built from ``pk_oracle.cpp``
by ``oracle/Makefile``) with numpy.  It is the checker for the CUDA library:
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import it, and nothing on the product path may.

Layer and encoder composition is restated here from
``src/webgpu/encoder.ts:1869-2138`` (one Conformer layer: 15 logical dispatches
over two rotating slots) and ``encoder.ts:2140-2430`` (subsampling front end),
with the projector from ``encoder.ts:1489-1509``.

Parity status: palette packing/expansion are pinned to the reference's
known-answer tests (tests/golden); the floating-point kernels are
"parity unpinned" (the reference tests pin WGSL text, not outputs).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libpk_oracle.so"
_lib = None

FP16, FP32 = 0, 1
ACT = {"none": 0, "silu": 1, "relu": 2}


def build() -> Path:
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def reference_root() -> Path | None:
    """The reference checkout: $PARAKEET_REFERENCE, else a directory named
    ``reference`` beside this repository; None when neither exists."""
    env = os.environ.get("PARAKEET_REFERENCE")
    for cand in ([Path(env)] if env else []) + [_HERE.parents[1] / "reference"]:
        if (cand / "src" / "cpp" / "fbank" / "parakeet_fbank.cpp").exists():
            return cand
    return None


def build_reference() -> bool:
    """Build oracle/_ref (the reference's own log-mel front end) when the
    reference checkout is present; a no-op otherwise.  Returns availability."""
    root = reference_root()
    if root is not None:
        subprocess.run(["make", "-s", "-C", str(_HERE), "ref", f"REFERENCE={root}"], check=True)
    return (_HERE / "_ref" / "libparakeet_fbank.so").exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        i64, i32, vp, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
        _lib.or_tile_major_index.restype = i64
        _lib.or_tile_major_index.argtypes = [i64, i64, i64, i64]
        _lib.or_unpack_codes.argtypes = [vp, i32, i64, vp]
        _lib.or_pack_codes.argtypes = [vp, i32, i64, vp]
        _lib.or_palette_expand.argtypes = [vp, vp, i32, i32, i64, i64, i32, i64, i32, vp]
        _lib.or_palette_gemm.argtypes = [i32, i32, i64, i64, i64, vp, vp, vp, i32, i32, i64,
                                         vp, vp, f32, i32, vp]
        _lib.or_layernorm.argtypes = [i32, i64, i64, vp, vp, vp, f32, vp]
        _lib.or_rel_attention.argtypes = [i32, i64, i64, vp, vp, vp, vp, vp, vp]
        _lib.or_conformer_conv.argtypes = [i32, i64, i64, vp, vp, vp, vp, vp, vp]
        _lib.or_subsampling_conv0_dw2.argtypes = [i32, i64, vp, vp, vp, vp, vp, vp, vp]
        _lib.or_subsampling_depthwise.argtypes = [i32, i64, i64, i64, i64, vp, vp, vp, vp, i32, vp]
        _lib.or_subsampling_time_mask.argtypes = [i32, i64, i64, i64, i64, vp, vp, i32]
        _lib.or_logmel.argtypes = [i64, i64, vp, vp, vp]
        _lib.or_logmel_tables.argtypes = [vp] * 6 + [i32]
        _lib.or_logmel_tables.restype = i32
        _lib.or_hfma_selfcheck.argtypes = [i64, ctypes.c_uint64]
        _lib.or_hfma_selfcheck.restype = i64
        _lib.or_tdt_decode.argtypes = [i32, i64, i64, i64, vp, vp, vp, vp, vp] + [vp] * 9 + [vp] * 4
    return _lib


def set_threads(n: int) -> None:
    os.environ["OMP_NUM_THREADS"] = str(n)


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _prec(dtype) -> int:
    return FP16 if np.dtype(dtype) == np.float16 else FP32


# -- palette format ---------------------------------------------------------

def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """LSB-first u32 packing (model/convert.py:2130-2157)."""
    flat = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    per, words = (32, 5) if bits == 5 else (16, 3)
    assert flat.size % per == 0
    out = np.zeros((flat.size // per, words), dtype="<u4")
    lib().or_pack_codes(_p(flat), bits, flat.size, _p(out))
    return out


def unpack_codes(packed: np.ndarray, bits: int) -> np.ndarray:
    per, words = (32, 5) if bits == 5 else (16, 3)
    packed = np.ascontiguousarray(packed, dtype="<u4")
    scalars = packed.size // words * per
    out = np.empty(scalars, dtype=np.uint8)
    lib().or_unpack_codes(_p(packed), bits, scalars, _p(out))
    return out


def tile_major_index(scalar: int, inner: int, columns: int, tile_cols: int) -> int:
    return int(lib().or_tile_major_index(scalar, inner, columns, tile_cols))


def palette_expand(codes, palette, bits, inner, columns, palette_groups=None, layout=0):
    """paletteDequantWgslForScalar (src/model/palette-expander.ts:478-587)."""
    palette = np.ascontiguousarray(palette)
    groups = palette.shape[0] if palette_groups is None else palette_groups
    prec = _prec(palette.dtype)
    out = np.empty(inner * columns, dtype=palette.dtype)
    lib().or_palette_expand(_p(np.ascontiguousarray(codes, dtype="<u4")), _p(palette), prec, bits,
                            inner, columns, groups, columns // groups, layout, _p(out))
    return out


def palette_gemm(a, codes, palette, bits, columns, *, bias=None, residual=None,
                 residual_scale=1.0, activation="none", acc_mode=0):
    """Palette GEMM restating gemm.ts:1362-1716 / :2356-2599 (see pk_oracle.cpp)."""
    a = np.ascontiguousarray(a)
    palette = np.ascontiguousarray(palette)
    rows, inner = a.shape
    prec = _prec(a.dtype)
    assert _prec(palette.dtype) == prec
    groups = palette.shape[0]
    out = np.empty((rows, columns), dtype=a.dtype)
    if residual is not None:
        residual = np.ascontiguousarray(residual, dtype=a.dtype)
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
    lib().or_palette_gemm(prec, acc_mode, rows, inner, columns, _p(a),
                          _p(np.ascontiguousarray(codes, dtype="<u4")), _p(palette), bits, groups,
                          columns // groups, _p(bias), _p(residual), float(residual_scale),
                          ACT[activation], _p(out))
    return out


def layernorm(x, gamma, beta, eps=1e-5):
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    lib().or_layernorm(_prec(x.dtype), x.shape[0], x.shape[1], _p(x),
                       _p(np.ascontiguousarray(gamma, np.float32)),
                       _p(np.ascontiguousarray(beta, np.float32)), float(eps), _p(out))
    return out


def rel_attention(qkv, positions, bias_u, bias_v, lengths, batch, frames):
    qkv = np.ascontiguousarray(qkv)
    out = np.empty((batch * frames, 1024), dtype=qkv.dtype)
    lib().or_rel_attention(_prec(qkv.dtype), batch, frames, _p(qkv),
                           _p(np.ascontiguousarray(positions, qkv.dtype)),
                           _p(np.ascontiguousarray(bias_u, np.float32)),
                           _p(np.ascontiguousarray(bias_v, np.float32)),
                           _p(np.ascontiguousarray(lengths, np.uint32)), _p(out))
    return out


def conformer_conv(pointwise, dw, scale, shift, lengths, batch, frames):
    pointwise = np.ascontiguousarray(pointwise)
    out = np.empty((batch * frames, 1024), dtype=pointwise.dtype)
    lib().or_conformer_conv(_prec(pointwise.dtype), batch, frames, _p(pointwise),
                            _p(np.ascontiguousarray(dw, pointwise.dtype)),
                            _p(np.ascontiguousarray(scale, np.float32)),
                            _p(np.ascontiguousarray(shift, np.float32)),
                            _p(np.ascontiguousarray(lengths, np.uint32)), _p(out))
    return out


def subsampling_conv0_dw2(fbank, conv0_w, conv0_b, dw_w, dw_b, feature_lengths, dtype):
    batch = fbank.shape[0]
    out = np.empty((batch, 376, 32, 256), dtype=dtype)
    lib().or_subsampling_conv0_dw2(_prec(dtype), batch,
                                   _p(np.ascontiguousarray(fbank, np.float32)),
                                   _p(np.ascontiguousarray(conv0_w, dtype)),
                                   _p(np.ascontiguousarray(conv0_b, np.float32)),
                                   _p(np.ascontiguousarray(dw_w, dtype)),
                                   _p(np.ascontiguousarray(dw_b, np.float32)),
                                   _p(np.ascontiguousarray(feature_lengths, np.uint32)), _p(out))
    return out


def subsampling_depthwise(x, w, b, feature_lengths, steps):
    x = np.ascontiguousarray(x)
    batch, ih, iw, ch = x.shape
    oh, ow = (ih - 1) // 2 + 1, (iw - 1) // 2 + 1
    out = np.empty((batch, oh, ow, ch), dtype=x.dtype)
    lib().or_subsampling_depthwise(_prec(x.dtype), batch, ih, iw, ch, _p(x),
                                   _p(np.ascontiguousarray(w, x.dtype)),
                                   _p(np.ascontiguousarray(b, np.float32)),
                                   _p(np.ascontiguousarray(feature_lengths, np.uint32)), steps, _p(out))
    return out


def subsampling_time_mask(x, feature_lengths, steps):
    x = np.ascontiguousarray(x).copy()
    batch, h, w, ch = x.shape
    lib().or_subsampling_time_mask(_prec(x.dtype), batch, h, w, ch, _p(x),
                                   _p(np.ascontiguousarray(feature_lengths, np.uint32)), steps)
    return x


def sub_len(raw: int, steps: int) -> int:
    for _ in range(steps):
        raw = (raw + 1) // 2
    return raw


# -- composition ------------------------------------------------------------

def _matrix(weights, name):
    t = weights[name]
    return t["data"], weights[name + ".palette"]["data"], t["bits"]


def gemm_named(weights, name, a, columns, acc_mode, **kw):
    codes, palette, bits = _matrix(weights, name)
    return palette_gemm(a, codes, palette, bits, columns, acc_mode=acc_mode, **kw)


def conformer_layer(weights, layer, x, encoder_lengths, batch, frames, acc_mode=0):
    """One Macaron Conformer layer, restating encoder.ts:1869-2138 dispatch by dispatch."""
    p = f"encoder.layers.{layer}"
    d = lambda n: weights[f"{p}.{n}"]["data"]  # noqa: E731
    a = layernorm(x, d("norm_feed_forward1.weight"), d("norm_feed_forward1.bias"))
    h = gemm_named(weights, f"{p}.feed_forward1.linear1.weight", a, 4096, acc_mode, activation="silu")
    x1 = gemm_named(weights, f"{p}.feed_forward1.linear2.weight", h, 1024, acc_mode,
                    residual=x, residual_scale=0.5)
    a = layernorm(x1, d("norm_self_att.weight"), d("norm_self_att.bias"))
    qkv = gemm_named(weights, f"{p}.self_attn.qkv.weight", a, 3072, acc_mode)
    ctx = rel_attention(qkv, d("self_attn.projected_positions"), d("self_attn.bias_u"),
                        d("self_attn.bias_v"), encoder_lengths, batch, frames)
    x2 = gemm_named(weights, f"{p}.self_attn.o_proj.weight", ctx, 1024, acc_mode, residual=x1)
    a = layernorm(x2, d("norm_conv.weight"), d("norm_conv.bias"))
    g = gemm_named(weights, f"{p}.conv.pointwise_conv1.weight", a, 2048, acc_mode)
    c = conformer_conv(g, d("conv.depthwise_conv.weight"), d("conv.norm.scale"),
                       d("conv.norm.shift"), encoder_lengths, batch, frames)
    x3 = gemm_named(weights, f"{p}.conv.pointwise_conv2.weight", c, 1024, acc_mode, residual=x2)
    a = layernorm(x3, d("norm_feed_forward2.weight"), d("norm_feed_forward2.bias"))
    h = gemm_named(weights, f"{p}.feed_forward2.linear1.weight", a, 4096, acc_mode, activation="silu")
    x4 = gemm_named(weights, f"{p}.feed_forward2.linear2.weight", h, 1024, acc_mode,
                    residual=x3, residual_scale=0.5)
    return layernorm(x4, d("norm_out.weight"), d("norm_out.bias"))


def subsampling(weights, fbank, feature_lengths, dtype, acc_mode=0):
    """Subsampling front end, restating encoder.ts:2140-2430 (microbatching does
    not change the arithmetic; each window is independent)."""
    w = lambda n: weights[n]["data"]  # noqa: E731
    batch = fbank.shape[0]
    s376 = subsampling_conv0_dw2(fbank, w("encoder.subsampling.layers.0.weight"),
                                 w("encoder.subsampling.layers.0.bias"),
                                 w("encoder.subsampling.layers.2.weight"),
                                 w("encoder.subsampling.layers.2.bias"), feature_lengths, dtype)
    p376 = gemm_named(weights, "encoder.subsampling.layers.3.weight", s376.reshape(-1, 256), 256,
                      acc_mode, bias=w("encoder.subsampling.layers.3.bias"), activation="relu")
    s188 = subsampling_depthwise(p376.reshape(batch, 376, 32, 256),
                                 w("encoder.subsampling.layers.5.weight"),
                                 w("encoder.subsampling.layers.5.bias"), feature_lengths, 3)
    p188 = gemm_named(weights, "encoder.subsampling.layers.6.weight", s188.reshape(-1, 256), 256,
                      acc_mode, bias=w("encoder.subsampling.layers.6.bias"), activation="relu")
    p188 = subsampling_time_mask(p188.reshape(batch, 188, 16, 256), feature_lengths, 3)
    return gemm_named(weights, "encoder.subsampling.linear.weight", p188.reshape(batch * 188, 4096),
                      1024, acc_mode, bias=w("encoder.subsampling.linear.bias"))


def encoder(weights, fbank, feature_lengths, dtype, layers=24, acc_mode=0, return_layers=False):
    """Full encoder: subsampling, `layers` Conformer layers, projector (1024->640 + bias)."""
    batch = fbank.shape[0]
    lengths = np.array([sub_len(int(v), 3) for v in feature_lengths], dtype=np.uint32)
    x = subsampling(weights, fbank, feature_lengths, dtype, acc_mode)
    checkpoints = [x]
    for layer in range(layers):
        x = conformer_layer(weights, layer, x, lengths, batch, 188, acc_mode)
        checkpoints.append(x)
    proj = gemm_named(weights, "encoder_projector.weight", x, 640, acc_mode,
                      bias=weights["encoder_projector.bias"]["data"])
    if return_layers:
        return proj, lengths, checkpoints
    return proj, lengths


def rel_frobenius(actual: np.ndarray, expected: np.ndarray) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    denom = np.linalg.norm(e)
    return float(np.linalg.norm(a - e) / (denom if denom > 0 else 1.0))


DECODER_ORDER = ("decoder.embedding.weight", "decoder.lstm.weight_l0", "decoder.lstm.bias_l0",
                 "decoder.lstm.weight_l1", "decoder.lstm.bias_l1", "decoder.decoder_projector.weight",
                 "decoder.decoder_projector.bias", "joint.head.weight", "joint.head.bias")


def tdt_decode(enc, lengths, decoder, *, max_tokens=376, starts=None, ends=None, flush=None):
    """Greedy TDT decoding of ``enc`` [batch, frames, 640] (f16 -> FP16 package,
    f32 -> FP32) with the decoder tensors ``decoder`` (name -> array), restating
    src/webgpu/kernels/tdt-decoder.ts.  Returns (tokens, frames, durations,
    counts, status) with the first three u32 [batch, max_tokens]."""
    enc = np.ascontiguousarray(enc)
    prec = FP16 if enc.dtype == np.float16 else FP32
    batch, frames = enc.shape[0], enc.shape[1]
    u32 = lambda a, d: np.ascontiguousarray(np.full(batch, d, np.uint32) if a is None else np.asarray(a, np.uint32))
    lengths = u32(lengths, frames)
    starts, ends, flush = u32(starts, 0), u32(ends, frames), u32(flush, 0)
    ws = [np.ascontiguousarray(decoder[n]) for n in DECODER_ORDER]
    tokens = np.zeros((batch, max_tokens), np.uint32)
    tframes = np.zeros_like(tokens)
    durs = np.zeros_like(tokens)
    meta = np.zeros(2 * batch, np.uint32)
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    lib().or_tdt_decode(prec, batch, frames, max_tokens, ptr(enc), ptr(lengths), ptr(starts), ptr(ends),
                        ptr(flush), *[ptr(w) for w in ws], ptr(tokens), ptr(tframes), ptr(durs), ptr(meta))
    return tokens, tframes, durs, meta[:batch].copy(), meta[batch:].copy()


def logmel(samples, valid):
    """Log-mel features f32 [batch, 128, sample_count // 160 + 1] of PCM
    ``samples`` f32 [batch, sample_count] with ``valid`` samples per window
    (restating src/cpp/fbank/parakeet_fbank.cpp)."""
    samples = np.ascontiguousarray(samples, np.float32)
    b, n = samples.shape
    valid = np.ascontiguousarray(valid, np.uint32)
    out = np.zeros((b, 128, n // 160 + 1), np.float32)
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    lib().or_logmel(b, n, ptr(samples), ptr(valid), ptr(out))
    return out


_REF_FBANK = _HERE / "_ref" / "libparakeet_fbank.so"


def reference_fbank_available() -> bool:
    return _REF_FBANK.exists()


def reference_fbank(samples, valid):
    """The reference's own front end (oracle/_ref, built by ``make -C oracle ref``
    from src/cpp/fbank/parakeet_fbank.cpp): one parakeet_fbank_compute_item per
    window, no raw-frame reuse.  Same shapes as ``logmel``."""
    samples = np.ascontiguousarray(samples, np.float32)
    b, n = samples.shape
    L = ctypes.CDLL(str(_REF_FBANK))
    L.parakeet_fbank_input_ptr.restype = ctypes.c_void_p
    L.parakeet_fbank_output_ptr.restype = ctypes.c_void_p
    assert L.parakeet_fbank_init() == 1
    frames = n // 160 + 1
    out = np.zeros((b, 128, frames), np.float32)
    inp = (ctypes.c_float * 240000).from_address(L.parakeet_fbank_input_ptr())
    outp = (ctypes.c_float * (128 * 1501)).from_address(L.parakeet_fbank_output_ptr())
    for i in range(b):
        L.parakeet_fbank_reset_reuse()
        if L.parakeet_fbank_begin_batch(1, n) != frames:
            raise ValueError("reference rejected the window shape")
        ctypes.memmove(inp, samples[i].ctypes.data, n * 4)
        if L.parakeet_fbank_compute_item(0, int(valid[i]), 0) != frames:
            raise ValueError("reference rejected the window")
        out[i] = np.frombuffer(outp, np.float32, count=128 * frames).reshape(128, frames)
        L.parakeet_fbank_finish_batch()
    return out


def logmel_tables():
    """(hann [512], twiddle re [256], im [256], first [128], count [128], packed weights)."""
    h = np.zeros(512, np.float32)
    tr = np.zeros(256, np.float32)
    ti = np.zeros(256, np.float32)
    first = np.zeros(128, np.int32)
    count = np.zeros(128, np.int32)
    packed = np.zeros(2048, np.float32)
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    n = lib().or_logmel_tables(ptr(h), ptr(tr), ptr(ti), ptr(first), ptr(count), ptr(packed), 2048)
    return h, tr, ti, first, count, packed[:n].copy()
