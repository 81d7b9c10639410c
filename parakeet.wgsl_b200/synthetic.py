"""Seeded random-init weight packages in the reference's tensor inventory.

The benchmark configurations use random-init palettes (no checkpoint is
available), so this module produces what ``model/convert.py`` would produce
for the 24-layer FastConformer encoder: the same tensor names
(``src/webgpu/encoder.ts:1869-2512``), dtypes, logical shapes and layout
strings, with

* palette matrices as uniformly random 5- or 6-bit codes (uniform codes packed
  LSB-first are exactly uniform random u32 words) and per-group LUTs drawn
  from N(0, 0.02) and sorted; ``qkv`` carries three palette groups, one per
  Q/K/V block (encoder.ts:2494-2495); ``o_proj`` is 6-bit under the reference's
  mixed policy (encoder.ts:2465);
* LayerNorm gamma 1 + N(0, 0.02), beta N(0, 0.02); attention biases u, v
  N(0, 0.02); depthwise k9 weights N(0, 0.1); folded BN scale 1 + N(0, 0.02),
  shift N(0, 0.02);
* projected relative positions = the sinusoidal table projected in f32 by a
  random 6-bit palette weight and packed head-vector-position-vec4
  (convert.py:1143-1228);
* subsampling conv weights N(0, 0.1) (conv0 N(0, 0.3)), biases N(0, 0.02).

Each record is a dict: ``data`` (numpy), ``dtype`` ("float16" | "float32" |
"uint32"), ``shape`` (logical), ``layout``; palette matrices also carry
``bits``.
"""
from __future__ import annotations

import numpy as np

from . import runtime_plan as rp

LAYERS = 24
HIDDEN = 1024


def _np_dtype(precision: str):
    return np.float16 if precision == "fp16" else np.float32


def _dtype_name(arr: np.ndarray) -> str:
    return {np.dtype(np.float16): "float16", np.dtype(np.float32): "float32",
            np.dtype("<u4"): "uint32"}[arr.dtype]


def _rec(data: np.ndarray, shape, layout: str, **extra) -> dict:
    d = {"data": np.ascontiguousarray(data), "dtype": _dtype_name(np.asarray(data)), "shape": tuple(shape),
         "layout": layout}
    d.update(extra)
    return d


def palette_matrix(rng: np.random.Generator, inner: int, columns: int, bits: int, groups: int, precision: str,
                   lut_std: float = 0.02) -> tuple[dict, dict]:
    """(packed-code record, palette record) for a random [K, N] palette matrix."""
    per, words = rp.code_group(bits)
    packed = rng.integers(0, 1 << 32, size=(inner * columns // per, words), dtype=np.uint64).astype("<u4")
    lut = np.sort(rng.normal(0.0, lut_std, size=(groups, 1 << bits)), axis=1).astype(_np_dtype(precision))
    return (_rec(packed, (inner, columns), rp.palette_layout(bits), bits=bits),
            _rec(lut, (groups, 1 << bits), rp.PALETTE_LUT_LAYOUT))


def matrix_bits(name: str, policy: str) -> int:
    if policy == "all5":
        return 5
    if policy == "all6":
        return 6
    return 6 if name.endswith(".self_attn.o_proj.weight") else 5  # reference's mixed policy


def make_package(precision: str = "fp16", layers: int = LAYERS, bits_policy: str = "mixed", seed: int = 0) -> dict:
    """Random-init encoder package (subsampling, `layers` Conformer layers, projector)."""
    if precision not in ("fp16", "fp32"):
        raise ValueError("precision must be fp16 or fp32")
    rng = np.random.default_rng(seed)
    dt = _np_dtype(precision)
    pkg: dict[str, dict] = {}

    def add_matrix(name, inner, columns, groups=1):
        codes, lut = palette_matrix(rng, inner, columns, matrix_bits(name, bits_policy), groups, precision)
        pkg[name] = codes
        pkg[name + ".palette"] = lut

    def f32(shape, mean=0.0, std=0.02):
        return (mean + rng.normal(0.0, std, size=shape)).astype(np.float32)

    # Subsampling (encoder.ts:2162-2245).
    pkg["encoder.subsampling.layers.0.weight"] = _rec(rng.normal(0, 0.3, (3, 3, 256)).astype(dt), (3, 3, 256),
                                                      "kh-kw-output-channel-vec4")
    pkg["encoder.subsampling.layers.0.bias"] = _rec(f32(256), (256,), "output-channel")
    pkg["encoder.subsampling.layers.2.weight"] = _rec(rng.normal(0, 0.1, (3, 3, 256)).astype(dt), (3, 3, 256),
                                                      "kh-kw-channel-vec4")
    pkg["encoder.subsampling.layers.2.bias"] = _rec(f32(256), (256,), "output-channel")
    add_matrix("encoder.subsampling.layers.3.weight", 256, 256)
    pkg["encoder.subsampling.layers.3.bias"] = _rec(f32(256), (256,), "output-channel")
    pkg["encoder.subsampling.layers.5.weight"] = _rec(rng.normal(0, 0.1, (3, 3, 256)).astype(dt), (3, 3, 256),
                                                      "kh-kw-channel-vec4")
    pkg["encoder.subsampling.layers.5.bias"] = _rec(f32(256), (256,), "output-channel")
    add_matrix("encoder.subsampling.layers.6.weight", 256, 256)
    pkg["encoder.subsampling.layers.6.bias"] = _rec(f32(256), (256,), "output-channel")
    add_matrix("encoder.subsampling.linear.weight", 4096, HIDDEN)
    pkg["encoder.subsampling.linear.bias"] = _rec(f32(HIDDEN), (HIDDEN,), "output-channel")

    table = rp.build_relative_positions()
    for layer in range(layers):
        p = f"encoder.layers.{layer}."
        for norm in ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"):
            pkg[p + norm + ".weight"] = _rec(f32(HIDDEN, 1.0), (HIDDEN,), "channel")
            pkg[p + norm + ".bias"] = _rec(f32(HIDDEN), (HIDDEN,), "channel")
        add_matrix(p + "feed_forward1.linear1.weight", HIDDEN, 4096)
        add_matrix(p + "feed_forward1.linear2.weight", 4096, HIDDEN)
        add_matrix(p + "self_attn.qkv.weight", HIDDEN, 3 * HIDDEN, groups=3)
        add_matrix(p + "self_attn.o_proj.weight", HIDDEN, HIDDEN)
        add_matrix(p + "conv.pointwise_conv1.weight", HIDDEN, 2 * HIDDEN)
        add_matrix(p + "conv.pointwise_conv2.weight", HIDDEN, HIDDEN)
        add_matrix(p + "feed_forward2.linear1.weight", HIDDEN, 4096)
        add_matrix(p + "feed_forward2.linear2.weight", 4096, HIDDEN)
        # Positional projection: random 6-bit palette weight, projected in f32.
        pos_codes, pos_lut = palette_matrix(rng, HIDDEN, HIDDEN, 6, 1, "fp32")
        w_in_out = rp.expand(pos_codes["data"], pos_lut["data"], 6, HIDDEN, HIDDEN)  # runtime [in, out]
        projected = rp.project_relative_positions(table, w_in_out.T, dtype=dt)
        pkg[p + "self_attn.projected_positions"] = _rec(rp.pack_projected_relative_positions(projected),
                                                        (375, HIDDEN), "head-vector-position-vec4")
        pkg[p + "self_attn.bias_u"] = _rec(f32((8, 128)), (8, 128), "head-by-channel")
        pkg[p + "self_attn.bias_v"] = _rec(f32((8, 128)), (8, 128), "head-by-channel")
        pkg[p + "conv.depthwise_conv.weight"] = _rec(rng.normal(0, 0.1, (9, HIDDEN)).astype(dt), (9, HIDDEN),
                                                     "kernel-channel-vec4")
        pkg[p + "conv.norm.scale"] = _rec(f32(HIDDEN, 1.0), (HIDDEN,), "channel")
        pkg[p + "conv.norm.shift"] = _rec(f32(HIDDEN), (HIDDEN,), "channel")

    add_matrix("encoder_projector.weight", HIDDEN, 640)
    pkg["encoder_projector.bias"] = _rec(f32(640), (640,), "output-channel")
    return pkg


def make_features(batch: int, seed: int = 0, mean: float = -4.0, std: float = 2.0) -> np.ndarray:
    """Log-mel features f32 [batch, 128, 1501] feature-major, i.i.d. N(mean, std^2)."""
    rng = np.random.default_rng(seed)
    return rng.normal(mean, std, size=(batch, 128, 1501)).astype(np.float32)


# Decoder tensors read by the persistent TDT decoder (src/webgpu/kernels/tdt-decoder.ts:367-420;
# packed by model/convert.py:1608-1703): name -> (logical shape, layout, weight dtype?).
DECODER_HIDDEN = 640
DECODER_TOKENS = 1025          # 1024 vocabulary tokens + blank (id 1024)
DECODER_HEAD_OUTPUTS = 1032    # 1025 tokens + 5 durations, padded to a multiple of 4
DECODER_TENSORS = {
    "decoder.embedding.weight": ((1025, 640), "token-by-channel-row-major", True),
    "decoder.lstm.weight_l0": ((1280, 2560), "input-hidden-k-by-ifgo-row-major-vec4", True),
    "decoder.lstm.bias_l0": ((2560,), "ifgo-gates", False),
    "decoder.lstm.weight_l1": ((1280, 2560), "input-hidden-k-by-ifgo-row-major-vec4", True),
    "decoder.lstm.bias_l1": ((2560,), "ifgo-gates", False),
    "decoder.decoder_projector.weight": ((640, 640), "k-by-output-row-major-vec4", True),
    "decoder.decoder_projector.bias": ((640,), "output-channel", False),
    "joint.head.weight": ((640, 1032), "k-by-output-row-major-vec4", True),
    "joint.head.bias": ((1032,), "output-channel-padded-vec4", False),
}


def make_decoder(precision: str = "fp16", seed: int = 0, blank_bias: float = 1.5) -> dict:
    """Random-init TDT decoder tensors (prediction net + joint head).

    LSTM weights U(+-1/sqrt(640)) (PyTorch's LSTM default), embedding N(0, 1),
    projector U(+-1/sqrt(640)), head N(0, 0.1); the blank logit's bias is raised
    by ``blank_bias`` so greedy decoding emits a realistic mix of blanks and
    tokens.  The two padding outputs of the head are zero."""
    rng = np.random.default_rng(seed)
    dt = _np_dtype(precision)
    a = 1.0 / np.sqrt(DECODER_HIDDEN)
    head = rng.normal(0.0, 0.1, size=(640, 1032)).astype(np.float32)
    head[:, 1030:] = 0.0
    head_bias = rng.normal(0.0, 0.1, size=1032).astype(np.float32)
    head_bias[1024] += blank_bias
    head_bias[1030:] = 0.0
    data = {
        "decoder.embedding.weight": rng.normal(0.0, 1.0, size=(1025, 640)).astype(dt),
        "decoder.lstm.weight_l0": rng.uniform(-a, a, size=(1280, 2560)).astype(dt),
        "decoder.lstm.bias_l0": rng.uniform(-2 * a, 2 * a, size=2560).astype(np.float32),
        "decoder.lstm.weight_l1": rng.uniform(-a, a, size=(1280, 2560)).astype(dt),
        "decoder.lstm.bias_l1": rng.uniform(-2 * a, 2 * a, size=2560).astype(np.float32),
        "decoder.decoder_projector.weight": rng.uniform(-a, a, size=(640, 640)).astype(dt),
        "decoder.decoder_projector.bias": rng.uniform(-a, a, size=640).astype(np.float32),
        "joint.head.weight": head.astype(dt),
        "joint.head.bias": head_bias,
    }
    return {name: _rec(data[name], shape, layout) for name, (shape, layout, _) in DECODER_TENSORS.items()}


def make_pcm(seconds: float, seed: int = 0, sample_rate: int = 16_000) -> np.ndarray:
    """Seeded synthetic speech-band audio as 16 kHz f32 PCM with PCM16
    quantization: pink (1/f) noise plus six amplitude-modulated tones between
    100 and 4000 Hz (the benchmark's stand-in for real recordings)."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * sample_rate))
    spec = np.fft.rfft(rng.standard_normal(n))
    f = np.fft.rfftfreq(n, 1.0 / sample_rate)
    spec[1:] /= np.sqrt(f[1:])
    spec[0] = 0.0
    pink = np.fft.irfft(spec, n)
    pink /= max(np.abs(pink).max(), 1e-12)
    t = np.arange(n) / sample_rate
    tones = np.zeros(n)
    for freq in rng.uniform(100.0, 4000.0, size=6):
        am = 0.5 * (1.0 + np.sin(2 * np.pi * rng.uniform(0.5, 4.0) * t + rng.uniform(0, 2 * np.pi)))
        tones += am * np.sin(2 * np.pi * freq * t + rng.uniform(0, 2 * np.pi))
    tones /= 6.0
    x = 0.3 * pink + 0.4 * tones
    pcm16 = np.clip(np.round(x * 32767.0), -32768, 32767).astype(np.int16)
    return pcm16.astype(np.float32) / 32768.0
