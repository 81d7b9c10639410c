"""Operator API of the encoder hot path, mirroring the reference's kernel layer.

The reference's operators follow one pattern (src/webgpu/kernels/*.ts):
``XKernel.create(device, arena, ..., profile)`` -> ``kernel.createDispatch(
descriptor)`` (synchronous validation, throws ``Error``/``RangeError``) ->
``dispatch.encode(encoder, timestampWrites?, shape?)`` -> ``destroy()``.
This module keeps that shape in Python over libpk_b200.so:

* ``create`` / ``create_dispatch`` validate exactly what the reference
  validates (shape, layout, fixed production signature) and raise
  ``RangeError`` (a ``ValueError``) or ``ParakeetError`` (a ``RuntimeError``);
* ``encode(stream=None, shape=None)`` launches on a CUDA stream (default: the
  current torch stream) instead of recording into a GPUCommandEncoder;
  ``shape={"rows": n}`` / ``{"batch_size": b}`` selects the active prefix as
  ``EncoderDispatchShape`` does (src/webgpu/kernels/execution-shape.ts:1-4);
* buffers are torch CUDA tensors (the "arena slices"); weights are
  ``GpuTensor`` records (src/model/package.ts:45).

Every launch goes through the C ABI; there is no CPU or framework fallback.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from . import _lib
from . import runtime_plan as rp

try:  # torch is the device-memory / stream plumbing
    import torch
except ImportError:  # pragma: no cover - the package requires torch at run time
    torch = None


class RangeError(ValueError):
    """The reference's RangeError: an argument outside its supported range."""


class ParakeetError(RuntimeError):
    """The reference's Error: invalid layout, signature or state."""


# F16_SUBGROUP_PRODUCTION_SPECIALIZATIONS (src/webgpu/kernels/gemm.ts:204-356)
# and the FP32 twin (:2154-2306): (label, rows, inner, columns, activation,
# has_bias, residual_scale, tile_major).
PRODUCTION_SPECIALIZATIONS = (
    ("encoder-layer-ff-expand", 7520, 1024, 4096, "silu", False, None, True),
    ("encoder-layer-ff-contract", 7520, 4096, 1024, "none", False, 0.5, True),
    ("encoder-layer-attention-qkv", 7520, 1024, 3072, "none", False, None, True),
    ("encoder-layer-residual-1024", 7520, 1024, 1024, "none", False, 1.0, True),
    ("encoder-layer-convolution-expand", 7520, 1024, 2048, "none", False, None, True),
    ("encoder-projector", 7520, 1024, 640, "none", True, None, False),
    ("subsampling-pointwise3", 12032, 256, 256, "relu", True, None, False),
    ("subsampling-pointwise3-b2", 24064, 256, 256, "relu", True, None, False),
    ("subsampling-pointwise3-b3", 36096, 256, 256, "relu", True, None, False),
    ("subsampling-pointwise6", 3008, 256, 256, "relu", True, None, False),
    ("subsampling-pointwise6-b2", 6016, 256, 256, "relu", True, None, False),
    ("subsampling-pointwise6-b3", 9024, 256, 256, "relu", True, None, False),
    ("subsampling-flatten-project", 188, 4096, 1024, "none", True, None, False),
    ("subsampling-flatten-project-b2", 376, 4096, 1024, "none", True, None, False),
    ("subsampling-flatten-project-b3", 564, 4096, 1024, "none", True, None, False),
)


def _stream_handle(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    if hasattr(stream, "cuda_stream"):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


def _ptr(t) -> ctypes.c_void_p | None:
    if t is None:
        return None
    if isinstance(t, GpuTensor):
        t = t.tensor
    if not t.is_cuda or not t.is_contiguous():
        raise ParakeetError("operands must be contiguous CUDA tensors")
    return ctypes.c_void_p(t.data_ptr())


def _precision(profile: str) -> int:
    if profile not in ("fp16", "fp32"):
        raise ParakeetError(f"unknown execution profile precision {profile!r}")
    return _lib.FP16 if profile == "fp16" else _lib.FP32


def _scalar_dtype(profile: str):
    return torch.float16 if profile == "fp16" else torch.float32


@dataclass
class GpuTensor:
    """A resident package tensor: runtime record + device buffer."""
    name: str
    dtype: str                 # "float16" | "float32" | "uint32"
    shape: tuple               # logical shape
    layout: str
    tensor: Any = field(repr=False)

    @staticmethod
    def from_record(name: str, record: dict, device: str = "cuda") -> "GpuTensor":
        data = np.ascontiguousarray(record["data"])
        if data.dtype == np.dtype("<u4"):
            t = torch.from_numpy(data.view(np.int32)).to(device)
        else:
            t = torch.from_numpy(data).to(device)
        return GpuTensor(name, record["dtype"], tuple(record["shape"]), record["layout"], t.contiguous())


class Device:
    """A pk_device handle (pk_device_open / pk_device_close)."""

    def __init__(self, ordinal: int = 0):
        handle = ctypes.c_void_p()
        _lib.call("pk_device_open", ordinal, ctypes.byref(handle))
        self.handle = handle
        self.ordinal = ordinal

    def status(self) -> int:
        bits = ctypes.c_uint32(0)
        _lib.call("pk_device_status", self.handle, ctypes.byref(bits))
        return bits.value

    def close(self) -> None:
        if self.handle:
            _lib.load().pk_device_close(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


class _Dispatch:
    def __init__(self, label: str):
        self.label = label
        self._destroyed = False

    def _alive(self):
        if self._destroyed:
            raise ParakeetError(f"{self.label} was destroyed")

    def destroy(self) -> None:
        self._destroyed = True  # idempotent, like the reference


# --------------------------------------------------------------------- palette expansion

class PaletteWeightExpander:
    """PaletteWeightExpander (src/model/palette-expander.ts:160-310): bit-exact expansion."""

    def __init__(self, device: Device, profile: str):
        self.device = device
        self.profile = profile

    @staticmethod
    def create(device: Device, profile: str = "fp16") -> "PaletteWeightExpander":
        _precision(profile)
        return PaletteWeightExpander(device, profile)

    def create_pooled_dispatch(self, descriptor: dict) -> _Dispatch:
        """descriptor: label, source (u32 tensor), palette, target, scalar_count, columns,
        palette_bits, palette_group_columns, palette_groups, runtime_layout."""
        d = descriptor
        bits = d["palette_bits"]
        per, words = rp.code_group(bits)
        esize = 2 if self.profile == "fp16" else 4
        count, columns = d["scalar_count"], d["columns"]
        if (count <= 0 or count % per or columns <= 0 or count % columns or d["palette_group_columns"] <= 0
                or columns % d["palette_group_columns"]
                or d["palette_group_columns"] * d["palette_groups"] != columns
                or d["source"].numel() * 4 != count // per * words * 4
                or d["palette"].numel() * esize != d["palette_groups"] * (1 << bits) * esize
                or d["target"].numel() != count):
            raise ParakeetError(f"{d['label']} has invalid transient palette geometry")
        layout = d["runtime_layout"]
        f16_layouts = (rp.ROW_MAJOR_F16_LAYOUT, rp.TILE_MAJOR_F16_LAYOUT)
        f32_layouts = (rp.ROW_MAJOR_F32_LAYOUT, rp.TILE_MAJOR_F32_LAYOUT)
        if layout not in (f16_layouts if self.profile == "fp16" else f32_layouts):
            raise ParakeetError(f"{d['label']} has a mismatched palette execution layout")
        tile = layout in (rp.TILE_MAJOR_F16_LAYOUT, rp.TILE_MAJOR_F32_LAYOUT)
        desc = _lib.PaletteDesc(_precision(self.profile), bits, count // columns, columns, d["palette_groups"],
                                d["palette_group_columns"],
                                _lib.LAYOUT_TILE_MAJOR if tile else _lib.LAYOUT_ROW_MAJOR,
                                _ptr(d["source"]), _ptr(d["palette"]), _ptr(d["target"]))
        device = self.device
        disp = _Dispatch(d["label"])

        def encode(stream=None):
            disp._alive()
            _lib.call("pk_palette_expand", device.handle, ctypes.byref(desc), _stream_handle(stream))

        disp.encode = encode
        return disp


# --------------------------------------------------------------------- GEMM

@dataclass
class GemmDescriptor:
    """GemmDescriptor (src/webgpu/kernels/gemm.ts:358-373)."""
    label: str
    a: Any
    b: GpuTensor
    output: Any
    rows: int
    inner: int
    columns: int
    b_palette: GpuTensor | None = None
    palette_group_columns: int | None = None
    bias: GpuTensor | None = None
    residual: Any = None
    residual_scale: float | None = None
    activation: str = "none"


class GemmDispatch(_Dispatch):
    def __init__(self, kernel: "F16GemmKernel", d: GemmDescriptor, bits: int, groups: int):
        super().__init__(d.label)
        self.kernel, self.d, self.bits, self.groups = kernel, d, bits, groups
        self.output = d.output

    def encode(self, stream=None, timestamp_writes=None, shape: dict | None = None) -> None:
        self._alive()
        d = self.d
        rows = d.rows
        if shape is not None:
            rows = shape.get("rows", rows)
            if not isinstance(rows, int) or rows <= 0 or rows > d.rows:
                raise RangeError(f"{d.label} active rows must be in [1, {d.rows}]")
        desc = _lib.GemmDesc(
            _precision(self.kernel.profile), rows, d.inner, d.columns, self.bits, self.groups,
            d.columns // self.groups, _lib.ACT[d.activation], int(d.residual is not None),
            float(1.0 if d.residual_scale is None else d.residual_scale), _ptr(d.bias), _ptr(d.residual),
            _ptr(d.a), _ptr(d.b), _ptr(d.b_palette), _ptr(d.output))
        _lib.call("pk_palette_gemm", self.kernel.device.handle, ctypes.byref(desc), _stream_handle(stream))


class F16GemmKernel:
    """Fixed-shape palette GEMM owner (gemm.ts:483-855; FP32 twin :2974-3340).

    Unlike the reference, no expanded-weight scratch exists: the CUDA kernels
    decode the packed codes on chip."""

    PROFILE = "fp16"

    def __init__(self, device: Device, profile: str):
        self.device = device
        self.profile = profile
        self._destroyed = False

    @classmethod
    def create(cls, device: Device, arena=None, profile: str | None = None):
        profile = profile or cls.PROFILE
        if profile != cls.PROFILE:
            raise ParakeetError(f"Parakeet {cls.PROFILE.upper()} GEMM requires an {cls.PROFILE.upper()} "
                                "execution profile")
        return cls(device, profile)

    def create_dispatch(self, d: GemmDescriptor) -> GemmDispatch:
        if self._destroyed:
            raise ParakeetError("Parakeet GEMM kernel was destroyed")
        # requireGemmShape (gemm.ts:1069-1119)
        if (not isinstance(d.rows, int) or d.rows <= 0 or not isinstance(d.inner, int) or d.inner <= 0
                or d.inner % 32 or not isinstance(d.columns, int) or d.columns <= 0 or d.columns % 8):
            raise RangeError(f"Unsupported GEMM shape for {d.label}")
        if tuple(d.b.shape) != (d.inner, d.columns):
            raise ParakeetError(f"{d.label} weight package does not match K={d.inner}, N={d.columns}")
        bits = rp.palette_bits_for_layout(d.b.layout)
        if bits is None or d.b.dtype != "uint32":
            raise ParakeetError(f"{d.label} has an unsupported weight format")
        per, words = rp.code_group(bits)
        if (d.inner * d.columns) % per:
            raise ParakeetError(f"{d.label} palette codes are not group aligned")
        if d.b.tensor.numel() != d.inner * d.columns // per * words:
            raise ParakeetError(f"{d.label} has invalid packed palette indices")
        # requireProductionSpecialization (gemm.ts:1140-1180)
        if d.residual is None and d.residual_scale is not None:
            raise ParakeetError(f"{d.label} supplies a residual scale without a residual")
        signature = (d.rows, d.inner, d.columns, d.activation, d.bias is not None,
                     None if d.residual is None else (1.0 if d.residual_scale is None else d.residual_scale))
        if not any(s[1:7] == signature for s in PRODUCTION_SPECIALIZATIONS):
            raise ParakeetError(
                f"{d.label} is not a fixed production GEMM signature: M={d.rows}, K={d.inner}, N={d.columns}, "
                f"activation={d.activation}, bias={d.bias is not None}, residualScale={signature[5] or 'none'}")
        # requireRuntimeWeight (gemm.ts:1182-1272)
        pal = d.b_palette
        scalar = "float16" if self.profile == "fp16" else "float32"
        if (pal is None or pal.dtype != scalar or pal.layout != rp.PALETTE_LUT_LAYOUT or len(pal.shape) != 2
                or pal.shape[1] != 1 << bits or d.palette_group_columns is None
                or d.palette_group_columns <= 0 or d.palette_group_columns * pal.shape[0] != d.columns):
            raise ParakeetError(f"{d.label} has invalid transient palette weights")
        return GemmDispatch(self, d, bits, pal.shape[0])

    def destroy(self) -> None:
        self._destroyed = True


class F32GemmKernel(F16GemmKernel):
    PROFILE = "fp32"


# --------------------------------------------------------------------- LayerNorm

class LayerNormKernel:
    """LayerNormKernel (src/webgpu/kernels/layernorm.ts:73-240)."""

    def __init__(self, device: Device, profile: str):
        self.device, self.profile = device, profile

    @staticmethod
    def create(device: Device, arena=None, capacity: int = 0, profile: str = "fp16") -> "LayerNormKernel":
        _precision(profile)
        return LayerNormKernel(device, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d: label, input, output, gamma, beta, rows, channels, epsilon=1e-5."""
        rows, channels = d["rows"], d["channels"]
        if rows <= 0 or channels <= 0 or channels % 4:
            raise RangeError(f"Unsupported LayerNorm shape for {d['label']}")
        disp = _Dispatch(d["label"])
        disp.output = d["output"]
        kernel = self

        def encode(stream=None, timestamp_writes=None, shape=None):
            disp._alive()
            r = rows if shape is None else shape.get("rows", rows)
            if r <= 0 or r > rows:
                raise RangeError(f"{d['label']} active rows must be in [1, {rows}]")
            _lib.call("pk_layernorm", kernel.device.handle, _precision(kernel.profile), r, channels,
                      _ptr(d["input"]), _ptr(d["gamma"]), _ptr(d["beta"]), float(d.get("epsilon", 1e-5)),
                      _ptr(d["output"]), _stream_handle(stream))

        disp.encode = encode
        return disp


# --------------------------------------------------------------------- attention

class RelativeAttentionKernel:
    """RelativeAttentionKernel (src/webgpu/kernels/attention.ts:105-321)."""

    def __init__(self, device: Device, profile: str):
        self.device, self.profile = device, profile

    @staticmethod
    def create(device: Device, arena=None, capacity: int = 0, profile: str = "fp16"):
        _precision(profile)
        return RelativeAttentionKernel(device, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d: label, qkv, projected_positions, bias_u, bias_v, valid_lengths, output, batch_size, frames."""
        b, t = d["batch_size"], d["frames"]
        if b <= 0 or t <= 0 or t > 192:
            raise RangeError(f"Unsupported attention shape for {d['label']}")
        esize = 2 if self.profile == "fp16" else 4
        if d["qkv"].numel() * esize < b * t * 3072 * esize:
            raise RangeError(f"{d['label']} QKV needs {b * t * 3072 * esize} bytes")
        pos = d["projected_positions"]
        if (pos.layout != "head-vector-position-vec4" or tuple(pos.shape) != (2 * t - 1, 1024)):
            raise ParakeetError("Projected positions must be head-vector-position-vec4, "
                                f"logical [{2 * t - 1},1024]")
        for key in ("bias_u", "bias_v"):
            bias = d[key]
            if bias.dtype != "float32" or tuple(bias.shape) != (8, 128) or bias.layout != "head-by-channel":
                raise ParakeetError(f"{d['label']} {key} must be float32 head-by-channel logical/storage [8,128]")
        disp = _Dispatch(d["label"])
        disp.output = d["output"]
        kernel = self

        def encode(stream=None, timestamp_writes=None, shape=None):
            disp._alive()
            batch = b if shape is None else shape.get("batch_size", b)
            if batch <= 0 or batch > b:
                raise RangeError(f"{d['label']} active batch must be in [1, {b}]")
            _lib.call("pk_rel_attention", kernel.device.handle, _precision(kernel.profile), batch, t,
                      _ptr(d["qkv"]), _ptr(pos), _ptr(d["bias_u"]), _ptr(d["bias_v"]), _ptr(d["valid_lengths"]),
                      _ptr(d["output"]), _stream_handle(stream))

        disp.encode = encode
        return disp


# --------------------------------------------------------------------- log-mel front end

PARAKEET_FBANK_HOP_SAMPLES = 160
PARAKEET_FBANK_BINS = 128
PARAKEET_FBANK_MAX_SAMPLES = 240_000


def parakeet_feature_frame_count(sample_count: int) -> int:
    """parakeetFeatureFrameCount (src/audio/fbank-wasm.ts:133-139)."""
    if not isinstance(sample_count, int) or sample_count < 0:
        raise RangeError("sampleCount must be a non-negative safe integer")
    return sample_count // PARAKEET_FBANK_HOP_SAMPLES + 1


def parakeet_valid_feature_frame_count(sample_count: int) -> int:
    """parakeetValidFeatureFrameCount (src/audio/fbank-wasm.ts:141-147)."""
    if not isinstance(sample_count, int) or sample_count < 0:
        raise RangeError("sampleCount must be a non-negative safe integer")
    return sample_count // PARAKEET_FBANK_HOP_SAMPLES


class ParakeetFbank:
    """The log-mel front end (ParakeetFbankWasm, src/audio/fbank-wasm.ts:158)
    on the GPU: a whole batch of windows per call instead of one item at a time."""

    def __init__(self, device: Device):
        self.device = device

    def compute_batch(self, samples, valid_samples, out=None, stream=None):
        """samples: CUDA f32 [batch, sample_count]; valid_samples: CUDA int32/uint32
        [batch]; returns (or fills) CUDA f32 [batch, 128, sample_count // 160 + 1]."""
        if samples.dim() != 2 or samples.dtype != torch.float32:
            raise RangeError("samples must be f32 [batch, sample_count]")
        batch, count = samples.shape
        if count < PARAKEET_FBANK_HOP_SAMPLES or count > PARAKEET_FBANK_MAX_SAMPLES:
            raise RangeError("sampleCount must be in [160, 240000]")
        if valid_samples.numel() < batch:
            raise RangeError("validSampleCount needs one entry per window")
        frames = parakeet_feature_frame_count(count)
        if out is None:
            out = torch.empty((batch, PARAKEET_FBANK_BINS, frames), dtype=torch.float32, device=samples.device)
        _lib.call("pk_logmel", self.device.handle, batch, count, _ptr(samples), _ptr(valid_samples), _ptr(out),
                  _stream_handle(stream))
        return out


# --------------------------------------------------------------------- TDT decoder

# requireDecoderWeights (src/webgpu/kernels/tdt-decoder.ts:367-420): name ->
# (weight dtype follows the profile?, storage shape, layout).
TDT_DECODER_TENSORS = {
    "decoder.embedding.weight": (True, (1025, 640), "token-by-channel-row-major"),
    "decoder.lstm.weight_l0": (True, (1280, 2560), "input-hidden-k-by-ifgo-row-major-vec4"),
    "decoder.lstm.bias_l0": (False, (2560,), "ifgo-gates"),
    "decoder.lstm.weight_l1": (True, (1280, 2560), "input-hidden-k-by-ifgo-row-major-vec4"),
    "decoder.lstm.bias_l1": (False, (2560,), "ifgo-gates"),
    "decoder.decoder_projector.weight": (True, (640, 640), "k-by-output-row-major-vec4"),
    "decoder.decoder_projector.bias": (False, (640,), "output-channel"),
    "joint.head.weight": (True, (640, 1032), "k-by-output-row-major-vec4"),
    "joint.head.bias": (False, (1032,), "output-channel-padded-vec4"),
}
TDT_DECODER_OVERFLOW = 1


def plan_tdt_decoder_execution(batch_size: int) -> dict:
    """planTdtDecoderExecution (tdt-decoder.ts:39-52), restated for this engine:
    one 4-CTA cluster per window; the predictor state stays on chip."""
    if not isinstance(batch_size, int) or batch_size <= 0:
        raise RangeError("TDT decoder batchSize must be a positive integer")
    return {"clusters": batch_size, "ctas": 4 * batch_size, "predictor_scratch_bytes": 0}


class PersistentTdtDecoderKernel:
    """PersistentTdtDecoderKernel (src/webgpu/kernels/tdt-decoder.ts:155-330):
    greedy TDT decoding of whole windows in one persistent launch."""

    def __init__(self, device: Device, weights: dict, profile: str):
        self.device, self.weights, self.profile = device, weights, profile

    @staticmethod
    def create(device: Device, arena=None, model: dict | None = None,
               profile: str = "fp16") -> "PersistentTdtDecoderKernel":
        """model: name -> GpuTensor holding the decoder tensors of the package."""
        _precision(profile)
        if model is None:
            raise ParakeetError("TDT decoder requires the decoder tensors of a package")
        wdtype = "float16" if profile == "fp16" else "float32"
        resident = {}
        for name, (profiled, shape, layout) in TDT_DECODER_TENSORS.items():
            if name not in model:
                raise ParakeetError(f"Missing decoder tensor {name}")
            t = model[name]
            want = wdtype if profiled else "float32"
            if t.dtype != want or tuple(t.shape) != shape or t.layout != layout:
                raise ParakeetError(f"Unexpected decoder tensor {t.layout} [{','.join(map(str, t.shape))}]")
            resident[name] = t
        return PersistentTdtDecoderKernel(device, resident, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d (TdtDecoderDescriptor, tdt-decoder.ts:54-82): label, encoder_projected,
        encoded_lengths, decode_starts, decode_ends, flush_finals, tokens, token_frames,
        token_durations, metadata, batch_size, frames, max_tokens."""
        for key in ("batch_size", "frames", "max_tokens"):
            v = d[key]
            if not isinstance(v, int) or v <= 0:
                raise RangeError(f"Invalid TDT decoder {key}")
        b, t, m = d["batch_size"], d["frames"], d["max_tokens"]
        esize = 2 if self.profile == "fp16" else 4
        need = {"encoder_projected": b * t * 640 * esize, "encoded_lengths": b * 4, "decode_starts": b * 4,
                "decode_ends": b * 4, "flush_finals": b * 4, "tokens": b * m * 4, "token_frames": b * m * 4,
                "token_durations": b * m * 4, "metadata": b * 2 * 4}
        for key, nbytes in need.items():
            buf = d[key]
            if buf.numel() * buf.element_size() < nbytes:
                raise RangeError(f"{key} is too small for TDT decoding")
        disp = _Dispatch(d.get("label", "parakeet-persistent-tdt-decode"))
        kernel = self
        w = self.weights

        def encode(stream=None, timestamp_writes=None, active_batch_size: int | None = None):
            disp._alive()
            batch = b if active_batch_size is None else active_batch_size
            if not isinstance(batch, int) or batch <= 0 or batch > b:
                raise RangeError(f"{disp.label} active batch must be in [1, {b}]")
            desc = _lib.TdtDesc(_precision(kernel.profile), batch, t, m, *[_ptr(x) for x in (
                d["encoder_projected"], d["encoded_lengths"], d["decode_starts"], d["decode_ends"],
                d["flush_finals"], w["decoder.embedding.weight"], w["decoder.lstm.weight_l0"],
                w["decoder.lstm.bias_l0"], w["decoder.lstm.weight_l1"], w["decoder.lstm.bias_l1"],
                w["decoder.decoder_projector.weight"], w["decoder.decoder_projector.bias"],
                w["joint.head.weight"], w["joint.head.bias"], d["tokens"], d["token_frames"],
                d["token_durations"], d["metadata"])])
            _lib.call("pk_tdt_decode", kernel.device.handle, ctypes.byref(desc), _stream_handle(stream))

        disp.encode = encode
        return disp


# --------------------------------------------------------------------- conformer conv

class FusedConformerConvKernel:
    """FusedConformerConvKernel (src/webgpu/kernels/conformer-conv.ts:174-351)."""

    def __init__(self, device: Device, profile: str):
        self.device, self.profile = device, profile

    @staticmethod
    def create(device: Device, arena=None, capacity: int = 0, profile: str = "fp16"):
        _precision(profile)
        return FusedConformerConvKernel(device, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d: label, pointwise_input, depthwise_weights, batch_norm_scale, batch_norm_shift,
        valid_lengths, output, batch_size, frames."""
        b, t = d["batch_size"], d["frames"]
        if not isinstance(b, int) or b <= 0:
            raise RangeError("batchSize must be a positive integer")
        if not isinstance(t, int) or t <= 0:
            raise RangeError("frames must be a positive integer")
        dw = d["depthwise_weights"]
        if dw.layout != "kernel-channel-vec4" or tuple(dw.shape) != (9, 1024):
            raise ParakeetError(f"{d['label']} depthwise weights must be kernel-channel-vec4 [9,1024]")
        disp = _Dispatch(d["label"])
        disp.output = d["output"]
        kernel = self

        def encode(stream=None, timestamp_writes=None, shape=None):
            disp._alive()
            batch = b if shape is None else shape.get("batch_size", b)
            if batch <= 0 or batch > b:
                raise RangeError(f"{d['label']} active batch must be in [1, {b}]")
            _lib.call("pk_conformer_conv", kernel.device.handle, _precision(kernel.profile), batch, t,
                      _ptr(d["pointwise_input"]), _ptr(dw), _ptr(d["batch_norm_scale"]),
                      _ptr(d["batch_norm_shift"]), _ptr(d["valid_lengths"]), _ptr(d["output"]),
                      _stream_handle(stream))

        disp.encode = encode
        return disp


# --------------------------------------------------------------------- subsampling

class FusedSubsamplingConv0Depthwise2Kernel:
    """FusedSubsamplingConv0Depthwise2Kernel (src/webgpu/kernels/subsampling.ts:620-)."""

    def __init__(self, device: Device, profile: str):
        self.device, self.profile = device, profile

    @staticmethod
    def create(device: Device, arena=None, capacity: int = 0, profile: str = "fp16"):
        _precision(profile)
        return FusedSubsamplingConv0Depthwise2Kernel(device, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d: label, input (f32 [B,128,1501]), conv0_weights, conv0_bias, depthwise_weights,
        depthwise_bias, output ([B,376,32,256]), valid_lengths, batch_size."""
        b = d["batch_size"]
        if b <= 0:
            raise RangeError("batchSize must be a positive integer")
        disp = _Dispatch(d["label"])
        disp.output = d["output"]
        kernel = self

        def encode(stream=None):
            disp._alive()
            _lib.call("pk_subsampling_conv0_dw2", kernel.device.handle, _precision(kernel.profile), b,
                      _ptr(d["input"]), _ptr(d["conv0_weights"]), _ptr(d["conv0_bias"]),
                      _ptr(d["depthwise_weights"]), _ptr(d["depthwise_bias"]), _ptr(d["valid_lengths"]),
                      _ptr(d["output"]), _stream_handle(stream))

        disp.encode = encode
        return disp


class DepthwiseSubsamplingKernel:
    """DepthwiseSubsamplingKernel (src/webgpu/kernels/subsampling.ts:438-)."""

    def __init__(self, device: Device, profile: str):
        self.device, self.profile = device, profile

    @staticmethod
    def create(device: Device, arena=None, capacity: int = 0, profile: str = "fp16"):
        _precision(profile)
        return DepthwiseSubsamplingKernel(device, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d: label, input, weights, bias, output, valid_lengths, valid_length_subsampling_steps,
        batch_size, input_height, input_width, channels."""
        disp = _Dispatch(d["label"])
        disp.output = d["output"]
        kernel = self
        if min(d["batch_size"], d["input_height"], d["input_width"], d["channels"]) <= 0:
            raise RangeError("subsampling dimensions must be positive integers")

        def encode(stream=None):
            disp._alive()
            _lib.call("pk_subsampling_depthwise", kernel.device.handle, _precision(kernel.profile),
                      d["batch_size"], d["input_height"], d["input_width"], d["channels"], _ptr(d["input"]),
                      _ptr(d["weights"]), _ptr(d["bias"]), _ptr(d["valid_lengths"]),
                      d["valid_length_subsampling_steps"], _ptr(d["output"]), _stream_handle(stream))

        disp.encode = encode
        return disp


class SubsamplingTimeMaskKernel:
    """SubsamplingTimeMaskKernel (src/webgpu/kernels/subsampling.ts:250-)."""

    def __init__(self, device: Device, profile: str):
        self.device, self.profile = device, profile

    @staticmethod
    def create(device: Device, arena=None, capacity: int = 0, profile: str = "fp16"):
        _precision(profile)
        return SubsamplingTimeMaskKernel(device, profile)

    def create_dispatch(self, d: dict) -> _Dispatch:
        """d: label, values, valid_lengths, batch_size, height, width, channels, valid_length_subsampling_steps."""
        disp = _Dispatch(d["label"])
        kernel = self

        def encode(stream=None):
            disp._alive()
            _lib.call("pk_subsampling_time_mask", kernel.device.handle, _precision(kernel.profile),
                      d["batch_size"], d["height"], d["width"], d["channels"], _ptr(d["values"]),
                      _ptr(d["valid_lengths"]), d["valid_length_subsampling_steps"], _stream_handle(stream))

        disp.encode = encode
        return disp


def set_gemm_route(route: str) -> None:
    """Test hook: "auto", "simt" (CUDA cores), "tensor" (tcgen05),
    "tensor-single" (tcgen05, single-CTA tiles only) or "tensor-pair"
    (tcgen05 CTA pairs wherever N is a multiple of 256)."""
    routes = {"auto": 0, "simt": 1, "tensor": 2, "tensor-single": 3, "tensor-pair": 4}
    _lib.call("pk_debug_set_gemm_route", routes[route])


def set_reference_arithmetic(enable: bool) -> None:
    """Test hook: FP16 operators (and encoder graphs recorded while it is on)
    replay the reference shaders' arithmetic on the CUDA cores -- f16 GEMM
    accumulation, sequential f32 reductions, correctly rounded exp -- for
    value-by-value comparison with the CPU restatement's reference mode."""
    _lib.call("pk_debug_set_reference_arithmetic", int(bool(enable)))


def set_gemm_tile(tile: int) -> None:
    """Test hook: force the tensor-core GEMM token tile (0 = automatic;
    128/192/256 single-CTA; -256/-384/-512 CTA pair)."""
    _lib.call("pk_debug_set_gemm_tile", int(tile))


def set_attention_route(route: str) -> None:
    """Test hook: "auto" (tensor cores for FP16), "simt" (CUDA cores), "mma"
    (the mma.sync kernel) or "tcgen05-rowmajor" (the tcgen05 kernel, with the
    positions argument given row-major [8][2T-1][128])."""
    _lib.call("pk_debug_set_attention_route", {"auto": 0, "simt": 1, "mma": 2, "tcgen05-rowmajor": 3}[route])


def set_decoder_route(route: str) -> None:
    """Test hook: "auto" (the resident FP16 decoder where it applies),
    "cluster" (one 4-CTA cluster per window) or "resident"."""
    _lib.call("pk_debug_set_decoder_route", {"auto": 0, "cluster": 1, "resident": 2}[route])
