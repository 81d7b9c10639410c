"""Encoder graph API, mirroring ParakeetEncoderGraph (src/webgpu/encoder.ts:1200-1862).

``ParakeetEncoderGraph.create(device, model, profile)`` uploads a weight
package (``pk_weights_upload``) and builds the fixed-shape 24-layer graph
(``pk_encoder_create``).  ``encode(features, valid_feature_lengths)`` runs
subsampling, the Conformer layers and the projector for 1..40 windows and
returns the [B*188, 640] decoder input plus the encoder valid lengths
(``deriveEncoderValidLengths``, encoder.ts:441-479).  The whole device side of
a forward is one CUDA graph launch per call.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .kernels import Device, ParakeetError, RangeError, _precision, _stream_handle

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

FEATURE_BINS = 128
FEATURE_FRAMES = 1501
ENCODER_FRAMES = 188
ENCODER_CHANNELS = 1024
PROJECTED_CHANNELS = 640
ENCODER_LAYERS = 24
BATCH_CAPACITY = 40

_DTYPES = {"float16": _lib.DTYPE_F16, "float32": _lib.DTYPE_F32, "uint32": _lib.DTYPE_U32}


def subsampling_output_dimension(n: int) -> int:
    """floor((n + 2*1 - 3) / 2) + 1 (src/webgpu/kernels/subsampling.ts:119-122)."""
    if n <= 0:
        raise RangeError("subsampling input dimension must be a positive integer")
    return (n + 2 - 3) // 2 + 1


def derive_encoder_valid_length(feature_length: int) -> int:
    if not 0 < feature_length <= FEATURE_FRAMES:
        raise RangeError(f"featureLength must be in [1, {FEATURE_FRAMES}]")
    n = feature_length
    for _ in range(3):
        n = subsampling_output_dimension(n)
    return n


class ModelWeights:
    """Device-resident package (pk_weights); keeps host buffers alive during upload."""

    def __init__(self, device: Device, package: dict):
        descs = (_lib.TensorDesc * len(package))()
        keep = []
        for i, (name, rec) in enumerate(package.items()):
            data = np.ascontiguousarray(rec["data"])
            keep.append(data)
            shape = list(rec["shape"])
            if len(shape) > 4:
                raise ParakeetError(f"{name} has rank {len(shape)} > 4")
            name_b, layout_b = name.encode(), rec["layout"].encode()
            keep += [name_b, layout_b]
            descs[i].name = name_b
            descs[i].dtype = _DTYPES[rec["dtype"]]
            descs[i].ndim = len(shape)
            for j, s in enumerate(shape):
                descs[i].shape[j] = int(s)
            descs[i].layout = layout_b
            descs[i].data = data.ctypes.data
            descs[i].bytes = data.nbytes
        handle = ctypes.c_void_p()
        _lib.call("pk_weights_upload", device.handle, descs, len(package), ctypes.byref(handle))
        self.handle = handle
        self.device = device

    def release(self) -> None:
        if self.handle:
            _lib.load().pk_weights_release(self.handle)
            self.handle = None


class ParakeetEncoderGraph:
    def __init__(self, device: Device, weights: ModelWeights, profile: str, capacity: int, handle):
        self.device, self.weights, self.profile = device, weights, profile
        self.batch_size = capacity
        self.handle = handle
        self._destroyed = False
        dt = torch.float16 if profile == "fp16" else torch.float32
        self._output = torch.empty((capacity * ENCODER_FRAMES, PROJECTED_CHANNELS), dtype=dt,
                                   device=f"cuda:{device.ordinal}")
        self._checkpoints = False

    @staticmethod
    def create(device: Device, model, profile: str = "fp16", capacity: int = BATCH_CAPACITY):
        """model: a package dict (name -> record) or an uploaded ModelWeights."""
        if not 0 < capacity <= BATCH_CAPACITY:
            raise RangeError(f"Encoder batch capacity must be in [1, {BATCH_CAPACITY}]")
        owned = not isinstance(model, ModelWeights)
        weights = ModelWeights(device, model) if owned else model
        handle = ctypes.c_void_p()
        try:
            _lib.call("pk_encoder_create", device.handle, weights.handle, _precision(profile), capacity,
                      ctypes.byref(handle))
        except Exception:
            if owned:
                weights.release()
            raise
        return ParakeetEncoderGraph(device, weights, profile, capacity, handle)

    def _alive(self):
        if self._destroyed:
            raise ParakeetError("Parakeet encoder graph was destroyed")

    def set_checkpoints(self, enable: bool) -> None:
        self._alive()
        _lib.call("pk_encoder_set_checkpoints", self.handle, int(enable))
        self._checkpoints = enable

    def encode(self, features, valid_feature_lengths, stream=None, out=None):
        """features: f32 [B, 128, 1501] (CUDA tensor or host numpy/torch); returns
        (decoder input [B*188, 640] CUDA tensor, encoder valid lengths u32 [B])."""
        self._alive()
        lengths = np.ascontiguousarray(np.asarray(valid_feature_lengths, dtype=np.int64))
        batch = int(lengths.shape[0])
        if not 0 < batch <= self.batch_size:
            raise RangeError(f"Encoder active batch must be in [1, {self.batch_size}]")
        for i, v in enumerate(lengths):
            if not 0 < int(v) <= FEATURE_FRAMES:
                raise RangeError(f"Feature length {i} must be in [1, {FEATURE_FRAMES}]")
        lengths_u32 = lengths.astype(np.uint32)
        on_device = isinstance(features, torch.Tensor) and features.is_cuda
        if isinstance(features, np.ndarray):
            features = np.ascontiguousarray(features, dtype=np.float32)
            if features.shape != (batch, FEATURE_BINS, FEATURE_FRAMES):
                raise RangeError(f"Expected features [{batch}, 128, 1501], got {features.shape}")
            feat_ptr = features.ctypes.data
        else:
            if tuple(features.shape) != (batch, FEATURE_BINS, FEATURE_FRAMES) or features.dtype != torch.float32:
                raise RangeError("Expected f32 features [B, 128, 1501]")
            features = features.contiguous()
            feat_ptr = features.data_ptr()
        enc = np.zeros(batch, dtype=np.uint32)
        target = self._output if out is None else out
        _lib.call("pk_encoder_forward", self.handle, ctypes.c_void_p(feat_ptr), int(on_device),
                  lengths_u32.ctypes.data_as(ctypes.c_void_p), batch, ctypes.c_void_p(target.data_ptr()),
                  int(target.is_cuda), enc.ctypes.data_as(ctypes.c_void_p), _stream_handle(stream))
        return target[: batch * ENCODER_FRAMES], enc

    def checkpoint(self, layer: int, stream=None):
        """Output of `layer` (-1 = subsampling) from the last encode, [capacity*188, 1024]."""
        self._alive()
        dt = torch.float16 if self.profile == "fp16" else torch.float32
        out = torch.empty((self.batch_size * ENCODER_FRAMES, ENCODER_CHANNELS), dtype=dt,
                          device=f"cuda:{self.device.ordinal}")
        _lib.call("pk_encoder_checkpoint", self.handle, layer, ctypes.c_void_p(out.data_ptr()),
                  _stream_handle(stream))
        return out

    def decoder_input(self):
        """The projected [capacity*188, 640] buffer (ParakeetEncoderGraph.decoderInput)."""
        return self._output

    def destroy(self) -> None:
        if not self._destroyed:
            _lib.load().pk_encoder_destroy(self.handle)
            self._destroyed = True
