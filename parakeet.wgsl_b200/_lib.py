"""ctypes binding of libpk_b200.so (the C ABI declared in include/pk_b200.h).

The library is built in-tree by ``build.py``.  There is no fallback: if the
shared object is missing or cannot be loaded, every entry point raises
``PkError`` -- the operators never fall back to CPU or framework code.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpk_b200.so"

PK_OK = 0
STATUS_NAMES = {
    -1: "PK_E_INVALID", -2: "PK_E_SHAPE", -3: "PK_E_LAYOUT", -4: "PK_E_SIGNATURE",
    -5: "PK_E_CUDA", -6: "PK_E_OOM", -7: "PK_E_TIMEOUT", -8: "PK_E_DESTROYED", -9: "PK_E_NOT_FOUND",
}
FP16, FP32 = 0, 1
ACT = {"none": 0, "silu": 1, "relu": 2}
LAYOUT_ROW_MAJOR, LAYOUT_TILE_MAJOR = 0, 1
DTYPE_F16, DTYPE_F32, DTYPE_U32 = 0, 1, 2

# Every symbol include/pk_b200.h declares.
EXPORTED = (
    "pk_last_error", "pk_version", "pk_device_open", "pk_device_close", "pk_device_status",
    "pk_palette_expand", "pk_palette_gemm", "pk_layernorm", "pk_rel_attention", "pk_rel_attention_noalloc",
    "pk_conformer_conv",
    "pk_subsampling_conv0_dw2", "pk_subsampling_depthwise", "pk_subsampling_time_mask", "pk_tdt_decode",
    "pk_logmel",
    "pk_weights_upload", "pk_weights_release", "pk_encoder_create", "pk_encoder_forward",
    "pk_encoder_set_checkpoints", "pk_encoder_checkpoint", "pk_encoder_destroy", "pk_debug_set_gemm_route",
    "pk_debug_set_gemm_tile", "pk_debug_set_attention_route", "pk_debug_set_decoder_route",
    "pk_debug_wait_probe", "pk_stitch_create", "pk_stitch_destroy", "pk_stitch_append", "pk_stitch_append_tdt",
    "pk_stitch_extend", "pk_stitch_counts", "pk_stitch_read", "pk_stitch_read_run",
    "pk_debug_set_reference_arithmetic",
)
STITCH_COLLECT_TRACE, STITCH_RECORD_RUN = 1, 2


class StitchRun(ctypes.Structure):
    """pk_stitch_run: a run of windows merged on its own (another rank's)."""
    _fields_ = [
        ("window_meta", ctypes.c_void_p), ("windows", ctypes.c_int64), ("window_tokens", ctypes.c_void_p),
        ("merged", ctypes.c_void_p), ("tokens", ctypes.c_int64), ("trace", ctypes.c_void_p),
        ("trace_entries", ctypes.c_int64), ("guard", ctypes.c_int64), ("local_ok", ctypes.c_int),
    ]


class PkError(RuntimeError):
    """An entry point returned a negative pk_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class PaletteDesc(ctypes.Structure):
    _fields_ = [
        ("precision", ctypes.c_int), ("bits", ctypes.c_int), ("inner", ctypes.c_int64),
        ("columns", ctypes.c_int64), ("palette_groups", ctypes.c_int),
        ("palette_group_columns", ctypes.c_int64), ("layout", ctypes.c_int),
        ("codes", ctypes.c_void_p), ("palette", ctypes.c_void_p), ("target", ctypes.c_void_p),
    ]


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("precision", ctypes.c_int), ("rows", ctypes.c_int64), ("inner", ctypes.c_int64),
        ("columns", ctypes.c_int64), ("bits", ctypes.c_int), ("palette_groups", ctypes.c_int),
        ("palette_group_columns", ctypes.c_int64), ("activation", ctypes.c_int),
        ("has_residual", ctypes.c_int), ("residual_scale", ctypes.c_float),
        ("bias", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("a", ctypes.c_void_p),
        ("codes", ctypes.c_void_p), ("palette", ctypes.c_void_p), ("c", ctypes.c_void_p),
    ]


class TdtDesc(ctypes.Structure):
    _fields_ = [
        ("precision", ctypes.c_int), ("batch", ctypes.c_int), ("frames", ctypes.c_int),
        ("max_tokens", ctypes.c_int),
    ] + [(n, ctypes.c_void_p) for n in (
        "encoder_projected", "encoded_lengths", "decode_starts", "decode_ends", "flush_finals", "embedding",
        "lstm_weight0", "lstm_bias0", "lstm_weight1", "lstm_bias1", "projector_weight", "projector_bias",
        "head_weight", "head_bias", "tokens", "token_frames", "token_durations", "metadata")]


class TensorDesc(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
        ("shape", ctypes.c_int64 * 4), ("layout", ctypes.c_char_p), ("data", ctypes.c_void_p),
        ("bytes", ctypes.c_size_t),
    ]


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libpk_b200.so once; raise PkError (never fall back) if unavailable."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise PkError(-5, f"{LIB_PATH} is not built (run parakeet.wgsl_b200/build.py)")
        lib = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
        sig = {
            "pk_last_error": [ctypes.c_char_p, sz],
            "pk_version": [],
            "pk_device_open": [i32, ctypes.POINTER(vp)],
            "pk_device_close": [vp],
            "pk_device_status": [vp, ctypes.POINTER(ctypes.c_uint32)],
            "pk_palette_expand": [vp, ctypes.POINTER(PaletteDesc), vp],
            "pk_palette_gemm": [vp, ctypes.POINTER(GemmDesc), vp],
            "pk_layernorm": [vp, i32, i64, i64, vp, vp, vp, f32, vp, vp],
            "pk_rel_attention": [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp],
            "pk_rel_attention_noalloc": [i32, i32, vp, vp, vp, vp, vp, vp, ctypes.POINTER(ctypes.c_uint32), vp],
            "pk_conformer_conv": [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp],
            "pk_subsampling_conv0_dw2": [vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp],
            "pk_subsampling_depthwise": [vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, i32, vp, vp],
            "pk_subsampling_time_mask": [vp, i32, i32, i32, i32, i32, vp, vp, i32, vp],
            "pk_tdt_decode": [vp, ctypes.POINTER(TdtDesc), vp],
            "pk_logmel": [vp, i32, i32, vp, vp, vp, vp],
            "pk_weights_upload": [vp, ctypes.POINTER(TensorDesc), i32, ctypes.POINTER(vp)],
            "pk_weights_release": [vp],
            "pk_encoder_create": [vp, vp, i32, i32, ctypes.POINTER(vp)],
            "pk_encoder_forward": [vp, vp, i32, vp, i32, vp, i32, vp, vp],
            "pk_encoder_set_checkpoints": [vp, i32],
            "pk_encoder_checkpoint": [vp, i32, vp, vp],
            "pk_encoder_destroy": [vp],
            "pk_debug_set_gemm_route": [i32],
            "pk_debug_set_gemm_tile": [i32],
            "pk_debug_set_reference_arithmetic": [i32],
            "pk_debug_set_attention_route": [i32],
            "pk_debug_set_decoder_route": [i32],
            "pk_debug_wait_probe": [vp, i32, ctypes.c_uint32, vp],
            "pk_stitch_create": [i32, ctypes.POINTER(vp)],
            "pk_stitch_destroy": [vp],
            "pk_stitch_append": [vp, vp, vp, i64],
            "pk_stitch_append_tdt": [vp, vp, vp, vp, vp, i64],
            "pk_stitch_extend": [vp, ctypes.POINTER(StitchRun)],
            "pk_stitch_counts": [vp, vp],
            "pk_stitch_read": [vp, i32, vp, vp],
            "pk_stitch_read_run": [vp, vp, vp, vp],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().pk_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != PK_OK:
        raise PkError(status, last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
