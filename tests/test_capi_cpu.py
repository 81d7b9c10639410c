"""CPU-side checks of the C ABI and of the host mirror of the operator API.

No compute runs here: the library must load, export every symbol the public
header declares, and the Python operator classes must reject what the
reference's createDispatch rejects before any GPU work."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "pk_b200.h").read_text()
    return sorted(set(re.findall(r"^int (pk_\w+)\(", text, flags=re.M)))


def test_library_loads_and_exports_every_header_symbol(pk):
    lib = pk._lib.load()
    syms = header_symbols()
    assert len(syms) >= 20
    for name in syms:
        assert hasattr(lib, name), name
    assert set(syms) == set(pk._lib.EXPORTED)
    assert lib.pk_version() == 1


def test_library_has_only_sm100a_device_code():
    import subprocess

    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", str(ROOT / "parakeet.wgsl_b200" /
                                                                              "libpk_b200.so")],
                         capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert arches == {"100a"}, arches


def test_last_error_roundtrip(pk):
    lib = pk._lib.load()
    handle = ctypes.c_void_p()
    st = lib.pk_device_open(-1, ctypes.byref(handle))
    assert st < 0
    assert pk._lib.last_error()
    with pytest.raises(pk.PkError):
        pk._lib.call("pk_device_open", -1, ctypes.byref(handle))


def test_null_arguments_are_rejected_without_a_gpu(pk):
    lib = pk._lib.load()
    assert lib.pk_palette_gemm(None, None, None) == -1
    assert lib.pk_layernorm(None, 0, 1, 1024, None, None, None, 1e-5, None, None) == -1
    assert lib.pk_encoder_forward(None, None, 0, None, 1, None, 0, None, None) == -1


class _FakeDevice:
    handle = None
    ordinal = 0


def _tensor(pk, name, shape, layout, dtype="uint32", numel=None):
    import torch

    n = numel if numel is not None else int(np.prod(shape))
    return pk.kernels.GpuTensor(name, dtype, tuple(shape), layout, torch.zeros(n))


def _desc(pk, **kw):
    import torch

    rp = pk.runtime_plan
    inner, columns = kw.pop("inner", 1024), kw.pop("columns", 4096)
    bits = kw.pop("bits", 5)
    per, words = rp.code_group(bits)
    b = _tensor(pk, "w", (inner, columns), rp.palette_layout(bits), numel=inner * columns // per * words)
    pal = _tensor(pk, "w.palette", (kw.pop("groups", 1), 1 << bits), rp.PALETTE_LUT_LAYOUT, dtype="float16")
    d = dict(label="t", a=torch.zeros(1), b=b, output=torch.zeros(1), rows=7520, inner=inner, columns=columns,
             b_palette=pal, palette_group_columns=columns // pal.shape[0], activation="silu")
    d.update(kw)
    return pk.kernels.GemmDescriptor(**d)


def test_gemm_create_dispatch_accepts_production_signature(pk):
    k = pk.kernels.F16GemmKernel.create(_FakeDevice())
    disp = k.create_dispatch(_desc(pk))
    assert disp.label == "t"
    disp.destroy()
    disp.destroy()  # idempotent
    with pytest.raises(pk.kernels.ParakeetError, match="destroyed"):
        disp.encode()


def test_gemm_rejects_like_the_reference(pk):
    K = pk.kernels
    k = K.F16GemmKernel.create(_FakeDevice())
    with pytest.raises(K.RangeError, match="Unsupported GEMM shape"):
        k.create_dispatch(_desc(pk, inner=1000))
    with pytest.raises(K.ParakeetError, match="not a fixed production GEMM signature"):
        k.create_dispatch(_desc(pk, activation="relu"))
    with pytest.raises(K.ParakeetError, match="residual scale without a residual"):
        k.create_dispatch(_desc(pk, activation="none", residual_scale=0.5))
    with pytest.raises(K.ParakeetError, match="weight package does not match"):
        bad = _desc(pk)
        bad.b.shape = (1024, 2048)
        k.create_dispatch(bad)
    with pytest.raises(K.ParakeetError, match="invalid transient palette weights"):
        k.create_dispatch(_desc(pk, palette_group_columns=100))
    with pytest.raises(K.ParakeetError, match="requires an FP32"):
        K.F32GemmKernel.create(_FakeDevice(), profile="fp16")


def test_qkv_signature_with_three_palette_groups(pk):
    k = pk.kernels.F16GemmKernel.create(_FakeDevice())
    d = _desc(pk, columns=3072, groups=3, activation="none")
    assert k.create_dispatch(d).groups == 3


def test_encoder_length_derivation(pk):
    enc = pk.encoder
    assert enc.derive_encoder_valid_length(1501) == 188
    assert enc.derive_encoder_valid_length(1500) == 188
    assert enc.derive_encoder_valid_length(1) == 1
    assert enc.derive_encoder_valid_length(700) == 88
    with pytest.raises(pk.kernels.RangeError):
        enc.derive_encoder_valid_length(1502)


def test_synthetic_package_inventory(pk):
    pkg = pk.synthetic.make_package("fp16", layers=1, seed=0)
    assert pkg["encoder.layers.0.self_attn.o_proj.weight"]["bits"] == 6
    assert pkg["encoder.layers.0.feed_forward1.linear1.weight"]["bits"] == 5
    assert pkg["encoder.layers.0.self_attn.qkv.weight.palette"]["shape"] == (3, 32)
    assert pkg["encoder.layers.0.self_attn.projected_positions"]["data"].shape == (8, 32, 375, 4)
    lut = pkg["encoder.layers.0.conv.pointwise_conv1.weight.palette"]["data"]
    assert np.all(np.diff(lut.astype(np.float32), axis=1) >= 0)  # sorted LUT
    # Packed byte length matches the reference's storage contract.
    w = pkg["encoder.layers.0.feed_forward1.linear2.weight"]
    assert w["data"].nbytes == 4096 * 1024 // 32 * 5 * 4
