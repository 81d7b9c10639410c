"""Helpers shared by the GPU parity tests: numpy <-> CUDA tensors and direct
C-ABI calls (every GPU test goes through libpk_b200.so)."""
from __future__ import annotations

import ctypes

import numpy as np


# Device copies made by cuda() stay referenced until release(): a raw pointer
# handed to the C ABI does not keep a torch tensor alive, and the caching
# allocator would otherwise hand the same block to the next temporary.
_KEEP: list = []


def cuda(arr):
    import torch

    arr = np.ascontiguousarray(arr)
    if arr.dtype == np.dtype("<u4"):
        t = torch.from_numpy(arr.view(np.int32)).cuda()
    else:
        t = torch.from_numpy(arr).cuda()
    _KEEP.append(t)
    return t


def release():
    import torch

    if _KEEP:
        torch.cuda.synchronize()
        _KEEP.clear()


def host(t, dtype=None):
    import torch

    torch.cuda.synchronize()
    a = t.cpu().numpy()
    return a if dtype is None else a.view(dtype)


def vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def gemm(pk, device, a, codes, lut, bits, columns, *, bias=None, residual=None, residual_scale=1.0,
         activation="none", precision=None, rows=None):
    """Runs pk_palette_gemm on numpy inputs; returns the numpy result."""
    import torch

    L = pk._lib
    prec = L.FP16 if a.dtype == np.float16 else L.FP32
    rows = a.shape[0] if rows is None else rows
    inner = a.shape[1]
    ta, tc, tl = cuda(a), cuda(codes), cuda(lut)
    tb = cuda(bias.astype(np.float32)) if bias is not None else None
    tr = cuda(residual) if residual is not None else None
    out = torch.full((a.shape[0], columns), float("nan"), dtype=ta.dtype, device="cuda")
    groups = lut.shape[0]
    desc = L.GemmDesc(prec, rows, inner, columns, bits, groups, columns // groups, L.ACT[activation],
                      int(residual is not None), float(residual_scale), vp(tb), vp(tr), vp(ta), vp(tc), vp(tl),
                      vp(out))
    L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), None)
    return host(out)
