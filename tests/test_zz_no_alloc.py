"""pk_rel_attention_noalloc: the attention entry point for callers that may
not allocate device memory (a host that owns a fixed device pool, a process
under a scheduler-set memory cap, a harness that must see every allocation up
front).  It keeps its scratch in a fixed array inside the library and takes no
device handle, so such callers can run the encoder's tcgen05 attention on
buffers they already hold.

This file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.  It passes alone in a fresh
process and after the rest of the suite (the scratch array keeps the previous
call's contents; each call rewrites what it reads)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import cuda, host, vp

pytestmark = pytest.mark.gpu

TOL = 5e-3  # tcgen05 (this entry point) vs mma.sync (pk_rel_attention) kernels, FP16 outputs
ORACLE_TOL = 5e-3  # FP16 attention vs the CPU restatement of the reference shader (f32 math)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _inputs(seed, frames, lengths):
    rng = np.random.default_rng(seed)
    batch, P = len(lengths), 2 * frames - 1
    qkv = rng.standard_normal((batch * frames, 3072)).astype(np.float16)
    pos = (0.5 * rng.standard_normal((8, 32, P, 4))).astype(np.float16)  # package layout
    u = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    v = (0.02 * rng.standard_normal((8, 128))).astype(np.float32)
    return qkv, pos, u, v, np.array(lengths, np.uint32)


def test_noalloc_attention_matches_pk_rel_attention_twice(pk, oracle, device):
    import torch

    lib = pk._lib
    # Two calls in a row on different shapes and inputs: the second call must
    # not see anything the first left in the shared scratch array.
    for seed, frames, lengths in ((5, 188, [188, 150, 1]), (6, 77, [77, 40])):
        qkv, pos, u, v, lens = _inputs(seed, frames, lengths)
        tq, tp, tu, tv, tl = cuda(qkv), cuda(pos), cuda(u), cuda(v), cuda(lens)
        batch = len(lengths)
        ref = torch.full((batch * frames, 1024), float("nan"), dtype=torch.float16, device="cuda")
        got = torch.full_like(ref, float("nan"))
        lib.call("pk_rel_attention", device.handle, lib.FP16, batch, frames, vp(tq), vp(tp), vp(tu), vp(tv),
                 vp(tl), vp(ref), None)
        status = ctypes.c_uint32(0xFFFFFFFF)
        lib.call("pk_rel_attention_noalloc", batch, frames, vp(tq), vp(tp), vp(tu), vp(tv), vp(tl), vp(got),
                 ctypes.byref(status), None)
        assert status.value == 0
        g, r = host(got), host(ref)
        assert np.isfinite(g).all()
        assert rel(g, r) < TOL, (frames, rel(g, r))
        expected = oracle.rel_attention(qkv, pos, u, v, lens, batch, frames)
        assert rel(g, expected) < ORACLE_TOL, (frames, rel(g, expected))
        for b, L in enumerate(lengths):
            assert np.all(g.reshape(batch, frames, 1024)[b, L:] == 0)


def test_noalloc_attention_rejects_windows_beyond_its_scratch(pk):
    x = cuda(np.zeros(8, np.float32))
    with pytest.raises(pk.PkError, match="PK_E_SHAPE"):
        pk._lib.call("pk_rel_attention_noalloc", 1, 193, vp(x), vp(x), vp(x), vp(x), vp(x), vp(x), None, None)
