"""Failure detection on the GPU without a GPU fault: the library's bounded
waits (the mbarrier wait behind the GEMM, attention and decoder kernels, and
the resident decoder's grid barrier) are made to run out on purpose through
pk_debug_wait_probe -- an mbarrier nothing arrives on, a CTA that returns
before the grid barrier -- with a limit of a quarter second.  Each must give
up after its limit, surface as PK_E_TIMEOUT with its status bit through
pk_device_status (the reference's uncapturederror / throwGpuError path,
src/runtime/webgpu-engine.ts:274, :959), and leave the context usable: the
next real operator runs and matches the oracle.  Nothing here traps, faults
or hangs a GPU."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from gpu_util import cuda, host, vp

pytestmark = pytest.mark.gpu

LIMIT_MS = 250
MBAR_BIT, GRID_BIT = 1, 32


def _status(pk, dev):
    bits = ctypes.c_uint32(0)
    rc = pk._lib.load().pk_device_status(dev.handle, ctypes.byref(bits))
    return rc, bits.value


@pytest.fixture
def own_device(pk):
    """A device handle of its own, so its status word is this test's alone."""
    dev = pk.kernels.Device(0)
    yield dev
    dev.close()


@pytest.mark.parametrize("kind, bit", [(1, MBAR_BIT), (3, GRID_BIT)])
def test_expired_wait_reports_timeout_and_context_survives(pk, oracle, own_device, kind, bit):
    import torch

    dev = own_device
    assert _status(pk, dev) == (0, 0)
    t0 = time.perf_counter()
    pk._lib.call("pk_debug_wait_probe", dev.handle, kind, LIMIT_MS, None)
    elapsed = time.perf_counter() - t0
    assert elapsed >= LIMIT_MS / 1e3 * 0.9, elapsed
    assert elapsed < 10.0, elapsed
    rc, bits = _status(pk, dev)
    assert rc == -7 and bits == bit, (rc, bits)  # PK_E_TIMEOUT
    assert _status(pk, dev) == (0, 0)  # read-and-clear

    # The context is intact: a real operator runs and matches the oracle.
    rng = np.random.default_rng(kind)
    x = rng.standard_normal((64, 1024)).astype(np.float16)
    gamma = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    tx, tg, tb = cuda(x), cuda(gamma), cuda(beta)
    out = torch.empty_like(tx)
    pk._lib.call("pk_layernorm", dev.handle, pk._lib.FP16, 64, 1024, vp(tx), vp(tg), vp(tb), 1e-5, vp(out), None)
    torch.cuda.synchronize()
    ref = oracle.layernorm(x, gamma, beta, 1e-5)
    got = host(out).astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref.astype(np.float64)) < 1e-3  # the layernorm test's bar
    assert _status(pk, dev) == (0, 0)


@pytest.mark.parametrize("kind", [0, 2])
def test_completed_wait_sets_no_status(pk, own_device, kind):
    t0 = time.perf_counter()
    pk._lib.call("pk_debug_wait_probe", own_device.handle, kind, 2000, None)
    assert time.perf_counter() - t0 < 1.0
    assert _status(pk, own_device) == (0, 0)


def test_probe_rejects_bad_arguments(pk, own_device):
    for kind, limit in ((4, 10), (-1, 10), (1, 0), (1, 2001)):  # nothing launches
        with pytest.raises(pk.PkError, match="PK_E_INVALID"):
            pk._lib.call("pk_debug_wait_probe", own_device.handle, kind, limit, None)


def test_engine_raises_on_expired_wait(pk, own_device):
    """A bounded wait that ran out (here: the probe, before a transcription)
    makes the engine raise PK_E_TIMEOUT instead of returning tokens; the read
    clears the word, and the next transcription on the same engine is clean."""
    package = pk.synthetic.make_package("fp16", bits_policy="all5", seed=0)
    package.update(pk.synthetic.make_decoder("fp16", seed=0))
    eng = pk.engine.ParakeetEngine(own_device, package, "fp16", capacity=2)
    try:
        pcm = pk.synthetic.make_pcm(20.0, seed=3)
        clean = eng.transcribe(pcm)
        pk._lib.call("pk_debug_wait_probe", own_device.handle, 1, LIMIT_MS, None)
        with pytest.raises(pk.PkError, match="PK_E_TIMEOUT"):
            eng.transcribe(pcm)
        again = eng.transcribe(pcm)
        assert again.tokens == clean.tokens
        assert _status(pk, own_device) == (0, 0)
    finally:
        eng.destroy()
