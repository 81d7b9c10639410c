"""GPU log-mel front end (pk_logmel) against the oracle and the reference's
fixtures, through the C ABI.

The kernel replays the reference's operations with the same rounding; only
the double-precision log comes from a different math library, so a value can
differ in its last f32 bit when the two logs straddle a rounding boundary.
Bar: at least 99.99 % of values bit-identical, and every value within 1e-5 of
the oracle (normalized features are O(1))."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from gpu_util import cuda, host

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "logmel_ref.npz"


def _gpu(pk, device, x, valid):
    fb = pk.kernels.ParakeetFbank(device)
    out = fb.compute_batch(cuda(np.ascontiguousarray(x, np.float32)), cuda(np.asarray(valid, np.uint32)))
    return host(out)


def _check(got, ref):
    assert got.shape == ref.shape
    same = np.mean(got.view(np.uint32) == ref.view(np.uint32))
    print(f"logmel: bit-identical fraction {same:.6f}, max abs diff {np.abs(got - ref).max():.3e}")
    assert same >= 0.9999
    assert np.abs(got - ref).max() <= 1e-5


def test_logmel_full_windows_match_oracle(pk, oracle, device):
    rng = np.random.default_rng(8)
    x = (0.2 * rng.standard_normal((3, 240_000))).astype(np.float32)
    valid = [240_000, 100_007, 159]
    got = _gpu(pk, device, x, valid)
    ref = oracle.logmel(x, valid)
    _check(got, ref)
    assert not np.any(got[2])
    assert not np.any(got[1][:, 100_007 // 160:])


def test_logmel_matches_reference_fixtures(pk, device):
    g = np.load(GOLDEN)
    for i in range(3):
        x = (g[f"pcm_{i}"].astype(np.float32) / 32768.0)[None, :]
        _check(_gpu(pk, device, x, g[f"valid_{i}"])[0], g[f"features_{i}"])


def test_logmel_rejects_bad_shapes(pk, device):
    x = cuda(np.zeros((1, 100), np.float32))
    v = cuda(np.zeros(1, np.uint32))
    with pytest.raises(pk.kernels.RangeError):
        pk.kernels.ParakeetFbank(device).compute_batch(x, v)
