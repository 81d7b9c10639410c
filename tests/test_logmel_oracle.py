"""The log-mel oracle against the reference's own front end: the committed
fixtures (tests/golden/logmel_ref.npz, made by make_logmel_golden.py from
src/cpp/fbank/parakeet_fbank.cpp) and, where oracle/_ref is built, live
full-length windows."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden" / "logmel_ref.npz"


def test_oracle_matches_reference_fixtures_bit_exactly(oracle):
    g = np.load(GOLDEN)
    for i in range(3):
        x = (g[f"pcm_{i}"].astype(np.float32) / 32768.0)[None, :]
        got = oracle.logmel(x, g[f"valid_{i}"])[0]
        ref = g[f"features_{i}"]
        assert got.shape == ref.shape
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_short_valid_length_is_all_zero(oracle):
    g = np.load(GOLDEN)
    assert not np.any(g["features_2"])  # 159 valid samples: no valid frame


def test_oracle_matches_live_reference_full_windows(oracle):
    if not oracle.reference_fbank_available():
        pytest.skip("oracle/_ref (the reference front end) is not built here")
    rng = np.random.default_rng(3)
    x = (0.2 * rng.standard_normal((2, 240_000))).astype(np.float32)
    valid = [240_000, 187_523]
    got = oracle.logmel(x, valid)
    ref = oracle.reference_fbank(x, valid)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
