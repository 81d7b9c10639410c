"""Pins the oracle and the host-side format code to the reference's golden vectors.

Fixtures in tests/golden/ were produced by tests/golden/make_golden.py from the
reference converter (model/convert.py); the word values of palette_kat.json are
the known answers of model/tests/test_convert.py:447-479.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"

# model/tests/test_convert.py:449-463 (exact LSB-first words for codes 0..N-1).
REFERENCE_KAT = {
    5: [0x8A418820, 0xC5A92839, 0xCA307B9A, 0x38BDAB49, 0xFFBBCDEB],
    6: [0x440C2040, 0xA2481C61, 0x3CE34C2C],
}


@pytest.fixture(scope="module")
def fixtures():
    return np.load(GOLDEN / "converter_fixtures.npz")


def test_kat_fixture_matches_reference_test_literals():
    kat = json.loads((GOLDEN / "palette_kat.json").read_text())
    for bits, words in REFERENCE_KAT.items():
        assert kat[str(bits)] == words


@pytest.mark.parametrize("bits,count", [(5, 32), (6, 16)])
def test_oracle_and_host_packing_reproduce_kat(oracle, pk, bits, count):
    codes = np.arange(count, dtype=np.uint8)
    expected = np.array(REFERENCE_KAT[bits], dtype="<u4")
    np.testing.assert_array_equal(oracle.pack_codes(codes, bits).reshape(-1), expected)
    np.testing.assert_array_equal(pk.runtime_plan.pack_codes(codes, bits).reshape(-1), expected)
    np.testing.assert_array_equal(oracle.unpack_codes(expected, bits), codes)
    np.testing.assert_array_equal(pk.runtime_plan.unpack_codes(expected, bits), codes)
    assert expected[0].tobytes() == int(REFERENCE_KAT[bits][0]).to_bytes(4, "little")


@pytest.mark.parametrize("bits", [5, 6])
def test_random_k_major_codes_match_reference_packer(oracle, pk, fixtures, bits):
    codes, words = fixtures[f"codes{bits}"], fixtures[f"words{bits}"]
    np.testing.assert_array_equal(oracle.pack_codes(codes, bits), words)
    np.testing.assert_array_equal(pk.runtime_plan.pack_codes(codes, bits), words)
    np.testing.assert_array_equal(oracle.unpack_codes(words, bits), codes.reshape(-1))


def test_relative_position_table_matches_converter(pk, fixtures):
    table = pk.runtime_plan.build_relative_positions()
    assert table.shape == (375, 1024) and table.dtype == np.float32
    np.testing.assert_array_equal(table[fixtures["relpos_rows"]], fixtures["relpos_sampled"])
    assert hashlib.sha256(table.tobytes()).digest() == fixtures["relpos_sha256"].tobytes()
    # test_convert.py:812-814: position 0 row is sin(0)=0 / cos(0)=1.
    np.testing.assert_array_equal(table[187, 0::2], 0)
    np.testing.assert_array_equal(table[187, 1::2], 1)


def test_projected_positions_match_converter(pk, fixtures):
    rp = pk.runtime_plan
    seed = int(fixtures["projection_weight_seed"][0])
    weight = (np.random.default_rng(seed).standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    projected = rp.project_relative_positions(rp.build_relative_positions(), weight, dtype=np.float16)
    packed = rp.pack_projected_relative_positions(projected)
    assert packed.shape == (8, 32, 375, 4)
    np.testing.assert_array_equal(packed[0], fixtures["projected_head0"])
    assert hashlib.sha256(packed.tobytes()).digest() == fixtures["projected_sha256"].tobytes()


def test_projection_orientation_kat(pk):
    # test_convert.py:817-826
    out = pk.runtime_plan.project_relative_positions(np.array([[1, 2], [3, 4]], np.float32),
                                                     np.array([[1, 3], [2, 4]], np.float32))
    np.testing.assert_array_equal(out, np.array([[7, 10], [15, 22]], dtype=np.float16))


def test_head_vector_packing_kat(pk):
    # test_convert.py:828-840
    projected = np.arange(16, dtype=np.float16).reshape(2, 8)
    packed = pk.runtime_plan.pack_projected_relative_positions(projected, heads=2)
    assert packed.shape == (2, 1, 2, 4)
    np.testing.assert_array_equal(packed[0, 0, 0], projected[0, 0:4])
    np.testing.assert_array_equal(packed[0, 0, 1], projected[1, 0:4])
    np.testing.assert_array_equal(packed[1, 0, 0], projected[0, 4:8])
    np.testing.assert_array_equal(packed[1, 0, 1], projected[1, 4:8])


def test_conv_weight_layouts_match_converter(fixtures):
    # kernel-channel-vec4: [9, C] = source[:, 0, :].T (convert.py:1893-1918)
    np.testing.assert_array_equal(fixtures["dw_packed"].reshape(9, 1024),
                                  fixtures["dw_source"][:, 0, :].T.astype(np.float16))
    # kh-kw-output-channel-vec4: [3, 3, C] = source[:, 0].transpose(1, 2, 0) (convert.py:1839-1878)
    np.testing.assert_array_equal(fixtures["conv0_packed"].reshape(3, 3, 256),
                                  fixtures["conv0_source"][:, 0].transpose(1, 2, 0).astype(np.float16))
