"""Generate the golden fixtures in this directory from the reference's own code.

Run in a container that has the reference checkout (read-only) at
``$PARAKEET_REFERENCE`` (default: a ``reference`` directory beside this repository):

    python tests/golden/make_golden.py

It imports the reference's converter (``model/convert.py``) -- the only part of
the reference's path that is executable without a browser -- and records:

* ``palette_kat.json``: the exact LSB-first words of the reference's
  known-answer test (``model/tests/test_convert.py:447-479``), re-derived by
  calling ``convert.pack_palette_codes_lsb`` on codes 0..31 / 0..15;
* ``converter_fixtures.npz``:
  - seeded random 5-bit [64, 256] and 6-bit [64, 128] code matrices with the
    words ``pack_palette_codes_lsb`` produces for them (K-major code order,
    ``model/convert.py:2130-2157``);
  - the relative-position table ``build_relative_positions()`` (375 x 1024,
    ``model/convert.py:1143-1165``) sampled at a few rows plus the SHA-256 of
    the whole table;
  - a seeded projection + head-vector packing of that table
    (``project_relative_positions`` / ``pack_projected_relative_positions``,
    ``model/convert.py:1168-1228``) for an 8-head, 1024-channel weight;
  - ``pack_conformer_depthwise_kernel`` / ``pack_conv0_kernel`` layouts for a
    small seeded source (``model/convert.py:1839-1918``).

The tests only read these files; nothing in the reference checkout is touched
at test time.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PROJECTION_SEED = 7  # weight = default_rng(7).standard_normal((1024, 1024)) * 0.02, f32
REFERENCE = Path(os.environ.get("PARAKEET_REFERENCE", str(HERE.parents[2] / "reference")))


def main() -> None:
    sys.path.insert(0, str(REFERENCE / "model"))
    import convert  # type: ignore  # the reference converter

    kat = {}
    for bits, count in ((5, 32), (6, 16)):
        words = convert.pack_palette_codes_lsb(np.arange(count, dtype=np.uint8), bits=bits)
        kat[str(bits)] = [int(w) for w in words.reshape(-1)]
    (HERE / "palette_kat.json").write_text(json.dumps(kat, indent=1) + "\n")

    rng = np.random.default_rng(20261201)
    codes5 = rng.integers(0, 32, size=(64, 256), dtype=np.uint8)
    codes6 = rng.integers(0, 64, size=(64, 128), dtype=np.uint8)
    words5 = convert.pack_palette_codes_lsb(codes5, bits=5)
    words6 = convert.pack_palette_codes_lsb(codes6, bits=6)

    table = convert.build_relative_positions()
    rows = np.array([0, 1, 93, 186, 187, 188, 300, 374])
    weight = (np.random.default_rng(PROJECTION_SEED).standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    projected = convert.project_relative_positions(table, weight, float_dtype="float16")
    packed_positions = convert.pack_projected_relative_positions(projected, float_dtype="float16")

    dw_source = rng.standard_normal((1024, 1, 9)).astype(np.float32)
    dw_packed, _ = convert.pack_conformer_depthwise_kernel(dw_source, float_dtype="float16")
    conv0_source = rng.standard_normal((256, 1, 3, 3)).astype(np.float32)
    conv0_packed, _ = convert.pack_conv0_kernel(conv0_source, float_dtype="float16")

    np.savez_compressed(
        HERE / "converter_fixtures.npz",
        codes5=codes5, words5=words5, codes6=codes6, words6=words6,
        relpos_rows=rows, relpos_sampled=table[rows],
        relpos_sha256=np.frombuffer(hashlib.sha256(table.tobytes()).digest(), dtype=np.uint8),
        projection_weight_seed=np.array([PROJECTION_SEED]),
        projected_head0=packed_positions[0],
        projected_sha256=np.frombuffer(hashlib.sha256(packed_positions.tobytes()).digest(), dtype=np.uint8),
        dw_source=dw_source, dw_packed=dw_packed,
        conv0_source=conv0_source, conv0_packed=conv0_packed,
    )
    print("wrote", HERE / "palette_kat.json", HERE / "converter_fixtures.npz")


if __name__ == "__main__":
    main()
