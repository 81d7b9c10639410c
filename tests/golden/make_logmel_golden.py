"""Generate ``logmel_ref.npz`` from the reference's own log-mel front end.

Run in a container that has the reference checkout at ``$PARAKEET_REFERENCE``
(default: a ``reference`` directory beside this repository):

    python tests/golden/make_logmel_golden.py

It builds ``src/cpp/fbank/parakeet_fbank.cpp`` with ``make -C oracle ref``
(the source compiled where it lies, two Emscripten headers replaced by
``oracle/ref_shim``), feeds it seeded PCM16 windows through its exported
``parakeet_fbank_begin_batch`` / ``parakeet_fbank_compute_item`` entry points
and records inputs and outputs.  The tests only read the file.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]

# (physical sample count, valid samples) of each recorded window.
CASES = ((12_000, 12_000), (16_000, 11_111), (4_000, 159))


def pcm16(seed: int, n: int) -> np.ndarray:
    """Seeded PCM16: two tones plus noise, as int16."""
    rng = np.random.default_rng(seed)
    t = np.arange(n) / 16_000.0
    x = 0.3 * np.sin(2 * np.pi * 440.0 * t) + 0.1 * np.sin(2 * np.pi * 3100.0 * t) + 0.05 * rng.standard_normal(n)
    return np.clip(np.round(x * 32767.0), -32768, 32767).astype(np.int16)


def main() -> None:
    env = dict(os.environ)
    env.setdefault("REFERENCE", os.environ.get("PARAKEET_REFERENCE", str(ROOT.parent / "reference")))
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "ref", f"REFERENCE={env['REFERENCE']}"], check=True)
    sys.path.insert(0, str(ROOT))
    from oracle import oracle

    record = {}
    for i, (count, valid) in enumerate(CASES):
        pcm = pcm16(1000 + i, count)
        x = (pcm.astype(np.float32) / 32768.0)[None, :]
        record[f"pcm_{i}"] = pcm
        record[f"valid_{i}"] = np.array([valid], np.uint32)
        record[f"features_{i}"] = oracle.reference_fbank(x, [valid])[0]
    np.savez_compressed(HERE / "logmel_ref.npz", **record)
    print("wrote", HERE / "logmel_ref.npz")


if __name__ == "__main__":
    main()
