"""CPU checks of the oracle's TDT decoder control flow (tdt-decoder.ts:1702-1990)
on decoders whose every choice is known in advance."""
from __future__ import annotations

import numpy as np
import pytest

from decoder_util import forced_decoder


def _enc(batch, frames, dt, seed=0):
    return np.random.default_rng(seed).normal(0, 1, (batch, frames, 640)).astype(dt)


def test_blank_with_duration_skips_frames(pk, oracle):
    dec = forced_decoder(pk, "fp32", 1024, 3)  # blank, advance 3 frames per step
    tok, fr, du, cnt, st = oracle.tdt_decode(_enc(2, 20, np.float32), [20, 7], dec, max_tokens=8)
    assert list(cnt) == [0, 0] and list(st) == [0, 0]


def test_nonblank_duration_zero_caps_at_ten_symbols_per_frame(pk, oracle):
    dec = forced_decoder(pk, "fp32", 7, 0)  # token 7, duration 0: forced advance after 10
    tok, fr, du, cnt, st = oracle.tdt_decode(_enc(1, 4, np.float32), [4], dec, max_tokens=64)
    assert cnt[0] == 40 and st[0] == 0
    assert np.all(tok[0, :40] == 7) and np.all(du[0, :40] == 0)
    assert list(fr[0, :40]) == [f for f in range(4) for _ in range(10)]


def test_overflow_sets_the_status_flag(pk, oracle):
    dec = forced_decoder(pk, "fp32", 7, 0)
    tok, fr, du, cnt, st = oracle.tdt_decode(_enc(1, 4, np.float32), [4], dec, max_tokens=15)
    assert cnt[0] == 15 and st[0] == 1


def test_flush_emits_bounded_continuation(pk, oracle):
    # Token 9 with duration 2: main loop emits at frames 0, 2, 4; the flush
    # then probes up to 10 more symbols (no blanks), frames clamped to L-1.
    dec = forced_decoder(pk, "fp32", 9, 2)
    tok, fr, du, cnt, st = oracle.tdt_decode(_enc(1, 6, np.float32), [6], dec, max_tokens=32, flush=[1])
    assert cnt[0] == 3 + 10
    assert list(fr[0, :3]) == [0, 2, 4]
    assert list(fr[0, 3:13]) == [5] * 10


def test_start_end_window(pk, oracle):
    dec = forced_decoder(pk, "fp32", 5, 1)  # one token per frame
    tok, fr, du, cnt, st = oracle.tdt_decode(_enc(1, 30, np.float32), [30], dec, max_tokens=40,
                                             starts=[4], ends=[12])
    assert cnt[0] == 8 and list(fr[0, :8]) == list(range(4, 12))


@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_random_decoder_emits_a_mix(pk, oracle, precision):
    dt = np.float16 if precision == "fp16" else np.float32
    dec = {k: v["data"] for k, v in pk.synthetic.make_decoder(precision, seed=1).items()}
    tok, fr, du, cnt, st = oracle.tdt_decode(_enc(1, 40, dt, seed=2), [40], dec, max_tokens=200)
    assert 0 < cnt[0] < 200 and st[0] == 0
    assert np.all(tok[0, :cnt[0]] < 1024) and np.all(du[0, :cnt[0]] <= 4)
    assert np.all(np.diff(fr[0, :cnt[0]].astype(np.int64)) >= 0)
