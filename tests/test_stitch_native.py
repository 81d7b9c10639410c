"""The native overlap merge (pk_stitch_*, libpk_b200.so host code) against
the Python restatement of src/runtime/stitch.ts, which the reference's own
known answers pin (test_stitch.py): the same tokens, trace and errors on the
reference's cases, on thousands of randomized plans, and for partial runs
joined at rank seams.  Runs on the CPU (the merge is host code)."""
from __future__ import annotations

import numpy as np
import pytest

from test_stitch import _random_decoded_windows, ids, pair, tok, win


@pytest.fixture(scope="module")
def st(pk):
    return pk.stitch


def native_stitch(st, windows):
    acc = st.NativeStitchAccumulator(collect_trace=True)
    for w in sorted(windows, key=lambda w: (w.start_sample, w.index)):
        acc.append(w)
    return acc.snapshot()


def test_reference_cases_without_pieces(st):
    cases = [
        ([tok(st, 1, 190_000), tok(st, 2, 212_000), tok(st, 3, 224_000)],
         [tok(st, 2, 213_000), tok(st, 3, 225_000), tok(st, 4, 250_000)], [1, 2, 3, 4], "contiguous"),
        ([tok(st, 1, 190_000), tok(st, 2, 210_000), tok(st, 9, 218_000), tok(st, 3, 225_000), tok(st, 4, 235_000)],
         [tok(st, 2, 211_000), tok(st, 3, 226_000), tok(st, 8, 232_000), tok(st, 4, 236_000), tok(st, 5, 250_000)],
         [1, 2, 9, 3, 8, 4, 5], "lcs"),
        ([tok(st, 1, 210_000), tok(st, 2, 230_000)], [tok(st, 3, 215_000), tok(st, 4, 240_000)], [1, 4], "midpoint"),
    ]
    for left, right, want, method in cases:
        wins = [win(st, 0, 0, 240_000, left), win(st, 1, 208_000, 448_000, right)]
        got = native_stitch(st, wins)
        assert ids(got) == want and got.trace[0].method == method
        assert got == st.stitch_token_windows(wins)


def test_randomized_plans_equal_python_merge(st, pk):
    methods = set()
    for trial in range(300):
        wins = _random_decoded_windows(st, pk.windows, np.random.default_rng(5000 + trial))
        ref = st.stitch_token_windows(wins)
        got = native_stitch(st, wins)
        assert got.tokens == ref.tokens and got.trace == ref.trace, trial
        methods.update(t.method for t in ref.trace)
    assert methods == {"disjoint", "contiguous", "lcs", "midpoint"}


def test_backward_timestamps_clamped(st):
    wins = pair(st, [tok(st, 1, 200_000), tok(st, 2, 236_000)], [tok(st, 7, 207_000), tok(st, 2, 235_000),
                                                                 tok(st, 3, 236_000)])
    assert native_stitch(st, wins) == st.stitch_token_windows(wins)


def test_append_tdt_equals_globalized_append(st, pk):
    rng = np.random.default_rng(3)
    plans = pk.windows.plan_stateless_windows(200 * 16_000)
    py = st.IncrementalStitchAccumulator(collect_trace=True)
    nat = st.NativeStitchAccumulator(collect_trace=True)
    for p in plans:
        n = int(rng.integers(0, 400))
        frames = np.sort(rng.integers(0, 188, n)).astype(np.int32)
        toks = rng.integers(0, 40, n).astype(np.int32)
        durs = rng.integers(0, 5, n).astype(np.int32)
        toks_g = st.globalize_tdt_arrays(toks, frames, durs, p)
        py.append(st.DecodedTokenWindow(p.index, p.emission_start_sample, p.emission_end_sample, tuple(toks_g)))
        nat.append_tdt(p, toks, frames, durs)
    assert nat.snapshot() == py.snapshot()


def test_partial_runs_joined_at_rank_seams(st, pk):
    wp = pk.windows
    spliced = 0
    for trial in range(150):
        wins = _random_decoded_windows(st, wp, np.random.default_rng(trial))
        ref = st.stitch_token_windows(wins)
        for world in (2, 3, 8):
            acc = st.NativeStitchAccumulator(collect_trace=True)
            for r in range(world):
                b = st.NativePartialStitchBuilder()
                for i in wp.shard_windows(len(wins), world, r):
                    b.append(wins[i])
                part = b.finish()
                py_part = st.stitch_partial([wins[i] for i in wp.shard_windows(len(wins), world, r)])
                assert part.guard == py_part.guard and part.local_ok == py_part.local_ok
                np.testing.assert_array_equal(part.tokens, py_part.tokens)
                assert part.trace == py_part.trace
                spliced += part.local_ok
                kind, back = st.unpack_partial(st.pack_partial(part))
                assert kind == "ok"
                acc.extend(back)
            got = acc.snapshot()
            assert got.tokens == ref.tokens and got.trace == ref.trace, (trial, world)
    assert spliced > 100


def test_error_payload_round_trip(st):
    assert st.unpack_partial(st.pack_error("rank 3: PkError: PK_E_TIMEOUT: wait")) == (
        "error", "rank 3: PkError: PK_E_TIMEOUT: wait")


def test_rejects_out_of_order_and_unsorted(st):
    acc = st.NativeStitchAccumulator()
    acc.append(win(st, 1, 100, 200, []))
    with pytest.raises(ValueError, match="chronological order"):
        acc.append(win(st, 0, 50, 200, []))
    with pytest.raises(ValueError, match="sorted by startSample"):
        st.NativeStitchAccumulator().append(win(st, 0, 0, 10_000, [tok(st, 1, 500), tok(st, 2, 400)]))
    with pytest.raises(ValueError, match="must not precede"):
        st.NativeStitchAccumulator().append(win(st, 0, 300, 200, []))
