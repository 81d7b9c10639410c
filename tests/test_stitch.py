"""Host overlap merge (stitch.py) against the reference's own known answers:
every expectation below is the one test/runtime/stitch.test.ts asserts for
the same inputs (src/runtime/stitch.ts)."""
from __future__ import annotations

import math

import pytest


@pytest.fixture(scope="module")
def st(pk):
    return pk.stitch


def tok(st, token_id, start, end=None):
    end = start if end is None else end
    return st.TimedToken(token_id, start, end, max(1, math.ceil((end - start) / 1280)))


def ftok(st, token_id, frame):
    return tok(st, token_id, frame * 1280, frame * 1280 + 1280)


def win(st, index, start, end, tokens):
    return st.DecodedTokenWindow(index, start, end, tuple(tokens))


def pair(st, left, right):
    return [win(st, 0, 0, 240_000, left), win(st, 1, 206_080, 446_080, right)]


def ids(result):
    return [t.token_id for t in result.tokens]


def resolver(vocab):
    return lambda tid: vocab.get(tid)


def test_contiguous_splice(st):
    r = st.stitch_token_windows([
        win(st, 0, 0, 240_000, [tok(st, 1, 190_000), tok(st, 2, 212_000), tok(st, 3, 224_000)]),
        win(st, 1, 208_000, 448_000, [tok(st, 2, 213_000), tok(st, 3, 225_000), tok(st, 4, 250_000)])])
    assert ids(r) == [1, 2, 3, 4]
    assert [t.method for t in r.trace] == ["contiguous"]


def test_lcs_pivot(st):
    r = st.stitch_token_windows([
        win(st, 0, 0, 240_000, [tok(st, 1, 190_000), tok(st, 2, 210_000), tok(st, 9, 218_000),
                                tok(st, 3, 225_000), tok(st, 4, 235_000)]),
        win(st, 1, 208_000, 448_000, [tok(st, 2, 211_000), tok(st, 3, 226_000), tok(st, 8, 232_000),
                                      tok(st, 4, 236_000), tok(st, 5, 250_000)])])
    assert r.trace[0].method == "lcs"
    assert ids(r) == [1, 2, 9, 3, 8, 4, 5]


def test_midpoint_without_matches(st):
    r = st.stitch_token_windows([
        win(st, 0, 0, 240_000, [tok(st, 1, 210_000), tok(st, 2, 230_000)]),
        win(st, 1, 208_000, 448_000, [tok(st, 3, 215_000), tok(st, 4, 240_000)])])
    assert r.trace[0].method == "midpoint"
    assert ids(r) == [1, 4]


def test_midpoint_keeps_right_window_without_safe_token(st):
    v = resolver({1: "▁hello", 511: "▁world", 549: "pre", 550: "ne", 551: "ta", 552: "tion"})
    r = st.stitch_token_windows(pair(st, [ftok(st, 1, 120), ftok(st, 511, 140)],
                                     [ftok(st, 549, 140), ftok(st, 550, 141), ftok(st, 551, 142),
                                      ftok(st, 552, 143)]), v)
    assert r.trace[0].method == "midpoint"
    assert ids(r) == [1, 511, 550, 551, 552]


def test_continuation_tail_mid_word(st):
    v = resolver({1: "▁hello", 424: "▁fan", 425: "tas", 426: "ti", 427: "cal"})
    r = st.stitch_token_windows(pair(st, [ftok(st, 1, 120), ftok(st, 424, 130), ftok(st, 425, 131)],
                                     [ftok(st, 425, 131), ftok(st, 426, 132), ftok(st, 427, 133)]), v)
    assert ids(r) == [1, 424, 425, 426, 427]


def test_case_only_variants_anchor(st):
    v = resolver({10: "▁the", 20: "▁meeting", 21: "▁Meeting", 30: "▁was", 40: "▁good"})
    r = st.stitch_token_windows(pair(st, [ftok(st, 10, 128), ftok(st, 30, 130), ftok(st, 20, 132)],
                                     [ftok(st, 10, 128), ftok(st, 30, 130), ftok(st, 21, 132),
                                      ftok(st, 40, 134)]), v)
    assert r.trace[0].method == "contiguous"
    assert ids(r) == [10, 30, 20, 40]


def test_orphaned_right_continuation(st):
    v = resolver({10: "▁hello", 20: "▁wor", 21: "ld", 30: "▁there", 50: "ne", 60: "▁o"})
    r = st.stitch_token_windows(pair(st, [ftok(st, 10, 120), ftok(st, 20, 133), ftok(st, 21, 135)],
                                     [ftok(st, 60, 134), ftok(st, 50, 136), ftok(st, 30, 138)]), v)
    assert r.trace[0].method == "midpoint"
    assert ids(r) == [10, 20, 21, 30]


def test_enforce_monotonic(st):
    same = [ftok(st, 100, 40), ftok(st, 101, 40), ftok(st, 102, 40)]
    out = st.enforce_monotonic_token_times(same)
    assert [t.token_id for t in out] == [100, 101, 102]
    assert [t.start_sample for t in out] == [51_200] * 3
    mono = [ftok(st, 1, 10), ftok(st, 2, 12), ftok(st, 3, 12), ftok(st, 4, 20)]
    assert st.enforce_monotonic_token_times(mono) == mono
    assert st.enforce_monotonic_token_times([]) == []


def _five_windows(st):
    return [
        win(st, 0, 0, 240_000, [tok(st, 100, 100_000), tok(st, 1, 190_000), tok(st, 2, 212_000),
                                tok(st, 3, 224_000)]),
        win(st, 1, 208_000, 448_000, [tok(st, 2, 213_000), tok(st, 3, 225_000), tok(st, 4, 300_000),
                                      tok(st, 10, 390_000), tok(st, 20, 410_000), tok(st, 99, 418_000),
                                      tok(st, 30, 425_000), tok(st, 40, 435_000)]),
        win(st, 2, 416_000, 656_000, [tok(st, 20, 411_000), tok(st, 30, 426_000), tok(st, 88, 432_000),
                                      tok(st, 40, 436_000), tok(st, 50, 500_000)]),
        win(st, 3, 624_000, 864_000, [tok(st, 60, 630_000), tok(st, 61, 810_000), tok(st, 62, 850_000)]),
        win(st, 4, 832_000, 1_072_000, [tok(st, 70, 835_000), tok(st, 71, 870_000)]),
    ]


PREFIXES = [
    [100, 1, 2, 3],
    [100, 1, 2, 3, 4, 10, 20, 99, 30, 40],
    [100, 1, 2, 3, 4, 10, 20, 99, 30, 88, 40, 50],
    [100, 1, 2, 3, 4, 10, 20, 99, 30, 88, 40, 50, 60, 61, 62],
    [100, 1, 2, 3, 4, 10, 20, 99, 30, 88, 40, 50, 60, 61, 71],
]
METHODS = ["contiguous", "lcs", "disjoint", "midpoint"]
TRACE = [(0, 1, "contiguous", 208_000, 240_000), (1, 2, "lcs", 416_000, 448_000),
         (2, 3, "disjoint", 624_000, 656_000), (3, 4, "midpoint", 832_000, 864_000)]


def test_incremental_matches_one_shot_prefixes(st):
    windows = _five_windows(st)
    pieces = resolver({tid: f"▁token-{tid}" for prefix in PREFIXES for tid in prefix})
    for piece in (None, pieces):
        acc = st.IncrementalStitchAccumulator(token_piece=piece, collect_trace=True)
        for i, w in enumerate(windows):
            acc.append(w)
            snap = acc.snapshot()
            assert snap == st.stitch_token_windows(windows[:i + 1], piece)
            assert ids(snap) == PREFIXES[i]
            assert [t.method for t in snap.trace] == METHODS[:i]
            assert [(t.left_window_index, t.right_window_index, t.method, t.overlap_start_sample,
                     t.overlap_end_sample) for t in snap.trace] == TRACE[:i]


def test_snapshot_cleanup_stays_out_of_merge_state(st):
    pieces = resolver({1: "▁ha", 2: "ve", 3: "▁Ha", 7: "▁after"})
    acc = st.IncrementalStitchAccumulator(token_piece=pieces, collect_trace=True)
    first = win(st, 0, 0, 240_000, [ftok(st, 1, 100), ftok(st, 2, 101), ftok(st, 3, 102), ftok(st, 2, 103)])
    second = win(st, 1, 400_000, 640_000, [ftok(st, 7, 320)])
    acc.append(first)
    assert ids(acc.snapshot()) == [1, 2]
    acc.append(second)
    assert acc.snapshot() == st.stitch_token_windows([first, second], pieces)


def test_backward_timestamp_clamped_in_text_order(st):
    acc = st.IncrementalStitchAccumulator(collect_trace=True)
    acc.append(win(st, 0, 0, 240_000, [ftok(st, 10, 158), ftok(st, 20, 160)]))
    acc.append(win(st, 1, 206_080, 446_080, [ftok(st, 20, 159), ftok(st, 30, 159)]))
    snap = acc.snapshot()
    assert ids(snap) == [10, 20, 30]
    assert [t.start_sample for t in snap.tokens] == [202_240, 204_800, 204_800]
    assert snap.tokens[2].end_sample == 206_080 and snap.tokens[2].duration_frames == 1
    acc.append(win(st, 2, 500_000, 740_000, [ftok(st, 40, 400)]))
    assert ids(acc.snapshot()) == [10, 20, 30, 40]
    assert ids(snap) == [10, 20, 30]


def test_rejects_out_of_order_windows(st):
    w = _five_windows(st)
    acc = st.IncrementalStitchAccumulator()
    acc.append(w[1])
    with pytest.raises(ValueError, match="chronological order"):
        acc.append(w[0])
    same = st.IncrementalStitchAccumulator()
    same.append(win(st, 2, 0, 240_000, []))
    with pytest.raises(ValueError, match="chronological order"):
        same.append(win(st, 1, 0, 240_000, []))
    assert st.stitch_token_windows([w[1], w[0]]) == st.stitch_token_windows([w[0], w[1]])


PIECES = {1: "▁ha", 2: "ve", 3: "▁Ha", 4: "▁ei", 5: "ther", 6: "▁Ei", 7: "▁a", 9: ".", 20: "continuation", 21: ","}


def test_splice_safe_classification(st):
    p = resolver(PIECES)
    assert st.is_splice_safe_token(1, p) and st.is_splice_safe_token(21, p)
    assert not st.is_splice_safe_token(20, p)


def test_seam_duplicate_collapse(st):
    p = resolver(PIECES)
    f = lambda seq: [ftok(st, tid, 100 + i) for i, tid in enumerate(seq)]  # noqa: E731
    assert [t.token_id for t in st.collapse_seam_word_duplicates(f([1, 2, 3, 2, 7]), p)] == [1, 2, 7]
    assert [t.token_id for t in st.collapse_seam_word_duplicates(f([6, 5, 4, 5, 7]), p)] == [4, 5, 7]
    assert [t.token_id for t in st.collapse_seam_word_duplicates(f([1, 2, 1, 2]), p)] == [1, 2, 1, 2]
    assert [t.token_id for t in st.collapse_seam_word_duplicates(f([1, 2, 9, 3, 2, 7]), p)] == [1, 2, 9, 3, 2, 7]


def test_clamp_before_duplicate_collapse(st):
    p = resolver(PIECES)
    r = st.stitch_token_windows(pair(st, [ftok(st, 1, 158), ftok(st, 2, 160)],
                                     [ftok(st, 2, 159), ftok(st, 3, 159), ftok(st, 2, 160), ftok(st, 7, 162)]), p)
    assert ids(r) == [1, 2, 7]
    assert [t.start_sample for t in r.tokens] == [202_240, 204_800, 207_360]


def test_globalize_end_aligned_window(st, pk):
    final = pk.windows.plan_stateless_windows(34 * 16_000)[2]
    g = st.globalize_tdt_tokens([st.EmittedToken(1, 80, 1), st.EmittedToken(2, 89, 2)], final)
    assert len(g) == 1
    assert (g[0].token_id, g[0].start_sample, g[0].end_sample) == (2, 419_840, 422_400)


def test_globalize_frame_samples(st, pk):
    w = pk.windows.plan_stateless_windows(384_000)[0]
    g = st.globalize_tdt_tokens([st.EmittedToken(7, 10, 2)], w)
    assert (g[0].start_sample, g[0].end_sample) == (12_800, 15_360)


def test_half_overlap_timestamp_tolerance(st):
    r = st.stitch_token_windows([
        win(st, 0, 0, 240_000, [tok(st, 1, 210_000), tok(st, 2, 220_000)]),
        win(st, 1, 208_000, 448_000, [tok(st, 1, 211_400), tok(st, 2, 221_400)])])
    assert r.trace[0].method == "contiguous"


def test_globalize_arrays_equals_per_token_globalize(st, pk):
    import numpy as np

    rng = np.random.default_rng(7)
    plans = pk.windows.plan_stateless_windows(16_000 * 95 + 1234)
    for plan in plans:
        n = int(rng.integers(0, 400))
        frames = np.sort(rng.integers(0, 188, n)).astype(np.int32)
        ids = rng.integers(0, 1030, n).astype(np.int32)
        durs = rng.integers(0, 5, n).astype(np.int32)
        emitted = [st.EmittedToken(int(a), int(b), int(c)) for a, b, c in zip(ids, frames, durs)]
        assert st.globalize_tdt_arrays(ids, frames, durs, plan) == st.globalize_tdt_tokens(emitted, plan)


def _lcs_plain(m):
    """Textbook LCS table over a boolean match matrix, then the merge's
    backtracking (diagonal on a match; up only when strictly larger)."""
    n, k = len(m), len(m[0]) if m else 0
    table = [[0] * (k + 1) for _ in range(n + 1)]
    for i in range(1, n + 1):
        for j in range(1, k + 1):
            table[i][j] = table[i - 1][j - 1] + 1 if m[i - 1][j - 1] else max(table[i - 1][j], table[i][j - 1])
    out, i, j = [], n, k
    while i > 0 and j > 0:
        if m[i - 1][j - 1]:
            out.append((i - 1, j - 1))
            i, j = i - 1, j - 1
        elif table[i - 1][j] > table[i][j - 1]:
            i -= 1
        else:
            j -= 1
    return out[::-1]


def test_bit_parallel_lcs_equals_textbook_table(st):
    import numpy as np

    rng = np.random.default_rng(3)
    for trial in range(400):
        n, k = int(rng.integers(1, 70)), int(rng.integers(1, 70))
        m = rng.random((n, k)) < (0.04, 0.3, 0.85)[trial % 3]
        assert st._longest_common_subsequence(m) == _lcs_plain(m.tolist()), trial


def test_small_and_large_contiguous_runs_agree(st):
    import numpy as np

    def plain(m):
        n, k = m.shape
        best, at = 0, None
        for i in range(n):  # row-major: the first start of the longest run
            for j in range(k):
                run = 0
                while i + run < n and j + run < k and m[i + run, j + run]:
                    run += 1
                if run > best:
                    best, at = run, (i, j)
        return [] if at is None else [(at[0] + d, at[1] + d) for d in range(best)]

    rng = np.random.default_rng(11)
    for trial in range(300):
        n, k = int(rng.integers(1, 60)), int(rng.integers(1, 60))
        m = rng.random((n, k)) < (0.05, 0.4, 0.9)[trial % 3]
        assert st._longest_contiguous(m) == plain(m), trial


def test_monotonic_clamp_equals_sequential_rule(st):
    import random

    random.seed(4)
    for _ in range(200):
        toks = [st.TimedToken(random.randint(0, 9), s, s + random.randint(0, 3000), 1)
                for s in (random.randint(0, 50_000) for _ in range(random.randint(0, 60)))]
        expect, last = [], None
        for t in toks:
            if last is None or t.start_sample >= last:
                expect.append(t)
                last = t.start_sample
            else:
                expect.append(st.TimedToken(t.token_id, last, t.end_sample + last - t.start_sample,
                                            t.duration_frames))
        assert st.enforce_monotonic_token_times(toks) == expect


def _random_decoded_windows(st, wp, rng):
    """Windows of a random-length plan with random tokens inside each
    emission range: empty, sparse, speech-like and dense windows, some with a
    silent head or tail."""
    import numpy as np

    plans = wp.plan_stateless_windows(int(rng.uniform(20, 300) * 16_000))
    density = rng.choice([0.0, 0.05, 0.3, 1.0, 3.0])
    out = []
    for p in plans:
        lo, hi = p.emission_start_sample, p.emission_end_sample
        n = int(rng.poisson(density * (hi - lo) / 1280))
        if rng.random() < 0.2:
            cut = int(rng.integers(lo, hi))
            starts = np.sort(rng.integers(lo, cut, n) if rng.random() < 0.5 else rng.integers(cut, hi, n))
        else:
            starts = np.sort(rng.integers(lo, hi, n))
        ids = rng.integers(0, int(rng.choice([3, 30, 1024])), n)
        toks = tuple(st.TimedToken(int(a), int(s), int(min(s + 1280 * int(rng.integers(0, 5)), hi)), 1)
                     for a, s in zip(ids, starts))
        out.append(st.DecodedTokenWindow(p.index, lo, hi, toks))
    return out


def test_partial_streams_joined_at_rank_seams_equal_one_fold(st, pk):
    """stitch_partial per contiguous shard + IncrementalStitchAccumulator.extend
    (the multi-rank merge) gives exactly the one-rank merge: tokens and trace."""
    import numpy as np

    wp = pk.windows
    spliced = 0
    for trial in range(120):
        wins = _random_decoded_windows(st, wp, np.random.default_rng(trial))
        ref = st.stitch_token_windows(wins)
        for world in (2, 3, 8):
            acc = st.IncrementalStitchAccumulator(collect_trace=True)
            for r in range(world):
                part = st.stitch_partial([wins[i] for i in wp.shard_windows(len(wins), world, r)])
                spliced += part.local_ok
                acc.extend(part)
            got = acc.snapshot()
            assert got.tokens == ref.tokens and got.trace == ref.trace, (trial, world)
    assert spliced > 100  # the splice path itself is exercised, not only the window-by-window fallback


def test_partial_streams_with_token_pieces_equal_one_fold(st, pk):
    import numpy as np

    vocab = ["\u2581a", "\u2581A", "b", "\u2581c", ",", "\u2581C", "d", "\u2581e", "f"]
    piece = lambda tid: vocab[tid % len(vocab)]  # noqa: E731
    for trial in range(40):
        wins = _random_decoded_windows(st, pk.windows, np.random.default_rng(1000 + trial))
        ref = st.stitch_token_windows(wins, piece)
        for world in (2, 5):
            acc = st.IncrementalStitchAccumulator(token_piece=piece, collect_trace=True)
            for r in range(world):
                acc.extend(st.stitch_partial([wins[i] for i in pk.windows.shard_windows(len(wins), world, r)],
                                             piece))
            got = acc.snapshot()
            assert got.tokens == ref.tokens and got.trace == ref.trace, (trial, world)


def test_partial_stitch_round_trips_windows(st, pk):
    import numpy as np

    wins = _random_decoded_windows(st, pk.windows, np.random.default_rng(5))
    part = st.stitch_partial(wins)
    assert part.windows() == wins
    assert part.window(-1, with_tokens=True) == wins[-1]
    acc = st.IncrementalStitchAccumulator(collect_trace=True)
    acc.extend(part)
    assert acc.snapshot() == st.stitch_token_windows(wins)
