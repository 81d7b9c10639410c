"""Host-side merge of independently decoded windows into one token stream.

Restates ``src/runtime/stitch.ts`` (the reference's port of FluidAudio's
ChunkProcessor merge): window-local TDT emissions are placed on the source
timeline (``globalize_tdt_tokens``, stitch.ts:69-99), then consecutive windows
are spliced at their 2 s overlap by the first applicable method -- disjoint
(no overlap), the longest contiguous run of matching tokens, their longest
common subsequence, or a timestamp midpoint (``merge_token_streams``,
:247-343) -- with word-boundary-aware splicing when token pieces are known
(:470-592).  ``snapshot`` clamps timestamps to be non-decreasing
(:209-237) and collapses case-only duplicate words at seams (:641-713).

This is the host half of the multi-GPU design: windows are encoded and
decoded on whichever GPU holds them, and only their token lists meet here.
``PartialStitchBuilder`` and ``IncrementalStitchAccumulator.extend`` have no
reference counterpart (the reference merges on one thread): each rank merges
its own contiguous windows, and rank 0 splices the runs in at the rank seams,
with the same tokens and trace as one merge of every window.

``NativeStitchAccumulator`` / ``NativePartialStitchBuilder`` run the same
merge (streams without word pieces, which is what the engine decodes) in
libpk_b200.so's native implementation (``pk_stitch_*``) on int64 token rows:
no per-token Python objects are built until a caller asks for them.
"""
from __future__ import annotations

import ctypes
import gc
import unicodedata
from contextlib import contextmanager
from itertools import chain
from dataclasses import dataclass
from typing import Callable, NamedTuple, Optional, Sequence

import numpy as np

from . import _lib
from .windows import ENCODER_FRAME_SAMPLES, OVERLAP_SAMPLES, WindowPlan

TokenPieceResolver = Callable[[int], Optional[str]]


class TimedToken(NamedTuple):
    """One token on the source timeline (an immutable record; a named tuple
    because a long-form merge builds hundreds of thousands of them)."""
    token_id: int
    start_sample: int
    end_sample: int
    duration_frames: int  # raw TDT duration (seam-gap repair keeps it)


class EmittedToken(NamedTuple):
    """One decoder emission in window-local encoder frames (TdtEmittedToken)."""
    token_id: int
    frame_index: int
    duration_frames: int


@contextmanager
def _gc_paused():
    """Bulk record construction without the cyclic collector's passes (the
    records hold only ints, so they cannot form cycles)."""
    was_enabled = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was_enabled:
            gc.enable()


@dataclass(frozen=True)
class DecodedTokenWindow:
    index: int
    start_sample: int  # logical emission range, not the physical read range
    end_sample: int
    tokens: tuple


@dataclass(frozen=True)
class StitchTrace:
    left_window_index: int
    right_window_index: int
    method: str  # "disjoint" | "contiguous" | "lcs" | "midpoint"
    overlap_start_sample: int
    overlap_end_sample: int


@dataclass(frozen=True)
class StitchedTokens:
    tokens: tuple
    trace: tuple


def globalize_tdt_tokens(tokens: Sequence[EmittedToken], window: WindowPlan) -> list[TimedToken]:
    """Window-local frames -> source samples (1 280 per encoder frame); tokens
    outside the window's logical emission range (hidden context, an end-aligned
    window's backfill) are dropped and ends clamp to the range."""
    out = []
    for t in tokens:
        start = window.timestamp_offset_sample + t.frame_index * ENCODER_FRAME_SAMPLES
        end = start + t.duration_frames * ENCODER_FRAME_SAMPLES
        if start < window.emission_start_sample or start >= window.emission_end_sample:
            continue
        out.append(TimedToken(t.token_id, start, min(end, window.emission_end_sample), t.duration_frames))
    return out


def globalize_tdt_arrays(token_ids, frames, durations, window: WindowPlan) -> list[TimedToken]:
    """globalize_tdt_tokens on the decoder's output arrays (token ids,
    window-local frames, durations; one entry per emission): the same tokens,
    without building an EmittedToken per emission first."""
    frames = np.asarray(frames, dtype=np.int64)
    durations = np.asarray(durations, dtype=np.int64)
    start = window.timestamp_offset_sample + frames * ENCODER_FRAME_SAMPLES
    end = np.minimum(start + durations * ENCODER_FRAME_SAMPLES, window.emission_end_sample)
    keep = (start >= window.emission_start_sample) & (start < window.emission_end_sample)
    ids = np.asarray(token_ids, dtype=np.int64)[keep].tolist()
    with _gc_paused():
        return list(map(TimedToken._make, zip(ids, start[keep].tolist(), end[keep].tolist(),
                                              durations[keep].tolist())))


def stitch_token_windows(windows: Sequence[DecodedTokenWindow],
                         token_piece: Optional[TokenPieceResolver] = None) -> StitchedTokens:
    ordered = sorted(windows, key=lambda w: (w.start_sample, w.index))
    acc = IncrementalStitchAccumulator(token_piece=token_piece, collect_trace=True)
    for w in ordered:
        acc.append(w)
    return acc.snapshot()


class IncrementalStitchAccumulator:
    """Streaming form of ``stitch_token_windows`` for windows appended in
    (start_sample, index) order; ``snapshot`` finalizes a copy."""

    def __init__(self, token_piece: Optional[TokenPieceResolver] = None, collect_trace: bool = False):
        self._piece = token_piece if token_piece is not None else (lambda _tid: None)
        self._has_pieces = token_piece is not None
        self._trace: Optional[list] = [] if collect_trace else None
        self._merged: list = []
        # start_sample and token_id of every merged token, in list order (the
        # first len(self._merged) entries): the overlap scans of each merge
        # read these arrays instead of the growing token list.
        self._starts = np.zeros(1024, dtype=np.int64)
        self._ids = np.zeros(1024, dtype=np.int64)
        self._previous: Optional[DecodedTokenWindow] = None

    def append(self, window: DecodedTokenWindow) -> None:
        _validate_window(window)
        self._merge_in(window, list(window.tokens))

    def _merge_in(self, window: DecodedTokenWindow, right: list) -> int:
        """Merges `right` -- `window`'s tokens, or a partial stream that
        starts with `window` -- after the previous window; returns the merge's
        keep count (-1 for the first window)."""
        prev = self._previous
        if prev is None:
            self._merged = right
            self._set_starts(0)
            self._previous = window
            return -1
        if (prev.start_sample, prev.index) > (window.start_sample, window.index):
            raise ValueError("incremental stitch windows must be appended in chronological order")
        n = len(self._merged)
        method, keep = _merge_token_streams(self._merged, self._starts[:n], self._ids[:n], right, self._piece,
                                            self._has_pieces)
        self._set_starts(keep)
        if self._trace is not None:
            self._trace.append(StitchTrace(prev.index, window.index, method, window.start_sample,
                                           min(prev.end_sample, window.end_sample)))
        self._previous = window
        return keep

    def extend(self, part: "PartialStitch") -> None:
        """Appends a run of windows that `stitch_partial` merged on its own
        (on another rank, with the same token_piece); the result is exactly
        that of appending the run's windows one by one.  The partial stream is
        spliced in at its first seam when that seam and the run's own merges
        cannot see each other's tokens (checked here and in stitch_partial);
        otherwise the run's windows are appended one by one."""
        count = part.window_meta.shape[0]
        if not count:
            return
        n = len(self._merged)
        # Splicing is exact outright into an empty stream (the run's own fold,
        # or a disjoint join) and for a one-window run (an append); otherwise
        # it needs the locality conditions.
        splice = self._previous is None or n == 0 or count == 1 or (
            part.local_ok and not self._has_pieces
            and int(self._starts[:n].max()) <= part.guard
            and self._merged[-1].start_sample + ENCODER_FRAME_SAMPLES + OVERLAP_SAMPLES <= part.guard + 1)
        if not splice:
            for w in part.windows():
                self.append(w)
            return
        first, last = part.window(0, with_tokens=False), part.window(-1, with_tokens=False)
        self._merge_in(first, part.token_list())
        if self._trace is not None:
            self._trace.extend(part.trace)
        self._previous = last

    def _set_starts(self, keep: int) -> None:
        """Refreshes the start array after a merge left the first `keep`
        merged tokens in place."""
        n = len(self._merged)
        if n > self._starts.shape[0]:
            size = max(n, 2 * self._starts.shape[0])
            for name in ("_starts", "_ids"):
                grown = np.zeros(size, dtype=np.int64)
                grown[:keep] = getattr(self, name)[:keep]
                setattr(self, name, grown)
        tail = _token_rows(self._merged[keep:])
        self._starts[keep:n] = tail[:, 1]
        self._ids[keep:n] = tail[:, 0]

    def snapshot(self) -> StitchedTokens:
        tokens = enforce_monotonic_token_times(self._merged, self._starts[:len(self._merged)])
        if len(tokens) > 1 and self._has_pieces:
            tokens = collapse_seam_word_duplicates(tokens, self._piece)
        return StitchedTokens(tuple(tokens), tuple(self._trace) if self._trace is not None else ())


@dataclass(frozen=True)
class PartialStitch:
    """A contiguous run of decoded windows merged on its own, packed as
    arrays for sending between ranks (see stitch_partial).

    window_meta: int64 [windows, 4] (index, start_sample, end_sample, token
    count); window_tokens / tokens: int64 [n, 4] (token_id, start_sample,
    end_sample, duration_frames) of the windows' own tokens and of the merged
    run; trace: the run's internal StitchTrace entries.  `guard` and
    `local_ok` are the splice conditions of IncrementalStitchAccumulator.extend."""
    window_meta: np.ndarray
    window_tokens: np.ndarray
    tokens: np.ndarray
    trace: tuple
    guard: int
    local_ok: bool

    def token_list(self) -> list:
        with _gc_paused():
            return list(map(TimedToken._make, self.tokens.tolist()))

    def window(self, i: int, with_tokens: bool = True) -> DecodedTokenWindow:
        index, start, end, count = self.window_meta[i].tolist()
        toks = ()
        if with_tokens:
            offset = int(self.window_meta[:i % self.window_meta.shape[0], 3].sum())
            toks = tuple(map(TimedToken._make, self.window_tokens[offset:offset + count].tolist()))
        return DecodedTokenWindow(index, start, end, toks)

    def windows(self) -> list:
        out, offset = [], 0
        with _gc_paused():
            for index, start, end, count in self.window_meta.tolist():
                rows = self.window_tokens[offset:offset + count].tolist()
                out.append(DecodedTokenWindow(index, start, end, tuple(map(TimedToken._make, rows))))
                offset += count
        return out


def _token_rows(tokens, count: Optional[int] = None) -> np.ndarray:
    """int64 [n, 4] rows of TimedTokens (4-field named tuples), read as one
    flat run of ints."""
    n = len(tokens) if count is None else count
    return np.fromiter(chain.from_iterable(tokens), dtype=np.int64, count=4 * n).reshape(n, 4)


class PartialStitchBuilder:
    """Incremental form of stitch_partial: windows are appended in order (as
    their batches finish decoding) and `finish` packs the run."""

    def __init__(self, token_piece: Optional[TokenPieceResolver] = None):
        self._acc = IncrementalStitchAccumulator(token_piece, collect_trace=True)
        self._windows: list = []
        self._ok = token_piece is None
        self._guard = 0
        self._head = 0

    def append(self, window: DecodedTokenWindow) -> None:
        self._acc.append(window)
        self._windows.append(window)
        if len(self._windows) == 2 and self._ok:
            self._guard = window.start_sample - OVERLAP_SAMPLES - ENCODER_FRAME_SAMPLES
            first = self._windows[0].tokens
            self._head = sum(1 for t in first if t.start_sample <= self._guard)
            self._ok = 1 <= self._head < len(first)
        if len(self._windows) > 1 and self._ok and len(self._acc._merged) <= self._head:
            self._ok = False

    def finish(self) -> PartialStitch:
        windows = self._windows
        meta = np.array([(w.index, w.start_sample, w.end_sample, len(w.tokens)) for w in windows],
                        dtype=np.int64).reshape(-1, 4)
        raw = _token_rows(chain.from_iterable(w.tokens for w in windows), int(meta[:, 3].sum()))
        ok = self._ok and len(windows) > 1
        if ok:
            lo, hi = (np.repeat(meta[:, c], meta[:, 3]) for c in (1, 2))
            ok = bool(np.all((lo <= raw[:, 1]) & (raw[:, 1] < hi)))
        return PartialStitch(meta, raw, _token_rows(self._acc._merged), tuple(self._acc._trace),
                             int(self._guard), bool(ok))


def stitch_partial(windows: Sequence[DecodedTokenWindow],
                   token_piece: Optional[TokenPieceResolver] = None) -> PartialStitch:
    """Merges a contiguous, chronological run of windows on its own, for a
    later IncrementalStitchAccumulator.extend.  Splicing the run's merged
    stream in at its first seam gives the same tokens and trace as appending
    its windows one by one when (checked here; `local_ok`):

    * every token lies inside its window's [start_sample, end_sample);
    * with G = (second window's start_sample) - overlap - one frame (`guard`),
      the run's later merges never look at tokens starting at or before G,
      so the first window's tokens up to G -- its first h tokens -- stay
      the run's first h tokens; h >= 1 and the first window has tokens after G;
    * every merge of the run leaves more than h tokens;

    and (checked by extend) the stream it joins starts no token after G and
    its last token's overlap reach ends by G.  Without token pieces only."""
    builder = PartialStitchBuilder(token_piece)
    for w in windows:
        builder.append(w)
    return builder.finish()


def enforce_monotonic_token_times(tokens: Sequence[TimedToken],
                                  starts: Optional[np.ndarray] = None) -> list[TimedToken]:
    """Keep the merged text order; shift any token that starts before its
    predecessor forward by the difference (start and end together).  Each
    token's new start is the running maximum of the starts so far.
    `starts`, when given, holds the tokens' start samples."""
    if not tokens:
        return []
    if starts is None:
        starts = _start_array(tokens)
    clamped = np.maximum.accumulate(starts)
    out = list(tokens)
    with _gc_paused():
        for i in np.flatnonzero(clamped != starts).tolist():
            t = out[i]
            shift = int(clamped[i]) - t.start_sample
            out[i] = TimedToken(t.token_id, t.start_sample + shift, t.end_sample + shift, t.duration_frames)
    return out


def _start_array(tokens) -> np.ndarray:
    return np.fromiter((t.start_sample for t in tokens), dtype=np.int64, count=len(tokens))


def _merge_token_streams(left, left_starts, left_ids, right, piece, has_pieces):
    """Merges `right` (one window's tokens) into the merged stream `left` in
    place; `left_starts` / `left_ids` hold left's start samples and token
    ids.  Returns (method, keep): the first `keep` tokens of the result are
    left's own first `keep`."""
    if not left:
        left.extend(right)
        return "disjoint", 0
    if not right:
        return "disjoint", len(left)
    left_end = left[-1].start_sample + ENCODER_FRAME_SAMPLES
    right_start = right[0].start_sample
    if left_end <= right_start:
        keep = len(left)
        left.extend(right)
        return "disjoint", keep
    right_rows = _token_rows(right)
    ov_left = np.flatnonzero(left_starts + ENCODER_FRAME_SAMPLES > right_start - OVERLAP_SAMPLES)
    ov_right = np.flatnonzero(right_rows[:, 1] < left_end + OVERLAP_SAMPLES)
    if len(ov_left) < 2 or len(ov_right) < 2:
        return "midpoint", _merge_by_midpoint(left, left_starts, right, right_rows[:, 1], left_end, right_start,
                                              piece, has_pieces)

    m = _match_matrix(left_ids[ov_left], left_starts[ov_left], right_rows[ov_right, 0], right_rows[ov_right, 1],
                      piece, has_pieces)
    ov_left, ov_right = ov_left.tolist(), ov_right.tolist()
    run = _longest_contiguous(m)
    if len(run) >= max(len(ov_left) // 2, 1):
        return "contiguous", _merge_using_matches(run, ov_left, ov_right, left, right, piece, has_pieces)
    lcs = _longest_common_subsequence(m)
    if not lcs:
        return "midpoint", _merge_by_midpoint(left, left_starts, right, right_rows[:, 1], left_end, right_start,
                                              piece, has_pieces)
    return "lcs", _merge_using_matches(lcs, ov_left, ov_right, left, right, piece, has_pieces)


def _match_matrix(lid, ls, rid, rs, piece, has_pieces) -> np.ndarray:
    """m[i, j]: overlap tokens i (left: ids `lid`, starts `ls`) and j (right)
    match -- same id (or the same piece ignoring case) and starts less than
    half the overlap apart."""
    same = lid[:, None] == rid[None, :]
    if has_pieces:
        codes: dict = {}

        def code(tid):
            p = piece(tid)
            return -1 if p is None else codes.setdefault(p.lower(), len(codes))

        lc = np.array([code(t) for t in lid.tolist()], dtype=np.int64)
        rc = np.array([code(t) for t in rid.tolist()], dtype=np.int64)
        same |= (lc[:, None] == rc[None, :]) & (lc[:, None] >= 0)
    return same & (np.abs(ls[:, None] - rs[None, :]) * 2 < OVERLAP_SAMPLES)


def _longest_contiguous(m: np.ndarray):
    """The longest diagonal run of matches; among equal lengths the first run
    start in row-major scan order (the reference's scan keeps the first)."""
    n, k = m.shape
    if n * k <= 1024:  # small overlaps: plain lists beat per-row numpy calls
        rows = m.tolist()
        below = [0] * (k + 1)
        best, bi, bj = 0, n, 0
        for i in range(n - 1, -1, -1):
            row, here = rows[i], [0] * (k + 1)
            for j in range(k):
                if row[j]:
                    run = below[j + 1] + 1
                    here[j] = run
                    # rows are visited bottom-up, columns left to right: the
                    # first run start in row-major order wins a tie
                    if run > best or (run == best and i < bi):
                        best, bi, bj = run, i, j
            below = here
        return [(bi + d, bj + d) for d in range(best)]
    runs = np.zeros((n + 1, k + 1), dtype=np.int32)
    hits = m.astype(np.int32)
    for i in range(n - 1, -1, -1):  # in place: run = (run below-right + 1) * match
        row = runs[i, :k]
        np.add(runs[i + 1, 1:], 1, out=row)
        np.multiply(row, hits[i], out=row)
    best = int(runs[:n, :k].max(initial=0))
    if best == 0:
        return []
    flat = int(np.argmax(runs[:n, :k] == best))
    i, j = divmod(flat, k)
    return [(i + d, j + d) for d in range(best)]


def _longest_common_subsequence(m: np.ndarray):
    """LCS of the match matrix with the reference's backtracking tie rule.
    The DP table L is held as one bit row per left token (Hyyro's
    bit-parallel LCS): bit j of row i is set when L(i, j+1) == L(i, j), so
    L(i, j) = j - popcount(row_i & (2^j - 1)); a row follows from the
    previous one in three big-integer operations."""
    n, k = m.shape
    full = (1 << k) - 1
    packed = np.packbits(m, axis=1, bitorder="little")
    rows = [full]
    v = full
    for i in range(n):
        u = v & int.from_bytes(packed[i].tobytes(), "little")
        v = ((v + u) | (v - u)) & full
        rows.append(v)

    def table(i, j):
        return j - (rows[i] & ((1 << j) - 1)).bit_count()

    rev = []
    lc, rc = n, k
    while lc > 0 and rc > 0:
        if m[lc - 1, rc - 1]:
            rev.append((lc - 1, rc - 1))
            lc -= 1
            rc -= 1
        elif table(lc - 1, rc) > table(lc, rc - 1):
            lc -= 1
        else:
            rc -= 1  # backtracking tie rule
    rev.reverse()
    return rev


def _merge_using_matches(pairs, ov_left, ov_right, out, right, piece, has_pieces):
    """Splices `right` into `out` (the merged stream, edited in place) at the
    matched pairs (rows of ov_left / ov_right, the overlap tokens' indices);
    returns how many leading tokens of `out` are unchanged."""
    base = ov_left[pairs[0][0]]
    left = out[base:]  # left[x] below is the stream's token base + x
    del out[base:]
    li = [ov_left[a] - base for a, _ in pairs]
    ri = [ov_right[b] for _, b in pairs]
    keep = base + 1  # the first matched token follows the untouched prefix, unless the seam-word pop cuts into it
    for m in range(len(pairs)):
        out.append(left[li[m]])
        if m == len(pairs) - 1:
            continue
        lgap = left[li[m] + 1:li[m + 1]]
        rgap = right[ri[m] + 1:ri[m + 1]]
        out.extend(rgap if len(rgap) > len(lgap) else lgap)
    last_right = ri[-1]
    if last_right + 1 >= len(right):
        return keep
    tail = right[last_right + 1:]
    if not has_pieces or is_splice_safe_token(tail[0].token_id, piece):
        out.extend(tail)
        return keep
    word_start = _word_initial_index(right, last_right, piece)
    if word_start is not None and _pop_seam_word(out, piece):
        keep = min(keep, len(out))
        out.extend(right[word_start:])
        return keep
    cursor = li[-1] + 1
    while cursor < len(left) and not is_splice_safe_token(left[cursor].token_id, piece):
        out.append(left[cursor])
        cursor += 1
    resume = next((i for i, t in enumerate(tail) if is_splice_safe_token(t.token_id, piece)), -1)
    out.extend(tail[resume:] if resume >= 0 else tail)  # a glued word beats dropping the tail
    return keep


def _word_initial_index(stream, ending_at, piece):
    for i in range(ending_at, -1, -1):
        if is_splice_safe_token(stream[i].token_id, piece):
            return i
    return None


def _pop_seam_word(out, piece) -> bool:
    for i in range(len(out) - 1, -1, -1):
        if is_splice_safe_token(out[i].token_id, piece):
            del out[i:]
            return True
    return False


def _merge_by_midpoint(left, left_starts, right, right_starts, left_end, right_start, piece, has_pieces):
    """Cuts `left` (edited in place) and `right` at the timestamp midpoint of
    their overlap; returns how many leading tokens of `left` are unchanged."""
    cutoff = (left_end + right_start) / 2
    at_or_after = np.flatnonzero(left_starts >= cutoff)
    le = int(at_or_after[0]) if at_or_after.size else len(left)
    at_or_after = np.flatnonzero(right_starts >= cutoff)
    rs = int(at_or_after[0]) if at_or_after.size else len(right)
    if has_pieces and le > 0:
        while le < len(left) and not is_splice_safe_token(left[le].token_id, piece):
            le += 1
    if has_pieces:
        safe = rs
        while safe < len(right) and not is_splice_safe_token(right[safe].token_id, piece):
            safe += 1
        if safe < len(right):  # keep the original cutoff when no safe right token exists
            rs = safe
    del left[le:]
    left.extend(right[rs:])
    return le


def _is_punct_or_symbol(ch: str) -> bool:
    return unicodedata.category(ch)[0] in ("P", "S")


def _starts_word(piece: str) -> bool:
    return piece.startswith("▁") or piece.startswith(" ")


def is_splice_safe_token(token_id: int, piece: TokenPieceResolver) -> bool:
    p = piece(token_id)
    if not p:
        return False
    return _starts_word(p) or all(_is_punct_or_symbol(c) for c in p)


def is_punctuation_only_token(token_id: int, piece: TokenPieceResolver) -> bool:
    p = piece(token_id)
    return bool(p) and all(_is_punct_or_symbol(c) for c in p)


def token_ids_match(a: int, b: int, piece: TokenPieceResolver) -> bool:
    if a == b:
        return True
    pa, pb = piece(a), piece(b)
    return pa is not None and pb is not None and pa.lower() == pb.lower()


def collapse_seam_word_duplicates(tokens: Sequence[TimedToken], piece: TokenPieceResolver) -> list[TimedToken]:
    """Drop one of two adjacent words that differ only in case and start within
    the overlap of each other (keeping the lowercase form when it comes
    second), unless the first ends a sentence."""
    if len(tokens) < 2:
        return list(tokens)
    words = []
    for t in tokens:
        p = piece(t.token_id) or ""
        if not words or _starts_word(p):
            words.append({"tokens": [t], "start": t.start_sample})
        else:
            words[-1]["tokens"].append(t)
    for w in words:
        text = "".join(_strip_prefix(piece(t.token_id) or "") for t in w["tokens"])
        core = text
        while core and (unicodedata.category(core[0])[0] == "P" or core[0].isspace()):
            core = core[1:]
        while core and (unicodedata.category(core[-1])[0] == "P" or core[-1].isspace()):
            core = core[:-1]
        w["core"] = core
        w["ends"] = text.endswith((".", "?", "!", ":"))
    keep = [True] * len(words)
    last = -1
    for i, cur in enumerate(words):
        if last < 0:
            last = i
            continue
        prev = words[last]
        dup = (prev["core"] and cur["core"] and prev["core"] != cur["core"]
               and prev["core"].lower() == cur["core"].lower()
               and unicodedata.category(cur["core"][0])[0] == "L" and not prev["ends"]
               and cur["start"] - prev["start"] <= OVERLAP_SAMPLES)
        if not dup:
            last = i
            continue
        if cur["core"] == cur["core"].lower() and prev["core"] != prev["core"].lower():
            keep[last] = False
            last = i
        else:
            keep[i] = False
    out = []
    for i, w in enumerate(words):
        if keep[i]:
            out.extend(w["tokens"])
    return out


def _strip_prefix(p: str) -> str:
    return p[1:] if _starts_word(p) else p


def _validate_window(w: DecodedTokenWindow) -> None:
    for name, v in (("window index", w.index), ("window startSample", w.start_sample),
                    ("window endSample", w.end_sample)):
        if not isinstance(v, int) or v < 0:
            raise ValueError(f"{name} must be a non-negative safe integer")
    if w.end_sample < w.start_sample:
        raise ValueError("window endSample must not precede startSample")
    prev = -1
    for t in w.tokens:
        a, start, end, dur = t.token_id, t.start_sample, t.end_sample, t.duration_frames
        # Fast path: plain ints in order; anything else takes the full check.
        if not (type(a) is int and type(start) is int and type(end) is int and type(dur) is int
                and a >= 0 and dur >= 0 and prev <= start <= end):
            _check_token(t, prev)
        prev = start


def _check_token(t: TimedToken, prev: int) -> None:
    for name, v in (("tokenId", t.token_id), ("token startSample", t.start_sample),
                    ("token endSample", t.end_sample), ("token durationFrames", t.duration_frames)):
        if not isinstance(v, int) or v < 0:
            raise ValueError(f"{name} must be a non-negative safe integer")
    if t.end_sample < t.start_sample:
        raise ValueError("token endSample must not precede startSample")
    if t.start_sample < prev:
        raise ValueError("tokens must be sorted by startSample")


# ------------------------------------------------------------------ native merge

STITCH_METHODS = ("disjoint", "contiguous", "lcs", "midpoint")


class StitchedTokenArrays:
    """StitchedTokens held as arrays: ``token_rows`` int64 [n, 4] (token_id,
    start_sample, end_sample, duration_frames; monotonic clamp applied) and
    ``trace_rows`` int64 [m, 5].  ``tokens`` / ``trace`` build the record
    tuples on first use; equality compares those with any StitchedTokens."""

    def __init__(self, token_rows: np.ndarray, trace_rows: np.ndarray):
        self.token_rows = token_rows
        self.trace_rows = trace_rows
        self._tokens = None
        self._trace = None

    @property
    def tokens(self) -> tuple:
        if self._tokens is None:
            with _gc_paused():
                self._tokens = tuple(map(TimedToken._make, self.token_rows.tolist()))
        return self._tokens

    @property
    def trace(self) -> tuple:
        if self._trace is None:
            self._trace = _trace_records(self.trace_rows)
        return self._trace

    def __len__(self) -> int:
        return int(self.token_rows.shape[0])

    def __eq__(self, other) -> bool:
        return self.tokens == other.tokens and self.trace == other.trace


def _trace_records(rows: np.ndarray) -> tuple:
    return tuple(StitchTrace(int(a), int(b), STITCH_METHODS[int(m)], int(s0), int(s1))
                 for a, b, m, s0, s1 in rows.tolist())


def _trace_rows(trace) -> np.ndarray:
    if isinstance(trace, np.ndarray):
        return np.ascontiguousarray(trace, dtype=np.int64).reshape(-1, 5)
    return np.array([(t.left_window_index, t.right_window_index, STITCH_METHODS.index(t.method),
                      t.overlap_start_sample, t.overlap_end_sample) for t in trace], dtype=np.int64).reshape(-1, 5)


def _vp(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a.size else None


class NativeStitchAccumulator:
    """IncrementalStitchAccumulator for streams without word pieces, on the
    native merge (pk_stitch_*): the same tokens, trace and errors."""

    def __init__(self, collect_trace: bool = False, record_run: bool = False):
        flags = (_lib.STITCH_COLLECT_TRACE if collect_trace else 0) | (_lib.STITCH_RECORD_RUN if record_run else 0)
        handle = ctypes.c_void_p()
        self._call("pk_stitch_create", flags, ctypes.byref(handle))
        self._h = handle

    @staticmethod
    def _call(name, *args) -> None:
        try:
            _lib.call(name, *args)
        except _lib.PkError as exc:
            if exc.status == -1:  # PK_E_INVALID: the reference's RangeError
                raise ValueError(str(exc).split(": ", 1)[-1]) from None
            raise

    def append(self, window: DecodedTokenWindow) -> None:
        rows = _token_rows(window.tokens) if window.tokens else np.zeros((0, 4), np.int64)
        self.append_rows(window.index, window.start_sample, window.end_sample, rows)

    def append_rows(self, index: int, start_sample: int, end_sample: int, rows: np.ndarray) -> None:
        win = np.array([index, start_sample, end_sample], dtype=np.int64)
        rows = np.ascontiguousarray(rows, dtype=np.int64).reshape(-1, 4)
        self._call("pk_stitch_append", self._h, _vp(win), _vp(rows), rows.shape[0])

    def append_tdt(self, plan: WindowPlan, token_ids, frames, durations) -> None:
        """Globalizes one window's decoder output (token ids, window-local
        encoder frames, durations) and appends it."""
        win = np.array([plan.index, plan.emission_start_sample, plan.emission_end_sample,
                        plan.timestamp_offset_sample], dtype=np.int64)
        arrs = [np.ascontiguousarray(a, dtype=np.int32) for a in (token_ids, frames, durations)]
        self._call("pk_stitch_append_tdt", self._h, _vp(win), *[_vp(a) for a in arrs], arrs[0].shape[0])

    def extend(self, part: "PartialStitch") -> None:
        """IncrementalStitchAccumulator.extend: splices a run merged on its
        own (on another rank) in at its first seam where that is exact."""
        meta = np.ascontiguousarray(part.window_meta, dtype=np.int64)
        raw = np.ascontiguousarray(part.window_tokens, dtype=np.int64)
        merged = np.ascontiguousarray(part.tokens, dtype=np.int64)
        trace = _trace_rows(part.trace)
        run = _lib.StitchRun(_vp(meta), meta.shape[0], _vp(raw), _vp(merged), merged.shape[0], _vp(trace),
                             trace.shape[0], int(part.guard), int(bool(part.local_ok)))
        self._call("pk_stitch_extend", self._h, ctypes.byref(run))

    def counts(self) -> tuple:
        c = np.zeros(4, np.int64)
        self._call("pk_stitch_counts", self._h, _vp(c))
        return tuple(int(v) for v in c)

    def _read(self, clamp: bool):
        n, t, _, _ = self.counts()
        tokens = np.zeros((n, 4), np.int64)
        trace = np.zeros((t, 5), np.int64)
        self._call("pk_stitch_read", self._h, int(clamp), _vp(tokens), _vp(trace))
        return tokens, trace

    def snapshot(self) -> StitchedTokenArrays:
        return StitchedTokenArrays(*self._read(True))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().pk_stitch_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


class NativePartialStitchBuilder:
    """PartialStitchBuilder on the native merge (no word pieces): windows are
    appended in order and ``finish`` packs the run with its splice
    conditions."""

    def __init__(self):
        self._acc = NativeStitchAccumulator(collect_trace=True, record_run=True)

    def append(self, window: DecodedTokenWindow) -> None:
        self._acc.append(window)

    def append_tdt(self, plan: WindowPlan, token_ids, frames, durations) -> None:
        self._acc.append_tdt(plan, token_ids, frames, durations)

    def finish(self) -> "PartialStitch":
        merged, trace = self._acc._read(False)
        _, _, windows, raw_count = self._acc.counts()
        meta = np.zeros((windows, 4), np.int64)
        raw = np.zeros((raw_count, 4), np.int64)
        cond = np.zeros(2, np.int64)
        self._acc._call("pk_stitch_read_run", self._acc._h, _vp(meta), _vp(raw), _vp(cond))
        self._acc.close()
        return PartialStitch(meta, raw, merged, _trace_records(trace), int(cond[0]), bool(cond[1]))


# Flat int64 form of a rank's result, for a gather of plain arrays:
# ok:    [0, windows, raw tokens, merged tokens, trace entries, guard, local_ok]
#        + window_meta + window_tokens + tokens + trace (row-major);
# error: [1, message bytes] + the UTF-8 message, zero-padded to 8 bytes.
def pack_partial(part: "PartialStitch") -> np.ndarray:
    trace = _trace_rows(part.trace)
    head = np.array([0, part.window_meta.shape[0], part.window_tokens.shape[0], part.tokens.shape[0],
                     trace.shape[0], part.guard, int(part.local_ok)], dtype=np.int64)
    return np.concatenate([head, np.asarray(part.window_meta, np.int64).ravel(),
                           np.asarray(part.window_tokens, np.int64).ravel(),
                           np.asarray(part.tokens, np.int64).ravel(), trace.ravel()])


def pack_error(message: str) -> np.ndarray:
    raw = message.encode()
    padded = raw + b"\0" * (-len(raw) % 8)
    return np.concatenate([np.array([1, len(raw)], np.int64), np.frombuffer(padded, dtype=np.int64)])


def unpack_partial(flat: np.ndarray):
    """("ok", PartialStitch) or ("error", message) from pack_partial / pack_error."""
    flat = np.asarray(flat, dtype=np.int64)
    if int(flat[0]) == 1:
        n = int(flat[1])
        return "error", flat[2:].tobytes()[:n].decode(errors="replace")
    w, nw, n, t, guard, ok = (int(v) for v in flat[1:7])
    sizes = (4 * w, 4 * nw, 4 * n, 5 * t)
    parts, off = [], 7
    for size in sizes:
        parts.append(flat[off:off + size])
        off += size
    meta, raw, merged, trace = (p.reshape(-1, c) for p, c in zip(parts, (4, 4, 4, 5)))
    return "ok", PartialStitch(meta, raw, merged, _trace_records(trace), guard, bool(ok))
