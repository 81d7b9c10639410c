// stitch.cpp -- native overlap merge of independently decoded windows.
//
// Host code (no GPU): the long-form merge the engine runs while the GPU decodes
// the next batch, and the per-rank partial merges of sharded transcription.
// It restates the reference's merge for token streams without word pieces
// (src/runtime/stitch.ts, itself a port of FluidAudio's ChunkProcessor):
//   * IncrementalStitchAccumulator.append / snapshot (stitch.ts:135-213);
//   * mergeTokenStreams (:247-359): disjoint, longest contiguous run of
//     matches, longest common subsequence, timestamp midpoint, in that order;
//   * longestContiguousMatches (:372-405): first run in row-major scan order
//     wins a tie;  longestCommonSubsequence (:407-461) with its backtracking
//     tie rule;  mergeUsingMatches (:463-520, the no-piece branch);
//     mergeByMidpoint (:568-606, no pieces);
//   * enforceMonotonicTokenTimes (:230-262).
// Word-piece-aware splicing needs the tokenizer's pieces and stays in the
// Python module; every merge here is the no-piece form.
//
// Layout: a token is 4 int64 (token_id, start_sample, end_sample,
// duration_frames); a trace entry 5 int64 (left window index, right window
// index, method 0 disjoint / 1 contiguous / 2 lcs / 3 midpoint, overlap start
// sample, overlap end sample); a window 3 int64 (index, start_sample,
// end_sample) -- its logical emission range.
//
// Beyond the reference (which merges on one thread): a pk_stitch created with
// PK_STITCH_RECORD_RUN keeps the windows it merged and the splice conditions
// of its run, and pk_stitch_extend joins such a run -- merged on another rank
// -- at its first seam.  The result equals appending the run's windows one by
// one; the conditions under which the splice is exact are checked on both
// sides (see pk_stitch_extend).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

#include "pk_internal.h"

namespace {

constexpr int64_t kFrame = 1280;    // PARAKEET_ENCODER_FRAME_SAMPLES (8 x 160-sample hops)
constexpr int64_t kOverlap = 32000; // PARAKEET_OVERLAP_SAMPLES (2 s at 16 kHz)

struct Tok {
  int64_t id, start, end, dur;
};
struct Win {
  int64_t index, start, end;
};
struct Trace {
  int64_t left, right, method, ov_start, ov_end;
};

enum { kDisjoint = 0, kContiguous = 1, kLcs = 2, kMidpoint = 3 };

}  // namespace

struct pk_stitch {
  bool collect_trace = false;
  bool record_run = false;
  std::vector<Tok> merged;
  std::vector<int64_t> pmax;  // pmax[i] = max start_sample of merged[0..i]
  bool has_prev = false;
  Win prev{};
  std::vector<Trace> trace;
  // Run record (PK_STITCH_RECORD_RUN): the windows and their own tokens, and
  // the splice conditions (guard, head count, locality).
  std::vector<Win> windows;
  std::vector<int64_t> window_counts;
  std::vector<Tok> window_tokens;
  bool run_ok = true;
  int64_t guard = 0, head = 0;
  // scratch
  std::vector<int64_t> ovl, ovr, order, mrow, mcols, run, stamp;
  std::vector<uint64_t> bits, lcs;
  std::vector<std::pair<int64_t, int64_t>> pairs, rowbuf;
  std::vector<Tok> tail, globalized;
};

namespace {

using pk::set_error;

int validate_window(const Win& w, const Tok* t, int64_t n) {
  if (w.index < 0) return set_error(PK_E_INVALID, "window index must be a non-negative safe integer");
  if (w.start < 0) return set_error(PK_E_INVALID, "window startSample must be a non-negative safe integer");
  if (w.end < 0) return set_error(PK_E_INVALID, "window endSample must be a non-negative safe integer");
  if (w.end < w.start) return set_error(PK_E_INVALID, "window endSample must not precede startSample");
  int64_t prev = -1;
  for (int64_t i = 0; i < n; ++i) {
    if (t[i].id < 0) return set_error(PK_E_INVALID, "tokenId must be a non-negative safe integer");
    if (t[i].start < 0) return set_error(PK_E_INVALID, "token startSample must be a non-negative safe integer");
    if (t[i].end < 0) return set_error(PK_E_INVALID, "token endSample must be a non-negative safe integer");
    if (t[i].dur < 0) return set_error(PK_E_INVALID, "token durationFrames must be a non-negative safe integer");
    if (t[i].end < t[i].start) return set_error(PK_E_INVALID, "token endSample must not precede startSample");
    if (t[i].start < prev) return set_error(PK_E_INVALID, "tokens must be sorted by startSample");
    prev = t[i].start;
  }
  return PK_OK;
}

void refresh_pmax(pk_stitch* s, int64_t from) {
  const int64_t n = (int64_t)s->merged.size();
  s->pmax.resize(n);
  int64_t m = from > 0 ? s->pmax[from - 1] : INT64_MIN;
  for (int64_t i = from; i < n; ++i) {
    m = std::max(m, s->merged[i].start);
    s->pmax[i] = m;
  }
}

// First index i with merged[i].start > thr (== first i with pmax[i] > thr).
int64_t first_start_above(const pk_stitch* s, int64_t thr) {
  return std::upper_bound(s->pmax.begin(), s->pmax.end(), thr) - s->pmax.begin();
}

// mergeByMidpoint without pieces: cut both streams at the overlap's timestamp
// midpoint (left_end + right_start) / 2; returns the kept prefix of `merged`.
int64_t merge_midpoint(pk_stitch* s, const Tok* right, int64_t nr, int64_t left_end, int64_t right_start) {
  // start >= (left_end + right_start) / 2  <=>  start >= ceil_half (integers)
  const int64_t ceil_half = (left_end + right_start + 1) / 2;
  const int64_t cut = first_start_above(s, ceil_half - 1);
  int64_t rs = 0;
  while (rs < nr && right[rs].start < ceil_half) ++rs;
  s->merged.resize(cut);
  s->merged.insert(s->merged.end(), right + rs, right + nr);
  return cut;
}

// mergeUsingMatches without pieces; pairs index ovl / ovr.  Returns the kept
// prefix of `merged`.
int64_t merge_matches(pk_stitch* s, const Tok* right, int64_t nr) {
  const auto& pairs = s->pairs;
  const int64_t base = s->ovl[pairs[0].first];
  s->tail.assign(s->merged.begin() + base, s->merged.end());  // left[base:]
  s->merged.resize(base);
  const size_t np = pairs.size();
  for (size_t m = 0; m < np; ++m) {
    const int64_t li = s->ovl[pairs[m].first] - base, ri = s->ovr[pairs[m].second];
    s->merged.push_back(s->tail[li]);
    if (m + 1 == np) continue;
    const int64_t li2 = s->ovl[pairs[m + 1].first] - base, ri2 = s->ovr[pairs[m + 1].second];
    const int64_t lgap = li2 - li - 1, rgap = ri2 - ri - 1;
    if (rgap > lgap)
      s->merged.insert(s->merged.end(), right + ri + 1, right + ri2);
    else
      s->merged.insert(s->merged.end(), s->tail.begin() + li + 1, s->tail.begin() + li2);
  }
  const int64_t last_right = s->ovr[pairs[np - 1].second];
  if (last_right + 1 < nr) s->merged.insert(s->merged.end(), right + last_right + 1, right + nr);
  return base + 1;
}

// mergeTokenStreams without pieces; `merged` is edited in place.  Returns the
// method and sets *keep to the number of leading tokens left unchanged.
int merge_streams(pk_stitch* s, const Tok* right, int64_t nr, int64_t* keep) {
  auto& left = s->merged;
  const int64_t nl = (int64_t)left.size();
  if (nl == 0) {
    left.assign(right, right + nr);
    *keep = 0;
    return kDisjoint;
  }
  if (nr == 0) {
    *keep = nl;
    return kDisjoint;
  }
  const int64_t left_end = left[nl - 1].start + kFrame;
  const int64_t right_start = right[0].start;
  if (left_end <= right_start) {
    left.insert(left.end(), right, right + nr);
    *keep = nl;
    return kDisjoint;
  }
  // Overlap tokens: left starts with start + frame > right_start - overlap,
  // right starts with start < left_end + overlap (every index, in order).
  const int64_t thr = right_start - kOverlap - kFrame;
  s->ovl.clear();
  for (int64_t i = first_start_above(s, thr); i < nl; ++i)
    if (left[i].start > thr) s->ovl.push_back(i);
  s->ovr.clear();
  for (int64_t j = 0; j < nr; ++j)
    if (right[j].start < left_end + kOverlap) s->ovr.push_back(j);
  const int64_t a = (int64_t)s->ovl.size(), b = (int64_t)s->ovr.size();
  if (a < 2 || b < 2) {
    *keep = merge_midpoint(s, right, nr, left_end, right_start);
    return kMidpoint;
  }
  // Matches: same token id, starts less than half the overlap apart.  Held
  // sparsely -- per left overlap token its matching right overlap tokens, in
  // increasing order (s->mcols, row i at mrow[i]..mrow[i+1]) -- and as one bit
  // row per left token (s->bits, `words` 64-bit words) for the LCS.
  s->order.resize(b);
  for (int64_t j = 0; j < b; ++j) s->order[j] = j;
  std::sort(s->order.begin(), s->order.end(), [&](int64_t x, int64_t y) {
    const int64_t ix = right[s->ovr[x]].id, iy = right[s->ovr[y]].id;
    return ix != iy ? ix < iy : x < y;
  });
  const int64_t words = (b + 63) / 64;
  s->bits.assign((size_t)a * words, 0);
  s->mrow.assign(a + 1, 0);
  s->mcols.clear();
  for (int64_t i = 0; i < a; ++i) {
    const Tok& l = left[s->ovl[i]];
    auto lo = std::lower_bound(s->order.begin(), s->order.end(), l.id,
                               [&](int64_t x, int64_t id) { return right[s->ovr[x]].id < id; });
    for (auto it = lo; it != s->order.end() && right[s->ovr[*it]].id == l.id; ++it) {
      const int64_t d = l.start - right[s->ovr[*it]].start;
      if ((d < 0 ? -d : d) * 2 < kOverlap) {
        s->mcols.push_back(*it);
        s->bits[(size_t)i * words + (*it >> 6)] |= 1ull << (*it & 63);
      }
    }
    s->mrow[i + 1] = (int64_t)s->mcols.size();
  }
  auto match = [&](int64_t i, int64_t j) { return (s->bits[(size_t)i * words + (j >> 6)] >> (j & 63)) & 1; };
  // Longest diagonal run; the first run start in row-major order wins ties.
  // run(i, j) = match(i, j) ? run(i + 1, j + 1) + 1 : 0, rows bottom-up; a
  // row's runs live in `run` with `stamp` naming the row they belong to.
  s->run.assign(b + 1, 0);
  s->stamp.assign(b + 1, -1);
  int64_t best = 0, bi = a, bj = 0;
  for (int64_t i = a - 1; i >= 0; --i) {
    // Row i's runs read row i+1's at j+1 > j: walk j upwards, writing as we go
    // into a small buffer, then publish (row i+1's entries stay readable).
    s->rowbuf.clear();
    for (int64_t k = s->mrow[i]; k < s->mrow[i + 1]; ++k) {
      const int64_t j = s->mcols[k];
      const int64_t below = s->stamp[j + 1] == i + 1 ? s->run[j + 1] : 0;
      const int64_t r = below + 1;
      s->rowbuf.emplace_back(j, r);
      if (r > best || (r == best && i < bi)) {
        best = r;
        bi = i;
        bj = j;
      }
    }
    for (const auto& jr : s->rowbuf) {
      s->run[jr.first] = jr.second;
      s->stamp[jr.first] = i;
    }
  }
  s->pairs.clear();
  if (best >= std::max<int64_t>(a / 2, 1)) {
    for (int64_t d = 0; d < best; ++d) s->pairs.emplace_back(bi + d, bj + d);
    *keep = merge_matches(s, right, nr);
    return kContiguous;
  }
  if (best == 0) {  // no match at all: the LCS is empty
    *keep = merge_midpoint(s, right, nr, left_end, right_start);
    return kMidpoint;
  }
  // Longest common subsequence by the bit-parallel recurrence (Hyyro): bit j
  // of row i is set when L(i, j+1) == L(i, j), so L(i, j) = j - popcount of
  // row i's bits below j; row i+1 = (v + u) | (v - u), u = v & match row i,
  // as multi-word integers.  Then the reference's backtrack.
  s->lcs.assign((size_t)(a + 1) * words, ~0ull);
  const uint64_t top = (b & 63) ? (1ull << (b & 63)) - 1 : ~0ull;
  s->lcs[words - 1] = top;
  for (int64_t i = 0; i < a; ++i) {
    const uint64_t* v = &s->lcs[(size_t)i * words];
    const uint64_t* m = &s->bits[(size_t)i * words];
    uint64_t* nx = &s->lcs[(size_t)(i + 1) * words];
    unsigned char carry = 0, borrow = 0;
    for (int64_t k = 0; k < words; ++k) {
      const uint64_t u = v[k] & m[k];
      const uint64_t sum = v[k] + u + carry;
      carry = (sum < v[k] || (carry && sum == v[k])) ? 1 : 0;
      const uint64_t diff = v[k] - u - borrow;
      borrow = (v[k] < u || (borrow && v[k] == u)) ? 1 : 0;
      nx[k] = sum | diff;
    }
    nx[words - 1] &= top;
  }
  auto table = [&](int64_t i, int64_t j) {
    const uint64_t* row = &s->lcs[(size_t)i * words];
    int64_t zeros = 0;
    for (int64_t k = 0; k < (j >> 6); ++k) zeros += __builtin_popcountll(row[k]);
    if (j & 63) zeros += __builtin_popcountll(row[j >> 6] & ((1ull << (j & 63)) - 1));
    return j - zeros;
  };
  int64_t lc = a, rc = b;
  while (lc > 0 && rc > 0) {
    if (match(lc - 1, rc - 1)) {
      s->pairs.emplace_back(lc - 1, rc - 1);
      --lc;
      --rc;
    } else if (table(lc - 1, rc) > table(lc, rc - 1)) {
      --lc;
    } else {
      --rc;  // backtracking tie rule
    }
  }
  std::reverse(s->pairs.begin(), s->pairs.end());
  *keep = merge_matches(s, right, nr);
  return kLcs;
}

// Merges `right` -- window w's tokens, or a run's merged stream that starts
// with window w -- after the previous window.
int merge_in(pk_stitch* s, const Win& w, const Tok* right, int64_t nr) {
  if (!s->has_prev) {
    s->merged.assign(right, right + nr);
    refresh_pmax(s, 0);
    s->has_prev = true;
    s->prev = w;
    return PK_OK;
  }
  if (s->prev.start > w.start || (s->prev.start == w.start && s->prev.index > w.index))
    return set_error(PK_E_INVALID, "incremental stitch windows must be appended in chronological order");
  int64_t keep = 0;
  const int method = merge_streams(s, right, nr, &keep);
  refresh_pmax(s, std::min<int64_t>(keep, (int64_t)s->merged.size()));
  if (s->collect_trace) s->trace.push_back({s->prev.index, w.index, method, w.start, std::min(s->prev.end, w.end)});
  s->prev = w;
  return PK_OK;
}

// One window appended (validated); updates the run record.
int append_window(pk_stitch* s, const Win& w, const Tok* t, int64_t n) {
  int st = validate_window(w, t, n);
  if (st) return st;
  if ((st = merge_in(s, w, t, n))) return st;
  if (s->record_run) {
    s->windows.push_back(w);
    s->window_counts.push_back(n);
    s->window_tokens.insert(s->window_tokens.end(), t, t + n);
    // Splice conditions of the run (see pk_stitch_extend): with G = second
    // window's start - overlap - one frame, the first window holds h >= 1
    // tokens at or before G and at least one after it, and every later merge
    // leaves more than h tokens.
    if (s->windows.size() == 2 && s->run_ok) {
      s->guard = w.start - kOverlap - kFrame;
      const int64_t n0 = s->window_counts[0];
      int64_t h = 0;
      for (int64_t i = 0; i < n0; ++i) h += s->window_tokens[i].start <= s->guard;
      s->head = h;
      s->run_ok = h >= 1 && h < n0;
    }
    if (s->windows.size() > 1 && s->run_ok && (int64_t)s->merged.size() <= s->head) s->run_ok = false;
  }
  return PK_OK;
}

}  // namespace

extern "C" {

int pk_stitch_create(int flags, pk_stitch** out) {
  if (!out) return set_error(PK_E_INVALID, "null argument");
  if (flags & ~(PK_STITCH_COLLECT_TRACE | PK_STITCH_RECORD_RUN)) return set_error(PK_E_INVALID, "unknown stitch flags");
  auto* s = new (std::nothrow) pk_stitch();
  if (!s) return set_error(PK_E_OOM, "stitch accumulator allocation failed");
  s->collect_trace = flags & PK_STITCH_COLLECT_TRACE;
  s->record_run = flags & PK_STITCH_RECORD_RUN;
  *out = s;
  return PK_OK;
}

int pk_stitch_destroy(pk_stitch* s) {
  delete s;
  return PK_OK;
}

int pk_stitch_append(pk_stitch* s, const int64_t* window, const int64_t* tokens, int64_t count) {
  if (!s || !window || (count > 0 && !tokens) || count < 0) return set_error(PK_E_INVALID, "null argument");
  const Win w{window[0], window[1], window[2]};
  return append_window(s, w, reinterpret_cast<const Tok*>(tokens), count);
}

int pk_stitch_append_tdt(pk_stitch* s, const int64_t* window, const int32_t* token_ids, const int32_t* frames,
                         const int32_t* durations, int64_t count) {
  if (!s || !window || count < 0 || (count > 0 && (!token_ids || !frames || !durations)))
    return set_error(PK_E_INVALID, "null argument");
  const Win w{window[0], window[1], window[2]};
  const int64_t offset = window[3];
  // globalizeTdtTokens (stitch.ts:69-99): local encoder frames -> source
  // samples; emissions outside the logical range are dropped, ends clamp.
  std::vector<Tok>& buf = s->globalized;
  buf.clear();
  buf.reserve((size_t)count);
  for (int64_t i = 0; i < count; ++i) {
    const int64_t start = offset + (int64_t)frames[i] * kFrame;
    if (start < w.start || start >= w.end) continue;
    const int64_t end = std::min(start + (int64_t)durations[i] * kFrame, w.end);
    buf.push_back({(int64_t)token_ids[i], start, end, (int64_t)durations[i]});
  }
  return append_window(s, w, buf.data(), (int64_t)buf.size());
}

int pk_stitch_extend(pk_stitch* s, const pk_stitch_run* run) {
  if (!s || !run || run->windows < 0 || run->tokens < 0 || run->trace_entries < 0)
    return set_error(PK_E_INVALID, "null argument");
  if (run->windows == 0) return PK_OK;
  const auto* meta = run->window_meta;  // [windows, 4]: index, start, end, token count
  const Tok* wt = reinterpret_cast<const Tok*>(run->window_tokens);
  const int64_t nl = (int64_t)s->merged.size();
  // Splicing is exact outright into an empty stream and for a one-window run;
  // otherwise the run's own conditions (local_ok, guard) must hold and the
  // stream it joins may start no token after G, its last token's overlap
  // reach ending by G.
  bool splice = !s->has_prev || nl == 0 || run->windows == 1;
  if (!splice && run->local_ok) {
    splice = s->pmax[nl - 1] <= run->guard && s->merged[nl - 1].start + kFrame + kOverlap <= run->guard + 1;
  }
  if (!splice) {
    int64_t off = 0;
    for (int64_t i = 0; i < run->windows; ++i) {
      const Win w{meta[4 * i], meta[4 * i + 1], meta[4 * i + 2]};
      const int st = append_window(s, w, wt + off, meta[4 * i + 3]);
      if (st) return st;
      off += meta[4 * i + 3];
    }
    return PK_OK;
  }
  const Win first{meta[0], meta[1], meta[2]};
  const int64_t L = run->windows - 1;
  const Win last{meta[4 * L], meta[4 * L + 1], meta[4 * L + 2]};
  int st = merge_in(s, first, reinterpret_cast<const Tok*>(run->merged), run->tokens);
  if (st) return st;
  if (s->collect_trace) {
    const auto* tr = reinterpret_cast<const Trace*>(run->trace);
    s->trace.insert(s->trace.end(), tr, tr + run->trace_entries);
  }
  s->prev = last;
  return PK_OK;
}

int pk_stitch_counts(const pk_stitch* s, int64_t* counts) {
  if (!s || !counts) return set_error(PK_E_INVALID, "null argument");
  counts[0] = (int64_t)s->merged.size();
  counts[1] = (int64_t)s->trace.size();
  counts[2] = (int64_t)s->windows.size();
  counts[3] = (int64_t)s->window_tokens.size();
  return PK_OK;
}

int pk_stitch_read(const pk_stitch* s, int clamp, int64_t* tokens, int64_t* trace) {
  if (!s) return set_error(PK_E_INVALID, "null argument");
  if (tokens) {
    Tok* out = reinterpret_cast<Tok*>(tokens);
    int64_t last = INT64_MIN;
    for (size_t i = 0; i < s->merged.size(); ++i) {
      Tok t = s->merged[i];
      if (clamp && i > 0 && t.start < last) {  // enforceMonotonicTokenTimes
        const int64_t shift = last - t.start;
        t.start += shift;
        t.end += shift;
      }
      last = t.start;
      out[i] = t;
    }
  }
  if (trace && !s->trace.empty()) std::memcpy(trace, s->trace.data(), s->trace.size() * sizeof(Trace));
  return PK_OK;
}

int pk_stitch_read_run(const pk_stitch* s, int64_t* window_meta, int64_t* window_tokens, int64_t* conditions) {
  if (!s || !s->record_run) return set_error(PK_E_INVALID, "stitch accumulator does not record its run");
  if (window_meta)
    for (size_t i = 0; i < s->windows.size(); ++i) {
      window_meta[4 * i] = s->windows[i].index;
      window_meta[4 * i + 1] = s->windows[i].start;
      window_meta[4 * i + 2] = s->windows[i].end;
      window_meta[4 * i + 3] = s->window_counts[i];
    }
  if (window_tokens && !s->window_tokens.empty())
    std::memcpy(window_tokens, s->window_tokens.data(), s->window_tokens.size() * sizeof(Tok));
  if (conditions) {
    bool ok = s->run_ok && s->windows.size() > 1;
    if (ok) {  // every token inside its window's range
      size_t off = 0;
      for (size_t i = 0; i < s->windows.size() && ok; ++i) {
        for (int64_t k = 0; k < s->window_counts[i]; ++k) {
          const int64_t st = s->window_tokens[off + k].start;
          if (st < s->windows[i].start || st >= s->windows[i].end) {
            ok = false;
            break;
          }
        }
        off += (size_t)s->window_counts[i];
      }
    }
    conditions[0] = s->guard;
    conditions[1] = ok ? 1 : 0;
  }
  return PK_OK;
}

}  // extern "C"
