"""Inference engine: PCM windows in, decoded tokens out, on one GPU.

Mirrors the engine seam the reference's worker runtime calls
(``ParakeetInferenceEngine``, src/runtime/worker.ts:114-153) as implemented
by ``createRawWebGpuParakeetEngine(...).transcribeWindows``
(src/runtime/webgpu-engine.ts:578-880): per batch of at most ``capacity``
windows the PCM arena is copied in, the log-mel front end, the 24-layer
encoder graph and the persistent TDT decoder run back to back on one stream,
and the token lists come back to the host.  ``transcribe`` adds the
reference's long-form flow around it: the stateless window plan
(src/runtime/chunking.ts:174-302), batching, timestamp globalization and the
overlap merge (src/runtime/stitch.ts).  ``transcribe_sharded`` splits the
window plan across ranks (one GPU each); only the token lists travel to rank
0, which merges them -- the hot path has no collective.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from . import stitch as st
from . import windows as wp
from .encoder import ModelWeights, ParakeetEncoderGraph, derive_encoder_valid_length
from .kernels import (Device, GpuTensor, ParakeetFbank, PersistentTdtDecoderKernel, RangeError,
                      TDT_DECODER_TENSORS)

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

WINDOW_SAMPLES = wp.WINDOW_SAMPLES
MAX_TOKENS_PER_WINDOW = 2048  # src/runtime/webgpu-engine.ts:84
BATCH_CAPACITY = 40  # windows per batch, the reference's encoder capacity (src/webgpu/encoder.ts:68)


@dataclass(frozen=True)
class WindowResult:
    """EngineWindowResult: one window's emissions in window-local frames."""
    tokens: tuple  # of stitch.EmittedToken
    overflow: bool


class ParakeetEngine:
    def __init__(self, device: Device, package: dict, precision: str = "fp16", capacity: int = BATCH_CAPACITY,
                 max_tokens: int = MAX_TOKENS_PER_WINDOW, keep_intermediates: bool = False):
        """package: encoder + decoder tensors (name -> record), as produced by
        the reference converter or ``synthetic.make_package`` + ``make_decoder``."""
        self.device, self.precision, self.capacity, self.max_tokens = device, precision, capacity, max_tokens
        dec_names = set(TDT_DECODER_TENSORS)
        missing = sorted(dec_names - set(package))
        if missing:
            raise RangeError(f"package lacks decoder tensors: {', '.join(missing)}")
        self.weights = ModelWeights(device, {k: v for k, v in package.items() if k not in dec_names})
        self.graph = ParakeetEncoderGraph.create(device, self.weights, precision, capacity)
        cuda = f"cuda:{device.ordinal}"
        self._decoder_tensors = {n: GpuTensor.from_record(n, package[n], cuda) for n in dec_names}
        self.decoder = PersistentTdtDecoderKernel.create(device, None, self._decoder_tensors, precision)
        self.fbank = ParakeetFbank(device)
        i32 = dict(dtype=torch.int32, device=cuda)
        self._pcm = torch.zeros((capacity, WINDOW_SAMPLES), dtype=torch.float32, device=cuda)
        self._control = torch.zeros((5, capacity), **i32)
        self._features = torch.zeros((capacity, 128, 1501), dtype=torch.float32, device=cuda)
        self._tokens = torch.zeros((3, capacity, max_tokens), **i32)
        self._meta = torch.zeros(2 * capacity, **i32)
        # Two pinned host slots: while the GPU runs one batch, the host stages
        # the next batch's PCM in the other (decode_plans pipelines batches).
        # Control rows: valid samples, encoder lengths, decode starts, decode
        # ends, flush flags.
        self._slots = [dict(
            pcm=torch.zeros((capacity, WINDOW_SAMPLES), dtype=torch.float32).pin_memory(),
            control=torch.zeros((5, capacity), dtype=torch.int32).pin_memory(),
            tokens=torch.zeros((3, capacity, max_tokens), dtype=torch.int32).pin_memory(),
            meta=torch.zeros(2 * capacity, dtype=torch.int32).pin_memory(),
            done=torch.cuda.Event()) for _ in range(2)]
        for slot in self._slots:
            slot["pcm_np"] = slot["pcm"].numpy()
        self._copy_pool = ThreadPoolExecutor(max_workers=_staging_threads())
        self._dispatch = self.decoder.create_dispatch(dict(
            encoder_projected=self.graph.decoder_input(), encoded_lengths=self._control[1],
            decode_starts=self._control[2], decode_ends=self._control[3], flush_finals=self._control[4],
            tokens=self._tokens[0], token_frames=self._tokens[1], token_durations=self._tokens[2],
            metadata=self._meta, batch_size=capacity, frames=188, max_tokens=max_tokens))
        self.keep_intermediates = keep_intermediates
        self.last: dict = {}

    def transcribe_windows(self, windows: Sequence[tuple], stream=None) -> list[WindowResult]:
        """windows: (samples f32 [<= 240 000], WindowPlan) per window, 1..capacity."""
        out = []
        for tok, fr, du, overflow in self._run_batch(windows, stream):
            out.append(WindowResult(tuple(map(st.EmittedToken._make, zip(tok.tolist(), fr.tolist(), du.tolist()))),
                                    overflow))
        return out

    def _run_batch(self, windows: Sequence[tuple], stream=None) -> list:
        """One batch through log-mel, encoder and decoder; per window its
        (token ids, frames, durations) arrays and overflow flag."""
        out = self._collect(self._submit(windows, stream, 0))
        self._check_status()
        return out

    def _check_status(self) -> None:
        """Raises PkError(PK_E_TIMEOUT) when a bounded device wait of this
        device expired since the last check (the kernel that gave up returned
        early, so its batch's tokens are not valid).  Called once no batch is
        in flight: reading the status word clears it."""
        self.device.status()

    def _submit(self, windows: Sequence[tuple], stream, slot: int, decode: bool = True):
        """Stages a batch in host slot `slot` and queues its copies and
        kernels on `stream` without waiting for them (without the decoder
        and the token read-back when `decode` is False)."""
        b = len(windows)
        if not 0 < b <= self.capacity:
            raise RangeError(f"Engine batch must contain 1-{self.capacity} windows")
        stream = torch.cuda.current_stream() if stream is None else stream
        host = self._slots[slot]
        pcm, ctrl = host["pcm"], host["control"]
        arena = host["pcm_np"]
        lengths = []
        copies = []
        for i, (samples, plan) in enumerate(windows):
            samples = np.asarray(samples, dtype=np.float32)
            if samples.ndim != 1 or samples.shape[0] > WINDOW_SAMPLES or plan.valid_sample_count > samples.shape[0]:
                raise RangeError(f"Window {i} must hold its {plan.valid_sample_count} valid samples in at most "
                                 f"{WINDOW_SAMPLES}")
            copies.append((i, samples))
            feature_frames = max(1, plan.valid_sample_count // wp.HOP_SAMPLES)
            enc_len = derive_encoder_valid_length(feature_frames)
            if plan.decode_start_frame > enc_len:
                raise RangeError(f"Window {i} decoder start exceeds its {enc_len} encoder frames")
            lengths.append(feature_frames)
            ctrl[0, i] = plan.valid_sample_count
            ctrl[1, i] = enc_len
            ctrl[2, i] = plan.decode_start_frame
            ctrl[3, i] = plan.decode_end_frame
            ctrl[4, i] = int(plan.flush_final)
        # The PCM copies into the pinned slot run on a few host threads (numpy
        # releases the GIL while copying): at one batch per rank they are not
        # hidden behind a previous batch's GPU work.
        list(self._copy_pool.map(lambda job: _stage_window(arena, *job), copies))
        with torch.cuda.stream(stream):
            self._pcm[:b].copy_(pcm[:b], non_blocking=True)
            self._control.copy_(ctrl, non_blocking=True)
            self.fbank.compute_batch(self._pcm[:b], self._control[0, :b], out=self._features[:b], stream=stream)
            projected, _ = self.graph.encode(self._features[:b], lengths, stream=stream)
            if decode:
                self._dispatch.encode(stream, active_batch_size=b)
                host["tokens"][:, :b].copy_(self._tokens[:, :b], non_blocking=True)
                host["meta"].copy_(self._meta, non_blocking=True)
            host["done"].record(stream)
        if self.keep_intermediates:
            stream.synchronize()
            self.last = {"features": self._features[:b].cpu().numpy(),
                         "projected": projected.view(b, 188, 640).cpu().numpy(),
                         "encoded_lengths": ctrl[1, :b].numpy().copy()}
        return slot, b

    def _collect(self, ticket) -> list:
        """Waits for a submitted batch and reads its tokens from its slot."""
        slot, b = ticket
        host = self._slots[slot]
        host["done"].synchronize()
        tok, fr, du = (host["tokens"][k, :b].numpy() for k in range(3))
        counts = host["meta"][:b].numpy()
        flags = host["meta"][self.capacity:self.capacity + b].numpy()
        out = []
        for i in range(b):
            n = min(int(counts[i]), self.max_tokens)
            out.append((tok[i, :n].copy(), fr[i, :n].copy(), du[i, :n].copy(), bool(flags[i] & 1)))
        return out

    def batches(self, count: int, limit: int | None = None) -> list[range]:
        """Splits `count` windows into the fewest batches of at most
        `limit` (default: capacity) windows, as equal in size as possible (35
        windows at capacity 32 run as 18 + 17, not 32 + 3: a decoder batch
        costs about as much as its longest window, whatever its size)."""
        cap = min(self.capacity, limit or self.capacity)
        n = -(-count // cap) if count else 0
        edges = [round(k * count / n) for k in range(n + 1)] if n else [0]
        return [range(a, b) for a, b in zip(edges, edges[1:])]

    def decode_plans(self, pcm: np.ndarray, plans: Sequence[wp.WindowPlan], stream=None, on_window=None,
                     on_tdt=None) -> list:
        """Runs `plans` in balanced batches of at most `capacity` windows;
        returns a DecodedTokenWindow per plan.  Batches are pipelined: batch
        i+1 is staged on the host and queued while the GPU runs batch i, and
        batch i's tokens are read, globalized and handed to `on_window` (in
        plan order; a merge, for instance) while batch i+1 runs.  With
        `on_tdt`, each window's raw decoder output (plan, token ids, frames,
        durations) goes to `on_tdt` instead and nothing is returned (no
        per-token Python objects are built)."""
        decoded = []

        def finish(chunk, ticket):
            for plan, (tok, fr, du, _) in zip(chunk, self._collect(ticket)):
                if on_tdt is not None:
                    on_tdt(plan, tok, fr, du)
                    continue
                toks = st.globalize_tdt_arrays(tok, fr, du, plan)
                window = st.DecodedTokenWindow(plan.index, plan.emission_start_sample, plan.emission_end_sample,
                                               tuple(toks))
                decoded.append(window)
                if on_window is not None:
                    on_window(window)

        pending = None
        for k, rows in enumerate(self.batches(len(plans))):
            chunk = plans[rows.start:rows.stop]
            batch = [(pcm[p.source_start_sample:p.source_end_sample], p) for p in chunk]
            ticket = self._submit(batch, stream, k % 2)
            if pending is not None:
                finish(*pending)
            pending = (chunk, ticket)
        if pending is not None:
            finish(*pending)
        self._check_status()
        return decoded

    def encode_plans(self, pcm: np.ndarray, plans: Sequence[wp.WindowPlan], stream=None,
                     batch: int | None = None) -> int:
        """Log-mel front end and encoder only, for `plans` in balanced
        batches of at most `batch` (default: capacity) windows with the same
        two-slot pipelining as decode_plans; each batch's projected encoder
        output is left on the device (where the decoder would read it).
        Returns the number of windows encoded."""
        pending = None
        for k, rows in enumerate(self.batches(len(plans), batch)):
            chunk = plans[rows.start:rows.stop]
            ticket = self._submit([(pcm[p.source_start_sample:p.source_end_sample], p) for p in chunk], stream,
                                  k % 2, decode=False)
            if pending is not None:
                self._slots[pending[0]]["done"].synchronize()
            pending = ticket
        if pending is not None:
            self._slots[pending[0]]["done"].synchronize()
        self._check_status()
        return len(plans)

    def transcribe(self, pcm: np.ndarray, token_piece=None, stream=None):
        """Long-form transcription of 16 kHz mono f32 PCM on this GPU; returns
        StitchedTokens (StitchedTokenArrays from the native merge when no
        token pieces are given)."""
        pcm = np.ascontiguousarray(pcm, dtype=np.float32)
        plans = wp.plan_stateless_windows(int(pcm.shape[0]))
        acc = _accumulator(token_piece)
        _decode_into(self, pcm, plans, acc, stream)
        return acc.snapshot()

    def destroy(self) -> None:
        self._copy_pool.shutdown(wait=True)
        self.graph.destroy()
        self.weights.release()


def _staging_threads() -> int:
    """Host threads for staging PCM: the cores this process may use, shared
    among the ranks of this node (LOCAL_WORLD_SIZE), at most 8."""
    import os

    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        cores = os.cpu_count() or 1
    ranks = int(os.environ.get("LOCAL_WORLD_SIZE", "1") or 1)
    return max(1, min(8, cores // max(1, ranks)))


def _stage_window(arena: np.ndarray, i: int, samples: np.ndarray) -> None:
    n = samples.shape[0]
    np.copyto(arena[i, :n], samples)
    if n < WINDOW_SAMPLES:
        arena[i, n:] = 0.0


def _accumulator(token_piece):
    """The merge: native (no word pieces) or the Python restatement (pieces)."""
    if token_piece is None:
        return st.NativeStitchAccumulator(collect_trace=True)
    return st.IncrementalStitchAccumulator(token_piece=token_piece, collect_trace=True)


def _decode_into(engine, pcm, plans, sink, stream=None) -> None:
    """Decodes `plans` and feeds each window to `sink` (an accumulator, a
    partial-run builder, or a function of a DecodedTokenWindow) in the
    merge's (emission start, index) order -- as each batch finishes, while
    the GPU runs the next one, when the plan is already in that order.
    Sinks with ``append_tdt`` take the decoder's arrays directly."""
    keys = [(p.emission_start_sample, p.index) for p in plans]
    ordered = all(a <= b for a, b in zip(keys, keys[1:]))
    if hasattr(sink, "append_tdt"):
        if ordered:
            engine.decode_plans(pcm, plans, stream, on_tdt=sink.append_tdt)
            return
        out = []
        engine.decode_plans(pcm, plans, stream, on_tdt=lambda *w: out.append(w))
        for w in sorted(out, key=lambda w: (w[0].emission_start_sample, w[0].index)):
            sink.append_tdt(*w)
        return
    append = sink.append if hasattr(sink, "append") else sink
    if ordered:
        engine.decode_plans(pcm, plans, stream, on_window=append)
        return
    for w in sorted(engine.decode_plans(pcm, plans, stream), key=lambda w: (w.start_sample, w.index)):
        append(w)


class ShardFailure(RuntimeError):
    """A sharded transcription failed on one or more ranks, or its gather did.
    ``failures`` maps each failed rank to its error ("ErrorType: message");
    a failed gather (a rank that left, a collective that timed out) has the
    key None."""

    def __init__(self, failures: dict):
        self.failures = dict(failures)
        super().__init__("; ".join(("gather" if r is None else f"rank {r}") + f": {m}"
                                   for r, m in sorted(self.failures.items(), key=lambda kv: (kv[0] is None, kv[0]))))


def transcribe_sharded(engine, pcm: np.ndarray, rank: int, world_size: int, gather, token_piece=None,
                       timings: dict | None = None):
    """Multi-GPU long-form transcription: this rank decodes its contiguous
    share of the window plan with its own `engine` (its own GPU) and merges
    its own windows as they finish decoding (a partial run); `gather(array)`
    brings every rank's run, packed as one flat int64 array
    (stitch.pack_partial), to rank 0 (see ``array_gather``), which joins
    them at the rank seams (extend -- the same tokens and trace as merging
    every window on one rank).  Returns the merged tokens on rank 0 and None
    elsewhere.  With world_size 1 it is ``engine.transcribe`` (no gather;
    errors propagate as they are).  `timings`, when given, receives this
    rank's host wall time per phase: decode_s (decode and the rank's own
    merge, overlapped), gather_s, merge_s (rank 0: joining the runs and the
    snapshot).

    Failures do not hang the other ranks: a rank whose decode raises (a
    PkError such as PK_E_TIMEOUT from a bounded device wait, a RangeError)
    still takes the gather step, carrying its error instead of its windows,
    and then re-raises; rank 0 raises ShardFailure naming every failed rank.
    A gather that itself fails (a rank that exited, a process-group timeout)
    raises ShardFailure on the ranks that see it."""
    import time

    clock = time.perf_counter
    t0 = clock()
    pcm = np.ascontiguousarray(pcm, dtype=np.float32)
    plans = wp.plan_stateless_windows(int(pcm.shape[0]))
    if world_size == 1:
        acc = _accumulator(token_piece)
        _decode_into(engine, pcm, plans, acc)
        t1 = clock()
        out = acc.snapshot()
        if timings is not None:
            timings.update(decode_s=t1 - t0, gather_s=0.0, merge_s=clock() - t1)
        return out
    mine = [plans[i] for i in wp.shard_windows(len(plans), world_size, rank)]
    error = None
    try:
        builder = st.NativePartialStitchBuilder() if token_piece is None else st.PartialStitchBuilder(token_piece)
        if mine:
            _decode_into(engine, pcm, mine, builder)
        payload = st.pack_partial(builder.finish())
    except Exception as exc:  # reported through the gather, re-raised below
        error = exc
        payload = st.pack_error(f"{type(exc).__name__}: {exc}")
    t1 = clock()
    try:
        gathered = gather(payload)
    except Exception as exc:
        raise ShardFailure({None: f"{type(exc).__name__}: {exc}"}) from exc
    t2 = clock()
    if timings is not None:
        timings.update(decode_s=t1 - t0, gather_s=t2 - t1, merge_s=0.0)
    if rank != 0:
        if error is not None:
            raise error
        return None
    parts = [st.unpack_partial(flat) for flat in gathered]
    failures = {r: part[1] for r, part in enumerate(parts) if part[0] != "ok"}
    if failures:
        raise ShardFailure(failures) from error
    acc = _accumulator(token_piece)
    for _, part in parts:  # rank order is window order: the shards are contiguous
        acc.extend(part)
    out = acc.snapshot()
    if timings is not None:
        timings["merge_s"] = clock() - t2
    return out


def array_gather(rank: int, world_size: int, device=None):
    """A `gather` for transcribe_sharded over torch.distributed: every rank's
    flat int64 array reaches rank 0 as plain tensors -- the lengths first,
    then one padded all-gather (the communicator's collective channels; a
    point-to-point gather would set up peer connections on first use).  NCCL
    tensors on `device`, CPU tensors for gloo.  Returns a list of arrays on
    rank 0 and None elsewhere."""
    import torch.distributed as dist

    def gather(flat: np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(flat, dtype=np.int64))
        if device is not None:
            t = t.to(device, non_blocking=False)
        n = torch.tensor([t.numel()], dtype=torch.int64, device=t.device)
        sizes = torch.zeros(world_size, dtype=torch.int64, device=t.device)
        dist.all_gather_into_tensor(sizes, n)
        sizes = sizes.tolist()
        width = max(sizes)
        padded = torch.zeros(width, dtype=torch.int64, device=t.device)
        padded[:t.numel()] = t
        everything = torch.empty(world_size * width, dtype=torch.int64, device=t.device)
        dist.all_gather_into_tensor(everything, padded)
        if rank != 0:
            return None
        host = everything.cpu().numpy()
        return [host[r * width:r * width + k] for r, k in enumerate(sizes)]

    return gather
