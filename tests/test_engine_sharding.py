"""Sharded long-form transcription on the host (engine.transcribe_sharded):
world_size-2 gloo ranks on CPU, each decoding its contiguous share of the
window plan with a deterministic stand-in engine; rank 0's merge equals the
single-rank merge.  Failure detection, made on the host: a rank whose engine
returns an injected PK_E_TIMEOUT, and a rank that exits before the gather --
rank 0 reports ShardFailure and no process hangs.  The GPU engine itself is
covered by test_gpu_engine.py; the device side of a timeout by
test_gpu_fault.py."""
from __future__ import annotations

import os

import numpy as np


class FakeEngine:
    """decode_plans without a GPU: three tokens per window, two in its overlap."""

    def __init__(self, pk):
        self.pk = pk

    def decode_plans(self, pcm, plans, stream=None, on_window=None, on_tdt=None):
        st = self.pk.stitch
        out = []
        for p in plans:
            ids, frames, durs = np.array([100 + p.index, 7, 8]), np.array([5, 150, 170]), np.array([1, 2, 1])
            if on_tdt is not None:
                on_tdt(p, ids, frames, durs)
                continue
            toks = [st.EmittedToken(int(a), int(f), int(d)) for a, f, d in zip(ids, frames, durs)]
            g = st.globalize_tdt_tokens(toks, p)
            out.append(st.DecodedTokenWindow(p.index, p.emission_start_sample, p.emission_end_sample, tuple(g)))
            if on_window is not None:
                on_window(out[-1])
        return out


def _rank(rank, world, port, result_path):
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pk = __graft_entry__.load()
    pcm = np.zeros(16_000 * 100, np.float32)
    timings = {}
    res = pk.engine.transcribe_sharded(FakeEngine(pk), pcm, rank, world, pk.engine.array_gather(rank, world),
                                       timings=timings)
    assert set(timings) == {"decode_s", "gather_s", "merge_s"}
    if rank == 0:
        with open(result_path, "w") as f:
            f.write(repr([(t.token_id, t.start_sample) for t in res.tokens]))
    dist.destroy_process_group()


def test_two_rank_merge_equals_single_rank(pk, tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "merged.txt"
    mp.start_processes(_rank, args=(2, port, str(out)), nprocs=2, join=True, start_method="spawn")
    got = eval(out.read_text())  # noqa: S307 - written by this test
    pcm = np.zeros(16_000 * 100, np.float32)
    single = pk.engine.transcribe_sharded(FakeEngine(pk), pcm, 0, 1, lambda obj: [obj])
    plans = pk.windows.plan_stateless_windows(len(pcm))
    sequential = pk.stitch.stitch_token_windows(FakeEngine(pk).decode_plans(pcm, plans))
    assert got == [(t.token_id, t.start_sample) for t in single.tokens]
    assert single.tokens == sequential.tokens and single.trace == sequential.trace
    assert len(got) > 0


class FailingEngine(FakeEngine):
    """decode_plans that fails the way a bounded device wait reports it."""

    def decode_plans(self, pcm, plans, stream=None, on_window=None, on_tdt=None):
        raise self.pk.PkError(-7, "injected: a bounded device wait expired (status bits 0x1)")


def _failing_rank(rank, world, port, out_dir, mode):
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    pk = __graft_entry__.load()
    outcome = "returned"
    if mode == "exits" and rank == 1:
        outcome = "left"  # leaves between steps: nothing of this rank is in flight
    else:
        engine = FailingEngine(pk) if (mode == "raises" and rank == 1) else FakeEngine(pk)
        try:
            pk.engine.transcribe_sharded(engine, np.zeros(16_000 * 100, np.float32), rank, world,
                                         pk.engine.array_gather(rank, world))
        except Exception as exc:  # recorded for the test
            outcome = f"{type(exc).__name__}|{exc}"
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(outcome)
    if outcome == "returned":
        dist.destroy_process_group()


def _run_ranks(tmp_path, mode, deadline_s=60.0):
    import socket
    import time

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.start_processes(_failing_rank, args=(2, port, str(tmp_path), mode), nprocs=2, join=False,
                             start_method="spawn")
    t0 = time.monotonic()
    while not ctx.join(timeout=1.0):
        if time.monotonic() - t0 > deadline_s:
            for p in ctx.processes:
                p.kill()
            raise AssertionError(f"ranks still running after {deadline_s} s ({mode})")
    return [(tmp_path / f"rank{r}.txt").read_text() for r in range(2)], time.monotonic() - t0


def test_rank_with_injected_timeout_is_reported_on_rank0(tmp_path):
    (r0, r1), _ = _run_ranks(tmp_path, "raises")
    kind, msg = r0.split("|", 1)
    assert kind == "ShardFailure"
    assert msg.startswith("rank 1: PkError: PK_E_TIMEOUT: injected"), msg
    assert r1.startswith("PkError|PK_E_TIMEOUT")


def test_rank_that_exits_before_the_gather_is_detected(tmp_path):
    (r0, r1), elapsed = _run_ranks(tmp_path, "exits")
    assert r1 == "left"
    assert r0.startswith("ShardFailure|gather: "), r0
    assert elapsed < 60.0


def test_shard_failure_message_orders_ranks_then_gather(pk):
    err = pk.engine.ShardFailure({3: "B", None: "C", 1: "A"})
    assert str(err) == "rank 1: A; rank 3: B; gather: C"


def test_decode_into_streams_in_merge_order(pk):
    """engine._decode_into hands windows to the merge as batches finish when
    the plan is in (emission start, index) order, and sorts them first when
    it is not; both give the one-shot merge."""
    pcm = np.zeros(16_000 * 100, np.float32)
    plans = pk.windows.plan_stateless_windows(len(pcm))
    fake = FakeEngine(pk)
    expect = pk.stitch.stitch_token_windows(fake.decode_plans(pcm, plans))
    for order in (plans, list(reversed(plans))):
        seen = []
        acc = pk.stitch.IncrementalStitchAccumulator(collect_trace=True)

        def sink(w, seen=seen, acc=acc):
            seen.append(w.index)
            acc.append(w)

        pk.engine._decode_into(fake, pcm, order, sink)
        assert seen == sorted(seen)
        got = acc.snapshot()
        assert got.tokens == expect.tokens and got.trace == expect.trace


def test_decode_into_native_sink_equals_python_merge(pk):
    """The native accumulator fed the decoder's arrays (on_tdt) merges as the
    Python accumulator fed globalized windows, in and out of plan order."""
    pcm = np.zeros(16_000 * 100, np.float32)
    plans = pk.windows.plan_stateless_windows(len(pcm))
    fake = FakeEngine(pk)
    expect = pk.stitch.stitch_token_windows(fake.decode_plans(pcm, plans))
    for order in (plans, list(reversed(plans))):
        acc = pk.stitch.NativeStitchAccumulator(collect_trace=True)
        pk.engine._decode_into(fake, pcm, order, acc)
        assert acc.snapshot() == expect


def test_batches_are_balanced(pk):
    eng = object.__new__(pk.engine.ParakeetEngine)
    eng.capacity = 32
    assert [len(r) for r in eng.batches(35)] == [18, 17]
    assert [len(r) for r in eng.batches(280)] == [31, 31, 31, 31, 32, 31, 31, 31, 31]
    assert [len(r) for r in eng.batches(32)] == [32]
    assert eng.batches(0) == []
    eng.capacity = 40
    assert [len(r) for r in eng.batches(35)] == [35]
    assert [len(r) for r in eng.batches(280)] == [40] * 7
