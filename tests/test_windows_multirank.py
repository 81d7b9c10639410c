"""Window planning (chunking.ts) known answers and the multi-rank partition.

Known answers are the reference's own (test/runtime/chunking.test.ts:57-67,
:95-120).  The multi-rank test runs world_size-2 gloo ranks on CPU: every rank
plans the same windows, takes its contiguous shard, and an all_gather proves
the shards tile the plan exactly once with no data-path collective needed.
"""
from __future__ import annotations

import os

import pytest


def test_reference_known_answers(pk):
    w = pk.windows
    plans = w.plan_stateless_windows(58_134_779)
    assert len(plans) == 282
    last = plans[-1]
    assert (last.logical_start_sample, last.logical_end_sample, last.source_start_sample,
            last.source_end_sample, last.timestamp_offset_sample, last.emission_start_sample,
            last.decode_start_frame, last.decode_end_frame) == (
        57_908_480, 58_134_779, 57_896_960, 58_134_779, 57_896_960, 57_908_480, 0, 186)
    full = w.plan_stateless_windows(w.WINDOW_SAMPLES)
    assert [(p.index, p.source_start_sample, p.source_end_sample) for p in full] == [
        (0, 0, w.PRIMARY_VISIBLE_SAMPLES), (1, full[1].source_start_sample, w.WINDOW_SAMPLES)]
    assert full[0].read_sample_count == w.PRIMARY_VISIBLE_SAMPLES
    last34 = w.plan_stateless_windows(34 * 16_000)[-1]
    assert (last34.source_start_sample, last34.source_end_sample, last34.timestamp_offset_sample,
            last34.logical_start_sample, last34.valid_sample_count, last34.decode_end_frame) == (
        305_920, 544_000, 305_920, 412_160, 238_080, 186)
    plans34 = w.plan_stateless_windows(34 * 16_000)
    assert plans34[1].source_start_sample == w.WINDOW_STRIDE_SAMPLES - w.PRIMARY_CONTEXT_SAMPLES
    assert plans34[1].decode_start_frame == 1
    assert plans34[0].logical_end_sample - plans34[1].logical_start_sample == w.OVERLAP_SAMPLES


def test_backfilled_final_window_ends_at_speech(pk):
    total = 34 * 16_000
    speech_end = total - 40 * 1_280
    final = pk.windows.plan_stateless_windows(total, speech_end)[-1]
    assert (final.logical_start_sample, final.logical_end_sample, final.source_end_sample,
            final.decode_start_frame, final.decode_end_frame, final.flush_final) == (
        412_160, speech_end, speech_end, 0, 186, False)


def test_every_length_is_covered(pk):
    w = pk.windows
    for n in (1, 159, 160, 1_280, 238_080, 238_081, 240_000, 1_000_003, 3_600 * 16_000):
        plans = w.plan_stateless_windows(n)
        assert plans[0].logical_start_sample == 0 and plans[-1].logical_end_sample == n
        assert all(p.index == i and p.logical_start_sample == i * w.WINDOW_STRIDE_SAMPLES
                   for i, p in enumerate(plans))
        assert all(0 < p.read_sample_count <= w.WINDOW_SAMPLES for p in plans)
    assert len(w.plan_stateless_windows(3_600 * 16_000)) == 280  # 1 h of audio


@pytest.mark.parametrize("count,world", [(280, 8), (7, 3), (2, 4), (0, 2)])
def test_shards_tile_the_plan(pk, count, world):
    shards = [pk.windows.shard_windows(count, world, r) for r in range(world)]
    flat = [i for s in shards for i in s]
    assert flat == list(range(count))
    sizes = [len(s) for s in shards]
    assert max(sizes) - min(sizes) <= 1
    for s in shards:
        for b in pk.windows.batches(s, 40):
            assert 0 < len(b) <= 40


def _rank_main(rank, world, port, result_path):
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__

    pk = __graft_entry__.load()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    plans = pk.windows.plan_stateless_windows(3_600 * 16_000)
    mine = pk.windows.shard_windows(len(plans), world, rank)
    frames = [plans[i].valid_feature_frames for i in mine]
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, list(mine), frames))
    if rank == 0:
        with open(result_path, "w") as f:
            f.write(repr(gathered))
    dist.destroy_process_group()


def test_two_gloo_ranks_partition_one_hour(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "gathered.txt"
    mp.start_processes(_rank_main, args=(2, port, str(out)), nprocs=2, join=True, start_method="spawn")
    gathered = eval(out.read_text())  # noqa: S307 - written by this test
    indices = [i for _, mine, _ in sorted(gathered) for i in mine]
    assert indices == list(range(280))
    frames = [f for _, _, fr in sorted(gathered) for f in fr]
    assert all(1 <= f <= 1500 for f in frames)
    assert frames[0] == 238_080 // 160 and frames[1] == (238_080 + 1_280) // 160
