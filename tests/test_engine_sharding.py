"""Sharded long-form transcription on the host (engine.transcribe_sharded):
world_size-2 gloo ranks on CPU, each decoding its contiguous share of the
window plan with a deterministic stand-in engine; rank 0's merge equals the
single-rank merge.  The GPU engine itself is covered by test_gpu_engine.py."""
from __future__ import annotations

import os

import numpy as np


class FakeEngine:
    """decode_plans without a GPU: three tokens per window, two in its overlap."""

    def __init__(self, pk):
        self.pk = pk

    def decode_plans(self, pcm, plans, stream=None):
        st = self.pk.stitch
        out = []
        for p in plans:
            toks = [st.EmittedToken(100 + p.index, 5, 1), st.EmittedToken(7, 150, 2), st.EmittedToken(8, 170, 1)]
            g = st.globalize_tdt_tokens(toks, p)
            out.append(st.DecodedTokenWindow(p.index, p.emission_start_sample, p.emission_end_sample, tuple(g)))
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

    def gather(obj):
        parts = [None] * world if rank == 0 else None
        dist.gather_object(obj, parts, dst=0)
        return parts

    res = pk.engine.transcribe_sharded(FakeEngine(pk), pcm, rank, world, gather)
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
    assert got == [(t.token_id, t.start_sample) for t in single.tokens]
    assert len(got) > 0
