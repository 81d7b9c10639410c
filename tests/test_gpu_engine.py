"""The single-GPU engine (engine.ParakeetEngine: log-mel -> encoder ->
TDT decoder per batch, then globalization and the overlap merge) against the
oracle, stage by stage on the same inputs:

* front end: features within the log-mel bar of test_gpu_logmel.py;
* encoder: the GPU's projected output within 2e-2 relative Frobenius of the
  oracle's wide-accumulation encoder run on the GPU's features;
* decoder + merge: the oracle decoder run on the GPU encoder's own output,
  globalized and stitched, gives exactly the engine's tokens.

Synthetic 16 kHz audio (pink noise + modulated tones) and random-init
weights stand in for recordings and a checkpoint."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_engine_matches_oracle_stage_by_stage(pk, oracle, device, precision):
    dtype = np.float16 if precision == "fp16" else np.float32
    package = pk.synthetic.make_package(precision, seed=0)
    decoder = pk.synthetic.make_decoder(precision, seed=0)
    package.update(decoder)
    eng = pk.engine.ParakeetEngine(device, package, precision, capacity=4, keep_intermediates=True)
    try:
        pcm = pk.synthetic.make_pcm(20.0, seed=3)
        result = eng.transcribe(pcm)
        plans = pk.windows.plan_stateless_windows(len(pcm))
        assert len(plans) == 2 and len(eng.last["features"]) == 2
        arena = np.zeros((2, 240_000), np.float32)
        valid = np.array([p.valid_sample_count for p in plans], np.uint32)
        for i, p in enumerate(plans):
            arena[i, : p.read_sample_count] = pcm[p.source_start_sample:p.source_end_sample]
        feats = eng.last["features"]
        ref_feats = oracle.logmel(arena, valid)
        assert np.mean(feats.view(np.uint32) == ref_feats.view(np.uint32)) >= 0.9999
        assert np.abs(feats - ref_feats).max() <= 1e-5

        lengths = [max(1, int(v) // 160) for v in valid]
        proj = eng.last["projected"]
        ref_proj, ref_lens = oracle.encoder(package, feats, lengths, dtype, acc_mode=1)
        err = oracle.rel_frobenius(proj.reshape(-1, 640), ref_proj)
        print(f"engine {precision}: encoder rel-Frobenius {err:.2e} vs wide oracle")
        assert err < 2e-2
        assert list(eng.last["encoded_lengths"]) == [int(v) for v in ref_lens]

        dec = {n: r["data"] for n, r in decoder.items()}
        tok, fr, du, cnt, flags = oracle.tdt_decode(
            proj.astype(dtype), eng.last["encoded_lengths"], dec, max_tokens=eng.max_tokens,
            starts=[p.decode_start_frame for p in plans], ends=[p.decode_end_frame for p in plans],
            flush=[int(p.flush_final) for p in plans])
        st = pk.stitch
        windows = []
        for i, p in enumerate(plans):
            emitted = [st.EmittedToken(int(tok[i, j]), int(fr[i, j]), int(du[i, j])) for j in range(int(cnt[i]))]
            windows.append(st.DecodedTokenWindow(p.index, p.emission_start_sample, p.emission_end_sample,
                                                 tuple(st.globalize_tdt_tokens(emitted, p))))
        ref = st.stitch_token_windows(windows)
        print(f"engine {precision}: {len(result.tokens)} merged tokens, methods {[t.method for t in result.trace]}")
        assert result.tokens == ref.tokens
        assert result.trace == ref.trace
        assert device.status() == 0
    finally:
        eng.destroy()


def test_pipelined_batches_equal_one_batch_at_a_time(pk, device):
    """decode_plans queues batch i+1 before reading batch i (two host slots);
    every window's tokens equal a synchronous transcribe_windows of its
    batch, and the encoder's length staging is not overwritten in flight."""
    package = pk.synthetic.make_package("fp16", seed=0, bits_policy="all5")
    package.update(pk.synthetic.make_decoder("fp16", seed=0))
    eng = pk.engine.ParakeetEngine(device, package, "fp16", capacity=3)
    try:
        pcm = pk.synthetic.make_pcm(100.0, seed=9)
        plans = pk.windows.plan_stateless_windows(len(pcm))
        assert len(plans) >= 7  # at least three batches of up to 3
        piped = eng.decode_plans(pcm, plans)
        one_by_one = []
        for start in range(0, len(plans), 3):
            chunk = plans[start:start + 3]
            res = eng.transcribe_windows([(pcm[p.source_start_sample:p.source_end_sample], p) for p in chunk])
            for p, r in zip(chunk, res):
                one_by_one.append(pk.stitch.DecodedTokenWindow(
                    p.index, p.emission_start_sample, p.emission_end_sample,
                    tuple(pk.stitch.globalize_tdt_tokens(r.tokens, p))))
        assert piped == one_by_one
        assert device.status() == 0
    finally:
        eng.destroy()
