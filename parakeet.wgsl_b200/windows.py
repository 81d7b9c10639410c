"""Long-form window plan and its partition across GPUs.

Restates ``planStatelessWindows`` (src/runtime/chunking.ts:174-302): fixed 15 s
(240 000-sample) model windows on a 206 080-sample stride (238 080 visible
samples minus a 2 s overlap), a one-encoder-frame (1 280-sample) decoder
context prefix for non-first windows, and an end-aligned, frame-aligned
backfill for the final window.  ``shard_windows`` partitions the plan into
contiguous, balanced ranges, one per rank: windows are independent, so a
multi-GPU run needs no collective on the hot path (each rank encodes its range;
the host merges overlaps afterwards).
"""
from __future__ import annotations

from dataclasses import dataclass

SAMPLE_RATE = 16_000
HOP_SAMPLES = 160
WINDOW_SAMPLES = 15 * SAMPLE_RATE                     # 240 000
ENCODER_FRAME_SAMPLES = 8 * HOP_SAMPLES               # 1 280
PRIMARY_CONTEXT_SAMPLES = ENCODER_FRAME_SAMPLES
PRIMARY_VISIBLE_SAMPLES = (WINDOW_SAMPLES - PRIMARY_CONTEXT_SAMPLES - HOP_SAMPLES) \
    // ENCODER_FRAME_SAMPLES * ENCODER_FRAME_SAMPLES  # 238 080
OVERLAP_SAMPLES = 2 * SAMPLE_RATE
WINDOW_STRIDE_SAMPLES = PRIMARY_VISIBLE_SAMPLES - OVERLAP_SAMPLES  # 206 080

assert WINDOW_SAMPLES // HOP_SAMPLES == 1500 and PRIMARY_VISIBLE_SAMPLES == 238_080
assert WINDOW_STRIDE_SAMPLES == 206_080


@dataclass(frozen=True)
class WindowPlan:
    index: int
    window_sample_count: int
    logical_start_sample: int
    logical_end_sample: int
    source_start_sample: int
    source_end_sample: int
    read_sample_count: int
    timestamp_offset_sample: int
    emission_start_sample: int
    emission_end_sample: int
    decode_start_frame: int
    decode_end_frame: int
    flush_final: bool
    valid_sample_count: int

    @property
    def valid_feature_frames(self) -> int:
        """parakeetValidFeatureFrameCount (src/audio/fbank-wasm.ts:141-147), at most 1500."""
        return min(self.valid_sample_count // HOP_SAMPLES, 1500)


def _ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def plan_stateless_windows(total_samples: int, speech_end_sample: int | None = None) -> list[WindowPlan]:
    if speech_end_sample is None:
        speech_end_sample = total_samples
    if total_samples < 0 or speech_end_sample < 0:
        raise ValueError("sample counts must be non-negative")
    if speech_end_sample > total_samples:
        raise ValueError("speechEndSample must not exceed totalSamples")
    plans: list[WindowPlan] = []
    logical_start, index = 0, 0
    while logical_start < total_samples:
        remaining_speech = min(speech_end_sample, total_samples) - logical_start
        reaches_eof = logical_start + PRIMARY_VISIBLE_SAMPLES >= total_samples
        backfill = 0
        if reaches_eof and remaining_speech > 0 and logical_start > 0:
            requested = (PRIMARY_VISIBLE_SAMPLES - remaining_speech) // ENCODER_FRAME_SAMPLES \
                * ENCODER_FRAME_SAMPLES
            if requested > 0:
                available = logical_start // ENCODER_FRAME_SAMPLES * ENCODER_FRAME_SAMPLES
                backfill = min(available, requested)
        visible = max(ENCODER_FRAME_SAMPLES, PRIMARY_VISIBLE_SAMPLES - backfill)
        candidate_end = logical_start + visible
        is_last = candidate_end >= total_samples
        logical_end = total_samples if is_last else candidate_end
        if logical_end <= logical_start:
            break
        source_end = min(logical_end, speech_end_sample) if is_last else logical_end
        if source_end <= logical_start:
            break
        context = 0 if (backfill > 0 or index == 0) else PRIMARY_CONTEXT_SAMPLES
        source_start = logical_start - max(backfill, context)
        read = source_end - source_start
        if read <= 0 or read > WINDOW_SAMPLES:
            raise RuntimeError("Invalid stateless source-window geometry")
        plans.append(WindowPlan(
            index=index, window_sample_count=WINDOW_SAMPLES, logical_start_sample=logical_start,
            logical_end_sample=logical_end, source_start_sample=source_start, source_end_sample=source_end,
            read_sample_count=read,
            timestamp_offset_sample=logical_start if context > 0 else source_start,
            emission_start_sample=logical_start, emission_end_sample=source_end,
            decode_start_frame=context // ENCODER_FRAME_SAMPLES,
            decode_end_frame=_ceil_div(read - context, ENCODER_FRAME_SAMPLES),
            flush_final=is_last, valid_sample_count=read))
        if is_last:
            break
        logical_start += WINDOW_STRIDE_SAMPLES
        index += 1
    return plans


def shard_windows(count: int, world_size: int, rank: int) -> range:
    """Contiguous, balanced window range of `rank` (sizes differ by at most one)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must be in [0, world_size)")
    base, extra = divmod(count, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def batches(indices: range, capacity: int) -> list[range]:
    """Split a rank's window range into encoder batches of at most `capacity`."""
    return [range(s, min(s + capacity, indices.stop)) for s in range(indices.start, indices.stop, capacity)]
