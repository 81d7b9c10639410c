"""Benchmark: encoder audio-seconds per second on B200.

Workload per GPU (weak scaling): the full FP16 encoder -- subsampling, 24
Macaron Conformer layers, projector -- on a batch of 32 independent 15 s
windows (log-mel f32 [32, 128, 1501] ~ N(-4, 2^2), feature length 1500 ->
188 encoder frames), random-init 5/6-bit palette weights (o_proj 6-bit, the
reference's mixed policy).  One step = one encoder forward of the batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

* ``value``: audio seconds encoded per second over all ranks, inputs resident
  in HBM, timed with CUDA events on the launching stream (max over ranks);
* ``e2e``: the same metric through the public API with host buffers: every
  step's features copied in from pinned host memory and its projected
  output copied out, the copies on a second stream overlapping the
  neighbouring steps' encoder work;
* ``roofline``: the palette GEMMs (the dominant kernel, tcgen05 tensor
  cores) -- algorithmic FLOPs of one step's GEMM launches / their summed
  CUDA-event time (each shape back to back over rotating operand sets larger
  than twice the L2), against the measured bf16 peak;
* ``cpu_baseline``: the CPU oracle (a port of the reference's shader math,
  f16-accumulating GEMMs) on one window, scaled to audio-s/s;
* ``config1_config2``: BASELINE configs 1 (the FP32 6-bit GEMM) and 2 (one
  FP16 block, 8 windows) on the GPU, GFLOP/s, beside the oracle on the host;
* ``fp32_encoder``: the FP32 package's encoder against the FFMA peak;
* ``decoder`` / ``logmel`` / ``transcribe``: the TDT decoder on the step's
  encoder output, the log-mel front end on 32 windows of PCM, and 60 s of PCM
  through ``ParakeetEngine.transcribe`` (config 4);
* ``longform``: config 5 -- an hour (FP16) or ten minutes (FP32) of PCM
  through ``engine.transcribe_sharded`` on all ranks, host PCM in and merged
  tokens out, for mixed and all-5-bit palettes (max over ranks), with the
  phases (decode, gather, rank-0 merge); ``longform_encoder``: the same hour
  through log-mel and the encoder only, sharded the same way.

``--impl reference`` times that CPU port on all host cores (rank 0 only):
the reference's own WGSL path cannot run here (no browser / WebGPU stack).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WINDOW_SECONDS = 15.0
BATCH = 32
FEATURE_LENGTH = 1500
FRAMES = 188
METRIC = "encoder audio-sec/sec (RTFx)"
UNIT = "audio-s/s"
# Kernel launches of one encoder step: subsampling (conv0+dw2, pw3 GEMM, dw5,
# pw6 GEMM with the time mask in its epilogue, flatten GEMM), 14 per layer (the
# out-LN of one layer and the FF1 LN of the next share one dual-LayerNorm
# launch), the last layer's own out-LN and the projector: 343, as counted by
# ncu's launch list of a step.
LAUNCHES_PER_STEP = 5 + 24 * 14 + 1 + 1
# DRAM bytes (read + write) of one step's palette-GEMM launches: per-launch bytes from one ncu
# capture of each bench.gemm_shapes(32) shape run alone, times its launches per step (the
# per-shape table and the command are kept with the other ncu summaries under profiles/).
GEMM_DRAM_BYTES_PER_STEP = 6173968384


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def gemm_shapes(batch: int):
    """(rows, inner, columns, bits, groups, activation, epilogue, launches per step) of every
    palette GEMM of one step, with the epilogue each one runs in the encoder."""
    rows = batch * FRAMES
    return [
        (batch * 376 * 32, 256, 256, 5, 1, "relu", "bias", 1),   # subsampling pointwise 3
        (batch * 188 * 16, 256, 256, 5, 1, "relu", "bias", 1),   # subsampling pointwise 6
        (rows, 4096, 1024, 5, 1, "none", "bias", 1),             # flatten projection
        (rows, 1024, 4096, 5, 1, "silu", "plain", 48),           # ff1/ff2 linear1
        (rows, 4096, 1024, 5, 1, "none", "residual", 48),        # ff1/ff2 linear2 (+0.5 residual)
        (rows, 1024, 3072, 5, 3, "none", "plain", 24),           # qkv (3 palette groups)
        (rows, 1024, 1024, 6, 1, "none", "residual", 24),        # o_proj (6-bit, + residual)
        (rows, 1024, 2048, 5, 1, "none", "plain", 24),           # pointwise conv 1
        (rows, 1024, 1024, 5, 1, "none", "residual", 24),        # pointwise conv 2 (+ residual)
        (rows, 1024, 640, 5, 1, "none", "bias", 1),              # projector
    ]


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms)}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["bf16_tflops"]), float(d.get("hbm_gbs", 6451.5)), "measured"
    return 1590.0, 6650.0, "fallback"


def gemm_operands(pk, rng, rows, inner, columns, bits, groups, act, epi, precision="fp16"):
    """Device operands and the pk_gemm_desc of one palette GEMM of the step
    (random activations, codes and palettes; the encoder's epilogue), FP16 or
    FP32 package."""
    import torch

    L = pk._lib
    dt = torch.float16 if precision == "fp16" else torch.float32
    codes, lut = pk.synthetic.palette_matrix(rng, inner, columns, bits, groups, precision)
    keep = {
        "a": torch.randn((rows, inner), dtype=dt, device="cuda"),
        "c": torch.empty((rows, columns), dtype=dt, device="cuda"),
        "res": torch.randn((rows, columns), dtype=dt, device="cuda") if epi == "residual" else None,
        "bias": torch.randn(columns, dtype=torch.float32, device="cuda") if epi == "bias" else None,
        "codes": torch.from_numpy(codes["data"].view(np.int32)).cuda(),
        "lut": torch.from_numpy(lut["data"]).cuda(),
    }
    ptr = lambda name: None if keep[name] is None else keep[name].data_ptr()  # noqa: E731
    desc = L.GemmDesc(L.FP16 if precision == "fp16" else L.FP32, rows, inner, columns, bits, groups,
                      columns // groups, L.ACT[act],
                      int(epi == "residual"), 0.5, ptr("bias"), ptr("res"), ptr("a"), ptr("codes"), ptr("lut"),
                      ptr("c"))
    return desc, keep


def time_gemms(pk, device, batch, stream, min_reps=8):
    """CUDA-event time of each distinct palette GEMM of a step, on `stream`.
    Launches run back to back as in the encoder step, cycling through enough
    independent operand sets (activations, codes, palettes, outputs,
    residuals) that together they exceed 256 MB, twice the L2: no launch
    starts with its own inputs in L2."""
    import ctypes

    import torch

    L = pk._lib
    rng = np.random.default_rng(0)
    total_flops = total_ms = 0.0
    detail = []
    for rows, inner, columns, bits, groups, act, epi, launches in gemm_shapes(batch):
        per_set = 2 * rows * (inner + columns * (2 if epi == "residual" else 1)) + inner * columns * bits // 8
        sets = [gemm_operands(pk, rng, rows, inner, columns, bits, groups, act, epi)
                for _ in range(max(1, -(-(256 << 20) // per_set)))]
        reps = len(sets) * max(1, -(-min_reps // len(sets)))
        h = ctypes.c_void_p(stream.cuda_stream)
        for desc, _ in sets:
            L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), h)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for r in range(reps):
            L.call("pk_palette_gemm", device.handle, ctypes.byref(sets[r % len(sets)][0]), h)
        end.record(stream)
        end.synchronize()
        ms = start.elapsed_time(end) / reps
        del sets
        flops = 2.0 * rows * inner * columns
        total_flops += flops * launches
        total_ms += ms * launches
        detail.append({"m": rows, "k": inner, "n": columns, "bits": bits, "epilogue": f"{epi}+{act}",
                       "launches": launches,
                       "us": round(ms * 1e3, 2), "tflops": round(flops / (ms * 1e-3) / 1e12, 1)})
    return total_flops, total_ms, detail


MAX_TOKENS_PER_WINDOW = 2048  # the reference engine's decoder capacity (src/runtime/webgpu-engine.ts:84)


def decoder_buffers(pk, device, enc, precision="fp16", seed=0):
    """PersistentTdtDecoderKernel over `enc` [batch, frames, 640] with synthetic
    decoder weights; returns (dispatch, descriptor dict)."""
    import torch

    K = pk.kernels
    b, t = enc.shape[0], enc.shape[1]
    dec = pk.synthetic.make_decoder(precision, seed=seed)
    model = {n: K.GpuTensor.from_record(n, r) for n, r in dec.items()}
    kern = K.PersistentTdtDecoderKernel.create(device, None, model, precision)
    u32 = lambda v: torch.full((b,), v, dtype=torch.int32, device="cuda")  # noqa: E731
    out = lambda: torch.zeros((b, MAX_TOKENS_PER_WINDOW), dtype=torch.int32, device="cuda")  # noqa: E731
    d = dict(encoder_projected=enc, encoded_lengths=u32(t), decode_starts=u32(0), decode_ends=u32(t),
             flush_finals=u32(0), tokens=out(), token_frames=out(), token_durations=out(),
             metadata=torch.zeros(2 * b, dtype=torch.int32, device="cuda"), batch_size=b, frames=t,
             max_tokens=MAX_TOKENS_PER_WINDOW, model=model)
    return kern.create_dispatch(d), d


def time_decoder(pk, device, enc, stream, reps=3):
    """CUDA-event time of one greedy TDT decode of the batch on `stream`."""
    import torch

    disp, d = decoder_buffers(pk, device, enc)
    with torch.cuda.stream(stream):
        disp.encode(stream)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            disp.encode(stream)
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / reps
    b = enc.shape[0]
    counts = d["metadata"][:b].cpu().numpy()
    return {"kernel": "tdt_resident_kernel (FP16 weights resident on 128 co-resident CTAs, windows in lockstep)",
            "windows": b,
            "ms_per_batch": round(ms, 3), "windows_per_s": round(b / (ms * 1e-3), 1),
            "audio_s_per_s": round(b * WINDOW_SECONDS / (ms * 1e-3), 1),
            "tokens_per_window": round(float(counts.mean()), 1), "joint_steps_bound": "<= 10 x 188 per window",
            "weights": "synthetic random-init decoder (blank-biased head)"}


def time_logmel(pk, device, stream, reps=5):
    """CUDA-event time of the log-mel front end for one batch of 15 s windows."""
    import torch

    pcm = (0.1 * torch.randn((BATCH, 240_000), device="cuda")).contiguous()
    valid = torch.full((BATCH,), 240_000, dtype=torch.int32, device="cuda")
    feats = torch.empty((BATCH, 128, 1501), dtype=torch.float32, device="cuda")
    fb = pk.kernels.ParakeetFbank(device)
    with torch.cuda.stream(stream):
        fb.compute_batch(pcm, valid, out=feats, stream=stream)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            fb.compute_batch(pcm, valid, out=feats, stream=stream)
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / reps
    moved = pcm.numel() * 4 + 3 * feats.numel() * 4  # PCM read, raw write, normalize read + write
    return {"kernels": "logmel_raw_kernel + logmel_normalize_kernel", "windows": BATCH,
            "us_per_batch": round(ms * 1e3, 1), "audio_s_per_s": round(BATCH * WINDOW_SECONDS / (ms * 1e-3), 1),
            "hbm_bytes_per_batch": moved, "achieved_gbs": round(moved / (ms * 1e-3) / 1e9, 1)}


def time_transcribe(pk, device, package, seconds=60.0, reps=2):
    """Wall time of engine.transcribe on `seconds` of synthetic PCM (host
    buffers in and out; window plan, log-mel, encoder, decoder, merge)."""
    import torch

    full = dict(package)
    full.update(pk.synthetic.make_decoder("fp16", seed=0))
    eng = pk.engine.ParakeetEngine(device, full, "fp16", capacity=BATCH)
    pcm = pk.synthetic.make_pcm(seconds, seed=4)
    eng.transcribe(pcm)  # warm-up
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(reps):
        res = eng.transcribe(pcm)
    dt = (time.perf_counter() - t0) / reps
    windows = len(pk.windows.plan_stateless_windows(len(pcm)))
    eng.destroy()
    return {"workload": f"config4: {seconds:.0f} s synthetic PCM (pink noise + modulated tones), {windows} windows",
            "s_per_run": round(dt, 4), "audio_s_per_s": round(seconds / dt, 1), "tokens": len(res),
            "note": "random-init weights; the decoder's token count (not real speech) sets most of the time"}


# Config 5 variants: (precision, palette policy, seconds of audio).  FP32 runs a
# shorter stretch so the default benchmark stays within minutes.
LONGFORM_VARIANTS = (("fp16", "mixed", 3600.0), ("fp16", "all5", 3600.0), ("fp32", "mixed", 3600.0),
                     ("fp32", "all5", 3600.0))
LONGFORM_CAPACITY = 40  # windows per engine batch (the reference's encoder capacity)


def encoder_batch(windows: int, capacity: int) -> int:
    """Encoder-only leg: batches of up to `capacity` windows, but at least two
    batches per rank, so one batch's host staging overlaps the other's GPU
    work (one hour on one GPU: 7 x 40; on eight: 18 + 17)."""
    return max(1, min(capacity, -(-windows // 2)))


def longform_pcm(pk, seconds, seed=5, distinct=5):
    """`seconds` of synthetic PCM built from `distinct` different 60 s
    make_pcm blocks in rotation (a full-length make_pcm of an hour costs
    about 40 s of host time)."""
    blocks = [pk.synthetic.make_pcm(60.0, seed=seed + i) for i in range(distinct)]
    n = int(round(seconds * 16_000))
    reps = -(-n // blocks[0].shape[0])
    return np.concatenate([blocks[i % distinct] for i in range(reps)])[:n]


def time_longform(pk, device, rank, world, stream, capacity=None):
    """engine.transcribe_sharded on synthetic audio, host PCM in and merged
    tokens out: each rank decodes its contiguous share of the window plan on
    its own GPU and merges its own windows as they finish (native merge);
    the runs meet on rank 0 as flat int64 arrays (a gather of plain tensors,
    no collective on the hot path), which joins them at the rank seams.
    Time: CUDA events on each rank's stream around its share, the gather and
    the merge; max over ranks.  Per phase (host wall time, max over ranks):
    decode (decode + the rank's own merge, overlapped), gather, rank-0 merge."""
    import torch
    import torch.distributed as dist

    capacity = capacity or LONGFORM_CAPACITY
    gather = (lambda flat: [flat]) if world == 1 else pk.engine.array_gather(rank, world, torch.device("cuda"))

    def max_over_ranks(values):
        if world == 1:
            return values
        t = torch.tensor(values, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    out = []
    # One generation serves every variant: the shorter runs take its prefix,
    # which is exactly what longform_pcm makes for their length.
    longest = longform_pcm(pk, max(v[2] for v in LONGFORM_VARIANTS))
    for precision, policy, seconds in LONGFORM_VARIANTS:
        package = pk.synthetic.make_package(precision, bits_policy=policy, seed=0)
        package.update(pk.synthetic.make_decoder(precision, seed=0))
        eng = pk.engine.ParakeetEngine(device, package, precision, capacity=capacity)
        del package
        pcm = longest[: int(round(seconds * 16_000))]
        timings = {}
        plans = pk.windows.plan_stateless_windows(len(pcm))
        mine = [plans[i] for i in pk.windows.shard_windows(len(plans), world, rank)]
        with torch.cuda.stream(stream):
            eng.transcribe(pcm[:30 * 16_000])  # warm-up
            for size in sorted({len(r) for r in eng.batches(len(mine))}):  # record every graph size used
                eng.encode_plans(pcm, mine[:size])
            if world > 1:
                gather(np.zeros(8, np.int64))  # the gather's buffers and channels exist before timing
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            res = pk.engine.transcribe_sharded(eng, pcm, rank, world, gather, timings=timings)
            end.record(stream)
            end.synchronize()
        ms, decode_s, gather_s, merge_s = max_over_ranks(
            [start.elapsed_time(end), timings["decode_s"], timings["gather_s"], timings["merge_s"]])
        windows = len(pk.windows.plan_stateless_windows(len(pcm)))
        batches = [len(r) for r in eng.batches(len(pk.windows.shard_windows(windows, world, rank)))]
        eng.destroy()
        out.append({"precision": precision, "palette_bits": policy, "audio_s": seconds, "windows": windows,
                    "s": round(ms / 1e3, 3), "audio_s_per_s": round(seconds / (ms / 1e3), 1),
                    "tokens": None if res is None else len(res),
                    "rank_batches": batches,
                    "phases_s": {"decode": round(decode_s, 4), "gather": round(gather_s, 4),
                                 "merge_rank0": round(merge_s, 4)}})
    return {"workload": "config5: synthetic PCM (five 60 s pink-noise + tone blocks in rotation), window plan "
                        "sharded over ranks, host PCM in, merged tokens out",
            "n_gpus": world, "capacity": capacity, "variants": out,
            "note": "random-init weights; decoded token counts are not real speech and set most of the time"}


def time_longform_encoder(pk, device, rank, world, stream, capacity=None, seconds=3600.0):
    """The encoder alone on an hour of synthetic audio (BASELINE config 5's
    workload, FP16, mixed palettes): each rank takes its contiguous share of
    the window plan and runs log-mel + the 24-layer encoder on it in balanced
    batches, host PCM in, projected encoder output left on the device.  CUDA
    events around each rank's share, max over ranks."""
    import torch
    import torch.distributed as dist

    capacity = capacity or LONGFORM_CAPACITY
    package = pk.synthetic.make_package("fp16", seed=0)
    package.update(pk.synthetic.make_decoder("fp16", seed=0))
    eng = pk.engine.ParakeetEngine(device, package, "fp16", capacity=capacity)
    del package
    pcm = longform_pcm(pk, seconds)
    plans = pk.windows.plan_stateless_windows(len(pcm))
    mine = [plans[i] for i in pk.windows.shard_windows(len(plans), world, rank)]
    batch = encoder_batch(len(mine), capacity)
    with torch.cuda.stream(stream):
        for rows in eng.batches(len(mine), batch):  # warm-up: every graph size is recorded
            eng.encode_plans(pcm, mine[rows.start:rows.stop])
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        eng.encode_plans(pcm, mine, batch=batch)
        end.record(stream)
        end.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    eng.destroy()
    return {"workload": "config5 encoder only: one hour of synthetic PCM, window plan sharded over ranks, "
                        "log-mel + 24-layer FP16 encoder (mixed palettes), host PCM in, encoder output on device",
            "n_gpus": world, "audio_s": seconds, "windows": len(plans),
            "rank_batches": [len(r) for r in eng.batches(len(mine), batch)],
            "s": round(ms / 1e3, 4), "audio_s_per_s": round(seconds / (ms / 1e3), 1)}


def time_e2e_pipelined(pk, graph, features, lengths, stream, steps):
    """``value``'s metric through the public API with host buffers, every
    step copying its features in from pinned host memory and its projected
    output back out, with the copies of one step overlapping the encoder
    work of its neighbours: two device input / output buffers, uploads and
    read-backs each on a stream of their own (ParakeetEncoderGraph.encode
    reads the device buffer).  CUDA events bracket the whole run on the
    launching stream, which joins both copy streams at the end.  Returns ms
    per step."""
    import torch

    copy = torch.cuda.Stream()     # host -> device
    drain = torch.cuda.Stream()    # device -> host (its own stream, so a step's read-back
                                   # never queues ahead of the next step's upload)
    pinned_in = torch.from_numpy(features).pin_memory()
    rows = features.shape[0] * FRAMES
    dev_in = [torch.empty(features.shape, dtype=torch.float32, device="cuda") for _ in range(2)]
    dev_out = [torch.empty((rows, 640), dtype=torch.float16, device="cuda") for _ in range(2)]
    host_out = [torch.empty((rows, 640), dtype=torch.float16).pin_memory() for _ in range(2)]
    landed = [torch.cuda.Event() for _ in range(2)]   # features of a buffer on the device
    computed = [torch.cuda.Event() for _ in range(2)]  # outputs of a buffer written
    drained = [torch.cuda.Event() for _ in range(2)]   # outputs of a buffer read back

    def run(n):
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(copy):
                if i >= 2:
                    copy.wait_event(computed[b])  # the encoder of step i-2 has read dev_in[b]
                dev_in[b].copy_(pinned_in, non_blocking=True)
                landed[b].record(copy)
            stream.wait_event(landed[b])
            if i >= 2:
                stream.wait_event(drained[b])  # step i-2's output left dev_out[b]
            with torch.cuda.stream(stream):
                graph.encode(dev_in[b], lengths, stream=stream, out=dev_out[b])
                computed[b].record(stream)
            with torch.cuda.stream(drain):
                drain.wait_event(computed[b])
                host_out[b].copy_(dev_out[b], non_blocking=True)
                drained[b].record(drain)
        stream.wait_stream(copy)
        stream.wait_stream(drain)

    run(3)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    copy.wait_event(start)
    drain.wait_event(start)
    run(steps)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps, int(pinned_in.numel() * 4), int(host_out[0].numel() * 2)


# FFMA peak of the FP32 package's GEMMs: SMs x 128 FP32 lanes x 2 FLOP per FMA x clock.
FFMA_LANES_PER_SM = 128
# Dense TF32 tensor-core rate of one B200 (NVIDIA's 2:4-sparse figure halved);
# nominal, not measured -- the FP32 package's GEMMs do not use it (each output
# must be the reference's fp32 fma chain), it is reported for scale.
TF32_DENSE_TFLOPS_NOMINAL = 1100.0


def time_config1(pk, device, stream, reps=50):
    """the FP32 palette GEMM [188 x 1024] . [1024 x 4096]
    (6-bit, 64-entry f32 LUT ~ N(0, 0.02) sorted, seed 0), raw product and
    the SiLU epilogue; CUDA events, inputs resident (operands total 20 MB,
    timed back to back: this single GEMM's figure includes L2 reuse)."""
    import ctypes

    import torch

    L = pk._lib
    rng = np.random.default_rng(0)
    a = torch.from_numpy(rng.standard_normal((188, 1024)).astype(np.float32)).cuda()
    codes, lut = pk.synthetic.palette_matrix(rng, 1024, 4096, 6, 1, "fp32")
    tc = torch.from_numpy(codes["data"].view(np.int32)).cuda()
    tl = torch.from_numpy(lut["data"]).cuda()
    out = torch.empty((188, 4096), dtype=torch.float32, device="cuda")
    res = {}
    h = ctypes.c_void_p(stream.cuda_stream)
    for act in ("none", "silu"):
        desc = L.GemmDesc(L.FP32, 188, 1024, 4096, 6, 1, 4096, L.ACT[act], 0, 1.0, None, None, a.data_ptr(),
                          tc.data_ptr(), tl.data_ptr(), out.data_ptr())
        for _ in range(5):
            L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), h)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), h)
        end.record(stream)
        end.synchronize()
        us = start.elapsed_time(end) / reps * 1e3
        res[act] = {"us": round(us, 2), "gflops": round(2 * 188 * 1024 * 4096 / (us * 1e-6) / 1e9, 1)}
    return {"workload": "config1: FP32 palette GEMM 188x1024x4096, 6-bit, CUDA-core fp32 fma chain "
                        "(bit-exact with the reference's order)", **res}


def block_launcher(pk, device, weights, batch, stream):
    """The 15 launches of one Macaron Conformer block (src/webgpu/encoder.ts:
    1869-2138) on the production kernels, through the C ABI, for `batch`
    188-frame windows: returns (launch function, device buffers).  The
    attention takes the positions re-laid out row-major, as the encoder does."""
    import ctypes

    import torch

    L = pk._lib
    rows = batch * FRAMES
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    w = {n: (dev(r["data"].view(np.int32)) if r["data"].dtype == np.dtype("<u4") else dev(r["data"]))
         for n, r in weights.items() if n.startswith("encoder.layers.0.")}
    p = "encoder.layers.0."
    f16 = lambda cols: torch.randn((rows, cols), dtype=torch.float16, device="cuda")  # noqa: E731
    buf = {"x": f16(1024), "a": f16(1024), "h": f16(4096), "x1": f16(1024), "qkv": f16(3072), "ctx": f16(1024),
           "x2": f16(1024), "g": f16(2048), "c": f16(1024), "x3": f16(1024), "x4": f16(1024), "y": f16(1024)}
    pos = weights[p + "self_attn.projected_positions"]["data"].reshape(8, 32, 375, 4)
    w["pos_rm"] = dev(np.ascontiguousarray(pos.transpose(0, 2, 1, 3).reshape(8, 375, 128)))
    lens = dev(np.full(batch, FRAMES, np.uint32).view(np.int32))
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    h = ctypes.c_void_p(stream.cuda_stream)
    descs = []

    def gemm(name, src, dst, cols, act="none", res=None, scale=1.0):
        rec = weights[p + name + ".weight"]
        groups = weights[p + name + ".weight.palette"]["data"].shape[0]
        d = L.GemmDesc(L.FP16, rows, src.shape[1], cols, rec["bits"], groups, cols // groups, L.ACT[act],
                       int(res is not None), scale, None, None if res is None else res.data_ptr(), src.data_ptr(),
                       w[p + name + ".weight"].data_ptr(), w[p + name + ".weight.palette"].data_ptr(), dst.data_ptr())
        descs.append(d)
        return lambda: L.call("pk_palette_gemm", device.handle, ctypes.byref(d), h)

    def norm(name, src, dst):
        return lambda: L.call("pk_layernorm", device.handle, L.FP16, rows, 1024, vp(src), vp(w[p + name + ".weight"]),
                              vp(w[p + name + ".bias"]), 1e-5, vp(dst), h)

    b = buf
    ops = [norm("norm_feed_forward1", b["x"], b["a"]), gemm("feed_forward1.linear1", b["a"], b["h"], 4096, "silu"),
           gemm("feed_forward1.linear2", b["h"], b["x1"], 1024, res=b["x"], scale=0.5),
           norm("norm_self_att", b["x1"], b["a"]), gemm("self_attn.qkv", b["a"], b["qkv"], 3072),
           lambda: L.call("pk_rel_attention", device.handle, L.FP16, batch, FRAMES, vp(b["qkv"]), vp(w["pos_rm"]),
                          vp(w[p + "self_attn.bias_u"]), vp(w[p + "self_attn.bias_v"]), vp(lens), vp(b["ctx"]), h),
           gemm("self_attn.o_proj", b["ctx"], b["x2"], 1024, res=b["x1"]), norm("norm_conv", b["x2"], b["a"]),
           gemm("conv.pointwise_conv1", b["a"], b["g"], 2048),
           lambda: L.call("pk_conformer_conv", device.handle, L.FP16, batch, FRAMES, vp(b["g"]),
                          vp(w[p + "conv.depthwise_conv.weight"]), vp(w[p + "conv.norm.scale"]),
                          vp(w[p + "conv.norm.shift"]), vp(lens), vp(b["c"]), h),
           gemm("conv.pointwise_conv2", b["c"], b["x3"], 1024, res=b["x2"]),
           norm("norm_feed_forward2", b["x3"], b["a"]), gemm("feed_forward2.linear1", b["a"], b["h"], 4096, "silu"),
           gemm("feed_forward2.linear2", b["h"], b["x4"], 1024, res=b["x3"], scale=0.5),
           norm("norm_out", b["x4"], b["y"])]

    def launch():
        for op in ops:
            op()

    return launch, (w, buf, lens, descs)


def time_config2(pk, device, stream, batch=8, reps=50):
    """one FP16 FastConformer block, batch 8 x 188 frames,
    mixed 5/6-bit palettes, inputs N(0, 1); its 15 launches captured in a
    CUDA graph (the attention on the tcgen05 route with row-major positions,
    as in the encoder), CUDA events over `reps` replays."""
    import torch

    weights = pk.synthetic.make_package("fp16", layers=1, seed=21)
    pk.kernels.set_attention_route("tcgen05-rowmajor")
    try:
        launch, keep = block_launcher(pk, device, weights, batch, stream)
        with torch.cuda.stream(stream):
            for _ in range(3):
                launch()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            launch()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                g.replay()
        end.record(stream)
        end.synchronize()
    finally:
        pk.kernels.set_attention_route("auto")
    us = start.elapsed_time(end) / reps * 1e3
    flops = 2.0 * batch * FRAMES * 24117248 + 3 * 2 * batch * FRAMES ** 2 * 1024
    del keep, g
    return {"workload": "config2: one FP16 block, 8 x 188 frames, mixed palettes (15 launches in one CUDA graph)",
            "us_per_block": round(us, 1), "gflops": round(flops / (us * 1e-6) / 1e9, 1),
            "flop_per_block": flops}


def cpu_config12(pk):
    """CPU baselines of configs 1 and 2: the oracle's reference mode (FP32
    fma chain for config 1; f16-accumulating GEMMs for config 2) on the
    host's cores; config 2 on one window (of the 8), scaled per block."""
    from oracle import oracle

    rng = np.random.default_rng(0)
    a = rng.standard_normal((188, 1024)).astype(np.float32)
    codes, lut = pk.synthetic.palette_matrix(rng, 1024, 4096, 6, 1, "fp32")
    oracle.palette_gemm(a, codes["data"], lut["data"], 6, 4096, acc_mode=0)
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        oracle.palette_gemm(a, codes["data"], lut["data"], 6, 4096, acc_mode=0)
    c1 = (time.perf_counter() - t0) / reps
    weights = pk.synthetic.make_package("fp16", layers=1, seed=21)
    x = rng.standard_normal((FRAMES, 1024)).astype(np.float16)
    t0 = time.perf_counter()
    oracle.conformer_layer(weights, 0, x, np.array([FRAMES], np.uint32), 1, FRAMES, acc_mode=0)
    c2 = time.perf_counter() - t0
    c2_flops = 2.0 * FRAMES * 24117248 + 3 * 2 * FRAMES ** 2 * 1024
    return {"config1": {"s": round(c1, 4), "gflops": round(2 * 188 * 1024 * 4096 / c1 / 1e9, 2)},
            "config2": {"s_per_window": round(c2, 3), "gflops": round(c2_flops / c2 / 1e9, 2),
                        "sample": "1 window of the 8 (windows are independent)"}}


def time_fp32_encoder(pk, device, stream, batch=8, reps=5):
    """The FP32 package's 24-layer encoder (f32 activations and LUTs, CUDA-core
    fp32 fma-chain GEMMs in the reference's order) on `batch` 15 s windows:
    audio-s/s and the GEMMs' FLOP rate against the FFMA peak."""
    import torch

    package = pk.synthetic.make_package("fp32", seed=7)
    g = pk.encoder.ParakeetEncoderGraph.create(device, package, "fp32", capacity=batch)
    feats = torch.from_numpy(pk.synthetic.make_features(batch, seed=8)).cuda()
    lengths = [FEATURE_LENGTH] * batch
    with torch.cuda.stream(stream):
        for _ in range(2):
            g.encode(feats, lengths, stream=stream)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            g.encode(feats, lengths, stream=stream)
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / reps
    g.destroy()
    g.weights.release()
    props = torch.cuda.get_device_properties(device.ordinal)
    gemm_flops = sum(2.0 * (m // BATCH) * batch * k * n * launches
                     for m, k, n, _, _, _, _, launches in gemm_shapes(BATCH))
    rate = gemm_flops / (ms * 1e-3) / 1e12
    ffma_peak = props.multi_processor_count * FFMA_LANES_PER_SM * 2 * 1.965e9 / 1e12
    return {"workload": f"FP32 package encoder, {batch} x 15 s windows", "ms_per_step": round(ms, 2),
            "audio_s_per_s": round(batch * WINDOW_SECONDS / (ms * 1e-3), 1),
            "gemm_tflop_per_step": round(gemm_flops / 1e12, 3),
            "gemm_tflops_if_all_time": round(rate, 2),
            "ffma_peak_tflops_at_max_clock": round(ffma_peak, 1),
            "frac_of_ffma_peak": round(rate / ffma_peak, 3),
            "tf32_dense_tflops_nominal": TF32_DENSE_TFLOPS_NOMINAL,
            "frac_of_tf32_nominal": round(rate / TF32_DENSE_TFLOPS_NOMINAL, 4),
            "peak_note": "FFMA: SMs x 128 FP32 lanes x 2 FLOP x 1965 MHz (clocks.max.sm); TF32: nominal dense tensor "
                         "rate, unused by these bit-exact fp32 chains; the GEMM rate counts the whole step's time, so "
                         "both fractions are lower bounds"}


def cpu_baseline(pk, package, window_count=1):
    """Oracle (reference algorithm, f16-accumulating GEMMs) on `window_count` windows."""
    from oracle import oracle

    fb = pk.synthetic.make_features(window_count, seed=1)
    t0 = time.perf_counter()
    oracle.encoder(package, fb, [FEATURE_LENGTH] * window_count, np.float16, acc_mode=0)
    dt = time.perf_counter() - t0
    return window_count * WINDOW_SECONDS / dt, dt


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    import __graft_entry__

    pk = __graft_entry__.load()
    from oracle import oracle

    oracle.build()
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    package = pk.synthetic.make_package("fp16", seed=0)
    for _ in range(args.warmup):
        cpu_baseline(pk, package, 1)
    times = []
    for _ in range(args.steps):
        _, dt = cpu_baseline(pk, package, 1)
        times.append(dt)
    value = WINDOW_SECONDS * args.steps / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sum(times) / args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "config3: 24-layer FP16 encoder, 15 s windows (1 window per step on CPU)",
                   "batch_per_step": 1, "precision": "fp16", "palette_bits": "mixed 5/6"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "1 window x 24 layers per step, oracle reference mode (f16 accumulation)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference WGSL path needs a browser WebGPU stack: unavailable on this box; timed its CPU port",
    }
    print(json.dumps(line))
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    import __graft_entry__

    pk = __graft_entry__.load()
    device = pk.kernels.Device(local)
    package = pk.synthetic.make_package("fp16", seed=0)
    graph = pk.encoder.ParakeetEncoderGraph.create(device, package, "fp16", capacity=BATCH)
    features = pk.synthetic.make_features(BATCH, seed=100 + rank)
    lengths = [FEATURE_LENGTH] * BATCH
    stream = torch.cuda.Stream()
    dev_features = torch.from_numpy(features).cuda()
    out = torch.empty((BATCH * FRAMES, 640), dtype=torch.float16, device="cuda")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing (value)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            graph.encode(dev_features, lengths, stream=stream, out=out)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            graph.encode(dev_features, lengths, stream=stream, out=out)
    end.record(stream)
    end.synchronize()
    barrier()
    clock_info = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    status = device.status()

    # ---- end to end through the public API with host buffers (copies overlapped with compute)
    barrier()
    e2e_ms, h2d_bytes, d2h_bytes = time_e2e_pipelined(pk, graph, features, lengths, stream, args.steps)
    barrier()
    e2e_ms = max_over_ranks(e2e_ms)

    legs = set(args.legs.split(","))

    # ---- BASELINE configs 1 and 2 on the GPU, and the FP32 package's encoder
    c12_info = None
    if "config12" in legs:
        c12_info = {"config1": time_config1(pk, device, stream), "config2": time_config2(pk, device, stream)}
    barrier()
    fp32_info = time_fp32_encoder(pk, device, stream) if "fp32" in legs else None
    barrier()

    # ---- log-mel front end for this batch (32 x 240 000 samples of PCM)
    lm_info = time_logmel(pk, device, stream) if "logmel" in legs else None
    barrier()

    # ---- TDT greedy decoding of this batch's encoder output (synthetic decoder weights)
    dec_info = None
    if "decoder" in legs:
        dec_info = time_decoder(pk, device, out.view(BATCH, FRAMES, 640), stream, reps=max(1, min(args.steps, 5)))
    barrier()

    # ---- end-to-end transcription (config 4): 60 s of PCM through the engine
    tr_info = time_transcribe(pk, device, package) if rank == 0 and "transcribe" in legs else None
    barrier()

    # ---- long-form (config 5): one hour's window plan sharded across all ranks
    lf_info = None if args.skip_longform or "longform" not in legs else time_longform(pk, device, rank, world, stream)
    barrier()

    # ---- the encoder alone on config 5's hour, sharded across all ranks
    lfe_info = None if "longform" not in legs else time_longform_encoder(pk, device, rank, world, stream)
    barrier()

    # ---- dominant kernel: palette GEMMs of one step, timed live
    gemm_flops, gemm_ms, gemm_detail = 0.0, 1.0, []
    if "gemm" in legs:
        with torch.cuda.stream(stream):
            gemm_flops, gemm_ms, gemm_detail = time_gemms(pk, device, BATCH, stream)
    barrier()

    if rank == 0:
        peak_tf, _, peak_kind = measured_peaks()
        achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12
        audio = world * BATCH * WINDOW_SECONDS
        cores = os.cpu_count() or 1
        cpu_value, cpu_dt = (None, None)
        if world == 1 and not args.skip_cpu_baseline:
            os.environ.setdefault("OMP_NUM_THREADS", str(cores))
            cpu_value, cpu_dt = cpu_baseline(pk, package, 1)
            if c12_info is not None:
                c12_info["cpu"] = cpu_config12(pk)
                c12_info["cpu"]["cores"] = int(os.environ.get("OMP_NUM_THREADS", cores))
        traffic = GEMM_DRAM_BYTES_PER_STEP
        line = {
            "metric": METRIC, "value": round(audio / (ms * 1e-3), 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "config3: full 24-layer FP16 encoder, batch 32 x 15 s windows per GPU",
                       "global_batch": world * BATCH, "seq_len": FRAMES, "parallelism": f"window-shard x{world}",
                       "palette_bits": "mixed (o_proj 6-bit, rest 5-bit)",
                       "audio_seconds": "each of the 32 independent 15 s windows counts 15 s (window-seconds); "
                                        "the longform legs count source audio",
                       "l2": "working set per step > 126 MB L2 (weights 365 MB packed + activations); "
                             "roofline GEMMs timed back to back over rotating operand sets > 256 MB"},
            "e2e": {"value": round(audio / (e2e_ms * 1e-3), 1), "unit": UNIT,
                    "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
                    "note": "ParakeetEncoderGraph.encode per step; each step's pinned H2D features and D2H "
                            "projected output on an upload and a read-back stream, overlapping the "
                            "neighbouring steps' encoder work"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": round(achieved / peak_tf, 4), "traffic": traffic,
                         "kernel": "palette GEMMs (tc2_/tc_palette_gemm, all launches of one step)",
                         "traffic_unit": "DRAM bytes per step (ncu, each shape captured alone)",
                         "peak_kind": f"bf16 dense burst, {peak_kind}",
                         "gemm_ms_per_step": round(gemm_ms, 3), "gemm_tflop_per_step": round(gemm_flops / 1e12, 3)},
            "gemm_shapes": gemm_detail,
            "config1_config2": c12_info,
            "fp32_encoder": fp32_info,
            "decoder": dec_info,
            "logmel": lm_info,
            "transcribe": tr_info,
            "longform": lf_info,
            "longform_encoder": lfe_info,
            "cpu_baseline": None if cpu_value is None else {
                "value": round(cpu_value, 3), "unit": UNIT, "cores": int(os.environ.get("OMP_NUM_THREADS", cores)),
                "kind": "port", "sample": f"1 window x 24 layers, oracle reference mode, {cpu_dt:.1f} s"},
            "clocks": clock_info,
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "device_status": status,
        }
        print(json.dumps(line))
    graph.destroy()
    device.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_kernel(args):
    """Profiling target: launch one operator `--steps` times at the C3 shapes
    (no JSON line).  `--kernel gemm --shape M,K,N,BITS` picks the GEMM shape."""
    import ctypes

    import torch

    import __graft_entry__

    pk = __graft_entry__.load()
    L = pk._lib
    device = pk.kernels.Device(0)
    rng = np.random.default_rng(0)
    keep = []

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int32) if a.dtype == np.dtype("<u4") else a).cuda()
        keep.append(t)
        return ctypes.c_void_p(t.data_ptr())

    if args.kernel in ("gemm", "gemm-fp32"):
        m, k, n, bits = (int(x) for x in args.shape.split(","))
        desc, keep_gemm = gemm_operands(pk, rng, m, k, n, bits, 1, args.act, args.epi,
                                        "fp32" if args.kernel == "gemm-fp32" else "fp16")
        launch = lambda: L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), None)  # noqa: E731
    elif args.kernel == "gemm-step":
        # Each distinct palette GEMM of a config-3 step once per launch() call.
        step = [gemm_operands(pk, rng, *shape[:7]) for shape in gemm_shapes(BATCH)]

        def launch():
            for desc, _ in step:
                L.call("pk_palette_gemm", device.handle, ctypes.byref(desc), None)
    elif args.kernel in ("attention", "attention-mma"):
        # "attention": the tcgen05 kernel on row-major positions (the encoder's
        # path); "attention-mma": the mma.sync kernel on the package layout.
        b = int(args.shape or BATCH)
        qkv = torch.randn((b * FRAMES, 3072), dtype=torch.float16, device="cuda")
        ctx = torch.empty((b * FRAMES, 1024), dtype=torch.float16, device="cuda")
        pos_np = (0.5 * rng.standard_normal((8, 32, 375, 4))).astype(np.float16)
        if args.kernel == "attention":
            pos_np = np.ascontiguousarray(pos_np.transpose(0, 2, 1, 3).reshape(8, 375, 128))
        pk.kernels.set_attention_route("tcgen05-rowmajor" if args.kernel == "attention" else "mma")
        pos = dev(pos_np)
        u = dev((0.02 * rng.standard_normal((8, 128))).astype(np.float32))
        v = dev((0.02 * rng.standard_normal((8, 128))).astype(np.float32))
        lens = dev(np.full(b, FRAMES, np.uint32))
        launch = lambda: L.call("pk_rel_attention", device.handle, L.FP16, b, FRAMES,  # noqa: E731
                                ctypes.c_void_p(qkv.data_ptr()), pos, u, v, lens, ctypes.c_void_p(ctx.data_ptr()),
                                None)
    elif args.kernel == "layernorm":
        rows = int(args.shape or BATCH * FRAMES)
        x = torch.randn((rows, 1024), dtype=torch.float16, device="cuda")
        y = torch.empty_like(x)
        g = dev(np.ones(1024, np.float32))
        bb = dev(np.zeros(1024, np.float32))
        launch = lambda: L.call("pk_layernorm", device.handle, L.FP16, rows, 1024,  # noqa: E731
                                ctypes.c_void_p(x.data_ptr()), g, bb, 1e-5, ctypes.c_void_p(y.data_ptr()), None)
    elif args.kernel == "subsampling":
        b = int(args.shape or BATCH)
        fb = torch.randn((b, 128, 1501), dtype=torch.float32, device="cuda")
        out = torch.empty((b, 376, 32, 256), dtype=torch.float16, device="cuda")
        w0 = dev((0.3 * rng.standard_normal((3, 3, 256))).astype(np.float16))
        b0 = dev((0.02 * rng.standard_normal(256)).astype(np.float32))
        wd = dev((0.1 * rng.standard_normal((3, 3, 256))).astype(np.float16))
        bd = dev((0.02 * rng.standard_normal(256)).astype(np.float32))
        lens = dev(np.full(b, 1501, np.uint32))
        launch = lambda: L.call("pk_subsampling_conv0_dw2", device.handle, L.FP16, b,  # noqa: E731
                                ctypes.c_void_p(fb.data_ptr()), w0, b0, wd, bd, lens,
                                ctypes.c_void_p(out.data_ptr()), None)
    elif args.kernel == "depthwise":
        # The subsampling's second depthwise 3x3 / 2 (channel-last FP16, 376 x 32 -> 188 x 16 x 256).
        b = int(args.shape or BATCH)
        x = torch.randn((b, 376, 32, 256), dtype=torch.float16, device="cuda")
        out = torch.empty((b, 188, 16, 256), dtype=torch.float16, device="cuda")
        wd = dev((0.1 * rng.standard_normal((3, 3, 256))).astype(np.float16))
        bd = dev((0.02 * rng.standard_normal(256)).astype(np.float32))
        lens = dev(np.full(b, 1501, np.uint32))
        launch = lambda: L.call("pk_subsampling_depthwise", device.handle, L.FP16, b, 376, 32, 256,  # noqa: E731
                                ctypes.c_void_p(x.data_ptr()), wd, bd, lens, 3, ctypes.c_void_p(out.data_ptr()),
                                None)
    elif args.kernel == "conv":
        b = int(args.shape or BATCH)
        gin = torch.randn((b * FRAMES, 2048), dtype=torch.float16, device="cuda")
        out = torch.empty((b * FRAMES, 1024), dtype=torch.float16, device="cuda")
        dw = dev((0.1 * rng.standard_normal((9, 1024))).astype(np.float16))
        sc = dev(np.ones(1024, np.float32))
        sh = dev(np.zeros(1024, np.float32))
        lens = dev(np.full(b, FRAMES, np.uint32))
        launch = lambda: L.call("pk_conformer_conv", device.handle, L.FP16, b, FRAMES,  # noqa: E731
                                ctypes.c_void_p(gin.data_ptr()), dw, sc, sh, lens, ctypes.c_void_p(out.data_ptr()),
                                None)
    elif args.kernel == "logmel":
        b = int(args.shape or BATCH)
        pcm = (0.1 * torch.randn((b, 240_000), device="cuda")).contiguous()
        valid = torch.full((b,), 240_000, dtype=torch.int32, device="cuda")
        fb = pk.kernels.ParakeetFbank(device)
        feats = torch.empty((b, 128, 1501), dtype=torch.float32, device="cuda")
        launch = lambda: fb.compute_batch(pcm, valid, out=feats)  # noqa: E731
    elif args.kernel == "decoder":
        b = int(args.shape or BATCH)
        enc = torch.randn((b, FRAMES, 640), dtype=torch.float16, device="cuda")
        disp, d = decoder_buffers(pk, device, enc)
        launch = lambda: disp.encode()  # noqa: E731
    else:
        raise SystemExit(f"unknown kernel {args.kernel}")
    for _ in range(args.steps):
        launch()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        launch()
    end.record()
    end.synchronize()
    print(f"{args.kernel} {args.shape}: {start.elapsed_time(end) / args.steps * 1e3:.1f} us/launch, "
          f"status {device.status()}")
    device.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=250)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-longform", action="store_true")
    ap.add_argument("--legs", default="logmel,decoder,transcribe,longform,gemm,config12,fp32",
                    help="comma-separated extra legs to run besides the encoder step (a subset for quick runs)")
    ap.add_argument("--kernel", choices=["gemm", "gemm-fp32", "gemm-step", "attention", "attention-mma", "layernorm", "conv",
                                         "subsampling", "depthwise", "decoder", "logmel"],
                    help="profiling target: launch one operator only")
    ap.add_argument("--shape", default="", help="gemm: M,K,N,BITS; attention/conv/decoder: batch; layernorm: rows")
    ap.add_argument("--act", default="none", choices=["none", "silu", "relu"])
    ap.add_argument("--epi", default="plain", choices=["plain", "bias", "residual"],
                    help="gemm: epilogue (residual: + 0.5 x a random residual)")
    args = ap.parse_args()
    if args.kernel:
        return run_kernel(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
