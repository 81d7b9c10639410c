"""The bench's own arithmetic, on the CPU: the roofline's FLOP count is the
algorithmic count of one config-3 step (per 188-frame window: 24 layers of
2 x 188 x 24 117 248 FLOP, the three subsampling GEMMs and the projector),
the launch count matches the step's structure, and the long-form PCM is
seeded and sized as asked."""
from __future__ import annotations

import numpy as np

import bench


def test_roofline_flops_are_the_algorithmic_count():
    per_layer_params = 4 * 4_194_304 + 3_145_728 + 1_048_576 + 2_097_152 + 1_048_576  # ff1, ff2, qkv, o, pw1, pw2
    assert per_layer_params == 24_117_248
    window = 24 * 2 * 188 * per_layer_params  # 24 Conformer layers
    window += 2 * (376 * 32) * 256 * 256 + 2 * (188 * 16) * 256 * 256  # pw3, pw6 (per output position)
    window += 2 * 188 * 4096 * 1024 + 2 * 188 * 1024 * 640  # flatten projection, projector
    step = sum(2.0 * m * k * n * launches for m, k, n, _, _, _, _, launches in bench.gemm_shapes(32))
    assert step == 32 * window
    assert abs(step / 1e12 - 7.086) < 1e-3  # TFLOP per step, as the bench line reports


def test_launch_count_matches_the_step_structure():
    shapes = bench.gemm_shapes(32)
    assert sum(s[-1] for s in shapes if s[0] == 32 * 188) == 1 + 48 + 48 + 24 + 24 + 24 + 24 + 1
    assert bench.LAUNCHES_PER_STEP == 343


def test_longform_pcm_is_seeded_and_sized(pk):
    a = bench.longform_pcm(pk, 130.0)
    b = bench.longform_pcm(pk, 130.0)
    assert a.shape == (130 * 16_000,) and a.dtype == np.float32
    assert np.array_equal(a, b)
    assert not np.array_equal(a[: 60 * 16_000], a[60 * 16_000: 120 * 16_000])  # distinct blocks rotate


def test_longform_prefix_equals_shorter_generation(pk):
    hour = bench.longform_pcm(pk, 200.0)
    assert np.array_equal(hour[: 70 * 16_000], bench.longform_pcm(pk, 70.0))
