"""GPU parity of the persistent TDT decoder (pk_tdt_decode) against the CPU
oracle, through the C ABI and the operator mirror.

Bar (north_star): greedy TDT tokens agree on >= 99% of encoder frames.  The
kernel replays the shader's arithmetic (f16 FMA chains with the same split
and order, f32 projection chain, same skip and tie rules), so the sequences
are expected to be identical; the test reports exact agreement and asserts
the frame bar."""
from __future__ import annotations

import numpy as np
import pytest

from decoder_util import forced_decoder, frame_agreement
from gpu_util import cuda, host

pytestmark = pytest.mark.gpu

FRAME_BAR = 0.99


def _run_gpu(pk, device, enc, lengths, dec, precision, max_tokens, starts=None, ends=None, flush=None):
    import torch

    K = pk.kernels
    b, t = enc.shape[0], enc.shape[1]
    u32 = lambda a, d: cuda(np.asarray(np.full(b, d) if a is None else a, np.uint32))
    wdtype = "float16" if precision == "fp16" else "float32"
    model = {name: K.GpuTensor(name, wdtype if profiled else "float32", shape, layout, cuda(dec[name]))
             for name, (profiled, shape, layout) in K.TDT_DECODER_TENSORS.items()}
    kern = K.PersistentTdtDecoderKernel.create(device, None, model, precision)
    out = lambda: torch.full((b, max_tokens), 0xEEEE, dtype=torch.int32, device="cuda")
    d = dict(encoder_projected=cuda(enc), encoded_lengths=u32(lengths, t), decode_starts=u32(starts, 0),
             decode_ends=u32(ends, t), flush_finals=u32(flush, 0), tokens=out(), token_frames=out(),
             token_durations=out(), metadata=torch.full((2 * b,), -1, dtype=torch.int32, device="cuda"),
             batch_size=b, frames=t, max_tokens=max_tokens)
    disp = kern.create_dispatch(d)
    disp.encode()
    u = np.uint32
    meta = host(d["metadata"], u)
    return host(d["tokens"], u), host(d["token_frames"], u), host(d["token_durations"], u), meta[:b], meta[b:]


def _compare(got, ref, lengths):
    tok, fr, du, cnt, st = got
    rtok, rfr, rdu, rcnt, rst = ref
    agree = frame_agreement(tok, fr, cnt, rtok, rfr, rcnt, lengths)
    exact = all(cnt[b] == rcnt[b] and np.array_equal(tok[b, :cnt[b]], rtok[b, :rcnt[b]]) and
                np.array_equal(fr[b, :cnt[b]], rfr[b, :rcnt[b]]) and np.array_equal(du[b, :cnt[b]], rdu[b, :rcnt[b]])
                for b in range(len(lengths)))
    print(f"decoder: frame agreement {agree:.4f}, exact {exact}, counts {list(cnt)} vs {list(rcnt)}")
    return agree, exact


@pytest.fixture(params=["cluster", "resident"])
def route(pk, request):
    pk.kernels.set_decoder_route(request.param)
    yield request.param
    pk.kernels.set_decoder_route("auto")


@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_tdt_decoder_matches_oracle(pk, oracle, device, precision, route):
    if route == "resident" and precision == "fp32":
        pytest.skip("the resident decoder holds FP16 weights only")
    dt = np.float16 if precision == "fp16" else np.float32
    rng = np.random.default_rng(11)
    enc = rng.normal(0, 1, (4, 188, 640)).astype(dt)
    dec = {k: v["data"] for k, v in pk.synthetic.make_decoder(precision, seed=3).items()}
    kw = dict(starts=[0, 0, 10, 0], ends=[188, 188, 100, 188], flush=[0, 1, 0, 1])
    lengths = [188, 150, 188, 5]
    got = _run_gpu(pk, device, enc, lengths, dec, precision, 400, **kw)
    ref = oracle.tdt_decode(enc, lengths, dec, max_tokens=400, **kw)
    assert device.status() == 0
    assert list(got[4]) == list(ref[4])
    agree, _ = _compare(got, ref, [min(L, e) for L, e in zip(lengths, kw["ends"])])
    assert agree >= FRAME_BAR


def test_tdt_decoder_skip_rule_with_nonfinite_head_weights(pk, oracle, device, route):
    """Head weights that are not all finite: the shader's +0 skip rule decides
    whether an infinite weight meets a zero input, so the kernels must apply it
    (the resident kernel takes its masked path in the CTAs that hold such a
    column).  Tokens, frames, durations and counts equal the oracle's."""
    rng = np.random.default_rng(17)
    enc = rng.normal(0, 1, (4, 40, 640)).astype(np.float16)
    dec = {k: v["data"].copy() for k, v in pk.synthetic.make_decoder("fp16", seed=3).items()}
    hw = dec["joint.head.weight"].reshape(640, -1)
    hw[5, 100] = np.inf     # a token column (CTA 12)
    hw[7, 1024] = -np.inf   # the blank (CTA 0)
    hw[9, 1026] = np.inf    # duration 1 (CTA 2)
    lengths = [40, 33, 40, 7]
    got = _run_gpu(pk, device, enc, lengths, dec, "fp16", 200, flush=[1, 0, 1, 0])
    ref = oracle.tdt_decode(enc, lengths, dec, max_tokens=200, flush=[1, 0, 1, 0])
    assert device.status() == 0
    assert list(got[3]) == list(ref[3]) and list(got[4]) == list(ref[4])
    for b in range(4):
        n = int(ref[3][b])
        assert np.array_equal(got[0][b, :n], ref[0][b, :n]) and np.array_equal(got[1][b, :n], ref[1][b, :n])
        assert np.array_equal(got[2][b, :n], ref[2][b, :n])
    print(f"decoder (non-finite head weights, {route}): counts {list(got[3])}")


@pytest.mark.parametrize("token,duration,max_tokens,flush", [(1024, 3, 8, 0), (7, 0, 64, 0), (7, 0, 15, 0),
                                                             (9, 2, 32, 1)])
def test_tdt_decoder_control_paths(pk, oracle, device, token, duration, max_tokens, flush, route):
    """Blank skipping, the 10-symbol cap, overflow and the end-of-stream flush."""
    enc = np.random.default_rng(4).normal(0, 1, (2, 12, 640)).astype(np.float16)
    dec = forced_decoder(pk, "fp16", token, duration)
    got = _run_gpu(pk, device, enc, [12, 5], dec, "fp16", max_tokens, flush=[flush, flush])
    ref = oracle.tdt_decode(enc, [12, 5], dec, max_tokens=max_tokens, flush=[flush, flush])
    assert list(got[3]) == list(ref[3]) and list(got[4]) == list(ref[4])
    for b in range(2):
        n = int(ref[3][b])
        assert np.array_equal(got[0][b, :n], ref[0][b, :n]) and np.array_equal(got[1][b, :n], ref[1][b, :n])


def test_tdt_decoder_rejects_bad_descriptors(pk, device):
    K = pk.kernels
    with pytest.raises(K.RangeError):
        K.plan_tdt_decoder_execution(0)
    import ctypes

    desc = pk._lib.TdtDesc(0, 0, 188, 10)
    with pytest.raises(pk.PkError, match="PK_E_SHAPE"):
        pk._lib.call("pk_tdt_decode", device.handle, ctypes.byref(desc), None)


@pytest.mark.parametrize("b", [40, 32, 7])
def test_resident_and_cluster_decoders_agree(pk, device, b):
    """40 windows (the resident kernel's capacity, the reference's batch
    capacity), 32 and an odd count, with ragged lengths, start / end ranges
    and flushes: both kernels return identical tokens, frames, durations,
    counts and flags."""
    rng = np.random.default_rng(21 + b)
    enc = rng.normal(0, 1, (b, 188, 640)).astype(np.float16)
    dec = {k: v["data"] for k, v in pk.synthetic.make_decoder("fp16", seed=5).items()}
    lengths = rng.integers(1, 189, size=b).tolist()
    starts = [int(rng.integers(0, 3)) for _ in range(b)]
    ends = [int(rng.integers(150, 189)) for _ in range(b)]
    flush = [int(i % 3 == 0) for i in range(b)]
    outs = []
    for r in ("cluster", "resident"):
        pk.kernels.set_decoder_route(r)
        try:
            outs.append(_run_gpu(pk, device, enc, lengths, dec, "fp16", 2048, starts=starts, ends=ends, flush=flush))
        finally:
            pk.kernels.set_decoder_route("auto")
    assert device.status() == 0
    (t0, f0, d0, c0, s0), (t1, f1, d1, c1, s1) = outs
    assert list(c0) == list(c1) and list(s0) == list(s1)
    for w in range(b):
        n = int(c0[w])
        assert np.array_equal(t0[w, :n], t1[w, :n]) and np.array_equal(f0[w, :n], f1[w, :n])
        assert np.array_equal(d0[w, :n], d1[w, :n])
    print(f"decoder: {b}-window agreement, {int(np.sum(c0))} tokens")
