"""Decoder inputs shared by the CPU and GPU decoder tests."""
from __future__ import annotations

import numpy as np


def forced_decoder(pkg, precision: str, token: int, duration: int) -> dict:
    """Synthetic decoder tensors whose head always picks `token` (1024 = blank)
    and duration index `duration`: head weights zero, biases favour the pair."""
    dec = {k: v["data"].copy() for k, v in pkg.synthetic.make_decoder(precision, seed=7).items()}
    dec["joint.head.weight"][:] = 0
    hb = np.zeros(1032, np.float32)
    hb[token] = 5.0
    hb[1025 + duration] = 5.0
    dec["joint.head.bias"] = hb
    return dec


def frame_agreement(tok_a, fr_a, cnt_a, tok_b, fr_b, cnt_b, lengths) -> float:
    """Fraction of encoder frames whose emitted token sequence agrees."""
    agree = total = 0
    for b, L in enumerate(lengths):
        ea = {}
        eb = {}
        for i in range(int(cnt_a[b])):
            ea.setdefault(int(fr_a[b, i]), []).append(int(tok_a[b, i]))
        for i in range(int(cnt_b[b])):
            eb.setdefault(int(fr_b[b, i]), []).append(int(tok_b[b, i]))
        for f in range(int(L)):
            total += 1
            agree += ea.get(f, []) == eb.get(f, [])
    return agree / max(total, 1)
