"""Hand-worked known-answer cases of the decomposed-rel-pos attention, independent of the float64 restatement in
tests/golden/make_golden.py and of the C oracle.

The inputs are built from the reference's own statement of the op (src/kernels.rs:8, the doc comment of
`relpos_softmax`; the table index `qi + size - 1 - ki` of its tensor fallback, src/kernels.rs:21-29):

    P[r, k] = softmax_k( scale * q_r . kt[:, k] + q_r . Th[i - kh + H - 1] + q_r . Tw[j - kw + W - 1] ),
    r = i W + j,  k = kh W + kw,  Th = table[0 : 2H-1],  Tw = table[2H-1 :],   out_r = sum_k P[r, k] v_k

with q_r = (1, 1, 0, ...), Th[m] = (ln a_m, 0, ...), Tw[m] = (0, ln b_m, ...) and kt[:, k] = (ln d_k / scale, 0, ...)
for positive integers a, b, d. Every logit is then the log of an integer product, so
P[r, k] = a[i-kh+H-1] b[j-kw+W-1] d_k / Z_r exactly, and with integer v the expected output is an exact rational,
computed here with fractions.Fraction by plain loops over the formula. A swapped h / w, a mirrored index
(kh - i instead of i - kh) or a wrong table split changes the answer by far more than the tolerance."""
import math
from fractions import Fraction

import numpy as np
import pytest

from oracle import oracle


def handworked(h, w, hd, with_scores):
    """Inputs (float32 arrays) and the exact expected output (Fractions) of one head."""
    n = h * w
    scale = 0.125
    a = [1 + (m * 7) % 5 for m in range(2 * h - 1)]        # small positive integers per Th row
    b = [1 + (m * 3) % 4 for m in range(2 * w - 1)]        # per Tw row
    d = [1 + (k * 5) % 3 if with_scores else 1 for k in range(n)]
    q = np.zeros((1, n, hd), np.float32)
    q[0, :, 0] = 1.0
    q[0, :, 1] = 1.0
    kt = np.zeros((1, hd, n), np.float32)
    kt[0, 0, :] = [math.log(x) / scale for x in d]
    table = np.zeros((2 * h - 1 + 2 * w - 1, hd), np.float32)
    table[:2 * h - 1, 0] = [math.log(x) for x in a]
    table[2 * h - 1:, 1] = [math.log(x) for x in b]
    v = np.zeros((1, n, hd), np.float32)
    vint = [((k * 13) % 7 - 3, (k * 5) % 11 - 5) for k in range(n)]
    v[0, :, 0] = [x for x, _ in vint]
    v[0, :, 1] = [y for _, y in vint]
    out = []
    for i in range(h):
        for j in range(w):
            wts = [Fraction(a[i - kh + h - 1] * b[j - kw + w - 1] * d[kh * w + kw])
                   for kh in range(h) for kw in range(w)]
            z = sum(wts)
            out.append((sum(wt * vint[k][0] for k, wt in enumerate(wts)) / z,
                        sum(wt * vint[k][1] for k, wt in enumerate(wts)) / z))
    return q, kt, v, table, scale, out


CASES = [(2, 3, 2, True), (3, 2, 2, True), (5, 4, 8, True), (14, 14, 64, False), (7, 11, 80, True)]


def expected_array(out, n, hd):
    e = np.zeros((1, n, hd), np.float64)
    e[0, :, 0] = [float(x) for x, _ in out]
    e[0, :, 1] = [float(y) for _, y in out]
    return e


@pytest.mark.parametrize("h,w,hd,scores", CASES)
def test_oracle_matches_handworked(h, w, hd, scores):
    q, kt, v, table, scale, out = handworked(h, w, hd, scores)
    got = oracle.attention_relpos(q, kt, v, table, h, w, scale)
    want = expected_array(out, h * w, hd)
    assert np.abs(got - want).max() <= 2e-6 * max(1.0, np.abs(want).max())


@pytest.mark.gpu
@pytest.mark.parametrize("h,w,hd,scores", CASES + [(64, 64, 64, False)])
def test_kernels_match_handworked(samrs, cuda, h, w, hd, scores):
    """The f32 path of the library (SIMT kernel) against the exact answer."""
    import torch
    q, kt, v, table, scale, out = handworked(h, w, hd, scores)
    dev = [torch.from_numpy(x).to(cuda) for x in (q, kt, v, table)]
    got = samrs.attention_relpos(*dev, h, w, scale).double().cpu().numpy()
    assert samrs.device_status() == 0
    want = expected_array(out, h * w, hd)
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())
