"""The block encoders the quantizer tests compare against (tests/golden/synth_model.py), checked on
the CPU: every K-quant encoding decodes through gguf-py 0.19's dequantizers (the published block
layouts, as ggml reads them) to within its format's step, and the legacy types come from gguf-py's
own quantizers, which restate ggml's reference quantizers bit for bit."""
import numpy as np
import pytest

import synth_model as sm
from synth_model import QT

# largest |error| allowed per value, in units of the row block's largest |value|
# (Q4_0 / Q5_0 map the block's largest magnitude to -8 / -16 steps, so the other end can be off by a
# whole step; a K-quant's sub-block scales are themselves quantized to 4 or 6 bits, so its bound is a few steps;
# a misplaced bit in a layout gives errors of the order of the block's largest value)
STEP = {QT.Q2_K: 0.7, QT.Q3_K: 0.35, QT.Q4_K: 0.15, QT.Q5_K: 0.1, QT.Q6_K: 0.08,
        QT.Q8_0: 0.005, QT.Q4_0: 0.13, QT.Q4_1: 0.07, QT.Q5_0: 0.065, QT.Q5_1: 0.035}


@pytest.mark.parametrize("qt", list(STEP))
def test_encoders_decode_within_their_step(qt):
    rng = np.random.default_rng(int(qt))
    w = rng.standard_normal((16, 512)).astype(np.float32)
    w[3] = 0.0                                  # an all-zero row
    w[5, :7] *= 40.0                            # an outlier block
    blocks = sm.quantize_rows(w, qt)
    back = sm.dequantize_rows(blocks, qt, 512)
    bs = 256 if qt in (QT.Q2_K, QT.Q3_K, QT.Q4_K, QT.Q5_K, QT.Q6_K) else 32
    amax = np.abs(w.reshape(-1, bs)).max(1, keepdims=True)
    err = np.abs(back.reshape(-1, bs) - w.reshape(-1, bs))
    assert np.all(err <= STEP[qt] * amax + 1e-6), float((err / np.maximum(amax, 1e-30)).max())
    assert np.all(back[3] == 0.0)
