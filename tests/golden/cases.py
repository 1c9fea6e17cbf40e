"""Seeded op-level input cases shared by the fixture script and the tests.

Each case returns plain numpy inputs; the reference (oracle/_ref), the oracle
and the GPU library are all run on exactly these arrays.
"""
from __future__ import annotations

import numpy as np

import synth_model as sm
from gguf import GGMLQuantizationType as QT

# ragged documents: a length-1 document, lengths below / above the conv kernel,
# not multiples of the HRA block or of 8
LENGTHS_SMALL = np.array([1, 7, 33, 2, 64, 5, 130], np.int32)
# one document long enough for the reference's blocked attention branch (>= 2048 keys)
LENGTHS_ATTN = np.array([1, 9, 300, 2100, 64, 17], np.int32)

WEIGHT_TYPES = [QT.Q8_0, QT.Q4_0, QT.Q4_1, QT.Q5_0, QT.Q5_1, QT.Q4_K, QT.Q5_K, QT.Q6_K]


def rng(seed):
    return np.random.default_rng(seed)


def weight_case(qt, n_out=64, n_in=512, seed=0):
    """A quantized weight: (raw blocks, n_in, n_out)."""
    w = (0.02 * rng(seed).standard_normal((n_out, n_in))).astype(np.float32)
    if seed % 3 == 1:
        w[3, :] = 0.0                     # an all-zero row: amax 0 -> scale 0
        w[5, 256:] = 0.0                  # a zero second block
    return sm.quantize_rows(w, qt), n_in, n_out


def linear_case(T=13, K=512, N=64, seed=0, qt=QT.Q8_0, residual=True):
    """Activations, weight blocks and an optional residual for one int8 linear."""
    r = rng(seed)
    x = r.standard_normal((T, K)).astype(np.float32)
    x[min(2, T - 1), :] = 0.0             # an all-zero activation row
    w = (0.02 * r.standard_normal((N, K))).astype(np.float32)
    res = r.standard_normal((T, N)).astype(np.float32) if residual else None
    return x, sm.quantize_rows(w, qt), qt, res


# name -> (T, K, N, weight type, residual, seed): token counts not a multiple of 4
# and row counts not a multiple of 12 reach the reference's 4x1 edge kernel
LINEAR_CASES = {"lin_a": (13, 512, 64, QT.Q8_0, True, 11),
                "lin_b": (7, 64, 1024, QT.Q5_0, False, 12),
                "lin_c": (33, 2304, 128, QT.Q6_K, True, 13)}


def cfg1_case():
    """Config 1: X [128, 1024] ~ N(0,1), W [4096, 1024] ~ N(0, 0.02), W in Q8_0."""
    r = rng(1)
    x = r.standard_normal((128, 1024)).astype(np.float32)
    w = (0.02 * r.standard_normal((4096, 1024))).astype(np.float32)
    return x, sm.quantize_rows(w, QT.Q8_0)


def rows_case(T=29, C=512, seed=0):
    r = rng(seed)
    x = (2.0 * r.standard_normal((T, C))).astype(np.float32)
    x[1, :] = 0.0
    x[4, 7] = 1e4                          # one large outlier in a block
    return x


def conv_case(C=256, k=5, seed=0, lengths=LENGTHS_SMALL):
    r = rng(seed)
    T = int(lengths.sum())
    x = r.standard_normal((T, C)).astype(np.float32)
    res = r.standard_normal((T, C)).astype(np.float32)
    b = r.standard_normal((T, C)).astype(np.float32)
    taps = (0.3 * r.standard_normal((k, C))).astype(np.float32)
    return x, res, b, taps


def qk_case(H=4, D=64, seed=0, lengths=LENGTHS_SMALL):
    r = rng(seed)
    T = int(lengths.sum())
    x = (0.7 * r.standard_normal((T, H * D))).astype(np.float32)
    x[0, :5] = [0.0, 0.05, -0.05, 30.0, -30.0]   # the tanh series branch and saturation
    alpha = (1.0 + 0.1 * r.standard_normal(D)).astype(np.float32)
    beta = (1.0 + 0.1 * r.standard_normal(D)).astype(np.float32)
    return x, alpha, beta


def attn_case(H=4, G=2, D=64, seed=0, lengths=LENGTHS_ATTN):
    r = rng(seed)
    T = int(lengths.sum())
    q = r.standard_normal((T, H * D)).astype(np.float32)
    k = r.standard_normal((G, T, D)).astype(np.float32)
    v = r.standard_normal((G, T, D)).astype(np.float32)
    scale = (0.125 * (1.0 + 0.2 * r.random(len(lengths)))).astype(np.float32)
    return q, k, v, scale


def model_batch(n_vocab, seed=0, lengths=LENGTHS_SMALL):
    T = int(lengths.sum())
    return sm.random_tokens(T, n_vocab, seed=seed), lengths
