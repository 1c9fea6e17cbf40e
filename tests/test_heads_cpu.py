"""The heads on the CPU checkers (no GPU).

* oracle/vecdot.c (ggml's mul_mat restated: activation conversion to the weight
  type's vec_dot type, integer block dots) against an independent numpy
  restatement of the conversion, bit for bit, and against the product of the
  gguf-py-dequantized weights with the converted activation;
* the reference's own head entry points (oracle/_ref: nextera_pooler_output,
  nextera_classify, nextera_mlm_logits) against the head graphs composed from
  the checkers' ops, bit for bit: this pins which rows, weights and ops each
  head uses (src/nexterabert.cpp:1296-1317, :1963-2011), the graph the GPU
  library mirrors.
"""
from __future__ import annotations

import numpy as np
import pytest

import heads_util as hu
import synth_model as sm
from gguf import GGMLQuantizationType as QT


def _rows(K, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((6, K)).astype(np.float32)
    x[1, :256] = 0.0                          # an all-zero block
    x[2, 3], x[2, 10] = -2.5, 2.5             # equal magnitudes: the first one sets the sign
    x[2, :256] = np.clip(x[2, :256], -2.0, 2.0)
    x[2, 3], x[2, 10] = -2.5, 2.5
    x[3] *= 1e-30                             # tiny values
    x[4, ::7] = 0.5                           # rounding ties after scaling are possible
    return x


@pytest.mark.parametrize("qt", hu.MUL_MAT_TYPES, ids=lambda q: q.name)
def test_act_conversion_matches_numpy(oracle, qt):
    K = 512
    x = _rows(K, 1)
    got = oracle.quantize_act(int(qt), x)
    for m in range(x.shape[0]):
        want = hu.act_numpy(qt, x[m])
        assert got.shape[1] == want.size
        np.testing.assert_array_equal(got[m], want, err_msg=f"row {m}")


@pytest.mark.parametrize("qt", hu.MUL_MAT_TYPES, ids=lambda q: q.name)
def test_mul_mat_equals_dequantized_product(oracle, qt):
    """Integer block dots with their scales = dequantized weights . converted activation."""
    N, K = 24, 512
    w = hu.weight_rows(qt, N, K, seed=int(qt))
    x = _rows(K, 2)
    got = oracle.mul_mat(int(qt), w, N, K, x).astype(np.float64)
    wd = hu.dequant_rows(qt, w, K)
    act = oracle.quantize_act(int(qt), x)
    for m in range(x.shape[0]):
        xd = hu.act_dequant(qt, act[m], K)
        want = wd @ xd
        scale = np.abs(wd) @ np.abs(xd) + 1e-30
        # fp32 accumulation; Q8_1 stores s = d * sum(codes) as fp16 (2^-11 relative)
        tol = 2e-3 if hu.FAMILY[qt] == "q8_1" else 2e-6
        err = np.abs(got[m] - want) / scale
        assert err.max() <= tol, (m, err.max())


def _lengths_tokens(n_vocab, seed=3):
    lengths = np.array([1, 5, 17, 40], np.int32)
    return lengths, sm.random_tokens(int(lengths.sum()), n_vocab, seed=seed)


HEAD_MODELS = [
    ("seq", dict(cls_task="sequence-classification", n_labels=3), "Q4_K_M"),
    ("tok", dict(cls_task="token-classification", n_labels=40, cls_f16=True, untied_decoder=True), "Q8_0"),
    ("mc", dict(cls_task="multiple-choice", n_labels=1), "Q5_K_M"),
    ("qa", dict(cls_task="question-answering", n_labels=2), "Q4_K_M"),
    ("pool", dict(pooler=True), "Q6_K"),
]


@pytest.fixture(scope="module")
def head_models():
    return {k: sm.cached_model("tiny_" + k, sm.tiny_hparams(**kw), preset, seed=11) for k, kw, preset in HEAD_MODELS}


@pytest.mark.parametrize("key", [m[0] for m in HEAD_MODELS])
def test_reference_heads_follow_their_graph(reflib, oracle, head_models, key):
    path = head_models[key]
    h = reflib.load(path, 4)
    try:
        lengths, toks = _lengths_tokens(1000)
        hidden, _ = reflib.encode(h, toks, lengths, normalize=False, hidden=True)
        hp = dict((m[0], m[1]) for m in HEAD_MODELS)[key]
        if hp.get("cls_task") in sm.POOLED_TASKS or hp.get("pooler"):
            got = reflib.pooler_output(h, toks, lengths)
            want = hu.head_graph(reflib, oracle, path, hidden, lengths, head="pooler")
            np.testing.assert_array_equal(got, want)
        if hp.get("cls_task"):
            got = reflib.classify(h, toks, lengths)
            want = hu.head_graph(reflib, oracle, path, hidden, lengths, head="classify")
            assert got.shape == want.shape
            np.testing.assert_array_equal(got, want)
        # MLM on one sequence: positions with repeats, first and last rows
        seq = toks[:40]
        pos = np.array([0, 39, 7, 7, 22], np.int32)
        hid1, _ = reflib.encode(h, seq, np.array([40], np.int32), normalize=False, hidden=True)
        got = reflib.mlm_logits(h, seq, pos)
        want = hu.head_graph(reflib, oracle, path, hid1, positions=pos, head="mlm")
        np.testing.assert_array_equal(got, want)
    finally:
        reflib.L.nextera_free(h)
