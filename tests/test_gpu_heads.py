"""The heads on a B200: pooler_output, classify and mlm_logits through the public
C API, and their kernels (nxk_mul_mat, nxk_gelu_norm, nxk_gather_rows), against
the CPU checkers.

Bars:
* the activation conversion of nxk_mul_mat (Q8_K / Q8_0 / Q8_1 codes and scales,
  F16 / BF16 rounding) is bit-identical to ggml's restated in oracle/vecdot.c;
* nxk_mul_mat's outputs: the integer chunk dots are exact and only the fp32 sums
  of the chunk terms run in another order, so |got - want| <= 1e-5 * sum|w||x|;
* the head entry points against the reference's own (oracle/_ref, on the host
  CPU): the int8 path is bit-exact, GELU uses CUDA's erff where the reference
  uses the C library's (they may differ in the last place), and that can flip an
  activation code of the MLM decoder's Q8_K conversion: max error <= 1e-3 and
  mean error <= 2e-5 of the largest |output|, cosine >= 0.99999 per row.
"""
import ctypes

import numpy as np
import pytest

import heads_util as hu
import synth_model as sm
from test_heads_cpu import HEAD_MODELS, _lengths_tokens, _rows

pytestmark = pytest.mark.gpu

i32 = ctypes.POINTER(ctypes.c_int32)
f32 = ctypes.POINTER(ctypes.c_float)


@pytest.fixture(scope="module")
def lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpulib import load_lib
    return load_lib()


def _mul_mat_gpu(L, qt, w, N, K, x, bias=None):
    import torch
    from gpulib import P, dev, host, stream_ptr
    M = x.shape[0]
    ws = L.nxk_mul_mat_workspace(int(qt), K, M)
    assert ws > 0
    work = torch.zeros(ws, dtype=torch.uint8, device="cuda")
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    rc = L.nxk_mul_mat(int(qt), P(dev(w)), N, K, P(dev(x)), M, P(dev(bias)) if bias is not None else None,
                       P(work), P(out), stream_ptr())
    assert rc == 0
    assert L.nxk_take_error(stream_ptr()) == 0
    return host(work).reshape(M, -1), host(out)


@pytest.mark.parametrize("K", [768, 2304])
@pytest.mark.parametrize("qt", hu.MUL_MAT_TYPES, ids=lambda q: q.name)
def test_mul_mat_kernel(lib, oracle, qt, K):
    N = 300
    w = hu.weight_rows(qt, N, K, seed=int(qt) + K)
    x = np.concatenate([_rows(K, 5), np.random.default_rng(6).standard_normal((7, K)).astype(np.float32)])
    bias = (0.02 * np.random.default_rng(7).standard_normal(N)).astype(np.float32)
    act, got = _mul_mat_gpu(lib, qt, w, N, K, x, bias)
    want_act = oracle.quantize_act(int(qt), x)
    np.testing.assert_array_equal(act[:, :want_act.shape[1]], want_act)
    want = oracle.mul_mat(int(qt), w, N, K, x) + bias
    wd = hu.dequant_rows(qt, w, K)
    for m in range(x.shape[0]):
        scale = np.abs(wd) @ np.abs(hu.act_dequant(qt, want_act[m], K)) + np.abs(bias) + 1e-30
        err = np.abs(got[m].astype(np.float64) - want[m]) / scale
        assert err.max() <= 1e-5, (m, err.max())


def test_mul_mat_rejects_bad_shapes(lib):
    from gpulib import stream_ptr
    assert lib.nxk_mul_mat_workspace(99, 256, 4) == 0
    # K-quants need K % 256 == 0; everything needs K % 32 == 0
    assert lib.nxk_mul_mat(int(sm.QT.Q4_K), ctypes.c_void_p(16), 8, 96, ctypes.c_void_p(16), 1, None,
                           ctypes.c_void_p(16), ctypes.c_void_p(16), stream_ptr()) != 0
    assert lib.nxk_mul_mat(int(sm.QT.Q8_0), ctypes.c_void_p(16), 8, 40, ctypes.c_void_p(16), 1, None,
                           ctypes.c_void_p(16), ctypes.c_void_p(16), stream_ptr()) != 0


@pytest.mark.parametrize("C", [256, 1024])
def test_gelu_norm_kernel(lib, oracle, C):
    import torch
    from gpulib import P, dev, host, stream_ptr
    rng = np.random.default_rng(C)
    x = (2.0 * rng.standard_normal((37, C))).astype(np.float32)
    g = (1.0 + 0.05 * rng.standard_normal(C)).astype(np.float32)
    out = torch.empty((37, C), dtype=torch.float32, device="cuda")
    assert lib.nxk_gelu_norm(P(dev(x)), P(dev(g)), 1e-5, 37, C, P(out), stream_ptr()) == 0
    got = host(out)
    want = oracle.layer_norm(oracle.gelu_erf(x), g, None, 1e-5)
    # CUDA's erff and the C library's may differ in the last place; the rest is exact
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6)
    # in place (out == x), as the library runs it
    xd = dev(x)
    assert lib.nxk_gelu_norm(P(xd), P(dev(g)), 1e-5, 37, C, P(xd), stream_ptr()) == 0
    np.testing.assert_array_equal(host(xd), got)


def test_gather_rows_kernel(lib):
    import torch
    from gpulib import P, dev, host, stream_ptr
    x = np.random.default_rng(0).standard_normal((50, 256)).astype(np.float32)
    idx = np.array([49, 0, 7, 7, 31], np.int32)
    out = torch.empty((5, 256), dtype=torch.float32, device="cuda")
    assert lib.nxk_gather_rows(P(dev(x)), 256, P(dev(idx)), 5, P(out), stream_ptr()) == 0
    np.testing.assert_array_equal(host(out), x[idx])


class Heads:
    def __init__(self, L, path):
        self.L = L
        self.h = L.nextera_load(str(path).encode(), L.nextera_default_params())
        assert self.h, f"nextera_load failed for {path}"
        self.C = L.nextera_n_embd(self.h)

    def pooler_output(self, toks, lengths):
        out = np.full((len(lengths), self.C), np.nan, np.float32)
        rc = self.L.nextera_pooler_output(self.h, toks.ctypes.data_as(i32), None, lengths.ctypes.data_as(i32),
                                          len(lengths), out.ctypes.data_as(f32))
        return rc, out

    def classify(self, toks, lengths):
        task = self.L.nextera_classifier_task(self.h).decode()
        rows = len(lengths) if task in sm.POOLED_TASKS else int(lengths.sum())
        out = np.full((rows, max(self.L.nextera_n_labels(self.h), 1)), np.nan, np.float32)
        rc = self.L.nextera_classify(self.h, toks.ctypes.data_as(i32), None, lengths.ctypes.data_as(i32),
                                     len(lengths), out.ctypes.data_as(f32))
        return rc, out

    def mlm_logits(self, toks, pos):
        out = np.full((max(len(pos), 1), self.L.nextera_n_vocab(self.h)), np.nan, np.float32)
        rc = self.L.nextera_mlm_logits(self.h, toks.ctypes.data_as(i32), len(toks), pos.ctypes.data_as(i32),
                                       len(pos), out.ctypes.data_as(f32))
        return rc, out

    def close(self):
        self.L.nextera_free(self.h)


def close_enough(got, want, what):
    assert got.shape == want.shape, what
    assert np.isfinite(got).all(), what
    top = float(np.abs(want).max())
    d = np.abs(got.astype(np.float64) - want)
    assert d.max() <= 1e-3 * top, (what, d.max() / top)
    assert d.mean() <= 2e-5 * top, (what, d.mean() / top)
    cos = (got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1) + 1e-30)
    assert cos.min() >= 0.99999, (what, cos.min())


@pytest.fixture(scope="module")
def head_models():
    return {k: sm.cached_model("tiny_" + k, sm.tiny_hparams(**kw), preset, seed=11) for k, kw, preset in HEAD_MODELS}


@pytest.mark.parametrize("key", [m[0] for m in HEAD_MODELS])
def test_heads_match_reference(lib, reflib, head_models, key):
    path = head_models[key]
    hp = dict((m[0], m[1]) for m in HEAD_MODELS)[key]
    m = Heads(lib, path)
    r = reflib.load(path, 0)
    try:
        lengths, toks = _lengths_tokens(1000)
        if hp.get("cls_task") in sm.POOLED_TASKS or hp.get("pooler"):
            rc, got = m.pooler_output(toks, lengths)
            assert rc == 0
            close_enough(got, reflib.pooler_output(r, toks, lengths), "pooler_output")
        else:
            rc, _ = m.pooler_output(toks, lengths)
            assert rc == 1                                   # no pooler in this file
        if hp.get("cls_task"):
            rc, got = m.classify(toks, lengths)
            assert rc == 0
            close_enough(got, reflib.classify(r, toks, lengths), "classify")
        else:
            rc, _ = m.classify(toks, lengths)
            assert rc == 1
        seq = toks[:40]
        pos = np.array([0, 39, 7, 7, 22], np.int32)
        rc, got = m.mlm_logits(seq, pos)
        assert rc == 0
        close_enough(got, reflib.mlm_logits(r, seq, pos), "mlm_logits")
        # bad positions and empty position lists are input errors (:1970-1973)
        assert m.mlm_logits(seq, np.array([40], np.int32))[0] == 1
        assert m.mlm_logits(seq, np.array([-1], np.int32))[0] == 1
        assert m.mlm_logits(seq, np.zeros(0, np.int32))[0] == 1
        assert m.mlm_logits(np.array([5000], np.int32), np.array([0], np.int32))[0] == 1
    finally:
        m.close()
        reflib.L.nextera_free(r)


def test_mlm_logits_q4km_full_width(lib, reflib):
    """The tied decoder over a 50368 x 1024 Q4_K table (the published model's widths, 2 layers)."""
    hp = sm.full_hparams(n_layer=2, block_types=["lily", "swa"])
    path = sm.cached_model("full2", hp, "Q4_K_M", seed=2)
    m = Heads(lib, path)
    r = reflib.load(path, 0)
    try:
        seq = sm.random_tokens(300, hp.n_vocab, seed=9)
        pos = np.array([0, 5, 150, 299], np.int32)
        rc, got = m.mlm_logits(seq, pos)
        assert rc == 0
        close_enough(got, reflib.mlm_logits(r, seq, pos), "mlm_logits full width")
    finally:
        m.close()
        reflib.L.nextera_free(r)
