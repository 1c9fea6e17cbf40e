"""Pins the CPU oracle (oracle/liboracle.so) bit-for-bit.

Two anchors:
* tests/golden/ref_vectors.npz -- outputs of the reference's own code, compiled
  here from its sources (oracle/_ref, written by tests/golden/make_ref_vectors.py);
* the live reference build, when this host has it (same comparisons plus more).
Block dequantization, which the reference leaves to ggml, is pinned to gguf-py.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

import cases
import synth_model as sm
from gguf import GGMLQuantizationType as QT

GOLD = Path(__file__).resolve().parent / "golden" / "ref_vectors.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def check_gold(gold, name, a):
    a = np.ascontiguousarray(a)
    if name in gold.files:
        g = gold[name]
        assert g.dtype == a.dtype and g.shape == a.shape, name
        assert np.array_equal(g, a), f"{name}: differs from the reference's output"
    else:
        want = bytes(gold[name + ".sha"]).decode()
        head = gold[name + ".head"]
        assert np.array_equal(head, a.reshape(-1)[:head.size]), f"{name}: leading values differ"
        assert hashlib.sha256(a.tobytes()).hexdigest() == want, f"{name}: differs from the reference's output"


def test_act_max(gold):
    assert int(gold["act_max"][0]) == 127      # AVX-VNNI / AVX512-VNNI build of the reference


@pytest.mark.parametrize("qt", [QT.Q8_0, QT.Q4_0, QT.Q4_1, QT.Q5_0, QT.Q5_1, QT.Q4_K, QT.Q5_K, QT.Q6_K])
def test_dequant_matches_gguf_py(oracle, qt):
    w = (0.02 * np.random.default_rng(int(qt)).standard_normal((16, 512))).astype(np.float32)
    blocks = sm.quantize_rows(w, qt)
    want = sm.dequantize_rows(blocks, qt, 512)
    for r in range(16):
        got = oracle.dequant_row(int(qt), np.ascontiguousarray(blocks[r]), 512)
        assert np.array_equal(got, want[r])


def test_dequant_k_quants_gguf_py_extra(oracle):
    # Q2_K / Q3_K blocks from random bytes with finite scales
    rng = np.random.default_rng(3)
    for qt, nbytes, dpos in ((QT.Q2_K, 84, [80, 82]), (QT.Q3_K, 110, [108])):
        raw = rng.integers(0, 256, (8, nbytes), dtype=np.uint8)
        for p in dpos:
            raw[:, p:p + 2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
        want = sm.dequantize_rows(raw, qt, 256)
        for r in range(8):
            assert np.array_equal(oracle.dequant_row(int(qt), np.ascontiguousarray(raw[r]), 256), want[r])


@pytest.mark.parametrize("i,qt", list(enumerate(cases.WEIGHT_TYPES)))
def test_build_i8_weight(oracle, gold, i, qt):
    blocks, n_in, n_out = cases.weight_case(qt, seed=i)
    w, sc, off = oracle.build_i8_weight(int(qt), blocks, n_in, n_out)
    check_gold(gold, f"i8w.{qt.name}.w", w)
    check_gold(gold, f"i8w.{qt.name}.scale", sc)
    check_gold(gold, f"i8w.{qt.name}.off", off)
    assert np.all(np.abs(w.astype(np.int32)) <= 127)


def test_quantize_rows(oracle, gold):
    q, sx = oracle.quantize_rows(cases.rows_case())
    check_gold(gold, "quant.q", q)
    check_gold(gold, "quant.sx", sx)


@pytest.mark.parametrize("name", list(cases.LINEAR_CASES))
def test_linear_i8(oracle, gold, name):
    T, K, N, qt, resid, seed = cases.LINEAR_CASES[name]
    x, blocks, qt_, res = cases.linear_case(T, K, N, seed=seed, qt=qt, residual=resid)
    w, sw, _ = oracle.build_i8_weight(int(qt_), blocks, K, N)
    xq, xs = oracle.quantize_rows(x)
    out, bs = oracle.linear_i8(xq, xs, w, sw, res, block_sums=True)
    check_gold(gold, f"{name}.out", out)
    # block sums are the integer dot products of s8 codes
    ref_bs = np.einsum("tk,nk->tn", xq[:, :256].astype(np.int64), w[:, :256].astype(np.int64))
    assert np.array_equal(bs[:, :, 0], ref_bs)


def test_cfg1_linear(oracle, gold):
    x, wb = cases.cfg1_case()
    w, sw, _ = oracle.build_i8_weight(int(QT.Q8_0), wb, 1024, 4096)
    xq, xs = oracle.quantize_rows(x)
    check_gold(gold, "cfg1.out", oracle.linear_i8(xq, xs, w, sw, None))


def test_row_ops(oracle, gold):
    xr = cases.rows_case()
    gain = (1.0 + 0.05 * np.random.default_rng(5).standard_normal(xr.shape[1])).astype(np.float32)
    y = oracle.rms_norm(xr, gain, 1e-8)
    check_gold(gold, "rms.out", y)
    q, sx = oracle.quantize_rows(y)
    check_gold(gold, "rms.q", q)
    check_gold(gold, "rms.sx", sx)
    q, sx = oracle.quantize_rows(oracle.relu_sqr(xr))
    check_gold(gold, "relu.q", q)
    check_gold(gold, "relu.sx", sx)
    g = cases.rows_case(seed=9)
    y = oracle.gate(g, xr)
    check_gold(gold, "gate.out", y)
    q, sx = oracle.quantize_rows(y)
    check_gold(gold, "gate.q", q)
    check_gold(gold, "gate.sx", sx)


def test_conv_ops(oracle, gold):
    L = cases.LENGTHS_SMALL
    xc, rc, bc, taps = cases.conv_case()
    check_gold(gold, "dwconv.out", oracle.dwconv(xc, rc, taps, L))
    q, sx = oracle.quantize_rows(oracle.dwconv(xc, None, taps, L))
    check_gold(gold, "dwconv.q", q)
    check_gold(gold, "dwconv.sx", sx)
    x64, r64, _, t64 = cases.conv_case(C=64, seed=2)
    q, sx = oracle.quantize_rows(oracle.dwconv(x64, r64, t64, L))
    check_gold(gold, "dwconv64.q", q)
    check_gold(gold, "dwconv64.sx", sx)
    y = oracle.lily_state(xc, rc, bc, taps, L)
    check_gold(gold, "lily.out", y)
    q, sx = oracle.quantize_rows(y)
    check_gold(gold, "lily.q", q)
    check_gold(gold, "lily.sx", sx)


def test_qk_prep_and_rope(oracle, gold):
    L = cases.LENGTHS_SMALL
    x, alpha, beta = cases.qk_case()
    check_gold(gold, "qk.row", oracle.qk_prep(x, alpha, beta, 100000.0, L, 4, 64, False))
    check_gold(gold, "qk.head", oracle.qk_prep(x, alpha, beta, 10000.0, L, 4, 64, True))
    c, s = oracle.rope_table(int(L.max()), 100000.0, 64)
    check_gold(gold, "rope.cos", c)
    check_gold(gold, "rope.sin", s)
    check_gold(gold, "head_major", oracle.head_major(x, 4, 64))


def test_hra_ops(oracle, gold):
    L = cases.LENGTHS_SMALL
    xc, rc, bc, _ = cases.conv_case()
    y = oracle.block_mean(xc, bc, L, 4)
    check_gold(gold, "bmean.out", y)
    q, sx = oracle.quantize_rows(y)
    check_gold(gold, "bmean.q", q)
    check_gold(gold, "bmean.sx", sx)
    ybm = oracle.block_mean(xc, None, L, 4)
    check_gold(gold, "bmean_nog.out", ybm)
    check_gold(gold, "upsample.out", oracle.upsample_add(ybm, rc, L, 4))


def test_attention(oracle, gold):
    q, k, v, scale = cases.attn_case()
    check_gold(gold, "attn.swa", oracle.attention(q, k, v, 4, 2, 64, 8, scale, cases.LENGTHS_ATTN))
    check_gold(gold, "attn.full", oracle.attention(q, k, v, 4, 2, 64, -1, scale, cases.LENGTHS_ATTN))


@pytest.mark.parametrize("tag,preset,seed", [("tiny_q4km", "Q4_K_M", 0), ("tiny_q8", "Q8_0", 1)])
def test_whole_model(oracle, gold, tag, preset, seed):
    path = sm.cached_model("tiny", sm.tiny_hparams(), preset, seed=seed)
    m = oracle.load(path)
    tok, lens = cases.model_batch(1000, seed=7)
    hid, pooled = m.encode(tok, lens)
    check_gold(gold, f"{tag}.hidden", hid)
    check_gold(gold, f"{tag}.pooled", pooled)
    _, pooled_raw = m.encode(tok, lens, normalize=False, hidden=False)
    check_gold(gold, f"{tag}.pooled_raw", pooled_raw)
    m.close()


# -- against the live reference build (skipped where oracle/_ref is absent) --

def test_live_ops_random(oracle, reflib):
    rng = np.random.default_rng(123)
    for C in (64, 256, 1024, 2304):
        x = (3.0 * rng.standard_normal((11, C))).astype(np.float32)
        q1, s1 = oracle.quantize_rows(x)
        q2, s2 = reflib.quantize_rows(x)
        assert np.array_equal(q1, q2) and np.array_equal(s1, s2)
    L = np.array([3, 1, 40, 9], np.int32)
    x, r, b, taps = cases.conv_case(C=1024, k=3, seed=4, lengths=L)
    assert np.array_equal(oracle.lily_state(x, r, b, taps, L), reflib.lily_state(x, r, b, taps, L))
    assert np.array_equal(oracle.dwconv(x, r, taps, L), reflib.dwconv(x, r, taps, L))


def test_live_whole_model_segments_and_layers(oracle, reflib):
    hp = sm.tiny_hparams(n_types=2, ssmax_mode="ssmax", ntk_train_len=64)
    path = sm.cached_model("tiny_seg", hp, "Q5_K_M", seed=4)
    m = oracle.load(path)
    h = reflib.load(path, 4)
    L = np.array([200], np.int32)          # beyond ntk_train_len: dynamic NTK base stretch
    tok = sm.random_tokens(200, hp.n_vocab, seed=1)
    types = (np.arange(200) >= 100).astype(np.int32)
    ho, po = m.encode(tok, L, types=types)
    hr, pr = reflib.encode(h, tok, L, types=types)
    assert np.array_equal(ho, hr) and np.array_equal(po, pr)
    reflib.L.nextera_debug_set_layers(h, 2)
    ho, _ = m.encode(tok, L, types=types, n_layers=2)
    hr, _ = reflib.encode(h, tok, L, types=types)
    assert np.array_equal(ho, hr)
    reflib.L.nextera_free(h)
    m.close()
