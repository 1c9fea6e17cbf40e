"""GPU kernels against the CPU oracle, one kernel at a time (needs a B200).

Bar: bit-identical for everything integer and for every fp32 row op (they
perform the reference's operations in the reference's order).  Attention also
follows the reference's order; its softmax tail exp is correctly rounded where
the reference calls glibc's expf, so it must be within 1e-4 of the output's
largest magnitude (the configuration's bar) and bit-identical almost everywhere.
"""
import ctypes

import numpy as np
import pytest

import cases
import synth_model as sm
from gguf import GGMLQuantizationType as QT

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpulib import Ops, load_lib
    return Ops(load_lib())


def test_library_reports_no_error(ops):
    assert ops.L.nxk_take_error(None) == 0


@pytest.mark.parametrize("i,qt", list(enumerate(cases.WEIGHT_TYPES + [QT.Q2_K, QT.Q3_K])))
def test_expand_weight_bit_exact(ops, oracle, i, qt):
    if qt in (QT.Q2_K, QT.Q3_K):
        rng = np.random.default_rng(i)
        nbytes = {QT.Q2_K: 84, QT.Q3_K: 110}[qt]
        raw = rng.integers(0, 256, (64 * 2, nbytes), dtype=np.uint8)
        for p in ([80, 82] if qt == QT.Q2_K else [108]):
            raw[:, p:p + 2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
        blocks, n_in, n_out = raw.reshape(64, -1), 512, 64
    else:
        blocks, n_in, n_out = cases.weight_case(qt, seed=i)
    w, sc, off = ops.expand_weight(int(qt), blocks, n_in, n_out)
    w2, sc2, off2 = oracle.build_i8_weight(int(qt), blocks, n_in, n_out)
    assert np.array_equal(w, w2)
    assert np.array_equal(sc, sc2)
    assert np.array_equal(off, off2)


def test_expand_weight_k64_and_full_rows(ops, oracle):
    # a 64-input weight (one partial block, Q5_0 as in Q4_K_M's ltc_conv.out_proj) and 2304 inputs
    for qt, n_in, n_out in ((QT.Q5_0, 64, 1024), (QT.Q6_K, 2304, 128), (QT.Q4_K, 1024, 2304)):
        w = (0.02 * np.random.default_rng(n_in).standard_normal((n_out, n_in))).astype(np.float32)
        blocks = sm.quantize_rows(w, qt)
        a = ops.expand_weight(int(qt), blocks, n_in, n_out)
        b = oracle.build_i8_weight(int(qt), blocks, n_in, n_out)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)


@pytest.mark.parametrize("name", list(cases.LINEAR_CASES))
def test_linear_bit_exact(ops, oracle, name):
    T, K, N, qt, resid, seed = cases.LINEAR_CASES[name]
    x, blocks, qt_, res = cases.linear_case(T, K, N, seed=seed, qt=qt, residual=resid)
    w, sw, _ = oracle.build_i8_weight(int(qt_), blocks, K, N)
    xq, xs = oracle.quantize_rows(x)
    want, bs = oracle.linear_i8(xq, xs, w, sw, res, block_sums=True)
    assert np.array_equal(ops.block_sums(xq, w), bs)            # int32 block dot products
    got = ops.linear(xq, xs, w, sw, res)
    assert np.array_equal(got, want), f"max diff {np.abs(got - want).max()}"
    assert np.array_equal(ops.linear(xq, xs, w, sw, res, simt=True), want)


def test_cfg1_linear_bit_exact(ops, oracle):
    """Config 1: X [128, 1024], W [4096, 1024] in Q8_0."""
    x, wb = cases.cfg1_case()
    w, sw, _ = oracle.build_i8_weight(int(QT.Q8_0), wb, 1024, 4096)
    xq, xs = oracle.quantize_rows(x)
    want, bs = oracle.linear_i8(xq, xs, w, sw, None, block_sums=True)
    assert np.array_equal(ops.block_sums(xq, w), bs)
    got = ops.linear(xq, xs, w, sw)
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= 1e-5
    assert np.array_equal(got, want)


@pytest.mark.parametrize("T,K,N", [(1, 1024, 64), (129, 64, 1024), (300, 2304, 1024), (1000, 1024, 2304),
                                   (4097, 1024, 512)])
def test_linear_shapes(ops, oracle, T, K, N):
    rng = np.random.default_rng(T + K + N)
    x = rng.standard_normal((T, K)).astype(np.float32)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    res = rng.standard_normal((T, N)).astype(np.float32)
    w8, sw, _ = oracle.build_i8_weight(int(QT.Q8_0), sm.quantize_rows(w, QT.Q8_0), K, N)
    xq, xs = oracle.quantize_rows(x)
    want = oracle.linear_i8(xq, xs, w8, sw, res)
    assert np.array_equal(ops.linear(xq, xs, w8, sw, res), want)


@pytest.mark.parametrize("T,K,N", [(1, 256, 256), (300, 1024, 512), (129, 2304, 1024), (1000, 1024, 2304),
                                   (4097, 1024, 256)])
def test_linear_fused_row_op_quantize_bit_exact(ops, oracle, T, K, N):
    """linear + relu^2 + quantize and linear + gate + quantize in one kernel: the codes and scales of the
    separate ops (rows past the last full tile, a single row, 1 to 9 quantization blocks)"""
    import torch
    from gpulib import P, dev, host, stream_ptr
    rng = np.random.default_rng(7 * T + K + N)
    x = rng.standard_normal((T, K)).astype(np.float32)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    z = rng.standard_normal((T, N)).astype(np.float32)
    w8, sw, _ = oracle.build_i8_weight(int(QT.Q8_0), sm.quantize_rows(w, QT.Q8_0), K, N)
    xq, xs = oracle.quantize_rows(x)
    y = oracle.linear_i8(xq, xs, w8, sw, None)
    args = [P(dev(xq)), P(dev(xs)), T, P(dev(w8)), P(dev(sw)), K, N]
    for name, want_v, extra in (("nxk_linear_i8_relu_sqr_q", oracle.relu_sqr(y), []),
                                ("nxk_linear_i8_gate_q", oracle.gate(y, z), [P(dev(z))])):
        q, sq = ops.quant_out(T, N)
        q.fill_(0x55)
        sq.fill_(float("nan"))
        ops._ok(getattr(ops.L, name)(*args, *extra, P(q), P(sq), stream_ptr()), name)
        wq, ws = oracle.quantize_rows(want_v)
        gq, gs = host(q), host(sq)
        assert np.array_equal(gq, wq), f"{name}: {np.count_nonzero(gq != wq)} codes differ"
        assert np.array_equal(gs, ws), f"{name}: scales differ"


@pytest.mark.parametrize("C", [512, 352])
def test_quantize_and_row_ops_bit_exact(ops, oracle, C):
    """C = 352: a partial last 256-column block"""
    from gpulib import P, dev
    xr = cases.rows_case(C=C)
    T, C = xr.shape
    gain = (1.0 + 0.05 * np.random.default_rng(5).standard_normal(C)).astype(np.float32)
    qq, ss = ops.quant_out(T, C)
    ops._ok(ops.L.nxk_quantize(P(dev(xr)), T, C, P(qq), P(ss), None), "quantize")
    from gpulib import host
    want_q, want_s = oracle.quantize_rows(xr)
    assert np.array_equal(host(qq), want_q) and np.array_equal(host(ss), want_s)

    want = oracle.rms_norm(xr, gain, 1e-8)
    assert np.array_equal(ops.rows("nxk_rms_norm", [P(dev(xr)), P(dev(gain)), 1e-8, T, C], T, C, False), want)
    q, s = ops.rows("nxk_rms_norm", [P(dev(xr)), P(dev(gain)), 1e-8, T, C], T, C, True)
    wq, ws = oracle.quantize_rows(want)
    assert np.array_equal(q, wq) and np.array_equal(s, ws)

    want = oracle.relu_sqr(xr)
    assert np.array_equal(ops.rows("nxk_relu_sqr", [P(dev(xr)), T, C], T, C, False), want)
    q, s = ops.rows("nxk_relu_sqr", [P(dev(xr)), T, C], T, C, True)
    wq, ws = oracle.quantize_rows(want)
    assert np.array_equal(q, wq) and np.array_equal(s, ws)

    g = cases.rows_case(C=C, seed=9)
    want = oracle.gate(g, xr)
    assert np.array_equal(ops.rows("nxk_gate", [P(dev(g)), P(dev(xr)), T, C], T, C, False), want)
    q, s = ops.rows("nxk_gate", [P(dev(g)), P(dev(xr)), T, C], T, C, True)
    wq, ws = oracle.quantize_rows(want)
    assert np.array_equal(q, wq) and np.array_equal(s, ws)


@pytest.mark.parametrize("C,k", [(256, 5), (64, 5), (1024, 3), (32, 5), (128, 3), (64, 7)])
def test_conv_ops_bit_exact(ops, oracle, C, k):
    from gpulib import P, dev
    L = cases.LENGTHS_SMALL
    x, r, b, taps = cases.conv_case(C=C, k=k, seed=C + k)
    start, ln, rd = ops.layout(L)
    T = int(L.sum())
    lay = [P(dev(rd)), P(dev(start)), P(dev(ln))]
    want = oracle.dwconv(x, r, taps, L)
    assert np.array_equal(ops.rows("nxk_dwconv", [P(dev(x)), P(dev(r)), P(dev(taps)), k, *lay, T, C], T, C, False), want)
    want = oracle.dwconv(x, None, taps, L)
    q, s = ops.rows("nxk_dwconv", [P(dev(x)), None, P(dev(taps)), k, *lay, T, C], T, C, True)
    wq, ws = oracle.quantize_rows(want)
    assert np.array_equal(q, wq) and np.array_equal(s, ws)
    want = oracle.lily_state(x, r, b, taps, L)
    assert np.array_equal(ops.rows("nxk_lily_state", [P(dev(x)), P(dev(r)), P(dev(b)), P(dev(taps)), k, *lay, T, C],
                                   T, C, False), want)
    # x and r as the two column ranges of one [T][2C] matrix, as the fused in_proj | A linear writes them
    xr = dev(np.ascontiguousarray(np.concatenate([x, r], axis=1)))
    px, pr = ctypes.c_void_p(xr.data_ptr()), ctypes.c_void_p(xr.data_ptr() + 4 * C)
    args = [px, pr, 2 * C, P(dev(taps)), k, 0, *lay, T, C]
    want = oracle.dwconv(x, r, taps, L)
    assert np.array_equal(ops.rows("nxk_dwconv_halo_ld", args, T, C, False), want)
    q, s = ops.rows("nxk_dwconv_halo_ld", args, T, C, True)
    wq, ws = oracle.quantize_rows(want)
    assert np.array_equal(q, wq) and np.array_equal(s, ws)


@pytest.mark.parametrize("C,k", [(64, 5), (256, 5), (128, 7)])
def test_conv_halo_shard_bit_exact(ops, oracle, C, k):
    """One shard of a longer document, as the sharded path runs it on one GPU: rows [off, off + T)
    of a document of Ltot rows, the document starting before row 0 (start = -off) and the inputs
    holding the halo rows around the shard; the outputs equal the whole document's rows."""
    from gpulib import P, dev
    Ltot, off, T = 300, 100, 100
    h = k // 2
    x, r, b, taps = cases.conv_case(C=C, k=k, seed=3 * C + k, lengths=np.array([Ltot], np.int32))
    lay = [P(dev(np.zeros(T, np.int32))), P(dev(np.array([-off], np.int32))), P(dev(np.array([Ltot], np.int32)))]
    dx, dr, db, dt = dev(x), dev(r), dev(b), dev(taps)
    row = lambda t: ctypes.c_void_p(t.data_ptr() + 4 * off * t.shape[1])          # row `off` of a matrix
    want = oracle.dwconv(x, r, taps, [Ltot])[off:off + T]
    got = ops.rows("nxk_dwconv_halo", [row(dx), row(dr), P(dt), k, h, *lay, T, C], T, C, False)
    assert np.array_equal(got, want)
    # the strided entry point: x and r side by side in one [Ltot][2C] matrix
    xr = dev(np.ascontiguousarray(np.concatenate([x, r], axis=1)))
    px = ctypes.c_void_p(xr.data_ptr() + 4 * off * 2 * C)
    got = ops.rows("nxk_dwconv_halo_ld", [px, ctypes.c_void_p(px.value + 4 * C), 2 * C, P(dt), k, h, *lay, T, C],
                   T, C, False)
    assert np.array_equal(got, want)
    want = oracle.lily_state(x, r, b, taps, [Ltot])[off:off + T]
    got = ops.rows("nxk_lily_state_halo", [row(dx), row(dr), row(db), P(dt), k, h, *lay, T, C], T, C, False)
    assert np.array_equal(got, want)


def test_qk_prep_and_head_major_bit_exact(ops, oracle):
    import torch
    from gpulib import P, dev, host
    L = cases.LENGTHS_SMALL
    x, alpha, beta = cases.qk_case()
    T = x.shape[0]
    start, ln, rd = ops.layout(L)
    for base, hm in ((100000.0, 0), (10000.0, 1)):
        c, s = oracle.rope_table(int(L.max()), base, 64)
        out = torch.empty((4, T, 64) if hm else (T, 256), dtype=torch.float32, device="cuda")
        ops._ok(ops.L.nxk_qk_prep(P(dev(x)), P(dev(alpha)), P(dev(beta)), P(dev(c)), P(dev(s)), P(dev(rd)),
                                  P(dev(start)), T, 4, 64, hm, P(out), None), "qk_prep")
        assert np.array_equal(host(out), oracle.qk_prep(x, alpha, beta, base, L, 4, 64, hm))
    out = torch.empty((4, T, 64), dtype=torch.float32, device="cuda")
    ops._ok(ops.L.nxk_head_major(P(dev(x)), T, 4, 64, P(out), None), "head_major")
    assert np.array_equal(host(out), oracle.head_major(x, 4, 64))


def test_qkv_prep_bit_exact(ops, oracle):
    """the fused q/k/v pass equals qk_prep (q token-major, k head-major) and head_major on the split columns"""
    import torch
    from gpulib import P, dev, host
    L = cases.LENGTHS_SMALL
    T = int(L.sum())
    H, G, D = 4, 2, 64
    rng = np.random.default_rng(77)
    x = rng.standard_normal((T, (H + 2 * G) * D)).astype(np.float32)
    qa, qb, ka, kb = (rng.uniform(0.2, 1.5, D).astype(np.float32) for _ in range(4))
    start, ln, rd = ops.layout(L)
    base = 10000.0
    c, s = oracle.rope_table(int(L.max()), base, D)
    q = torch.empty((T, H * D), dtype=torch.float32, device="cuda")
    k = torch.empty((G, T, D), dtype=torch.float32, device="cuda")
    v = torch.empty((G, T, D), dtype=torch.float32, device="cuda")
    ops._ok(ops.L.nxk_qkv_prep(P(dev(x)), x.shape[1], P(dev(qa)), P(dev(qb)), P(dev(ka)), P(dev(kb)), P(dev(c)),
                               P(dev(s)), P(dev(rd)), P(dev(start)), T, H, G, D, P(q), P(k), P(v), None), "qkv_prep")
    xq = np.ascontiguousarray(x[:, :H * D])
    xk = np.ascontiguousarray(x[:, H * D:(H + G) * D])
    xv = np.ascontiguousarray(x[:, (H + G) * D:])
    assert np.array_equal(host(q), oracle.qk_prep(xq, qa, qb, base, L, H, D, 0))
    assert np.array_equal(host(k), oracle.qk_prep(xk, ka, kb, base, L, G, D, 1))
    assert np.array_equal(host(v), oracle.head_major(xv, G, D))
    # the sharded layout: k and v at rows koff .. koff + T - 1 of buffers of Tk rows per head, the
    # rows around them (halo or other shards' rows) left as they were
    koff, Tk = 5, T + 9
    q2 = torch.empty((T, H * D), dtype=torch.float32, device="cuda")
    k2 = torch.full((G, Tk, D), 7.0, dtype=torch.float32, device="cuda")
    v2 = torch.full((G, Tk, D), 7.0, dtype=torch.float32, device="cuda")
    ops._ok(ops.L.nxk_qkv_prep_kv(P(dev(x)), x.shape[1], P(dev(qa)), P(dev(qb)), P(dev(ka)), P(dev(kb)), P(dev(c)),
                                  P(dev(s)), P(dev(rd)), P(dev(start)), T, H, G, D, Tk, koff, P(q2), P(k2), P(v2),
                                  None), "qkv_prep_kv")
    assert np.array_equal(host(q2), host(q))
    for got, want in ((host(k2), host(k)), (host(v2), host(v))):
        assert np.array_equal(got[:, koff:koff + T], want)
        assert np.all(got[:, :koff] == 7.0) and np.all(got[:, koff + T:] == 7.0)


def test_hra_ops_bit_exact(ops, oracle):
    from gpulib import P, dev
    L = cases.LENGTHS_SMALL
    x, r, b, _ = cases.conv_case()
    C = x.shape[1]
    start, ln, rd = ops.layout(L)
    nb = (ln + 3) // 4
    bstart, _, brd = ops.layout(nb)
    NB = int(nb.sum())
    args = [P(dev(x)), P(dev(b)), C, 4, P(dev(start)), P(dev(ln)), P(dev(bstart)), P(dev(brd)), NB]
    want = oracle.block_mean(x, b, L, 4)
    assert np.array_equal(ops.rows("nxk_block_mean", args, NB, C, False), want)
    q, s = ops.rows("nxk_block_mean", args, NB, C, True)
    wq, ws = oracle.quantize_rows(want)
    assert np.array_equal(q, wq) and np.array_equal(s, ws)
    y = oracle.block_mean(x, None, L, 4)
    want = oracle.upsample_add(y, r, L, 4)
    import torch
    from gpulib import host
    out = torch.empty_like(dev(r))
    ops._ok(ops.L.nxk_upsample_add(P(dev(y)), P(dev(r)), C, 4, int(L.sum()), P(dev(rd)), P(dev(start)),
                                   P(dev(bstart)), P(out), None), "upsample")
    assert np.array_equal(host(out), want)


def run_attention(ops, q, k, v, H, G, half, scale, lengths):
    import torch
    from gpulib import P, dev, host
    T = q.shape[0]
    start, ln, rd = ops.layout(lengths)
    ws_bytes = ops.L.nxk_attention_workspace(ln.ctypes.data_as(ops.L.nxk_attention_workspace.argtypes[0]),
                                             len(ln), half)
    ws = torch.empty(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    out = torch.empty((T, H * 64), dtype=torch.float32, device="cuda")
    i32 = ops.L.nxk_attention.argtypes[13]
    ops._ok(ops.L.nxk_attention(P(dev(q)), P(dev(k)), P(dev(v)), T, H, G, 64, half, P(dev(np.asarray(scale, np.float32))),
                                P(dev(rd)), P(dev(start)), P(dev(ln)), len(ln), start.ctypes.data_as(i32),
                                ln.ctypes.data_as(i32), P(ws), ws.numel(), P(out), None), "attention")
    return host(out)


@pytest.mark.parametrize("half", [8, -1])
def test_attention_vs_oracle(ops, oracle, half):
    q, k, v, scale = cases.attn_case()
    got = run_attention(ops, q, k, v, 4, 2, half, scale, cases.LENGTHS_ATTN)
    want = oracle.attention(q, k, v, 4, 2, 64, half, scale, cases.LENGTHS_ATTN)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-4, err
    same = float(np.mean(got == want))
    print(f"attention half={half}: max rel err {err:.2e}, bit-identical fraction {same:.6f}")
    assert same >= 0.999


@pytest.mark.parametrize("half", [64, -1])
def test_cfg2_attention(ops, oracle, half):
    """Config 2 shapes: 64 documents, lengths U[16, 2048], H=16, G=4, D=64; swa window 128 and global."""
    lengths = sm.uniform_lengths(64, 16, 2048, seed=0)
    T = int(lengths.sum())
    assert T == 67328
    rng = np.random.default_rng(2)
    q = rng.standard_normal((T, 16 * 64)).astype(np.float32)
    k = rng.standard_normal((4, T, 64)).astype(np.float32)
    v = rng.standard_normal((4, T, 64)).astype(np.float32)
    scale = np.full(64, 0.125, np.float32)
    got = run_attention(ops, q, k, v, 16, 4, half, scale, lengths)
    # the scalar oracle checks a sample of documents (the whole set takes minutes on one core)
    start, _, _ = ops.layout(lengths)
    for d in (0, 7, int(np.argmax(lengths)), 63):
        s0, n = int(start[d]), int(lengths[d])
        want = oracle.attention(q[s0:s0 + n], np.ascontiguousarray(k[:, s0:s0 + n]),
                                np.ascontiguousarray(v[:, s0:s0 + n]), 16, 4, 64, half, scale[d:d + 1],
                                np.array([n], np.int32))
        err = np.abs(got[s0:s0 + n] - want).max() / np.abs(want).max()
        assert err <= 1e-4, (d, err)
        assert float(np.mean(got[s0:s0 + n] == want)) >= 0.999, d


@pytest.mark.parametrize("half", [8, -1])
def test_attention_on_a_shard_matches_the_whole_document(ops, half):
    """One shard of a long document on one GPU, as the sharded path runs it: query rows [off, off + T)
    of a document of Ltot rows (off not a multiple of the 64-query tile), the document starting before
    query row 0, with K / V gathered from the whole document (global: Tk = Ltot, koff = off) or a
    halo-extended slice of it (band: Tk = T + 2 half, koff = half).  Bit-identical to the same rows of
    the whole document through nxk_attention, which the tests above check against the oracle."""
    import torch
    from gpulib import P, dev, host
    rng = np.random.default_rng(21)
    H, G, D = 4, 2, 64
    Ltot, off, T = 700, 250, 192
    q = rng.standard_normal((Ltot, H * D)).astype(np.float32)
    k = rng.standard_normal((G, Ltot, D)).astype(np.float32)
    v = rng.standard_normal((G, Ltot, D)).astype(np.float32)
    scale = np.full(1, 0.125, np.float32)
    whole = run_attention(ops, q, k, v, H, G, half, scale, np.array([Ltot], np.int32))
    if half < 0:
        Tk, koff, ks, vs = Ltot, off, k, v
    else:
        Tk, koff = T + 2 * half, half
        ks = np.ascontiguousarray(k[:, off - half:off + T + half])
        vs = np.ascontiguousarray(v[:, off - half:off + T + half])
    hs, hl = np.array([-off], np.int32), np.array([Ltot], np.int32)
    i32 = ops.L.nxk_attention_kv.argtypes[14]
    ws_bytes = int(ops.L.nxk_attention_workspace(hl.ctypes.data_as(i32), 1, half))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    out = torch.empty((T, H * D), dtype=torch.float32, device="cuda")
    dq, dk, dv = dev(np.ascontiguousarray(q[off:off + T])), dev(ks), dev(vs)
    ops._ok(ops.L.nxk_attention_kv(P(dq), P(dk), P(dv), T, Tk, koff, H, G, D, half, P(dev(scale)), P(dev(hs)),
                                   P(dev(hl)), 1, hs.ctypes.data_as(i32), hl.ctypes.data_as(i32), P(ws), ws.numel(),
                                   P(out), None), "attention_kv")
    assert np.array_equal(host(out), whole[off:off + T])


def test_pool_over_shards_matches_the_whole(ops, oracle):
    """The pooled sum carried over three shards in order (nxk_pool_continue), then nxk_pool_finish,
    equals pooling the whole document, bit for bit."""
    import torch
    from gpulib import P, dev, host
    rng = np.random.default_rng(12)
    n, C = 300, 256
    x = rng.standard_normal((n, C)).astype(np.float32)
    dx = dev(x)
    for normalize in (0, 1):
        pooled = torch.zeros(C, dtype=torch.float32, device="cuda")
        for a, b in ((0, 100), (100, 250), (250, n)):
            ops._ok(ops.L.nxk_pool_continue(ctypes.c_void_p(dx.data_ptr() + 4 * a * C), b - a, C, P(pooled), None),
                    "pool_continue")
        ops._ok(ops.L.nxk_pool_finish(n, C, normalize, P(pooled), None), "pool_finish")
        assert np.array_equal(host(pooled), oracle.pool(x, np.array([n], np.int32), normalize)[0])


def test_layer_norm_and_pool(ops, oracle):
    import torch
    from gpulib import P, dev, host
    rng = np.random.default_rng(11)
    L = cases.LENGTHS_SMALL
    T, C = int(L.sum()), 256
    x = rng.standard_normal((T, C)).astype(np.float32)
    w = rng.standard_normal(C).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    out = torch.empty((T, C), dtype=torch.float32, device="cuda")
    ops._ok(ops.L.nxk_layer_norm(P(dev(x)), P(dev(w)), P(dev(b)), 1e-5, T, C, P(out), None), "layer_norm")
    want = oracle.layer_norm(x, w, b, 1e-5)
    assert np.abs(host(out) - want).max() <= 1e-6 * np.abs(want).max()
    start, ln, _ = ops.layout(L)
    for normalize in (0, 1):
        pooled = torch.empty((len(L), C), dtype=torch.float32, device="cuda")
        ops._ok(ops.L.nxk_pool(P(dev(x)), P(dev(start)), P(dev(ln)), len(L), C, normalize, P(pooled), None), "pool")
        assert np.array_equal(host(pooled), oracle.pool(x, L, normalize))


def test_embed_bit_exact(ops, oracle):
    import torch
    from gpulib import P, dev, host
    C, V = 256, 50
    rng = np.random.default_rng(3)
    table = (0.02 * rng.standard_normal((V, C))).astype(np.float32)
    types_t = (0.02 * rng.standard_normal((2, C))).astype(np.float32)
    tok = rng.integers(0, V, 37).astype(np.int32)
    ty = rng.integers(0, 2, 37).astype(np.int32)
    for qt in (QT.Q4_K, QT.Q8_0, QT.Q6_K):
        blocks = sm.quantize_rows(table, qt)
        out = torch.empty((37, C), dtype=torch.float32, device="cuda")
        ops._ok(ops.L.nxk_embed(int(qt), P(dev(blocks.reshape(-1))), V, C, P(dev(tok)), 37, 0, P(dev(types_t)), 2,
                                P(dev(ty)), P(out), None), "embed")
        deq = sm.dequantize_rows(blocks, qt, C)
        assert np.array_equal(host(out), deq[tok] + types_t[ty])
    # an id outside the table: zero row and the device error word, no read past the table
    bad = tok.copy()
    bad[5] = V + 3
    out = torch.empty((37, C), dtype=torch.float32, device="cuda")
    rc = ops.L.nxk_embed(int(QT.Q8_0), P(dev(sm.quantize_rows(table, QT.Q8_0).reshape(-1))), V, C, P(dev(bad)), 37,
                         0, None, 0, None, P(out), None)
    assert rc == 0
    assert ops.L.nxk_take_error(None) != 0
    assert np.all(host(out)[5] == 0)


def test_bounded_wait_reports_timeout(ops, oracle):
    """A pipeline wait that runs out ends the kernel with an error word, not a hang; the context
    stays usable (the GEMM after it is still bit-exact)."""
    L = ops.L
    assert L.nxk_take_error(None) == 0
    assert L.nxk_selftest_wait(0, None) != 0                     # limits outside (0, 1 s] are refused
    assert L.nxk_selftest_wait(20_000_000, None) == 0            # 20 ms on an mbarrier nothing completes
    assert L.nxk_take_error(None) == 0x1FF
    assert L.nxk_take_error(None) == 0                           # reading clears it
    rng = np.random.default_rng(3)
    x = rng.standard_normal((300, 1024)).astype(np.float32)
    w = (0.02 * rng.standard_normal((512, 1024))).astype(np.float32)
    w8, sw, _ = oracle.build_i8_weight(int(QT.Q8_0), sm.quantize_rows(w, QT.Q8_0), 1024, 512)
    xq, xs = oracle.quantize_rows(x)
    assert np.array_equal(ops.linear(xq, xs, w8, sw), oracle.linear_i8(xq, xs, w8, sw))
