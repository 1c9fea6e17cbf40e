"""nxk_attention_noalloc: attention for callers that cannot allocate device memory.

Some hosts of this library hand it device pointers from a pool they manage
themselves and forbid cudaMalloc once serving has started; others run on a path
where an allocation that may block is not allowed.  For them the library
offers one attention entry point that takes no workspace and allocates
nothing: its work plan lives in a fixed array compiled into the library.  This
file checks it through the C ABI against nxk_attention (which takes a
workspace) on two calls in a row, to the attention tolerance the other tests
use, and that a batch beyond the fixed array's capacity is refused.  It sits
last in collection order so a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu

TOL = 1e-4           # attention bar: max |diff| over max |reference output|


@pytest.fixture(scope="module")
def lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpulib import load_lib
    L = load_lib()
    L.nxk_attention_noalloc.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [ctypes.c_void_p] * 3 + \
        [ctypes.c_int, ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p, ctypes.c_void_p]
    L.nxk_attention_noalloc.restype = ctypes.c_int
    return L


def _inputs(seed, lengths, H, G):
    rng = np.random.default_rng(seed)
    T = int(lengths.sum())
    q = rng.standard_normal((T, H * 64)).astype(np.float32)
    k = rng.standard_normal((G, T, 64)).astype(np.float32)
    v = rng.standard_normal((G, T, 64)).astype(np.float32)
    scale = (0.125 * (1.0 + 0.2 * rng.random(len(lengths)))).astype(np.float32)
    return q, k, v, scale


def _run_both(L, q, k, v, scale, lengths, H, G, half):
    import torch
    from gpulib import P, dev, host
    T = q.shape[0]
    lengths = np.ascontiguousarray(lengths, np.int32)
    start = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
    row_doc = np.repeat(np.arange(len(lengths), dtype=np.int32), lengths).astype(np.int32)
    i32 = ctypes.POINTER(ctypes.c_int32)
    dq, dk, dv, ds = dev(q), dev(k), dev(v), dev(scale)
    dstart, dlen, drow = dev(start), dev(lengths), dev(row_doc)
    # the existing entry point, with its workspace
    ws_bytes = int(L.nxk_attention_workspace(lengths.ctypes.data_as(i32), len(lengths), half))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    want = torch.empty((T, H * 64), dtype=torch.float32, device="cuda")
    rc = L.nxk_attention(P(dq), P(dk), P(dv), T, H, G, 64, half, P(ds), P(drow), P(dstart), P(dlen), len(lengths),
                         start.ctypes.data_as(i32), lengths.ctypes.data_as(i32), P(ws), ws.numel(), P(want), None)
    assert rc == 0
    got = torch.full((T, H * 64), float("nan"), dtype=torch.float32, device="cuda")
    rc = L.nxk_attention_noalloc(P(dq), P(dk), P(dv), T, H, G, 64, half, P(ds), P(dstart), P(dlen), len(lengths),
                                 lengths.ctypes.data_as(i32), P(got), None)
    assert rc == 0
    assert L.nxk_take_error(None) == 0
    return host(got), host(want)


def test_no_alloc_matches_workspace_entry_point_twice(lib):
    # two calls in a row on different batches: the second reuses the fixed plan array
    for seed, lengths, H, G, half in ((1, cases.LENGTHS_ATTN, 4, 2, 8),
                                      (2, np.array([700, 3, 64, 129, 1], np.int32), 16, 4, -1)):
        q, k, v, scale = _inputs(seed, lengths, H, G)
        got, want = _run_both(lib, q, k, v, scale, lengths, H, G, half)
        assert np.all(np.isfinite(got))
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err <= TOL, err


def test_no_alloc_rejects_batches_beyond_its_fixed_plan(lib):
    lengths = np.full(131073, 1, np.int32)        # one tile more than the plan holds
    i32 = ctypes.POINTER(ctypes.c_int32)
    rc = lib.nxk_attention_noalloc(None, None, None, int(lengths.sum()), 4, 2, 64, -1, None, None, None,
                                   len(lengths), lengths.ctypes.data_as(i32), None, None)
    assert rc == -1


def test_no_alloc_accepts_exactly_its_fixed_plan(lib):
    # 131072 one-row documents fill the plan exactly; a one-key softmax weighs its value row by 1,
    # so every output row is the value row of its KV head
    from gpulib import P, dev, host
    import torch
    H, G, n = 4, 2, 131072
    lengths = np.ones(n, np.int32)
    rng = np.random.default_rng(7)
    q = rng.standard_normal((n, H * 64)).astype(np.float32)
    k = rng.standard_normal((G, n, 64)).astype(np.float32)
    v = rng.standard_normal((G, n, 64)).astype(np.float32)
    scale = np.full(n, 0.125, np.float32)
    start = np.arange(n, dtype=np.int32)
    i32 = ctypes.POINTER(ctypes.c_int32)
    out = torch.full((n, H * 64), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.nxk_attention_noalloc(P(dev(q)), P(dev(k)), P(dev(v)), n, H, G, 64, -1, P(dev(scale)), P(dev(start)),
                                   P(dev(lengths)), n, lengths.ctypes.data_as(i32), P(out), None)
    assert rc == 0
    assert lib.nxk_take_error(None) == 0
    got = host(out).reshape(n, H, 64)
    for h in range(H):
        assert np.array_equal(got[:, h], v[h // (H // G)])


def test_no_alloc_rejects_documents_past_T(lib):
    # the documents hold 10 rows but T says 9: refused on the host, nothing launched
    lengths = np.array([4, 6], np.int32)
    i32 = ctypes.POINTER(ctypes.c_int32)
    rc = lib.nxk_attention_noalloc(None, None, None, 9, 4, 2, 64, -1, None, None, None, len(lengths),
                                   lengths.ctypes.data_as(i32), None, None)
    assert rc == -1


def test_no_alloc_device_lengths_that_disagree_set_the_error_word(lib):
    # the device copy of the lengths asks for more tiles than the host copy counted: the planner
    # writes empty entries, the output stays untouched and the error word reports it
    from gpulib import P, dev, host
    import torch
    H, G = 4, 2
    h_len = np.array([40, 30], np.int32)
    d_len = np.array([40, 70], np.int32)          # 70 rows would run past T = 70
    T = int(h_len.sum())
    q, k, v, scale = _inputs(3, h_len, H, G)
    start = np.array([0, 40], np.int32)
    i32 = ctypes.POINTER(ctypes.c_int32)
    out = torch.full((T, H * 64), 7.0, dtype=torch.float32, device="cuda")
    rc = lib.nxk_attention_noalloc(P(dev(q)), P(dev(k)), P(dev(v)), T, H, G, 64, -1, P(dev(scale)), P(dev(start)),
                                   P(dev(d_len)), 2, h_len.ctypes.data_as(i32), P(out), None)
    assert rc == 0
    assert lib.nxk_take_error(None) == 0x301
    assert np.all(host(out) == 7.0)
    # the next, consistent call plans and runs normally
    got, want = _run_both(lib, q, k, v, scale, h_len, H, G, -1)
    assert np.abs(got - want).max() <= TOL * np.abs(want).max()
