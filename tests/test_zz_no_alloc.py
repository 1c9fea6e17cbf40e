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
