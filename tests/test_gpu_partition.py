"""One batch of sequences partitioned over GPUs (nextera_partition / nextera_encode_partitioned*).

The reference's batch contract (src/nexterabert.h:69-84) says a sequence's result does not depend
on the rest of the batch, so the sequences of one batch may run on different GPUs.  Checked here:
  * the partition covers every sequence and balances the estimated device time;
  * on one GPU, the parts encoded separately and put back in batch order are bit-identical to the
    whole batch, through the host and the device entry points;
  * on 2, 4 and 8 GPUs (one process each, NCCL), rank 0's gathered pooled rows are bit-identical
    to the whole batch on one GPU (skipped when the box has fewer GPUs).
"""
from __future__ import annotations

import ctypes
import multiprocessing as mp

import numpy as np
import pytest

import cases
import synth_model as sm

pytestmark = pytest.mark.gpu
i32 = ctypes.POINTER(ctypes.c_int32)
f32 = ctypes.POINTER(ctypes.c_float)


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.fixture(scope="module")
def lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpulib import load_lib
    return load_lib()


def doc_cost(L: int, blocks, half=128, qt=64, hra=4) -> float:
    """Restatement of the library's cost estimate (tokens + 3.9e-4 x attention tile-keys)."""
    tiles = -(-L // qt)
    keys = 0.0
    for bt in blocks:
        if bt == "swa":
            for i in range(tiles):
                q0, q1 = i * qt, min(L, i * qt + qt)
                keys += qt * (min(L, q1 + half) - max(0, q0 - half))
        elif bt == "attn":
            keys += tiles * qt * L
        elif bt == "hra":
            nb = -(-L // hra)
            keys += -(-nb // qt) * qt * nb
    return L + 3.9e-4 * keys


def test_partition_balances_the_mixed_length_batch(lib):
    path = sm.cached_model("full", sm.full_hparams(), "Q4_K_M", seed=0)
    h = lib.nextera_load(str(path).encode(), lib.nextera_default_params())
    assert h
    lens = np.ascontiguousarray(sm.throughput_lengths(4096, 16, 2048, seed=0), np.int32)
    cost = np.array([doc_cost(int(x), sm.FULL_BLOCKS) for x in lens])
    for parts in (1, 2, 4, 8):
        part = np.full(len(lens), -1, np.int32)
        assert lib.nextera_partition(h, lens.ctypes.data_as(i32), len(lens), parts, part.ctypes.data_as(i32)) == 0
        assert part.min() == 0 and part.max() == parts - 1
        load = np.array([cost[part == r].sum() for r in range(parts)])
        assert load.max() <= 1.002 * load.mean(), load / load.mean()
        again = np.empty_like(part)
        lib.nextera_partition(h, lens.ctypes.data_as(i32), len(lens), parts, again.ctypes.data_as(i32))
        assert np.array_equal(part, again)
    bad = np.array([5, 0], np.int32)
    assert lib.nextera_partition(h, bad.ctypes.data_as(i32), 2, 2, part.ctypes.data_as(i32)) == 1
    lib.nextera_free(h)


def test_parts_encoded_separately_match_the_whole_batch(lib):
    import torch
    path = sm.cached_model("tiny", sm.tiny_hparams(), "Q4_K_M", seed=0)
    h = lib.nextera_load(str(path).encode(), lib.nextera_default_params())
    assert h
    C = lib.nextera_n_embd(h)
    tok, lens = cases.model_batch(1000, seed=7)
    tok = np.ascontiguousarray(tok, np.int32)
    lens = np.ascontiguousarray(lens, np.int32)
    n = len(lens)
    want = np.empty((n, C), np.float32)
    assert lib.nextera_encode(h, tok.ctypes.data_as(i32), lens.ctypes.data_as(i32), n, None,
                              want.ctypes.data_as(f32), 1) == 0
    start = np.concatenate([[0], np.cumsum(lens)])
    for parts in (2, 3, 8):
        part = np.empty(n, np.int32)
        assert lib.nextera_partition(h, lens.ctypes.data_as(i32), n, parts, part.ctypes.data_as(i32)) == 0
        got = np.full((n, C), np.nan, np.float32)
        for r in range(parts):
            idx = np.flatnonzero(part == r)
            if len(idx) == 0:
                continue
            t = np.ascontiguousarray(np.concatenate([tok[start[i]:start[i + 1]] for i in idx]), np.int32)
            ln = np.ascontiguousarray(lens[idx], np.int32)
            out = np.empty((len(idx), C), np.float32)
            assert lib.nextera_encode(h, t.ctypes.data_as(i32), ln.ctypes.data_as(i32), len(idx), None,
                                      out.ctypes.data_as(f32), 1) == 0
            got[idx] = out
        assert np.array_equal(got, want), parts
    # without a shard group the partitioned entry points run the whole batch here
    got = np.full((n, C), np.nan, np.float32)
    assert lib.nextera_encode_partitioned(h, tok.ctypes.data_as(i32), None, lens.ctypes.data_as(i32), n,
                                          got.ctypes.data_as(f32), 1) == 0
    assert np.array_equal(got, want)
    d_tok = torch.from_numpy(tok).cuda()
    d_pool = torch.full((n, C), float("nan"), device="cuda")
    rc = lib.nextera_encode_partitioned_device(h, ctypes.c_void_p(d_tok.data_ptr()), lens.ctypes.data_as(i32), n,
                                               ctypes.c_void_p(d_pool.data_ptr()), 1,
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == 0
    assert np.array_equal(d_pool.cpu().numpy(), want)
    lib.nextera_free(h)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_partitioned_over_ranks_matches_one_gpu(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    from gpulib import load_lib, shard_id
    import shard_worker

    path = sm.cached_model("full", sm.full_hparams(), "Q4_K_M", seed=0)
    lens = sm.throughput_lengths(96, 16, 2048, seed=3)
    tokens = sm.random_tokens(int(lens.sum()), 50368, seed=12)
    L = load_lib()
    nid = shard_id(L, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=shard_worker.run_partitioned,
                         args=(r, world, str(path), nid, tokens.tolist(), lens.tolist(), q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=900))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join()
    for r in sorted(results):
        assert r[1] == "ok", r
        if r[0] == 0:
            _, _, host_eq, host_diff, dev_eq, dev_diff, counts = r
            assert sum(counts) == len(lens) and min(counts) > 0, counts
            assert host_eq, f"host entry point: gathered rows differ (max |diff| {host_diff})"
            assert dev_eq, f"device entry point: gathered rows differ (max |diff| {dev_diff})"
