"""One rank of the sharded-encode GPU test (tests/test_gpu_shard.py), run in its own process.

The rank encodes its part of the sequence with nextera_encode_sharded and, on the same GPU, the
whole sequence with nextera_encode_device; it reports whether its rows and the pooled vector are
bit-identical.
"""
from __future__ import annotations


def run(rank: int, world: int, model_path: str, nccl_id: bytes, tokens, out_q) -> None:
    import ctypes

    import numpy as np
    import torch

    from gpulib import load_lib

    try:
        torch.cuda.set_device(rank)
        L = load_lib()
        p = L.nextera_default_params()
        h = L.nextera_load(model_path.encode(), p)
        if not h:
            out_q.put((rank, "error", "nextera_load failed"))
            return
        C = L.nextera_n_embd(h)
        n_total = len(tokens)
        n_local = n_total // world
        rc = L.nextera_shard_init(h, rank, world, nccl_id)
        if rc != 0:
            out_q.put((rank, "error", f"shard_init {rc}"))
            return
        stream = torch.cuda.current_stream().cuda_stream
        tok = torch.tensor(np.asarray(tokens, np.int32), device="cuda")
        hid = torch.empty((n_local, C), device="cuda")
        pooled = torch.empty(C, device="cuda")
        rc = L.nextera_encode_sharded(h, ctypes.c_void_p(tok[rank * n_local:].data_ptr()), n_local, n_total,
                                      ctypes.c_void_p(hid.data_ptr()), ctypes.c_void_p(pooled.data_ptr()), 1,
                                      ctypes.c_void_p(stream))
        torch.cuda.synchronize()
        if rc != 0:
            out_q.put((rank, "error", f"encode_sharded {rc}"))
            return
        hid_all = torch.empty((n_total, C), device="cuda")
        pooled_all = torch.empty(C, device="cuda")
        lens = (ctypes.c_int32 * 1)(n_total)
        rc = L.nextera_encode_device(h, ctypes.c_void_p(tok.data_ptr()), None, lens, 1,
                                     ctypes.c_void_p(hid_all.data_ptr()), ctypes.c_void_p(pooled_all.data_ptr()), 1,
                                     ctypes.c_void_p(stream))
        torch.cuda.synchronize()
        if rc != 0:
            out_q.put((rank, "error", f"encode_device {rc}"))
            return
        a = hid.cpu().numpy()
        b = hid_all[rank * n_local:(rank + 1) * n_local].cpu().numpy()
        pa, pb = pooled.cpu().numpy(), pooled_all.cpu().numpy()
        out_q.put((rank, "ok", bool(np.array_equal(a, b)), float(np.max(np.abs(a - b))),
                   bool(np.array_equal(pa, pb)), float(np.max(np.abs(pa - pb)))))
        L.nextera_free(h)
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, "error", repr(e)))


def run_partitioned(rank: int, world: int, model_path: str, nccl_id: bytes, tokens, lengths, out_q) -> None:
    """One rank of the partitioned-batch GPU test (tests/test_gpu_partition.py): the batch split over
    the ranks with nextera_encode_partitioned (host arrays) and nextera_encode_partitioned_device
    (this rank's ids on its GPU); rank 0 also encodes the whole batch alone and reports whether the
    gathered pooled rows are bit-identical to it."""
    import ctypes

    import numpy as np
    import torch

    from gpulib import load_lib

    try:
        torch.cuda.set_device(rank)
        L = load_lib()
        h = L.nextera_load(model_path.encode(), L.nextera_default_params())
        if not h:
            out_q.put((rank, "error", "nextera_load failed"))
            return
        C = L.nextera_n_embd(h)
        tok = np.ascontiguousarray(tokens, np.int32)
        lens = np.ascontiguousarray(lengths, np.int32)
        n = len(lens)
        i32 = ctypes.POINTER(ctypes.c_int32)
        f32 = ctypes.POINTER(ctypes.c_float)
        rc = L.nextera_shard_init(h, rank, world, nccl_id)
        if rc != 0:
            out_q.put((rank, "error", f"shard_init {rc}"))
            return
        got = np.full((n, C), np.nan, np.float32)
        rc = L.nextera_encode_partitioned(h, tok.ctypes.data_as(i32), None, lens.ctypes.data_as(i32), n,
                                          got.ctypes.data_as(f32) if rank == 0 else None, 1)
        if rc != 0:
            out_q.put((rank, "error", f"encode_partitioned {rc}"))
            return
        # the device variant: this rank's ids only, in batch order
        part = np.empty(n, np.int32)
        assert L.nextera_partition(h, lens.ctypes.data_as(i32), n, world, part.ctypes.data_as(i32)) == 0
        start = np.concatenate([[0], np.cumsum(lens)])
        mine = np.concatenate([tok[start[i]:start[i + 1]] for i in range(n) if part[i] == rank] or
                              [np.zeros(0, np.int32)])
        d_tok = torch.from_numpy(np.ascontiguousarray(mine, np.int32)).cuda() if len(mine) else \
            torch.zeros(1, dtype=torch.int32, device="cuda")
        d_pool = torch.full((n, C), float("nan"), device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        rc = L.nextera_encode_partitioned_device(h, ctypes.c_void_p(d_tok.data_ptr()), lens.ctypes.data_as(i32), n,
                                                 ctypes.c_void_p(d_pool.data_ptr()), 1, ctypes.c_void_p(stream))
        torch.cuda.synchronize()
        if rc != 0:
            out_q.put((rank, "error", f"encode_partitioned_device {rc}"))
            return
        if rank == 0:
            want = np.empty((n, C), np.float32)
            rc = L.nextera_encode(h, tok.ctypes.data_as(i32), lens.ctypes.data_as(i32), n, None,
                                  want.ctypes.data_as(f32), 1)
            if rc != 0:
                out_q.put((rank, "error", f"encode {rc}"))
                return
            dev_rows = d_pool.cpu().numpy()
            out_q.put((rank, "ok", bool(np.array_equal(got, want)), float(np.nanmax(np.abs(got - want))),
                       bool(np.array_equal(dev_rows, want)), float(np.nanmax(np.abs(dev_rows - want))),
                       [int(np.sum(part == r)) for r in range(world)]))
        else:
            out_q.put((rank, "ok", True, 0.0, True, 0.0, []))
        L.nextera_free(h)
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, "error", repr(e)))
