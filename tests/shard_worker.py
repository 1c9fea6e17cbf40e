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
