"""ctypes access to libnexterabert.so for the tests (kernel layer + public API).

Device buffers come from torch (plumbing only); every computation runs in the
library's own kernels, called through its C ABI (include/nextera_kernels.h,
include/nexterabert.h).
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "nexterabert.cpp_b200"
LIB_PATH = PKG / "libnexterabert.so"

vp, c_int, c_float, c_size = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
i32p = ctypes.POINTER(ctypes.c_int32)
f32p = ctypes.POINTER(ctypes.c_float)


def header_symbols():
    """Every function declared in include/*.h, plus the reference's unexported-but-bound debug symbols."""
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names.update(re.findall(r"NEXTERA_API\s+[\w\s\*]+?\b((?:nextera|nxk)_\w+)\s*\(", text))
    return sorted(names)


class Params(ctypes.Structure):
    _fields_ = [("n_threads", ctypes.c_int32), ("use_int8", ctypes.c_int32),
                ("use_repack", ctypes.c_int32), ("verbosity", ctypes.c_int32)]


def load_lib(path=None):
    path = Path(path) if path else LIB_PATH
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run __graft_entry__.build())")
    L = ctypes.CDLL(str(path))
    sig = {
        "nxk_take_error": ([vp], ctypes.c_int32),
        "nxk_selftest_wait": ([ctypes.c_int64, vp], c_int),
        "nxk_i8_mma_rate_probe": ([c_int, c_int, vp], c_int),
        "nxk_expand_weight": ([c_int, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_embed": ([c_int, vp, c_int, c_int, vp, c_int, c_int, vp, c_int, vp, vp, vp], c_int),
        "nxk_linear_i8": ([vp, vp, c_int, vp, vp, c_int, c_int, vp, vp, vp], c_int),
        "nxk_linear_i8_simt": ([vp, vp, c_int, vp, vp, c_int, c_int, vp, vp, vp], c_int),
        "nxk_block_sums": ([vp, c_int, vp, c_int, c_int, vp, vp], c_int),
        "nxk_linear_i8_relu_sqr_q": ([vp, vp, c_int, vp, vp, c_int, c_int, vp, vp, vp], c_int),
        "nxk_linear_i8_gate_q": ([vp, vp, c_int, vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_quantize": ([vp, c_int, c_int, vp, vp, vp], c_int),
        "nxk_rms_norm": ([vp, vp, c_float, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_relu_sqr": ([vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_gate": ([vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_dwconv": ([vp, vp, vp, c_int, vp, vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_lily_state": ([vp, vp, vp, vp, c_int, vp, vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_dwconv_halo_ld": ([vp, vp, c_int, vp, c_int, c_int, vp, vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_dwconv_halo": ([vp, vp, vp, c_int, c_int, vp, vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_lily_state_halo": ([vp, vp, vp, vp, c_int, c_int, vp, vp, vp, c_int, c_int, vp, vp, vp, vp], c_int),
        "nxk_qk_prep": ([vp, vp, vp, vp, vp, vp, vp, c_int, c_int, c_int, c_int, vp, vp], c_int),
        "nxk_head_major": ([vp, c_int, c_int, c_int, vp, vp], c_int),
        "nxk_qkv_prep": ([vp, c_int, vp, vp, vp, vp, vp, vp, vp, vp, c_int, c_int, c_int, c_int, vp, vp, vp, vp],
                         c_int),
        "nxk_qkv_prep_kv": ([vp, c_int, vp, vp, vp, vp, vp, vp, vp, vp, c_int, c_int, c_int, c_int, c_int, c_int, vp, vp,
                             vp, vp], c_int),
        "nxk_block_mean": ([vp, vp, c_int, c_int, vp, vp, vp, vp, c_int, vp, vp, vp, vp], c_int),
        "nxk_upsample_add": ([vp, vp, c_int, c_int, c_int, vp, vp, vp, vp, vp], c_int),
        "nxk_layer_norm": ([vp, vp, vp, c_float, c_int, c_int, vp, vp], c_int),
        "nxk_pool": ([vp, vp, vp, c_int, c_int, c_int, vp, vp], c_int),
        "nxk_pool_continue": ([vp, c_int, c_int, vp, vp], c_int),
        "nxk_pool_finish": ([c_int, c_int, c_int, vp, vp], c_int),
        "nxk_attention_kv": ([vp, vp, vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, vp, vp, vp, c_int, i32p, i32p,
                              vp, c_size, vp, vp], c_int),
        "nxk_attention_workspace": ([i32p, c_int, c_int], c_size),
        "nxk_attention": ([vp, vp, vp, c_int, c_int, c_int, c_int, c_int, vp, vp, vp, vp, c_int, i32p, i32p,
                           vp, c_size, vp, vp], c_int),
        "nxk_gelu_norm": ([vp, vp, c_float, c_int, c_int, vp, vp], c_int),
        "nxk_gather_rows": ([vp, c_int, vp, c_int, vp, vp], c_int),
        "nxk_mul_mat_workspace": ([c_int, c_int, c_int], c_size),
        "nxk_mul_mat": ([c_int, vp, c_int, c_int, vp, c_int, vp, vp, vp, vp], c_int),
        "nextera_default_params": ([], Params),
        "nextera_load": ([ctypes.c_char_p, Params], vp),
        "nextera_free": ([vp], None),
        "nextera_n_embd": ([vp], ctypes.c_int32),
        "nextera_n_vocab": ([vp], ctypes.c_int32),
        "nextera_n_layer": ([vp], ctypes.c_int32),
        "nextera_encode": ([vp, i32p, i32p, ctypes.c_int32, f32p, f32p, ctypes.c_int32], ctypes.c_int32),
        "nextera_encode_segments": ([vp, i32p, i32p, i32p, ctypes.c_int32, f32p, f32p, ctypes.c_int32],
                                    ctypes.c_int32),
        "nextera_encode_device": ([vp, vp, vp, i32p, ctypes.c_int32, vp, vp, ctypes.c_int32, vp], ctypes.c_int32),
        "nextera_system_info": ([vp], ctypes.c_char_p),
        "nextera_n_labels": ([vp], ctypes.c_int32),
        "nextera_has_pooler": ([vp], ctypes.c_int32),
        "nextera_has_mlm_head": ([vp], ctypes.c_int32),
        "nextera_classifier_task": ([vp], ctypes.c_char_p),
        "nextera_pooler_output": ([vp, i32p, i32p, i32p, ctypes.c_int32, f32p], ctypes.c_int32),
        "nextera_classify": ([vp, i32p, i32p, i32p, ctypes.c_int32, f32p], ctypes.c_int32),
        "nextera_mlm_logits": ([vp, i32p, ctypes.c_int32, i32p, ctypes.c_int32, f32p], ctypes.c_int32),
        "nextera_ftype": ([vp], ctypes.c_char_p),
        "nextera_last_ms": ([vp], ctypes.c_double),
        "nextera_debug_set_layers": ([vp, ctypes.c_int32], None),
        "nextera_debug_profile": ([vp, ctypes.c_int32], None),
        "nextera_debug_profile_print": ([vp], None),
        "nextera_debug_launches": ([vp], ctypes.c_int64),
        "nextera_debug_profile_get": ([vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)],
                                      ctypes.c_int64),
        "nextera_shard_unique_id": ([ctypes.c_char_p], ctypes.c_int32),
        "nextera_shard_init": ([vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_char_p], ctypes.c_int32),
        "nextera_encode_sharded": ([vp, vp, ctypes.c_int32, ctypes.c_int32, vp, vp, ctypes.c_int32, vp],
                                   ctypes.c_int32),
        "nextera_partition": ([vp, i32p, ctypes.c_int32, ctypes.c_int32, i32p], ctypes.c_int32),
        "nextera_quantize": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int32,
                              ctypes.POINTER(ctypes.c_char_p)], ctypes.c_int32),
        "nxk_quantize_rows": ([c_int, vp, ctypes.c_int64, ctypes.c_int64, vp, vp], c_int),
        "nextera_encode_partitioned": ([vp, i32p, i32p, i32p, ctypes.c_int32, f32p, ctypes.c_int32],
                                       ctypes.c_int32),
        "nextera_encode_partitioned_device": ([vp, vp, i32p, ctypes.c_int32, vp, ctypes.c_int32, vp],
                                              ctypes.c_int32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes, fn.restype = args, res
    return L


def shard_id(L, rank: int, dist=None) -> bytes:
    """The 128-byte NCCL id of a sharded group: made by rank 0 through the library, handed to the
    other ranks over `dist` (torch.distributed, any backend) when given."""
    buf = ctypes.create_string_buffer(128)
    if rank == 0:
        rc = L.nextera_shard_unique_id(buf)
        if rc != 0:
            raise RuntimeError(f"nextera_shard_unique_id returned {rc}")
    if dist is not None:
        import torch
        t = torch.frombuffer(bytearray(buf.raw), dtype=torch.uint8).clone()
        if dist.get_backend() == "nccl":
            t = t.cuda()
        dist.broadcast(t, 0)
        return bytes(t.cpu().numpy().tobytes())
    return buf.raw


# -- torch plumbing -------------------------------------------------------------

# Device copies made by dev() stay referenced here until the test ends
# (tests/conftest.py releases them), so a raw pointer taken from a temporary
# tensor is never recycled by torch's caching allocator while still in use.
_KEEP: list = []


def dev(a: np.ndarray):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def release():
    import torch
    torch.cuda.synchronize()
    _KEEP.clear()


def empty(shape, dtype):
    import torch
    return torch.empty(shape, dtype=dtype, device="cuda")


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def host(t) -> np.ndarray:
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def stream_ptr():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class Ops:
    """The kernel layer on numpy inputs (host -> device -> kernel -> host)."""

    def __init__(self, L):
        self.L = L

    def _ok(self, rc, what):
        assert rc == 0, f"{what} returned {rc}"
        err = self.L.nxk_take_error(stream_ptr())
        assert err == 0, f"{what}: device error word {err:#x}"

    def expand_weight(self, qtype, blocks, n_in, n_out):
        import torch
        n_blk = (n_in + 255) // 256
        b = dev(np.ascontiguousarray(blocks).view(np.uint8).reshape(-1))
        w = empty((n_out, n_in), torch.int8)
        sc = empty((n_blk, n_out), torch.float32)
        off = empty((n_blk, n_out), torch.int32)
        self._ok(self.L.nxk_expand_weight(int(qtype), P(b), n_in, n_out, P(w), P(sc), P(off), stream_ptr()), "expand")
        return host(w), host(sc), host(off)

    def quant_out(self, T, C):
        import torch
        return empty((T, C), torch.int8), empty((T, (C + 255) // 256), torch.float32)

    def linear(self, xq, sx, w, sw, res=None, simt=False):
        import torch
        T, K = xq.shape
        N = w.shape[0]
        out = empty((T, N), torch.float32)
        out.fill_(float("nan"))             # every output must be written
        fn = self.L.nxk_linear_i8_simt if simt else self.L.nxk_linear_i8
        self._ok(fn(P(dev(xq)), P(dev(sx)), T, P(dev(w)), P(dev(sw)), K, N, P(None if res is None else dev(res)),
                    P(out), stream_ptr()), "linear")
        return host(out)

    def block_sums(self, xq, w):
        import torch
        T, K = xq.shape
        N = w.shape[0]
        s = empty((T, N, (K + 255) // 256), torch.int32)
        self._ok(self.L.nxk_block_sums(P(dev(xq)), T, P(dev(w)), K, N, P(s), stream_ptr()), "block_sums")
        return host(s)

    def rows(self, fn_name, args, T, C, quant):
        import torch
        if quant:
            q, sx = self.quant_out(T, C)
            self._ok(getattr(self.L, fn_name)(*args, None, P(q), P(sx), stream_ptr()), fn_name)
            return host(q), host(sx)
        out = empty((T, C), torch.float32)
        self._ok(getattr(self.L, fn_name)(*args, P(out), None, None, stream_ptr()), fn_name)
        return host(out)

    @staticmethod
    def layout(lengths):
        lengths = np.asarray(lengths, np.int32)
        start = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
        row_doc = np.repeat(np.arange(len(lengths), dtype=np.int32), lengths).astype(np.int32)
        return start, lengths, row_doc
