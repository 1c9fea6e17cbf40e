"""ctypes access to the CPU checkers (test infrastructure).

* ``Oracle``  -- oracle/liboracle.so, the C restatement of the reference's arithmetic.
* ``RefLib``  -- oracle/_ref/libnexterabert_ref_*.so, the reference's own
  src/nexterabert.cpp compiled here against the ggml stand-in; it exports the
  reference's C API and op-level entry points (oracle/ref_ops.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this module.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"

f32p = ctypes.POINTER(ctypes.c_float)
i32p = ctypes.POINTER(ctypes.c_int32)
i8p = ctypes.POINTER(ctypes.c_int8)
vp = ctypes.c_void_p
c_int, c_float = ctypes.c_int, ctypes.c_float


def ptr(a, t=None):
    if a is None:
        return None
    if t is None:
        t = {np.float32: ctypes.c_float, np.int32: ctypes.c_int32, np.int8: ctypes.c_int8,
             np.uint8: ctypes.c_uint8}[a.dtype.type]
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(t))


def default_ref_dir() -> Path:
    """The reference checkout: $REF_DIR, else a sibling of this repository named `reference`."""
    env = os.environ.get("REF_DIR")
    return Path(env) if env else ORACLE_DIR.parent.parent / "reference"


def build_oracle(ref: bool = False) -> None:
    """Runs oracle/Makefile (the reference build only when its sources exist)."""
    import subprocess
    targets = ["all"]
    ref_dir = os.environ.get("REF_DIR") or str(default_ref_dir())
    if ref and Path(ref_dir, "src", "nexterabert.cpp").exists():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), f"REF_DIR={ref_dir}", *targets], check=True)


def cpu_flags() -> set:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def ref_library_path() -> Path | None:
    """The reference build matching this host's int8 ISA, or None."""
    flags = cpu_flags()
    cands = []
    if "avx_vnni" in flags:
        cands.append(ORACLE_DIR / "_ref" / "libnexterabert_ref_avxvnni.so")
    if {"avx512_vnni", "avx512vl"} <= flags:
        cands.append(ORACLE_DIR / "_ref" / "libnexterabert_ref_avx512vnni.so")
    for c in cands:
        if c.exists():
            return c
    return None


class Oracle:
    def __init__(self, path: str | os.PathLike | None = None):
        path = Path(path) if path else ORACLE_DIR / "liboracle.so"
        if not path.exists():
            build_oracle()
        L = ctypes.CDLL(str(path))
        self.L = L
        L.or_load.restype = vp
        L.or_load.argtypes = [ctypes.c_char_p]
        L.or_free.argtypes = [vp]
        L.or_n_embd.argtypes = [vp]
        L.or_encode.argtypes = [vp, i32p, i32p, i32p, c_int, f32p, f32p, c_int, c_int]
        L.or_get_i8.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                ctypes.POINTER(i8p), ctypes.POINTER(f32p), ctypes.POINTER(i32p)]
        L.or_exp8.restype = c_float
        L.or_exp8.argtypes = [c_float]
        L.or_tanh8.restype = c_float
        L.or_tanh8.argtypes = [c_float]
        L.or_sigmoid8.restype = c_float
        L.or_sigmoid8.argtypes = [c_float]
        L.or_dot_f32.restype = c_float
        L.or_dot_f32.argtypes = [f32p, f32p, c_int]
        L.or_dequant_row.argtypes = [c_int, vp, f32p, ctypes.c_int64]
        L.or_build_i8_weight.argtypes = [c_int, vp, c_int, c_int, i8p, f32p, i32p]
        L.or_quantize_rows.argtypes = [f32p, c_int, c_int, i8p, f32p]
        L.or_linear_i8.argtypes = [i8p, f32p, c_int, i8p, f32p, c_int, c_int, f32p, f32p, i32p]
        L.or_rms_norm.argtypes = [f32p, f32p, c_float, c_int, c_int, f32p]
        L.or_relu_sqr.argtypes = [f32p, c_int, c_int, f32p]
        L.or_gate.argtypes = [f32p, f32p, c_int, c_int, f32p]
        L.or_dwconv.argtypes = [f32p, f32p, f32p, c_int, i32p, i32p, i32p, c_int, c_int, f32p]
        L.or_lily_state.argtypes = [f32p, f32p, f32p, f32p, c_int, i32p, i32p, i32p, c_int, c_int, f32p]
        L.or_qk_prep.argtypes = [f32p, f32p, f32p, f32p, f32p, i32p, i32p, c_int, c_int, c_int, c_int, f32p]
        L.or_head_major.argtypes = [f32p, c_int, c_int, c_int, f32p]
        L.or_block_mean.argtypes = [f32p, f32p, c_int, c_int, i32p, i32p, i32p, i32p, c_int, f32p]
        L.or_upsample_add.argtypes = [f32p, f32p, c_int, c_int, c_int, i32p, i32p, i32p, f32p]
        L.or_attention.argtypes = [f32p, f32p, f32p, c_int, c_int, c_int, c_int, c_int, f32p, i32p, i32p, i32p, f32p]
        L.or_layer_norm.argtypes = [f32p, f32p, f32p, c_float, c_int, c_int, f32p]
        L.or_pool.argtypes = [f32p, i32p, c_int, c_int, c_int, f32p]
        L.or_rope_table.argtypes = [c_int, c_float, c_int, f32p, f32p]
        L.or_set_threads.argtypes = [c_int]
        L.or_act_bytes.restype = ctypes.c_size_t
        L.or_act_bytes.argtypes = [c_int, ctypes.c_int64]
        L.or_quantize_act.argtypes = [c_int, f32p, ctypes.c_int64, vp]
        L.or_mul_mat.argtypes = [c_int, vp, ctypes.c_int64, ctypes.c_int64, f32p, ctypes.c_int64, f32p]
        L.or_gelu_erf.argtypes = [f32p, ctypes.c_int64, f32p]

    # -- ops -----------------------------------------------------------------
    def dequant_row(self, qtype: int, data: np.ndarray, n: int) -> np.ndarray:
        y = np.empty(n, np.float32)
        rc = self.L.or_dequant_row(qtype, data.ctypes.data, ptr(y), n)
        assert rc == 0
        return y

    def build_i8_weight(self, qtype: int, data: np.ndarray, n_in: int, n_out: int):
        n_blk = (n_in + 255) // 256
        w = np.empty((n_out, n_in), np.int8)
        sc = np.empty((n_blk, n_out), np.float32)
        off = np.empty((n_blk, n_out), np.int32)
        rc = self.L.or_build_i8_weight(qtype, np.ascontiguousarray(data).ctypes.data, n_in, n_out,
                                       ptr(w), ptr(sc), ptr(off))
        assert rc == 0
        return w, sc, off

    def quantize_rows(self, x: np.ndarray):
        T, C = x.shape
        n_blk = (C + 255) // 256
        q = np.empty((T, C), np.int8)
        sx = np.empty((T, n_blk), np.float32)
        self.L.or_quantize_rows(ptr(x), T, C, ptr(q), ptr(sx))
        return q, sx

    def linear_i8(self, xq, sx, w, sw, res=None, block_sums=False):
        T, K = xq.shape
        N = w.shape[0]
        n_blk = (K + 255) // 256
        out = np.empty((T, N), np.float32)
        bs = np.empty((T, N, n_blk), np.int32) if block_sums else None
        self.L.or_linear_i8(ptr(xq), ptr(sx), T, ptr(w), ptr(sw), K, N, ptr(res), ptr(out), ptr(bs))
        return (out, bs) if block_sums else out

    def rms_norm(self, x, gain, eps):
        T, C = x.shape
        out = np.empty_like(x)
        self.L.or_rms_norm(ptr(x), ptr(gain), eps, T, C, ptr(out))
        return out

    def relu_sqr(self, x):
        out = np.empty_like(x)
        self.L.or_relu_sqr(ptr(x), x.shape[0], x.shape[1], ptr(out))
        return out

    def gate(self, g, y):
        out = np.empty_like(g)
        self.L.or_gate(ptr(g), ptr(y), g.shape[0], g.shape[1], ptr(out))
        return out

    @staticmethod
    def layout(lengths):
        lengths = np.asarray(lengths, np.int32)
        start = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
        row_doc = np.repeat(np.arange(len(lengths), dtype=np.int32), lengths).astype(np.int32)
        return start, lengths, row_doc

    def dwconv(self, x, r, taps, lengths):
        T, C = x.shape
        start, ln, rd = self.layout(lengths)
        out = np.empty_like(x)
        self.L.or_dwconv(ptr(x), ptr(r), ptr(taps), taps.shape[0], ptr(rd), ptr(start), ptr(ln), T, C, ptr(out))
        return out

    def lily_state(self, a, x, b, taps, lengths):
        T, C = x.shape
        start, ln, rd = self.layout(lengths)
        out = np.empty_like(x)
        self.L.or_lily_state(ptr(a), ptr(x), ptr(b), ptr(taps), taps.shape[0], ptr(rd), ptr(start), ptr(ln),
                             T, C, ptr(out))
        return out

    def rope_table(self, n_pos, base, D):
        c = np.empty((n_pos, D // 2), np.float32)
        s = np.empty((n_pos, D // 2), np.float32)
        self.L.or_rope_table(n_pos, base, D, ptr(c), ptr(s))
        return c, s

    def qk_prep(self, x, alpha, beta, base, lengths, H, D, head_major):
        T = x.shape[0]
        start, ln, rd = self.layout(lengths)
        c, s = self.rope_table(int(max(lengths)), base, D)
        out = np.empty((H, T, D) if head_major else (T, H * D), np.float32)
        self.L.or_qk_prep(ptr(x), ptr(alpha), ptr(beta), ptr(c), ptr(s), ptr(rd), ptr(start), T, H, D,
                          int(head_major), ptr(out))
        return out

    def head_major(self, x, H, D):
        T = x.shape[0]
        out = np.empty((H, T, D), np.float32)
        self.L.or_head_major(ptr(x), T, H, D, ptr(out))
        return out

    def block_mean(self, h, g, lengths, block):
        T, C = h.shape
        start, ln, rd = self.layout(lengths)
        nb = (ln + block - 1) // block
        bstart, _, brd = self.layout(nb)
        out = np.empty((int(nb.sum()), C), np.float32)
        self.L.or_block_mean(ptr(h), ptr(g), C, block, ptr(start), ptr(ln), ptr(bstart), ptr(brd),
                             int(nb.sum()), ptr(out))
        return out

    def upsample_add(self, y, r, lengths, block):
        T, C = r.shape
        start, ln, rd = self.layout(lengths)
        nb = (ln + block - 1) // block
        bstart, _, _ = self.layout(nb)
        out = np.empty_like(r)
        self.L.or_upsample_add(ptr(y), ptr(r), C, block, T, ptr(rd), ptr(start), ptr(bstart), ptr(out))
        return out

    def attention(self, q, k, v, H, G, D, half, scale, lengths):
        T = q.shape[0]
        start, ln, rd = self.layout(lengths)
        out = np.empty((T, H * D), np.float32)
        self.L.or_attention(ptr(q), ptr(k), ptr(v), T, H, G, D, half, ptr(np.asarray(scale, np.float32)),
                            ptr(rd), ptr(start), ptr(ln), ptr(out))
        return out

    def act_bytes(self, qtype: int, K: int) -> int:
        return int(self.L.or_act_bytes(qtype, K))

    def quantize_act(self, qtype: int, x: np.ndarray) -> np.ndarray:
        """Rows of x in the weight type's vec_dot type (oracle/vecdot.c layout), one row per line."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, x.shape[-1])
        K = x.shape[1]
        out = np.zeros((x.shape[0], self.act_bytes(qtype, K)), np.uint8)
        for m in range(x.shape[0]):
            assert self.L.or_quantize_act(qtype, ptr(x[m]), K, out[m].ctypes.data) == 0
        return out

    def mul_mat(self, qtype: int, w: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
        """ggml_mul_mat: out[m][n] = W[n] . x[m], W in GGUF blocks of qtype."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty((x.shape[0], N), np.float32)
        assert self.L.or_mul_mat(qtype, np.ascontiguousarray(w).ctypes.data, N, K, ptr(x), x.shape[0], ptr(out)) == 0
        return out

    def gelu_erf(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.L.or_gelu_erf(ptr(x), x.size, ptr(out))
        return out

    def layer_norm(self, x, w, b, eps):
        out = np.empty_like(x)
        self.L.or_layer_norm(ptr(x), ptr(w), ptr(b), eps, x.shape[0], x.shape[1], ptr(out))
        return out

    def pool(self, hidden, lengths, normalize):
        lengths = np.asarray(lengths, np.int32)
        C = hidden.shape[1]
        out = np.empty((len(lengths), C), np.float32)
        self.L.or_pool(ptr(hidden), ptr(lengths), len(lengths), C, int(normalize), ptr(out))
        return out

    # -- model ---------------------------------------------------------------
    def load(self, path) -> "OracleModel":
        h = self.L.or_load(str(path).encode())
        if not h:
            raise RuntimeError(f"oracle failed to load {path}")
        return OracleModel(self, h)


class OracleModel:
    def __init__(self, o: Oracle, h):
        self.o, self.h = o, h
        self.n_embd = o.L.or_n_embd(h)

    def close(self):
        if self.h:
            self.o.L.or_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, tokens, lengths, types=None, normalize=True, hidden=True, n_layers=-1):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lengths = np.ascontiguousarray(lengths, np.int32)
        types = None if types is None else np.ascontiguousarray(types, np.int32)
        T = int(lengths.sum())
        hid = np.empty((T, self.n_embd), np.float32) if hidden else None
        pooled = np.empty((len(lengths), self.n_embd), np.float32)
        rc = self.o.L.or_encode(self.h, ptr(tokens), ptr(types), ptr(lengths), len(lengths), ptr(hid),
                                ptr(pooled), int(normalize), n_layers)
        if rc != 0:
            raise RuntimeError(f"or_encode failed ({rc})")
        return hid, pooled

    def i8(self, name: str):
        n_in, n_out = c_int(), c_int()
        w, s, o = i8p(), f32p(), i32p()
        if self.o.L.or_get_i8(self.h, name.encode(), ctypes.byref(n_in), ctypes.byref(n_out),
                              ctypes.byref(w), ctypes.byref(s), ctypes.byref(o)) != 0:
            return None
        n_blk = (n_in.value + 255) // 256
        W = np.ctypeslib.as_array(w, (n_out.value, n_in.value)).copy()
        S = np.ctypeslib.as_array(s, (n_blk, n_out.value)).copy()
        O = np.ctypeslib.as_array(o, (n_blk, n_out.value)).copy()
        return W, S, O


class RefLib:
    """The reference's own code (oracle/_ref): C API plus op-level entry points."""

    def __init__(self, path=None):
        path = Path(path) if path else ref_library_path()
        if path is None or not path.exists():
            raise FileNotFoundError("oracle/_ref is not built for this host")
        L = ctypes.CDLL(str(path))
        self.L = L
        self.path = path
        L.ref_act_max.restype = c_int
        L.ref_build_i8_weight.argtypes = [c_int, vp, c_int, c_int, i8p, f32p, i32p]
        L.ref_quantize_rows.argtypes = [f32p, c_int, c_int, i8p, f32p]
        L.ref_linear_i8.argtypes = [i8p, f32p, c_int, i8p, f32p, i32p, c_int, c_int, f32p, f32p]
        L.ref_rms_norm.argtypes = [f32p, f32p, c_float, c_int, c_int, f32p, i8p, f32p]
        L.ref_relu_sqr.argtypes = [f32p, c_int, c_int, f32p, i8p, f32p]
        L.ref_gate.argtypes = [f32p, f32p, c_int, c_int, f32p, i8p, f32p]
        L.ref_dwconv.argtypes = [f32p, f32p, f32p, c_int, i32p, c_int, c_int, f32p, i8p, f32p]
        L.ref_lily_state.argtypes = [f32p, f32p, f32p, f32p, c_int, i32p, c_int, c_int, f32p, i8p, f32p]
        L.ref_qk_prep.argtypes = [f32p, f32p, f32p, c_float, i32p, c_int, c_int, c_int, c_int, f32p]
        L.ref_rope_table.argtypes = [c_int, c_float, c_int, f32p, f32p]
        L.ref_head_major.argtypes = [f32p, c_int, c_int, c_int, f32p]
        L.ref_block_mean.argtypes = [f32p, f32p, c_int, c_int, i32p, c_int, f32p, i8p, f32p]
        L.ref_upsample_add.argtypes = [f32p, f32p, c_int, c_int, i32p, c_int, f32p]
        L.ref_attention.argtypes = [f32p, f32p, f32p, c_int, c_int, c_int, c_int, f32p, i32p, c_int, f32p]
        # the reference's public API (src/nexterabert.h)
        class Params(ctypes.Structure):
            _fields_ = [("n_threads", ctypes.c_int32), ("use_int8", ctypes.c_int32),
                        ("use_repack", ctypes.c_int32), ("verbosity", ctypes.c_int32)]
        self.Params = Params
        L.nextera_default_params.restype = Params
        L.nextera_load.restype = vp
        L.nextera_load.argtypes = [ctypes.c_char_p, Params]
        L.nextera_free.argtypes = [vp]
        L.nextera_n_embd.argtypes = [vp]
        L.nextera_encode_segments.argtypes = [vp, i32p, i32p, i32p, c_int, f32p, f32p, c_int]
        L.nextera_encode_segments.restype = ctypes.c_int32
        L.nextera_debug_set_layers.argtypes = [vp, c_int]
        L.nextera_set_n_threads.argtypes = [vp, c_int]
        L.nextera_get_n_threads.argtypes = [vp]
        L.nextera_last_ms.argtypes = [vp]
        L.nextera_last_ms.restype = ctypes.c_double
        L.nextera_system_info.argtypes = [vp]
        L.nextera_system_info.restype = ctypes.c_char_p
        L.nextera_n_vocab.argtypes = [vp]
        L.nextera_n_labels.argtypes = [vp]
        L.nextera_classifier_task.argtypes = [vp]
        L.nextera_classifier_task.restype = ctypes.c_char_p
        L.nextera_pooler_output.argtypes = [vp, i32p, i32p, i32p, c_int, f32p]
        L.nextera_classify.argtypes = [vp, i32p, i32p, i32p, c_int, f32p]
        L.nextera_mlm_logits.argtypes = [vp, i32p, c_int, i32p, c_int, f32p]

    @staticmethod
    def _q(T, C, quant):
        if not quant:
            return None, None
        return np.empty((T, C), np.int8), np.empty((T, (C + 255) // 256), np.float32)

    def build_i8_weight(self, qtype, data, n_in, n_out):
        n_blk = (n_in + 255) // 256
        w = np.empty((n_out, n_in), np.int8)
        sc = np.empty((n_blk, n_out), np.float32)
        off = np.empty((n_blk, n_out), np.int32)
        self.L.ref_build_i8_weight(qtype, np.ascontiguousarray(data).ctypes.data, n_in, n_out, ptr(w), ptr(sc), ptr(off))
        return w, sc, off

    def quantize_rows(self, x):
        T, C = x.shape
        q, sx = self._q(T, C, True)
        self.L.ref_quantize_rows(ptr(x), T, C, ptr(q), ptr(sx))
        return q, sx

    def linear_i8(self, xq, sx, w, sw, off, res=None):
        T, K = xq.shape
        N = w.shape[0]
        out = np.empty((T, N), np.float32)
        self.L.ref_linear_i8(ptr(xq), ptr(sx), T, ptr(w), ptr(sw), ptr(off), K, N, ptr(res), ptr(out))
        return out

    def rms_norm(self, x, gain, eps, quant=False):
        T, C = x.shape
        q, sx = self._q(T, C, quant)
        out = None if quant else np.empty_like(x)
        self.L.ref_rms_norm(ptr(x), ptr(gain), eps, T, C, ptr(out), ptr(q), ptr(sx))
        return (q, sx) if quant else out

    def relu_sqr(self, x, quant=False):
        T, C = x.shape
        q, sx = self._q(T, C, quant)
        out = None if quant else np.empty_like(x)
        self.L.ref_relu_sqr(ptr(x), T, C, ptr(out), ptr(q), ptr(sx))
        return (q, sx) if quant else out

    def gate(self, g, y, quant=False):
        T, C = g.shape
        q, sx = self._q(T, C, quant)
        out = None if quant else np.empty_like(g)
        self.L.ref_gate(ptr(g), ptr(y), T, C, ptr(out), ptr(q), ptr(sx))
        return (q, sx) if quant else out

    def dwconv(self, x, r, taps, lengths, quant=False):
        T, C = x.shape
        lengths = np.ascontiguousarray(lengths, np.int32)
        q, sx = self._q(T, C, quant)
        out = None if quant else np.empty_like(x)
        self.L.ref_dwconv(ptr(x), ptr(r), ptr(taps), taps.shape[0], ptr(lengths), len(lengths), C, ptr(out),
                          ptr(q), ptr(sx))
        return (q, sx) if quant else out

    def lily_state(self, a, x, b, taps, lengths, quant=False):
        T, C = x.shape
        lengths = np.ascontiguousarray(lengths, np.int32)
        q, sx = self._q(T, C, quant)
        out = None if quant else np.empty_like(x)
        self.L.ref_lily_state(ptr(a), ptr(x), ptr(b), ptr(taps), taps.shape[0], ptr(lengths), len(lengths), C,
                              ptr(out), ptr(q), ptr(sx))
        return (q, sx) if quant else out

    def qk_prep(self, x, alpha, beta, base, lengths, H, D, head_major):
        T = x.shape[0]
        lengths = np.ascontiguousarray(lengths, np.int32)
        out = np.empty((H, T, D) if head_major else (T, H * D), np.float32)
        self.L.ref_qk_prep(ptr(x), ptr(alpha), ptr(beta), base, ptr(lengths), len(lengths), H, D,
                           int(head_major), ptr(out))
        return out

    def rope_table(self, n_pos, base, D):
        c = np.empty((n_pos, D // 2), np.float32)
        s = np.empty((n_pos, D // 2), np.float32)
        self.L.ref_rope_table(n_pos, base, D, ptr(c), ptr(s))
        return c, s

    def head_major(self, x, H, D):
        T = x.shape[0]
        out = np.empty((H, T, D), np.float32)
        self.L.ref_head_major(ptr(x), T, H, D, ptr(out))
        return out

    def block_mean(self, h, g, lengths, block, quant=False):
        C = h.shape[1]
        lengths = np.ascontiguousarray(lengths, np.int32)
        nb = int(((lengths + block - 1) // block).sum())
        q, sx = self._q(nb, C, quant)
        out = None if quant else np.empty((nb, C), np.float32)
        self.L.ref_block_mean(ptr(h), ptr(g), C, block, ptr(lengths), len(lengths), ptr(out), ptr(q), ptr(sx))
        return (q, sx) if quant else out

    def upsample_add(self, y, r, lengths, block):
        lengths = np.ascontiguousarray(lengths, np.int32)
        out = np.empty_like(r)
        self.L.ref_upsample_add(ptr(y), ptr(r), r.shape[1], block, ptr(lengths), len(lengths), ptr(out))
        return out

    def attention(self, q, k, v, H, G, D, half, scale, lengths):
        lengths = np.ascontiguousarray(lengths, np.int32)
        out = np.empty((q.shape[0], H * D), np.float32)
        self.L.ref_attention(ptr(q), ptr(k), ptr(v), H, G, D, half, ptr(np.asarray(scale, np.float32)),
                             ptr(lengths), len(lengths), ptr(out))
        return out

    # -- the reference's C API ---------------------------------------------
    def load(self, path, n_threads=0):
        p = self.L.nextera_default_params()
        p.n_threads = n_threads
        p.verbosity = 0
        h = self.L.nextera_load(str(path).encode(), p)
        if not h:
            raise RuntimeError(f"reference failed to load {path}")
        return h

    def encode(self, h, tokens, lengths, types=None, normalize=True, hidden=True):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lengths = np.ascontiguousarray(lengths, np.int32)
        types = None if types is None else np.ascontiguousarray(types, np.int32)
        C = self.L.nextera_n_embd(h)
        T = int(lengths.sum())
        hid = np.empty((T, C), np.float32) if hidden else None
        pooled = np.empty((len(lengths), C), np.float32)
        rc = self.L.nextera_encode_segments(h, ptr(tokens), ptr(types), ptr(lengths), len(lengths), ptr(hid),
                                            ptr(pooled), int(normalize))
        if rc != 0:
            raise RuntimeError(f"reference encode failed ({rc})")
        return hid, pooled

    # -- heads (nextera_pooler_output / nextera_classify / nextera_mlm_logits) --
    def pooler_output(self, h, tokens, lengths, types=None):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lengths = np.ascontiguousarray(lengths, np.int32)
        types = None if types is None else np.ascontiguousarray(types, np.int32)
        out = np.empty((len(lengths), self.L.nextera_n_embd(h)), np.float32)
        rc = self.L.nextera_pooler_output(h, ptr(tokens), ptr(types), ptr(lengths), len(lengths), ptr(out))
        if rc != 0:
            raise RuntimeError(f"reference pooler_output failed ({rc})")
        return out

    def classify(self, h, tokens, lengths, types=None):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lengths = np.ascontiguousarray(lengths, np.int32)
        types = None if types is None else np.ascontiguousarray(types, np.int32)
        task = self.L.nextera_classifier_task(h).decode()
        rows = len(lengths) if task in ("sequence-classification", "multiple-choice") else int(lengths.sum())
        out = np.empty((rows, self.L.nextera_n_labels(h)), np.float32)
        rc = self.L.nextera_classify(h, ptr(tokens), ptr(types), ptr(lengths), len(lengths), ptr(out))
        if rc != 0:
            raise RuntimeError(f"reference classify failed ({rc})")
        return out

    def mlm_logits(self, h, tokens, positions):
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        out = np.empty((len(positions), self.L.nextera_n_vocab(h)), np.float32)
        rc = self.L.nextera_mlm_logits(h, ptr(tokens), len(tokens), ptr(positions), len(positions), ptr(out))
        if rc != 0:
            raise RuntimeError(f"reference mlm_logits failed ({rc})")
        return out
