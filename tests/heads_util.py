"""Shared pieces of the head tests (test infrastructure).

* ``weight_rows``  -- N rows of K weights in GGUF blocks of any type the heads accept;
* ``act_numpy``    -- a numpy restatement of ggml's activation conversion to the
  weight type's vec_dot type (Q8_K / Q8_0 / Q8_1 codes, F16 / BF16 rounding),
  laid out as oracle/vecdot.c lays it out (codes | d | s | bsum);
* ``raw_tensor``   -- a tensor's file bytes from a GGUF file (gguf-py reader);
* ``head_graph``   -- the reference's head graphs (src/nexterabert.cpp:1296-1317,
  :1963-2011) composed from the CPU checkers' ops.
"""
from __future__ import annotations

import numpy as np

import gguf
from gguf import GGMLQuantizationType as QT

import synth_model as sm

# every weight type ggml_mul_mat takes on the heads' path
MUL_MAT_TYPES = [QT.F32, QT.F16, QT.BF16, QT.Q4_0, QT.Q4_1, QT.Q5_0, QT.Q5_1, QT.Q8_0,
                 QT.Q2_K, QT.Q3_K, QT.Q4_K, QT.Q5_K, QT.Q6_K]
FAMILY = {QT.F32: "f32", QT.F16: "f16", QT.BF16: "bf16", QT.Q4_0: "q8_0", QT.Q5_0: "q8_0", QT.Q8_0: "q8_0",
          QT.Q4_1: "q8_1", QT.Q5_1: "q8_1", QT.Q2_K: "q8_k", QT.Q3_K: "q8_k", QT.Q4_K: "q8_k",
          QT.Q5_K: "q8_k", QT.Q6_K: "q8_k"}


def weight_rows(qt, N: int, K: int, seed: int = 0) -> np.ndarray:
    """N rows of K weights ~ N(0, 0.02) as GGUF bytes (one row per line).

    Q2_K and Q3_K have no encoder in this environment: their blocks are random
    bytes with the fp16 scales set to small finite values (any bit pattern of the
    code and sub-scale bytes is a valid block)."""
    rng = np.random.default_rng(seed)
    if qt in (QT.Q2_K, QT.Q3_K):
        bs, ts = gguf.GGML_QUANT_SIZES[qt]
        nb = N * K // bs
        blocks = rng.integers(0, 256, (nb, ts), dtype=np.uint8)
        d = (0.002 * (1.0 + rng.random(nb))).astype(np.float16).view(np.uint8).reshape(nb, 2)
        if qt == QT.Q2_K:
            blocks[:, 80:82] = d
            blocks[:, 82:84] = (0.001 * (1.0 + rng.random(nb))).astype(np.float16).view(np.uint8).reshape(nb, 2)
        else:
            blocks[:, 108:110] = d
        return blocks.reshape(N, -1)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    if qt == QT.F32:
        return w.view(np.uint8).reshape(N, -1)
    if qt == QT.F16:
        return w.astype(np.float16).view(np.uint8).reshape(N, -1)
    if qt == QT.BF16:
        return gguf.quants.quantize(w, QT.BF16).view(np.uint8).reshape(N, -1)
    return np.ascontiguousarray(sm.quantize_rows(w, qt)).view(np.uint8).reshape(N, -1)


def dequant_rows(qt, rows: np.ndarray, K: int) -> np.ndarray:
    if qt == QT.F32:
        return rows.view(np.float32).reshape(-1, K).astype(np.float64)
    if qt == QT.F16:
        return rows.view(np.float16).reshape(-1, K).astype(np.float64)
    return gguf.quants.dequantize(rows, qt).reshape(-1, K).astype(np.float64)


def _f16(v):
    return np.asarray(v, np.float32).astype(np.float16).astype(np.float32)


def _bf16(v):
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + (0x7FFF + ((u >> 16) & 1))) & 0xFFFF0000).astype(np.uint32)
    return u.view(np.float32)


def act_numpy(qt, x: np.ndarray) -> np.ndarray:
    """One converted activation row of K floats, as bytes (oracle/vecdot.c layout)."""
    x = np.asarray(x, np.float32)
    K = x.size
    fam = FAMILY[qt]
    if fam == "f32":
        return x.view(np.uint8).copy()
    if fam == "f16":
        return _f16(x).view(np.uint8).copy()
    if fam == "bf16":
        return _bf16(x).view(np.uint8).copy()
    f32 = np.float32
    if fam in ("q8_0", "q8_1"):
        xb = x.reshape(-1, 32)
        q = np.zeros_like(xb, dtype=np.int8)
        d = np.zeros(len(xb), np.float32)
        s = np.zeros(len(xb), np.float32)
        for b, row in enumerate(xb):
            amax = f32(np.abs(row).max())
            db = f32(amax / f32(127))
            idv = f32(f32(127) / amax) if amax != 0 else f32(0)
            qi = np.rint(row * idv).astype(np.int32)
            q[b] = qi.astype(np.int8)
            d[b] = _f16(db)
            s[b] = _f16(f32(db * f32(qi.sum())))
        parts = [q.reshape(-1).view(np.uint8), d.view(np.uint8)]
        if fam == "q8_1":
            parts.append(s.view(np.uint8))
        return np.concatenate(parts)
    xb = x.reshape(-1, 256)
    q = np.zeros_like(xb, dtype=np.int8)
    d = np.zeros(len(xb), np.float32)
    bsum = np.zeros((len(xb), 16), np.int32)
    for b, row in enumerate(xb):
        ax = np.abs(row)
        if ax.max() == 0:
            continue
        mx = row[int(np.argmax(ax))]              # first of the largest magnitude
        iscale = f32(f32(-127) / mx)
        qi = np.minimum(np.rint(iscale * row).astype(np.int32), 127)
        q[b] = qi.astype(np.int8)
        bsum[b] = qi.reshape(16, 16).sum(1)
        d[b] = f32(f32(1) / iscale)
    return np.concatenate([q.reshape(-1).view(np.uint8), d.view(np.uint8), bsum.reshape(-1).view(np.uint8)])


def act_dequant(qt, act: np.ndarray, K: int) -> np.ndarray:
    """The values a converted row stands for (codes times scales), float64."""
    fam = FAMILY[qt]
    if fam in ("f32", "f16", "bf16"):
        return act[:4 * K].view(np.float32).astype(np.float64)
    q = act[:K].view(np.int8).astype(np.float64)
    if fam in ("q8_0", "q8_1"):
        d = act[K:K + 4 * (K // 32)].view(np.float32).astype(np.float64)
        return q * np.repeat(d, 32)
    d = act[K:K + 4 * (K // 256)].view(np.float32).astype(np.float64)
    return q * np.repeat(d, 256)


def raw_tensor(path, name: str):
    """(type, rows of bytes, ne0, ne1) of one tensor of a GGUF file."""
    r = gguf.GGUFReader(str(path))
    for t in r.tensors:
        if t.name == name:
            ne0 = int(t.shape[0])
            ne1 = int(t.shape[1]) if len(t.shape) > 1 else 1
            data = np.ascontiguousarray(t.data).view(np.uint8).reshape(ne1, -1)
            return int(t.tensor_type), data, ne0, ne1
    raise KeyError(name)


def f32_tensor(path, name: str) -> np.ndarray:
    typ, data, ne0, ne1 = raw_tensor(path, name)
    assert typ == 0
    return data.view(np.float32).reshape(-1) if ne1 == 1 else data.view(np.float32).reshape(ne1, ne0)


def head_graph(reflib, oracle, path, hidden, lengths=None, positions=None, head="pooler", eps=1e-5):
    """The reference's head graph from the checkers' ops, on the encoder output `hidden`.

    head: "pooler" (pooler_output), "classify" (pooled or per-token by the file's task)
    or "mlm" (rows `positions` of a single sequence)."""
    import gguf as _g
    rd = _g.GGUFReader(str(path))
    task = ""
    f = rd.fields.get("nexterabert.classifier.task")
    if f is not None:
        task = bytes(f.parts[f.data[0]]).decode()
    pooled = head == "pooler" or task in sm.POOLED_TASKS

    def linear(name, x):
        typ, data, ne0, ne1 = raw_tensor(path, name)
        if typ not in (0, 1, 30):                       # quantized: the int8 path
            w, sw, off = reflib.build_i8_weight(typ, data, ne0, ne1)
            xq, sx = reflib.quantize_rows(np.ascontiguousarray(x, np.float32))
            return reflib.linear_i8(xq, sx, w, sw, off)
        return oracle.mul_mat(typ, data, ne1, ne0, x)

    def transform(pre, x):
        y = oracle.gelu_erf(linear(pre + "dense.weight", x))
        return oracle.layer_norm(y, f32_tensor(path, pre + "norm.weight"), None, eps)

    if head == "mlm":
        h = transform("mlm.", hidden[np.asarray(positions)])
        try:
            typ, data, ne0, ne1 = raw_tensor(path, "mlm.decoder.weight")
        except KeyError:
            typ, data, ne0, ne1 = raw_tensor(path, "embedding.weight")
        return oracle.mul_mat(typ, data, ne1, ne0, h) + f32_tensor(path, "mlm.bias")
    x = oracle.pool(hidden, lengths, 0) if pooled else hidden
    h = transform("pooler." if pooled else "head.", x)
    if head == "pooler":
        return h
    typ, data, ne0, ne1 = raw_tensor(path, "classifier.weight")
    return oracle.mul_mat(typ, data, ne1, ne0, h) + f32_tensor(path, "classifier.bias")
