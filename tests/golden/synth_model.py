"""Seeded synthetic NexteraBERT GGUF files (test and benchmark infrastructure).

No checkpoint of the real model exists in this environment, so every parity test
and benchmark runs on random-init models that have the real architecture:

* metadata keys and tensor names follow the reference converter
  (python/convert_hf_to_gguf.py:178-209) and the tensors the reference loader
  requires (src/nexterabert.cpp:1483-1516);
* 2-D weights are drawn N(0, 0.02); the 1-D parameters (norm gains, DyT curves,
  conv taps, SSMax scalars, LayerNorm) use the fixed choices in `_small_params`;
* file types follow the reference quantizer (tools/quantize.cpp:33-98): a matrix
  is a 2-D ``*.weight`` other than the classifier with both dims >= 32;
  ``_M`` presets keep the residual writers, c_v, c_gate and the head transforms
  at Q6_K (``wants_more_bits``, quantize.cpp:79-83); K-quant rows whose length is
  not a multiple of 256 fall back per ``fallback_for_row`` (quantize.cpp:87-98).

Q8_0, Q4_0, Q4_1, Q5_0 and Q5_1 blocks are written by gguf-py's own quantizers
(gguf 0.19.0, ``gguf.quants``).  gguf-py has no K-quant encoder, so Q4_K, Q5_K
and Q6_K blocks are encoded here from the published GGUF block layout (the
inverse of ``gguf.quants.Q4_K/Q5_K/Q6_K.dequantize_blocks``).  Any valid
encoding serves: the oracle and the GPU library read the same file.  These
files are therefore not byte-identical to ``nexterabert-quantize`` output.
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass, field, asdict
from pathlib import Path

import numpy as np

import gguf
from gguf import GGMLQuantizationType as QT

ARCH = "nexterabert"

# llama.cpp general.file_type numbers used by the reference (nexterabert.cpp:1390-1410)
FTYPES = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q8_0": 7, "Q5_0": 8, "Q5_1": 9,
          "Q4_K_S": 14, "Q4_K_M": 15, "Q5_K_S": 16, "Q5_K_M": 17, "Q6_K": 18}

# preset -> (base type, "more bits" type), quantize.cpp:33-45
PRESETS = {
    "F32": (QT.F32, QT.F32), "F16": (QT.F16, QT.F16), "Q8_0": (QT.Q8_0, QT.Q8_0),
    "Q6_K": (QT.Q6_K, QT.Q6_K), "Q5_K_M": (QT.Q5_K, QT.Q6_K), "Q5_K_S": (QT.Q5_K, QT.Q5_K),
    "Q5_0": (QT.Q5_0, QT.Q5_0), "Q4_K_M": (QT.Q4_K, QT.Q6_K), "Q4_K_S": (QT.Q4_K, QT.Q4_K),
    "Q4_0": (QT.Q4_0, QT.Q4_0), "Q4_1": (QT.Q4_1, QT.Q4_1), "Q5_1": (QT.Q5_1, QT.Q5_1),
}
PRESET_FTYPE = {"F32": 0, "F16": 1, "Q8_0": 7, "Q6_K": 18, "Q5_K_M": 17, "Q5_K_S": 16,
                "Q5_0": 8, "Q4_K_M": 15, "Q4_K_S": 14, "Q4_0": 2, "Q4_1": 3, "Q5_1": 9}


@dataclass
class HParams:
    n_vocab: int = 50368
    n_embd: int = 1024
    n_layer: int = 18
    n_inter: int = 2304
    n_head: int = 16
    n_kv_head: int = 8
    lily_kernel: int = 5
    hra_block: int = 4
    swa_window: int = 256
    ntk_train_len: int = 0
    rope_base: float = 100000.0
    swa_rope_base: float = 10000.0
    ssmax_mode: str = "sssmax"
    ssmax_base: float = 0.1
    block_types: list = field(default_factory=list)
    mlm_head: bool = True
    n_types: int = 0
    cls_id: int = 50281
    sep_id: int = 50282
    pad_id: int = 50283
    mask_id: int = 50284
    # heads (python/convert_hf_to_gguf.py:39-66, :125-166): a classifier task
    # ("sequence-classification", "multiple-choice", "token-classification",
    # "question-answering") with n_labels outputs; a pooler kept without one;
    # an untied MLM decoder; a classifier written by an f16 conversion
    cls_task: str = ""
    n_labels: int = 0
    pooler: bool = False
    untied_decoder: bool = False
    cls_f16: bool = False
    # embed a word-level tokenizer.json ("w<id>" words; the special ids as [CLS] [SEP] [PAD] [MASK])
    # under tokenizer.huggingface.json, as the converter embeds the real one (convert_hf_to_gguf.py:204)
    tokenizer: bool = False


# fields added after the first fixtures: left out of the cache key at their defaults
_LATE_FIELDS = {"cls_task": "", "n_labels": 0, "pooler": False, "untied_decoder": False, "cls_f16": False,
                "tokenizer": False}
POOLED_TASKS = ("sequence-classification", "multiple-choice")


# 8 lily, 6 swa, 2 attn, 2 hra: the published block mix (141 int8 linears with mlm.dense).
# The real layer order is not in this environment; this order is fixed here.
FULL_BLOCKS = ["lily", "swa", "lily", "swa", "lily", "attn", "lily", "swa", "hra",
               "lily", "swa", "lily", "swa", "lily", "attn", "lily", "swa", "hra"]


def full_hparams(**kw) -> HParams:
    hp = HParams(block_types=list(FULL_BLOCKS))
    for k, v in kw.items():
        setattr(hp, k, v)
    return hp


def tiny_hparams(**kw) -> HParams:
    """A small model with every mixer kind, sized so the scalar oracle runs in seconds."""
    hp = HParams(n_vocab=1000, n_embd=256, n_layer=4, n_inter=512, n_head=4, n_kv_head=2,
                 swa_window=16, block_types=["lily", "swa", "attn", "hra"],
                 cls_id=996, sep_id=997, pad_id=998, mask_id=999)
    for k, v in kw.items():
        setattr(hp, k, v)
    return hp


# ---------------------------------------------------------------------------
# block encoders
# ---------------------------------------------------------------------------

def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16)


def _pack_k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """8 six-bit scales and 8 six-bit mins -> 12 bytes (inverse of Q4_K.get_scale_min)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out


def _affine_k(x: np.ndarray, levels: int):
    """Per 32-value sub-block affine fit for Q4_K / Q5_K.  x: (nb, 256)."""
    nb = x.shape[0]
    xb = x.reshape(nb, 8, 32)
    lo = np.minimum(xb.min(-1), 0.0)
    hi = xb.max(-1)
    scale = (hi - lo) / levels
    mins = 0.0 - lo                                     # +0 (not -0) when lo is 0
    d = _f16(scale.max(-1) / 63.0)
    dmin = _f16(mins.max(-1) / 63.0)
    df = d.astype(np.float32)[:, None]
    dmf = dmin.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.clip(np.rint(scale / df), 0, 63), 0).astype(np.uint8)
        mq = np.where(dmf > 0, np.clip(np.rint(mins / dmf), 0, 63), 0).astype(np.uint8)
    dsub = (df * sc.astype(np.float32))[:, :, None]
    dm = (dmf * mq.astype(np.float32))[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(dsub > 0, np.clip(np.rint((xb + dm) / dsub), 0, levels), 0).astype(np.uint8)
    return d, dmin, sc, mq, q


def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d, dmin, sc, mq, q = _affine_k(x, 15)
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(nb, 128)
    return np.concatenate([d.reshape(nb, 1).view(np.uint8), dmin.reshape(nb, 1).view(np.uint8),
                           _pack_k_scales(sc, mq), qs], axis=1)


def quantize_q5_k(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d, dmin, sc, mq, q = _affine_k(x, 31)
    lo = q & 15
    qs = (lo[:, 0::2, :] | (lo[:, 1::2, :] << 4)).reshape(nb, 128)
    hb = (q >> 4) & 1                                   # (nb, 8, 32)
    qh = np.zeros((nb, 32), dtype=np.uint8)
    for j in range(8):
        qh |= (hb[:, j, :] << j).astype(np.uint8)
    return np.concatenate([d.reshape(nb, 1).view(np.uint8), dmin.reshape(nb, 1).view(np.uint8),
                           _pack_k_scales(sc, mq), qh, qs], axis=1)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    xb = x.reshape(nb, 16, 16)
    s = np.abs(xb).max(-1) / 31.0
    d = _f16(s.max(-1) / 127.0)
    df = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.clip(np.rint(s / df), -128, 127), 0).astype(np.int8)
    dsub = (df * sc.astype(np.float32))[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(dsub != 0, np.clip(np.rint(xb / dsub), -32, 31), 0).astype(np.int16) + 32
    q = q.astype(np.uint8).reshape(nb, 2, 128)         # [half][r]
    ql = np.zeros((nb, 2, 64), dtype=np.uint8)
    qh = np.zeros((nb, 2, 32), dtype=np.uint8)
    for s_ in range(2):
        ql |= ((q[:, :, 64 * s_:64 * s_ + 64] & 15) << (4 * s_)).astype(np.uint8)
    for k in range(4):
        qh |= (((q[:, :, 32 * k:32 * k + 32] >> 4) & 3) << (2 * k)).astype(np.uint8)
    return np.concatenate([ql.reshape(nb, 128), qh.reshape(nb, 64), sc.view(np.uint8),
                           d.reshape(nb, 1).view(np.uint8)], axis=1)


def quantize_q2_k(x: np.ndarray) -> np.ndarray:
    """16 sub-blocks of 16, affine: 4-bit scale and minimum codes under fp16 d / dmin, 2-bit codes."""
    nb = x.shape[0]
    xb = x.reshape(nb, 16, 16)
    lo = np.minimum(xb.min(-1), 0.0)
    hi = xb.max(-1)
    scale = (hi - lo) / 3
    mins = 0.0 - lo                                     # +0 (not -0) when lo is 0
    d = _f16(scale.max(-1) / 15.0)
    dmin = _f16(mins.max(-1) / 15.0)
    df = d.astype(np.float32)[:, None]
    dmf = dmin.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.clip(np.rint(scale / df), 0, 15), 0).astype(np.uint8)
        mq = np.where(dmf > 0, np.clip(np.rint(mins / dmf), 0, 15), 0).astype(np.uint8)
    dsub = (df * sc.astype(np.float32))[:, :, None]
    dm = (dmf * mq.astype(np.float32))[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(dsub > 0, np.clip(np.rint((xb + dm) / dsub), 0, 3), 0).astype(np.uint8)
    q = q.reshape(nb, 2, 4, 32)                          # [half][shift][position]
    qs = np.zeros((nb, 2, 32), dtype=np.uint8)
    for k in range(4):
        qs |= (q[:, :, k, :] << (2 * k)).astype(np.uint8)
    return np.concatenate([sc | (mq << 4), qs.reshape(nb, 64), d.reshape(nb, 1).view(np.uint8),
                           dmin.reshape(nb, 1).view(np.uint8)], axis=1)


def quantize_q3_k(x: np.ndarray) -> np.ndarray:
    """16 sub-blocks of 16, symmetric: 6-bit scales (stored + 32) under an fp16 d, 3-bit codes in
    [-4, 3] stored + 4 (low 2 bits in qs, bit 2 in hmask)."""
    nb = x.shape[0]
    xb = x.reshape(nb, 16, 16)
    s = np.abs(xb).max(-1) / 4.0
    d = _f16(s.max(-1) / 31.0)
    df = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.clip(np.rint(s / df), -32, 31), 0).astype(np.int16)
    dsub = (df * sc.astype(np.float32))[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = (np.where(dsub != 0, np.clip(np.rint(xb / dsub), -4, 3), 0) + 4).astype(np.uint8)
    q = q.reshape(nb, 2, 4, 32)
    hmask = np.zeros((nb, 32), dtype=np.uint8)
    qs = np.zeros((nb, 2, 32), dtype=np.uint8)
    for h in range(2):
        for k in range(4):
            hmask |= (((q[:, h, k, :] >> 2) & 1) << (4 * h + k)).astype(np.uint8)
            qs[:, h, :] |= ((q[:, h, k, :] & 3) << (2 * k)).astype(np.uint8)
    sc6 = (sc + 32).astype(np.uint8)
    scb = np.zeros((nb, 12), dtype=np.uint8)
    for j in range(16):
        if j < 8:
            scb[:, j] |= sc6[:, j] & 15
        else:
            scb[:, j - 8] |= ((sc6[:, j] & 15) << 4).astype(np.uint8)
        scb[:, 8 + j % 4] |= (((sc6[:, j] >> 4) & 3) << (2 * (j // 4))).astype(np.uint8)
    return np.concatenate([hmask, qs.reshape(nb, 64), scb, d.reshape(nb, 1).view(np.uint8)], axis=1)


_K_ENCODERS = {QT.Q2_K: quantize_q2_k, QT.Q3_K: quantize_q3_k, QT.Q4_K: quantize_q4_k, QT.Q5_K: quantize_q5_k,
               QT.Q6_K: quantize_q6_k}


def quantize_rows(w: np.ndarray, qt) -> np.ndarray:
    """(rows, n) float32 -> (rows, row_bytes) uint8 blocks of type `qt`."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, n = w.shape
    if qt in _K_ENCODERS:
        blocks = _K_ENCODERS[qt](w.reshape(-1, 256))
        return np.ascontiguousarray(blocks.reshape(rows, -1))
    return gguf.quants.quantize(w, qt)


def dequantize_rows(data: np.ndarray, qt, n: int) -> np.ndarray:
    return gguf.quants.dequantize(data, qt).reshape(-1, n)


def fallback_for_row(qt, n_per_row: int):
    """tools/quantize.cpp:87-98."""
    bs = gguf.GGML_QUANT_SIZES[qt][0]
    if n_per_row % bs == 0:
        return qt
    fb = {QT.Q2_K: QT.Q4_0, QT.Q3_K: QT.Q4_0, QT.Q4_K: QT.Q5_0, QT.Q5_K: QT.Q5_1, QT.Q6_K: QT.Q8_0}
    qt = fb.get(qt, qt)
    return qt if n_per_row % gguf.GGML_QUANT_SIZES[qt][0] == 0 else QT.F32


def wants_more_bits(name: str) -> bool:
    """tools/quantize.cpp:79-83."""
    return (name.endswith(".attn.c_proj.weight") or name.endswith(".mlp.c_proj.weight")
            or name.endswith(".attn.c_v.weight") or name.endswith(".attn.c_gate.weight")
            or name in ("mlm.dense.weight", "head.dense.weight", "pooler.dense.weight"))


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------

def tensor_specs(hp: HParams):
    """Ordered (name, numpy shape, kind) of every tensor the model carries.

    numpy shape is (ne[1], ne[0]): a linear weight is (n_out, n_in)."""
    C, I, H, G = hp.n_embd, hp.n_inter, hp.n_head, hp.n_kv_head
    D = C // H
    r = D  # lily low rank = expand * n_embd / n_head with expand = 1
    k = hp.lily_kernel
    out = [("embedding.weight", (hp.n_vocab, C), "w")]
    for l, bt in enumerate(hp.block_types):
        blk, pre = f"blocks.{l}.", f"blocks.{l}.attn."
        out += [(blk + "attn_norm.weight", (C,), "gain"), (blk + "mlp_norm.weight", (C,), "gain"),
                (blk + "mlp.c_fc.weight", (I, C), "w"), (blk + "mlp.c_proj.weight", (C, I), "w"),
                (pre + "c_proj.weight", (C, C), "w")]
        if bt == "lily":
            out += [(pre + "ltc_conv.in_proj.weight", (r, C), "w"), (pre + "ltc_conv.A.weight", (r, C), "w"),
                    (pre + "ltc_conv.kernel", (r, k), "taps"), (pre + "ltc_conv.out_proj.weight", (C, r), "w"),
                    (pre + "x_proj.weight", (C, C), "w"), (pre + "B_proj.weight", (C, C), "w"),
                    (pre + "state_conv.depthwise.weight", (C, k), "taps")]
            continue
        out += [(pre + "c_q.weight", (H * D, C), "w"), (pre + "c_k.weight", (G * D, C), "w"),
                (pre + "c_v.weight", (G * D, C), "w"), (pre + "c_gate.weight", (C, H * D), "w"),
                (pre + "q_norm.alpha", (D,), "alpha"), (pre + "q_norm.beta", (D,), "beta"),
                (pre + "k_norm.alpha", (D,), "alpha"), (pre + "k_norm.beta", (D,), "beta")]
        if bt == "hra":
            out += [(pre + "qkv_in.weight", (C, C), "w"), (pre + "qkv_gate.weight", (C, C), "w"),
                    (pre + "c_C.weight", (C, C), "w"), (pre + "qkv_conv.depthwise.weight", (C, k), "taps"),
                    (pre + "c_o.depthwise.weight", (C, k), "taps")]
        if bt != "swa" and hp.ssmax_mode != "none":
            out += [(pre + "scalable_factor.s", (1,), "ss_s")]
            if hp.ssmax_mode == "sssmax":
                out += [(pre + "scalable_factor.b", (1,), "ss_b")]
    out += [("out_norm.weight", (C,), "gain"), ("out_norm.bias", (C,), "bias")]
    if hp.n_types > 0:
        out += [("token_type_embeddings.weight", (hp.n_types, C), "w")]
    if hp.mlm_head:
        out += [("mlm.dense.weight", (C, C), "w"), ("mlm.norm.weight", (C,), "gain"),
                ("mlm.bias", (hp.n_vocab,), "bias")]
        if hp.untied_decoder:
            out += [("mlm.decoder.weight", (hp.n_vocab, C), "w")]
    if hp.cls_task in POOLED_TASKS or hp.pooler:
        out += [("pooler.dense.weight", (C, C), "w"), ("pooler.norm.weight", (C,), "gain")]
    if hp.cls_task and hp.cls_task not in POOLED_TASKS:
        out += [("head.dense.weight", (C, C), "w"), ("head.norm.weight", (C,), "gain")]
    if hp.cls_task:
        out += [("classifier.weight", (hp.n_labels, C), "w"), ("classifier.bias", (hp.n_labels,), "bias")]
    return out


def _small_params(kind: str, shape, rng: np.random.Generator) -> np.ndarray:
    """The builder's stated choice for every non-matrix parameter."""
    if kind == "gain":
        return (1.0 + 0.05 * rng.standard_normal(shape)).astype(np.float32)
    if kind == "bias":
        return (0.02 * rng.standard_normal(shape)).astype(np.float32)
    if kind == "alpha":
        return (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
    if kind == "beta":
        return (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
    if kind == "taps":
        return (0.3 * rng.standard_normal(shape)).astype(np.float32)
    if kind == "ss_s":
        return np.array([0.3], dtype=np.float32)
    if kind == "ss_b":
        return np.array([0.05], dtype=np.float32)
    raise ValueError(kind)


def tensor_type(name: str, shape, preset: str, cls_f16: bool = False):
    """Storage type of one tensor under `preset` (quantize.cpp:195-206)."""
    base, more = PRESETS[preset]
    if name == "classifier.weight":
        # the quantizer keeps it as converted (quantize.cpp:171-175); the converter writes a
        # matrix with both dims >= 32 as f16 under --outtype f16 (convert_hf_to_gguf.py:216-218)
        return QT.F16 if (cls_f16 or preset == "F16") and min(shape) >= 32 else QT.F32
    is_matrix = (len(shape) == 2 and name.endswith(".weight")
                 and shape[1] >= 32 and shape[0] >= 32)
    if not is_matrix:
        return QT.F32
    t = more if wants_more_bits(name) else base
    return fallback_for_row(t, shape[1])


def write_model(path: str | os.PathLike, hp: HParams, preset: str, seed: int = 0) -> Path:
    """Write a random-init model quantized with `preset` to `path`."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(str(path) + ".tmp", ARCH)
    w.add_name("nexterabert-synthetic")
    w.add_file_type(PRESET_FTYPE[preset])
    w.add_quantization_version(gguf.GGML_QUANT_VERSION)
    k = f"{ARCH}."
    w.add_uint32(k + "vocab_size", hp.n_vocab)
    w.add_uint32(k + "embedding_length", hp.n_embd)
    w.add_uint32(k + "block_count", hp.n_layer)
    w.add_uint32(k + "feed_forward_length", hp.n_inter)
    w.add_uint32(k + "attention.head_count", hp.n_head)
    w.add_uint32(k + "attention.head_count_kv", hp.n_kv_head)
    w.add_array(k + "block_types", list(hp.block_types))
    w.add_uint32(k + "lily.low_rank", hp.n_embd // hp.n_head)
    w.add_uint32(k + "lily.kernel_size", hp.lily_kernel)
    w.add_uint32(k + "hra.block_size", hp.hra_block)
    w.add_uint32(k + "swa.window", hp.swa_window)
    w.add_float32(k + "rope.freq_base", hp.rope_base)
    w.add_float32(k + "swa.rope.freq_base", hp.swa_rope_base)
    w.add_uint32(k + "rope.ntk_train_length", hp.ntk_train_len)
    w.add_string(k + "ssmax.mode", hp.ssmax_mode)
    w.add_float32(k + "ssmax.base", hp.ssmax_base)
    w.add_float32(k + "rms_norm_epsilon", 1e-8)
    w.add_float32(k + "layer_norm_epsilon", 1e-5)
    w.add_bool(k + "mlm_head", hp.mlm_head)
    if hp.cls_task:
        w.add_string(k + "classifier.task", hp.cls_task)
        w.add_array(k + "classifier.labels", [f"LABEL_{i}" for i in range(hp.n_labels)])
    w.add_uint32("tokenizer.ggml.cls_token_id", hp.cls_id)
    w.add_uint32("tokenizer.ggml.seperator_token_id", hp.sep_id)
    w.add_uint32("tokenizer.ggml.padding_token_id", hp.pad_id)
    w.add_uint32("tokenizer.ggml.mask_token_id", hp.mask_id)
    if hp.tokenizer:
        w.add_string("tokenizer.huggingface.json", word_tokenizer_json(hp))
    for name, shape, kind in tensor_specs(hp):
        if kind == "w":
            arr = (0.02 * rng.standard_normal(shape)).astype(np.float32)
        else:
            arr = _small_params(kind, shape, rng)
        qt = tensor_type(name, shape, preset, hp.cls_f16)
        if qt == QT.F32:
            w.add_tensor(name, np.ascontiguousarray(arr))
        elif qt == QT.F16:
            w.add_tensor(name, np.ascontiguousarray(arr.astype(np.float16)))
        else:
            w.add_tensor(name, quantize_rows(arr, qt), raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    os.replace(str(path) + ".tmp", path)
    return path


def word_tokenizer_json(hp: HParams) -> str:
    """A Hugging Face tokenizer.json for a synthetic model: whitespace-split words "w<id>" map to
    their ids, the special ids are [CLS] [SEP] [PAD] [MASK], single texts become [CLS] text [SEP]
    and pairs [CLS] a [SEP] b [SEP] with segment ids 0 / 1 (the layout of a BERT tokenizer)."""
    special = {hp.cls_id: "[CLS]", hp.sep_id: "[SEP]", hp.pad_id: "[PAD]", hp.mask_id: "[MASK]"}
    vocab = {special.get(i, f"w{i}"): i for i in range(hp.n_vocab)}
    unk = "[PAD]"
    tok = {
        "version": "1.0", "truncation": None, "padding": None,
        "added_tokens": [{"id": i, "content": t, "single_word": False, "lstrip": False, "rstrip": False,
                          "normalized": False, "special": True} for i, t in sorted(special.items())],
        "normalizer": None,
        "pre_tokenizer": {"type": "WhitespaceSplit"},
        "post_processor": {
            "type": "TemplateProcessing",
            "single": [{"SpecialToken": {"id": "[CLS]", "type_id": 0}}, {"Sequence": {"id": "A", "type_id": 0}},
                       {"SpecialToken": {"id": "[SEP]", "type_id": 0}}],
            "pair": [{"SpecialToken": {"id": "[CLS]", "type_id": 0}}, {"Sequence": {"id": "A", "type_id": 0}},
                     {"SpecialToken": {"id": "[SEP]", "type_id": 0}}, {"Sequence": {"id": "B", "type_id": 1}},
                     {"SpecialToken": {"id": "[SEP]", "type_id": 1}}],
            "special_tokens": {t: {"id": t, "ids": [i], "tokens": [t]} for i, t in special.items()}},
        "decoder": None,
        "model": {"type": "WordLevel", "vocab": vocab, "unk_token": unk},
    }
    return json.dumps(tok)


def model_cache_dir() -> Path:
    d = os.environ.get("NEXTERA_MODEL_CACHE")
    if d:
        return Path(d)
    return Path(__file__).resolve().parent / "_models"


def cached_model(name: str, hp: HParams, preset: str, seed: int = 0) -> Path:
    """Path of a generated model, written on first use (the key covers every setting)."""
    d = asdict(hp)
    for k, v in _LATE_FIELDS.items():
        if d.get(k) == v:
            del d[k]
    key = json.dumps({"hp": d, "preset": preset, "seed": seed, "v": 1}, sort_keys=True)
    h = hashlib.sha256(key.encode()).hexdigest()[:12]
    p = model_cache_dir() / f"{name}-{preset}-{h}.gguf"
    if not p.exists():
        write_model(p, hp, preset, seed)
    return p


# ---------------------------------------------------------------------------
# synthetic batches (seeded)
# ---------------------------------------------------------------------------

def throughput_lengths(n_docs: int = 4096, lo: int = 16, hi: int = 2048, seed: int = 0) -> np.ndarray:
    """Log-uniform lengths in [lo, hi] (the mixed-length throughput batch).

    With the defaults: 4096 documents, 1,685,650 tokens."""
    rng = np.random.default_rng(seed)
    return np.exp(rng.uniform(np.log(lo), np.log(hi + 1), n_docs)).astype(np.int64).clip(lo, hi).astype(np.int32)


def uniform_lengths(n_docs: int = 64, lo: int = 16, hi: int = 2048, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, n_docs).astype(np.int32)


def random_tokens(n: int, n_vocab: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, n_vocab, n).astype(np.int32)
