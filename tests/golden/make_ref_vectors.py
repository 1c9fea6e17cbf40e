"""Writes tests/golden/ref_vectors.npz: outputs of the reference's own code.

Run here, where the reference source exists:  python tests/golden/make_ref_vectors.py

The reference (Rikka-Botan/NexteraBERT.cpp, src/nexterabert.cpp) is compiled
from its sources by oracle/Makefile into oracle/_ref; this script runs its ops
and its C API on the seeded inputs of cases.py and stores the results.  Arrays
up to 64K elements are stored whole; larger ones as a SHA-256 of their bytes
plus a leading slice.  tests/test_oracle_pin.py checks the oracle against
these vectors, so the oracle stays pinned on machines without the reference.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))

import cases  # noqa: E402
import synth_model as sm  # noqa: E402
from oracle_lib import RefLib, build_oracle  # noqa: E402

OUT = HERE / "ref_vectors.npz"
WHOLE_LIMIT = 1 << 14


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def put(store: dict, name: str, a: np.ndarray) -> None:
    a = np.ascontiguousarray(a)
    if a.size <= WHOLE_LIMIT:
        store[name] = a
    else:
        store[name + ".sha"] = np.frombuffer(digest(a).encode(), np.uint8)
        store[name + ".head"] = a.reshape(-1)[:4096]


def generate(ref: RefLib) -> dict:
    s: dict = {}
    s["act_max"] = np.array([ref.L.ref_act_max()], np.int32)
    for i, qt in enumerate(cases.WEIGHT_TYPES):
        blocks, n_in, n_out = cases.weight_case(qt, seed=i)
        w, sc, off = ref.build_i8_weight(int(qt), blocks, n_in, n_out)
        put(s, f"i8w.{qt.name}.w", w)
        put(s, f"i8w.{qt.name}.scale", sc)
        put(s, f"i8w.{qt.name}.off", off)

    x = cases.rows_case()
    q, sx = ref.quantize_rows(x)
    put(s, "quant.q", q)
    put(s, "quant.sx", sx)

    for name, (T, K, N, qt, resid, seed) in cases.LINEAR_CASES.items():
        xa, blocks, qt_, res = cases.linear_case(T, K, N, seed=seed, qt=qt, residual=resid)
        w, sw, off = ref.build_i8_weight(int(qt_), blocks, K, N)
        xq, xs = ref.quantize_rows(xa)
        put(s, f"{name}.out", ref.linear_i8(xq, xs, w, sw, off, res))

    x1, wb = cases.cfg1_case()
    w, sw, off = ref.build_i8_weight(int(cases.QT.Q8_0), wb, 1024, 4096)
    xq, xs = ref.quantize_rows(x1)
    put(s, "cfg1.out", ref.linear_i8(xq, xs, w, sw, off, None))

    xr = cases.rows_case()
    gain = (1.0 + 0.05 * np.random.default_rng(5).standard_normal(xr.shape[1])).astype(np.float32)
    put(s, "rms.out", ref.rms_norm(xr, gain, 1e-8))
    q, sx = ref.rms_norm(xr, gain, 1e-8, quant=True)
    put(s, "rms.q", q)
    put(s, "rms.sx", sx)
    q, sx = ref.relu_sqr(xr, quant=True)
    put(s, "relu.q", q)
    put(s, "relu.sx", sx)
    g = cases.rows_case(seed=9)
    put(s, "gate.out", ref.gate(g, xr))
    q, sx = ref.gate(g, xr, quant=True)
    put(s, "gate.q", q)
    put(s, "gate.sx", sx)

    L = cases.LENGTHS_SMALL
    xc, rc, bc, taps = cases.conv_case()
    put(s, "dwconv.out", ref.dwconv(xc, rc, taps, L))
    q, sx = ref.dwconv(xc, None, taps, L, quant=True)
    put(s, "dwconv.q", q)
    put(s, "dwconv.sx", sx)
    x64, r64, _, t64 = cases.conv_case(C=64, seed=2)
    q, sx = ref.dwconv(x64, r64, t64, L, quant=True)
    put(s, "dwconv64.q", q)
    put(s, "dwconv64.sx", sx)
    put(s, "lily.out", ref.lily_state(xc, rc, bc, taps, L))
    q, sx = ref.lily_state(xc, rc, bc, taps, L, quant=True)
    put(s, "lily.q", q)
    put(s, "lily.sx", sx)

    xq_, alpha, beta = cases.qk_case()
    put(s, "qk.row", ref.qk_prep(xq_, alpha, beta, 100000.0, L, 4, 64, False))
    put(s, "qk.head", ref.qk_prep(xq_, alpha, beta, 10000.0, L, 4, 64, True))
    c, sn = ref.rope_table(int(L.max()), 100000.0, 64)
    put(s, "rope.cos", c)
    put(s, "rope.sin", sn)
    put(s, "head_major", ref.head_major(xq_, 4, 64))

    put(s, "bmean.out", ref.block_mean(xc, bc, L, 4))
    q, sx = ref.block_mean(xc, bc, L, 4, quant=True)
    put(s, "bmean.q", q)
    put(s, "bmean.sx", sx)
    ybm = ref.block_mean(xc, None, L, 4)
    put(s, "bmean_nog.out", ybm)
    put(s, "upsample.out", ref.upsample_add(ybm, rc, L, 4))

    qa, ka, va, scale = cases.attn_case()
    put(s, "attn.swa", ref.attention(qa, ka, va, 4, 2, 64, 8, scale, cases.LENGTHS_ATTN))
    put(s, "attn.full", ref.attention(qa, ka, va, 4, 2, 64, -1, scale, cases.LENGTHS_ATTN))

    for tag, path in {"tiny_q4km": sm.cached_model("tiny", sm.tiny_hparams(), "Q4_K_M", seed=0),
                      "tiny_q8": sm.cached_model("tiny", sm.tiny_hparams(), "Q8_0", seed=1)}.items():
        h = ref.load(path, 4)
        tok, lens = cases.model_batch(1000, seed=7)
        hid, pooled = ref.encode(h, tok, lens)
        put(s, f"{tag}.hidden", hid)
        put(s, f"{tag}.pooled", pooled)
        _, pooled_raw = ref.encode(h, tok, lens, normalize=False, hidden=False)
        put(s, f"{tag}.pooled_raw", pooled_raw)
        ref.L.nextera_free(h)
    return s


def main() -> int:
    build_oracle(ref=True)
    s = generate(RefLib())
    np.savez_compressed(OUT, **s)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KiB, {len(s)} arrays)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
