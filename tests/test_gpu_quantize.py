"""The quantizer on the GPU (nxk_quantize_rows, nextera_quantize, nexterabert-quantize), the
counterpart of the reference's tools/quantize.cpp.

  * block level: every type, on rows with zeros and outliers, bit-identical to the CPU encoders -
    gguf-py's quantizers for the legacy types (which restate ggml's reference quantizers) and
    tests/golden/synth_model.py's fits for the K-quants;
  * file level: an F32 file re-encoded to a preset equals, tensor for tensor, the file the fixture
    generator writes for that preset from the same weights (same per-tensor types: the "_M" extra
    bits, the fallback for 64-wide rows, the classifier kept), and it loads and encodes to the same
    bits; --tensor-type overrides and the command line work; bad arguments return 1.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import gguf
import numpy as np
import pytest

import synth_model as sm
from synth_model import QT

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
CLI = ROOT / "nexterabert.cpp_b200" / "nexterabert-quantize"
TYPES = [QT.F16, QT.Q8_0, QT.Q4_0, QT.Q4_1, QT.Q5_0, QT.Q5_1, QT.Q2_K, QT.Q3_K, QT.Q4_K, QT.Q5_K, QT.Q6_K]


@pytest.fixture(scope="module")
def lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpulib import load_lib
    return load_lib()


def cpu_blocks(w, qt):
    if qt == QT.F16:
        return np.ascontiguousarray(w.astype(np.float16)).view(np.uint8).reshape(w.shape[0], -1)
    return sm.quantize_rows(w, qt)


@pytest.mark.parametrize("qt", TYPES, ids=lambda t: t.name)
def test_blocks_bit_identical(lib, qt):
    import torch
    from gpulib import P, host
    rng = np.random.default_rng(100 + int(qt))
    rows, n = 37, 768
    w = (rng.standard_normal((rows, n)) * rng.uniform(0.01, 3.0, (rows, 1))).astype(np.float32)
    w[2] = 0.0                                   # an all-zero row
    w[4, 5] = 250.0                              # an outlier
    w[6, :64] = -1.5                             # a constant run (max = min inside blocks)
    want = cpu_blocks(w, qt)
    x = torch.from_numpy(w).cuda()
    out = torch.full((rows, want.shape[1]), 0xAB, dtype=torch.uint8, device="cuda")
    assert lib.nxk_quantize_rows(int(qt), P(x), n, rows, P(out), None) == 0
    got = host(out)
    assert np.array_equal(got, want), f"{(got != want).sum()} bytes differ"


def test_blocks_reject_bad_shapes(lib):
    assert lib.nxk_quantize_rows(int(QT.Q4_K), None, 512, 1, None, None) == -1
    assert lib.nxk_quantize_rows(int(QT.Q8_0), ctypes.c_void_p(16), 48, 1, ctypes.c_void_p(16), None) == -1   # not a multiple of 32
    assert lib.nxk_quantize_rows(int(QT.Q4_K), ctypes.c_void_p(16), 64, 1, ctypes.c_void_p(16), None) == -1   # not a multiple of 256
    assert lib.nxk_quantize_rows(15, ctypes.c_void_p(16), 256, 1, ctypes.c_void_p(16), None) == -1           # Q8_K: not a file type


def tensors(path):
    r = gguf.GGUFReader(str(path))
    return {t.name: (int(t.tensor_type), np.asarray(t.data).view(np.uint8).tobytes()) for t in r.tensors}


def quantize(lib, src, dst, ftype, overrides=()):
    arr = (ctypes.c_char_p * max(1, len(overrides)))(*[o.encode() for o in overrides])
    return lib.nextera_quantize(str(src).encode(), str(dst).encode(), ftype.encode(), len(overrides), arr)


@pytest.mark.parametrize("preset", ["Q4_K_M", "Q8_0", "Q5_K_M", "F16", "Q4_0"])
def test_file_matches_the_preset_fixture(lib, tmp_path, preset):
    hp = sm.tiny_hparams(cls_task="sequence-classification", n_labels=3, pooler=True)
    src = sm.cached_model("tiny_qsrc", hp, "F32", seed=4)
    want_path = sm.cached_model("tiny_qsrc", hp, preset, seed=4)
    out = tmp_path / f"q-{preset}.gguf"
    assert quantize(lib, src, out, preset) == 0
    got, want = tensors(out), tensors(want_path)
    assert got.keys() == want.keys()
    for name in want:
        assert got[name][0] == want[name][0], (name, got[name][0], want[name][0])
        assert got[name][1] == want[name][1], name
    r = gguf.GGUFReader(str(out))
    assert int(r.fields["general.file_type"].parts[-1][0]) == sm.PRESET_FTYPE[preset]
    assert bytes(r.fields["general.architecture"].parts[-1]).decode() == "nexterabert"
    if preset == "F16":
        return                                   # float encoder matrices are refused at load (f2)
    from test_gpu_model import Model
    import cases
    tok, lens = cases.model_batch(1000, seed=9)
    a, b = Model(lib, out), Model(lib, want_path)
    ra, ha, pa = a.encode(tok, lens)
    rb, hb, pb = b.encode(tok, lens)
    assert ra == 0 and rb == 0
    assert np.array_equal(ha, hb) and np.array_equal(pa, pb)
    a.close()
    b.close()


def test_overrides_cli_and_errors(lib, tmp_path):
    hp = sm.tiny_hparams()
    src = sm.cached_model("tiny_qsrc2", hp, "F32", seed=5)
    out = tmp_path / "o.gguf"
    # every mixer's c_q to Q8_0, the MLP up-projection to Q2_K, on top of Q3_K_M
    assert quantize(lib, src, out, "Q3_K_M", [".attn.c_q.weight=Q8_0", "mlp.c_fc=q2_k"]) == 0
    got = tensors(out)
    w = {k: v for k, v in tensors(src).items()}
    for name, (typ, data) in got.items():
        t_src = w[name][0]
        if "attn.c_q.weight" in name:
            assert typ == int(QT.Q8_0), name
        elif "mlp.c_fc.weight" in name:
            assert typ == int(QT.Q2_K), name
    # a tensor's bytes follow from its type and the F32 weights
    r = gguf.GGUFReader(str(src))
    for t in r.tensors:
        if t.name.endswith("mlp.c_fc.weight"):
            f = np.asarray(t.data).astype(np.float32).reshape(int(t.shape[1]), int(t.shape[0]))
            assert got[t.name][1] == sm.quantize_rows(f, QT.Q2_K).tobytes()
    # the command line, with the reference tool's arguments
    if CLI.exists():
        out2 = tmp_path / "cli.gguf"
        p = subprocess.run([str(CLI), str(src), str(out2), "Q4_K_M", "4"], capture_output=True, text=True, timeout=300)
        assert p.returncode == 0, p.stderr
        assert "-> Q4_K" in p.stdout and "(Q4_K_M)" in p.stdout
        assert tensors(out2) == tensors(sm.cached_model("tiny_qsrc2", hp, "Q4_K_M", seed=5))
    # errors
    assert quantize(lib, src, tmp_path / "x.gguf", "Q9_Z") == 1
    assert quantize(lib, src, tmp_path / "x.gguf", "Q4_K_M", ["c_q=NOPE"]) == 1
    assert quantize(lib, tmp_path / "missing.gguf", tmp_path / "x.gguf", "Q4_K_M") == 1
    assert not (tmp_path / "x.gguf").exists()
