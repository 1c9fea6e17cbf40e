"""The reference's own front ends, unmodified, against this library (the drop-in claim).

oracle/Makefile's `front` target compiles the reference's tools/cli.cpp against
include/nexterabert.h and links it to libnexterabert.so, and stages the reference's
python/nexterabert_cpp.py beside it (oracle/_ref/front/; built where the reference sources are,
and carried with the library).  Here:
  * the CLI runs --info, --ids (one and two sequences, --full), --classify and
    --bench 128 --batch 2 --profile (tools/cli.cpp:155-204, including the two debug exports the
    CLI links, src/nexterabert.cpp:1818-1841);
  * the binding loads the library through $NEXTERABERT_LIB (python/nexterabert_cpp.py:32-90) and
    runs encode_ids, encode (its tokenizer read out of the GGUF), classify, logits_ids,
    pooler_output and fill_mask.
Outputs are compared with the reference compiled here (oracle/_ref) on the same file and ids.
"""
from __future__ import annotations

import importlib.util
import os
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import synth_model as sm

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
FRONT = ROOT / "oracle" / "_ref" / "front"
CLI = FRONT / "nexterabert-cli"
BINDING = FRONT / "nexterabert_cpp.py"
LIB = ROOT / "nexterabert.cpp_b200" / "libnexterabert.so"


@pytest.fixture(scope="module")
def gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def cls_model():
    # the CLI's --bench draws ids from [1000, min(vocab, 40000)) (tools/cli.cpp:180), so the file's
    # vocabulary must exceed 1000 ids
    hp = sm.tiny_hparams(n_vocab=4096, cls_task="sequence-classification", n_labels=3, pooler=True,
                         tokenizer=True)
    return sm.cached_model("tiny_front", hp, "Q4_K_M", seed=21)


def rel_close(got, want, tol=1e-3):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert rel <= tol, rel
    return rel


def run_cli(*args):
    if not CLI.exists():
        pytest.skip("oracle/_ref/front is not built (the reference sources were absent at build time)")
    p = subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True, timeout=600)
    return p.returncode, p.stdout, p.stderr


def parse_rows(out: str):
    rows = []
    for line in out.splitlines():
        m = re.match(r"\[(\d+)\] (?:\((\d+) tokens\)|token \d+:)(.*)", line)
        if m:
            rows.append([float(x) for x in m.group(3).replace("...", "").split()])
    return np.array(rows, np.float32)


def test_cli_info_ids_classify_bench(gpu, reflib, cls_model):
    rc, out, err = run_cli("-m", cls_model, "--info")
    assert rc == 0, err
    assert "int8" in out + err
    seqs = [[996, 5, 17, 300, 997], [996, 42, 997]]
    ids_args = [a for s in seqs for a in ("--ids", ",".join(map(str, s)))]
    toks = np.array([t for s in seqs for t in s], np.int32)
    lens = np.array([len(s) for s in seqs], np.int32)
    r = reflib.load(cls_model, 0)
    try:
        rc, out, err = run_cli("-m", cls_model, *ids_args, "--full")
        assert rc == 0, err
        got = parse_rows(out)
        _, want = reflib.encode(r, toks, lens, hidden=False)
        assert np.abs(got - want).max() <= 1e-6          # printed with 6 decimals
        rc, out, err = run_cli("-m", cls_model, *ids_args, "--classify")
        assert rc == 0, err
        got = parse_rows(out)
        want = reflib.classify(r, toks, lens)
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())
        rc, out, err = run_cli("-m", cls_model, *ids_args, "--pooler")
        assert rc == 0, err
        rel_close(parse_rows(out), reflib.pooler_output(r, toks, lens)[:, :8])
    finally:
        reflib.L.nextera_free(r)
    rc, out, err = run_cli("-m", cls_model, "--bench", 128, "--batch", 2, "--reps", 3, "--profile")
    assert rc == 0, err
    assert re.search(r"bench: .* T=128\s+batch=2 .* tokens/s", out), out
    assert "profile over" in err and "int8 linear" in err, err


def load_binding():
    if not BINDING.exists():
        pytest.skip("oracle/_ref/front is not built (the reference sources were absent at build time)")
    os.environ["NEXTERABERT_LIB"] = str(LIB)
    spec = importlib.util.spec_from_file_location("nexterabert_cpp", BINDING)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_python_binding_unchanged(gpu, reflib, cls_model):
    nb = load_binding()
    m = nb.NexteraBERT(cls_model)
    r = reflib.load(cls_model, 0)
    try:
        assert "int8" in m.system_info
        assert m.task == "sequence-classification" and m.n_labels == 3
        ids = [[996, 5, 17, 300, 997], [996, 42, 997], [996] + list(range(10, 200)) + [997]]
        toks = np.array([t for s in ids for t in s], np.int32)
        lens = np.array([len(s) for s in ids], np.int32)
        pooled, hidden = m.encode_ids(ids, return_hidden=True)
        want_h, want_p = reflib.encode(r, toks, lens)
        rel_close(pooled, want_p)
        rel_close(np.concatenate(hidden), want_h)
        # text in: the tokenizer comes out of the GGUF (tokenizer.huggingface.json)
        texts = ["w5 w17 w300", "w42", "w7 w8 w9 w10"]
        emb = m.encode(texts)
        tids = m.tokenize(texts)
        assert tids[0] == [996, 5, 17, 300, 997]
        for i, t in enumerate(tids):
            _, p = reflib.encode(r, np.array(t, np.int32), np.array([len(t)], np.int32), hidden=False)
            rel_close(emb[i], p[0])
        logits = m.logits_ids(ids)
        want = reflib.classify(r, toks, lens)
        rel_close(logits, want, 1e-5)
        labels = m.classify(texts)
        wl = reflib.classify(r, np.concatenate([np.array(t, np.int32) for t in tids]),
                             np.array([len(t) for t in tids], np.int32))
        probs = np.exp(wl - wl.max(1, keepdims=True))
        probs /= probs.sum(1, keepdims=True)
        for (lab, pr), row in zip(labels, probs):
            assert lab == f"LABEL_{int(row.argmax())}"
            assert abs(pr - row.max()) <= 1e-5
        rel_close(m.pooler_output(ids), reflib.pooler_output(r, toks, lens))
        cand = m.fill_mask("w5 [MASK] w300")
        seq = np.array(m.tokenize(["w5 [MASK] w300"])[0], np.int32)
        ml = reflib.mlm_logits(r, seq, np.array([2], np.int32))
        assert cand[0][0][0] == m.tokenizer.decode([int(ml[0].argmax())])
    finally:
        m.close()
        reflib.L.nextera_free(r)
