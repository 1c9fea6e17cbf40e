"""One sequence encoded by two, four or eight GPUs (nextera_shard_init / nextera_encode_sharded).

Each rank's rows of the last hidden state and the pooled vector must be bit-identical to the whole
sequence encoded on one GPU: the token convolutions read their neighbours' halo rows, the band
attention the neighbours' K / V rows, the full attention (and HRA) every rank's K / V, and the
pooled sum runs over the ranks in the sequence's order.  Needs two (four, eight) GPUs; skipped otherwise.
"""
from __future__ import annotations

import multiprocessing as mp
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import synth_model as sm  # noqa: E402

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _run_ranks(model_path: Path, tokens: np.ndarray, world: int):
    from gpulib import load_lib, shard_id
    import shard_worker

    L = load_lib()
    nid = shard_id(L, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=shard_worker.run, args=(r, world, str(model_path), nid, tokens.tolist(), q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=600))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join()
    return sorted(results)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("which", ["tiny", "full"])
def test_sharded_sequence_matches_one_gpu(which, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    if which == "tiny":
        path = sm.cached_model("tiny", sm.tiny_hparams(), "Q4_K_M", seed=0)
        n, vocab = 512, 1000
    else:
        path = sm.cached_model("full", sm.full_hparams(), "Q4_K_M", seed=0)
        n, vocab = 2048, 50368
    tokens = sm.random_tokens(n, vocab, seed=11)
    res = _run_ranks(path, tokens, world)
    for r in res:
        assert r[1] == "ok", r
        rank, _, hid_eq, hid_diff, pool_eq, pool_diff = r
        assert hid_eq, f"rank {rank}: hidden rows differ (max |diff| {hid_diff})"
        assert pool_eq, f"rank {rank}: pooled differs (max |diff| {pool_diff})"
