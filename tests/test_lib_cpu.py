"""CPU-side checks of libnexterabert.so: it loads without a GPU, exports every
symbol include/*.h declares (plus the reference's debug exports its CLI and
Python binding bind), and fails cleanly where no device exists."""
import ctypes
import subprocess
from pathlib import Path

import pytest

from gpulib import LIB_PATH, header_symbols, load_lib

ROOT = Path(__file__).resolve().parent.parent

# the reference's public API (src/nexterabert.h) and its extra exports (nexterabert.cpp:1818-1841)
REFERENCE_API = [
    "nextera_default_params", "nextera_load", "nextera_free", "nextera_n_embd", "nextera_n_vocab",
    "nextera_n_layer", "nextera_has_mlm_head", "nextera_has_pooler", "nextera_n_token_types",
    "nextera_classifier_task", "nextera_n_labels", "nextera_label", "nextera_token_cls", "nextera_token_sep",
    "nextera_token_pad", "nextera_token_mask", "nextera_tokenizer_json", "nextera_ftype", "nextera_system_info",
    "nextera_set_n_threads", "nextera_get_n_threads", "nextera_encode", "nextera_encode_segments",
    "nextera_pooler_output", "nextera_classify", "nextera_mlm_logits", "nextera_last_ms",
    "nextera_debug_set_layers", "nextera_debug_profile", "nextera_debug_profile_print",
]


@pytest.fixture(scope="module")
def built():
    if not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(LIB_PATH.parent)], check=True)
    return LIB_PATH


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_exports_every_declared_symbol(built):
    syms = exported(built)
    declared = header_symbols()
    assert len(declared) >= 45
    missing = [s for s in declared if s not in syms]
    assert not missing, missing


def test_exports_the_reference_api(built):
    syms = exported(built)
    assert not [s for s in REFERENCE_API if s not in syms]


def test_no_internal_symbols_leak(built):
    syms = exported(built)
    leaked = [s for s in syms if not (s.startswith("nextera_") or s.startswith("nxk_"))
              and not s.startswith("_") and "cuda" not in s.lower()]
    assert not leaked, leaked[:20]


def test_loads_and_binds_without_gpu(built):
    L = load_lib(built)
    p = L.nextera_default_params()
    assert (p.n_threads, p.use_int8, p.use_repack, p.verbosity) == (0, 1, 1, 0)


def test_load_without_device_fails_cleanly(built, tiny_model_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    L = load_lib(built)
    assert not L.nextera_load(str(tiny_model_path).encode(), L.nextera_default_params())


def test_load_rejects_bad_files(built, tmp_path):
    L = load_lib(built)
    bad = tmp_path / "x.gguf"
    bad.write_bytes(b"not a gguf file")
    assert not L.nextera_load(str(bad).encode(), L.nextera_default_params())
    assert not L.nextera_load(str(tmp_path / "missing.gguf").encode(), L.nextera_default_params())


def test_kernel_layer_rejects_unsupported_shapes(built):
    L = load_lib(built)
    # argument checks happen before any device work
    assert L.nxk_linear_i8(None, None, 4, None, None, 1024, 100, None, None, None) == -1   # N not a multiple of 64
    assert L.nxk_rms_norm(None, None, 1e-8, 4, 100, None, None, None, None) == -1         # C not a multiple of 32
    assert L.nxk_attention(None, None, None, 4, 16, 2, 64, -1, None, None, None, None, 1, None, None,
                           None, 0, None, None) == -1                                     # 8 heads per KV head
    # the strided dwconv: rows closer than C floats, or not 16-byte aligned (the output pointer is
    # a placeholder; the checks reject the call before it is used)
    fake = ctypes.c_void_p(256)
    for ld in (60, 66):
        assert L.nxk_dwconv_halo_ld(None, None, ld, None, 5, 0, None, None, None, 4, 64, fake, None, None,
                                    None) == -1


def test_shard_id_without_gpu():
    """The NCCL id of a sharded group is made on the host (no GPU needed): 128 bytes, fresh each call."""
    from gpulib import load_lib, shard_id
    L = load_lib()
    a, b = shard_id(L, 0), shard_id(L, 0)
    assert len(a) == 128 and len(b) == 128 and a != b


def _shard_id_rank(rank, port, q):
    import os
    import torch.distributed as dist
    from gpulib import load_lib, shard_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        q.put((rank, shard_id(load_lib(), rank, dist)))
    finally:
        dist.destroy_process_group()


def test_shard_id_exchange_gloo():
    """Two ranks (gloo, CPU): rank 0's id reaches rank 1 unchanged, as bench.py hands it out."""
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_shard_id_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[0] == got[1] and len(got[0]) == 128


def test_bench_linear_floor_covers_the_counted_linears():
    """bench.py's linear floor walks the same linears as its op count: with a memory rate so high
    that every linear is compute-bound, the floor is the op count at the tcgen05 rate."""
    import importlib.util
    import numpy as np
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    lengths = np.array([16, 17, 100, 511, 2048], dtype=np.int64)
    peak = 4000.0
    floor, comp, mem = bench.linear_floor_ms(lengths, peak, 1e12)
    assert mem == 0.0 and abs(comp - floor) < 1e-12
    assert abs(floor - bench.linear_ops(lengths) / (peak * 1e12) * 1e3) < 1e-9 * floor
    # at the measured rates the fp32-output linears are memory-bound
    floor2, comp2, mem2 = bench.linear_floor_ms(lengths, 4571.0, 6509.4)
    assert mem2 > comp2 and floor2 > floor
