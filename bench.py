#!/usr/bin/env python
"""Throughput benchmark: encoded tokens/s on the mixed-length batch (config 4).

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference] [--preset Q4_K_M]

Workload: one batch of 4096 documents with lengths log-uniform in [16, 2048]
(1,685,650 tokens at seed 0), token ids uniform over the vocabulary, through the
random-init NexteraBERT model (18 layers, hidden 1024) quantized to Q4_K_M (or
--preset Q8_0); pooled, L2-normalised embeddings out.  A step encodes the whole
batch.  With N GPUs the batch is partitioned over the ranks by sequence
(nextera_partition: longest-first, balanced on estimated device time), every rank
encodes its share on its own model replica, and the pooled rows are gathered to
rank 0 in batch order over NCCL inside the step: the total work is fixed as N
grows ("scaling": "strong").  A weak-scaling figure (every rank its own
4096-document batch, no exchange) is reported beside it at N > 1.

  value   tokens/s of the batch, each rank's ids already in HBM
          (nextera_encode_partitioned_device), K steps timed with CUDA events on the
          launching stream, barrier and synchronize on both sides, max over ranks
  e2e     the same metric through the public host API (nextera_encode_partitioned):
          every rank passes the batch from pinned host memory, rank 0 gets every
          pooled row back in its host buffer, per step
  roofline, shares: per-kind device time from the library's profiler (one extra
          untimed step; rank 0's share at N > 1), the dominant kind against its peak
  cpu_baseline: the reference's own C++ (oracle/_ref, compiled from its sources)
          on this host's cores over a bounded sample of the same batch (rank 0, N=1)

--impl reference times only that CPU implementation (rank 0; other ranks exit).

--config 5 [--seq-len 65536]: one long sequence instead (its own metric, strong scaling): one GPU
encodes it whole; N ranks share it with nextera_encode_sharded (halo rows and K/V all-gather over
NCCL), value = sequence tokens / step time, max over ranks; the reference encodes a prefix of it
on the host cores (--cpu-prefix).
--config 1: one int8 linear (T=128, K=1024, N=4096, Q8_0), TOPS per launch with an L2 flush before
each, against the measured tcgen05 kind::i8 rate; the model's linear shapes at 131,072 rows beside it.
--config 2: attention alone (64 documents, H=16, G=4; band 128 and full), TFLOP/s per launch.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tests"))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

METRIC = "encoded tokens/s (mixed-length batch, Q4_K_M)"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# The result line is the only thing this program writes to its standard output.  Libraries
# print there too (NCCL announces its version at initialisation when NCCL_DEBUG asks for it),
# so main() points file descriptor 1 at standard error and keeps a copy of the original for emit().
_RESULT_OUT = None


def emit(line: dict) -> None:
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


# ---------------------------------------------------------------- workload
def workload(rank: int, n_docs: int):
    import synth_model as sm
    lengths = sm.throughput_lengths(n_docs, 16, 2048, seed=rank)
    tokens = sm.random_tokens(int(lengths.sum()), 50368, seed=1000 + rank)
    return tokens, lengths


def model_path(preset: str, rank: int, world: int, dist):
    import synth_model as sm
    hp = sm.full_hparams()
    if rank == 0:
        p = sm.cached_model("full", hp, preset, seed=0)
    if world > 1:
        dist.barrier()
    if rank != 0:
        p = sm.cached_model("full", hp, preset, seed=0)
    return p


def linear_ops(lengths) -> float:
    """Algorithmic int8 multiply-adds x 2 of one step (every linear layer, full model)."""
    C, I, H, G, D, r = 1024, 2304, 16, 8, 64, 64
    T = float(np.sum(lengths))
    nb = float(np.sum((lengths + 3) // 4))
    import synth_model as sm
    macs = 0.0
    for bt in sm.FULL_BLOCKS:
        if bt == "lily":
            macs += T * (2 * r * C + C * r + 3 * C * C)
        elif bt in ("swa", "attn"):
            macs += T * (H * D * C + 2 * G * D * C + C * H * D + C * C)
        else:
            macs += T * 5 * C * C + nb * (H * D * C + 2 * G * D * C)
        macs += T * 2 * C * I
    return 2.0 * macs


def linear_floor_ms(lengths, peak_tops: float, hbm_gbs: float):
    """Time floor of one step's int8 linears: per linear, the larger of its multiply-adds at the
    tcgen05 rate and its HBM bytes at the measured copy rate.  Bytes per row: int8 codes in (K, plus
    one fp32 scale per 256 inputs); out fp32 (4N), fp32 read and written again when the linear adds
    into the residual (8N), or int8 codes and scales (c_fc's relu² epilogue).  Weights stay in L2
    and are not counted.  Returns (floor ms, ms of the compute-bound linears, ms of the memory-bound)."""
    C, I, H, G, D, r = 1024, 2304, 16, 8, 64, 64
    T = float(np.sum(lengths))
    nb = float(np.sum((lengths + 3) // 4))
    import synth_model as sm
    F32, RES, CODES = 0, 1, 2
    lins = []                                    # (rows, K, N, output)
    for bt in sm.FULL_BLOCKS:
        if bt == "lily":
            lins += [(T, C, r, F32), (T, C, r, F32), (T, r, C, F32), (T, C, C, F32), (T, C, C, F32),
                     (T, C, C, RES)]
        elif bt in ("swa", "attn"):
            lins += [(T, C, H * D + 2 * G * D, F32), (T, H * D, C, F32), (T, C, C, RES)]
        else:
            lins += [(T, C, C, F32), (T, C, C, F32), (nb, C, H * D + 2 * G * D, F32), (T, C, C, F32),
                     (T, C, C, F32), (T, C, C, RES)]
        lins += [(T, C, I, CODES), (T, I, C, RES)]
    floor = comp = mem = 0.0
    for rows, K, N, kind in lins:
        t_ops = 2.0 * rows * N * K / (peak_tops * 1e12)
        out_b = {F32: 4.0 * N, RES: 8.0 * N, CODES: N + 4.0 * N / 256}[kind]
        t_mem = rows * (K + 4.0 * K / 256 + out_b) / (hbm_gbs * 1e9)
        floor += max(t_ops, t_mem)
        if t_ops >= t_mem:
            comp += t_ops
        else:
            mem += t_mem
    return floor * 1e3, comp * 1e3, mem * 1e3


def attention_work(lengths):
    """(fp32 FLOPs of scores + weighted values, algorithmic bytes of q/k/v/out) of one step."""
    H, G, D, half = 16, 8, 64, 128
    import synth_model as sm
    L = lengths.astype(np.float64)
    nb = np.ceil(L / 4)
    flops, bytes_ = 0.0, 0.0
    for bt in sm.FULL_BLOCKS:
        if bt == "lily":
            continue
        if bt == "swa":
            # keys per query: min(L, t + half + 1) - max(0, t - half), summed over t
            keys = 0.0
            for n in lengths:
                t = np.arange(n)
                keys += float(np.sum(np.minimum(n, t + half + 1) - np.maximum(0, t - half)))
            rows = float(L.sum())
        elif bt == "attn":
            keys, rows = float(np.sum(L * L)), float(L.sum())
        else:
            keys, rows = float(np.sum(nb * nb)), float(nb.sum())
        flops += 4.0 * H * D * keys
        bytes_ += 4.0 * rows * (2 * H * D + 2 * G * D)
    return flops, bytes_


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", gpu_id, "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- CPU reference
def reference_runner():
    """(encode function, cores, kind): the reference compiled here, else the oracle port."""
    from oracle_lib import Oracle, RefLib, ref_library_path
    cores = os.cpu_count() or 1
    if ref_library_path() is not None:
        ref = RefLib()
        state = {}

        def run(path, tokens, lengths):
            if "h" not in state:
                state["h"] = ref.load(path, cores)
            ref.encode(state["h"], tokens, lengths, hidden=False)
        return run, cores, "reference"
    o = Oracle()
    o.L.or_set_threads(cores)
    state = {}

    def run(path, tokens, lengths):
        if "m" not in state:
            state["m"] = o.load(path)
        state["m"].encode(tokens, lengths, hidden=False)
    return run, cores, "port"


def cpu_sample(run, path, tokens, lengths, target_s: float):
    """Docs from the front of the batch whose encode takes about target_s seconds."""
    start = np.concatenate([[0], np.cumsum(lengths)])
    n = 8
    run(path, tokens[:start[n]], lengths[:n])           # load + warm
    t0 = time.perf_counter()
    run(path, tokens[:start[n]], lengths[:n])
    dt = max(time.perf_counter() - t0, 1e-3)
    per_tok = dt / float(start[n])
    want = int(target_s / per_tok)
    n = int(np.searchsorted(start, want))
    n = max(8, min(n, len(lengths)))
    return tokens[:start[n]], lengths[:n]


def time_cpu(run, path, tokens, lengths, steps: int, warmup: int):
    for _ in range(warmup):
        run(path, tokens, lengths)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run(path, tokens, lengths)
        ts.append(time.perf_counter() - t0)
    return float(np.sum(lengths)) / (sum(ts) / len(ts)), 1000.0 * sum(ts) / len(ts)


def base_line(args, world):
    return {"metric": METRIC, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8+fp32",
            "data": "synthetic (seeded lengths and token ids; random-init weights N(0,0.02), Q4_K_M)"}


def config(args, world, tokens):
    return {"workload": f"cfg4 mixed-length batch: {args.docs} docs, lengths log-uniform [16, 2048], "
                        f"{args.preset} random-init NexteraBERT (18 layers, hidden 1024), one batch partitioned "
                        f"over {world} GPU(s)",
            "model": "NexteraBERT-synthetic (8 lily / 6 swa / 2 attn / 2 hra)", "preset": args.preset,
            "docs": args.docs, "tokens_per_step": int(tokens),
            "global_batch": args.docs, "seq_len": "16-2048 (unpadded)",
            "parallelism": f"dp{world}: sequences of one batch partitioned longest-first by estimated cost "
                           "(nextera_partition), replicated weights, pooled rows gathered to rank 0 over NCCL"
                           if world > 1 else "one GPU",
            "l2": "inputs larger than L2 (each activation tensor ~6.9 GB at one GPU, ~0.9 GB per GPU at 8)"}


LONG_METRIC = "encoded tokens/s (one 65,536-token sequence, Q4_K_M)"


def run_long(args, rank, world, local_rank, dist):
    """Config 5: one sequence of args.seq_len ids; N ranks share it (nextera_encode_sharded), so the
    total work is fixed as N grows ("scaling": "strong")."""
    import torch
    import synth_model as sm
    from gpulib import load_lib, shard_id

    torch.cuda.set_device(local_rank)
    dev_uuid = str(torch.cuda.get_device_properties(local_rank).uuid)
    gpu_id = dev_uuid if dev_uuid.startswith("GPU-") else f"GPU-{dev_uuid}"
    L = load_lib()
    path = model_path(args.preset, rank, world, dist)
    n_total = args.seq_len
    if n_total % (4 * world):
        raise SystemExit(f"--seq-len must be a multiple of 4 x {world}")
    n_local = n_total // world
    tokens = sm.random_tokens(n_total, 50368, seed=5)
    h = L.nextera_load(str(path).encode(), L.nextera_default_params())
    assert h, "nextera_load failed"
    C = 1024
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    local = np.ascontiguousarray(tokens[rank * n_local:(rank + 1) * n_local])
    d_tok = torch.from_numpy(local).cuda()
    d_pool = torch.empty(C, dtype=torch.float32, device="cuda")
    lens = (ctypes.c_int32 * 1)(n_total)
    if world > 1:
        rc = L.nextera_shard_init(h, rank, world, shard_id(L, rank, dist))
        assert rc == 0, f"nextera_shard_init returned {rc}"

    def step(tok):
        if world == 1:
            rc = L.nextera_encode_device(h, ctypes.c_void_p(tok.data_ptr()), None, lens, 1, None,
                                         ctypes.c_void_p(d_pool.data_ptr()), 1, sptr)
        else:
            rc = L.nextera_encode_sharded(h, ctypes.c_void_p(tok.data_ptr()), n_local, n_total, None,
                                          ctypes.c_void_p(d_pool.data_ptr()), 1, sptr)
        assert rc == 0, f"encode returned {rc}"

    if args.profile_run:
        step(d_tok)
        torch.cuda.synchronize()
        return
    for _ in range(args.warmup):
        step(d_tok)
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = L.nextera_debug_launches(h)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step(d_tok)
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = int(L.nextera_debug_launches(h) - l0)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = n_total / (ms_step * 1e-3)

    # e2e: this rank's ids from pinned host memory, the pooled vector back to the host, every step
    h_tok = torch.from_numpy(local).pin_memory()
    h_pool = torch.empty(C, dtype=torch.float32).pin_memory()
    d_tok2 = torch.empty_like(d_tok)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        d_tok2.copy_(h_tok, non_blocking=True)
        step(d_tok2)
        h_pool.copy_(d_pool, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / args.steps
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": n_total / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(4 * n_local),
           "d2h_bytes_per_step": int(4 * C), "ms_per_step": 1000.0 * e2e_s,
           "api": "nextera_encode_device / nextera_encode_sharded with pinned host copies in the timed loop"}
    L.nextera_free(h)
    log(f"rank {rank}: {ms_step:.1f} ms/step, {value:.0f} tokens/s, e2e {e2e['value']:.0f} tokens/s")
    # the reference on this box's cores: one sequence made of the first --cpu-prefix ids (the whole
    # 65,536-token sequence takes the reference about 99 s on 18 cores, so a prefix stands in)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        run, cores, kindname = reference_runner()
        n_pre = min(args.cpu_prefix, n_total)
        pre = np.ascontiguousarray(tokens[:n_pre])
        pl = np.array([n_pre], np.int32)
        run(path, pre[:512], np.array([512], np.int32))          # load + warm
        t0 = time.perf_counter()
        run(path, pre, pl)
        cs = time.perf_counter() - t0
        cpu = {"value": n_pre / cs, "unit": "tokens/s", "cores": cores, "kind": kindname, "ms": 1e3 * cs,
               "sample": f"one sequence of the first {n_pre} ids of the {n_total}-token sequence, one timed encode "
                         "(attention cost per token grows with length, so the full sequence runs slower)"}
    if world > 1:
        dist.barrier()
    if rank == 0:
        att_flops, _ = attention_work(np.array([n_total]))
        line = {"metric": LONG_METRIC, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "int8+fp32", "data": "synthetic (seeded token ids; random-init weights N(0,0.02))",
                "value": value, "ms_per_step": ms_step, "e2e": e2e, "clocks": clocks, "gpu_launches": launches,
                "cpu_baseline": cpu,
                "config": {"workload": f"cfg5: one sequence of {n_total} ids, {args.preset} random-init NexteraBERT "
                                       "(18 layers, hidden 1024)",
                           "seq_len": n_total, "tokens_per_gpu_step": n_local,
                           "parallelism": f"sequence sharded over {world} GPU(s): halo rows and K/V all-gather "
                                          "over NCCL" if world > 1 else "one GPU",
                           "linear_int_ops_per_step": linear_ops(np.array([n_total])),
                           "attention_flop_per_step": att_flops}}
        emit(line)


# ---------------------------------------------------------------- main
def run_reference(args, rank, world, dist):
    if rank != 0:
        return
    path = model_path(args.preset, 0, 1, None)
    tokens, lengths = workload(0, args.docs)
    run, cores, kind = reference_runner()
    st, sl = cpu_sample(run, path, tokens, lengths, target_s=8.0)
    v, ms = time_cpu(run, path, st, sl, args.steps, args.warmup)
    sample = f"first {len(sl)} docs ({int(sl.sum())} tokens) of the rank-0 batch per step"
    line = base_line(args, world)
    line.update({"impl": "reference", "value": v, "ms_per_step": ms, "n_gpus": world,
                 "config": config(args, world, int(lengths.sum())),
                 "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample},
                 "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    emit(line)


def hbm_peak():
    """(GB/s, source): the driver-measured copy bandwidth, else the earlier measurement on this pool."""
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    if "hbm_gbs" in peaks:
        return float(peaks["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    return 6650.0, "6650 GB/s, an earlier copy measurement on this pool (of fallback: MEASURED_PEAKS.json absent)"


def int8_peak_tops(torch) -> float:
    """Measured dense int8 throughput of the library GEMM (cuBLASLt via torch._int_mm), TOPS."""
    n = 8192
    a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = 1e30
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def fp32_peak_tflops(torch) -> float:
    """Measured fp32 FMA throughput: cuBLAS SGEMM with TF32 off (CUDA-core FFMA), 8192^3, TFLOP/s."""
    n = 8192
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(2):
        torch.matmul(a, b)
    best = 1e30
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def run_b200(args, rank, world, local_rank, dist):
    import torch
    from gpulib import load_lib, shard_id

    torch.cuda.set_device(local_rank)
    dev_uuid = str(torch.cuda.get_device_properties(local_rank).uuid)
    gpu_id = dev_uuid if dev_uuid.startswith("GPU-") else f"GPU-{dev_uuid}"
    L = load_lib()
    path = model_path(args.preset, rank, world, dist)
    # one batch for the whole job (strong scaling): every rank holds the same lengths and ids and
    # encodes the share nextera_partition gives it
    tokens, lengths = workload(0, args.docs)
    T, n_docs, C = int(lengths.sum()), len(lengths), 1024
    h = L.nextera_load(str(path).encode(), L.nextera_default_params())
    assert h, "nextera_load failed"
    if world > 1:
        rc = L.nextera_shard_init(h, rank, world, shard_id(L, rank, dist))
        assert rc == 0, f"nextera_shard_init returned {rc}"
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    lens = np.ascontiguousarray(lengths, np.int32)
    i32 = ctypes.POINTER(ctypes.c_int32)
    lens_p = lens.ctypes.data_as(i32)
    part = np.empty(n_docs, np.int32)
    assert L.nextera_partition(h, lens_p, n_docs, world, part.ctypes.data_as(i32)) == 0
    starts = np.concatenate([[0], np.cumsum(lengths)])
    mine = np.flatnonzero(part == rank)
    my_tok = np.ascontiguousarray(np.concatenate([tokens[starts[i]:starts[i + 1]] for i in mine]), np.int32)
    d_tok = torch.from_numpy(my_tok).cuda()
    d_pool = torch.empty((n_docs, C), dtype=torch.float32, device="cuda") if rank == 0 else None
    pool_p = ctypes.c_void_p(d_pool.data_ptr()) if rank == 0 else None

    def step():
        rc = L.nextera_encode_partitioned_device(h, ctypes.c_void_p(d_tok.data_ptr()), lens_p, n_docs, pool_p, 1,
                                                 sptr)
        assert rc == 0, f"nextera_encode_partitioned_device returned {rc}"

    if args.profile_run:
        step()
        torch.cuda.synchronize()
        return

    def timed(fn, steps):
        """K calls between CUDA events on the launching stream, barrier + synchronize on both
        sides; (ms per step, max over ranks; launches of this rank)."""
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        l0 = L.nextera_debug_launches(h)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(steps):
            fn()
        ev1.record(stream)
        torch.cuda.synchronize()
        launches_ = int(L.nextera_debug_launches(h) - l0)
        if world > 1:
            dist.barrier()
        ms_ = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([ms_], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_ = float(t.item())
        return ms_ / steps, launches_

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    ms_step, launches = timed(step, args.steps)
    clocks = sampler.stop()
    value = T / (ms_step * 1e-3)
    my_ms = None
    if world > 1:
        # this rank's own share alone (no gather), to show the balance of the partition
        lens_mine = np.ascontiguousarray(lengths[mine], np.int32)
        d_mine_pool = torch.empty((len(mine), C), dtype=torch.float32, device="cuda")

        def local():
            assert L.nextera_encode_device(h, ctypes.c_void_p(d_tok.data_ptr()), None,
                                           lens_mine.ctypes.data_as(i32), len(mine), None,
                                           ctypes.c_void_p(d_mine_pool.data_ptr()), 1, sptr) == 0
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            local()
        e1.record(stream)
        torch.cuda.synchronize()
        mine_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device="cuda")
        allms = [torch.zeros_like(mine_ms) for _ in range(world)]
        dist.all_gather(allms, mine_ms)
        my_ms = [float(x.item()) for x in allms]
        del d_mine_pool

    # e2e through the host API: every rank passes the whole batch from pinned host memory; rank 0
    # gets every pooled row back in batch order
    h_tok = torch.from_numpy(tokens).pin_memory().numpy()
    h_pool = torch.empty((n_docs, C), dtype=torch.float32).pin_memory().numpy()
    f32 = ctypes.POINTER(ctypes.c_float)

    def host_call():
        rc = L.nextera_encode_partitioned(h, h_tok.ctypes.data_as(i32), None, lens_p, n_docs,
                                          h_pool.ctypes.data_as(f32) if rank == 0 else None, 1)
        assert rc == 0, f"nextera_encode_partitioned returned {rc}"
    host_call()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_call()
    e2e_s = (time.perf_counter() - t0) / args.steps
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": T / e2e_s, "unit": "tokens/s",
           "h2d_bytes_per_step": int(4 * T + 4 * (3 * T + (T + 3) // 4 + 4 * n_docs)),
           "d2h_bytes_per_step": int(4 * n_docs * C), "ms_per_step": 1000.0 * e2e_s,
           "api": "nextera_encode_partitioned (host buffers; every rank passes the batch, rank 0 receives "
                  "all pooled rows)"}

    # weak scaling beside it: every rank encodes its own whole batch (seed = rank), no exchange
    weak = None
    if world > 1 and not args.no_weak:
        wt, wl = workload(rank, args.docs)
        wlens = np.ascontiguousarray(wl, np.int32)
        d_wtok = torch.from_numpy(wt).cuda()
        d_wpool = torch.empty((len(wl), C), dtype=torch.float32, device="cuda")

        def wstep():
            assert L.nextera_encode_device(h, ctypes.c_void_p(d_wtok.data_ptr()), None, wlens.ctypes.data_as(i32),
                                           len(wl), None, ctypes.c_void_p(d_wpool.data_ptr()), 1, sptr) == 0
        for _ in range(max(1, args.warmup - 1)):
            wstep()
        wms, _ = timed(wstep, args.steps)
        tt = torch.tensor([float(wl.sum())], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        weak = {"value": float(tt.item()) / (wms * 1e-3), "unit": "tokens/s", "ms_per_step": wms,
                "scaling": "weak", "docs_per_gpu": args.docs,
                "how": "every rank encodes its own 4096-document batch (seed = rank) with nextera_encode_device; "
                       "tokens of all ranks / max-over-ranks step time"}
        del d_wtok, d_wpool

    # per-kind device time (one extra, untimed, profiled step)
    L.nextera_debug_profile(h, 1)
    host_call()
    kind = (ctypes.c_double * 3)()
    tot = ctypes.c_double()
    L.nextera_debug_profile_get(h, kind, ctypes.byref(tot))
    L.nextera_debug_profile(h, 0)
    k_ms = {"int8_linear": kind[0], "attention": kind[1], "row_ops": kind[2]}
    dev_ms = sum(k_ms.values())
    shares = {k: v / dev_ms for k, v in k_ms.items()}
    hbm_pk, hbm_src = hbm_peak()
    # the profiled call's work: this rank's share of the batch (rank 0 reports)
    lin_ops = linear_ops(lengths[mine])
    att_flops, att_bytes = attention_work(lengths[mine])
    top = max(k_ms, key=k_ms.get)
    roof = None
    if rank == 0:
        i8_peak = i8_mma_peak(torch, L, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        lin = {"bound": "tensor", "achieved": lin_ops / (k_ms["int8_linear"] * 1e-3) / 1e12, "peak": i8_peak,
               "unit": "TOPS", "kernel": "gemm_i8_tc (int8 linear layers)",
               "peak_source": "tcgen05 kind::i8 rate measured in this run (nxk_i8_mma_rate_probe: operands "
                              "resident in shared memory, one CTA per SM, burst)",
               "library_int8_gemm_tops": int8_peak_tops(torch),
               "library_source": "cuBLASLt dense int8 (torch._int_mm 8192^3) in this run",
               "algorithmic": "sum over the step's 141-per-token int8 linears of 2*T*N*K"}
        lin["frac"] = lin["achieved"] / lin["peak"]
        fl, fl_c, fl_m = linear_floor_ms(lengths[mine], i8_peak, hbm_pk)
        lin["floor_ms"] = fl
        lin["frac_of_floor"] = fl / k_ms["int8_linear"]
        lin["floor"] = (f"per linear the larger of its multiply-adds at the tcgen05 rate and its HBM bytes "
                        f"(int8 codes in; fp32 out, residual read and written, or codes out) at {hbm_src}: "
                        f"{fl_c:.1f} ms from compute-bound linears, {fl_m:.1f} ms from memory-bound ones")
        f32_peak = fp32_peak_tflops(torch)
        # the attention's arithmetic is fixed fp32 fused multiply-add chains in the reference's
        # order, which tensor cores cannot reproduce: its ceiling is the CUDA-core FMA pipe
        att = {"bound": "fp32", "achieved": att_flops / (k_ms["attention"] * 1e-3) / 1e12, "peak": f32_peak,
               "unit": "TFLOP/s", "kernel": "attn_tiled_kernel (exact varlen GQA)",
               "peak_source": "fp32 FMA throughput measured in this run (cuBLAS SGEMM, TF32 off, 8192^3)",
               "algorithmic": "2 * 64 multiply-adds per (query, head, key) for the scores and again for the "
                              "weighted values, keys in each query's range",
               "hbm_gbs": att_bytes / (k_ms["attention"] * 1e-3) / 1e9, "hbm_peak_gbs": hbm_pk,
               "hbm_peak_source": hbm_src,
               "hbm_algorithmic": "q + k + v read, output written once per attention layer (fp32)"}
        att["frac"] = att["achieved"] / att["peak"]
        roof = lin if top == "int8_linear" else att if top == "attention" else None
        if roof is None:
            roof = {"bound": "hbm", "achieved": None, "peak": hbm_pk, "unit": "GB/s", "frac": None,
                    "kernel": "row ops", "peak_source": hbm_src}
        tf = ROOT / "profiles" / "traffic.json"
        roof["traffic"] = None
        if tf.exists():
            try:
                tr = json.loads(tf.read_text())
                roof["traffic"] = tr.get(roof["kernel"].split()[0], {}).get("bytes_per_launch")
            except ValueError:
                pass
        roof = dict(roof)
        roof["by_kind"] = {"int8_linear": dict(lin), "attention": dict(att)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        run, cores, kindname = reference_runner()
        st, sl = cpu_sample(run, path, tokens, lengths, target_s=6.0)
        cv, cms = time_cpu(run, path, st, sl, 1, 0)
        cpu = {"value": cv, "unit": "tokens/s", "cores": cores, "kind": kindname,
               "sample": f"first {len(sl)} docs ({int(sl.sum())} tokens) of the batch, one timed encode"}
    L.nextera_free(h)
    log(f"rank {rank}: {ms_step:.1f} ms/step, {value:.0f} tokens/s, e2e {e2e['value']:.0f} tokens/s, kinds {k_ms}")
    if rank == 0:
        line = base_line(args, world)
        line.update({"value": value, "ms_per_step": ms_step, "config": config(args, world, T),
                     "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
                     "gpu_launches": launches, "device_ms_by_kind": k_ms, "shares": shares,
                     "device_ms_by_kind_rank0": "rank 0's share of the batch, one profiled host call"})
        if my_ms is not None:
            line["rank_ms_alone"] = my_ms
            line["partition"] = {"docs_per_rank": [int(np.sum(part == r)) for r in range(world)],
                                 "tokens_per_rank": [int(lengths[part == r].sum()) for r in range(world)]}
        if weak is not None:
            line["weak_scaling"] = weak
        emit(line)


# ---------------------------------------------------------------- configs 1 and 2 (one kernel each)
def flush_l2(torch, buf):
    """Writes a buffer larger than L2 (126 MB) so the next launch starts with a cold cache."""
    buf.fill_(1)


def event_times(torch, stream, fn, steps, flush=None):
    """ms of each of `steps` launches of fn, each between its own CUDA events on `stream`, an L2
    flush before each (outside the events) when given."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        if flush is not None:
            flush()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def i8_mma_peak(torch, L, sptr):
    """Measured tcgen05 kind::i8 rate with operands resident in shared memory (one CTA per SM, the
    GEMM's M 128 x N 256 x K 32 MMAs, no copies, no epilogue): TOPS, burst."""
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    iters = 20000
    ops = 2.0 * 128 * 256 * 128 * iters * sms
    assert L.nxk_i8_mma_rate_probe(sms, iters, sptr) == 0
    torch.cuda.synchronize()
    ts = event_times(torch, torch.cuda.current_stream(), lambda: L.nxk_i8_mma_rate_probe(sms, iters, sptr), 5)
    assert L.nxk_take_error(sptr) == 0
    return ops / (min(ts) * 1e-3) / 1e12


def run_cfg1(args):
    """Config 1: one int8 linear, X [128, 1024] ~ N(0,1), W [4096, 1024] ~ N(0, 0.02) in Q8_0 (expanded
    on the device by nxk_expand_weight, X quantized by nxk_quantize), timed per launch with an L2 flush
    before each; the model's own linear shapes at 131,072 rows beside it."""
    import torch
    import cases
    from gpulib import load_lib
    from synth_model import QT
    torch.cuda.set_device(0)
    L = load_lib()
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    x, wb = cases.cfg1_case()
    T, K, N = 128, 1024, 4096
    d_blocks = torch.from_numpy(np.ascontiguousarray(wb).view(np.uint8).reshape(-1)).cuda()
    w8 = torch.empty((N, K), dtype=torch.int8, device="cuda")
    sw = torch.empty(((K + 255) // 256, N), dtype=torch.float32, device="cuda")
    assert L.nxk_expand_weight(int(QT.Q8_0), P(d_blocks), K, N, P(w8), P(sw), None, sptr) == 0
    d_x = torch.from_numpy(x).cuda()
    xq = torch.empty((T, K), dtype=torch.int8, device="cuda")
    sx = torch.empty((T, K // 256), dtype=torch.float32, device="cuda")
    assert L.nxk_quantize(P(d_x), T, K, P(xq), P(sx), sptr) == 0
    out = torch.empty((T, N), dtype=torch.float32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def lin():
        assert L.nxk_linear_i8(P(xq), P(sx), T, P(w8), P(sw), K, N, None, P(out), sptr) == 0
    for _ in range(args.warmup):
        lin()
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_uuid(torch, 0))
    time.sleep(0.3)
    ts = event_times(torch, stream, lin, args.steps, flush=lambda: flush_l2(torch, flush))
    warm = event_times(torch, stream, lin, args.steps)
    clocks = sampler.stop()
    assert L.nxk_take_error(sptr) == 0
    ms = statistics.median(ts)
    ops = 2.0 * T * N * K
    tops = ops / (ms * 1e-3) / 1e12
    peak = i8_mma_peak(torch, L, sptr)
    lib_peak = int8_peak_tops(torch)

    # the model's linear shapes at 131,072 rows (inputs > L2): plain, residual, relu^2 + quantize
    big = []
    Tb = 131072
    for (Kb, Nb, kind) in ((1024, 1024, "plain"), (1024, 1024, "residual"), (2304, 1024, "residual"),
                           (1024, 2304, "relu2_q")):
        xb = torch.randint(-127, 128, (Tb, Kb), dtype=torch.int8, device="cuda")
        sxb = torch.rand((Tb, Kb // 256), device="cuda") * 0.01
        wb8 = torch.randint(-127, 128, (Nb, Kb), dtype=torch.int8, device="cuda")
        swb = torch.rand((Kb // 256 + (1 if Kb % 256 else 0), Nb), device="cuda") * 0.01
        if kind == "relu2_q":
            qo = torch.empty((Tb, Nb), dtype=torch.int8, device="cuda")
            so = torch.empty((Tb, Nb // 256), dtype=torch.float32, device="cuda")
            fn = lambda: L.nxk_linear_i8_relu_sqr_q(P(xb), P(sxb), Tb, P(wb8), P(swb), Kb, Nb, P(qo), P(so), sptr)  # noqa
        else:
            ob = torch.zeros((Tb, Nb), dtype=torch.float32, device="cuda")
            res = ob if kind == "residual" else None
            fn = lambda: L.nxk_linear_i8(P(xb), P(sxb), Tb, P(wb8), P(swb), Kb, Nb, P(res), P(ob), sptr)  # noqa
        for _ in range(3):
            assert fn() == 0
        tb = statistics.median(event_times(torch, stream, lambda: fn(), 10))
        big.append({"T": Tb, "K": Kb, "N": Nb, "epilogue": kind, "ms": tb,
                    "tops": 2.0 * Tb * Kb * Nb / (tb * 1e-3) / 1e12,
                    "frac_of_mma_peak": 2.0 * Tb * Kb * Nb / (tb * 1e-3) / 1e12 / peak})
        del xb, sxb, wb8, swb
    assert L.nxk_take_error(sptr) == 0

    cpu = None
    if not args.no_cpu_baseline:
        from oracle_lib import RefLib, ref_library_path
        if ref_library_path() is not None:
            r = RefLib()
            w_h, sw_h, off_h = r.build_i8_weight(int(QT.Q8_0), wb, K, N)
            xq_h, sx_h = r.quantize_rows(x)
            r.linear_i8(xq_h, sx_h, w_h, sw_h, off_h)
            cts = []
            for _ in range(max(3, args.steps)):
                t0 = time.perf_counter()
                r.linear_i8(xq_h, sx_h, w_h, sw_h, off_h)
                cts.append(time.perf_counter() - t0)
            cms = 1e3 * statistics.median(cts)
            cpu = {"value": ops / (cms * 1e-3) / 1e12, "unit": "TOPS", "ms": cms, "cores": os.cpu_count() or 1,
                   "kind": "reference", "sample": "the whole cfg-1 linear (op_linear_i8 of oracle/_ref, all threads)"}
    emit({"metric": "int8 GEMM TOPS (cfg1: one linear, T=128, K=1024, N=4096, Q8_0)", "unit": "TOPS",
          "value": tops, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
          "scaling": "none", "vs_baseline": None, "dtype": "int8 (s8 x s8 -> s32, fp32 epilogue)",
          "data": "synthetic (seeded X ~ N(0,1), W ~ N(0, 0.02) in Q8_0)", "ms_per_step": ms,
          "us_per_launch": 1e3 * ms, "us_per_launch_warm_l2": 1e3 * statistics.median(warm),
          "config": {"workload": "cfg1: X [128, 1024] int8 (row-quantized) x W [4096, 1024] int8 (Q8_0 expanded)",
                     "l2": "flushed before every timed launch (256 MB write)"},
          "roofline": {"bound": "tensor", "achieved": tops, "peak": peak, "unit": "TOPS", "frac": tops / peak,
                       "traffic": None,
                       "peak_source": "tcgen05 kind::i8 rate measured in this run (nxk_i8_mma_rate_probe: operands "
                                      "resident in shared memory, one CTA per SM, burst)",
                       "library_int8_gemm_tops": lib_peak,
                       "library_source": "cuBLASLt dense int8 (torch._int_mm 8192^3) in this run"},
          "model_shapes": big, "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": args.steps * 2})


def run_cfg2(args):
    """Config 2: attention alone over 64 documents (lengths U[16, 2048], 67,328 tokens), H=16, G=4, D=64;
    a band layer (window 128) and a full layer, each timed per launch."""
    import torch
    import synth_model as sm
    from gpulib import load_lib
    torch.cuda.set_device(0)
    L = load_lib()
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    H, G, D = 16, 4, 64
    lengths = np.ascontiguousarray(sm.uniform_lengths(64, 16, 2048, seed=0), np.int32)
    T = int(lengths.sum())
    rng = np.random.default_rng(2)
    q = rng.standard_normal((T, H * D)).astype(np.float32)
    k = rng.standard_normal((G, T, D)).astype(np.float32)
    v = rng.standard_normal((G, T, D)).astype(np.float32)
    scale = np.full(64, 0.125, np.float32)
    start = np.ascontiguousarray(np.concatenate([[0], np.cumsum(lengths)[:-1]]), np.int32)
    row_doc = np.repeat(np.arange(64, dtype=np.int32), lengths)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    ds, dst, dlen, drow = (torch.from_numpy(a).cuda() for a in (scale, start, lengths, row_doc))
    out = torch.empty((T, H * D), dtype=torch.float32, device="cuda")
    i32 = ctypes.POINTER(ctypes.c_int32)
    peak = fp32_peak_tflops(torch)
    hbm, hbm_src = hbm_peak()
    res = {}
    sampler = ClockSampler(gpu_uuid(torch, 0))
    time.sleep(0.3)
    for name, half in (("swa_window128", 64), ("global", -1)):
        wsb = int(L.nxk_attention_workspace(lengths.ctypes.data_as(i32), 64, half))
        ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device="cuda")

        def att():
            assert L.nxk_attention(P(dq), P(dk), P(dv), T, H, G, D, half, P(ds), P(drow), P(dst), P(dlen), 64,
                                   start.ctypes.data_as(i32), lengths.ctypes.data_as(i32), P(ws), ws.numel(),
                                   P(out), sptr) == 0
        for _ in range(args.warmup):
            att()
        ms = statistics.median(event_times(torch, stream, att, args.steps))
        keys = 0.0
        for n in lengths.astype(np.int64):
            t = np.arange(n)
            keys += float(np.sum(np.minimum(n, t + half + 1) - np.maximum(0, t - half))) if half >= 0 else float(n * n)
        flops = 4.0 * H * D * keys
        byts = 4.0 * T * (2 * H * D + 2 * G * D)
        res[name] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "frac_fp32_peak": flops / (ms * 1e-3) / 1e12 / peak,
                     "gbs": byts / (ms * 1e-3) / 1e9, "frac_hbm": byts / (ms * 1e-3) / 1e9 / hbm,
                     "flop": flops, "algorithmic_bytes": byts}
        del ws
    clocks = sampler.stop()
    assert L.nxk_take_error(sptr) == 0
    cpu = None
    if not args.no_cpu_baseline:
        from oracle_lib import RefLib, ref_library_path
        if ref_library_path() is not None:
            r = RefLib()
            cpu = {}
            n_s = 6                                            # the first documents, about 6,000 tokens
            Ts = int(lengths[:n_s].sum())
            for name, half in (("swa_window128", 64), ("global", -1)):
                args_ = (q[:Ts], np.ascontiguousarray(k[:, :Ts]), np.ascontiguousarray(v[:, :Ts]), H, G, D, half,
                         scale[:n_s], lengths[:n_s])
                t0 = time.perf_counter()
                r.attention(*args_)
                cs = time.perf_counter() - t0
                keys = 0.0
                for n in lengths[:n_s].astype(np.int64):
                    t = np.arange(n)
                    keys += float(np.sum(np.minimum(n, t + half + 1) - np.maximum(0, t - half))) if half >= 0 \
                        else float(n * n)
                cpu[name] = {"value": 4.0 * H * D * keys / cs / 1e12, "unit": "TFLOP/s", "ms": 1e3 * cs}
            cpu.update({"cores": os.cpu_count() or 1, "kind": "reference",
                        "sample": f"first {n_s} documents ({Ts} tokens) through op_attention of oracle/_ref"})
    tot_ms = res["swa_window128"]["ms"] + res["global"]["ms"]
    tot_flop = res["swa_window128"]["flop"] + res["global"]["flop"]
    emit({"metric": "attention TFLOP/s (cfg2: 64 docs, H=16, G=4, D=64; band 128 + full)", "unit": "TFLOP/s",
          "value": tot_flop / (tot_ms * 1e-3) / 1e12, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
          "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "fp32",
          "data": "synthetic (seeded q, k, v ~ N(0,1))", "ms_per_step": tot_ms, "variants": res,
          "config": {"workload": f"cfg2: {T} tokens in 64 documents, lengths U[16, 2048] (seed 0)",
                     "l2": "inputs larger than L2 (q alone 276 MB)"},
          "roofline": {"bound": "fp32", "achieved": tot_flop / (tot_ms * 1e-3) / 1e12, "peak": peak,
                       "unit": "TFLOP/s", "frac": tot_flop / (tot_ms * 1e-3) / 1e12 / peak, "traffic": None,
                       "peak_source": "cuBLAS SGEMM, TF32 off, 8192^3, measured in this run"},
          "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": 2 * args.steps})


def gpu_uuid(torch, i):
    u = str(torch.cuda.get_device_properties(i).uuid)
    return u if u.startswith("GPU-") else f"GPU-{u}"



HEADS_METRIC = "classified documents/s (mixed-length batch, sequence classification, Q4_K_M)"


def run_heads(args):
    """--heads (one GPU): the task heads on the full-size model with a 2-label sequence classifier.

    * classify: nextera_classify over the config-4 batch (host API, wall clock around each call,
      which returns after the logits are on the host), beside nextera_encode on the same batch;
    * mlm_logits: fill-mask shape, one 512-token sequence with 77 masked positions (host API);
    * the decoder alone: nxk_mul_mat over the 50368 x 1024 Q4_K embedding table for 8, 77 and 512
      rows, CUDA events on the launching stream, against the HBM peak (table bytes + output);
    * the reference (oracle/_ref) on the host cores for mlm_logits of the same shape."""
    import torch
    import heads_util as hu
    import synth_model as sm
    from gpulib import load_lib

    torch.cuda.set_device(0)
    L = load_lib()
    hp = sm.full_hparams(cls_task="sequence-classification", n_labels=2)
    path = sm.cached_model("full_cls", hp, args.preset, seed=0)
    tokens, lengths = workload(0, args.docs)
    T, n_docs = int(lengths.sum()), len(lengths)
    h = L.nextera_load(str(path).encode(), L.nextera_default_params())
    assert h, "nextera_load failed"
    i32 = ctypes.POINTER(ctypes.c_int32)
    f32 = ctypes.POINTER(ctypes.c_float)
    tok = np.ascontiguousarray(tokens, np.int32)
    lens = np.ascontiguousarray(lengths, np.int32)
    logits = np.empty((n_docs, 2), np.float32)
    pooled = np.empty((n_docs, 1024), np.float32)

    def wall(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return sum(ts) / len(ts)

    def classify():
        assert L.nextera_classify(h, tok.ctypes.data_as(i32), None, lens.ctypes.data_as(i32), n_docs,
                                  logits.ctypes.data_as(f32)) == 0

    def encode():
        assert L.nextera_encode(h, tok.ctypes.data_as(i32), lens.ctypes.data_as(i32), n_docs, None,
                                pooled.ctypes.data_as(f32), 1) == 0

    t_cls = wall(classify, args.steps, args.warmup)
    t_enc = wall(encode, args.steps, args.warmup)
    log(f"classify {t_cls * 1e3:.1f} ms, encode {t_enc * 1e3:.1f} ms per batch")

    seq = sm.random_tokens(512, hp.n_vocab, seed=77)
    pos = np.ascontiguousarray(np.sort(np.random.default_rng(78).choice(512, 77, replace=False)), np.int32)
    ml = np.empty((77, hp.n_vocab), np.float32)

    def mlm():
        assert L.nextera_mlm_logits(h, seq.ctypes.data_as(i32), 512, pos.ctypes.data_as(i32), 77,
                                    ml.ctypes.data_as(f32)) == 0

    t_mlm = wall(mlm, 10, 3)
    L.nextera_free(h)

    # the decoder kernel alone
    typ, table, ne0, ne1 = hu.raw_tensor(path, "embedding.weight")
    d_tab = torch.from_numpy(np.ascontiguousarray(table)).cuda()
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    peak, peak_src = hbm_peak()
    dec = []
    for M in (8, 77, 512):
        x = torch.randn((M, ne0), dtype=torch.float32, device="cuda")
        ws = torch.empty(L.nxk_mul_mat_workspace(typ, ne0, M), dtype=torch.uint8, device="cuda")
        out = torch.empty((M, ne1), dtype=torch.float32, device="cuda")

        def launch(sp):
            assert L.nxk_mul_mat(typ, ctypes.c_void_p(d_tab.data_ptr()), ne1, ne0, ctypes.c_void_p(x.data_ptr()),
                                 M, None, ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                 sp) == 0
        # 20 calls captured in a CUDA graph, so host launch overhead does not enter the time
        gs = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(gs):
            gsp = ctypes.c_void_p(gs.cuda_stream)
            for _ in range(3):
                launch(gsp)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=gs):
                for _ in range(20):
                    launch(gsp)
        for _ in range(3):
            graph.replay()
        n = 10
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(n):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (20 * n)
        byts = table.nbytes + 4.0 * M * ne1 + 4.0 * M * ne0
        dec.append({"rows": M, "us": us, "bytes": byts, "gbs": byts / us * 1e-3, "frac_hbm": byts / us * 1e-3 / peak,
                    "int_macs_per_s": M * ne1 * ne0 / (us * 1e-6)})
        log(f"decoder M={M}: {us:.1f} us, {byts / us * 1e-3:.0f} GB/s")

    # the reference on the host cores, same mlm_logits call
    ref = None
    if not args.no_cpu_baseline:
        from oracle_lib import RefLib, ref_library_path
        if ref_library_path() is not None:
            r = RefLib()
            cores = os.cpu_count() or 1
            rh = r.load(path, cores)
            r.mlm_logits(rh, seq, pos)
            t0 = time.perf_counter()
            r.mlm_logits(rh, seq, pos)
            ref = {"ms": 1e3 * (time.perf_counter() - t0), "cores": cores, "kind": "reference"}
            r.L.nextera_free(rh)

    emit({"metric": HEADS_METRIC, "unit": "documents/s", "value": n_docs / t_cls, "n_gpus": 1,
          "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "int8+fp32",
          "data": "synthetic (seeded lengths and ids; random-init weights N(0,0.02), Q4_K_M, 2-label classifier)",
          "config": {"workload": f"cfg4 batch ({n_docs} docs, {T} tokens) through nextera_classify; "
                                 "fill-mask: 512 tokens, 77 positions through nextera_mlm_logits",
                     "model": "NexteraBERT-synthetic + pooler + classifier + tied MLM head"},
          "classify": {"ms_per_batch": 1e3 * t_cls, "tokens_per_s": T / t_cls,
                       "encode_ms_per_batch": 1e3 * t_enc, "head_overhead": t_cls / t_enc - 1.0,
                       "api": "nextera_classify (host buffers, wall clock)"},
          "mlm_logits": {"ms_per_call": 1e3 * t_mlm, "tokens": 512, "positions": 77,
                         "api": "nextera_mlm_logits (host buffers, wall clock)", "reference": ref},
          "decoder_kernel": {"type": "Q4_K", "table_bytes": int(table.nbytes), "launches": dec,
                             "peak_hbm_gbs": peak, "peak_source": peak_src}})


def main() -> int:
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--preset", default="Q4_K_M")
    ap.add_argument("--docs", type=int, default=4096)
    ap.add_argument("--config", type=int, choices=[1, 2, 4, 5], default=4,
                    help="4: mixed-length batch (the headline); 5: one long sequence, sharded over the GPUs; "
                         "1: one int8 linear; 2: attention alone")
    ap.add_argument("--seq-len", type=int, default=65536, help="config 5 sequence length")
    ap.add_argument("--cpu-prefix", type=int, default=8192,
                    help="config 5: ids of the sequence the reference encodes on the host cores")
    ap.add_argument("--profile-run", action="store_true", help="one untimed step (for profilers)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-weak", action="store_true", help="skip the weak-scaling extra measurement (N > 1)")
    ap.add_argument("--heads", action="store_true", help="time the task heads instead (one GPU)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if args.impl == "reference":
        run_reference(args, rank, world, dist)
        return 0
    if args.heads:
        run_heads(args)
        return 0
    if args.config in (1, 2):
        if rank == 0:
            (run_cfg1 if args.config == 1 else run_cfg2)(args)
        return 0
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local_rank}"))
    try:
        if args.config == 5:
            run_long(args, rank, world, local_rank, dist)
        else:
            run_b200(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
