#!/usr/bin/env python
"""Benchmark of the hot path: embedded tokens/s of the ModernBERT-base varlen encoder on 1..8 B200s.

``python bench.py --gpus N --steps K --warmup W`` (torchrun for N > 1, one rank per GPU).

Workload (default): ModernBERT-base in bf16 (22 layers, hidden 768, 12 heads
x 64, GeGLU 1152, global attention every 3rd layer with RoPE theta 160000, 128-token sliding
window with theta 10000 elsewhere), random-init N(0, 0.02) weights; 4096 chunks per GPU with
lengths uniform in [64, 512] and token ids uniform over the 50368-token vocabulary, packed varlen
with cu_seqlens.  One step = the encoder forward over all 4096 chunks of the rank (mean-pooled,
L2-normalised 768-d outputs).  Chunks shard by data parallelism with no collective (weak scaling:
every rank embeds its own 4096 chunks).

* ``value``: tokens/s with the ids already in HBM (``rv_embed_varlen_device``), CUDA events on
  the launching stream around each step, L2 flushed between steps, max over ranks.
* ``e2e``: the same through ``rv_embed_varlen`` with pinned host buffers (ids H2D and the
  embeddings D2H inside the timed region), host clock around the synchronous call, max over ranks.
* ``roofline``: the tcgen05 projection GEMMs, timed live by the library's own CUDA events on its
  stream over the timed region; algorithmic FLOPs 2*M*N*K per launch.
* ``cpu_baseline``: the numpy port of the reference fp32 CPU path (``oracle/``) on a bounded
  sample of the same chunks, rank 0, N = 1.
* ``parity``: min / p50 cosine of 16 chunks of the timed output against that port.
* ``sweep_tokens_per_s`` (config 4, strong scaling): 100k log-normal chunks sharded over the
  ranks by token count, max over ranks of the device time.
* ``long_tokens_per_s`` (config 3, weak scaling): ModernBERT-base in fp16 over 512 chunks of
  U[2048, 8192] tokens per rank, max over ranks; on one GPU with the longest chunk's cosine
  against the fp32 port.
* ``classic_tokens_per_s`` (config 1, weak scaling): BERT-small ClassicBert over 64 chunks of
  U[32, 256] tokens per rank, with all 64 chunks' cosine against the fp32 port on rank 0.
* ``scan_step_ms`` (config 5): one 1024-query top-100 step over a 10M x 768 bf16 database
  row-sharded over the ranks, through ``rv_index_topk_sharded`` (the library's NCCL all-gather
  of the per-shard lists and device merge).

``--impl reference`` times that CPU port as the reference arm (rank 0 only).  Other workloads:
``--workload long`` (config 3, fp16, 512 chunks of 2048..8192 tokens), ``--workload sweep``
(config 4, 1M log-normal chunks sharded by token count), ``--workload scan`` (config 5, exact
top-100 over a 10M x 768 bf16 database, 1024 queries by default or a list such as
``--queries 1,16,64,128``; with several ranks through ``rv_index_topk_sharded``),
``--workload turboquant`` (``rank_turboquant`` over 4-bit PolarQuant codes of the same database),
``--workload duplicates`` (``find_duplicates`` over 200k x 768 rows: every pair scored),
``--workload cascade`` (``rank_cascade`` over the 10M x 768 database truncated to 256 dimensions),
``--workload classic`` (config 1: BERT-small over 64 chunks, with its cosine against the fp32 oracle).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "embedded tokens/sec (ModernBERT-base varlen)"
UNIT = "tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["encoder", "long", "sweep", "scan", "turboquant", "duplicates",
                                           "cascade", "classic"], default="encoder")
    ap.add_argument("--chunks", type=int, default=None, help="override chunks per GPU")
    ap.add_argument("--max-batch-tokens", type=int, default=1 << 19)
    ap.add_argument("--scan-rows", type=int, default=10_000_000,
                    help="database rows of the scan workload (smaller only for profiling)")
    ap.add_argument("--queries", default="1024",
                    help="queries per step of the scan workload, or a comma-separated list (one JSON line "
                         "each, same database); the roofline is HBM below ~210 queries, tensor above")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the 16-chunk oracle check of the timed output")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config 1, 3, 4 and 5 keys of the encoder line (classic, long, sweep, scan)")
    ap.add_argument("--sweep-chunks", type=int, default=100_000,
                    help="chunks of the strong-scaling sweep key (log-normal lengths, all ranks together)")
    return ap.parse_args()


# ------------------------------------------------------------------ environment / ranks
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sus": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sus": 1400.0, "source": "fallback"}


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local])
        except (ValueError, IndexError):
            return local
    return local


# ------------------------------------------------------------------ workloads
def encoder_workload(args, rank):
    from ripvec_b200 import MODERNBERT_BASE, synth

    if args.workload == "long":
        n = args.chunks or 512
        lengths = synth.uniform_lengths(n, 2048, 8192, seed=2000 + rank)
        name, dtype = "modernbert_base_long_fp16", "f16"
        desc = f"{n} chunks, lengths U[2048,8192]"
    else:
        n = args.chunks or 4096
        lengths = synth.uniform_lengths(n, 64, 512, seed=1000 + rank)
        name, dtype = "modernbert_base_varlen", "bf16"
        desc = f"{n} chunks, lengths U[64,512]"
    ids, cu = synth.packed_ids(lengths, MODERNBERT_BASE.vocab, seed=3000 + rank)
    return MODERNBERT_BASE, name, dtype, desc, lengths, ids, cu


def sweep_shard(rank, world, n_chunks):
    """1M log-normal chunks (median 180, sigma 0.8, clip [16,1024]) sharded by token count."""
    from ripvec_b200 import shard, synth

    lengths = synth.lognormal_lengths(n_chunks, 180.0, 0.8, 16, 1024, seed=4242)
    return lengths, shard.shard_by_tokens(lengths, world)[rank]


# ------------------------------------------------------------------ reference arm (CPU port)
def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def pin_blas_threads() -> int:
    """Gives the BLAS pool every host core this process may run on and returns the count.

    torchrun exports OMP_NUM_THREADS=1, which OpenBLAS reads when it loads, so without this the
    reference arm of a multi-rank launch would run on one core."""
    n = host_cores()
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n, user_api="blas")
    except Exception:
        pass
    return blas_threads()


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return os.cpu_count() or 1


def cpu_encoder_rate(spec, w, lengths, ids, cu, budget_s: float, dtype=np.float32):
    """Tokens/s of the numpy port of the reference fp32 CPU path over a bounded sample (whole
    chunks in workload order until ``budget_s`` of CPU work, at least one chunk)."""
    from oracle import modern_bert

    cfg = modern_bert.ModernBertConfig(
        hidden=spec.hidden, num_layers=spec.num_layers, num_heads=spec.num_heads, intermediate=spec.intermediate,
        vocab=spec.vocab, max_position=spec.max_position, global_every_n=spec.global_every_n,
        local_window=spec.local_window, global_rope_theta=spec.global_rope_theta,
        local_rope_theta=spec.local_rope_theta, norm_eps=spec.norm_eps)
    t0 = time.perf_counter()
    tok = 0
    n = 0
    while n < len(lengths):
        modern_bert.embed_sequence(w, cfg, ids[cu[n]:cu[n + 1]], dtype)
        tok += int(lengths[n])
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return tok / dt, n, tok, dt


def cpu_embed_one(spec, w, ids_one):
    """One chunk's embedding from the numpy fp32 port of the reference CPU path (f64 result)."""
    from oracle import modern_bert

    cfg = modern_bert.ModernBertConfig(
        hidden=spec.hidden, num_layers=spec.num_layers, num_heads=spec.num_heads, intermediate=spec.intermediate,
        vocab=spec.vocab, max_position=spec.max_position, global_every_n=spec.global_every_n,
        local_window=spec.local_window, global_rope_theta=spec.global_rope_theta,
        local_rope_theta=spec.local_rope_theta, norm_eps=spec.norm_eps)
    return modern_bert.embed_sequence(w, cfg, ids_one).astype(np.float64)


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return
    if args.workload == "scan":
        return run_reference_scan(args)
    from ripvec_b200 import synth

    spec, name, dtype, desc, lengths, ids, cu = encoder_workload(args, 0)
    w = synth.random_weights(spec, seed=1)
    cores = pin_blas_threads()
    step_budget = 4.0
    rates, samples = [], []
    for s in range(args.warmup + args.steps):
        # each step: a bounded sample of the workload's chunks, rotating through the workload
        off = (s * 7) % max(1, len(lengths) - 16)
        r, n, tok, dt = cpu_encoder_rate(spec, w, lengths[off:], ids[cu[off]:], cu[off:] - cu[off], step_budget)
        if s >= args.warmup:
            rates.append((tok, dt))
            samples.append(n)
    tok = sum(t for t, _ in rates)
    dt = sum(d for _, d in rates)
    value = tok / dt
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random token ids, random-init N(0,0.02) weights)",
            "config": {"workload": name, "model": "ModernBERT-base", "chunks_per_gpu": len(lengths),
                       "lengths": desc, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{sum(samples)} whole chunks ({tok} tokens) of the workload over {args.steps} steps"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_scan_baseline(n_rows, dim, steps=1, warmup=0):
    """The reference's exact search (``rank``: f32 GEMV + full sort, ``index.rs:172-186``) on the
    host cores over a 200k-row sample, scaled to ``n_rows``: (queries/s, ms per sampled step,
    cpu_baseline dict)."""
    from oracle import scan as oscan
    from ripvec_b200 import synth

    cores = pin_blas_threads()
    sample = 200_000
    db = synth.normalized_gaussian(sample, dim, seed=77)
    q = synth.normalized_gaussian(8, dim, seed=78)
    times = []
    for s in range(warmup + steps):
        t0 = time.perf_counter()
        for qi in range(q.shape[0]):
            oscan.rank(db, q[qi], -1.0)
        if s >= warmup:
            times.append(time.perf_counter() - t0)
    qps = 1.0 / (sum(times) / (steps * q.shape[0] * sample) * n_rows)
    return qps, 1e3 * sum(times) / steps, {
        "value": qps, "unit": "queries/s", "cores": cores, "kind": "port",
        "sample": f"{q.shape[0]} queries x {sample} rows per step (f32 GEMV + full sort), scaled to {n_rows} rows"}


def cpu_turboquant_baseline(n_rows, dim, top_k):
    """``rank_turboquant`` (``index.rs:196-234``: LUT scan of the codes, top 10·top_k, exact
    re-rank) by the oracle port on a 20k-row sample with its codes built beforehand (index build,
    untimed), the per-query time scaled by rows."""
    from oracle import turbo_quant as otq
    from ripvec_b200 import synth

    cores = pin_blas_threads()
    sample = 20_000
    rows = synth.normalized_gaussian(sample, dim, seed=81)
    rot = otq.generate_rotation(dim, 42)
    codes = otq.encode(rows, rot)
    q = synth.normalized_gaussian(4, dim, seed=82)
    t0 = time.perf_counter()
    for qi in range(q.shape[0]):
        otq.rank_turboquant(rows, q[qi], top_k, float("-inf"), rot, codes=codes)
    per_q = (time.perf_counter() - t0) / q.shape[0] * (n_rows / sample)
    return {"value": 1.0 / per_q, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{q.shape[0]} queries x {sample} rows (codes built untimed), scaled to {n_rows} rows"}


def cpu_cascade_baseline(n_rows, dim, t_dim, top_k):
    """``rank_cascade``'s query work (``index.rs:245-297``) in the reference's f32 arithmetic on a
    100k-row sample whose truncated matrix is built beforehand (untimed), scaled by rows."""
    from oracle import scan as oscan
    from ripvec_b200 import synth

    cores = pin_blas_threads()
    sample = 100_000
    rows = synth.normalized_gaussian(sample, dim, seed=83)
    tr = oscan.ln_truncate(rows, t_dim)
    q = synth.normalized_gaussian(8, dim, seed=84)
    t0 = time.perf_counter()
    for qi in range(q.shape[0]):
        oscan.rank_cascade_f32(rows, tr, q[qi], top_k, float("-inf"), t_dim)
    per_q = (time.perf_counter() - t0) / q.shape[0] * (n_rows / sample)
    return {"value": 1.0 / per_q, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{q.shape[0]} queries x {sample} rows (truncated matrix built untimed), scaled to {n_rows} rows"}


def cpu_duplicates_baseline(dim):
    """``find_duplicates`` in the reference's arithmetic (f32 BLAS similarity matrix, upper
    triangle, threshold, sort) over a 16k-row sample: pair scores per second."""
    from oracle import scan as oscan
    from ripvec_b200 import synth

    cores = pin_blas_threads()
    sample = 16_384
    rows = synth.normalized_gaussian(sample, dim, seed=85)
    t0 = time.perf_counter()
    oscan.find_duplicates_f32(rows, 0.85, 20)
    pps = sample * (sample - 1) / 2 / (time.perf_counter() - t0)
    return {"value": pps, "unit": "pairs/s", "cores": cores, "kind": "port",
            "sample": f"{sample} rows ({sample * (sample - 1) // 2} pairs), f32 BLAS upper triangle"}


def run_reference_scan(args):
    n_rows, dim, nq = 10_000_000, 768, 1024
    qps, ms, base = cpu_scan_baseline(n_rows, dim, args.steps, args.warmup)
    line = {"metric": "exact cosine top-100 queries/sec (10M x 768 bf16)", "value": qps, "unit": "queries/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic normalised Gaussian rows",
            "config": {"workload": "scan_topk", "rows": n_rows, "dim": dim, "queries": nq},
            "cpu_baseline": base,
            "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def traffic_per_flop():
    """DRAM bytes per algorithmic GEMM FLOP from the committed ncu summary, or None."""
    p = ROOT / "profiles" / "gemm_tc_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d["dram_bytes"] / d["flops"]


def make_shard_comm(dist, rank, world, local):
    """The library's NCCL communicator for the sharded search: rank 0's unique id reaches every
    rank through the harness's process group (the caller's own channel, as the C ABI expects)."""
    import torch

    from ripvec_b200 import _lib as L
    from ripvec_b200.index import ShardComm

    if dist is None:
        uid = ShardComm.new_unique_id()
    else:
        t = torch.zeros(L.RV_COMM_ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            t.copy_(torch.frombuffer(bytearray(ShardComm.new_unique_id()), dtype=torch.uint8))
        dist.broadcast(t, 0)
        uid = bytes(t.cpu().numpy().tobytes())
    return ShardComm(uid, rank, world, device=local, timeout_ms=120000)


def device_database_shard(torch, lo, hi, dim, seed):
    """Rows [lo, hi) of the synthetic database: Gaussian, L2-normalised, bf16, made on the device
    in blocks (seeded per rank)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    shard = torch.empty(hi - lo, dim, device="cuda", dtype=torch.bfloat16)
    for s in range(0, hi - lo, 1 << 20):
        e = min(hi - lo, s + (1 << 20))
        x = torch.randn(e - s, dim, device="cuda", generator=gen)
        shard[s:e] = (x / x.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    return shard


def sweep_extra(args, torch, be, spec, barrier, max_over_ranks, rank, world, stream):
    """Config 4 as a strong-scaling key: a fixed set of log-normal chunks (median 180, sigma 0.8,
    clip [16, 1024]) sharded over the ranks by token count; each rank embeds its shard with ids
    in HBM; time = max over ranks of the CUDA-event time of the whole shard."""
    from ripvec_b200 import synth

    n_total = args.sweep_chunks
    all_len, mine = sweep_shard(rank, world, n_total)
    lengths = all_len[mine]
    ids, cu = synth.packed_ids(lengths, spec.vocab, seed=5000 + rank)
    ids_dev = torch.from_numpy(ids).cuda()
    out = torch.empty(len(lengths), spec.hidden, device="cuda", dtype=torch.float32)
    w = min(len(lengths), 2000)
    be.embed_device(ids_dev, cu[:w + 1], out, stream=stream.cuda_stream)  # warm-up on a prefix
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    be.embed_device(ids_dev, cu, out, stream=stream.cuda_stream)
    b.record(stream)
    barrier()
    ms = max_over_ranks(a.elapsed_time(b))
    total_tokens = int(all_len.sum())
    return {"tokens_per_s": total_tokens / (ms / 1e3), "ms": ms, "chunks": n_total, "tokens": total_tokens,
            "scaling": "strong", "sharding": "shard_by_tokens (longest first to the rank with the fewest tokens)",
            "lengths": "log-normal median 180 sigma 0.8 clip [16,1024]",
            "rank0_chunks": int(len(lengths)), "rank0_tokens": int(cu[-1])}


def timed_device_passes(torch, be, ids_dev, cu, out, stream, steps, flush):
    """Device time (ms) of ``steps`` encoder passes over one packed set with the ids in HBM, CUDA
    events on the launching stream, L2 flushed before each pass (outside the events)."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s in range(steps):
        flush.zero_()
        evs[s][0].record(stream)
        be.embed_device(ids_dev, cu, out, stream=stream.cuda_stream)
        evs[s][1].record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs)


def long_extra(args, torch, local, barrier, max_over_ranks, rank, world, stream, flush):
    """Config 3 as a key of the encoder line: ModernBERT-base in fp16 over 512 chunks of U[2048, 8192]
    tokens per rank (weak scaling, the ``--workload long`` set), one warm-up pass and two timed
    passes with the ids in HBM, max over ranks.  On one GPU the longest chunk of the set (RoPE
    positions up to about 8192) is checked against the fp32 oracle at the fp16 bar; that check
    costs about a minute of host time, so the multi-GPU runs leave it to the tests."""
    from ripvec_b200 import MODERNBERT_BASE, EmbedBackend, synth

    n = 512
    lengths = synth.uniform_lengths(n, 2048, 8192, seed=2000 + rank)
    ids, cu = synth.packed_ids(lengths, MODERNBERT_BASE.vocab, seed=3000 + rank)
    w = synth.random_weights(MODERNBERT_BASE, seed=1)
    be = EmbedBackend(MODERNBERT_BASE, w, dtype="f16", device=local, max_batch_tokens=args.max_batch_tokens)
    ids_dev = torch.from_numpy(ids).cuda()
    out = torch.empty(n, MODERNBERT_BASE.hidden, device="cuda", dtype=torch.float32)
    be.embed_device(ids_dev, cu, out, stream=stream.cuda_stream)
    barrier()
    steps = 2
    ms = max_over_ranks(timed_device_passes(torch, be, ids_dev, cu, out, stream, steps, flush) / steps)
    barrier()
    res = {"tokens_per_s": int(cu[-1]) * world / (ms / 1e3), "ms_per_step": ms, "chunks_per_gpu": n,
           "tokens_per_gpu": int(cu[-1]), "lengths": "U[2048,8192]", "dtype": "f16", "steps": steps, "warmup": 1,
           "scaling": "weak", "l2": "flushed between passes"}
    if rank == 0 and world == 1 and not args.no_parity:
        b = int(np.argmax(lengths))
        pin_blas_threads()
        ref = cpu_embed_one(MODERNBERT_BASE, w, ids[cu[b]:cu[b + 1]])
        g = out[b].double().cpu().numpy()
        cos = float(g @ ref / max(np.linalg.norm(g) * np.linalg.norm(ref), 1e-300))
        res["parity"] = {"min_cos": cos, "bar": 0.9999, "chunks": 1, "sample_lengths": [int(lengths[b])],
                         "against": "numpy fp32 port of the reference CPU path, the longest chunk of the set"}
        if cos < 0.9999:
            raise RuntimeError(f"config-3 parity below the fp16 bar: {res['parity']}")
    be.close()
    return res


def classic_extra(args, torch, local, barrier, max_over_ranks, rank, world, stream, flush):
    """Config 1 as a key of the encoder line: BERT-small ClassicBert (f16 storage, mean pooling)
    over the 64 chunks of U[32, 256] tokens on every rank (weak scaling), five timed passes with
    the ids in HBM, max over ranks; rank 0 checks all 64 chunks against the fp32 oracle (bar
    0.9999)."""
    from ripvec_b200 import EmbedBackend

    spec, w, lengths, ids, cu = classic_workload()
    n = len(lengths)
    be = EmbedBackend(spec, w, dtype="f16", device=local, pooling="mean")
    ids_dev = torch.from_numpy(ids).cuda()
    out = torch.empty(n, spec.hidden, device="cuda", dtype=torch.float32)
    for _ in range(3):
        be.embed_device(ids_dev, cu, out, stream=stream.cuda_stream)
    barrier()
    steps = 5
    ms = max_over_ranks(timed_device_passes(torch, be, ids_dev, cu, out, stream, steps, flush) / steps)
    barrier()
    res = {"tokens_per_s": int(cu[-1]) * world / (ms / 1e3), "ms_per_step": ms, "chunks_per_gpu": n,
           "tokens_per_gpu": int(cu[-1]), "lengths": "U[32,256]", "dtype": "f16", "pooling": "mean",
           "steps": steps, "warmup": 3, "scaling": "weak", "l2": "flushed between passes"}
    if rank == 0 and not args.no_parity:
        pin_blas_threads()
        ref, _ = classic_oracle(spec, w, ids, cu)
        a = out.double().cpu().numpy()
        b = ref.astype(np.float64)
        cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
        res["parity"] = {"min_cos": float(cos.min()), "p50_cos": float(np.median(cos)), "bar": 0.9999, "chunks": n,
                         "against": "numpy fp32 port of the reference CPU path, all 64 chunks"}
        if cos.min() < 0.9999:
            raise RuntimeError(f"config-1 parity below the bar: {res['parity']}")
    be.close()
    return res


def scan_extra(args, torch, dist, rank, world, local, barrier, max_over_ranks, stream):
    """Config 5 as a key of the encoder line: one 1024-query top-100 step over a 10M x 768 bf16
    database row-sharded across the ranks, through rv_index_topk_sharded (shard top-k, one NCCL
    all-gather inside the library, device merge).  Time = max over ranks of CUDA events."""
    from ripvec_b200 import shard as shard_mod
    from ripvec_b200 import synth
    from ripvec_b200.index import SearchIndex, topk_sharded

    n_rows, dim, nq, k = args.scan_rows, 768, 1024, 100
    lo, hi = shard_mod.row_ranges(n_rows, world)[rank]
    db = device_database_shard(torch, lo, hi, dim, 100 + rank)
    idx = SearchIndex(db, device=local, base=lo)
    del db
    comm = make_shard_comm(dist, rank, world, local)
    q = torch.from_numpy(synth.normalized_gaussian(nq, dim, seed=99)).cuda()
    oi = torch.empty(nq, k, dtype=torch.int64, device="cuda")
    os_ = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    o64 = torch.empty(nq, k, dtype=torch.float64, device="cuda")
    steps = 5
    for _ in range(3):
        topk_sharded(idx, comm, q, k, oi, os_, o64, stream=stream.cuda_stream)
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s in range(steps):
        evs[s][0].record(stream)
        topk_sharded(idx, comm, q, k, oi, os_, o64, stream=stream.cuda_stream)
        evs[s][1].record(stream)
    barrier()
    ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / steps)
    comm.close()
    idx.close()
    return {"step_ms": ms, "queries_per_s": nq / (ms / 1e3), "rows": n_rows, "dim": dim, "queries": nq, "k": k,
            "rows_per_rank": hi - lo, "entry_point": "rv_index_topk_sharded (NCCL all-gather + device merge)",
            "steps": steps, "warmup": 3}


def run_encoder(args):
    import torch

    from ripvec_b200 import EmbedBackend, synth
    from ripvec_b200 import _lib as L

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    if args.workload == "sweep":
        from ripvec_b200 import MODERNBERT_BASE

        n_total = args.chunks or 1_000_000
        all_len, mine = sweep_shard(rank, world, n_total)
        lengths = all_len[mine]
        ids, cu = synth.packed_ids(lengths, MODERNBERT_BASE.vocab, seed=5000 + rank)
        spec, name, dtype = MODERNBERT_BASE, "modernbert_base_index_sweep", "bf16"
        desc = f"{n_total} chunks total, log-normal median 180 sigma 0.8 clip [16,1024], sharded by token count"
    else:
        spec, name, dtype, desc, lengths, ids, cu = encoder_workload(args, rank)
    tokens = int(cu[-1])
    n = len(lengths)
    w = synth.random_weights(spec, seed=1)
    be = EmbedBackend(spec, w, dtype=dtype, device=local, max_batch_tokens=args.max_batch_tokens)
    del w

    stream = torch.cuda.current_stream()
    ids_dev = torch.from_numpy(ids).cuda()
    out_dev = torch.empty(n, spec.hidden, device="cuda", dtype=torch.float32)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > 126 MB L2

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        be.embed_device(ids_dev, cu, out_dev, stream=stream.cuda_stream)
    barrier()

    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    be._lib.rv_reset_profile(be._h)
    be._lib.rv_set_profiling(be._h, 1)
    launches0 = be.kernel_launches()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    for s in range(args.steps):
        flush.zero_()  # L2 flush between timed steps (outside the events)
        evs[s][0].record(stream)
        be.embed_device(ids_dev, cu, out_dev, stream=stream.cuda_stream)
        evs[s][1].record(stream)
    barrier()
    launches = be.kernel_launches() - launches0
    be._lib.rv_set_profiling(be._h, 0)
    clocks = sampler.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = max_over_ranks(sum(step_ms))
    value = (tokens * args.steps * world) / (total_ms / 1e3)

    prof = {}
    import ctypes as C

    for k, kname in enumerate(L.KIND_NAMES):
        ms, cnt, fl = C.c_double(), C.c_int64(), C.c_double()
        be._lib.rv_get_profile(be._h, k, C.byref(ms), C.byref(cnt), C.byref(fl))
        prof[kname] = {"ms": ms.value, "launches": cnt.value, "flops": fl.value}
    kern_total = sum(v["ms"] for v in prof.values()) or 1.0
    pk = peaks()
    g = prof["gemm_tc"]
    gemm_ms_per_launch = g["ms"] / max(1, g["launches"])
    gemm_flops_per_launch = g["flops"] / max(1, g["launches"])
    achieved = gemm_flops_per_launch / (gemm_ms_per_launch / 1e3) / 1e12 if g["launches"] else 0.0
    tpf = traffic_per_flop()
    roofline = {"kernel": "gemm_tc (tcgen05 projection GEMMs, all four per layer)", "bound": "tensor",
                "achieved": achieved, "peak": pk["bf16_sus"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_sus"],
                "peak_source": f"{pk['source']} bf16_tflops_sustained (kernel timed inside a long step)",
                "traffic": (tpf * gemm_flops_per_launch) if tpf else None,
                "flops_per_launch": gemm_flops_per_launch, "ms_per_launch": gemm_ms_per_launch}
    att = prof["attention_varlen"]
    whole_flops = sum(v["flops"] for v in prof.values()) / args.steps
    kernels = {k: {"ms_per_step": v["ms"] / args.steps, "share": v["ms"] / kern_total,
                   "launches_per_step": v["launches"] / args.steps} for k, v in prof.items()}

    # ---------------------------------------------------------------- e2e through the host API
    e2e = None
    if not args.no_e2e:
        ids_h = torch.from_numpy(ids).pin_memory()
        cu_h = np.ascontiguousarray(cu, np.int32)
        out_h = torch.empty(n, spec.hidden, dtype=torch.float32).pin_memory()
        ids_np = ids_h.numpy()
        out_np = out_h.numpy()
        for _ in range(max(1, min(args.warmup, 2))):
            be.embed_packed(ids_np, cu_h, out_np)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            be.embed_packed(ids_np, cu_h, out_np)
        torch.cuda.synchronize()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        nb = -(-tokens // args.max_batch_tokens) + 1
        h2d = tokens * 4 + 8 * (n + nb)
        e2e = {"value": tokens * args.steps * world / e2e_s, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(n * spec.hidden * 4),
               "how": "rv_embed_varlen with pinned host ids / cu_seqlens / output, host clock around the synchronous call"}
        if np.abs(np.linalg.norm(out_np, axis=1) - 1).max() > 1e-3:
            raise RuntimeError("e2e outputs are not unit-norm")

    cpu = None
    parity = None
    if rank == 0 and not args.no_parity:
        # Parity of the timed workload itself: the device-resident path's output of the last timed
        # step against the numpy fp32 port of the reference CPU path, on 16 chunks (4 of the long
        # workload) spread evenly over the rank's chunks, after the timed region.
        w = synth.random_weights(spec, seed=1)
        pin_blas_threads()
        out_last = out_dev.cpu().numpy()
        n_pick = 4 if args.workload == "long" else 16  # long chunks cost ~10 s each in the oracle
        pick = np.unique(np.linspace(0, n - 1, min(n_pick, n)).astype(np.int64))
        cos = []
        for b in pick:
            ref = cpu_embed_one(spec, w, ids[cu[b]:cu[b + 1]])
            g = out_last[b].astype(np.float64)
            cos.append(float(g @ ref / max(np.linalg.norm(g) * np.linalg.norm(ref), 1e-300)))
        bar = 0.999 if dtype == "bf16" else 0.9999
        parity = {"min_cos": min(cos), "p50_cos": float(np.median(cos)), "bar": bar, "chunks": len(pick),
                  "sample_lengths": [int(lengths[b]) for b in pick],
                  "against": "numpy fp32 port of the reference CPU path (oracle/modern_bert.py), device-resident "
                             "output of the last timed step"}
        if min(cos) < bar:
            raise RuntimeError(f"parity below the bar on the timed workload: {parity}")
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ("encoder", "long"):
        w = synth.random_weights(spec, seed=1)
        cores = pin_blas_threads()
        r, nc, tok, dt = cpu_encoder_rate(spec, w, lengths, ids, cu, 12.0)
        cpu = {"value": r, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"first {nc} chunks of the workload ({tok} tokens, {dt:.1f} s), numpy fp32 port of the reference CPU path"}

    sweep = scan = long_ = classic = None
    if args.workload == "encoder" and not args.no_extras:
        sweep = sweep_extra(args, torch, be, spec, barrier, max_over_ranks, rank, world, stream)
        be.close()
        del ids_dev, out_dev
        long_ = long_extra(args, torch, local, barrier, max_over_ranks, rank, world, stream, flush)
        classic = classic_extra(args, torch, local, barrier, max_over_ranks, rank, world, stream, flush)
        scan = scan_extra(args, torch, dist, rank, world, local, barrier, max_over_ranks, stream)

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
                "scaling": "weak" if args.workload != "sweep" else "strong", "vs_baseline": None, "dtype": dtype,
                "data": "synthetic (seeded random token ids, random-init N(0,0.02) weights)",
                "config": {"workload": name, "model": "ModernBERT-base (22L, H768, 12x64, GeGLU 1152, window 128)",
                           "chunks_per_gpu": n, "lengths": desc, "tokens_per_gpu": tokens,
                           "global_batch": n * world, "seq_len": "varlen", "parallelism": f"dp{world}",
                           "max_batch_tokens": args.max_batch_tokens, "l2": "flushed between steps (256 MiB write)"},
                "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline, "cpu_baseline": cpu,
                "parity": parity, "clocks": clocks, "kernels": kernels,
                "whole_step_tflops": whole_flops / (total_ms / args.steps / 1e3) / 1e12,
                "attention_tflops": (att["flops"] / (att["ms"] / 1e3) / 1e12) if att["ms"] else None}
        if sweep is not None:
            line["sweep_tokens_per_s"] = sweep["tokens_per_s"]
            line["sweep"] = sweep
        if long_ is not None:
            line["long_tokens_per_s"] = long_["tokens_per_s"]
            line["long"] = long_
        if classic is not None:
            line["classic_tokens_per_s"] = classic["tokens_per_s"]
            line["classic"] = classic
        if scan is not None:
            line["scan_step_ms"] = scan["step_ms"]
            line["scan"] = scan
        print(json.dumps(line), flush=True)
    be.close()
    if dist is not None:
        dist.destroy_process_group()


def run_scan(args):
    import torch

    from ripvec_b200 import synth
    from ripvec_b200.index import SearchIndex

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    n_rows, dim, k = args.scan_rows, 768, 100
    from ripvec_b200 import shard as shard_mod

    lo, hi = shard_mod.row_ranges(n_rows, world)[rank]
    # shard rows generated on the device in blocks (normalised Gaussian, rounded to bf16 by the index)
    shard = device_database_shard(torch, lo, hi, dim, 100 + rank)
    idx = SearchIndex(shard, device=local, base=lo)
    del shard
    comm = make_shard_comm(dist, rank, world, local) if world > 1 else None
    stream = torch.cuda.current_stream()
    # The database shard (15.4 GB at 10M rows on one GPU) is larger than L2, so every step
    # streams it from HBM: no flush is needed between steps.
    lines = [scan_line(args, torch, dist, idx, comm, synth, stream, rank, world, local, n_rows, dim, nq, k)
             for nq in [int(v) for v in str(args.queries).split(",")]]
    # The CPU sample runs after every GPU measurement, so it cannot disturb one.  One query at a
    # time on the CPU: the same baseline for every batch size.
    if rank == 0:
        cpu_base = None if world > 1 or args.no_cpu_baseline else cpu_scan_baseline(n_rows, dim)[2]
        for line in lines:
            if cpu_base is not None:
                line["cpu_baseline"] = cpu_base
            print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    idx.close()
    if dist is not None:
        dist.destroy_process_group()


def scan_line(args, torch, dist, idx, comm, synth, stream, rank, world, local, n_rows, dim, nq, k):
    """Times ``args.steps`` exact top-k steps of ``nq`` queries and returns the JSON line (rank 0;
    None on the other ranks).
    With several ranks a step is ``rv_index_topk_sharded``: the shard's top-k, the library's
    NCCL all-gather of the lists and the device merge."""
    from ripvec_b200.index import topk_sharded

    q = torch.from_numpy(synth.normalized_gaussian(nq, dim, seed=99)).cuda()
    oi = torch.empty(nq, k, dtype=torch.int64, device="cuda")
    os_ = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    o64 = torch.empty(nq, k, dtype=torch.float64, device="cuda")

    def step():
        if comm is None:
            idx.topk_device(q, k, oi, os_, o64, stream=stream.cuda_stream)
        else:
            topk_sharded(idx, comm, q, k, oi, os_, o64, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(physical_gpu(local))
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    launches0 = idx.kernel_launches()
    for s in range(args.steps):
        evs[s][0].record(stream)
        step()
        evs[s][1].record(stream)
    torch.cuda.synchronize()
    launches = idx.kernel_launches() - launches0
    clocks = sampler.stop() if rank == 0 else None
    ms = sum(a.elapsed_time(b) for a, b in evs)
    # End to end with host buffers: host queries in, host results out, host clock per step.  One
    # GPU: the public host-buffer call (rv_index_topk).  Several: pinned copies around the
    # sharded call, every rank timing its own steps (max over ranks below).
    qh = synth.normalized_gaussian(nq, dim, seed=99)
    e2e_t = []
    if comm is None:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            idx.topk(qh, k, with_f64=True)
            e2e_t.append(time.perf_counter() - t0)
        d2h = nq * k * (8 + 4 + 8) + nq * 4
    else:
        qp = torch.from_numpy(qh).pin_memory()
        oi_h = torch.empty(nq, k, dtype=torch.int64).pin_memory()
        o64_h = torch.empty(nq, k, dtype=torch.float64).pin_memory()
        dist.barrier()
        for _ in range(args.steps):
            t0 = time.perf_counter()
            q.copy_(qp, non_blocking=True)
            step()
            oi_h.copy_(oi, non_blocking=True)
            o64_h.copy_(o64, non_blocking=True)
            stream.synchronize()
            e2e_t.append(time.perf_counter() - t0)
        d2h = nq * k * (8 + 8)
    e2e_ms = 1e3 * sum(e2e_t) / len(e2e_t)
    if dist is not None:
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0].item()), float(t[1].item())
    if rank != 0:
        return None
    pk = peaks()
    db_bytes = (n_rows // world) * dim * 2
    line = {"metric": "exact cosine top-100 queries/sec (10M x 768 bf16)", "value": nq * args.steps / (ms / 1e3),
            "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic normalised Gaussian rows",
            "config": {"workload": "scan_topk", "rows": n_rows, "dim": dim, "queries": nq, "k": k,
                       "parallelism": f"rows{world}", "l2": "database shard larger than L2, no flush"},
            "db_gbs_per_rank": db_bytes / (ms / args.steps / 1e3) / 1e9, "hbm_peak_gbs": pk["hbm_gbs"],
            "clocks": clocks, "gpu_launches": launches,
            "e2e": {"value": nq / (e2e_ms / 1e3), "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                    "d2h_bytes_per_step": d2h,
                    "how": "rv_index_topk with host queries and results" if comm is None else
                           "pinned host copies around rv_index_topk_sharded, host clock, max over ranks"}}
    # Every database byte feeds nq / 2 multiply-adds.  Above the ridge point (peak FLOP/s over
    # HBM bytes/s, about 213 FLOP per byte here, i.e. ~210 queries) the scan is bound by the
    # tensor cores (2 * nq * rows * dim FLOP per step per rank); below it by streaming the
    # database shard from HBM once per step (rows * dim * 2 bytes).
    flops = 2.0 * nq * (n_rows // world) * dim
    sec = ms / args.steps / 1e3
    kern = "scan step (fused tcgen05 filter GEMM + merges + exact rescoring)"
    if flops / db_bytes > pk["bf16_sus"] * 1e12 / (pk["hbm_gbs"] * 1e9):
        ach = flops / sec / 1e12
        line["roofline"] = {"kernel": kern, "bound": "tensor", "achieved": ach, "peak": pk["bf16_sus"],
                            "unit": "TFLOP/s", "frac": ach / pk["bf16_sus"],
                            "peak_source": f"{pk['source']} bf16_tflops_sustained",
                            "traffic": None, "flops_per_step": flops}
    else:
        ach = db_bytes / sec / 1e9
        line["roofline"] = {"kernel": kern, "bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"],
                            "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                            "peak_source": f"{pk['source']} hbm_gbs", "traffic": None,
                            "bytes_per_step": db_bytes}
    return line


def run_turboquant(args):
    """rank_turboquant over PolarQuant codes of a 10M x 768 database (1 GPU): one step = one
    call for the query batch, top_k 100 (1000 rows re-scored exactly per query)."""
    import torch

    from ripvec_b200 import synth
    from ripvec_b200.index import SearchIndex, polar_rotation

    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    n_rows, dim, top_k = args.scan_rows, 768, 100
    gen = torch.Generator(device="cuda").manual_seed(100)
    db = torch.empty(n_rows, dim, device="cuda", dtype=torch.bfloat16)
    for s in range(0, n_rows, 1 << 20):
        e = min(n_rows, s + (1 << 20))
        x = torch.randn(e - s, dim, device="cuda", generator=gen)
        db[s:e] = (x / x.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    idx = SearchIndex(db, device=local)
    del db
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    idx.build_turboquant(polar_rotation(dim, 42))
    build_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream()
    pk = peaks()
    lines = []
    for nq in [int(v) for v in str(args.queries).split(",")]:
        qh = synth.normalized_gaussian(nq, dim, seed=99)
        q = torch.from_numpy(qh).cuda()
        oi = torch.empty(nq, top_k, dtype=torch.int64, device="cuda")
        os_ = torch.empty(nq, top_k, dtype=torch.float32, device="cuda")

        def step():
            idx.topk_turboquant_device(q, top_k, oi, os_, stream=stream.cuda_stream)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        sampler = ClockSampler(physical_gpu(local))
        sampler.start()
        time.sleep(0.3)
        launches0 = idx.kernel_launches()
        for st in range(args.steps):
            evs[st][0].record(stream)
            step()
            evs[st][1].record(stream)
        torch.cuda.synchronize()
        launches = idx.kernel_launches() - launches0
        clocks = sampler.stop()
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        # end to end: the host-buffer call (rv_index_rank_turboquant), host clock
        e2e_t = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            idx.topk_turboquant(qh, top_k)
            e2e_t.append(time.perf_counter() - t0)
        e2e_s = sum(e2e_t) / len(e2e_t)
        # passes over the codes: the scan shares each code word among up to 8 queries (then 4, 2, 1
        # for the rest), as scan_qb in turbo_quant.cu
        passes, left = 0, nq
        while left > 0:
            qb = 8
            while qb > left:
                qb //= 2
            left -= qb
            passes += 1
        code_bytes = passes * n_rows * (dim // 2) * 5
        ach = code_bytes / (ms / 1e3) / 1e9
        line = {"metric": "rank_turboquant queries/sec (PolarQuant 4-bit, 10M x 768)", "value": nq / (ms / 1e3),
                "unit": "queries/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic normalised Gaussian rows",
                "config": {"workload": "rank_turboquant", "rows": n_rows, "dim": dim, "queries": nq, "top_k": top_k,
                           "bits": 4, "l2": "codes (19.2 GB) larger than L2, no flush"},
                "build_s": build_s, "clocks": clocks, "gpu_launches": launches,
                "e2e": {"value": nq / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                        "d2h_bytes_per_step": nq * top_k * 12 + nq * 4,
                        "how": "rv_index_rank_turboquant with host queries and results, host clock"},
                "roofline": {"kernel": "rank_turboquant step (code scan + selection + exact rescoring)",
                             "bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": ach / pk["hbm_gbs"], "peak_source": f"{pk['source']} hbm_gbs",
                             "traffic": None, "bytes_per_step": code_bytes}}
        lines.append(line)
    # the CPU sample after every GPU measurement
    cpu_base = None if args.no_cpu_baseline else cpu_turboquant_baseline(n_rows, dim, top_k)
    for line in lines:
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), flush=True)
    idx.close()


def run_duplicates(args):
    """find_duplicates over a 200k x 768 database (1 GPU; ``--scan-rows`` to change n): one step
    = one call at the reference's default threshold 0.85 and 20 pairs, with 64 planted near-copies.
    Algorithmic work: the n (n - 1) / 2 pair scores, 2 * dim FLOP each."""
    import torch

    from ripvec_b200.index import SearchIndex

    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    n = args.scan_rows if args.scan_rows != 10_000_000 else 200_000
    dim = 768
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(n, dim, device="cuda", generator=gen)
    x[n // 2:n // 2 + 64] = x[:64] + 0.05 * torch.randn(64, dim, device="cuda", generator=gen)
    db = (x / x.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    del x
    idx = SearchIndex(db, device=local)
    del db
    for _ in range(args.warmup):
        idx.duplicate_pairs(0.85, 20)
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    times = []
    launches0 = idx.kernel_launches()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        a, b, s, s64 = idx.duplicate_pairs(0.85, 20)  # synchronous: host results at return
        times.append(time.perf_counter() - t0)
    launches = idx.kernel_launches() - launches0
    clocks = sampler.stop()
    sec = sum(times) / len(times)
    flops = float(n) * (n - 1) / 2 * 2 * dim
    pk = peaks()
    ach = flops / sec / 1e12
    line = {"metric": "find_duplicates pair scores/sec (200k x 768 bf16)", "value": n * (n - 1) / 2 / sec,
            "unit": "pairs/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sec,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic normalised Gaussian rows with 64 planted near-copies",
            "config": {"workload": "find_duplicates", "rows": n, "dim": dim, "threshold": 0.85, "max_pairs": 20,
                       "timing": "host clock around the synchronous call (results on the host)"},
            "pairs_found": int(len(a)), "clocks": clocks, "gpu_launches": launches,
            "e2e": {"value": n * (n - 1) / 2 / sec, "unit": "pairs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": int(len(a)) * 28,
                    "how": "the timed call itself: rv_index_find_duplicates returns host arrays"},
            "roofline": {"kernel": "find_duplicates (tcgen05 strip GEMMs + pair filter + exact rescoring)",
                         "bound": "tensor", "achieved": ach, "peak": pk["bf16_sus"], "unit": "TFLOP/s",
                         "frac": ach / pk["bf16_sus"], "peak_source": f"{pk['source']} bf16_tflops_sustained",
                         "traffic": None, "flops_per_step": flops}}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_duplicates_baseline(dim)
    print(json.dumps(line), flush=True)
    idx.close()


def classic_workload():
    """BERT-small (12 layers, hidden 384, 12 heads, FFN 1536, learned positions,
    post-LN), random-init N(0, 0.02) weights, 64 chunks of U[32, 256] tokens, mean pooling."""
    from ripvec_b200 import BERT_SMALL, synth

    lengths = synth.uniform_lengths(64, 32, 256, seed=1100)
    ids, cu = synth.packed_ids(lengths, BERT_SMALL.vocab, seed=1200)
    return BERT_SMALL, synth.random_weights(BERT_SMALL, seed=1), lengths, ids, cu


def classic_oracle(spec, w, ids, cu):
    """The numpy port of the reference's fp32 ClassicBert CPU path over every chunk, timed."""
    from oracle import classic_bert

    cfg = classic_bert.ClassicBertConfig(hidden=spec.hidden, num_layers=spec.num_layers, num_heads=spec.num_heads,
                                         intermediate=spec.intermediate, vocab=spec.vocab,
                                         max_position=spec.max_position, type_vocab=spec.type_vocab,
                                         norm_eps=spec.norm_eps)
    t0 = time.perf_counter()
    ref = classic_bert.embed_batch(w, cfg, ids, cu, "mean")
    return ref, time.perf_counter() - t0


def run_classic(args):
    """BASELINE config 1 on the GPU (f16 storage, f32 accumulation) next to the reference's fp32
    CPU path: tokens/s device-resident and through rv_embed_varlen, and the per-chunk cosine of
    the GPU embeddings against the fp32 oracle (bar 0.9999 for this fp32 configuration)."""
    import torch

    from ripvec_b200 import EmbedBackend

    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    spec, w, lengths, ids, cu = classic_workload()
    tokens, n = int(cu[-1]), len(lengths)
    be = EmbedBackend(spec, w, dtype="f16", device=local, pooling="mean")
    stream = torch.cuda.current_stream()
    ids_dev = torch.from_numpy(ids).cuda()
    out_dev = torch.empty(n, spec.hidden, device="cuda", dtype=torch.float32)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > 126 MB L2
    for _ in range(args.warmup):
        be.embed_device(ids_dev, cu, out_dev, stream=stream.cuda_stream)
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    launches0 = be.kernel_launches()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for st in range(args.steps):
        flush.zero_()
        evs[st][0].record(stream)
        be.embed_device(ids_dev, cu, out_dev, stream=stream.cuda_stream)
        evs[st][1].record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = be.kernel_launches() - launches0
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    out_h = np.empty((n, spec.hidden), np.float32)
    cu_h = np.ascontiguousarray(cu, np.int32)
    be.embed_packed(ids, cu_h, out_h)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        be.embed_packed(ids, cu_h, out_h)
    e2e_s = (time.perf_counter() - t0) / args.steps
    be.close()
    ref, cpu_s = classic_oracle(spec, w, ids, cu)
    a = out_h.astype(np.float64)
    b = ref.astype(np.float64)
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    line = {"metric": "embedded tokens/sec (BERT-small ClassicBert, 64 chunks)", "value": tokens / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random token ids, random-init N(0,0.02) weights)",
            "config": {"workload": "classicbert_small_config1", "model": "BERT-small (12L, H384, 12x32, FFN 1536)",
                       "chunks": n, "lengths": "U[32,256]", "tokens": tokens, "pooling": "mean",
                       "l2": "flushed between steps (256 MiB write)"},
            "e2e": {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(tokens * 4 + 4 * (n + 1)),
                    "d2h_bytes_per_step": int(n * spec.hidden * 4),
                    "how": "rv_embed_varlen with host ids / cu_seqlens / output, host clock around the call"},
            "gpu_launches": int(launches), "clocks": clocks,
            "parity": {"min_cos": float(cos.min()), "p50_cos": float(np.median(cos)), "bar": 0.9999,
                       "against": "numpy fp32 port of the reference CPU path, all 64 chunks"},
            "cpu_baseline": {"value": tokens / cpu_s, "unit": "tokens/s", "cores": blas_threads(), "kind": "port",
                             "sample": f"all {n} chunks ({tokens} tokens, {cpu_s:.1f} s), numpy fp32 port"}}
    print(json.dumps(line), flush=True)


def run_cascade(args):
    """rank_cascade over a 10M x 768 database truncated to 256 dimensions (1 GPU): one step = one
    call for the query batch, top_k 10 (first phase: the exact top 100 of the truncated rows;
    second phase: exact re-rank with the full rows).  Host buffers, host clock around the call."""
    import torch

    from ripvec_b200 import synth
    from ripvec_b200.index import SearchIndex

    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    n_rows, dim, t_dim, top_k = args.scan_rows, 768, 256, 10
    gen = torch.Generator(device="cuda").manual_seed(100)
    db = torch.empty(n_rows, dim, device="cuda", dtype=torch.bfloat16)
    for s in range(0, n_rows, 1 << 20):
        e = min(n_rows, s + (1 << 20))
        x = torch.randn(e - s, dim, device="cuda", generator=gen)
        db[s:e] = (x / x.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    idx = SearchIndex(db, device=local, cascade_dim=t_dim)
    build_s = time.perf_counter() - t0
    del db
    pk = peaks()
    lines = []
    for nq in [int(v) for v in str(args.queries).split(",")]:
        q = synth.normalized_gaussian(nq, dim, seed=99)
        for _ in range(args.warmup):
            idx.topk_cascade(q, top_k)
        torch.cuda.synchronize()
        sampler = ClockSampler(physical_gpu(local))
        sampler.start()
        times = []
        launches0 = idx.kernel_launches()
        for _ in range(args.steps):
            t1 = time.perf_counter()
            idx.topk_cascade(q, top_k)
            times.append(time.perf_counter() - t1)
        launches = idx.kernel_launches() - launches0
        clocks = sampler.stop()
        sec = sum(times) / len(times)
        trunc_bytes = n_rows * t_dim * 2
        ach = trunc_bytes / sec / 1e9
        line = {"metric": "rank_cascade queries/sec (MRL 256 of 768, 10M rows)", "value": nq / sec,
                "unit": "queries/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sec,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic normalised Gaussian rows",
                "config": {"workload": "rank_cascade", "rows": n_rows, "dim": dim, "truncated_dim": t_dim,
                           "queries": nq, "top_k": top_k,
                           "timing": "host clock around the synchronous call (host queries and results)"},
                "build_s": build_s, "clocks": clocks, "gpu_launches": launches,
                "e2e": {"value": nq / sec, "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                        "d2h_bytes_per_step": nq * top_k * 12 + nq * 4,
                        "how": "the timed call itself: rv_index_rank_cascade with host queries and results"},
                "roofline": {"kernel": "rank_cascade step (exact scan of the truncated rows + full re-rank)",
                             "bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": ach / pk["hbm_gbs"], "peak_source": f"{pk['source']} hbm_gbs",
                             "traffic": None, "bytes_per_step": trunc_bytes}}
        lines.append(line)
    cpu_base = None if args.no_cpu_baseline else cpu_cascade_baseline(n_rows, dim, t_dim, top_k)
    for line in lines:
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), flush=True)
    idx.close()


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "scan":
        return run_scan(args)
    if args.workload == "turboquant":
        return run_turboquant(args)
    if args.workload == "duplicates":
        return run_duplicates(args)
    if args.workload == "cascade":
        return run_cascade(args)
    if args.workload == "classic":
        return run_classic(args)
    return run_encoder(args)


if __name__ == "__main__":
    main()
