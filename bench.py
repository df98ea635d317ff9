#!/usr/bin/env python
"""Ragged-batch decode throughput of the B200 engine (and of the reference).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE config "Llama-3-8B-shaped Q4_K"): vocab 128256, d_model
4096, 32 layers, 32/8 heads (head_dim 128), FFN 14336, RoPE theta 5e5,
Q4_K projections, Q8_0 embedding and output head.  512 ragged requests share
a 1024-token system prefix through the radix prefix cache; each has a unique
suffix of U(64, 2048) positions and has generated U(0, output) of its
U(64, 512) output tokens.  One step = one decode token for all 512 requests
in a single tvara_batch_step call.  Synthetic data: weights are seeded random
Q4_K/Q8_0 blocks; the shared prefix's K/V is computed by the engine (a real
1024-token prefill); every request's unique positions hold seeded random K/V
written into the pool (the decode step's work does not depend on their
values).  KV is F16.  N > 1 runs tensor parallel (NCCL allreduce after
o_proj and down_proj) over the same 512 requests: strong scaling.

Reported: value = decode tokens/s over the timed steps (device time on the
engine stream, max over ranks); e2e = wall-clock tokens/s of the same call a
serving loop makes (tvara_batch_step with host token arrays in and the next
tokens -- device argmax with the finiteness check -- back in host memory,
exactly what tvara_b200.scheduler.BatchedSchedulerBackend issues), and
e2e_full_logits = the same with every full-vocabulary F32 logit row copied to
the host; the dominant kernel's roofline (DRAM traffic from the committed ncu
captures) and the step roofline of the survey's convention (sum over kernels
of max(bytes / HBM peak, flops / tensor peak), shared prefix counted per
reader, over the measured step time); the reference CPU engine timed on this
host; SM clocks.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (read + write) from small-case ncu captures (profiles/), scaled to the benchmark's launches:
# attention per distinct K/V position of a launch (its traffic grows with the positions it reads), and the
# four projection launches of one layer at 512 tokens (their traffic does not depend on the layer count).
# DRAM bytes from small ncu captures (profiles/), scaled by the units a launch
# processes: attention per distinct K/V position per layer launch (2-layer,
# 64-request case), the Q4_K projections per layer at 512 tokens (1-layer case:
# QKV, o_proj, gate/up, down)
NCU_TRAFFIC = {"attention_per_distinct_position": {"f16": 4150.0, "i8": 2150.0}, "projections_per_layer": 226.4e6}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="llama8b")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (same per-layer shapes; small cases for ncu captures)")
    ap.add_argument("--requests", type=int, default=512)
    ap.add_argument("--prefix", type=int, default=1024)
    ap.add_argument("--suffix", type=int, nargs=2, default=(64, 2048), metavar=("MIN", "MAX"),
                    help="unique suffix length range per request")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--kv", choices=["f16", "f32", "i8"], default="f16")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-standalone", action="store_true", help="skip the standalone GEMV / matmul figures")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the timed decode step: no parity check, standalone kernels or other configs")
    ap.add_argument("--planes", choices=["auto", "hilo", "off", "q4kplane"], default="auto",
                    help="tensor-core weight form: auto (Q4_K read packed with side arrays, other types hi/lo), "
                         "hilo, off, q4kplane (Q4_K as a prebuilt FP16 plane of sc*q)")
    ap.add_argument("--standalone-only", action="store_true",
                    help="only the standalone GEMV / matmul figures (one JSON line; used for kernel profiles)")
    ap.add_argument("--cpu-tokens", type=int, default=2, help="tokens the reference CPU engine decodes")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model-dir", default=os.environ.get("TVARA_BENCH_DIR", "/tmp/tvara_bench"))
    ap.add_argument("--cpu-worker", default=None, help=argparse.SUPPRESS)
    return ap.parse_args()


# ----------------------------------------------------------------- workload
def model_config(args) -> dict:
    from tvara_b200 import gguf
    cfg = gguf.model_config(args.config)
    if args.layers:
        cfg["layers"] = args.layers
    return cfg


def model_path(args) -> Path:
    depth = f"_l{args.layers}" if args.layers else ""
    return Path(args.model_dir) / f"{args.config}{depth}_s{args.seed}.gguf"


def ensure_model(args, rank):
    from tvara_b200 import gguf
    path = model_path(args)
    if rank == 0 and not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        gguf.make_llama(tmp, model_config(args), seed=args.seed, random_packed=args.config != "tiny")
        tmp.rename(path)
    return path


def workload(args, vocab):
    rng = np.random.default_rng(args.seed + 1)
    n = args.requests
    prefix = rng.integers(0, vocab, args.prefix)
    suffix = rng.integers(args.suffix[0], args.suffix[1] + 1, n)
    out_len = rng.integers(64, 513, n)
    done = (rng.random(n) * out_len).astype(np.int64)
    first = rng.integers(0, vocab, n)
    return prefix, suffix, done, first


class DeviceView:
    """__cuda_array_interface__ over a raw device pointer (the KV pool)."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def fill_pool_random(model, seed):
    import torch
    info = model.kv_pool()
    n = info["max_blocks"] * info["block_elements"]
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    chunk = 1 << 28
    if info["kv_dtype"] == 2:  # int8 codes and one F32 scale per row of head_dim
        t = torch.as_tensor(DeviceView(info["base"], n, "|i1"), device="cuda")
        for i in range(0, n, chunk):
            t[i:i + chunk].random_(-127, 128, generator=g)
        rows = n // info["head_dim"]
        sc = torch.as_tensor(DeviceView(info["scales"], rows, "<f4"), device="cuda")
        sc.uniform_(0.005, 0.02, generator=g)
    else:
        t = torch.as_tensor(DeviceView(info["base"], n, "<f2" if info["kv_dtype"] == 1 else "<f4"), device="cuda")
        for i in range(0, n, chunk):
            t[i:i + chunk].normal_(0.0, 1.0, generator=g)
    torch.cuda.synchronize()


# ------------------------------------------------------------------- clocks
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(tempfile.mkdtemp()) / "clocks.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) > 8 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 8 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) > 8:
                for name, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------ CPU baseline
def cpu_worker(spec: str):
    """Reference engine (oracle/_ref) on the bench GGUF: decode tokens of one
    sequence and print tokens/s.  Runs in its own process."""
    path, tokens = spec.rsplit(":", 1)
    tokens = int(tokens)
    from oracle.model import RefEngine
    t0 = time.perf_counter()
    eng = RefEngine(path, max_blocks=4, block_tokens=16)
    load = time.perf_counter() - t0
    s = eng.create()
    eng.decode(s, 1)
    t0 = time.perf_counter()
    for i in range(tokens):
        eng.decode(s, 2 + i)
    dt = time.perf_counter() - t0
    print(json.dumps({"tokens": tokens, "seconds": dt, "load_seconds": load}))


def start_reference_cpu(path, tokens):
    """Starts the reference engine in a child process (it loads for minutes:
    the GPU work runs meanwhile)."""
    from oracle import oracle as O
    if O.ref_capi() is None:
        return None
    proc = subprocess.Popen([sys.executable, __file__, "--cpu-worker", f"{path}:{tokens}"], stdout=subprocess.PIPE,
                            text=True)
    return proc, tokens, time.perf_counter()


def reference_attention_seconds(cfg, context, seed=0):
    """The reference's fused_paged_attention (attention.hpp:57-83, compiled
    from its sources) for one query row of one layer over `context` cached
    positions of this model's head shape: median seconds of a few calls."""
    from oracle import oracle as O
    R = O.ref()
    if R is None:
        return None
    H, HKV, D = cfg["heads"], cfg["kv_heads"], cfg["hidden"] // cfg["heads"]
    tpb = 16
    c = R.ref_cache_new(1, HKV, D, tpb, context // tpb + 2)
    rng = np.random.default_rng(seed)
    s = R.ref_cache_create(c)
    kv = rng.standard_normal((context, 2, HKV * D), dtype=np.float32)
    for p in range(context):
        assert R.ref_cache_append(c, s, kv[p, 0], kv[p, 1]) == 0
    q = rng.standard_normal(H * D, dtype=np.float32)
    out = np.empty(H * D, np.float32)
    times = []
    for _ in range(5):
        t0 = time.perf_counter()
        assert R.ref_paged_attention(c, s, 0, H, q, None, None, 0, out) == 0
        times.append(time.perf_counter() - t0)
    R.ref_cache_free(c)
    return float(np.median(times))


def reference_cpu(path, cfg, mean_context, started):
    """Reference CPU engine on this host, one core (it runs one thread per
    model handle): seconds per token = the measured decode time per token at
    a context of a few positions (every projection, the LM head, norms) plus
    `layers` x the measured fused_paged_attention time of one query row at
    the workload's mean context.  tok/s = 1 / that."""
    if started is None:
        return None
    proc, tokens, t0 = started
    out = json.loads(proc.communicate()[0].strip().splitlines()[-1])
    wall = time.perf_counter() - t0
    short = out["seconds"] / out["tokens"]
    attn = reference_attention_seconds(cfg, int(round(mean_context)))
    per_token = short + (cfg["layers"] * attn if attn is not None else 0.0)
    return {"value": 1.0 / per_token, "unit": "tok/s", "cores": 1, "kind": "reference",
            "sample": (f"the reference engine (oracle/_ref, compiled from its sources; one thread, as it serves one "
                       f"handle) decoding {tokens} tokens of one sequence at context <= {tokens + 1} on the same GGUF "
                       f"(weights expanded to F32 as the reference does): {short:.3f} s/token; plus "
                       f"{cfg['layers']} x its fused_paged_attention for one query row at the workload's mean context "
                       f"{mean_context:.0f} ({attn if attn is not None else float('nan'):.4f} s/layer)"),
            "seconds_per_token_short_context": short, "attention_seconds_per_layer": attn,
            "mean_context": mean_context, "load_seconds": out["load_seconds"], "wall_seconds": wall}


# --------------------------------------------------------------------- runs
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = ensure_model(args, 0)
    cfg = model_config(args)
    from tvara_b200 import gguf
    vocab = len(gguf.GGUFFile(path).metadata["tokenizer.ggml.tokens"])
    prefix, suffix, done, _ = workload(args, vocab)
    mean_ctx = float(np.mean(args.prefix + suffix + done + 1))
    res = reference_cpu(path, cfg, mean_ctx, start_reference_cpu(path, args.cpu_tokens))
    line = {"impl": "reference", "metric": "ragged-batch decode tok/s (8B-shape Q4_K)", "unit": "tok/s",
            "higher_is_better": True, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"{args.config} decode, reference CPU engine at the workload's mean context",
                       "model": args.config}}
    if res is None:
        line["unavailable"] = "reference library oracle/_ref/libtvara_capi.so not built"
    else:
        line.update({"value": res["value"], "cpu_baseline": res,
                     "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    emit(line)


def standalone_cpu(kind, raw, rows, cols, weight_bytes):
    """The reference's fastest CPU path for the same projection at one token
    (int8 activations, KernelDispatch -- AVX2 on this host -- rows split over
    its ThreadPool; ref_matmul_dispatch over the reference's headers), on 1
    thread and on every host thread: median of a few calls, GB/s of packed
    weights."""
    from oracle import oracle as O
    R = O.ref()
    if R is None:
        return None
    x = np.random.default_rng(5).standard_normal(cols, dtype=np.float32)
    y = np.empty(rows, np.float32)
    out = {}
    for threads in (1, os.cpu_count() or 1):
        times = []
        for _ in range(5 if threads > 1 else 3):
            t0 = time.perf_counter()
            assert R.ref_matmul_dispatch(kind, raw, raw.size, rows, cols, x, 1, y, threads) == 0
            times.append(time.perf_counter() - t0)
        ms = float(np.median(times)) * 1e3
        out[f"threads{threads}"] = {"ms": round(ms, 3), "gbs": round(weight_bytes / ms / 1e6, 2), "cores": threads}
    return out


def standalone_gemv(lib, hbm_gbs, cpu=True):
    """Quantised GEMV (M = 1) and matmul (M = 8 ... 512) on the survey's
    standalone shape, 11008 x 4096, for Q4_K, Q8_0 and Q4_0, through the
    kernel-level ABI: GB/s of packed weights per launch over CUDA events.
    Eight weight copies (> L2) are used in turn, so every launch reads its
    weights from DRAM.  Beside each type, the reference's CPU path on this
    host (one token)."""
    import torch
    from tvara_b200 import gguf
    rows, cols, copies = 11008, 4096, 8
    rng = np.random.default_rng(11)
    out = {}
    for name, kind in (("q4_k", gguf.Q4_K), ("q8_0", gguf.Q8_0), ("q4_0", gguf.Q4_0)):
        nbytes = lib.tvara_packed_bytes(kind, rows, cols)
        host_raw = np.frombuffer(gguf.random_blocks(kind, rows, cols, rng), dtype=np.uint8).copy()
        raw = torch.from_numpy(host_raw).cuda()
        mats = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(copies)]
        for m in mats:
            assert lib.tvara_pack(kind, C.c_void_p(raw.data_ptr()), rows, cols, C.c_void_p(m.data_ptr()), None) == 0
        weight_bytes = rows * cols // {gguf.Q4_K: 256, gguf.Q8_0: 32, gguf.Q4_0: 32}[kind] * \
            {gguf.Q4_K: 144, gguf.Q8_0: 34, gguf.Q4_0: 18}[kind]
        res = {}
        for M in (1, 8, 32, 128, 512):
            x = torch.randn(M, cols, device="cuda")
            y = torch.empty(M, rows, device="cuda")
            ws_n = lib.tvara_quant_matmul_workspace(cols, M)
            ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device="cuda")

            def call(m, stream):
                assert lib.tvara_quant_matmul(kind, C.c_void_p(m.data_ptr()), rows, cols, C.c_void_p(x.data_ptr()),
                                              M, C.c_void_p(y.data_ptr()), C.c_void_p(ws.data_ptr()), ws_n,
                                              C.c_void_p(stream)) == 0
            # the calls are captured in a CUDA graph and replayed, so the
            # figure is device time, not the host cost of 64 ctypes calls
            side = torch.cuda.Stream()
            with torch.cuda.stream(side):
                for m in mats:
                    call(m, side.cuda_stream)
            torch.cuda.synchronize()
            reps = 64
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side, capture_error_mode="relaxed"):
                for i in range(reps):
                    call(mats[i % copies], side.cuda_stream)
            graph.replay()
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            graph.replay()
            s1.record()
            s1.synchronize()
            us = s0.elapsed_time(s1) * 1e3 / reps
            del graph
            moved = weight_bytes + M * cols * 4 + M * rows * 4
            res[f"m{M}"] = {"us": round(us, 2), "gbs": round(moved / us / 1e3, 1),
                            "frac_hbm": round(moved / us / 1e3 / hbm_gbs, 3),
                            "tflops": round(2.0 * M * rows * cols / us / 1e6, 2)}
        res["weight_bytes"] = weight_bytes
        if cpu:
            res["cpu_baseline_m1"] = standalone_cpu(kind, host_raw, rows, cols, weight_bytes)
        out[name] = res
    return {"shape": f"{rows}x{cols}", "weights": "seeded random packed blocks, 8 copies used in turn (> L2)",
            "note": "kernel-level ABI (tvara_quant_matmul), 64 calls replayed from a CUDA graph (device time); "
                    "frac_hbm counts packed weights + F32 activations in and out once",
            **out}


# ------------------------------------------------------- the other configs
def guard(fn, *args, **kw):
    """Runs one single-rank measurement; an exception is reported in the
    result line (and on stderr) instead of losing the whole line."""
    import traceback
    try:
        return fn(*args, **kw)
    except Exception as e:  # noqa: BLE001 -- reported, not swallowed
        traceback.print_exc()
        return {"error": f"{type(e).__name__}: {e}"}


def nccl_unique_id(rank, world):
    """A fresh NCCL unique id, made on rank 0 and shared over torch.distributed."""
    import torch.distributed as dist
    if world == 1:
        return None
    lib = C.CDLL("libnccl.so.2")
    buf = C.create_string_buffer(128)
    if rank == 0:
        assert lib.ncclGetUniqueId(buf) == 0
    obj = [buf.raw]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def allreduce_standalone(world, n=512 * 4096, reps=20):
    """NCCL's allreduce of the step's residual (512 x 4096 F32 = 8 MB) on
    its own, through torch.distributed: device time per call (CUDA events,
    max over ranks) and the bus bandwidth 2 (N-1)/N x bytes / time."""
    import torch
    import torch.distributed as dist
    x = torch.ones(n, device="cuda")
    for _ in range(5):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        dist.all_reduce(x)
    e1.record()
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / reps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    return {"bytes": n * 4, "us": round(us, 1), "bus_gbs": round(2 * (world - 1) / world * n * 4 / us / 1e3, 1),
            "note": "torch.distributed NCCL allreduce alone, 20 calls back to back; the engine's own residual "
                    "allreduce (kernels.collective) runs over NVLink peer memory unless TVARA_ALLREDUCE=nccl"}


def parity_check(args, rank, world, local, barrier):
    """The checker, outside every timed region: a 2-layer model with the
    benchmark's widths (llama8b shape, Q4_K / Q8_0), split over the same ranks
    as the benchmark, runs one ragged step of 64 sequences that share a
    1000-position radix prefix (copy-on-write of its tail) and hold 64..1000
    positions of their own, 1..8 tokens each; rank 0 compares every row's
    logits with the CPU oracle (oracle/parity.py)."""
    from oracle import parity
    from tvara_b200 import gguf
    from tvara_b200.native import NativeModel
    path = Path(args.model_dir) / "llama8b_l2_parity_s0.gguf"
    if rank == 0 and not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        gguf.make_llama(tmp, gguf.model_config("llama8b", layers=2), seed=0, random_packed=True)
        tmp.rename(path)
    barrier()
    requests, prefix, suffix = 64, 1000, (64, 1000)
    blocks = requests * ((prefix + suffix[1] + 24) // 16 - prefix // 16 + 1) + prefix // 16 + 8
    t0 = time.perf_counter()
    model = NativeModel(path, max_blocks=blocks, block_tokens=16, kv_dtype=args.kv, device=local,
                        max_step_tokens=2048, tp_rank=rank, tp_size=world, nccl_id=nccl_unique_id(rank, world))
    try:
        case = parity.build_step(model, seed=args.seed + 31, requests=requests, prefix=prefix, suffix=suffix,
                                 extra_rows=8, rank=rank, world=world)
        got, _ = model.batch_step(case["seqs"], case["tokens"], all_logits=True)
    finally:
        model.close()
    res = None
    if rank == 0:
        f16 = (lambda x: x.astype(np.float16).astype(np.float32)) if args.kv == "f16" else None
        want = parity.oracle_rows(path, case, max_positions=prefix + suffix[1] + 16, kv_round=f16)
        res = parity.compare(got, want) if f16 is None else parity.compare(got, want, parity.F16_ATOL, parity.F16_RTOL)
        if f16 is not None:  # distance of the F16-stored rows from the reference's F32 KV
            ref = parity.oracle_rows(path, case, max_positions=prefix + suffix[1] + 16)
            res["vs_f32_reference"] = {"max_abs": float(np.abs(got - ref).max()),
                                       "note": "the oracle above stores the step's new K/V rows in F16 as the pool "
                                               "does; this is the same rows against the reference's F32 KV"}
        res.update({"case": f"llama8b widths, 2 layers, tp{world}, {args.kv} KV, {requests} sequences sharing a "
                            f"{prefix}-position radix prefix + U({suffix[0]},{suffix[1]}) own positions, "
                            f"{len(want)} rows in one step",
                    "seconds": round(time.perf_counter() - t0, 1)})
    barrier()
    return res


def smollm2_replicas(args, rank, world, local, barrier, dist):
    """SmolLM2-135M-shaped Q8_0 served as replicas: 256 requests (prompts
    U(32,1024), outputs U(16,256), seeded) divided least-loaded over the
    ranks; each rank serves its share with continuous batching (512-token
    prefill chunks, one tvara_batch_step per iteration, argmax back) on its
    own full model and F32 KV pool.  Time: max over ranks of the serving wall
    time (host token lists in, next tokens out, every iteration)."""
    import torch
    from tvara_b200 import gguf
    from tvara_b200.native import NativeModel
    from tvara_b200.serving import ContinuousBatcher, shard_requests, synthetic_requests
    path = Path(args.model_dir) / "smollm2_s0.gguf"
    if rank == 0 and not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        gguf.make_llama(tmp, "smollm2", seed=0, random_packed=True)
        tmp.rename(path)
    barrier()
    cfg = gguf.model_config("smollm2")
    reqs = synthetic_requests(256, cfg["vocab"], prompt=(32, 1024), output=(16, 256), seed=args.seed + 7)
    mine = [reqs[i] for i in shard_requests(reqs, world)[rank]]
    tpb = 16
    blocks = sum(-(-r.work // tpb) for r in mine) + 64
    model = NativeModel(path, max_blocks=blocks, block_tokens=tpb, device=local, max_step_tokens=8192)
    try:
        warm = synthetic_requests(16, cfg["vocab"], prompt=(32, 600), output=(4, 8), seed=99)
        ContinuousBatcher(model, kv_blocks=blocks, block_tokens=tpb, prefill_chunk=512).run(warm)
        torch.cuda.synchronize()
        barrier()
        batcher = ContinuousBatcher(model, kv_blocks=blocks, block_tokens=tpb, prefill_chunk=512)
        launches0 = model._library.tvara_kernel_launches()
        t0 = time.perf_counter()
        batcher.run(mine)
        secs = time.perf_counter() - t0
        launches = model._library.tvara_kernel_launches() - launches0
    finally:
        model.close()
    if world > 1:
        t = torch.tensor([secs], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    out_tokens = sum(r.max_tokens for r in reqs)
    all_tokens = out_tokens + sum(len(r.prompt) for r in reqs)
    weights = 142.9e6
    return {"metric": "served output tok/s (SmolLM2-135M-shaped Q8_0, 256 requests, replicas)",
            "value": out_tokens / secs, "unit": "tok/s", "n_gpus": world, "scaling": "strong",
            "seconds": secs, "tokens_per_s_incl_prompt": all_tokens / secs,
            "rank0": {"requests": len(mine), "steps": batcher.steps, "prefill_tokens": batcher.prefill_tokens,
                      "decode_tokens": batcher.decode_tokens, "gpu_launches": int(launches),
                      "weight_gb_per_s": round(batcher.steps * weights / secs / 1e9, 1)},
            "config": {"workload": "256 requests, prompts U(32,1024), outputs U(16,256), chunked prefill 512, "
                                   "F32 KV, least-loaded sharding of requests over replicas",
                       "parallelism": f"replicas{world}"},
            "timing": "wall clock of the serving loop on each rank (max over ranks); e2e by construction"}


def tiny_generate(args, local):
    """Tiny Llama Q8_0: one sequence, a 64-token
    seeded prompt then 64 greedy tokens (NativeModel.generate: one device
    step for the prompt, one per token, argmax on the device), F32 KV."""
    from tvara_b200 import gguf
    from tvara_b200.native import NativeModel
    path = Path(args.model_dir) / "tiny_s0.gguf"
    if not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        gguf.make_llama(path, "tiny", seed=0)
    prompt = np.random.default_rng(1).integers(0, 512, 64).tolist()
    with NativeModel(path, max_blocks=16, block_tokens=16, device=local) as m:
        m.generate(prompt, max_new_tokens=8)
        times = []
        for _ in range(5):
            t0 = time.perf_counter()
            toks = m.generate(prompt, max_new_tokens=64)
            times.append(time.perf_counter() - t0)
    secs = float(np.median(times))
    return {"metric": "greedy decode tok/s (tiny Llama Q8_0, 64-token prompt, 64 tokens)",
            "value": 64 / secs, "unit": "tok/s", "ms_per_token": secs / 64 * 1e3, "tokens": len(toks),
            "note": "median of 5 generate calls, wall clock incl. the prompt step; latency-bound (5 MB of "
                    "weights per token)", "reference_published": "8,770 tok/s on the reference's own 4-core host"}


def attention_config(lib, hbm_gbs, seed=0, cpu=True):
    """Standalone fused paged GQA attention: 64
    sequences, contexts log-uniform in [128, 8192], 32/8 heads of 128, block
    size 16; block tables drawn from a random permutation of a 40,000-block
    pool, 10% of each sequence's blocks shared copy-on-write with its pair
    sequence; Q and K/V ~ N(0, 1).  Decode: one query row per sequence.
    Chunked prefill: the last 512 positions of each sequence as query rows
    (row i sees the first context-512+i+1 positions).  Per call through
    tvara_paged_attention (which uploads the tables and waits for the
    kernels' error word): median device time between CUDA events around the
    call.  KV bytes: every visible position's K and V read once per query row
    that sees it (decode: once per sequence)."""
    import torch
    from tvara_b200._bindings import AttentionArgs
    rng = np.random.default_rng(seed)
    H, HKV, D, tpb, pool_blocks = 32, 8, 128, 16, 40000
    ctx = np.exp(rng.uniform(np.log(128), np.log(8192), 64)).astype(np.int64)
    perm = list(rng.permutation(pool_blocks))
    tables = []
    for n in ctx:
        tables.append([int(perm.pop()) for _ in range(-(-int(n) // tpb))])
    for i in range(0, 64, 2):  # 10% of the blocks of each pair shared (copy-on-write prefix)
        k = max(1, int(0.1 * min(len(tables[i]), len(tables[i + 1]))))
        tables[i + 1][:k] = tables[i][:k]
    flat = np.ascontiguousarray([b for t in tables for b in t], np.int32)
    offs = np.cumsum([0] + [len(t) for t in tables])[:-1].astype(np.uint32)
    res = {"sequences": 64, "mean_context": float(ctx.mean()), "pool_blocks": pool_blocks}
    for kv, es in (("f16", 2), ("f32", 4)):
        pool = torch.empty(pool_blocks * 2 * HKV * tpb * D, dtype=torch.float16 if kv == "f16" else torch.float32,
                           device="cuda").normal_()
        out_kv = {}
        for mode in ("decode", "prefill512"):
            if mode == "decode":
                vis = ctx.astype(np.uint32)
                off = offs
            else:
                rows = [(i, int(n) - min(512, int(n)) + j + 1) for i, n in enumerate(ctx) for j in range(min(512, int(n)))]
                vis = np.array([v for _, v in rows], np.uint32)
                off = offs[[i for i, _ in rows]]
            q = torch.randn(len(vis), H * D, device="cuda")
            out = torch.empty_like(q)
            a = AttentionArgs()
            a.struct_size = C.sizeof(AttentionArgs)
            a.kv_dtype = 1 if kv == "f16" else 0
            a.heads, a.kv_heads, a.head_dim, a.block_tokens, a.layers, a.layer = H, HKV, D, tpb, 1, 0
            a.max_blocks, a.n_queries = pool_blocks, len(vis)
            a.q, a.out, a.pool = q.data_ptr(), out.data_ptr(), pool.data_ptr()
            a.tables, a.tables_len = flat.ctypes.data, len(flat)
            vis = np.ascontiguousarray(vis)
            off = np.ascontiguousarray(off, np.uint32)
            a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
            n = lib.tvara_paged_attention_workspace(C.byref(a))
            ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")
            stream = torch.cuda.current_stream()
            times = []
            for rep in range(6):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                assert lib.tvara_paged_attention(C.byref(a), C.c_void_p(ws.data_ptr()), n,
                                                 C.c_void_p(stream.cuda_stream)) == 0, lib.tvara_last_error()
                e1.record(stream)
                e1.synchronize()
                if rep:
                    times.append(e0.elapsed_time(e1) * 1e3)
            us = float(np.median(times))
            kv_bytes = float(np.sum(vis.astype(np.float64))) * 2 * HKV * D * es
            flops = 4.0 * float(np.sum(vis.astype(np.float64))) * D * H
            out_kv[mode] = {"us": round(us, 1), "rows": int(len(vis)), "kv_bytes_per_reader": kv_bytes,
                            "gbs_per_reader": round(kv_bytes / us / 1e3, 1),
                            "frac_hbm_per_reader": round(kv_bytes / us / 1e3 / hbm_gbs, 3),
                            "tflops": round(flops / us / 1e6, 2)}
        res[kv] = out_kv
        del pool
        torch.cuda.empty_cache()
    if cpu:
        cfg = {"heads": H, "kv_heads": HKV, "hidden": H * D, "layers": 1}
        per = [reference_attention_seconds(cfg, int(n), seed=i) for i, n in enumerate(ctx[:16])]
        if per[0] is not None:
            scale = float(ctx.sum() / ctx[:16].sum())
            res["cpu_baseline_decode"] = {"us": round(sum(per) * scale * 1e6, 1), "cores": 1, "kind": "reference",
                                          "sample": "fused_paged_attention (attention.hpp:57-83) of the first 16 "
                                                    "sequences at their contexts, F32 KV, scaled to all 64 by "
                                                    "total context"}
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist
    from tvara_b200.native import NativeModel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    path = ensure_model(args, rank)
    barrier()
    # the reference CPU engine loads for minutes: it runs beside the GPU work
    # on one host core and is collected at the end
    cpu_job = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_job = start_reference_cpu(path, args.cpu_tokens)
    nccl_id = nccl_unique_id(rank, world)
    from tvara_b200 import gguf
    g = gguf.GGUFFile(path)
    vocab = len(g.metadata["tokenizer.ggml.tokens"])
    prefix, suffix, done, first = workload(args, vocab)
    total_steps = args.warmup + 2 * args.steps + 2 * args.e2e_steps + 2
    tpb = 16
    unique = suffix + done + total_steps
    blocks = int(np.sum((args.prefix + unique + tpb - 1) // tpb - args.prefix // tpb)) + args.prefix // tpb + 64
    model = NativeModel(path, max_blocks=blocks, block_tokens=tpb, kv_dtype=args.kv, device=local,
                        max_step_tokens=max(2048, args.prefix), tp_rank=rank, tp_size=world, nccl_id=nccl_id,
                        weight_planes=None if args.planes == "auto" else args.planes)
    wbytes = model.weight_bytes()
    fill_pool_random(model, args.seed + 2 + rank)
    seq0 = model._new_sequence()
    model.batch_step([seq0], [prefix.tolist()], logits=False)  # real prefill of the shared prefix
    node = model.prefix_insert(prefix.tolist(), seq0)
    seqs = []
    for i in range(args.requests):
        s, reused = model.prefix_reuse(prefix.tolist() + [int(first[i])])
        assert reused == args.prefix, reused
        model.reserve(s, int(suffix[i] + done[i]))
        seqs.append(s)
    model.prefix_pin(node)
    lens0 = np.array([model.sequence_length(s) for s in seqs])
    seqs = np.array(seqs, dtype=np.uint64)
    tokens = np.asarray(first, dtype=np.uint32).copy()

    def step(logits=False):
        out, am = model.batch_step(seqs, tokens, logits=logits, argmax=True, finite_argmax=True)
        tokens[:] = am
        return out

    for _ in range(args.warmup):
        step()
    ext = torch.cuda.ExternalStream(model.stream)
    lib = model._library
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    torch.cuda.synchronize()
    barrier()
    clocks.start()
    launches0 = lib.tvara_kernel_launches()
    start.record(ext)
    for _ in range(args.steps):
        step()
    end.record(ext)
    end.synchronize()
    launches = lib.tvara_kernel_launches() - launches0
    clk = clocks.stop()
    torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end)
    # kernel-class breakdown: the same number of steps again, with CUDA events
    # around each launch group (kept out of the timed region above)
    lib.tvara_model_profile(model._handle, 1)
    for _ in range(args.steps):
        step()
    prof_ms = (C.c_double * 6)()
    prof_n = (C.c_uint64 * 6)()
    lib.tvara_model_profile_read(model._handle, prof_ms, prof_n, 6)
    lib.tvara_model_profile(model._handle, 0)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = args.requests * args.steps / (ms / 1e3)

    # ---- e2e: the same call from the host, wall clock (next tokens back; then full logits back)
    caller_h2d = args.requests * (4 + 8) + (args.requests + 1) * 4  # tokens, sequence ids, cu_tokens

    def e2e(logits):
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            step(logits=logits)
        secs = time.perf_counter() - t0
        h2d, d2h = C.c_uint64(), C.c_uint64()
        lib.tvara_model_step_bytes(model._handle, C.byref(h2d), C.byref(d2h))
        if world > 1:
            t = torch.tensor([secs], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            secs = float(t.item())
        return {"value": args.requests * args.e2e_steps / secs, "unit": "tok/s",
                "h2d_bytes_per_step": int(h2d.value) + caller_h2d, "d2h_bytes_per_step": int(d2h.value)}

    e2e_tokens = e2e(False)
    e2e_tokens["note"] = ("tvara_batch_step: host token / sequence arrays in, next tokens (device argmax, "
                          "finiteness checked) out -- the BatchedSchedulerBackend call")
    e2e_logits = e2e(True)
    e2e_logits["note"] = "same, plus every full-vocabulary F32 logit row copied to host memory"

    # ---- roofline of the dominant kernel class
    pk, pk_kind = peaks()
    cfg = model_config(args)
    L, H, HKV, D = cfg["layers"], cfg["heads"], cfg["kv_heads"], cfg["hidden"]
    dh = D // H
    tp = world
    es = {"f16": 2, "f32": 4, "i8": 1}[args.kv]
    mean_ctx = float(np.mean(lens0 + args.warmup + args.steps + 1 + (args.steps - 1) / 2))  # profiled pass
    row_scale = 4 if args.kv == "i8" else 0  # int8 pools: one F32 scale per K/V row
    pos_bytes = 2 * (HKV // tp) * (dh * es + row_scale)  # K and V of one position, this rank's heads
    qo_bytes = args.requests * 2 * (H // tp) * dh * 4
    # per reader: every visible position once per request that attends to it (the shared prefix 512 times)
    attn_bytes = args.requests * mean_ctx * pos_bytes + qo_bytes
    # compulsory: every distinct position once (the prefix once, each request's own positions once)
    distinct = args.prefix + args.requests * (mean_ctx - args.prefix)
    attn_bytes_compulsory = distinct * pos_bytes + qo_bytes
    attn_launches = int(prof_n[0])
    attn_ms = float(prof_ms[0])
    proj_launches = int(prof_n[1])
    proj_ms = float(prof_ms[1])
    params = L * (D * D * 2 + 2 * D * (HKV * dh) + 3 * D * cfg["ffn"]) / tp
    proj_flops_step = 2.0 * args.requests * params
    kernels = {
        "attention": {"ms_per_step": attn_ms / args.steps, "launches_per_step": attn_launches / args.steps,
                      "bytes_per_launch": attn_bytes_compulsory, "bytes_per_launch_per_reader": attn_bytes,
                      "achieved_gbs": attn_bytes_compulsory / (attn_ms / attn_launches * 1e-3) / 1e9
                      if attn_launches else None},
        "projections": {"ms_per_step": proj_ms / args.steps, "flops_per_step": proj_flops_step,
                        "achieved_tflops": proj_flops_step / (proj_ms / args.steps * 1e-3) / 1e12 if proj_ms else None},
        "head": {"ms_per_step": prof_ms[2] / args.steps},
        "other": {"ms_per_step": prof_ms[3] / args.steps},
        "collective": {"ms_per_step": prof_ms[4] / args.steps},
        "host_gap": {"ms_per_step": prof_ms[5] / args.steps,
                     "note": "stream idle on the host between steps (previous results back -> next step's first copy)"},
    }
    hbm, tensor = pk["hbm_gbs"], pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    ach = kernels["attention"]["achieved_gbs"]
    attn_kernel = {"f16": "attn_mma_kernel", "i8": "attn_mma_i8_kernel"}.get(args.kv, "attn_kernel")
    per_pos = NCU_TRAFFIC["attention_per_distinct_position"].get(args.kv)
    roof_attn = {"kernel": f"{attn_kernel} (paged attention, one launch per layer)", "bound": "hbm",
                 "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm if ach else None,
                 "traffic": per_pos * distinct if per_pos and tp == 1 else None, "peak_source": pk_kind,
                 "algorithmic_bytes_per_launch": attn_bytes_compulsory,
                 "per_reader": {"bytes_per_launch": attn_bytes,
                                "achieved_gbs": attn_bytes / (attn_ms / attn_launches * 1e-3) / 1e9
                                if attn_launches else None},
                 "note": "achieved = compulsory bytes (each distinct K/V position of the launch once: the shared "
                         "prefix once, every request's own positions once) / mean launch time; per_reader counts the "
                         "prefix once per request (L2 serves the repeats); traffic = ncu DRAM bytes per distinct "
                         "position from a small capture (profiles/), times this launch's distinct positions"}
    ach = kernels["projections"]["achieved_tflops"]
    per_row = NCU_TRAFFIC["projections_per_layer"]
    roof_proj = {"kernel": "tc_gemm_q4kp_kernel (the Q4_K projections of a step)", "bound": "tensor", "achieved": ach,
                 "peak": tensor, "unit": "TFLOP/s", "frac": ach / tensor if ach else None,
                 "traffic": per_row / 4 if per_row and tp == 1 and args.requests == 512 else None,
                 "peak_source": pk_kind,
                 "algorithmic_flops_per_step": proj_flops_step, "tensor_work_multiplier": 2,
                 "note": "useful flops 2*T*rows*cols; the Q4_K form issues 2 FP16 MMAs per product (plane of "
                         "sc*q times the hi and lo activation parts) plus the min term (1/32 of the K range)"}
    roof = roof_attn if attn_ms >= proj_ms else roof_proj
    # survey convention: sum over kernels of max(bytes/BW, flops/P) over the measured step time
    head_bytes = cfg["vocab"] * D * 34 / 32
    t_attn = L * max(attn_bytes / (hbm * 1e9), 4.0 * args.requests * mean_ctx * dh * (H // tp) / (tensor * 1e12))
    weight_bytes = params * 0.5625 + head_bytes
    t_proj = max(weight_bytes / (hbm * 1e9), (proj_flops_step + 2.0 * args.requests * cfg["vocab"] * D) / (tensor * 1e12))
    t_roof_ms = (t_attn + t_proj) * 1e3
    step_roof = {"t_roof_ms": t_roof_ms, "measured_ms": ms_per_step, "frac": t_roof_ms / ms_per_step,
                 "convention": "sum over kernels of max(bytes/HBM, flops/tensor peak); shared prefix per reader"}

    model.close()
    torch.cuda.empty_cache()
    single = rank == 0 and world == 1
    extras = not args.no_extras
    gemv = guard(standalone_gemv, lib, hbm, cpu=cpu_job is not None) \
        if single and not args.no_standalone and extras else None
    cpu = guard(reference_cpu, path, cfg, mean_ctx, cpu_job) if cpu_job else None
    parity = parity_check(args, rank, world, local, barrier) if extras else None
    if world > 1:
        kernels["collective"]["nccl_allreduce_8mb_alone"] = allreduce_standalone(world)
        kernels["collective"]["implementation"] = ("NCCL allreduce" if os.environ.get("TVARA_ALLREDUCE") == "nccl"
                                                   else "two-shot allreduce over NVLink peer memory (p2p_allreduce.cu)")
        kernels["collective"]["calls_per_step"] = 2 * cfg["layers"]
    other = {}
    if extras:
        other["smollm2"] = smollm2_replicas(args, rank, world, local, barrier, dist)
        if single:
            other["tiny"] = guard(tiny_generate, args, local)
            other["attention"] = guard(attention_config, lib, hbm, cpu=cpu_job is not None)
    line = {
        "metric": "ragged-batch decode tok/s (8B-shape Q4_K)", "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": f"f32 (Q4_K/Q8_0 weights, {args.kv} KV)",
        "data": "synthetic",
        "config": {"workload": f"{args.config} ragged decode, {args.requests} requests, shared {args.prefix}-token "
                               f"prefix + U({args.suffix[0]},{args.suffix[1]}) suffix + U(0,out) generated, "
                               "1 token/request/step",
                   "model": args.config + (f" ({args.layers} layers)" if args.layers else ""),
                   "global_batch": args.requests, "seq_len": float(np.mean(lens0)),
                   "parallelism": f"tp{world}", "kv": args.kv, "block_tokens": tpb,
                   "weights_gb": {"packed": round(wbytes["packed"] / 1e9, 2),
                                  "tensor_core_forms": round(wbytes["planes"] / 1e9, 2)},
                   "tensor_core_weight_form": {"auto": "Q4_K: packed rows, sc*q built per K-step in tensor memory or "
                                                       "shared memory (chosen per launch), block scales + minima in "
                                                       "side arrays (2 MMAs per K-step); other types: exact hi/lo "
                                                       "FP16 planes",
                                               "q4kplane": "Q4_K: prebuilt FP16 plane of sc*q (2 MMAs per K-step); "
                                                           "other types: exact hi/lo FP16 planes",
                                               "hilo": "exact hi/lo FP16 planes (3 MMAs per K-step)",
                                               "off": "packed rows dequantised by producer warps"}[args.planes],
                   "l2": "inputs larger than L2 (KV ~%.0f GB, weights ~4.5 GB)" % (blocks * 2 * 2 ** 20 / 1e9)},
        "e2e": e2e_tokens, "e2e_full_logits": e2e_logits,
        "roofline": roof, "rooflines": {"attention": roof_attn, "projections": roof_proj}, "step_roofline": step_roof,
        "kernels": kernels, "standalone_kernels": gemv, "gpu_launches": int(launches), "clocks": clk,
        "cpu_baseline": cpu, "parity": parity, "other_configs": other,
    }
    if rank == 0:
        emit(line)
    if world > 1:
        dist.destroy_process_group()


_RESULT = None  # the original stdout, kept for the one result line


def emit(line: dict) -> None:
    """Writes the result JSON line to the process's original stdout."""
    out = _RESULT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _RESULT
    args = parse()
    if args.cpu_worker:
        cpu_worker(args.cpu_worker)
        return
    # Libraries (NCCL's version banner, warnings) may print to stdout; the
    # contract is ONE JSON line there, so fd 1 is pointed at stderr and the
    # result goes to a duplicate of the original stdout.
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.standalone_only:
        from tvara_b200 import load_library
        emit({"standalone_kernels": standalone_gemv(load_library(), peaks()[0]["hbm_gbs"])})
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
