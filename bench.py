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

# DRAM bytes (read + write) per launch from ncu captures of this workload
# (profiles/attn_mma_llama8b_decode512.txt for F16 KV, profiles/attn_mma_i8_llama8b_decode512.txt for int8 KV,
# profiles/tc_gemm_q4k_llama8b_512tok.txt: the average over the four projection launches of a layer).
NCU_TRAFFIC = {"attention": {"f16": 2.63e9, "i8": 1.41e9}, "projections": 1.42e8}


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
    ap.add_argument("--planes", choices=["auto", "hilo", "off"], default="auto",
                    help="tensor-core weight form: auto (Q4_K plane of sc*q, other types hi/lo), hilo, off")
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


def start_reference_cpu(path, tokens, processes):
    from oracle import oracle as O
    if O.ref_capi() is None:
        return None
    procs = [subprocess.Popen([sys.executable, __file__, "--cpu-worker", f"{path}:{tokens}"], stdout=subprocess.PIPE,
                              text=True) for _ in range(processes)]
    return procs, tokens, time.perf_counter()


def reference_cpu(path, tokens, processes, started=None):
    started = started or start_reference_cpu(path, tokens, processes)
    if started is None:
        return None
    procs, tokens, t0 = started
    outs = [json.loads(p.communicate()[0].strip().splitlines()[-1]) for p in procs]
    wall = time.perf_counter() - t0
    total = sum(o["tokens"] for o in outs)
    slowest = max(o["seconds"] for o in outs)
    return {"value": total / slowest, "unit": "tok/s", "cores": processes, "kind": "reference",
            "sample": (f"{processes} process(es) of the reference engine (oracle/_ref, compiled from its sources; "
                       f"one thread per handle) each decoding {tokens} tokens of one sequence after a 1-token prompt "
                       f"on the same GGUF (weights expanded to F32 as the reference does); context <= {tokens + 1}, "
                       "so the reference's attention cost at the workload's contexts is not included"),
            "load_seconds": max(o["load_seconds"] for o in outs), "wall_seconds": wall}


def cpu_processes():
    try:
        mem = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    except (ValueError, OSError):
        mem = 64 << 30
    per = 40 << 30  # the reference expands the 8B model to ~36 GB of F32
    return max(1, min(os.cpu_count() or 1, int(mem * 0.6 // per), 8))


# --------------------------------------------------------------------- runs
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = ensure_model(args, 0)
    procs = cpu_processes()
    res = reference_cpu(path, args.cpu_tokens, procs)
    line = {"impl": "reference", "metric": "ragged-batch decode tok/s (8B-shape Q4_K)", "unit": "tok/s",
            "higher_is_better": True, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"{args.config} decode, reference CPU engine", "model": args.config}}
    if res is None:
        line["unavailable"] = "reference library oracle/_ref/libtvara_capi.so not built"
    else:
        line.update({"value": res["value"], "cpu_baseline": res,
                     "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    emit(line)


def standalone_gemv(lib, hbm_gbs):
    """Quantised GEMV (M = 1) and small-M matmul on the survey's standalone
    shape, 11008 x 4096, through the kernel-level ABI: GB/s of packed weights
    per launch over CUDA events.  Eight weight copies (> L2) are used in turn,
    so every launch reads its weights from DRAM."""
    import torch
    from tvara_b200 import gguf
    rows, cols, copies = 11008, 4096, 8
    rng = np.random.default_rng(11)
    out = {}
    for name, kind in (("q4_k", gguf.Q4_K), ("q8_0", gguf.Q8_0), ("q4_0", gguf.Q4_0)):
        nbytes = lib.tvara_packed_bytes(kind, rows, cols)
        raw = torch.from_numpy(np.frombuffer(gguf.random_blocks(kind, rows, cols, rng), dtype=np.uint8).copy()).cuda()
        mats = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(copies)]
        for m in mats:
            assert lib.tvara_pack(kind, C.c_void_p(raw.data_ptr()), rows, cols, C.c_void_p(m.data_ptr()), None) == 0
        weight_bytes = rows * cols // {gguf.Q4_K: 256, gguf.Q8_0: 32, gguf.Q4_0: 32}[kind] * \
            {gguf.Q4_K: 144, gguf.Q8_0: 34, gguf.Q4_0: 18}[kind]
        res = {}
        for M in ((1, 8, 32, 128, 512) if kind == gguf.Q4_K else (1,)):
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
        out[name] = res
    return {"shape": f"{rows}x{cols}", "weights": "seeded random packed blocks, 8 copies used in turn (> L2)",
            "note": "kernel-level ABI, 64 calls replayed from a CUDA graph (device time); M <= 4 CUDA-core GEMV, "
                    "M >= 5 tensor cores on the packed (producer) path incl. the activation split",
            **out}


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
        cpu_job = start_reference_cpu(path, args.cpu_tokens, 1)
    nccl_id = None
    if world > 1:
        lib = C.CDLL("libnccl.so.2")
        buf = C.create_string_buffer(128)
        if rank == 0:
            assert lib.ncclGetUniqueId(buf) == 0
        obj = [buf.raw]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
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
    attn_bytes = args.requests * (mean_ctx * 2 * (HKV // tp) * (dh * es + row_scale) + 2 * (H // tp) * dh * 4)
    attn_launches = int(prof_n[0])
    attn_ms = float(prof_ms[0])
    proj_launches = int(prof_n[1])
    proj_ms = float(prof_ms[1])
    params = L * (D * D * 2 + 2 * D * (HKV * dh) + 3 * D * cfg["ffn"]) / tp
    proj_flops_step = 2.0 * args.requests * params
    kernels = {
        "attention": {"ms_per_step": attn_ms / args.steps, "launches_per_step": attn_launches / args.steps,
                      "bytes_per_launch": attn_bytes,
                      "achieved_gbs": attn_bytes / (attn_ms / attn_launches * 1e-3) / 1e9 if attn_launches else None},
        "projections": {"ms_per_step": proj_ms / args.steps, "flops_per_step": proj_flops_step,
                        "achieved_tflops": proj_flops_step / (proj_ms / args.steps * 1e-3) / 1e12 if proj_ms else None},
        "head": {"ms_per_step": prof_ms[2] / args.steps},
        "other": {"ms_per_step": prof_ms[3] / args.steps},
        "collective": {"ms_per_step": prof_ms[4] / args.steps},
        "host_gap": {"ms_per_step": prof_ms[5] / args.steps,
                     "note": "stream idle on the host between steps (previous results back -> next step's first copy)"},
    }
    full = args.layers is None and tp == 1 and args.requests == 512
    hbm, tensor = pk["hbm_gbs"], pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    ach = kernels["attention"]["achieved_gbs"]
    attn_kernel = {"f16": "attn_mma_kernel", "i8": "attn_mma_i8_kernel"}.get(args.kv, "attn_kernel")
    roof_attn = {"kernel": f"{attn_kernel} (paged attention, one launch per layer)", "bound": "hbm",
                 "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm if ach else None,
                 "traffic": NCU_TRAFFIC["attention"].get(args.kv) if full else None, "peak_source": pk_kind,
                 "algorithmic_bytes_per_launch": attn_bytes,
                 "note": "algorithmic bytes count the shared 1024-token prefix once per reader; DRAM traffic "
                         "reads it once (L2 serves the rest), so frac can exceed 1"}
    ach = kernels["projections"]["achieved_tflops"]
    roof_proj = {"kernel": "tc_gemm_q4k_kernel (the Q4_K projections of a step)", "bound": "tensor", "achieved": ach,
                 "peak": tensor, "unit": "TFLOP/s", "frac": ach / tensor if ach else None,
                 "traffic": NCU_TRAFFIC["projections"] if full else None, "peak_source": pk_kind,
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

    gemv = standalone_gemv(lib, hbm) if rank == 0 and world == 1 and not args.no_standalone else None
    cpu = reference_cpu(path, args.cpu_tokens, 1, cpu_job) if cpu_job else None
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
                   "tensor_core_weight_form": {"auto": "Q4_K: FP16 plane of sc*q + block scales + minima "
                                                       "(2 MMAs per K-step); other types: exact hi/lo FP16 planes",
                                               "hilo": "exact hi/lo FP16 planes (3 MMAs per K-step)",
                                               "off": "packed rows dequantised by producer warps"}[args.planes],
                   "l2": "inputs larger than L2 (KV ~%.0f GB, weights ~4.5 GB)" % (blocks * 2 * 2 ** 20 / 1e9)},
        "e2e": e2e_tokens, "e2e_full_logits": e2e_logits,
        "roofline": roof, "rooflines": {"attention": roof_attn, "projections": roof_proj}, "step_roofline": step_roof,
        "kernels": kernels, "standalone_kernels": gemv, "gpu_launches": int(launches), "clocks": clk,
        "cpu_baseline": cpu,
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
