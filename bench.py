#!/usr/bin/env python
"""Benchmark: MOSS-TTS-Nano per-frame LLM step on B200, frames/s for the whole job.

Workload: per GPU, 64 independent streams with KV lengths drawn
uniformly from 64..1024 (seeded), paged fp16 KV with 16-token pages.  One step = one full
audio frame for every stream: the 17-step local decoder with the W8A8 end gate and 16
greedy codes (repetition penalty 1.2), then the 12-layer global decode step that appends one
KV position.  Weights: the reference architecture with seeded synthetic N(0,0.02) weights in
the reference's Q8_0_4X4 format; KV ~ N(0,1) fp16.  The KV working set (about 1.3 GB per GPU)
is far larger than L2, so no explicit L2 flush is needed between steps.

  value   K frames per stream on the device (mossgpu_step_frames, no host round trip per
          frame), CUDA events on the engine's stream, max over ranks.
  e2e     the same K frames as K calls of mossgpu_step through the C ABI with host buffers
          (control block H2D and codes/flags/gate D2H every frame), wall clock, max over ranks.
  roofline: the kernel class with the largest device time, timed live with CUDA events
          recorded between the kernels of the captured frame graph (a separate pass);
          `rooflines` gives the same figures for every class, `traffic` the DRAM bytes per
          launch of the committed ncu capture of that kernel (profiles/traffic.json).

--impl reference runs the reference's own CPU implementation (oracle/_ref, compiled from the
reference sources; the C port in oracle/ when that is absent) on a bounded sample of the
same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "dsh-moss-tts_b200"
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
METRIC = "LLM frames/sec (whole box)"


def load_package():
    if "moss_b200" in sys.modules:
        return sys.modules["moss_b200"]
    spec = importlib.util.spec_from_file_location("moss_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moss_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    if PEAKS.exists():
        d = json.loads(PEAKS.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {**FALLBACK_PEAKS, "source": "fallback"}


def q8x4_bytes(rows, cols):
    return rows // 4 * cols // 32 * 136


# ----------------------------------------------------------------------------- clocks

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.path = Path(tempfile.gettempdir()) / f"moss_clocks_{os.getpid()}.csv"
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(device)], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                "samples": len(rows), "reasons": reasons}


# ----------------------------------------------------------------------------- CPU legs

def cpu_frames_per_s(weights: str, lens: list[int], budget_s: float, max_frames: int, threads: int):
    """Time whole frames of the reference (oracle/_ref) or, failing that, of the C port on
    states with the given KV lengths.  Returns (frames/s, kind, threads, sample description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle_py
    rng = np.random.default_rng(7)
    use_ref = oracle_py.RefModel.available()
    frames = 0
    elapsed = 0.0
    per_stream = []
    for L in lens:
        k = rng.standard_normal((12, L, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
        v = rng.standard_normal((12, L, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
        h = rng.standard_normal(768, dtype=np.float32)
        if use_ref:
            m = oracle_py.RefModel(weights, threads=threads)
            fn = m.lib.ref_frames
        else:
            m = oracle_py.Oracle(weights, max_ctx=L + max_frames + 8)
            fn = m.lib.or_frames
            threads = 1
        fn.argtypes = [C.c_void_p, C.c_int, C.c_float, np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")]
        m.set_state(k, v, h)
        codes = np.zeros((1, 16), np.int32)
        fn(m.h, 1, 1.2, codes)  # warm-up frame (first touch of the weights)
        n = 0
        t0 = time.perf_counter()
        while n < max_frames and (n == 0 or time.perf_counter() - t0 < budget_s / len(lens)):
            fn(m.h, 1, 1.2, codes)
            n += 1
        dt = time.perf_counter() - t0
        frames += n
        elapsed += dt
        per_stream.append(n)
        m.close()
    kind = "reference" if use_ref else "port"
    sample = (f"{frames} frames ({'+'.join(map(str, per_stream))}) over {len(lens)} streams with KV lengths "
              f"{lens} drawn from the same U(64,1024) distribution, one frame = local decoder + 16 codes + "
              f"global step")
    return frames / elapsed, kind, threads, sample


def run_reference_arm(args, rank):
    if rank != 0:
        return
    pkg = load_package()
    from moss_b200 import mossfile
    weights = mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0)
    rng = np.random.default_rng(1234)
    lens = [int(x) for x in rng.integers(args.lmin, args.lmax + 1, 2)]
    threads = os.cpu_count() or 1
    # each step is one frame for each sampled stream; bound the run to a few minutes
    budget = min(120.0, 0.5 * (args.steps + args.warmup))
    fps, kind, cores, sample = cpu_frames_per_s(weights, lens, budget, max(2, args.steps), threads)
    line = {"impl": "reference", "metric": METRIC, "value": round(fps, 3), "unit": "frames/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * len(lens) / fps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": round(fps, 3), "unit": "frames/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": round(fps, 3), "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(args):
    return {"workload": f"configs[1]: {args.streams} ragged streams per GPU, full per-frame step "
                        f"(17-step local decoder + gate + 16 greedy codes + 12-layer global decode)",
            "streams_per_gpu": args.streams, "kv_len": [args.lmin, args.lmax], "page_tokens": 16,
            "model": "MOSS-TTS-Nano LLM (reference architecture, Q8_0_4X4 weights, synthetic)",
            "compute": "int8 weights x fp32 activations (W8A16 as the reference's MOSS_A16), fp32 accumulate, fp16 KV",
            "l2": "not flushed: KV working set per GPU >> 126 MB L2", "parallelism": f"dp{args.gpus} (streams sharded)"}


# ----------------------------------------------------------------------------- GPU arm

def run_ours(args, rank, world, local_rank, dist):
    import torch
    torch.cuda.set_device(local_rank)
    pkg = load_package()
    if rank == 0:
        pkg.build()
    if dist is not None:
        dist.barrier()
    from moss_b200 import mossfile
    weights = mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0)
    B, K, W = args.streams, args.steps, args.warmup
    prof_frames = min(K, 16)
    max_ctx = args.lmax + W + 2 * K + prof_frames + 64
    eng = pkg.Engine(weights, device=local_rank, max_streams=B + 1, max_ctx=max_ctx)
    eng.set_cuda_stream(torch.cuda.current_stream().cuda_stream)
    # one workload of B streams per GPU, KV lengths U{lmin..lmax}, sharded across the ranks
    # by total KV length (rank 0 decides, every rank gets B streams)
    import importlib
    sharding = importlib.import_module("moss_b200.sharding")
    all_lens = [int(x) for x in np.random.default_rng(1234).integers(args.lmin, args.lmax + 1, B * world)]
    lens = [all_lens[i] for i in sharding.agree_shards(dist, all_lens, per_rank=B)[rank]]
    sids = [eng.open() for _ in lens]

    def reset_states():
        # every measured phase starts from the same cached lengths (lmin..lmax), not from
        # where the previous phase left the streams
        for i, (s, L) in enumerate(zip(sids, lens)):
            eng.fill_state_random(s, L, seed=1000 * rank + i)
            eng.generate_begin(s, 0)
        torch.cuda.synchronize()

    reset_states()
    params = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)
    if args.profile_prefill:  # one warm-up batch, then one batch of N prompts x 256 rows (ncu)
        eng.close()
        run_prefill(pkg, weights, local_rank, torch, n_prompts=args.profile_prefill, rows=256)
        return
    if args.profile_frames:  # the short run the ncu captures use: one warm-up frame, then N
        eng.step_frames(sids, params, 1, want_codes=False)
        eng.step_frames(sids, params, args.profile_frames, want_codes=False)
        torch.cuda.synchronize()
        eng.close()
        return

    # warm-up: captures both the multi-frame and the single-frame graphs
    eng.step_frames(sids, params, W)
    eng.step(sids, params)
    torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        return sharding.max_over_ranks(dist, x, device="cuda")

    reset_states()
    clocks = Clocks(local_rank)
    # ---- value: K frames resident on the device
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _, done = eng.step_frames(sids, params, K, want_codes=False)
    e1.record()
    torch.cuda.synchronize()
    dev_ms = max_over_ranks(e0.elapsed_time(e1))
    launches = eng.last_launch_count()
    assert int(done.min()) == K, "a stream stopped during the timed region"
    # ---- e2e: K calls through the C ABI, host buffers in and out every frame
    reset_states()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(K):
        codes, stop, gate, _ = eng.step(sids, params)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    clk = clocks.stop()

    # ---- per-kernel device time (separate pass, events inside the frame graph)
    reset_states()
    eng.kernel_profile(True)
    base_pos = [eng.position(s) for s in sids]
    eng.step_frames(sids, params, prof_frames, want_codes=False)
    prof = eng.kernel_profile_read()
    eng.kernel_profile(False)

    # ---- batch-1 global step (configs[0] shape: L = 128 cached positions)
    s1 = eng.open()
    eng.fill_state_random(s1, 128, seed=99)
    x1 = np.random.default_rng(5).standard_normal((1, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
    for _ in range(5):
        eng.global_step_embed([s1], x1, want_hidden=False)
    eng.fill_state_random(s1, 128, seed=99)
    n1 = 50
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    for _ in range(n1):
        eng.global_step_embed([s1], x1, want_hidden=False)
    b1.record()
    torch.cuda.synchronize()
    b1_us = 1000 * b0.elapsed_time(b1) / n1
    b1_bytes = 12 * (q8x4_bytes(2304, 768) + q8x4_bytes(768, 768) + q8x4_bytes(3072, 768) + q8x4_bytes(768, 3072)) \
        + 485_376 + 36_864 * (128 + n1 // 2 + 1) + 36_864
    pk = peaks()

    # ---- prefill: 16 prompts x 256 rows (192 text + 64 voice-frame embeddings,
    # N(0,1) rounded to fp16) in one 4096-row pass through the 12 layers on the tensor cores,
    # writing the fp16 KV; embeddings are copied from host memory inside the timing
    for s_ in sids + [s1]:
        eng.close_stream(s_)
    pf = run_prefill(pkg, weights, local_rank, torch, n_prompts=16, rows=256)
    pf["frac_of_bf16_peak"] = round(pf["tflops"] / pk["bf16_tflops"], 4)

    # ---- rooflines.  Classes run on the tcgen05 GEMM (R > 8) or the CUDA-core GEMV (R <= 8);
    # algorithmic bytes = weights (Q8_0_4X4) + bias + activations in and out, FLOPs = 2 rows K R.
    R = B
    mean_ctx = float(np.mean(base_pos)) + prof_frames / 2.0 + 1.0  # attended positions per row
    act = 4  # bytes per input element: fp32 rows, or the tensor-core image's two fp16 parts
    gemm = {  # class -> (rows, K, output bytes per row)
        "qkv_global": (2304, 768, 768 * 4 + 1536 * 2), "proj_global": (768, 768, 768 * 8),
        "fc_in_global": (3072, 768, 3072 * 4), "fc_out_global": (768, 3072, 768 * 8),
        "qkv_local": (2304, 768, 768 * 4 + 1536 * 4), "proj_local": (768, 768, 768 * 8),
        "fc_in_local": (3072, 768, 3072 * 4), "fc_out_local": (768, 3072, 768 * 8),
        "audio_heads": (1024, 768, 1024 * 4),
    }
    algo = {k: q8x4_bytes(m, kk) + m * 4 + R * (kk * act + ob) for k, (m, kk, ob) in gemm.items()}
    flops = {k: 2.0 * m * kk * R for k, (m, kk, _) in gemm.items()}
    algo.update({
        "attn_decode_paged": R * mean_ctx * 12 * 64 * 2 * 2 + R * 768 * 8,
        "attn_combine": R * 12 * 8 * 68 * 4 + R * 768 * 4,
        "attn_local": R * 9 * 768 * 8 + R * 768 * 8,
        "build_activation_image": R * 768 * 4 + max(16, R) * 768 * 4,
        "sample_greedy": R * 1024 * 4 + R * 1024 * 2,
    })
    tf = Path(__file__).resolve().parent / "profiles" / "traffic.json"
    traffic_db = json.loads(tf.read_text()) if tf.exists() else {}  # dram bytes per launch, committed ncu captures
    rooflines = {}
    for k, (tot, nl) in prof.items():
        if nl and k in algo:
            us = 1000 * tot / nl
            r_ = {"avg_launch_us": round(us, 2), "achieved_gbs": round(algo[k] / (us / 1e6) / 1e9, 1),
                  "frac_of_hbm": round(algo[k] / (us / 1e6) / 1e9 / pk["hbm_gbs"], 4)}
            if k in flops:
                r_["achieved_tflops"] = round(flops[k] / (us / 1e6) / 1e12, 2)
            if k in traffic_db:
                r_["traffic"] = traffic_db[k]["dram_bytes_per_launch"]
            rooflines[k] = r_
    # the dominant kernel: the kernel function with the most device time in the profiled
    # frames; the weight-matrix roles all run one function (k_gemm_tc above 8 rows, else k_gemv)
    fn_of = {k: ("k_gemm_tc" if R > 8 else "k_gemv") for k in gemm}
    fns = {}
    for k, (tot, nl) in prof.items():
        if nl and k in algo:
            f = fn_of.get(k, k)
            e = fns.setdefault(f, [0.0, 0, 0.0, []])
            e[0] += tot
            e[1] += nl
            e[2] += algo[k] * nl
            e[3].append(k)
    name, (tot_ms, nl, bytes_all, classes) = max(fns.items(), key=lambda kv: kv[1][0])
    avg_ms = tot_ms / max(nl, 1)
    algo_launch = bytes_all / max(nl, 1)  # mean algorithmic bytes per launch of that function
    achieved = algo_launch / (avg_ms / 1e3) / 1e9
    traffic = traffic_db.get(name, {}).get("dram_bytes_per_launch")
    step_ms = dev_ms / K
    value = B * world * K / (dev_ms / 1e3)
    e2e = B * world * K / e2e_s
    h2d = eng_ctl_bytes(B)
    d2h = B * (16 * 4 + 4 + 8)
    breakdown = {k: {"ms_per_frame": round(v[0] / prof_frames, 4), "launches_per_frame": v[1] // prof_frames}
                 for k, v in sorted(prof.items(), key=lambda kv: -kv[1][0]) if v[1]}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_frames_per_s(weights, lens[:2], budget_s=20.0, max_frames=64, threads=os.cpu_count() or 1)
        cpu_baseline = {"value": round(cpu[0], 3), "unit": "frames/s", "cores": cpu[2], "kind": cpu[1], "sample": cpu[3]}
    else:
        cpu_baseline = None

    line = {"metric": METRIC, "value": round(value, 2), "unit": "frames/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,0.02) Q8_0_4X4 weights, N(0,1) fp16 KV)",
            "config": workload_config(args),
            "roofline": {"kernel": name, "classes": sorted(classes), "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": traffic, "algorithmic_bytes_per_launch": round(algo_launch),
                         "launches_per_frame": nl // prof_frames,
                         "avg_launch_us": round(1000 * avg_ms, 3), "peak_source": pk["source"]},
            "rooflines": rooflines,
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": round(e2e, 2), "unit": "frames/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "mossgpu_step (C ABI), one call per frame, host buffers"},
            "gpu_launches": launches,
            "clocks": clk,
            "prefill": pf,
            "batch1_global_step": {"us": round(b1_us, 2), "kv_len": 128, "algorithmic_bytes": b1_bytes,
                                   "achieved_gbs": round(b1_bytes / (b1_us / 1e6) / 1e9, 1),
                                   "frac_of_hbm": round(b1_bytes / (b1_us / 1e6) / 1e9 / pk["hbm_gbs"], 4)},
            "kernel_breakdown_ms_per_frame": breakdown}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()


# model FLOPs per prefilled row: 2 x the 84,934,656 weights of the 12 layers; causal attention
# adds 12 layers x 2 (scores, weighted sum) x 2 x 768 per attended position
PREFILL_FLOPS_PER_ROW = 2 * 12 * (2304 * 768 + 768 * 768 + 3072 * 768 + 768 * 3072)


def run_prefill(pkg, weights, device, torch, n_prompts: int, rows: int, warmup: int = 1) -> dict:
    """All prompts in one mossgpu_prefill_embeds_batch call: one pass of n_prompts x rows rows
    through the layers (an engine sized for it: max_rows = n_prompts x rows)."""
    eng = pkg.Engine(weights, device=device, max_streams=n_prompts, max_ctx=rows + 16, max_rows=n_prompts * rows)
    eng.set_cuda_stream(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(2024)
    # the embeddings live in pinned host memory, as a serving host keeps its staging buffers
    x = torch.empty((n_prompts * rows, 768), dtype=torch.float32, pin_memory=True).numpy()
    x[:] = rng.standard_normal((n_prompts * rows, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
    m = np.full(n_prompts, rows, np.int32)
    sids = [eng.open() for _ in range(n_prompts)]
    for _ in range(warmup):
        eng.prefill_embeds_batch(sids, x, m=m)
        for s in sids:
            eng.reset(s)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    eng.prefill_embeds_batch(sids, x, m=m)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    eng.close()
    attn = n_prompts * 12 * 2 * 2 * 768 * rows * (rows + 1) / 2
    flops = n_prompts * rows * PREFILL_FLOPS_PER_ROW + attn
    return {"prompts": n_prompts, "rows": rows, "ms": round(ms, 3), "gflop": round(flops / 1e9, 1),
            "tflops": round(flops / (ms / 1e3) / 1e12, 2), "rows_per_s": round(n_prompts * rows / (ms / 1e3), 1)}


def run_sweep(args, rank, world, local_rank, dist):
    """Long-form streaming: every stream generates `frames` frames from a
    starting KV length drawn from U{256..4096}, appending one position per frame.  Streams are
    sharded over the ranks by KV length; each GPU steps its streams in groups of <= 256 rows
    through mossgpu_step (C ABI, host buffers).  value = all frames of all streams / the
    slowest rank's wall time; p50 / p99 = per-call latency of one frame for one group."""
    import importlib
    import math
    import torch
    torch.cuda.set_device(local_rank)
    pkg = load_package()
    if rank == 0:
        pkg.build()
    if dist is not None:
        dist.barrier()
    from moss_b200 import mossfile
    sharding = importlib.import_module("moss_b200.sharding")
    weights = mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0)
    frames, n_all, warm = args.sweep_frames, args.sweep_streams, 2
    all_lens = [int(x) for x in np.random.default_rng(4096).integers(256, 4097, n_all)]
    mine = [all_lens[i] for i in sharding.agree_shards(dist, all_lens, per_rank=math.ceil(n_all / world))[rank]]
    pages = sum((L + frames + warm + kPAGE) // kPAGE + 1 for L in mine) + 16
    eng = pkg.Engine(weights, device=local_rank, max_streams=len(mine) + 1, max_ctx=4096 + frames + warm + 32,
                     kv_pages=pages)
    sids = [eng.open() for _ in mine]
    for i, (s, L) in enumerate(zip(sids, mine)):
        eng.fill_state_random(s, L, seed=7000 + 1000 * rank + i)
        eng.generate_begin(s, 0)
    groups = [sids[i:i + 256] for i in range(0, len(sids), 256)]
    params = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)
    for _ in range(warm):
        for g in groups:
            eng.step(g, params)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    lat = []
    t0 = time.perf_counter()
    for _ in range(frames):
        for g in groups:
            c0 = time.perf_counter()
            eng.step(g, params)  # returns after the frame's codes reached the host
            lat.append(time.perf_counter() - c0)
    wall = sharding.max_over_ranks(dist, time.perf_counter() - t0, device="cuda")
    p50 = sharding.max_over_ranks(dist, float(np.percentile(lat, 50)), device="cuda")
    p99 = sharding.max_over_ranks(dist, float(np.percentile(lat, 99)), device="cuda")
    kv_end = sum(L + warm + frames for L in all_lens) * 36_864
    line = {"metric": "long-form streaming frames/sec (whole box)", "value": round(n_all * frames / wall, 1),
            "unit": "frames/s", "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            "config": {"workload": "configs[4]: long-form sweep", "streams": n_all, "frames_per_stream": frames,
                       "start_kv_len": [256, 4096], "rows_per_step_call": 256, "streams_per_gpu": len(mine)},
            "p50_step_ms": round(1000 * p50, 3), "p99_step_ms": round(1000 * p99, 3),
            "wall_s": round(wall, 3), "kv_bytes_at_end": kv_end, "dtype": "f32", "data": "synthetic"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()


kPAGE = 16


def eng_ctl_bytes(B: int) -> int:
    """Bytes of the engine's per-call control block (engine.h off_* layout): slots, positions,
    frames, forced codes, page updates, FrameCtl (12 ints), active flags, frame counter."""
    r_max = max(B + 1, 256)
    return 4 * (22 * r_max + 1 + 12 + r_max + 4)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--streams", type=int, default=64)
    ap.add_argument("--lmin", type=int, default=64)
    ap.add_argument("--lmax", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE configs[4] instead: 512 streams from KV lengths U{256..4096}, 400 frames each, "
                         "sharded over the ranks; sustained frames/s and p50/p99 step latency")
    ap.add_argument("--sweep-frames", type=int, default=400)
    ap.add_argument("--sweep-streams", type=int, default=512)
    ap.add_argument("--profile-prefill", type=int, default=0,
                    help="prefill this many 256-row prompts after one warm-up prompt and exit (ncu captures)")
    ap.add_argument("--profile-frames", type=int, default=0,
                    help="run this many frames of the N=1 workload after one warm-up frame and exit "
                         "(the command the ncu captures under profiles/ use)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    try:
        if args.sweep:
            run_sweep(args, rank, world, local_rank, dist)
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
