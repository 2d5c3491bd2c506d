#!/usr/bin/env python
"""Benchmark: MOSS-TTS-Nano per-frame LLM step on B200, frames/s for the whole box.

Default workload (the long-form streaming sweep, strong scaling):
512 independent streams for the whole job with starting KV lengths drawn uniformly from
256..4096 (seeded), sharded over the N ranks by total KV length (512/N streams per GPU), paged
fp16 KV with 16-token pages.  One step = one audio frame for every stream: the 17-step local
decoder with the W8A8 end gate and 16 greedy codes (repetition penalty 1.2), then the 12-layer
global decode step that appends one KV position.  Weights: the reference architecture with
seeded synthetic N(0,0.02) weights in the reference's Q8_0_4X4 format; KV ~ N(0,1) fp16.  The
KV working set (~41 GB for the whole job) is far larger than L2, so no L2 flush is needed.
`--workload configs1` runs BASELINE configs[1] instead: 64 streams per GPU, KV U{64..1024}
(weak scaling).

  value   K frames of every stream on the device (one mossgpu_step_frames call: no host
          round trip per frame), CUDA events on the engine's stream, max over ranks.
  e2e     the same K frames as K calls of mossgpu_step through the C ABI with host buffers
          (control block H2D, codes/flags/gate D2H every frame), wall clock, max over ranks;
          p50/p99 of that per-frame call latency per GPU are gathered in `stats`.
  roofline: the kernel function with the largest device time in a separate profiled pass
          (CUDA events recorded between the kernels of the captured frame graph).  Event
          separation breaks the launch overlap and adds a gap to every launch; that gap is
          taken as one overhead per launch ((event time - frame time) / launches) and
          subtracted, so that launches x time adds up to the frame.
  stats   one all_gather of per-GPU frames, device time, e2e time and per-frame latency
          percentiles (the only collective besides the shard broadcast and the max).

--impl reference runs the reference's own CPU implementation (oracle/_ref, compiled from the
reference sources; the C port in oracle/ when that is absent) as K independent single-thread
processes on K physical cores, one stream each at the quantiles of the same KV distribution, on
rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib
import importlib.util
import json
import math
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
kPAGE = 16
POS_BYTES = 36_864  # fp16 K and V of one position, all 12 layers


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


# ----------------------------------------------------------------------------- workload

def workload(args, world):
    """(all stream lengths of the job, streams per rank, scaling)."""
    if args.workload == "configs4":
        lens = [int(x) for x in np.random.default_rng(4096).integers(args.lmin, args.lmax + 1, args.streams_total)]
        return lens, math.ceil(len(lens) / world), "strong"
    lens = [int(x) for x in np.random.default_rng(1234).integers(args.lmin, args.lmax + 1, args.streams * world)]
    return lens, args.streams, "weak"


def workload_config(args, world=1):
    if args.workload == "configs4":
        w = (f"configs[4]: {args.streams_total} streams for the whole box, start KV U{{{args.lmin}..{args.lmax}}}, "
             f"sharded over the GPUs (strong scaling); step = one full frame of every stream "
             f"(17-step local decoder + gate + 16 greedy codes + 12-layer global decode)")
        shape = {"streams_total": args.streams_total, "streams_per_gpu": math.ceil(args.streams_total / world)}
    else:
        w = (f"configs[1]: {args.streams} ragged streams per GPU, full per-frame step "
             f"(17-step local decoder + gate + 16 greedy codes + 12-layer global decode)")
        shape = {"streams_per_gpu": args.streams}
    return {"workload": w, **shape, "kv_len": [args.lmin, args.lmax], "page_tokens": kPAGE,
            "model": "MOSS-TTS-Nano LLM (reference architecture, Q8_0_4X4 weights, synthetic)",
            "compute": "int8 weights x fp32 activations (W8A16 as the reference's MOSS_A16), fp32 accumulate, fp16 KV",
            "l2": "not flushed: KV working set per GPU >> 126 MB L2", "parallelism": f"dp{world} (streams sharded)"}


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

def host_cpus() -> dict:
    """Physical cores this process may use (distinct (package, core) pairs among the CPUs of
    its affinity mask, capped by a cgroup CPU quota), logical CPUs and the CPU model."""
    affinity = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(os.cpu_count() or 1))
    model, pairs, cur = "", {}, {}
    try:
        for line in open("/proc/cpuinfo"):
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "processor":
                cur = {"cpu": int(v)}
            elif k == "model name":
                model = model or v
                cur["model"] = v
            elif k == "physical id":
                cur["pkg"] = v
            elif k == "core id":
                cur["core"] = v
                pairs[cur["cpu"]] = (cur.get("pkg"), v)
    except OSError:
        pass
    physical = len({pairs[c] for c in affinity if c in pairs}) or len(affinity)
    quota = None
    try:
        q, period = Path("/sys/fs/cgroup/cpu.max").read_text().split()[:2]
        if q != "max":
            quota = max(1, int(int(q) / int(period)))
    except (OSError, ValueError):
        pass
    usable = min(physical, quota) if quota else physical
    return {"physical_cores": usable, "logical_cpus": len(affinity), "cpu_model": model or "unknown",
            "cgroup_cpu_quota": quota}


def _cpu_stream_worker(job):
    """One single-thread reference process: one stream with a random fp16 N(0,1) KV state of
    length L, greedy frames with repetition penalty 1.2 (MOSS_A16=decode, the product mode)
    through the reference's own LlmModel::generate, for about budget_s seconds."""
    weights, L, budget_s, seed, threads = job
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle_py
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((12, L, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((12, L, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
    h = rng.standard_normal(768, dtype=np.float32)
    if oracle_py.RefModel.available():
        m, kind = oracle_py.RefModel(weights, threads=threads, a16_mode="decode"), "reference"
        run = lambda n: m.generate(n, greedy=True, rep=1.2, min_frames=1 << 30)  # noqa: E731
    else:
        m, kind = oracle_py.Oracle(weights, max_ctx=min(4608, L + 4096)), "port"
        sp = oracle_py.sample_params(greedy=True, rep=1.2, min_frames=1 << 30)
        run = lambda n: m.generate(n, sp)  # noqa: E731
    room = m.max_ctx - L - 2
    m.set_state(k, v, h)
    del k, v
    t0 = time.perf_counter()
    run(2)  # warm-up (first touch of the weights); also sizes the timed call
    per = (time.perf_counter() - t0) / 2
    n = int(max(2, min(room - 2, budget_s / max(per, 1e-4))))
    t0 = time.perf_counter()
    got = run(n)[0].shape[0]
    dt = time.perf_counter() - t0
    m.close()
    return got, dt, kind


def cpu_throughput(weights: str, lmin: int, lmax: int, budget_s: float, procs: int | None = None) -> dict:
    """The reference CPU engine's throughput mode: P independent single-thread processes on P
    physical cores, one stream each with KV lengths at the P quantiles of U{lmin..lmax}."""
    import multiprocessing as mp
    cpus = host_cpus()
    P = procs or max(1, min(cpus["physical_cores"], 32))
    lens = [int(round(lmin + (i + 0.5) / P * (lmax - lmin))) for i in range(P)]
    with mp.get_context("spawn").Pool(P) as pool:
        res = pool.map(_cpu_stream_worker, [(weights, L, budget_s, 7 + i, 1) for i, L in enumerate(lens)])
    fps = sum(f / dt for f, dt, _ in res)
    frames = sum(f for f, _, _ in res)
    kind = res[0][2]
    return {"value": round(fps, 3), "unit": "frames/s", "cores": P, "kind": kind,
            "sample": (f"{P} single-thread {'reference' if kind == 'reference' else 'C-port'} processes on {P} physical "
                       f"cores ({cpus['cpu_model']}; {cpus['logical_cpus']} logical CPUs usable), one stream each, "
                       f"KV lengths at the {P} quantiles of U{{{lmin}..{lmax}}} ({min(lens)}..{max(lens)}), "
                       f"{frames} greedy frames in ~{budget_s:.0f} s per process through LlmModel::generate, "
                       f"MOSS_A16=decode"),
            "host": cpus}


def _cpu_codec_worker(job):
    """One reference audio-decoder process (AudioDecoder::decode_chunk, decoder.cpp:211-225)
    on one stream: a 4-frame first chunk, then 8-frame chunks (engine.cpp:482-486) for about
    budget_s seconds."""
    path, budget_s, seed, threads = job
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle_py
    if oracle_py.REF_SO.exists():
        dec, kind = oracle_py.RefCodec(path, threads=threads), "reference"
    else:
        import codec_oracle
        dec, kind = codec_oracle.CodecOracle(path), "port"
    rng = np.random.default_rng(seed)
    dec.decode_chunk(rng.integers(0, 1024, (16, 4)).astype(np.int32))
    frames, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        dec.decode_chunk(rng.integers(0, 1024, (16, 8)).astype(np.int32))
        frames += 8
    return frames, time.perf_counter() - t0, kind


def cpu_codec_throughput(path: str, budget_s: float, procs: int | None = None) -> dict:
    """The reference codec decoder's throughput mode: P single-thread processes on P physical
    cores, one stream each."""
    import multiprocessing as mp
    cpus = host_cpus()
    P = procs or max(1, min(cpus["physical_cores"], 32))
    with mp.get_context("spawn").Pool(P) as pool:
        res = pool.map(_cpu_codec_worker, [(path, budget_s, 31 + i, 1) for i in range(P)])
    fps = sum(f / dt for f, dt, _ in res)
    kind = res[0][2]
    return {"value": round(fps, 3), "unit": "codec frames/s", "cores": P, "kind": kind,
            "sample": (f"{P} single-thread {'reference' if kind == 'reference' else 'numpy-port'} AudioDecoder "
                       f"processes on {P} physical cores ({cpus['cpu_model']}), one stream each: a 4-frame chunk, "
                       f"then 8-frame decode_chunk calls for ~{budget_s:.0f} s (rings filling from empty, so "
                       f"attention is shorter than in the GPU leg's full-ring steady state)")}


def run_codec(pkg, device, torch, n: int, K: int, peaks_: dict, chunk: int = 8, fill_chunks: int = 16,
              cpu_budget_s: float = 0.0) -> dict:
    """The audio codec decoder (mossgpu_codec_*) on n codec streams, one chunk of `chunk`
    frames per stream per call (the reference engine's chunk, engine.cpp:482-486).  The rings
    are filled first (16 chunks = 128 frames > the longest ring, 500 rows = 125 frames), so the
    timed calls run at the steady state of long-form streaming.  value: K calls with device
    codes and output, CUDA events; e2e: K calls of mossgpu_codec_decode_batch with host codes
    and host samples (the samples' D2H inside the timed region), wall clock."""
    from moss_b200 import codecfile
    path = codecfile.ensure_synth_decoder(Path(tempfile.gettempdir()) / "moss_b200_dec1.moss", 1)
    codec = pkg.Codec(path, device, max_streams=n, max_batch_frames=n * chunk)
    stream = torch.cuda.current_stream()
    codec.set_cuda_stream(stream.cuda_stream)
    sids = [codec.open() for _ in range(n)]
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    codes = torch.randint(0, 1024, (fill_chunks + 2 * K + 2, n, 16, chunk), dtype=torch.int32, device="cuda",
                          generator=g)
    out = torch.empty((n, chunk * codec.samples_per_frame), dtype=torch.float32, device="cuda")
    for i in range(fill_chunks):
        codec.decode_batch_device(sids, codes[i].data_ptr(), chunk, out.data_ptr())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        codec.decode_batch_device(sids, codes[fill_chunks + i].data_ptr(), chunk, out.data_ptr())
    e1.record(stream)
    e1.synchronize()
    dev_ms = e0.elapsed_time(e1) / K
    # per-class device time of one more call (events between launches; one gap per launch removed)
    codec.profile(True)
    codec.decode_batch_device(sids, codes[fill_chunks + K].data_ptr(), chunk, out.data_ptr())
    prof = codec.profile_read()
    codec.profile(False)
    nl_all = sum(v[1] for v in prof.values())
    gap = max(0.0, (sum(v[0] for v in prof.values()) - dev_ms) / max(nl_all, 1))
    # e2e through the host entry point
    hcodes = codes[fill_chunks + K + 1:fill_chunks + 2 * K + 1].cpu().numpy()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(K):
        pcm = codec.decode_batch(sids, hcodes[i])
    e2e_s = (time.perf_counter() - t0) / K
    assert pcm.shape == (n, chunk * codec.samples_per_frame) and np.isfinite(pcm[:, :64]).all()
    launches = codec.launches_per_call()
    codec.close()
    frames = n * chunk
    # algorithmic FLOPs per call: the GEMMs, and the attention at full rings
    rows_f, gemm_macs, attn_macs = 1, 512 * 1024, 0
    cin = 1024
    for s, (p, L, ctx, cout) in enumerate(((4, 4, 500, 512), (2, 2, 800, 512), (2, 2, 1200, 512), (2, 4, 1600, 240))):
        rows_f *= p
        gemm_macs += rows_f * (256 * cin // p + L * (768 * 256 + 256 * 256 + 2 * 1024 * 256) + cout * 256)
        attn_macs += rows_f * L * 4 * ctx * 64 * 2
        cin = cout
    flops = {"k_gemm_mma": 2.0 * gemm_macs * frames, "k_window_attn": 2.0 * attn_macs * frames}
    classes = {}
    for k, (ms, nl) in prof.items():
        if nl:
            t = max(ms - gap * nl, 0.05 * ms)
            classes[k] = {"ms_per_call": round(t, 4), "launches": nl, "share": round(t / dev_ms, 4)}
            if k in flops:
                classes[k]["achieved_tflops"] = round(flops[k] / (t / 1e3) / 1e12, 2)
    top = max((k for k in classes if k in flops), key=lambda k: classes[k]["ms_per_call"])
    r = {"api": "mossgpu_codec_decode_batch_device (value) / mossgpu_codec_decode_batch (e2e)",
         "streams": n, "chunk_frames": chunk, "ms_per_call": round(dev_ms, 3),
         "value": round(frames / (dev_ms / 1e3), 1), "unit": "codec frames/s",
         "e2e": {"value": round(frames / e2e_s, 1), "unit": "codec frames/s", "ms_per_call": round(1e3 * e2e_s, 3),
                 "h2d_bytes_per_step": int(n * 16 * chunk * 4),
                 "d2h_bytes_per_step": int(n * chunk * codec.samples_per_frame * 4)},
         "audio_seconds_per_s": round(frames * 0.08 / (dev_ms / 1e3), 1),
         "gpu_launches_per_call": launches,
         "gflop_per_call": round(sum(flops.values()) / 1e9, 1),
         "roofline": {"kernel": top, "bound": "tensor", "achieved": classes[top]["achieved_tflops"],
                      "peak": peaks_["bf16_tflops"], "unit": "TFLOP/s",
                      "frac": round(classes[top]["achieved_tflops"] / peaks_["bf16_tflops"], 4),
                      "tensor_products_per_flop": 2 if top == "k_gemm_mma" else 3,
                      "note": ("algorithmic FLOPs; each product runs as 2 (GEMM: W.x_hi + W.x_lo) or 3 "
                               "(attention: hi/lo of both operands) fp16 tensor products"),
                      "peak_source": peaks_["source"]},
         "kernels": classes, "profile_gap_us": round(1000 * gap, 2)}
    if cpu_budget_s > 0:
        r["cpu_baseline"] = cpu_codec_throughput(path, cpu_budget_s)
    return r


def cpu_single_stream(weights: str, L: int, budget_s: float) -> dict:
    """One stream, one process, all logical CPUs as the reference's --threads (single-stream mode)."""
    import multiprocessing as mp
    cpus = host_cpus()
    T = cpus["logical_cpus"]
    with mp.get_context("spawn").Pool(1) as pool:
        f, dt, kind = pool.map(_cpu_stream_worker, [(weights, L, budget_s, 99, T)])[0]
    return {"frames_per_s": round(f / dt, 3), "ms_per_frame": round(1000 * dt / f, 2), "threads": T, "kv_len": L,
            "kind": kind}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    load_package()
    from moss_b200 import mossfile
    weights = str(mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0))
    budget = min(60.0, max(10.0, 0.6 * (args.steps + args.warmup)))
    cb = cpu_throughput(weights, args.lmin, args.lmax, budget)
    single = cpu_single_stream(weights, (args.lmin + args.lmax) // 2, min(budget, 15.0))
    lens, per_rank, scaling = workload(args, world)
    n_streams = len(lens)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * n_streams / cb["value"], 3),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "cpu_host": cb["host"], "single_stream_all_threads": single,
            "e2e": {"value": cb["value"], "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm

SL_ATTN_PHASES = ["issue pre-wait copies", "dependency wait", "x in + LN1", "QKV + RoPE, pushed to the head's CTAs",
                  "cluster barrier 1", "attention + CTA merge, pushed", "cluster barrier 2",
                  "merge of the pushed partials", "proj + accumulator adds + KV append", "exit"]
SL_MLP_PHASES = ["issue pre-wait copies", "dependency wait", "x in + LN2", "fc_in + GELU",
                 "fc_out partials, pushed", "cluster barrier", "sum of the pushed partials", "accumulator adds",
                 "exit"]


def phase_stats(st, step_us) -> dict:
    """Per-phase medians (µs) of the small-layer phase stamps st[steps][24 launches][96 CTAs][12]
    (ns; launch p = 2 layer + {0: attention half, 1: MLP half}; stamp 2 = the dependency wait
    returned, the last stamp = the CTA's end).  after_wait: from a launch's median wait return
    to its last CTA's end; handoff: from a launch's last CTA end to the next launch's median
    wait return; layers_us: from the first launch's first CTA start to the last launch's end."""
    st = np.asarray(st, dtype=np.int64)
    out = {"steps": int(st.shape[0]), "step_us_events": round(float(np.median(step_us)), 2)}
    last = {0: len(SL_ATTN_PHASES), 1: len(SL_MLP_PHASES)}
    for half, names in ((0, SL_ATTN_PHASES), (1, SL_MLP_PHASES)):
        key = "attn" if half == 0 else "mlp"
        ph = st[:, half::2]  # [steps][12][96][12]
        d = np.diff(ph[..., : last[half] + 1], axis=-1) / 1000.0
        out[key] = {n: round(float(np.median(d[..., i])), 3) for i, n in enumerate(names)}
        span = (ph[..., last[half]].max(axis=-1) - np.median(ph[..., 2], axis=-1)) / 1000.0
        out[key + "_after_wait_us"] = round(float(np.median(span)), 3)
    nl = st.shape[1]
    ends = np.where(np.arange(nl)[None, :, None] % 2 == 0, st[..., last[0]], st[..., last[1]]).max(axis=-1)
    release = np.median(st[..., 2], axis=-1)
    out["handoff_us"] = round(float(np.median((release[:, 1:] - ends[:, :-1]) / 1000.0)), 3)
    out["layers_us"] = round(float(np.median((ends[:, -1] - st[:, 0, :, 0].min(axis=-1)) / 1000.0)), 2)
    return out


def run_phase_stamps(steps: int, stamps: bool = True):
    """Batch-1 global step (one stream, 128 cached positions) on the library built with phase
    stamps: thread 0 of every CTA of the 24 small-layer launches stamps %globaltimer at each
    phase boundary.  Per phase: the median over CTAs, launches and steps; per launch: the
    hand-off (the predecessor's last CTA ends -> this launch's median CTA leaves its wait)."""
    import torch
    if stamps:
        os.environ["MOSSGPU_LIB_VARIANT"] = "stamps"
    pkg = load_package()
    pkg.build()
    from moss_b200 import mossfile
    weights = str(mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0))
    eng = pkg.Engine(weights, device=0, max_streams=2, max_ctx=128 + steps + 64)
    s1 = eng.open()
    x1 = np.random.default_rng(5).standard_normal((1, 768), dtype=np.float32).astype(np.float16).astype(np.float32)
    eng.fill_state_random(s1, 128, seed=99)
    for _ in range(5):
        eng.global_step_embed([s1], x1, want_hidden=False)
    eng.fill_state_random(s1, 128, seed=99)
    st, step_us = [], []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        eng.global_step_embed([s1], x1, want_hidden=False)
        b.record()
        torch.cuda.synchronize()
        step_us.append(1000 * a.elapsed_time(b))
        if stamps:
            st.append(eng.small_layer_stamps().astype(np.int64))
    eng.close()
    if not stamps:
        return
    out = {"workload": "configs[0] batch-1 global step, 128 cached positions", **phase_stats(np.stack(st), step_us)}
    print(json.dumps(out), flush=True)


def kernel_classes(R: int):
    """Algorithmic bytes and FLOPs per launch of each kernel class at R batch rows."""
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
    return gemm, algo, flops


def run_ours(args, rank, world, local_rank, dist):
    import torch
    torch.cuda.set_device(local_rank)
    pkg = load_package()
    if rank == 0:
        pkg.build()
    if dist is not None:
        dist.barrier()
    from moss_b200 import mossfile
    sharding = importlib.import_module("moss_b200.sharding")
    weights = str(mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0))
    K, W = args.steps, args.warmup
    prof_frames = min(K, 16)
    all_lens, per_rank, scaling = workload(args, world)
    lens = [all_lens[i] for i in sharding.agree_shards(dist, all_lens, per_rank=per_rank)[rank]]
    B = len(lens)
    extra = max(W + 1, K, prof_frames) + 2  # positions a phase appends before the next reset
    b1_extra = 128 + 64
    pages = sum((L + extra + kPAGE - 1) // kPAGE + 1 for L in lens) + (b1_extra + kPAGE - 1) // kPAGE + 16
    eng = pkg.Engine(weights, device=local_rank, max_streams=B + 2, max_ctx=max(lens) + extra + 32, kv_pages=pages,
                     max_rows=max(B + 2, 256))
    eng.set_cuda_stream(torch.cuda.current_stream().cuda_stream)
    if args.tc_direct_min is not None:
        eng.set_tc_policy(args.tc_direct_min, args.tc_direct_rows)
    if args.local_path is not None:
        eng.set_local_path(args.local_path)
    sids = [eng.open() for _ in lens]

    def reset_states():
        # every measured phase starts from the same cached lengths, not from where the
        # previous phase left the streams
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
    my_dev_ms = e0.elapsed_time(e1)
    dev_ms = max_over_ranks(my_dev_ms)
    launches = eng.last_launch_count()
    assert int(done.min()) == K, "a stream stopped during the timed region"
    # ---- e2e: K calls through the C ABI, host buffers in and out every frame
    reset_states()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    lat = []
    t0 = time.perf_counter()
    for _ in range(K):
        c0 = time.perf_counter()
        eng.step(sids, params)  # returns after the frame's codes reached the host
        lat.append(time.perf_counter() - c0)
    torch.cuda.synchronize()
    my_e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(my_e2e_s)
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
    # one step at a time with L2 flushed before each (the 96 MB of weights would otherwise stay
    # in the 126 MB L2): the call's latency through the C ABI, CUDA events around the call (host
    # copies, the launched step and the host sync included)
    n1 = 30
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    api_us = []
    eng.fill_state_random(s1, 128, seed=99)
    for _ in range(n1):
        flush.fill_(1)
        b0.record()
        eng.global_step_embed([s1], x1, want_hidden=False)
        b1.record()
        torch.cuda.synchronize()
        api_us.append(1000 * b0.elapsed_time(b1))
    del flush
    b1_us = float(np.median(api_us))
    b1_bytes = 12 * (q8x4_bytes(2304, 768) + q8x4_bytes(768, 768) + q8x4_bytes(3072, 768) + q8x4_bytes(768, 3072)) \
        + 485_376 + POS_BYTES * (128 + n1 // 2 + 1) + POS_BYTES
    pk = peaks()
    h2d = eng_ctl_bytes(B)
    d2h = B * (16 * 4 + 4 + 8)
    eng.close()

    # ---- configs[1] frame (64 streams per GPU, KV U{64..1024}) and configs[2] prefill:
    # reported beside the headline, each in an engine of its own
    c1 = pf = codec = pipe = None
    if not args.frame_only:
        c1 = run_configs1_frame(pkg, weights, local_rank, torch, rank, K, W, args.local_path) \
            if args.workload == "configs4" else None
        pf = run_prefill(pkg, weights, local_rank, torch, n_prompts=16, rows=256)
        pf["frac_of_bf16_peak"] = round(pf["tflops"] / pk["bf16_tflops"], 4)
        # ---- the audio codec decoder on this rank's streams (8-frame chunks, full rings), then
        # the LLM and the codec together on this GPU (per-GPU figures: rank 0's streams)
        codec = run_codec(pkg, local_rank, torch, B, min(K, 8), pk,
                          cpu_budget_s=10.0 if (rank == 0 and world == 1 and not args.no_cpu_baseline) else 0.0)
        pipe = run_pipeline(pkg, weights, local_rank, torch, lens, K=max(2, min(K // 8, 4)), overlap=False)
        codec["scope"] = pipe["scope"] = "one GPU (rank 0's streams)"

    # ---- rooflines
    R = B
    step_ms = dev_ms / K
    mean_ctx = float(np.mean(base_pos)) + prof_frames / 2.0 + 1.0  # attended positions per row
    gemm, algo, flops = kernel_classes(R)
    algo.update({
        "attn_decode_paged": R * mean_ctx * 12 * 64 * 2 * 2 + R * 768 * 8,
        "attn_combine": R * 12 * 8 * 68 * 4 + R * 768 * 4,
        "attn_local": R * 9 * 768 * 8 + R * 768 * 8,
        "build_activation_image": R * 768 * 4 + max(16, R) * 768 * 4,
        "sample_greedy": R * 1024 * 4 + R * 1024 * 2,
    })
    tf = ROOT / "profiles" / "traffic.json"
    traffic_db = json.loads(tf.read_text()) if tf.exists() else {}  # dram bytes per launch, committed captures
    # Event-separated class times each carry the launch gap that the graph overlaps.  Take
    # that gap as one overhead per launch: delta = (event time - frame time) / launches, and
    # each launch's time = its event time - delta, so that launches x time add up to the frame.
    event_ms_per_frame = sum(tot for tot, nl in prof.values() if nl) / prof_frames
    launches_per_frame = sum(nl for _, nl in prof.values()) / prof_frames
    delta_ms = max(0.0, (event_ms_per_frame - step_ms) / max(launches_per_frame, 1))

    def launch_ms(tot, nl):  # apportioned mean time of one launch of a class
        return max(tot / nl - delta_ms, 0.05 * tot / nl)

    rooflines = {}
    for k, (tot, nl) in prof.items():
        if nl and k in algo:
            us = 1000 * launch_ms(tot, nl)
            r_ = {"avg_launch_us": round(us, 2), "achieved_gbs": round(algo[k] / (us / 1e6) / 1e9, 1),
                  "frac_of_hbm": round(algo[k] / (us / 1e6) / 1e9 / pk["hbm_gbs"], 4)}
            if k in flops:
                r_["achieved_tflops"] = round(flops[k] / (us / 1e6) / 1e12, 2)
            rooflines[k] = r_
    direct = args.tc_direct_min if args.tc_direct_min is not None else 256  # the engine's default
    # from `direct` rows on, launch_tc picks the form per matrix (k_gemm_tp tiles or k_gemm_tc
    # split-K): the GEMM classes are then reported as one function name covering both
    gemm_fn = "k_gemm_tp|k_gemm_tc" if (direct > 0 and R >= direct) else ("k_gemm_tc" if R > 8 else "k_gemv")
    attn_fn = "k_attn_decode" if R > 96 else "k_attn_rows"
    fn_of = {**{k: gemm_fn for k in gemm}, "attn_decode_paged": attn_fn}
    fns = {}
    for k, (tot, nl) in prof.items():
        if nl and k in algo:
            e = fns.setdefault(fn_of.get(k, k), [0.0, 0, 0.0, []])
            e[0] += tot
            e[1] += nl
            e[2] += algo[k] * nl
            e[3].append(k)
    name, (tot_ms, nl, bytes_all, classes) = max(fns.items(), key=lambda kv: kv[1][0])
    avg_ms = launch_ms(tot_ms, max(nl, 1))
    algo_launch = bytes_all / max(nl, 1)  # mean algorithmic bytes per launch of that function
    achieved = algo_launch / (avg_ms / 1e3) / 1e9
    tentry = traffic_db.get(f"{name}@{args.workload}", {})  # committed ncu capture of that kernel
    traffic = tentry.get("dram_bytes_per_launch")
    if traffic is None and "dram_per_algorithmic_byte" in tentry:  # captured on a smaller case, scaled by units
        traffic = round(tentry["dram_per_algorithmic_byte"] * algo_launch)
    value = len(all_lens) * K / (dev_ms / 1e3)
    e2e = len(all_lens) * K / e2e_s
    breakdown = {k: {"ms_per_frame": round(launch_ms(v[0], v[1]) * v[1] / prof_frames, 4),
                     "launches_per_frame": v[1] // prof_frames}
                 for k, v in sorted(prof.items(), key=lambda kv: -kv[1][0]) if v[1]}

    # ---- stats gather: per-GPU frames, device ms, e2e s, per-frame call latency p50/p99 (ms)
    mine = [float(B * K), my_dev_ms, my_e2e_s, 1000 * float(np.percentile(lat, 50)),
            1000 * float(np.percentile(lat, 99)), float(sum(lens))]
    per_gpu = gather_stats(dist, mine)
    stats = {"per_gpu": [{"rank": i, "streams": int(g[0] // K), "frames": int(g[0]), "device_ms": round(g[1], 3),
                          "e2e_s": round(g[2], 4), "p50_frame_ms": round(g[3], 3), "p99_frame_ms": round(g[4], 3),
                          "kv_positions": int(g[5])} for i, g in enumerate(per_gpu)],
             "device_ms_max_over_min": round(max(g[1] for g in per_gpu) / min(g[1] for g in per_gpu), 4),
             "p50_frame_ms": round(max(g[3] for g in per_gpu), 3), "p99_frame_ms": round(max(g[4] for g in per_gpu), 3)}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_throughput(weights, args.lmin, args.lmax, budget_s=15.0)
        cpu_baseline = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        if codec and codec.get("cpu_baseline"):
            # the reference's LLM and codec each measured on all the cores; run together they
            # share them, so the pipeline's rate is the harmonic combination of the two
            lv, cv = cb["value"], codec["cpu_baseline"]["value"]
            pipe["cpu_reference_frames_per_s"] = round(1.0 / (1.0 / lv + 1.0 / cv), 2)
            pipe["cpu_reference_note"] = ("1 / (1 / LLM + 1 / codec) of the two measured reference arms on the same "
                                          f"{cb['cores']} cores ({lv} and {cv} frames/s)")
    else:
        cpu_baseline = None

    line = {"metric": METRIC, "value": round(value, 2), "unit": "frames/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,0.02) Q8_0_4X4 weights, N(0,1) fp16 KV)",
            "config": workload_config(args, world),
            "roofline": {"kernel": name, "classes": sorted(classes), "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": traffic, "algorithmic_bytes_per_launch": round(algo_launch),
                         "launches_per_frame": nl // prof_frames, "avg_launch_us": round(1000 * avg_ms, 3),
                         "avg_launch_us_event_separated": round(1000 * tot_ms / max(nl, 1), 3),
                         "launch_overhead_us": round(1000 * delta_ms, 3), "peak_source": pk["source"]},
            "rooflines": rooflines,
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": round(e2e, 2), "unit": "frames/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "mossgpu_step (C ABI), one call per frame for all of a GPU's streams, host buffers"},
            "gpu_launches": launches,
            "clocks": clk,
            "stats": stats,
            "configs1_frame": c1,
            "prefill": pf,
            "codec": codec,
            "pipeline": pipe,
            "batch1_global_step": {"us": round(b1_us, 2), "kv_len": 128, "algorithmic_bytes": b1_bytes,
                                   "l2": "flushed before every step",
                                   "achieved_gbs": round(b1_bytes / (b1_us / 1e6) / 1e9, 1),
                                   "frac_of_hbm": round(b1_bytes / (b1_us / 1e6) / 1e9 / pk["hbm_gbs"], 4),
                                   "path": "two-launch layers (layer_small.cuh); one C-ABI call with host copies "
                                           "and sync per step (profiles/small_layers_b1.md: 131 us of it on the "
                                           "device)"},
            "kernel_breakdown_ms_per_frame": breakdown}
    if rank == 0:
        print(json.dumps(line), flush=True)


def gather_stats(dist, values: list[float]) -> list[list[float]]:
    """One all_gather of a small float vector per rank (the end-of-run stats gather)."""
    if dist is None or not dist.is_initialized():
        return [list(values)]
    import torch
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.cpu().tolist() for o in out]


def run_configs1_frame(pkg, weights, device, torch, rank, K, W, local_path=None) -> dict:
    """configs[1] on this GPU: 64 streams, KV U{64..1024}, K frames on the device."""
    lens = [int(x) for x in np.random.default_rng(1234 + rank).integers(64, 1025, 64)]
    eng = pkg.Engine(weights, device=device, max_streams=65, max_ctx=1024 + W + K + 32)
    eng.set_cuda_stream(torch.cuda.current_stream().cuda_stream)
    if local_path is not None:
        eng.set_local_path(local_path)
    sids = [eng.open() for _ in lens]
    p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)

    def reset():
        for i, (s, L) in enumerate(zip(sids, lens)):
            eng.fill_state_random(s, L, seed=i)
            eng.generate_begin(s, 0)

    reset()
    eng.step_frames(sids, p, W, want_codes=False)
    reset()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    eng.step_frames(sids, p, K, want_codes=False)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    eng.close()
    return {"streams": 64, "kv_len": [64, 1024], "ms_per_frame": round(ms, 4), "frames_per_s_per_gpu": round(64 / ms * 1e3, 1)}


def run_pipeline(pkg, weights, device, torch, lens, K: int, chunk: int = 8, fill_chunks: int = 16,
                 overlap: bool = False) -> dict:
    """The LLM and the codec decoder on one GPU, as a serving loop runs them: per chunk, one
    mossgpu_step_frames call of `chunk` frames for every stream (codes to the host), and one
    mossgpu_codec_decode_batch_device call that turns every stream's block into samples (codes
    back to the device, samples kept there).  overlap: the codec runs on a second CUDA stream,
    so chunk k's decode overlaps chunk k+1's LLM frames (the host enqueues the decode, then
    steps the LLM); otherwise both run in turn on one stream.  The codec streams' rings are
    filled first, so the codec runs at its long-form steady state; the LLM streams start at the
    workload's KV lengths.  Timed: K chunks, wall clock around the host loop until both
    streams are idle."""
    from moss_b200 import codecfile
    dec = codecfile.ensure_synth_decoder(Path(tempfile.gettempdir()) / "moss_b200_dec1.moss", 1)
    B = len(lens)
    extra = (K + 2) * chunk + 32
    pages = sum((L + extra + kPAGE - 1) // kPAGE + 1 for L in lens) + 16
    eng = pkg.Engine(weights, device=device, max_streams=B + 2, max_ctx=max(lens) + extra, kv_pages=pages,
                     max_rows=max(B + 2, 256))
    codec = pkg.Codec(dec, device, max_streams=B, max_batch_frames=B * chunk)
    stream = torch.cuda.current_stream()
    cstream = torch.cuda.Stream() if overlap else stream
    eng.set_cuda_stream(stream.cuda_stream)
    codec.set_cuda_stream(cstream.cuda_stream)
    sids = [eng.open() for _ in lens]
    csids = [codec.open() for _ in lens]
    for i, (s, L) in enumerate(zip(sids, lens)):
        eng.fill_state_random(s, L, seed=i)
        eng.generate_begin(s, 0)
    p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    warm = torch.randint(0, 1024, (B, 16, chunk), dtype=torch.int32, device="cuda", generator=g)
    pcm = torch.empty((B, chunk * codec.samples_per_frame), dtype=torch.float32, device="cuda")
    for _ in range(fill_chunks):
        codec.decode_batch_device(csids, warm.data_ptr(), chunk, pcm.data_ptr())
    # two code buffers: chunk k's block is read by the decode on the codec's stream, chunk k+1's
    # is written after it in the same stream's order
    codes_dev = [torch.empty((B, 16, chunk), dtype=torch.int32, device="cuda") for _ in range(2)]

    def llm_chunk(k):  # frames of chunk k -> codes_dev[k % 2] (on the codec's stream)
        codes, done = eng.step_frames(sids, p, chunk)  # [chunk][B][16], host; syncs the LLM stream
        assert (done == chunk).all()
        with torch.cuda.stream(cstream):
            codes_dev[k % 2].copy_(torch.from_numpy(np.ascontiguousarray(codes.transpose(1, 2, 0))))

    def codec_chunk(k):  # enqueued only: runs on the codec's stream
        codec.decode_batch_device(csids, codes_dev[k % 2].data_ptr(), chunk, pcm.data_ptr())

    llm_chunk(0)  # warm-up: graphs captured, caches hot
    codec_chunk(0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    llm_chunk(1)
    for k in range(1, K + 1):
        codec_chunk(k)  # chunk k's samples ...
        if k < K:
            llm_chunk(k + 1)  # ... while chunk k+1's frames run on the LLM's stream
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    assert codec.status() == 0
    eng.close()
    codec.close()
    frames = B * chunk * K
    return {"api": "mossgpu_step_frames (LLM, codes to the host) + mossgpu_codec_decode_batch_device (codec)",
            "streams": B, "chunk_frames": chunk, "chunks": K, "overlap": overlap,
            "frames_per_s": round(frames / wall, 1), "audio_seconds_per_s": round(frames * 0.08 / wall, 1),
            "ms_per_chunk": round(1e3 * wall / K, 3)}


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
    """Long-form streaming sustained over the whole 400 frames: every
    stream generates `frames` frames from its starting KV length, appending one position per
    frame.  Streams are sharded over the ranks by KV length; each GPU steps all its streams in
    one mossgpu_step call per frame (C ABI, host buffers).  value = all frames of all streams /
    the slowest rank's wall time; p50 / p99 = per-call latency of one frame of a GPU's streams."""
    import torch
    torch.cuda.set_device(local_rank)
    pkg = load_package()
    if rank == 0:
        pkg.build()
    if dist is not None:
        dist.barrier()
    from moss_b200 import mossfile
    sharding = importlib.import_module("moss_b200.sharding")
    weights = str(mossfile.ensure_synth_weights(Path(tempfile.gettempdir()) / "moss_b200_w0.moss", 0))
    frames, n_all, warm = args.sweep_frames, args.streams_total, 2
    all_lens = [int(x) for x in np.random.default_rng(4096).integers(args.lmin, args.lmax + 1, n_all)]
    mine = [all_lens[i] for i in sharding.agree_shards(dist, all_lens, per_rank=math.ceil(n_all / world))[rank]]
    pages = sum((L + frames + warm + kPAGE) // kPAGE + 1 for L in mine) + 16
    eng = pkg.Engine(weights, device=local_rank, max_streams=len(mine) + 1, max_ctx=args.lmax + frames + warm + 32,
                     kv_pages=pages, max_rows=max(len(mine) + 1, 256))
    if args.tc_direct_min is not None:
        eng.set_tc_policy(args.tc_direct_min, args.tc_direct_rows)
    sids = [eng.open() for _ in mine]
    for i, (s, L) in enumerate(zip(sids, mine)):
        eng.fill_state_random(s, L, seed=7000 + 1000 * rank + i)
        eng.generate_begin(s, 0)
    params = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)
    for _ in range(warm):
        eng.step(sids, params)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    lat = []
    t0 = time.perf_counter()
    for _ in range(frames):
        c0 = time.perf_counter()
        eng.step(sids, params)  # returns after the frame's codes reached the host
        lat.append(time.perf_counter() - c0)
    my_wall = time.perf_counter() - t0
    wall = sharding.max_over_ranks(dist, my_wall, device="cuda")
    per_gpu = gather_stats(dist, [float(len(mine) * frames), my_wall, 1000 * float(np.percentile(lat, 50)),
                                  1000 * float(np.percentile(lat, 99))])
    kv_end = sum(L + warm + frames for L in all_lens) * POS_BYTES
    line = {"metric": "long-form streaming frames/sec (whole box)", "value": round(n_all * frames / wall, 1),
            "unit": "frames/s", "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            "config": {"workload": "configs[4]: long-form sweep", "streams": n_all, "frames_per_stream": frames,
                       "start_kv_len": [args.lmin, args.lmax], "streams_per_gpu": len(mine)},
            "p50_step_ms": round(max(g[2] for g in per_gpu), 3), "p99_step_ms": round(max(g[3] for g in per_gpu), 3),
            "per_gpu": [{"rank": i, "frames": int(g[0]), "wall_s": round(g[1], 3), "p50_ms": round(g[2], 3),
                         "p99_ms": round(g[3], 3)} for i, g in enumerate(per_gpu)],
            "wall_s": round(wall, 3), "kv_bytes_at_end": kv_end, "dtype": "f32", "data": "synthetic"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()


def eng_ctl_bytes(B: int) -> int:
    """Bytes of the engine's per-call control block (engine.h off_* layout): slots, positions,
    frames, forced codes, page updates, FrameCtl (12 ints), active flags, frame counter."""
    r_max = max(B + 2, 256)
    return 4 * (22 * r_max + 1 + 12 + r_max + 4)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["configs4", "configs1"], default="configs4",
                    help="configs4 (default): 512 streams for the whole box, KV U{256..4096}, strong scaling; "
                         "configs1: 64 streams per GPU, KV U{64..1024}, weak scaling")
    ap.add_argument("--streams-total", type=int, default=512, help="configs4: streams of the whole job")
    ap.add_argument("--streams", type=int, default=64, help="configs1: streams per GPU")
    ap.add_argument("--lmin", type=int, default=None)
    ap.add_argument("--lmax", type=int, default=None)
    ap.add_argument("--tc-direct-min", type=int, default=None,
                    help="batch rows from which the GEMMs use the direct tile form (mossgpu_set_tc_policy)")
    ap.add_argument("--tc-direct-rows", type=int, default=0,
                    help="batch rows per tile of the direct form (mossgpu_set_tc_policy; 0 = by batch size)")
    ap.add_argument("--local-path", type=int, default=None,
                    help="local decoder: 0 = fused cluster kernel for greedy frames, 1 = per-step kernels "
                         "(mossgpu_set_local_path; default: the engine's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--frame-only", action="store_true",
                    help="the headline frame only: skip the configs1, prefill, codec and pipeline legs (sweeps)")
    ap.add_argument("--sweep", action="store_true",
                    help="configs[4] sustained: every stream runs --sweep-frames frames (400), per-frame latency")
    ap.add_argument("--sweep-frames", type=int, default=400)
    ap.add_argument("--profile-prefill", type=int, default=0,
                    help="prefill this many 256-row prompts after one warm-up prompt and exit (ncu captures)")
    ap.add_argument("--profile-codec", type=int, default=0,
                    help="codec: fill the rings of this many streams (16 chunks of 8 frames), decode one more "
                         "chunk and exit (the command the codec ncu captures use)")
    ap.add_argument("--profile-frames", type=int, default=0,
                    help="run this many frames of the workload after one warm-up frame and exit "
                         "(the command the ncu captures under profiles/ use)")
    ap.add_argument("--profile-batch1", type=int, default=0,
                    help="run this many batch-1 global steps (configs[0]) after 5 warm-up steps and exit "
                         "(the command of the small-layer ncu captures)")
    ap.add_argument("--phase-stamps", type=int, default=0,
                    help="batch-1 global step (configs[0]) on the phase-stamp build: per-phase times "
                         "of the two-launch layers over this many steps (profiles/small_layers_b1.md)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.lmin is None:
        args.lmin = 256 if args.workload == "configs4" else 64
    if args.lmax is None:
        args.lmax = 4096 if args.workload == "configs4" else 1024
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.phase_stamps or args.profile_batch1:
        run_phase_stamps(args.phase_stamps or args.profile_batch1, stamps=bool(args.phase_stamps))
        return
    if args.profile_codec:
        import torch
        pkg = load_package()
        pkg.build()
        from moss_b200 import codecfile
        path = codecfile.ensure_synth_decoder(Path(tempfile.gettempdir()) / "moss_b200_dec1.moss", 1)
        n = args.profile_codec
        codec = pkg.Codec(path, 0, max_streams=n, max_batch_frames=n * 8)
        sids = [codec.open() for _ in range(n)]
        codes = torch.randint(0, 1024, (n, 16, 8), dtype=torch.int32, device="cuda")
        out = torch.empty((n, 8 * codec.samples_per_frame), dtype=torch.float32, device="cuda")
        for _ in range(17):
            codec.decode_batch_device(sids, codes.data_ptr(), 8, out.data_ptr())
        torch.cuda.synchronize()
        codec.close()
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
