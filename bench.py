#!/usr/bin/env python
"""Benchmark: Gemma 4 E2B vision and audio tower throughput on B200.

Default workload (the batched configurations of the benchmark spec):
- vision: a job of 64 seeded 768x768 images (2304 patches, 256 tokens, all
  16 layers, pooler, embedder), sharded by image across the N ranks;
- audio: a job of 128 seeded clips, lengths U[1,30] s, LPT-balanced across
  the ranks by encoder rows.
The job is fixed as N grows ("strong" scaling); `--scaling weak` makes
--images / --clips per-GPU counts instead.  One process per GPU under
torchrun, no data-path collective (items are independent).

A step is one pass of the tower over this rank's share of the job.  `value`
is device-timed: CUDA events on the launching stream around every timed
step, inputs resident in HBM, L2 flushed (a 256 MB write) before each step
outside the events, max over ranks.  `e2e` is the same metric through the
C ABI batch call with pinned host buffers (host->device inputs and
device->host embeddings inside the timed region).  `--impl reference` times
the CPU restatement of the reference's CPU path (the oracle) instead, one
encoder layer of a full image (or clip) per step.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "gemma-4-webgpu-kernels-multimodal_b200"

HIDDEN, FF, HEADS, HD, TEXT = 768, 3072, 12, 64, 1536
AUDIO_D, AUDIO_FF, AUDIO_OUT = 1024, 4096, 1536
VISION_METRIC = "images/s (vision tower 768x768, 16 layers, + embedder)"
AUDIO_METRIC = "audio-sec/s (audio tower, 12 layers, + embedder)"
FLUSH_BYTES = 256 << 20
sharding = None  # the package's sharding module, imported with the package


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def s_in_mode(quant: str):
    """input_activation_scale of every QAT linear: 0 (no static input
    quantisation) or the fixed per-linear absmax/127 table ("calibrated")."""
    return "calibrated" if quant == "calibrated" else 0.0


QUANT_DESC = {"none": "none (input_activation_scale 0: fp16 hi/lo activations, two-term GEMMs)",
              "calibrated": "calibrated (input_activation_scale = absmax/127 per linear: int8 codes, kind::i8 GEMMs)"}


def job_images(args, world: int) -> int:
    return args.images if args.scaling == "strong" else args.images * world


def job_clips(args, world: int) -> int:
    return args.clips if args.scaling == "strong" else args.clips * world


def vision_config(args, world: int) -> dict:
    """The workload both arms report (one definition, so the lines match)."""
    n = job_images(args, world)
    per = (f"{n} images in the job, sharded by image over the ranks" if args.scaling == "strong"
           else f"{args.images} images per GPU")
    return {"workload": f"batched vision: {per}; 768x768 (2304 patches, 256 tokens), 16 layers + pooler + embedder",
            "job_images": n, "image": "768x768", "layers": 16, "parallelism": f"dp{world} (replicas)",
            "l2": "L2 flushed (256 MB write) before every timed step, outside the timed events",
            "activation_quant": QUANT_DESC[args.quant]}


def audio_config(args, world: int) -> dict:
    n = job_clips(args, world)
    per = (f"{n} clips in the job" if args.scaling == "strong" else f"{args.clips} clips per GPU")
    return {"workload": f"batched audio: {per}, lengths U[1,30] s (seeded), packed rows (no padding), clips "
                        "LPT-balanced over the ranks by encoder rows; 12 layers + output projection + embedder",
            "job_clips": n, "layers": 12, "parallelism": f"dp{world} (replicas)",
            "l2": "L2 flushed (256 MB write) before every timed step, outside the timed events",
            "activation_quant": QUANT_DESC[args.quant]}


def weights_path(tower: str, layers: int, quant: str, rank: int, barrier) -> str:
    syn = importlib.import_module(PKG + ".synthetic")
    d = os.path.join(os.environ.get("TMPDIR", "/tmp"), "g4m_bench")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, f"{tower}{layers}_seed0_{quant}.safetensors")
    if rank == 0 and not os.path.exists(p):
        tmp = p + f".tmp{os.getpid()}"
        make = syn.vision_weights if tower == "vision" else syn.audio_weights
        syn.write_safetensors(tmp, make(0, layers=layers, s_in=s_in_mode(quant)))
        os.replace(tmp, p)
    barrier()
    return p


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling.  nvidia-smi runs for the
    whole process at a 50 ms period with timestamps; only samples that fall
    inside the timed windows (window() around each timed region) count."""
    FIELDS = ("timestamp,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 50

    def __init__(self, uuid: str, index: int):
        self.uuid = uuid.lower().replace("gpu-", "")
        self.index = index
        self.all = []
        self.windows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", str(self.PERIOD_MS)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        import datetime
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                try:
                    t = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                self.all.append([t] + parts[1:])

    class _Window:
        def __init__(self, owner):
            self.owner = owner

        def __enter__(self):
            self.t0 = time.time()

        def __exit__(self, *exc):
            self.owner.windows.append((self.t0, time.time()))
            return False

    def window(self):
        """Context manager marking one timed region."""
        return ClockSampler._Window(self)

    def stop(self):
        if self.proc:
            time.sleep(2 * self.PERIOD_MS / 1000.0)  # the samples of the last window's end
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        mine = [r for r in self.all if self.uuid and self.uuid in r[1].lower()]
        if not mine and self.all:  # UUID formats differ: fall back to the device ordinal
            uuids = sorted({r[1] for r in self.all})
            pick = uuids[self.index] if self.index < len(uuids) else uuids[0]
            mine = [r for r in self.all if r[1] == pick]
        slack = self.PERIOD_MS / 1000.0
        rows = [r for r in mine if any(t0 - slack <= r[0] <= t1 + slack for t0, t1 in self.windows)]
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[6 + i] and "Not" not in r[6 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "timed_windows": len(self.windows),
                "timed_s": round(sum(t1 - t0 for t0, t1 in self.windows), 3)}


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def tensor_peak():
    """(peak TFLOP/s, source): the measured sustained bf16 figure (kernels
    timed inside seconds-long steps), else the recipe's fallback."""
    p = measured_peaks().get("bf16_tflops_sustained")
    return (float(p), "measured (bf16 cuBLAS, sustained)") if p else (1400.0, "fallback")


def int8_peak():
    """(peak TOP/s, source) for the kind::i8 GEMMs: twice the bf16 figure --
    a kind::i8 MMA retires twice the multiply-adds per cycle of a kind::f16
    one of the same shape (16384 against 8192 per cycle per SM, measured on
    this part with single-thread MMA issue loops)."""
    p, src = tensor_peak()
    return 2.0 * p, "2x " + src


def traffic_per_launch(kernel: str, key: str):
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "traffic_per_launch.json")))
        return tr.get(kernel, {}).get(key)
    except Exception:
        return None


def vision_kernel_flops(B: int, N: int, tokens: int):
    """Algorithmic FLOPs per launch of each profiled kernel (2*M*N*K for a
    linear, 4*n^2*d per head for attention), counted once (not per split
    term)."""
    M = B * N
    return {
        "gemm_qkv": 2.0 * M * 3 * HIDDEN * HIDDEN,
        "gemm_o": 2.0 * M * HIDDEN * HIDDEN,
        "gemm_gate_up": 2.0 * M * 2 * FF * HIDDEN,
        "gemm_down": 2.0 * M * FF * HIDDEN,
        "attention": 4.0 * B * HEADS * N * N * HD,
        "gemm_patch": 2.0 * M * HIDDEN * 768,
        "gemm_embed": 2.0 * B * tokens * TEXT * HIDDEN,
    }


def audio_kernel_flops(M: int):
    """Algorithmic FLOPs per launch of the audio GEMMs over M packed rows."""
    return {
        "gemm_ffw1": 2.0 * M * AUDIO_FF * AUDIO_D,
        "gemm_ffw2": 2.0 * M * AUDIO_D * AUDIO_FF,
        "gemm_qkv": 2.0 * M * 3 * AUDIO_D * AUDIO_D,
        "gemm_post": 2.0 * M * AUDIO_D * AUDIO_D,
        "gemm_lconv_start": 2.0 * M * 2 * AUDIO_D * AUDIO_D,
        "gemm_lconv_end": 2.0 * M * AUDIO_D * AUDIO_D,
        "gemm_in_proj": 2.0 * M * AUDIO_D * AUDIO_D,
        "gemm_out_proj": 2.0 * M * AUDIO_OUT * AUDIO_D,
        "gemm_embed": 2.0 * M * 1536 * AUDIO_OUT,
    }


def audio_rows(n: int) -> int:
    return sharding.encoder_rows(n)


# ------------------------------------------------------------ CPU (oracle)


class CpuVisionSteps:
    """The oracle (CPU restatement of the reference's CPU twins) on one
    768x768 image, one encoder layer per step: the patch embedding runs with
    layer 0 and the pooler / embedder with layer 15, so 16 consecutive steps
    are exactly one image through the whole tower."""
    DESC = ("one 768x768 image through the oracle, one of the 16 encoder layers per step (patch embedding with "
            "layer 0, pooler + embedder with layer 15; 16 steps = one image)")

    def __init__(self, threads: int, quant: str):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        syn = importlib.import_module(PKG + ".synthetic")
        O.set_threads(threads)
        self.O = O
        self.W = syn.vision_weights(0, layers=16, s_in=s_in_mode(quant))
        pre = O.preprocess_image_pixels(syn.image_pixels(0, 768, 768))
        self.patches, self.pos = O.valid_image_patch_input(pre)
        self.i = 0
        self.h = None

    def step(self) -> float:
        O, layer = self.O, self.i % 16
        t0 = time.perf_counter()
        if layer == 0:
            self.h = O.vision_patch_embeddings(self.W, self.patches, self.pos)
        self.h = O.vision_layer(self.W, layer, self.h, self.pos)
        if layer == 15:
            O.embedder(O.vision_pooler(self.h, self.pos, 256), self.W["model.embed_vision.embedding_projection.weight"])
        self.i += 1
        return time.perf_counter() - t0


class CpuAudioSteps:
    """The oracle on one 10 s clip (250 encoder rows), one conformer layer per
    step: log-mel and subsample run with layer 0, the output projection and
    embedder with layer 11, so 12 consecutive steps are one clip."""
    DESC = ("one 10 s clip through the oracle, one of the 12 conformer layers per step (log-mel + subsample with "
            "layer 0, output projection + embedder with layer 11; 12 steps = one clip)")
    SECONDS = 10.0

    def __init__(self, threads: int, quant: str):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        syn = importlib.import_module(PKG + ".synthetic")
        O.set_threads(threads)
        self.O = O
        self.W = syn.audio_weights(0, layers=12, s_in=s_in_mode(quant))
        self.x = syn.audio_samples(0, 160000)
        self.i = 0
        self.h = None

    def step(self) -> float:
        O, W, layer = self.O, self.W, self.i % 12
        t0 = time.perf_counter()
        if layer == 0:
            pre = O.preprocess_audio(self.x, pad_to_multiple_of=None)
            self.h, _ = O.audio_subsample(W, pre["inputFeatures"], pre["inputFeaturesMask"])
        self.h = O.audio_layer(W, layer, self.h)
        if layer == 11:
            proj = O.add_bias_rows(O.f32_linear_rows(self.h, W["model.audio_tower.output_proj.weight"]),
                                   W["model.audio_tower.output_proj.bias"])
            O.embedder(proj, W["model.embed_audio.embedding_projection.weight"])
        self.i += 1
        return time.perf_counter() - t0


def cpu_rate(make, steps: int, units_per_cycle: float, cycle: int):
    """Run `steps` oracle steps; rate = units processed / seconds, where a
    cycle of `cycle` steps processes `units_per_cycle` units."""
    runner = make()
    secs = [runner.step() for _ in range(steps)]
    return units_per_cycle * steps / cycle / sum(secs), secs, runner.DESC


def run_reference(args):
    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    v = CpuVisionSteps(threads, args.quant)
    for _ in range(args.warmup):
        v.step()
    secs = [v.step() for _ in range(args.steps)]
    value = (args.steps / 16.0) / sum(secs)
    line = {
        "impl": "reference", "metric": VISION_METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(secs) / len(secs),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32 (JS number / Math.fround semantics)", "data": "synthetic",
        "config": vision_config(args, world),
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "port", "sample": v.DESC},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    if not args.no_audio:
        a = CpuAudioSteps(threads, args.quant)
        a.step()
        k = max(args.steps, 12)
        a_secs = [a.step() for _ in range(k)]
        av = CpuAudioSteps.SECONDS * (k / 12.0) / sum(a_secs)
        line["audio"] = {"metric": AUDIO_METRIC, "value": av, "unit": "audio-s/s",
                         "ms_per_step": 1000.0 * sum(a_secs) / k, "config": audio_config(args, world),
                         "cpu_baseline": {"value": av, "unit": "audio-s/s", "cores": threads, "kind": "port",
                                          "sample": a.DESC},
                         "e2e": {"value": av, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- device arm


def timed_steps(step, stream, steps: int, flush):
    """Device time of `steps` calls of step(): each call bracketed by its own
    CUDA events on `stream`; the L2 flush before it runs outside them."""
    import torch
    evs = []
    for _ in range(steps):
        with torch.cuda.stream(stream):
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs)


def run_audio(args, native, syn, rank, world, dist, barrier, flush, clocks):
    """Batched audio: the job's clips, lengths U[1, 30] s, packed without
    padding rows, this rank's LPT share.  Returns the sub-object of the JSON
    line (rank 0)."""
    import numpy as np
    import torch
    p = weights_path("audio", 12, args.quant, rank, barrier)
    ctx = native.Context([torch.cuda.current_device()])
    ctx.load_weights(p)
    job_lens = syn.audio_batch_lengths(1000, job_clips(args, world))
    mine = sorted(sharding.lpt_assign([audio_rows(int(L)) for L in job_lens], world)[rank])
    lens = job_lens[mine]
    n = len(mine)
    job_seconds = float(job_lens.sum()) / 16000.0
    total = int(lens.sum())
    host = torch.empty(max(total, 1), dtype=torch.float32).pin_memory()
    offs = np.zeros(n, np.int64)
    o = 0
    for j, (i, L) in enumerate(zip(mine, lens)):
        host[o:o + int(L)] = torch.from_numpy(syn.audio_samples(5000 + i, int(L)))
        offs[j] = o
        o += int(L)
    dev = host.cuda()
    rows = sum(audio_rows(int(L)) for L in lens)
    out = torch.empty((max(rows, 1), 1536), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    step = lambda: ctx.audio_embed_device(dev.data_ptr(), offs, lens, out.data_ptr(), stream=stream.cuda_stream)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    launches0 = native.kernel_launches()
    with clocks.window():
        ms = timed_steps(step, stream, args.steps, flush)
    launches = native.kernel_launches() - launches0
    ms = sharding.max_over_ranks(ms, dist, "cuda")
    value = job_seconds * args.steps / (ms / 1000.0)
    ctx.profile_begin()
    step()
    prof = ctx.profile_end()
    flops = audio_kernel_flops(rows)
    gem = {k: v for k, v in prof.items() if k in flops}
    dom = max(gem, key=lambda k: gem[k][1])
    peak, peak_src = tensor_peak()
    ach = flops[dom] / (gem[dom][1] / gem[dom][0] / 1000.0) / 1e12
    traffic = traffic_per_launch(dom, "bytes_per_launch_audio128") if n == 128 else None
    # end to end with pinned host clips through the C ABI batch call
    clips = [host[int(offs[i]):int(offs[i]) + int(lens[i])].numpy() for i in range(n)]
    out_pin = torch.empty((max(rows, 1), 1536), dtype=torch.float32).pin_memory()
    outs, r0 = [], 0
    for L in lens:
        r = audio_rows(int(L))
        outs.append(out_pin[r0:r0 + r].numpy())
        r0 += r
    ctx.audio_embed(clips, 16000, 12, outs=outs)
    barrier()
    k_e2e = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(k_e2e):
        ctx.audio_embed(clips, 16000, 12, outs=outs)
    te = sharding.max_over_ranks(time.perf_counter() - t0, dist, "cuda")
    res = {
        "metric": AUDIO_METRIC, "value": value, "unit": "audio-s/s", "ms_per_step": ms / args.steps,
        "config": dict(audio_config(args, world), clips_this_rank=n, audio_seconds_job=job_seconds,
                       audio_seconds_this_rank=total / 16000.0, encoder_rows_this_rank=rows),
        "gpu_launches": launches,
        "e2e": {"value": job_seconds * k_e2e / te, "unit": "audio-s/s",
                "h2d_bytes_per_step": total * 4, "d2h_bytes_per_step": rows * 1536 * 4},
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                     "frac": ach / peak, "peak_source": peak_src, "traffic": traffic,
                     "launch_ms": gem[dom][1] / gem[dom][0], "flop_per_launch": flops[dom]},
        "kernel_ms_per_step": {k: round(v[1], 4) for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, _, desc = cpu_rate(lambda: CpuAudioSteps(threads, args.quant), 12, CpuAudioSteps.SECONDS, 12)
        res["cpu_baseline"] = {"value": rate, "unit": "audio-s/s", "cores": threads, "kind": "port", "sample": desc}
    ctx.close()
    return res


def qat_sweep(native, syn, peak, steps=10):
    """The int8 QAT linear (768 -> 768, per-channel scales, bias) on
    device-resident activations at M = 256, 18432 (8 images) and 147456
    (64 images): per-launch CUDA-event time of the tensor-core GEMM,
    algorithmic TFLOP/s and the fraction of the measured peak."""
    import ctypes
    import torch
    L = native.lib()
    ctx = native.Context([torch.cuda.current_device()])
    out = {}
    try:
        _, w, s, b = syn.qat_linear_case(0, rows=1)
        h = ctypes.c_void_p()
        native.check(L.g4m_linear_prepare(ctx.h, 0, native.ptr(w), 0, 768, 768, native.ptr(s), 0.0, 0.0,
                                          native.ptr(b), ctypes.byref(h)))
        try:
            for M in (256, 18432, 147456):
                x = torch.randn((M, 768), dtype=torch.float32, device="cuda")
                y = torch.empty((M, 768), dtype=torch.float32, device="cuda")
                st = torch.cuda.current_stream().cuda_stream
                run = lambda: native.check(L.g4m_linear_run(h, ctypes.c_void_p(x.data_ptr()), M,
                                                            ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(st)))
                for _ in range(3):
                    run()
                torch.cuda.synchronize()
                ctx.profile_begin()
                for _ in range(steps):
                    run()
                prof = ctx.profile_end()
                cnt, tot = prof["gemm_qat"]
                ms = tot / cnt
                tf = 2.0 * M * 768 * 768 / (ms / 1000.0) / 1e12
                out[str(M)] = {"gemm_ms": round(ms, 5), "tflops": round(tf, 1), "frac": round(tf / peak, 4),
                               "operand_ms": round(prof["prep_a"][1] / prof["prep_a"][0], 5)}
        finally:
            L.g4m_linear_free(h)
    finally:
        ctx.close()
    return {"workload": "int8 QAT linear 768x768 (+bias), activations resident; algorithmic 2*M*768*768",
            "peak": peak, "by_rows": out}


def qat_cfg0(native, syn, steps=20):
    """The single int8 QAT linear of the benchmark spec (x f32 [256, 768]
    ~N(0,1), W int8 [768, 768] U[-127, 127], per-channel scales, bias, seed
    0): latency through g4m_qat_linear with host buffers (weights uploaded
    and converted inside the call, as the reference's one-shot runner takes
    them), the resident form (g4m_linear_run on device buffers, CUDA events),
    and the oracle on the host's cores.  Parity against the oracle is
    reported beside the times."""
    import ctypes

    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    x, w, s, b = syn.qat_linear_case(0)
    ctx = native.Context([torch.cuda.current_device()])
    try:
        for _ in range(3):
            y = ctx.qat_linear(x, w, s, bias=b)
        lat = []
        for _ in range(steps):
            t0 = time.perf_counter()
            y = ctx.qat_linear(x, w, s, bias=b)
            lat.append(time.perf_counter() - t0)
        L = native.lib()
        h = ctypes.c_void_p()
        native.check(L.g4m_linear_prepare(ctx.h, 0, native.ptr(w), 0, 768, 768, native.ptr(s), 0.0, 0.0,
                                          native.ptr(b), ctypes.byref(h)))
        try:
            xd = torch.from_numpy(x).cuda()
            yd = torch.empty((256, 768), dtype=torch.float32, device="cuda")
            st = torch.cuda.current_stream()
            run = lambda: native.check(L.g4m_linear_run(h, ctypes.c_void_p(xd.data_ptr()), 256,
                                                        ctypes.c_void_p(yd.data_ptr()), ctypes.c_void_p(st.cuda_stream)))
            for _ in range(3):
                run()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(steps):
                run()
            e1.record(st)
            e1.synchronize()
            resident_ms = e0.elapsed_time(e1) / steps
        finally:
            L.g4m_linear_free(h)
    finally:
        ctx.close()
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    cpu = []
    for _ in range(5):
        t0 = time.perf_counter()
        ref = O.add_bias_rows(O.qat_i8_linear(x, w, s), b)
        cpu.append(time.perf_counter() - t0)
    rms = float(np.sqrt((ref.astype(np.float64) ** 2).mean()))
    cos = ((ref * y).sum(1) / (np.linalg.norm(ref, axis=1) * np.linalg.norm(y, axis=1))).min()
    return {"workload": "int8 QAT linear 256x768 -> 768 + bias, seed 0 (x ~N(0,1), W U[-127,127])",
            "flop": 2.0 * 256 * 768 * 768,
            "e2e_ms": round(1000 * statistics.median(lat), 4),
            "e2e_note": "g4m_qat_linear: host x / W / scales / bias in, host y out; weight upload and fp16 "
                        "conversion inside every call (the reference's runner takes its weights per call)",
            "resident_ms": round(resident_ms, 5),
            "resident_note": "g4m_linear_run: weights prepared once, device x / y, CUDA events",
            "cpu_ms": round(1000 * statistics.median(cpu), 4), "cpu_cores": threads, "cpu_kind": "port",
            "max_abs_over_rms": float(np.abs(y - ref).max() / rms), "min_row_cos": float(cos)}


def run_ours(args):
    import numpy as np
    import torch

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    native = importlib.import_module(PKG + "._native")
    syn = importlib.import_module(PKG + ".synthetic")
    global sharding
    sharding = importlib.import_module(PKG + ".sharding")
    H, Wd, layers, max_soft = 768, 768, 16, 280
    N, tokens = (H // 16) * (Wd // 16), 256
    n_job = job_images(args, world)
    mine = list(sharding.image_shard(n_job, world, rank))
    B = len(mine)
    path = weights_path("vision", layers, args.quant, rank, barrier)
    ctx = native.Context([local])
    ctx.load_weights(path)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    pix_host = torch.empty((max(B, 1), H, Wd, 3), dtype=torch.float32).pin_memory()
    for i, seed in enumerate(mine):  # this rank's images of the job
        pix_host[i] = torch.from_numpy(syn.image_pixels(seed, H, Wd))
    pix = pix_host.cuda()
    out = torch.empty((max(B, 1) * tokens, TEXT), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()  # a real stream: the library launches on it, the events bracket it

    def step():
        ctx.vision_embed_device(pix.data_ptr(), B, H, Wd, out.data_ptr(), max_soft, layers, stream.cuda_stream)

    clocks = ClockSampler(str(torch.cuda.get_device_properties(local).uuid), local)
    clocks.start()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    barrier()
    launches0 = native.kernel_launches()
    with clocks.window():
        ms = timed_steps(step, stream, args.steps, flush)
    launches = native.kernel_launches() - launches0
    barrier()
    ms_max = sharding.max_over_ranks(ms, dist, "cuda")
    value = n_job * args.steps / (ms_max / 1000.0)

    # roofline of the dominant kernel: per-launch CUDA-event times of one step
    ctx.profile_begin()
    step()
    prof = ctx.profile_end()
    flops = vision_kernel_flops(B, N, tokens)
    dom = max((k for k in prof if k in flops), key=lambda k: prof[k][1])
    cnt, tot = prof[dom]
    peak, peak_src = tensor_peak()
    achieved = flops[dom] / (tot / cnt / 1000.0) / 1e12
    traffic = traffic_per_launch(dom, "bytes_per_launch_b64") if B == 64 else None
    # split-operand factor: executed tensor FLOPs per algorithmic FLOP (three S products and
    # four P*V products for attention; two or one terms for the QAT linears)
    factor = {"attention": 3.5}.get(dom, 1.0 if args.quant == "calibrated" else 2.0)
    roofline = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": peak_src, "traffic": traffic,
                "launch_ms": tot / cnt, "flop_per_launch": flops[dom],
                "executed_tflops": achieved * factor, "executed_frac": achieved * factor / peak,
                "note": "achieved/frac count one term (2*M*N*K, 4*n^2*d); executed_* include the fp16 hi/lo "
                        "split products the tensor pipe runs for fp32-grade results"}
    kernel_ms = {k: round(v[1], 4) for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])}
    # the int8 QAT linears together (the metric's "int8-linear tensor-pipe % of peak")
    qat = [k for k in ("gemm_qkv", "gemm_o", "gemm_gate_up", "gemm_down") if k in prof]
    qat_flop = sum(flops[k] * prof[k][0] for k in qat)
    qat_ms = sum(prof[k][1] for k in qat)
    qat_ach = qat_flop / (qat_ms / 1000.0) / 1e12
    if args.quant == "calibrated":
        qpeak, qsrc = int8_peak()
        qat_linear = {"kernels": qat, "achieved": qat_ach, "peak": qpeak, "unit": "TOP/s", "frac": qat_ach / qpeak,
                      "peak_source": qsrc, "ms_per_step": qat_ms,
                      "note": "algorithmic 2*M*N*K per linear on int8 codes x int8 weights (kind::i8, one term)"}
    else:
        qat_linear = {"kernels": qat, "achieved": qat_ach, "peak": peak, "unit": "TFLOP/s", "frac": qat_ach / peak,
                      "peak_source": peak_src, "ms_per_step": qat_ms,
                      "note": "algorithmic 2*M*N*K per linear (one term); the split operands execute 2x that on "
                              "the tensor pipe (fp16 hi and lo planes of the activations)"}

    # end to end through the C ABI with pinned host buffers
    out_pin = torch.empty((max(B, 1), tokens, TEXT), dtype=torch.float32).pin_memory()
    out_host = [out_pin[i].numpy() for i in range(B)]
    in_host = [pix_host[i].numpy() for i in range(B)]
    ctx.vision_embed(in_host, max_soft, layers, outs=out_host)
    barrier()
    k_e2e = max(1, min(args.steps, 5))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(k_e2e):
        ctx.vision_embed(in_host, max_soft, layers, outs=out_host)
    t_e2e = time.perf_counter() - t0
    e2e_value = n_job * k_e2e / sharding.max_over_ranks(t_e2e, dist, "cuda")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, _, desc = cpu_rate(lambda: CpuVisionSteps(threads, args.quant), 16, 1.0, 16)
        cpu = {"value": rate, "unit": "images/s", "cores": threads, "kind": "port", "sample": desc}

    sweep = qat_sweep(native, syn, peak) if rank == 0 else None
    cfg0 = qat_cfg0(native, syn) if rank == 0 and not args.no_cpu_baseline else None
    audio = None
    if not args.no_audio:
        ctx.close()
        audio = run_audio(args, native, syn, rank, world, dist, barrier, flush, clocks)
    clk = clocks.stop()

    if rank == 0:
        line = {
            "impl": "g4m", "metric": VISION_METRIC, "value": value,
            "unit": "images/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None,
            "dtype": ("f32-grade (fp16 hi/lo split operands on tcgen05, f32 accumulate)" if args.quant == "none" else
                      "int8 activation codes x int8 weights on tcgen05 kind::i8, exact int32 accumulate"),
            "data": "synthetic (seeded U[0,1] pixels, random-init weights with the reference dtypes)",
            "config": dict(vision_config(args, world), images_this_rank=B),
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": B * H * Wd * 3 * 4,
                    "d2h_bytes_per_step": B * tokens * TEXT * 4},
            "gpu_launches": launches,
            "roofline": roofline,
            "qat_linear": qat_linear,
            "qat_linear_sweep": sweep,
            "qat_cfg0": cfg0,
            "kernel_ms_per_step": kernel_ms,
            "cpu_baseline": cpu,
            "clocks": clk,  # samples inside the timed windows of both towers
        }
        if audio:
            line["audio"] = audio
        print(json.dumps(line), flush=True)
    if args.no_audio:
        ctx.close()
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: --images / --clips are the job's totals, sharded over the ranks; weak: per GPU")
    ap.add_argument("--images", type=int, default=64, help="images in the job (strong) or per GPU (weak)")
    ap.add_argument("--clips", type=int, default=128, help="audio clips in the job (strong) or per GPU (weak)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-audio", action="store_true", help="skip the batched-audio half of the metric")
    ap.add_argument("--quant", default="none", choices=["none", "calibrated"],
                    help="static input-activation quantisation of the QAT linears")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
