#!/usr/bin/env python
"""bench.py -- throughput of the B200 spectral path (chunking -> STFT -> mask -> iSTFT -> OLA).

Metric: audio-seconds per second of the whole separation, whole job over
all GPUs; plus the dominant kernel's achieved HBM bandwidth against the measured peak (the
fused kernel for RoFormer and TFC-TDF, the back kernel for HTDemucs).

Workload (default ``cfg1``, the headline configuration): Mel-Band RoFormer (Kim) front/back
end on 60 s of seeded stereo 44.1 kHz audio: chunks of 352800 samples, num_overlap 4
(36 chunks), STFT n_fft 2048 / hop 441 (801 frames, 1025 bins), 60 mel bands (1979
band-bin entries, duplicates averaged), complex mask N(0, 0.5) in the network's band-major
layout, iSTFT, windowed overlap-add across chunks. One step = one such track. The mask
(913 MB) and the mix are resident in HBM before the timed region; they exceed the 126 MB
L2, so no flush is needed between steps. Other workloads: cfg0, cfg2, cfg3, cfg4 (the
BASELINE configurations), vr3band and io48k (see WORKLOADS).

Multi-GPU (torchrun, one process per GPU): every rank separates its own track; there is no
data-path collective (weak scaling). NCCL is used only for the barrier and the max-over-
ranks of the device-timed duration. ``--split-track`` splits one track's output samples
across the ranks instead (strong scaling, still without an exchange).

``--impl reference`` times the reference's CPU implementation of the same path on this
box's host cores (rank 0 only): the reference's own stft.h compiled from its sources
(oracle/_ref) under the restated host loops of src/roformer.cpp, with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SR = 44100

WORKLOADS = {
    "cfg1": dict(arch="roformer", bands="mel", seconds=60, chunk=352800, num_overlap=4, n_fft=2048,
                 hop=441, zero_dc=False, sigma=0.5, seed=1,
                 desc="Mel-Band RoFormer (Kim) front/back end, 60 s stereo, chunk 352800, overlap 4"),
    "cfg2": dict(arch="roformer", bands="bs", seconds=180, chunk=352800, num_overlap=2, n_fft=2048,
                 hop=441, zero_dc=True, sigma=0.5, seed=2,
                 desc="BS-RoFormer (viperx 317) front/back end, 180 s stereo, chunk 352800, overlap 2"),
    "cfg0": dict(arch="htdemucs", seconds=20, segment=343980, sources=4, sigma=1.0, seed=0,
                 desc="HTDemucs spectral path, 20 s stereo, 4 stems, segments of 7.8 s, 25% overlap"),
    "cfg3": dict(arch="tfc", seconds=180, n_fft=7680, hop=1024, dim_f=3072, dim_t=256, zero_bins=3,
                 overlap=0.5, sigma=1.0, seed=3,
                 desc="MDX TFC-TDF (Kim_Vocal_2) framing, 180 s stereo, n_fft 7680, UVR 50% overlap"),
    "cfg4": dict(arch="htdemucs", seconds=240, segment=343980, sources=4, sigma=1.0, seed=4, tracks=64,
                 desc="batch of 64 tracks of 240 s through the HTDemucs spectral path, round-robin over GPUs"),
    # VR (src/vr.cpp): no BASELINE config; a three-band layout of the reference's kind (bands at
    # 7.35 / 14.7 / 44.1 kHz, n_fft 320 / 512 / 960, equal frame durations), 180 s
    "vr3band": dict(arch="vr", seconds=180, seed=10, bins=608, pre=(500, 600), bands=[
        dict(sr=7350, hop=80, nfft=320, start=0, stop=100, lp_start=80, lp_stop=100),
        dict(sr=14700, hop=160, nfft=512, start=50, stop=200, hp_start=60, hp_stop=50, lp_start=180, lp_stop=200),
        dict(sr=44100, hop=480, nfft=960, start=150, stop=481, hp_start=170, hp_stop=150)],
        desc="VR spectral path, 3 bands (7.35/14.7/44.1 kHz, n_fft 320/512/960), 180 s stereo, 2 stems"),
    # the request-side conversions around separate() (src/libstems.cpp:160-199): not a
    # BASELINE config; measured so the row that feeds the path has its own number
    "io48k": dict(arch="io", seconds=180, rate=48000, stems=4, seed=9,
                  desc="interleaved stereo 48 kHz -> planar 44.1 kHz (Kaiser sinc), 4 stereo stems back to "
                       "48 kHz pinned to the input length, 180 s"),
}


def load_pkg():
    import __graft_entry__
    return __graft_entry__.load_package()


def synth_audio(seed, length, channels=2):
    """The benchmark mix: 8 seeded sines (50-8000 Hz, amp 0.05-0.2) + N(0, 0.01) noise, clipped."""
    rng = np.random.default_rng(seed)
    t = np.arange(length, dtype=np.float64) / SR
    out = np.empty((channels, length), np.float32)
    for c in range(channels):
        f, a, ph = rng.uniform(50, 8000, 8), rng.uniform(0.05, 0.2, 8), rng.uniform(0, 2 * np.pi, 8)
        x = np.zeros(length)
        for k in range(8):
            x += a[k] * np.sin(2 * np.pi * f[k] * t + ph[k])
        x += 0.01 * rng.standard_normal(length)
        out[c] = np.clip(x, -1, 1)
    return out


def make_plan(pkg, eng, w, length):
    if w["arch"] == "roformer":
        sizes, freqs = pkg.bands.mel_bands() if w["bands"] == "mel" else pkg.bands.bs_bands()
        return eng.plan_roformer(length, sizes, freqs, chunk=w["chunk"], num_overlap=w["num_overlap"],
                                 n_fft=w["n_fft"], hop=w["hop"], zero_dc=w["zero_dc"])
    if w["arch"] == "htdemucs":
        return eng.plan_htdemucs(length, n_sources=w["sources"], segment=w["segment"])
    return eng.plan_tfc(length, n_fft=w["n_fft"], hop=w["hop"], dim_f=w["dim_f"], dim_t=w["dim_t"],
                        zero_bins=w["zero_bins"], overlap=w["overlap"])


def kernel_algorithmic_bytes(plan, w):
    """(the dominant kernel, the bytes it must move once per launch), 4-byte floats.
    RoFormer / TFC-TDF, the fused kernel: each chunk's audio window in, the masks in, each
    chunk's separated output out (TFC-TDF at n_fft 7680 with an even hop: the fused kernel on CTA
    pairs). HTDemucs, the back kernel: each segment's spectra (2048 bins x T frames x 2
    channels, complex) in, the masks in, the segment outputs out."""
    if w["arch"] == "htdemucs":
        lc = w["segment"]
        z = plan.n_chunks * plan.n_frames * 2048 * 4
        return "back_kernel", 4 * (z + plan.mask_floats + plan.n_chunks * plan.n_out_sources * plan.n_channels * lc)
    lc = w["chunk"] if w["arch"] == "roformer" else w["hop"] * (w["dim_t"] - 1)
    n_src = plan.n_out_sources
    pair = w["arch"] == "tfc" and w["n_fft"] == 7680 and w["hop"] % 2 == 0
    return "fused_pair_kernel" if pair else "fused_kernel", 4 * (plan.n_chunks * plan.n_channels * lc + plan.mask_floats
                                + plan.n_chunks * n_src * plan.n_channels * lc)


def path_algorithmic_bytes(plan, w):
    """The path's algorithmic bytes per track: audio in per chunk window + masks in + stems out once."""
    lc = {"roformer": w.get("chunk"), "htdemucs": w.get("segment")}.get(w["arch"]) or w["hop"] * (w["dim_t"] - 1)
    return 4 * (plan.n_chunks * plan.n_channels * lc + plan.mask_floats + plan.out_floats)


# ---- clocks during the timed region (NVML, the source nvidia-smi reads) -----------------------
class ClockSampler:
    BAD = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")

    def __init__(self, device_index, period_s=0.005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period, self._stop, self._t, self.ok = period_s, threading.Event(), None, False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
                "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, b in bits.items():
                    if r & b:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._t:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}

    def rejected(self):
        return any(r in self.reasons for r in self.BAD)


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(kernel, workload):
    """DRAM bytes per launch of the kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.txt")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


# ---- CPU baselines -------------------------------------------------------------------------
def cpu_info():
    """The host's CPU model and core counts (the CPU figures' context)."""
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    logical = os.cpu_count() or 1
    try:
        import psutil
        physical = psutil.cpu_count(logical=False) or logical
    except Exception:
        physical = logical
    return {"cpu_model": model, "logical_cores": logical, "physical_cores": physical}


def cpu_threads():
    """Threads of the multi-threaded CPU figure: one per physical core, as the plan says."""
    return cpu_info()["physical_cores"]


def cpu_repeat(fn, min_s=10.0, max_reps=30):
    """Run fn() (returns (seconds, kind)) until about min_s seconds of CPU work are timed;
    returns the mean seconds per run, the kind, and the number of runs."""
    times, kind = [], None
    while not times or (sum(times) < min_s and len(times) < max_reps):
        dt, kind = fn()
        times.append(dt)
    return statistics.mean(times), kind, len(times)


def cpu_run(w, length, mix, mask_host, n_sample, threads):
    """Time the CPU path on the first n_sample chunks of one track; returns (seconds, kind)."""
    import oracle
    kind = "reference" if oracle.use_reference(True) else "port"
    if w["arch"] == "roformer":
        pkg = load_pkg()
        sizes, freqs = pkg.bands.mel_bands() if w["bands"] == "mel" else pkg.bands.bs_bands()
        p = oracle.rf_params(sizes, freqs, chunk=w["chunk"], num_overlap=w["num_overlap"],
                             n_fft=w["n_fft"], hop=w["hop"], zero_dc=int(w["zero_dc"]),
                             sample_first=0, sample_count=n_sample, threads=threads)
        fn = oracle.rf_separate
    elif w["arch"] == "htdemucs":
        p = oracle.ht_params(n_sources=w["sources"], segment=w["segment"], mono_norm=1, cac_norm=1,
                             sample_first=0, sample_count=n_sample, threads=threads)
        fn = oracle.ht_separate
    else:
        p = oracle.tfc_params(n_fft=w["n_fft"], hop=w["hop"], dim_f=w["dim_f"], dim_t=w["dim_t"],
                              zero_bins=w["zero_bins"], overlap=w["overlap"], sample_first=0,
                              sample_count=n_sample, threads=threads)
        fn = oracle.tfc_separate
    t0 = time.perf_counter()
    fn(p, mix, mask_host)
    return time.perf_counter() - t0, kind


class CpuSample:
    """The CPU baseline's workload, shared by the reference arm and the cpu_baseline leg: the
    chunks of one whole track (every chunk the GPU step runs for one track), their masks, and
    the audio-seconds they stand for."""

    def __init__(self, w, threads):
        self.w = w
        self.threads = threads
        self.length = w["seconds"] * SR
        self.n_chunks = _n_chunks(w, self.length)
        self.n_sample = self.n_chunks
        self.mix = synth_audio(w["seed"], self.length)
        self.mask = _host_mask(w, self.n_sample)
        self.audio_s = w["seconds"] * self.n_sample / self.n_chunks
        self.desc = f"all {self.n_chunks} chunks of one {w['seconds']} s track"

    def run(self, threads=None, n_sample=None):
        return cpu_run(self.w, self.length, self.mix, self.mask, n_sample or self.n_sample, threads or self.threads)


def cpu_baseline_record(w, min_s=10.0, single=True):
    """The cpu_baseline object: the shared sample on one thread per physical core, timed for
    about min_s seconds, and (single) the same chunks' first few on one thread."""
    smp = CpuSample(w, cpu_threads())
    dt, kind, reps = cpu_repeat(smp.run, min_s=min_s)
    rec = {"value": smp.audio_s / dt, "unit": "audio-s/s", "cores": smp.threads, "kind": kind,
           "sample": f"{smp.desc}, timed {reps} times", **cpu_info()}
    if single:
        n1 = max(1, min(smp.n_sample, 2))
        dt1, _, reps1 = cpu_repeat(lambda: smp.run(threads=1, n_sample=n1), min_s=min_s / 2)
        rec["single_thread"] = {"value": w["seconds"] * n1 / smp.n_chunks / dt1, "unit": "audio-s/s", "cores": 1,
                                "sample": f"the first {n1} of the {smp.n_chunks} chunks, timed {reps1} times"}
    return rec


def workload_config(w, name, world, split=False):
    """The config object of a RoFormer / HTDemucs / TFC-TDF workload's bench line, computed on
    the host, so that both arms print the same one."""
    length = w["seconds"] * SR
    n_chunks = _n_chunks(w, length)
    if w["arch"] == "roformer":
        frames = w["chunk"] // w["hop"] + 1
    elif w["arch"] == "htdemucs":
        frames = (w["segment"] + 1023) // 1024
    else:
        frames = w["dim_t"]
    tracks = 1 if split else w.get("tracks", world)
    return {"workload": name, "desc": w["desc"], "tracks_per_step": tracks, "chunks_per_track": n_chunks,
            "frames_per_chunk": frames, "mask_bytes_per_track": 4 * n_chunks * _mask_floats_per_chunk(w),
            "l2": "inputs larger than L2 (no flush needed)",
            "parallelism": f"one track split by samples x{world}" if split else f"replicas x{world}"}


def run_reference(args, w, rank):
    """The reference's CPU implementation of the path (its compiled stft.h under the restated
    loops) on this box's host cores: one step = the same sample the cpu_baseline leg times."""
    if rank != 0:
        return 0
    if w["arch"] in ("io", "vr"):
        sample_s = 5.0
        times, kind = [], "port"
        fn = cpu_io if w["arch"] == "io" else cpu_vr
        for k in range(args.warmup + args.steps):
            dt, kind = fn(w, sample_s)
            if k >= args.warmup:
                times.append(dt)
        value = sample_s / statistics.mean(times)
        print(json.dumps({
            "metric": "audio_seconds_per_second", "value": value, "unit": "audio-s/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(times), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["desc"]},
            "cpu_baseline": {"value": value, "unit": "audio-s/s", "cores": 1, "kind": kind,
                             "sample": f"{sample_s:.0f} s of the {w['seconds']} s request per step", **cpu_info()},
            "e2e": {"value": value, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return 0
    smp = CpuSample(w, cpu_threads())
    times, kind = [], "port"
    for k in range(args.warmup + args.steps):
        dt, kind = smp.run()
        if k >= args.warmup:
            times.append(dt)
    value = smp.audio_s / statistics.mean(times)
    line = {"metric": "audio_seconds_per_second", "value": value, "unit": "audio-s/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": workload_config(w, args.workload, int(os.environ.get("WORLD_SIZE", "1")), args.split_track),
            "cpu_baseline": {"value": value, "unit": "audio-s/s", "cores": smp.threads, "kind": kind,
                             "sample": f"{smp.desc} per step", **cpu_info()},
            "e2e": {"value": value, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def _n_chunks(w, length):
    import oracle
    if w["arch"] == "roformer":
        pkg = load_pkg()
        sizes, freqs = pkg.bands.mel_bands() if w["bands"] == "mel" else pkg.bands.bs_bands()
        return oracle.rf_n_chunks(oracle.rf_params(sizes, freqs, chunk=w["chunk"], num_overlap=w["num_overlap"]), length)
    if w["arch"] == "htdemucs":
        return oracle.ht_n_segments(oracle.ht_params(n_sources=w["sources"], segment=w["segment"]), length)
    return oracle.tfc_n_chunks(oracle.tfc_params(n_fft=w["n_fft"], hop=w["hop"], dim_f=w["dim_f"],
                                                 dim_t=w["dim_t"], overlap=w["overlap"]), length)


def _mask_floats_per_chunk(w):
    if w["arch"] == "roformer":
        pkg = load_pkg()
        sizes, _ = pkg.bands.mel_bands() if w["bands"] == "mel" else pkg.bands.bs_bands()
        return int(sizes.sum()) * 2 * 2 * (w["chunk"] // w["hop"] + 1)
    if w["arch"] == "htdemucs":
        return w["sources"] * 4 * 2048 * ((w["segment"] + 1023) // 1024)
    return 4 * w["dim_f"] * w["dim_t"]


def _host_mask(w, n_chunks):
    """Masks for the first n_chunks chunks (the CPU legs only touch the chunks they time)."""
    rng = np.random.default_rng(w["seed"] + 1000)
    n = n_chunks * _mask_floats_per_chunk(w)
    return (w["sigma"] * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)


# ---- the request-side conversions (workload io48k) ----------------------------------------
def _io_inputs(w):
    n = w["seconds"] * w["rate"]
    x = synth_audio(w["seed"], n)                          # planar, at the request's rate
    inter = np.ascontiguousarray(x.T).reshape(-1)           # the request's interleaved frames
    return n, inter


def run_ours_io(args, w, rank, world, local_rank):
    import torch
    pkg = load_pkg()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    eng = pkg.Engine(local_rank)
    n, inter = _io_inputs(w)
    rows = w["stems"] * 2
    m = pkg.resampled_length(n, w["rate"], SR)
    d_in = torch.from_numpy(inter).to(dev)
    d_prep = torch.empty((2, m), device=dev)
    d_stems = torch.randn((rows, m), device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    d_back = torch.empty((rows, n), device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        eng.prepare_input(d_in, 2, w["rate"], out=d_prep, stream=stream)
        eng.restore_output(d_stems, SR, w["rate"], n, out=d_back, stream=stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local_rank])

    def timed(fn, k):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clk:
            e0.record(stream)
            for _ in range(k):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        return e0.elapsed_time(e1) / k, clk

    ms, clk = timed(step, args.steps)
    remeasured = False
    if clk.rejected():
        ms, clk = timed(step, args.steps)
        remeasured = True
    ms = pkg.sharding.max_over_ranks(ms, device=dev)
    prep_ms, _ = timed(lambda: eng.prepare_input(d_in, 2, w["rate"], out=d_prep, stream=stream), args.steps)
    # end to end: the request's frames from pinned host memory in, the stems' frames out
    h_in = torch.from_numpy(inter).pin_memory()
    h_stems = d_stems.cpu().pin_memory()
    h_back = torch.empty((rows, n)).pin_memory()

    def e2e_step():
        d_in.copy_(h_in, non_blocking=True)
        d_stems.copy_(h_stems, non_blocking=True)
        step()
        h_back.copy_(d_back, non_blocking=True)
    e2e_ms, _ = timed(e2e_step, max(1, min(args.steps, 10)))
    e2e_ms = pkg.sharding.max_over_ranks(e2e_ms, device=dev)
    bytes_step = 4 * (2 * n + 2 * m + rows * m + rows * n)
    peak, peak_kind = measured_peak()
    achieved = bytes_step / (ms / 1e3) / 1e9
    audio_s = w["seconds"] * world
    eng.close()
    if rank != 0:
        return None
    return {
        "metric": "audio_seconds_per_second", "value": audio_s / (ms / 1e3), "unit": "audio-s/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded sines + noise at 48 kHz; N(0, 1) stems)",
        "config": {"workload": args.workload, "desc": w["desc"], "rows_back": rows, "samples_in": n,
                   "samples_model": m, "l2": "inputs larger than L2 (no flush needed)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "kernel": "resample_kernel", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                     "algorithmic_bytes_per_step": bytes_step, "prepare_ms": prep_ms,
                     "note": "the kernel does ~70 double-precision taps per output sample; it is bound by "
                             "FP64 issue, not by HBM"},
        "clocks": dict(clk.summary(), remeasured=remeasured),
        "e2e": {"value": audio_s / (e2e_ms / 1e3), "unit": "audio-s/s",
                "h2d_bytes_per_step": 4 * (2 * n + rows * m), "d2h_bytes_per_step": 4 * rows * n},
        "gpu_launches": 2 * args.steps,
    }


def _vr_setup(w):
    import oracle
    p = oracle.vr_params(w["bands"], bins=w["bins"], pre_start=w["pre"][0], pre_stop=w["pre"][1])
    rates = sorted({x["sr"] for x in w["bands"]})
    firs = {(s, d): oracle.vr_fir(s, d) for s in rates for d in rates if s != d}
    bands = [dict(sample_rate=x["sr"], hop=x["hop"], n_fft=x["nfft"], crop_start=x["start"], crop_stop=x["stop"],
                  hpf_start=x.get("hp_start", -1), hpf_stop=x.get("hp_stop", -1), lpf_start=x.get("lp_start", -1),
                  lpf_stop=x.get("lp_stop", -1)) for x in w["bands"]]
    return p, firs, bands


def cpu_vr(w, seconds):
    """The VR path restated in C (oracle, one thread, as the reference runs it) on a sample."""
    import oracle
    p, _, _ = _vr_setup(w)
    n = int(seconds * SR)
    T = oracle.vr_n_frames(p, n)
    mask = np.random.default_rng(11).uniform(0, 1, (2, w["bins"] + 1, T)).astype(np.float32)
    mix = synth_audio(w["seed"], n)
    t0 = time.perf_counter()
    oracle.vr_separate(p, mix, mask)
    return time.perf_counter() - t0, "port"


def run_ours_vr(args, w, rank, world, local_rank):
    import torch
    pkg = load_pkg()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    eng = pkg.Engine(local_rank)
    _, firs, bands = _vr_setup(w)
    n = w["seconds"] * SR
    plan = eng.plan_vr(n, bands, firs, bins=w["bins"], pre_filter_start=w["pre"][0], pre_filter_stop=w["pre"][1])
    mix_h = synth_audio(w["seed"] + 7 * rank, n)
    d_mix = torch.from_numpy(mix_h).to(dev)
    d_mask = torch.rand(plan.mask_shape, device=dev, generator=torch.Generator(device=dev).manual_seed(12))
    d_out = torch.empty(plan.out_shape, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        plan.separate(d_mix, d_mask, d_out, stream=stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local_rank])

    def timed(fn, k):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clk:
            e0.record(stream)
            for _ in range(k):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        return e0.elapsed_time(e1) / k, clk

    ms, clk = timed(step, args.steps)
    remeasured = False
    if clk.rejected():
        ms, clk = timed(step, args.steps)
        remeasured = True
    ms = pkg.sharding.max_over_ranks(ms, device=dev)
    h_mix = torch.from_numpy(mix_h).pin_memory()
    h_mask = d_mask.cpu().pin_memory()
    h_out = torch.empty(plan.out_shape).pin_memory()

    def e2e_step():
        d_mix.copy_(h_mix, non_blocking=True)
        d_mask.copy_(h_mask, non_blocking=True)
        step()
        h_out.copy_(d_out, non_blocking=True)
    e2e_ms, _ = timed(e2e_step, max(1, min(args.steps, 10)))
    e2e_ms = pkg.sharding.max_over_ranks(e2e_ms, device=dev)
    mask_b = 4 * d_mask.numel()
    bytes_step = 4 * 2 * n + mask_b + 4 * 4 * n
    peak, peak_kind = measured_peak()
    achieved = bytes_step / (ms / 1e3) / 1e9
    # front: resamples between the B distinct rates, B STFTs, the assembly; each stem: B band
    # parts, B iSTFT back + combine, B - 1 sums, B - 1 resamples, the crop
    launches = 2 * len(bands) + 2 * (5 * len(bands) - 1)
    plan.close()
    eng.close()
    if rank != 0:
        return None
    return {
        "metric": "audio_seconds_per_second", "value": w["seconds"] * world / (ms / 1e3), "unit": "audio-s/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded sines + noise; U(0, 1) masks standing in for the network)",
        "config": {"workload": args.workload, "desc": w["desc"], "frames": plan.n_frames,
                   "mask_bytes_per_track": mask_b, "l2": "inputs larger than L2 (no flush needed)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "kernel": "the VR path (all its kernels)", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                     "algorithmic_bytes_per_step": bytes_step},
        "clocks": dict(clk.summary(), remeasured=remeasured),
        "e2e": {"value": w["seconds"] * world / (e2e_ms / 1e3), "unit": "audio-s/s",
                "h2d_bytes_per_step": 4 * 2 * n + mask_b, "d2h_bytes_per_step": 4 * 4 * n},
        "gpu_launches": launches * args.steps,
    }


def cpu_io(w, seconds):
    """The reference's resample_planar (compiled, one thread as libstems calls it) on a
    `seconds` sample of the io48k workload: both directions; returns (seconds taken, kind)."""
    import oracle
    R = oracle.ref_lib()
    kind = "reference" if R is not None else "port"
    n = int(seconds * w["rate"])
    x = synth_audio(w["seed"], n)
    stems = np.random.default_rng(5).standard_normal((w["stems"] * 2, oracle.resampled_length(n, w["rate"], SR)),
                                                     dtype=np.float32)
    t0 = time.perf_counter()
    oracle.prepare_input(np.ascontiguousarray(x.T).reshape(-1), True, 2, w["rate"], 2, SR, impl=R)
    oracle.restore_output(stems, SR, w["rate"], n, impl=R)
    return time.perf_counter() - t0, kind


# ---- our arm -----------------------------------------------------------------------------
def run_ours(args, w, rank, world, local_rank, name=None, steps=None, warmup=None, split=None, e2e_steps=None):
    """One workload through the C ABI on this rank's GPU: the device-resident step (the
    headline value), the kernel timing behind the roofline, and end to end from pinned host
    memory. Returns rank 0's line (None elsewhere). Every rank takes the same collective steps."""
    import torch
    import torch.distributed as dist

    name = name or args.workload
    steps = steps or args.steps
    warmup = max(3, warmup or args.warmup)
    split = args.split_track if split is None else split
    pkg = load_pkg()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    eng = pkg.Engine(local_rank)
    length = w["seconds"] * SR
    plan = make_plan(pkg, eng, w, length)
    mix_h = synth_audio(w["seed"] + 7 * rank, length)
    d_mix = torch.from_numpy(mix_h).to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    d_mask = torch.randn(plan.mask_floats, generator=gen, device=dev, dtype=torch.float32).mul_(w["sigma"])
    d_out = torch.empty(plan.out_shape, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x):
        return pkg.sharding.max_over_ranks(x, device=dev)

    # tracks this rank separates per step: one replica of the single-track workloads, or its
    # round-robin share of a batch (the buffers are reused; the kernels do not look at values)
    n_tracks = w.get("tracks", world)
    mine = len(pkg.sharding.tracks_for_rank(n_tracks, rank, world))
    split = split and "tracks" not in w
    if split:   # one track, its output samples split across the ranks (strong scaling)
        n_tracks = 1
        part = pkg.sharding.sample_range_for_rank(length, rank, world)

    def step():
        if split:
            plan.separate_part(d_mix, d_mask, d_out, part[0], part[1], stream=stream)
            return
        for _ in range(mine):
            plan.separate(d_mix, d_mask, d_out, stream=stream)

    def timed_region():
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clk:
            e0.record(stream)
            for _ in range(steps):
                step()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps, clk

    ms, clk = timed_region()
    remeasured = False
    if clk.rejected():
        ms, clk = timed_region()
        remeasured = True
    ms = max_over_ranks(ms)

    # Kernel-level timing on the launching stream (events recorded inside the engine).
    eng.set_profiling(True)
    prep, fused, comb = [], [], []
    for _ in range(max(3, min(steps, 20))):
        plan.separate(d_mix, d_mask, d_out, stream=stream)
        a, b, c, n_launch = plan.last_timing_detail()
        prep.append(a)
        fused.append(b)
        comb.append(c)
    eng.set_profiling(False)
    prep_ms = statistics.mean(prep)
    fused_ms = statistics.mean(fused)
    combine_ms = statistics.mean(comb)

    # End to end through the public host-buffer entry point (pinned host memory): one track per
    # e2e step on every rank.
    h_mix = torch.from_numpy(mix_h).pin_memory()
    h_mask = d_mask.cpu().pin_memory()
    h_out = torch.empty(plan.out_shape, dtype=torch.float32).pin_memory()
    e2e_steps = e2e_steps or max(1, min(steps, 10))
    plan.separate_host_ptr(h_mix.data_ptr(), h_mask.data_ptr(), h_out.data_ptr(), stream=stream.cuda_stream)
    torch.cuda.synchronize(dev)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        plan.separate_host_ptr(h_mix.data_ptr(), h_mask.data_ptr(), h_out.data_ptr(), stream=stream.cuda_stream)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    e2e_s = max_over_ranks(e2e_s)
    barrier()
    # the same bytes copied and nothing else: the PCIe bound of the e2e number
    d_in_mix, d_in_mask = torch.empty_like(h_mix, device=dev), torch.empty_like(h_mask, device=dev)
    d_res = torch.empty(plan.out_shape, dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            d_in_mix.copy_(h_mix, non_blocking=True)
            d_in_mask.copy_(h_mask, non_blocking=True)
            h_out.copy_(d_res, non_blocking=True)
            stream.synchronize()
    copy_s = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
    del d_in_mix, d_in_mask, d_res
    barrier()

    audio_s = w["seconds"] * n_tracks
    value = audio_s / (ms / 1e3)
    peak, peak_kind = measured_peak()
    kname, fbytes = kernel_algorithmic_bytes(plan, w)
    achieved = fbytes / (fused_ms / 1e3) / 1e9
    traffic = profiled_traffic(kname, name)
    h2d = 4 * (plan.n_channels * plan.n_samples + plan.mask_floats)
    d2h = 4 * plan.out_floats
    line = None
    if rank == 0:
        config = workload_config(w, name, world, split)
        assert (config["chunks_per_track"], config["frames_per_chunk"]) == (plan.n_chunks, plan.n_frames), config
        line = {
            "metric": "audio_seconds_per_second", "value": value, "unit": "audio-s/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if split else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded sines + noise; N(0, sigma) masks standing in for the network)",
            "config": config,
            "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "algorithmic_bytes_per_launch": fbytes,
                         "fused_ms": fused_ms, "combine_ms": combine_ms, "prep_ms": prep_ms},
            "path": {"algorithmic_bytes_per_step": path_algorithmic_bytes(plan, w),
                     "gbs": path_algorithmic_bytes(plan, w) / (ms / 1e3) / 1e9},
            "clocks": dict(clk.summary(), remeasured=remeasured),
            "e2e": {"value": w["seconds"] * world / e2e_s, "unit": "audio-s/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "per_gpu_h2d_gbs": h2d / e2e_s / 1e9, "aggregate_h2d_gbs": world * h2d / e2e_s / 1e9,
                    "tracks_per_e2e_step": world,
                    "copies_only": w["seconds"] * world / copy_s,
                    "copies_only_note": "the same host<->device copies alone, no kernels: the PCIe bound"},
            "gpu_launches": n_launch * steps * mine,
        }
    plan.close()
    eng.close()
    return line


BASELINE_WORKLOADS = ("cfg0", "cfg1", "cfg2", "cfg3", "cfg4")


def workload_summary(line):
    """The per-workload record of the default bench line's `workloads` object."""
    keep = {"value": line["value"], "unit": line["unit"], "ms_per_step": line["ms_per_step"], "steps": line["steps"],
            "kernel": line["roofline"]["kernel"], "frac": line["roofline"]["frac"],
            "fused_ms": line["roofline"]["fused_ms"], "e2e": line["e2e"]["value"],
            "e2e_copies_only": line["e2e"]["copies_only"], "clocks_sm_mhz": line["clocks"].get("sm_mhz"),
            "config": line["config"]}
    if "cpu_baseline" in line:
        keep["cpu_baseline"] = line["cpu_baseline"]
    return keep


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg1", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="only the headline workload (no `workloads` / `strong` records)")
    ap.add_argument("--split-track", action="store_true",
                    help="one track per step, its output samples split across the ranks (strong scaling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    w = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, w, rank)

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        # stdout carries the one JSON line: keep NCCL's version banner off it unless asked for
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    extra = {}
    try:
        line = {"io": run_ours_io, "vr": run_ours_vr}.get(w["arch"], run_ours)(args, w, rank, world, local_rank)
        headline = args.workload in BASELINE_WORKLOADS and not args.split_track and not args.no_extra
        if headline:
            # the other BASELINE configurations in the same run (fewer steps), and one track of
            # cfg2 split by samples over this run's GPUs (strong scaling; at one GPU, one track)
            if world == 1:
                for name in BASELINE_WORKLOADS:
                    if name == args.workload:
                        continue
                    wx = WORKLOADS[name]
                    r = run_ours(args, wx, rank, world, local_rank, name=name, steps=min(args.steps, 10),
                                 warmup=3, split=False, e2e_steps=3)
                    if rank == 0 and not args.no_cpu_baseline:
                        r["cpu_baseline"] = cpu_baseline_record(wx, min_s=5.0, single=False)
                    extra[name] = r
            strong = run_ours(args, WORKLOADS["cfg2"], rank, world, local_rank, name="cfg2",
                              steps=min(args.steps, 10), warmup=3, split=True, e2e_steps=2)
            extra["strong"] = strong
    finally:
        if world > 1:
            dist.barrier(device_ids=[local_rank])
            dist.destroy_process_group()
    if rank != 0:
        return 0
    if w["arch"] in ("io", "vr"):
        if world == 1 and not args.no_cpu_baseline:
            dt, kind, reps = cpu_repeat(lambda: (cpu_io if w["arch"] == "io" else cpu_vr)(w, 5.0))
            line["cpu_baseline"] = {"value": 5.0 / dt, "unit": "audio-s/s", "cores": 1, "kind": kind,
                                    "sample": f"5 s of the {w['seconds']} s input (one thread, as the reference "
                                              f"runs it), timed {reps} times", **cpu_info()}
        print(json.dumps(line))
        return 0
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_record(w)
    if extra:
        line["workloads"] = {n: workload_summary(r) for n, r in extra.items() if n != "strong"}
        st = extra["strong"]
        line["strong"] = {"workload": "cfg2", "value": st["value"], "unit": st["unit"], "n_gpus": world,
                          "ms_per_step": st["ms_per_step"], "scaling": "strong",
                          "parallelism": st["config"]["parallelism"],
                          "note": "one 180 s BS-RoFormer track per step, its output samples split across the GPUs "
                                  "(the chunks at a range's edge run on both neighbours; nothing is exchanged)"}
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
