"""Benchmark of the AudioVAE2 decoder hot path on B200.

Workloads (``--workload``; the default is what the headline line reports):

  stream40ms  every GPU decodes 512 independent streams (the per-GPU shard of
              cfg5's 4096 streams on 8 GPUs) on 1-frame (40 ms, 1920-sample)
              chunks with carried history, bf16 plan. One step = one chunk for
              all 512 streams (23 kernel launches). Weak scaling.
  cfg3        256 streams x 2-frame (80 ms) chunks per step, bf16. Weak scaling.
  int8        stream40ms's shape on the int8 (W8A8) plan (cfg5's precision).
  cfg1        batch decode of one clip [1,64,25] (1 s of audio) per step.
  cfg4        batch decode of 64 clips [1,64,750] (30 s each) per step, the
              clips sharded over the ranks: strong scaling.

Latents are seeded N(0,1) (one seed per stream or clip) standing in for the
reference's speech latents; coefficients are the seeded random init.

Reported (one JSON line, rank 0):
  value     aggregate audio-s/s, inputs resident in HBM, device time (CUDA
            events around the K timed steps, max over ranks);
  e2e       the same metric through the public API (host numpy chunks in, host
            audio out: ``CUDADecoder.decode_streams`` / ``decode_many``), host
            wall time, max over ranks; plus p50/p99 step latency;
  tensor_roofline  the step's 706.7 MFLOP per latent frame of dense
            contraction (the 25 GEMMs) over the device and e2e times, against
            the measured sustained bf16 peak;
  roofline  the longest kernel's algorithmic FLOPs and bytes per launch over
            its CUDA-event duration against MEASURED_PEAKS.json, with a
            CUDA-core (FP32 / SFU) ceiling for the kernels whose work is not a
            contraction, and the ncu DRAM traffic of that launch
            (bench_traffic.json) when the workload matches the capture;
  gpu_launches  kernel launches in the timed region, counted from a CUDA graph
            capture of one step;
  cpu_baseline  the fp32 oracle port of the reference decoder (int8: the int8
            recipe oracle) on the host cores, on a bounded sample.

``--impl reference`` times the reference decoder's CPU implementation (the
oracle port of ``mps_decoder.py``; rank 0 only) on a bounded sample of the
same workload and prints the same line with ``"impl": "reference"``.
``--ingest-ncu CSV`` turns an ncu launch list of one default step
(``gpu__time_duration.sum``, ``dram__bytes_read.sum``, ``dram__bytes_write.sum``)
into bench_traffic.json.
"""
from __future__ import annotations

import argparse
import csv
import ctypes as ct
import json
import os
import subprocess
import sys
import threading
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "fast-audiovae_b200"))
sys.path.insert(0, str(ROOT))

FRAME_SECONDS = 1920 / 48000
RATES = (8, 6, 5, 2, 2, 2)
FLOPS_PER_FRAME = 706_740_224  # 2 x 353,370,112 MAC of the 25 GEMMs per latent frame
TRAFFIC_FILE = ROOT / "bench_traffic.json"


def fused_stage(i, precision=0):
    """Stages whose three residual units and the next conv's planes run as one
    fused kernel: 2, 3 and 4 (bf16 units), stage 4 only in the int8 plan."""
    return i == 4 or (i in (2, 3) and precision == 0)


def kernel_names(precision=0):
    """Kernels of one step, in launch order of the per-layer timing: the stem,
    per stage a transposed conv and three residual units (``stageI.units`` for
    a fused stage), stage 5's transposed conv and the fused tail (three
    residual units + final conv)."""
    names = ["stem"]
    for i in range(5):
        names.append(f"stage{i}.transpose")
        names += [f"stage{i}.units"] if fused_stage(i, precision) else [f"stage{i}.res{j}" for j in range(3)]
    return names + ["stage5.transpose", "stage5.tail"]


@dataclass(frozen=True)
class Workload:
    kind: str          # "stream" or "batch"
    metric: str
    text: str
    streams: int = 0   # stream: streams per GPU
    frames: int = 1    # stream: frames per chunk; batch: frames per clip
    clips: int = 0     # batch: clips per step (all ranks together when strong)
    chunk: int = 0     # batch: frames per internal step
    precision: int = 0
    strong: bool = False


WORKLOADS = {
    "stream40ms": Workload("stream", "aggregate audio-s/s (RTF^-1), 40 ms streaming chunks",
                           "stream40ms: {S} streams/GPU x 1-frame (40 ms) chunks, carried history", streams=512),
    "cfg3": Workload("stream", "aggregate audio-s/s (RTF^-1), 80 ms streaming chunks",
                     "cfg3: {S} streams/GPU x 2-frame (80 ms) chunks, carried history", streams=256, frames=2),
    "int8": Workload("stream", "aggregate audio-s/s (RTF^-1), 40 ms streaming chunks, int8 W8A8 plan",
                     "int8: {S} streams/GPU x 1-frame (40 ms) chunks on the int8 (W8A8) plan", streams=512,
                     precision=1),
    "cfg1": Workload("batch", "aggregate audio-s/s (RTF^-1), batch decode of 1 s clips",
                     "cfg1: batch decode of {C} clip(s) [1,64,25] per GPU per step", frames=25, clips=1, chunk=25),
    "cfg4": Workload("batch", "aggregate audio-s/s (RTF^-1), batch decode of 30 s clips",
                     "cfg4: batch decode of 64 clips [1,64,750] per step, sharded over the GPUs ({C} on this rank)",
                     frames=750, clips=64, chunk=128, strong=True),
}


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="stream40ms")
    p.add_argument("--streams", type=int, default=0, help="override the stream workloads' streams per GPU")
    p.add_argument("--cpu-seconds", type=float, default=8.0, help="budget per CPU baseline leg")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--ingest-ncu", metavar="CSV", help="write bench_traffic.json from an ncu launch list")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        d = json.loads(path.read_text())
        mhz = d.get("sm_max_mhz", 1965.0)
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "sm_mhz": mhz,
                "source": "measured (MEASURED_PEAKS.json; bf16 sustained)"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "sm_mhz": 1965.0, "source": "fallback"}


# ------------------------------------------------------------------ algorithmic cost
def layer_costs(precision=0):
    """Per kernel of ``kernel_names(precision)``, per latent frame: algorithmic FLOPs (2*MAC
    of the contractions), HBM bytes of this design's data layout (each
    activation read and written once), CUDA-core work (FP32 instructions and
    special-function sines), and per-launch weight bytes and per-stream history
    bytes (read + write).

    Layout (bf16 plan): a transposed conv reads its input as split-bf16 planes
    (hi + lo, 4 B per element) twice (as they are, and one time step later for
    its second tap) and writes y in fp32 (plus Snake_pre(y) at stages 0-1,
    whose units read it); stages 0-1's units read Snake_pre(y), write their
    f16 operand once and read it back. A fused stage (2-4) reads its input y
    once and writes the next conv's two plane copies; the fused stage-5 tail
    reads its input once and writes audio; their intermediates stay on chip.
    (The int8 plan's stages 2-3 run their units as per-layer launches.)

    CUDA-core work per element of a residual unit: two Snakes (4 FP32 + 1 sine
    each), the depthwise k=7 tap chain with its bias (8) and the skip/bias add
    (2); the unit feeding a transposed conv adds the stage affine, the next
    Snake and the bf16 split (9 FP32 + 1 sine)."""
    out = []
    n = 1  # rows per frame at the current layer input
    out.append(dict(flops=2 * 2048 * 64, act=64 * 4 + 2048 * 8, weights=2048 * 64 * 4,
                    hist=6 * 64 * 4 * 2 + 2048 * 4 * 2, fp32=2048 * 10 + 64 * 8, sfu=2048))
    cin = 2048
    for i, s in enumerate(RATES):
        cout = cin // 2
        y_only = i == 5 or fused_stage(i, precision)
        out_elems = n * s * cout
        out.append(dict(flops=2 * cin * cout * 2 * s * n, act=n * cin * 8 + out_elems * (4 if y_only else 8),
                        weights=cin * cout * 2 * s * 4, hist=0,
                        fp32=out_elems * (1 if y_only else 6), sfu=0 if y_only else out_elems))
        n *= s
        if i == 5:
            rows = n
            out.append(dict(flops=rows * 3 * 2 * cout * cout, act=rows * (cout * 4 + 4), weights=3 * cout * cout * 2,
                            hist=(6 + 18 + 54 + 6) * cout * 4 * 2, fp32=rows * 2090, sfu=rows * 225))
            break
        elems = n * cout
        if fused_stage(i, precision):
            out.append(dict(flops=3 * 2 * cout * cout * n, act=elems * (4 + 8), weights=3 * cout * cout * 2,
                            hist=(6 + 18 + 54) * cout * 4 * 2 + cout * 4 * 2,
                            fp32=elems * (3 * 18 + 9), sfu=elems * (3 * 2 + 1)))
            cin = cout
            continue
        for j, d in enumerate((1, 3, 9)):
            last = j == 2
            if precision == 0 and i >= 2:
                act = elems * (4 + (8 if last else 4))
            else:
                act = elems * (4 + 2 + 2 + 4 + 8)
            out.append(dict(flops=2 * cout * cout * n, act=act, weights=cout * cout * 2,
                            hist=6 * d * cout * 4 * 2 + (cout * 4 * 2 if last else 0),
                            fp32=elems * (18 + (9 if last else 0)), sfu=elems * (2 + (1 if last else 0))))
        cin = cout
    assert len(out) == len(kernel_names(precision))
    return out


def pipe_peaks(pk):
    """Nominal CUDA-core issue rates at the measured maximum SM clock: 148 SMs x
    128 FP32 lanes, and 148 x 16 special-function (sine) results per clock."""
    hz = pk["sm_mhz"] * 1e6
    return {"fp32": 148 * 128 * hz, "sfu": 148 * 16 * hz}


def stored_traffic(workload, streams, frames):
    """DRAM bytes (read + write) per launch of each kernel from bench_traffic.json,
    when that capture was taken on this workload and shape."""
    if not TRAFFIC_FILE.is_file():
        return None
    d = json.loads(TRAFFIC_FILE.read_text())
    if d.get("workload") != workload or d.get("streams") != streams or d.get("frames") != frames:
        return None
    return d


def roofline(layer_ms, frames_per_launch, streams, pk, workload, frames, precision):
    costs = layer_costs(precision)
    names = kernel_names(precision)
    dom = int(np.argmax(layer_ms))
    c = costs[dom]
    flops = c["flops"] * frames_per_launch
    bytes_ = c["act"] * frames_per_launch + c["weights"] + c["hist"] * streams
    pp = pipe_peaks(pk)
    fp32, sfu = c["fp32"] * frames_per_launch, c["sfu"] * frames_per_launch
    t_tensor = flops / (pk["tflops"] * 1e12)
    t_hbm = bytes_ / (pk["hbm_gbs"] * 1e9)
    t_core = max(fp32 / pp["fp32"], sfu / pp["sfu"])
    sec = layer_ms[dom] / 1e3
    if t_tensor >= t_hbm:
        achieved, peak, unit, bound = flops / sec / 1e12, pk["tflops"], "TFLOP/s", "tensor"
    else:
        achieved, peak, unit, bound = bytes_ / sec / 1e9, pk["hbm_gbs"], "GB/s", "hbm"
    binding = max((t_tensor, "tensor"), (t_hbm, "hbm"), (t_core, "cuda_core"))[1]
    tr = stored_traffic(workload, streams, frames)
    traffic = tr["layers"].get(names[dom]) if tr else None
    return {"kernel": names[dom], "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum ({TRAFFIC_FILE.name}: "
                              f"{tr['source']})" if traffic else None,
            "binding": binding,
            "cuda_core": {"fp32_instr": fp32, "sines": sfu, "ceiling_ms": round(1e3 * t_core, 4),
                          "frac": round(t_core / sec, 4),
                          "peaks": "nominal: 148 SMs x 128 FP32 lanes and x 16 SFU results per clock at "
                                   f"{pk['sm_mhz']:.0f} MHz"},
            "share_of_step": round(float(layer_ms[dom] / np.sum(layer_ms)), 4),
            "algorithmic_per_launch": {"flops": flops, "bytes": bytes_}, "peak_source": pk["source"],
            "layer_ms": {names[i]: round(float(v), 4) for i, v in enumerate(layer_ms)}}


def tensor_roofline(frames, dev_s, e2e_s, pk):
    """The whole step's dense-contraction rate (706.7 MFLOP per latent frame)
    against the measured sustained bf16 tensor-core peak."""
    dev = frames * FLOPS_PER_FRAME / dev_s / 1e12
    e2e = frames * FLOPS_PER_FRAME / e2e_s / 1e12
    return {"flops_per_frame": FLOPS_PER_FRAME, "device_tflops": round(dev, 2),
            "device_frac": round(dev / pk["tflops"], 4), "e2e_tflops": round(e2e, 2),
            "e2e_frac": round(e2e / pk["tflops"], 4), "peak_tflops": pk["tflops"], "peak_source": pk["source"]}


def kernel_ms(layer_ms26, precision=0):
    """Per-kernel durations (``kernel_names(precision)``) from the 26 per-layer
    event intervals of ``fav_step_profile``: interval 0 is the stem, 1 + 4i
    stage i's transposed conv, 2 + 4i + j its residual unit j (a fused stage's
    kernel spans its three), 21 stage 5's conv and 22-25 the fused tail."""
    v = np.asarray(layer_ms26, dtype=np.float64)
    out = [v[0]]
    for i in range(5):
        out.append(v[1 + 4 * i])
        units = v[2 + 4 * i:5 + 4 * i]
        out += [units.sum()] if fused_stage(i, precision) else list(units)
    return np.array(out + [v[21], v[22:].sum()])


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons of one GPU while the timed region runs:
    read through NVML (read-only queries) every 5 ms from a background thread,
    so a timed region of tens of milliseconds still gets several samples;
    ``nvidia-smi -lms 100`` is the fallback when NVML cannot be used."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index):
        self.proc = self.thread = None
        self.rows, self.done = [], threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            handle = self._handle(pynvml, index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))

            def run():
                while not self.done.is_set():
                    self.rows.append((float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)),
                                      int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))))
                    self.done.wait(0.005)
            self.rows.append((float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)),
                              int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))))
            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:  # no NVML binding or device: the nvidia-smi loop instead
            self.rows = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    @staticmethod
    def _handle(pynvml, index):
        """NVML handle of CUDA device ``index`` (by UUID; the index as listed
        in CUDA_VISIBLE_DEVICES otherwise)."""
        import torch
        try:
            return pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(torch.cuda.get_device_properties(index).uuid)).encode())
        except Exception:
            visible = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
            if index < len(visible) and visible[index].strip().isdigit():
                index = int(visible[index])
            return pynvml.nvmlDeviceGetHandleByIndex(index)

    def stop(self):
        if self.thread is not None:
            self.done.set()
            self.thread.join(timeout=5)
            rows = list(self.rows)
            busy = [mhz for mhz, _ in rows if mhz > 0]
            reasons = sorted({name for _, bits in rows for name, bit in self.REASONS if bits & bit})
            return {"sm_mhz": float(np.median(busy)) if busy else None, "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(rows), "source": "nvml, 5 ms"}
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, col in (("hw_slowdown", 5), ("hw_thermal_slowdown", 6), ("sw_thermal_slowdown", 7),
                              ("sw_power_cap", 8)):
                if r[col].strip() == "Active":
                    reasons.add(name)
        busy = [v for v in sm if v > 0]
        return {"sm_mhz": float(np.median(busy)) if busy else None, "sm_max_mhz": float(rows[0][2]),
                "reasons": sorted(reasons), "samples": len(rows), "source": "nvidia-smi, 100 ms"}


# ------------------------------------------------------------------ CPU legs
def cpu_stream_rate(streams, budget_s, threads, frames=1, int8=False):
    """Oracle port (fp32 reference decoder, or the int8 recipe oracle) streaming
    ``frames``-frame chunks for ``streams`` streams on CPU: (audio-s/s, frames, s)."""
    import torch
    from fast_audiovae import weights as W
    from oracle.decoder import Decoder
    torch.set_num_threads(threads)
    if int8:
        from oracle.int8_recipe import Int8RecipeDecoder
        dec = Int8RecipeDecoder(W.seeded_weights(0))
    else:
        dec = Decoder(W.seeded_weights(0))
    latents = [W.seeded_latents(s, 4096) for s in range(streams)]
    states = [None] * streams
    for s in range(streams):  # warm-up step
        _, states[s] = dec.decode(latents[s][..., :frames], states[s])
    done, t0, step = 0, time.perf_counter(), 1
    while True:
        for s in range(streams):
            _, states[s] = dec.decode(latents[s][..., step * frames:(step + 1) * frames], states[s])
            done += frames
        step += 1
        el = time.perf_counter() - t0
        if el >= budget_s or step * frames >= 4000:
            break
    return done * FRAME_SECONDS / el, done, el


def cpu_clip_rate(frames, budget_s, threads):
    """fp32 oracle batch decode of whole ``frames``-frame clips on CPU, repeated
    within the budget (at least once): (audio-s/s, frames, s)."""
    import torch
    from fast_audiovae import weights as W
    from oracle.decoder import Decoder
    torch.set_num_threads(threads)
    dec = Decoder(W.seeded_weights(0))
    dec.decode(W.seeded_latents(0, min(frames, 4)))  # warm-up
    done, t0, k = 0, time.perf_counter(), 0
    while True:
        dec.decode(W.seeded_latents(k, frames))
        done += frames
        k += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return done * FRAME_SECONDS / el, done, el


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(wl, budget):
    cores = host_cores()
    if wl.kind == "stream":
        sample_streams = 1 if wl.precision else 8
        rate, done, el = cpu_stream_rate(sample_streams, budget, cores, wl.frames, wl.precision == 1)
        rate1, _, _ = cpu_stream_rate(1 if wl.precision else 2, budget, 1, wl.frames, wl.precision == 1)
        what = "int8 recipe oracle" if wl.precision else "fp32 oracle decoder"
        sample = (f"{what}, {sample_streams} stream(s) x {done // sample_streams} {wl.frames}-frame chunks with "
                  f"carried history, {cores} threads (~{el:.0f} s)")
    else:
        frames = min(wl.frames, 250)
        rate, done, el = cpu_clip_rate(frames, budget, cores)
        rate1, _, _ = cpu_clip_rate(frames, budget, 1)
        sample = f"fp32 oracle decoder, {done // frames} clip(s) of {frames} frames, {cores} threads (~{el:.0f} s)"
    return {"value": round(rate, 3), "unit": "audio-s/s", "cores": cores, "kind": "port", "sample": sample,
            "value_1thread": round(rate1, 3)}


# ------------------------------------------------------------------ distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def dist_max(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ reference arm
def run_reference(args, wl, world, rank):
    if rank != 0:
        return
    cores = host_cores()
    per_step = max(1.0, min(20.0, 120.0 / max(1, args.steps)))
    total_frames, total_time = 0, 0.0
    if wl.kind == "stream":
        streams = 1 if wl.precision else min(wl.streams, 8)
        for _ in range(args.warmup):
            cpu_stream_rate(streams, 0.5, cores, wl.frames, wl.precision == 1)
        for _ in range(args.steps):
            _, done, el = cpu_stream_rate(streams, per_step, cores, wl.frames, wl.precision == 1)
            total_frames += done
            total_time += el
        sample = f"{streams} streams x {wl.frames}-frame chunks with carried history, ~{per_step:.1f} s per step"
    else:
        frames = min(wl.frames, 250)
        for _ in range(min(args.warmup, 1)):
            cpu_clip_rate(min(frames, 25), 0.1, cores)
        for _ in range(args.steps):
            _, done, el = cpu_clip_rate(frames, per_step, cores)
            total_frames += done
            total_time += el
        sample = f"clips of {frames} frames decoded whole, ~{per_step:.1f} s per step"
    value = total_frames * FRAME_SECONDS / total_time
    line = {"impl": "reference", "metric": wl.metric, "value": round(value, 3), "unit": "audio-s/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * total_time / args.steps, 3), "higher_is_better": True,
            "scaling": "strong" if wl.strong else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": args.workload,
                       "implementation": ("reference int8 recipe (precision.cpp restated, torch CPU)" if wl.precision
                                          else "reference fp32 decoder (mps_decoder.py restated, torch CPU)")},
            "cpu_baseline": {"value": round(value, 3), "unit": "audio-s/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def count_kernels(torch, launch):
    """Kernel launches of one call of ``launch(stream_handle)``, counted from a
    CUDA graph capture of it (kernel nodes)."""
    from cuda.bindings import runtime as rt
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph(keep_graph=True)  # captured, never instantiated or run
    with torch.cuda.graph(graph, stream=side):
        launch(ct.c_void_p(side.cuda_stream))
    torch.cuda.current_stream().wait_stream(side)
    err, _, n = rt.cudaGraphGetNodes(graph.raw_cuda_graph(), 0)
    err, nodes, n = rt.cudaGraphGetNodes(graph.raw_cuda_graph(), n)
    kernels = 0
    for node in nodes:
        err, kind = rt.cudaGraphNodeGetType(node)
        kernels += kind == rt.cudaGraphNodeType.cudaGraphNodeTypeKernel
    del graph
    return int(kernels)


def profile_layers(lib, _native, plan, S, F, z_dev, audio, ws, ws_bytes, status, stream, precision, reps=20, warm=3):
    """Per-kernel CUDA-event durations (ms) of a step of S streams x F frames:
    the median over ``reps`` profiled steps after ``warm`` uncounted ones."""
    import torch
    pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
    fresh = torch.tensor([(s << 2) | 2 for s in range(S)], dtype=torch.int32, device="cuda")
    parity = [torch.tensor([(s << 2) | p for s in range(S)], dtype=torch.int32, device="cuda") for p in (0, 1)]
    P = lambda t: ct.c_void_p(t.data_ptr())
    buf = (ct.c_float * 26)()
    runs = []
    for r in range(warm + reps):  # call 0 starts the streams (fresh); call r reads table r % 2
        codes = fresh if r == 0 else parity[r & 1]
        _native.check(lib, lib.fav_step_profile(plan.handle, P(pool), S, P(codes), S, F, P(z_dev), P(audio), P(ws),
                                                ws_bytes, P(status), buf, stream))
        if r >= warm:
            runs.append(np.array(buf[:]))
    return kernel_ms(np.median(np.stack(runs), axis=0), precision)


def run_stream(args, wl, world, rank, local):
    import torch
    from fast_audiovae import _native
    from fast_audiovae import weights as W
    from fast_audiovae.cuda import CUDADecoder

    torch.cuda.set_device(local)  # the plan, buffers and every ABI call on this rank's GPU
    S = args.streams or wl.streams
    F = wl.frames
    K, Wm = args.steps, args.warmup
    weights = W.seeded_weights(0)
    dec = CUDADecoder(weights, {}, "streaming", max_streams=S, device=local, precision=wl.precision)
    be = dec._backend
    lib = be.lib
    total_frames = (K + Wm) * F
    first = rank * S
    lat = np.stack([W.seeded_latents(first + s, total_frames)[0] for s in range(S)])  # [S,64,frames]
    steps_host = np.ascontiguousarray(lat.reshape(S, 64, K + Wm, F).transpose(2, 0, 1, 3))  # [step][S][64][F]
    z_dev = torch.from_numpy(steps_host).cuda()
    audio = torch.empty(S, 1920 * F, device="cuda")
    ws_bytes = int(lib.fav_plan_workspace_bytes(be.plan.handle, S, F))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
    codes = [torch.tensor([(s << 2) | p for s in range(S)], dtype=torch.int32, device="cuda") for p in (0, 1)]
    fresh = torch.tensor([(s << 2) | 2 for s in range(S)], dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())

    def step(i, on=None):
        c = fresh if i == 0 else codes[i % 2]
        _native.check(lib, lib.fav_step(be.plan.handle, P(pool), S, P(c), S, F, P(z_dev[i]), P(audio), P(ws),
                                        ws_bytes, P(status), on or stream))

    for i in range(Wm):
        step(i)
    torch.cuda.synchronize()
    launches = count_kernels(torch, lambda h: step(Wm, h))  # capture only: nothing runs
    barrier(world)
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for i in range(Wm, Wm + K):
        step(i)
    stop.record()
    torch.cuda.synchronize()
    dev_s = dist_max(start.elapsed_time(stop) / 1e3, world)
    clock_info = clocks.stop() if clocks else None
    assert status.item() == 0, "kernel status %x" % status.item()
    barrier(world)
    layer_ms = profile_layers(lib, _native, be.plan, S, F, z_dev[Wm], audio, ws, ws_bytes, status, stream,
                              wl.precision)

    # end to end through the public API: host chunks in, host audio out
    streams = [dec.stream() for _ in range(S)]
    chunks = [[lat[s:s + 1, :, i * F:(i + 1) * F].copy() for s in range(S)] for i in range(K + Wm)]
    for i in range(Wm):
        dec.decode_streams(streams, chunks[i])
    torch.cuda.synchronize()
    barrier(world)
    lat_ms = []
    t0 = time.perf_counter()
    for i in range(Wm, Wm + K):
        t = time.perf_counter()
        dec.decode_streams(streams, chunks[i])
        lat_ms.append(1e3 * (time.perf_counter() - t))
    torch.cuda.synchronize()
    e2e_s = dist_max(time.perf_counter() - t0, world)
    for s in streams:
        s.close()

    # single-stream chunk latency (the reference's GPU packet latency)
    one = CUDADecoder(weights, {}, "streaming", max_streams=1, device=local, precision=wl.precision)
    single = []
    with one.stream() as s1:
        zl = W.seeded_latents(first, 60 * F)
        for i in range(60):
            t = time.perf_counter()
            s1.decode_chunk(zl[..., i * F:(i + 1) * F])
            if i >= 10:
                single.append(1e3 * (time.perf_counter() - t))

    frames_total = world * S * F * K
    audio_s = frames_total * FRAME_SECONDS
    if rank == 0:
        pk = peaks()
        line = base_line(args, wl, world, K, Wm, dev_s, audio_s, "weak")
        line["config"].update(workload=wl.text.format(S=S), streams_per_gpu=S, frames_per_chunk=F)
        line["e2e"] = {"value": round(audio_s / e2e_s, 2), "unit": "audio-s/s", "h2d_bytes_per_step": S * 64 * F * 4,
                       "d2h_bytes_per_step": S * 1920 * F * 4}
        line["latency_ms"] = {"p50": round(float(np.percentile(lat_ms, 50)), 3),
                              "p99": round(float(np.percentile(lat_ms, 99)), 3), "chunk": f"{40 * F} ms",
                              "streams_per_step": S}
        line["latency_1stream_ms"] = {"p50": round(float(np.percentile(single, 50)), 3),
                                      "p99": round(float(np.percentile(single, 99)), 3)}
        line["gpu_launches"] = launches * K
        line["launches_per_step"] = launches
        line["tensor_roofline"] = tensor_roofline(frames_total, dev_s, e2e_s, pk)
        line["roofline"] = roofline(layer_ms, S * F, S, pk, args.workload, F, wl.precision)
        line["cpu_baseline"] = (cpu_baseline(wl, args.cpu_seconds) if world == 1 and not args.no_cpu_baseline
                                else None)
        line["clocks"] = clock_info
        print(json.dumps(line), flush=True)
    barrier(world)


def run_batch(args, wl, world, rank, local):
    import torch
    from fast_audiovae import _native, shard
    from fast_audiovae import weights as W
    from fast_audiovae.cuda import CUDADecoder

    torch.cuda.set_device(local)  # the plan, buffers and every ABI call on this rank's GPU
    K, Wm = args.steps, args.warmup
    T = wl.frames
    if wl.strong:
        lo, hi = shard.shard_range(wl.clips, world, rank)
    else:
        lo, hi = rank * wl.clips, (rank + 1) * wl.clips
    n = hi - lo
    weights = W.seeded_weights(0)
    dec = CUDADecoder(weights, {}, "batch", device=local, batch_chunk_frames=wl.chunk, precision=wl.precision)
    be = dec._backend
    lib = be.lib
    chunk = min(wl.chunk, T)
    clips = [W.seeded_latents(c, T) for c in range(lo, hi)]
    z_dev = torch.from_numpy(np.concatenate(clips, 0)).cuda()
    audio = torch.empty(n, 1920 * T, device="cuda")
    ws_bytes = int(lib.fav_plan_batch_workspace_bytes(be.plan.handle, n, chunk))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())

    def step(on=None):
        _native.check(lib, lib.fav_decode_batch(be.plan.handle, P(z_dev), n, T, chunk, P(audio), P(ws), ws_bytes,
                                                P(status), on or stream))

    for _ in range(Wm):
        step()
    torch.cuda.synchronize()
    launches = count_kernels(torch, step)
    barrier(world)
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(K):
        step()
    stop.record()
    torch.cuda.synchronize()
    dev_s = dist_max(start.elapsed_time(stop) / 1e3, world)
    clock_info = clocks.stop() if clocks else None
    assert status.item() == 0, "kernel status %x" % status.item()
    barrier(world)
    # the dominant kernel of one internal step (n clips x chunk frames)
    zc = torch.from_numpy(np.ascontiguousarray(np.concatenate(clips, 0)[..., :chunk])).cuda()
    ac = torch.empty(n, 1920 * chunk, device="cuda")
    wsc_bytes = int(lib.fav_plan_workspace_bytes(be.plan.handle, n, chunk))
    wsc = torch.empty(wsc_bytes, dtype=torch.uint8, device="cuda")
    layer_ms = profile_layers(lib, _native, be.plan, n, chunk, zc, ac, wsc, wsc_bytes, status, stream,
                              wl.precision)
    del zc, ac, wsc

    # end to end through the public API (shard.decode_clips -> decode_many)
    all_clips = [W.seeded_latents(c, T) for c in range(wl.clips * (1 if wl.strong else world))] \
        if wl.strong else clips
    for _ in range(Wm):
        shard.decode_clips(dec, all_clips, gather=False) if wl.strong else dec.decode_many(clips)
    barrier(world)
    lat_ms = []
    t0 = time.perf_counter()
    for _ in range(K):
        t = time.perf_counter()
        shard.decode_clips(dec, all_clips, gather=False) if wl.strong else dec.decode_many(clips)
        lat_ms.append(1e3 * (time.perf_counter() - t))
    e2e_s = dist_max(time.perf_counter() - t0, world)

    frames_total = (wl.clips if wl.strong else world * n) * T * K
    audio_s = frames_total * FRAME_SECONDS
    if rank == 0:
        pk = peaks()
        line = base_line(args, wl, world, K, Wm, dev_s, audio_s, "strong" if wl.strong else "weak")
        line["config"].update(workload=wl.text.format(C=n), clips_per_step=wl.clips if wl.strong else n,
                              frames_per_clip=T, chunk_frames=chunk)
        line["e2e"] = {"value": round(audio_s / e2e_s, 2), "unit": "audio-s/s", "h2d_bytes_per_step": n * 64 * T * 4,
                       "d2h_bytes_per_step": n * 1920 * T * 4}
        line["latency_ms"] = {"p50": round(float(np.percentile(lat_ms, 50)), 3),
                              "p99": round(float(np.percentile(lat_ms, 99)), 3),
                              "call": f"{n} clip(s) x {T} frames"}
        line["gpu_launches"] = launches * K
        line["launches_per_step"] = launches
        line["tensor_roofline"] = tensor_roofline(frames_total, dev_s, e2e_s, pk)
        line["roofline"] = roofline(layer_ms, n * chunk, n, pk, args.workload, chunk, wl.precision)
        line["cpu_baseline"] = (cpu_baseline(wl, args.cpu_seconds) if world == 1 and not args.no_cpu_baseline
                                else None)
        line["clocks"] = clock_info
        print(json.dumps(line), flush=True)
    barrier(world)


def base_line(args, wl, world, K, Wm, dev_s, audio_s, scaling):
    operands = ("W8A8 int8 (s8 tensor cores, per-row weight and per-time-step activation scales) on the projections "
                "with min(rows, cols) >= 128; the rest as the bf16 plan" if wl.precision else
                "split-bf16 stem (4 MMAs) and transposed convs (3 MMAs), f16 residual 1x1s, fp32 activations and "
                "accumulation")
    return {"metric": wl.metric, "value": round(audio_s / dev_s, 2), "unit": "audio-s/s", "n_gpus": world,
            "steps": K, "warmup": Wm, "ms_per_step": round(1e3 * dev_s / K, 4), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None,
            "dtype": "int8 W8A8 + bf16 (fp32 accumulate)" if wl.precision else "bf16+f16 (fp32 accumulate)",
            "data": "synthetic",
            "config": {"weights": "seeded random init (seed 0)",
                       "l2": "working set larger than L2 (126 MB) between timed steps: 183 MB weights plus "
                             "activations and histories; no flush",
                       "operands": operands}}


# ------------------------------------------------------------------ ncu ingest
LAUNCH_ORDER = (["stem"]
                + [x for i in (0, 1) for x in [f"stage{i}.transpose"]
                   + [y for j in range(3) for y in (f"stage{i}.res{j}", f"stage{i}.res{j}")]]
                + [x for i in (2, 3, 4) for x in (f"stage{i}.transpose", f"stage{i}.units")]
                + ["stage5.transpose", "stage5.tail"])


def ingest_ncu(path):
    """bench_traffic.json from an ncu launch list (csv) of one default step: the
    launches in order (stem, per stage 0-1 a conv and each unit's depthwise
    pre-pass + GEMM, per stage 2-4 a conv and the fused stage, stage 5's conv
    and tail), DRAM bytes per kernel (a unit's two launches summed)."""
    rows = {}
    with open(path) as f:
        lines = [l for l in f if l.startswith('"')]
    for rec in csv.DictReader(lines):
        key = rec["ID"]
        rows.setdefault(key, {"name": rec["Kernel Name"]})
        unit = rec["Metric Unit"]
        val = float(rec["Metric Value"].replace(",", ""))
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "ns": 1e-3, "nsecond": 1e-3, "us": 1, "usecond": 1,
                 "ms": 1e3, "msecond": 1e3}
        rows[key][rec["Metric Name"]] = val * scale.get(unit, 1)
    launches = [rows[k] for k in sorted(rows, key=int)]
    if len(launches) != len(LAUNCH_ORDER):
        raise SystemExit(f"expected {len(LAUNCH_ORDER)} launches, found {len(launches)}")
    layers = {}
    for name, rec in zip(LAUNCH_ORDER, launches):
        layers[name] = layers.get(name, 0) + int(rec.get("dram__bytes_read.sum", 0) + rec.get("dram__bytes_write.sum", 0))
    out = {"workload": "stream40ms", "streams": 512, "frames": 1,
           "source": "ncu launch list of one step of `python bench.py --steps 2 --warmup 3 --no-cpu-baseline` "
                     "(profiles/step_launches_stream40ms_512.md)",
           "layers": layers}
    TRAFFIC_FILE.write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out))


def main():
    args = parse()
    if args.ingest_ncu:
        ingest_ncu(args.ingest_ncu)
        return
    wl = WORKLOADS[args.workload]
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, wl, world, rank)
        elif wl.kind == "stream":
            run_stream(args, wl, world, rank, local)
        else:
            run_batch(args, wl, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
