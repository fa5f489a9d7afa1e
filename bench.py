"""Benchmark of the AudioVAE2 decoder hot path on B200: 40 ms streaming chunks.

Workload ("stream40ms"): every GPU decodes S independent streams (default 512,
the per-GPU shard of 4096 streams on 8 GPUs) that each receive one-frame
(40 ms, 1920-sample) latent chunks ~N(0,1) with per-stream seeds, carrying
causal history across steps; decoder coefficients are the seeded random init.
One step = one chunk for all S streams (29 kernel launches: stem, then per
stage a transposed conv and three residual units, stages 0-1's units as a
depthwise pre-pass plus the GEMM, stage 5's units and the final conv fused into
one kernel). Weak scaling:
each rank owns S streams, no collective on the data path.

Reported (one JSON line, rank 0):
  value   aggregate audio-s/s, inputs resident in HBM, device time (CUDA events,
          max over ranks);
  e2e     the same metric through the public API (``CUDADecoder.decode_streams``
          with host numpy chunks: validation, pinned H2D, step (audio written
          device-to-host into mapped pinned memory by the final kernel), finite
          check), host wall time, max over ranks; plus p50/p99 chunk latency;
  roofline  the dominant kernel's algorithmic FLOPs or bytes per launch over its
          CUDA-event duration, against MEASURED_PEAKS.json;
  cpu_baseline  the fp32 oracle port of the reference decoder on the host cores.

``--impl reference`` times the reference decoder's CPU implementation (the
oracle port of ``mps_decoder.py``; rank 0 only) on a bounded sample of the
same workload and prints the same line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "fast-audiovae_b200"))
sys.path.insert(0, str(ROOT))

FRAME_SECONDS = 1920 / 48000
RATES = (8, 6, 5, 2, 2, 2)
METRIC = "aggregate audio-s/s (RTF^-1), 40 ms streaming chunks"
# Kernels of one step, in launch order: the stem, per stage a transposed conv
# and three residual units (stage 5: its transposed conv and the fused tail =
# three residual units + final conv).
LAYER_NAMES = ["stem"] + [f"stage{i}.{k}" for i in range(5) for k in ("transpose", "res0", "res1", "res2")] + \
    ["stage5.transpose", "stage5.tail"]
# The residual units of stages 0-1 are two launches each (depthwise pre-pass, then the GEMM).
LAUNCHES_PER_STEP = len(LAYER_NAMES) + 6


def kernel_ms(layer_ms26):
    """Per-kernel durations from the 26 per-layer event intervals of
    ``fav_step_profile`` (the fused tail spans layers 22-25)."""
    v = np.asarray(layer_ms26, dtype=np.float64)
    return np.concatenate([v[:22], [v[22:].sum()]])


def parse():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--streams", type=int, default=512, help="streams per GPU")
    p.add_argument("--frames", type=int, default=1, help="latent frames per chunk (1 = 40 ms)")
    p.add_argument("--cpu-seconds", type=float, default=8.0, help="budget per CPU baseline leg")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured (MEASURED_PEAKS.json; bf16 sustained)"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "source": "fallback"}


# ------------------------------------------------------------------ algorithmic cost
def layer_costs():
    """Per kernel of ``LAYER_NAMES``, per latent frame: algorithmic FLOPs (2*MAC
    of the contractions) and HBM bytes of this design's data layout (each
    activation read and written once), plus per-launch weight bytes and
    per-stream history bytes (read + write). Activations: fp32 y and Snake(y)
    between residual units; the split-bf16 planes a transposed conv reads,
    written twice (as they are, and one time step later for the second tap).
    The fused stage-5 tail reads its input y once and writes audio; its
    intermediates stay on chip."""
    out = []
    n = 1  # rows per frame at the current layer input
    out.append(dict(flops=2 * 2048 * 64, act=64 * 4 + 2048 * 8, weights=2048 * 64 * 4,
                    hist=6 * 64 * 4 * 2 + 2048 * 4 * 2))
    cin = 2048
    for i, s in enumerate(RATES):
        cout = cin // 2
        y_bytes = 4 if i == 5 else 8  # stage 5's transposed conv writes y only (the tail applies Snake_pre)
        out.append(dict(flops=2 * cin * cout * 2 * s * n, act=n * cin * 8 + n * s * cout * y_bytes,
                        weights=cin * cout * 2 * s * 4, hist=0))
        n *= s
        if i == 5:
            out.append(dict(flops=n * (3 * 2 * cout * cout + 2 * cout * 7), act=n * cout * 4 + n * 4,
                            weights=3 * cout * cout * 2, hist=(6 + 18 + 54 + 6) * cout * 4 * 2))
            break
        for j, d in enumerate((1, 3, 9)):
            nxt = 0 if j < 2 else cout * 4 * 2  # next transposed conv's history row
            pre = n * cout * 4 if i <= 1 else 0  # stages 0-1: the f16 A operand written and read once
            out.append(dict(flops=2 * cout * cout * n, act=n * cout * 16 + pre, weights=cout * cout * 2,
                            hist=6 * d * cout * 4 * 2 + nxt))
        cin = cout
    assert len(out) == len(LAYER_NAMES)
    return out


def measured_traffic(layer, streams, frames):
    """DRAM bytes (read + write) of one launch of ``layer`` from the committed
    ncu launch list, which was captured on this workload (512 streams x 1 frame)."""
    path = ROOT / "profiles" / "step_launches_stream40ms_512.md"
    if streams != 512 or frames != 1 or not path.is_file():
        return None
    text = path.read_text()
    block = text.split("```csv", 1)[-1].split("```", 1)[0]
    for line in block.strip().splitlines()[1:]:
        name, _, rd, wr = line.split(",")
        if name == layer:
            return int(rd) + int(wr)
    return None


def roofline(layer_ms, frames_per_launch, streams, pk, frames=1):
    costs = layer_costs()
    dom = int(np.argmax(layer_ms))
    c = costs[dom]
    flops = c["flops"] * frames_per_launch
    bytes_ = c["act"] * frames_per_launch + c["weights"] + c["hist"] * streams
    t_tensor = flops / (pk["tflops"] * 1e12)
    t_hbm = bytes_ / (pk["hbm_gbs"] * 1e9)
    sec = layer_ms[dom] / 1e3
    if t_tensor >= t_hbm:
        achieved, peak, unit, bound = flops / sec / 1e12, pk["tflops"], "TFLOP/s", "tensor"
    else:
        achieved, peak, unit, bound = bytes_ / sec / 1e9, pk["hbm_gbs"], "GB/s", "hbm"
    share = float(layer_ms[dom] / np.sum(layer_ms))
    traffic = measured_traffic(LAYER_NAMES[dom], streams, frames)
    return {"kernel": LAYER_NAMES[dom], "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                              "profiles/step_launches_stream40ms_512.md" if traffic else None,
            "share_of_step": round(share, 4),
            "algorithmic_per_launch": {"flops": flops, "bytes": bytes_}, "peak_source": pk["source"],
            "layer_ms": {LAYER_NAMES[i]: round(float(v), 4) for i, v in enumerate(layer_ms)}}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
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
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------ CPU legs
def cpu_rate(streams, budget_s, threads, frames=1):
    """Oracle port (fp32 reference decoder) streaming 1-frame chunks on CPU: audio-s/s."""
    import torch
    from fast_audiovae import weights as W
    from oracle.decoder import Decoder
    torch.set_num_threads(threads)
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


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ distributed
def dist_setup(args):
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
def run_reference(args, world, rank):
    if rank != 0:
        return
    cores = host_cores()
    total_frames, total_time = 0, 0.0
    streams = min(args.streams, 8)
    for _ in range(args.warmup):
        cpu_rate(streams, 0.5, cores)
    per_step = max(1.0, min(20.0, 120.0 / max(1, args.steps)))
    for _ in range(args.steps):
        rate, done, el = cpu_rate(streams, per_step, cores)
        total_frames += done
        total_time += el
    value = total_frames * FRAME_SECONDS / total_time
    sample = f"{streams} streams x 1-frame chunks with carried history, ~{per_step:.1f} s per step"
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "audio-s/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * total_time / args.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"stream40ms: {args.streams} streams/GPU x {args.frames}-frame chunks",
                       "implementation": "reference fp32 decoder (mps_decoder.py restated, torch CPU)"},
            "cpu_baseline": {"value": round(value, 3), "unit": "audio-s/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    import torch
    from fast_audiovae import _native
    from fast_audiovae import weights as W
    from fast_audiovae.cuda import CUDADecoder

    torch.cuda.set_device(local)
    S, F = args.streams, args.frames
    K, Wm = args.steps, args.warmup
    weights = W.seeded_weights(0)
    dec = CUDADecoder(weights, {}, "streaming", max_streams=S, device=local)
    be = dec._backend
    lib = be.lib
    total_frames = (K + Wm) * F
    first = rank * S
    lat = np.stack([W.seeded_latents(first + s, total_frames)[0] for s in range(S)])  # [S,64,frames]
    steps_host = np.ascontiguousarray(lat.reshape(S, 64, K + Wm, F).transpose(2, 0, 1, 3))  # [step][S][64][F]
    z_dev = torch.from_numpy(steps_host).cuda()
    audio = torch.empty(S, 1920 * F, device="cuda")
    ws_bytes = int(lib.fav_step_workspace_bytes(S, F))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    pool = torch.zeros(lib.fav_state_pool_bytes(S) // 4, device="cuda")
    codes = [torch.tensor([(s << 2) | p for s in range(S)], dtype=torch.int32, device="cuda") for p in (0, 1)]
    fresh = torch.tensor([(s << 2) | 2 for s in range(S)], dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())

    def step(i):
        c = fresh if i == 0 else codes[i % 2]
        _native.check(lib, lib.fav_step(be.plan.handle, P(pool), S, P(c), S, F, P(z_dev[i]), P(audio), P(ws),
                                        ws_bytes, P(status), stream))

    for i in range(Wm):
        step(i)
    torch.cuda.synchronize()
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

    # per-layer durations (CUDA events on the launching stream) for the roofline
    layer_ms = np.zeros(26)
    buf = (ct.c_float * 26)()
    reps = 5
    for r in range(reps):
        i = Wm + (r % K)
        _native.check(lib, lib.fav_step_profile(be.plan.handle, P(pool), S, P(codes[i % 2]), S, F, P(z_dev[i]),
                                                P(audio), P(ws), ws_bytes, P(status), buf, stream))
        layer_ms += np.array(buf[:])
    layer_ms = kernel_ms(layer_ms / reps)

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

    # single-stream 40 ms chunk latency (the reference's GPU packet latency)
    one = CUDADecoder(weights, {}, "streaming", max_streams=1, device=local)
    single = []
    with one.stream() as s1:
        zl = W.seeded_latents(first, 60)
        for i in range(60):
            t = time.perf_counter()
            s1.decode_chunk(zl[..., i:i + 1])
            if i >= 10:
                single.append(1e3 * (time.perf_counter() - t))

    audio_s = world * S * F * K * FRAME_SECONDS
    result = None
    if rank == 0:
        pk = peaks()
        rl = roofline(layer_ms, S * F, S, pk, F)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cores = host_cores()
            rate_all, done_all, _ = cpu_rate(8, args.cpu_seconds, cores)
            rate_one, done_one, _ = cpu_rate(2, args.cpu_seconds, 1)
            cpu = {"value": round(rate_all, 3), "unit": "audio-s/s", "cores": cores, "kind": "port",
                   "sample": f"fp32 oracle decoder, 8 streams x {done_all // 8} one-frame chunks with carried "
                             f"history, {cores} threads (~{args.cpu_seconds:.0f} s)",
                   "value_1thread": round(rate_one, 3)}
        result = {
            "metric": METRIC, "value": round(audio_s / dev_s, 2), "unit": "audio-s/s", "n_gpus": world,
            "steps": K, "warmup": Wm, "ms_per_step": round(1e3 * dev_s / K, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16+f16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"stream40ms: {S} streams/GPU x {F}-frame (40 ms) chunks, carried history",
                       "streams_per_gpu": S, "frames_per_chunk": F, "weights": "seeded random init (seed 0)",
                       "l2": "working set larger than L2: 183 MB weights + %d MB histories per GPU"
                             % (2 * S * 647424 // 2**20),
                       "operands": "split-bf16 (3 MMAs) stem/transposed, f16 residual 1x1, fp32 activations"},
            "e2e": {"value": round(audio_s / e2e_s, 2), "unit": "audio-s/s", "h2d_bytes_per_step": S * 64 * F * 4,
                    "d2h_bytes_per_step": S * 1920 * F * 4},
            "latency_ms": {"p50": round(float(np.percentile(lat_ms, 50)), 3),
                           "p99": round(float(np.percentile(lat_ms, 99)), 3), "chunk": "40 ms",
                           "streams_per_step": S},
            "latency_1stream_ms": {"p50": round(float(np.percentile(single, 50)), 3),
                                   "p99": round(float(np.percentile(single, 99)), 3)},
            "gpu_launches": LAUNCHES_PER_STEP * K,
            "roofline": rl,
            "cpu_baseline": cpu,
            "clocks": clock_info,
        }
        print(json.dumps(result), flush=True)
    barrier(world)
    return result


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
