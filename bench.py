#!/usr/bin/env python
"""htdemucs_6s source separation throughput on B200 (the 240 s track workload).

One step = the whole of dc_apply_model (apply.c:179-306) on a 240 s synthetic stereo track:
shifts = 1, 7.8 s segments at overlap 0.25, batches of 8 segments -> 42 segment forwards of
the full htdemucs_6s model (random-init fp16 weights), transition-weighted overlap-add.
With N GPUs (one process each, torchrun) rank 0's packed weight block is NCCL-broadcast
once to ranks that hold only the layout, the segments are split into N contiguous blocks
(strong scaling: the track is fixed), each rank computes its weighted stems over its own
output window only, and rank 0 gathers the windows (NCCL) and overlap-adds them.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line (rank 0).  value = audio seconds separated per second of device time
(max over ranks) with the input resident in HBM; e2e = the same through the public API with
the track copied host->device and the stems device->host inside every timed step.
--impl reference times the reference's own CPU implementation (oracle/_ref, backend_cpu.c
with the reference model code) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "audio sec/sec (7.8 s segs, fp16)"
UNIT = "audio-s/s"
CACHE = os.environ.get("DCB_BENCH_CACHE", "/tmp/demucs_b200_bench")
REF_BIN = os.path.join(ROOT, "oracle", "_ref", "dcref")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def model_files():
    from demucs_cuda_b200 import synth
    return synth.write_model(os.path.join(CACHE, "full_s1"), synth.FULL, seed=1)


def short_config(weights_dir):
    """The same weights with 1 s segments (valid_length 44100): the bounded CPU sample."""
    from demucs_cuda_b200 import synth
    path = os.path.join(weights_dir, "model_1s.json")
    if not os.path.exists(path):
        with open(path, "w") as f:
            f.write(synth.SHORT.to_json())
    return path


def track(seconds):
    from demucs_cuda_b200 import synth
    os.makedirs(CACHE, exist_ok=True)
    path = os.path.join(CACHE, f"track_{seconds:g}s.npy")
    if os.path.exists(path):
        return np.load(path)
    x = synth.track_input(seconds, 44100, seed=0)
    np.save(path + ".tmp.npy", x)
    os.replace(path + ".tmp.npy", path)
    return x


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling during the timed region (clocks, power, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = []
        for ln in open(self.f.name):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                if int(parts[0]) not in self.gpus:
                    continue
                rows.append(parts)
            except ValueError:
                continue
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(float(r[1]) for r in rows)
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].lower() in ("active", "1", "yes")})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows
                                                        if r[3].replace(".", "").isdigit())
                if any(r[3].replace(".", "").isdigit() for r in rows) else None}


# ------------------------------------------------------------------ CPU reference
def run_reference_cpu(weights, config_1s, reps, procs, seconds=1.0):
    """procs parallel single-thread processes of the reference CPU forward (oracle/_ref,
    unmodified backend_cpu.c + model code), each timing `reps` forwards of one 1 s
    segment.  Returns the per-repeat aggregate throughput in audio-s/s."""
    from demucs_cuda_b200 import synth
    mix = synth.segment_input(synth.SHORT, 1, 0)
    os.makedirs(CACHE, exist_ok=True)
    mpath = os.path.join(CACHE, "mix_1s.f32")
    mix.astype("<f4").tofile(mpath)
    T = mix.shape[-1]
    ps = [subprocess.Popen([REF_BIN, "time", weights, config_1s, mpath, "1", "2", str(T),
                            str(reps)], stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                           text=True) for _ in range(procs)]
    times = []
    for p in ps:
        out, err = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"reference CPU run failed: {err.strip()[-300:]}")
        times.append(json.loads(out.strip().splitlines()[-1])["times_s"])
    times = np.array(times)  # [procs, reps]
    per_rep = (seconds / times).sum(axis=0)  # audio seconds per second, all processes
    return per_rep, times


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if not os.path.exists(REF_BIN):
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/dcref was not built (reference sources absent)"}))
        return 0
    w, _ = model_files()
    c1 = short_config(os.path.dirname(w))
    procs = host_cores()
    per_rep, times = run_reference_cpu(w, c1, args.warmup + args.steps, procs)
    timed = per_rep[args.warmup:]
    value = float(np.mean(timed))
    sample = (f"{procs} parallel single-thread processes (one per host core) of the reference "
              f"CPU forward (backend_cpu.c + htdemucs.c, unmodified) on 1 s segments of the "
              f"same htdemucs_6s weights; each step = one forward per process")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": float(np.mean(times[:, args.warmup:].max(axis=0)) * 1e3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded U[-0.5,0.5] segment, random-init weights)",
        "config": {"workload": "htdemucs_6s segment forwards, 1 s segments (bounded CPU sample "
                               "of the 240 s / 7.8 s-segment workload)", "host_cores": procs},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": procs, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------ B200 arm
def cuda_array(ptr, nbytes):
    """Zero-copy uint8 torch view of a device allocation owned by the library."""
    import torch

    class _CAI:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                    "data": (ptr, False), "version": 3}

    return torch.as_tensor(_CAI(), device="cuda")


def b200_arm(args):
    import torch
    import torch.distributed as dist
    import datetime

    import demucs_cuda_b200 as dcb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dcb.require_gpu()
    if rank == 0:
        w, c = model_files()
    if world > 1:
        dist.barrier()
    w, c = model_files()
    # weights: rank 0 reads and packs the file; the other ranks build the same layout from
    # the safetensors header alone (a zeroed device block) and receive rank 0's packed
    # block through one NCCL broadcast, checked word for word afterwards
    model = dcb.Model(w, c, layout_only=(world > 1 and rank != 0))
    bcast_ms = None
    if world > 1:
        ptr, nbytes = model.weight_block()
        view = cuda_array(ptr, nbytes)
        torch.cuda.synchronize()
        t0 = time.time()
        dist.broadcast(view, src=0)
        torch.cuda.synchronize()
        bcast_ms = (time.time() - t0) * 1e3
        words = view[: nbytes // 4 * 4].view(torch.int32).to(torch.int64)
        pos = torch.arange(words.numel(), device="cuda", dtype=torch.int64) % 65521 + 1
        ck = torch.stack([words.sum(), (words * pos).sum()])
        del words, pos
        allck = [torch.empty_like(ck) for _ in range(world)]
        dist.all_gather(allck, ck)
        if any(not torch.equal(a, allck[0]) for a in allck):
            raise RuntimeError("weight block differs from rank 0's after the broadcast")
    x = track(args.seconds)
    T = x.shape[-1]
    mix_host = torch.from_numpy(x).pin_memory()
    mix = mix_host.cuda()
    out = torch.empty((1, model.n_sources, 2, T), device="cuda", dtype=torch.float32)
    out_host = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
    kw = dict(shifts=args.shifts, overlap=args.overlap, batch_size=args.batch,
              shard_index=rank, shard_count=world)
    nfw, nbatched = model.apply_plan(T, **kw)
    rows = model.n_sources * 2
    if world > 1:
        # each rank's share is non-zero only on its output window: ranks write their window,
        # rank 0 gathers them (NCCL over NVLink) and overlap-adds them into the stems
        spans = [model.apply_window(T, **dict(kw, shard_index=r)) for r in range(world)]
        wmax = max(h - l for l, h in spans)
        win = torch.empty((rows, wmax), device="cuda", dtype=torch.float32)
        gbuf = (torch.empty((world, rows, wmax), device="cuda", dtype=torch.float32)
                if rank == 0 else None)
        glist = list(gbuf.unbind(0)) if rank == 0 else None

    def step():
        if world == 1:
            model.apply(mix, out=out, **kw)
            return
        model.apply_shard(mix, win, **kw)
        dist.gather(win, gather_list=glist, dst=0)
        if rank == 0:
            dcb.merge_windows(out, gbuf, [l for l, _ in spans], [h for _, h in spans])

    def step_e2e():
        if world == 1:
            # the public host-buffer call: the track's spans go up just before the batches
            # that read them and finished stretches of the stems come back while later
            # batches compute (dcb_apply_host)
            model.apply_host(mix_host, out_host, **kw)
            return
        mix.copy_(mix_host, non_blocking=True)
        step()
        if rank == 0:
            out_host.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def timed(fn, steps, trace=False):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = dcb.kernel_launches()
        if trace:
            dcb.trace_start()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        tr = dcb.trace_stop() if trace else None
        if trace and args.trace_csv and rank == 0:
            dcb.trace_dump(args.trace_csv)
        launches = dcb.kernel_launches() - n0
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms, launches, tr

    # the segment forward runs as a replayed CUDA graph (captured during the warm-up)
    dcb.set_option("graphs", 0 if args.no_graphs else 1)
    dcb.set_option("streams", 0 if args.one_stream else 1)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    gpus = [int(g) for g in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if g.strip()]
    clk = Clocks(set(gpus[:world]) if gpus else set(range(world)))
    clk.start()
    ms, launches, _ = timed(step, args.steps)
    clocks = clk.stop()
    # end to end through the public API: host input -> device -> stems -> host
    step_e2e()
    ms_e2e, _, _ = timed(step_e2e, args.steps)
    # per-kernel-class CUDA events for the roofline: a separate eager pass (tracing
    # bypasses the graph), so the headline numbers above carry no event overhead; it runs
    # on one stream, so no event pair also times a kernel of the other branch
    dcb.set_option("streams", 0)
    step()
    ms_tr, _, tr = timed(step, args.steps, trace=True)
    dcb.set_option("streams", 0 if args.one_stream else 1)
    fault = dcb.device_fault()

    audio = float(args.seconds) * max(1, 1)  # one track per step, whole job
    value = audio / (ms / 1e3)
    e2e = audio / (ms_e2e / 1e3)
    hbm, tflops_burst, tflops_sus, pk_kind = peaks()
    # dominant kernel class of the timed region (CUDA events around its launches); the
    # memory-bound glue classes are reported separately (bytes only)
    glue = {k: v for k, v in tr.items() if v["launches"] and k in dcb.GLUE_CLASSES}
    kinds = {k: v for k, v in tr.items() if v["launches"] and k not in dcb.GLUE_CLASSES}
    dom = max(kinds, key=lambda k: kinds[k]["ms"])
    d = kinds[dom]
    per_launch_ms = d["ms"] / d["launches"]
    fl_launch = d["flops"] / d["launches"]
    by_launch = d["bytes"] / d["launches"]
    ai = d["flops"] / max(d["bytes"], 1.0)
    tensor_bound = ai * hbm / 1e3 > tflops_sus  # ridge point of the measured peaks
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        traffic = json.load(open(tpath)).get(dom)
    if tensor_bound:
        achieved = fl_launch / (per_launch_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": tflops_sus, "unit": "TFLOP/s",
                "frac": achieved / tflops_sus}
    else:
        achieved = by_launch / (per_launch_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm}
    roof.update({"traffic": traffic, "kernel": dom, "peak_kind": f"{pk_kind} "
                 f"({'bf16 dense sustained' if tensor_bound else 'HBM copy'})",
                 "launches": d["launches"], "ms_per_launch": per_launch_ms,
                 "algorithmic_flops_per_launch": fl_launch,
                 "algorithmic_bytes_per_launch": by_launch})
    # shares: each class's kernel time per step (CUDA events around its launches in the
    # traced one-stream eager pass) over the graph-replayed step time of the headline value,
    # whose two branch streams overlap kernels (so the shares can sum above 1); the traced
    # pass itself runs host-bound (eager launches plus two events per traced launch)
    classes = {k: {"share_of_step": v["ms"] / args.steps / ms,
                   "tflops": v["flops"] / (v["ms"] * 1e-3) / 1e12 if v["ms"] else 0.0,
                   "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9 if v["ms"] else 0.0,
                   "launches_per_step": v["launches"] / args.steps} for k, v in kinds.items()}
    glue_rep = {k: {"share_of_step": v["ms"] / args.steps / ms,
                    "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9 if v["ms"] else 0.0,
                    "frac_of_hbm": (v["bytes"] / (v["ms"] * 1e-3) / 1e9) / hbm if v["ms"] else 0.0,
                    "launches_per_step": v["launches"] / args.steps,
                    "mb_per_step": v["bytes"] / args.steps / 1e6} for k, v in glue.items()}
    gemm_flops = sum(v["flops"] for v in kinds.values()) / args.steps
    gemm_ms = sum(v["ms"] for v in kinds.values()) / args.steps

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and os.path.exists(REF_BIN):
        try:
            procs = host_cores()
            per_rep, _ = run_reference_cpu(w, short_config(os.path.dirname(w)), 1, procs)
            cpu = {"value": float(per_rep[0]), "unit": UNIT, "cores": procs,
                   "kind": "reference",
                   "sample": f"{procs} parallel single-thread reference CPU forwards "
                             "(oracle/_ref: backend_cpu.c + htdemucs.c) of one 1 s segment "
                             "each, same weights"}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                   "sample": f"failed: {ex}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16",
            "data": "synthetic: 240 s seeded 40-sinusoid + noise stereo track, random-init "
                    "htdemucs_6s weights (Kaiming-uniform, seed 1)",
            "config": {"workload": f"dc_apply_model on a {args.seconds:g} s track: shifts "
                                   f"{args.shifts}, overlap {args.overlap}, batch "
                                   f"{args.batch}, {nfw} segment forwards in {nbatched} "
                                   "forward calls (this rank)",
                       "model": "htdemucs_6s", "segment_samples": 343980,
                       "parallelism": f"segment data parallel x{world}" + (
                           f": contiguous segment blocks per rank, output windows of at most "
                           f"{wmax} samples gathered to rank 0 (NCCL) and overlap-added"
                           if world > 1 else ""),
                       "l2": "inputs and activations larger than L2 (126 MB) every step",
                       "weight_broadcast_ms": bcast_ms},
            "e2e": {"value": e2e, "unit": UNIT, "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": int(mix_host.numel() * 4),
                    "d2h_bytes_per_step": int(out_host.numel() * 4)},
            "gpu_launches": int(launches),
            "cuda_graphs": not args.no_graphs,
            "branch_streams": 1 if args.one_stream else 2,
            "roofline": roof,
            "gemm": {"tflops": gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None,
                     "frac_of_peak": (gemm_flops / (gemm_ms * 1e-3) / 1e12) / tflops_sus
                     if gemm_ms else None, "peak_tflops": tflops_sus,
                     "share_of_step": gemm_ms / ms, "traced_ms_per_step": ms_tr,
                     "classes": classes},
            "glue": glue_rep,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "device_fault": fault,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seconds", type=float, default=240.0)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--shifts", type=int, default=1)
    ap.add_argument("--overlap", type=float, default=0.25)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--one-stream", action="store_true",
                    help="issue the time branch on the same stream as the frequency branch")
    ap.add_argument("--no-graphs", action="store_true",
                    help="launch every kernel eagerly instead of replaying the captured "
                         "segment forward")
    ap.add_argument("--trace-csv", default="", help="write every traced GEMM-family launch "
                    "of the timed region (class, ms, FLOPs, bytes, M, N, K) to this CSV")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    return b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())
