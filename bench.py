#!/usr/bin/env python3
"""Benchmark of the B200 HAT backend on the reference's headline workload.

Workload: HAT-S x4, one seeded synthetic 512x512 RGB image
per GPU, seeded random weights in the reference's checkpoint layout, fp32-parity mode.
Metric: output Mpix/s (BASELINE.json `metric`). One process per GPU; for N > 1 every
rank runs its own image (the batch is split per GPU, no collective on the data path),
so scaling is weak.

`--shard strip` measures the other multi-GPU mode instead:
ONE HAT-L x4 1024x1024 image split into window-aligned row strips over the N GPUs, with
NCCL halo exchange between neighbours; scaling is strong (the same image at every N).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--shard batch|strip]

`value`: K timed steps of `hat_b200_forward_device` with the input already in HBM, each
step timed with CUDA events on the launching stream, L2 flushed between steps; the max
over ranks. `e2e`: the same metric through `hat_b200_forward` from pinned host memory
to host memory (H2D of the image and D2H of the result inside the timed region).
`--impl reference` times the CPU oracle port of the reference's forward on the host
cores (the reference's Rust CPU path cannot be built on these machines).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "hat-rs_b200"))
sys.path.insert(0, str(ROOT))

# The two workloads: (variant, scale, H, W, config id, algorithmic FLOPs per padded input
# pixel with QK^T and PV counted once).
WORKLOADS = {
    "batch": ("hat-s", 4, 512, 512, 2, 26.67e6),
    "strip": ("hat-l", 4, 1024, 1024, 4, 99.12e6),
}
VARIANT, SCALE, H, W, CFG_ID, FLOPS_PER_PIX = WORKLOADS["batch"]
WEIGHT_SEED = 2024
REF_GPU_S = 8.6  # seconds, README.md:18 of the reference (HAT-S x4 512x512, GPU, hardware unstated)


def select_workload(shard: str):
    global VARIANT, SCALE, H, W, CFG_ID, FLOPS_PER_PIX
    VARIANT, SCALE, H, W, CFG_ID, FLOPS_PER_PIX = WORKLOADS[shard]


def metric_name(mode: str = "parity") -> str:
    return f"output Mpix/s, {VARIANT.upper()} x{SCALE} {H}x{W} input (fp32-{mode} mode)" if mode == "parity" \
        else f"output Mpix/s, {VARIANT.upper()} x{SCALE} {H}x{W} input ({mode} mode)"


def baseline_mpixs():
    """The reference's published number for this metric, when there is one."""
    if (VARIANT, SCALE, H, W) == ("hat-s", 4, 512, 512):
        return (H * SCALE) * (W * SCALE) / 1e6 / REF_GPU_S
    return None
# DRAM bytes (read + write) per launch of a kernel kind at this workload, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum); profiles/ holds the capture's
# summary and command. Kinds without a capture report null.
NCU_TRAFFIC_BYTES = {"attn.window": 583.3e6}  # profiles/k_attn_tc_window_hats_x4_512.md


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, dev: int):
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(dev), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_oracle_sample(ck: str, img: np.ndarray, crop: int):
    """One oracle forward of a crop of the workload image; returns (seconds, out Mpix)."""
    from oracle import hat_oracle as O
    m = O.Model.load(ck)
    t = time.perf_counter()
    y = O.forward(m, img[:, :crop, :crop])
    dt = time.perf_counter() - t
    assert y.shape == (3, crop * SCALE, crop * SCALE)
    return dt, (crop * SCALE) ** 2 / 1e6


def make_checkpoint(directory: str) -> str:
    from hat_b200 import checkpoint
    p = os.path.join(directory, f"{VARIANT}_x{SCALE}_{WEIGHT_SEED}.safetensors")
    if not os.path.exists(p):
        checkpoint.make_checkpoint(p, VARIANT, SCALE, WEIGHT_SEED)
    return p


def arm_config(args, ws):
    """The workload description both arms print (the reference arm samples a crop of it)."""
    strip = args.shard == "strip"
    return {"workload": (f"{VARIANT.upper()} x{SCALE}, one {H}x{W} image split into row strips over "
                         f"{ws} GPU(s) (configs[3])") if strip else
                        f"{VARIANT.upper()} x{SCALE}, one {H}x{W} image per GPU (configs[1])",
            "variant": VARIANT, "scale": SCALE, "h": H, "w": W,
            "images_per_gpu": (1.0 / ws) if strip else 1,
            "mode": args.mode,
            "parallelism": (f"strip{ws} (row strips, NCCL halo exchange)" if strip
                            else f"dp{ws} (independent images)"),
            "l2": "256 MB buffer written between timed steps (> 126 MB L2)"}


def run_reference(args):
    """The reference arm: the CPU oracle port on all host cores, one crop per step."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from hat_b200 import synth
    crop = args.ref_crop
    with tempfile.TemporaryDirectory() as d:
        ck = make_checkpoint(d)
        img = synth.image(H, W, CFG_ID * 1000)
        for _ in range(args.warmup):
            cpu_oracle_sample(ck, img, crop)
        ts = []
        for _ in range(args.steps):
            dt, mpix = cpu_oracle_sample(ck, img, crop)
            ts.append(dt)
    t = float(np.mean(ts))
    value = mpix / t
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": metric_name(args.mode), "value": value, "unit": "Mpix/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong" if args.shard == "strip" else "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": arm_config(args, ws),
        "cpu_baseline": {"value": value, "unit": "Mpix/s", "cores": cores, "kind": "port",
                         "sample": f"numpy/OpenBLAS float32 restatement of the reference forward "
                                   f"(oracle/hat_oracle.py) on a {crop}x{crop} crop of the workload image per "
                                   f"step, {args.steps} steps"},
        "e2e": {"value": value, "unit": "Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    import hat_b200
    from hat_b200 import synth

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))

    def barrier():
        if ws > 1:
            dist.barrier()

    tmp = tempfile.mkdtemp()
    ck = make_checkpoint(tmp)
    mode = hat_b200.MODE_FAST if args.mode == "fast" else hat_b200.MODE_PARITY
    be = hat_b200.B200(ck, device=local, mode=mode, use_graph=True)
    strip = args.shard == "strip"
    if strip and ws > 1:
        # One NCCL communicator for the library's halo exchange; rank 0 makes its id.
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(hat_b200.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        be.attach_strip(rank, ws, bytes(uid.cpu().numpy().tobytes()))
    # Batch: every rank its own image. Strip: every rank the same image, its own rows.
    img = synth.image(H, W, CFG_ID * 1000 + (0 if strip else rank))
    # A dedicated stream: the library's kernels run on it and the timing events are
    # recorded on it (torch's default stream is the legacy NULL stream).
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    d_in = torch.from_numpy(img).cuda()
    d_out = torch.empty((3, H * SCALE, W * SCALE), device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")  # > 126 MB L2

    def step():
        be.forward_device(d_in.data_ptr(), d_out.data_ptr(), 1, H, W, st.cuda_stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    assert torch.isfinite(d_out).all().item(), "non-finite output"

    clocks = Clocks(local)
    launches0 = be.launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        flush.fill_(1.0)
        a.record(st)
        step()
        b.record(st)
    torch.cuda.synchronize()
    barrier()
    launches = be.launch_count() - launches0
    clk = clocks.stop()
    t_dev = sum(a.elapsed_time(b) for a, b in evs) / 1e3  # seconds for K steps, this rank
    if ws > 1:
        tt = torch.tensor([t_dev], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_dev = float(tt.item())
    out_mpix = (H * SCALE) * (W * SCALE) / 1e6
    images = 1 if strip else ws  # images the whole job finishes per step
    value = images * args.steps * out_mpix / t_dev

    d2h_rows = H * SCALE
    if strip and ws > 1:
        r0, r1 = hat_b200.strip_rows(H, ws, rank)
        d2h_rows = min(r1 * SCALE, H * SCALE) - r0 * SCALE
    # e2e: the public host entry point from pinned host memory, wall clock around it.
    h_in = torch.from_numpy(img).pin_memory()
    h_out = torch.empty((3, H * SCALE, W * SCALE)).pin_memory()

    def host_step():
        from hat_b200 import lib, _err, _check
        import ctypes
        e = _err()
        _check(lib().hat_b200_forward(be._h, 1, H, W, ctypes.c_void_p(h_in.data_ptr()),
                                      ctypes.c_void_p(h_out.data_ptr()), e, len(e)), e)

    host_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_step()
    t_e2e = time.perf_counter() - t0
    if ws > 1:
        tt = torch.tensor([t_e2e], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = float(tt.item())
    e2e = images * args.steps * out_mpix / t_e2e

    # Roofline of the dominant kernel, from an event-timed eager pass on this stream.
    prof = be.profile(H, W)
    top_kind, top = max(((k, v) for k, v in prof.items() if v["flops"] > 0 or v["bytes"] > 0),
                        key=lambda kv: kv[1]["ms"])
    hbm, tf, src = peaks()
    total_ms = sum(v["ms"] for v in prof.values())
    if top["flops"] > 0:
        achieved = top["flops"] / (top["ms"] / 1e3) / 1e12
        # Parity mode issues every product as 3 MMAs: fp16 pairs (kind::f16, the bf16 rate)
        # when the width is a multiple of 8, else tf32 pairs (kind::tf32, half that rate);
        # fast mode one tf32 MMA. pipe_frac is the tensor pipe's own utilisation.
        parity = mode == hat_b200.MODE_PARITY
        from hat_b200 import checkpoint as ck_mod
        h16 = parity and ck_mod.VARIANTS[VARIANT]["embed_dim"] % 8 == 0
        terms = 3 if parity else 1
        pipe_peak = tf if h16 else tf / 2
        roof = {"kernel": top_kind, "bound": "tensor", "achieved": achieved, "peak": tf,
                "unit": "TFLOP/s", "frac": achieved / tf, "traffic": None,
                "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
                "pipe_frac": terms * achieved / pipe_peak,
                "pipe_kind": "f16" if h16 else "tf32",
                "share_of_pass": top["ms"] / total_ms, "launches": top["launches"]}
    else:
        achieved = top["bytes"] / (top["ms"] / 1e3) / 1e9
        roof = {"kernel": top_kind, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": None, "peak_source": f"{src} HBM copy",
                "share_of_pass": top["ms"] / total_ms, "launches": top["launches"]}
    if top_kind in NCU_TRAFFIC_BYTES and not strip and (VARIANT, H, W) == ("hat-s", 512, 512):
        roof["traffic"] = NCU_TRAFFIC_BYTES[top_kind]
        roof["alg_bytes_per_launch"] = top["bytes"] / max(top["launches"], 1)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        dt, mpix = cpu_oracle_sample(ck, img, args.ref_crop)
        cpu = {"value": mpix / dt, "unit": "Mpix/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"oracle/hat_oracle.py (numpy float32) on a {args.ref_crop}x{args.ref_crop} "
                         f"crop of the workload image, one forward, {dt:.1f} s"}
    if rank == 0:
        line = {
            "metric": metric_name(args.mode), "value": value, "unit": "Mpix/s", "n_gpus": ws,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong" if strip else "weak",
            "vs_baseline": value / baseline_mpixs() if baseline_mpixs() else None,
            "dtype": "fp32" if mode == 0 else "tf32",
            "data": "synthetic",
            "config": arm_config(args, ws),
            # per rank: the whole input image in, this rank's output rows out (all of them
            # unless strip-sharded)
            "e2e": {"value": e2e, "unit": "Mpix/s", "h2d_bytes_per_step": 3 * H * W * 4,
                    "d2h_bytes_per_step": 3 * d2h_rows * W * SCALE * 4},
            "gpu_launches": launches,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk,
            "kernel_ms_per_pass": {k: round(v["ms"], 3) for k, v in sorted(prof.items())},
            "alg_tflops_per_s": images * FLOPS_PER_PIX * H * W / (t_dev / args.steps) / 1e12,
        }
        print(json.dumps(line), flush=True)
    be.close()
    if ws > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="parity", choices=["parity", "fast"])
    ap.add_argument("--ref-crop", type=int, default=96)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--shard", default="batch", choices=["batch", "strip"])
    args = ap.parse_args()
    select_workload(args.shard)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
