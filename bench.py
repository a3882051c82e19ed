#!/usr/bin/env python3
"""Benchmark of the B200 HAT backend on the reference's headline workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|2|3|4] [--shard strip|batch] [--mode parity|fast]

Workloads (BASELINE.json `configs`; seeded synthetic images and seeded weights in the
reference's checkpoint layout, no dataset or released checkpoint on these machines):
  --config 1 (default)  HAT-S x4, one 512x512 image: the whole image on 1 GPU, split into
                        window-aligned row strips with per-layer NCCL halo exchange at N > 1
                        (strong scaling: the same image at every N).
  --config 2            HAT x4, eight 256x256 images per GPU (the batch split per GPU, weak).
  --config 3            HAT-L x4, one 1024x1024 image, row strips over the N GPUs (strong).
  --config 4            HAT-S x3, four 333x500 images per GPU (weak).
`--shard batch` with config 1 or 3 gives every rank its own image instead (weak).

Metric: output Mpix/s of the whole job. `value`: K timed steps of
`hat_b200_forward_device` with the inputs already in HBM, each step timed with CUDA events
on the launching stream with a 256 MB buffer (> 126 MB L2) written before it; the max over
ranks. `e2e`: the same metric through `hat_b200_forward` from pinned host memory to host
memory (the H2D of the inputs and the D2H of the outputs inside the timed region).
After timing, the outputs are checked against the fp32 reference (the oracle's torch
twin on the same GPU, TF32 off): `max_abs_err_vs_fp32_ref`, max over ranks; parity mode
must stay within the reference's 1e-4 (src/main.rs:310), fast mode above 50 dB PSNR.
`--impl reference` times the fp32 restatement of the reference forward (the oracle's
torch twin) on all host cores, one bounded crop of the workload per step: the
reference's own CPU path is Rust plus an un-vendored CUDA crate and cannot be built on
these machines.
"""
from __future__ import annotations

import argparse
import datetime
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

# BASELINE.json configs[i]: variant, scale, input size, images per rank (batch mode),
# default sharding, algorithmic FLOPs per padded input pixel (QK^T and PV counted once),
# the crop side the CPU legs time per step.
CONFIGS = {
    1: dict(variant="hat-s", scale=4, h=512, w=512, n=1, shard="strip", flops=26.67e6, crop=128),
    2: dict(variant="hat", scale=4, h=256, w=256, n=8, shard="batch", flops=50.72e6, crop=96),
    3: dict(variant="hat-l", scale=4, h=1024, w=1024, n=1, shard="strip", flops=99.12e6, crop=64),
    4: dict(variant="hat-s", scale=3, h=333, w=500, n=4, shard="batch", flops=25.83e6, crop=128),
}
WEIGHT_SEED = 2024
REF_GPU_S = 8.6      # seconds, README.md:18 of the reference (HAT-S x4 512x512, GPU, hardware unstated)
# DRAM bytes (read + write) per launch of a kernel kind, each from one ncu capture of the
# configuration-1 workload whose summary is committed under profiles/ (dram__bytes_read.sum +
# dram__bytes_write.sum); reported as the roofline's `traffic` when that kind is the top one.
TRAFFIC = {
    "attn.window": (454.2e6 + 129.6e6, "profiles/k_attn_tc_window_hats_x4_512.md"),
    "attn.overlap": (453.4e6 + 133.3e6, "profiles/k_attn_tc_overlap_hats_x4_512.md"),
    "mlp.fused": (302.5e6 + 109.8e6, "profiles/k_mlp_fused_hats_x4_512.md"),
    "linear.qkv": (151.4e6 + 399.8e6, "profiles/k_umma_linear_qkv_hats_x4_512.md"),
    "layernorm": (151.0e6 + 98.9e6, "profiles/k_layernorm_bulk_hats_x4_512.md"),
}
PARITY_TOL = 1e-4    # src/main.rs:310 VERIFY_TOL
PSNR_MIN = 50.0      # fast-mode bar


class Workload:
    def __init__(self, cfg: int, shard: str | None, mode: str, ws: int):
        c = CONFIGS[cfg]
        self.cfg, self.mode, self.ws = cfg, mode, ws
        self.variant, self.scale, self.h, self.w = c["variant"], c["scale"], c["h"], c["w"]
        self.shard = shard or c["shard"]
        self.strip = self.shard == "strip" and ws > 1
        # images each rank runs per step (strip: one image shared by all ranks)
        self.n = c["n"] if self.shard == "batch" else 1
        self.flops_per_pix = c["flops"]
        self.crop = c["crop"]
        self.hp, self.wp = -(-self.h // 16) * 16, -(-self.w // 16) * 16

    def metric(self) -> str:
        if self.cfg == 1 and self.mode == "parity":
            # BASELINE.json's `metric`, verbatim
            return "output Mpix/s, HAT-S x4 512² input at 1/2/4/8 B200; max abs err vs fp32 ref"
        m = "fp32-parity" if self.mode == "parity" else "fast (tf32)"
        return f"output Mpix/s, {self.variant.upper()} x{self.scale} {self.h}x{self.w} input ({m} mode)"

    def images_per_step(self) -> int:
        """Images the whole job finishes per step."""
        return 1 if self.strip else self.n * self.ws

    def out_mpix(self) -> float:
        return (self.h * self.scale) * (self.w * self.scale) / 1e6

    def config(self) -> dict:
        if self.shard == "strip" and self.ws == 1:
            what = (f"{self.variant.upper()} x{self.scale}, one {self.h}x{self.w} image on one GPU "
                    f"(configs[{self.cfg}]; split into row strips over the GPUs at N > 1)")
            par = "single GPU (row strips with NCCL halo exchange at N > 1)"
        elif self.shard == "strip":
            what = (f"{self.variant.upper()} x{self.scale}, one {self.h}x{self.w} image split into window-aligned "
                    f"row strips over {self.ws} GPUs (configs[{self.cfg}])")
            par = f"strip{self.ws} (row strips, NCCL halo exchange)"
        else:
            what = (f"{self.variant.upper()} x{self.scale}, {self.n} {self.h}x{self.w} image(s) per GPU "
                    f"(configs[{self.cfg}])")
            par = f"dp{self.ws} (independent images)"
        return {"workload": what, "variant": self.variant, "scale": self.scale, "h": self.h, "w": self.w,
                "images_per_gpu": (1.0 / self.ws) if self.strip else self.n, "mode": self.mode,
                "parallelism": par, "l2": "256 MB buffer written between timed steps (> 126 MB L2)"}

    def images(self, rank: int) -> np.ndarray:
        """`[n][3][h][w]`: this rank's inputs (strip: the shared image)."""
        from hat_b200 import synth
        if self.shard == "strip":
            return synth.image(self.h, self.w, self.cfg * 1000)[None]
        return np.stack([synth.image(self.h, self.w, self.cfg * 1000 + rank * self.n + i) for i in range(self.n)])


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


def make_checkpoint(directory: str, wl: Workload) -> str:
    from hat_b200 import checkpoint
    p = os.path.join(directory, f"{wl.variant}_x{wl.scale}_{WEIGHT_SEED}.safetensors")
    if not os.path.exists(p):
        checkpoint.make_checkpoint(p, wl.variant, wl.scale, WEIGHT_SEED)
    return p


def cpu_numpy_sample(ck: str, img: np.ndarray, crop: int, scale: int):
    """One numpy-oracle forward of a crop of the workload image: (seconds, out Mpix)."""
    from oracle import hat_oracle as O
    m = O.Model.load(ck)
    t = time.perf_counter()
    y = O.forward(m, img[:, :crop, :crop])
    dt = time.perf_counter() - t
    assert y.shape == (3, crop * scale, crop * scale)
    return dt, (crop * scale) ** 2 / 1e6


def run_reference(args, wl: Workload):
    """The reference arm: the fp32 torch restatement of the reference forward on all host
    cores (torch CPU), one crop of the workload per step; rank 0 only."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import torch
    from oracle import hat_torch as T
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    crop = args.ref_crop or wl.crop
    with tempfile.TemporaryDirectory() as d:
        ck = make_checkpoint(d, wl)
        wt = T.Weights.load(ck, "cpu")
        img = wl.images(0)[0][:, :crop, :crop]
        for _ in range(args.warmup):
            T.forward(wt, img)
        ts = []
        for _ in range(args.steps):
            t = time.perf_counter()
            y = T.forward(wt, img)
            ts.append(time.perf_counter() - t)
        assert y.shape == (3, crop * wl.scale, crop * wl.scale)
    t = float(np.mean(ts))
    value = (crop * wl.scale) ** 2 / 1e6 / t
    cfg = wl.config()
    cfg.update({"mode": "fp32 (torch CPU, strict fp32)", "parallelism": f"one host process, {threads} threads",
                "l2": "n/a (CPU)"})
    line = {
        "impl": "reference", "metric": wl.metric(), "value": value, "unit": "Mpix/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong" if wl.shard == "strip" else "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": value, "unit": "Mpix/s", "cores": threads, "kind": "port",
                         "sample": f"oracle/hat_torch.py (the reference forward restated with torch CPU ops, "
                                   f"fp32) on a {crop}x{crop} crop of the workload image per step, "
                                   f"{args.steps} steps"},
        "e2e": {"value": value, "unit": "Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def verify(wl: Workload, ck: str, imgs: np.ndarray, outs: np.ndarray, rank: int):
    """Max abs error and min PSNR of this rank's outputs against the fp32 reference (the
    oracle's torch twin on this GPU); strip mode compares this rank's own rows."""
    import hat_b200
    from oracle import hat_torch as T
    wt = T.Weights.load(ck, "cuda")
    rows = slice(0, wl.h * wl.scale)
    if wl.strip:
        r0, r1 = hat_b200.strip_rows(wl.h, wl.ws, rank)
        rows = slice(r0 * wl.scale, min(r1 * wl.scale, wl.h * wl.scale))
    err, psnr = 0.0, float("inf")
    for i in range(imgs.shape[0]):
        want = T.forward(wt, imgs[i])[:, rows]
        got = outs[i][:, rows]
        err = max(err, float(np.abs(got - want).max()))
        mse = float(((got.astype(np.float64) - want) ** 2).mean())
        psnr = min(psnr, 10 * np.log10(1.0 / max(mse, 1e-30)))
    del wt
    import torch
    torch.cuda.empty_cache()
    return err, psnr


def run_ours(args, wl: Workload):
    import torch
    import torch.distributed as dist
    import hat_b200

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))

    def barrier():
        if ws > 1:
            dist.barrier()

    def allmax(v: float) -> float:
        if ws == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    tmp = tempfile.mkdtemp()
    ck = make_checkpoint(tmp, wl)
    mode = hat_b200.MODE_FAST if args.mode == "fast" else hat_b200.MODE_PARITY
    be = hat_b200.B200(ck, device=local, mode=mode, use_graph=True)
    if wl.strip:
        # One NCCL communicator for the library's halo exchange; rank 0 makes its id.
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(hat_b200.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        be.attach_strip(rank, ws, bytes(uid.cpu().numpy().tobytes()))
    imgs = wl.images(rank)
    n, H, W, S = imgs.shape[0], wl.h, wl.w, wl.scale
    # A dedicated stream: the library's kernels run on it and the timing events are
    # recorded on it (torch's default stream is the legacy NULL stream).
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    d_in = torch.from_numpy(imgs).cuda()
    d_out = torch.zeros((n, 3, H * S, W * S), device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")  # > 126 MB L2

    def step():
        be.forward_device(d_in.data_ptr(), d_out.data_ptr(), n, H, W, st.cuda_stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    be.sync()

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
    be.sync()
    t_dev = allmax(sum(a.elapsed_time(b) for a, b in evs) / 1e3)  # seconds for K steps
    value = wl.images_per_step() * args.steps * wl.out_mpix() / t_dev
    outs = d_out.cpu().numpy()

    d2h_rows = H * S
    if wl.strip:
        r0, r1 = hat_b200.strip_rows(H, ws, rank)
        d2h_rows = min(r1 * S, H * S) - r0 * S
    # e2e: the public host entry point from pinned host memory, wall clock around it.
    h_in = torch.from_numpy(imgs).pin_memory()
    h_out = torch.empty((n, 3, H * S, W * S)).pin_memory()

    def host_step():
        from hat_b200 import lib, _err, _check
        import ctypes
        e = _err()
        _check(lib().hat_b200_forward(be._h, n, H, W, ctypes.c_void_p(h_in.data_ptr()),
                                      ctypes.c_void_p(h_out.data_ptr()), e, len(e)), e)

    host_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_step()
    t_e2e = allmax(time.perf_counter() - t0)
    e2e = wl.images_per_step() * args.steps * wl.out_mpix() / t_e2e

    # Roofline of the dominant kernel, from an event-timed eager pass on this stream
    # (every rank takes part: a strip-sharded pass has collectives).
    prof = be.profile(H, W)
    top_kind, top = max(((k, v) for k, v in prof.items() if v["flops"] > 0 or v["bytes"] > 0),
                        key=lambda kv: kv[1]["ms"])
    hbm, tf, src = peaks()
    total_ms = sum(v["ms"] for v in prof.values())
    traffic, traffic_src = TRAFFIC.get(top_kind, (None, None)) if wl.cfg == 1 and mode == hat_b200.MODE_PARITY \
        else (None, None)
    parity = mode == hat_b200.MODE_PARITY
    h16 = be.fp16_pairs()
    if top["flops"] > 0:
        achieved = top["flops"] / (top["ms"] / 1e3) / 1e12
        # Parity mode issues every product as 3 MMAs: fp16 pairs (kind::f16, the bf16 rate)
        # or tf32 pairs (kind::tf32, half that rate); fast mode one tf32 MMA. pipe_frac is
        # the tensor pipe's own utilisation.
        terms = 3 if parity else 1
        pipe_peak = tf if h16 else tf / 2
        roof = {"kernel": top_kind, "bound": "tensor", "achieved": achieved, "peak": tf,
                "unit": "TFLOP/s", "frac": achieved / tf, "traffic": traffic, "traffic_source": traffic_src,
                "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
                "pipe_frac": terms * achieved / pipe_peak, "pipe_kind": "f16" if h16 else "tf32",
                "share_of_pass": top["ms"] / total_ms, "launches": top["launches"],
                "alg_bytes_per_launch": top["bytes"] / max(top["launches"], 1),
                "alg_flops_per_launch": top["flops"] / max(top["launches"], 1)}
    else:
        achieved = top["bytes"] / (top["ms"] / 1e3) / 1e9
        roof = {"kernel": top_kind, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic, "traffic_source": traffic_src,
                "peak_source": f"{src} HBM copy",
                "share_of_pass": top["ms"] / total_ms, "launches": top["launches"],
                "alg_bytes_per_launch": top["bytes"] / max(top["launches"], 1)}

    # Correctness of the timed outputs against the fp32 reference (outside the timed region).
    err, psnr = (None, None)
    if not args.no_verify:
        err, psnr = verify(wl, ck, imgs, outs, rank)
        err = allmax(err)
        psnr = -allmax(-psnr)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        dt, mpix = cpu_numpy_sample(ck, imgs[0], args.ref_crop or wl.crop, S)
        cpu = {"value": mpix / dt, "unit": "Mpix/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"oracle/hat_oracle.py (numpy float32, OpenBLAS on all host cores) on a "
                         f"{args.ref_crop or wl.crop}x{args.ref_crop or wl.crop} crop of the workload "
                         f"image, one forward, {dt:.1f} s"}
    if rank == 0:
        line = {
            "metric": wl.metric(), "value": value, "unit": "Mpix/s", "n_gpus": ws,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong" if wl.shard == "strip" else "weak",
            "vs_baseline": (value / ((H * S) * (W * S) / 1e6 / REF_GPU_S)) if wl.cfg == 1 else None,
            "dtype": ("fp32 via fp16 hi/lo pairs (3 MMAs per product)" if h16 else
                      "fp32 via tf32 hi/lo pairs (3 MMAs per product)") if parity else "tf32",
            "data": "synthetic",
            "config": wl.config(),
            "max_abs_err_vs_fp32_ref": err,
            "psnr_db_vs_fp32_ref": psnr,
            "parity_tol": PARITY_TOL if parity else None,
            "parity_ok": (err is not None and err <= PARITY_TOL) if parity else
                         (psnr is not None and psnr >= PSNR_MIN),
            # per rank: its inputs in, its outputs out (strip: the whole image in, its own rows out)
            "e2e": {"value": e2e, "unit": "Mpix/s", "h2d_bytes_per_step": int(imgs.nbytes),
                    "d2h_bytes_per_step": 3 * n * d2h_rows * W * S * 4},
            "gpu_launches": launches,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk,
            "kernel_ms_per_pass": {k: round(v["ms"], 3) for k, v in sorted(prof.items())},
            "alg_tflops_per_s": wl.images_per_step() * wl.flops_per_pix * wl.hp * wl.wp / (t_dev / args.steps) / 1e12,
        }
        print(json.dumps(line), flush=True)
    be.close()
    if ws > 1:
        dist.destroy_process_group()
    if parity and err is not None and err > PARITY_TOL:
        print(f"bench: max abs error {err:.3e} exceeds {PARITY_TOL}", file=sys.stderr)
        return 1
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="parity", choices=["parity", "fast"])
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--shard", default=None, choices=["batch", "strip"])
    ap.add_argument("--ref-crop", type=int, default=0, help="crop side of the CPU legs (0: per config)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    args = ap.parse_args()
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    wl = Workload(args.config, args.shard, args.mode, ws)
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    sys.exit(main())
