#!/usr/bin/env python3
"""Generate the golden fixtures from the reference's own network definition.

Run in a container where the reference checkout is available (it is not on the GPU
machines, which only read the committed outputs):

    python tests/golden/make_golden.py --reference <path to hat-rs checkout>

For every case below this builds upstream HAT (`tools/hat_arch.py`, through the
reference's `tools/make_fixture.py:build`), loads the seeded weights that
`hat_b200.checkpoint.generate` draws for (variant, scale, seed, perturb), runs the
seeded synthetic image through it exactly as the reference engine's `Backend`
contract does (edge-replicated padding to a window multiple, src/backend.rs:71-89;
crop after, src/backend.rs:94-109), and writes a HATF v1 fixture (the format of
src/fixture.rs:44-78: magic, u32 version/h/w/c/scale/win/flags/reserved, the f32
input, the f32 expected output). `manifest.json` records how each case was made.

It also records the reference's own geometry: HAT's `calculate_rpi_sa`,
`calculate_rpi_oca` and `calculate_mask` outputs for a few plane sizes, in
`geometry.npz`, so the oracle's index maps are checked against them.
"""
import argparse
import json
import struct
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "hat-rs_b200"))

from hat_b200 import checkpoint, synth  # noqa: E402

# (name, variant, scale, h, w, weight seed, perturb, input config id)
CASES = [
    ("hats_x4_48x48_p", "hat-s", 4, 48, 48, 11, True, 101),
    ("hats_x4_37x29_p", "hat-s", 4, 37, 29, 12, True, 102),
    ("hats_x3_48x32_p", "hat-s", 3, 48, 32, 13, True, 103),
    ("hat_x4_32x48", "hat", 4, 32, 48, 14, False, 104),
    ("hatl_x4_16x16_p", "hat-l", 4, 16, 16, 15, True, 105),
    ("hats_x2_32x16_p", "hat-s", 2, 32, 16, 16, True, 106),
]
GEOMETRIES = [(16, 16), (32, 32), (48, 48), (32, 48), (64, 32)]
CFG_KEYS = {"hat-s": "s", "hat": "m", "hat-l": "l"}


def write_hatf(path, h, w, scale, win, x, y):
    head = struct.pack("<4sIIIIIIII", b"HATF", 1, h, w, 3, scale, win, 0, 0)
    with open(path, "wb") as f:
        f.write(head)
        f.write(np.ascontiguousarray(x, "<f4").tobytes())
        f.write(np.ascontiguousarray(y, "<f4").tobytes())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="hat-rs checkout (read only)")
    args = ap.parse_args()
    tools = Path(args.reference) / "tools"
    sys.path.insert(0, str(tools))
    import timm_shim  # noqa: E402
    timm_shim.install()
    import make_fixture  # noqa: E402

    torch.set_num_threads(8)
    manifest = []
    for name, variant, scale, h, w, seed, perturb, cfg in CASES:
        model = make_fixture.build(CFG_KEYS[variant], scale).eval()
        arch = checkpoint.arch_of(variant, scale)
        t = checkpoint.generate(arch, seed, perturb)
        sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in t.items()}
        missing, unexpected = model.load_state_dict(sd, strict=True), None
        img = synth.image(h, w, cfg * 1000)
        win = arch.window
        hp, wp = -(-h // win) * win, -(-w // win) * win
        padded = np.pad(img, ((0, 0), (0, hp - h), (0, wp - w)), mode="edge")
        with torch.no_grad():
            y = model(torch.from_numpy(padded)[None])[0].numpy()
        y = y[:, :h * scale, :w * scale]
        write_hatf(HERE / f"{name}.bin", h, w, scale, win, img, y)
        manifest.append(dict(name=name, variant=variant, scale=scale, h=h, w=w, seed=seed,
                             perturb=perturb, input_seed=cfg * 1000))
        print(f"{name}: out {y.shape} range [{y.min():.4f}, {y.max():.4f}]")
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")

    geo = {}
    m = make_fixture.build("s", 4)
    geo["rpi_sa"] = m.calculate_rpi_sa().numpy().astype(np.int64)
    geo["rpi_oca"] = m.calculate_rpi_oca().numpy().astype(np.int64)
    for (gh, gw) in GEOMETRIES:
        mask = m.calculate_mask((gh, gw)).numpy()
        geo[f"mask_{gh}x{gw}"] = mask.astype(np.float32)
    np.savez_compressed(HERE / "geometry.npz", **geo)
    print("wrote geometry.npz")


if __name__ == "__main__":
    main()
