"""Seeded synthetic RGB inputs for the benchmark and parity configurations.

No image dataset is available on the GPU machines, so every configuration runs on
images drawn here: per image and channel, 0.5 plus a sum of three sinusoids
`a_k sin(2 pi (fx_k x / w + fy_k y / h) + phi_k)` with (a, f, phi) drawn from a
seeded PCG64 generator, plus uniform noise in (-0.05, 0.05), clamped to [0, 1] and
quantised to k/255 like an 8-bit PNG decoded by the reference's image loader
(src/image.rs:43-96). The seed of image `i` of configuration `cfg` is
`cfg * 1000 + i`, so every process that asks for the same image gets the same
bytes.
"""
from __future__ import annotations

import numpy as np


def image(h: int, w: int, seed: int) -> np.ndarray:
    """One planar `[3][h][w]` float32 image in [0, 1], quantised to k/255."""
    rng = np.random.Generator(np.random.PCG64(seed))
    y = np.arange(h, dtype=np.float64)[:, None]
    x = np.arange(w, dtype=np.float64)[None, :]
    out = np.empty((3, h, w), np.float32)
    for ch in range(3):
        v = np.full((h, w), 0.5)
        for _ in range(3):
            a = rng.uniform(0.05, 0.2)
            fx, fy = rng.uniform(0.5, 8.0, 2)
            phi = rng.uniform(0.0, 2 * np.pi)
            v += a * np.sin(2 * np.pi * (fx * x / w + fy * y / h) + phi)
        v += rng.uniform(-0.05, 0.05, (h, w))
        out[ch] = (np.round(np.clip(v, 0.0, 1.0) * 255.0) / 255.0).astype(np.float32)
    return out


def batch(n: int, h: int, w: int, cfg: int) -> np.ndarray:
    """`[n][3][h][w]` float32: image `i` is `image(h, w, cfg * 1000 + i)`."""
    return np.stack([image(h, w, cfg * 1000 + i) for i in range(n)])
