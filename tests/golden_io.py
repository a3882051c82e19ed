"""Readers for the committed golden fixtures (tests/golden/)."""
import json
import struct
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def read_hatf(path):
    """HATF v1 (the reference's src/fixture.rs:44-78 format): header, input, expected."""
    raw = Path(path).read_bytes()
    magic, ver, h, w, c, scale, win, flags, _ = struct.unpack("<4sIIIIIIII", raw[:36])
    assert magic == b"HATF" and ver == 1 and flags == 0 and c == 3
    n_in = 3 * h * w
    x = np.frombuffer(raw[36:36 + 4 * n_in], "<f4").reshape(3, h, w).astype(np.float32)
    y = np.frombuffer(raw[36 + 4 * n_in:], "<f4").reshape(3, h * scale, w * scale).astype(np.float32)
    assert len(raw) == 36 + 4 * (n_in + 3 * h * scale * w * scale)
    return dict(h=h, w=w, scale=scale, win=win, input=x, expected=y)


def cases():
    return json.loads((GOLDEN / "manifest.json").read_text())


def checkpoint_for(case, directory):
    """Write the seeded checkpoint a golden case was made with; returns its path."""
    from hat_b200 import checkpoint
    p = Path(directory) / f"{case['name']}.safetensors"
    if not p.exists():
        checkpoint.make_checkpoint(str(p), case["variant"], case["scale"], case["seed"], case["perturb"])
    return str(p)
