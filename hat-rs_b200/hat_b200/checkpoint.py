"""Seeded HAT checkpoints in the reference's safetensors layout.

The reference engine loads a `.safetensors` written by its `tools/convert.py`
(convert.py:106-258): every f32 tensor of HAT's `state_dict` under its PyTorch
name, the two int64 relative-position index buffers, and an `__metadata__` block
naming the architecture (convert.py:205-221, read back by src/weights.rs:60-129).
The released checkpoints are not available on this machine, so the benchmarks and
parity tests run on weights drawn here from a seeded generator with the same
initialisation rules HAT's constructor applies (hat_arch.py:873-880 for Linear and
LayerNorm, PyTorch's default Conv2d init, trunc-normal std 0.02 for the bias
tables), written in that same layout so the C-ABI reader sees an ordinary file.

`perturb=True` additionally randomises the LayerNorm affine parameters and the
Linear biases, which HAT's init leaves at 1/0. Parity tests use it so that a
kernel which drops a LayerNorm bias or a Linear bias cannot pass by accident.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field

import numpy as np

# The released configurations (tools/convert.py:55-63, tools/make_fixture.py:42-50).
VARIANTS = {
    "hat-s": dict(depths=[6] * 6, embed_dim=144, num_heads=6, mlp_ratio=2,
                  compress_ratio=24, squeeze_factor=24),
    "hat": dict(depths=[6] * 6, embed_dim=180, num_heads=6, mlp_ratio=2,
                compress_ratio=3, squeeze_factor=30),
    "hat-l": dict(depths=[6] * 12, embed_dim=180, num_heads=6, mlp_ratio=2,
                  compress_ratio=3, squeeze_factor=30),
}
WINDOW = 16
OVERLAP = 0.5
CONV_SCALE = 0.01
IMG_RANGE = 1.0
RGB_MEAN = (0.4488, 0.4371, 0.4040)
HEAD_FEAT = 64


@dataclass
class Arch:
    variant: str
    scale: int
    depths: list
    embed: int
    heads: int
    mlp_ratio: int
    compress_ratio: int
    squeeze_factor: int
    window: int = WINDOW
    overlap: float = OVERLAP
    conv_scale: float = CONV_SCALE
    img_range: float = IMG_RANGE
    mean: tuple = RGB_MEAN
    feat: int = HEAD_FEAT
    extra: dict = field(default_factory=dict)

    @property
    def owin(self) -> int:
        return self.window + int(self.window * self.overlap)

    @property
    def compressed(self) -> int:
        return self.embed // self.compress_ratio

    @property
    def squeezed(self) -> int:
        return self.embed // self.squeeze_factor

    def up_blocks(self):
        """(factor, widened channels) per upsampling block (src/weights.rs:290-305)."""
        if self.scale == 3:
            return [(3, 9 * self.feat)]
        s, n = self.scale, 0
        while s > 1 and s % 2 == 0:
            s //= 2
            n += 1
        if s != 1:
            raise ValueError(f"scale {self.scale}: HAT's Upsample builds 2^n and 3 only")
        return [(2, 4 * self.feat)] * n


def arch_of(variant: str, scale: int) -> Arch:
    v = VARIANTS[variant]
    return Arch(variant=variant, scale=scale, depths=list(v["depths"]), embed=v["embed_dim"],
                heads=v["num_heads"], mlp_ratio=v["mlp_ratio"],
                compress_ratio=v["compress_ratio"], squeeze_factor=v["squeeze_factor"])


def tensor_shapes(a: Arch):
    """Every f32 tensor of the checkpoint with its shape, in state_dict order
    (the list src/weights.rs:133-241 validates)."""
    c, win, owin = a.embed, a.window, a.owin
    out = [("conv_first.weight", (c, 3, 3, 3)), ("conv_first.bias", (c,)),
           ("patch_embed.norm.weight", (c,)), ("patch_embed.norm.bias", (c,))]
    for li, depth in enumerate(a.depths):
        for b in range(depth):
            p = f"layers.{li}.residual_group.blocks.{b}"
            out += [(f"{p}.norm1.weight", (c,)), (f"{p}.norm1.bias", (c,)),
                    (f"{p}.attn.relative_position_bias_table", ((2 * win - 1) ** 2, a.heads)),
                    (f"{p}.attn.qkv.weight", (3 * c, c)), (f"{p}.attn.qkv.bias", (3 * c,)),
                    (f"{p}.attn.proj.weight", (c, c)), (f"{p}.attn.proj.bias", (c,)),
                    (f"{p}.conv_block.cab.0.weight", (a.compressed, c, 3, 3)),
                    (f"{p}.conv_block.cab.0.bias", (a.compressed,)),
                    (f"{p}.conv_block.cab.2.weight", (c, a.compressed, 3, 3)),
                    (f"{p}.conv_block.cab.2.bias", (c,)),
                    (f"{p}.conv_block.cab.3.attention.1.weight", (a.squeezed, c, 1, 1)),
                    (f"{p}.conv_block.cab.3.attention.1.bias", (a.squeezed,)),
                    (f"{p}.conv_block.cab.3.attention.3.weight", (c, a.squeezed, 1, 1)),
                    (f"{p}.conv_block.cab.3.attention.3.bias", (c,)),
                    (f"{p}.norm2.weight", (c,)), (f"{p}.norm2.bias", (c,)),
                    (f"{p}.mlp.fc1.weight", (a.mlp_ratio * c, c)),
                    (f"{p}.mlp.fc1.bias", (a.mlp_ratio * c,)),
                    (f"{p}.mlp.fc2.weight", (c, a.mlp_ratio * c)), (f"{p}.mlp.fc2.bias", (c,))]
        p = f"layers.{li}.residual_group.overlap_attn"
        out += [(f"{p}.relative_position_bias_table", ((win + owin - 1) ** 2, a.heads)),
                (f"{p}.norm1.weight", (c,)), (f"{p}.norm1.bias", (c,)),
                (f"{p}.qkv.weight", (3 * c, c)), (f"{p}.qkv.bias", (3 * c,)),
                (f"{p}.proj.weight", (c, c)), (f"{p}.proj.bias", (c,)),
                (f"{p}.norm2.weight", (c,)), (f"{p}.norm2.bias", (c,)),
                (f"{p}.mlp.fc1.weight", (a.mlp_ratio * c, c)),
                (f"{p}.mlp.fc1.bias", (a.mlp_ratio * c,)),
                (f"{p}.mlp.fc2.weight", (c, a.mlp_ratio * c)), (f"{p}.mlp.fc2.bias", (c,)),
                (f"layers.{li}.conv.weight", (c, c, 3, 3)), (f"layers.{li}.conv.bias", (c,))]
    out += [("norm.weight", (c,)), ("norm.bias", (c,)),
            ("conv_after_body.weight", (c, c, 3, 3)), ("conv_after_body.bias", (c,)),
            ("conv_before_upsample.0.weight", (a.feat, c, 3, 3)),
            ("conv_before_upsample.0.bias", (a.feat,))]
    for i, (_r, widened) in enumerate(a.up_blocks()):
        out += [(f"upsample.{2 * i}.weight", (widened, a.feat, 3, 3)),
                (f"upsample.{2 * i}.bias", (widened,))]
    out += [("conv_last.weight", (3, a.feat, 3, 3)), ("conv_last.bias", (3,))]
    return out


def rpi_sa(win: int) -> np.ndarray:
    """`HAT.calculate_rpi_sa` (hat_arch.py:882-895): row = query, column = key,
    `(qy - ky + win - 1) * (2 win - 1) + (qx - kx + win - 1)`."""
    y, x = np.divmod(np.arange(win * win), win)
    dy = y[:, None] - y[None, :] + win - 1
    dx = x[:, None] - x[None, :] + win - 1
    return (dy * (2 * win - 1) + dx).astype(np.int64)


def rpi_oca(win: int, owin: int) -> np.ndarray:
    """`HAT.calculate_rpi_oca` (hat_arch.py:897-919): key minus query, shifted by
    `win - owin + 1`, so the buffer holds negative entries that PyTorch's indexing
    wraps modulo the table's `(win + owin - 1)^2` rows."""
    qy, qx = np.divmod(np.arange(win * win), win)
    ky, kx = np.divmod(np.arange(owin * owin), owin)
    dy = ky[None, :] - qy[:, None] + win - owin + 1
    dx = kx[None, :] - qx[:, None] + win - owin + 1
    return (dy * (win + owin - 1) + dx).astype(np.int64)


def _trunc_normal(rng, shape, std):
    return np.clip(rng.standard_normal(shape) * std, -2 * std, 2 * std).astype(np.float32)


def generate(a: Arch, seed: int, perturb: bool = False) -> dict:
    """Seeded weights for every tensor of `a`, following HAT's initialisation."""
    rng = np.random.Generator(np.random.PCG64(seed))
    shapes = tensor_shapes(a)
    by_name = dict(shapes)
    out = {}
    for name, shape in shapes:
        stem, last = name.rsplit(".", 1)
        conv_w = by_name.get(stem + ".weight")
        if name.endswith("relative_position_bias_table"):
            t = _trunc_normal(rng, shape, 0.02)
        elif conv_w is not None and len(conv_w) == 4:
            # Conv2d weight and bias: kaiming_uniform(a=sqrt 5), i.e. U(+-1/sqrt(fan_in)).
            bound = 1.0 / np.sqrt(conv_w[1] * conv_w[2] * conv_w[3])
            t = rng.uniform(-bound, bound, shape).astype(np.float32)
        elif len(shape) == 2:  # Linear weight
            t = _trunc_normal(rng, shape, 0.02)
        elif "norm" in stem:  # LayerNorm: weight 1, bias 0
            t = np.full(shape, 1.0 if last == "weight" else 0.0, np.float32)
            if perturb:
                span = 0.5 if last == "weight" else 0.2
                t = t + rng.uniform(-span, span, shape).astype(np.float32)
        else:  # Linear bias: 0
            t = np.zeros(shape, np.float32)
            if perturb:
                t = t + rng.uniform(-0.05, 0.05, shape).astype(np.float32)
        out[name] = np.ascontiguousarray(t, dtype=np.float32)
    out["relative_position_index_SA"] = rpi_sa(a.window)
    out["relative_position_index_OCA"] = rpi_oca(a.window, a.owin)
    return out


def metadata(a: Arch, source: str) -> dict:
    """The `__metadata__` keys src/weights.rs:64-66 requires (convert.py:205-221)."""
    return {
        "variant": a.variant, "scale": str(a.scale), "window_size": str(a.window),
        "overlap_ratio": str(a.overlap), "embed_dim": str(a.embed),
        "num_heads": str(a.heads), "mlp_ratio": str(a.mlp_ratio),
        "depths": ",".join(str(d) for d in a.depths),
        "compress_ratio": str(a.compress_ratio), "squeeze_factor": str(a.squeeze_factor),
        "conv_scale": str(a.conv_scale), "img_range": str(a.img_range),
        "rgb_mean": ",".join(str(m) for m in a.mean), "source": source, "format": "pt",
    }


def write_safetensors(path: str, tensors: dict, meta: dict) -> None:
    """A plain safetensors container: u64 header length, JSON header with
    `dtype`/`shape`/`data_offsets` per tensor plus `__metadata__`, then the data."""
    names = sorted(tensors)
    header, off, blobs = {}, 0, []
    for n in names:
        t = np.ascontiguousarray(tensors[n])
        dt = {np.dtype(np.float32): "F32", np.dtype(np.int64): "I64"}[t.dtype]
        raw = t.astype(t.dtype.newbyteorder("<")).tobytes()
        header[n] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    header["__metadata__"] = meta
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((-(8 + len(hj))) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def make_checkpoint(path: str, variant: str, scale: int, seed: int, perturb: bool = False) -> Arch:
    """Write a seeded checkpoint for `variant` at `scale` and return its arch."""
    a = arch_of(variant, scale)
    t = generate(a, seed, perturb)
    write_safetensors(path, t, metadata(a, f"seeded:{variant}:x{scale}:{seed}:{int(perturb)}"))
    return a
