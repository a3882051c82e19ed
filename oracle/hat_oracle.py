"""CPU oracle for the HAT forward pass — TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA backend is held against. Only the tests, the
smoke entry point and the benchmark's CPU-baseline leg may import it; the product
path never calls it and has no CPU fallback.

It is a float32 numpy restatement of the reference's forward: the network defined by
upstream `tools/hat_arch.py` (whose output is what the reference's `--verify`
fixtures hold) in the order the reference's own CPU backend evaluates it
(`src/cpu.rs`). Activations are token-major `[H][W][C]` planes. Each function names
the reference lines it follows. Parity of this oracle is pinned against outputs of
`tools/hat_arch.py` itself (the committed fixtures under `tests/golden/`, made by
`tests/golden/make_golden.py`) and against the reference's shipped scale-3 fixture.
"""
from __future__ import annotations

import json
import struct

import numpy as np
from scipy.special import erf

EPS = 1e-5      # nn.LayerNorm default (src/gpu.rs:65)
LEAKY = 0.01    # nn.LeakyReLU default (src/gpu.rs:72)
MASK = -100.0   # calculate_mask fill (hat_arch.py:921-941)


# --------------------------------------------------------------------------- weights

def load_safetensors(path: str):
    """Tensors and `__metadata__` of a safetensors file (F32 and I64 only)."""
    with open(path, "rb") as f:
        raw = f.read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + hlen])
    meta = header.pop("__metadata__", {})
    base = 8 + hlen
    out = {}
    for name, info in header.items():
        dt = {"F32": np.float32, "I64": np.int64}[info["dtype"]]
        a, b = info["data_offsets"]
        out[name] = np.frombuffer(raw[base + a:base + b], dtype=np.dtype(dt).newbyteorder("<")) \
            .reshape(info["shape"]).astype(dt)
    return out, meta


class Model:
    """The checkpoint plus the architecture its metadata names (src/weights.rs:60-129)."""

    def __init__(self, tensors: dict, meta: dict):
        self.t = tensors
        self.variant = meta["variant"]
        self.scale = int(meta["scale"])
        self.win = int(meta["window_size"])
        self.owin = self.win + int(self.win * float(meta["overlap_ratio"]))
        self.c = int(meta["embed_dim"])
        self.heads = int(meta["num_heads"])
        self.depths = [int(d) for d in meta["depths"].split(",")]
        self.conv_scale = float(meta["conv_scale"])
        self.img_range = float(meta["img_range"])
        self.mean = np.array([float(m) for m in meta["rgb_mean"].split(",")], np.float32)
        self.feat = tensors["conv_before_upsample.0.weight"].shape[0]

    @classmethod
    def load(cls, path: str) -> "Model":
        return cls(*load_safetensors(path))

    def up_blocks(self):
        """src/weights.rs:290-305."""
        if self.scale == 3:
            return [(3, 9 * self.feat)]
        n, s = 0, self.scale
        while s > 1:
            s //= 2
            n += 1
        return [(2, 4 * self.feat)] * n


# --------------------------------------------------------------------------- ops

def layer_norm(x, g, b):
    """nn.LayerNorm over the channel axis, biased variance, eps 1e-5
    (src/cpu.rs:563-581)."""
    mu = x.mean(-1, keepdims=True, dtype=np.float32)
    d = x - mu
    var = (d * d).mean(-1, keepdims=True, dtype=np.float32)
    return (d / np.sqrt(var + np.float32(EPS)) * g + b).astype(np.float32)


def gelu(x):
    """Exact erf GELU, nn.GELU's default (src/cpu.rs:584-603)."""
    return (0.5 * x * (1.0 + erf(x * np.float32(1 / np.sqrt(2))))).astype(np.float32)


def conv3x3(x, w, b):
    """Conv2d(k=3, s=1, p=1) on a `[H][W][Cin]` plane with PyTorch `[Cout][Cin][3][3]`
    weights (src/cpu.rs:304-422): nine shifted matmuls over the zero-padded plane."""
    h, wd, _ = x.shape
    xp = np.pad(x, ((1, 1), (1, 1), (0, 0)))
    out = np.broadcast_to(b.astype(np.float32), (h, wd, w.shape[0])).copy()
    for dy in range(3):
        for dx in range(3):
            out += xp[dy:dy + h, dx:dx + wd, :] @ w[:, :, dy, dx].T
    return out


def linear(x, w, b):
    """nn.Linear on token rows (src/cpu.rs:456-555)."""
    return (x @ w.T + b).astype(np.float32)


def rpi_sa(win):
    """hat_arch.py:882-895 / src/plan.rs:357-372."""
    y, x = np.divmod(np.arange(win * win), win)
    return (y[:, None] - y[None, :] + win - 1) * (2 * win - 1) + (x[:, None] - x[None, :] + win - 1)


def rpi_oca(win, owin):
    """hat_arch.py:897-919 / src/plan.rs:397-416 (negative entries wrap)."""
    qy, qx = np.divmod(np.arange(win * win), win)
    ky, kx = np.divmod(np.arange(owin * owin), owin)
    dy = ky[None, :] - qy[:, None] + win - owin + 1
    dx = kx[None, :] - qx[:, None] + win - owin + 1
    return dy * (win + owin - 1) + dx


def mask_labels(hp, wp, win, shift):
    """Region label of every pixel of the shifted frame, `band(y) * 3 + band(x)` with
    bands `[0, hp-win)`, `[hp-win, hp-shift)`, `[hp-shift, hp)` (calculate_mask,
    hat_arch.py:921-941; src/plan.rs:300-334)."""
    def band(size):
        b = np.zeros(size, np.int32)
        b[max(size - win, 0):] = 1
        b[max(size - shift, 0):] = 2
        return b
    return band(hp)[:, None] * 3 + band(wp)[None, :]


def partition(x, win):
    """window_partition (hat_arch.py:95-107): `[H][W][C]` → `[nw][win*win][C]`."""
    h, w, c = x.shape
    return x.reshape(h // win, win, w // win, win, c).transpose(0, 2, 1, 3, 4) \
        .reshape(-1, win * win, c)


def reverse(x, win, h, w):
    """window_reverse (hat_arch.py:110-125)."""
    c = x.shape[-1]
    return x.reshape(h // win, w // win, win, win, c).transpose(0, 2, 1, 3, 4).reshape(h, w, c)


def softmax_attention(q, k, v, bias, mask=None, chunk=64):
    """`softmax(q*scale @ k^T + bias (+ mask)) @ v` per window and head, with q already
    scaled (hat_arch.py:165-196, 392-438; src/cpu.rs:772-844). q `[nw][h][nq][d]`,
    k/v `[nw][h][nk][d]`, bias `[h][nq][nk]`, mask `[nw][nq][nk]`."""
    out = np.empty(q.shape, np.float32)
    for s in range(0, q.shape[0], chunk):
        e = slice(s, s + chunk)
        a = q[e] @ k[e].transpose(0, 1, 3, 2) + bias[None]
        if mask is not None:
            a = a + mask[e][:, None]
        a = a - a.max(-1, keepdims=True)
        np.exp(a, out=a)
        a /= a.sum(-1, keepdims=True)
        out[e] = a @ v[e]
    return out


def split_heads(x, heads):
    nw, n, c = x.shape
    return x.reshape(nw, n, heads, c // heads).transpose(0, 2, 1, 3)


def merge_heads(x):
    nw, h, n, d = x.shape
    return x.transpose(0, 2, 1, 3).reshape(nw, n, h * d)


# --------------------------------------------------------------------------- blocks

class Forward:
    """One forward pass over a padded plane (src/cpu.rs:1318-1368)."""

    def __init__(self, m: Model, hp: int, wp: int):
        self.m, self.hp, self.wp = m, hp, wp
        win, owin = m.win, m.owin
        self.shift = win // 2
        self.idx_sa = rpi_sa(win) % ((2 * win - 1) ** 2)
        self.idx_oca = rpi_oca(win, owin) % ((win + owin - 1) ** 2)
        lab = partition(mask_labels(hp, wp, win, self.shift)[:, :, None], win)[..., 0]
        self.mask = np.where(lab[:, :, None] != lab[:, None, :], np.float32(MASK),
                             np.float32(0)).astype(np.float32)

    def w(self, name):
        return self.m.t[name]

    def cab(self, x, p):
        """conv → GELU → conv → channel attention, NO residual (hat_arch.py:40-74,
        src/cpu.rs:918-960)."""
        y = gelu(conv3x3(x, self.w(f"{p}.cab.0.weight"), self.w(f"{p}.cab.0.bias")))
        y = conv3x3(y, self.w(f"{p}.cab.2.weight"), self.w(f"{p}.cab.2.bias"))
        pooled = y.reshape(-1, y.shape[-1]).mean(0, dtype=np.float32)
        s = self.w(f"{p}.cab.3.attention.1.weight")[:, :, 0, 0] @ pooled \
            + self.w(f"{p}.cab.3.attention.1.bias")
        s = np.maximum(s, 0)
        g = self.w(f"{p}.cab.3.attention.3.weight")[:, :, 0, 0] @ s \
            + self.w(f"{p}.cab.3.attention.3.bias")
        g = (1.0 / (1.0 + np.exp(-g))).astype(np.float32)
        return (y * g).astype(np.float32)

    def mlp(self, x, p):
        """`x + fc2(gelu(fc1(norm2(x))))` (src/gpu.rs:449-466)."""
        n = layer_norm(x, self.w(f"{p}.norm2.weight"), self.w(f"{p}.norm2.bias"))
        hdn = gelu(linear(n, self.w(f"{p}.mlp.fc1.weight"), self.w(f"{p}.mlp.fc1.bias")))
        return x + linear(hdn, self.w(f"{p}.mlp.fc2.weight"), self.w(f"{p}.mlp.fc2.bias"))

    def hab(self, x, stage, blk):
        """HAB.forward (hat_arch.py:266-309; src/cpu.rs:1090-1166)."""
        m = self.m
        p = f"layers.{stage}.residual_group.blocks.{blk}"
        c, heads, win = m.c, m.heads, m.win
        d = c // heads
        n = layer_norm(x, self.w(f"{p}.norm1.weight"), self.w(f"{p}.norm1.bias"))
        conv_x = self.cab(n, f"{p}.conv_block")
        s = self.shift if blk % 2 == 1 else 0
        xs = np.roll(n, (-s, -s), axis=(0, 1)) if s else n
        win_t = partition(xs, win)
        qkv = linear(win_t, self.w(f"{p}.attn.qkv.weight"), self.w(f"{p}.attn.qkv.bias"))
        q = split_heads(qkv[..., :c], heads) * np.float32(d ** -0.5)
        k = split_heads(qkv[..., c:2 * c], heads)
        v = split_heads(qkv[..., 2 * c:], heads)
        tab = self.w(f"{p}.attn.relative_position_bias_table")
        bias = tab[self.idx_sa.reshape(-1)].reshape(win * win, win * win, heads) \
            .transpose(2, 0, 1)
        a = merge_heads(softmax_attention(q, k, v, bias, self.mask if s else None))
        a = linear(a, self.w(f"{p}.attn.proj.weight"), self.w(f"{p}.attn.proj.bias"))
        a = reverse(a, win, self.hp, self.wp)
        if s:
            a = np.roll(a, (s, s), axis=(0, 1))
        # `shortcut + attn_x + conv_x * conv_scale`, in that order (hat_arch.py:305).
        x = (x + a) + conv_x * np.float32(m.conv_scale)
        return self.mlp(x, p)

    def ocab(self, x, stage):
        """OCAB.forward (hat_arch.py:392-438; src/cpu.rs:983-1055): 16x16 queries
        against the 24x24 `nn.Unfold(stride 16, padding 4)` neighbourhood of k and v,
        zero outside the plane, relative-position bias, no mask."""
        m = self.m
        p = f"layers.{stage}.residual_group.overlap_attn"
        c, heads, win, owin = m.c, m.heads, m.win, m.owin
        d = c // heads
        pad = (owin - win) // 2
        n = layer_norm(x, self.w(f"{p}.norm1.weight"), self.w(f"{p}.norm1.bias"))
        qkv = linear(n, self.w(f"{p}.qkv.weight"), self.w(f"{p}.qkv.bias"))
        q = split_heads(partition(qkv[..., :c], win), heads) * np.float32(d ** -0.5)
        kvp = np.pad(qkv[..., c:], ((pad, pad), (pad, pad), (0, 0)))
        ny, nx = self.hp // win, self.wp // win
        kv = np.empty((ny * nx, owin * owin, 2 * c), np.float32)
        for wy in range(ny):
            for wx in range(nx):
                kv[wy * nx + wx] = kvp[wy * win:wy * win + owin, wx * win:wx * win + owin] \
                    .reshape(owin * owin, 2 * c)
        k = split_heads(kv[..., :c], heads)
        v = split_heads(kv[..., c:], heads)
        tab = self.w(f"{p}.relative_position_bias_table")
        bias = tab[self.idx_oca.reshape(-1)].reshape(win * win, owin * owin, heads) \
            .transpose(2, 0, 1)
        a = merge_heads(softmax_attention(q, k, v, bias))
        a = reverse(a, win, self.hp, self.wp)
        x = linear(a, self.w(f"{p}.proj.weight"), self.w(f"{p}.proj.bias")) + x
        return self.mlp(x, p)

    def run(self, x0):
        """`x0` is the padded, mean-adjusted `[hp][wp][3]` plane; returns the padded
        output plane `[hp*s][wp*s][3]` in network units (hat_arch.py:971-984)."""
        m = self.m
        body = conv3x3(x0, self.w("conv_first.weight"), self.w("conv_first.bias"))
        x = layer_norm(body, self.w("patch_embed.norm.weight"), self.w("patch_embed.norm.bias"))
        for stage, depth in enumerate(m.depths):
            resi = x
            for blk in range(depth):
                x = self.hab(x, stage, blk)
            x = self.ocab(x, stage)
            x = conv3x3(x, self.w(f"layers.{stage}.conv.weight"),
                        self.w(f"layers.{stage}.conv.bias")) + resi
        x = layer_norm(x, self.w("norm.weight"), self.w("norm.bias"))
        x = conv3x3(x, self.w("conv_after_body.weight"), self.w("conv_after_body.bias")) + body
        h = conv3x3(x, self.w("conv_before_upsample.0.weight"),
                    self.w("conv_before_upsample.0.bias"))
        h = np.where(h > 0, h, h * np.float32(LEAKY)).astype(np.float32)
        for i, (r, _wd) in enumerate(m.up_blocks()):
            h = conv3x3(h, self.w(f"upsample.{2 * i}.weight"), self.w(f"upsample.{2 * i}.bias"))
            hh, ww, cr = h.shape
            # PixelShuffle: channel `c*r*r + i*r + j` → (c, r*y + i, r*x + j)
            # (src/cpu.rs:1285-1301).
            h = h.reshape(hh, ww, cr // (r * r), r, r).transpose(0, 3, 1, 4, 2) \
                .reshape(hh * r, ww * r, cr // (r * r))
        return conv3x3(h, self.w("conv_last.weight"), self.w("conv_last.bias"))


def pre(m: Model, img: np.ndarray, win: int):
    """Pad to the next window multiple by EDGE REPLICATION and apply
    `(x - mean) * img_range` (src/backend.rs:71-89). `img` is planar `[3][h][w]`."""
    _, h, w = img.shape
    hp, wp = -(-h // win) * win, -(-w // win) * win
    x = np.pad(img, ((0, 0), (0, hp - h), (0, wp - w)), mode="edge")
    x = (x - m.mean[:, None, None]) * np.float32(m.img_range)
    return np.ascontiguousarray(x.transpose(1, 2, 0), dtype=np.float32), hp, wp


def finish(m: Model, out: np.ndarray, h: int, w: int):
    """Crop to `h*s x w*s` and denormalise (src/backend.rs:94-109): planar output."""
    s = m.scale
    y = out[:h * s, :w * s, :].transpose(2, 0, 1)
    return np.ascontiguousarray(y / np.float32(m.img_range) + m.mean[:, None, None],
                                dtype=np.float32)


def forward(m: Model, img: np.ndarray) -> np.ndarray:
    """`Backend::forward` (src/backend.rs:29-36): planar `[3][h][w]` in [0, 1] →
    planar `[3][h*s][w*s]`."""
    _, h, w = img.shape
    x0, hp, wp = pre(m, img.astype(np.float32), m.win)
    return finish(m, Forward(m, hp, wp).run(x0), h, w)
