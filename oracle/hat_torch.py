"""fp32 PyTorch twin of the CPU oracle — TEST INFRASTRUCTURE ONLY.

The same forward as `oracle/hat_oracle.py` (upstream `tools/hat_arch.py` evaluated in
the order of the reference's `src/cpu.rs`), written with torch tensor ops so that it
runs on any torch device. On a GPU it is the fp32 reference for the sizes the numpy
oracle cannot reach in seconds (512x512 and up, batches of 333x500): every matmul and
convolution runs in IEEE fp32 with TF32 switched off for the duration of the call.

It is a checker, never the thing measured or shipped: only the tests, `smoke()` and
`bench.py`'s error report call it. Its parity is pinned the same way as the numpy
oracle's: against the committed fixtures made by the reference's own
`tools/hat_arch.py` (`tests/golden/`) and against the numpy oracle itself
(`tests/test_oracle.py`).
"""
from __future__ import annotations

import contextlib

import numpy as np
import torch
import torch.nn.functional as F

from . import hat_oracle as O

EPS = O.EPS
LEAKY = O.LEAKY
MASK = O.MASK


@contextlib.contextmanager
def strict_fp32():
    """IEEE fp32 matmuls and convolutions (no TF32) inside the block."""
    m, c = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    prec = torch.get_float32_matmul_precision()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = m
        torch.backends.cudnn.allow_tf32 = c
        torch.set_float32_matmul_precision(prec)


class Weights:
    """The checkpoint's tensors on `device` (the same safetensors file as the oracle's
    `Model.load`, src/weights.rs:60-129)."""

    def __init__(self, m: O.Model, device):
        self.m = m
        self.t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device)
                  for k, v in m.t.items() if v.dtype == np.float32}
        self.device = device

    @classmethod
    def load(cls, path: str, device="cpu") -> "Weights":
        return cls(O.Model.load(path), device)


def layer_norm(x, g, b):
    """nn.LayerNorm over channels, biased variance, eps 1e-5 (src/cpu.rs:563-581)."""
    return F.layer_norm(x, (x.shape[-1],), g, b, EPS)


def gelu(x):
    """Exact erf GELU (src/cpu.rs:584-603)."""
    return F.gelu(x)


def conv3x3(x, w, b):
    """Conv2d(k=3, s=1, p=1) on a `[H][W][Cin]` plane (src/cpu.rs:304-422)."""
    y = F.conv2d(x.permute(2, 0, 1)[None], w, b, padding=1)
    return y[0].permute(1, 2, 0).contiguous()


def linear(x, w, b):
    """nn.Linear on token rows (src/cpu.rs:456-555)."""
    return F.linear(x, w, b)


def partition(x, win):
    """window_partition (hat_arch.py:95-107): `[H][W][C]` → `[nw][win*win][C]`."""
    h, w, c = x.shape
    return x.reshape(h // win, win, w // win, win, c).permute(0, 2, 1, 3, 4).reshape(-1, win * win, c)


def reverse(x, win, h, w):
    """window_reverse (hat_arch.py:110-125)."""
    c = x.shape[-1]
    return x.reshape(h // win, w // win, win, win, c).permute(0, 2, 1, 3, 4).reshape(h, w, c)


def split_heads(x, heads):
    nw, n, c = x.shape
    return x.reshape(nw, n, heads, c // heads).permute(0, 2, 1, 3)


def merge_heads(x):
    nw, h, n, d = x.shape
    return x.permute(0, 2, 1, 3).reshape(nw, n, h * d)


def softmax_attention(q, k, v, bias, mask=None, chunk=256):
    """`softmax(q @ k^T + bias (+ mask)) @ v` with q already scaled
    (hat_arch.py:165-196, 392-438; src/cpu.rs:772-844), in chunks of windows."""
    out = torch.empty_like(q)
    for s in range(0, q.shape[0], chunk):
        e = slice(s, s + chunk)
        a = q[e] @ k[e].transpose(-1, -2) + bias[None]
        if mask is not None:
            a = a + mask[e][:, None]
        out[e] = torch.softmax(a, -1) @ v[e]
    return out


class Forward:
    """One forward pass over a padded plane (src/cpu.rs:1318-1368), as the numpy
    oracle's `Forward`."""

    def __init__(self, wt: Weights, hp: int, wp: int):
        m = wt.m
        self.wt, self.m, self.hp, self.wp = wt, m, hp, wp
        win, owin = m.win, m.owin
        dev = wt.device
        self.shift = win // 2
        self.idx_sa = torch.from_numpy(O.rpi_sa(win) % ((2 * win - 1) ** 2)).to(dev)
        self.idx_oca = torch.from_numpy(O.rpi_oca(win, owin) % ((win + owin - 1) ** 2)).to(dev)
        lab = O.partition(O.mask_labels(hp, wp, win, self.shift)[:, :, None], win)[..., 0]
        lab = torch.from_numpy(lab.astype(np.int64)).to(dev)
        self.mask = torch.where(lab[:, :, None] != lab[:, None, :], torch.tensor(MASK, device=dev),
                                torch.tensor(0.0, device=dev)).float()

    def w(self, name):
        return self.wt.t[name]

    def cab(self, x, p):
        """conv → GELU → conv → channel attention, no residual (hat_arch.py:40-74)."""
        y = gelu(conv3x3(x, self.w(f"{p}.cab.0.weight"), self.w(f"{p}.cab.0.bias")))
        y = conv3x3(y, self.w(f"{p}.cab.2.weight"), self.w(f"{p}.cab.2.bias"))
        pooled = y.reshape(-1, y.shape[-1]).mean(0)
        s = self.w(f"{p}.cab.3.attention.1.weight")[:, :, 0, 0] @ pooled + self.w(f"{p}.cab.3.attention.1.bias")
        s = torch.relu(s)
        g = self.w(f"{p}.cab.3.attention.3.weight")[:, :, 0, 0] @ s + self.w(f"{p}.cab.3.attention.3.bias")
        return y * torch.sigmoid(g)

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
        xs = torch.roll(n, (-s, -s), dims=(0, 1)) if s else n
        qkv = linear(partition(xs, win), self.w(f"{p}.attn.qkv.weight"), self.w(f"{p}.attn.qkv.bias"))
        q = split_heads(qkv[..., :c], heads) * np.float32(d ** -0.5)
        k = split_heads(qkv[..., c:2 * c], heads)
        v = split_heads(qkv[..., 2 * c:], heads)
        tab = self.w(f"{p}.attn.relative_position_bias_table")
        bias = tab[self.idx_sa.reshape(-1)].reshape(win * win, win * win, heads).permute(2, 0, 1)
        a = merge_heads(softmax_attention(q, k, v, bias, self.mask if s else None))
        a = linear(a, self.w(f"{p}.attn.proj.weight"), self.w(f"{p}.attn.proj.bias"))
        a = reverse(a, win, self.hp, self.wp)
        if s:
            a = torch.roll(a, (s, s), dims=(0, 1))
        # `shortcut + attn_x + conv_x * conv_scale`, in that order (hat_arch.py:305).
        x = (x + a) + conv_x * np.float32(m.conv_scale)
        return self.mlp(x, p)

    def ocab(self, x, stage):
        """OCAB.forward (hat_arch.py:392-438): 16x16 queries against the 24x24
        `nn.Unfold(stride 16, padding 4)` of k and v, zero outside the plane."""
        m = self.m
        p = f"layers.{stage}.residual_group.overlap_attn"
        c, heads, win, owin = m.c, m.heads, m.win, m.owin
        d = c // heads
        pad = (owin - win) // 2
        n = layer_norm(x, self.w(f"{p}.norm1.weight"), self.w(f"{p}.norm1.bias"))
        qkv = linear(n, self.w(f"{p}.qkv.weight"), self.w(f"{p}.qkv.bias"))
        q = split_heads(partition(qkv[..., :c], win), heads) * np.float32(d ** -0.5)
        kvp = F.pad(qkv[..., c:], (0, 0, pad, pad, pad, pad))
        # [ny][nx][owin][owin][2c] by two strided unfolds of the padded plane
        kv = kvp.unfold(0, owin, win).unfold(1, owin, win)  # [ny][nx][2c][owin][owin]
        kv = kv.permute(0, 1, 3, 4, 2).reshape(-1, owin * owin, 2 * c)
        k = split_heads(kv[..., :c], heads)
        v = split_heads(kv[..., c:], heads)
        tab = self.w(f"{p}.relative_position_bias_table")
        bias = tab[self.idx_oca.reshape(-1)].reshape(win * win, owin * owin, heads).permute(2, 0, 1)
        a = merge_heads(softmax_attention(q, k, v, bias, chunk=128))
        a = reverse(a, win, self.hp, self.wp)
        x = linear(a, self.w(f"{p}.proj.weight"), self.w(f"{p}.proj.bias")) + x
        return self.mlp(x, p)

    def run(self, x0):
        """Padded, mean-adjusted `[hp][wp][3]` → padded `[hp*s][wp*s][3]` in network
        units (hat_arch.py:971-984)."""
        m = self.m
        body = conv3x3(x0, self.w("conv_first.weight"), self.w("conv_first.bias"))
        x = layer_norm(body, self.w("patch_embed.norm.weight"), self.w("patch_embed.norm.bias"))
        for stage, depth in enumerate(m.depths):
            resi = x
            for blk in range(depth):
                x = self.hab(x, stage, blk)
            x = self.ocab(x, stage)
            x = conv3x3(x, self.w(f"layers.{stage}.conv.weight"), self.w(f"layers.{stage}.conv.bias")) + resi
        x = layer_norm(x, self.w("norm.weight"), self.w("norm.bias"))
        x = conv3x3(x, self.w("conv_after_body.weight"), self.w("conv_after_body.bias")) + body
        h = conv3x3(x, self.w("conv_before_upsample.0.weight"), self.w("conv_before_upsample.0.bias"))
        h = F.leaky_relu(h, LEAKY)
        for i, (r, _wd) in enumerate(m.up_blocks()):
            h = conv3x3(h, self.w(f"upsample.{2 * i}.weight"), self.w(f"upsample.{2 * i}.bias"))
            hh, ww, cr = h.shape
            # PixelShuffle: channel `c*r*r + i*r + j` → (c, r*y + i, r*x + j) (src/cpu.rs:1285-1301)
            h = h.reshape(hh, ww, cr // (r * r), r, r).permute(0, 3, 1, 4, 2).reshape(hh * r, ww * r, cr // (r * r))
        return conv3x3(h, self.w("conv_last.weight"), self.w("conv_last.bias"))


def forward(wt: Weights, img) -> np.ndarray:
    """`Backend::forward` (src/backend.rs:29-36): planar `[3][h][w]` in [0, 1] (numpy
    or torch) → planar `[3][h*s][w*s]` float32 numpy, edge-replicated padding to a
    window multiple and the crop + denormalisation after (src/backend.rs:71-109)."""
    m = wt.m
    x = torch.as_tensor(np.asarray(img, np.float32)).to(wt.device)
    _, h, w = x.shape
    win = m.win
    hp, wp = -(-h // win) * win, -(-w // win) * win
    with torch.no_grad(), strict_fp32():
        xp = F.pad(x[None], (0, wp - w, 0, hp - h), mode="replicate")[0]
        mean = torch.from_numpy(m.mean).to(wt.device)
        x0 = ((xp - mean[:, None, None]) * np.float32(m.img_range)).permute(1, 2, 0).contiguous()
        y = Forward(wt, hp, wp).run(x0)
        s = m.scale
        y = y[:h * s, :w * s, :].permute(2, 0, 1) / np.float32(m.img_range) + mean[:, None, None]
        return y.contiguous().float().cpu().numpy()
