"""CPU restatement of the strip-sharded pass (test infrastructure).

The engine's strip mode (hat-rs_b200/csrc/engine.cu: exchange / conv_res / the CAB
all-reduce, and the AttnGeom window placement in k_attn_tc.cu) written again in numpy on
top of the oracle's primitives, one rank per process with the halo exchange and the
channel-sum all-reduce done over torch.distributed (gloo), or one rank per thread over an
in-process exchange (LocalNet). Run on every rank, it returns this rank's output rows; stacked over ranks they must equal the
unsharded oracle forward. That checks the sharding scheme itself (strip bounds, halo
depth and wrap, window origins in strip coordinates, the shift mask in global
coordinates, OCAB zero padding at the image edge only, conv padding at the image edge,
the channel-attention mean over the whole image) without a GPU.
"""
import threading

import numpy as np

from oracle import hat_oracle as O

HALO = 8


class GlooNet:
    """Point-to-point exchange and all-reduce over the default torch.distributed group."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist

    def exchange(self, rank, n, up, down, send_top, send_bot):
        torch, dist = self.torch, self.dist
        st, sb = torch.from_numpy(send_top), torch.from_numpy(send_bot)
        rb, rt = torch.empty_like(st), torch.empty_like(st)
        # Tags keep the two messages between the same pair of ranks apart.
        reqs = [dist.isend(st, up, tag=1), dist.isend(sb, down, tag=2),
                dist.irecv(rb, down, tag=1), dist.irecv(rt, up, tag=2)]
        for r in reqs:
            r.wait()
        return rt.numpy(), rb.numpy()

    def allreduce(self, rank, v):
        t = self.torch.from_numpy(v)
        self.dist.all_reduce(t)
        return t.numpy()


class LocalNet:
    """The same two operations between threads of one process (one thread per rank)."""

    def __init__(self, n):
        self.n = n
        self.bar = threading.Barrier(n)
        self.box = {}

    def exchange(self, rank, n, up, down, send_top, send_bot):
        self.box[(rank, "top")] = send_top
        self.box[(rank, "bot")] = send_bot
        self.bar.wait()
        got_top, got_bot = self.box[(up, "bot")].copy(), self.box[(down, "top")].copy()
        self.bar.wait()
        return got_top, got_bot

    def allreduce(self, rank, v):
        self.box[("sum", rank)] = v
        self.bar.wait()
        total = self.box[("sum", 0)].copy()
        for r in range(1, self.n):
            total += self.box[("sum", r)]
        self.bar.wait()
        return total


def strip_rows(hp, win, rank, n):
    """Plan::make_strip: window rows as equal as possible, the first ny % n ranks one more."""
    ny = hp // win
    base, extra = divmod(ny, n)
    wy0 = rank * base + min(rank, extra)
    wy1 = wy0 + base + (1 if rank < extra else 0)
    return wy0 * win, wy1 * win


class Strip:
    def __init__(self, m, h, w, rank, n, net):
        self.m, self.h, self.w, self.rank, self.n, self.net = m, h, w, rank, n, net
        win = m.win
        self.hp, self.wp = -(-h // win) * win, -(-w // win) * win
        self.r0, self.r1 = strip_rows(self.hp, win, rank, n)
        self.own = self.r1 - self.r0
        self.rows = self.own + 2 * HALO
        self.gy0 = self.r0 - HALO
        self.f = O.Forward(m, self.hp, self.wp)  # for the bias index tables

    def w_(self, name):
        return self.m.t[name]

    # ---------------------------------------------------------------- communication
    def exchange(self, plane, res, nrows):
        """Engine::exchange: own top rows to the rank above, own bottom rows to the rank
        below (wrapping around), halos filled from the neighbours."""
        top, bot = HALO * res, (HALO + self.own) * res
        up, down = (self.rank - 1) % self.n, (self.rank + 1) % self.n
        send_top = np.ascontiguousarray(plane[top:top + nrows])
        send_bot = np.ascontiguousarray(plane[bot - nrows:bot])
        if self.n == 1:
            got_top, got_bot = send_bot, send_top
        else:
            got_top, got_bot = self.net.exchange(self.rank, self.n, up, down, send_top, send_bot)
        plane[bot:bot + nrows] = got_bot
        plane[top - nrows:top] = got_top

    def allreduce(self, v):
        v = np.ascontiguousarray(v, dtype=np.float32)
        return self.net.allreduce(self.rank, v) if self.n > 1 else v

    # ---------------------------------------------------------------- layers
    def view(self, res):
        lo, hi = 0, self.rows * res
        if self.r0 == 0:
            lo = HALO * res
        if self.r1 == self.hp:
            hi = (HALO + self.own) * res
        return lo, hi

    def conv(self, x, name, res):
        """conv_res: the conv over the rows that hold image data (zero padding past the
        image's top / bottom), the whole local plane written (halo rows are scratch)."""
        lo, hi = self.view(res)
        out = np.zeros(x.shape[:2] + (self.w_(name + ".weight").shape[0],), np.float32)
        out[lo:hi] = O.conv3x3(x[lo:hi], self.w_(name + ".weight"), self.w_(name + ".bias"))
        return out

    def cab(self, n, p):
        m = self.m
        y = O.gelu(self.conv(n, f"{p}.cab.0", 1))
        y = self.conv(y, f"{p}.cab.2", 1)
        own = y[HALO:HALO + self.own].reshape(-1, y.shape[-1])
        pooled = self.allreduce(own.sum(0, dtype=np.float32)) / np.float32(self.hp * self.wp)
        s = np.maximum(self.w_(f"{p}.cab.3.attention.1.weight")[:, :, 0, 0] @ pooled
                       + self.w_(f"{p}.cab.3.attention.1.bias"), 0)
        g = self.w_(f"{p}.cab.3.attention.3.weight")[:, :, 0, 0] @ s + self.w_(f"{p}.cab.3.attention.3.bias")
        g = (1.0 / (1.0 + np.exp(-g))).astype(np.float32)
        return (y * g).astype(np.float32)

    def window_attention(self, qkv, p, shifted):
        """AttnGeom in strip mode: unshifted windows at local rows HALO + 16k; shifted
        windows at HALO - 8 + 16k (k <= own/16), columns rolled by 8, the mask labels
        taken in the rolled frame of the whole image."""
        m = self.m
        c, heads, win = m.c, m.heads, m.win
        d = c // heads
        s = win // 2
        if shifted:
            oy, nwy = HALO - s, self.own // win + 1
            plane = np.roll(qkv, -s, axis=1)
        else:
            oy, nwy = HALO, self.own // win
            plane = qkv
        rows = plane[oy:oy + nwy * win]
        t = O.partition(rows, win)
        q = O.split_heads(t[..., :c], heads) * np.float32(d ** -0.5)
        k = O.split_heads(t[..., c:2 * c], heads)
        v = O.split_heads(t[..., 2 * c:], heads)
        tab = self.w_(f"{p}.attn.relative_position_bias_table")
        bias = tab[self.f.idx_sa.reshape(-1)].reshape(win * win, win * win, heads).transpose(2, 0, 1)
        mask = None
        if shifted:
            labels = O.mask_labels(self.hp, self.wp, win, s)  # rolled-frame labels
            yr = (self.r0 - 2 * s + np.arange(nwy * win)) % self.hp
            lab = O.partition(labels[yr][:, :, None], win)[..., 0]
            mask = np.where(lab[:, :, None] != lab[:, None, :], np.float32(O.MASK), np.float32(0))
        a = O.merge_heads(O.softmax_attention(q, k, v, bias, mask))
        out = np.zeros(qkv.shape[:2] + (c,), np.float32)
        out[oy:oy + nwy * win] = O.reverse(a, win, nwy * win, self.wp)
        if shifted:
            out = np.roll(out, s, axis=1)
        return out

    def hab(self, x, stage, blk):
        m = self.m
        p = f"layers.{stage}.residual_group.blocks.{blk}"
        self.exchange(x, 1, HALO)
        n = O.layer_norm(x, self.w_(f"{p}.norm1.weight"), self.w_(f"{p}.norm1.bias"))
        conv_x = self.cab(n, f"{p}.conv_block")
        qkv = O.linear(n, self.w_(f"{p}.attn.qkv.weight"), self.w_(f"{p}.attn.qkv.bias"))
        a = self.window_attention(qkv, p, blk % 2 == 1)
        a = O.linear(a, self.w_(f"{p}.attn.proj.weight"), self.w_(f"{p}.attn.proj.bias"))
        x = (x + a) + conv_x * np.float32(m.conv_scale)
        return self.mlp(x, p)

    def mlp(self, x, p):
        n = O.layer_norm(x, self.w_(f"{p}.norm2.weight"), self.w_(f"{p}.norm2.bias"))
        hdn = O.gelu(O.linear(n, self.w_(f"{p}.mlp.fc1.weight"), self.w_(f"{p}.mlp.fc1.bias")))
        return x + O.linear(hdn, self.w_(f"{p}.mlp.fc2.weight"), self.w_(f"{p}.mlp.fc2.bias"))

    def ocab(self, x, stage):
        """Own query windows at local rows HALO + 16k; keys 4 rows / columns further out,
        zero outside the padded image (global rows), as the OCAB's nn.Unfold pads."""
        m = self.m
        p = f"layers.{stage}.residual_group.overlap_attn"
        c, heads, win, owin = m.c, m.heads, m.win, m.owin
        d = c // heads
        pad = (owin - win) // 2
        self.exchange(x, 1, HALO)
        n = O.layer_norm(x, self.w_(f"{p}.norm1.weight"), self.w_(f"{p}.norm1.bias"))
        qkv = O.linear(n, self.w_(f"{p}.qkv.weight"), self.w_(f"{p}.qkv.bias"))
        g = self.gy0 + np.arange(self.rows)
        kvl = np.where(((g >= 0) & (g < self.hp))[:, None, None], qkv[..., c:], np.float32(0))
        kvp = np.pad(kvl, ((0, 0), (pad, pad), (0, 0)))
        nwy, nx = self.own // win, self.wp // win
        q = O.split_heads(O.partition(qkv[HALO:HALO + self.own, :, :c], win), heads) * np.float32(d ** -0.5)
        kv = np.empty((nwy * nx, owin * owin, 2 * c), np.float32)
        for wy in range(nwy):
            y0 = HALO + wy * win - pad
            for wx in range(nx):
                kv[wy * nx + wx] = kvp[y0:y0 + owin, wx * win:wx * win + owin].reshape(owin * owin, 2 * c)
        k = O.split_heads(kv[..., :c], heads)
        v = O.split_heads(kv[..., c:], heads)
        tab = self.w_(f"{p}.relative_position_bias_table")
        bias = tab[self.f.idx_oca.reshape(-1)].reshape(win * win, owin * owin, heads).transpose(2, 0, 1)
        a = np.zeros(x.shape, np.float32)
        a[HALO:HALO + self.own] = O.reverse(O.merge_heads(O.softmax_attention(q, k, v, bias)), win, self.own,
                                             self.wp)
        x = O.linear(a, self.w_(f"{p}.proj.weight"), self.w_(f"{p}.proj.bias")) + x
        return self.mlp(x, p)

    def run(self, img):
        """This rank's output rows [scale*r0, scale*r1) (cropped to the image), planar."""
        m = self.m
        h, w = self.h, self.w
        # k_pre: edge replication at the image, clamped rows for the halo beyond it.
        yy = np.clip(self.gy0 + np.arange(self.rows), 0, h - 1)
        xx = np.minimum(np.arange(self.wp), w - 1)
        x0 = img[:, yy][:, :, xx]
        x0 = ((x0 - m.mean[:, None, None]) * np.float32(m.img_range)).transpose(1, 2, 0)
        x0 = np.ascontiguousarray(x0, dtype=np.float32)
        body = self.conv(x0, "conv_first", 1)
        x = O.layer_norm(body, self.w_("patch_embed.norm.weight"), self.w_("patch_embed.norm.bias"))
        for stage, depth in enumerate(m.depths):
            resi = x
            for blk in range(depth):
                x = self.hab(x, stage, blk)
            x = self.ocab(x, stage)
            self.exchange(x, 1, 1)
            x = self.conv(x, f"layers.{stage}.conv", 1) + resi
        x = O.layer_norm(x, self.w_("norm.weight"), self.w_("norm.bias"))
        self.exchange(x, 1, 1)
        x = self.conv(x, "conv_after_body", 1) + body
        self.exchange(x, 1, 1)
        hd = self.conv(x, "conv_before_upsample.0", 1)
        hd = np.where(hd > 0, hd, hd * np.float32(O.LEAKY)).astype(np.float32)
        res = 1
        for i, (r, _wd) in enumerate(m.up_blocks()):
            self.exchange(hd, res, 1)
            hd = self.conv(hd, f"upsample.{2 * i}", res)
            hh, ww, cr = hd.shape
            hd = hd.reshape(hh, ww, cr // (r * r), r, r).transpose(0, 3, 1, 4, 2).reshape(hh * r, ww * r, cr // (r * r))
            res *= r
        self.exchange(hd, res, 1)
        out = self.conv(hd, "conv_last", res)
        s = m.scale
        a, b = self.r0 * s, min(self.r1 * s, h * s)
        y = out[HALO * s:HALO * s + (b - a), :w * s, :].transpose(2, 0, 1)
        return a, b, np.ascontiguousarray(y / np.float32(m.img_range) + m.mean[:, None, None], dtype=np.float32)
