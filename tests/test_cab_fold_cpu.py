"""The identities behind the CAB fold (k_ca_gate, k_cab_rowstat / k_cab_pool, k_proj_cab in
hat-rs_b200/csrc), restated in numpy and checked against the oracle's own 3x3 conv
(oracle/hat_oracle.py, src/cpu.rs:304-422) on the CPU.

* The pool: the sum over a block of output rows of conv3x3(x) equals
  P * b + sum_{tap, ci} w[n][ci][tap] * T[tap][ci], with T taken from the per-row channel
  sums and first / last pixels of x, the row range shifted by one for dy = -1 / +1, exactly
  as k_cab_pool combines them; for the whole plane and for strip views (rows outside the
  view are the conv's zero padding, the output rows a sub-range of the view).
* The fold: proj(attn) + conv_scale * gate * conv3x3(cmid) equals one GEMM over the
  concatenated K (attention channels, then tap-major cmid channels) with the folded weight
  W'[n][tap * cinp + ci] = conv_scale * gate[n] * w[n][ci][tap] and bias bp + conv_scale *
  gate * b2, as k_ca_gate writes them and k_proj_cab accumulates them.
* The tiling: k_proj_cab's 8x16 patches, its K loop (the attention output's 64-byte k-blocks,
  then (tap, chunk) of the middle plane's view with zero fill outside it) and the folded
  weight's K layout, on one GPU's plane and on strip views, reproduce proj + gated conv +
  residual on the output rows and leave the other rows alone.
"""
import numpy as np
import pytest

from oracle import hat_oracle as O


def _pool(x, w, b, y0, y1):
    """k_cab_rowstat + k_cab_pool: x [R][W][cc] (the view), output rows [y0, y1)."""
    R, W, cc = x.shape
    r_lo, r_hi = max(0, y0 - 1), min(R, y1 + 1)
    stat = {r: np.concatenate([x[r].sum(0, dtype=np.float64), x[r, 0], x[r, W - 1]]) for r in range(r_lo, r_hi)}
    row = lambda r: stat[r] if r_lo <= r < r_hi else np.zeros(3 * cc)
    S = sum((stat[r] for r in range(y0, y1)), np.zeros(3 * cc))
    T = np.zeros((9, cc))
    for tap in range(9):
        dy, dx = tap // 3 - 1, tap % 3 - 1
        v = S.copy()
        if dy < 0:
            v = v - row(y1 - 1) + row(y0 - 1)
        if dy > 0:
            v = v - row(y0) + row(y1)
        a, first, last = v[:cc], v[cc:2 * cc], v[2 * cc:]
        T[tap] = a - (last if dx < 0 else 0) - (first if dx > 0 else 0)
    wt = w.reshape(w.shape[0], cc, 9).astype(np.float64)  # [n][ci][tap]
    return (y1 - y0) * W * b.astype(np.float64) + np.einsum("nct,tc->n", wt, T)


@pytest.mark.parametrize("R,W,cc,c,y0,y1", [
    (16, 32, 6, 12, 0, 16),   # the whole plane (one GPU)
    (24, 16, 6, 8, 8, 16),    # a middle strip: the view's halo rows on both sides
    (16, 16, 5, 4, 0, 8),     # a strip at the top edge (the view starts at the image)
    (16, 16, 5, 4, 8, 16),    # a strip at the bottom edge
    (9, 7, 3, 3, 4, 5),       # one output row
])
def test_pool_from_row_sums_equals_conv_sums(R, W, cc, c, y0, y1):
    rng = np.random.default_rng(R * 100 + y0)
    x = rng.standard_normal((R, W, cc)).astype(np.float32)
    w = rng.standard_normal((c, cc, 3, 3)).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    want = O.conv3x3(x.astype(np.float64), w.astype(np.float64), b.astype(np.float64))[y0:y1].sum((0, 1))
    got = _pool(x, w, b, y0, y1)
    # the oracle's conv accumulates in fp32 (as the reference's CPU backend does)
    assert np.abs(got - want).max() <= 2e-6 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("cc,cinp", [(6, 16), (60, 64)])
def test_fold_is_one_gemm_over_concatenated_k(cc, cinp):
    rng = np.random.default_rng(cc)
    H, W, c, cs = 8, 16, 24, 0.01
    attn = rng.standard_normal((H, W, c))
    cmid = rng.standard_normal((H, W, cc))
    wp, bp = rng.standard_normal((c, c)), rng.standard_normal(c)
    w2, b2 = rng.standard_normal((c, cc, 3, 3)), rng.standard_normal(c)
    gate = rng.random(c)
    want = O.linear(attn, wp, bp) + cs * gate * O.conv3x3(cmid, w2, b2)
    # k_ca_gate: the folded weight in the conv's tensor-core K layout, and the folded bias
    wf = np.zeros((c, 9 * cinp))
    for tap in range(9):
        wf[:, tap * cinp:tap * cinp + cc] = cs * gate[:, None] * w2[:, :, tap // 3, tap % 3]
    bias = bp + cs * gate * b2
    # k_proj_cab: A = [attention channels | the nine shifted cmid views, tap-major, padded to cinp]
    pad = np.pad(cmid, ((1, 1), (1, 1), (0, cinp - cc)))
    taps = [pad[t // 3:t // 3 + H, t % 3:t % 3 + W] for t in range(9)]
    a = np.concatenate([attn] + taps, axis=-1)
    got = a @ np.concatenate([wp, wf], axis=1).T + bias
    assert np.abs(got - want).max() <= 2e-6 * max(1.0, np.abs(want).max())


def _box(plane, c0, x0, y0, inner):
    """A 3-D TMA box {inner channels, 16 pixels, 8 rows} at (c0, x0, y0) of a [R][W][C] plane,
    zero outside the plane (the hardware's fill), as the [128][inner] rows k_proj_cab reads."""
    R, W, C = plane.shape
    out = np.zeros((8, 16, inner))
    ys, xs = np.arange(y0, y0 + 8), np.arange(x0, x0 + 16)
    yv, xv = (ys >= 0) & (ys < R), (xs >= 0) & (xs < W)
    cs = np.arange(c0, c0 + inner)
    cv = cs < C
    sub = plane[np.ix_(ys[yv], xs[xv], cs[cv])]
    out[np.ix_(np.where(yv)[0], np.where(xv)[0], np.where(cv)[0])] = sub
    return out.reshape(128, inner)


@pytest.mark.parametrize("rows,W,c,cc,cin_plane,es,vlo,vhi,ylo,yhi", [
    (16, 32, 20, 6, 16, 2, 0, 16, 0, 16),    # one GPU, fp16 pairs (HAT-S's middle plane: 16 channels)
    (32, 16, 20, 6, 16, 2, 8, 32, 8, 24),    # a strip at the top edge: the view starts at row 8
    (32, 16, 12, 60, 60, 4, 0, 24, 8, 24),   # bottom edge, tf32 (HAT: cc = 60): the chunk is half a 128-byte row
])
def test_proj_cab_tiling_against_direct(rows, W, c, cc, cin_plane, es, vlo, vhi, ylo, yhi):
    """k_proj_cab's patch / K-loop arithmetic (umma_proj_cab's geometry, the producer's box
    coordinates, the folded weight's K layout) reproduces proj + gated conv + residual on the
    output rows [ylo, yhi) and writes no other row."""
    rng = np.random.default_rng(rows + cc)
    attn, res = rng.standard_normal((rows, W, c)), rng.standard_normal((rows, W, c))
    cm = rng.standard_normal((rows, W, cin_plane))
    cm[:, :, cc:] = 0  # channels past cc are written as zeros
    wp, bp = rng.standard_normal((c, c)), rng.standard_normal(c)
    w2, b2 = rng.standard_normal((c, cc, 3, 3)), rng.standard_normal(c)
    gate, cs = rng.random(c), 0.01
    # plan_gemm_w's conv layout and the launcher's chunking (64-byte rows at most)
    ckb = (128 if cin_plane >= 64 else 32) if es == 2 else (32 if cc <= 8 else 128)
    chunk = ckb // es
    cinp = -(-cc // chunk) * chunk
    kel, kstep, cke = 64 // es, 32 // es, min(ckb, 64) // es
    assert cinp == -(-cc // cke) * cke  # umma_proj_cab_ok
    kba, cchunks = -(-c // kel), -(-cc // cke)
    wf = np.zeros((c, 9 * cinp))  # k_ca_gate's folded weight
    for tap in range(9):
        wf[:, tap * cinp:tap * cinp + cc] = cs * gate[:, None] * w2[:, :, tap // 3, tap % 3]
    bias = bp + cs * gate * b2
    view = cm[vlo:vhi]
    out = np.full((rows, W, c), np.nan)
    tx = W // 16
    for mt in range((yhi - ylo) // 8 * tx):
        py, px = ylo // 8 + mt // tx, mt % tx
        acc = np.zeros((128, c))
        for kb in range(kba):  # the attention output at the patch, kel channels a k-block
            a = _box(attn, kb * kel, px * 16, py * 8, kel)
            b = np.zeros((c, kel))
            n = min(kel, c - kb * kel)
            b[:, :n] = wp[:, kb * kel:kb * kel + n]
            acc += a @ b.T
        for kb2 in range(9 * cchunks):  # (tap, chunk) of the middle plane's view
            tap, ch = divmod(kb2, cchunks)
            a = _box(view, ch * cke, px * 16 + tap % 3 - 1, py * 8 + tap // 3 - 1 - vlo, cke)
            acc += a @ wf[:, kb2 * cke:(kb2 + 1) * cke].T
        for r in range(128):
            y, x = py * 8 + r // 16, px * 16 + r % 16
            out[y, x] = res[y, x] + (acc[r] + bias)
    cz = np.zeros_like(cm)
    cz[vlo:vhi] = cm[vlo:vhi]
    conv = O.conv3x3(cz[:, :, :cc], w2, b2)
    want = res + O.linear(attn, wp, bp) + cs * gate * conv
    assert np.abs(out[ylo:yhi] - want[ylo:yhi]).max() <= 2e-5
    assert np.isnan(out[:ylo]).all() and np.isnan(out[yhi:]).all()
