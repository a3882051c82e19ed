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
