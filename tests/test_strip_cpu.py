"""Strip sharding on the CPU: the sharding scheme of the engine's multi-GPU mode, run as
world_size 2 and 3 gloo process groups (tests/strip_emul.py restates the engine's
strip schedule in numpy), against the reference's own outputs; plus the strip bounds
the library computes (hat_b200_strip_rows, no device needed)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import hat_b200
from golden_io import GOLDEN, cases, checkpoint_for, read_hatf


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, n, port, ckpt, fixture, q):
    import torch.distributed as dist
    from oracle import hat_oracle as O
    from strip_emul import Strip
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=n)
    try:
        from strip_emul import GlooNet
        fx = read_hatf(fixture)
        m = O.Model.load(ckpt)
        a, b, y = Strip(m, fx["h"], fx["w"], rank, n, GlooNet()).run(fx["input"])
        q.put((rank, a, b, y))
    except Exception as e:  # reported to the parent instead of leaving it waiting
        q.put((rank, repr(e), None, None))
    finally:
        dist.destroy_process_group()


def _assemble(fx, parts):
    out = np.full_like(fx["expected"], np.nan)
    for a, b, y in parts:
        out[:, a:b] = y
    assert np.isfinite(out).all(), "some output rows were not produced by any rank"
    # The unsharded oracle sits below 2.4e-7 of the reference; sharding changes only the
    # order of the channel-attention sums.
    err = float(np.abs(out - fx["expected"]).max())
    assert err < 2e-6, err


def test_strip_scheme_gloo_two_ranks(tmp_path):
    """world_size 2 over gloo, one process per rank, a ragged image (37x29 -> 48x32)."""
    name, n = "hats_x4_37x29_p", 2
    case = next(c for c in cases() if c["name"] == name)
    ckpt = checkpoint_for(case, tmp_path)
    fixture = str(GOLDEN / f"{name}.bin")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, n, port, ckpt, fixture, q)) for r in range(n)]
    for p in procs:
        p.start()
    try:
        parts = [q.get(timeout=300) for _ in range(n)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    bad = [pt for pt in parts if pt[2] is None]
    assert not bad, bad
    _assemble(read_hatf(fixture), [pt[1:] for pt in parts])


@pytest.mark.parametrize("name,n", [("hats_x4_48x48_p", 3), ("hats_x3_48x32_p", 2), ("hats_x4_48x48_p", 1)])
def test_strip_scheme_threads(name, n, tmp_path):
    """The same scheme with one thread per rank (middle ranks, x3, and one rank that wraps
    onto itself)."""
    import threading
    from oracle import hat_oracle as O
    from strip_emul import LocalNet, Strip
    case = next(c for c in cases() if c["name"] == name)
    fx = read_hatf(GOLDEN / f"{name}.bin")
    m = O.Model.load(checkpoint_for(case, tmp_path))
    net = LocalNet(n)
    parts, errors = [None] * n, []

    def run(r):
        try:
            parts[r] = Strip(m, fx["h"], fx["w"], r, n, net).run(fx["input"])
        except Exception as e:  # surfaced below
            errors.append(e)
            net.bar.abort()

    ts = [threading.Thread(target=run, args=(r,)) for r in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    assert not errors, errors
    _assemble(fx, parts)


@pytest.mark.parametrize("height,n", [(48, 2), (48, 3), (512, 8), (1024, 8), (1000, 7), (33, 3)])
def test_strip_rows_cover_the_image(height, n):
    hp = -(-height // 16) * 16
    spans = [hat_b200.strip_rows(height, n, r) for r in range(n)]
    assert spans[0][0] == 0 and spans[-1][1] == hp
    for (a0, b0), (a1, b1) in zip(spans, spans[1:]):
        assert b0 == a1
    sizes = [b - a for a, b in spans]
    assert all(s % 16 == 0 and s >= 16 for s in sizes)
    assert max(sizes) - min(sizes) <= 16


def test_strip_rows_refuses_too_many_ranks():
    with pytest.raises(hat_b200.HatError):
        hat_b200.strip_rows(32, 3, 0)  # two window rows for three ranks
