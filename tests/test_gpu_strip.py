"""Strip sharding on 2+ GPUs (one process per GPU, NCCL halo exchange) against the
reference's own output and against the unsharded pass on one GPU. Skipped with fewer
than two GPUs."""
import numpy as np
import pytest
import torch.multiprocessing as mp

import hat_b200
from golden_io import GOLDEN, cases, checkpoint_for, read_hatf

pytestmark = pytest.mark.gpu


def _n_gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _rank_main(rank, n, ckpt, img, mode, q_id, q_out):
    try:
        import torch
        torch.cuda.set_device(rank)
        be = hat_b200.B200(ckpt, device=rank, mode=mode)
        if rank == 0:
            uid = hat_b200.nccl_unique_id()
            for _ in range(n - 1):
                q_id.put(uid)
        else:
            uid = q_id.get(timeout=120)
        be.attach_strip(rank, n, uid)
        h, w = img.shape[1:]
        out = be.forward(h, w, img)
        r0, r1 = hat_b200.strip_rows(h, n, rank)
        s = be.info["scale"]
        a, b = r0 * s, min(r1 * s, h * s)
        q_out.put((rank, a, b, np.ascontiguousarray(out[:, a:b])))
        be.close()
    except Exception as e:  # reported to the parent instead of leaving it waiting
        q_out.put((rank, repr(e), None, None))


def _strip_forward(ckpt, img, n, mode=hat_b200.MODE_PARITY):
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, n, ckpt, img, mode, q_id, q_out)) for r in range(n)]
    for p in procs:
        p.start()
    try:
        parts = [q_out.get(timeout=600) for _ in range(n)]
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    bad = [pt for pt in parts if pt[2] is None]
    assert not bad, bad
    h, w = img.shape[1:]
    scale = parts[0][3].shape[2] // w
    out = np.full((3, h * scale, w * scale), np.nan, np.float32)
    for _r, a, b, y in parts:
        out[:, a:b] = y
    assert np.isfinite(out).all(), "output rows missing"
    return out


@pytest.mark.skipif(_n_gpus() < 2, reason="needs two GPUs")
def test_strip_two_gpus_matches_reference(tmp_path):
    case = next(c for c in cases() if c["name"] == "hats_x4_48x48_p")
    fx = read_hatf(GOLDEN / "hats_x4_48x48_p.bin")
    out = _strip_forward(checkpoint_for(case, tmp_path), fx["input"], 2)
    err = float(np.abs(out - fx["expected"]).max())
    assert err <= 1e-4, err


@pytest.mark.skipif(_n_gpus() < 2, reason="needs two GPUs")
def test_strip_two_gpus_matches_one_gpu(tmp_path):
    from hat_b200 import checkpoint, synth
    ck = str(tmp_path / "hats.safetensors")
    checkpoint.make_checkpoint(ck, "hat-s", 4, 7, True)
    img = synth.image(200, 136, 4242)
    one = hat_b200.B200(ck, device=0, mode=hat_b200.MODE_PARITY)
    ref = one.forward(200, 136, img)
    one.close()
    out = _strip_forward(ck, img, 2)
    # The same kernels on the same data, except the channel-attention sums, which are
    # added per strip and then across GPUs.
    err = float(np.abs(out - ref).max())
    assert err <= 2e-5, err
