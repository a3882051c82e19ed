"""One handle over several GPUs (hat_b200_opts.ngpus), and a strip rank that stops
calling. Skipped with fewer than two GPUs.

* BATCH: the call's images divided among the GPUs; every image equals the one-GPU pass
  bit for bit (the same kernels on the same data).
* STRIP: every image split into row strips over the GPUs with NCCL halo exchange; equal
  to the one-GPU pass up to the order of the channel-attention sums, and within the
  reference's 1e-4 of the fp32 reference (the oracle's torch twin).
* A rank of a strip-sharded job (one process per GPU) that stops calling between steps
  (after two joint steps: the eager pass and the captured one): the other rank's next call
  comes back with an error once its deadline passes instead of blocking. The ranks meet on
  the host before a pass enqueues any exchange, so nothing was launched: the communicator
  stays intact, a repeated call fails the same way, and when the silent rank calls again
  both run the pass and get the same output as before. NCCL's NVLS is off in these
  processes, and the silent rank stays alive.
"""
import os

import numpy as np
import pytest
import torch.multiprocessing as mp

import hat_b200
from hat_b200 import checkpoint, synth

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _n_gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


needs2 = pytest.mark.skipif(_n_gpus() < 2, reason="needs two GPUs")


@pytest.fixture(scope="module")
def ckdir(tmp_path_factory):
    return tmp_path_factory.mktemp("ckmulti")


def _ck(ckdir, variant, scale, seed, perturb=True):
    p = ckdir / f"{variant}_{scale}_{seed}.safetensors"
    if not p.exists():
        checkpoint.make_checkpoint(str(p), variant, scale, seed, perturb)
    return str(p)


@needs2
def test_batch_over_two_gpus_equals_one_gpu(ckdir):
    p = _ck(ckdir, "hat-s", 4, 31)
    imgs = synth.batch(5, 48, 64, 31)
    one = hat_b200.B200(p)
    ref = one.forward_batch(imgs)
    one.close()
    two = hat_b200.B200(p, devices=[0, 1], shard=hat_b200.SHARD_BATCH)
    assert two.gpu_count() == 2
    got = two.forward_batch(imgs)
    assert two.launch_count() > 0
    two.close()
    assert np.array_equal(got, ref)


@needs2
@pytest.mark.parametrize("variant,scale,h,w", [("hat-s", 4, 512, 512), ("hat-l", 4, 96, 80), ("hat-s", 3, 333, 500)])
def test_strip_over_two_gpus_one_handle(ckdir, variant, scale, h, w):
    from oracle import hat_torch as T
    p = _ck(ckdir, variant, scale, 32)
    img = synth.image(h, w, 3200 + h)
    one = hat_b200.B200(p)
    ref = one.forward(h, w, img)
    one.close()
    two = hat_b200.B200(p, devices=[0, 1], shard=hat_b200.SHARD_STRIP, timeout_ms=60000)
    got = two.forward(h, w, img)
    again = two.forward(h, w, img)  # the captured graph's replay
    two.close()
    assert np.array_equal(got, again)
    assert float(np.abs(got - ref).max()) <= 2e-5
    want = T.forward(T.Weights.load(p, "cuda"), img)
    err = float(np.abs(got - want).max())
    print(f"{variant} x{scale} {h}x{w} strip2: max {err:.3e} vs fp32")
    assert err <= TOL


def _silent_rank_main(rank, ckpt, img, q_id, q_out, q_resume, q_done):
    """One rank of a 2-rank strip job; every stage is reported to the parent as it ends."""
    def leave():
        q_out.close()
        q_out.join_thread()  # the queue's feeder thread delivers what was put before the exit
        os._exit(0)

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import faulthandler
    faulthandler.enable()
    try:
        import time
        import torch
        torch.cuda.set_device(rank)
        be = hat_b200.B200(ckpt, device=rank)  # the first call sets up NCCL: default deadline
        if rank == 0:
            uid = hat_b200.nccl_unique_id()
            q_id.put(uid)
        else:
            uid = q_id.get(timeout=120)
        be.attach_strip(rank, 2, uid)
        h, w = img.shape[1:]
        s = be.scale
        r0, r1 = hat_b200.strip_rows(h, 2, rank)
        mine = slice(r0 * s, min(r1, h) * s)  # the output rows this rank writes
        t0 = time.perf_counter()
        be.forward(h, w, img)  # two steps together: the eager pass, then the captured one
        first = be.forward(h, w, img)[:, mine]
        q_out.put((rank, "step", time.perf_counter() - t0))
        be.set_timeout(3000)
        if rank == 1:
            # stops calling: stays alive and issues nothing until rank 0 has had its errors
            q_resume.get(timeout=300)
            faulthandler.dump_traceback_later(30)
            out = be.forward(h, w, img)[:, mine]
            faulthandler.cancel_dump_traceback_later()
            q_out.put((rank, "resumed", bool(np.array_equal(out, first))))
            q_done.get(timeout=300)
            leave()
        for stage in ("error", "again"):
            t = time.perf_counter()
            try:
                be.forward(h, w, img)
                q_out.put((rank, "no error", stage))
                leave()
            except hat_b200.HatError as e:
                q_out.put((rank, stage, (e.code, str(e), time.perf_counter() - t)))
        q_resume.put(1)
        faulthandler.dump_traceback_later(30)
        out = be.forward(h, w, img)[:, mine]
        faulthandler.cancel_dump_traceback_later()
        q_out.put((rank, "resumed", bool(np.array_equal(out, first))))
        leave()
    except Exception as e:
        q_out.put((rank, "exception", repr(e)))


@needs2
def test_strip_rank_that_stops_calling_ends_in_an_error(ckdir):
    p = _ck(ckdir, "hat-s", 4, 33)
    img = synth.image(64, 48, 3300)
    ctx = mp.get_context("spawn")
    q_id, q_out, q_resume, q_done = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_silent_rank_main, args=(r, p, img, q_id, q_out, q_resume, q_done))
             for r in range(2)]
    for pr in procs:
        pr.start()
    got = {}
    try:
        # two "step" reports, rank 0's "error" and "again", then both ranks' "resumed"
        for _ in range(6):
            rank, stage, val = q_out.get(timeout=120)
            got[(rank, stage)] = val
            if stage in ("exception", "no error"):
                break
    finally:
        print("stages:", got)
        q_done.put(1)
        q_resume.put(1)
        for pr in procs:
            pr.join(timeout=60)
            if pr.exitcode is None:
                pr.kill()
        print("exit codes:", [pr.exitcode for pr in procs])
    assert (0, "step") in got and (1, "step") in got, got
    for stage in ("error", "again"):
        code, msg, waited = got[(0, stage)]
        assert code == hat_b200.E_CUDA
        assert "did not start pass" in msg and "intact" in msg, msg
        assert 2.5 <= waited <= 30, waited
    assert got[(0, "resumed")] is True and got[(1, "resumed")] is True, got
