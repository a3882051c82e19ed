"""Parity at every benchmark configuration's own size, on a B200, through the C ABI.

The reference's check is `--verify`: max abs error <= 1e-4 on [0, 1] pixels against the
fp32 output of its own network definition (src/main.rs:310-326). At these sizes the
fp32 reference is the torch twin of the oracle (oracle/hat_torch.py) run on the same
GPU in IEEE fp32 (TF32 off); the twin is pinned to the reference's fixtures and to the
numpy oracle on the CPU (tests/test_oracle_torch.py).

Workloads: synthetic sinusoid + noise images quantised to k/255 and seeded weights in
the reference's checkpoint layout (no dataset or released checkpoint on these
machines), at the shapes of the benchmark configurations:
* HAT-S x4, 512x512 (parity and fast mode);
* HAT x4, 256x256 images (the eight one GPU gets), and a 96x96 one;
* HAT-L x4, 1024x1024 on one GPU, and smaller multi-window planes;
* HAT-S x3, a batch of four 333x500 images (padded to 336x512 by edge
  replication), parity and fast mode, each image also against its own single forward.
"""
import numpy as np
import pytest

import hat_b200
from hat_b200 import checkpoint, synth

pytestmark = pytest.mark.gpu
TOL = 1e-4   # src/main.rs:310 VERIFY_TOL
PSNR_MIN = 50.0  # fast-mode bar


@pytest.fixture(scope="module")
def ckdir(tmp_path_factory):
    return tmp_path_factory.mktemp("ckcfg")


@pytest.fixture(scope="module")
def twin():
    import torch
    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    from oracle import hat_torch as T
    return T


def ck(ckdir, variant, scale, seed, perturb):
    p = ckdir / f"{variant}_x{scale}_{seed}_{int(perturb)}.safetensors"
    if not p.exists():
        checkpoint.make_checkpoint(str(p), variant, scale, seed, perturb)
    return str(p)


def psnr(a, b):
    mse = float(((a.astype(np.float64) - b) ** 2).mean())
    return 10 * np.log10(1.0 / max(mse, 1e-30))


def check(name, got, want):
    err = np.abs(got - want)
    print(f"{name}: max {err.max():.3e} mean {err.mean():.3e}")
    assert got.shape == want.shape
    assert float(err.max()) <= TOL, name


@pytest.mark.parametrize("perturb", [False, True], ids=["bench_weights", "perturbed"])
def test_config1_hats_x4_512(ckdir, twin, perturb):
    p = ck(ckdir, "hat-s", 4, 2024, perturb)
    img = synth.image(512, 512, 2000)
    want = twin.forward(twin.Weights.load(p, "cuda"), img)
    be = hat_b200.B200(p)
    check("hat-s x4 512 parity", be.forward(512, 512, img), want)
    be.close()
    fast = hat_b200.B200(p, mode=hat_b200.MODE_FAST)
    got = fast.forward(512, 512, img)
    print(f"hat-s x4 512 fast: PSNR {psnr(got, want):.1f} dB")
    assert psnr(got, want) >= PSNR_MIN
    fast.close()


@pytest.mark.parametrize("h,w", [(64, 64), (96, 80), (45, 70)])
def test_hatl_x4_multi_window(ckdir, twin, h, w):
    """HAT-L: 12 stages, several window rows, the OCAB's real neighbours, tf32 pairs."""
    p = ck(ckdir, "hat-l", 4, 77, True)
    img = synth.image(h, w, 7700 + h)
    want = twin.forward(twin.Weights.load(p, "cuda"), img)
    be = hat_b200.B200(p)
    check(f"hat-l x4 {h}x{w}", be.forward(h, w, img), want)
    be.close()


def test_hat_x4_96(ckdir, twin):
    p = ck(ckdir, "hat", 4, 78, True)
    img = synth.image(96, 96, 7800)
    want = twin.forward(twin.Weights.load(p, "cuda"), img)
    be = hat_b200.B200(p)
    check("hat x4 96x96", be.forward(96, 96, img), want)
    be.close()


def test_config2_hat_x4_256_batch8(ckdir, twin):
    """configs[2]'s per-GPU share: eight 256x256 images in one call."""
    p = ck(ckdir, "hat", 4, 2024, False)
    imgs = synth.batch(8, 256, 256, 3)
    be = hat_b200.B200(p)
    got = be.forward_batch(imgs)
    be.close()
    wt = twin.Weights.load(p, "cuda")
    for i in range(8):
        check(f"hat x4 256 image {i}", got[i], twin.forward(wt, imgs[i]))


def test_config3_hatl_x4_1024(ckdir, twin):
    """configs[3]'s image on one GPU (the strip-sharded runs are held to this pass)."""
    p = ck(ckdir, "hat-l", 4, 2024, False)
    img = synth.image(1024, 1024, 4000)
    be = hat_b200.B200(p)
    got = be.forward(1024, 1024, img)
    be.close()
    check("hat-l x4 1024", got, twin.forward(twin.Weights.load(p, "cuda"), img))


def test_config4_hats_x3_333x500_batch4(ckdir, twin):
    """HAT-S x3, four 333x500 images, parity and fast mode; every image of
    the batch also equals its own single-image forward."""
    p = ck(ckdir, "hat-s", 3, 2024, False)
    imgs = synth.batch(4, 333, 500, 5)
    wt = twin.Weights.load(p, "cuda")
    wants = [twin.forward(wt, imgs[i]) for i in range(4)]
    be = hat_b200.B200(p)
    got = be.forward_batch(imgs)
    assert got.shape == (4, 3, 999, 1500)
    for i in range(4):
        check(f"hat-s x3 333x500 image {i}", got[i], wants[i])
        assert np.array_equal(got[i], be.forward(333, 500, imgs[i]))
    be.close()
    fast = hat_b200.B200(p, mode=hat_b200.MODE_FAST)
    gotf = fast.forward_batch(imgs)
    fast.close()
    for i in range(4):
        v = psnr(gotf[i], wants[i])
        print(f"hat-s x3 333x500 fast image {i}: PSNR {v:.1f} dB")
        assert v >= PSNR_MIN
