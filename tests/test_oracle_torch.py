"""The torch fp32 twin of the oracle (oracle/hat_torch.py) pinned on the CPU.

The GPU tests and the benchmark's error report use the twin as the fp32 reference at
sizes the numpy oracle cannot reach in seconds, so it is held here to the same bar as
the numpy oracle: every golden fixture made by the reference's own `tools/hat_arch.py`,
and the numpy oracle itself on a ragged multi-window image of each variant.
"""
import numpy as np
import pytest

from golden_io import GOLDEN, cases, checkpoint_for, read_hatf
from oracle import hat_oracle as O
from oracle import hat_torch as T


@pytest.fixture(scope="module")
def ckdir(tmp_path_factory):
    return tmp_path_factory.mktemp("ckt")


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_torch_twin_matches_reference_fixture(case, ckdir):
    fx = read_hatf(GOLDEN / f"{case['name']}.bin")
    got = T.forward(T.Weights.load(checkpoint_for(case, ckdir)), fx["input"])
    assert got.shape == fx["expected"].shape
    assert float(np.abs(got - fx["expected"]).max()) < 2e-6


@pytest.mark.parametrize("variant,scale,h,w", [("hat-s", 3, 37, 50), ("hat-l", 4, 40, 33), ("hat", 2, 33, 40)])
def test_torch_twin_matches_numpy_oracle(variant, scale, h, w, ckdir):
    """Several window rows and columns, a ragged edge, real OCAB neighbours."""
    from hat_b200 import checkpoint, synth
    p = str(ckdir / f"{variant}_{scale}.safetensors")
    checkpoint.make_checkpoint(p, variant, scale, 41, perturb=True)
    img = synth.image(h, w, 4242)
    want = O.forward(O.Model.load(p), img)
    got = T.forward(T.Weights.load(p), img)
    assert float(np.abs(got - want).max()) < 2e-6


def test_strict_fp32_restores_flags():
    import torch
    before = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    with T.strict_fp32():
        assert not torch.backends.cuda.matmul.allow_tf32 and not torch.backends.cudnn.allow_tf32
    assert (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32) == before
