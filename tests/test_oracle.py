"""The CPU oracle pinned against the reference's own outputs (no GPU).

* every committed golden fixture (made by tests/golden/make_golden.py from upstream
  `tools/hat_arch.py`) at the reference's verify tolerance and well below it;
* HAT's own index maps and shift mask (`calculate_rpi_sa`, `calculate_rpi_oca`,
  `calculate_mask`, saved in golden/geometry.npz);
* the reference's shipped scale-3 fixture `tests/data/hats_x3_48x48.bin`, when the
  reference checkout is present (its weights come from torch's seed-5 init, which
  only the reference's own model constructor reproduces).
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

from golden_io import GOLDEN, cases, checkpoint_for, read_hatf
from oracle import hat_oracle as O

# The reference checkout: $HAT_REFERENCE, else a `reference` directory beside this repository.
REFERENCE = Path(os.environ.get("HAT_REFERENCE", Path(__file__).resolve().parents[2] / "reference"))


@pytest.fixture(scope="module")
def ckdir(tmp_path_factory):
    return tmp_path_factory.mktemp("ck")


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_fixture(case, ckdir):
    fx = read_hatf(GOLDEN / f"{case['name']}.bin")
    m = O.Model.load(checkpoint_for(case, ckdir))
    got = O.forward(m, fx["input"])
    assert got.shape == fx["expected"].shape
    err = float(np.abs(got - fx["expected"]).max())
    # The reference's verify tolerance is 1e-4 (src/main.rs:310); the oracle is a
    # float32 restatement of the same graph, so it sits far below that.
    assert err < 2e-6, err


def test_geometry_matches_hat():
    g = np.load(GOLDEN / "geometry.npz")
    assert np.array_equal(O.rpi_sa(16), g["rpi_sa"])
    assert np.array_equal(O.rpi_oca(16, 24), g["rpi_oca"])
    # The known answers the reference's own tests pin (tests/plan.rs:189-205).
    assert list(O.rpi_sa(16).reshape(-1)[:4]) == [480, 479, 478, 477]
    assert list((O.rpi_oca(16, 24) % 1521).reshape(-1)[:4]) == [1241, 1242, 1243, 1244]
    assert (O.rpi_oca(16, 24) < 0).any()
    for key in g.files:
        if not key.startswith("mask_"):
            continue
        h, w = map(int, key[5:].split("x"))
        lab = O.partition(O.mask_labels(h, w, 16, 8)[:, :, None], 16)[..., 0]
        mask = np.where(lab[:, :, None] != lab[:, None, :], -100.0, 0.0)
        assert np.array_equal(mask, g[key]), key


def test_mask_is_not_zero_on_window_multiples():
    # T5: the bands are offset from the window grid, so even a 32x32 plane masks.
    lab = O.mask_labels(32, 32, 16, 8)
    assert len(np.unique(lab)) == 9


@pytest.mark.skipif(not (REFERENCE / "tests/data/hats_x3_48x48.bin").exists(),
                    reason="reference checkout not present")
def test_oracle_matches_shipped_x3_fixture():
    import torch
    sys.path.insert(0, str(REFERENCE / "tools"))
    import timm_shim
    timm_shim.install()
    import make_fixture
    from hat_b200 import checkpoint

    # tests/parity.rs:30-37: weights from `make_fixture.py --config s --scale 3 --seed 5`.
    torch.manual_seed(5)
    model = make_fixture.build("s", 3)
    sd = {k: v.numpy() for k, v in model.state_dict().items()}
    m = O.Model(sd, checkpoint.metadata(checkpoint.arch_of("hat-s", 3), "seed5"))
    fx = read_hatf(REFERENCE / "tests/data/hats_x3_48x48.bin")
    got = O.forward(m, fx["input"])
    assert float(np.abs(got - fx["expected"]).max()) < 2e-6


def test_padding_is_edge_replication():
    # T9: Pre::adjust pads by replicating the last row/column (src/backend.rs:71-89).
    from hat_b200 import checkpoint
    m = O.Model(checkpoint.generate(checkpoint.arch_of("hat-s", 4), 0),
                checkpoint.metadata(checkpoint.arch_of("hat-s", 4), "t"))
    img = np.random.default_rng(0).random((3, 17, 5), dtype=np.float32)
    x0, hp, wp = O.pre(m, img, 16)
    assert (hp, wp) == (32, 16)
    assert np.allclose(x0[31, 15], img[:, 16, 4] - m.mean)
    assert np.allclose(x0[20, 2], img[:, 16, 2] - m.mean)
