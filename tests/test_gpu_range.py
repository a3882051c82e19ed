"""Parity-mode operands beyond fp16's range, on a B200.

HAT-S runs its parity mode on fp16 hi/lo operand pairs, which carry fp32's 22
significant bits but not its exponent range: an operand of 65504 or more does not
fit. The reference computes such inputs in fp32 and answers them, so the backend must
too. These checkpoints are the seeded HAT-S weights with one layer's output scaled by a
power of two (2^14 for LayerNorm's, 2^20 for v) and the consuming weights by its
inverse: exact in fp32, so the network computes the same function while an operand
plane goes past 65504. The pass must match the oracle at the reference's 1e-4 and leave
the handle on tf32 pairs.
"""
import numpy as np
import pytest

import hat_b200
from hat_b200 import checkpoint, synth
from oracle import hat_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-4
BIG = np.float32(2.0 ** 14)
HUGE = np.float32(2.0 ** 20)


def scaled_checkpoint(path, kind):
    a = checkpoint.arch_of("hat-s", 4)
    t = checkpoint.generate(a, 61, perturb=True)
    b = "layers.0.residual_group.blocks.1"
    if kind == "norm":
        # LN1's output (the qkv linear's and the CAB conv's operand) times 2^14.
        t[f"{b}.norm1.weight"] = t[f"{b}.norm1.weight"] * BIG
        t[f"{b}.norm1.bias"] = t[f"{b}.norm1.bias"] * BIG
        t[f"{b}.attn.qkv.weight"] = t[f"{b}.attn.qkv.weight"] / BIG
        t[f"{b}.conv_block.cab.0.weight"] = t[f"{b}.conv_block.cab.0.weight"] / BIG
    else:
        # v (an attention operand, |v| up to about 1 here) times 2^20, proj's weight times 2^-20.
        c = a.embed
        t[f"{b}.attn.qkv.weight"][2 * c:] *= HUGE
        t[f"{b}.attn.qkv.bias"][2 * c:] *= HUGE
        t[f"{b}.attn.proj.weight"] = t[f"{b}.attn.proj.weight"] / HUGE
    checkpoint.write_safetensors(path, t, checkpoint.metadata(a, f"range-{kind}"))
    return path


@pytest.mark.parametrize("kind", ["norm", "value"])
def test_operand_beyond_fp16_range_falls_back_to_tf32_pairs(tmp_path, kind):
    p = scaled_checkpoint(str(tmp_path / f"{kind}.safetensors"), kind)
    img = synth.image(48, 48, 6100)
    want = O.forward(O.Model.load(p), img)
    be = hat_b200.B200(p)
    assert be.fp16_pairs()
    got = be.forward(48, 48, img)
    assert not be.fp16_pairs(), "the pass should have moved to tf32 operand pairs"
    err = float(np.abs(got - want).max())
    print(f"{kind}: max {err:.3e} after the fallback")
    assert err <= TOL
    # The handle stays on tf32 pairs: the next call needs no retry and agrees.
    assert np.array_equal(be.forward(48, 48, img), got)
    be.close()


def test_device_entry_reports_range_error_on_sync(tmp_path):
    """forward_device does not retry; the condition surfaces at sync() as ECUDA."""
    import torch
    p = scaled_checkpoint(str(tmp_path / "dev.safetensors"), "norm")
    img = synth.image(32, 32, 6200)
    be = hat_b200.B200(p, use_graph=False)
    x = torch.from_numpy(img).cuda()
    y = torch.empty((3, 128, 128), device="cuda")
    be.forward_device(x.data_ptr(), y.data_ptr(), 1, 32, 32)
    with pytest.raises(hat_b200.HatError, match="fp16's range") as e:
        be.sync()
    assert e.value.code == hat_b200.E_CUDA
    be.sync()  # the error word was cleared
    be.close()


def test_unscaled_weights_stay_on_fp16_pairs(tmp_path):
    p = str(tmp_path / "plain.safetensors")
    checkpoint.make_checkpoint(p, "hat-s", 4, 61, perturb=True)
    img = synth.image(48, 48, 6100)
    be = hat_b200.B200(p)
    got = be.forward(48, 48, img)
    assert be.fp16_pairs()
    assert float(np.abs(got - O.forward(O.Model.load(p), img)).max()) <= TOL
    be.close()
