"""The C-ABI library without a GPU: it loads, exports every declared symbol, and its
checkpoint reader validates the way src/weights.rs does."""
import ctypes
import json
import re
import struct
from pathlib import Path

import numpy as np
import pytest

import hat_b200
from hat_b200 import checkpoint

HEADER = Path(__file__).resolve().parent.parent / "include" / "hat_b200.h"


def declared_symbols():
    return sorted(set(re.findall(r"HAT_B200_API\s+[\w\s\*]+?\b(hat_b200_\w+)\s*\(", HEADER.read_text())))


def test_library_exports_every_declared_symbol():
    lib = hat_b200.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    # and the Python binding covers every one of them
    assert set(names) == set(hat_b200.SIGNATURES)


def test_inspect_reads_a_converted_checkpoint(tmp_path):
    p = tmp_path / "s.safetensors"
    checkpoint.make_checkpoint(str(p), "hat-s", 4, 3)
    info = hat_b200.inspect(p)
    assert info["variant"] == "hat-s" and info["scale"] == 4 and info["embed"] == 144
    assert info["n_blocks"] == 36 and info["compressed"] == 6 and info["squeezed"] == 6
    p3 = tmp_path / "l3.safetensors"
    checkpoint.make_checkpoint(str(p3), "hat-l", 3, 3)
    info = hat_b200.inspect(p3)
    assert info["n_stages"] == 12 and info["head_dim"] == 30 and info["scale"] == 3


def _rewrite(src, dst, edit_header=None, drop=None):
    raw = Path(src).read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    head = json.loads(raw[8:8 + n])
    if drop:
        del head[drop]
    if edit_header:
        edit_header(head)
    hj = json.dumps(head).encode()
    hj += b" " * ((-(8 + len(hj))) % 8)
    Path(dst).write_bytes(struct.pack("<Q", len(hj)) + hj + raw[8 + n:])


def test_inspect_rejects_what_the_reference_rejects(tmp_path):
    p = tmp_path / "s.safetensors"
    checkpoint.make_checkpoint(str(p), "hat-s", 4, 3)
    bad = tmp_path / "bad.safetensors"
    # no architecture metadata (src/weights.rs:64-76)
    _rewrite(p, bad, edit_header=lambda h: h.pop("__metadata__"))
    with pytest.raises(hat_b200.HatError, match="__metadata__") as e:
        hat_b200.inspect(bad)
    assert e.value.code == hat_b200.E_IO
    # a missing tensor names the tensor
    _rewrite(p, bad, drop="layers.2.residual_group.blocks.3.norm2.bias")
    with pytest.raises(hat_b200.HatError, match="blocks.3.norm2.bias"):
        hat_b200.inspect(bad)

    # metadata that disagrees with the tensors (hat-s weights labelled embed 180)
    def relabel(h):
        h["__metadata__"]["embed_dim"] = "180"
    _rewrite(p, bad, edit_header=relabel)
    with pytest.raises(hat_b200.HatError, match="expected"):
        hat_b200.inspect(bad)

    # a scale the reference's Upsample does not build
    def scale5(h):
        h["__metadata__"]["scale"] = "5"
    _rewrite(p, bad, edit_header=scale5)
    with pytest.raises(hat_b200.HatError, match="scale 5"):
        hat_b200.inspect(bad)
    with pytest.raises(hat_b200.HatError):
        hat_b200.inspect(tmp_path / "missing.safetensors")


def test_checkpoint_layout_matches_the_reference_tensor_list():
    # 864 tensors for HAT-S (862 f32 + the two int64 index buffers)
    a = checkpoint.arch_of("hat-s", 4)
    t = checkpoint.generate(a, 0)
    assert len(t) == 864
    assert t["relative_position_index_OCA"].dtype == np.int64
    assert t["layers.0.residual_group.overlap_attn.relative_position_bias_table"].shape == (1521, 6)


@pytest.mark.skipif(hat_b200.probe(), reason="a B200 is present")
def test_no_silent_cpu_fallback_without_a_gpu(tmp_path):
    p = tmp_path / "s.safetensors"
    checkpoint.make_checkpoint(str(p), "hat-s", 2, 3)
    with pytest.raises(hat_b200.HatError) as e:
        hat_b200.B200(p)
    assert e.value.code == hat_b200.E_CUDA
