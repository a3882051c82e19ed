"""hat_b200_linear_noalloc (scratch in a fixed device array) against hat_b200_linear.

Collected last (file name) so it also runs after every other GPU test has used the
device; it passes on its own as well. Two calls in a row check that the shared scratch
is fully rewritten by each call.
"""
import pytest

import hat_b200

pytestmark = pytest.mark.gpu
# Same tolerance as the kernel-level linear tests: both entry points run the same kernels.
TOL = {hat_b200.MODE_SIMT: 2e-5, hat_b200.MODE_PARITY: 2e-5, hat_b200.MODE_FAST: 5e-3}


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    return torch


@pytest.mark.parametrize("mode", [hat_b200.MODE_SIMT, hat_b200.MODE_PARITY, hat_b200.MODE_FAST],
                         ids=["simt", "tcgen05_3xtf32", "tcgen05_tf32"])
def test_noalloc_matches_linear_twice(torch_cuda, mode):
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(11)
    shapes = [(1000, 432, 144), (777, 540, 180)]  # the second call reuses the scratch at another size
    for m, n, k in shapes:
        x = torch.randn(m, k, device="cuda", generator=g)
        w = torch.randn(n, k, device="cuda", generator=g) * 0.05
        b = torch.randn(n, device="cuda", generator=g)
        want = torch.empty(m, n, device="cuda")
        got = torch.full((m, n), float("nan"), device="cuda")
        hat_b200.linear(mode, x.data_ptr(), w.data_ptr(), b.data_ptr(), want.data_ptr(), m, n, k)
        hat_b200.linear_noalloc(mode, x.data_ptr(), w.data_ptr(), b.data_ptr(), got.data_ptr(), m, n, k)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert float((got - want).abs().max()) <= TOL[mode]


def test_noalloc_refuses_beyond_scratch(torch_cuda):
    torch = torch_cuda
    m, n, k = 20000, 144, 144  # parity split of x alone is 2*m*k*4 = 23 MB > 8 MiB
    x = torch.zeros(m, k, device="cuda")
    w = torch.zeros(n, k, device="cuda")
    y = torch.zeros(m, n, device="cuda")
    with pytest.raises(hat_b200.HatError) as ei:
        hat_b200.linear_noalloc(hat_b200.MODE_PARITY, x.data_ptr(), w.data_ptr(), 0, y.data_ptr(), m, n, k)
    assert ei.value.code == 1
    assert "limit" in str(ei.value)


def test_noalloc_leaves_free_device_memory_unchanged(torch_cuda):
    """The property the entry point exists for: after a first call (which may load the
    library's device code on this GPU), further calls change neither the device's free
    memory nor torch's allocator."""
    torch = torch_cuda
    m, n, k = 1000, 432, 144
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(m, k, device="cuda", generator=g)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.05
    b = torch.randn(n, device="cuda", generator=g)
    y = torch.empty(m, n, device="cuda")
    hat_b200.linear_noalloc(hat_b200.MODE_PARITY, x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), m, n, k)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_reserved()
    for mode in (hat_b200.MODE_PARITY, hat_b200.MODE_FAST, hat_b200.MODE_SIMT):
        hat_b200.linear_noalloc(mode, x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), m, n, k)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert torch.cuda.memory_reserved() == alloc0
