"""The torch operator registrations (w4a16/ops.py): on CPU, the operators exist and their
fake implementations give shapes and dtypes; on the GPU, each operator equals the Python op
it wraps, bit for bit."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import w4a16 as K  # noqa: F401  (registers the operators)


def test_operators_registered_with_fake_shapes():
    ops = torch.ops.w4a16
    for name in ("gemv", "gemv_rmsnorm", "gemv_swiglu", "dequant"):
        assert hasattr(ops, name)
    with FakeTensorMode():
        packed = torch.empty(300, 1024, dtype=torch.uint8)
        scale = torch.empty(300, 16)
        y = ops.gemv(packed, scale, torch.empty(2048, dtype=torch.float16), 128)
        assert y.shape == (300,) and y.dtype == torch.float32
        y = ops.gemv(packed, scale, torch.empty(5, 2048, dtype=torch.float16), 128)
        assert y.shape == (5, 300)
        y = ops.gemv_rmsnorm(packed, scale, torch.empty(2048), torch.empty(2048), 1e-5, 128)
        assert y.shape == (300,) and y.dtype == torch.float32
        y = ops.gemv_swiglu(packed, scale, torch.empty(4096, dtype=torch.float16), 128)
        assert y.shape == (300,)
        w = ops.dequant(packed, scale, 128)
        assert w.shape == (300, 2048) and w.dtype == torch.float16


@pytest.mark.gpu
def test_operators_match_python_ops():
    torch.manual_seed(0)
    w = torch.randn(1000, 2048, device="cuda") * 0.02
    packed, scale = K.quantize_pack(w, group=128)
    x = torch.randn(2048, device="cuda").half()
    assert torch.equal(torch.ops.w4a16.gemv(packed, scale, x, 128), K.gemv(packed, scale, x, group=128))
    h, gamma = torch.randn(2048, device="cuda"), torch.rand(2048, device="cuda")
    assert torch.equal(torch.ops.w4a16.gemv_rmsnorm(packed, scale, h, gamma, 1e-5, 128),
                       K.gemv_rmsnorm(packed, scale, h, gamma, 1e-5, group=128))
    gu = torch.randn(4096, device="cuda").half()
    assert torch.equal(torch.ops.w4a16.gemv_swiglu(packed, scale, gu, 128),
                       K.gemv_swiglu(packed, scale, gu, group=128))
    assert torch.equal(torch.ops.w4a16.dequant(packed, scale, 128), K.dequant_int4(packed, scale, group=128))
