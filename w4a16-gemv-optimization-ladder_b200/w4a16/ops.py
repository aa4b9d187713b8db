"""The library's products as registered torch operators (namespace `w4a16`).

The reference exposes its kernels only through a pybind11 module (kernels/w4a16_kernels.cu:
189-195), invisible to torch's dispatcher.  Registering them lets torch code call
`torch.ops.w4a16.gemv(...)` and trace models that use them (the fake implementations give
output shapes and dtypes without running anything); the implementations call the C ABI
through w4a16.kernels, on the current stream.

    torch.ops.w4a16.gemv(packed, scale, x, group) -> fp32 [rows] or [batch, rows]
    torch.ops.w4a16.gemv_rmsnorm(packed, scale, h, gamma, eps, group) -> fp32 [rows]
    torch.ops.w4a16.gemv_swiglu(packed, scale, gate_up, group) -> fp32 [rows]
    torch.ops.w4a16.dequant(packed, scale, group) -> fp16 [rows, cols]
"""
import torch

from . import kernels as K


@torch.library.custom_op("w4a16::gemv", mutates_args=())
def gemv(packed: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, group: int) -> torch.Tensor:
    return K.gemv(packed, scale, x, group=group)


@gemv.register_fake
def _(packed, scale, x, group):
    rows = packed.shape[0]
    shape = (rows,) if x.dim() == 1 else (x.shape[0], rows)
    return packed.new_empty(shape, dtype=torch.float32)


@torch.library.custom_op("w4a16::gemv_rmsnorm", mutates_args=())
def gemv_rmsnorm(packed: torch.Tensor, scale: torch.Tensor, h: torch.Tensor, gamma: torch.Tensor,
                 eps: float, group: int) -> torch.Tensor:
    return K.gemv_rmsnorm(packed, scale, h, gamma, eps, group=group)


@gemv_rmsnorm.register_fake
def _(packed, scale, h, gamma, eps, group):
    return packed.new_empty((packed.shape[0],), dtype=torch.float32)


@torch.library.custom_op("w4a16::gemv_swiglu", mutates_args=())
def gemv_swiglu(packed: torch.Tensor, scale: torch.Tensor, gate_up: torch.Tensor, group: int) -> torch.Tensor:
    return K.gemv_swiglu(packed, scale, gate_up, group=group)


@gemv_swiglu.register_fake
def _(packed, scale, gate_up, group):
    return packed.new_empty((packed.shape[0],), dtype=torch.float32)


@torch.library.custom_op("w4a16::dequant", mutates_args=())
def dequant(packed: torch.Tensor, scale: torch.Tensor, group: int) -> torch.Tensor:
    return K.dequant_int4(packed, scale, group=group)


@dequant.register_fake
def _(packed, scale, group):
    return packed.new_empty((packed.shape[0], packed.shape[1] * 2), dtype=torch.float16)
