"""W4A16 GEMV for NVIDIA B200 (sm_100a).

Drop-in for the Python surface of the reference package `w4a16`
(src/w4a16/__init__.py:1-13): the same names, arguments and outputs, backed by
hand-written sm_100a kernels behind the C ABI of libw4a16_b200.so.
"""
from .kernels import (
    decode_attention,
    dequant_int4,
    gemm,
    gemv,
    gemv_rmsnorm,
    gemv_staged,
    gemv_swiglu,
    matvec_byte,
    matvec_champ,
    matvec_fp16,
    matvec_h2f32,
    matvec_u32,
    matvec_u32_v4,
    matvec_uint4,
    quantize_pack,
    read_device_error,
    new_workspace,
    reserve_workspace,
    w4a16_gemv,
    w4a16_gemv_g128,
)
from . import ops  # noqa: F401  (registers torch.ops.w4a16.*)
from .checkpoint import load_quantized, save_quantized
from .linear import W4A16Linear, replace_linear_with_w4a16
from .quant import (
    dequant_ref,
    dequant_ref_group,
    pack_int4,
    pack_int4_interleaved,
    quantize_int4_group,
    quantize_int4_symmetric,
    unpack_int4,
)

__all__ = [
    # reference names (src/w4a16/__init__.py:8-13)
    "matvec_byte", "matvec_u32", "matvec_u32_v4", "matvec_champ",
    "matvec_uint4", "matvec_h2f32", "w4a16_gemv", "w4a16_gemv_g128", "matvec_fp16",
    "quantize_int4_symmetric", "quantize_int4_group", "pack_int4", "pack_int4_interleaved",
    "dequant_ref", "dequant_ref_group", "W4A16Linear", "replace_linear_with_w4a16",
    # additions
    "gemv", "gemv_staged", "gemv_rmsnorm", "gemv_swiglu", "decode_attention", "new_workspace",
    "dequant_int4", "gemm", "quantize_pack", "unpack_int4", "reserve_workspace", "save_quantized",
    "load_quantized",
    "read_device_error",
]
