"""nn.Linear drop-in over the W4A16 kernels, and the recursive module swapper.

W4A16Linear keeps the reference's constructor (weight_fp16, bias, packed, scale) and
forward contract (src/w4a16/kernels.py:105-124): x [..., in] -> [..., out] in x's
dtype.  Differences, all opt-in or invisible to callers:
  * batches of up to 64 rows run on the int4 tensor-core kernel (16 rows per pass)
    instead of the dense fp16 fallback the reference used for any batch > 1;
  * bias add and the cast to fp16 happen in the kernel epilogue;
  * scale may be group-128 ([out, in/128]) as well as per-row ([out]);
  * weight_fp16 may be None (no dense copy kept); larger batches then run the int4
    tensor-core GEMM (tcgen05, the dequantised weight formed in shared memory only:
    the same fp16 weight dequant_int4 gives, fp32 sums), or, for shapes it does not
    take (K not a multiple of 64 / 128), dequantise to fp16 on the GPU and call a
    dense GEMM.
"""
import torch
import torch.nn as nn

from . import kernels as K
from .quant import GROUP, pack_int4_interleaved, quantize_int4_group, quantize_int4_symmetric

SMALL_BATCH_MAX = 64


class W4A16Linear(nn.Module):
    def __init__(self, weight_fp16, bias, packed, scale):
        super().__init__()
        if weight_fp16 is not None:
            self.register_buffer("dense_weight", weight_fp16)
        else:
            self.dense_weight = None
        self.register_buffer("packed", packed)  # interleaved packing
        self.register_buffer("scale", scale)
        self.bias = bias
        self.out_features = packed.shape[0]
        self.in_features = packed.shape[1] * 2
        self.group = GROUP if scale.dim() == 2 else 0
        self.register_buffer("bias_f32", None if bias is None else bias.detach().float().contiguous(),
                             persistent=False)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"group={self.group}, dense_copy={self.dense_weight is not None}")

    def forward(self, x):
        lead = x.shape[:-1]
        xf = x.reshape(-1, self.in_features)
        m = xf.shape[0]
        if m <= SMALL_BATCH_MAX:
            xh = xf if xf.dtype == torch.float16 and xf.is_contiguous() else xf.half().contiguous()
            odt = torch.float16 if x.dtype == torch.float16 else torch.float32
            vec = xh[0] if m == 1 else xh
            y = K.gemv(self.packed, self.scale, vec, group=self.group, bias=self.bias_f32,
                       out_dtype=odt)
            return y.to(x.dtype).view(*lead, self.out_features)
        if self.dense_weight is None and self.in_features % (GROUP if self.group else 64) == 0:
            xh = xf if xf.dtype == torch.float16 and xf.is_contiguous() else xf.half().contiguous()
            odt = torch.float16 if x.dtype == torch.float16 else torch.float32
            # fp16 scales widen to fp32 exactly: the same dequantised weight either way
            sc = self.scale if self.scale.dtype == torch.float32 else self.scale.float()
            y = K.gemm(self.packed, sc, xh, group=self.group, bias=self.bias_f32, out_dtype=odt)
            return y.to(x.dtype).view(*lead, self.out_features)
        if self.dense_weight is not None:
            w = self.dense_weight
        else:
            w = K.dequant_int4(self.packed, self.scale, group=self.group)
        y = (xf.to(w.dtype) @ w.t()).float()
        if self.bias_f32 is not None:
            y = y + self.bias_f32
        return y.to(x.dtype).view(*lead, self.out_features)


def replace_linear_with_w4a16(module, group=0, keep_dense=True, scale_dtype=torch.float32,
                              device=None, quantizer="torch"):
    """Swap every nn.Linear under `module` for a W4A16Linear (reference kernels.py:127-137).

    Defaults match the reference: per-row scales, the dense fp16 weight kept for large
    batches, buffers on the GPU.  group=128 uses group-wise scales; keep_dense=False
    drops the dense copy; device places the buffers (default: the weight's CUDA
    device, else the current one).  quantizer="gpu" quantises and packs each weight in
    one kernel launch on the target GPU (bit-identical codes and fp32 scales) instead of
    the reference's torch ops."""
    if quantizer not in ("torch", "gpu"):
        raise ValueError("quantizer must be 'torch' or 'gpu'")
    for name, child in module.named_children():
        if isinstance(child, nn.Linear):
            w = child.weight.data
            if device is not None:
                dev = torch.device(device)
            else:
                dev = w.device if w.is_cuda else torch.device("cuda", torch.cuda.current_device())
            if quantizer == "gpu":
                if dev.type != "cuda":
                    raise ValueError("quantizer='gpu' needs a CUDA device")
                packed, scale = K.quantize_pack(w.to(dev).float().contiguous(), group=group,
                                                scale_dtype=scale_dtype)
            else:
                if group:
                    q, scale = quantize_int4_group(w.float(), group=group)
                else:
                    q, scale = quantize_int4_symmetric(w.float())
                packed = pack_int4_interleaved(q).to(dev)
                scale = scale.to(scale_dtype).to(dev)
            dense = w.half().to(dev) if keep_dense else None
            setattr(module, name, W4A16Linear(dense, child.bias, packed, scale))
        else:
            replace_linear_with_w4a16(child, group=group, keep_dense=keep_dense,
                                      scale_dtype=scale_dtype, device=device, quantizer=quantizer)
    return module
