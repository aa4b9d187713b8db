"""W4A16 GEMV ops for B200 (sm_100a): the reference's Python op surface over the C ABI.

Every function here keeps the name, arguments, output shape and dtype of its
counterpart in the reference's src/w4a16/kernels.py:33-43 and launches one of the
hand-written sm_100a kernels of libw4a16_b200.so on the current CUDA stream:

    w4a16_gemv(packed, scale, vec)       interleaved packing, per-row scale   (:40)
    w4a16_gemv_g128(packed, scale, vec)  interleaved packing, group-128 scale (:41)
    matvec_byte/u32/u32_v4/champ/uint4   simple packing, per-row scale     (:33-37)
    matvec_h2f32                         simple packing, fp16 products (lossy) (:38)
    matvec_fp16(mat, vec)                dense fp16 baseline                 (:43)

Inputs are validated before launch (the reference checked nothing): a wrong dtype,
device, layout or shape raises RuntimeError and launches nothing.  `vec` may also be
a [batch, cols] matrix, giving a [batch, rows] output.

gemv() is the general form (fp16 or fp32 scales, fp16 or fp32 output, fused bias,
split-K workspace) that W4A16Linear uses.
"""
import ctypes

import torch

from . import _lib
from .quant import (  # noqa: F401  (re-exported, as in the reference module)
    GROUP,
    dequant_ref,
    dequant_ref_group,
    pack_int4,
    pack_int4_interleaved,
    quantize_int4_group,
    quantize_int4_symmetric,
    unpack_int4,
)

_SCALE_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16}
_OUT_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16}
_PACKINGS = {"interleaved": _lib.PACK_INTERLEAVED, "simple": _lib.PACK_SIMPLE}


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _need(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_packed(packed):
    _need(isinstance(packed, torch.Tensor) and packed.is_cuda, "packed must be a CUDA tensor")
    _need(packed.dtype == torch.uint8, f"packed must be uint8, got {packed.dtype}")
    _need(packed.dim() == 2 and packed.is_contiguous(), "packed must be a contiguous [rows, cols/2] tensor")


def _check_vec(vec, cols, device):
    _need(isinstance(vec, torch.Tensor) and vec.device == device,
          f"vec must be a CUDA tensor on {device}")
    _need(vec.dtype == torch.float16, f"vec must be float16, got {vec.dtype}")
    _need(vec.dim() in (1, 2) and vec.shape[-1] == cols and vec.is_contiguous(),
          f"vec must be a contiguous [{cols}] or [batch, {cols}] tensor, got {tuple(vec.shape)}")


# ------------------------------------------------------------------ workspace

_WORKSPACE = {}


def _workspace(device, batch, rows, cols):
    """Per-device zero-filled buffer for the split-K path (the kernels re-zero its counters).

    Grown outside stream capture only; during capture a too-small buffer just turns
    split-K off for that call."""
    need = int(_lib.lib().w4a16_gemv_workspace_bytes(batch, rows, cols))
    key = device.index
    buf = _WORKSPACE.get(key)
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            return buf
        buf = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACE[key] = buf
    return buf


def reserve_workspace(device, batch, rows, cols):
    """Grow the split-K workspace ahead of CUDA-graph capture."""
    _workspace(torch.device(device), batch, rows, cols)


def new_workspace(device, batch=1):
    """A zero-filled workspace of its own for the split-K path (any rows and cols).

    Chained launches (pdl=True) overlap two consecutive kernels, so consecutive calls
    must use different workspaces; alternate two of these."""
    need = int(_lib.lib().w4a16_gemv_workspace_bytes(batch, 1, 1))
    return torch.zeros(need, dtype=torch.uint8, device=torch.device(device))


# --------------------------------------------------------------- general entry

def gemv(packed, scale, x, *, group=0, packing="interleaved", bias=None, out_dtype=torch.float32,
         out=None, split_k=True):
    """out[b, r] = sum_k q[r, k] * scale(r, k) * x[b, k] (+ bias[r]).

    packed   uint8 [rows, cols/2] (interleaved or simple packing)
    scale    fp32 or fp16, [rows] (group=0) or [rows, cols/128] (group=128)
    x        fp16 [cols] or [batch, cols]
    bias     optional fp32 [rows]
    returns  out_dtype [rows] or [batch, rows]
    """
    _check_packed(packed)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    dev = packed.device
    _check_vec(x, cols, dev)
    _need(packing in _PACKINGS, f"packing must be one of {list(_PACKINGS)}")
    _need(group in (0, GROUP), f"group must be 0 or {GROUP}")
    _need(isinstance(scale, torch.Tensor) and scale.device == dev and scale.dtype in _SCALE_DTYPES,
          "scale must be a float32/float16 CUDA tensor on the weights' device")
    want = (rows,) if group == 0 else (rows, cols // GROUP)
    _need(tuple(scale.shape) == want and scale.is_contiguous(),
          f"scale must be contiguous {want}, got {tuple(scale.shape)}")
    _need(out_dtype in _OUT_DTYPES, "out_dtype must be float32 or float16")
    if bias is not None:
        _need(bias.device == dev and bias.dtype == torch.float32 and tuple(bias.shape) == (rows,)
              and bias.is_contiguous(), "bias must be a contiguous float32 [rows] tensor")
    batch = 1 if x.dim() == 1 else x.shape[0]
    shape = (rows,) if x.dim() == 1 else (batch, rows)
    if out is None:
        out = torch.empty(shape, dtype=out_dtype, device=dev)
    else:
        _need(out.device == dev and out.dtype == out_dtype and tuple(out.shape) == shape
              and out.is_contiguous(), "out has the wrong device, dtype, shape or layout")
    ws = _workspace(dev, batch, rows, cols) if split_k else None
    with torch.cuda.device(dev):
        status = _lib.lib().w4a16_gemv(
            _ptr(packed), _PACKINGS[packing], _ptr(scale), _SCALE_DTYPES[scale.dtype], group,
            _ptr(x), batch, rows, cols, _ptr(out), _OUT_DTYPES[out_dtype], _ptr(bias),
            _ptr(ws), ws.numel() if ws is not None else 0, _stream(dev))
    _lib.check(status, "w4a16_gemv")
    return out


def _fused(prologue, packed, scale, src, gamma, eps, group, bias, out, out_dtype, split_k, pdl,
           workspace, swiglu_out=False):
    _check_packed(packed)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    dev = packed.device
    _need(group in (0, GROUP), f"group must be 0 or {GROUP}")
    _need(isinstance(scale, torch.Tensor) and scale.device == dev and scale.dtype in _SCALE_DTYPES
          and scale.is_contiguous(), "scale must be a contiguous float32/float16 CUDA tensor")
    if swiglu_out:
        _need(rows % 16 == 0 and bias is None, "swiglu_out needs rows % 16 == 0 and no bias")
    n_out = rows // 2 if swiglu_out else rows
    if out is None:
        out = torch.empty(n_out, dtype=out_dtype, device=dev)
    _need(out.device == dev and out.dtype in _OUT_DTYPES and tuple(out.shape) == (n_out,)
          and out.is_contiguous(), f"out must be a contiguous fp32/fp16 [{n_out}] tensor")
    if bias is not None:
        _need(bias.device == dev and bias.dtype == torch.float32 and tuple(bias.shape) == (rows,)
              and bias.is_contiguous(), "bias must be a contiguous float32 [rows] tensor")
    if workspace is not None:
        _need(workspace.device == dev and workspace.dtype == torch.uint8 and workspace.is_contiguous(),
              "workspace must be a contiguous uint8 tensor on the weights' device (new_workspace)")
        ws = workspace if split_k else None
    else:
        ws = _workspace(dev, 1, rows, cols) if split_k else None
    with torch.cuda.device(dev):
        status = _lib.lib().w4a16_gemv_fused(
            _ptr(packed), _ptr(scale), _SCALE_DTYPES[scale.dtype], group, prologue, _ptr(src),
            _ptr(gamma), float(eps), rows, cols, _ptr(out), _OUT_DTYPES[out.dtype], _ptr(bias),
            _ptr(ws), ws.numel() if ws is not None else 0,
            (_lib.LAUNCH_PDL if pdl else 0) | (_lib.LAUNCH_SWIGLU_OUT if swiglu_out else 0),
            _stream(dev))
    _lib.check(status, "w4a16_gemv_fused")
    return out


_CHAIN_DOC = """
    Chaining: pdl=True launches with programmatic dependent launch, so the kernel loads
    its first weights while the previous kernel in the stream finishes; consecutive
    chained calls must then use different split-K workspaces (pass two buffers from
    new_workspace alternately); workspace=None uses the per-device default."""


def gemv_staged(packed, scale, x, *, group=0, bias=None, out=None, out_dtype=torch.float32,
                split_k=True, pdl=False, workspace=None):
    """W @ x (+ bias) for one fp16 vector x [cols] staged in shared memory.

    The decode-step GEMV without a prologue (out may alias bias: in-place residual)."""
    cols = packed.shape[1] * 2
    _check_vec(x, cols, packed.device)
    _need(x.dim() == 1, "gemv_staged takes one activation vector")
    return _fused(_lib.PROLOGUE_NONE, packed, scale, x, None, 0.0, group, bias, out, out_dtype,
                  split_k, pdl, workspace)


def gemv_rmsnorm(packed, scale, h, gamma, eps=1e-5, *, group=0, bias=None, out=None,
                 out_dtype=torch.float32, split_k=True, pdl=False, workspace=None, swiglu_out=False):
    """W @ fp16(h * rsqrt(mean(h^2) + eps) * gamma) (+ bias): RMSNorm fused into the GEMV.

    h, gamma: fp32 [cols] on the weights' device.  out may alias bias (in-place residual).
    swiglu_out: W holds gate / up row pairs in blocks of 16 (interleave_gate_up's layout:
    8 gate rows, then their 8 up rows) and out[rows // 2] = silu(gate) * up of the fp32
    sums, the activation of a Llama MLP applied in the epilogue (no bias)."""
    cols = packed.shape[1] * 2
    for name, t in (("h", h), ("gamma", gamma)):
        _need(isinstance(t, torch.Tensor) and t.device == packed.device and t.dtype == torch.float32
              and tuple(t.shape) == (cols,) and t.is_contiguous(), f"{name} must be fp32 [{cols}]")
    return _fused(_lib.PROLOGUE_RMSNORM, packed, scale, h, gamma, eps, group, bias, out, out_dtype,
                  split_k, pdl, workspace, swiglu_out)


def gemv_swiglu(packed, scale, gate_up, *, group=0, bias=None, out=None, out_dtype=torch.float32,
                split_k=True, pdl=False, workspace=None):
    """W @ fp16(silu(gate) * up) (+ bias) with gate_up = [gate | up] fp16 [2 * cols]."""
    cols = packed.shape[1] * 2
    _need(isinstance(gate_up, torch.Tensor) and gate_up.device == packed.device
          and gate_up.dtype == torch.float16 and tuple(gate_up.shape) == (2 * cols,)
          and gate_up.is_contiguous(), f"gate_up must be fp16 [{2 * cols}]")
    return _fused(_lib.PROLOGUE_SWIGLU, packed, scale, gate_up, None, 0.0, group, bias, out, out_dtype,
                  split_k, pdl, workspace)


for _f in (gemv_staged, gemv_rmsnorm, gemv_swiglu):
    _f.__doc__ += _CHAIN_DOC


_ATTN_SCRATCH = {}


def decode_attention(qkv, cos, sin, pos, k_cache, v_cache, *, heads, kv_heads, out=None, splits=None,
                     pdl=False):
    """One decode token's attention with rotary and the KV-cache write in one launch.

    qkv fp16 [(heads + 2 kv_heads) * 64] (q | k | v); cos, sin fp32 [max_len, 64]
    (rotate-half tables); pos int64 [1] on the device; k_cache, v_cache fp16
    [kv_heads, max_len, 64] (this layer's).  Writes k_cache/v_cache at pos and returns
    out fp16 [heads * 64].  splits: CTAs per kv head over the positions (default one per
    32 positions; splits=1 with max_len <= 512 and 1, 2, 4 or 8 query heads per kv head
    runs one 16-warp CTA per kv head that combines in shared memory).  The zeroed scratch is kept per device and shape; allocate it (one
    eager call) before capturing the op in a CUDA graph.  pdl: programmatic dependent
    launch (see gemv_staged)."""
    dev = qkv.device
    D = 64
    max_len = k_cache.shape[1]
    _need(qkv.dtype == torch.float16 and qkv.is_cuda and qkv.is_contiguous()
          and tuple(qkv.shape) == ((heads + 2 * kv_heads) * D,), "qkv must be fp16 [(heads + 2 kv_heads) * 64]")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        _need(t.device == dev and t.dtype == torch.float16 and t.is_contiguous()
              and tuple(t.shape) == (kv_heads, max_len, D), f"{name} must be fp16 [kv_heads, max_len, 64]")
    for name, t in (("cos", cos), ("sin", sin)):
        _need(t.device == dev and t.dtype == torch.float32 and t.is_contiguous()
              and t.dim() == 2 and t.shape[1] == D and t.shape[0] >= max_len, f"{name} must be fp32 [>= max_len, 64]")
    _need(pos.device == dev and pos.dtype == torch.int64 and pos.numel() == 1, "pos must be int64 [1] on the device")
    if splits is None:  # one CTA per 32 positions (the fastest measured split for one token)
        splits = max(1, (max_len + 31) // 32)
    if out is None:
        out = torch.empty(heads * D, dtype=torch.float16, device=dev)
    _need(out.device == dev and out.dtype == torch.float16 and tuple(out.shape) == (heads * D,)
          and out.is_contiguous(), "out must be fp16 [heads * 64]")
    L = _lib.lib()
    need = L.w4a16_decode_attention_scratch_bytes(heads, kv_heads, splits)
    key = (dev.index, heads, kv_heads, splits)
    scratch = _ATTN_SCRATCH.get(key)
    if scratch is None:
        _need(not torch.cuda.is_current_stream_capturing(),
              "decode_attention scratch must exist before capture: call it once eagerly")
        scratch = torch.zeros(need, dtype=torch.uint8, device=dev)
        _ATTN_SCRATCH[key] = scratch
    with torch.cuda.device(dev):
        status = L.w4a16_decode_attention(
            _ptr(qkv), _ptr(cos), _ptr(sin), _ptr(pos), _ptr(k_cache), _ptr(v_cache), _ptr(out),
            _ptr(scratch), scratch.numel(), heads, kv_heads, D, max_len, splits,
            _lib.LAUNCH_PDL if pdl else 0, _stream(dev))
    _lib.check(status, "w4a16_decode_attention")
    return out


# ------------------------------------------------------- reference-named ops

def _ref_call(name, packed, scale, vec, group, packing):
    _check_packed(packed)
    _need(isinstance(scale, torch.Tensor) and scale.dtype == torch.float32,
          f"scale must be float32, got {getattr(scale, 'dtype', type(scale))}")
    if vec.dim() == 2:  # batched extension of the reference's 1-D vec
        return gemv(packed, scale, vec, group=group, packing=packing)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    _check_vec(vec, cols, packed.device)
    want = (rows,) if group == 0 else (rows, cols // GROUP)
    _need(scale.device == packed.device and tuple(scale.shape) == want and scale.is_contiguous(),
          f"scale must be a contiguous CUDA tensor of shape {want}")
    out = torch.empty(rows, dtype=torch.float32, device=packed.device)
    with torch.cuda.device(packed.device):
        status = getattr(_lib.lib(), name)(_ptr(packed), _ptr(scale), _ptr(vec), _ptr(out), rows,
                                           cols, _stream(packed.device))
    _lib.check(status, name)
    return out


def w4a16_gemv(packed, scale, vec):
    """Per-row int4 GEMV on the interleaved packing (reference kernels.py:40).

    Runs the same kernel as the C entry w4a16_marlin_cuda, through w4a16_gemv so that
    layers with few rows can use split-K.  fp16 scales are accepted too."""
    _check_packed(packed)
    return gemv(packed, scale, vec, group=0)


def w4a16_gemv_g128(packed, scale, vec):
    """Group-128 int4 GEMV on the interleaved packing (reference kernels.py:41);
    the C entry w4a16_marlin_g128_cuda runs the same kernel without split-K."""
    _check_packed(packed)
    _need((packed.shape[1] * 2) % GROUP == 0, f"cols must be a multiple of {GROUP} for group-128 scales")
    return gemv(packed, scale, vec, group=GROUP)


def matvec_byte(packed, scale, vec):
    """Simple-packing per-row GEMV (reference kernels.py:33)."""
    return _ref_call("w4a16_byte_cuda", packed, scale, vec, 0, "simple")


def matvec_u32(packed, scale, vec):
    """Simple-packing per-row GEMV (reference kernels.py:34)."""
    return _ref_call("w4a16_u32_cuda", packed, scale, vec, 0, "simple")


def matvec_u32_v4(packed, scale, vec):
    """Simple-packing per-row GEMV (reference kernels.py:35)."""
    return _ref_call("w4a16_u32_v4_cuda", packed, scale, vec, 0, "simple")


def matvec_champ(packed, scale, vec):
    """Simple-packing per-row GEMV (reference kernels.py:36)."""
    return _ref_call("w4a16_champ_cuda", packed, scale, vec, 0, "simple")


def matvec_uint4(packed, scale, vec):
    """Simple-packing per-row GEMV (reference kernels.py:37)."""
    return _ref_call("w4a16_uint4_cuda", packed, scale, vec, 0, "simple")


def matvec_h2f32(packed, scale, vec):
    """Lossy simple-packing GEMV: fp16 products summed in fp16 per packed word
    (reference kernels.py:38).  Expect ~1e-2 absolute error on N(0,1) weights."""
    _need(vec.dim() == 1, "matvec_h2f32 takes a 1-D vec")
    return _ref_call("w4a16_h2f32_cuda", packed, scale, vec, 0, "simple")


def matvec_fp16(mat, vec):
    """Dense fp16 GEMV with fp32 accumulation (reference kernels.py:43)."""
    _need(isinstance(mat, torch.Tensor) and mat.is_cuda and mat.dtype == torch.float16
          and mat.dim() == 2 and mat.is_contiguous(), "mat must be a contiguous fp16 CUDA matrix")
    rows, cols = mat.shape
    _check_vec(vec, cols, mat.device)
    _need(vec.dim() == 1, "matvec_fp16 takes a 1-D vec")
    out = torch.empty(rows, dtype=torch.float32, device=mat.device)
    with torch.cuda.device(mat.device):
        status = _lib.lib().w4a16_fp16_cuda(_ptr(mat), _ptr(vec), _ptr(out), rows, cols,
                                            _stream(mat.device))
    _lib.check(status, "w4a16_fp16_cuda")
    return out


# ------------------------------------------------------------ data-format ops

def dequant_int4(packed, scale, group=0, packing="interleaved"):
    """fp16 [rows, cols] = fp16(fp32(q) * fp32(scale)) on the GPU; bit-identical to
    (q.float() * scale_expanded).half() (the reference's dequant formula)."""
    _check_packed(packed)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    _need(scale.device == packed.device and scale.dtype in _SCALE_DTYPES and scale.is_contiguous(),
          "scale must be a contiguous float32/float16 tensor on the weights' device")
    out = torch.empty(rows, cols, dtype=torch.float16, device=packed.device)
    with torch.cuda.device(packed.device):
        status = _lib.lib().w4a16_dequant(_ptr(packed), _PACKINGS[packing], _ptr(scale),
                                          _SCALE_DTYPES[scale.dtype], group, rows, cols, _ptr(out),
                                          _stream(packed.device))
    _lib.check(status, "w4a16_dequant")
    return out


_GEMM_WS = {}


def _gemm_workspace(dev, m, n, k):
    """The per-device split-K workspace for a GEMM of this size (zero-filled when made, grown
    outside stream capture only), or None when the call does not split K."""
    need = int(_lib.lib().w4a16_gemm_workspace_bytes(m, n, k))
    if need == 0:
        return None
    ws = _GEMM_WS.get(dev)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            return None  # no allocation during capture: that call runs unsplit
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        _GEMM_WS[dev] = ws
    return ws


def gemm(packed, scale, x, *, group=0, bias=None, out_dtype=torch.float32, out=None, workspace=None):
    """y [M, N] = x [M, K] @ dequant_int4(packed, scale, group).T (+ bias), fp32 sums, on the
    tensor cores (tcgen05, accumulators in tensor memory); the dequantised weight is formed
    on chip only.  For many activation rows (prefill): the GEMV above is the batch 1..64
    path.  Interleaved packing, fp32 scales; K a multiple of 64 (128 with group 128).
    workspace: a zero-filled uint8 CUDA tensor of at least w4a16_gemm_workspace_bytes, None
    for this device's shared one (calls on several streams at once need their own), or False
    for no split of K.  Raises RuntimeError on bad input and launches nothing."""
    _check_packed(packed)
    n, k = packed.shape[0], packed.shape[1] * 2
    dev = packed.device
    _need(isinstance(x, torch.Tensor) and x.device == dev and x.dtype == torch.float16 and x.dim() == 2
          and x.shape[1] == k and x.is_contiguous() and x.data_ptr() % 16 == 0,
          f"x must be a contiguous 16-byte aligned fp16 [M, {k}] tensor on the weights' device")
    _need(packed.data_ptr() % 16 == 0, "packed must be 16-byte aligned")
    _need(group in (0, GROUP), f"group must be 0 or {GROUP}")
    want = (n,) if group == 0 else (n, k // GROUP)
    _need(isinstance(scale, torch.Tensor) and scale.device == dev and scale.dtype == torch.float32
          and tuple(scale.shape) == want and scale.is_contiguous(),
          f"scale must be a contiguous float32 {want} tensor on the weights' device")
    _need(k % (GROUP if group else 64) == 0, f"K={k} must be a multiple of {GROUP if group else 64}")
    _need(out_dtype in _OUT_DTYPES, "out_dtype must be float32 or float16")
    if bias is not None:
        _need(bias.device == dev and bias.dtype == torch.float32 and tuple(bias.shape) == (n,)
              and bias.is_contiguous(), "bias must be a contiguous float32 [N] tensor")
    m = x.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=dev)
    _need(out.dtype == out_dtype and tuple(out.shape) == (m, n) and out.is_contiguous() and out.device == dev,
          "out must be a contiguous [M, N] tensor of out_dtype on the weights' device")
    if m == 0:
        return out
    with torch.cuda.device(dev):
        if workspace is None:
            workspace = _gemm_workspace(dev, m, n, k)
        elif workspace is False:
            workspace = None
        else:
            _need(isinstance(workspace, torch.Tensor) and workspace.device == dev
                  and workspace.dtype == torch.uint8 and workspace.is_contiguous(),
                  "workspace must be a contiguous uint8 tensor on the weights' device")
        wsb = workspace.numel() if workspace is not None else 0
        status = _lib.lib().w4a16_gemm(_ptr(packed), _ptr(scale), group, _ptr(x),
                                       _ptr(bias) if bias is not None else None, m, n, k, _ptr(out),
                                       _OUT_DTYPES[out_dtype], _ptr(workspace), wsb, _stream(dev))
    _lib.check(status, "w4a16_gemm")
    return out


def quantize_pack(w, group=0, packing="interleaved", scale_dtype=torch.float32):
    """Quantise (symmetric int4, per-row or group-128) and pack on the GPU in one launch.

    Returns (packed uint8 [rows, cols/2], scale [rows] or [rows, cols/128]).  For fp32
    input the codes and fp32 scales equal quantize_int4_* followed by the packer."""
    _need(isinstance(w, torch.Tensor) and w.is_cuda and w.dim() == 2 and w.is_contiguous()
          and w.dtype in (torch.float32, torch.float16), "w must be a contiguous fp32/fp16 CUDA matrix")
    rows, cols = w.shape
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=w.device)
    sshape = (rows,) if group == 0 else (rows, cols // GROUP)
    scale = torch.empty(sshape, dtype=scale_dtype, device=w.device)
    with torch.cuda.device(w.device):
        status = _lib.lib().w4a16_quantize_pack(
            _ptr(w), _SCALE_DTYPES[w.dtype], rows, cols, group, _PACKINGS[packing], _ptr(packed),
            _ptr(scale), _SCALE_DTYPES[scale_dtype], _stream(w.device))
    _lib.check(status, "w4a16_quantize_pack")
    return packed, scale


def read_device_error(device=None):
    """Read and clear the device error word (non-zero if a kernel gave up on a wait).

    A kernel that gave up may have left split-K counters set, so after a non-zero code the
    workspaces this module owns on the device (the GEMV's and the GEMM's) are zero-filled
    again; workspaces a caller passed in must be zero-filled by the caller."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    code = ctypes.c_int(0)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().w4a16_read_device_error(ctypes.byref(code), _stream(dev)),
                   "w4a16_read_device_error")
        if code.value:
            for buf in (_WORKSPACE.get(dev.index), _GEMM_WS.get(dev)):
                if buf is not None:
                    buf.zero_()
    return code.value
