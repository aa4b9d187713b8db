"""Symmetric int4 quantisers, nibble packers and the dequant-then-matmul helpers.

Same functions, arguments and outputs as the reference's src/w4a16/kernels.py:46-101;
codes, scales and packed bytes are bit-identical to it (pinned by the golden vectors
under tests/golden).  All functions are plain torch and run on any device.

One deliberate difference: an all-zero row (or group) has scale 0, for which the
reference divides 0 by 0 and casts NaN to int8 (undefined).  Here such codes are 0.
"""
import torch

GROUP = 128

# Nibble slot i of a packed 32-bit word holds column _INTERLEAVE[i] of its 8 columns
# (src/w4a16/kernels.py:73).  Byte b of the word is slot 2b | slot 2b+1 << 4, so the
# low and high nibble of byte b come from these columns:
_INTERLEAVE = [0, 2, 4, 6, 1, 3, 5, 7]
_BYTE_LO_COLS = [_INTERLEAVE[2 * b] for b in range(4)]       # [0, 4, 1, 5]
_BYTE_HI_COLS = [_INTERLEAVE[2 * b + 1] for b in range(4)]   # [2, 6, 3, 7]


def _codes(w, scale):
    """round-half-even(w / scale) clamped to [-8, 7] as int8; scale 0 gives code 0."""
    zero = scale == 0
    div = torch.where(zero, torch.ones_like(scale), scale)
    q = torch.round(w / div).clamp(-8, 7)
    return torch.where(zero, torch.zeros_like(q), q).to(torch.int8)


def quantize_int4_symmetric(w):
    """Per-row symmetric int4 (kernels.py:47-50): scale[r] = max_k |w[r,k]| / 7.

    Returns (codes int8 [rows, cols], scale [rows] in w's dtype)."""
    scale = w.abs().amax(dim=1, keepdim=True) / 7.0
    return _codes(w, scale), scale.squeeze(1)


def quantize_int4_group(w, group=GROUP):
    """Group-wise symmetric int4 (kernels.py:52-60): one scale per `group` consecutive
    columns of a row.  Returns (codes int8 [rows, cols], scales [rows, cols/group])."""
    rows, cols = w.shape
    assert cols % group == 0, f"cols {cols} not divisible by group {group}"
    wg = w.reshape(rows, cols // group, group)
    scale = wg.abs().amax(dim=2, keepdim=True) / 7.0
    q = _codes(wg, scale).reshape(rows, cols)
    return q, scale.reshape(rows, cols // group).contiguous()


def pack_int4(q):
    """Simple packing (kernels.py:64-70): byte c = (q[2c]+8) << 4 | (q[2c+1]+8)."""
    n = (q + 8).to(torch.uint8)
    return ((n[:, 0::2] << 4) | n[:, 1::2]).contiguous()


def pack_int4_interleaved(q):
    """Interleaved packing (kernels.py:73-91): within each group of 8 columns, nibble
    slot i of the little-endian u32 holds column [0,2,4,6,1,3,5,7][i].  Built with
    uint8 arithmetic only (the reference goes through int64 temporaries)."""
    rows, cols = q.shape
    assert cols % 8 == 0, "interleaved packing requires cols % 8 == 0"
    n = ((q + 8) & 0xF).to(torch.uint8).view(rows, cols // 8, 8)
    lo = n[:, :, _BYTE_LO_COLS]
    hi = n[:, :, _BYTE_HI_COLS]
    return (lo | (hi << 4)).reshape(rows, cols // 2)


def unpack_int4(packed, interleaved=True):
    """Inverse of the packers: uint8 [rows, cols/2] -> int8 codes [rows, cols]."""
    rows, half = packed.shape
    lo = (packed & 0xF).to(torch.int8) - 8
    hi = (packed >> 4).to(torch.int8) - 8
    if not interleaved:
        return torch.stack([hi, lo], dim=2).reshape(rows, half * 2)
    lo = lo.view(rows, half // 4, 4)
    hi = hi.view(rows, half // 4, 4)
    out = torch.empty(rows, half // 4, 8, dtype=torch.int8, device=packed.device)
    out[:, :, _BYTE_LO_COLS] = lo
    out[:, :, _BYTE_HI_COLS] = hi
    return out.reshape(rows, half * 2)


def dequant_ref(q, scale, vec):
    """Packing-independent fp32 reference (kernels.py:94-96): (q * scale) @ vec."""
    return (q.float() * scale.float()[:, None]).matmul(vec.float())


def dequant_ref_group(q, scale_group, vec, group=GROUP):
    """Group-wise fp32 reference (kernels.py:98-101)."""
    full = scale_group.float().repeat_interleave(group, dim=1)
    return (q.float() * full).matmul(vec.float())
