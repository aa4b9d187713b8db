"""TEST INFRASTRUCTURE ONLY — the oracle for the W4A16 GEMV path.

A CPU restatement, in numpy, of the reference's quantise / pack / dequant-then-matmul
algorithm (src/w4a16/kernels.py of emirabayer/w4a16-gemv-optimization-ladder).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import it, and
only as the checker: the library never calls it and has no CPU fallback.

Pinned against the reference itself: tests/golden/*.npz were produced by running the
reference's own Python functions (tests/golden/make_golden.py) and
tests/test_oracle_golden.py checks every function below against them bit for bit
(integer and packed data) or to fp32 rounding (GEMV sums).

Conventions: weights/scales float32, codes int8 in [-8, 7], packed uint8 [rows, cols/2],
activations float16.
"""
import numpy as np

GROUP = 128
# Column held by nibble slot i of a packed 32-bit word (kernels.py:73).
INTERLEAVE = (0, 2, 4, 6, 1, 3, 5, 7)


def _codes(w, scale):
    """round-half-even(w / scale) clamped to [-8, 7] (kernels.py:49 and :59);
    scale 0 (all-zero row or group) gives code 0."""
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.rint(w / scale)
    r = np.where(scale == 0, 0.0, r)
    return np.clip(r, -8, 7).astype(np.int8)


def quantize_int4_symmetric(w):
    """Per-row symmetric int4, kernels.py:47-50: scale = max|w| / 7 over each row."""
    w = np.asarray(w, dtype=np.float32)
    scale = (np.abs(w).max(axis=1, keepdims=True) / np.float32(7.0)).astype(np.float32)
    return _codes(w, scale), scale[:, 0]


def quantize_int4_group(w, group=GROUP):
    """Group-wise symmetric int4, kernels.py:52-60: scale per `group` consecutive columns."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    assert cols % group == 0
    wg = w.reshape(rows, cols // group, group)
    scale = (np.abs(wg).max(axis=2, keepdims=True) / np.float32(7.0)).astype(np.float32)
    q = _codes(wg, scale).reshape(rows, cols)
    return q, scale[:, :, 0]


def pack_int4(q):
    """Simple packing, kernels.py:64-70: byte c = (q[2c]+8) << 4 | (q[2c+1]+8)."""
    q = np.asarray(q, dtype=np.int16)
    hi = ((q[:, 0::2] + 8) & 0xF).astype(np.uint8)
    lo = ((q[:, 1::2] + 8) & 0xF).astype(np.uint8)
    return (hi << 4) | lo


def pack_int4_interleaved(q):
    """Interleaved packing, kernels.py:73-91: build each little-endian u32 word from
    its 8 columns (slot i <- column INTERLEAVE[i]) and split it into 4 bytes."""
    q = np.asarray(q, dtype=np.int64)
    rows, cols = q.shape
    assert cols % 8 == 0
    n = (q + 8) & 0xF
    g = n.reshape(rows, cols // 8, 8)
    word = np.zeros((rows, cols // 8), dtype=np.int64)
    for slot, col in enumerate(INTERLEAVE):
        word |= g[:, :, col] << (4 * slot)
    out = np.stack([(word >> (8 * b)) & 0xFF for b in range(4)], axis=2)
    return out.reshape(rows, cols // 2).astype(np.uint8)


def unpack_int4(packed, interleaved=True):
    """Codes back from packed bytes (inverse of the two packers)."""
    packed = np.asarray(packed, dtype=np.uint8)
    rows, half = packed.shape
    if not interleaved:
        out = np.empty((rows, half * 2), dtype=np.int8)
        out[:, 0::2] = (packed >> 4).astype(np.int8) - 8
        out[:, 1::2] = (packed & 0xF).astype(np.int8) - 8
        return out
    word = packed.reshape(rows, half // 4, 4).astype(np.int64)
    word = word[:, :, 0] | (word[:, :, 1] << 8) | (word[:, :, 2] << 16) | (word[:, :, 3] << 24)
    out = np.empty((rows, half // 4, 8), dtype=np.int8)
    for slot, col in enumerate(INTERLEAVE):
        out[:, :, col] = ((word >> (4 * slot)) & 0xF).astype(np.int8) - 8
    return out.reshape(rows, half * 2)


def expand_scale(scale, cols, group=0):
    """Scale per element, fp32 [rows, cols] (kernels.py:96 and :100)."""
    scale = np.asarray(scale, dtype=np.float32)
    if group == 0:
        return np.broadcast_to(scale[:, None], (scale.shape[0], cols))
    return np.repeat(scale, group, axis=1)


def dequant_f32(q, scale, group=0):
    """fp32(q) * fp32(scale): the dequantised matrix of kernels.py:96 / :100-101."""
    q = np.asarray(q)
    return q.astype(np.float32) * expand_scale(scale, q.shape[1], group)


def dequant_f16(q, scale, group=0):
    """fp16(fp32(q) * fp32(scale)) with round-to-nearest-even: the fp16 dequant target."""
    return dequant_f32(q, scale, group).astype(np.float16)


def gemv(q, scale, x, group=0):
    """y[b, r] = sum_k dequant_f32(q, scale)[r, k] * fp32(x[b, k]), summed in float64.

    The reference's dequant_ref / dequant_ref_group (kernels.py:94-101) sum in fp32;
    float64 here makes the oracle the more accurate side of every comparison."""
    w = dequant_f32(q, scale, group).astype(np.float64)
    xf = np.asarray(x, dtype=np.float32).astype(np.float64)
    y = xf @ w.T if xf.ndim == 2 else w @ xf
    return y


def gemv_packed(packed, scale, x, group=0, interleaved=True):
    """gemv() starting from packed bytes."""
    return gemv(unpack_int4(packed, interleaved), scale, x, group)


def gemv_h2f32(q, scale, x):
    """The reference's deliberately lossy h2f32 kernel (kernels/w4a16_kernels.cu:161-171),
    every floating-point operation emulated in its order, so the result is bit-exact.

    q: signed codes [rows, cols] (cols a multiple of 8), scale: fp32 per row, x: fp16.
    Lane l of a row's warp takes packed words l, l+32, ... in order.  Per word, pairs
    (2k, 2k+1) run two fp16 chains: even = f16(q0*x0), f16(q2*x2 + even), f16(q4*x4 +
    even), f16(q6*x6 + even), likewise odd over columns 1,3,5,7 (mul.rn then fma.rn,
    each rounded once; the float64 intermediates here are exact).  The lane sum is
    p = p + (f32(even) + f32(odd)) in fp32; then p = p * scale, and the warp's shuffle
    tree p += shfl_down(p, o) for o = 16, 8, 4, 2, 1 leaves lane 0's value.
    """
    q = np.asarray(q)
    rows, cols = q.shape
    words = cols // 8
    qw = q.reshape(rows, words, 8).astype(np.float64)
    xw = np.asarray(x, dtype=np.float16).astype(np.float64).reshape(words, 8)

    def f16(v):
        return v.astype(np.float16).astype(np.float64)

    with np.errstate(over="ignore", invalid="ignore"):
        chains = []
        for c0 in (0, 1):
            t = f16(qw[:, :, c0] * xw[:, c0])
            for c in (c0 + 2, c0 + 4, c0 + 6):
                t = f16(qw[:, :, c] * xw[:, c] + t)
            chains.append(t.astype(np.float32))
        wsum = chains[0] + chains[1]                      # float32 add
        lanes = np.zeros((rows, 32), dtype=np.float32)
        for g0 in range(0, words, 32):
            n = min(32, words - g0)
            lanes[:, :n] = lanes[:, :n] + wsum[:, g0:g0 + n]
        lanes = lanes * np.asarray(scale, dtype=np.float32)[:, None]
        for o in (16, 8, 4, 2, 1):
            shifted = lanes.copy()
            shifted[:, :32 - o] = lanes[:, o:]            # shfl_down keeps its own value past lane 31-o
            lanes = lanes + shifted
    return lanes[:, 0]
