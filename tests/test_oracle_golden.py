"""Pins the oracle (numpy and C restatements) to the reference's own outputs.

tests/golden/reference_golden.npz was produced by running the reference's Python
functions (tests/golden/make_golden.py).  Integer and packed data must match bit for
bit; GEMV sums (the oracle sums in float64, the reference in fp32) within fp32
rounding."""
import numpy as np
import pytest

from oracle import c_oracle
from oracle import w4a16_oracle as O


def _cases(golden, group=None):
    names = [str(n) for n in golden["cases"]]
    if group is None:
        return names
    return [n for n in names if int(golden[f"{n}.group"]) == group]


def test_known_answer(golden):
    q = golden["known_q"]
    assert O.pack_int4_interleaved(q).tolist() == [[0x64, 0xA8, 0x75, 0xB9]]
    assert O.pack_int4(q).tolist() == [[0x45, 0x67, 0x89, 0xAB]]
    np.testing.assert_array_equal(O.pack_int4_interleaved(q), golden["known_inter"])
    np.testing.assert_array_equal(O.pack_int4(q), golden["known_simple"])


@pytest.mark.parametrize("group", [0, 128])
def test_quantize_matches_reference(golden, group):
    for n in _cases(golden, group):
        w = golden[f"{n}.w"].astype(np.float32)
        q, s = O.quantize_int4_group(w, group) if group else O.quantize_int4_symmetric(w)
        np.testing.assert_array_equal(q, golden[f"{n}.q"], err_msg=n)
        np.testing.assert_array_equal(s, golden[f"{n}.s"], err_msg=n)


def test_pack_and_unpack_match_reference(golden):
    for n in _cases(golden):
        q = golden[f"{n}.q"]
        np.testing.assert_array_equal(O.pack_int4(q), golden[f"{n}.simple"], err_msg=n)
        np.testing.assert_array_equal(O.unpack_int4(golden[f"{n}.simple"], interleaved=False), q)
        if f"{n}.inter" in golden:
            np.testing.assert_array_equal(O.pack_int4_interleaved(q), golden[f"{n}.inter"], err_msg=n)
            np.testing.assert_array_equal(O.unpack_int4(golden[f"{n}.inter"]), q)


def test_dequant_f16_bit_exact(golden):
    for n in _cases(golden):
        group = int(golden[f"{n}.group"])
        d = O.dequant_f16(golden[f"{n}.q"], golden[f"{n}.s"], group)
        np.testing.assert_array_equal(d.view(np.uint16), golden[f"{n}.deq16"].view(np.uint16), err_msg=n)


def test_fakequant_formula(golden):
    # benchmarks/perplexity.py:22-25: per-row q*scale in fp32, then fp16.  There q stays
    # a float, so round() of a small negative weight gives -0.0 and the product -0.0;
    # from int8 codes it is +0.0.  Every value is equal (and bit-equal except the sign
    # of those zeros).
    w = golden["fakequant.w"].astype(np.float32)
    q, s = O.quantize_int4_symmetric(w)
    mine = O.dequant_f16(q, s)
    ref = golden["fakequant.deq16"]
    np.testing.assert_array_equal(mine, ref)
    nz = ref != 0
    np.testing.assert_array_equal(mine.view(np.uint16)[nz], ref.view(np.uint16)[nz])


def test_gemv_matches_reference(golden):
    for n in _cases(golden):
        group = int(golden[f"{n}.group"])
        y = O.gemv(golden[f"{n}.q"], golden[f"{n}.s"], golden[f"{n}.x"], group)
        ref = golden[f"{n}.y"].astype(np.float64)
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * max(1.0, np.abs(ref).max()),
                                   err_msg=n)


def test_c_oracle_matches_reference(golden):
    c_oracle.build()
    for n in _cases(golden):
        group = int(golden[f"{n}.group"])
        w = golden[f"{n}.w"].astype(np.float32)
        for interleaved, key in ((True, "inter"), (False, "simple")):
            if f"{n}.{key}" not in golden:
                continue
            packed, s = c_oracle.quantize_pack(w, group=group, interleaved=interleaved, threads=2)
            np.testing.assert_array_equal(packed, golden[f"{n}.{key}"], err_msg=n)
            np.testing.assert_array_equal(s, golden[f"{n}.s"], err_msg=n)
            y = c_oracle.gemv(packed, s, golden[f"{n}.x"], group=group, interleaved=interleaved,
                              threads=2)
            ref = golden[f"{n}.y"]
            np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * max(1.0, np.abs(ref).max()),
                                       err_msg=n)


def test_c_oracle_fp32_accumulate_close_to_f64():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 2048)) * 0.02).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(2048).astype(np.float16)
    packed, s = c_oracle.quantize_pack(w, group=128)
    y64 = c_oracle.gemv(packed, s, x, group=128, accumulate_f64=True)
    y32 = c_oracle.gemv(packed, s, x, group=128, accumulate_f64=False)
    np.testing.assert_allclose(y32, y64, rtol=1e-4, atol=1e-5)


def test_oracle_batched_matches_rows():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, 256)).astype(np.float16)
    q, s = O.quantize_int4_symmetric(w)
    yb = O.gemv(q, s, x)
    for b in range(3):
        np.testing.assert_allclose(yb[b], O.gemv(q, s, x[b]), rtol=0, atol=1e-12)
    packed = O.pack_int4_interleaved(q)
    yc = c_oracle.gemv(packed, s, x, threads=2)
    np.testing.assert_allclose(yc, yb, rtol=1e-6, atol=1e-7)


def _h2f32_scalar(q, scale, x):
    """The reference's k_h2f32 (kernels/w4a16_kernels.cu:161-171) as scalar loops: lane l
    sums words l, l+32, ...; per word two fp16 chains over the column pairs (mul, then fma
    rounded once each); fp32 lane sums scaled, then reduced by shfl_down."""
    rows, cols = q.shape
    out = []
    for r in range(rows):
        lanes = []
        for lane in range(32):
            p = np.float32(0)
            for g in range(lane, cols // 8, 32):
                t = [None, None]
                for k in range(4):
                    for h in (0, 1):
                        c = 8 * g + 2 * k + h
                        prod = float(q[r, c]) * float(x[c])
                        t[h] = np.float16(prod if k == 0 else prod + float(t[h]))
                p = np.float32(p + np.float32(np.float32(t[0]) + np.float32(t[1])))
            lanes.append(np.float32(p * scale[r]))
        for o in (16, 8, 4, 2, 1):
            lanes = [np.float32(lanes[i] + (lanes[i + o] if i + o < 32 else lanes[i])) for i in range(32)]
        out.append(lanes[0])
    return np.array(out, dtype=np.float32)


@pytest.mark.parametrize("cols,vscale", [(560, 3.0), (2048, 1.0), (64, 1200.0)])
def test_h2f32_oracle_matches_scalar_restatement(cols, vscale):
    rng = np.random.default_rng(cols)
    q = rng.integers(-8, 8, size=(6, cols))
    x = (rng.standard_normal(cols) * vscale).astype(np.float16)
    s = rng.random(6).astype(np.float32)
    got = O.gemv_h2f32(q, s, x)
    want = _h2f32_scalar(q, s, x)
    assert np.array_equal(got, want) or np.array_equal(np.isnan(got), np.isnan(want)) and \
        np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])
    if vscale < 10:  # lossy: fp16 rounding of every product shows against the exact sum
        exact = (q * x.astype(np.float64)).sum(1) * s
        assert 0 < np.abs(got - exact).max() < 0.5
