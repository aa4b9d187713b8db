"""GPU parity of the sm_100a kernels, called through the C ABI, against the oracle.

The first block mirrors the reference's own suite (tests/test_kernels.py:25-144:
same shapes, seeds, distributions and tolerances).  The rest compares against the
CPU oracle (oracle/, pinned to the reference's golden vectors) with the tolerance the
W4A16 path is held to:

    |y - y_oracle| <= ATOL + RTOL * |y_oracle|,  ATOL = RTOL = 1e-3   (fp32 outputs)

covering the golden fixtures, the full-size configurations (262144x2048 per-row and
group-128 with and without outliers, lm_head 128256x2048, 8192x2048, the 2048x8192
split-K layer), batches 1..33, fp16 scales, the fp16+bias epilogue, ragged and
minimal shapes, the generic fallback, bit-exact dequantisation and GPU quantisation.
"""
import ctypes

import numpy as np
import pytest
import torch

import w4a16 as K
from oracle import c_oracle
from oracle import w4a16_oracle as O

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-3           # the W4A16 path's tolerance vs the fp32 oracle
REF_ATOL, REF_RTOL = 1e-3, 1e-2  # the reference suite's tolerance (tests/test_kernels.py:19)
SHAPES = [(4096, 2048), (2048, 4096), (8192, 2048)]
SIMPLE = [("byte", K.matvec_byte), ("u32", K.matvec_u32), ("u32_v4", K.matvec_u32_v4),
          ("champ", K.matvec_champ), ("uint4", K.matvec_uint4)]
DEV = "cuda"


def _sid(s):
    return f"{s[0]}x{s[1]}"


def assert_close(y, ref, atol=ATOL, rtol=RTOL, what=""):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(y - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    idx = np.flatnonzero(bad)[:8]
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance, "
                           f"max abs err {err.max():.3e}; first bad flat indices {idx.tolist()} "
                           f"got {y.ravel()[idx].tolist()} want {ref.ravel()[idx].tolist()}")


def _setup(rows, cols, seed=0):
    # the reference's _setup (tests/test_kernels.py:41-48): N(0,1) weights
    torch.manual_seed(seed)
    mat = torch.randn(rows, cols, device=DEV).half()
    vec = torch.randn(cols, device=DEV).half()
    q, scale = K.quantize_int4_symmetric(mat.float())
    scale = scale.float().cuda()
    ref = K.dequant_ref(q.cuda(), scale, vec)
    return q, scale, vec, mat, ref


# ------------------------------------------------- the reference's suite, as-is

@pytest.mark.parametrize("shape", SHAPES, ids=_sid)
@pytest.mark.parametrize("name,fn", SIMPLE, ids=[k[0] for k in SIMPLE])
def test_simple_packing_kernels(name, fn, shape):
    q, scale, vec, _, ref = _setup(*shape)
    out = fn(K.pack_int4(q).cuda(), scale, vec)
    assert torch.allclose(out, ref, atol=REF_ATOL, rtol=REF_RTOL), \
        f"{name} {_sid(shape)} max abs err {(out - ref).abs().max().item():.3e}"


@pytest.mark.parametrize("shape", SHAPES, ids=_sid)
def test_marlin_interleaved(shape):
    q, scale, vec, _, ref = _setup(*shape)
    out = K.w4a16_gemv(K.pack_int4_interleaved(q).cuda(), scale, vec)
    assert torch.allclose(out, ref, atol=REF_ATOL, rtol=REF_RTOL)


@pytest.mark.parametrize("shape", SHAPES, ids=_sid)
def test_marlin_group128(shape):
    rows, cols = shape
    torch.manual_seed(0)
    mat = torch.randn(rows, cols, device=DEV).half()
    vec = torch.randn(cols, device=DEV).half()
    q, scale_g = K.quantize_int4_group(mat.float(), group=128)
    out = K.w4a16_gemv_g128(K.pack_int4_interleaved(q).cuda(), scale_g.float().cuda(), vec)
    ref = K.dequant_ref_group(q.cuda(), scale_g.float().cuda(), vec, group=128)
    assert torch.allclose(out, ref, atol=REF_ATOL, rtol=REF_RTOL)


@pytest.mark.parametrize("shape", SHAPES, ids=_sid)
def test_h2f32_is_documented_lossy(shape):
    q, scale, vec, _, ref = _setup(*shape)
    out = K.matvec_h2f32(K.pack_int4(q).cuda(), scale, vec)
    assert out.shape == ref.shape and torch.isfinite(out).all()
    err = (out - ref).abs().max().item()
    assert err < 5e-1, f"h2f32 error {err:.3e} unexpectedly large"
    assert not torch.allclose(out, ref, atol=REF_ATOL), "h2f32 passes the tight tolerance"


@pytest.mark.parametrize("rows,cols,vscale", [(4096, 2048, 1.0), (1037, 560, 1.0), (64, 20480, 1.0),
                                              (300, 4096, 1500.0), (7, 8, 1.0)],
                         ids=lambda v: str(v))
def test_h2f32_bit_exact_vs_oracle(rows, cols, vscale):
    # every fp16 rounding, the per-lane fp32 order and the shuffle tree of the
    # reference's kernel, emulated; vscale 1500 drives some fp16 sums into overflow (inf)
    rng = np.random.default_rng(rows + cols)
    q = rng.integers(-8, 8, size=(rows, cols)).astype(np.int8)
    x = (rng.standard_normal(cols) * vscale).astype(np.float16)
    scale = (rng.random(rows) * 0.1 + 0.01).astype(np.float32)
    packed = K.pack_int4(torch.from_numpy(q)).cuda()
    out = K.matvec_h2f32(packed, torch.from_numpy(scale).cuda(), torch.from_numpy(x).cuda())
    want = O.gemv_h2f32(q, scale, x)
    got = out.cpu().numpy()
    same = (got == want) | (np.isnan(got) & np.isnan(want))
    assert same.all(), (f"{(~same).sum()} of {rows} rows differ; first "
                        f"{np.flatnonzero(~same)[:4].tolist()}: got {got[~same][:4]} want {want[~same][:4]}")


def test_marlin_matches_champ_exactly_enough():
    q, scale, vec, _, _ = _setup(8192, 2048)
    out_c = K.matvec_champ(K.pack_int4(q).cuda(), scale, vec)
    out_m = K.w4a16_gemv(K.pack_int4_interleaved(q).cuda(), scale, vec)
    assert torch.allclose(out_c, out_m, atol=REF_ATOL, rtol=REF_RTOL)


@pytest.mark.parametrize("packer", [K.pack_int4, K.pack_int4_interleaved], ids=["simple", "interleaved"])
def test_pack_roundtrip(packer):
    torch.manual_seed(0)
    w = torch.randn(64, 128, device=DEV)
    q, _ = K.quantize_int4_symmetric(w)
    packed = packer(q)
    assert packed.dtype == torch.uint8 and packed.shape == (64, 64)
    assert torch.equal(K.unpack_int4(packed, interleaved=packer is K.pack_int4_interleaved), q)


def test_quant_error_regression():
    torch.manual_seed(0)
    w = torch.randn(4096, 4096, device=DEV)
    q, scale = K.quantize_int4_symmetric(w)
    frob = (torch.norm(w - q.float() * scale.unsqueeze(1)) / torch.norm(w)).item()
    assert 0.10 < frob < 0.20


# ------------------------------------------------------------ golden fixtures

def _golden_cases(golden):
    return [str(n) for n in golden["cases"]]


def test_golden_cases_through_every_entry_point(golden):
    for n in _golden_cases(golden):
        group = int(golden[f"{n}.group"])
        ref = golden[f"{n}.y"]
        s = torch.from_numpy(golden[f"{n}.s"]).to(DEV)
        x = torch.from_numpy(golden[f"{n}.x"]).to(DEV)
        if f"{n}.inter" in golden:
            p = torch.from_numpy(golden[f"{n}.inter"]).to(DEV)
            y = K.w4a16_gemv_g128(p, s, x) if group else K.w4a16_gemv(p, s, x)
            assert_close(y.cpu(), ref, what=f"{n} interleaved")
            y16 = K.gemv(p, s.half(), x, group=group)
            ref16 = O.gemv(golden[f"{n}.q"], golden[f"{n}.s"].astype(np.float16), golden[f"{n}.x"], group)
            assert_close(y16.cpu(), ref16, what=f"{n} fp16 scales")
        ps = torch.from_numpy(golden[f"{n}.simple"]).to(DEV)
        y = K.gemv(ps, s, x, group=group, packing="simple")
        assert_close(y.cpu(), ref, what=f"{n} simple")
        if not group:
            assert_close(K.matvec_champ(ps, s, x).cpu(), ref, what=f"{n} champ")


def test_golden_dequant_bit_exact(golden):
    for n in _golden_cases(golden):
        group = int(golden[f"{n}.group"])
        s = torch.from_numpy(golden[f"{n}.s"]).to(DEV)
        want = golden[f"{n}.deq16"].view(np.uint16)
        for packing, key in (("interleaved", "inter"), ("simple", "simple")):
            if f"{n}.{key}" not in golden:
                continue
            p = torch.from_numpy(golden[f"{n}.{key}"]).to(DEV)
            d = K.dequant_int4(p, s, group=group, packing=packing)
            np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), want, err_msg=f"{n} {packing}")


def test_golden_gpu_quantize_pack_bit_exact(golden):
    for n in _golden_cases(golden):
        group = int(golden[f"{n}.group"])
        w = torch.from_numpy(golden[f"{n}.w"]).to(DEV)
        for packing, key in (("interleaved", "inter"), ("simple", "simple")):
            if f"{n}.{key}" not in golden:
                continue
            for wt in (w.float(), w):  # fp32 and fp16 input give the same codes here
                p, s = K.quantize_pack(wt, group=group, packing=packing)
                np.testing.assert_array_equal(p.cpu().numpy(), golden[f"{n}.{key}"], err_msg=n)
                np.testing.assert_array_equal(s.cpu().numpy(), golden[f"{n}.s"], err_msg=n)


# ------------------------------------------------------- full-size configurations

def _weights(rows, cols, seed, outliers=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = torch.randn(rows, cols, device=DEV, generator=g) * 0.02
    if outliers:  # 0.1% of weights scaled x20
        n = rows * cols // 1000
        idx = torch.randint(0, rows * cols, (n,), device=DEV, generator=g)
        w.view(-1)[idx] *= 20.0
    w = w.half()
    x = torch.randn(cols, device=DEV, generator=g).half()
    return w, x


FULL = [
    (262144, 2048, 0, False), (262144, 2048, 128, False),
    (262144, 2048, 0, True), (262144, 2048, 128, True),
    (128256, 2048, 0, False), (128256, 2048, 128, False),
    (8192, 2048, 0, False), (8192, 2048, 128, False),
    (2048, 8192, 0, False), (2048, 8192, 128, False),
]


@pytest.mark.parametrize("rows,cols,group,outliers", FULL,
                         ids=[f"{r}x{c}-g{g}{'-outl' if o else ''}" for r, c, g, o in FULL])
def test_full_size_vs_oracle(rows, cols, group, outliers):
    w, x = _weights(rows, cols, seed=rows + cols + group, outliers=outliers)
    packed, scale = K.quantize_pack(w, group=group)
    # the GPU quantiser against the C oracle's (the reference's CPU semantics: true
    # fp32 division; torch on CUDA divides by the scalar 7 through a reciprocal, so the
    # reference quantiser run on a GPU tensor can differ from its CPU run in the last
    # bit of a scale)
    p_o, s_o = c_oracle.quantize_pack(w.float().cpu().numpy(), group=group)
    np.testing.assert_array_equal(packed.cpu().numpy(), p_o)
    np.testing.assert_array_equal(scale.cpu().numpy(), s_o)
    del p_o, s_o
    y = K.w4a16_gemv_g128(packed, scale, x) if group else K.w4a16_gemv(packed, scale, x)
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy(), group=group)
    assert_close(y.cpu().numpy(), ref, what=f"{rows}x{cols} g{group}")
    # the reference-named C entries without split-K give the same sums
    out = torch.empty_like(y)
    fn = K._lib.lib().w4a16_marlin_g128_cuda if group else K._lib.lib().w4a16_marlin_cuda
    st = fn(ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(scale.data_ptr()),
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), rows, cols,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    assert_close(out.cpu().numpy(), ref, what="C entry")


def test_split_k_deterministic_and_equal():
    w, x = _weights(2048, 8192, seed=7)
    packed, scale = K.quantize_pack(w, group=128)
    y1 = K.gemv(packed, scale, x, group=128)
    y2 = K.gemv(packed, scale, x, group=128)
    assert torch.equal(y1, y2), "split-K reduction is not deterministic"
    y0 = K.gemv(packed, scale, x, group=128, split_k=False)
    assert_close(y1.cpu(), y0.cpu().numpy(), atol=1e-5, rtol=1e-5, what="split vs no split")
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy(), group=128)
    assert_close(y1.cpu(), ref)


# ----------------------------------------------------------------- batch, dtypes

@pytest.mark.parametrize("batch", [1, 2, 3, 4, 8, 9, 16, 17, 33])
@pytest.mark.parametrize("group", [0, 128])
def test_batched_vs_oracle(batch, group):
    w, _ = _weights(3000, 2048, seed=batch * 3 + group)
    x = torch.randn(batch, 2048, device=DEV).half()
    packed, scale = K.quantize_pack(w, group=group)
    y = K.gemv(packed, scale, x, group=group)
    assert y.shape == (batch, 3000)
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy(), group=group)
    assert_close(y.cpu(), ref, what=f"batch {batch}")


@pytest.mark.parametrize("rows,batch,group,sdt", [(128256, 16, 128, torch.float32), (14208, 12, 0, torch.float32),
                                                  (20000, 16, 128, torch.float16), (128256, 4, 128, torch.float32)])
def test_batched_many_tiles_vs_oracle(rows, batch, group, sdt):
    # 9..16 activation rows on a matrix of many 32-row tiles take the wide geometry (6 warps,
    # 32-row tiles; 14208 rows is the smallest that does on 148 SMs), the ragged last tile
    # included (20000 = 625 x 32)
    w, _ = _weights(rows, 2048, seed=rows + batch)
    x = torch.randn(batch, 2048, device=DEV).half()
    packed, scale = K.quantize_pack(w, group=group, scale_dtype=sdt)
    del w
    y = K.gemv(packed, scale, x, group=group)
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.float().cpu().numpy(), x.cpu().numpy(), group=group)
    assert_close(y.cpu(), ref, what=f"{rows} rows, batch {batch}")


@pytest.mark.parametrize("rows,cols,group", [(4096, 14336, 128), (1000, 18432, 0), (3000, 12288, 128),
                                             (2048, 11264, 128)])
def test_long_rows_vs_oracle(rows, cols, group):
    # one activation vector too long to sit beside twelve warps' rings: staged beside nine
    # (Llama-3-8B's down projection is 4096 x 14336)
    w, x = _weights(rows, cols, seed=rows + cols)
    packed, scale = K.quantize_pack(w, group=group)
    y = K.gemv(packed, scale, x, group=group)
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy(), group=group)
    assert_close(y.cpu(), ref, what=f"{rows}x{cols}")


@pytest.mark.parametrize("group", [0, 128])
def test_fp16_scales_and_fp16_bias_epilogue(group):
    w, x = _weights(4100, 4096, seed=11)
    packed, scale = K.quantize_pack(w, group=group, scale_dtype=torch.float16)
    bias = torch.randn(4100, device=DEV) * 0.1
    y = K.gemv(packed, scale, x, group=group, bias=bias, out_dtype=torch.float16)
    assert y.dtype == torch.float16
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.float().cpu().numpy(), x.cpu().numpy(),
                        group=group) + bias.cpu().numpy()
    # fp16 output: add one fp16 rounding (2^-11 relative) to the tolerance
    assert_close(y.float().cpu(), ref, atol=ATOL, rtol=RTOL + 2 ** -11, what="fp16 out")


# ------------------------------------------------------------- edge shapes

EDGE = [(1, 256, 0), (17, 256, 0), (33, 512, 128), (5, 8, 0), (3, 24, 0), (7, 136, 0),
        (4, 128, 128), (19, 384, 128), (100, 768, 0), (1000, 11008, 0), (300, 14336, 128),
        (70, 16384, 0)]


@pytest.mark.parametrize("rows,cols,group", EDGE, ids=[f"{r}x{c}-g{g}" for r, c, g in EDGE])
@pytest.mark.parametrize("packing", ["interleaved", "simple"])
def test_edge_shapes(rows, cols, group, packing):
    w, x = _weights(rows, cols, seed=rows * 31 + cols)
    packed, scale = K.quantize_pack(w, group=group, packing=packing)
    y = K.gemv(packed, scale, x, group=group, packing=packing)
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy(), group=group,
                        interleaved=packing == "interleaved")
    assert_close(y.cpu(), ref, what=f"{rows}x{cols}")


def test_misaligned_weights_take_generic_path():
    w, x = _weights(64, 2048, seed=3)
    packed, scale = K.quantize_pack(w)
    buf = torch.empty(packed.numel() + 16, dtype=torch.uint8, device=DEV)
    view = buf[4:4 + packed.numel()].view(64, 1024)  # 4-byte aligned, not 16
    view.copy_(packed)
    y = K.gemv(view, scale, x)
    ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy())
    assert_close(y.cpu(), ref)


def test_empty_rows_is_noop():
    packed = torch.empty(0, 1024, dtype=torch.uint8, device=DEV)
    y = K.w4a16_gemv(packed, torch.empty(0, device=DEV), torch.randn(2048, device=DEV).half())
    assert y.shape == (0,)


def test_bad_inputs_raise():
    packed = torch.zeros(16, 128, dtype=torch.uint8, device=DEV)
    s = torch.ones(16, device=DEV)
    x = torch.randn(256, device=DEV).half()
    with pytest.raises(RuntimeError):
        K.w4a16_gemv(packed, s, x.float())           # fp32 activations
    with pytest.raises(RuntimeError):
        K.w4a16_gemv(packed.cpu(), s, x)             # CPU weights
    with pytest.raises(RuntimeError):
        K.w4a16_gemv(packed, s, x[:128])             # wrong length
    with pytest.raises(RuntimeError):
        K.w4a16_gemv(packed.float(), s, x)           # wrong packed dtype
    with pytest.raises(RuntimeError):
        K.w4a16_gemv_g128(packed, s, x)              # per-row scale to g128
    with pytest.raises(RuntimeError):
        K.matvec_byte(packed, s.half(), x)           # the ladder takes fp32 scales


# ------------------------------------------------------------- other kernels

def test_matvec_fp16_vs_fp32_reference():
    torch.manual_seed(0)
    mat = torch.randn(8192, 2048, device=DEV).half()
    vec = torch.randn(2048, device=DEV).half()
    out = K.matvec_fp16(mat, vec)
    ref = mat.float() @ vec.float()
    assert torch.allclose(out, ref, atol=1e-3, rtol=1e-4)


def test_dequant_full_size_vs_oracle():
    w, _ = _weights(8192, 2048, seed=5)
    for group in (0, 128):
        for sdt in (torch.float32, torch.float16):
            packed, scale = K.quantize_pack(w, group=group, scale_dtype=sdt)
            d = K.dequant_int4(packed, scale, group=group)
            q = O.unpack_int4(packed.cpu().numpy())
            want = O.dequant_f16(q, scale.float().cpu().numpy(), group)
            np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_no_device_error_recorded():
    assert K.read_device_error() == 0
