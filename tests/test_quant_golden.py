"""The package's quantisers, packers and fp32 helpers against the reference's outputs
(bit for bit), on CPU.  These are the host-side half of the drop-in surface."""
import numpy as np
import pytest
import torch

import w4a16 as K


def _cases(golden, group=None):
    names = [str(n) for n in golden["cases"]]
    return [n for n in names if group is None or int(golden[f"{n}.group"]) == group]


def test_exports_match_reference_names():
    ref_names = [
        "matvec_byte", "matvec_u32", "matvec_u32_v4", "matvec_champ",
        "matvec_uint4", "matvec_h2f32", "w4a16_gemv", "w4a16_gemv_g128", "matvec_fp16",
        "quantize_int4_symmetric", "quantize_int4_group", "pack_int4", "pack_int4_interleaved",
        "dequant_ref", "dequant_ref_group", "W4A16Linear", "replace_linear_with_w4a16",
    ]
    for n in ref_names:
        assert hasattr(K, n), n
        assert n in K.__all__
    from w4a16 import kernels
    for n in ref_names:  # `from w4a16.kernels import X` works as in the reference
        assert hasattr(kernels, n) or n in ("W4A16Linear", "replace_linear_with_w4a16")


def test_known_answer(golden):
    q = torch.from_numpy(golden["known_q"])
    assert K.pack_int4_interleaved(q)[0].tolist() == [0x64, 0xA8, 0x75, 0xB9]
    assert K.pack_int4(q)[0].tolist() == [0x45, 0x67, 0x89, 0xAB]


@pytest.mark.parametrize("group", [0, 128])
def test_quantizers_bit_exact(golden, group):
    for n in _cases(golden, group):
        w = torch.from_numpy(golden[f"{n}.w"]).float()
        q, s = K.quantize_int4_group(w, group=group) if group else K.quantize_int4_symmetric(w)
        assert q.dtype == torch.int8
        np.testing.assert_array_equal(q.numpy(), golden[f"{n}.q"], err_msg=n)
        np.testing.assert_array_equal(s.numpy(), golden[f"{n}.s"], err_msg=n)


def test_packers_bit_exact_and_roundtrip(golden):
    for n in _cases(golden):
        q = torch.from_numpy(golden[f"{n}.q"])
        ps = K.pack_int4(q)
        assert ps.dtype == torch.uint8 and ps.shape == (q.shape[0], q.shape[1] // 2)
        np.testing.assert_array_equal(ps.numpy(), golden[f"{n}.simple"], err_msg=n)
        assert torch.equal(K.unpack_int4(ps, interleaved=False), q)
        if f"{n}.inter" in golden:
            pi = K.pack_int4_interleaved(q)
            np.testing.assert_array_equal(pi.numpy(), golden[f"{n}.inter"], err_msg=n)
            assert torch.equal(K.unpack_int4(pi), q)


def test_pack_roundtrip_all_codes():
    # every code value in every column position, both packings (the reference's
    # tests/test_kernels.py:122-133 only checked dtype and shape)
    q = torch.arange(-8, 8, dtype=torch.int8).repeat(16, 1)
    q = torch.stack([q.roll(i, dims=1) for i in range(8)]).reshape(-1, 16)
    for interleaved in (True, False):
        p = K.pack_int4_interleaved(q) if interleaved else K.pack_int4(q)
        assert torch.equal(K.unpack_int4(p, interleaved=interleaved), q)


def test_interleaved_requires_cols_multiple_of_8():
    with pytest.raises(AssertionError):
        K.pack_int4_interleaved(torch.zeros(2, 12, dtype=torch.int8))
    with pytest.raises(AssertionError):
        K.quantize_int4_group(torch.zeros(2, 96), group=128)


def test_dequant_ref_matches_reference(golden):
    for n in _cases(golden):
        group = int(golden[f"{n}.group"])
        q = torch.from_numpy(golden[f"{n}.q"])
        s = torch.from_numpy(golden[f"{n}.s"])
        x = torch.from_numpy(golden[f"{n}.x"])
        y = K.dequant_ref_group(q, s, x, group=group) if group else K.dequant_ref(q, s, x)
        np.testing.assert_allclose(y.numpy(), golden[f"{n}.y"], rtol=1e-6, atol=1e-6, err_msg=n)


def test_quant_error_regression():
    # reference tests/test_kernels.py:136-144 (CPU here): per-row int4 on N(0,1)
    torch.manual_seed(0)
    w = torch.randn(4096, 4096)
    q, scale = K.quantize_int4_symmetric(w)
    frob = (torch.norm(w - q.float() * scale[:, None]) / torch.norm(w)).item()
    assert 0.10 < frob < 0.20


def test_zero_row_gets_zero_codes():
    w = torch.zeros(3, 256)
    w[1] = torch.linspace(-1, 1, 256)
    q, s = K.quantize_int4_symmetric(w)
    assert s[0] == 0 and s[2] == 0 and (q[0] == 0).all() and (q[2] == 0).all()
    qg, sg = K.quantize_int4_group(w)
    assert (sg[0] == 0).all() and (qg[0] == 0).all()
