"""GPU parity of the tensor-core W4A16 GEMM (w4a16_gemm, many activation rows).

The GEMM's contract is y = x @ dequant_int4(packed, scale).T (+ bias) with fp32 sums: the
fp16 dequantised weight bit for bit (the reference's dequant formula,
src/w4a16/kernels.py:94-101) times the fp16 activations.  Checked against torch fp32 on
that weight (only the order of the fp32 sums differs) and against the float64 oracle on the
int4 codes (which adds the fp16 rounding of q * scale), at ragged and minimal shapes,
per-row and group-128 scales, fp32 and fp16 outputs, with a bias.
"""
import ctypes

import numpy as np
import pytest
import torch

import w4a16 as K
from w4a16 import _lib
from oracle import w4a16_oracle as O

pytestmark = pytest.mark.gpu

CASES = [  # M, N, K, group
    (128, 256, 1024, 0),
    (200, 1000, 2048, 128),
    (1, 384, 512, 0),
    (300, 128, 64, 0),
    (512, 4096, 4096, 128),
    (77, 130, 256, 128),
    (600, 16384, 512, 0),     # 256-row activation tiles (enough tiles for every SM), ragged M
    (1000, 9500, 1024, 128),  # 256-row tiles, ragged M and N
    (128, 4096, 4096, 128),   # split K: 32 tiles, 4 splits
    (96, 1000, 1024, 0),      # split K, ragged N, per-row scales
    (200, 640, 8192, 128),    # split K: 10 tiles, 8 splits
]


def _weights(n, k, group, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    return K.quantize_pack(w.half(), group=group)


def _device_error():
    code = ctypes.c_int(-1)
    assert _lib.lib().w4a16_read_device_error(ctypes.byref(code), None) == 0
    return code.value


@pytest.mark.parametrize("m,n,k,group", CASES, ids=lambda v: str(v))
def test_gemm_matches_dequantised_weight(m, n, k, group):
    p, s = _weights(n, k, group, m + n + k)
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(m, k, device="cuda", generator=g).half()
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    w16 = K.dequant_int4(p, s, group=group).float()
    ref = x.float() @ w16.t() + bias
    y = K.gemm(p, s, x, group=group, bias=bias)
    torch.cuda.synchronize()
    assert _device_error() == 0
    err = (y - ref).abs()
    bound = 1e-3 + 1e-3 * ref.abs()
    assert (err <= bound).all(), f"max abs err {err.max().item():.3e}"
    # fp32 sum order only: far inside the path's tolerance
    assert err.max().item() <= 1e-4 * max(1.0, ref.abs().max().item())
    y16 = K.gemm(p, s, x, group=group, bias=bias, out_dtype=torch.float16)
    assert y16.dtype == torch.float16
    assert ((y16.float() - ref).abs() <= 2e-3 + 2e-3 * ref.abs()).all()


def test_gemm_matches_oracle_codes():
    m, n, k, group = 96, 640, 1024, 128
    p, s = _weights(n, k, group, 3)
    x = torch.randn(m, k, device="cuda").half()
    y = K.gemm(p, s, x, group=group).cpu().numpy()
    q = O.unpack_int4(p.cpu().numpy())
    ref = O.gemv(q, s.cpu().numpy(), x.cpu().numpy(), group)
    err = np.abs(y - ref)
    assert (err <= 1e-3 + 1e-3 * np.abs(ref)).all(), err.max()


def test_gemm_repeated_calls_and_linear_layer():
    # W4A16Linear without a dense copy sends batches above 64 rows to the GEMM
    torch.manual_seed(4)
    lin = torch.nn.Linear(1024, 768, bias=True).half().cuda()
    model = torch.nn.Sequential(lin)
    K.replace_linear_with_w4a16(model, group=128, keep_dense=False)
    layer = model[0]
    x = torch.randn(2, 100, 1024, device="cuda").half()
    y1 = layer(x)
    y2 = layer(x)
    torch.cuda.synchronize()
    assert y1.shape == (2, 100, 768) and y1.dtype == torch.float16
    assert torch.equal(y1, y2)  # deterministic: no split of K across CTAs
    w16 = K.dequant_int4(layer.packed, layer.scale, group=128).float()
    ref = x.reshape(-1, 1024).float() @ w16.t() + layer.bias_f32
    assert ((y1.reshape(-1, 768).float() - ref).abs() <= 2e-3 + 2e-3 * ref.abs()).all()
    assert _device_error() == 0


@pytest.mark.parametrize("m,n,k", [(128, 4096, 4096), (200, 640, 8192)], ids=lambda v: str(v))
def test_gemm_split_k_is_deterministic_and_matches_unsplit(m, n, k):
    lib = _lib.lib()
    assert lib.w4a16_gemm_workspace_bytes(m, n, k) > 0  # these shapes split K
    p, s = _weights(n, k, 128, 11)
    x = torch.randn(m, k, device="cuda").half()
    ys = [K.gemm(p, s, x, group=128) for _ in range(3)]  # shared workspace, counters re-armed
    whole = K.gemm(p, s, x, group=128, workspace=False)
    torch.cuda.synchronize()
    assert _device_error() == 0
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])  # fixed summation order
    assert ((ys[0] - whole).abs() <= 1e-4 * (1.0 + whole.abs())).all()


@pytest.mark.parametrize("m,n,k", [(128, 4096, 4096), (640, 2048, 1024)], ids=lambda v: str(v))
def test_gemm_in_cuda_graph(m, n, k):
    # the first call sizes the workspace outside capture; replays re-arm the split counters
    p, s = _weights(n, k, 128, 21)
    x = torch.randn(m, k, device="cuda").half()
    want = K.gemm(p, s, x, group=128).clone()
    out = torch.empty(m, n, device="cuda")
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        K.gemm(p, s, x, group=128, out=out)
    torch.cuda.current_stream().wait_stream(st)
    with torch.cuda.graph(g):
        K.gemm(p, s, x, group=128, out=out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert _device_error() == 0
