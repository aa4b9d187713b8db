"""Decode-step kernels around the GEMV (GPU): the RMSNorm / SwiGLU prologues fused into
the GEMV, and the rotary + KV-cache write + attention kernel.

The prologues are checked against an fp32 restatement of the activation (numpy) fed to
the oracle GEMV; the activation is rounded to fp16 on both sides, so a difference can
only come from an fp16 rounding tie landing the other way (one ulp on a handful of
elements) and from the GEMV's summation order.  Attention is checked against an fp32
torch evaluation of rotate-half rotary, the cache update and softmax attention."""
import numpy as np
import pytest
import torch

import w4a16 as K
from oracle import c_oracle

pytestmark = pytest.mark.gpu


def _weights(rows, cols, group, seed, scale_dtype=torch.float32):
    torch.manual_seed(seed)
    w = torch.randn(rows, cols, device="cuda") * 0.02
    packed, scale = K.quantize_pack(w, group=group, scale_dtype=scale_dtype)
    return packed, scale, packed.cpu().numpy(), scale.float().cpu().numpy()


def _oracle(pk, s, x, group):
    return c_oracle.gemv(pk, s, x, group=group).astype(np.float64)


def _rmsnorm_np(h, gamma, eps):
    h = h.astype(np.float32)
    r = np.float32(1.0) / np.sqrt(np.mean(h * h, dtype=np.float32) + np.float32(eps), dtype=np.float32)
    return (h * r * gamma.astype(np.float32)).astype(np.float16)


def _swiglu_np(gu):
    k = gu.shape[0] // 2
    g, u = gu[:k].astype(np.float32), gu[k:].astype(np.float32)
    return (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float16)


def _close(got, ref, rel=2e-3):
    err = np.abs(got.astype(np.float64) - ref)
    tol = rel * np.abs(ref).max() + 1e-6
    assert (err <= tol).all(), (err.max(), tol)


@pytest.mark.parametrize("rows,cols,group", [(3072, 2048, 128), (16384, 2048, 128), (128256, 2048, 128),
                                             (300, 512, 0), (4096, 8192, 128)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_gemv_rmsnorm_matches_oracle(rows, cols, group, out_dtype):
    packed, scale, pk, s = _weights(rows, cols, group, seed=rows + cols)
    torch.manual_seed(7)
    h = torch.randn(cols, device="cuda") * 3.0
    gamma = torch.rand(cols, device="cuda") + 0.5
    y = K.gemv_rmsnorm(packed, scale, h, gamma, 1e-5, group=group, out_dtype=out_dtype)
    assert y.dtype == out_dtype and y.shape == (rows,)
    x = _rmsnorm_np(h.cpu().numpy(), gamma.cpu().numpy(), 1e-5)
    ref = _oracle(pk, s, x, group)
    _close(y.float().cpu().numpy(), ref, rel=2e-3 if out_dtype == torch.float32 else 4e-3)


@pytest.mark.parametrize("rows,cols,group", [(16384, 2048, 128), (3072, 2048, 128), (512, 256, 0),
                                             (57344, 4096, 128)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_gemv_rmsnorm_swiglu_out_matches_oracle(rows, cols, group, out_dtype):
    """Gate|up projection with the SwiGLU epilogue: rows 16b..16b+7 are gate rows and
    16b+8..16b+15 their up rows; out[8b+i] = silu(y[16b+i]) * y[16b+8+i] of the oracle
    GEMV's sums (decode-step gate/up with CTA-local reduction, a small per-row matrix, and
    Llama-3-8B's 2 x 14336 rows on whole-tile schedules)."""
    packed, scale, pk, s = _weights(rows, cols, group, seed=5 * rows + cols)
    torch.manual_seed(9)
    h = torch.randn(cols, device="cuda") * 3.0
    gamma = torch.rand(cols, device="cuda") + 0.5
    y = K.gemv_rmsnorm(packed, scale, h, gamma, 1e-5, group=group, out_dtype=out_dtype, swiglu_out=True)
    assert y.dtype == out_dtype and y.shape == (rows // 2,)
    full = _oracle(pk, s, _rmsnorm_np(h.cpu().numpy(), gamma.cpu().numpy(), 1e-5), group).reshape(-1, 2, 8)
    g, u = full[:, 0].reshape(-1), full[:, 1].reshape(-1)
    ref = g / (1.0 + np.exp(-g)) * u
    _close(y.float().cpu().numpy(), ref, rel=2e-3 if out_dtype == torch.float32 else 4e-3)
    with pytest.raises(RuntimeError):
        K.gemv_rmsnorm(packed, scale, h, gamma, 1e-5, group=group, bias=torch.zeros(rows, device="cuda"),
                       swiglu_out=True)


@pytest.mark.parametrize("rows,cols,group", [(2048, 8192, 128), (2048, 2048, 0), (512, 10752, 128)])  # 10752: the longest group-128 vector that fits
def test_gemv_swiglu_matches_oracle(rows, cols, group):
    packed, scale, pk, s = _weights(rows, cols, group, seed=3 * rows + cols)
    torch.manual_seed(8)
    gu = (torch.randn(2 * cols, device="cuda") * 2.0).half()
    y = K.gemv_swiglu(packed, scale, gu, group=group)
    ref = _oracle(pk, s, _swiglu_np(gu.cpu().numpy()), group)
    _close(y.cpu().numpy(), ref)


@pytest.mark.parametrize("split_k", [True, False])
def test_fused_in_place_residual(split_k):
    # h += W_down swiglu(gu) with out aliasing bias, as the decode step does
    rows, cols = 2048, 8192
    packed, scale, pk, s = _weights(rows, cols, 128, seed=11)
    torch.manual_seed(9)
    gu = torch.randn(2 * cols, device="cuda").half()
    h = torch.randn(rows, device="cuda")
    h0 = h.cpu().numpy().astype(np.float64)
    out = K.gemv_swiglu(packed, scale, gu, group=128, bias=h, out=h, split_k=split_k)
    assert out.data_ptr() == h.data_ptr()
    ref = h0 + _oracle(pk, s, _swiglu_np(gu.cpu().numpy()), 128)
    _close(h.cpu().numpy(), ref)
    # RMSNorm prologue with an in-place residual on a different vector
    packed2, scale2, pk2, s2 = _weights(cols, rows, 128, seed=12)
    acc = torch.randn(cols, device="cuda")
    acc0 = acc.cpu().numpy().astype(np.float64)
    gamma = torch.ones(rows, device="cuda")
    K.gemv_rmsnorm(packed2, scale2, h, gamma, group=128, bias=acc, out=acc, split_k=split_k)
    ref2 = acc0 + _oracle(pk2, s2, _rmsnorm_np(h.cpu().numpy(), gamma.cpu().numpy(), 1e-5), 128)
    _close(acc.cpu().numpy(), ref2)


def test_fused_fp16_scales_and_determinism():
    packed, scale, pk, s = _weights(8192, 2048, 128, seed=13, scale_dtype=torch.float16)
    h = torch.randn(2048, device="cuda")
    gamma = torch.rand(2048, device="cuda")
    a = K.gemv_rmsnorm(packed, scale, h, gamma, group=128)
    b = K.gemv_rmsnorm(packed, scale, h, gamma, group=128)
    assert torch.equal(a, b)
    _close(a.cpu().numpy(), _oracle(pk, s, _rmsnorm_np(h.cpu().numpy(), gamma.cpu().numpy(), 1e-5), 128))


def test_fused_rejects_unsupported_shapes():
    packed, scale, _, _ = _weights(64, 384, 128, seed=14)         # cols % 256 != 0
    with pytest.raises(RuntimeError, match="256"):
        K.gemv_rmsnorm(packed, scale, torch.randn(384, device="cuda"), torch.ones(384, device="cuda"),
                       group=128)
    packed, scale, _, _ = _weights(16, 131072, 128, seed=15)      # vector too long for shared memory
    with pytest.raises(RuntimeError, match="cols <="):
        K.gemv_swiglu(packed, scale, torch.randn(2 * 131072, device="cuda").half(), group=128)
    packed, scale, _, _ = _weights(256, 256, 128, seed=16)
    src = torch.randn(512, device="cuda")
    with pytest.raises(RuntimeError, match="overlaps"):           # out overlaps the source vector
        K.gemv_rmsnorm(packed, scale, src[:256], torch.ones(256, device="cuda"), group=128, out=src[128:384])


# --------------------------------------------------------------------- attention

def _rope_tables(max_len, theta=500000.0, D=64):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device="cuda").float() / D))
    ang = torch.arange(max_len, device="cuda").float()[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.cos()], 1).contiguous(), torch.cat([ang.sin(), ang.sin()], 1).contiguous()


def _attention_ref(qkv, cos, sin, pos, kc, vc, heads, kv_heads):
    D = 64
    x = qkv.float()
    q = x[: heads * D].view(heads, D)
    k = x[heads * D:(heads + kv_heads) * D].view(kv_heads, D)
    v = x[(heads + kv_heads) * D:].view(kv_heads, D)

    def rope(t):
        rot = torch.cat([-t[:, D // 2:], t[:, : D // 2]], 1)
        return t * cos[pos] + rot * sin[pos]

    q, k = rope(q), rope(k)
    kc, vc = kc.float().clone(), vc.float().clone()
    kc[:, pos] = k.half().float()
    vc[:, pos] = v
    rep = heads // kv_heads
    keys = kc[:, : pos + 1].repeat_interleave(rep, 0)
    vals = vc[:, : pos + 1].repeat_interleave(rep, 0)
    p = torch.softmax((keys @ q.unsqueeze(-1)).squeeze(-1) / 8.0, -1)
    return (p.unsqueeze(1) @ vals).reshape(-1), k.half()


@pytest.mark.parametrize("heads,kv_heads,max_len,pos,splits", [
    (32, 8, 512, 511, None), (32, 8, 512, 0, None), (32, 8, 512, 200, 1), (32, 8, 128, 63, 128),
    (8, 8, 256, 100, 3), (4, 1, 96, 95, 5), (32, 1, 64, 40, 2), (32, 8, 4096, 3000, None),
    # one CTA per kv head (splits 1, cache <= 512, 1/2/4/8 query heads per kv head)
    (8, 1, 512, 300, 1), (16, 8, 384, 383, 1), (8, 8, 64, 10, 1), (32, 8, 512, 33, 1)])
def test_decode_attention_matches_fp32_reference(heads, kv_heads, max_len, pos, splits):
    torch.manual_seed(heads + max_len + pos)
    qkv = torch.randn((heads + 2 * kv_heads) * 64, device="cuda").half()
    kc = torch.randn(kv_heads, max_len, 64, device="cuda").half()
    vc = torch.randn(kv_heads, max_len, 64, device="cuda").half()
    kc0, vc0 = kc.clone(), vc.clone()
    cos, sin = _rope_tables(max_len)
    p = torch.tensor([pos], device="cuda")
    ref, k_new = _attention_ref(qkv, cos, sin, pos, kc0, vc0, heads, kv_heads)
    out = K.decode_attention(qkv, cos, sin, p, kc, vc, heads=heads, kv_heads=kv_heads, splits=splits)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out.shape == (heads * 64,)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-3 + 1e-2 * ref.abs().max().item(), err
    # the cache changed at pos only: v exactly, k up to one fp16 ulp (rounding of the rotation)
    v_new = qkv[(heads + kv_heads) * 64:].view(kv_heads, 64)
    assert torch.equal(vc[:, pos], v_new)
    assert ((kc[:, pos].float() - k_new.float()).abs() <= 1e-3 * k_new.float().abs() + 1e-7).all()
    keep = torch.ones(max_len, dtype=torch.bool, device="cuda")
    keep[pos] = False
    assert torch.equal(kc[:, keep], kc0[:, keep]) and torch.equal(vc[:, keep], vc0[:, keep])


def test_decode_attention_repeatable_and_scratch_left_zeroed():
    heads, kv_heads, max_len = 32, 8, 512
    qkv = torch.randn((heads + 2 * kv_heads) * 64, device="cuda").half()
    kc = torch.randn(kv_heads, max_len, 64, device="cuda").half()
    vc = torch.randn_like(kc)
    cos, sin = _rope_tables(max_len)
    p = torch.tensor([300], device="cuda")
    a = K.decode_attention(qkv, cos, sin, p, kc, vc, heads=heads, kv_heads=kv_heads, splits=1).clone()
    b = K.decode_attention(qkv, cos, sin, p, kc, vc, heads=heads, kv_heads=kv_heads, splits=1).clone()
    assert torch.equal(a, b)
    b = K.decode_attention(qkv, cos, sin, p, kc, vc, heads=heads, kv_heads=kv_heads, splits=16).clone()
    c = K.decode_attention(qkv, cos, sin, p, kc, vc, heads=heads, kv_heads=kv_heads, splits=16).clone()
    assert torch.equal(b, c)                                      # split path: repeatable too
    assert (a.float() - b.float()).abs().max().item() < 2e-3      # and equal to the one-CTA path
    scratch = K.kernels._ATTN_SCRATCH[(0, heads, kv_heads, 16)]
    assert int(scratch[-kv_heads * 4:].count_nonzero()) == 0   # per-kv-head counters back at zero


def test_decode_attention_position_out_of_range():
    heads, kv_heads, max_len = 8, 2, 64
    qkv = torch.randn((heads + 2 * kv_heads) * 64, device="cuda").half()
    kc = torch.randn(kv_heads, max_len, 64, device="cuda").half()
    vc = torch.randn_like(kc)
    kc0, vc0 = kc.clone(), vc.clone()
    cos, sin = _rope_tables(max_len)
    for bad in (max_len, -1):
        for splits in (4, 1):  # the split kernel and the one-CTA kernel
            out = K.decode_attention(qkv, cos, sin, torch.tensor([bad], device="cuda"), kc, vc,
                                     heads=heads, kv_heads=kv_heads, splits=splits)
            torch.cuda.synchronize()
            assert torch.isnan(out).all()
            assert torch.equal(kc, kc0) and torch.equal(vc, vc0)
    good = K.decode_attention(qkv, cos, sin, torch.tensor([10], device="cuda"), kc, vc,
                              heads=heads, kv_heads=kv_heads, splits=4)
    assert torch.isfinite(good).all()


# ------------------------------------------------------------ chained launches

# (2048, 2048) and (1000, 1536): two windows per CTA, so 4 warps share each window (slabs
# split between them; 1536 columns leave two parts of the second window empty);
# (3000, 4096): 4-8 windows per CTA and a partial last tile
@pytest.mark.parametrize("rows,cols", [(2048, 2048), (3000, 4096), (1000, 1536), (64, 512)])
def test_gemv_staged_matches_oracle(rows, cols):
    packed, scale, pk, s = _weights(rows, cols, 128, seed=rows + 5)
    x = torch.randn(cols, device="cuda").half()
    bias = torch.randn(rows, device="cuda")
    y = K.gemv_staged(packed, scale, x, group=128, bias=bias)
    _close(y.cpu().numpy(), _oracle(pk, s, x.cpu().numpy(), 128) + bias.cpu().numpy().astype(np.float64))


def _chain(layers, h, gu_buf, attn_x, pdl, ws):
    """A residual chain like the decode step: h += Wo x; gu = Wgu rmsnorm(h); h += Wd swiglu(gu)."""
    for (po, so), (pg, sg), (pd, sd), gamma in layers:
        K.gemv_staged(po, so, attn_x, group=128, bias=h, out=h, pdl=pdl, workspace=ws[1])
        K.gemv_rmsnorm(pg, sg, h, gamma, group=128, out=gu_buf, pdl=pdl, workspace=ws[0])
        K.gemv_swiglu(pd, sd, gu_buf, group=128, bias=h, out=h, pdl=pdl, workspace=ws[1])
        attn_x = gu_buf[: attn_x.numel()]
    return h


def test_pdl_chain_equals_plain_chain_eager_and_graph():
    H, I = 2048, 4096
    layers = []
    for i in range(3):
        po, so, _, _ = _weights(H, H, 128, seed=100 + i)
        pg, sg, _, _ = _weights(2 * I, H, 128, seed=200 + i)
        pd, sd, _, _ = _weights(H, I, 128, seed=300 + i)
        layers.append(((po, so), (pg, sg), (pd, sd), torch.rand(H, device="cuda") + 0.5))
    torch.manual_seed(5)
    h0 = torch.randn(H, device="cuda")
    x0 = torch.randn(H, device="cuda").half()
    ws = [K.new_workspace("cuda"), K.new_workspace("cuda")]
    outs = {}
    for pdl in (False, True):
        h = h0.clone()
        gu = torch.empty(2 * I, dtype=torch.float16, device="cuda")
        outs[pdl] = _chain(layers, h, gu, x0.clone(), pdl, ws).clone()
    torch.cuda.synchronize()
    assert torch.equal(outs[False], outs[True])
    # captured in a graph and replayed: the same result each time, workspaces left zeroed
    h = h0.clone()
    gu = torch.empty(2 * I, dtype=torch.float16, device="cuda")
    x = x0.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _chain(layers, h, gu, x, True, ws)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _chain(layers, h, gu, x, True, ws)
    for _ in range(3):
        h.copy_(h0)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(h, outs[True])
    # the counter block at the start of each workspace is back at zero (the partial
    # sums behind it are scratch)
    assert all(int(w[:16384].count_nonzero()) == 0 for w in ws)
    assert K.read_device_error() == 0
