"""W4A16Linear and replace_linear_with_w4a16 (reference src/w4a16/kernels.py:105-137).

CPU: the swap bookkeeping (which modules, buffers, shapes) on a small random Llama.
GPU: forward parity of the swapped layers against the oracle, the reference's
113-Linear swap count on a random-init Llama-3.2-1B-architecture model, and the
batch paths (kernel for <= 64 rows, dense or dequantised fallback above)."""
import copy

import numpy as np
import pytest
import torch
import torch.nn as nn

import w4a16 as K
from oracle import w4a16_oracle as O

LLAMA_1B = dict(hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                num_attention_heads=32, num_key_value_heads=8, head_dim=64, vocab_size=128256,
                tie_word_embeddings=True, max_position_embeddings=4096)


def _llama(**kw):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    return LlamaForCausalLM(LlamaConfig(**kw))


def test_swap_structure_on_cpu_model():
    model = nn.Sequential(nn.Linear(64, 32), nn.ReLU(), nn.Sequential(nn.Linear(32, 16, bias=False)))
    ref_w = model[0].weight.data.clone()
    n_before = sum(isinstance(m, nn.Linear) for m in model.modules())
    K.replace_linear_with_w4a16(model, device="cpu")
    swapped = [m for m in model.modules() if isinstance(m, K.W4A16Linear)]
    assert len(swapped) == n_before == 2
    assert not any(isinstance(m, nn.Linear) for m in model.modules())
    first = swapped[0]
    assert first.packed.shape == (32, 32) and first.packed.dtype == torch.uint8
    assert first.scale.shape == (32,) and first.scale.dtype == torch.float32
    assert first.dense_weight.dtype == torch.float16 and first.group == 0
    assert first.in_features == 64 and first.out_features == 32
    q, s = K.quantize_int4_symmetric(ref_w.float())
    assert torch.equal(first.packed, K.pack_int4_interleaved(q)) and torch.equal(first.scale, s)
    assert swapped[1].bias is None and swapped[0].bias_f32.dtype == torch.float32
    g = nn.Sequential(nn.Linear(256, 8))
    K.replace_linear_with_w4a16(g, group=128, keep_dense=False, device="cpu")
    assert g[0].scale.shape == (8, 2) and g[0].dense_weight is None and g[0].group == 128
    assert set(g.state_dict()) == {"0.packed", "0.scale", "0.bias"}


def test_llama_small_swap_count_cpu():
    model = _llama(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                   num_key_value_heads=2, head_dim=16, vocab_size=256, tie_word_embeddings=True)
    n_before = sum(isinstance(m, nn.Linear) for m in model.modules())
    K.replace_linear_with_w4a16(model, device="cpu")
    assert sum(isinstance(m, K.W4A16Linear) for m in model.modules()) == n_before == 2 * 7 + 1


@pytest.mark.gpu
def test_swap_count_llama_3_2_1b_architecture():
    # reference tests/test_kernels.py:147-164 (needs the real checkpoint there)
    model = _llama(**LLAMA_1B).half().cuda().eval()
    n_before = sum(isinstance(m, nn.Linear) for m in model.modules())
    K.replace_linear_with_w4a16(model, group=128, keep_dense=False)
    n_swapped = sum(isinstance(m, K.W4A16Linear) for m in model.modules())
    n_after = sum(isinstance(m, nn.Linear) for m in model.modules())
    assert n_swapped == 113 and n_swapped == n_before and n_after == 0
    with torch.no_grad():
        out = model(torch.tensor([[1, 2, 3]], device="cuda"), use_cache=False)
    assert torch.isfinite(out.logits).all()


@pytest.mark.gpu
@pytest.mark.parametrize("group,keep_dense", [(0, True), (128, False)])
@pytest.mark.parametrize("batch", [1, 4, 16, 80])
def test_linear_forward_matches_oracle(group, keep_dense, batch):
    torch.manual_seed(1)
    lin = nn.Linear(1024, 3000, bias=True).half().cuda()
    model = nn.Sequential(lin)
    K.replace_linear_with_w4a16(model, group=group, keep_dense=keep_dense)
    layer = model[0]
    x = torch.randn(batch, 1024, device="cuda").half()
    y = layer(x).detach()
    assert y.shape == (batch, 3000) and y.dtype == torch.float16
    q = O.unpack_int4(layer.packed.cpu().numpy())
    ref = O.gemv(q, layer.scale.float().cpu().numpy(), x.cpu().numpy(), group) + lin.bias.detach().float().cpu().numpy()
    if batch > 64 and keep_dense:
        # the reference's prefill fallback multiplies by the dense fp16 weight
        ref = (x.float() @ lin.weight.detach().float().t() + lin.bias.detach().float()).cpu().numpy()
        tol = 2e-2
    else:
        tol = 2e-3
    err = np.abs(y.float().cpu().numpy() - ref)
    assert (err <= tol + 2e-3 * np.abs(ref)).all(), err.max()


@pytest.mark.gpu
def test_linear_three_dim_input_and_bf16():
    torch.manual_seed(2)
    lin = nn.Linear(512, 256, bias=False).cuda().to(torch.bfloat16)
    model = nn.Sequential(lin)
    K.replace_linear_with_w4a16(model, group=128, keep_dense=False)
    x = torch.randn(2, 3, 512, device="cuda", dtype=torch.bfloat16)
    y = model(x).detach()
    assert y.shape == (2, 3, 256) and y.dtype == torch.bfloat16
    layer = model[0]
    q = O.unpack_int4(layer.packed.cpu().numpy())
    ref = O.gemv(q, layer.scale.cpu().numpy(), x.reshape(6, 512).half().cpu().numpy(), 128)
    assert np.abs(y.reshape(6, 256).float().cpu().numpy() - ref).max() < 3e-2  # bf16 output rounding


@pytest.mark.gpu
@pytest.mark.parametrize("group,scale_dtype", [(0, torch.float32), (128, torch.float32), (128, torch.float16)])
def test_gpu_quantizer_swap_is_bit_identical(group, scale_dtype):
    # replace_linear_with_w4a16(quantizer="gpu") quantises and packs in one launch per layer
    # against the torch quantiser on the host (the reference's path; torch's CUDA division
    # is not always correctly rounded, the kernel's is)
    torch.manual_seed(4)
    base = nn.Sequential(nn.Linear(2048, 3072), nn.Sequential(nn.Linear(3072, 256, bias=False))).half()
    a = copy.deepcopy(base)          # weights on the CPU: torch quantises there, buffers go to cuda
    b = copy.deepcopy(base).cuda()
    K.replace_linear_with_w4a16(a, group=group, keep_dense=False, scale_dtype=scale_dtype, device="cuda")
    K.replace_linear_with_w4a16(b, group=group, keep_dense=False, scale_dtype=scale_dtype, quantizer="gpu")
    for la, lb in ((a[0], b[0]), (a[1][0], b[1][0])):
        assert torch.equal(la.packed, lb.packed)
        assert la.scale.dtype == lb.scale.dtype == scale_dtype and torch.equal(la.scale, lb.scale)
