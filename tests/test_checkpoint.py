"""Quantised checkpoints (w4a16/checkpoint.py) on CPU: a swapped model saved as packed codes,
scales and biases loads into a freshly initialised model of the same architecture without
quantising again, and the loaded layers and the rest of the state equal the saved ones."""
import pytest
import torch
import torch.nn as nn

import w4a16 as K


def _toy(seed, width=64):
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(256, width), nn.LayerNorm(width),
                         nn.Sequential(nn.Linear(width, 32, bias=False)))


def _layers(model):
    return {n: m for n, m in model.named_modules() if isinstance(m, K.W4A16Linear)}


@pytest.mark.parametrize("group", [0, 128])
def test_roundtrip_toy_model(tmp_path, group):
    width = 128 if group else 64  # group-128 needs in_features % 128 == 0
    src = _toy(0, width)
    with torch.no_grad():  # a LayerNorm that differs from a fresh one
        src[1].weight.normal_()
        src[1].bias.normal_()
    K.replace_linear_with_w4a16(src, group=group, keep_dense=False, device="cpu")
    path = tmp_path / "q.pt"
    K.save_quantized(src, path)
    dst = K.load_quantized(_toy(1, width), path, device="cpu")
    a, b = _layers(src), _layers(dst)
    assert set(a) == set(b) == {"0", "2.0"}
    for n in a:
        assert torch.equal(a[n].packed, b[n].packed) and torch.equal(a[n].scale, b[n].scale)
        assert a[n].group == b[n].group and b[n].dense_weight is None
        assert (a[n].bias is None) == (b[n].bias is None)
        if a[n].bias is not None:
            assert torch.equal(a[n].bias, b[n].bias) and torch.equal(b[n].bias_f32, a[n].bias_f32)
    # the LayerNorm came from the checkpoint, not from the fresh initialisation
    assert torch.equal(dst[1].weight, src[1].weight) and torch.equal(dst[1].bias, src[1].bias)
    # nothing dense was written: the file holds the packed codes, scales and small state
    assert path.stat().st_size < 256 * width * 2


def test_roundtrip_small_llama(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=32, vocab_size=512, tie_word_embeddings=True)
    torch.manual_seed(0)
    src = LlamaForCausalLM(cfg)
    K.replace_linear_with_w4a16(src, group=128, keep_dense=False, device="cpu")
    path = tmp_path / "llama.pt"
    K.save_quantized(src, path)
    torch.manual_seed(1)
    dst = K.load_quantized(LlamaForCausalLM(cfg), path, device="cpu")
    a, b = _layers(src), _layers(dst)
    assert len(a) == len(b) == 2 * 7 + 1
    for n in a:
        assert torch.equal(a[n].packed, b[n].packed) and torch.equal(a[n].scale, b[n].scale)
    sa, sb = src.state_dict(), dst.state_dict()
    for k in ("model.embed_tokens.weight", "model.norm.weight", "model.layers.1.input_layernorm.weight"):
        assert torch.equal(sa[k], sb[k])


def test_rejects_mismatches(tmp_path):
    src = _toy(0)
    K.replace_linear_with_w4a16(src, keep_dense=False, device="cpu")
    path = tmp_path / "q.pt"
    K.save_quantized(src, path)
    other = nn.Sequential(nn.Linear(256, 48), nn.LayerNorm(48), nn.Sequential(nn.Linear(48, 32, bias=False)))
    with pytest.raises(ValueError, match="does not match"):
        K.load_quantized(other, path, device="cpu")
    with pytest.raises(KeyError, match="not a Linear"):
        K.load_quantized(nn.Sequential(nn.LayerNorm(64)), path, device="cpu")
    with pytest.raises(ValueError, match="no W4A16Linear"):
        K.save_quantized(_toy(2), tmp_path / "plain.pt")
    torch.save({"format": "other"}, tmp_path / "bad.pt")
    with pytest.raises(ValueError, match="checkpoint"):
        K.load_quantized(_toy(3), tmp_path / "bad.pt", device="cpu")


@pytest.mark.gpu
def test_loaded_model_gives_the_same_logits_on_gpu(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=1024, tie_word_embeddings=True)
    torch.manual_seed(0)
    src = LlamaForCausalLM(cfg).half().cuda().eval()
    K.replace_linear_with_w4a16(src, group=128, keep_dense=False, quantizer="gpu")
    path = tmp_path / "llama.pt"
    K.save_quantized(src, path)
    torch.manual_seed(1)
    dst = K.load_quantized(LlamaForCausalLM(cfg).half().cuda().eval(), path)
    ids = torch.tensor([[3, 14, 15, 92]], device="cuda")
    with torch.no_grad():
        la = src(ids, use_cache=False).logits
        lb = dst(ids, use_cache=False).logits
    assert torch.isfinite(la).all() and torch.equal(la, lb)
