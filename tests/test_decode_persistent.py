"""The one-kernel decode step (w4a16_decode_step through DecodePlan) on the GPU.

The persistent kernel runs the same arithmetic as the step built from separate fused
kernels (fp16 activations into exact int4 x fp16 products, fp32 group sums, fp32 residual
and softmax), so its logits must agree with that step and with the fp32 torch evaluation
from the dequantised weights; the cache rows it writes must match too."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg(layers=2, vocab=4096, max_len=128):
    from w4a16.decode import LlamaDecodeConfig

    return LlamaDecodeConfig(layers=layers, vocab=vocab, max_len=max_len)


def _pair(cfg, seed, fill):
    """The same random model as a fused-kernel step and as a persistent step."""
    from w4a16.decode import W4A16LlamaDecoder

    fused = W4A16LlamaDecoder(cfg, seed=seed, fused=True)
    pers = W4A16LlamaDecoder(cfg, seed=seed, persistent=True)
    fused.fill_cache(fill)
    pers.fill_cache(fill)
    return fused, pers


@pytest.mark.parametrize("pos", [0, 1, 31, 32, 63, 127])
def test_persistent_step_matches_fused_step_and_fp32(pos):
    import w4a16 as K

    fused, pers = _pair(_cfg(), seed=3, fill=pos)
    ref = pers.reference_logits(token=17, pos=pos)
    a = fused.step(token=17, pos=pos).clone()
    b = pers.step(token=17, pos=pos).clone()
    torch.cuda.synchronize()
    scale = ref.abs().max().item()
    assert (b - a).abs().max().item() <= 1e-3 * scale, (b - a).abs().max().item()
    assert (b - ref).abs().max().item() <= 2e-2 * scale
    # the rotated key and the value written at pos (fp16: the two steps sum the QKV GEMV's
    # windows in a different order, so a value may round to the neighbouring fp16)
    for pc, fc in ((pers.k_cache, fused.k_cache), (pers.v_cache, fused.v_cache)):
        assert torch.allclose(pc[:, :, pos].float(), fc[:, :, pos].float(), atol=2e-3, rtol=2e-3)
        assert torch.equal(pc[:, :, :pos], fc[:, :, :pos])   # the rows before pos are untouched
    assert K.read_device_error() == 0


def test_persistent_graph_replay_and_generation():
    from w4a16.decode import W4A16LlamaDecoder

    cfg = _cfg()
    dec = W4A16LlamaDecoder(cfg, seed=4, persistent=True)
    dec.fill_cache(40)
    k0, v0 = dec.k_cache.clone(), dec.v_cache.clone()
    eager = dec.step(token=5, pos=40).clone()
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    dec.capture()
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    replay = dec.replay(token=5, pos=40).clone()
    torch.cuda.synchronize()
    assert torch.equal(replay, eager)
    # greedy generation by graph replays equals the same steps launched one by one
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    toks = dec.generate(token=11, pos=20, n=10)
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    want, t = [], 11
    for i in range(10):
        t = int(dec.step(token=t, pos=20 + i).argmax())
        want.append(t)
    assert toks.tolist() == want


def test_persistent_step_bad_position_or_token_gives_nan_and_no_cache_write():
    import w4a16 as K
    from w4a16.decode import W4A16LlamaDecoder

    cfg = _cfg()
    dec = W4A16LlamaDecoder(cfg, seed=5, persistent=True)
    dec.fill_cache(cfg.max_len)
    k0, v0 = dec.k_cache.clone(), dec.v_cache.clone()
    for token, pos in ((3, cfg.max_len), (3, -1), (cfg.vocab, 10), (-2, 10)):
        out = dec.step(token=token, pos=pos)
        torch.cuda.synchronize()
        assert torch.isnan(out).all(), (token, pos)
        assert torch.equal(dec.k_cache, k0) and torch.equal(dec.v_cache, v0)
    assert torch.isfinite(dec.step(token=3, pos=10)).all()   # the plan still works
    assert K.read_device_error() == 0


def test_persistent_full_size_step_matches_fused():
    import w4a16 as K
    from w4a16.decode import LLAMA_3_2_1B

    fused, pers = _pair(LLAMA_3_2_1B, seed=0, fill=511)
    ref = pers.reference_logits(token=1, pos=511)
    a = fused.step(token=1, pos=511).clone()
    b = pers.step(token=1, pos=511).clone()
    torch.cuda.synchronize()
    assert torch.isfinite(b).all()
    scale = ref.abs().max().item()
    # 16 layers of fp16 rounding in different summation orders: the two kernel paths stay
    # within a few 1e-3 of each other and as close to the fp32 evaluation as each other
    d_ab = (b - a).abs().max().item()
    d_a, d_b = (a - ref).abs().max().item(), (b - ref).abs().max().item()
    print(f"full-size logits: |pers - fused| {d_ab:.2e}, |fused - fp32| {d_a:.2e}, |pers - fp32| {d_b:.2e}, "
          f"max |logit| {scale:.3f}")
    assert d_ab <= 5e-3 * scale
    assert d_b <= 2e-2 * scale and d_b <= 2 * d_a + 1e-3 * scale
    assert K.read_device_error() == 0
