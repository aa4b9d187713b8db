"""Decode step of the Llama-architecture model on the W4A16 kernels (GPU).

The graph-replayed step must equal the eager step, and both must match an fp32 torch
evaluation of the same step from the dequantised weights (the decoder itself rounds the
GEMV inputs and outputs to fp16, as the reference's fp16 models do)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _small():
    from w4a16.decode import LlamaDecodeConfig

    return LlamaDecodeConfig(layers=2, vocab=4096, max_len=128)


@pytest.mark.parametrize("dense,fused", [(False, True), (False, False), (True, False)])
def test_eager_step_matches_fp32_reference(dense, fused):
    from w4a16.decode import W4A16LlamaDecoder

    dec = W4A16LlamaDecoder(_small(), dense=dense, fused=fused, seed=3)
    dec.fill_cache(63)
    ref = dec.reference_logits(token=17, pos=63)
    out = dec.step(token=17, pos=63).clone()
    err = (out - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err


def test_graph_replay_equals_eager_and_advances_cache():
    from w4a16.decode import W4A16LlamaDecoder

    dec = W4A16LlamaDecoder(_small(), seed=4)
    dec.fill_cache(40)
    k0 = dec.k_cache.clone()
    v0 = dec.v_cache.clone()
    eager = dec.step(token=5, pos=40).clone()
    k_eager = dec.k_cache[:, :, 40].clone()
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    dec.capture()
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    replay = dec.replay(token=5, pos=40).clone()
    torch.cuda.synchronize()
    assert torch.equal(replay, eager)
    assert torch.equal(dec.k_cache[:, :, 40], k_eager)
    nxt = dec.replay(token=int(replay.argmax()), pos=41).clone()   # the next position
    assert torch.isfinite(nxt).all() and not torch.equal(nxt, replay)
    assert not torch.equal(dec.k_cache[:, :, 41], k0[:, :, 41])


def test_full_size_weight_bytes():
    from w4a16.decode import LLAMA_3_2_1B, W4A16LlamaDecoder

    dec = W4A16LlamaDecoder(LLAMA_3_2_1B, seed=0)
    # 113 Linears of Llama-3.2-1B (q,k,v,o,gate,up,down x 16 + lm_head) at 0.5 B/weight plus
    # fp32 group-128 scales (4 B per 128 weights)
    weights = 16 * (2048 * 3072 + 2048 * 2048 + 2048 * 16384 + 8192 * 2048) + 128256 * 2048
    assert dec.weight_bytes() == weights // 2 + weights // 128 * 4
    dec.fill_cache(511)
    dec.capture()
    logits = dec.replay(token=1, pos=511)
    torch.cuda.synchronize()
    assert torch.isfinite(logits).all()


def test_chained_launches_change_nothing():
    # the fused step with programmatic dependent launch equals the one without, bit for bit
    from w4a16.decode import W4A16LlamaDecoder

    outs = []
    for pdl in (False, True):
        dec = W4A16LlamaDecoder(_small(), seed=6, pdl=pdl)
        assert dec.pdl == pdl
        dec.fill_cache(70)
        outs.append(dec.step(token=9, pos=70).clone())
        dec.capture()
        outs.append(dec.replay(token=9, pos=70).clone())
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_greedy_generation_on_device_matches_eager_loop():
    from w4a16.decode import W4A16LlamaDecoder

    dec = W4A16LlamaDecoder(_small(), seed=7)
    dec.fill_cache(20)
    k0, v0 = dec.k_cache.clone(), dec.v_cache.clone()
    toks = dec.generate(token=11, pos=20, n=12)            # graph replays, argmax fed back on device
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    want, t = [], 11
    for i in range(12):                                      # the same steps launched one by one
        t = int(dec.step(token=t, pos=20 + i).argmax())
        want.append(t)
    assert toks.tolist() == want
    with pytest.raises(ValueError):
        dec.generate(token=1, pos=120, n=20)
