"""The decode step against Hugging Face's LlamaForCausalLM (transformers), the model the
reference's end-to-end benchmark runs (benchmarks/end_to_end.py:24-42).

A small random-init Llama (2 layers, hidden 1024, 16 query / 4 kv heads of 64, SwiGLU 2048,
vocab 4096, default rotary) is loaded into W4A16LlamaDecoder, which quantises every Linear to
int4 with group-128 scales; the Hugging Face model then gets exactly those weights back
(dequantised) and the fp16 embedding, so both sides compute the same network.  A greedy run
over a short prompt must give the same logits (within 1e-2 absolute; the decoder rounds its
GEMV inputs, q/k/v and the attention output to fp16) and the same tokens.  This pins the
rotary convention, the GQA head mapping, the RMSNorm epsilon and weight, the q|k|v and
gate|up layouts and the untied head."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _hf_model(seed):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(seed)
    c = LlamaConfig(vocab_size=4096, hidden_size=1024, intermediate_size=2048, num_hidden_layers=2,
                    num_attention_heads=16, num_key_value_heads=4, head_dim=64, max_position_embeddings=128,
                    rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=True,
                    attn_implementation="eager")
    model = LlamaForCausalLM(c).float().cuda().eval()
    with torch.no_grad():  # norm weights other than one, so that they are exercised
        for lyr in model.model.layers:
            lyr.input_layernorm.weight.uniform_(0.5, 1.5)
            lyr.post_attention_layernorm.weight.uniform_(0.5, 1.5)
        model.model.norm.weight.uniform_(0.5, 1.5)
    return model


def _give_hf_the_quantised_weights(dec, model):
    from w4a16.decode import split_gate_up

    cfg = dec.cfg
    nq, nk = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    with torch.no_grad():
        for lyr, L in zip(model.model.layers, dec.layers):
            qkv = L["qkv"].dequantized()
            lyr.self_attn.q_proj.weight.copy_(qkv[:nq])
            lyr.self_attn.k_proj.weight.copy_(qkv[nq:nq + nk])
            lyr.self_attn.v_proj.weight.copy_(qkv[nq + nk:])
            lyr.self_attn.o_proj.weight.copy_(L["o"].dequantized())
            gu = L["gu"].dequantized()
            gate, up = split_gate_up(gu, cfg.intermediate, dec.gu_interleaved)
            lyr.mlp.gate_proj.weight.copy_(gate)
            lyr.mlp.up_proj.weight.copy_(up)
            lyr.mlp.down_proj.weight.copy_(L["down"].dequantized())
        # the lookup uses the fp16 embedding, the head its int4 quantisation: untie them
        model.model.embed_tokens.weight.copy_(dec.embed.float())
        model.lm_head.weight = torch.nn.Parameter(dec.lm_head.dequantized().clone())


@pytest.mark.parametrize("mode", ["fused", "persistent"])
def test_greedy_decode_matches_hugging_face_llama(mode):
    import w4a16 as K
    from w4a16.decode import W4A16LlamaDecoder

    model = _hf_model(seed=1)
    dec = W4A16LlamaDecoder.from_hf(model, max_len=128, fused=mode == "fused", persistent=mode == "persistent")
    _give_hf_the_quantised_weights(dec, model)
    prompt = [1, 517, 33, 2048, 77, 9]       # then six greedy tokens
    seq, nxt, worst = [], None, 0.0
    for step in range(12):
        tok = prompt[step] if step < len(prompt) else nxt
        seq.append(tok)
        with torch.no_grad():
            ref = model(torch.tensor([seq], device="cuda")).logits[0, -1].float()
        ours = dec.step(token=tok, pos=step).clone()   # one token at a time through the cache
        torch.cuda.synchronize()
        err = (ours - ref).abs().max().item()
        worst = max(worst, err)
        assert err <= 1e-2, f"step {step}: max |logit diff| {err:.3e} (max |logit| {ref.abs().max().item():.3f})"
        if step >= len(prompt) - 1:  # from the last prompt token on: both pick the same next token
            nxt = int(ref.argmax())
            assert int(ours.argmax()) == nxt
    print(f"{mode}: worst |logit diff| over 12 steps {worst:.2e}")
    assert K.read_device_error() == 0


def test_prefill_through_the_int4_gemm_matches_hugging_face():
    """A 100-token prefill of the Hugging Face model after replace_linear_with_w4a16 with no
    dense copy: every projection (batch 100 > 64 rows) runs the tensor-core int4 GEMM, whose
    contract is x @ dequant(W).T in fp32 sums.  The same model with those dequantised weights
    copied back (fp16 model, torch matmuls) must give the same logits within fp16 rounding."""
    import copy

    import w4a16 as K

    base = _hf_model(5).half()
    quant = copy.deepcopy(base)
    K.replace_linear_with_w4a16(quant, group=128, keep_dense=False)
    ref = base
    qmods = dict(quant.named_modules())
    with torch.no_grad():  # the reference model gets the quantised weights, dequantised
        for (name, mod) in list(ref.named_modules()):
            if isinstance(mod, torch.nn.Linear):
                q = qmods[name]
                # a new parameter, not a copy: the head is tied to the embedding, which the
                # int4 model keeps in fp16
                mod.weight = torch.nn.Parameter(K.dequant_int4(q.packed, q.scale, group=128))
    ids = torch.randint(0, 4096, (1, 100), device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))
    with torch.no_grad():
        got = quant(ids).logits.float()
        want = ref(ids).logits.float()
    assert torch.isfinite(got).all()
    err = (got - want).abs().max().item()
    assert err <= 2e-2 * max(1.0, want.abs().max().item()), err
    assert (got.argmax(-1) == want.argmax(-1)).float().mean().item() > 0.9
