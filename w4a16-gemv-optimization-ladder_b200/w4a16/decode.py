"""One-token decode step of a Llama-architecture model on the W4A16 kernels.

The reference measures end-to-end decode by swapping the Linears of a Hugging Face
Llama-3.2-1B and looping `model(next_token, past_key_values=...)` from Python
(benchmarks/end_to_end.py:24-42): every token drives ~113 GEMVs plus the model's
other kernels from the host.  Here the same architecture (random weights; there is no
checkpoint offline) runs as a fixed sequence of device operations over a static KV
cache, captured once in a CUDA graph and replayed per token.  With `fused=True` (the
default for int4 weights) a layer is five launches:

  qkv = W_qkv fp16(rmsnorm(h))           gemv_rmsnorm  (norm in the GEMV prologue)
  attn = attention(rotary(q, k), cache)  decode_attention (also writes k, v at pos)
  h += W_o attn                          gemv          (residual in the epilogue)
  gu = W_gu fp16(rmsnorm(h))             gemv_rmsnorm
  h += W_down fp16(silu(g) * u)          gemv_swiglu   (activation in the prologue)

and the head is logits = W_lm fp16(rmsnorm(h)) (gemv_rmsnorm).  All projections are
int4 with group-128 scales; the residual stream h is fp32.  `fused=False` runs the
same GEMVs with the norms, rotary, cache write, attention (SDPA) and SwiGLU as torch
ops in between; `dense=True` builds the model with fp16 weights on cuBLAS (`F.linear`)
and the torch ops, for comparison.
"""
import ctypes
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import kernels as K

GROUP = 128


@dataclass
class LlamaDecodeConfig:
    hidden: int = 2048
    intermediate: int = 8192
    layers: int = 16
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 64
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5
    max_len: int = 512          # KV cache length

    @property
    def qkv_rows(self):
        return (self.heads + 2 * self.kv_heads) * self.head_dim


LLAMA_3_2_1B = LlamaDecodeConfig()


class _Proj:
    """One projection: int4 packed + group-128 scales, or a dense fp16 weight."""

    def __init__(self, w, dense):
        self.rows, self.cols = w.shape
        self.dense = dense
        if dense:
            self.w = w.half().contiguous()
        else:
            self.packed, self.scale = K.quantize_pack(w.contiguous(), group=GROUP)

    def bytes(self):
        if self.dense:
            return self.w.numel() * 2
        return self.packed.numel() + self.scale.numel() * self.scale.element_size()

    def dequantized(self):
        if self.dense:
            return self.w.float()
        return K.dequant_int4(self.packed, self.scale, group=GROUP).float()

    def __call__(self, x, out=None, residual=None, out_dtype=torch.float16):
        """out = W x (+ residual); x fp16 [cols].  residual (fp32 [rows]) may alias out."""
        if self.dense:
            y = F.linear(x.view(1, -1), self.w).view(-1)
            if residual is not None:
                out.copy_(residual + y.float())
                return out
            return y if out is None else out.copy_(y)
        if out is None:
            out = torch.empty(self.rows, dtype=out_dtype, device=x.device)
        return K.gemv(self.packed, self.scale, x, group=GROUP, bias=residual, out=out,
                      out_dtype=out.dtype)


def interleave_gate_up(w, inter):
    """[gate (inter rows) | up (inter rows)] -> blocks of 8 gate rows followed by the
    matching 8 up rows (the layout the one-kernel step applies SwiGLU to in its epilogue)."""
    rest = w.shape[1:]
    return w.view(2, inter // 8, 8, *rest).transpose(0, 1).reshape(2 * inter, *rest).contiguous()


def split_gate_up(v, inter, interleaved):
    """(gate, up) halves of a gate|up projection output (or of its weight rows) in either
    row layout."""
    if not interleaved:
        return v[:inter], v[inter:]
    rest = v.shape[1:]
    b = v.view(inter // 8, 2, 8, *rest)
    return b[:, 0].reshape(inter, *rest), b[:, 1].reshape(inter, *rest)


class _G128Weight(ctypes.Structure):
    _fields_ = [("packed", ctypes.c_void_p), ("scale", ctypes.c_void_p)]


class _LlamaDesc(ctypes.Structure):
    """w4a16_llama_desc of include/w4a16_b200.h."""
    _fields_ = [("layers", ctypes.c_int), ("hidden", ctypes.c_int), ("intermediate", ctypes.c_int),
                ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("vocab", ctypes.c_int), ("max_len", ctypes.c_int), ("eps", ctypes.c_float),
                ("qkv", ctypes.POINTER(_G128Weight)), ("o", ctypes.POINTER(_G128Weight)),
                ("gate_up", ctypes.POINTER(_G128Weight)), ("down", ctypes.POINTER(_G128Weight)),
                ("norm_attn", ctypes.POINTER(ctypes.c_void_p)), ("norm_mlp", ctypes.POINTER(ctypes.c_void_p)),
                ("lm_head", _G128Weight), ("norm_final", ctypes.c_void_p), ("embed", ctypes.c_void_p),
                ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p), ("gate_up_interleaved", ctypes.c_int)]


class DecodePlan:
    """The one-kernel decode step of the C ABI (w4a16_decode_plan_create / w4a16_decode_step)
    for a decoder's int4 weights: every layer and the head in one persistent launch."""

    def __init__(self, dec):
        from . import _lib

        cfg = dec.cfg
        self.lib = _lib.lib()
        self._check = _lib.check
        self.device = dec.device

        def wt(p):
            return _G128Weight(p.packed.data_ptr(), p.scale.data_ptr())

        L = cfg.layers
        arrs = {name: (_G128Weight * L)(*[wt(layer[name]) for layer in dec.layers])
                for name in ("qkv", "o", "gu", "down")}
        na = (ctypes.c_void_p * L)(*[layer["norm_attn"].data_ptr() for layer in dec.layers])
        nm = (ctypes.c_void_p * L)(*[layer["norm_mlp"].data_ptr() for layer in dec.layers])
        d = _LlamaDesc(L, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab,
                       cfg.max_len, cfg.eps, arrs["qkv"], arrs["o"], arrs["gu"], arrs["down"], na, nm,
                       wt(dec.lm_head), dec.norm_final.data_ptr(), dec.embed.data_ptr(), dec.cos.data_ptr(),
                       dec.sin.data_ptr(), 8 if dec.gu_interleaved else 0)
        self.plan = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            self._check(self.lib.w4a16_decode_plan_create(ctypes.byref(d), ctypes.byref(self.plan)),
                        "w4a16_decode_plan_create")

    def step(self, token, pos, k_cache, v_cache, logits):
        """Launch one step on the current stream (token, pos: device int64 [1])."""
        with torch.cuda.device(self.device):
            st = self.lib.w4a16_decode_step(self.plan, ctypes.c_void_p(token.data_ptr()),
                                            ctypes.c_void_p(pos.data_ptr()), ctypes.c_void_p(k_cache.data_ptr()),
                                            ctypes.c_void_p(v_cache.data_ptr()), ctypes.c_void_p(logits.data_ptr()),
                                            K._stream(self.device))
        self._check(st, "w4a16_decode_step")
        return logits

    def timeline(self, enable=True):
        """Start (enable=True) recording the per-CTA %globaltimer timeline of each step, or
        stop it.  Returns the number of entries a record holds."""
        n = ctypes.c_size_t(0)
        with torch.cuda.device(self.device):
            self._check(self.lib.w4a16_decode_plan_timeline(self.plan, int(enable), None, 0, ctypes.byref(n),
                                                            K._stream(self.device)), "w4a16_decode_plan_timeline")
        return n.value

    def read_timeline(self, grid):
        """The last step's record as an int64 tensor [3 * (barriers + 1), grid] (ns): rows
        3b, 3b + 1, 3b + 2 are barrier b's arrival, departure and the next phase's staged
        input (b = 0: start, end, first phase staged)."""
        import numpy as np

        n = self.timeline(True)
        buf = np.zeros(n, dtype=np.uint64)
        with torch.cuda.device(self.device):
            self._check(self.lib.w4a16_decode_plan_timeline(self.plan, 1, ctypes.c_void_p(buf.ctypes.data), n, None,
                                                            K._stream(self.device)), "w4a16_decode_plan_timeline")
        return torch.from_numpy(buf.astype(np.int64)).view(-1, grid)

    def close(self):
        if self.plan:
            self.lib.w4a16_decode_plan_destroy(self.plan)
            self.plan = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class W4A16LlamaDecoder:
    """Random-init Llama decoder for one-token steps (batch 1) over a static KV cache.

    fused: the step as the fused GEMV / attention kernels (one launch each, ~5 per layer);
    persistent: the whole step as one persistent kernel (DecodePlan), int4 weights only."""

    def __init__(self, cfg=LLAMA_3_2_1B, device="cuda", seed=0, dense=False, std=0.02, fused=None,
                 pdl=None, persistent=False, weights=None):
        """weights: None for random N(0, std) projections and unit norms, or a dict with
        embed [vocab, hidden], lm_head (None: tied to embed), norm_final [hidden] and
        layers: a list of dicts with q, k, v, o, gate, up, down (the nn.Linear weight
        matrices, [out, in]) and norm_attn, norm_mlp (see from_hf)."""
        self.cfg = cfg
        self.dense = dense
        self.persistent = bool(persistent)
        if self.persistent and (dense or cfg.head_dim != 64):
            raise ValueError("the persistent step needs int4 weights and head_dim 64")
        self.fused = (not dense and not self.persistent) if fused is None else bool(fused)
        if self.fused and (dense or cfg.head_dim != 64):
            raise ValueError("the fused step needs int4 weights and head_dim 64")
        # the one-kernel step keeps gate and up rows interleaved by 8 (SwiGLU in the epilogue)
        # the one-kernel step and the fused launches apply SwiGLU to gate / up row pairs in
        # the gate|up epilogue
        self.gu_interleaved = self.persistent or self.fused
        # chained launches (each kernel starts while the previous one finishes)
        self.pdl = self.fused if pdl is None else bool(pdl) and self.fused
        dev = torch.device(device)
        self.device = dev
        g = torch.Generator(device=dev).manual_seed(seed)
        H, I, D = cfg.hidden, cfg.intermediate, cfg.head_dim

        def rnd(*shape):
            return (torch.randn(*shape, device=dev, generator=g) * std).half()

        def gate_up(w):
            return interleave_gate_up(w, I) if self.gu_interleaved else w

        self.layers = []
        if weights is None:
            self.embed = rnd(cfg.vocab, H)
            for _ in range(cfg.layers):
                self.layers.append(dict(
                    qkv=_Proj(rnd(cfg.qkv_rows, H), dense),
                    o=_Proj(rnd(H, cfg.heads * D), dense),
                    gu=_Proj(gate_up(rnd(2 * I, H)), dense),
                    down=_Proj(rnd(H, I), dense),
                    norm_attn=torch.ones(H, device=dev),
                    norm_mlp=torch.ones(H, device=dev),
                ))
            self.norm_final = torch.ones(H, device=dev)
            self.lm_head = _Proj(self.embed, dense)  # tied to the embedding, as in Llama-3.2-1B
        else:
            def t(x):
                return x.detach().to(dev).float().contiguous()

            self.embed = t(weights["embed"]).half()
            for lw in weights["layers"]:
                self.layers.append(dict(
                    qkv=_Proj(torch.cat([t(lw["q"]), t(lw["k"]), t(lw["v"])]), dense),
                    o=_Proj(t(lw["o"]), dense),
                    gu=_Proj(gate_up(torch.cat([t(lw["gate"]), t(lw["up"])])), dense),
                    down=_Proj(t(lw["down"]), dense),
                    norm_attn=t(lw["norm_attn"]),
                    norm_mlp=t(lw["norm_mlp"]),
                ))
            self.norm_final = t(weights["norm_final"])
            head = weights.get("lm_head")
            self.lm_head = _Proj(self.embed if head is None else t(head), dense)
        # rotary tables (Llama's rotate-half convention)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=dev).float() / D))
        ang = torch.arange(cfg.max_len, device=dev).float()[:, None] * inv[None, :]
        self.cos = torch.cat([ang.cos(), ang.cos()], dim=1)   # [L, D]
        self.sin = torch.cat([ang.sin(), ang.sin()], dim=1)
        # static state
        self.k_cache = torch.zeros(cfg.layers, cfg.kv_heads, cfg.max_len, D, dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.token = torch.zeros(1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.h = torch.empty(H, dtype=torch.float32, device=dev)
        self.qkv = torch.empty(cfg.qkv_rows, dtype=torch.float16, device=dev)
        self.gu = torch.empty(2 * I, dtype=torch.float16, device=dev)
        self.act = torch.empty(I, dtype=torch.float16, device=dev)  # silu(gate) * up (fused step)
        self.attn = torch.empty(cfg.heads * D, dtype=torch.float16, device=dev)
        # two split-K workspaces, alternated so that overlapping neighbours never share one
        self.ws = [K.new_workspace(dev), K.new_workspace(dev)] if self.fused else None
        self.logits = torch.empty(cfg.vocab, dtype=torch.float32, device=dev)
        self.graph = None
        self.plan = DecodePlan(self) if self.persistent else None
        # greedy generation on the device: the next token and position are written by the
        # graph itself, generated tokens collected in gen_tokens
        self.gen_tokens = torch.zeros(cfg.max_len, dtype=torch.long, device=dev)
        self.gen_idx = torch.zeros(1, dtype=torch.long, device=dev)
        self.gen_graph = None

    # ------------------------------------------------------------------ pieces

    @classmethod
    def from_hf(cls, model, device="cuda", max_len=512, **kw):
        """A decoder with the weights of a Hugging Face LlamaForCausalLM (default rotary,
        head_dim 64): every Linear is quantised to int4 with group-128 scales here (the
        model's own weights are left untouched)."""
        c = model.config
        head_dim = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
        cfg = LlamaDecodeConfig(hidden=c.hidden_size, intermediate=c.intermediate_size,
                                layers=c.num_hidden_layers, heads=c.num_attention_heads,
                                kv_heads=c.num_key_value_heads, head_dim=head_dim, vocab=c.vocab_size,
                                rope_theta=float(getattr(c, "rope_theta", None)
                                                 or c.rope_parameters["rope_theta"]),
                                eps=c.rms_norm_eps, max_len=max_len)
        m = model.model
        layers = []
        for lyr in m.layers:
            a, f = lyr.self_attn, lyr.mlp
            layers.append(dict(q=a.q_proj.weight, k=a.k_proj.weight, v=a.v_proj.weight, o=a.o_proj.weight,
                               gate=f.gate_proj.weight, up=f.up_proj.weight, down=f.down_proj.weight,
                               norm_attn=lyr.input_layernorm.weight, norm_mlp=lyr.post_attention_layernorm.weight))
        tied = model.lm_head.weight.data_ptr() == m.embed_tokens.weight.data_ptr()
        weights = dict(embed=m.embed_tokens.weight, norm_final=m.norm.weight, layers=layers,
                       lm_head=None if tied else model.lm_head.weight)
        return cls(cfg, device=device, weights=weights, **kw)

    def weight_bytes(self):
        per = sum(p.bytes() for L in self.layers for p in (L["qkv"], L["o"], L["gu"], L["down"]))
        return per + self.lm_head.bytes()

    def fill_cache(self, length, seed=1):
        """Random keys/values for positions [0, length) (a stand-in for a prompt)."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        self.k_cache[:, :, :length].normal_(generator=g)
        self.v_cache[:, :, :length].normal_(generator=g)

    def _rmsnorm(self, h, w):
        return (h * torch.rsqrt(h.pow(2).mean() + self.cfg.eps) * w).half()

    def _rope(self, x, heads):
        D = self.cfg.head_dim
        x = x.view(heads, D).float()
        cos = self.cos.index_select(0, self.pos)    # [1, D]
        sin = self.sin.index_select(0, self.pos)
        rot = torch.cat([-x[:, D // 2:], x[:, :D // 2]], dim=1)
        return (x * cos + rot * sin).half()

    def _attention(self, q, li):
        cfg = self.cfg
        L = cfg.max_len
        kc = self.k_cache[li].view(1, cfg.kv_heads, L, cfg.head_dim)
        vc = self.v_cache[li].view(1, cfg.kv_heads, L, cfg.head_dim)
        mask = torch.where(torch.arange(L, device=self.device) <= self.pos, 0.0, float("-inf"))
        out = F.scaled_dot_product_attention(q.view(1, cfg.heads, 1, cfg.head_dim), kc, vc,
                                             attn_mask=mask.view(1, 1, 1, L).half(), enable_gqa=True)
        return out.reshape(-1)

    def _step_fused(self):
        cfg = self.cfg
        G, pdl, ws = GROUP, self.pdl, self.ws
        self.h.copy_(self.embed.index_select(0, self.token).view(-1))
        for li, L in enumerate(self.layers):
            qkv, o, gu, down = L["qkv"], L["o"], L["gu"], L["down"]
            # GEMVs alternate workspaces: qkv ws0, o ws1, gu ws0, down ws1 (attention has its own)
            K.gemv_rmsnorm(qkv.packed, qkv.scale, self.h, L["norm_attn"], cfg.eps, group=G, out=self.qkv,
                           pdl=pdl, workspace=ws[0])
            K.decode_attention(self.qkv, self.cos, self.sin, self.pos, self.k_cache[li], self.v_cache[li],
                               heads=cfg.heads, kv_heads=cfg.kv_heads, out=self.attn, pdl=pdl)
            K.gemv_staged(o.packed, o.scale, self.attn, group=G, bias=self.h, out=self.h, pdl=pdl,
                          workspace=ws[1])
            K.gemv_rmsnorm(gu.packed, gu.scale, self.h, L["norm_mlp"], cfg.eps, group=G, out=self.act,
                           pdl=pdl, workspace=ws[0], swiglu_out=True)
            K.gemv_staged(down.packed, down.scale, self.act, group=G, bias=self.h, out=self.h, pdl=pdl,
                          workspace=ws[1])
        head = self.lm_head
        K.gemv_rmsnorm(head.packed, head.scale, self.h, self.norm_final, cfg.eps, group=G, out=self.logits,
                       pdl=pdl, workspace=ws[0])
        return self.logits

    def _step(self):
        if self.persistent:
            return self.plan.step(self.token, self.pos, self.k_cache, self.v_cache, self.logits)
        if self.fused:
            return self._step_fused()
        cfg = self.cfg
        nq, nk = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        self.h.copy_(self.embed.index_select(0, self.token).view(-1).float())
        for li, L in enumerate(self.layers):
            x = self._rmsnorm(self.h, L["norm_attn"])
            L["qkv"](x, out=self.qkv)
            q = self._rope(self.qkv[:nq], cfg.heads)
            k = self._rope(self.qkv[nq:nq + nk], cfg.kv_heads)
            v = self.qkv[nq + nk:].view(cfg.kv_heads, cfg.head_dim)
            self.k_cache[li].index_copy_(1, self.pos, k.view(cfg.kv_heads, 1, cfg.head_dim))
            self.v_cache[li].index_copy_(1, self.pos, v.view(cfg.kv_heads, 1, cfg.head_dim))
            attn = self._attention(q, li)
            L["o"](attn, out=self.h, residual=self.h)
            x = self._rmsnorm(self.h, L["norm_mlp"])
            L["gu"](x, out=self.gu)
            a = (F.silu(self.gu[:cfg.intermediate].float()) * self.gu[cfg.intermediate:].float()).half()
            L["down"](a, out=self.h, residual=self.h)
        x = self._rmsnorm(self.h, self.norm_final)
        self.lm_head(x, out=self.logits)
        return self.logits

    # ------------------------------------------------------------------- public

    def step(self, token, pos):
        """Eager step: logits (fp32 [vocab]) for `token` at position `pos`."""
        self.token.fill_(int(token))
        self.pos.fill_(int(pos))
        return self._step()

    def capture(self):
        """Record one decode step in a CUDA graph (token and pos are read on the device)."""
        K.reserve_workspace(self.device, 1, self.cfg.vocab, self.cfg.hidden)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside capture
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        return self.graph

    def _greedy_step(self):
        logits = self._step()
        nxt = torch.argmax(logits).view(1)
        self.gen_tokens.index_copy_(0, self.gen_idx, nxt)
        self.token.copy_(nxt)
        self.pos.add_(1)
        self.gen_idx.add_(1)

    def capture_generate(self):
        """Record one greedy step in a CUDA graph: the step, the argmax of the logits fed
        back as the next token, the position advanced; replays need no host round trip."""
        K.reserve_workspace(self.device, 1, self.cfg.vocab, self.cfg.hidden)
        saved = (self.token.clone(), self.pos.clone(), self.gen_idx.clone(), self.k_cache.clone(),
                 self.v_cache.clone())
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside capture (restored below)
                self.pos.zero_()
                self.gen_idx.zero_()
                self._greedy_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.gen_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.gen_graph):
            self._greedy_step()
        for t, v in zip((self.token, self.pos, self.gen_idx, self.k_cache, self.v_cache), saved):
            t.copy_(v)
        return self.gen_graph

    def generate(self, token, pos, n):
        """Greedy continuation of `token` at position `pos` for n tokens (graph replays);
        returns the n generated token ids on the host."""
        if pos + n > self.cfg.max_len:
            raise ValueError(f"pos + n = {pos + n} exceeds the cache length {self.cfg.max_len}")
        if self.gen_graph is None:
            self.capture_generate()
        self.token.fill_(int(token))
        self.pos.fill_(int(pos))
        self.gen_idx.zero_()
        for _ in range(n):
            self.gen_graph.replay()
        return self.gen_tokens[:n].cpu()

    def replay(self, token, pos):
        """Graph step: set token/pos on the device, replay, return the logits buffer."""
        self.token.fill_(int(token))
        self.pos.fill_(int(pos))
        self.graph.replay()
        return self.logits

    def reference_logits(self, token, pos):
        """The same step in fp32 torch from the dequantised weights (test reference).

        Uses and updates a copy of the caches, so the decoder's own state is unchanged."""
        cfg = self.cfg
        D, nq, nk = cfg.head_dim, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        kc, vc = self.k_cache.float().clone(), self.v_cache.float().clone()
        p = int(pos)
        h = self.embed[int(token)].float()

        def norm(v, w):
            return v * torch.rsqrt(v.pow(2).mean() + cfg.eps) * w

        def rope(v, heads):
            v = v.view(heads, D)
            rot = torch.cat([-v[:, D // 2:], v[:, :D // 2]], dim=1)
            return v * self.cos[p] + rot * self.sin[p]

        for li, L in enumerate(self.layers):
            x = norm(h, L["norm_attn"]).half().float()
            qkv = L["qkv"].dequantized() @ x
            q, k = rope(qkv[:nq], cfg.heads), rope(qkv[nq:nq + nk], cfg.kv_heads)
            kc[li, :, p] = k
            vc[li, :, p] = qkv[nq + nk:].view(cfg.kv_heads, D)
            rep = cfg.heads // cfg.kv_heads
            keys = kc[li, :, : p + 1].repeat_interleave(rep, 0)      # [heads, p+1, D]
            vals = vc[li, :, : p + 1].repeat_interleave(rep, 0)
            att = torch.softmax((keys @ q.unsqueeze(-1)).squeeze(-1) / D ** 0.5, dim=-1)
            attn = (att.unsqueeze(1) @ vals).reshape(-1)
            h = h + L["o"].dequantized() @ attn
            x = norm(h, L["norm_mlp"]).half().float()
            gate, up = split_gate_up(L["gu"].dequantized() @ x, cfg.intermediate, self.gu_interleaved)
            a = F.silu(gate) * up
            h = h + L["down"].dequantized() @ a
        return self.lm_head.dequantized() @ norm(h, self.norm_final)


PHASES = ("qkv", "attention", "o", "gate_up", "down")


def timeline_summary(dec, layers):
    """One eager step of the one-kernel decode with its per-CTA %globaltimer record, reduced
    to where the time goes.  Phase p (five per layer: qkv, attention, o, gate_up, down, then
    the head) runs from the departure of barrier p (the kernel start for p = 0) to the arrival
    at barrier p + 1 (the kernel end for the head).  Per phase kind, summed over layers, in µs:
    work = median over CTAs of the phase's span, wait = median over CTAs of the barrier wait
    that ends it, staged = median time from a barrier's departure until the next phase's input
    vector is in shared memory; plus the step's span (start of the first CTA to the end of the
    last)."""
    plan = dec.plan
    nb = 5 * layers
    grid = plan.timeline(True) // (3 * (nb + 1))
    dec._step()
    torch.cuda.synchronize()
    t = plan.read_timeline(grid).double()
    plan.timeline(False)
    start, end = t[0], t[1]

    def dep(b):
        return start if b == 0 else t[3 * b + 1]

    def arr(b):
        return end if b == nb + 1 else t[3 * b]

    out = {k: {"work_us": 0.0, "wait_us": 0.0, "staged_us": 0.0} for k in PHASES + ("head",)}
    for ph in range(nb + 1):
        kind = "head" if ph == nb else PHASES[ph % 5]
        out[kind]["work_us"] += float((arr(ph + 1) - dep(ph)).median()) / 1e3
        out[kind]["staged_us"] += float((t[3 * ph + 2] - dep(ph)).median()) / 1e3
        if ph < nb:
            out[kind]["wait_us"] += float((t[3 * (ph + 1) + 1] - t[3 * (ph + 1)]).median()) / 1e3
    out = {k: {kk: round(vv, 1) for kk, vv in v.items()} for k, v in out.items()}
    out["span_us"] = round(float(end.max() - start.min()) / 1e3, 1)
    out["barriers"] = nb
    return out


def main(argv=None):
    """Time one decode step (graph replay, or eager launches) of the Llama-3.2-1B
    architecture: the counterpart of the reference's benchmarks/end_to_end.py."""
    import argparse
    import json

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--mode", choices=["persistent", "fused", "unfused", "dense"], default="persistent")
    ap.add_argument("--no-pdl", action="store_true", help="fused mode without chained launches")
    ap.add_argument("--layers", type=int, default=LLAMA_3_2_1B.layers)
    ap.add_argument("--max-len", type=int, default=LLAMA_3_2_1B.max_len)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--eager", action="store_true", help="launch op by op (no CUDA graph)")
    ap.add_argument("--timeline", action="store_true",
                    help="persistent mode: record one step's per-CTA timeline and report where its time goes")
    ap.add_argument("--generate", type=int, default=0,
                    help="also generate this many tokens greedily on the device and report tokens/s")
    a = ap.parse_args(argv)
    cfg = LlamaDecodeConfig(layers=a.layers, max_len=a.max_len)
    dec = W4A16LlamaDecoder(cfg, dense=a.mode == "dense", fused=a.mode == "fused",
                            pdl=False if a.no_pdl else None, persistent=a.mode == "persistent")
    pos = cfg.max_len - 1
    dec.fill_cache(pos)
    dec.token.fill_(1)
    dec.pos.fill_(pos)
    if a.eager:
        run = dec._step
    else:
        dec.capture()
        run = dec.graph.replay
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(a.steps):
        run()
    en.record()
    torch.cuda.synchronize()
    us = st.elapsed_time(en) * 1000.0 / max(a.steps, 1)
    res = {"mode": a.mode, "pdl": dec.pdl, "graph": not a.eager, "layers": cfg.layers,
           "kv_len": pos + 1, "step_us": round(us, 2), "weight_bytes": dec.weight_bytes(),
           "weight_gbs": round(dec.weight_bytes() / us / 1e3, 1)}
    if a.timeline:
        if a.mode != "persistent":
            raise SystemExit("--timeline needs --mode persistent")
        res["timeline"] = timeline_summary(dec, cfg.layers)
    if a.generate:
        n = min(a.generate, cfg.max_len - 1)
        dec.capture_generate()
        dec.generate(1, 0, 4)  # warm
        torch.cuda.synchronize()
        st.record()
        toks = dec.generate(1, 0, n)
        en.record()
        torch.cuda.synchronize()
        res.update({"generated": n, "tokens_per_s": round(n / (st.elapsed_time(en) / 1000.0), 1),
                    "first_tokens": toks[:8].tolist()})
    print(json.dumps(res))


if __name__ == "__main__":
    main()
