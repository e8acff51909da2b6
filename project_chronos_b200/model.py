"""Chronos hybrid-attention MoE language model on the sm_100a kernels.

Drop-in for ``chronos/model/model_chronos.py`` (``ChronosForCausalLM`` ->
``ChronosModel`` -> ``ChronosBlock``) and ``chronos/model/hybrid_attention.py``
(``MLAAttention`` on even layers, ``SlidingWindowAttention`` on odd layers) of
FonaTech/Project_Chronos: same constructor (a Chronos config), same
submodule names and parameter shapes, so the reference's ``state_dict``
(``model.layers.{i}.self_attn.*``, ``.mlp.*``, ``model.lookahead_router.*``,
``lm_head.weight`` tied to ``model.embed_tokens.weight``) loads unchanged.
``forward(input_ids, past_key_values=..., use_cache=..., available_expert_masks=...)``
returns ``(output, lookahead_probs)`` as the reference does, with
``output.logits``, ``output.past_key_values``, ``output.aux_loss``.

Where each piece runs:

* the MoE feed-forward of every block: ``ChronosMOEFeedForward`` (the fused
  routing, grouped tcgen05 GEMMs and blend of this package);
* the lookahead router after block 0: its fused kernel;
* every RMSNorm (the block norms fused with the residual add that precedes
  them, and the per-head query/key norms): ``chronos_add_rmsnorm``;
* one-token decode steps with a cache: the MLA and sliding-window decode
  kernels (``include/chronos_attention.h``: per-head norms, RoPE, the cache
  append and the attention in one launch per layer), with the input
  projections as one GEMM per layer (cuBLAS) and o_proj;
* a prompt (several tokens on an empty cache): the reference's own tensor
  arithmetic on the device (projections, RoPE, ``scaled_dot_product_attention``),
  which also fills the caches the decode kernels read;
* ``GraphedDecoder``: a whole decode step (every layer, the lookahead router,
  the LM head and the greedy pick of the next token) captured once as a CUDA
  graph and replayed per token; the position advances on the device.

The cache (``HybridCache``) keeps, per MLA layer, the normalised latent c_t and
the rotated rope keys of every position, and per sliding-window layer a ring of
``sliding_window_size`` key/value slots; the reference's cut-to-window
semantics, including the rotary position of a new token being the cut cache's
length (``hybrid_attention.py:217-234``), are kept.  Inputs must be CUDA
tensors, eval mode, no attention mask (the reference's 2-D padding mask is not
supported here), and a prompt must start on an empty cache.
"""
from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .lookahead import LookaheadRouter
from .moe import ChronosMOEFeedForward


def precompute_freqs_cis(dim: int, end: int, rope_base: float = 1e6, rope_scaling=None):
    """Rotary tables [end, dim] in minimind's form: frequencies base^(-2i/dim),
    i < dim/2, each row (cos(t f), cos(t f)) and (sin(t f), sin(t f))."""
    if rope_scaling:
        raise NotImplementedError("rope_scaling is not supported")
    inv = 1.0 / (rope_base ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    ang = torch.outer(torch.arange(end).float(), inv)
    return torch.cat([torch.cos(ang), torch.cos(ang)], dim=-1), torch.cat([torch.sin(ang), torch.sin(ang)], dim=-1)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, heads, d], cos/sin [S, d] (minimind apply_rotary_pos_emb)."""
    return x * cos[:, None, :] + _rotate_half(x) * sin[:, None, :]


def _repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    b, s, nkv, d = x.shape
    return x[:, :, :, None, :].expand(b, s, nkv, n_rep, d).reshape(b, s, nkv * n_rep, d)


class RMSNorm(nn.Module):
    """minimind RMSNorm: x * rsqrt(mean(x^2) + eps) * weight, in fp32, rounded to
    x's type; runs in ``chronos_add_rmsnorm``."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                sum_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("RMSNorm (sm_100a kernel) needs CUDA tensors")
        return ops.add_rmsnorm(x.contiguous(), self.weight, self.eps, residual=residual, sum_out=sum_out)


class HybridCache:
    """Decode caches of every layer of one batch.

    MLA layers (even): ``a[l]`` latent [B, capacity, L], ``b[l]`` rotated rope
    keys [B, capacity, nKV, R].  Sliding-window layers (odd): ``a[l]`` keys and
    ``b[l]`` values, rings of [B, window, nKV, D].  ``length`` (host) and
    ``pos`` (device int32, read by the kernels) count the cached tokens."""

    def __init__(self, config, batch: int, capacity: int, device, dtype):
        nh = config.num_attention_heads
        nkv = config.num_key_value_heads or nh
        d = getattr(config, "head_dim", None) or config.hidden_size // nh
        lat = getattr(config, "kv_latent_dim", max(64, nkv * d // 8))
        rope = max(1, min(getattr(config, "rope_dim", min(64, d)), d - 1))
        win = int(getattr(config, "sliding_window_size", 2048))
        self.batch, self.capacity, self.window = int(batch), int(capacity), win
        self.a: List[torch.Tensor] = []
        self.b: List[torch.Tensor] = []
        for layer in range(config.num_hidden_layers):
            if layer % 2 == 0:
                self.a.append(torch.zeros(batch, capacity, lat, device=device, dtype=dtype))
                self.b.append(torch.zeros(batch, capacity, nkv, rope, device=device, dtype=dtype))
            else:
                self.a.append(torch.zeros(batch, win, nkv, d, device=device, dtype=dtype))
                self.b.append(torch.zeros(batch, win, nkv, d, device=device, dtype=dtype))
        self.length = 0
        self.pos = torch.zeros((), dtype=torch.int32, device=device)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.a + self.b)


class MLAAttention(nn.Module):
    """Multi-head latent attention (``hybrid_attention.py:62-179``)."""

    def __init__(self, config, layer_id: int):
        super().__init__()
        self.layer_id = layer_id
        self.n_heads = config.num_attention_heads
        self.n_kv_heads = config.num_key_value_heads or config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // self.n_heads
        self.n_rep = self.n_heads // self.n_kv_heads
        self.kv_latent_dim = getattr(config, "kv_latent_dim", max(64, self.n_kv_heads * self.head_dim // 8))
        self.rope_dim = max(1, min(getattr(config, "rope_dim", min(64, self.head_dim)), self.head_dim - 1))
        self.nope_dim = self.head_dim - self.rope_dim
        self.eps = config.rms_norm_eps
        H = config.hidden_size
        self.q_nope_proj = nn.Linear(H, self.n_heads * self.nope_dim, bias=False)
        self.q_rope_proj = nn.Linear(H, self.n_heads * self.rope_dim, bias=False)
        self.q_nope_norm = RMSNorm(self.nope_dim, eps=config.rms_norm_eps)
        self.q_rope_norm = RMSNorm(self.rope_dim, eps=config.rms_norm_eps)
        self.kv_down_proj = nn.Linear(H, self.kv_latent_dim, bias=False)
        self.kv_down_norm = RMSNorm(self.kv_latent_dim, eps=config.rms_norm_eps)
        self.k_nope_proj = nn.Linear(self.kv_latent_dim, self.n_kv_heads * self.nope_dim, bias=False)
        self.k_rope_proj = nn.Linear(self.kv_latent_dim, self.n_kv_heads * self.rope_dim, bias=False)
        self.v_proj = nn.Linear(self.kv_latent_dim, self.n_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.n_heads * self.head_dim, H, bias=False)
        self._cat = None

    def _in_weight(self) -> torch.Tensor:
        """[q_nope_proj; q_rope_proj; kv_down_proj] stacked: one GEMM per step."""
        ws = (self.q_nope_proj.weight, self.q_rope_proj.weight, self.kv_down_proj.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype) for w in ws)
        if self._cat is None or self._cat[0] != key:
            self._cat = (key, torch.cat([w.detach() for w in ws], dim=0).contiguous())
        return self._cat[1]

    def prefill(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache: HybridCache) -> torch.Tensor:
        B, S, _ = x.shape
        nh, nkv, R, nope = self.n_heads, self.n_kv_heads, self.rope_dim, self.nope_dim
        q_nope = self.q_nope_norm(self.q_nope_proj(x).view(B, S, nh, nope))
        q_rope = self.q_rope_norm(self.q_rope_proj(x).view(B, S, nh, R))
        cr, sr = cos[:S, :R], sin[:S, :R]
        q = torch.cat([q_nope, _rope(q_rope, cr, sr)], dim=-1)
        c_kv = self.kv_down_norm(self.kv_down_proj(x))
        k_nope = self.k_nope_proj(c_kv).view(B, S, nkv, nope)
        k_rope = _rope(self.k_rope_proj(c_kv).view(B, S, nkv, R), cr, sr)
        k = torch.cat([k_nope, k_rope], dim=-1)
        v = self.v_proj(c_kv).view(B, S, nkv, self.head_dim)
        cache.a[self.layer_id][:, :S].copy_(c_kv)
        cache.b[self.layer_id][:, :S].copy_(k_rope)
        q = q.transpose(1, 2)
        k = _repeat_kv(k, self.n_rep).transpose(1, 2)
        v = _repeat_kv(v, self.n_rep).transpose(1, 2)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=S > 1)
        return self.o_proj(out.transpose(1, 2).reshape(B, S, -1))

    def decode(self, x2: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache: HybridCache) -> torch.Tensor:
        proj = F.linear(x2, self._in_weight())
        out = ops.attn_decode(
            "mla", proj, cache.pos, cos, sin, cache.a[self.layer_id], cache.b[self.layer_id], self.n_heads,
            self.n_kv_heads, self.head_dim, self.rope_dim, self.kv_latent_dim, 0, self.eps,
            self.q_nope_norm.weight, self.q_rope_norm.weight, norm_kv=self.kv_down_norm.weight,
            w_krope=self.k_rope_proj.weight, w_knope=self.k_nope_proj.weight, w_v=self.v_proj.weight)
        return F.linear(out, self.o_proj.weight)


class SlidingWindowAttention(nn.Module):
    """Local attention over the last ``sliding_window_size`` tokens
    (``hybrid_attention.py:184-258``)."""

    def __init__(self, config, layer_id: int):
        super().__init__()
        self.layer_id = layer_id
        self.n_heads = config.num_attention_heads
        self.n_kv_heads = config.num_key_value_heads or config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // self.n_heads
        self.n_rep = self.n_heads // self.n_kv_heads
        self.window_size = int(getattr(config, "sliding_window_size", 2048))
        self.eps = config.rms_norm_eps
        H = config.hidden_size
        self.q_proj = nn.Linear(H, self.n_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(H, self.n_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(H, self.n_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.n_heads * self.head_dim, H, bias=False)
        self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self._cat = None

    def _in_weight(self) -> torch.Tensor:
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype) for w in ws)
        if self._cat is None or self._cat[0] != key:
            self._cat = (key, torch.cat([w.detach() for w in ws], dim=0).contiguous())
        return self._cat[1]

    def prefill(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache: HybridCache) -> torch.Tensor:
        B, S, _ = x.shape
        D, W = self.head_dim, self.window_size
        xq = self.q_norm(self.q_proj(x).view(B, S, self.n_heads, D))
        xk = self.k_norm(self.k_proj(x).view(B, S, self.n_kv_heads, D))
        xv = self.v_proj(x).view(B, S, self.n_kv_heads, D)
        xq, xk = _rope(xq, cos[:S], sin[:S]), _rope(xk, cos[:S], sin[:S])
        if S > W:  # the reference keeps the last `window` keys only
            xk, xv = xk[:, -W:], xv[:, -W:]
        T = xk.shape[1]
        slots = torch.arange(S - T, S, device=x.device) % W
        cache.a[self.layer_id][:, slots] = xk
        cache.b[self.layer_id][:, slots] = xv
        q = xq.transpose(1, 2)
        k = _repeat_kv(xk, self.n_rep).transpose(1, 2)
        v = _repeat_kv(xv, self.n_rep).transpose(1, 2)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=(T == S and S > 1))
        return self.o_proj(out.transpose(1, 2).reshape(B, S, -1))

    def decode(self, x2: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache: HybridCache) -> torch.Tensor:
        proj = F.linear(x2, self._in_weight())
        out = ops.attn_decode(
            "sw", proj, cache.pos, cos, sin, cache.a[self.layer_id], cache.b[self.layer_id], self.n_heads,
            self.n_kv_heads, self.head_dim, self.head_dim, 0, self.window_size, self.eps,
            self.q_norm.weight, self.k_norm.weight)
        return F.linear(out, self.o_proj.weight)


def make_attention(layer_id: int, config) -> nn.Module:
    """Even layers MLA, odd layers sliding window (``hybrid_attention.py:261-269``)."""
    return MLAAttention(config, layer_id) if layer_id % 2 == 0 else SlidingWindowAttention(config, layer_id)


class ChronosBlock(nn.Module):
    def __init__(self, layer_id: int, config):
        super().__init__()
        if not getattr(config, "use_hybrid_attention", True):
            raise NotImplementedError("only the hybrid attention blocks are implemented")
        self.layer_id = layer_id
        self.self_attn = make_attention(layer_id, config)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.mlp = ChronosMOEFeedForward(config)


@dataclasses.dataclass
class CausalLMOutput:
    logits: torch.Tensor
    past_key_values: Optional[HybridCache]
    aux_loss: torch.Tensor
    hidden_states: torch.Tensor
    loss: Optional[torch.Tensor] = None


class ChronosModel(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.vocab_size = config.vocab_size
        self.num_hidden_layers = config.num_hidden_layers
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.dropout = nn.Dropout(getattr(config, "dropout", 0.0))
        self.layers = nn.ModuleList([ChronosBlock(i, config) for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.lookahead_router = LookaheadRouter(config)
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        cos, sin = precompute_freqs_cis(head_dim, config.max_position_embeddings, config.rope_theta,
                                        getattr(config, "rope_scaling", None))
        self.register_buffer("freqs_cos", cos, persistent=False)
        self.register_buffer("freqs_sin", sin, persistent=False)

    def _blocks(self, hidden: torch.Tensor, cache: HybridCache, masks, decode: bool):
        """Every block on hidden [B, S, H]; the residual adds are fused into the
        next RMSNorm.  Returns (final normed hidden, lookahead probs)."""
        B, S, H = hidden.shape
        cos, sin = self.freqs_cos, self.freqs_sin
        pending = None           # last MoE output, not yet added to `hidden`
        look = None
        for i, layer in enumerate(self.layers):
            h_in = layer.input_layernorm(hidden) if pending is None else \
                layer.input_layernorm(pending, residual=hidden, sum_out=hidden)
            if decode:
                attn = layer.self_attn.decode(h_in.view(B, H), cos, sin, cache).view(B, 1, H)
            else:
                attn = layer.self_attn.prefill(h_in, cos, sin, cache)
            mlp_in = layer.post_attention_layernorm(attn, residual=hidden, sum_out=hidden)
            mask = masks[i] if masks else None
            if decode and i > 0 and hasattr(layer.mlp, "forward_acc"):
                # the next norm rounds the layer's fp32 accumulator itself (no finalize pass)
                pending = layer.mlp.forward_acc(mlp_in, mask)
            else:
                pending = layer.mlp(mlp_in, mask)
            if i == 0:   # the lookahead router reads block 0's output (model_chronos.py:155-156)
                hidden = hidden + pending
                pending = None
                look = self.lookahead_router(hidden)
        out = self.norm(hidden) if pending is None else self.norm(pending, residual=hidden, sum_out=hidden)
        return out, look

    def forward(self, input_ids, attention_mask=None, past_key_values: Optional[HybridCache] = None,
                use_cache: bool = False, available_expert_masks=None, cache_capacity: int = 4096, **kwargs):
        if attention_mask is not None:
            raise NotImplementedError("attention masks are not supported")
        if self.training and torch.is_grad_enabled():
            raise NotImplementedError("forward-only kernels: call under torch.no_grad() or in eval mode")
        B, S = input_ids.shape
        cache = past_key_values
        decode = cache is not None and cache.length > 0
        if decode:
            if S != 1:
                raise NotImplementedError("a cached step takes one token per row")
            if cache.length >= cache.capacity or cache.length >= self.freqs_cos.shape[0]:
                raise RuntimeError(f"cache full at {cache.length} tokens (capacity {cache.capacity}, "
                                   f"rotary table {self.freqs_cos.shape[0]})")
        else:
            if S > self.freqs_cos.shape[0]:
                raise RuntimeError("prompt longer than max_position_embeddings")
            if cache is None:
                cache = HybridCache(self.config, B, max(cache_capacity, S + 1), input_ids.device,
                                    self.embed_tokens.weight.dtype)
            elif S > cache.capacity:
                raise RuntimeError("prompt longer than the cache")
        hidden = self.dropout(self.embed_tokens(input_ids))
        out, look = self._blocks(hidden, cache, available_expert_masks, decode)
        cache.length += S
        if decode:
            cache.pos.add_(1)
        else:
            cache.pos.fill_(cache.length)
        aux = sum((layer.mlp.aux_loss for layer in self.layers), out.new_zeros(()))
        return out, (cache if use_cache or decode else None), aux, look


class ChronosForCausalLM(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.model = ChronosModel(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if getattr(config, "tie_word_embeddings", True):
            self.model.embed_tokens.weight = self.lm_head.weight

    @classmethod
    def on_device(cls, config, device, dtype) -> "ChronosForCausalLM":
        """A model with uninitialised parameters allocated straight on ``device`` in
        ``dtype`` (no host copy), rotary tables computed; fill the weights with
        ``load_state_dict`` or an initialiser."""
        with torch.device("meta"):
            m = cls(config)
        m = m.to_empty(device=device)
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        cos, sin = precompute_freqs_cis(head_dim, config.max_position_embeddings, config.rope_theta,
                                        getattr(config, "rope_scaling", None))
        m.model.freqs_cos, m.model.freqs_sin = cos.to(device), sin.to(device)
        return m.to(dtype)

    def forward(self, input_ids, attention_mask=None, past_key_values=None, use_cache=False,
                logits_to_keep: int = 0, labels=None, available_expert_masks=None, **kwargs):
        hidden, cache, aux, look = self.model(input_ids, attention_mask, past_key_values, use_cache,
                                              available_expert_masks=available_expert_masks, **kwargs)
        keep = slice(-logits_to_keep, None) if logits_to_keep > 0 else slice(None)
        logits = F.linear(hidden[:, keep, :], self.lm_head.weight)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[..., :-1, :].reshape(-1, logits.shape[-1]).float(),
                                   labels[..., 1:].reshape(-1), ignore_index=-100)
        return CausalLMOutput(logits, cache, aux, hidden, loss), look


class GraphedDecoder:
    """One greedy decode step of ``ChronosForCausalLM`` captured as a CUDA graph.

    The step embeds ``ids`` [B, 1], runs every block (attention decode kernels,
    MoE layers with the per-layer availability rows of ``masks`` [L, E]), the
    lookahead router and the LM head, picks the arg-max token of every row into
    ``next_ids``, copies it into ``ids`` (so consecutive replays generate
    greedily; a caller may write ``ids`` before a replay to teacher-force) and
    advances the cache position, all on the device.  Capture runs two warm-up
    steps at the current position first (they write that position's cache
    entries, which the first replay overwrites)."""

    def __init__(self, lm: ChronosForCausalLM, cache: HybridCache, masks: Optional[torch.Tensor] = None):
        if cache.length < 1:
            raise RuntimeError("prefill the cache before capturing decode steps")
        self.lm, self.cache = lm, cache
        dev = cache.pos.device
        L = lm.config.num_hidden_layers
        E = lm.config.num_experts
        self.ids = torch.zeros(cache.batch, 1, dtype=torch.long, device=dev)
        self.masks = masks if masks is not None else torch.ones(L, E, dtype=torch.float32, device=dev)
        self.next_ids = torch.zeros(cache.batch, dtype=torch.long, device=dev)
        for _ in range(2):
            self._body(advance=False)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        before = ops.kernel_launches()
        with torch.cuda.graph(self.graph):
            self.logits, self.lookahead = self._body(advance=True)
        # kernels of this package in one step (the graph replays exactly these)
        self.launches_per_step = ops.kernel_launches() - before

    def _body(self, advance: bool):
        m = self.lm.model
        hidden = m.embed_tokens(self.ids)
        out, look = m._blocks(hidden, self.cache, [self.masks[i] for i in range(len(m.layers))], decode=True)
        logits = F.linear(out[:, -1, :], self.lm.lm_head.weight)
        ops.argmax_rows(logits, out=self.next_ids)
        if advance:
            self.ids.copy_(self.next_ids.view(-1, 1))
            self.cache.pos.add_(1)
        return logits, look

    def step(self) -> torch.Tensor:
        c = self.cache
        if c.length >= c.capacity or c.length >= self.lm.model.freqs_cos.shape[0]:
            raise RuntimeError(f"cache full at {c.length} tokens")
        self.graph.replay()
        c.length += 1
        return self.next_ids
