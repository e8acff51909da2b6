"""Stand-in for the third-party ``model.model_minimind`` module — TEST INFRASTRUCTURE.

FonaTech/Project_Chronos imports ``MiniMindConfig``, ``FeedForward``,
``MOEFeedForward``, ``RMSNorm``, ``precompute_freqs_cis``, ``Attention``,
``apply_rotary_pos_emb`` and ``repeat_kv`` from minimind
(github.com/jingyaogong/minimind, branch ``master``, ``chronos/deps.py:17-18``),
which is not vendored in the reference and not installed here.  This file is
written for this project from the behaviour the reference relies on, so that
the reference's own ``ChronosMOEFeedForward`` can be imported and run on CPU to
produce golden vectors.  It is used only by ``tests/golden/make_golden.py``
(in the build container) and never on the product path.

The one piece whose arithmetic the MoE golden vectors depend on is
``FeedForward``: the bias-free SwiGLU ``down(act(gate(x)) * up(x))`` that the
reference restates itself at ``chronos/mlx/moe.py:13-23``.  Config defaults
that minimind would supply (``norm_topk_prob``, ``hidden_act``, …) are passed
explicitly by the golden generator, so they do not depend on this file.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from transformers import PretrainedConfig
from transformers.activations import ACT2FN


class MiniMindConfig(PretrainedConfig):
    model_type = "minimind"

    def __init__(self, dropout: float = 0.0, bos_token_id: int = 1, eos_token_id: int = 2,
                 hidden_act: str = "silu", hidden_size: int = 512,
                 intermediate_size: int | None = None, max_position_embeddings: int = 32768,
                 num_attention_heads: int = 8, num_hidden_layers: int = 8,
                 num_key_value_heads: int = 2, vocab_size: int = 6400,
                 rms_norm_eps: float = 1e-5, rope_theta: float = 1e6,
                 rope_scaling=None, flash_attn: bool = True, use_moe: bool = False,
                 num_experts: int = 4, num_experts_per_tok: int = 1,
                 moe_intermediate_size: int | None = None, norm_topk_prob: bool = True,
                 router_aux_loss_coef: float = 5e-4, head_dim: int | None = None,
                 tie_word_embeddings: bool = True, **kwargs):
        super().__init__(bos_token_id=bos_token_id, eos_token_id=eos_token_id,
                         tie_word_embeddings=tie_word_embeddings, **kwargs)
        self.dropout = dropout
        self.hidden_act = hidden_act
        self.hidden_size = hidden_size
        if intermediate_size is None:
            intermediate_size = 64 * ((int(hidden_size * 8 / 3) + 63) // 64)
        self.intermediate_size = intermediate_size
        self.max_position_embeddings = max_position_embeddings
        self.num_attention_heads = num_attention_heads
        self.num_hidden_layers = num_hidden_layers
        self.num_key_value_heads = num_key_value_heads
        self.vocab_size = vocab_size
        self.rms_norm_eps = rms_norm_eps
        self.rope_theta = rope_theta
        self.rope_scaling = rope_scaling
        self.flash_attn = flash_attn
        self.use_moe = use_moe
        self.num_experts = num_experts
        self.num_experts_per_tok = num_experts_per_tok
        self.moe_intermediate_size = (moe_intermediate_size if moe_intermediate_size is not None
                                      else intermediate_size)
        self.norm_topk_prob = norm_topk_prob
        self.router_aux_loss_coef = router_aux_loss_coef
        self.head_dim = head_dim if head_dim is not None else hidden_size // num_attention_heads


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (self.weight * xf).type_as(x)


def precompute_freqs_cis(dim: int, end: int = 32768, rope_base: float = 1e6, rope_scaling=None):
    inv = 1.0 / (rope_base ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    t = torch.arange(end).float()
    ang = torch.outer(t, inv)
    cos = torch.cat([torch.cos(ang), torch.cos(ang)], dim=-1)
    sin = torch.cat([torch.sin(ang), torch.sin(ang)], dim=-1)
    return cos, sin


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim: int = 1):
    c = cos.unsqueeze(unsqueeze_dim)
    s = sin.unsqueeze(unsqueeze_dim)
    return (q * c) + (_rotate_half(q) * s), (k * c) + (_rotate_half(k) * s)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    b, s, nkv, d = x.shape
    return x[:, :, :, None, :].expand(b, s, nkv, n_rep, d).reshape(b, s, nkv * n_rep, d)


class Attention(nn.Module):
    """Plain causal GQA attention with the (x, position_embeddings, past, use_cache,
    attention_mask) -> (out, present) calling convention the reference uses."""

    def __init__(self, config: MiniMindConfig):
        super().__init__()
        self.n_heads = config.num_attention_heads
        self.n_kv = config.num_key_value_heads or config.num_attention_heads
        self.n_rep = self.n_heads // self.n_kv
        self.head_dim = config.head_dim
        h = config.hidden_size
        self.q_proj = nn.Linear(h, self.n_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(h, self.n_kv * self.head_dim, bias=False)
        self.v_proj = nn.Linear(h, self.n_kv * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.n_heads * self.head_dim, h, bias=False)

    def forward(self, x, position_embeddings, past_key_value=None, use_cache=False,
                attention_mask=None):
        b, s, _ = x.shape
        xq = self.q_proj(x).view(b, s, self.n_heads, self.head_dim)
        xk = self.k_proj(x).view(b, s, self.n_kv, self.head_dim)
        xv = self.v_proj(x).view(b, s, self.n_kv, self.head_dim)
        start = past_key_value[0].shape[1] if past_key_value is not None else 0
        cos, sin = position_embeddings
        xq, xk = apply_rotary_pos_emb(xq, xk, cos[start:start + s], sin[start:start + s])
        if past_key_value is not None:
            xk = torch.cat([past_key_value[0], xk], dim=1)
            xv = torch.cat([past_key_value[1], xv], dim=1)
        present = (xk, xv) if use_cache else None
        q = xq.transpose(1, 2)
        k = repeat_kv(xk, self.n_rep).transpose(1, 2)
        v = repeat_kv(xv, self.n_rep).transpose(1, 2)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=(s > 1 and start == 0))
        return self.o_proj(out.transpose(1, 2).reshape(b, s, -1)), present


class FeedForward(nn.Module):
    """Bias-free SwiGLU expert (the form restated at chronos/mlx/moe.py:13-23)."""

    def __init__(self, config: MiniMindConfig, intermediate_size: int | None = None):
        super().__init__()
        inter = intermediate_size if intermediate_size is not None else config.intermediate_size
        self.gate_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.down_proj = nn.Linear(inter, config.hidden_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.dropout = nn.Dropout(config.dropout)
        self.act_fn = ACT2FN[config.hidden_act]

    def forward(self, x):
        return self.dropout(self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x)))


class MOEFeedForward(nn.Module):
    """Imported by the reference (moe_chronos.py:9) but never instantiated there."""

    def __init__(self, config: MiniMindConfig):
        super().__init__()
        self.experts = nn.ModuleList([FeedForward(config) for _ in range(config.num_experts)])

    def forward(self, x):  # pragma: no cover - unused by the reference
        raise NotImplementedError("MOEFeedForward is not used by Chronos")
