"""Seeded synthetic MoE-layer workloads (weights, hidden states, masks, router bias).

Every tensor comes from ONE ``torch.Generator`` seeded per workload and is
drawn in this fixed order:

1. router weight ``[E, H]``                     N(0, std)
2. for e in 0..E-1: gate ``[F, H]``, up ``[F, H]``, down ``[H, F]``   N(0, std)
3. for j in 0..S_h-1: shared gate, up, down     N(0, std)
4. hidden states ``[N, H]``                     N(0, 1)
5. availability mask ``[E]``                    Bernoulli(p) as ``rand < p``
6. router logit bias ``[E]`` (optional)         log p_e with p_e ∝ rank^-s over a
                                                seeded permutation (Zipf)

Values are drawn in fp32 and then cast to the requested dtype, so the bf16
tensors of two runs with the same seed are identical on any machine with the
same torch build.  Generation may run on the CPU (reproducible against the
committed golden fixtures) or on a CUDA device (fast, for benchmark-size
workloads; CUDA and CPU generators give different streams).

The named workloads mirror the benchmark configurations of the MoE layer:
``cpu_fp32`` (d_model 512, 8 experts top-2 + 1 shared, d_ff 1024, 256 tokens),
``decode`` (DeepSeek-MoE-16B shape: d_model 2048, 64 experts top-6 + 2 shared,
d_ff 1408, 1/8/32/64 tokens), ``prefill`` (same shape, 8192 tokens, Zipf s=1.1
router bias), ``ep`` (DeepSeek-V3 shape: d_model 7168, 256 experts top-8 + 1
shared, d_ff 2048, 4096 tokens per GPU) and ``e2e`` (8 layers of d_model 1024,
16 experts top-2 + 1 shared, d_ff 2048).
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch


@dataclasses.dataclass(frozen=True)
class MoEShape:
    hidden: int
    num_experts: int
    top_k: int
    ffn: int
    num_shared: int
    norm_topk: bool = True


WORKLOADS = {
    "cpu_fp32": dict(shape=MoEShape(512, 8, 2, 1024, 1), tokens=256, dtype=torch.float32,
                     avail_p=0.75, zipf_s=None),
    "decode": dict(shape=MoEShape(2048, 64, 6, 1408, 2), tokens=(1, 8, 32, 64),
                   dtype=torch.bfloat16, avail_p=0.9, zipf_s=None),
    "prefill": dict(shape=MoEShape(2048, 64, 6, 1408, 2), tokens=8192, dtype=torch.bfloat16,
                    avail_p=1.0, zipf_s=1.1),
    "ep": dict(shape=MoEShape(7168, 256, 8, 2048, 1), tokens=4096, dtype=torch.bfloat16,
               avail_p=1.0, zipf_s=None),
    "e2e": dict(shape=MoEShape(1024, 16, 2, 2048, 1), tokens=32, dtype=torch.bfloat16,
                avail_p=0.85, zipf_s=None),
}


@dataclasses.dataclass
class MoEWeights:
    router: torch.Tensor      # [E, H]
    gate: torch.Tensor        # [E, F, H]
    up: torch.Tensor          # [E, F, H]
    down: torch.Tensor        # [E, H, F]
    sh_gate: torch.Tensor     # [S, F, H]
    sh_up: torch.Tensor       # [S, F, H]
    sh_down: torch.Tensor     # [S, H, F]

    def to(self, device=None, dtype=None) -> "MoEWeights":
        return MoEWeights(*[getattr(self, f.name).to(device=device, dtype=dtype)
                            for f in dataclasses.fields(self)])


def _randn(g: torch.Generator, shape, std: float, device) -> torch.Tensor:
    t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t


def make_generator(seed: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def make_weights(shape: MoEShape, g: torch.Generator, dtype=torch.float32, device="cpu",
                 std: float = 0.02) -> MoEWeights:
    """Steps 1-3 of the draw order.  Stacked layouts: gate/up [E,F,H], down [E,H,F]."""
    e, h, f, s = shape.num_experts, shape.hidden, shape.ffn, shape.num_shared
    router = _randn(g, (e, h), std, device).to(dtype)
    gate = torch.empty(e, f, h, dtype=dtype, device=device)
    up = torch.empty(e, f, h, dtype=dtype, device=device)
    down = torch.empty(e, h, f, dtype=dtype, device=device)
    for i in range(e):
        gate[i].copy_(_randn(g, (f, h), std, device))
        up[i].copy_(_randn(g, (f, h), std, device))
        down[i].copy_(_randn(g, (h, f), std, device))
    sh_gate = torch.empty(s, f, h, dtype=dtype, device=device)
    sh_up = torch.empty(s, f, h, dtype=dtype, device=device)
    sh_down = torch.empty(s, h, f, dtype=dtype, device=device)
    for j in range(s):
        sh_gate[j].copy_(_randn(g, (f, h), std, device))
        sh_up[j].copy_(_randn(g, (f, h), std, device))
        sh_down[j].copy_(_randn(g, (h, f), std, device))
    return MoEWeights(router, gate, up, down, sh_gate, sh_up, sh_down)


def make_ep_weights(shape: MoEShape, rank: int, world: int, seed: int = 0, dtype=torch.bfloat16,
                    device="cpu", std: float = 0.02) -> MoEWeights:
    """Weights of one expert-parallel rank: the router and shared experts
    (replicated, from ``seed``) and ONLY this rank's routed experts
    ``[rank*E/G, (rank+1)*E/G)``, expert e drawn from its own generator
    (``seed * 1000003 + 1 + e``) so every rank agrees on every expert without
    materialising the others."""
    e, h, f, s = shape.num_experts, shape.hidden, shape.ffn, shape.num_shared
    epr = e // world
    g = make_generator(seed, device)
    router = _randn(g, (e, h), std, device).to(dtype)
    sh = [torch.empty(s, f, h, dtype=dtype, device=device), torch.empty(s, f, h, dtype=dtype, device=device),
          torch.empty(s, h, f, dtype=dtype, device=device)]
    for j in range(s):
        sh[0][j].copy_(_randn(g, (f, h), std, device))
        sh[1][j].copy_(_randn(g, (f, h), std, device))
        sh[2][j].copy_(_randn(g, (h, f), std, device))
    gate = torch.empty(epr, f, h, dtype=dtype, device=device)
    up = torch.empty(epr, f, h, dtype=dtype, device=device)
    down = torch.empty(epr, h, f, dtype=dtype, device=device)
    for i in range(epr):
        ge = make_generator(seed * 1000003 + 1 + rank * epr + i, device)
        gate[i].copy_(_randn(ge, (f, h), std, device))
        up[i].copy_(_randn(ge, (f, h), std, device))
        down[i].copy_(_randn(ge, (h, f), std, device))
    return MoEWeights(router, gate, up, down, sh[0], sh[1], sh[2])


def make_hidden(n: int, hidden: int, g: torch.Generator, dtype=torch.float32,
                device="cpu") -> torch.Tensor:
    """Step 4: hidden states N(0, 1), [N, H]."""
    return _randn(g, (n, hidden), 1.0, device).to(dtype)


def make_mask(num_experts: int, p: float, g: torch.Generator, device="cpu") -> torch.Tensor:
    """Step 5: availability mask, bool [E], True with probability p."""
    r = torch.rand(num_experts, generator=g, device=device, dtype=torch.float32)
    return r < p


def make_zipf_bias(num_experts: int, s: float, g: torch.Generator, device="cpu") -> torch.Tensor:
    """Step 6: per-expert router-logit offset log(p_e), p_e ∝ rank^-s over a seeded
    permutation of the experts (load imbalance for the prefill workload)."""
    perm = torch.randperm(num_experts, generator=g, device=device)
    ranks = torch.empty(num_experts, dtype=torch.float32, device=device)
    ranks[perm] = torch.arange(1, num_experts + 1, dtype=torch.float32, device=device)
    p = ranks.pow(-s)
    p = p / p.sum()
    return torch.log(p)


@dataclasses.dataclass
class Workload:
    shape: MoEShape
    weights: MoEWeights
    x: torch.Tensor                   # [N, H]
    mask: Optional[torch.Tensor]      # [E] bool or None
    bias: Optional[torch.Tensor]      # [E] fp32 or None


def make_workload(shape: MoEShape, tokens: int, seed: int = 0, dtype=torch.float32,
                  device="cpu", avail_p: Optional[float] = None,
                  zipf_s: Optional[float] = None, std: float = 0.02) -> Workload:
    g = make_generator(seed, device)
    w = make_weights(shape, g, dtype=dtype, device=device, std=std)
    x = make_hidden(tokens, shape.hidden, g, dtype=dtype, device=device)
    mask = make_mask(shape.num_experts, avail_p, g, device) if avail_p is not None else None
    bias = make_zipf_bias(shape.num_experts, zipf_s, g, device) if zipf_s else None
    return Workload(shape, w, x, mask, bias)


def named_workload(name: str, tokens: Optional[int] = None, seed: int = 0, device="cpu",
                   dtype=None) -> Workload:
    spec = WORKLOADS[name]
    n = tokens if tokens is not None else spec["tokens"]
    if isinstance(n, (tuple, list)):
        n = max(n)
    return make_workload(spec["shape"], int(n), seed=seed,
                         dtype=dtype if dtype is not None else spec["dtype"], device=device,
                         avail_p=spec["avail_p"] if spec["avail_p"] < 1.0 else None,
                         zipf_s=spec["zipf_s"])


def model_state(shapes, seed: int, std: float = 0.02, embed_std: float = 0.5,
                norm_std: float = 0.1) -> dict:
    """Seeded weights of a whole model by parameter name, drawn in sorted-name
    order from one CPU generator: RMSNorm weights (names ending in
    ``norm.weight``) 1 + N(0, norm_std), the token embedding N(0, embed_std),
    every other matrix N(0, std).  ``shapes``: {name: shape}; pass one name of
    a tied pair only."""
    g = make_generator(seed)
    out = {}
    for name in sorted(shapes):
        shp = tuple(shapes[name])
        if name.endswith("norm.weight"):
            out[name] = 1.0 + _randn(g, shp, norm_std, "cpu")
        elif "embed_tokens" in name:
            out[name] = _randn(g, shp, embed_std, "cpu")
        else:
            out[name] = _randn(g, shp, std, "cpu")
    return out


# The 8-layer Chronos model of the end-to-end decode workload (d_model 1024,
# 8 heads / 2 kv heads of 128, MLA latent 64 + rope 32 on even layers, a
# 2048-token window on odd layers, 16 experts top-2 + 1 shared, d_ff 2048,
# vocab 6400, tied LM head, lookahead router of 2 steps).
DECODE_MODEL = dict(vocab_size=6400, hidden_size=1024, num_hidden_layers=8, num_attention_heads=8,
                    num_key_value_heads=2, max_position_embeddings=32768, num_experts=16,
                    num_experts_per_tok=2, moe_intermediate_size=2048, num_shared_experts=1,
                    norm_topk_prob=True, kv_latent_dim=64, rope_dim=32, sliding_window_size=2048,
                    lookahead_steps=2, dropout=0.0, hidden_act="silu", rms_norm_eps=1e-5, rope_theta=1e6,
                    tie_word_embeddings=True, rope_scaling=None, use_hybrid_attention=True,
                    router_aux_loss_coef=5e-4, fallback_mask_prob=0.0, intermediate_size=2048, head_dim=128)


def init_model_(model, seed: int, device) -> None:
    """Seeded random init of a model's parameters on ``device``, in sorted-name
    order with one device generator (RMSNorm weights N(1, 0.1), the embedding
    N(0, 0.5), every other matrix N(0, 0.02))."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            if name.endswith("norm.weight"):
                p.normal_(1.0, 0.1, generator=g)
            elif "embed_tokens" in name:
                p.normal_(0.0, 0.5, generator=g)
            else:
                p.normal_(0.0, 0.02, generator=g)


def flops_per_token_routed(shape: MoEShape) -> float:
    """FLOPs of one routed or shared SwiGLU application to one token."""
    return 2.0 * 3.0 * shape.hidden * shape.ffn


def layer_flops(shape: MoEShape, tokens: int, routed_applications: Optional[int] = None) -> float:
    """Algorithmic FLOPs of one layer call: router GEMM + every expert application
    (routed applications default to N*k, i.e. all available) + shared experts."""
    if routed_applications is None:
        routed_applications = tokens * shape.top_k
    return (2.0 * tokens * shape.hidden * shape.num_experts
            + flops_per_token_routed(shape) * (routed_applications + tokens * shape.num_shared))


def expert_bytes(shape: MoEShape, elem_bytes: int = 2) -> int:
    return 3 * shape.hidden * shape.ffn * elem_bytes


def decode_bytes(shape: MoEShape, tokens: int, experts_read: int, elem_bytes: int = 2) -> int:
    """Algorithmic HBM bytes of one decode call: router weight, the weights of every
    expert read (selected-and-available routed experts plus the shared ones), x in
    and y out, router probabilities out."""
    return (elem_bytes * shape.hidden * shape.num_experts
            + expert_bytes(shape, elem_bytes) * (experts_read + shape.num_shared)
            + 2 * elem_bytes * tokens * shape.hidden
            + elem_bytes * tokens * shape.num_experts)


__all__ = ["MoEShape", "MoEWeights", "Workload", "WORKLOADS", "make_generator", "make_weights",
           "make_hidden", "make_mask", "make_zipf_bias", "make_workload", "named_workload",
           "layer_flops", "decode_bytes", "expert_bytes", "flops_per_token_routed", "make_ep_weights",
           "model_state", "DECODE_MODEL", "init_model_"]

