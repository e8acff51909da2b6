"""Generate golden vectors for the MoE layer from the REFERENCE implementation.

Run in the build container (the only place the reference tree exists):

    python tests/golden/make_golden.py [--ref /root/reference] [--only NAME]

It imports FonaTech/Project_Chronos's own ``chronos.model.moe_chronos``,
``chronos.model.lookahead_router`` and ``chronos.io.storage`` (unmodified)
with ``tests/golden/minimind_shim`` standing in for the absent third-party
minimind package and a stub ``chronos.deps`` that points the reference's
bootstrap at that shim instead of cloning from the network
(``chronos/deps.py:49-72``).  For every case below it rebuilds the seeded
inputs with ``project_chronos_b200.synthetic`` (CPU generator), runs the
reference on the CPU and stores the reference outputs in
``tests/golden/<case>.npz``; the case parameters go to ``cases.json``.
Inputs are NOT stored: tests regenerate them from the same seeds.

MoE cases.  Unavailable experts are replaced by the reference's
``LazyExpertPlaceholder`` (as ``tests/test_smoke.py:147-167`` of the reference
does), because in eval mode the reference only takes the shared-expert
fallback for placeholder experts (``moe_chronos.py:220-227``).  Cases with a
Zipf router bias (the prefill workload) give the reference's ``gate`` Linear a
bias of ``log p_e``: the logits are then ``x W^T + b`` as the layer's
``router_logit_bias`` adds them.

Stored per MoE case (all from the reference):
  y_ref        layer output in the case dtype, as fp32 (bf16 cases: the
               bf16 bit patterns, uint16, to keep the file small)   [N, H]
  y_ref_fp32   (bf16 cases) the reference run in fp32 on the same bf16-valued
               weights and inputs                                  [N, H]
  idx_ref      top-k indices per token, sorted ascending (fp32 run)   [N, k]
  w_ref        top-k weights aligned with idx_ref (fp32 run)         [N, k]
  probs_ref    router probabilities (fp32 run)                      [N, E]
  idx_lit      (bf16 cases) top-k sets of the LITERAL bf16 path: the bf16
               gate GEMM, bf16 softmax and torch.topk
               (``moe_chronos.py:112, 124-128``), sorted ascending  [N, k]
  probs_lit    (bf16 cases) that path's bf16 probabilities, uint16 bits [N, E]
  logits64     (bf16 cases) x W^T (+ b) in float64 on the bf16 values [N, E]
  logits64_lit (bf16 cases) the same with the bias rounded to bf16, as the
               literal path's bf16 gate parameter holds it          [N, E]
  keep_draws   (train_fallback) the uniform draws ``torch.rand(E)`` the
               reference made for its miss simulation (``:141``)     [E]
and in ``cases.json``: the bookkeeping lists and masses, ``aux_loss_raw`` /
``aux_loss`` (train cases), and for bf16 cases the mismatch count of the
literal bf16 routing against the fp32 routing contract, each mismatch
classified (``tests/_golden.py:classify_literal``).

Lookahead cases run the reference's ``LookaheadRouter`` (``probs_ref``
[B, S, K, E], plus ``probs_ref_fp32`` for bf16).  ``model_tf`` runs the
reference's ``ChronosForCausalLM`` (hybrid attention, MoE blocks, lookahead
router) teacher-forced: ``logits_{fp32,bf16}`` [steps+1, B, V] and
``lookahead_{fp32,bf16}`` [steps+1, B, K, E] at the last position of the
prompt and of every cached one-token step, and the token ids.
``attn_decode`` steps the reference's two attention modules alone, one token
at a time with their caches (``y_mla``, ``y_sw`` [steps, B, H], inputs ``x``).  The ``ctsr_ref`` directory
holds cluster files written by the reference's ``ClusterStorage.write_clusters``
(``chronos/io/storage.py:182-233``) for the readers here to load.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
SHIM = HERE / "minimind_shim"
sys.path.insert(0, str(REPO))

from tests._golden import bf16_bits, classify_literal, from_bf16_bits as G_from_bits  # noqa: E402

# Cases: shape (H, E, k, F, S_h), tokens as (B, S), dtype, seed, availability
# probability (None = no mask), mode: "eval" (placeholders for unavailable
# experts), "eval_stale" (mask given but every expert live), "train_mask"
# (train mode, dropout 0, float mask, no placeholders), "nomask",
# "train_nomask" (train mode, standard path, aux loss), "train_fallback"
# (train mode, no mask, fallback_mask_prob > 0: the reference's miss simulation).
CASES = [
    dict(name="cfg1_fp32", H=512, E=8, k=2, F=1024, S=1, norm=True, B=2, T=128,
         dtype="fp32", seed=0, avail_p=0.75, mode="eval"),
    dict(name="cfg1_fp32_nonorm", H=512, E=8, k=2, F=1024, S=1, norm=False, B=1, T=64,
         dtype="fp32", seed=1, avail_p=0.75, mode="eval"),
    dict(name="tiny_nomask", H=64, E=4, k=2, F=128, S=1, norm=True, B=1, T=8,
         dtype="fp32", seed=2, avail_p=None, mode="nomask"),
    dict(name="tiny_allmask", H=64, E=4, k=2, F=128, S=1, norm=True, B=1, T=8,
         dtype="fp32", seed=2, avail_p=1.01, mode="eval"),
    dict(name="tiny_k1_placeholder", H=64, E=2, k=1, F=128, S=1, norm=False, B=1, T=4,
         dtype="fp32", seed=3, avail_p=0.5, mode="eval", force_mask=[False, True]),
    dict(name="tiny_sh2_norm", H=128, E=6, k=3, F=128, S=2, norm=True, B=2, T=8,
         dtype="fp32", seed=4, avail_p=0.5, mode="eval"),
    dict(name="tiny_sh0", H=64, E=4, k=2, F=128, S=0, norm=False, B=1, T=12,
         dtype="fp32", seed=5, avail_p=0.5, mode="eval"),
    dict(name="eval_stale", H=64, E=4, k=2, F=128, S=1, norm=True, B=1, T=12,
         dtype="fp32", seed=6, avail_p=0.5, mode="eval_stale"),
    dict(name="train_mask", H=64, E=4, k=2, F=128, S=1, norm=False, B=1, T=12,
         dtype="fp32", seed=7, avail_p=None, mode="train_mask",
         float_mask=[0.0, 0.3, 1.0, 0.0]),
    dict(name="bf16_small", H=128, E=8, k=2, F=256, S=1, norm=True, B=4, T=16,
         dtype="bf16", seed=8, avail_p=0.75, mode="eval"),
    dict(name="decode_shape_bf16", H=2048, E=64, k=6, F=1408, S=2, norm=True, B=8, T=1,
         dtype="bf16", seed=9, avail_p=0.9, mode="eval"),
    # the decode workload's batch ends at full shape (DeepSeek-MoE-16B layer)
    dict(name="decode_b1_bf16", H=2048, E=64, k=6, F=1408, S=2, norm=True, B=1, T=1,
         dtype="bf16", seed=10, avail_p=0.9, mode="eval"),
    dict(name="decode_b64_bf16", H=2048, E=64, k=6, F=1408, S=2, norm=True, B=64, T=1,
         dtype="bf16", seed=11, avail_p=0.9, mode="eval"),
    # a 256-token slice of the prefill workload: Zipf(1.1)-biased router, all available
    dict(name="prefill_zipf256_bf16", H=2048, E=64, k=6, F=1408, S=2, norm=True, B=1, T=256,
         dtype="bf16", seed=12, avail_p=None, mode="nomask", zipf=1.1),
    # training-mode forwards: the load-balance aux loss (moe_chronos.py:175-188)
    dict(name="train_nomask_aux", H=64, E=8, k=2, F=128, S=1, norm=True, B=2, T=10,
         dtype="fp32", seed=13, avail_p=None, mode="train_nomask", aux_coef=0.01),
    # training-time miss simulation, fallback_mask_prob > 0 (moe_chronos.py:132-144)
    dict(name="train_fallback", H=64, E=8, k=2, F=128, S=1, norm=True, B=2, T=10,
         dtype="fp32", seed=14, avail_p=None, mode="train_fallback", fallback_p=0.5,
         rng_seed=3, aux_coef=0.01),
]

LOOKAHEAD_CASES = [
    dict(name="lookahead_fp32", H=256, E=16, steps=2, B=2, S=5, dtype="fp32", seed=30),
    dict(name="lookahead_bf16", H=1024, E=64, steps=2, B=1, S=8, dtype="bf16", seed=31),
    # the 8-layer decode model's shape: d_model 1024, 16 experts, batch 32
    dict(name="lookahead_decode_bf16", H=1024, E=16, steps=2, B=32, S=1, dtype="bf16", seed=32),
]

CTSR = dict(name="ctsr_ref", H=32, E=4, F=64, S=1, L=2, clusters=[[0, 2], [1, 3]], seeds=[40, 41])

# A small hybrid-attention model (MLA on even layers, sliding window on odd),
# run teacher-forced: a prompt, then one cached token per step past the window.
MODEL = dict(name="model_tf", seed=50, ids_seed=51, B=2, prompt=8, steps=8,
             config=dict(vocab_size=512, hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                         num_key_value_heads=2, max_position_embeddings=64, num_experts=8,
                         num_experts_per_tok=2, moe_intermediate_size=256, num_shared_experts=1,
                         norm_topk_prob=True, kv_latent_dim=64, rope_dim=32, sliding_window_size=12,
                         lookahead_steps=2, dropout=0.0, hidden_act="silu", flash_attn=True,
                         rms_norm_eps=1e-5, rope_theta=1e6, tie_word_embeddings=True,
                         fallback_mask_prob=0.0))


def import_reference(ref_root: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(SHIM))
    sys.path.insert(0, ref_root)
    deps = types.ModuleType("chronos.deps")
    deps.ensure_minimind = lambda: SHIM
    deps.get_tokenizer_path = lambda: str(SHIM / "model")
    deps._minimind_root = SHIM
    sys.modules["chronos.deps"] = deps
    from chronos.model.config import ChronosConfig
    from chronos.model.moe_chronos import ChronosMOEFeedForward, LazyExpertPlaceholder
    return ChronosConfig, ChronosMOEFeedForward, LazyExpertPlaceholder


def case_inputs(c):
    from project_chronos_b200 import synthetic as syn
    shape = syn.MoEShape(c["H"], c["E"], c["k"], c["F"], c["S"], c["norm"])
    n = c["B"] * c["T"]
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    wl = syn.make_workload(shape, n, seed=c["seed"], dtype=dt, avail_p=c["avail_p"],
                           zipf_s=c.get("zipf"))
    mask = wl.mask
    if c.get("force_mask") is not None:
        mask = torch.tensor(c["force_mask"], dtype=torch.bool)
    return shape, wl, mask


def build_module(refs, c, w, dtype, bias=None):
    ChronosConfig, ChronosMOEFeedForward, _ = refs
    cfg = ChronosConfig(hidden_size=c["H"], num_experts=c["E"], num_experts_per_tok=c["k"],
                        moe_intermediate_size=c["F"], num_shared_experts=c["S"],
                        norm_topk_prob=c["norm"], hidden_act="silu", dropout=0.0,
                        fallback_mask_prob=float(c.get("fallback_p", 0.0)),
                        router_aux_loss_coef=float(c.get("aux_coef", 5e-4)))
    m = ChronosMOEFeedForward(cfg).to(dtype)
    with torch.no_grad():
        if bias is not None:
            # the benchmark's logit offset, as a bias of the reference's own gate
            m.gate = torch.nn.Linear(c["H"], c["E"], bias=True).to(dtype)
            m.gate.bias.copy_(bias.to(dtype))
        m.gate.weight.copy_(w.router.to(dtype))
        for e in range(c["E"]):
            m.experts[e].gate_proj.weight.copy_(w.gate[e].to(dtype))
            m.experts[e].up_proj.weight.copy_(w.up[e].to(dtype))
            m.experts[e].down_proj.weight.copy_(w.down[e].to(dtype))
        for j in range(c["S"]):
            m.shared_experts[j].gate_proj.weight.copy_(w.sh_gate[j].to(dtype))
            m.shared_experts[j].up_proj.weight.copy_(w.sh_up[j].to(dtype))
            m.shared_experts[j].down_proj.weight.copy_(w.sh_down[j].to(dtype))
    return m, cfg


def run_reference(refs, c, wl, mask, dtype):
    _, _, LazyExpertPlaceholder = refs
    m, cfg = build_module(refs, c, wl.weights, dtype, bias=wl.bias)
    mode = c["mode"]
    fwd_mask = None
    if mode == "eval":
        m.eval()
        for e in range(c["E"]):
            if not bool(mask[e]):
                m.experts[e] = LazyExpertPlaceholder(c["H"], c["F"], dtype)
        fwd_mask = mask
    elif mode == "eval_stale":
        m.eval()
        fwd_mask = mask
    elif mode == "train_mask":
        m.train()
        fwd_mask = torch.tensor(c["float_mask"], dtype=torch.float32)
    elif mode in ("train_nomask", "train_fallback"):
        m.train()
    else:
        m.eval()
    x = wl.x.to(dtype).view(c["B"], c["T"], c["H"])
    if mode == "train_fallback":
        torch.manual_seed(c["rng_seed"])
    with torch.no_grad():
        y = m(x, available_expert_mask=fwd_mask)
    probs = m.last_router_probs.reshape(-1, c["E"]).float()
    return m, y.reshape(-1, c["H"]).float(), probs


def moe_case(refs, c):
    shape, wl, mask = case_inputs(c)
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    m, y, probs = run_reference(refs, c, wl, mask, dt)
    out = {}
    entry = dict(c)
    if c["dtype"] != "fp32":
        out["y_ref"] = bf16_bits(y)
        m32, y32, probs32 = run_reference(refs, c, wl, mask, torch.float32)
        out["y_ref_fp32"] = y32.numpy().astype(np.float32)
        # the literal bf16 routing: bf16 probabilities, torch.topk (moe_chronos.py:112, 124-128)
        lit = torch.topk(m.last_router_probs.reshape(-1, c["E"]), c["k"], dim=-1, sorted=False).indices
        out["idx_lit"] = np.sort(lit.numpy(), axis=1).astype(np.int32)
        out["probs_lit"] = bf16_bits(probs)
        l64 = wl.x.double() @ wl.weights.router.double().T
        l64_lit = l64
        if wl.bias is not None:
            # the literal path's gate bias is a bf16 parameter
            l64_lit = l64 + wl.bias.to(torch.bfloat16).double()
            l64 = l64 + wl.bias.double()
        out["logits64"] = l64.numpy()
        out["logits64_lit"] = l64_lit.numpy()
        m_book = m32
        probs = probs32
    else:
        out["y_ref"] = y.numpy().astype(np.float32)
        m_book = m
    topv, topi = torch.topk(probs, c["k"], dim=-1)
    order = torch.argsort(topi, dim=-1)
    idx_sorted = torch.gather(topi, 1, order)
    w_sorted = torch.gather(topv, 1, order)
    if c["norm"]:
        w_sorted = w_sorted / (w_sorted.sum(-1, keepdim=True) + 1e-20)
    out["idx_ref"] = idx_sorted.numpy().astype(np.int32)
    out["w_ref"] = w_sorted.numpy().astype(np.float32)
    out["probs_ref"] = probs.numpy().astype(np.float32)
    if c["mode"] == "train_fallback":
        torch.manual_seed(c["rng_seed"])
        draws = torch.rand(c["E"])  # the reference's first RNG use in forward (moe_chronos.py:141)
        keep = draws >= c["fallback_p"]
        if not bool(keep.any()):
            raise SystemExit(f"{c['name']}: pick another rng_seed (no expert kept)")
        out["keep_draws"] = draws.numpy().astype(np.float32)
        entry["keep"] = [bool(v) for v in keep.tolist()]
    np.savez_compressed(HERE / f"{c['name']}.npz", **out)
    entry["mask"] = None if mask is None else [bool(v) for v in mask.tolist()]
    entry["on_demand"] = list(m_book.last_on_demand_experts)
    entry["fallback"] = list(m_book.last_fallback_experts)
    entry["on_demand_mass"] = float(m_book.last_on_demand_weight_mass)
    entry["fallback_mass"] = float(m_book.last_fallback_weight_mass)
    if c["mode"].startswith("train"):
        entry["aux_loss_raw"] = float(m_book.aux_loss_raw)
        entry["aux_loss"] = float(m_book.aux_loss)
    if c["dtype"] != "fp32":
        entry["literal_bf16_routing"] = classify_literal(
            out["idx_lit"], out["idx_ref"], G_from_bits(out["probs_lit"]), out["logits64"],
            out["logits64_lit"])
    lit = entry.get("literal_bf16_routing")
    print(f"{c['name']}: y norm {float(y.norm()):.4f}  fallback {entry['fallback']} "
          f"on_demand {entry['on_demand']}" + (f"  literal-bf16 {lit}" if lit else ""))
    return entry


def lookahead_case(ref_root, c):
    from chronos.model.lookahead_router import LookaheadRouter
    cfg = types.SimpleNamespace(hidden_size=c["H"], num_experts=c["E"], lookahead_steps=c["steps"])
    g = torch.Generator().manual_seed(c["seed"])
    K = c["steps"] + 1
    w1 = (torch.randn(c["H"] // 4, c["H"], generator=g) * 0.05)
    w2 = (torch.randn(c["E"] * K, c["H"] // 4, generator=g) * 0.05)
    x = torch.randn(c["B"], c["S"], c["H"], generator=g)
    out = {}
    src = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    w1, w2, x = (t.to(src).float() for t in (w1, w2, x))   # the case's values
    for key, dt in (("probs_ref", src), ("probs_ref_fp32", torch.float32)):
        if key == "probs_ref_fp32" and c["dtype"] == "fp32":
            continue
        m = LookaheadRouter(cfg)
        with torch.no_grad():
            m.proj[0].weight.copy_(w1)
            m.proj[2].weight.copy_(w2)
        m = m.to(dt).eval()
        with torch.no_grad():
            out[key] = m(x.to(dt)).float().numpy()
    np.savez_compressed(HERE / f"{c['name']}.npz", **out)
    print(f"{c['name']}: probs {out['probs_ref'].shape}")
    return dict(c)


def ctsr_fixture(refs):
    from chronos.io.storage import ClusterStorage
    from project_chronos_b200 import synthetic as syn
    c = CTSR
    layers = []
    for li in range(c["L"]):
        cc = dict(H=c["H"], E=c["E"], k=2, F=c["F"], S=c["S"], norm=True)
        wl = syn.make_workload(syn.MoEShape(c["H"], c["E"], 2, c["F"], c["S"]), 1, seed=c["seeds"][li])
        m, _ = build_module(refs, cc, wl.weights, torch.float32)
        layers.append(m)
    out_dir = HERE / c["name"]
    if out_dir.exists():
        shutil.rmtree(out_dir)
    ClusterStorage.write_clusters(layers, c["clusters"], str(out_dir), c["L"], c["E"])
    print(f"{c['name']}: {sorted(os.listdir(out_dir))}")
    return dict(c)


ATTN = dict(name="attn_decode", B=2, steps=12, seed=60, x_seed=61,
            config=dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, kv_latent_dim=64,
                        rope_dim=32, sliding_window_size=5, max_position_embeddings=64, rms_norm_eps=1e-5,
                        dropout=0.0, flash_attn=True, rope_theta=1e6))


def attn_case(refs):
    """The reference's MLAAttention and SlidingWindowAttention
    (chronos/model/hybrid_attention.py:62-258) stepped one token at a time with
    their own caches (past the window), fp32: the output of every step."""
    from chronos.model.hybrid_attention import MLAAttention, SlidingWindowAttention
    from model.model_minimind import precompute_freqs_cis
    from project_chronos_b200 import synthetic as syn
    c = ATTN
    cfg = refs[0](**c["config"])
    cos, sin = precompute_freqs_cis(dim=cfg.head_dim, end=cfg.max_position_embeddings, rope_base=cfg.rope_theta)
    g = torch.Generator().manual_seed(c["x_seed"])
    xs = torch.randn(c["steps"], c["B"], 1, cfg.hidden_size, generator=g)
    out, shapes = {"x": xs.numpy()}, {}
    for tag, cls, seed in (("mla", MLAAttention, c["seed"]), ("sw", SlidingWindowAttention, c["seed"] + 1)):
        m = cls(cfg).eval()
        shp = {k: v.shape for k, v in m.state_dict().items()}
        shapes[tag] = {k: list(v) for k, v in shp.items()}
        m.load_state_dict(syn.model_state(shp, seed))
        past, ys = None, []
        with torch.no_grad():
            for t in range(c["steps"]):
                y, past = m(xs[t], (cos, sin), past, use_cache=True)
                ys.append(y[:, 0])
        out[f"y_{tag}"] = torch.stack(ys).numpy()
    np.savez_compressed(HERE / f"{c['name']}.npz", **out)
    print(f"{c['name']}: {out['y_mla'].shape} / {out['y_sw'].shape}")
    return dict(c, state_shapes=shapes, head_dim=cfg.head_dim)


def model_case(refs):
    """Teacher-forced logits of the reference's ChronosForCausalLM
    (chronos/model/model_chronos.py:166-222): the prompt's last position, then
    one cached token per step; in fp32 and in bf16 on the same bf16-valued weights."""
    from chronos.model.model_chronos import ChronosForCausalLM
    from project_chronos_b200 import synthetic as syn
    ChronosConfig = refs[0]
    c = MODEL
    cfg = ChronosConfig(**c["config"])
    ref = ChronosForCausalLM(cfg)
    shapes = {k: v.shape for k, v in ref.state_dict().items() if k != "lm_head.weight"}
    state = {k: v.to(torch.bfloat16).float() for k, v in syn.model_state(shapes, c["seed"]).items()}
    g = torch.Generator().manual_seed(c["ids_seed"])
    ids = torch.randint(0, cfg.vocab_size, (c["B"], c["prompt"] + c["steps"]), generator=g)
    out = {}
    for tag, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        m = ChronosForCausalLM(cfg)
        missing, unexpected = m.load_state_dict(state, strict=False)
        assert set(missing) <= {"lm_head.weight"} and not unexpected, (missing, unexpected)
        m = m.to(dt).eval()
        logits, look = [], []
        with torch.no_grad():
            o, lp = m(ids[:, :c["prompt"]], use_cache=True)
            logits.append(o.logits[:, -1].float())
            look.append(lp[:, -1].float())
            pkv = o.past_key_values
            for t in range(c["steps"]):
                j = c["prompt"] + t
                o, lp = m(ids[:, j:j + 1], past_key_values=pkv, use_cache=True)
                logits.append(o.logits[:, -1].float())
                look.append(lp[:, -1].float())
                pkv = o.past_key_values
        out[f"logits_{tag}"] = torch.stack(logits).numpy()
        out[f"lookahead_{tag}"] = torch.stack(look).numpy()
    out["ids"] = ids.numpy().astype(np.int64)
    np.savez_compressed(HERE / f"{c['name']}.npz", **out)
    rel = float(np.linalg.norm(out["logits_bf16"] - out["logits_fp32"]) / np.linalg.norm(out["logits_fp32"]))
    print(f"{c['name']}: logits {out['logits_fp32'].shape}, bf16 vs fp32 rel-L2 {rel:.3e}")
    return dict(c, reference_bf16_vs_fp32=rel,
                state_shapes={k: list(v.shape) for k, v in ref.state_dict().items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    refs = import_reference(args.ref)
    torch.manual_seed(0)
    path = HERE / "cases.json"
    old = json.load(open(path)) if path.exists() else {}
    moe = {c["name"]: c for c in old.get("cases", [])}
    look = {c["name"]: c for c in old.get("lookahead", [])}
    ctsr = old.get("ctsr")
    for c in CASES:
        if not args.only or c["name"] == args.only:
            moe[c["name"]] = moe_case(refs, c)
    for c in LOOKAHEAD_CASES:
        if not args.only or c["name"] == args.only:
            look[c["name"]] = lookahead_case(args.ref, c)
    if not args.only or args.only == CTSR["name"]:
        ctsr = ctsr_fixture(refs)
    attn = old.get("attn")
    if not args.only or args.only == ATTN["name"]:
        attn = attn_case(refs)
    model = old.get("model")
    if not args.only or args.only == MODEL["name"]:
        model = model_case(refs)
    with open(path, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                   "cases": [moe[c["name"]] for c in CASES if c["name"] in moe],
                   "lookahead": [look[c["name"]] for c in LOOKAHEAD_CASES if c["name"] in look],
                   "ctsr": ctsr, "attn": attn, "model": model}, f, indent=1)


if __name__ == "__main__":
    main()
