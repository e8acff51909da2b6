"""Generate golden vectors for the MoE layer from the REFERENCE implementation.

Run in the build container (the only place the reference tree exists):

    python tests/golden/make_golden.py [--ref /root/reference]

It imports FonaTech/Project_Chronos's own ``chronos.model.moe_chronos``
(unmodified) with ``tests/golden/minimind_shim`` standing in for the absent
third-party minimind package and a stub ``chronos.deps`` that points the
reference's bootstrap at that shim instead of cloning from the network
(``chronos/deps.py:49-72``).  For every case below it rebuilds the seeded
inputs with ``project_chronos_b200.synthetic`` (CPU generator), runs the
reference layer on the CPU in eval mode (or train mode where the case says so)
and stores the reference outputs in ``tests/golden/<case>.npz``; the case
parameters go to ``tests/golden/cases.json``.  Inputs are NOT stored: tests
regenerate them from the same seeds.

Unavailable experts are replaced by the reference's ``LazyExpertPlaceholder``
(as ``tests/test_smoke.py:147-167`` of the reference does), because in eval
mode the reference only takes the shared-expert fallback for placeholder
experts (``moe_chronos.py:220-227``).

Stored per case (all from the reference):
  y_ref        layer output in the case dtype, as fp32          [N, H]
  y_ref_fp32   (bf16 cases) the reference run in fp32 on the same bf16-valued
               weights and inputs                                [N, H]
  idx_ref      top-k indices per token, sorted ascending          [N, k]
  w_ref        top-k weights aligned with idx_ref (fp32 run)      [N, k]
  probs_ref    router probabilities (fp32 run)                    [N, E]
  on_demand / fallback   the reference's last_on_demand_experts /
               last_fallback_experts lists, and their weight masses.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
SHIM = HERE / "minimind_shim"

# Cases: shape (H, E, k, F, S_h), tokens as (B, S), dtype, seed, availability
# probability (None = no mask), mode: "eval" (placeholders for unavailable
# experts), "eval_stale" (mask given but every expert live), "train_mask"
# (train mode, dropout 0, float mask, no placeholders), "nomask".
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
]


def import_reference(ref_root: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(SHIM))
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(REPO))
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
    wl = syn.make_workload(shape, n, seed=c["seed"], dtype=dt, avail_p=c["avail_p"])
    mask = wl.mask
    if c.get("force_mask") is not None:
        mask = torch.tensor(c["force_mask"], dtype=torch.bool)
    return shape, wl, mask


def build_module(refs, c, w, dtype):
    ChronosConfig, ChronosMOEFeedForward, _ = refs
    cfg = ChronosConfig(hidden_size=c["H"], num_experts=c["E"], num_experts_per_tok=c["k"],
                        moe_intermediate_size=c["F"], num_shared_experts=c["S"],
                        norm_topk_prob=c["norm"], hidden_act="silu", dropout=0.0,
                        fallback_mask_prob=0.0)
    m = ChronosMOEFeedForward(cfg).to(dtype)
    with torch.no_grad():
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
    m, cfg = build_module(refs, c, wl.weights, dtype)
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
    else:
        m.eval()
    x = wl.x.to(dtype).view(c["B"], c["T"], c["H"])
    with torch.no_grad():
        y = m(x, available_expert_mask=fwd_mask)
    probs = m.last_router_probs.reshape(-1, c["E"]).float()
    return m, y.reshape(-1, c["H"]).float(), probs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    refs = import_reference(args.ref)
    torch.manual_seed(0)
    manifest = []
    for c in CASES:
        if args.only and c["name"] != args.only:
            continue
        shape, wl, mask = case_inputs(c)
        dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
        m, y, probs = run_reference(refs, c, wl, mask, dt)
        out = {"y_ref": y.numpy().astype(np.float32)}
        if c["dtype"] != "fp32":
            m32, y32, probs32 = run_reference(refs, c, wl, mask, torch.float32)
            out["y_ref_fp32"] = y32.numpy().astype(np.float32)
            probs = probs32
            m_book = m32
        else:
            m_book = m
        p = probs.numpy()
        topv, topi = torch.topk(probs, c["k"], dim=-1)
        order = torch.argsort(topi, dim=-1)
        idx_sorted = torch.gather(topi, 1, order)
        w_sorted = torch.gather(topv, 1, order)
        if c["norm"]:
            w_sorted = w_sorted / (w_sorted.sum(-1, keepdim=True) + 1e-20)
        out["idx_ref"] = idx_sorted.numpy().astype(np.int32)
        out["w_ref"] = w_sorted.numpy().astype(np.float32)
        out["probs_ref"] = p.astype(np.float32)
        np.savez_compressed(HERE / f"{c['name']}.npz", **out)
        entry = dict(c)
        entry["mask"] = None if mask is None else [bool(v) for v in mask.tolist()]
        entry["on_demand"] = list(m_book.last_on_demand_experts)
        entry["fallback"] = list(m_book.last_fallback_experts)
        entry["on_demand_mass"] = float(m_book.last_on_demand_weight_mass)
        entry["fallback_mass"] = float(m_book.last_fallback_weight_mass)
        manifest.append(entry)
        print(f"{c['name']}: y norm {float(y.norm()):.4f}  fallback {entry['fallback']} "
              f"on_demand {entry['on_demand']}")
    if not args.only:
        with open(HERE / "cases.json", "w") as f:
            json.dump({"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                       "cases": manifest}, f, indent=1)


if __name__ == "__main__":
    main()
