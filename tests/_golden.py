"""Helpers that rebuild the golden cases' inputs and load their reference outputs."""
import json
import os

import numpy as np
import torch

from project_chronos_b200 import synthetic as syn

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _manifest():
    with open(os.path.join(GOLDEN, "cases.json")) as f:
        return json.load(f)


def cases():
    return _manifest()["cases"]


def lookahead_cases():
    return _manifest()["lookahead"]


def ctsr_fixture():
    """(directory, parameters) of the cluster files the reference wrote."""
    c = _manifest()["ctsr"]
    return os.path.join(GOLDEN, c["name"]), c


def case(name):
    for c in cases() + lookahead_cases():
        if c["name"] == name:
            return c
    raise KeyError(name)


def bf16_bits(t) -> np.ndarray:
    """A float tensor rounded to bf16, as its uint16 bit patterns."""
    return t.detach().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def load(c):
    d = np.load(os.path.join(GOLDEN, f"{c['name']}.npz"))
    out = {k: d[k] for k in d.files}
    for k in ("y_ref", "probs_lit"):
        if k in out and out[k].dtype == np.uint16:
            out[k] = from_bf16_bits(out[k])
    return out


def inputs(c, device="cpu"):
    """The case's workload, generated on the CPU (as the fixtures were)."""
    shape = syn.MoEShape(c["H"], c["E"], c["k"], c["F"], c["S"], c["norm"])
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    wl = syn.make_workload(shape, c["B"] * c["T"], seed=c["seed"], dtype=dt,
                           avail_p=c["avail_p"], zipf_s=c.get("zipf"))
    if device != "cpu":
        wl = syn.Workload(wl.shape, wl.weights.to(device=device), wl.x.to(device),
                          wl.mask, None if wl.bias is None else wl.bias.to(device))
    return wl


def lookahead_inputs(c):
    """(w1, w2, x [B, S, H]) of a lookahead case, fp32, drawn as the generator drew them."""
    g = torch.Generator().manual_seed(c["seed"])
    K = c["steps"] + 1
    w1 = torch.randn(c["H"] // 4, c["H"], generator=g) * 0.05
    w2 = torch.randn(c["E"] * K, c["H"] // 4, generator=g) * 0.05
    x = torch.randn(c["B"], c["S"], c["H"], generator=g)
    return w1, w2, x


def effective_avail(c):
    """a_e the reference applies in the case's mode (moe_chronos.py:220-227)."""
    if c["mode"] == "eval":
        return np.array(c["mask"], dtype=np.float32)
    if c["mode"] == "train_mask":
        return (np.array(c["float_mask"], dtype=np.float32) > 0).astype(np.float32)
    if c["mode"] == "train_fallback":
        return np.array(c["keep"], dtype=np.float32)
    return None


def reference_y(c, d):
    return d["y_ref_fp32"] if "y_ref_fp32" in d else d["y_ref"]


def _bf16_round(a):
    return from_bf16_bits(bf16_bits(torch.from_numpy(np.ascontiguousarray(a, np.float32))))


def _bf16_ulp(v):
    e = np.floor(np.log2(np.maximum(np.abs(v), 1e-30)))
    return np.exp2(e - 7)


def classify_literal(idx_lit, idx_ref, probs_lit, logits64, logits64_lit=None) -> dict:
    """Tokens whose top-k set under the literal bf16 path (bf16 GEMM, bf16 softmax,
    torch.topk) differs from the fp32 routing contract, each explained:

    * ``bf16_tie``: the swapped experts have EQUAL bf16 probabilities, so the
      literal path's choice among them is arbitrary (torch.topk's tie order);
    * ``logit_rounding``: the logits rounded to bf16 order the pair the other
      way round from the exact logits (the literal path rounds the gate GEMM's
      output to bf16 before the softmax, and holds a gate bias in bf16:
      ``logits64_lit`` is the exact product plus that bf16 bias);
    * ``other``: neither; ``max_other_gap_ulps`` is the exact logit gap of such
      a pair in bf16 ulps of the larger logit.
    """
    probs_lit = np.asarray(probs_lit, np.float32)
    if probs_lit.ndim != 2:
        raise ValueError("probs_lit must be [N, E]")
    lit_src = logits64 if logits64_lit is None else logits64_lit
    lb = _bf16_round(np.asarray(lit_src, np.float64).astype(np.float32))
    n = idx_lit.shape[0]
    res = dict(tokens=int(n), mismatched_tokens=0, bf16_tie=0, logit_rounding=0, other=0,
               max_other_gap_ulps=0.0)
    for t in range(n):
        lit, ref = set(idx_lit[t].tolist()), set(idx_ref[t].tolist())
        if lit == ref:
            continue
        res["mismatched_tokens"] += 1
        a_only = sorted(lit - ref, key=lambda e: -probs_lit[t, e])
        b_only = sorted(ref - lit, key=lambda e: -probs_lit[t, e])
        worst = 0
        for a, b in zip(a_only, b_only):
            if probs_lit[t, a] == probs_lit[t, b]:
                cls = 0
            elif lb[t, a] > lb[t, b] and logits64[t, a] <= logits64[t, b]:
                cls = 1
            else:
                cls = 2
                gap = (logits64[t, b] - logits64[t, a]) / _bf16_ulp(max(abs(logits64[t, a]),
                                                                         abs(logits64[t, b])))
                res["max_other_gap_ulps"] = max(res["max_other_gap_ulps"], float(gap))
            worst = max(worst, cls)
        res[("bf16_tie", "logit_rounding", "other")[worst]] += 1
    return res


def model_case():
    return _manifest()["model"]


def attn_case():
    return _manifest()["attn"]


def model_config(cfg: dict):
    """A config namespace for this package's model from a golden case's
    ChronosConfig keyword arguments, with the defaults ChronosConfig and
    minimind's config supply for the fields not given."""
    import types
    d = dict(rope_scaling=None, use_hybrid_attention=True, router_aux_loss_coef=5e-4, lookahead_steps=2,
             num_shared_experts=1, kv_latent_dim=64, rope_dim=32, sliding_window_size=2048,
             tie_word_embeddings=True, rms_norm_eps=1e-5, rope_theta=1e6, dropout=0.0, hidden_act="silu",
             fallback_mask_prob=0.0, norm_topk_prob=True)
    d.update(cfg)
    d.setdefault("intermediate_size", d.get("moe_intermediate_size"))
    d.setdefault("head_dim", d["hidden_size"] // d["num_attention_heads"])
    return types.SimpleNamespace(**d)
