"""The CPU oracle against the golden vectors made by the reference itself."""
import numpy as np
import pytest
import torch

from tests import _golden as G

from oracle import moe_oracle as O  # noqa: E402


def _np(t):
    return t.float().numpy()


def _bias(wl):
    return None if wl.bias is None else _np(wl.bias)


@pytest.mark.parametrize("name", [c["name"] for c in G.cases()])
def test_oracle_matches_reference(name):
    c = G.case(name)
    d = G.load(c)
    wl = G.inputs(c)
    w = wl.weights
    y, idx, wt, probs = O.moe_forward(
        _np(wl.x), _np(w.router), _np(w.gate), _np(w.up), _np(w.down), _np(w.sh_gate),
        _np(w.sh_up), _np(w.sh_down), c["k"], c["norm"], avail=G.effective_avail(c), bias=_bias(wl))
    # routing: same expert set per token as the reference (bit-exact indices)
    assert np.array_equal(np.sort(idx, axis=1), d["idx_ref"])
    order = np.argsort(idx, axis=1)
    np.testing.assert_allclose(np.take_along_axis(wt, order, 1), d["w_ref"], rtol=2e-6,
                               atol=1e-7)
    np.testing.assert_allclose(probs, d["probs_ref"], rtol=2e-6, atol=1e-7)
    # output: fp32 reference (for bf16 cases: the reference in fp32 on the bf16 values)
    assert O.rel_l2(y, G.reference_y(c, d)) < 2e-6
    if "aux_loss_raw" in c:
        aux = O.aux_loss(idx, probs, c["E"])
        assert abs(aux - c["aux_loss_raw"]) <= 1e-5 * max(1.0, abs(c["aux_loss_raw"]))
        coef = c.get("aux_coef", 5e-4)
        assert abs(aux * coef - c["aux_loss"]) <= 1e-5 * max(abs(c["aux_loss"]), 1e-6)


@pytest.mark.parametrize("name", [c["name"] for c in G.cases() if c["dtype"] == "bf16"])
def test_literal_bf16_routing_mismatches_are_explained(name):
    """The reference's literal bf16 path (bf16 gate GEMM, bf16 softmax, torch.topk)
    against the fp32 routing contract: every token whose expert set differs is a
    bf16 tie or a bf16 rounding of the logits, and the counts are the published ones."""
    c = G.case(name)
    d = G.load(c)
    got = G.classify_literal(d["idx_lit"], d["idx_ref"], d["probs_lit"], d["logits64"],
                             d.get("logits64_lit"))
    assert got == c["literal_bf16_routing"]
    assert got["other"] == 0
    # and the contract's sets are exactly the oracle's
    wl = G.inputs(c)
    idx, _, _, _ = O.route(_np(wl.x), _np(wl.weights.router), c["k"], c["norm"], bias=_bias(wl))
    assert np.array_equal(np.sort(idx, axis=1), d["idx_ref"])


def test_fallback_draws_give_the_recorded_keep_mask():
    # moe_chronos.py:141-143: keep = rand(E) >= p (at least one kept)
    c = G.case("train_fallback")
    d = G.load(c)
    keep = d["keep_draws"] >= c["fallback_p"]
    assert keep.tolist() == c["keep"] and keep.any()
    torch.manual_seed(c["rng_seed"])
    assert np.array_equal(torch.rand(c["E"]).numpy(), d["keep_draws"])


@pytest.mark.parametrize("name", [c["name"] for c in G.lookahead_cases()])
def test_lookahead_oracle_matches_reference(name):
    c = G.case(name)
    d = G.load(c)
    w1, w2, x = G.lookahead_inputs(c)
    if c["dtype"] == "bf16":
        w1, w2, x = (t.to(torch.bfloat16).float() for t in (w1, w2, x))
    n = c["B"] * c["S"]
    got = O.lookahead(x.reshape(n, c["H"]).numpy(), w1.numpy(), w2.numpy(), c["E"], c["steps"] + 1)
    want = d["probs_ref_fp32" if c["dtype"] == "bf16" else "probs_ref"].reshape(n, c["steps"] + 1, c["E"])
    assert np.abs(got - want).max() < 2e-6
    if c["dtype"] == "bf16":
        # the reference's own bf16 run rounds every intermediate to bf16
        lit = d["probs_ref"].reshape(n, c["steps"] + 1, c["E"])
        assert np.abs(got - lit).max() < 1e-2


def test_oracle_rank_order_and_ties():
    # all-equal logits: ties go to the lower index, in rank order
    x = np.ones((3, 8), np.float32)
    w = np.zeros((5, 8), np.float32)
    idx, wt, probs, logits = O.route(x, w, 3, norm_topk=False)
    assert idx.tolist() == [[0, 1, 2]] * 3
    np.testing.assert_allclose(wt, 0.2, rtol=1e-6)
    # distinct logits: descending order
    w = np.arange(5, dtype=np.float32)[:, None] * np.ones((5, 8), np.float32)
    idx, wt, _, _ = O.route(x, w, 2, norm_topk=True)
    assert idx.tolist() == [[4, 3]] * 3
    np.testing.assert_allclose(wt.sum(1), 1.0, rtol=1e-6)


def test_oracle_logits_are_in_order_sums_of_chunk_fma_chains():
    # routing contract: partial = fmaf chain over each 128-wide chunk of h,
    # logit = in-order fp32 sum of the partials starting from 0
    import math
    rng = np.random.default_rng(0)
    h = 300
    x = rng.standard_normal((4, h)).astype(np.float32)
    w = rng.standard_normal((3, h)).astype(np.float32)
    _, _, _, logits = O.route(x, w, 1, norm_topk=False)

    def fma32(a, b, c):
        # exact fp32 product in double, correctly rounded sum, then fp32; this
        # double rounding differs from fmaf only on rare halfway cases (none here)
        return np.float32(math.fsum([float(a) * float(b), float(c)]))

    for t in range(4):
        for e in range(3):
            total = np.float32(0.0)
            for c0 in range(0, h, 128):
                acc = np.float32(0.0)
                for i in range(c0, min(h, c0 + 128)):
                    acc = fma32(x[t, i], w[e, i], acc)
                total = np.float32(total + acc)
            assert logits[t, e] == total


def test_bf16_rounding_helper():
    v = np.array([1.0, 1.00390625, 1.005859375, -3.0e-3, 65504.0], np.float32)
    want = torch.tensor(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.round_to_bf16(v), want)


def test_all_available_equals_no_mask():
    # moe_chronos.py masked path with an all-true mask == the standard path
    # (reference tests/test_smoke.py:1099-1115)
    a, b = G.load(G.case("tiny_allmask")), G.load(G.case("tiny_nomask"))
    assert np.abs(a["y_ref"] - b["y_ref"]).max() < 1e-6
