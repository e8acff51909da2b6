"""The CPU oracle against the golden vectors made by the reference itself."""
import os
import sys

import numpy as np
import pytest

from tests import _golden as G

from oracle import moe_oracle as O  # noqa: E402


def _np(t):
    return t.float().numpy()


@pytest.mark.parametrize("name", [c["name"] for c in G.cases()])
def test_oracle_matches_reference(name):
    c = G.case(name)
    d = G.load(c)
    wl = G.inputs(c)
    w = wl.weights
    y, idx, wt, probs = O.moe_forward(
        _np(wl.x), _np(w.router), _np(w.gate), _np(w.up), _np(w.down), _np(w.sh_gate),
        _np(w.sh_up), _np(w.sh_down), c["k"], c["norm"], avail=G.effective_avail(c))
    # routing: same expert set per token as the reference (bit-exact indices)
    assert np.array_equal(np.sort(idx, axis=1), d["idx_ref"])
    order = np.argsort(idx, axis=1)
    np.testing.assert_allclose(np.take_along_axis(wt, order, 1), d["w_ref"], rtol=2e-6,
                               atol=1e-7)
    np.testing.assert_allclose(probs, d["probs_ref"], rtol=2e-6, atol=1e-7)
    # output: fp32 reference (for bf16 cases: the reference in fp32 on the bf16 values)
    assert O.rel_l2(y, G.reference_y(c, d)) < 2e-6


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


def test_oracle_logits_are_a_sequential_fma_chain():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 33)).astype(np.float32)
    w = rng.standard_normal((3, 33)).astype(np.float32)
    _, _, _, logits = O.route(x, w, 1, norm_topk=False)
    for t in range(4):
        for e in range(3):
            acc = np.float32(0.0)
            for h in range(33):
                acc = np.float32(np.float64(x[t, h]) * np.float64(w[e, h]) + np.float64(acc))
            assert logits[t, e] == acc


def test_bf16_rounding_helper():
    v = np.array([1.0, 1.00390625, 1.005859375, -3.0e-3, 65504.0], np.float32)
    import torch
    want = torch.tensor(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.round_to_bf16(v), want)


def test_all_available_equals_no_mask():
    # moe_chronos.py masked path with an all-true mask == the standard path
    # (reference tests/test_smoke.py:1099-1115)
    a, b = G.load(G.case("tiny_allmask")), G.load(G.case("tiny_nomask"))
    assert np.abs(a["y_ref"] - b["y_ref"]).max() < 1e-6
