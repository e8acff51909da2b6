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
    import torch
    want = torch.tensor(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.round_to_bf16(v), want)


def test_all_available_equals_no_mask():
    # moe_chronos.py masked path with an all-true mask == the standard path
    # (reference tests/test_smoke.py:1099-1115)
    a, b = G.load(G.case("tiny_allmask")), G.load(G.case("tiny_nomask"))
    assert np.abs(a["y_ref"] - b["y_ref"]).max() < 1e-6
