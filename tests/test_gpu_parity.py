"""CUDA path vs the oracle and the reference's golden vectors (GPU; calls the C ABI).

Tolerances (written here, from the parity contract of the layer):
  * top-k indices: bit-exact against the oracle's routing (fp32 fmaf chain,
    ties -> lower index) and, as sets, against the reference's golden indices;
  * outputs: rel-L2 <= 1e-5 for fp32 layers, <= 1e-2 for bf16 layers, against
    the reference run in fp32 on the same (bf16-valued) inputs; bf16 results
    are also held to 3e-3 against the oracle's bf16-emulating mode, which
    rounds where the kernels round.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests import _golden as G

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from project_chronos_b200 import ops
    return ops


def _np(t):
    return t.detach().float().cpu().numpy()


def _run(wl, k, norm, avail=None, bias=None, **kw):
    ops = _ops()
    w = wl.weights
    return ops.moe_forward(wl.x, w.router, w.gate, w.up, w.down,
                           w.sh_gate if w.sh_gate.shape[0] else None,
                           w.sh_up if w.sh_up.shape[0] else None,
                           w.sh_down if w.sh_down.shape[0] else None, k, norm,
                           avail=avail, router_bias=bias, **kw)


def _oracle(wl, k, norm, avail=None, bias=None, rows=None, emulate=False):
    w = wl.weights
    x = _np(wl.x)
    if rows is not None:
        x = x[rows]
    dt = "bf16" if wl.x.dtype == torch.bfloat16 else ("fp16" if wl.x.dtype == torch.float16 else "fp32")
    return O.moe_forward(x, _np(w.router), _np(w.gate), _np(w.up), _np(w.down), _np(w.sh_gate),
                         _np(w.sh_up), _np(w.sh_down), k, norm,
                         avail=None if avail is None else _np(avail),
                         bias=None if bias is None else _np(bias), dtype=dt,
                         emulate_device=emulate)


@pytest.mark.parametrize("name", [c["name"] for c in G.cases()])
def test_golden_case(name):
    c = G.case(name)
    d = G.load(c)
    wl = G.inputs(c, device=DEV)
    a = G.effective_avail(c)
    avail = None if a is None else torch.tensor(a, device=DEV)
    out = _run(wl, c["k"], c["norm"], avail=avail, bias=wl.bias)
    torch.cuda.synchronize()
    _ops().check_status()
    idx = out["topk_idx"].cpu().numpy()
    # reference's expert set per token (bit-exact routing)
    assert np.array_equal(np.sort(idx, axis=1), d["idx_ref"])
    # oracle's rank order
    o_idx, o_w, o_probs, _ = O.route(_np(wl.x), _np(wl.weights.router), c["k"], c["norm"],
                                     bias=None if wl.bias is None else _np(wl.bias))
    assert np.array_equal(idx, o_idx)
    np.testing.assert_allclose(out["topk_weight"].cpu().numpy(), o_w, rtol=1e-5, atol=1e-6)
    y = _np(out["y"])
    ref = G.reference_y(c, d)
    tol = 1e-5 if c["dtype"] == "fp32" else 1e-2
    assert O.rel_l2(y, ref) <= tol, O.rel_l2(y, ref)
    if c["dtype"] != "fp32":
        emu, *_ = _oracle(wl, c["k"], c["norm"], avail=avail, bias=wl.bias, emulate=True)
        assert O.rel_l2(y, emu) <= 3e-3
        # the literal bf16 reference output (bf16 routing, bf16 index_add combine) on
        # the tokens whose expert set it shares with the routing contract
        same = (d["idx_lit"] == d["idx_ref"]).all(axis=1)
        assert O.rel_l2(y[same], d["y_ref"][same]) <= 1e-2


def _workload(h, e, k, f, s, n, dtype=torch.bfloat16, seed=0, avail_p=None, zipf=None):
    from project_chronos_b200 import synthetic as syn
    shape = syn.MoEShape(h, e, k, f, s)
    return syn.make_workload(shape, n, seed=seed, dtype=dtype, device=DEV, avail_p=avail_p,
                             zipf_s=zipf)


@pytest.mark.parametrize("n", [1, 2, 7, 16, 33, 64, 65, 200, 1100])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_path_token_counts(n, dtype):
    # covers every token-tile width (16/32/64/128), split-K decode and ragged tails
    wl = _workload(256, 16, 4, 192, 2, n, dtype=dtype, seed=n, avail_p=0.7)
    avail = wl.mask.to(torch.float32)
    out = _run(wl, 4, True, avail=avail)
    torch.cuda.synchronize()
    _ops().check_status()
    y = _np(out["y"])
    ref, o_idx, _, _ = _oracle(wl, 4, True, avail=avail)
    assert np.array_equal(out["topk_idx"].cpu().numpy(), o_idx)
    assert O.rel_l2(y, ref) <= 1e-2
    emu, *_ = _oracle(wl, 4, True, avail=avail, emulate=True)
    assert O.rel_l2(y, emu) <= 3e-3


@pytest.mark.parametrize("h,e,k,f,s", [(32, 4, 2, 48, 1), (96, 6, 3, 80, 0), (64, 9, 1, 64, 2),
                                       (128, 256, 8, 64, 1)])
def test_simt_and_odd_shapes(h, e, k, f, s):
    for dtype in (torch.float32, torch.bfloat16):
        wl = _workload(h, e, k, f, s, 37, dtype=dtype, seed=h + e, avail_p=0.6)
        avail = wl.mask.to(torch.float32)
        out = _run(wl, k, False, avail=avail)
        torch.cuda.synchronize()
        y = _np(out["y"])
        ref, o_idx, _, _ = _oracle(wl, k, False, avail=avail)
        assert np.array_equal(out["topk_idx"].cpu().numpy(), o_idx)
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        assert O.rel_l2(y, ref) <= tol


@pytest.mark.parametrize("n,h,e", [(256, 2048, 64), (257, 2048, 64), (300, 100, 256),
                                   (1000, 260, 40), (5, 100, 256)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_router_both_logit_kernels_bit_exact(n, h, e, dtype):
    # <= 256 tokens: chunk-partials kernel; larger: register-tiled kernel; odd H
    # and E exercise the ragged chunk / tile edges
    ops = _ops()
    g = torch.Generator(device=DEV)
    g.manual_seed(n + h + e)
    x = torch.randn(n, h, generator=g, device=DEV).to(dtype)
    w = (torch.randn(e, h, generator=g, device=DEV) * 0.02).to(dtype)
    k = min(8, e)
    r = ops.moe_route(x, w, k, True)
    torch.cuda.synchronize()
    o_idx, o_w, o_probs, _ = O.route(_np(x), _np(w), k, True)
    assert np.array_equal(r["topk_idx"].cpu().numpy(), o_idx)
    np.testing.assert_allclose(r["topk_weight"].cpu().numpy(), o_w, rtol=1e-5, atol=1e-6)
    counts = r["counts"].cpu().numpy()
    assert np.array_equal(counts, np.bincount(o_idx.ravel(), minlength=e))


def test_empty_input():
    wl = _workload(128, 8, 2, 128, 1, 0)
    out = _run(wl, 2, True)
    torch.cuda.synchronize()
    assert out["y"].shape == (0, 128)


def test_all_unavailable_is_shared_only():
    wl = _workload(128, 8, 2, 128, 2, 40, seed=3)
    avail = torch.zeros(8, device=DEV)
    out = _run(wl, 2, False, avail=avail)
    torch.cuda.synchronize()
    ref, *_ = _oracle(wl, 2, False, avail=avail)
    assert O.rel_l2(_np(out["y"]), ref) <= 1e-2


@pytest.mark.parametrize("n", [3, 40, 300])
def test_no_shared_experts_and_nothing_available_gives_zero(n):
    # S_h = 0 and every expert unavailable: the layer output is exactly zero
    wl = _workload(128, 8, 2, 128, 0, n, seed=n)
    out = _run(wl, 2, True, avail=torch.zeros(8, device=DEV))
    torch.cuda.synchronize()
    assert float(out["y"].float().abs().max()) == 0.0


@pytest.mark.parametrize("n,h", [(1000, 2560), (2000, 2624)])
def test_shared_experts_last_in_down_gemm(n, h):
    """Shapes whose shared-expert tiles cover the SMs: the shared experts run
    last in the down GEMM as one K = S_h * F product per tile and write the
    output rows (routed accumulator + shared term) themselves, with no
    finalize pass.  n = 1000: 128-column weight-major tiles; n = 2000:
    token-major tiles, ragged in tokens (2000 = 15 * 128 + 80) and in output
    columns (2624 = 10 * 256 + 64).  The output starts NaN-filled, so every
    row and column must be written."""
    wl = _workload(h, 16, 4, 192, 2, n, seed=n + h, avail_p=0.7)
    avail = wl.mask.to(torch.float32)
    y0 = torch.full((n, h), float("nan"), dtype=wl.x.dtype, device=DEV)
    out = _run(wl, 4, True, avail=avail, out=y0)
    torch.cuda.synchronize()
    _ops().check_status()
    y = _np(out["y"])
    assert np.isfinite(y).all()
    ref, o_idx, _, _ = _oracle(wl, 4, True, avail=avail)
    assert np.array_equal(out["topk_idx"].cpu().numpy(), o_idx)
    assert O.rel_l2(y, ref) <= 1e-2
    emu, *_ = _oracle(wl, 4, True, avail=avail, emulate=True)
    assert O.rel_l2(y, emu) <= 3e-3


@pytest.mark.parametrize("n,h", [(1000, 2560), (2000, 2624)])
def test_shared_experts_last_with_few_ctas(n, h):
    """The shared-last units wait until every CTA with routed units has counted
    itself in; with the GEMMs capped at 5 CTAs (the C ABI's max_ctas, e.g. to
    leave SMs to a concurrent all-to-all) each CTA walks many units before its
    shared-last ones and the count must still complete."""
    wl = _workload(h, 16, 4, 192, 2, n, seed=n + h + 1, avail_p=0.7)
    avail = wl.mask.to(torch.float32)
    out = _run(wl, 4, True, avail=avail, max_ctas=5)
    torch.cuda.synchronize()
    _ops().check_status()
    y = _np(out["y"])
    ref, o_idx, _, _ = _oracle(wl, 4, True, avail=avail)
    assert np.array_equal(out["topk_idx"].cpu().numpy(), o_idx)
    assert O.rel_l2(y, ref) <= 1e-2


@pytest.mark.parametrize("n", [1, 5, 64, 65, 700, 1300])
def test_one_choice_no_shared_direct_output(n):
    """k = 1, S_h = 0: the down GEMM stores the output rows itself (no fp32
    accumulator); tokens whose one expert is unavailable get exact zeros;
    fractional availability scales the row.  The output buffer starts as
    garbage (NaN-filled) so every row must be written."""
    wl = _workload(256, 8, 1, 192, 0, n, seed=40 + n)
    avail = torch.tensor([1.0, 0.0, 1.0, 0.5, 1.0, 0.0, 1.0, 1.0], device=DEV)
    y0 = torch.full((n, 256), float("nan"), dtype=wl.x.dtype, device=DEV)
    out = _run(wl, 1, False, avail=avail, out=y0)
    torch.cuda.synchronize()
    _ops().check_status()
    y = _np(out["y"])
    ref, o_idx, _, _ = _oracle(wl, 1, False, avail=avail)
    assert np.array_equal(out["topk_idx"].cpu().numpy(), o_idx)
    assert np.isfinite(y).all()
    dead = np.isin(o_idx[:, 0], [1, 5])
    assert (y[dead] == 0.0).all()
    assert O.rel_l2(y, ref) <= 1e-2
    emu, *_ = _oracle(wl, 1, False, avail=avail, emulate=True)
    assert O.rel_l2(y, emu) <= 3e-3


def test_fractional_availability_blend():
    # a_e in (0,1): y = sum w (a E + (1-a) S) + S  (chronos/mlx/moe.py:162)
    wl = _workload(128, 8, 2, 128, 1, 24, seed=5)
    avail = torch.linspace(0.0, 1.0, 8, device=DEV)
    out = _run(wl, 2, True, avail=avail)
    torch.cuda.synchronize()
    ref, *_ = _oracle(wl, 2, True, avail=avail)
    assert O.rel_l2(_np(out["y"]), ref) <= 1e-2


def test_routing_is_deterministic_and_prerouted_matches():
    wl = _workload(256, 64, 6, 128, 2, 300, seed=11)
    a = _run(wl, 6, True)
    b = _run(wl, 6, True)
    torch.cuda.synchronize()
    assert torch.equal(a["topk_idx"], b["topk_idx"])
    assert torch.equal(a["topk_weight"], b["topk_weight"])
    c = _run(wl, 6, True, topk=[a["topk_idx"], a["topk_weight"]])
    torch.cuda.synchronize()
    # the fp32 combine is summed in a run-dependent order (TMA reduce-adds), so
    # a few bf16 outputs may differ by one ulp between runs: bf16-level bound
    assert O.rel_l2(_np(c["y"]), _np(a["y"])) < 1e-3
    assert O.rel_l2(_np(b["y"]), _np(a["y"])) < 1e-3


def test_ready_flags_gate_selected_experts():
    ops = _ops()
    wl = _workload(128, 8, 2, 128, 1, 16, seed=2)
    flags = torch.ones(8, dtype=torch.int32, device=DEV)
    ok = _run(wl, 2, True, ready_flags=flags, ready_epoch=1)
    torch.cuda.synchronize()
    ops.check_status()
    ref, *_ = _oracle(wl, 2, True)
    assert O.rel_l2(_np(ok["y"]), ref) <= 1e-2
    # a flag nothing sets: the bounded wait runs out and the status word says so
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    flags[int(ok["topk_idx"][0, 0])] = 0
    _run(wl, 2, True, ready_flags=flags, ready_epoch=1, spin_limit_ns=2_000_000, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 4  # CHRONOS_ERR_EXPERT_NOT_READY
    # the context is still usable
    again = _run(wl, 2, True)
    torch.cuda.synchronize()
    assert O.rel_l2(_np(again["y"]), ref) <= 1e-2


def test_prefill_full_size_routing_bit_exact_and_sampled_output():
    from project_chronos_b200 import synthetic as syn
    wl = syn.named_workload("prefill", device=DEV)
    sh = wl.shape
    out = _run(wl, sh.top_k, sh.norm_topk, bias=wl.bias, want_stats=True)
    torch.cuda.synchronize()
    _ops().check_status()
    idx = out["topk_idx"].cpu().numpy()
    o_idx, o_w, _, _ = O.route(_np(wl.x), _np(wl.weights.router), sh.top_k, sh.norm_topk,
                               bias=_np(wl.bias))
    assert np.array_equal(idx, o_idx)
    counts = out["counts"].cpu().numpy()
    assert counts.sum() == wl.x.shape[0] * sh.top_k
    assert np.array_equal(counts, np.bincount(o_idx.ravel(), minlength=sh.num_experts))
    rows = np.random.default_rng(0).choice(wl.x.shape[0], 48, replace=False)
    ref, *_ = _oracle(wl, sh.top_k, sh.norm_topk, bias=wl.bias, rows=rows)
    assert O.rel_l2(_np(out["y"])[rows], ref) <= 1e-2


def test_custom_op_registration():
    ops = _ops()
    wl = _workload(128, 8, 2, 128, 1, 10, seed=9)
    w = wl.weights
    y, probs, idx, wt = torch.ops.chronos.moe_forward(wl.x, w.router, w.gate, w.up, w.down,
                                                      w.sh_gate, w.sh_up, w.sh_down, None, 2, True)
    torch.cuda.synchronize()
    ref = ops.moe_forward(wl.x, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up, w.sh_down, 2,
                          True)
    assert torch.equal(idx, ref["topk_idx"])
    assert O.rel_l2(_np(y), _np(ref["y"])) < 1e-3  # bf16, run-order-dependent combine


@pytest.mark.parametrize("n,h,e,k,s,dtype", [
    (1, 2048, 64, 6, 2, torch.bfloat16), (8, 2048, 64, 6, 2, torch.bfloat16),
    (33, 2048, 64, 6, 2, torch.bfloat16), (64, 2048, 64, 6, 2, torch.bfloat16),
    (32, 1024, 16, 2, 1, torch.bfloat16), (17, 256, 256, 8, 1, torch.bfloat16),
    (64, 4096, 64, 6, 0, torch.bfloat16), (3, 320, 8, 2, 1, torch.float32),
    (12, 512, 16, 1, 0, torch.bfloat16)])
def test_fused_decode_routing_matches_two_kernel_path(n, h, e, k, s, dtype):
    """Decode routing as one cluster launch (route_fused.cuh) against the logit +
    select/plan kernels: identical indices, weights, probabilities and
    statistics; the layer output equal up to the order of fp32 reduce-adds;
    indices equal to the oracle's."""
    ops = _ops()
    f = 64 if h % 64 == 0 else 48
    wl = _workload(h, e, k, f, s, n, dtype=dtype, seed=n * 7 + e, avail_p=0.8)
    avail = wl.mask.to(torch.float32)
    outs = []
    try:
        for fused in (0, 1):
            ops.set_option("fused_route", fused)
            outs.append(_run(wl, k, True, avail=avail, want_stats=True))
            torch.cuda.synchronize()
            ops.check_status()
    finally:
        ops.set_option("fused_route", 0)
    a, b = outs
    for key in ("topk_idx", "topk_weight", "probs", "counts"):
        assert torch.equal(a[key], b[key]), key
    # a float sum of atomics: its order (and last bits) is scheduling-dependent in both paths
    assert torch.allclose(a["mass"], b["mass"], rtol=1e-5, atol=1e-6)
    tol = 1e-5 if dtype == torch.float32 else 1e-3
    assert O.rel_l2(_np(b["y"]), _np(a["y"])) <= tol
    o_idx, _, _, _ = O.route(_np(wl.x), _np(wl.weights.router), k, True)
    assert np.array_equal(b["topk_idx"].cpu().numpy(), o_idx)


# shapes whose (128-token x 256-column) output tiles cover the SMs, so the shared
# experts run last in the token-major down GEMM
@pytest.mark.parametrize("n,h,e,k,f,s", [(4096, 2048, 32, 4, 256, 2), (2560, 2560, 16, 2, 128, 1),
                                         (8192, 1024, 64, 6, 192, 2)])
def test_two_phase_combine_matches_reduce_adds(n, h, e, k, f, s):
    """Large calls with the shared experts last in the token-major down GEMM:
    the two-phase combine (slot rows stored in the layer dtype, summed per token
    in choice order) against the fp32 reduce-add path and the oracle; the
    two-phase output is bitwise reproducible run to run."""
    ops = _ops()
    wl = _workload(h, e, k, f, s, n, seed=n + e, avail_p=0.85)
    avail = wl.mask.to(torch.float32)
    outs = []
    try:
        for two in (0, 1, 1):
            ops.set_option("two_phase_combine", two)
            outs.append(_run(wl, k, True, avail=avail))
            torch.cuda.synchronize()
            ops.check_status()
    finally:
        ops.set_option("two_phase_combine", 0)
    red, two, two_again = (_np(o["y"]) for o in outs)
    assert np.array_equal(two, two_again)
    assert O.rel_l2(two, red) <= 3e-3
    emu, *_ = _oracle(wl, k, True, avail=avail, emulate=True)
    assert O.rel_l2(two, emu) <= 3e-3
    ref, *_ = _oracle(wl, k, True, avail=avail)
    assert O.rel_l2(two, ref) <= 1e-2


@pytest.mark.parametrize("n", [1, 8, 33, 64, 200, 700])
def test_folded_finalize_matches_finalize_kernel(n):
    """Calls below 1024 tokens with shared experts: the down GEMM writing each
    output-column tile when its last contribution lands, against the separate
    finalize kernel and the oracle (several calls in a row: the tile counters
    are re-armed by every call's plan)."""
    ops = _ops()
    wl = _workload(512, 32, 4, 256, 2, n, seed=n + 5, avail_p=0.8)
    avail = wl.mask.to(torch.float32)
    outs = []
    try:
        for fold in (0, 1, 1, 1):
            ops.set_option("fold_finalize", fold)
            outs.append(_np(_run(wl, 4, True, avail=avail)["y"]))
            torch.cuda.synchronize()
            ops.check_status()
    finally:
        ops.set_option("fold_finalize", 0)
    for y in outs[1:]:
        assert O.rel_l2(y, outs[0]) <= 1e-3
    emu, idx, _, _ = _oracle(wl, 4, True, avail=avail, emulate=True)
    assert O.rel_l2(outs[-1], emu) <= 3e-3


@pytest.mark.parametrize("h,e,k,f,s,n", [
    (2048, 64, 6, 1408, 2, 1),    # the DeepSeek-MoE-16B decode shape, one token: 2-way split
    (2048, 64, 6, 512, 2, 1),     # few weight-row tiles: 4-way split
    (2048, 64, 6, 1408, 2, 2),
    (1024, 16, 2, 2048, 1, 1),
])
def test_gateup_k_split_matches_unsplit(h, e, k, f, s, n):
    """Decode calls whose gate/up units would not cover the SMs split the routed
    units along K; the split completing a tile sums the fp32 partials in split
    order.  Against the unsplit path, the oracle, and itself on consecutive calls
    (the tile counters are re-armed by every call's plan; the down GEMM's fp32
    reduce-adds land in any order, so repeated calls agree to rounding, not bitwise)."""
    ops = _ops()
    wl = _workload(h, e, k, f, s, n, seed=n + f, avail_p=0.8)
    avail = wl.mask.to(torch.float32)
    outs = []
    try:
        for split in (1, 1, 0):
            ops.set_option("gateup_split", split)
            outs.append(_np(_run(wl, k, True, avail=avail)["y"]))
            torch.cuda.synchronize()
            ops.check_status()
    finally:
        ops.set_option("gateup_split", 0)
    split, split_again, whole = outs
    assert O.rel_l2(split_again, split) <= 1e-3
    assert O.rel_l2(split, whole) <= 1e-3
    emu, *_ = _oracle(wl, k, True, avail=avail, emulate=True)
    assert O.rel_l2(split, emu) <= 3e-3


@pytest.mark.parametrize("h,e,k,f,s,n,avail_p", [
    (2048, 64, 6, 1408, 2, 32, 0.9),   # the DeepSeek-MoE-16B decode shape: two 32-expert mask words
    (2048, 64, 6, 1408, 2, 64, None),
    (1024, 16, 2, 2048, 1, 32, 0.85),  # the 8-layer model's MoE shape
    (512, 40, 4, 256, 0, 48, 0.5),     # no shared experts; most CTAs' guesses land on no unit
])
def test_gateup_l2_prefetch_is_only_a_hint(h, e, k, f, s, n, avail_p):
    """Batches that select nearly every expert let the gate/up GEMM's idle CTAs
    prefetch their first routed unit into L2 before the plan exists (a guess from
    the availability input).  The results must not depend on it: prefetch on
    (128 MB budget, the default), off, and a budget of one k tile, against the
    oracle."""
    ops = _ops()
    wl = _workload(h, e, k, f, s, n, seed=n + e, avail_p=avail_p)
    avail = None if wl.mask is None else wl.mask.to(torch.float32)
    outs = []
    try:
        for mb in (128, 0, 1):
            ops.set_option("gateup_prefetch_mb", mb)
            outs.append(_np(_run(wl, k, True, avail=avail)["y"]))
            torch.cuda.synchronize()
            ops.check_status()
    finally:
        ops.set_option("gateup_prefetch_mb", 128)
    on, off, small = outs
    assert O.rel_l2(on, off) <= 1e-3
    assert O.rel_l2(small, off) <= 1e-3
    emu, *_ = _oracle(wl, k, True, avail=avail, emulate=True)
    assert O.rel_l2(on, emu) <= 3e-3
