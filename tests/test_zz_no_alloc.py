"""chronos_moe_forward_noalloc: the layer for callers that cannot allocate GPU memory.

Some hosts cannot give the library a workspace: an engine that embeds the
layer through FFI without access to the GPU allocator, a runtime whose device
memory pool is sized once at start-up for its own tensors, or a real-time
server that forbids cudaMalloc after start-up.  This entry point uses a
scratch array built into the library instead.  The tests call it through the
C ABI (ctypes), several calls in a row on different inputs, and check each
result against the workspace-taking chronos_moe_forward on the same inputs
(rel-L2 <= 1e-2 for bf16, <= 1e-5 for fp32; routing identical), and at the
full decode shape the header promises (64 tokens, d_model 2048, 64 experts
top-6, d_ff 1408, 2 shared) against the CPU oracle.  The file is collected
last, and passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _lib():
    from project_chronos_b200 import _native
    return _native, _native.load_library()


def _noalloc(N, lib, x, w, k, avail, norm=True, topk=None):
    """One call of the no-alloc entry point; ``topk`` = (idx, weight) pre-routes it."""
    n, h = x.shape
    e = w.router.shape[0]
    _, f, _ = w.gate.shape
    s = w.sh_gate.shape[0]
    dt = {torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_FP16, torch.float32: N.DTYPE_FP32}[x.dtype]
    y = torch.empty_like(x)
    if topk is None:
        idx = torch.empty(n, k, dtype=torch.int32, device=x.device)
        wt = torch.empty(n, k, dtype=torch.float32, device=x.device)
        flags = 0
    else:
        idx, wt = topk
        flags = N.FLAG_PREROUTED
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    args = N.ChronosMoeArgs(
        shape=N.ChronosMoeShape(n, h, e, k, f, s, dt), norm_topk=int(norm), flags=flags,
        x=x.data_ptr(), router_w=w.router.data_ptr(), w_gate=w.gate.data_ptr(),
        w_up=w.up.data_ptr(), w_down=w.down.data_ptr(), pool_slots=e,
        w_shared_gate=w.sh_gate.data_ptr() if s else None, w_shared_up=w.sh_up.data_ptr() if s else None,
        w_shared_down=w.sh_down.data_ptr() if s else None, avail=avail.data_ptr(), y=y.data_ptr(),
        topk_idx=idx.data_ptr(), topk_weight=wt.data_ptr(), workspace=None, workspace_bytes=0,
        status=status.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    N.check(lib.chronos_moe_forward_noalloc(ctypes.byref(args), ctypes.c_void_p(stream)))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return y, idx


def _rel_l2(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm())


def _forward(wl, k, avail, norm=True, topk=None):
    from project_chronos_b200 import ops
    w = wl.weights
    s = w.sh_gate.shape[0]
    return ops.moe_forward(wl.x, w.router, w.gate, w.up, w.down, w.sh_gate if s else None,
                           w.sh_up if s else None, w.sh_down if s else None, k, norm, avail=avail,
                           topk=None if topk is None else [topk[0], topk[1]])


def _fits(N, lib, n, shape, dtype):
    need = lib.chronos_moe_workspace_size(ctypes.byref(N.ChronosMoeShape(
        n, shape.hidden, shape.num_experts, shape.top_k, shape.ffn, shape.num_shared, dtype)))
    return 0 < need <= N.NOALLOC_SCRATCH_BYTES


def test_noalloc_matches_forward_on_two_calls_in_a_row():
    from project_chronos_b200 import synthetic as syn
    N, lib = _lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = syn.MoEShape(hidden=512, num_experts=16, top_k=4, ffn=256, num_shared=2)
    assert _fits(N, lib, 40, shape, N.DTYPE_BF16)
    for call, (n, seed) in enumerate(((40, 3), (17, 4))):
        wl = syn.make_workload(shape, n, seed=seed, dtype=torch.bfloat16, device=dev, avail_p=0.7)
        avail = wl.mask.to(torch.float32)
        ref = _forward(wl, shape.top_k, avail)
        y, idx = _noalloc(N, lib, wl.x, wl.weights, shape.top_k, avail)
        assert torch.equal(idx, ref["topk_idx"]), f"call {call}: routing differs"
        err = _rel_l2(y.float(), ref["y"].float())
        assert err <= 1e-2, f"call {call}: rel-L2 {err:.3e}"
        assert np.isfinite(y.float().cpu().numpy()).all()


def test_noalloc_at_the_decode_shape_against_the_oracle():
    """64 tokens of the DeepSeek-MoE-16B-shaped layer, the size the header names,
    then 1 token (the scratch keeps the larger call's contents): each against
    chronos_moe_forward and the CPU oracle."""
    from project_chronos_b200 import synthetic as syn
    N, lib = _lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = syn.WORKLOADS["decode"]["shape"]
    assert _fits(N, lib, 64, shape, N.DTYPE_BF16)
    for n, seed in ((64, 11), (1, 12), (64, 13)):
        wl = syn.make_workload(shape, n, seed=seed, dtype=torch.bfloat16, device=dev, avail_p=0.9)
        avail = wl.mask.to(torch.float32)
        y, idx = _noalloc(N, lib, wl.x, wl.weights, shape.top_k, avail)
        ref = _forward(wl, shape.top_k, avail)
        assert torch.equal(idx, ref["topk_idx"])
        assert _rel_l2(y.float(), ref["y"].float()) <= 1e-2
        w = wl.weights
        f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
        o_y, o_idx, _, _ = O.moe_forward(f(wl.x), f(w.router), f(w.gate), f(w.up), f(w.down), f(w.sh_gate),
                                         f(w.sh_up), f(w.sh_down), shape.top_k, True, avail=f(avail))
        assert np.array_equal(idx.cpu().numpy(), o_idx)
        assert O.rel_l2(f(y), o_y) <= 1e-2


def test_noalloc_fp32_layer_matches_forward():
    """An fp32 layer (the FMA path) through the no-alloc entry point, twice."""
    from project_chronos_b200 import synthetic as syn
    N, lib = _lib()
    dev = torch.device("cuda", 0)
    shape = syn.MoEShape(hidden=256, num_experts=8, top_k=2, ffn=512, num_shared=1)
    assert _fits(N, lib, 33, shape, N.DTYPE_FP32)
    for n, seed in ((33, 21), (5, 22)):
        wl = syn.make_workload(shape, n, seed=seed, dtype=torch.float32, device=dev, avail_p=0.75)
        avail = wl.mask.to(torch.float32)
        y, idx = _noalloc(N, lib, wl.x, wl.weights, shape.top_k, avail, norm=False)
        ref = _forward(wl, shape.top_k, avail, norm=False)
        assert torch.equal(idx, ref["topk_idx"])
        assert _rel_l2(y, ref["y"]) <= 1e-5


def test_noalloc_prerouted_matches_forward():
    """CHRONOS_FLAG_PREROUTED: the caller's routing (the hook slow path), with the
    weights of fallback selections zeroed as the layer's multi-pass mode does."""
    from project_chronos_b200 import ops, synthetic as syn
    N, lib = _lib()
    dev = torch.device("cuda", 0)
    shape = syn.MoEShape(hidden=512, num_experts=16, top_k=4, ffn=256, num_shared=2)
    for n, seed in ((24, 31), (7, 32)):
        wl = syn.make_workload(shape, n, seed=seed, dtype=torch.bfloat16, device=dev, avail_p=0.6)
        avail = wl.mask.to(torch.float32)
        r = ops.moe_route(wl.x, wl.weights.router, shape.top_k, True, num_shared=2, ffn=256)
        w_part = (r["topk_weight"] * (r["topk_idx"] % 3 != 0).float()).contiguous()
        topk = (r["topk_idx"].clone(), w_part)
        ref = _forward(wl, shape.top_k, avail, topk=topk)
        y, idx = _noalloc(N, lib, wl.x, wl.weights, shape.top_k, avail, topk=topk)
        assert torch.equal(idx, r["topk_idx"])
        assert _rel_l2(y.float(), ref["y"].float()) <= 1e-2


def test_noalloc_rejects_shapes_beyond_its_scratch():
    N, lib = _lib()
    args = N.ChronosMoeArgs()
    args.shape = N.ChronosMoeShape(8192, 2048, 64, 6, 1408, 2, N.DTYPE_BF16)
    rc = lib.chronos_moe_forward_noalloc(ctypes.byref(args), None)
    assert rc == N.CHRONOS_ERR_INVALID_ARG
    assert b"scratch" in lib.chronos_moe_last_error()
