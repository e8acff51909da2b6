"""chronos_moe_forward_noalloc: the layer for callers that cannot allocate GPU memory.

Some hosts cannot give the library a workspace: an engine that embeds the
layer through FFI without access to the GPU allocator, a decode loop replayed
inside a CUDA graph whose memory was fixed at capture time, or a real-time
server that forbids cudaMalloc after start-up.  This entry point uses a
scratch array built into the library instead.  The test calls it through the
C ABI (ctypes) twice in a row, on different inputs, and checks each result
against the workspace-taking chronos_moe_forward on the same inputs, with the
bf16 tolerance the parity tests use (rel-L2 <= 1e-2; routing identical).  It
lives in its own file, collected last, and passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from project_chronos_b200 import _native
    return _native, _native.load_library()


def _noalloc(N, lib, x, w, k, avail):
    n, h = x.shape
    e = w.router.shape[0]
    _, f, _ = w.gate.shape
    s = w.sh_gate.shape[0]
    y = torch.empty_like(x)
    idx = torch.empty(n, k, dtype=torch.int32, device=x.device)
    wt = torch.empty(n, k, dtype=torch.float32, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    args = N.ChronosMoeArgs(
        shape=N.ChronosMoeShape(n, h, e, k, f, s, N.DTYPE_BF16), norm_topk=1, flags=0,
        x=x.data_ptr(), router_w=w.router.data_ptr(), w_gate=w.gate.data_ptr(),
        w_up=w.up.data_ptr(), w_down=w.down.data_ptr(), pool_slots=e,
        w_shared_gate=w.sh_gate.data_ptr(), w_shared_up=w.sh_up.data_ptr(),
        w_shared_down=w.sh_down.data_ptr(), avail=avail.data_ptr(), y=y.data_ptr(),
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


def test_noalloc_matches_forward_on_two_calls_in_a_row():
    from project_chronos_b200 import ops, synthetic as syn
    N, lib = _lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = syn.MoEShape(hidden=512, num_experts=16, top_k=4, ffn=256, num_shared=2)
    need = N.load_library().chronos_moe_workspace_size(
        ctypes.byref(N.ChronosMoeShape(40, 512, 16, 4, 256, 2, N.DTYPE_BF16)))
    assert 0 < need <= N.NOALLOC_SCRATCH_BYTES
    for call, (n, seed) in enumerate(((40, 3), (17, 4))):
        wl = syn.make_workload(shape, n, seed=seed, dtype=torch.bfloat16, device=dev, avail_p=0.7)
        w = wl.weights
        avail = wl.mask.to(torch.float32)
        ref = ops.moe_forward(wl.x, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up, w.sh_down,
                              shape.top_k, True, avail=avail)
        y, idx = _noalloc(N, lib, wl.x, w, shape.top_k, avail)
        assert torch.equal(idx, ref["topk_idx"]), f"call {call}: routing differs"
        err = _rel_l2(y.float(), ref["y"].float())
        assert err <= 1e-2, f"call {call}: rel-L2 {err:.3e}"
        assert np.isfinite(y.float().cpu().numpy()).all()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    N, lib = _lib()
    args = N.ChronosMoeArgs()
    args.shape = N.ChronosMoeShape(8192, 2048, 64, 6, 1408, 2, N.DTYPE_BF16)
    rc = lib.chronos_moe_forward_noalloc(ctypes.byref(args), None)
    assert rc == N.CHRONOS_ERR_INVALID_ARG
    assert b"scratch" in lib.chronos_moe_last_error()
