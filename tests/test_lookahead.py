"""Lookahead router (chronos/model/lookahead_router.py:36-55).

CPU: the oracle restatement against the reference's torch formulation (the
module's own ``proj`` run in fp32), state_dict compatibility, CPU inputs
rejected.  GPU: the fused kernel against the oracle and the torch fp32
reference, bf16 within 1e-2 absolute on probabilities, fp32 within 1e-5;
``predict_next_experts`` shape and agreement.
"""
import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import moe_oracle as O


def _cfg(H=256, E=16, steps=2):
    return types.SimpleNamespace(hidden_size=H, num_experts=E, lookahead_steps=steps)


def _torch_reference(m, x):
    """The reference's forward, restated with the module's own layers (fp32)."""
    B, S, H = x.shape
    K = m.lookahead_steps + 1
    logits = m.proj(x.float())
    return F.softmax(logits.view(B, S, K, m.num_experts), dim=-1)


def test_oracle_matches_torch_formulation():
    from project_chronos_b200 import LookaheadRouter
    torch.manual_seed(0)
    m = LookaheadRouter(_cfg())
    x = torch.randn(2, 5, 256)
    want = _torch_reference(m, x).detach().numpy().reshape(10, 3, 16)
    got = O.lookahead(x.view(10, 256).numpy(), m.proj[0].weight.detach().numpy(),
                      m.proj[2].weight.detach().numpy(), 16, 3)
    assert np.abs(got - want).max() < 1e-6


def test_state_dict_keys_and_cpu_rejected():
    from project_chronos_b200 import LookaheadRouter
    m = LookaheadRouter(_cfg())
    assert sorted(m.state_dict()) == ["proj.0.weight", "proj.2.weight"]
    assert tuple(m.proj[0].weight.shape) == (64, 256) and tuple(m.proj[2].weight.shape) == (48, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(1, 1, 256))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
@pytest.mark.parametrize("H,E,steps,n", [(256, 16, 2, 7), (1024, 64, 2, 32), (7168, 256, 1, 3),
                                         (96, 5, 3, 1), (100, 6, 2, 9), (512, 32, 2, 300)])
def test_kernel_matches_oracle(dtype, tol, H, E, steps, n):
    from project_chronos_b200 import LookaheadRouter
    torch.manual_seed(H + E)
    m = LookaheadRouter(_cfg(H, E, steps))
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0.0, 0.05)
    x = torch.randn(1, n, H)
    m = m.to("cuda", dtype).eval()
    xd = x.to("cuda", dtype)
    with torch.no_grad():
        got = m(xd).float().cpu().numpy()
    w1 = m.proj[0].weight.detach().float().cpu().numpy()
    w2 = m.proj[2].weight.detach().float().cpu().numpy()
    want = O.lookahead(xd.float().cpu().view(n, H).numpy(), w1, w2, E, steps + 1).reshape(1, n, steps + 1, E)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= tol
    assert np.allclose(got.sum(-1), 1.0, atol=tol * 4)
    with torch.no_grad():
        idx = m.predict_next_experts(xd, top_k=2)
    assert tuple(idx.shape) == (1, n, steps, 2)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["lookahead_fp32", "lookahead_bf16", "lookahead_decode_bf16"])
def test_kernel_matches_reference_golden(name):
    """The fused kernel against the reference's own LookaheadRouter
    (chronos/model/lookahead_router.py:36-42), golden vectors from
    tests/golden/make_golden.py: fp32 within 1e-5; bf16 within 5e-3 of the
    reference run in fp32 on the bf16 values and 1e-2 of its bf16 run."""
    from project_chronos_b200 import LookaheadRouter
    from tests import _golden as G
    c = G.case(name)
    d = G.load(c)
    w1, w2, x = G.lookahead_inputs(c)
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    m = LookaheadRouter(_cfg(c["H"], c["E"], c["steps"]))
    with torch.no_grad():
        m.proj[0].weight.copy_(w1)
        m.proj[2].weight.copy_(w2)
    m = m.to("cuda", dt).eval()
    with torch.no_grad():
        got = m(x.to("cuda", dt)).float().cpu().numpy()
    assert got.shape == d["probs_ref"].shape
    if dt == torch.float32:
        assert np.abs(got - d["probs_ref"]).max() <= 1e-5
    else:
        assert np.abs(got - d["probs_ref_fp32"]).max() <= 5e-3
        assert np.abs(got - d["probs_ref"]).max() <= 1e-2
