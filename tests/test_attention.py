"""Hybrid attention decode (chronos/model/hybrid_attention.py) and the model
around it (chronos/model/model_chronos.py).

CPU: the attention oracle against the reference's own MLAAttention /
SlidingWindowAttention stepped with their caches (golden vectors from
tests/golden/make_golden.py), the model's parameter names and shapes against
the reference's, argument checks of the C ABI.
GPU: the decode kernels against those goldens and the oracle (fp32 within
rel-L2 2e-5, bf16 within 1e-2; cache rings wrapping, every head grouping), the
fused add + RMSNorm against a torch fp32 restatement, the whole model
teacher-forced against the reference's logits and lookahead probabilities
(fp32 within 1e-4, bf16 within 1e-2 of the reference's fp32 run), and the
CUDA-graph decode step against eager steps.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as A
from oracle import moe_oracle as O
from tests import _golden as G


def _np(t):
    return t.detach().float().cpu().numpy()


def _tables(d, n):
    from project_chronos_b200.model import precompute_freqs_cis
    return precompute_freqs_cis(d, n, 1e6)


def _attn_state(c, tag):
    from project_chronos_b200 import synthetic as syn
    shapes = c["state_shapes"][tag]
    return syn.model_state({k: tuple(v) for k, v in shapes.items()}, c["seed"] + (tag == "sw"))


def _cat(st, names):
    return torch.cat([st[n] for n in names], dim=0)


MLA_IN = ("q_nope_proj.weight", "q_rope_proj.weight", "kv_down_proj.weight")
SW_IN = ("q_proj.weight", "k_proj.weight", "v_proj.weight")


def _oracle_for(tag, c, st, cos, sin):
    cfg = c["config"]
    nh, nkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], c["head_dim"]
    if tag == "mla":
        return A.MLADecodeOracle(nh, nkv, D, cfg["rope_dim"], cfg["kv_latent_dim"], cfg["rms_norm_eps"],
                                 st["q_nope_norm.weight"], st["q_rope_norm.weight"], st["kv_down_norm.weight"],
                                 st["k_nope_proj.weight"], st["k_rope_proj.weight"], st["v_proj.weight"],
                                 cos.numpy(), sin.numpy())
    return A.SlidingWindowDecodeOracle(nh, nkv, D, cfg["sliding_window_size"], cfg["rms_norm_eps"],
                                       st["q_norm.weight"], st["k_norm.weight"], cos.numpy(), sin.numpy())


@pytest.mark.parametrize("tag", ["mla", "sw"])
def test_oracle_matches_reference_attention_modules(tag):
    c = G.attn_case()
    d = np.load(f"{G.GOLDEN}/{c['name']}.npz")
    st = _attn_state(c, tag)
    cos, sin = _tables(c["head_dim"], c["config"]["max_position_embeddings"])
    w_in = _cat(st, MLA_IN if tag == "mla" else SW_IN).numpy()
    w_o = st["o_proj.weight"].numpy()
    for b in range(c["B"]):
        orc = _oracle_for(tag, c, st, cos, sin)
        for t in range(c["steps"]):
            y = orc.step(d["x"][t, b, 0] @ w_in.T) @ w_o.T
            assert O.rel_l2(y, d[f"y_{tag}"][t, b]) < 1e-5, (b, t)


def test_model_parameters_match_the_reference():
    from project_chronos_b200.model import ChronosForCausalLM
    c = G.model_case()
    m = ChronosForCausalLM(G.model_config(c["config"]))
    got = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert got == c["state_shapes"]
    assert m.model.embed_tokens.weight is m.lm_head.weight


def test_attention_abi_checks_arguments():
    from project_chronos_b200 import _native as N
    lib = N.load_library()
    a = N.ChronosAttnArgs(batch=0, heads=8, kv_heads=2, head_dim=128, rope_dim=32, latent=64, window=0,
                          max_len=768, table_len=1024, dtype=N.DTYPE_BF16, eps=1e-5)
    assert lib.chronos_mla_decode(ctypes.byref(a), None) == N.CHRONOS_OK
    a.heads = 7
    assert lib.chronos_mla_decode(ctypes.byref(a), None) == N.CHRONOS_ERR_INVALID_ARG
    assert b"kv_heads" in lib.chronos_moe_last_error()
    a.heads, a.rope_dim = 8, 128
    assert lib.chronos_mla_decode(ctypes.byref(a), None) == N.CHRONOS_ERR_INVALID_ARG
    assert b"rope_dim" in lib.chronos_moe_last_error()
    a.rope_dim, a.max_len = 32, 9000
    assert lib.chronos_mla_decode(ctypes.byref(a), None) == N.CHRONOS_ERR_INVALID_ARG
    s = N.ChronosAttnArgs(batch=0, heads=8, kv_heads=2, head_dim=128, rope_dim=128, latent=0, window=16,
                          max_len=16, table_len=1024, dtype=N.DTYPE_FP32, eps=1e-5)
    assert lib.chronos_sw_decode(ctypes.byref(s), None) == N.CHRONOS_OK
    s.max_len = 32
    assert lib.chronos_sw_decode(ctypes.byref(s), None) == N.CHRONOS_ERR_INVALID_ARG
    s.max_len, s.batch = 16, 1
    assert lib.chronos_sw_decode(ctypes.byref(s), None) == N.CHRONOS_ERR_INVALID_ARG   # NULL pointers
    n = N.ChronosNormArgs(rows=0, width=20000, dtype=N.DTYPE_BF16, eps=1e-5)
    assert lib.chronos_add_rmsnorm(ctypes.byref(n), None) == N.CHRONOS_ERR_INVALID_ARG


# ---------------------------------------------------------------------------- GPU
DEV = "cuda"


def _decode_run(tag, proj_steps, st, cfg, head_dim, cos, sin, dtype, batch):
    """Step the decode kernel over proj_steps [T, B, width]; returns outputs [T, B, nH*D]."""
    from project_chronos_b200 import ops
    nh, nkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], head_dim
    dev = lambda t: t.to(DEV, dtype).contiguous()  # noqa: E731
    c_d, s_d = dev(cos), dev(sin)
    T = proj_steps.shape[0]
    pos = torch.zeros((), dtype=torch.int32, device=DEV)
    outs = []
    if tag == "mla":
        L, R = cfg["kv_latent_dim"], cfg["rope_dim"]
        ca = torch.zeros(batch, T, L, device=DEV, dtype=dtype)
        cb = torch.zeros(batch, T, nkv, R, device=DEV, dtype=dtype)
        for t in range(T):
            outs.append(ops.attn_decode("mla", dev(proj_steps[t]), pos, c_d, s_d, ca, cb, nh, nkv, D, R, L, 0,
                                        cfg["rms_norm_eps"], dev(st["q_nope_norm.weight"]),
                                        dev(st["q_rope_norm.weight"]), norm_kv=dev(st["kv_down_norm.weight"]),
                                        w_krope=dev(st["k_rope_proj.weight"]),
                                        w_knope=dev(st["k_nope_proj.weight"]), w_v=dev(st["v_proj.weight"])))
            pos.add_(1)
    else:
        W = cfg["sliding_window_size"]
        ca = torch.zeros(batch, W, nkv, D, device=DEV, dtype=dtype)
        cb = torch.zeros(batch, W, nkv, D, device=DEV, dtype=dtype)
        for t in range(T):
            outs.append(ops.attn_decode("sw", dev(proj_steps[t]), pos, c_d, s_d, ca, cb, nh, nkv, D, D, 0, W,
                                        cfg["rms_norm_eps"], dev(st["q_norm.weight"]), dev(st["k_norm.weight"])))
            pos.add_(1)
    torch.cuda.synchronize()
    return torch.stack(outs).float().cpu()


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["mla", "sw"])
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 1e-2)])
def test_decode_kernels_match_reference_modules(tag, dtype, tol):
    c = G.attn_case()
    d = np.load(f"{G.GOLDEN}/{c['name']}.npz")
    st = _attn_state(c, tag)
    if dtype != torch.float32:   # compare on the values the bf16 layer holds
        st = {k: v.to(dtype).float() for k, v in st.items()}
    cos, sin = _tables(c["head_dim"], c["config"]["max_position_embeddings"])
    w_in = _cat(st, MLA_IN if tag == "mla" else SW_IN)
    x = torch.from_numpy(d["x"])[:, :, 0]                      # [T, B, H]
    if dtype != torch.float32:
        x = x.to(dtype).float()
    proj = torch.einsum("tbh,wh->tbw", x, w_in)
    if dtype != torch.float32:
        proj = proj.to(dtype).float()
    outs = _decode_run(tag, proj, st, c["config"], c["head_dim"], cos, sin, dtype, c["B"])
    y = torch.einsum("tbk,hk->tbh", outs, st["o_proj.weight"]).numpy()
    if dtype == torch.float32:
        assert O.rel_l2(y, d[f"y_{tag}"]) <= tol
    else:   # against the unfolded oracle on the same bf16 values
        for b in range(c["B"]):
            orc = _oracle_for(tag, c, st, cos.to(dtype).float(), sin.to(dtype).float())
            want = np.stack([orc.step(proj[t, b].numpy()) for t in range(c["steps"])])
            assert O.rel_l2(outs[:, b].numpy(), want) <= tol


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["mla", "sw"])
@pytest.mark.parametrize("nh,nkv,D,R,L,W,T,B", [
    (8, 2, 128, 32, 64, 16, 40, 3),     # the 8-layer decode model's attention shape
    (4, 4, 64, 16, 32, 3, 11, 2),       # one head per kv head, a 3-slot ring
    (8, 1, 128, 64, 128, 7, 20, 1),     # 8 heads per kv head
    (2, 1, 256, 64, 256, 1, 5, 2),      # widest head, a one-slot window
    (8, 2, 128, 32, 64, 64, 300, 1),    # 300 positions over a cluster of 8 CTAs; the ring wraps 4 times
])
def test_decode_kernels_match_oracle(tag, nh, nkv, D, R, L, W, T, B):
    torch.manual_seed(nh * 1000 + D + W)
    cfg = dict(num_attention_heads=nh, num_key_value_heads=nkv, kv_latent_dim=L, rope_dim=R,
               sliding_window_size=W, rms_norm_eps=1e-5)
    nope = D - R
    st = {"q_nope_norm.weight": 1 + 0.1 * torch.randn(nope), "q_rope_norm.weight": 1 + 0.1 * torch.randn(R),
          "kv_down_norm.weight": 1 + 0.1 * torch.randn(L), "k_nope_proj.weight": 0.1 * torch.randn(nkv * nope, L),
          "k_rope_proj.weight": 0.1 * torch.randn(nkv * R, L), "v_proj.weight": 0.1 * torch.randn(nkv * D, L),
          "q_norm.weight": 1 + 0.1 * torch.randn(D), "k_norm.weight": 1 + 0.1 * torch.randn(D)}
    cos, sin = _tables(D, max(64, T + 1))
    width = nh * (nope + R) + L if tag == "mla" else (nh + 2 * nkv) * D
    proj = torch.randn(T, B, width)
    outs = _decode_run(tag, proj, st, cfg, D, cos, sin, torch.float32, B)
    case = dict(config=cfg, head_dim=D)
    for b in range(B):
        orc = _oracle_for(tag, case, {k: v.numpy() for k, v in st.items()}, cos, sin)
        want = np.stack([orc.step(proj[t, b].numpy()) for t in range(T)])
        assert O.rel_l2(outs[:, b].numpy(), want) <= 2e-5, b


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_argmax_rows_matches_torch(dtype):
    from project_chronos_b200 import ops
    g = torch.Generator().manual_seed(7)
    x = torch.randn(37, 6400, generator=g).to(dtype)
    x[3, 100] = x[3, 5000] = 50.0        # a tie: the first index wins
    x[4, :] = 1.0                        # all equal
    x[5, 17] = float("nan")              # NaN counts as the maximum
    x[6, 9] = x[6, 11] = float("nan")    # the first NaN
    x[7, -1] = 60.0                      # the last column
    xd = x.to(DEV)
    got = ops.argmax_rows(xd)
    want = torch.argmax(xd, dim=-1)
    assert got.dtype == torch.int64 and got.shape == (37,)
    assert torch.equal(got.cpu(), want.cpu())
    assert got[3].item() == 100 and got[4].item() == 0 and got[5].item() == 17 and got[6].item() == 9
    y = torch.randn(2, 3, 129, device=DEV, dtype=dtype)
    assert torch.equal(ops.argmax_rows(y), torch.argmax(y, dim=-1))
    # rows longer than one pass of 4 x 256 8-element groups per block
    z = torch.randn(3, 8800, generator=g).to(dtype)
    z[0, 8799] = 70.0
    z[1, 8200] = z[1, 8300] = 70.0
    zd = z.to(DEV)
    assert torch.equal(ops.argmax_rows(zd).cpu(), torch.argmax(zd, dim=-1).cpu())


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_add_rmsnorm(dtype):
    from project_chronos_b200 import ops
    torch.manual_seed(0)
    x = torch.randn(37, 1024, device=DEV).to(dtype)
    r = torch.randn(37, 1024, device=DEV).to(dtype)
    w = (1 + 0.1 * torch.randn(1024, device=DEV)).to(dtype)
    s = (x.float() + r.float()).to(dtype)
    want = (w.float() * (s.float() * torch.rsqrt(s.float().pow(2).mean(-1, keepdim=True) + 1e-5))).to(dtype)
    got = ops.add_rmsnorm(x, w, 1e-5, residual=r, sum_out=r)      # the sum written over the residual
    torch.cuda.synchronize()
    assert torch.equal(r, s)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert (got.float() - want.float()).norm() / want.float().norm() <= tol
    plain = ops.add_rmsnorm(x, w, 1e-5)
    want2 = (w.float() * (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5))).to(dtype)
    assert (plain.float() - want2.float()).norm() / want2.float().norm() <= tol


@pytest.mark.gpu
@pytest.mark.parametrize("width", [1024, 2048, 4096])
def test_add_rmsnorm_reads_an_fp32_accumulator(width):
    """An fp32 x with a bf16 weight (a MoE layer's fp32 accumulator) is rounded
    to bf16 as it is read: bitwise the same as rounding it first."""
    from project_chronos_b200 import ops
    torch.manual_seed(width)
    acc = torch.randn(33, width, device=DEV) * 3
    r = torch.randn(33, width, device=DEV).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(width, device=DEV)).to(torch.bfloat16)
    r1, r2 = r.clone(), r.clone()
    got = ops.add_rmsnorm(acc, w, 1e-5, residual=r1, sum_out=r1)
    want = ops.add_rmsnorm(acc.to(torch.bfloat16), w, 1e-5, residual=r2, sum_out=r2)
    torch.cuda.synchronize()
    assert got.dtype == torch.bfloat16
    assert torch.equal(got, want) and torch.equal(r1, r2)


@pytest.mark.gpu
def test_moe_forward_acc_is_the_unrounded_output():
    """ChronosMOEFeedForward.forward_acc: the fp32 accumulator (CHRONOS_FLAG_ACC_OUT,
    no finalize pass) rounds to forward's output (to the order of the fp32 adds)."""
    import types
    from project_chronos_b200 import synthetic as syn
    from project_chronos_b200.moe import ChronosMOEFeedForward
    shape = syn.MoEShape(512, 16, 2, 256, 1)
    for n in (1, 32, 300):
        wl = syn.make_workload(shape, n, seed=n, dtype=torch.bfloat16, device=DEV, avail_p=0.8)
        w = wl.weights
        cfg = types.SimpleNamespace(hidden_size=512, num_experts=16, num_experts_per_tok=2,
                                    moe_intermediate_size=256, num_shared_experts=1, norm_topk_prob=True,
                                    router_aux_loss_coef=5e-4, fallback_mask_prob=0.0, hidden_act="silu",
                                    dropout=0.0, intermediate_size=256)
        m = ChronosMOEFeedForward.from_stacked(cfg, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up,
                                               w.sh_down).eval()
        m.mask_semantics = "residency"
        mask = wl.mask.to(DEV, torch.float32)
        with torch.no_grad():
            y = m(wl.x.view(1, n, 512), mask)
            acc = m.forward_acc(wl.x.view(1, n, 512), mask)
        torch.cuda.synchronize()
        assert acc.dtype == torch.float32 and acc.shape == y.shape
        rel = ((acc.to(torch.bfloat16).float() - y.float()).norm() / y.float().norm()).item()
        assert rel <= 1e-3, (n, rel)


def _model(dtype):
    from project_chronos_b200 import synthetic as syn
    from project_chronos_b200.model import ChronosForCausalLM
    c = G.model_case()
    m = ChronosForCausalLM(G.model_config(c["config"]))
    shapes = {k: tuple(v) for k, v in c["state_shapes"].items() if k != "lm_head.weight"}
    state = {k: v.to(torch.bfloat16).float() for k, v in syn.model_state(shapes, c["seed"]).items()}
    m.load_state_dict(state, strict=False)
    return c, m.to(DEV, dtype).eval()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 1e-2)])
def test_model_teacher_forced_matches_reference(dtype, tol):
    c, m = _model(dtype)
    d = np.load(f"{G.GOLDEN}/{c['name']}.npz")
    ids = torch.from_numpy(d["ids"]).to(DEV)
    P = c["prompt"]
    logits, look = [], []
    with torch.no_grad():
        o, lp = m(ids[:, :P], use_cache=True)
        logits.append(o.logits[:, -1].float())
        look.append(lp[:, -1].float())
        cache = o.past_key_values
        for t in range(c["steps"]):
            o, lp = m(ids[:, P + t:P + t + 1], past_key_values=cache, use_cache=True)
            logits.append(o.logits[:, -1].float())
            look.append(lp[:, -1].float())
    torch.cuda.synchronize()
    got = torch.stack(logits).cpu().numpy()
    for t in range(c["steps"] + 1):
        assert O.rel_l2(got[t], d["logits_fp32"][t]) <= tol, t
    assert np.abs(torch.stack(look).cpu().numpy() - d["lookahead_fp32"]).max() <= (1e-5 if tol < 1e-3 else 1e-2)
    assert cache.length == P + c["steps"]


@pytest.mark.gpu
def test_graphed_decoder_matches_eager_steps():
    from project_chronos_b200.model import GraphedDecoder
    c, m = _model(torch.bfloat16)
    d = np.load(f"{G.GOLDEN}/{c['name']}.npz")
    ids = torch.from_numpy(d["ids"]).to(DEV)
    P, T = c["prompt"], c["steps"]
    with torch.no_grad():
        o, _ = m(ids[:, :P], use_cache=True)
        eager_cache = o.past_key_values
        eager = []
        for t in range(T):
            o, _ = m(ids[:, P + t:P + t + 1], past_key_values=eager_cache, use_cache=True)
            eager.append(o.logits[:, -1].float().clone())
        o, _ = m(ids[:, :P], use_cache=True)
        gd = GraphedDecoder(m, o.past_key_values)
        graphed = []
        for t in range(T):
            gd.ids.copy_(ids[:, P + t:P + t + 1])        # teacher forcing
            gd.step()
            graphed.append(gd.logits.float().clone())
    torch.cuda.synchronize()
    for t in range(T):
        assert O.rel_l2(graphed[t].cpu().numpy(), eager[t].cpu().numpy()) <= 2e-3, t
        assert O.rel_l2(graphed[t].cpu().numpy(), d["logits_fp32"][t + 1]) <= 1e-2, t
    assert gd.cache.length == P + T
    # greedy: a replay feeds its own pick to the next
    with torch.no_grad():
        first = gd.step().clone()
        assert torch.equal(gd.ids.view(-1), first)


@pytest.mark.gpu
def test_model_steps_do_not_depend_on_programmatic_launch():
    """The norm, attention, lookahead and arg-max kernels launch early behind their
    predecessor (programmatic launch) and wait for it before touching memory; with
    the switch off they launch after it.  Teacher-forced eager steps agree."""
    from project_chronos_b200 import ops
    c, m = _model(torch.bfloat16)
    d = np.load(f"{G.GOLDEN}/{c['name']}.npz")
    ids = torch.from_numpy(d["ids"]).to(DEV)
    P, T = c["prompt"], c["steps"]
    runs = []
    try:
        for pdl in (1, 0):
            ops.set_option("model_pdl", pdl)
            with torch.no_grad():
                o, _ = m(ids[:, :P], use_cache=True)
                cache = o.past_key_values
                steps = []
                for t in range(T):
                    o, _ = m(ids[:, P + t:P + t + 1], past_key_values=cache, use_cache=True)
                    steps.append(o.logits[:, -1].float().cpu().numpy())
            runs.append(steps)
    finally:
        ops.set_option("model_pdl", 0)
    for t in range(T):
        assert O.rel_l2(runs[0][t], runs[1][t]) <= 2e-3, t
        assert O.rel_l2(runs[0][t], d["logits_fp32"][t + 1]) <= 1e-2, t
