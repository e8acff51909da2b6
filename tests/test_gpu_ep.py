"""Expert-parallel kernels and layer on the GPU.

* ``chronos_ep_dispatch`` / ``chronos_ep_combine`` against the oracle's
  restatement (oracle/ep_oracle.py): counts, shared weights and the combine
  exactly; send rows and metadata through ``pair_slot`` (the order inside a
  rank is unspecified);
* the layer on one rank (no exchange) == the single-device layer;
* two NCCL ranks on two GPUs (skipped with fewer): each rank's output == the
  single-device layer on its tokens.
"""
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests import _ep_worker

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _route(x, router, k):
    from project_chronos_b200 import ops
    return ops.moe_route(x, router, k, True, num_shared=1, ffn=64, want_probs=False)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("world,n,chunks,dedup", [(1, 7, 1, False), (2, 33, 1, False), (4, 300, 1, False),
                                                  (8, 1, 1, False), (2, 33, 4, False), (8, 300, 2, False),
                                                  (4, 5, 4, False), (1, 40, 16, False), (1, 7, 1, True),
                                                  (2, 33, 1, True), (4, 300, 1, True), (8, 300, 1, True),
                                                  (16, 64, 1, True)])
def test_dispatch_and_combine_match_oracle(dtype, world, n, chunks, dedup):
    from oracle.ep_oracle import CpuEpBackend
    from project_chronos_b200 import ops
    E, k, H = 16, 4, 256
    g = torch.Generator().manual_seed(world * 1000 + n)
    x = torch.randn(n, H, generator=g).to(DEV, dtype)
    router = (torch.randn(E, H, generator=g) * 0.05).to(DEV, dtype)
    avail = (torch.rand(E, generator=g) > 0.25).float()
    avail[3] = 0.5
    r = _route(x, router, k)
    d = ops.ep_dispatch(x, r["topk_idx"], r["topk_weight"], E, world, avail=avail.to(DEV), num_chunks=chunks,
                        dedup=dedup)
    ref = CpuEpBackend.ep_dispatch(x.cpu(), r["topk_idx"].cpu(), r["topk_weight"].cpu(), E, world, avail,
                                   num_chunks=chunks, dedup=dedup)
    assert d["pairs"] == ref["pairs"] == (min(k, E // world) if dedup else 1)
    assert d["send_counts"].cpu().tolist() == ref["send_counts"].tolist()
    assert torch.equal(d["shared_weight"].cpu(), ref["shared_weight"])
    ps = d["pair_slot"].cpu()
    assert torch.equal(ps < 0, ref["pair_slot"] < 0)
    n_send = int(ref["send_counts"].sum())
    # rows and metadata, matched through pair_slot
    sent = ps >= 0
    got_rows = d["send_x"].cpu()[ps[sent].long()]
    want_rows = ref["send_x"][ref["pair_slot"][sent].long()]
    assert torch.equal(got_rows, want_rows)
    assert torch.equal(d["send_meta"].cpu()[ps[sent].long()], ref["send_meta"][ref["pair_slot"][sent].long()])
    assert sorted(ps[sent].tolist()) == list(range(n_send))
    # rows of each (expert chunk, destination rank) are contiguous, chunk-major
    offs = np.concatenate([[0], np.cumsum(ref["send_counts"].numpy().ravel())])
    epr = E // world
    e_sent = r["topk_idx"].cpu().view(-1)[sent].numpy()
    key = ((e_sent % epr) // (epr // chunks)) * world + e_sent // epr
    slots = ps[sent].numpy()
    assert np.all((slots >= offs[key]) & (slots < offs[key + 1]))

    # combine: returned rows (any values), shared term
    rows = torch.randn(max(n_send, 1), H, generator=g).to(DEV, dtype)[:n_send]
    y_sh = torch.randn(n, H, generator=g).to(DEV, dtype)
    y = ops.ep_combine(rows, d["pair_slot"], k, y_shared=y_sh, num_tokens=n)
    want = CpuEpBackend.ep_combine(rows.cpu(), d["pair_slot"].cpu(), k, y_shared=y_sh.cpu(), num_tokens=n)
    assert torch.equal(y.cpu(), want)


@pytest.mark.parametrize("world,n,dedup,seg", [(2, 33, True, 40), (4, 300, True, 300), (8, 300, True, 512),
                                                (2, 33, False, 33 * 4), (4, 0, True, 8)])
def test_fixed_segments_match_oracle(world, n, dedup, seg):
    """Fixed all-to-all segments: rank g's rows start at g * seg, in the oracle's
    rows (matched through pair_slot), and every row past a segment's count carries
    padding metadata (expert -1, weight 0)."""
    from oracle.ep_oracle import CpuEpBackend
    from project_chronos_b200 import ops
    E, k, H = 16, 4, 256
    g = torch.Generator().manual_seed(world * 77 + n)
    x = torch.randn(max(n, 1), H, generator=g).to(DEV, torch.bfloat16)[:n]
    router = (torch.randn(E, H, generator=g) * 0.05).to(DEV, torch.bfloat16)
    avail = (torch.rand(E, generator=g) > 0.25).float()
    r = _route(x, router, k) if n else dict(topk_idx=torch.zeros(0, k, dtype=torch.int32, device=DEV),
                                             topk_weight=torch.zeros(0, k, device=DEV))
    d = ops.ep_dispatch(x, r["topk_idx"], r["topk_weight"], E, world, avail=avail.to(DEV), dedup=dedup,
                        seg_rows=seg)
    ref = CpuEpBackend.ep_dispatch(x.cpu(), r["topk_idx"].cpu(), r["topk_weight"].cpu(), E, world, avail,
                                   dedup=dedup, seg_rows=seg)
    assert d["send_x"].shape[0] == world * seg and d["send_meta"].shape[0] == world * seg
    counts = d["send_counts"].cpu().view(-1)
    assert counts.tolist() == ref["send_counts"].view(-1).tolist()
    ps = d["pair_slot"].cpu()
    sent = ps >= 0
    assert torch.equal(sent, ref["pair_slot"] >= 0)
    slots = ps[sent].long()
    assert torch.equal(d["send_x"].cpu()[slots], ref["send_x"][ref["pair_slot"][sent].long()])
    assert torch.equal(d["send_meta"].cpu()[slots], ref["send_meta"][ref["pair_slot"][sent].long()])
    meta = d["send_meta"].cpu()
    for gg in range(world):
        used = sorted(v - gg * seg for v in slots.tolist() if gg * seg <= v < (gg + 1) * seg)
        assert used == list(range(int(counts[gg])))
        pad = meta[gg * seg + int(counts[gg]):(gg + 1) * seg]
        assert bool((pad[..., 0] == -1).all()) and bool((pad[..., 1] == 0).all())


@pytest.mark.parametrize("dispatch", [False, True])
@pytest.mark.parametrize("masked", [False, True])
def test_single_rank_layer_matches_single_device(masked, dispatch):
    from project_chronos_b200 import ops
    from project_chronos_b200.ep import ExpertParallelMoE
    E, k, H, F, S, n = 16, 4, 256, 128, 1, 96
    w = {key: v.to(DEV, torch.bfloat16) for key, v in _ep_worker._weights(E, H, F, S).items()}
    x = torch.randn(n, H, generator=torch.Generator().manual_seed(5)).to(DEV, torch.bfloat16)
    mask = None
    if masked:
        mask = (torch.rand(E, generator=torch.Generator().manual_seed(6)) > 0.3).float().to(DEV)
    m = ExpertParallelMoE.from_stacked(_ep_worker._cfg(E, k, H, F, S), w["router"], w["gate"], w["up"],
                                       w["down"], w["sh_gate"], w["sh_up"], w["sh_down"],
                                       dispatch_single_rank=dispatch)
    y = m(x.view(2, n // 2, H), available_expert_mask=mask).view(n, H)
    full = ops.moe_forward(x, w["router"], w["gate"], w["up"], w["down"], w["sh_gate"], w["sh_up"],
                           w["sh_down"], k, True, avail=mask, want_probs=False)["y"]
    torch.cuda.synchronize()
    ops.check_status(torch.device(DEV))
    rel = (torch.linalg.vector_norm(y.float() - full.float()) / torch.linalg.vector_norm(full.float())).item()
    assert rel <= 1e-2
    assert m.last_send_counts == m.last_recv_counts
    if dispatch:
        # the same through fixed segments (padding rows travel, no host read of the counts)
        sent = m.last_send_counts
        m.segment_rows = n + 8
        y2 = m(x.view(2, n // 2, H), available_expert_mask=mask).view(n, H)
        torch.cuda.synchronize()
        ops.check_status(torch.device(DEV))
        rel2 = (torch.linalg.vector_norm(y2.float() - full.float()) /
                torch.linalg.vector_norm(full.float())).item()
        assert rel2 <= 1e-2
        assert m.last_send_counts is None and m.read_send_counts() == sent


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("seg", [0, 256])
def test_two_ranks_nccl_match_single_device(seg):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cfg = dict(E=16, k=4, H=512, F=256, S=1, n=200, seg=seg)
    procs = [ctx.Process(target=_ep_worker.gpu_rank, args=(r, 2, port, q, cfg)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in range(2):
            res.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join()
    res.sort(key=lambda r: r[1])
    for status, rank, val, sc, rc in res:
        assert status == "ok", val
        assert val <= 1e-2, (rank, val)
    if not seg:
        assert res[0][3][1] == res[1][4][0] and res[1][3][0] == res[0][4][1]


def test_mask_is_the_arithmetic_availability_in_eval():
    """ExpertParallelMoE applies the mask as a_e = mask[e] (the blend of
    chronos/mlx/moe.py:160-166) in eval too, while ChronosMOEFeedForward in eval
    runs a loaded expert even where the mask says unavailable
    (moe_chronos.py:221-227): on the same layer and mask the two differ, each
    as the oracle predicts."""
    import types
    from oracle import moe_oracle as O
    from project_chronos_b200 import ChronosMOEFeedForward
    from project_chronos_b200.ep import ExpertParallelMoE
    H, E, k, F = 256, 8, 2, 128
    cfg = types.SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                                moe_intermediate_size=F, num_shared_experts=1, norm_topk_prob=True,
                                router_aux_loss_coef=0.0, hidden_act="silu", dropout=0.0,
                                fallback_mask_prob=0.0, intermediate_size=F)
    torch.manual_seed(0)
    layer = ChronosMOEFeedForward(cfg)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.05)
    layer = layer.to(DEV).eval()
    ep = ExpertParallelMoE.from_layer(layer)
    x = torch.randn(1, 24, H, device=DEV)
    mask = torch.tensor([1, 0, 1, 1, 0, 1, 1, 1], dtype=torch.bool)
    with torch.no_grad():
        y_layer = layer(x, available_expert_mask=mask)
        y_ep = ep(x, available_expert_mask=mask)
    torch.cuda.synchronize()
    sd = {kk: v.float().cpu().numpy() for kk, v in layer.state_dict().items()}
    st = lambda n: np.stack([sd[f"experts.{e}.{n}.weight"] for e in range(E)])  # noqa: E731
    args = (x.cpu().numpy().reshape(-1, H), sd["gate.weight"], st("gate_proj"), st("up_proj"),
            st("down_proj"), sd["shared_experts.0.gate_proj.weight"][None],
            sd["shared_experts.0.up_proj.weight"][None], sd["shared_experts.0.down_proj.weight"][None],
            k, True)
    want_live, idx, _, _ = O.moe_forward(*args)
    want_blend, _, _, _ = O.moe_forward(*args, avail=mask.float().numpy())
    assert (np.isin(idx, [1, 4])).any()
    assert O.rel_l2(y_layer.cpu().numpy().reshape(-1, H), want_live) <= 1e-5
    assert O.rel_l2(y_ep.cpu().numpy().reshape(-1, H), want_blend) <= 1e-5
    assert O.rel_l2(want_live, want_blend) > 1e-3
