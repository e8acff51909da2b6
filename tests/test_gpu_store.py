"""Pooled expert store on the GPU: slots, H2D stream, device ready flags.

Mirrors the reference's lazy-loading tests (tests/test_smoke.py of
FonaTech/Project_Chronos: on-demand offload == full model, :429-488, with a
pool of ONE resident expert; CUDA double-stream pipeline, tests/test_smoke_cuda.py)
on the layer level, and checks what the device path adds: a forward issued
while its experts' copies are still queued on the H2D stream waits on the
per-(layer, expert) ready flags, not on the stream, and still matches.
"""
import types

import numpy as np
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cfg(E=8, H=128, F=256, S=1, k=2, budget_experts=4, flags=True):
    return types.SimpleNamespace(
        hidden_size=H, num_experts=E, num_experts_per_tok=k, moe_intermediate_size=F,
        num_shared_experts=S, norm_topk_prob=True, router_aux_loss_coef=5e-4, hidden_act="silu",
        dropout=0.0, fallback_mask_prob=0.0, intermediate_size=F,
        vram_budget_gb=budget_experts * 3 * H * F * 2 * 2 / (1024 ** 3),
        pinned_memory_max_fraction=0.25, device_ready_flags=flags)


class _Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        from project_chronos_b200 import ChronosMOEFeedForward
        self.mlp = ChronosMOEFeedForward(cfg)


class _Model(nn.Module):
    def __init__(self, cfg, layers):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([_Block(cfg) for _ in range(layers)])


def _pair(cfg, layers, dtype, seed=0):
    """(full model, lazy model, half-representable state) on the GPU."""
    torch.manual_seed(seed)
    src = _Model(cfg, layers)
    with torch.no_grad():
        for p in src.parameters():
            p.normal_(0.0, 0.05)
    state = {f"model.{k}": v.detach().half().float() for k, v in src.model.state_dict().items()}
    full = _Model(cfg, layers)
    full.load_state_dict(state)
    lazy = _Model(cfg, layers)
    lazy.load_state_dict(state)
    full = full.to(DEV, dtype).eval()
    lazy = lazy.to(DEV, dtype).eval()
    return full, lazy, state


def _selected(moe, x):
    from project_chronos_b200 import ops
    r = ops.moe_route(x.reshape(-1, x.shape[-1]), moe.gate.weight, moe.num_experts_per_tok, True,
                      num_shared=len(moe.shared_experts), ffn=moe.config.moe_intermediate_size)
    return sorted(set(r["topk_idx"].reshape(-1).tolist()))


def _tol(dtype):
    return 1e-5 if dtype == torch.float32 else 1e-2


def _rel(a, b):
    return (torch.linalg.vector_norm((a.float() - b.float())) /
            torch.linalg.vector_norm(b.float()).clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_store_layers_match_full_model(tmp_path, dtype):
    """Per layer: ensure_resident(the layer's experts) then the layer with the
    store's mask == the full layer.  Four slots for eight experts, two layers:
    slots are reused between layers (eviction events order the copies)."""
    from project_chronos_b200 import CacheManager
    cfg = _cfg()
    full, lazy, state = _pair(cfg, 2, dtype)
    mgr = CacheManager(lazy, cfg, ssd_dir=str(tmp_path / "c"))
    mgr.expert_store.offload_from_state_dict(state)
    x = torch.randn(1, 2, cfg.hidden_size, device=DEV, dtype=dtype)
    with torch.no_grad():
        for li in range(2):
            f_moe = full.model.layers[li].mlp
            l_moe = lazy.model.layers[li].mlp
            need = _selected(f_moe, x)
            assert len(need) <= 4
            mgr.ensure_resident(need)
            y_full = f_moe(x)
            y_lazy = l_moe(x, available_expert_mask=mgr.availability_mask())
            torch.cuda.synchronize()
            assert l_moe.last_fallback_experts == []
            assert _rel(y_lazy, y_full) <= _tol(dtype)
    assert mgr.stats()["vram_experts"] <= 4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_forward_waits_on_ready_flags_not_on_the_stream(tmp_path, dtype):
    """The H2D stream is held back (a sleep kernel) so the copies land well
    after the forward starts; the GEMMs must wait on the experts' flags."""
    from project_chronos_b200 import CacheManager, ops
    cfg = _cfg(budget_experts=8)
    full, lazy, state = _pair(cfg, 1, dtype, seed=1)
    mgr = CacheManager(lazy, cfg, ssd_dir=str(tmp_path / "d"))
    store = mgr.expert_store
    store.offload_from_state_dict(state)
    x = torch.randn(1, 5, cfg.hidden_size, device=DEV, dtype=dtype)
    f_moe, l_moe = full.model.layers[0].mlp, lazy.model.layers[0].mlp
    need = _selected(f_moe, x)
    store.prefetch_to_ram(need)
    torch.cuda.synchronize()
    with torch.cuda.stream(store._h2d_stream):
        torch.cuda._sleep(100_000_000)   # ~50 ms of the H2D stream
    with torch.no_grad():
        newly = mgr.ensure_resident(need)
        assert newly == need
        y_lazy = l_moe(x, available_expert_mask=mgr.availability_mask())
        launched_before_copies = not store._h2d_stream.query()
        y_full = f_moe(x)
    torch.cuda.synchronize()
    ops.check_status(torch.device(DEV))
    assert launched_before_copies
    assert (store._ready[0, need] == 1).all()
    assert l_moe.last_fallback_experts == []
    assert _rel(y_lazy, y_full) <= _tol(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_sync_on_demand_with_one_slot_matches_full(tmp_path, dtype):
    """Reference tests/test_smoke.py:429-488 on the layer: every expert cold,
    a pool of ONE slot, the runtime loader promotes each selected expert; the
    layer computes them in passes and matches the full model."""
    from project_chronos_b200 import ExpertStore
    cfg = _cfg(budget_experts=1)
    full, lazy, state = _pair(cfg, 1, dtype, seed=2)
    store = ExpertStore(lazy, cfg, ssd_dir=str(tmp_path / "e"))
    assert store.vram_capacity == 1
    store.offload_from_state_dict(state)
    loaded = []

    def loader(eid):
        ok = store.promote_to_vram(eid)
        loaded.append(eid)
        return {"ok": ok}

    l_moe = lazy.model.layers[0].mlp
    l_moe.runtime_miss_policy = "sync_on_demand"
    l_moe.runtime_on_demand_loader = loader
    x = torch.randn(1, 6, cfg.hidden_size, device=DEV, dtype=dtype)
    cold = torch.zeros(cfg.num_experts, dtype=torch.bool)
    with torch.no_grad():
        y_full = full.model.layers[0].mlp(x)
        y_lazy = l_moe(x, available_expert_mask=cold)
    torch.cuda.synchronize()
    need = _selected(full.model.layers[0].mlp, x)
    assert sorted(loaded) == need
    assert l_moe.last_on_demand_experts == need
    assert l_moe.last_fallback_experts == []
    assert len(store.vram_lru) <= 1
    assert _rel(y_lazy, y_full) <= _tol(dtype)


def test_event_wait_mode_without_flags(tmp_path):
    """device_ready_flags=False: ensure_resident makes the compute stream wait
    on the promoted experts' events (the reference's M3 path)."""
    from project_chronos_b200 import CacheManager
    cfg = _cfg(flags=False)
    full, lazy, state = _pair(cfg, 1, torch.bfloat16, seed=3)
    mgr = CacheManager(lazy, cfg, ssd_dir=str(tmp_path / "f"))
    mgr.expert_store.offload_from_state_dict(state)
    assert lazy.model.layers[0].mlp.expert_ready_flags is None
    x = torch.randn(1, 2, cfg.hidden_size, device=DEV, dtype=torch.bfloat16)
    need = _selected(full.model.layers[0].mlp, x)
    with torch.no_grad():
        mgr.ensure_resident(need)
        y_lazy = lazy.model.layers[0].mlp(x, available_expert_mask=mgr.availability_mask())
        y_full = full.model.layers[0].mlp(x)
    torch.cuda.synchronize()
    assert _rel(y_lazy, y_full) <= 1e-2


def test_cluster_cold_tier_promotes_from_pinned_views(tmp_path):
    """.ctsr clusters: one pinned buffer per cluster, promotion copies straight from it."""
    from project_chronos_b200 import CacheManager
    cfg = _cfg(budget_experts=8)
    cfg.storage_format = "safetensors"
    full, lazy, state = _pair(cfg, 1, torch.bfloat16, seed=4)
    mgr = CacheManager(lazy, cfg, ssd_dir=str(tmp_path / "g"))
    store = mgr.expert_store
    store.offload_all_to_ssd(clusters=[[0, 1, 2, 3], [4, 5, 6, 7]])
    store.replace_live_experts_with_placeholders()
    x = torch.randn(1, 3, cfg.hidden_size, device=DEV, dtype=torch.bfloat16)
    need = _selected(full.model.layers[0].mlp, x)
    with torch.no_grad():
        mgr.ensure_resident(need)
        y_lazy = lazy.model.layers[0].mlp(x, available_expert_mask=mgr.availability_mask())
        y_full = full.model.layers[0].mlp(x)
    torch.cuda.synchronize()
    assert store.stats()["cluster_aware"] is True
    assert _rel(y_lazy, y_full) <= 1e-2


def _engine_hooks(mgr, policy):
    """The hooks the reference's engine installs (inference_engine.py:118-167):
    a miss already warm (or any miss under sync_on_demand) is promoted; a cold
    miss under on_demand is queued for the background reader and falls back."""
    store = mgr.expert_store

    def load_one(eid):
        eid = int(eid)
        if store.vram_lru.contains(eid) or store.ram_lru.contains(eid) or policy == "sync_on_demand":
            mgr.ensure_resident([eid])
            return {"ok": store.vram_lru.contains(eid)}
        mgr.prefetch_experts_to_ram([eid])
        return {"ok": False}

    return load_one, store.touch_expert


@pytest.mark.parametrize("policy", ["sync_on_demand", "on_demand"])
def test_decode_loop_replay(tmp_path, monkeypatch, policy):
    """The reference's decode-step call sequence (inference_engine.py:600-663)
    against the drop-ins: prefetch_experts_to_ram and prefetch_for_next_step of
    the previous step's lookahead predictions, ensure_resident of the warm
    candidates, availability_masks_all_layers, then every layer's forward with
    the engine's runtime hooks.  The SSD is slowed to 100 ms per read: the
    prefetch calls must not wait for one (each stays under half a read, though
    the background reader competes for the host meanwhile).  sync_on_demand must reproduce the
    full-resident model; on_demand must equal the blend with the fallbacks the
    layer reports (cold misses go to the shared expert)."""
    import time
    from oracle import moe_oracle as O
    from project_chronos_b200 import CacheManager
    cfg = _cfg(E=8, budget_experts=4)
    cfg.lookahead_steps = 2
    L, B, dtype = 2, 2, torch.bfloat16
    full, lazy, state = _pair(cfg, L, dtype, seed=7)
    mgr = CacheManager(lazy, cfg, ssd_dir=str(tmp_path / "loop"))
    store = mgr.expert_store
    store.offload_from_state_dict(state)
    mgr.start()
    monkeypatch.setenv("CHRONOS_SIM_SSD_MS", "100")
    load_one, touch_one = _engine_hooks(mgr, policy)
    for blk in lazy.model.layers:
        blk.mlp.runtime_miss_policy = policy
        blk.mlp.runtime_on_demand_loader = load_one
        blk.mlp.runtime_touch_expert = touch_one
    g = torch.Generator(device=DEV).manual_seed(11)
    prev_lp = None
    slowest_prefetch = 0.0
    try:
        mgr.warm_up([0, 1])
        for step in range(6):
            if prev_lp is not None:
                # the previous step's kernels are done: the timed region holds the two
                # read-backs of the predictions and the queueing, not a wait on the GPU
                torch.cuda.synchronize()
                t0 = time.monotonic()
                ram_ids = sorted({e for ids in mgr.predicted_experts(prev_lp) for e in ids})
                mgr.prefetch_experts_to_ram(ram_ids)
                mgr.prefetch_for_next_step(prev_lp)
                slowest_prefetch = max(slowest_prefetch, time.monotonic() - t0)
                ready = [e for e in ram_ids if store.vram_lru.contains(e) or store.ram_lru.contains(e)]
                mgr.ensure_resident(ready[:store.vram_capacity])
            masks = mgr.availability_masks_all_layers()
            x = torch.randn(B, 1, cfg.hidden_size, device=DEV, generator=g).to(dtype)
            xl_full, xl_lazy = x, x
            with torch.no_grad():
                for li in range(L):
                    f_moe, l_moe = full.model.layers[li].mlp, lazy.model.layers[li].mlp
                    y_full = f_moe(xl_full)
                    y_lazy = l_moe(xl_lazy, available_expert_mask=masks[li])
                    torch.cuda.synchronize()
                    if policy == "sync_on_demand":
                        assert l_moe.last_fallback_experts == []
                        assert _rel(y_lazy, y_full) <= 1e-2, (step, li)
                    else:
                        a = np.ones(cfg.num_experts, np.float32)
                        a[l_moe.last_fallback_experts] = 0.0
                        sd = {k: v.float().cpu().numpy() for k, v in f_moe.state_dict().items()}
                        stack = lambda n: np.stack([sd[f"experts.{e}.{n}.weight"]  # noqa: E731
                                                    for e in range(cfg.num_experts)])
                        want, *_ = O.moe_forward(
                            xl_lazy.float().cpu().numpy().reshape(B, -1), sd["gate.weight"],
                            stack("gate_proj"), stack("up_proj"), stack("down_proj"),
                            sd["shared_experts.0.gate_proj.weight"][None],
                            sd["shared_experts.0.up_proj.weight"][None],
                            sd["shared_experts.0.down_proj.weight"][None], cfg.num_experts_per_tok, True,
                            avail=a)
                        got = y_lazy.float().cpu().numpy().reshape(B, -1)
                        assert O.rel_l2(got, want) <= 1e-2, (step, li)
                    xl_full = xl_full + y_full
                    xl_lazy = xl_lazy + (y_full if policy == "sync_on_demand" else y_lazy)
            prev_lp = torch.softmax(torch.randn(B, 1, cfg.lookahead_steps + 1, cfg.num_experts,
                                                device=DEV, generator=g), dim=-1)
        assert slowest_prefetch < 0.05, slowest_prefetch
        assert mgr.prefetcher.drain(10.0)
        st = mgr.stats()
        assert st["vram_experts"] <= store.vram_capacity and st["total_requests"] > 0
    finally:
        mgr.stop()
    ops_status = __import__("project_chronos_b200").ops.check_status(torch.device(DEV))
    assert ops_status == 0
