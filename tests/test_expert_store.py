"""Host logic of the pooled expert store and cache manager (CPU).

Mirrors the reference's store tests (tests/test_smoke.py of
FonaTech/Project_Chronos: ``test_lru_cache`` :127-134, ``test_expert_store_init``
:137-145) and checks the slot bookkeeping the device path relies on: slot
assignment and reuse under LRU eviction, the expert -> slot map, ready flags,
placeholders swapped in and out, the warm tier and the availability mask.
The copies run on CPU tensors here; the GPU tests cover the same flow with the
H2D stream, events and the kernels' ready-flag waits.
"""
import types

import numpy as np
import pytest
import torch
import torch.nn as nn


def _cfg(E=4, H=32, F=64, S=1, k=1, budget_experts=2):
    expert_fp16_bytes = 3 * H * F * 2
    return types.SimpleNamespace(
        hidden_size=H, num_experts=E, num_experts_per_tok=k, moe_intermediate_size=F,
        num_shared_experts=S, norm_topk_prob=False, router_aux_loss_coef=5e-4, hidden_act="silu",
        dropout=0.0, fallback_mask_prob=0.0, intermediate_size=F,
        # vram_capacity = budget * 0.5 / expert bytes
        vram_budget_gb=budget_experts * expert_fp16_bytes * 2 / (1024 ** 3),
        pinned_memory_max_fraction=0.25)


class _Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        from project_chronos_b200 import ChronosMOEFeedForward
        self.mlp = ChronosMOEFeedForward(cfg)


class _Model(nn.Module):
    """Stand-in with the reference model's ``model.layers[i].mlp`` structure."""

    def __init__(self, cfg, layers=2):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([_Block(cfg) for _ in range(layers)])


def _half_state(model):
    return {f"model.{k}": v.detach().half().float() for k, v in model.model.state_dict().items()}


def test_lru_cache():
    from project_chronos_b200 import LRUCache
    lru = LRUCache(capacity=3)
    lru.put(0); lru.put(1); lru.put(2)
    assert lru.put(3) == 0
    assert lru.contains(3) and not lru.contains(0)
    assert lru.put(3) is None
    lru.touch(1)
    assert lru.keys() == [2, 3, 1]
    lru.reorder_by_score({1: 0.1, 2: 0.9, 3: 0.5})
    assert lru.keys() == [1, 3, 2]
    assert lru.put(7) == 1
    lru.remove(3)
    assert len(lru) == 2


def test_expert_store_init(tmp_path):
    from project_chronos_b200 import ExpertStore
    cfg = _cfg()
    model = _Model(cfg)
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "cache"))
    s = store.stats()
    assert s["vram_capacity"] == 2
    assert s["ram_capacity_dynamic"] >= 1
    assert "available_ram_gb" in s
    assert store.num_layers == 2 and store.num_experts == 4


def test_offload_promote_evict_cycle(tmp_path):
    from project_chronos_b200 import ExpertStore, LazyExpertPlaceholder
    torch.manual_seed(0)
    cfg = _cfg()
    model = _Model(cfg)
    state = _half_state(model)
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "cache"))
    store.offload_from_state_dict(state)
    assert (tmp_path / "cache" / "expert_l1_e3.pt").exists()
    moes = store.moe_layers
    assert all(isinstance(m.experts[e], LazyExpertPlaceholder) for m in moes for e in range(4))
    assert store.vram_availability_mask().tolist() == [False] * 4

    assert store.promote_to_vram(2) is True
    assert store.promote_to_vram(0) is True
    slots = store.slot_of_expert()
    assert sorted([slots[2], slots[0]]) == [0, 1] and slots[1] == -1 and slots[3] == -1
    assert store.vram_availability_mask().tolist() == [True, False, True, False]
    assert store._slot_dev.tolist() == slots.tolist()
    assert store._ready[:, [0, 2]].eq(1).all() and store._ready[:, [1, 3]].eq(0).all()
    for li, m in enumerate(moes):
        ex = m.experts[2]
        assert not isinstance(ex, LazyExpertPlaceholder)
        want = state[f"model.layers.{li}.mlp.experts.2.up_proj.weight"]
        assert torch.equal(ex.up_proj.weight, want)
        # the live module's weight IS the slot of the pool (no separate copy)
        assert ex.up_proj.weight.data_ptr() == store._pools[li]["up"][slots[2]].data_ptr()

    # capacity 2: promoting a third expert evicts the least recent (2) and reuses its slot
    slot2 = int(slots[2])
    assert store.promote_to_vram(3) is True
    slots = store.slot_of_expert()
    assert slots[2] == -1 and slots[3] == slot2
    assert store._ready[:, 2].eq(0).all() and store._ready[:, 3].eq(1).all()
    assert all(isinstance(m.experts[2], LazyExpertPlaceholder) for m in moes)
    for li, m in enumerate(moes):
        want = state[f"model.layers.{li}.mlp.experts.3.down_proj.weight"]
        assert torch.equal(m.experts[3].down_proj.weight, want)
    assert store.ram_lru.contains(2)  # the evicted expert stays warm

    # re-promoting a resident expert keeps its slot and copies nothing
    before = store._pools[0]["gate"].clone()
    assert store.promote_to_vram(3) is True
    assert store.slot_of_expert()[3] == slot2
    assert torch.equal(before, store._pools[0]["gate"])

    # an id with no cold-tier file cannot be promoted
    assert store.promote_to_vram(99) is False


def test_eviction_without_warm_copy_writes_back(tmp_path):
    from project_chronos_b200 import ExpertStore
    torch.manual_seed(1)
    cfg = _cfg()
    model = _Model(cfg, layers=1)
    state = _half_state(model)
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "c"))
    store.offload_from_state_dict(state)
    store.promote_to_vram(1)
    store.ram_lru.remove(1)                 # warm copy gone
    assert store.ram_lru.get(1) is None
    for e in (2, 3):                        # evicts 1
        store.promote_to_vram(e)
    assert store.slot_of_expert()[1] == -1
    got = store.ram_lru.get(1)[0]["gate_proj.weight"]
    assert torch.equal(got, state["model.layers.0.mlp.experts.1.gate_proj.weight"])


def test_cache_manager_ensure_resident_and_masks(tmp_path):
    from project_chronos_b200 import CacheManager
    torch.manual_seed(2)
    cfg = _cfg(E=6, budget_experts=3)
    model = _Model(cfg)
    mgr = CacheManager(model, cfg, ssd_dir=str(tmp_path / "m"))
    mgr.expert_store.offload_from_state_dict(_half_state(model))
    mgr.warm_up([0, 1])
    assert mgr.availability_mask().tolist() == [True, True, False, False, False, False]
    newly = mgr.ensure_resident([1, 4, 5])
    assert newly == [4, 5]
    m = mgr.availability_mask().tolist()
    assert sum(m) == 3 and m[4] and m[5] and m[1]
    masks = mgr.availability_masks_all_layers()
    assert len(masks) == 2 and all(torch.equal(x, masks[0]) for x in masks)
    assert mgr.prefetch_experts_to_ram([3, 3, 2]) == [3, 2]
    st = mgr.stats()
    assert st["vram_experts"] == 3 and st["pool_slots"] == 3


def test_module_attached_pool_bookkeeping(tmp_path):
    """The layer adopts the store's pools: live experts = resident slots, the
    shared experts in the layer's own pool, the device slot map passed along."""
    from project_chronos_b200 import ExpertStore
    torch.manual_seed(3)
    cfg = _cfg()
    model = _Model(cfg, layers=1)
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "p"))
    store.offload_from_state_dict(_half_state(model))
    store.promote_to_vram(1)
    moe = store.moe_layers[0]
    moe._sync_pool(torch.device("cpu"), torch.float32)
    assert moe._live_np.tolist() == [0.0, 1.0, 0.0, 0.0]
    assert moe._pool["slot"] is store._slot_dev
    assert moe._pool["gate"] is store._pools[0]["gate"]
    assert moe.expert_ready_flags is None  # flags only on CUDA
    sh = moe.shared_experts[0].gate_proj.weight
    assert sh.data_ptr() == moe._pool["sh_gate"][0].data_ptr()
    with pytest.raises(RuntimeError, match="CUDA"):
        moe(torch.zeros(1, 1, cfg.hidden_size))
    np.testing.assert_array_equal(store.slot_of_expert(), [-1, 0, -1, -1])


# --------------------------------------------------------------------------
# clustered .ctsr cold tier (chronos/io/storage.py)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_tensor_file_format_is_safetensors(tmp_path, dtype):
    """Our writer and reader against the safetensors package, both directions."""
    st = pytest.importorskip("safetensors.torch")
    from project_chronos_b200.cluster_storage import read_tensor_file, write_tensor_file
    g = torch.Generator().manual_seed(0)
    tensors = {"l0_e1__gate_proj.weight": torch.randn(6, 5, generator=g).to(dtype),
               "l1_e0__down_proj.weight": torch.randn(3, 7, generator=g).to(dtype),
               "l0_e0__up_proj.weight": torch.randn(1, 2, generator=g).to(dtype)}
    ours = str(tmp_path / "ours.ctsr")
    write_tensor_file(ours, tensors)
    back = st.load_file(ours)
    assert set(back) == set(tensors) and all(torch.equal(back[k], tensors[k]) for k in tensors)
    theirs = str(tmp_path / "theirs.ctsr")
    st.save_file(tensors, theirs)
    got = read_tensor_file(theirs, pin=False)
    assert set(got) == set(tensors) and all(torch.equal(got[k], tensors[k]) for k in tensors)


def test_cluster_cold_tier_round_trip(tmp_path):
    from project_chronos_b200 import ExpertStore, LazyExpertPlaceholder
    from project_chronos_b200.cluster_storage import MANIFEST_FILENAME, ClusterStorage
    torch.manual_seed(4)
    cfg = _cfg(E=4)
    cfg.storage_format = "safetensors"
    model = _Model(cfg, layers=2)
    with torch.no_grad():  # fp16-representable weights: the cold tier stores fp16
        for p in model.parameters():
            p.copy_(p.half().float())
    want = {k: v.clone() for k, v in model.model.state_dict().items()}
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "cl"))
    store.offload_all_to_ssd(clusters=[[0, 2], [1, 3]])
    assert (tmp_path / "cl" / MANIFEST_FILENAME).exists()
    assert (tmp_path / "cl" / "cluster_1.ctsr").exists()
    cs = ClusterStorage(str(tmp_path / "cl"))
    nested = cs.load_cluster(1, pin=False)
    assert sorted(nested) == [1, 3] and sorted(nested[3]) == [0, 1]
    assert torch.equal(nested[3][1]["up_proj.weight"].float(), want["layers.1.mlp.experts.3.up_proj.weight"])
    store.replace_live_experts_with_placeholders()
    assert isinstance(store.moe_layers[0].experts[2], LazyExpertPlaceholder)
    store.prefetch_to_ram([2])                        # loads cluster 0: experts 0 and 2
    assert store.ram_lru.contains(0) and store.ram_lru.contains(2) and not store.ram_lru.contains(1)
    assert store.promote_to_vram(3) is True           # cluster 1 read on demand
    for li in range(2):
        got = store.moe_layers[li].experts[3].down_proj.weight
        assert torch.equal(got, want[f"layers.{li}.mlp.experts.3.down_proj.weight"])
    s = store.stats()
    assert s["cluster_aware"] is True and s["num_clusters"] == 2 and s["storage_format"] == "safetensors"


def test_bookkeeping_resolves_from_pending_statistics():
    """The fast path leaves the per-call statistics pending (device counts and
    weight mass, the availability used, and an on-demand mask built only when
    read); reading a bookkeeping attribute resolves them the way the reference
    fills its lists (moe_chronos.py:231-256): a selected expert that ran counts
    as on-demand when the mask marked it unavailable but it was live, a selected
    expert that did not run is a fallback."""
    from project_chronos_b200.moe import ChronosMOEFeedForward, _LazyOnDemand, _NO_ON_DEMAND
    cfg = _cfg(E=4)
    moe = ChronosMOEFeedForward(cfg)
    live = np.array([1, 1, 0, 1], dtype=np.float32)
    mask = np.array([1, 0, 0, 0], dtype=np.float32)
    counts = torch.tensor([3, 2, 1, 0], dtype=torch.int32)
    mass = torch.tensor([0.5, 0.25, 0.125, 0.0])
    lazy = _LazyOnDemand(mask, live)
    moe._stats_pending = dict(counts=counts, mass=mass, a=live.copy(), on_demand=lazy)
    assert lazy._v is None  # nothing computed until a bookkeeping attribute is read
    assert moe.last_on_demand_experts == [1]
    assert moe.last_fallback_experts == [2]
    assert moe.last_on_demand_weight_mass == pytest.approx(0.25)
    assert moe.last_fallback_weight_mass == pytest.approx(0.125)
    # without an eval-time mask nothing is on demand
    moe._stats_pending = dict(counts=counts, mass=mass, a=np.array([1, 1, 0, 1], np.float32),
                              on_demand=_NO_ON_DEMAND)
    assert moe.last_on_demand_experts == [] and moe.last_fallback_experts == [2]
    # a CUDA-less tensor mask is read back the same way
    lazy_t = _LazyOnDemand(torch.from_numpy(mask), live)
    assert [bool(lazy_t[e]) for e in range(4)] == [False, True, False, True]


def test_slot_table_capacity_and_order():
    """The device tier's residency record: slots reused coldest first, a lowered
    capacity applied at the next promotion, scores re-ordering the victims."""
    from project_chronos_b200.expert_store import SlotTable
    t = SlotTable(num_experts=6, num_slots=3, capacity=3)
    for e in (4, 1, 5):
        assert t.victims_for(e) == []
        t.occupy(e)
    assert t.keys() == [4, 1, 5] and len(t) == 3 and t.contains(1) and not t.contains(0)
    t.touch(4)
    assert t.victims_for(0) == [1]
    s1 = t.release(1)
    assert t.occupy(0) == s1 and t.slot_of[0] == s1 and t.slot_of[1] == -1
    t.reorder_by_score({5: 0.9, 4: 0.1, 0: 0.5})
    assert t.keys() == [4, 0, 5]
    t.capacity = 1
    assert t.victims_for(2) == [4, 0, 5]


def test_offload_from_state_reader_matches_state_dict(tmp_path):
    """offload_from_state_reader (expert_store.py:276-312) writes the same shards
    as offload_from_state_dict, reading each tensor through get_tensor."""
    from project_chronos_b200 import ExpertStore
    torch.manual_seed(5)
    cfg = _cfg()
    model = _Model(cfg)
    state = _half_state(model)
    reads = []

    class Reader:
        def keys(self):
            return list(state.keys())

        def get_tensor(self, key):
            reads.append(key)
            return state[key]

    a = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "a"))
    a.offload_from_state_reader(Reader(), replace_live=False)
    b = ExpertStore(_Model(cfg), cfg, ssd_dir=str(tmp_path / "b"))
    b.offload_from_state_dict(state, replace_live=False)
    assert a.storage_format == "pt"
    assert sorted(reads) == sorted(k for k in state if ".mlp.experts." in k)
    for li in range(2):
        for ei in range(4):
            x = torch.load(tmp_path / "a" / f"expert_l{li}_e{ei}.pt")
            y = torch.load(tmp_path / "b" / f"expert_l{li}_e{ei}.pt")
            assert sorted(x) == sorted(y) == ["down_proj.weight", "gate_proj.weight", "up_proj.weight"]
            assert all(torch.equal(x[k], y[k]) and x[k].dtype == torch.float16 for k in x)


def test_warm_loader_reads_in_background(tmp_path, monkeypatch):
    """prefetch_experts_to_ram returns without touching the disk once the loader
    runs (async_prefetcher.py:81-138): with 150 ms per simulated SSD read the
    call returns at once and the experts turn warm later."""
    import time
    from project_chronos_b200 import CacheManager
    torch.manual_seed(6)
    cfg = _cfg(E=6, budget_experts=3)
    model = _Model(cfg)
    mgr = CacheManager(model, cfg, ssd_dir=str(tmp_path / "w"))
    mgr.expert_store.offload_from_state_dict(_half_state(model))
    monkeypatch.setenv("CHRONOS_SIM_SSD_MS", "150")
    mgr.start()
    try:
        t0 = time.monotonic()
        assert mgr.prefetch_experts_to_ram([4, 5, 4]) == [4, 5]
        assert time.monotonic() - t0 < 0.1
        assert not mgr.expert_store.ram_lru.contains(4)
        assert mgr.prefetcher.wait_for(5, timeout=5.0)
        assert mgr.prefetcher.drain(5.0)
        assert mgr.expert_store.ram_lru.contains(4)
        st = mgr.stats()
        assert st["total_requests"] == 2 and st["prefetch_hits"] == 1 and "hit_rate" in st
    finally:
        mgr.stop()


def test_warm_loader_drops_the_oldest_request_when_full(tmp_path, monkeypatch):
    from project_chronos_b200.cache_manager import WarmLoader
    from project_chronos_b200 import ExpertStore
    cfg = _cfg(E=6, budget_experts=3)
    model = _Model(cfg)
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "q"))
    store.offload_from_state_dict(_half_state(model))
    monkeypatch.setenv("CHRONOS_SIM_SSD_MS", "200")
    loader = WarmLoader(store, queue_depth=1)
    loader.start()
    try:
        loader.submit([0])          # taken by the worker (busy ~200 ms)
        import time
        time.sleep(0.05)
        loader.submit([1])          # queued
        loader.submit([2])          # queue full: [1] dropped
        assert loader.drain(5.0)
        assert store.ram_lru.contains(0) and store.ram_lru.contains(2)
        assert not store.ram_lru.contains(1)
        assert loader.stats["dropped"] == 1
    finally:
        loader.stop()


def test_prefetch_for_next_step_and_step(tmp_path):
    """prefetch_for_next_step (cache_manager.py:94-98 -> async_prefetcher.py:198-223):
    per future step of the last token, the top-k experts of every row; step()
    promotes the current experts, queues the predictions and syncs."""
    from project_chronos_b200 import CacheManager
    cfg = _cfg(E=6, k=2, budget_experts=3)
    model = _Model(cfg)
    mgr = CacheManager(model, cfg, ssd_dir=str(tmp_path / "s"))
    mgr.expert_store.offload_from_state_dict(_half_state(model))
    lp = torch.zeros(2, 3, 3, 6)          # [B, S, K+1, E]
    lp[0, -1, 1, [5, 1]] = torch.tensor([0.6, 0.3])
    lp[1, -1, 1, [1, 2]] = torch.tensor([0.5, 0.4])
    lp[0, -1, 2, [0, 3]] = torch.tensor([0.7, 0.2])
    lp[1, -1, 2, [3, 4]] = torch.tensor([0.8, 0.1])
    lp[:, -1, 0, 2] = 1.0                 # the current step is not a prediction
    assert mgr.predicted_experts(lp) == [[1, 2, 5], [0, 3, 4]]
    assert mgr.prefetch_for_next_step(lp) == [1, 2, 5, 0, 3, 4]
    assert all(mgr.expert_store.ram_lru.contains(e) for e in (0, 1, 2, 3, 4, 5))  # not started: read inline
    assert mgr.prefetch_for_next_step(None) == []
    mgr.step(lp, [4, 0])
    assert mgr.availability_mask().tolist() == [True, False, False, False, True, False]


def test_reads_cluster_files_written_by_the_reference():
    """.ctsr files and manifest written by the reference's ClusterStorage.write_clusters
    (chronos/io/storage.py:182-233) load here with the weights they were given."""
    from project_chronos_b200 import synthetic as syn
    from project_chronos_b200.cluster_storage import ClusterStorage
    from tests import _golden as G
    root, c = G.ctsr_fixture()
    cs = ClusterStorage(root)
    m = cs.manifest
    assert m.num_experts == c["E"] and m.num_layers == c["L"]
    assert [cs.experts_in_cluster(i) for i in range(len(c["clusters"]))] == c["clusters"]
    want = [syn.make_workload(syn.MoEShape(c["H"], c["E"], 2, c["F"], c["S"]), 1, seed=s).weights
            for s in c["seeds"]]
    for cid, members in enumerate(c["clusters"]):
        nested = cs.load_cluster(cid, pin=False)
        assert sorted(nested) == sorted(members)
        for e in members:
            assert cs.cluster_for_expert(e) == cid
            for li in range(c["L"]):
                st = nested[e][li]
                assert st["gate_proj.weight"].dtype == torch.float16
                assert torch.equal(st["gate_proj.weight"], want[li].gate[e].half())
                assert torch.equal(st["up_proj.weight"], want[li].up[e].half())
                assert torch.equal(st["down_proj.weight"], want[li].down[e].half())


def test_store_serves_the_reference_written_clusters(tmp_path):
    """An ExpertStore attached to the reference-written cluster directory reads a
    whole cluster per request into the warm tier."""
    import shutil
    from project_chronos_b200 import ExpertStore
    from tests import _golden as G
    root, c = G.ctsr_fixture()
    cfg = _cfg(E=c["E"], H=c["H"], F=c["F"], budget_experts=2)
    cfg.storage_format = "safetensors"
    shutil.copytree(root, tmp_path / "ref")
    model = _Model(cfg, layers=c["L"])
    store = ExpertStore(model, cfg, ssd_dir=str(tmp_path / "ref"))
    assert store.stats()["cluster_aware"] is True
    store.replace_live_experts_with_placeholders()
    store.prefetch_to_ram([3])
    assert store.ram_lru.contains(1) and store.ram_lru.contains(3) and not store.ram_lru.contains(0)
    assert store.promote_to_vram(3) is True
    assert store.vram_availability_mask().tolist() == [False, False, False, True]


def test_bookkeeping_uses_the_mask_of_the_call():
    """The on-demand statistics are resolved lazily, but from the mask as it was
    at forward time: a caller that updates its mask in place afterwards does not
    change them (the reference fills its lists during forward)."""
    from project_chronos_b200.moe import _LazyOnDemand
    mask = torch.tensor([1.0, 0.0, 0.0, 1.0])
    live = np.array([1, 1, 0, 1], dtype=np.float32)
    snap = np.array(mask.detach().to(torch.float32).numpy(), copy=True)
    lazy = _LazyOnDemand(snap, live)
    mask.zero_()
    assert [bool(lazy[e]) for e in range(4)] == [False, True, False, False]
