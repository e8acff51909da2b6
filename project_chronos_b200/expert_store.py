"""Pooled expert store: residency of routed experts in fixed device slots.

Mirrors ``chronos/io/expert_store.py`` of FonaTech/Project_Chronos (class
``ExpertStore``, ``LRUCache``; same constructor, method names, arguments,
return values and stats keys) with the device tier rebuilt for the sm_100a
kernels:

* The reference keeps each resident expert as its own ``nn.Module`` and
  promotes it with ``load_state_dict`` (``expert_store.py:480-527``).  Here
  every MoE layer owns P = ``vram_capacity`` slots in stacked pools
  (gate/up ``[P, F, H]``, down ``[P, H, F]``), shared by all layers under one
  expert -> slot map (residency is per expert id across layers, as in the
  reference's ``vram_lru``).  Promotion is one pinned-host -> slot
  ``cudaMemcpyAsync`` per weight per layer on the dedicated H2D stream.
* Per-(layer, expert) device ready flags: after a layer's copies the H2D
  stream writes ``ready[layer, e] = 1``; the grouped GEMMs wait (bounded) on
  the flag of a SELECTED expert only, so a forward issued right after
  ``promote_to_vram`` computes every other expert while the copy lands, and
  layer 0 needs only its own slice.  ``wait_for_experts`` keeps the
  reference's per-expert event wait on the compute stream
  (``expert_store.py:529-543``) for callers that want it.
* Eviction (LRU, ``expert_store.py:499-501, 562-587``) frees the slot on the
  compute stream: slot map entry -1 and flags 0 are written there and an event
  recorded; the next copy into that slot waits on the event, so it never
  overwrites weights an earlier forward still reads.  The warm (RAM) tier keeps
  the weights, so nothing is copied back unless its RAM copy was dropped.
* Expert modules are still swapped between ``LazyExpertPlaceholder`` and a live
  ``FeedForward`` (whose weights are views of its slot), so residency checks
  written against the reference's modules keep working.

Disk formats (both the reference's): the clustered ``.ctsr`` layout
(``chronos/io/storage.py``, here ``cluster_storage.py``: a whole cluster read
with one sequential read into one pinned buffer) when the config's
``storage_format`` is ``"safetensors"`` (the reference's default) and a
manifest is present, else the legacy layout, one ``expert_l{L}_e{E}.pt`` per
(layer, expert) holding fp16 ``{gate,up,down}_proj.weight``
(``expert_store.py:233-243, 321-322``).  The warm tier holds pinned tensors in
the pool dtype so that promotion is a plain copy.
"""
from __future__ import annotations

import collections
import contextlib
import os
import threading
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.nn as nn

from .cluster_storage import ClusterStorage

_WEIGHTS = (("gate_proj.weight", "gate"), ("up_proj.weight", "up"), ("down_proj.weight", "down"))


class LRUCache:
    """Thread-safe LRU set of expert ids (``chronos/io/expert_store.py:34-82``)."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self._cache: "collections.OrderedDict[int, bool]" = collections.OrderedDict()
        self._lock = threading.Lock()

    def contains(self, key: int) -> bool:
        with self._lock:
            return key in self._cache

    def touch(self, key: int):
        with self._lock:
            if key in self._cache:
                self._cache.move_to_end(key)

    def put(self, key: int) -> Optional[int]:
        """Insert ``key`` as most recent; returns the evicted key when full."""
        with self._lock:
            if key in self._cache:
                self._cache.move_to_end(key)
                return None
            evicted = None
            if len(self._cache) >= self.capacity:
                evicted, _ = self._cache.popitem(last=False)
            self._cache[key] = True
            return evicted

    def remove(self, key: int):
        with self._lock:
            self._cache.pop(key, None)

    def keys(self) -> List[int]:
        with self._lock:
            return list(self._cache.keys())

    def reorder_by_score(self, scores: Dict[int, float]):
        """Coldest (lowest score, then lowest id) first, so they are evicted first."""
        with self._lock:
            order = sorted(self._cache.keys(), key=lambda k: (float(scores.get(k, 0.0)), k))
            self._cache = collections.OrderedDict((k, True) for k in order)

    def __len__(self):
        with self._lock:
            return len(self._cache)


def _moe_layers(model) -> list:
    from .moe import ChronosMOEFeedForward
    inner = getattr(model, "model", None)
    layers = getattr(inner, "layers", None)
    if layers is None:
        layers = getattr(model, "layers", [])
    return [blk.mlp for blk in layers if isinstance(getattr(blk, "mlp", None), ChronosMOEFeedForward)]


class ExpertStore:
    """Three tiers for routed-expert weights: device slots (hot), pinned host
    memory (warm), ``.pt`` files (cold).

        store = ExpertStore(model, config, ssd_dir="./expert_cache")
        store.offload_from_state_dict(state_dict)   # writes the cold tier, placeholders in
        store.prefetch_to_ram([0, 2])                # cold -> warm
        store.promote_to_vram(0)                     # warm -> slot (async, ready flag)
        mask = store.vram_availability_mask()        # [E] bool
    """

    def __init__(self, model, config, ssd_dir: str = "./expert_cache"):
        self.config = config
        self.ssd_dir = ssd_dir
        self.model = model
        self.device = next(model.parameters()).device
        os.makedirs(ssd_dir, exist_ok=True)
        self._cuda = self.device.type == "cuda"
        self._h2d_stream: Optional[torch.cuda.Stream] = (
            torch.cuda.Stream(device=self.device) if self._cuda else None)

        self.moe_layers = _moe_layers(model)
        self.num_experts = int(config.num_experts)
        self.num_layers = len(self.moe_layers)

        expert_bytes = self._expert_size_bytes()
        self._expert_bytes = expert_bytes
        self._expert_dtype_cached = self._expert_dtype()
        vram_bytes = float(getattr(config, "vram_budget_gb", 4.0)) * (1024 ** 3)
        # half the budget for routed experts (shared experts, KV cache get the rest),
        # as expert_store.py:127-130
        self.vram_capacity = max(1, int(vram_bytes * 0.5 / max(expert_bytes, 1)))
        max_fraction = getattr(config, "pinned_memory_max_fraction", 0.25)
        per_expert_ram = max(expert_bytes * self.num_layers, 1)
        ram_by_safety = max(1, int(self._physical_ram_bytes() * max_fraction / per_expert_ram))
        self.ram_capacity = min(self.vram_capacity * 4, ram_by_safety)

        self.vram_lru = LRUCache(capacity=self.vram_capacity)
        self.ram_lru = LRUCache(capacity=self.ram_capacity)
        self._ram_buffers: Dict[int, Dict[int, Dict[str, torch.Tensor]]] = {}
        self._ram_lock = threading.Lock()
        self._offloaded = False
        self._pending_events: Dict[int, "torch.cuda.Event"] = {}
        self._events_lock = threading.Lock()
        self.storage_format = getattr(config, "storage_format", "safetensors")
        self._cluster_storage: Optional[ClusterStorage] = None
        if self.storage_format == "safetensors" and ClusterStorage.has_manifest(ssd_dir):
            self._cluster_storage = ClusterStorage(ssd_dir)

        # device slot pools, created when the routed experts become placeholders
        self._pools: Optional[List[Dict[str, torch.Tensor]]] = None
        self._slot_host = np.full(self.num_experts, -1, dtype=np.int32)
        self._slot_dev: Optional[torch.Tensor] = None
        self._ready: Optional[torch.Tensor] = None        # [L, E] int32
        self._free_slots: List[int] = []
        self._slot_free_event: Dict[int, object] = {}     # slot -> event after its last reader
        self._flag_reset_event: Dict[int, object] = {}    # expert -> event after its flags reset
        self._one = None
        self.ready_timeout_ns = int(getattr(config, "expert_ready_timeout_ns", 0) or 0)
        self.device_ready_flags = bool(getattr(config, "device_ready_flags", True))

    # ------------------------------------------------------------------ sizes
    @staticmethod
    def _physical_ram_bytes() -> int:
        try:
            import psutil
            return int(psutil.virtual_memory().available)
        except ImportError:
            return 8 * (1024 ** 3)

    def _safe_ram_capacity(self) -> int:
        max_fraction = getattr(self.config, "pinned_memory_max_fraction", 0.25)
        per_expert_ram = max(self._expert_size_bytes() * self.num_layers, 1)
        return max(1, min(self.ram_capacity, self.vram_capacity * 4,
                          int(self._physical_ram_bytes() * max_fraction / per_expert_ram)))

    def _expert_size_bytes(self) -> int:
        """fp16 bytes of one expert in one layer (``expert_store.py:190-207``)."""
        hidden = int(getattr(self.config, "hidden_size", 0) or 0)
        inter = int(getattr(self.config, "moe_intermediate_size", 0) or 0)
        if self.moe_layers:
            size = sum(p.numel() * 2 for p in self.moe_layers[0].experts[0].parameters())
            if size:
                return size
        cached = getattr(self, "_expert_bytes", 0)
        if cached:
            return cached
        return 3 * hidden * inter * 2 if hidden and inter else 0

    def _expert_dtype(self) -> torch.dtype:
        if self.moe_layers:
            for p in self.moe_layers[0].experts[0].parameters():
                return p.dtype
            for p in self.moe_layers[0].shared_experts.parameters():
                return p.dtype
            return self.moe_layers[0].gate.weight.dtype
        return getattr(self, "_expert_dtype_cached", torch.float16)

    # ------------------------------------------------------------------ modules
    def _build_live_expert(self, layer_idx: int, slot: int) -> nn.Module:
        """A ``FeedForward`` whose weights are views of ``slot`` in the layer's pools."""
        from .moe import FeedForward
        with torch.device("meta"):
            ff = FeedForward(self.config, intermediate_size=self.config.moe_intermediate_size)
        pools = self._pools[layer_idx]
        ff.gate_proj.weight = nn.Parameter(pools["gate"][slot], requires_grad=False)
        ff.up_proj.weight = nn.Parameter(pools["up"][slot], requires_grad=False)
        ff.down_proj.weight = nn.Parameter(pools["down"][slot], requires_grad=False)
        return ff

    def _build_placeholder_expert(self):
        from .moe import LazyExpertPlaceholder
        return LazyExpertPlaceholder(self.config.hidden_size, self.config.moe_intermediate_size,
                                     self._expert_dtype_cached)

    def _replace_expert_module(self, layer_idx: int, expert_id: int, module: nn.Module):
        self.moe_layers[layer_idx].experts[expert_id] = module

    def _ensure_pools(self) -> None:
        """Allocate the slot pools and hand them to every layer (once)."""
        if self._pools is not None:
            return
        H = int(self.config.hidden_size)
        Fd = int(self.config.moe_intermediate_size)
        P = min(self.vram_capacity, self.num_experts)
        dt = self._expert_dtype_cached
        dev = self.device
        self._pools = [dict(gate=torch.zeros(P, Fd, H, device=dev, dtype=dt),
                            up=torch.zeros(P, Fd, H, device=dev, dtype=dt),
                            down=torch.zeros(P, H, Fd, device=dev, dtype=dt))
                       for _ in range(self.num_layers)]
        self._slot_dev = torch.full((self.num_experts,), -1, dtype=torch.int32, device=dev)
        self._ready = torch.zeros(self.num_layers, self.num_experts, dtype=torch.int32, device=dev)
        self._free_slots = list(range(P - 1, -1, -1))
        if self._cuda:
            self._one = torch.ones(1, dtype=torch.int32).pin_memory()
        for li, moe in enumerate(self.moe_layers):
            flags = self._ready[li] if (self._cuda and self.device_ready_flags) else None
            moe.attach_expert_pool(self._pools[li]["gate"], self._pools[li]["up"],
                                   self._pools[li]["down"], self._slot_dev, self._slot_host,
                                   ready_flags=flags, ready_timeout_ns=self.ready_timeout_ns)

    # ------------------------------------------------------------------ cold tier
    def _ssd_path(self, expert_id: int, layer_idx: int) -> str:
        return os.path.join(self.ssd_dir, f"expert_l{layer_idx}_e{expert_id}.pt")

    @staticmethod
    def _expert_state_from_checkpoint(state_dict: Dict[str, torch.Tensor], layer_idx: int,
                                      expert_id: int) -> Dict[str, torch.Tensor]:
        prefix = f"model.layers.{layer_idx}.mlp.experts.{expert_id}."
        return {k[len(prefix):]: v.detach().to(dtype=torch.float16, device="cpu").contiguous()
                for k, v in state_dict.items() if k.startswith(prefix)}

    def offload_from_state_dict(self, state_dict: Dict[str, torch.Tensor],
                                clusters: Optional[List[List[int]]] = None,
                                replace_live: bool = True):
        """Write the cold tier straight from a checkpoint (``expert_store.py:245-274``):
        one ``.pt`` file per (layer, expert), as the reference does (a raw checkpoint
        has no co-activation clusters)."""
        if self.storage_format == "safetensors" and clusters is None:
            self.storage_format = "pt"
            self._cluster_storage = None
        for li in range(self.num_layers):
            for ei in range(self.num_experts):
                path = self._ssd_path(ei, li)
                if os.path.exists(path):
                    continue
                state = self._expert_state_from_checkpoint(state_dict, li, ei)
                if state:
                    torch.save(state, path)
        if replace_live:
            self.replace_live_experts_with_placeholders()

    def offload_all_to_ssd(self, clusters: Optional[List[List[int]]] = None):
        """Write every live expert of every layer: ``.ctsr`` clusters + manifest when
        ``storage_format`` is ``"safetensors"`` (one all-expert cluster when
        ``clusters`` is None), else one ``.pt`` file per (layer, expert)
        (``expert_store.py:326-364``)."""
        if self.storage_format == "safetensors":
            if clusters is None:
                clusters = [list(range(self.num_experts))]
            ClusterStorage.write_clusters(self.moe_layers, clusters, self.ssd_dir, self.num_layers,
                                          self.num_experts)
            self._cluster_storage = ClusterStorage(self.ssd_dir)
            return
        for li, moe in enumerate(self.moe_layers):
            for ei, expert in enumerate(moe.experts):
                path = self._ssd_path(ei, li)
                if os.path.exists(path):
                    continue
                state = {k: v.detach().to(dtype=torch.float16, device="cpu").contiguous()
                         for k, v in expert.state_dict().items()}
                if state:
                    torch.save(state, path)

    def replace_live_experts_with_placeholders(self):
        """Drop every routed expert to a placeholder; the slot pools take over."""
        self._ensure_pools()
        for li in range(self.num_layers):
            for ei in range(self.num_experts):
                self._replace_expert_module(li, ei, self._build_placeholder_expert())
        self._offloaded = True

    def _load_from_ssd(self, expert_id: int) -> Dict[int, Dict[str, torch.Tensor]]:
        states: Dict[int, Dict[str, torch.Tensor]] = {}
        for li in range(self.num_layers):
            path = self._ssd_path(expert_id, li)
            if os.path.exists(path):
                states[li] = torch.load(path, map_location="cpu")
        return states

    # ------------------------------------------------------------------ warm tier
    def _pin_layer_states(self, layer_states: Dict[int, Dict[str, torch.Tensor]]
                          ) -> Dict[int, Dict[str, torch.Tensor]]:
        """Convert to the pool dtype once and pin, so promotion is a plain copy."""
        dt = self._expert_dtype_cached
        out: Dict[int, Dict[str, torch.Tensor]] = {}
        for li, state in layer_states.items():
            out[li] = {}
            for k, v in state.items():
                t = v.to(dtype=dt).contiguous()
                if self._cuda and not t.is_pinned():
                    try:
                        t = t.pin_memory()
                    except RuntimeError:
                        pass
                out[li][k] = t
        return out

    def attach_cluster_manifest(self, manifest_dir: Optional[str] = None) -> bool:
        """Use the ``.ctsr`` clusters under ``manifest_dir`` (default: the cache dir)."""
        root = manifest_dir or self.ssd_dir
        if not ClusterStorage.has_manifest(root):
            return False
        self._cluster_storage = ClusterStorage(root)
        self.storage_format = "safetensors"
        return True

    def prefetch_to_ram(self, expert_ids: List[int]):
        """Cold -> warm for each id not already warm (``expert_store.py:389-463``).
        With clusters, a request loads its whole cluster (one read per cluster)."""
        if self._cluster_storage is not None:
            self._prefetch_clustered(expert_ids or [])
            return
        for eid in expert_ids or []:
            eid = int(eid)
            if self.ram_lru.contains(eid):
                self.ram_lru.touch(eid)
                continue
            self.ram_lru.capacity = self._safe_ram_capacity()
            states = self._load_from_ssd(eid)
            if not states:
                continue
            pinned = self._pin_layer_states(states)
            with self._ram_lock:
                evicted = self.ram_lru.put(eid)
                if evicted is not None:
                    self._ram_buffers.pop(evicted, None)
                self._ram_buffers[eid] = pinned

    def _prefetch_clustered(self, expert_ids: List[int]) -> None:
        cs = self._cluster_storage
        to_load: List[int] = []
        for eid in expert_ids:
            eid = int(eid)
            if eid not in cs.manifest.expert_to_cluster:
                continue
            if self.ram_lru.contains(eid):
                self.ram_lru.touch(eid)
                continue
            cid = cs.cluster_for_expert(eid)
            if cid not in to_load:
                to_load.append(cid)
        for cid in to_load:
            nested = cs.load_cluster(cid)
            self.ram_lru.capacity = self._safe_ram_capacity()
            for eid, layer_states in nested.items():
                if self.ram_lru.contains(eid):
                    self.ram_lru.touch(eid)
                    continue
                pinned = self._pin_layer_states(layer_states)
                with self._ram_lock:
                    evicted = self.ram_lru.put(eid)
                    if evicted is not None:
                        self._ram_buffers.pop(evicted, None)
                    self._ram_buffers[eid] = pinned

    # ------------------------------------------------------------------ hot tier
    def promote_to_vram(self, expert_id: int, blocking: bool = False) -> bool:
        """Warm -> device slot.  Returns True when the expert is (being made) resident.

        The copies go on the H2D stream, each layer's followed by its ready
        flag; an event per expert is kept for ``wait_for_experts``.  With
        ``blocking=True`` the H2D stream is synchronised before returning."""
        expert_id = int(expert_id)
        if not self.ram_lru.contains(expert_id):
            self.prefetch_to_ram([expert_id])
        with self._ram_lock:
            layer_states = self._ram_buffers.get(expert_id)
        if layer_states is None:
            return False
        self._ensure_pools()
        if self._slot_host[expert_id] >= 0:
            # already resident: the slot holds its weights (no re-copy)
            self.vram_lru.put(expert_id)
            if blocking:
                self.sync_h2d()
            return True

        evicted = self.vram_lru.put(expert_id)
        if evicted is not None:
            self._evict_from_vram(evicted)
        if not self._free_slots:  # capacity lowered below the resident count
            for victim in self.vram_lru.keys():
                if victim != expert_id and self._slot_host[victim] >= 0:
                    self.vram_lru.remove(victim)
                    self._evict_from_vram(victim)
                    break
        slot = self._free_slots.pop()

        # mapping, visible to every forward issued after this call (stream order)
        self._slot_dev[expert_id:expert_id + 1].fill_(slot)
        self._slot_host[expert_id] = slot
        ctx = torch.cuda.stream(self._h2d_stream) if self._h2d_stream is not None \
            else contextlib.nullcontext()
        with ctx:
            if self._h2d_stream is not None:
                for ev in (self._slot_free_event.pop(slot, None),
                           self._flag_reset_event.pop(expert_id, None)):
                    if ev is not None:
                        self._h2d_stream.wait_event(ev)
            for li in range(self.num_layers):
                state = layer_states.get(li)
                if state is None:
                    continue
                pools = self._pools[li]
                for key, name in _WEIGHTS:
                    src = state.get(key)
                    if src is not None:
                        pools[name][slot].copy_(src, non_blocking=True)
                if self._one is not None:
                    self._ready[li, expert_id:expert_id + 1].copy_(self._one, non_blocking=True)
                else:
                    self._ready[li, expert_id] = 1
            if self._h2d_stream is not None:
                evt = torch.cuda.Event(blocking=False)
                evt.record(self._h2d_stream)
                with self._events_lock:
                    self._pending_events[expert_id] = evt
        for li in range(self.num_layers):
            self._replace_expert_module(li, expert_id, self._build_live_expert(li, slot))
        if blocking:
            self.sync_h2d()
        return True

    def wait_for_experts(self, expert_ids: List[int]) -> None:
        """Make the current stream wait for the named experts' copies only
        (``expert_store.py:529-543``); no host blocking."""
        if self._h2d_stream is None:
            return
        current = torch.cuda.current_stream(self.device)
        with self._events_lock:
            events = [self._pending_events.pop(int(e), None) for e in expert_ids]
        for evt in events:
            if evt is not None:
                current.wait_event(evt)

    def touch_expert(self, expert_id: int) -> None:
        self.vram_lru.touch(expert_id)
        self.ram_lru.touch(expert_id)

    def reprioritize_resident_experts(self, scores: Dict[int, float]) -> None:
        self.vram_lru.reorder_by_score(scores)
        self.ram_lru.reorder_by_score(scores)

    def sync_h2d(self):
        """Wait for every pending copy (``expert_store.py:555-560``)."""
        if self._h2d_stream is not None:
            self._h2d_stream.synchronize()
        with self._events_lock:
            self._pending_events.clear()

    def _evict_from_vram(self, expert_id: int):
        """Free the expert's slot, ordered after every forward issued so far."""
        expert_id = int(expert_id)
        slot = int(self._slot_host[expert_id])
        if slot >= 0:
            with self._ram_lock:
                have_ram = expert_id in self._ram_buffers
            if not have_ram:  # keep the weights: write the slot back to the warm tier
                states = {li: {key: self._pools[li][name][slot].detach().to("cpu").clone()
                               for key, name in _WEIGHTS} for li in range(self.num_layers)}
                with self._ram_lock:
                    self._ram_buffers[expert_id] = self._pin_layer_states(states)
            self._slot_dev[expert_id:expert_id + 1].fill_(-1)
            self._ready[:, expert_id].zero_()
            self._slot_host[expert_id] = -1
            if self._cuda:
                ev = torch.cuda.Event(blocking=False)
                ev.record(torch.cuda.current_stream(self.device))
                self._slot_free_event[slot] = ev
                self._flag_reset_event[expert_id] = ev
            self._free_slots.append(slot)
            with self._events_lock:
                self._pending_events.pop(expert_id, None)
        for li in range(self.num_layers):
            self._replace_expert_module(li, expert_id, self._build_placeholder_expert())
        with self._ram_lock:
            evicted = self.ram_lru.put(expert_id)
            if evicted is not None and evicted != expert_id:
                self._ram_buffers.pop(evicted, None)
        self.vram_lru.remove(expert_id)

    # ------------------------------------------------------------------ masks, stats
    def vram_availability_mask(self) -> torch.Tensor:
        """``[num_experts]`` bool, True for experts resident (or landing) in a slot."""
        mask = torch.zeros(self.num_experts, dtype=torch.bool)
        for eid in self.vram_lru.keys():
            if eid < self.num_experts:
                mask[eid] = True
        return mask

    def slot_of_expert(self) -> np.ndarray:
        """Host copy of the expert -> slot map (-1 = not resident)."""
        return self._slot_host.copy()

    def stats(self) -> dict:
        available_ram_gb = self._physical_ram_bytes() / (1024 ** 3)
        pinned_used_gb = len(self.ram_lru) * self._expert_size_bytes() * self.num_layers / (1024 ** 3)
        return {
            "vram_experts": len(self.vram_lru),
            "vram_capacity": self.vram_capacity,
            "ram_experts": len(self.ram_lru),
            "ram_capacity_dynamic": self._safe_ram_capacity(),
            "expert_size_kb": self._expert_size_bytes() // 1024,
            "pinned_ram_used_gb": round(pinned_used_gb, 3),
            "available_ram_gb": round(available_ram_gb, 1),
            "pinned_ram_fraction": round(pinned_used_gb / max(available_ram_gb, 1), 4),
            "h2d_stream": "dedicated" if self._h2d_stream is not None else "default",
            "storage_format": self.storage_format,
            "cluster_aware": self._cluster_storage is not None,
            "num_clusters": (len(self._cluster_storage.manifest.clusters)
                             if self._cluster_storage is not None else 0),
            "pool_slots": int(self._pools[0]["gate"].shape[0]) if self._pools else 0,
            "device_ready_flags": bool(self._cuda and self.device_ready_flags),
        }
