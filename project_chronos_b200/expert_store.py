"""Pooled expert store: residency of routed experts in fixed device slots.

Drop-in for ``chronos/io/expert_store.py`` of FonaTech/Project_Chronos: the
class ``ExpertStore`` keeps the reference's constructor, method names,
arguments, return values and ``stats()`` keys, and ``vram_lru`` / ``ram_lru``
answer the calls engine code makes on them (``contains``, ``touch``,
``keys``, ``len``, a settable ``capacity``; ``inference_engine.py:123-130,
243-255``).  The implementation is built around the device pool the sm_100a
kernels read:

* Hot tier.  Every MoE layer owns P = ``vram_capacity`` slots in stacked pools
  (gate/up ``[P, F, H]``, down ``[P, H, F]``).  ``SlotTable`` is the one
  residency record: expert -> slot (the host array the layers and the device
  slot map mirror), slot -> expert, and a last-use stamp per slot; the
  occupied slot with the oldest stamp is the one given up.  Residency is per
  expert id across layers, as in the reference.
* Promotion is one pinned-host -> slot ``cudaMemcpyAsync`` per weight per
  layer on the dedicated H2D stream, each layer's copies followed by a 4-byte
  copy that sets ``ready[layer, e] = 1``.  The grouped GEMMs wait (bounded) on
  the flag of a SELECTED expert only, so a forward issued right after
  ``promote_to_vram`` computes every other expert while the copy lands.
  ``wait_for_experts`` keeps the reference's per-expert event wait on the
  compute stream (``expert_store.py:529-543``) for callers that want it.
* Giving a slot up writes slot -1 and flags 0 on the compute stream and
  records an event; the next copy into that slot (and the expert's next
  flag write) waits on it, so no copy overwrites weights a forward issued
  earlier still reads.
* Warm tier.  ``WarmTier`` holds each warm expert's pinned host tensors (all
  layers, already in the pool dtype so promotion is a plain copy) under a
  stamp order of its own, bounded by ``ram_capacity``; an expert dropped from
  a slot stays warm, and one whose warm copy is gone is copied back from its
  slot first.  It is thread-safe: ``CacheManager``'s background loader fills
  it while the decode thread promotes from it.
* Expert modules are still swapped between ``LazyExpertPlaceholder`` and a live
  ``FeedForward`` whose weights are views of the slot, so residency checks
  written against the reference's modules keep working.

Cold tier (both of the reference's formats): the clustered ``.ctsr`` layout
(``chronos/io/storage.py``, here ``cluster_storage.py``: a whole cluster read
with one sequential read into one pinned buffer) when ``storage_format`` is
``"safetensors"`` and a manifest is present, else one ``expert_l{L}_e{E}.pt``
per (layer, expert) holding fp16 ``{gate,up,down}_proj.weight``
(``expert_store.py:233-243, 321-322``).  ``CHRONOS_SIM_SSD_MS`` adds that many
milliseconds per cold read unit (a cluster, or one legacy expert), the
reference's SSD-latency knob (``chronos/io/io_simulator.py:23-40``).
"""
from __future__ import annotations

import itertools
import os
import re
import threading
import time
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from .cluster_storage import ClusterStorage

# (state-dict parameter name, pool name)
_WEIGHTS = (("gate_proj.weight", "gate"), ("up_proj.weight", "up"), ("down_proj.weight", "down"))
_EXPERT_KEY = re.compile(r"^model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(.+)$")

LayerStates = Dict[int, Dict[str, torch.Tensor]]   # layer -> {param: tensor}


def _simulated_read_delay() -> None:
    """Sleep ``CHRONOS_SIM_SSD_MS`` milliseconds (unset or 0: nothing)."""
    try:
        ms = float(os.environ.get("CHRONOS_SIM_SSD_MS", "0") or 0.0)
    except ValueError:
        ms = 0.0
    if ms > 0.0:
        time.sleep(ms / 1000.0)


class ResidencySet:
    """Expert ids held by a tier, each with a last-use stamp (a global counter);
    the smallest stamp is the first to go.  ``capacity`` may be changed at any
    time and is applied at the next insertion."""

    def __init__(self, capacity: int):
        self.capacity = int(capacity)
        self._stamp: Dict[int, int] = {}
        self._clock = itertools.count(1)
        self._lock = threading.RLock()

    def contains(self, key: int) -> bool:
        return int(key) in self._stamp

    def touch(self, key: int) -> None:
        key = int(key)
        with self._lock:
            if key in self._stamp:
                self._stamp[key] = next(self._clock)

    def put(self, key: int) -> Optional[int]:
        """Hold ``key`` (most recent); returns the id given up to make room, if any."""
        evicted = self.insert(key)
        return evicted[0] if evicted else None

    def insert(self, key: int) -> List[int]:
        """Hold ``key``; returns every id given up to fit ``capacity``."""
        key = int(key)
        out: List[int] = []
        with self._lock:
            if key not in self._stamp:
                while self._stamp and len(self._stamp) >= max(1, self.capacity):
                    victim = min(self._stamp, key=self._stamp.__getitem__)
                    del self._stamp[victim]
                    out.append(victim)
            self._stamp[key] = next(self._clock)
        return out

    def remove(self, key: int) -> None:
        with self._lock:
            self._stamp.pop(int(key), None)

    def keys(self) -> List[int]:
        """Held ids, the next to go first."""
        with self._lock:
            return sorted(self._stamp, key=self._stamp.__getitem__)

    def reorder_by_score(self, scores: Dict[int, float]) -> None:
        """Re-stamp by score: the lowest score (then the lowest id) goes first."""
        with self._lock:
            for key in sorted(self._stamp, key=lambda k: (float(scores.get(k, 0.0)), k)):
                self._stamp[key] = next(self._clock)

    def __len__(self) -> int:
        return len(self._stamp)


# The reference's name for the tier bookkeeping class (chronos/io/expert_store.py).
LRUCache = ResidencySet


class SlotTable:
    """Which expert each device slot holds, and in what order slots are given up.

    ``slot_of`` ([E] int32, -1 = not resident) is the host copy of the map the
    kernels read; the layers hold a reference to this very array.  ``stamp``
    is a per-slot last-use counter: among the occupied slots the smallest is
    the first reused.  Offers the calls engine code makes on ``vram_lru``."""

    def __init__(self, num_experts: int, num_slots: int, capacity: int):
        self.slot_of = np.full(num_experts, -1, dtype=np.int32)
        self.expert_in = np.full(num_slots, -1, dtype=np.int32)
        self.stamp = np.zeros(num_slots, dtype=np.int64)
        self.capacity = int(capacity)
        self._clock = itertools.count(1)
        self._lock = threading.RLock()

    # -- the reference's residency queries --------------------------------
    def contains(self, expert: int) -> bool:
        e = int(expert)
        return 0 <= e < self.slot_of.shape[0] and self.slot_of[e] >= 0

    def touch(self, expert: int) -> None:
        with self._lock:
            s = self.slot_of[int(expert)] if 0 <= int(expert) < self.slot_of.shape[0] else -1
            if s >= 0:
                self.stamp[s] = next(self._clock)

    def keys(self) -> List[int]:
        with self._lock:
            used = np.nonzero(self.expert_in >= 0)[0]
            return [int(self.expert_in[s]) for s in used[np.argsort(self.stamp[used], kind="stable")]]

    def reorder_by_score(self, scores: Dict[int, float]) -> None:
        with self._lock:
            for e in sorted(self.keys(), key=lambda k: (float(scores.get(k, 0.0)), k)):
                self.stamp[self.slot_of[e]] = next(self._clock)

    def __len__(self) -> int:
        return int((self.expert_in >= 0).sum())

    # -- slot assignment ------------------------------------------------------
    def victims_for(self, expert: int) -> List[int]:
        """Resident experts to give up so that ``expert`` fits both the slots and
        ``capacity`` (coldest first)."""
        with self._lock:
            limit = max(1, min(self.capacity, self.expert_in.shape[0]))
            order = [e for e in self.keys() if e != expert]
            excess = len(order) + 1 - limit
            return order[:max(0, excess)]

    def occupy(self, expert: int) -> int:
        """Put ``expert`` in a free slot (the caller gave up ``victims_for`` first)."""
        with self._lock:
            free = np.nonzero(self.expert_in < 0)[0]
            if free.size == 0:
                raise RuntimeError("no free device slot (give up victims_for() first)")
            s = int(free[0])
            self.expert_in[s] = expert
            self.slot_of[expert] = s
            self.stamp[s] = next(self._clock)
            return s

    def release(self, expert: int) -> int:
        with self._lock:
            s = int(self.slot_of[expert])
            if s >= 0:
                self.expert_in[s] = -1
                self.slot_of[expert] = -1
                self.stamp[s] = 0
            return s


class WarmTier(ResidencySet):
    """Pinned host copies of experts (every layer), bounded by ``capacity``; the
    least recently used warm expert is dropped first.  Offers the calls engine
    code makes on ``ram_lru``."""

    def __init__(self, capacity: int):
        super().__init__(capacity)
        self._states: Dict[int, LayerStates] = {}

    def get(self, expert: int) -> Optional[LayerStates]:
        with self._lock:
            return self._states.get(int(expert))

    def hold(self, expert: int, states: LayerStates) -> List[int]:
        """Keep ``states`` as ``expert``'s warm copy; returns the ids dropped."""
        with self._lock:
            dropped = self.insert(expert)
            for d in dropped:
                self._states.pop(d, None)
            self._states[int(expert)] = states
            return dropped

    def remove(self, key: int) -> None:
        with self._lock:
            super().remove(key)
            self._states.pop(int(key), None)


class _CopyFences:
    """One CUDA event per expert, recorded after its latest promotion's copies."""

    def __init__(self):
        self._ev: Dict[int, "torch.cuda.Event"] = {}
        self._lock = threading.Lock()

    def record(self, expert: int, stream: "torch.cuda.Stream") -> None:
        ev = torch.cuda.Event(blocking=False)
        ev.record(stream)
        with self._lock:
            self._ev[int(expert)] = ev

    def wait(self, experts: Iterable[int], stream: "torch.cuda.Stream") -> None:
        with self._lock:
            evs = [self._ev.pop(int(e)) for e in experts if int(e) in self._ev]
        for ev in evs:
            stream.wait_event(ev)

    def drop(self, expert: int) -> None:
        with self._lock:
            self._ev.pop(int(expert), None)

    def clear(self) -> None:
        with self._lock:
            self._ev.clear()


def _moe_layers(model) -> list:
    from .moe import ChronosMOEFeedForward
    inner = getattr(model, "model", None)
    layers = getattr(inner, "layers", None)
    if layers is None:
        layers = getattr(model, "layers", [])
    return [blk.mlp for blk in layers if isinstance(getattr(blk, "mlp", None), ChronosMOEFeedForward)]


def _available_ram_bytes() -> int:
    try:
        import psutil
        return int(psutil.virtual_memory().available)
    except ImportError:
        return 8 * (1024 ** 3)


class ExpertStore:
    """Three tiers for routed-expert weights: device slots (hot), pinned host
    memory (warm), ``.ctsr`` clusters or ``.pt`` files (cold).

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
        self._h2d_stream = torch.cuda.Stream(device=self.device) if self._cuda else None
        self.moe_layers = _moe_layers(model)
        self.num_layers = len(self.moe_layers)
        self.num_experts = int(config.num_experts)
        self.device_ready_flags = bool(getattr(config, "device_ready_flags", True))
        self.ready_timeout_ns = int(getattr(config, "expert_ready_timeout_ns", 0) or 0)

        self._expert_bytes = self._layer_expert_bytes()
        self._expert_dtype_cached = self._pool_dtype()
        self.vram_capacity, self.ram_capacity = self._capacities()

        # hot tier: created with the pools (replace_live_experts_with_placeholders)
        self._pools: Optional[List[Dict[str, torch.Tensor]]] = None
        self._slots = SlotTable(self.num_experts, min(self.vram_capacity, self.num_experts),
                                self.vram_capacity)
        self._slot_dev: Optional[torch.Tensor] = None    # [E] int32, device mirror of slot_of
        self._ready: Optional[torch.Tensor] = None       # [L, E] int32 device ready flags
        self._one: Optional[torch.Tensor] = None         # pinned 1, the flag copies' source
        self._slot_reuse_after: Dict[int, object] = {}   # slot -> event after its last reader
        self._flags_reset_after: Dict[int, object] = {}  # expert -> event after its flag reset
        self._fences = _CopyFences()
        # warm tier
        self._warm = WarmTier(self.ram_capacity)
        self._offloaded = False
        # cold tier
        self.storage_format = getattr(config, "storage_format", "safetensors")
        self._cluster_storage: Optional[ClusterStorage] = None
        if self.storage_format == "safetensors" and ClusterStorage.has_manifest(ssd_dir):
            self._cluster_storage = ClusterStorage(ssd_dir)

    # ------------------------------------------------------------------ tiers
    @property
    def vram_lru(self) -> SlotTable:
        """Residency of the device tier (the slot table)."""
        return self._slots

    @property
    def ram_lru(self) -> WarmTier:
        """Residency of the warm tier."""
        return self._warm

    # ------------------------------------------------------------------ sizes
    def _layer_expert_bytes(self) -> int:
        """fp16 bytes of one expert in one layer (the unit of the VRAM budget,
        ``expert_store.py:190-207``)."""
        if self.moe_layers:
            n = sum(p.numel() for p in self.moe_layers[0].experts[0].parameters())
            if n:
                return 2 * n
        h = int(getattr(self.config, "hidden_size", 0) or 0)
        f = int(getattr(self.config, "moe_intermediate_size", 0) or 0)
        return 2 * 3 * h * f

    def _pool_dtype(self) -> torch.dtype:
        for m in self.moe_layers[:1]:
            for mod in (m.experts[0], m.shared_experts, m.gate):
                p = next(mod.parameters(), None)
                if p is not None:
                    return p.dtype
        return torch.float16

    def _capacities(self) -> Tuple[int, int]:
        """(device slots, warm experts).  Same budget rules as the reference
        (``expert_store.py:125-143``): half of ``vram_budget_gb`` holds routed
        experts; the warm tier holds at most 4x that, and no more than
        ``pinned_memory_max_fraction`` of the available RAM."""
        per_expert = max(self._expert_bytes, 1)
        budget = float(getattr(self.config, "vram_budget_gb", 4.0)) * 2 ** 30
        slots = max(1, int(0.5 * budget / per_expert))
        return slots, max(1, min(4 * slots, self._ram_limit()))

    def _ram_limit(self) -> int:
        fraction = float(getattr(self.config, "pinned_memory_max_fraction", 0.25))
        return max(1, int(_available_ram_bytes() * fraction / max(self._expert_bytes * self.num_layers, 1)))

    @staticmethod
    def _physical_ram_bytes() -> int:
        return _available_ram_bytes()

    def _safe_ram_capacity(self) -> int:
        return max(1, min(self.ram_capacity, 4 * self.vram_capacity, self._ram_limit()))

    def _expert_size_bytes(self) -> int:
        return self._expert_bytes

    # ------------------------------------------------------------------ modules
    def _live_module(self, layer_idx: int, slot: int) -> nn.Module:
        """A ``FeedForward`` whose weights are views of ``slot`` in the layer's pools."""
        from .moe import FeedForward
        with torch.device("meta"):
            ff = FeedForward(self.config, intermediate_size=self.config.moe_intermediate_size)
        pool = self._pools[layer_idx]
        for lin, name in ((ff.gate_proj, "gate"), (ff.up_proj, "up"), (ff.down_proj, "down")):
            lin.weight = nn.Parameter(pool[name][slot], requires_grad=False)
        return ff

    def _placeholder(self) -> nn.Module:
        from .moe import LazyExpertPlaceholder
        return LazyExpertPlaceholder(self.config.hidden_size, self.config.moe_intermediate_size,
                                     self._expert_dtype_cached)

    def _set_modules(self, expert_id: int, make: Callable[[int], nn.Module]) -> None:
        for li, moe in enumerate(self.moe_layers):
            moe.experts[expert_id] = make(li)

    def _ensure_pools(self) -> None:
        """Allocate the slot pools and hand them to every layer (once)."""
        if self._pools is not None:
            return
        h, f = int(self.config.hidden_size), int(self.config.moe_intermediate_size)
        p = self._slots.expert_in.shape[0]
        dt, dev = self._expert_dtype_cached, self.device
        self._pools = [{"gate": torch.zeros(p, f, h, device=dev, dtype=dt),
                        "up": torch.zeros(p, f, h, device=dev, dtype=dt),
                        "down": torch.zeros(p, h, f, device=dev, dtype=dt)}
                       for _ in range(self.num_layers)]
        self._slot_dev = torch.from_numpy(self._slots.slot_of.copy()).to(dev)
        self._ready = torch.zeros(self.num_layers, self.num_experts, dtype=torch.int32, device=dev)
        if self._cuda:
            self._one = torch.ones(1, dtype=torch.int32).pin_memory()
        use_flags = self._cuda and self.device_ready_flags
        for li, moe in enumerate(self.moe_layers):
            pool = self._pools[li]
            moe.attach_expert_pool(pool["gate"], pool["up"], pool["down"], self._slot_dev,
                                   self._slots.slot_of, ready_flags=self._ready[li] if use_flags else None,
                                   ready_timeout_ns=self.ready_timeout_ns)

    # ------------------------------------------------------------------ cold tier
    def _ssd_path(self, expert_id: int, layer_idx: int) -> str:
        return os.path.join(self.ssd_dir, f"expert_l{layer_idx}_e{expert_id}.pt")

    def _write_shards(self, keys: Iterable[str], fetch: Callable[[str], torch.Tensor]) -> None:
        """One fp16 ``.pt`` per (layer, expert) from checkpoint-style keys
        (``model.layers.{L}.mlp.experts.{E}.{param}``): the keys are grouped in
        one pass and each shard is materialised only while it is written.
        Existing files are kept."""
        groups: Dict[Tuple[int, int], List[Tuple[str, str]]] = {}
        for key in keys:
            m = _EXPERT_KEY.match(key)
            if m is None:
                continue
            li, ei = int(m.group(1)), int(m.group(2))
            if li < self.num_layers and ei < self.num_experts:
                groups.setdefault((li, ei), []).append((m.group(3), key))
        for (li, ei), members in sorted(groups.items()):
            path = self._ssd_path(ei, li)
            if not os.path.exists(path):
                torch.save({param: fetch(key).detach().to(device="cpu", dtype=torch.float16).contiguous()
                            for param, key in members}, path)

    def _use_legacy_layout_unless(self, clusters) -> None:
        # a checkpoint or export has no co-activation clusters: one shard per
        # (layer, expert) keeps every miss a small read (expert_store.py:256-262)
        if self.storage_format == "safetensors" and clusters is None:
            self.storage_format = "pt"
            self._cluster_storage = None

    def offload_from_state_dict(self, state_dict: Dict[str, torch.Tensor],
                                clusters: Optional[List[List[int]]] = None,
                                replace_live: bool = True):
        """Write the cold tier straight from a checkpoint (``expert_store.py:245-274``)."""
        self._use_legacy_layout_unless(clusters)
        self._write_shards(state_dict.keys(), state_dict.__getitem__)
        if replace_live:
            self.replace_live_experts_with_placeholders()

    def offload_from_state_reader(self, reader, clusters: Optional[List[List[int]]] = None,
                                  replace_live: bool = True):
        """Write the cold tier from a random-access export reader (``reader.keys()``,
        ``reader.get_tensor(key)``, e.g. a safetensors ``safe_open`` handle or the
        reference's GGUF reader; ``expert_store.py:276-312``): each tensor is read
        only while its shard is written."""
        self._use_legacy_layout_unless(clusters)
        self._write_shards(list(reader.keys()), reader.get_tensor)
        if replace_live:
            self.replace_live_experts_with_placeholders()

    def offload_all_to_ssd(self, clusters: Optional[List[List[int]]] = None):
        """Write every live expert of every layer: ``.ctsr`` clusters + manifest when
        ``storage_format`` is ``"safetensors"`` (one all-expert cluster when
        ``clusters`` is None), else one ``.pt`` file per (layer, expert)
        (``expert_store.py:326-364``)."""
        if self.storage_format == "safetensors":
            ClusterStorage.write_clusters(self.moe_layers, clusters or [list(range(self.num_experts))],
                                          self.ssd_dir, self.num_layers, self.num_experts)
            self._cluster_storage = ClusterStorage(self.ssd_dir)
            return
        self._write_shards(
            (f"model.layers.{li}.mlp.experts.{ei}.{p}" for li, moe in enumerate(self.moe_layers)
             for ei, ex in enumerate(moe.experts) for p in ex.state_dict()),
            lambda key: self._live_param(key))

    def _live_param(self, key: str) -> torch.Tensor:
        m = _EXPERT_KEY.match(key)
        return self.moe_layers[int(m.group(1))].experts[int(m.group(2))].state_dict()[m.group(3)]

    def replace_live_experts_with_placeholders(self):
        """Drop every routed expert to a placeholder; the slot pools take over."""
        self._ensure_pools()
        for ei in range(self.num_experts):
            self._set_modules(ei, lambda _li: self._placeholder())
        self._offloaded = True

    def _read_legacy(self, expert_id: int) -> LayerStates:
        _simulated_read_delay()
        out: LayerStates = {}
        for li in range(self.num_layers):
            path = self._ssd_path(expert_id, li)
            if os.path.exists(path):
                out[li] = torch.load(path, map_location="cpu")
        return out

    # ------------------------------------------------------------------ warm tier
    def _pin(self, states: LayerStates) -> LayerStates:
        """In the pool dtype and page-locked, so that promotion is a plain copy."""
        dt = self._expert_dtype_cached

        def prep(t: torch.Tensor) -> torch.Tensor:
            t = t.to(dtype=dt).contiguous()
            if self._cuda and not t.is_pinned():
                try:
                    t = t.pin_memory()
                except RuntimeError:
                    pass
            return t

        return {li: {k: prep(v) for k, v in s.items()} for li, s in states.items()}

    def _keep_warm(self, expert_id: int, states: LayerStates) -> None:
        self._warm.capacity = self._safe_ram_capacity()
        self._warm.hold(expert_id, self._pin(states))

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
        With clusters, a request loads its whole cluster, each cluster at most
        once per call.  Safe to call from a background thread."""
        ids = [int(e) for e in (expert_ids or [])]
        for e in ids:
            self._warm.touch(e)
        missing = [e for e in dict.fromkeys(ids) if not self._warm.contains(e)]
        if not missing:
            return
        cs = self._cluster_storage
        if cs is None:
            for e in missing:
                states = self._read_legacy(e)
                if states:
                    self._keep_warm(e, states)
            return
        e2c = cs.manifest.expert_to_cluster
        for cid in dict.fromkeys(e2c[e] for e in missing if e in e2c):
            _simulated_read_delay()
            for e, states in cs.load_cluster(cid).items():
                if self._warm.contains(e):
                    self._warm.touch(e)
                else:
                    self._keep_warm(e, states)

    # ------------------------------------------------------------------ hot tier
    def promote_to_vram(self, expert_id: int, blocking: bool = False) -> bool:
        """Warm -> device slot.  Returns True when the expert is (being made) resident.

        The copies go on the H2D stream, each layer's followed by its ready
        flag; an event per expert is kept for ``wait_for_experts``.  With
        ``blocking=True`` the H2D stream is synchronised before returning."""
        e = int(expert_id)
        if not 0 <= e < self.num_experts:
            return False
        self._ensure_pools()
        if not self._slots.contains(e):  # a resident expert's slot already holds it: no copy
            states = self._warm.get(e)
            if states is None:
                self.prefetch_to_ram([e])
                states = self._warm.get(e)
                if states is None:
                    return False
            for victim in self._slots.victims_for(e):
                self._evict_from_vram(victim)
            slot = self._slots.occupy(e)
            self._fill_slot(e, slot, states)
            self._set_modules(e, lambda li: self._live_module(li, slot))
        self._slots.touch(e)
        self._warm.touch(e)
        if blocking:
            self.sync_h2d()
        return True

    def _fill_slot(self, expert: int, slot: int, states: LayerStates) -> None:
        """Map the slot (compute stream order), then the copies and flags on the
        H2D stream after the slot's previous reader and the flags' last reset."""
        self._slot_dev[expert:expert + 1].fill_(slot)
        h2d = self._h2d_stream
        if h2d is None:
            for li, st in states.items():
                for key, name in _WEIGHTS:
                    if key in st:
                        self._pools[li][name][slot].copy_(st[key])
                self._ready[li, expert] = 1
            return
        with torch.cuda.stream(h2d):
            for ev in (self._slot_reuse_after.pop(slot, None), self._flags_reset_after.pop(expert, None)):
                if ev is not None:
                    h2d.wait_event(ev)
            for li, st in states.items():
                for key, name in _WEIGHTS:
                    if key in st:
                        self._pools[li][name][slot].copy_(st[key], non_blocking=True)
                self._ready[li, expert:expert + 1].copy_(self._one, non_blocking=True)
        self._fences.record(expert, h2d)

    def _evict_from_vram(self, expert_id: int):
        """Give up the expert's slot, ordered after every forward issued so far;
        its weights stay in (or are copied back to) the warm tier."""
        e = int(expert_id)
        slot = int(self._slots.slot_of[e])
        if slot >= 0:
            if self._warm.get(e) is None:
                back = {li: {key: self._pools[li][name][slot].detach().cpu().clone()
                             for key, name in _WEIGHTS} for li in range(self.num_layers)}
                self._keep_warm(e, back)
            else:
                self._warm.touch(e)  # the expert leaving a slot is the most recent warm one
            self._slot_dev[e:e + 1].fill_(-1)
            self._ready[:, e].zero_()
            if self._cuda:
                ev = torch.cuda.Event(blocking=False)
                ev.record(torch.cuda.current_stream(self.device))
                self._slot_reuse_after[slot] = ev
                self._flags_reset_after[e] = ev
            self._slots.release(e)
            self._fences.drop(e)
        self._set_modules(e, lambda _li: self._placeholder())

    def wait_for_experts(self, expert_ids: List[int]) -> None:
        """Make the current stream wait for the named experts' copies only
        (``expert_store.py:529-543``); no host blocking."""
        if self._h2d_stream is not None:
            self._fences.wait(expert_ids, torch.cuda.current_stream(self.device))

    def touch_expert(self, expert_id: int) -> None:
        self._slots.touch(expert_id)
        self._warm.touch(expert_id)

    def reprioritize_resident_experts(self, scores: Dict[int, float]) -> None:
        self._slots.reorder_by_score(scores)
        self._warm.reorder_by_score(scores)

    def sync_h2d(self):
        """Wait for every pending copy (``expert_store.py:555-560``)."""
        if self._h2d_stream is not None:
            self._h2d_stream.synchronize()
        self._fences.clear()

    # ------------------------------------------------------------------ masks, stats
    def vram_availability_mask(self) -> torch.Tensor:
        """``[num_experts]`` bool, True for experts resident (or landing) in a slot."""
        return torch.from_numpy(self._slots.slot_of >= 0)

    def slot_of_expert(self) -> np.ndarray:
        """Host copy of the expert -> slot map (-1 = not resident)."""
        return self._slots.slot_of.copy()

    def stats(self) -> dict:
        gib = float(1 << 30)
        avail = _available_ram_bytes() / gib
        pinned = len(self._warm) * self._expert_bytes * self.num_layers / gib
        cs = self._cluster_storage
        return dict(
            vram_experts=len(self._slots), vram_capacity=self.vram_capacity,
            ram_experts=len(self._warm), ram_capacity_dynamic=self._safe_ram_capacity(),
            expert_size_kb=self._expert_bytes // 1024, pinned_ram_used_gb=round(pinned, 3),
            available_ram_gb=round(avail, 1), pinned_ram_fraction=round(pinned / max(avail, 1.0), 4),
            h2d_stream="dedicated" if self._h2d_stream is not None else "default",
            storage_format=self.storage_format, cluster_aware=cs is not None,
            num_clusters=len(cs.manifest.clusters) if cs is not None else 0,
            pool_slots=int(self._slots.expert_in.shape[0]) if self._pools else 0,
            device_ready_flags=bool(self._cuda and self.device_ready_flags))
