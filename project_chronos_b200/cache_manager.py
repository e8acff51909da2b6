"""Cache manager over the pooled expert store.

Mirrors ``chronos/runtime/cache_manager.py`` of FonaTech/Project_Chronos
(``CacheManager``: same constructor, ``availability_mask``,
``availability_masks_all_layers``, ``warm_up``, ``ensure_resident``,
``prefetch_experts_to_ram``, ``start``/``stop``, ``stats``).

``ensure_resident`` promotes the missing experts with non-blocking copies.
With device ready flags on (the default on CUDA) it does not make the compute
stream wait on them: the expert GEMMs wait per selected expert on the flags,
so the copies overlap the layers' other work.  Without flags it waits on the
promoted experts' events, as the reference does (``cache_manager.py:107-118``).

The reference's background SSD prefetcher and lookahead scheduler
(``chronos/io/async_prefetcher.py``) are not part of this package:
``prefetch_experts_to_ram`` loads synchronously, ``start``/``stop`` are kept
for interface compatibility.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from .expert_store import ExpertStore


class CacheManager:
    def __init__(self, model, config, ssd_dir: str = "./expert_cache"):
        self.config = config
        self.expert_store = ExpertStore(model, config, ssd_dir=ssd_dir)
        self._num_layers = len(self.expert_store.moe_layers)
        self._prefetched = 0

    def start(self):
        """Kept for interface compatibility (no background thread)."""

    def stop(self):
        """Kept for interface compatibility (no background thread)."""

    def warm_up(self, initial_expert_ids: Optional[List[int]] = None):
        """Make the given experts (default 0..capacity-1) resident and wait for them."""
        store = self.expert_store
        if initial_expert_ids is None:
            initial_expert_ids = list(range(min(self.config.num_experts, store.vram_capacity)))
        store.prefetch_to_ram(initial_expert_ids)
        for eid in initial_expert_ids:
            store.promote_to_vram(eid)
        store.sync_h2d()

    def availability_mask(self) -> torch.Tensor:
        """``[num_experts]`` bool, True when the expert has a device slot."""
        return self.expert_store.vram_availability_mask()

    def availability_masks_all_layers(self) -> List[torch.Tensor]:
        mask = self.availability_mask()
        return [mask] * self._num_layers

    def prefetch_experts_to_ram(self, expert_ids: List[int]) -> List[int]:
        """Cold -> warm for the given ids (deduplicated, order kept)."""
        ids = list(dict.fromkeys(int(e) for e in expert_ids or []))
        if ids:
            self.expert_store.prefetch_to_ram(ids)
            self._prefetched += len(ids)
        return ids

    def ensure_resident(self, expert_ids: List[int]) -> List[int]:
        """Promote the ids that are not resident; returns those newly promoted."""
        store = self.expert_store
        newly = []
        for eid in expert_ids:
            if not store.vram_lru.contains(int(eid)):
                if store.promote_to_vram(int(eid), blocking=False):
                    newly.append(int(eid))
        if not (store._cuda and store.device_ready_flags):
            store.wait_for_experts(newly)
        return newly

    def stats(self) -> dict:
        return {**self.expert_store.stats(), "prefetch_submitted": self._prefetched}
