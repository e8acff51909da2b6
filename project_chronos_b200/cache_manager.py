"""Cache manager over the pooled expert store.

Drop-in for ``chronos/runtime/cache_manager.py`` of FonaTech/Project_Chronos:
``CacheManager`` keeps the reference's constructor, ``start``/``stop``,
``warm_up``, ``availability_mask``, ``availability_masks_all_layers``,
``step``, ``prefetch_for_next_step``, ``prefetch_experts_to_ram``,
``ensure_resident`` and ``stats`` (the calls the reference's decode loop makes,
``inference_engine.py:600-663``), and ``prefetcher`` answers ``submit`` /
``wait_for`` / ``stats`` as the reference's ``AsyncPrefetcher`` does
(``chronos/io/async_prefetcher.py:29-147``).

* ``ensure_resident`` promotes the missing experts with non-blocking copies.
  With device ready flags on (the default on CUDA) it does not make the compute
  stream wait: the expert GEMMs wait per selected expert on the flags, so the
  copies overlap the layers' other work.  Without flags it waits on the
  promoted experts' events, as the reference does (``cache_manager.py:107-118``).
* SSD -> RAM reads run on one background thread (``WarmLoader``): requests are
  batches of expert ids in a bounded queue; when it is full the OLDEST batch
  is dropped (the newest prediction is the one worth reading,
  ``async_prefetcher.py:81-96``).  The decode thread never reads the disk for
  ``prefetch_experts_to_ram`` / ``prefetch_for_next_step``.  Before ``start()``
  (and after ``stop()``) requests are read on the caller's thread.
* ``prefetch_for_next_step`` ranks the lookahead router's predictions on the
  device and reads them back once: for every future step k of the last
  token, the top-``num_experts_per_tok`` experts of every batch row, sorted
  and deduplicated per step, submitted step by step (t+1 first), as the
  reference's ``PrefetchScheduler.prefetch_only`` (``async_prefetcher.py:198-223``).
"""
from __future__ import annotations

import collections
import threading
import time
from typing import Deque, List, Optional

import torch

from .cluster_storage import ClusterStorage
from .expert_store import ExpertStore


class WarmLoader:
    """One daemon thread that reads requested experts into the warm tier."""

    def __init__(self, store: ExpertStore, queue_depth: int = 8, log_fn=None):
        self.store = store
        self.queue_depth = max(1, int(queue_depth))
        self.log_fn = log_fn or (lambda _msg: None)
        self._pending: Deque[List[int]] = collections.deque()
        self._cv = threading.Condition()
        self._thread: Optional[threading.Thread] = None
        self._running = False
        self._busy = False
        self._counts = {"prefetch_hits": 0, "prefetch_misses": 0, "total_requests": 0, "dropped": 0}

    # -- lifecycle -------------------------------------------------------------
    def start(self) -> None:
        with self._cv:
            if self._running:
                return
            self._running = True
        self._thread = threading.Thread(target=self._run, name="chronos-warm-loader", daemon=True)
        self._thread.start()

    def stop(self, timeout: float = 2.0) -> None:
        with self._cv:
            self._running = False
            self._cv.notify_all()
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None

    @property
    def running(self) -> bool:
        return self._running and self._thread is not None

    # -- requests --------------------------------------------------------------
    def submit(self, expert_ids: List[int]) -> None:
        """Queue one batch (non-blocking); a full queue gives up its oldest batch."""
        ids = [int(e) for e in expert_ids or []]
        if not ids:
            return
        if not self.running:
            self._load(ids)
            return
        with self._cv:
            while len(self._pending) >= self.queue_depth:
                self._pending.popleft()
                self._counts["dropped"] += 1
            self._pending.append(ids)
            self._cv.notify()

    def wait_for(self, expert_id: int, timeout: float = 0.05) -> bool:
        """True once the expert is warm or resident (polls until ``timeout`` s)."""
        deadline = time.monotonic() + timeout
        store = self.store
        while True:
            if store.ram_lru.contains(expert_id) or store.vram_lru.contains(expert_id):
                self._counts["prefetch_hits"] += 1
                return True
            if time.monotonic() >= deadline:
                self._counts["prefetch_misses"] += 1
                return False
            time.sleep(0.0005)

    def drain(self, timeout: float = 10.0) -> bool:
        """Wait until every queued batch has been read (tests, shutdown)."""
        deadline = time.monotonic() + timeout
        with self._cv:
            while self._pending or self._busy:
                left = deadline - time.monotonic()
                if left <= 0:
                    return False
                self._cv.wait(left)
        return True

    # -- worker ----------------------------------------------------------------
    def _load(self, ids: List[int]) -> None:
        self._counts["total_requests"] += len(ids)
        store = self.store
        cold = [e for e in ids if not (store.ram_lru.contains(e) or store.vram_lru.contains(e))]
        if cold:
            try:
                store.prefetch_to_ram(cold)
            except Exception as exc:  # a failed read leaves the expert cold; the layer falls back
                self.log_fn(f"[warm-loader] reading {cold} failed: {exc}")

    def _run(self) -> None:
        while True:
            with self._cv:
                while self._running and not self._pending:
                    self._cv.wait(0.05)
                if not self._running:
                    self._pending.clear()
                    self._cv.notify_all()
                    return
                batch = self._pending.popleft()
                self._busy = True
            try:
                self._load(batch)
            finally:
                with self._cv:
                    self._busy = False
                    self._cv.notify_all()

    @property
    def stats(self) -> dict:
        s = dict(self._counts)
        s["hit_rate"] = s["prefetch_hits"] / max(1, s["prefetch_hits"] + s["prefetch_misses"])
        return s


class CacheManager:
    def __init__(self, model, config, ssd_dir: str = "./expert_cache"):
        self.config = config
        self.expert_store = ExpertStore(model, config, ssd_dir=ssd_dir)
        self.prefetcher = WarmLoader(self.expert_store,
                                     queue_depth=int(getattr(config, "prefetch_queue_depth", 8) or 8))
        self._num_layers = len(self.expert_store.moe_layers)
        # a manifest named by the config wins over one in the cache directory
        # (cache_manager.py:42-49)
        override = getattr(config, "cluster_manifest_path", None)
        if override and ClusterStorage.has_manifest(override):
            self.expert_store.attach_cluster_manifest(override)
        elif ClusterStorage.has_manifest(ssd_dir):
            self.expert_store.attach_cluster_manifest(ssd_dir)

    def start(self):
        """Start the background SSD -> RAM reader."""
        self.prefetcher.start()

    def stop(self):
        """Stop the background reader (queued requests are dropped)."""
        self.prefetcher.stop()

    def warm_up(self, initial_expert_ids: Optional[List[int]] = None):
        """Make the given experts (default 0..capacity-1) resident and wait for them."""
        store = self.expert_store
        ids = initial_expert_ids
        if ids is None:
            ids = list(range(min(self.config.num_experts, store.vram_capacity)))
        store.prefetch_to_ram(ids)
        for eid in ids:
            store.promote_to_vram(eid)
        store.sync_h2d()

    def availability_mask(self) -> torch.Tensor:
        """``[num_experts]`` bool, True when the expert has a device slot."""
        return self.expert_store.vram_availability_mask()

    def availability_masks_all_layers(self) -> List[torch.Tensor]:
        return [self.availability_mask()] * self._num_layers

    def _promote(self, expert_ids: List[int], blocking: bool) -> List[int]:
        store = self.expert_store
        newly = []
        for eid in expert_ids:
            eid = int(eid)
            if not store.vram_lru.contains(eid) and store.promote_to_vram(eid, blocking=blocking):
                newly.append(eid)
        return newly

    def ensure_resident(self, expert_ids: List[int]) -> List[int]:
        """Promote the ids that are not resident; returns those newly promoted."""
        store = self.expert_store
        newly = self._promote(expert_ids, blocking=False)
        if not (store._cuda and store.device_ready_flags):
            store.wait_for_experts(newly)
        return newly

    def prefetch_experts_to_ram(self, expert_ids: List[int]) -> List[int]:
        """Queue these ids for the background reader (deduplicated, order kept)."""
        ids = list(dict.fromkeys(int(e) for e in expert_ids or []))
        self.prefetcher.submit(ids)
        return ids

    def predicted_experts(self, lookahead_probs) -> List[List[int]]:
        """Per future step (t+1, t+2, ...): the sorted ids the lookahead router
        ranks in the top ``num_experts_per_tok`` for the last token of any row."""
        if lookahead_probs is None or lookahead_probs.dim() != 4 or lookahead_probs.shape[2] < 2:
            return []
        k = max(1, min(int(getattr(self.config, "num_experts_per_tok", 1) or 1),
                       int(lookahead_probs.shape[-1])))
        top = torch.topk(lookahead_probs[:, -1, 1:, :], k=k, dim=-1).indices   # [B, K, k] on device
        top = top.transpose(0, 1).reshape(top.shape[1], -1).cpu()              # one read-back
        return [sorted(set(row.tolist())) for row in top]

    def prefetch_for_next_step(self, lookahead_probs) -> List[int]:
        """Queue the lookahead predictions for the background reader (non-blocking;
        call before the next forward).  Returns the ids submitted, t+1's first."""
        submitted: List[int] = []
        for ids in self.predicted_experts(lookahead_probs):
            if ids:
                self.prefetcher.submit(ids)
                submitted.extend(ids)
        return list(dict.fromkeys(submitted))

    def step(self, lookahead_probs, current_expert_ids: List[int]):
        """The reference's single-call step (``cache_manager.py:83-90``): promote the
        current experts and wait for them, queue the predictions, then wait for
        every copy."""
        self._promote(current_expert_ids, blocking=True)
        self.prefetch_for_next_step(lookahead_probs)
        self.expert_store.sync_h2d()

    def stats(self) -> dict:
        return {**self.expert_store.stats(), **self.prefetcher.stats}
