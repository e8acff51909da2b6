"""B200-native (sm_100a) Chronos MoE feed-forward layer.

Public API (mirrors chronos/model/moe_chronos.py of FonaTech/Project_Chronos):

* ``ChronosMOEFeedForward``, ``LazyExpertPlaceholder``, ``FeedForward`` — the
  drop-in layer (``project_chronos_b200.moe``);
* ``ops.moe_forward`` / ``ops.moe_route`` — torch-level calls of the C ABI in
  ``include/chronos_moe.h``;
* ``ExpertStore`` (``expert_store``; ``LRUCache`` is the reference's name for
  its residency sets) and ``CacheManager`` with its background SSD -> RAM
  reader ``WarmLoader`` (``cache_manager``) — pooled expert residency with
  device ready flags (mirrors chronos/io/expert_store.py,
  chronos/runtime/cache_manager.py and chronos/io/async_prefetcher.py);
* ``LookaheadRouter`` (``lookahead``) — the lookahead routing predictor
  (chronos/model/lookahead_router.py) as one fused kernel;
* ``synthetic`` — seeded workloads of the benchmark configurations.

Importing the package does not load the CUDA library; the first layer call
does, and raises if it is missing.
"""
from .moe import ChronosMOEFeedForward, FeedForward, LazyExpertPlaceholder  # noqa: F401
from .expert_store import ExpertStore, LRUCache, ResidencySet, SlotTable, WarmTier  # noqa: F401
from .cache_manager import CacheManager, WarmLoader  # noqa: F401
from .lookahead import LookaheadRouter  # noqa: F401

__all__ = ["ChronosMOEFeedForward", "FeedForward", "LazyExpertPlaceholder", "ExpertStore", "LRUCache",
           "ResidencySet", "SlotTable", "WarmTier", "CacheManager", "WarmLoader", "LookaheadRouter"]
