"""B200-native (sm_100a) Chronos MoE feed-forward layer.

Public API (mirrors chronos/model/moe_chronos.py of FonaTech/Project_Chronos):

* ``ChronosMOEFeedForward``, ``LazyExpertPlaceholder``, ``FeedForward`` — the
  drop-in layer (``project_chronos_b200.moe``);
* ``ops.moe_forward`` / ``ops.moe_route`` — torch-level calls of the C ABI in
  ``include/chronos_moe.h``;
* ``ExpertStore``, ``LRUCache`` (``expert_store``) and ``CacheManager``
  (``cache_manager``) — pooled expert residency with device ready flags
  (mirrors chronos/io/expert_store.py and chronos/runtime/cache_manager.py);
* ``LookaheadRouter`` (``lookahead``) — the lookahead routing predictor
  (chronos/model/lookahead_router.py) as one fused kernel;
* ``synthetic`` — seeded workloads of the benchmark configurations.

Importing the package does not load the CUDA library; the first layer call
does, and raises if it is missing.
"""
from .moe import ChronosMOEFeedForward, FeedForward, LazyExpertPlaceholder  # noqa: F401
from .expert_store import ExpertStore, LRUCache  # noqa: F401
from .cache_manager import CacheManager  # noqa: F401
from .lookahead import LookaheadRouter  # noqa: F401

__all__ = ["ChronosMOEFeedForward", "FeedForward", "LazyExpertPlaceholder", "ExpertStore", "LRUCache",
           "CacheManager", "LookaheadRouter"]
