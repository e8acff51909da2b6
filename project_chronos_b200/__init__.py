"""B200-native (sm_100a) Chronos MoE feed-forward layer.

Public API (mirrors chronos/model/moe_chronos.py of FonaTech/Project_Chronos):

* ``ChronosMOEFeedForward``, ``LazyExpertPlaceholder``, ``FeedForward`` — the
  drop-in layer (``project_chronos_b200.moe``);
* ``ops.moe_forward`` / ``ops.moe_route`` — torch-level calls of the C ABI in
  ``include/chronos_moe.h``;
* ``synthetic`` — seeded workloads of the benchmark configurations.

Importing the package does not load the CUDA library; the first layer call
does, and raises if it is missing.
"""
from .moe import ChronosMOEFeedForward, FeedForward, LazyExpertPlaceholder  # noqa: F401

__all__ = ["ChronosMOEFeedForward", "FeedForward", "LazyExpertPlaceholder"]
