"""Policy vocabulary and configuration checks of the eviction overlay.

Names, modes and the {name, budget, prefix, recent, seed} configuration follow
the reference overlay (code/cache_eviction/sglang_evict_runtime.py:4-8, 44-46,
625-637).  h2o_global_2048 is the one addition: one kept set per (layer, row)
shared by every KV head, ranked by the sum of the heads' H2O scores.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import capi

INTERVAL = 2048          # boundaries fall before queries 2048, 4096, ... (runtime:44)

# decode score mode per policy (runtime:45-46); h2o_global accumulates like head_sum
POLICIES = {"random_2048": 3, "random_reservoir_2048": 3,
            "prefix_sliding_2048": 3, "head_sum_2048": 1, "head_max_sum_2048": 2,
            "h2o_global_2048": 1}
SCORE_MODE = {"head_sum_2048": capi.CE_MODE_SUM, "head_max_sum_2048": capi.CE_MODE_MAX,
              "h2o_global_2048": capi.CE_MODE_SUM}
POLICY_IDS = {"prefix_sliding_2048": capi.CE_POLICY_PREFIX_SLIDING,
              "random_2048": capi.CE_POLICY_RANDOM,
              "random_reservoir_2048": capi.CE_POLICY_RESERVOIR,
              "head_sum_2048": capi.CE_POLICY_HEAD_SUM,
              "head_max_sum_2048": capi.CE_POLICY_HEAD_MAX,
              "h2o_global_2048": capi.CE_POLICY_H2O_GLOBAL}
# short names used by the ragged-batch configuration (benchmark configs 3 and 5)
ALIASES = {"recent": "prefix_sliding_2048", "random": "random_2048",
           "reservoir": "random_reservoir_2048", "h2o_per_head": "head_sum_2048",
           "h2o_max": "head_max_sum_2048", "h2o_global": "h2o_global_2048"}


def canonical(name: str) -> str:
    return ALIASES.get(name, name)


@dataclass(frozen=True)
class EvictionConfig:
    """Validated eviction settings of one request, in tokens."""
    name: str
    budget: int
    prefix: int
    recent: int
    seed: int = 0
    record: bool = False

    @property
    def mode(self) -> int:
        return POLICIES[self.name]

    @property
    def score_mode(self) -> int:
        return SCORE_MODE.get(self.name, capi.CE_MODE_NONE)

    @property
    def policy_id(self) -> int:
        return POLICY_IDS[self.name]

    def units(self, page_size: int) -> tuple[int, int, int]:
        return self.budget // page_size, self.prefix // page_size, self.recent // page_size


def validate(cfg: dict, page_size: int = 1) -> EvictionConfig:
    """The reference's checks (runtime:630-634) plus page alignment.

    Raises ValueError with the reference's messages.
    """
    try:
        name = canonical(cfg["name"])
        budget, prefix, recent = int(cfg["budget"]), int(cfg["prefix"]), int(cfg["recent"])
    except (KeyError, TypeError) as error:
        raise ValueError(str(error)) from error
    if name not in POLICIES or min(prefix, recent) < 0 or prefix + recent > budget:
        raise ValueError("invalid gstar eviction settings")
    if name == "prefix_sliding_2048" and prefix + recent != budget:
        raise ValueError("Prefix Sliding requires B = P + R")
    if page_size > 1 and (budget % page_size or prefix % page_size or recent % page_size):
        raise ValueError(f"budget, prefix and recent must be multiples of the page size {page_size}")
    return EvictionConfig(name, budget, prefix, recent, int(cfg.get("seed", 0)), bool(cfg.get("record", False)))


def sweep_split(budget: int, name: str) -> tuple[int, int]:
    """The study's convention P = R = B/4, Prefix Sliding R = 3B/4
    (code/cache_eviction/sglang_static.py:41-44)."""
    prefix = budget // 4
    recent = budget - prefix if canonical(name) == "prefix_sliding_2048" else budget // 4
    return prefix, recent
