"""hexo_bot_b200 — B200-native Shrimp leaf-evaluation forward.

The Shrimp policy/value network of Cmiller132/hexo-bot, served by hand-written
sm_100a kernels behind a C ABI (include/shrimp_b200.h). Public API:

- ShrimpNet (hexo_bot_b200.model): the reference module tree; forward_policy_value
  runs natively on CUDA tensors.
- ShrimpEvaluator (hexo_bot_b200.evaluator): the serve-side wire-ABI evaluator.
- featurize / positions: host-side input builders.
"""

from . import constants, geometry  # noqa: F401

__all__ = ["constants", "geometry"]
