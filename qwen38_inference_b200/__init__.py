"""B200-native (sm_100a) hybrid Gated-DeltaNet / gated-GQA ``forward_step``.

Drop-in for the reference API: ``Qwen38``, ``HybridCache``, ``forward_step``,
``generate`` and ``new_cache``. The GPU work runs in ``libqw200.so`` (C ABI in
include/qw200.h); build it with ``python -m qwen38_inference_b200.build``.
"""
from .model import HybridCache, Qwen38, forward_step, generate, new_cache  # noqa: F401

__all__ = ["Qwen38", "HybridCache", "forward_step", "generate", "new_cache"]
