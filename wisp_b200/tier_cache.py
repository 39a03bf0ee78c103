"""Next-token expert prediction from observed routing.

The reference's tier cache predicts which experts each layer will need from what its
router picked so far (wisp/runtime/tier_cache.py:118-177): per layer a frequency table
fed by the experts that fired (``observe``, or ``drain_engine_log`` from the engine's
access log), ``predict(layer)`` = the 2 * top_k most frequent experts, and
``prefetch_all_layers`` sends them as prefetch hints.  MoE routing is sticky within a
workload, so the frequent experts are the likely next ones.  Here the hints go to the
engine's prefetch queue (``wisp_expert_prefetch_hint``: SSD reads into the RAM tier
on its worker thread) or to the streaming cache (``StreamingStack.step(predictor=)``:
pinned-pool copies into HBM slots for the next layer).
"""

from __future__ import annotations

from collections import Counter


class ExpertPredictor:
    """Per-layer expert frequencies; optionally feeds a ``LearningCache``."""

    def __init__(self, num_layers: int, top_k: int, learning_cache=None):
        self.num_layers = num_layers
        self.top_k = top_k
        self.learning_cache = learning_cache
        self._freq = [Counter() for _ in range(num_layers)]
        self.dropped_observations = 0

    def observe(self, layer_idx: int, expert_ids) -> None:
        """The experts layer `layer_idx` routed to (negative ids: unrouted slots)."""
        freq = self._freq[layer_idx]
        ids = [int(e) for e in expert_ids if int(e) >= 0]
        for e in ids:
            freq[e] += 1
        if self.learning_cache is not None and ids:
            self.learning_cache.record_hits((layer_idx, e) for e in ids)

    def drain_engine_log(self, engine) -> int:
        """Feed the engine's access log (``core.drain_expert_log``); returns the
        number of accesses taken."""
        from . import core
        d = core.drain_expert_log(engine)
        self.dropped_observations += int(d.get("dropped", 0))
        hits = [(l, e) for l, e in d.get("hits", []) if 0 <= l < self.num_layers]
        for l, e in hits:
            self._freq[l][e] += 1
        if self.learning_cache is not None and hits:
            self.learning_cache.record_hits(hits)
        return len(hits)

    def predict(self, layer_idx: int) -> list[int]:
        """The 2 * top_k most frequent experts of the layer (the first seen first
        among equal counts); empty before any observation."""
        return [e for e, _ in self._freq[layer_idx].most_common(2 * self.top_k)]

    def prefetch_all_layers(self, engine) -> int:
        """Prefetch hints for every layer's predicted experts; returns hints sent."""
        from . import core
        n = 0
        for layer in range(self.num_layers):
            ids = self.predict(layer)
            if ids:
                core.expert_prefetch_hint(engine, layer, ids)
                n += len(ids)
        return n

    def clear(self) -> None:
        for c in self._freq:
            c.clear()


def prewarm_engine(engine, learning_cache, top_n: int) -> int:
    """The reference's warm start for the engine: the `top_n` hottest (layer, expert)
    pairs of a loaded ``LearningCache`` go to the engine's prefetch queue (its worker
    reads them from SSD into the RAM tier); returns the hints sent."""
    from . import core
    by_layer: dict[int, list[int]] = {}
    for layer, e in learning_cache.get_hot_experts(top_n):
        by_layer.setdefault(layer, []).append(e)
    for layer, ids in by_layer.items():
        core.expert_prefetch_hint(engine, layer, ids)
    return sum(len(v) for v in by_layer.values())
