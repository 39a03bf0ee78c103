"""Persistent expert-usage record for warm starts.

The reference keeps, per model directory, how often each (layer, expert) fired across
sessions (wisp/runtime/learning_cache.py:54-230): hits are counted in memory during a
session, merged into a JSON file (``.wisp_usage``) when the session saves, and at the
next start the hottest experts -- hit count blended with a recency decay -- are
returned for pre-warming the expert caches.  This module keeps that interface
(``load``, ``save``, ``record_hit``, ``record_hits``, ``get_hot_experts``,
``get_stats``, ``reset``) and the file format, so a usage file written by either
implementation loads in the other; here the pre-warm feeds the engine
(``wisp_expert_prefetch_hint``) or the streaming cache (``StreamingStack.prewarm``).
"""

from __future__ import annotations

import json
import os
import threading
import time
from collections import defaultdict
from dataclasses import dataclass
from pathlib import Path

USAGE_FORMAT_VERSION = 1
USAGE_FILE = ".wisp_usage"


@dataclass
class ExpertUsageRecord:
    """Accumulated use of one expert over all saved sessions."""
    layer_id: int
    expert_id: int
    hit_count: int = 0
    last_used: float = 0.0  # unix time of the last session that used it
    sessions: int = 0


class LearningCache:
    """Usage counts of a model directory's experts (see the module doc)."""

    USAGE_FILE = USAGE_FILE

    def __init__(self, model_dir, max_tracked: int = 5000):
        self.model_dir = Path(model_dir)
        self.usage_file = self.model_dir / self.USAGE_FILE
        self.max_tracked = max_tracked
        self.records: dict[tuple[int, int], ExpertUsageRecord] = {}
        self.session_hits: dict[tuple[int, int], int] = defaultdict(int)
        self._lock = threading.Lock()
        self._dirty = False

    def load(self) -> int:
        """Records read from the usage file; 0 (a cold start) when it is missing,
        unreadable or of another format version -- never an error."""
        try:
            with open(self.usage_file, encoding="utf-8") as f:
                data = json.load(f)
        except (OSError, ValueError):
            return 0
        if not isinstance(data, dict) or data.get("version") != USAGE_FORMAT_VERSION:
            return 0
        loaded: dict[tuple[int, int], ExpertUsageRecord] = {}
        try:
            for r in data.get("experts", []):
                k = (int(r["layer_id"]), int(r["expert_id"]))
                loaded[k] = ExpertUsageRecord(k[0], k[1], int(r.get("hit_count", 0)),
                                              float(r.get("last_used", 0.0)),
                                              int(r.get("sessions", 1)))
        except (KeyError, TypeError, ValueError):
            return 0
        self.records = loaded
        return len(loaded)

    def record_hit(self, layer_id: int, expert_id: int, count: int = 1) -> None:
        """One expert fired `count` times (in memory only)."""
        self.session_hits[(int(layer_id), int(expert_id))] += count
        self._dirty = True

    def record_hits(self, pairs) -> int:
        """Many (layer, expert) firings, e.g. a drained engine access log."""
        n = 0
        for layer_id, expert_id in pairs:
            self.session_hits[(int(layer_id), int(expert_id))] += 1
            n += 1
        if n:
            self._dirty = True
        return n

    def save(self) -> bool:
        """Merge this session's hits into the records and rewrite the file
        atomically (the most-used `max_tracked` records kept).  False when there was
        nothing new or the file could not be written."""
        if not self._dirty:
            return False
        now = time.time()
        with self._lock:
            for key, hits in self.session_hits.items():
                rec = self.records.get(key)
                if rec is None:
                    rec = self.records[key] = ExpertUsageRecord(key[0], key[1])
                rec.hit_count += hits
                rec.last_used = now
                rec.sessions += 1
            kept = sorted(self.records.values(), key=lambda r: r.hit_count,
                          reverse=True)[:self.max_tracked]
            payload = {
                "version": USAGE_FORMAT_VERSION,
                "model_dir": str(self.model_dir),
                "last_updated": now,
                "total_sessions": max((r.sessions for r in kept), default=0),
                "experts": [{"layer_id": r.layer_id, "expert_id": r.expert_id,
                             "hit_count": r.hit_count, "last_used": r.last_used,
                             "sessions": r.sessions} for r in kept],
            }
            self.session_hits.clear()
            self._dirty = False
        try:
            self.usage_file.parent.mkdir(parents=True, exist_ok=True)
            tmp = self.usage_file.with_name(self.usage_file.name + ".tmp")
            with open(tmp, "w", encoding="utf-8") as f:
                json.dump(payload, f)
            os.replace(tmp, self.usage_file)
        except OSError:
            return False
        return True

    def get_hot_experts(self, top_n: int, recency_weight: float = 0.3,
                        now: float | None = None) -> list[tuple[int, int]]:
        """The `top_n` (layer, expert) pairs most worth pre-warming, hottest first:
        score = hits * ((1 - w) + w * recency), recency = 1 / (1 + 0.1 * age in
        days); ties go to the lower layer, then the lower expert id."""
        if top_n <= 0 or not self.records:
            return []
        t = time.time() if now is None else now
        w = recency_weight

        def score(r: ExpertUsageRecord) -> float:
            age_days = max(0.0, (t - r.last_used) / 86400.0)
            return r.hit_count * ((1.0 - w) + w / (1.0 + 0.1 * age_days))

        ranked = sorted(self.records.values(),
                        key=lambda r: (-score(r), r.layer_id, r.expert_id))
        return [(r.layer_id, r.expert_id) for r in ranked[:top_n]]

    def get_stats(self) -> dict:
        if not self.records:
            return {"status": "empty", "experts_tracked": 0, "total_hits": 0,
                    "sessions": 0, "top_expert": None}
        top = max(self.records.values(), key=lambda r: r.hit_count)
        return {"status": "active", "experts_tracked": len(self.records),
                "total_hits": sum(r.hit_count for r in self.records.values()),
                "sessions": max(r.sessions for r in self.records.values()),
                "top_expert": top}

    def reset(self) -> None:
        """Forget everything, in memory and on disk."""
        self.records.clear()
        self.session_hits.clear()
        self._dirty = False
        try:
            self.usage_file.unlink()
        except FileNotFoundError:
            pass
