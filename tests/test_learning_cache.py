"""The learning cache and the frequency predictor (CPU): the usage file written by
the reference's own LearningCache (tests/golden/make_usage_golden.py) loads here with
the same ranking, and a file written here round-trips; recency, caps, bad files,
reset; the predictor's ranking and its feed into the learning cache."""

import json
from pathlib import Path

from wisp_b200.learning_cache import USAGE_FORMAT_VERSION, LearningCache
from wisp_b200.tier_cache import ExpertPredictor

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reference_usage_file_loads_with_the_reference_ranking():
    want = json.loads((GOLDEN / "usage_golden.json").read_text())
    lc = LearningCache(GOLDEN / "usage")
    assert lc.load() == want["records"]
    assert [list(p) for p in lc.get_hot_experts(100, recency_weight=0.0)] == want["hot_all"]
    assert [list(p) for p in lc.get_hot_experts(3, recency_weight=0.0)] == want["hot_3"]


def test_save_load_round_trip_and_session_merge(tmp_path):
    lc = LearningCache(tmp_path)
    assert lc.load() == 0 and lc.save() is False  # nothing yet
    lc.record_hits([(1, 2), (1, 2), (0, 4)])
    lc.record_hit(3, 3, count=5)
    assert lc.save() and lc.save() is False
    lc.record_hit(0, 4)
    assert lc.save()
    data = json.loads((tmp_path / LearningCache.USAGE_FILE).read_text())
    assert data["version"] == USAGE_FORMAT_VERSION and data["total_sessions"] == 2
    back = LearningCache(tmp_path)
    assert back.load() == 3
    rec = back.records[(0, 4)]
    assert rec.hit_count == 2 and rec.sessions == 2
    assert back.get_hot_experts(10, recency_weight=0.0) == [(3, 3), (0, 4), (1, 2)]
    assert back.get_stats()["total_hits"] == 9


def test_recency_decay_and_ties(tmp_path):
    lc = LearningCache(tmp_path)
    day = 86400.0
    now = 1_000 * day
    from wisp_b200.learning_cache import ExpertUsageRecord
    lc.records = {
        (0, 1): ExpertUsageRecord(0, 1, 10, now - 100 * day, 1),   # old and frequent
        (0, 2): ExpertUsageRecord(0, 2, 6, now, 1),                # fresh
        (1, 0): ExpertUsageRecord(1, 0, 6, now, 1),                # tie with (0, 2)
    }
    # pure frequency: the old expert first; full recency: 10/11 < 6, the fresh ones
    # first, the tie broken by the lower layer
    assert lc.get_hot_experts(3, recency_weight=0.0, now=now)[0] == (0, 1)
    assert lc.get_hot_experts(3, recency_weight=1.0, now=now) == [(0, 2), (1, 0), (0, 1)]


def test_cap_bad_files_and_reset(tmp_path):
    lc = LearningCache(tmp_path, max_tracked=2)
    lc.record_hits([(0, 0)] * 3 + [(0, 1)] * 2 + [(0, 2)])
    assert lc.save()
    assert LearningCache(tmp_path).load() == 2  # the least used record dropped
    f = tmp_path / LearningCache.USAGE_FILE
    f.write_text("{not json")
    assert LearningCache(tmp_path).load() == 0
    f.write_text(json.dumps({"version": 99, "experts": []}))
    assert LearningCache(tmp_path).load() == 0
    lc.reset()
    assert not f.exists() and lc.get_hot_experts(5) == []


def test_predictor_ranks_by_frequency_and_feeds_the_learning_cache(tmp_path):
    lc = LearningCache(tmp_path)
    p = ExpertPredictor(num_layers=2, top_k=2, learning_cache=lc)
    assert p.predict(0) == []
    p.observe(0, [5, 3, -1])
    p.observe(0, [3, 7])
    p.observe(0, [3, 5])
    p.observe(1, [1])
    # 2 * top_k experts, most frequent first, ties in first-seen order
    assert p.predict(0) == [3, 5, 7]
    assert p.predict(1) == [1]
    assert sum(lc.session_hits.values()) == 7
    p.clear()
    assert p.predict(0) == []
