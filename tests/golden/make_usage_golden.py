"""Writes tests/golden/usage/.wisp_usage with the reference's own LearningCache
(wisp/runtime/learning_cache.py, imported from a reference checkout given as the first
argument) and records its pure-frequency ranking (recency weight 0, independent of
the clock) in tests/golden/usage_golden.json.  Run once in a container that has the
reference; the GPU boxes only read the committed files."""

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from wisp.runtime.learning_cache import LearningCache
    d = HERE / "usage"
    d.mkdir(exist_ok=True)
    lc = LearningCache(d)
    lc.reset()
    # two sessions: (layer, expert) hit patterns with distinct totals and one tie
    first = [(0, 3)] * 7 + [(0, 5)] * 2 + [(1, 0)] * 4 + [(2, 9)] * 4 + [(1, 7)]
    second = [(0, 3)] * 1 + [(3, 1)] * 6 + [(0, 5)] * 3
    for batch in (first, second):
        lc.record_hits(batch)
        assert lc.save()
    # the file names its directory, which no reader uses: keep it machine-independent
    f = d / LearningCache.USAGE_FILE
    data = json.loads(f.read_text())
    data["model_dir"] = "usage"
    f.write_text(json.dumps(data, indent=2))
    back = LearningCache(d)
    n = back.load()
    golden = {"records": n, "hot_all": back.get_hot_experts(100, recency_weight=0.0),
              "hot_3": back.get_hot_experts(3, recency_weight=0.0)}
    (HERE / "usage_golden.json").write_text(json.dumps(golden, indent=1) + "\n")
    print(golden)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_usage_golden.py <reference checkout root>")
    main(sys.argv[1])
