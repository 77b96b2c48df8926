"""Writes tests/golden/fixture_t24_e16_top2.rrtrace: a small route-trace
fixture of our own (24 tokens, 16 experts, top-2; frames "uniform", "hot"
with half of the routes on expert 0, and "pairs" (t mod 16, t+5 mod 16))
in the reference's text format. Run from the repository root."""
import os
import sys

import numpy as np

sys.path.insert(0, os.getcwd())
from raggedroute_b200.route_trace import write_route_trace  # noqa: E402

rng = np.random.default_rng(2024)
frames = {}
for name, p in (("uniform", None), ("hot", np.array([0.5] + [0.5 / 15] * 15)), ("pairs", None)):
    ids = np.zeros((24, 2), np.int32)
    for t in range(24):
        ids[t] = [t % 16, (t + 5) % 16] if name == "pairs" else rng.choice(16, 2, replace=False, p=p)
    frames[name] = ids
write_route_trace("tests/golden/fixture_t24_e16_top2.rrtrace", "fixture_t24_e16_top2",
                  "synthetic_fixture", 16, frames)
