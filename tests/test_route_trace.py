"""Route-trace input on the CPU: the library's .rrtrace reader (the
reference loader's rules, include/raggedroute/benchmark/adapter_utils.h:
250-322) on our fixture, on the reference's own fixture when the reference
checkout is present (its text and JSON twins must agree), on every
rejection rule, and the logits builder (chain_adapter.cpp:222-228) checked
through the top-2 oracle."""
from __future__ import annotations

import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "fixture_t24_e16_top2.rrtrace")

from oracle.build_oracle import reference_checkout  # noqa: E402

REF_DIR = os.path.join(reference_checkout(), "configs", "workloads")


def test_read_fixture_frames(rrlib):
    from raggedroute_b200.route_trace import load_route_trace_frame
    names = []
    for f in range(3):
        fr = load_route_trace_frame(FIXTURE, f)
        assert (fr.tokens, fr.experts, fr.top_k, fr.frame_count) == (24, 16, 2, 3)
        assert fr.trace_id == "fixture_t24_e16_top2" and fr.source_kind == "synthetic_fixture"
        assert fr.expert_ids.shape == (24, 2)
        names.append(fr.frame_id)
    assert names == ["uniform", "hot", "pairs"]
    pairs = load_route_trace_frame(FIXTURE, 2).expert_ids
    t = np.arange(24)
    assert np.array_equal(pairs, np.stack([t % 16, (t + 5) % 16], 1))


@pytest.mark.skipif(not os.path.isdir(REF_DIR), reason="reference checkout not present")
def test_reference_fixture_text_and_json_agree(rrlib):
    from raggedroute_b200.route_trace import load_route_trace_frame, load_route_trace_json
    txt = os.path.join(REF_DIR, "synthetic_fixture.rrtrace")
    js = os.path.join(REF_DIR, "synthetic_fixture.route_trace.json")
    first = load_route_trace_frame(txt, 0)
    for f in range(first.frame_count):
        a = load_route_trace_frame(txt, f)
        b = load_route_trace_json(js, f)
        assert (a.trace_id, a.frame_id, a.tokens, a.experts, a.top_k) == \
            (b.trace_id, b.frame_id, b.tokens, b.experts, b.top_k)
        assert np.array_equal(a.expert_ids, b.expert_ids)


BAD = {
    "schema": "raggedroute.route_trace.v2\nx\nsynthetic_fixture\n2 4 2 1\nf 0 1 2 3\n",
    "trace_id": "raggedroute.route_trace.v1\nbad id\nsynthetic_fixture\n2 4 2 1\nf 0 1 2 3\n",
    "source": "raggedroute.route_trace.v1\nx\nmade_up\n2 4 2 1\nf 0 1 2 3\n",
    "top_k": "raggedroute.route_trace.v1\nx\ncaptured\n2 4 5 1\nf 0 1 2 3\n",
    "id_range": "raggedroute.route_trace.v1\nx\ncaptured\n2 4 2 1\nf 0 1 2 4\n",
    "repeat": "raggedroute.route_trace.v1\nx\ncaptured\n2 4 2 1\nf 0 0 2 3\n",
    "dup_frame": "raggedroute.route_trace.v1\nx\ncaptured\n2 4 2 2\nf 0 1 2 3\nf 1 0 3 2\n",
    "trailing": "raggedroute.route_trace.v1\nx\ncaptured\n2 4 2 1\nf 0 1 2 3\nextra\n",
    "short": "raggedroute.route_trace.v1\nx\ncaptured\n2 4 2 1\nf 0 1 2\n",
}


@pytest.mark.parametrize("case", sorted(BAD))
def test_reader_rejects(rrlib, tmp_path, case):
    from raggedroute_b200._lib import RaggedRouteError
    from raggedroute_b200.route_trace import load_route_trace_frame
    p = tmp_path / "t.rrtrace"
    p.write_text(BAD[case])
    with pytest.raises(RaggedRouteError):
        load_route_trace_frame(str(p), 0)


def test_reader_rejects_missing_frame_and_file(rrlib, tmp_path):
    from raggedroute_b200._lib import RaggedRouteError
    from raggedroute_b200.route_trace import load_route_trace_frame
    with pytest.raises(RaggedRouteError):
        load_route_trace_frame(FIXTURE, 3)
    with pytest.raises(RaggedRouteError):
        load_route_trace_frame(str(tmp_path / "missing.rrtrace"), 0)


def test_trace_logits_select_the_frame(rrlib, oracle):
    from raggedroute_b200.route_trace import load_route_trace_frame, trace_logits
    for f in range(3):
        fr = load_route_trace_frame(FIXTURE, f)
        logits = trace_logits(fr.expert_ids, fr.experts)
        ids, w = oracle.top2_f32(logits)
        assert np.array_equal(ids.reshape(-1, 2), fr.expert_ids)
        r = np.float32(np.exp(np.float32(-1.0)))
        w0 = np.float32(1.0) / (np.float32(1.0) + r)
        np.testing.assert_allclose(w.reshape(-1, 2), np.tile([w0, r * w0], (fr.tokens, 1)),
                                   rtol=1e-6)
