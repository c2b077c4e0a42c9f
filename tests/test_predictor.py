"""The route predictor of the streaming pool (qmoe_predictor_*), on the CPU.

The restatement (oracle/predictor.py) is pinned to golden vectors recorded from
the reference's own ExpertStore (tests/golden/predictor.json); the library's
predictor must issue the same prefetch requests in the same order, keep the
same counts and rank the same frequent experts, on those vectors and on longer
seeded sequences at the workload's 512 experts."""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "predictor.json")


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def _run(make, case):
    """Replays a golden case through a predictor object; returns what it saw."""
    p = make(case["num_layers"], case["num_experts"], case["depth"])
    reqs = []
    for st in case["steps"]:
        sel = p.record_route(st["layer"], st["routed"]) if hasattr(p, "record_route") else \
            p.record(st["layer"], st["routed"])
        assert list(sel) == st["selected"]
        pred = p.prefetch_predictions(st["layer"], st["selected"]) if hasattr(p, "prefetch_predictions") \
            else p.predict(st["layer"], st["selected"])
        reqs.append([list(r) for r in pred])
    return p, reqs


@pytest.mark.parametrize("ci", range(8))
def test_restatement_matches_reference_vectors(ci):
    from oracle.predictor import RoutePredictor
    case = _cases()[ci]
    p, reqs = _run(RoutePredictor, case)
    assert reqs == [st["requests"] for st in case["steps"]]
    assert p.routes == case["routes"]
    assert [list(f) for f in p.frequent(20)] == case["frequent"]


@pytest.mark.parametrize("ci", range(8))
def test_library_predictor_matches_reference_vectors(built, ci):
    import qmoe
    case = _cases()[ci]
    p, reqs = _run(qmoe.Predictor, case)
    for step, (got, st) in enumerate(zip(reqs, case["steps"])):
        assert got == st["requests"], (step, got, st["requests"])
    assert p.routes() == case["routes"]
    assert [list(f) for f in p.frequent(20)] == case["frequent"]
    for l in range(case["num_layers"]):
        assert [p.count(l, e) for e in range(case["num_experts"])] == case["counts"][l]


@pytest.mark.parametrize("E,L,k,tokens,depth,skew", [(512, 6, 10, (1, 1), 2, 1.1),
                                                     (512, 4, 10, (1, 64), 2, 1.1),
                                                     (64, 3, 4, (0, 8), 5, 0.3)])
def test_library_predictor_matches_restatement_at_scale(built, E, L, k, tokens, depth, skew):
    """Decode-like (one token a step) and batched steps over the workload's
    512 experts with a Zipf(1.1) skew, layer after layer."""
    import qmoe
    from oracle.predictor import RoutePredictor
    rng = np.random.default_rng(E + L + k)
    a, b = RoutePredictor(L, E, depth), qmoe.Predictor(L, E, depth)
    prob = 1.0 / np.arange(1, E + 1) ** skew
    prob /= prob.sum()
    perms = [rng.permutation(E) for _ in range(L)]
    for step in range(60 * L):
        layer = step % L
        n = int(rng.integers(tokens[0], tokens[1] + 1))
        routed = [int(perms[layer][i]) for _ in range(n)
                  for i in rng.choice(E, size=k, replace=False, p=prob)]
        sel = a.record_route(layer, routed)
        assert b.record(layer, routed) == list(sel)
        assert b.predict(layer, sel) == a.prefetch_predictions(layer, sel), step
    assert b.routes() == a.routes
    assert b.frequent(20) == a.frequent(20)


def test_route_counts_and_hot_marks(built):
    """tests/test_streaming.py:201-213: routes counts token assignments, the
    most routed expert leads the frequent list, and a cached expert routed
    four times is marked hot in the cache."""
    import ctypes as C

    import qmoe
    L = qmoe.lib()
    cache = L.qmoe_cache_new(4096, qmoe.QMOE_POLICY_ADAPTIVE, 1)
    try:
        assert L.qmoe_cache_put(cache, (0 << 32) | 1, 7, 1, 0, 0, None, 0, None) == 1
        p = qmoe.Predictor(1, 4, 0)
        assert p.record(0, [1, 1, 1, 1, 2], cache=cache) == [1, 2]
        assert p.routes() == 5
        assert p.frequent(1) == [(0, 1, 4)]
        assert L.qmoe_cache_stats_get(cache).hot == 1
        assert p.predict(0, [1, 2]) == []    # prefetch_count 0 predicts nothing
        # a later step with the expert routed less keeps it hot (count stays >= 4)
        p.record(0, [1], cache=cache)
        assert L.qmoe_cache_stats_get(cache).hot == 1
        v = C.c_uint64()
        assert L.qmoe_cache_peek(cache, (0 << 32) | 1, C.byref(v)) == 1 and v.value == 7
    finally:
        L.qmoe_cache_free(cache)


def test_out_of_range_experts_change_nothing(built):
    import qmoe
    p = qmoe.Predictor(2, 8, 2)
    p.record(0, [1, 2])
    with pytest.raises(ValueError):
        p.record(0, [3, 8])
    with pytest.raises(ValueError):
        p.predict(0, [-1])
    assert p.routes() == 2 and p.count(0, 3) == 0
    assert qmoe.lib().qmoe_predictor_record(p.h, None, 2, None, 0, None) == -1   # layer out of range
    # an empty step clears the previous selection: no transitions into the next step
    p.record(0, [])
    p.record(0, [5])
    assert p.predict(0, [5]) == [(0, 1), (0, 2)]   # falls back to the layer's counts


hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@st.composite
def step_sequences(draw):
    L = draw(st.integers(1, 4))
    E = draw(st.integers(1, 6))
    depth = draw(st.integers(0, 4))
    steps = draw(st.lists(st.tuples(st.integers(0, L - 1),
                                    st.lists(st.integers(0, E - 1), max_size=12)), max_size=30))
    return L, E, depth, steps


@settings(max_examples=300, deadline=None, suppress_health_check=list(HealthCheck))
@given(seq=step_sequences())
def test_library_predictor_matches_restatement_on_random_steps(built, seq):
    """Few experts, so nearly every ranking has ties; layers in any order;
    empty steps included."""
    import qmoe
    from oracle.predictor import RoutePredictor
    L, E, depth, steps = seq
    a, b = RoutePredictor(L, E, depth), qmoe.Predictor(L, E, depth)
    for layer, routed in steps:
        sel = a.record_route(layer, routed)
        assert b.record(layer, routed) == list(sel)
        assert b.predict(layer, sel) == a.prefetch_predictions(layer, sel)
    assert b.frequent(20) == a.frequent(20) and b.routes() == a.routes
    b.close()
