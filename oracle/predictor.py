"""TEST INFRASTRUCTURE ONLY: a pure-Python restatement of the reference's route
statistics and prefetch prediction (ExpertStore, src/colibri_runtime/
streaming.py), the checker of the library's qmoe_predictor_*.

- record_route           streaming.py:400-413
- prefetch_predictions   streaming.py:415-435 (returns the (layer, expert)
                         requests the reference issues, in order)
- frequent               streaming.py:445-453 (snapshot's frequent_experts)

Rankings use Counter.most_common, as the reference does: by count, ties in
first-insertion order. Pinned against the reference's own ExpertStore by the
vectors in tests/golden/predictor.json (tests/golden/make_predictor_golden.py).
"""
from __future__ import annotations

from collections import Counter, defaultdict


class RoutePredictor:
    def __init__(self, num_layers: int, num_experts: int, depth: int):
        self.L, self.E, self.depth = num_layers, num_experts, max(0, depth)
        self.freq: defaultdict[int, Counter] = defaultdict(Counter)   # layer -> expert counts
        self.last: dict[int, tuple[int, ...]] = {}                     # layer -> previous selection
        self.trans: defaultdict[tuple[int, int], Counter] = defaultdict(Counter)
        self.routes = 0
        self.hot: dict[tuple[int, int], bool] = {}                     # hot marks set

    def _check(self, experts):
        for e in experts:
            if not 0 <= e < self.E:
                raise ValueError(f"expert {e} out of range")

    def record_route(self, layer: int, routed) -> tuple[int, ...]:
        routed = tuple(int(e) for e in routed)
        self._check(routed)
        selected = tuple(sorted(set(routed)))
        for old in self.last.get(layer, ()):
            self.trans[(layer, old)].update(selected)
        self.freq[layer].update(routed)
        self.last[layer] = selected
        self.routes += len(routed)
        for e in selected:
            self.hot[(layer, e)] = self.freq[layer][e] >= 4
        return selected

    def prefetch_predictions(self, layer: int, selected) -> list[tuple[int, int]]:
        selected = [int(e) for e in selected]
        self._check(selected)
        if not self.depth:
            return []
        cand = Counter()
        for e in selected:
            cand.update(self.trans[(layer, e)])
        if not cand:
            cand.update(self.freq[layer])
        if layer + 1 < self.L:
            cand.update({e: n * 2 for e, n in self.freq[layer + 1].items()})
        out = [(layer, e) for e, _ in cand.most_common(self.depth)]
        if layer + 1 < self.L:
            out += [(layer + 1, e) for e, _ in self.freq[layer + 1].most_common(self.depth)]
        return out

    def frequent(self, n: int = 20) -> list[tuple[int, int, int]]:
        allc = Counter({(l, e): c for l, counts in self.freq.items() for e, c in counts.items()})
        return [(l, e, c) for (l, e), c in allc.most_common(n)]
