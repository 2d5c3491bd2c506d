"""Global layers of decode batches of <= 8 rows in two launches a layer (layer_small.cuh)
against the five-launch GEMV path and the C oracle (llm.cpp:248-255).

Covers: 1..8 ragged rows (each template width 1, 2, 4, 8 and the rows it leaves idle), page
edges, contexts whose pages exceed the 16 K/V slots a CTA stages in shared memory (those pages
are read from global memory), the KV row each step appends, run-to-run determinism of the
integer residual accumulators, and a prefill of <= 8 rows after small-layer steps (prefill
keeps the five-launch form, whose rows of one stream attend to each other).
"""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import global_state
from oracle_py import Oracle

pytestmark = pytest.mark.gpu
TOL = 2e-2        # north_star bound against the oracle (hidden states, KV rows)
PATH_TOL = 2e-3   # the two GPU forms against each other (fp32 sums in different orders)


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


@pytest.fixture(scope="module")
def eng(pkg, weights_path):
    e = pkg.Engine(weights_path, device=0, max_streams=8, max_ctx=4608)
    yield e
    e.set_small_layers(1)
    e.close()


def _step(eng, lens, seed, mode):
    """Set per-stream states of the given lengths, run one global step in `mode`; returns the
    hidden rows and the appended K/V rows of layers 0, 5 and 11."""
    eng.set_small_layers(mode)
    sids = [eng.open() for _ in lens]
    try:
        states = [global_state(L, seed=seed + i) for i, L in enumerate(lens)]
        for s, (k, v, h0, _), L in zip(sids, states, lens):
            if L > 0:  # a stream with no cached position starts at position 0
                eng.set_state(s, k, v, h0)
        x = np.stack([st[3] for st in states])
        h = eng.global_step_embed(sids, x)
        kv = [[eng.kv(s, layer, L, 1) for layer in (0, 5, 11)] for s, L in zip(sids, lens)]
        for s, L in zip(sids, lens):
            assert eng.position(s) == L + 1
        return h, kv, states
    finally:
        for s in sids:
            eng.close_stream(s)


@pytest.mark.parametrize("lens", [
    [128],                      # configs[0]: one stream at L = 128
    [1], [15], [16], [17],      # a single cached position, page edges
    [2047], [2048], [2100],     # the last fully staged context at one row (16 pages x 8 CTAs), past it
    [5, 300],                   # 2 rows
    [0, 33, 700],               # 3 rows (width 4, one idle row), a stream with no cached position
    [64, 1, 129, 257, 16],      # 5 rows (width 8)
    [900, 1000, 1100, 1200, 1300, 1400, 1500, 1600],  # 8 rows, most pages read from global memory
])
def test_small_layers_match_five_launch_form_and_oracle(eng, weights_path, lens):
    h1, kv1, states = _step(eng, lens, 300 + sum(lens) % 97, 1)
    h0, kv0, _ = _step(eng, lens, 300 + sum(lens) % 97, 0)
    assert np.abs(h1 - h0).max() < PATH_TOL
    for a, b in zip(kv1, kv0):
        for (ka, va), (kb, vb) in zip(a, b):
            assert np.abs(ka - kb).max() < PATH_TOL * 4 and np.abs(va - vb).max() < PATH_TOL * 4
    # the oracle, for the first and last stream of the batch
    for i in sorted({0, len(lens) - 1}):
        k, v, h, x = states[i]
        orc = Oracle(weights_path, max_ctx=max(lens) + 8)
        if lens[i] > 0:
            orc.set_state(k, v, h)
        ref = orc.global_step_embed(x)
        assert np.abs(h1[i] - ref).max() < TOL
        for j, layer in enumerate((0, 5, 11)):
            rk, rv = orc.kv(layer, lens[i], 1)
            assert np.abs(kv1[i][j][0] - rk).max() < TOL and np.abs(kv1[i][j][1] - rv).max() < TOL


def test_small_layers_are_deterministic(eng):
    lens = [3, 500, 77, 1024]
    a, kva, _ = _step(eng, lens, 11, 1)
    b, kvb, _ = _step(eng, lens, 11, 1)
    assert np.array_equal(a, b)
    for x, y in zip(kva, kvb):
        for (kx, vx), (ky, vy) in zip(x, y):
            assert np.array_equal(kx, ky) and np.array_equal(vx, vy)


def test_consecutive_steps_and_short_prefill(eng, weights_path):
    """Several small-layer steps in a row (the accumulators cycle across steps), then a 5-row
    prefill continuation of the same stream, each against the oracle."""
    eng.set_small_layers(1)
    s = eng.open()
    try:
        k, v, h0, x = global_state(40, seed=77)
        eng.set_state(s, k, v, h0)
        orc = Oracle(weights_path, max_ctx=128, a16_prefill=True)
        orc.set_state(k, v, h0)
        rng = np.random.default_rng(5)
        for _ in range(4):
            xi = rng.standard_normal(768).astype(np.float32)
            h = eng.global_step_embed([s], xi[None])[0]
            assert np.abs(h - orc.global_step_embed(xi)).max() < TOL
        xs = rng.standard_normal((5, 768)).astype(np.float32)
        eng.prefill_embeds(s, xs, start=44)
        orc.prefill_embeds(xs, start=44)
        assert np.abs(eng.hidden(s) - orc.hidden()).max() < TOL
        xi = rng.standard_normal(768).astype(np.float32)
        assert np.abs(eng.global_step_embed([s], xi[None])[0] - orc.global_step_embed(xi)).max() < TOL
    finally:
        eng.close_stream(s)
