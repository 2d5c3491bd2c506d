"""The device sampler (sample_token, sampler.cpp:9-77; end_reached, llm.cpp:30-35) against the
C oracle on the same seeds: per-stream xoshiro128** state seeded by generate_begin, one
draw per stochastic channel and one per sampled end decision, in the reference's order."""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import forced_codes, global_state
from oracle_py import Oracle, sample_params

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(weights_path):
    import moss_b200
    moss_b200.build()
    e = moss_b200.Engine(weights_path, device=0, max_streams=16, max_ctx=512)
    yield moss_b200, e
    e.close()


@pytest.mark.parametrize("gemm_path", [1, 2])
def test_stochastic_teacher_forced_codes_match_oracle(eng, weights_path, gemm_path):
    # product sampling (temperature 0.8, top-k 25, top-p 0.95, penalty 1.2); forcing keeps
    # the states equal, so every frame's 16 draws line up with the oracle's
    pkg, e = eng
    e.set_gemm_path(gemm_path)
    frames, seed = 6, 1234
    k, v, h0, _ = global_state(80, seed=41)
    forced = forced_codes(frames, seed=42)
    orc = Oracle(weights_path, max_ctx=256)
    orc.set_state(k, v, h0)
    op = sample_params(greedy=False, temperature=0.8, top_k=25, top_p=0.95, rep=1.2, min_frames=99)
    oc, _, _ = orc.generate(frames, op, seed=seed, forced=forced, want_logits=True)
    s = e.open()
    try:
        e.set_state(s, k, v, h0)
        e.generate_begin(s, seed)
        p = pkg.SampleParams.make(greedy=False, temperature=0.8, top_k=25, top_p=0.95, repetition_penalty=1.2,
                                  min_frames=99)
        got = np.stack([e.step([s], p, forced=forced[f])[0][0] for f in range(frames)])
        assert (got == oc).mean() >= 0.99
    finally:
        e.close_stream(s)
        e.set_gemm_path(0)


def test_sampled_end_decision_stops_where_the_oracle_stops(eng, weights_path):
    # greedy codes, sampled stop: one draw per frame against p(slot)
    pkg, e = eng
    for seed in (3, 17, 99):
        k, v, h0, _ = global_state(50, seed=seed)
        orc = Oracle(weights_path, max_ctx=256)
        orc.set_state(k, v, h0)
        oc, _, _ = orc.generate(24, sample_params(greedy=True, rep=1.2, end_greedy=False, min_frames=1), seed=seed,
                                want_logits=True)
        n_oracle = len(oc) if oc.ndim == 2 else 0
        s = e.open()
        try:
            e.set_state(s, k, v, h0)
            e.generate_begin(s, seed)
            p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, end_greedy=False, min_frames=1)
            codes, done = e.step_frames([s], p, 24)
            assert int(done[0]) == n_oracle, seed
            assert (codes[: n_oracle, 0, :] == oc[:n_oracle]).all()
        finally:
            e.close_stream(s)


def test_stochastic_first_free_frame_matches_oracle(eng, weights_path):
    pkg, e = eng
    k, v, h0, _ = global_state(64, seed=8)
    orc = Oracle(weights_path, max_ctx=256)
    orc.set_state(k, v, h0)
    oc, _, _ = orc.generate(2, sample_params(greedy=False, temperature=0.8, top_k=25, top_p=0.95, rep=1.2,
                                             min_frames=99), seed=77, want_logits=True)
    s = e.open()
    try:
        e.set_state(s, k, v, h0)
        e.generate_begin(s, 77)
        p = pkg.SampleParams.make(greedy=False, temperature=0.8, top_k=25, top_p=0.95, repetition_penalty=1.2,
                                  min_frames=99)
        codes, done = e.step_frames([s], p, 2)
        assert (codes[0, 0] == oc[0]).mean() >= 15 / 16
    finally:
        e.close_stream(s)
