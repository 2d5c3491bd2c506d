"""The fused local decoder (local_fused.cuh: one cluster kernel for step 0 and one for steps
1..16 of a greedy frame) against the per-step kernel chain it replaces and against the oracle,
on identical seeded states: logits within 2e-2 (the two GPU paths within 1e-3), identical codes,
gate values and next hidden states, over ragged batches whose last cluster is partly empty, a
single stream, repeated frames (the repetition history) and the multi-frame path."""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import forced_codes
from oracle_py import Oracle, sample_params

pytestmark = pytest.mark.gpu
TOL = 2e-2
PATH_TOL = 1e-3
GREEDY = dict(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


def states(eng, sids, lens, seed):
    for i, (s, L) in enumerate(zip(sids, lens)):
        eng.fill_state_random(s, L, seed=seed + i)
        eng.generate_begin(s, 0)


def read_state(eng, sid, L):
    k = np.empty((12, L, 768), np.float32)
    v = np.empty((12, L, 768), np.float32)
    for layer in range(12):
        k[layer], v[layer] = eng.kv(sid, layer, 0, L)
    return k, v, eng.hidden(sid)


@pytest.mark.parametrize("n", [1, 5, 37])
def test_fused_local_decoder_matches_the_kernel_chain(pkg, weights_path, n):
    lens = [int(x) for x in np.random.default_rng(n).integers(10, 300, n)]
    eng = pkg.Engine(weights_path, device=0, max_streams=n, max_ctx=320)
    try:
        sids = [eng.open() for _ in lens]
        p = pkg.SampleParams.make(**GREEDY)
        forced = [forced_codes(n, seed=70 + f) for f in range(3)]
        out = {}
        for path in (1, 0):
            eng.set_local_path(path)
            states(eng, sids, lens, seed=11)
            frames = []
            for f in range(3):  # three frames: the repetition history carries over
                c, stop, gate, lg = eng.step(sids, p, forced=forced[f], want_logits=True)
                assert not stop.any()
                frames.append((c, gate, lg))
            hid = np.stack([eng.hidden(s) for s in sids])
            out[path] = (frames, hid)
        for f in range(3):
            (c1, g1, l1), (c0, g0, l0) = out[1][0][f], out[0][0][f]
            assert np.abs(l0 - l1).max() <= PATH_TOL, f
            assert np.abs(g0 - g1).max() <= PATH_TOL, f
            assert (c0 == c1).all(), f
        assert np.abs(out[0][1] - out[1][1]).max() <= PATH_TOL
    finally:
        eng.close()


def test_fused_local_decoder_vs_oracle_and_free_running_frames(pkg, weights_path):
    """19 ragged streams: one teacher-forced frame against the oracle for three streams, then 4
    free-running frames through mossgpu_step_frames on both paths (identical codes)."""
    n = 19
    lens = [int(x) for x in np.random.default_rng(5).integers(30, 900, n)]
    eng = pkg.Engine(weights_path, device=0, max_streams=n, max_ctx=1024)
    try:
        sids = [eng.open() for _ in lens]
        p = pkg.SampleParams.make(**GREEDY)
        eng.set_local_path(0)
        states(eng, sids, lens, seed=200)
        sample = (0, 9, 18)
        st = {i: read_state(eng, sids[i], lens[i]) for i in sample}
        forced = forced_codes(n, seed=3)
        c, stop, gate, lg = eng.step(sids, p, forced=forced, want_logits=True)
        for i in sample:
            orc = Oracle(weights_path, max_ctx=lens[i] + 8)
            orc.set_state(*st[i])
            oc, ol, og = orc.generate(2, sample_params(greedy=True, rep=1.2, min_frames=1 << 30),
                                      forced=np.stack([forced[i], forced[i]]), want_logits=True)
            assert np.abs(lg[i] - ol[0]).max() <= TOL, i
            assert (c[i] == oc[0]).all(), i
            assert np.abs(gate[i] - og[0]).max() <= TOL, i
            assert np.abs(eng.hidden(sids[i]) - orc.hidden()).max() <= TOL, i
            orc.close()
        runs = {}
        for path in (0, 1):
            eng.set_local_path(path)
            states(eng, sids, lens, seed=300)
            codes, done = eng.step_frames(sids, p, 4)
            assert (done == 4).all()
            runs[path] = codes
        assert (runs[0] == runs[1]).all()
    finally:
        eng.close()


def test_stochastic_frames_keep_the_kernel_chain(pkg, weights_path):
    """The fused kernel samples greedily only; a stochastic frame takes the per-step kernels
    whatever the local path, so its codes do not depend on the setting."""
    n = 6
    lens = [40 + 13 * i for i in range(n)]
    eng = pkg.Engine(weights_path, device=0, max_streams=n, max_ctx=256)
    try:
        sids = [eng.open() for _ in lens]
        p = pkg.SampleParams.make(greedy=False, temperature=0.8, top_k=25, top_p=0.95, repetition_penalty=1.2,
                                  min_frames=1 << 30)
        got = []
        for path in (0, 1):
            eng.set_local_path(path)
            states(eng, sids, lens, seed=9)
            got.append(eng.step(sids, p)[0])
        assert (got[0] == got[1]).all()
    finally:
        eng.close()
