"""Failure detection without a GPU fault.

Every barrier wait in the engine's kernels is bounded (about a second): a wait that runs out
records a code in the engine's device error word, the kernel returns, and the host turns the
code into a non-zero C-ABI status with a message.  Here the test hook
mossgpu_debug_inject_wait_timeout makes one ring stage of the split-K decode attention stay
unfilled -- a flag that nothing sets; no copy is issued for it, so nothing is left in flight --
and the test checks that the step fails with the code, that the host state did not advance,
and that the engine steps correctly (against the oracle) once the hook is off.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from golden_inputs import forced_codes
from oracle_py import Oracle, sample_params

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


def test_attention_wait_timeout_is_reported_and_engine_recovers(pkg, weights_path):
    R = 100  # above 96 rows the tensor-core path runs the split-K attention (page ring)
    lens = [20 + (7 * i) % 60 for i in range(R)]
    eng = pkg.Engine(weights_path, device=0, max_streams=R, max_ctx=128)
    try:
        sids = [eng.open() for _ in range(R)]

        def init():
            for i, s in enumerate(sids):
                eng.fill_state_random(s, lens[i], seed=40 + i)
                eng.generate_begin(s, 0)

        init()
        p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=1 << 30)
        forced = forced_codes(R, seed=5)
        eng.debug_inject_wait_timeout(True)
        t0 = time.perf_counter()
        with pytest.raises(pkg.MossGpuError, match=r"wait timed out \(code 7\)"):
            eng.step(sids, p, forced=forced)
        dt = time.perf_counter() - t0
        eng.debug_inject_wait_timeout(False)
        assert dt < 30.0, dt  # bounded: about a second per waiting CTA, all in parallel
        assert [eng.position(s) for s in sids] == lens  # the failed frame advanced nothing

        # the same engine (and its captured frame graph) steps correctly afterwards
        init()
        sample = (0, 37, 99)
        states = {}
        for i in sample:
            k = np.empty((12, lens[i], 768), np.float32)
            v = np.empty((12, lens[i], 768), np.float32)
            for layer in range(12):
                k[layer], v[layer] = eng.kv(sids[i], layer, 0, lens[i])
            states[i] = (k, v, eng.hidden(sids[i]))
        codes, stop, gate, logits = eng.step(sids, p, forced=forced, want_logits=True)
        assert not stop.any()
        for i in sample:
            orc = Oracle(weights_path, max_ctx=lens[i] + 8)
            orc.set_state(*states[i])
            o_codes, o_logits, _ = orc.generate(2, sample_params(greedy=True, rep=1.2, min_frames=1 << 30),
                                                forced=np.stack([forced[i], forced[i]]), want_logits=True)
            assert np.abs(logits[i] - o_logits[0]).max() <= TOL, i
            assert (codes[i] == o_codes[0]).all(), i
            assert np.abs(eng.hidden(sids[i]) - orc.hidden()).max() < TOL, i
            orc.close()
    finally:
        eng.close()


def test_op_device_status_reads_clear_after_normal_calls(pkg):
    """The standalone ops' device status word (mossgpu_op_device_status) reads 0 when no wait
    ran out, and the query itself succeeds on a device that has run no op yet."""
    L = pkg.lib()
    code = ctypes.c_int(-1)
    assert L.mossgpu_op_device_status(ctypes.byref(code)) == 0, L.mossgpu_op_last_error()
    assert code.value == 0
    assert L.mossgpu_op_device_status(None) != 0
