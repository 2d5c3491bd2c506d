"""GPU parity of the tcgen05 tensor-core path (int8 weights dequantised to fp16 in shared
memory, fp16 activations, fp32 TMEM accumulators), forced on for every batch size, against
the C oracle and the reference's golden vectors.  Same tolerances as test_gpu_parity.py."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from golden_inputs import forced_codes, global_state, prompt_rows
from oracle_py import Oracle, sample_params
from test_gpu_parity import KL_TOL, TOL, kl_per_frame

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


@pytest.fixture(scope="module")
def eng(pkg, weights_path):
    e = pkg.Engine(weights_path, device=0, max_streams=24, max_ctx=1280)
    e.set_gemm_path(2)
    yield e
    e.close()


def test_tile_repack_is_a_byte_permutation(eng, weights_path):
    from moss_b200 import mossfile
    data, ents = mossfile.read_moss(weights_path)
    for name in ["g0.attn.w", "g7.fc_out.w", "local.proj.w", "aemb.3"]:
        t = ents[name]
        got = eng.matrix_tile_bytes(name, t.rows, t.cols)
        assert np.array_equal(got, np.frombuffer(data, np.uint8, t.nbytes, t.offset)), name


def test_tc_global_step_golden(eng):
    dec = np.load(G / "decode.npz")
    s = eng.open()
    try:
        k, v, h0, x = global_state(128)
        eng.set_state(s, k, v, h0)
        h = eng.global_step_embed([s], x[None])[0]
        assert np.abs(h - dec["gs_hidden1"]).max() < TOL
        for layer in (0, 5, 11):
            kk, vv = eng.kv(s, layer, 128, 1)
            assert np.abs(kk[0] - dec[f"gs_k{layer}"]).max() < TOL
            assert np.abs(vv[0] - dec[f"gs_v{layer}"]).max() < TOL
    finally:
        eng.close_stream(s)


def test_tc_prefill_a16_golden(eng):
    g = np.load(G / "prefill_a16.npz")
    s = eng.open()
    try:
        eng.prefill(s, g["rows"])
        assert np.abs(eng.hidden(s) - g["hidden"]).max() < TOL
        for layer in (0, 11):
            kk, vv = eng.kv(s, layer, 0, 64)
            assert np.abs(kk[[0, 31, 63]] - g[f"k{layer}"]).max() < TOL
            assert np.abs(vv[[0, 31, 63]] - g[f"v{layer}"]).max() < TOL
    finally:
        eng.close_stream(s)


def test_tc_teacher_forced_generate_vs_oracle(eng, pkg, weights_path):
    rows = prompt_rows(40, seed=3)
    frames = 12
    forced = forced_codes(frames, seed=4)
    orc = Oracle(weights_path, max_ctx=256, a16_prefill=True)
    orc.prefill_rows(rows)
    o_codes, o_logits, _ = orc.generate(frames, sample_params(greedy=True, rep=1.2, min_frames=99), forced=forced,
                                        want_logits=True)
    s = eng.open()
    try:
        eng.prefill(s, rows)
        eng.generate_begin(s, 0)
        p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=99)
        lg, cd = [], []
        for f in range(frames):
            c, stop, gate, logits = eng.step([s], p, forced=forced[f], want_logits=True, run_global=f + 1 < frames)
            lg.append(logits[0])
            cd.append(c[0])
        lg, cd = np.array(lg), np.array(cd)
        assert np.abs(lg - o_logits).max() <= TOL
        assert kl_per_frame(o_logits, lg).max() <= KL_TOL
        assert (cd == o_codes).all(-1).mean() >= 0.99
    finally:
        eng.close_stream(s)


@pytest.mark.parametrize("lens", [[5, 16, 31, 64, 100, 129, 257, 700, 33, 47, 1000, 2, 17, 300, 512, 90],
                                  [64] * 20])
def test_tc_ragged_batch_vs_oracle(eng, pkg, weights_path, lens):
    sids = [eng.open() for _ in lens]
    try:
        states = [global_state(L, seed=70 + i) for i, L in enumerate(lens)]
        for s, (k, v, h0, _) in zip(sids, states):
            eng.set_state(s, k, v, h0)
            eng.generate_begin(s, 0)
        forced = forced_codes(len(lens), seed=19)
        p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=99)
        codes, stop, gate, logits = eng.step(sids, p, forced=forced, want_logits=True)
        for i in range(0, len(lens), 3):  # every third stream against the oracle (CPU time)
            k, v, h0, _ = states[i]
            orc = Oracle(weights_path, max_ctx=1100)
            orc.set_state(k, v, h0)
            oc, ol, _ = orc.generate(2, sample_params(greedy=True, rep=1.2, min_frames=99),
                                     forced=np.stack([forced[i], forced[i]]), want_logits=True)
            assert np.abs(logits[i] - ol[0]).max() <= TOL
            assert kl_per_frame(ol[:1], logits[i][None]).max() <= KL_TOL
            assert np.abs(eng.hidden(sids[i]) - orc.hidden()).max() < TOL
    finally:
        for s in sids:
            eng.close_stream(s)


def test_tc_and_cuda_core_paths_agree_on_a_batch(pkg, weights_path):
    """The automatic switch-over (R = 8 vs R = 9) gives the same frame within tolerance."""
    e = pkg.Engine(weights_path, device=0, max_streams=16, max_ctx=512)
    try:
        lens = [40 + 13 * i for i in range(12)]
        out = {}
        for mode in (1, 2):
            e.set_gemm_path(mode)
            sids = [e.open() for _ in lens]
            for i, (s, L) in enumerate(zip(sids, lens)):
                e.fill_state_random(s, L, seed=i)
                e.generate_begin(s, 0)
            p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=99)
            _, _, _, logits = e.step(sids, p, forced=forced_codes(len(lens), seed=5), want_logits=True)
            out[mode] = (logits, np.stack([e.hidden(s) for s in sids]))
            for s in sids:
                e.close_stream(s)
        assert np.abs(out[1][0] - out[2][0]).max() <= TOL
        assert np.abs(out[1][1] - out[2][1]).max() <= TOL
    finally:
        e.close()
