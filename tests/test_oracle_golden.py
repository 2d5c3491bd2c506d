"""The C restatement (oracle/moss_oracle.c) against golden vectors made by the reference.

The fixtures in tests/golden/ were produced by the reference's own code (its numpy weight
writer and its C++ LlmModel built from its sources, tests/golden/make_golden.py).  The
restatement keeps the reference's operation order, so every comparison here is bit-exact.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from golden_inputs import (END_SEEDS, LONG_CTX, SAMPLER_SWEEP, forced_codes, global_state, prompt_rows, sampler_case,
                           sampler_sweep_case, sha)
from oracle_py import Oracle, lib, sample_params

G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def fmt():
    return np.load(G / "format.npz")


@pytest.fixture(scope="module")
def dec():
    return np.load(G / "decode.npz")


def test_weights_generator_matches_recorded_digest(weights_digest_ok):
    assert weights_digest_ok, "synthetic weights differ from the digest the golden fixtures were made with"


def test_pack_q8x4_matches_reference_writer(fmt):
    from moss_b200 import mossfile
    assert np.array_equal(mossfile.pack_q8x4(fmt["w"]), fmt["packed"])


def test_moss_container_matches_reference_writer(fmt, tmp_path):
    from moss_b200 import mossfile
    p = tmp_path / "tiny.moss"
    mossfile.write_moss(p, [("m", 4, (8, 64), fmt["packed"].tobytes()),
                            ("v", 3, (1, 5), np.arange(5, dtype=np.float32).tobytes())])
    assert np.array_equal(np.frombuffer(p.read_bytes(), np.uint8), fmt["container"])
    data, ents = mossfile.read_moss(p)
    assert ents["m"].rows == 8 and ents["m"].cols == 64 and ents["m"].offset % 32 == 0
    assert ents["v"].dtype == 3 and ents["v"].nbytes == 20


def test_half_to_float_all_inputs(fmt):
    L = lib()
    out = np.empty(65536, np.float32)
    L.or_half_to_float_n(np.arange(65536, dtype=np.uint16), 65536, out)
    assert sha(out) == str(fmt["h2f_sha"])
    assert np.array_equal(out[::97].view(np.uint32), fmt["h2f_sample"].view(np.uint32))


def test_float_to_half(fmt):
    L = lib()
    src = np.ascontiguousarray(fmt["f2h_in"])
    got = np.empty(src.size, np.uint16)
    L.or_float_to_half_n(src, src.size, got)
    assert np.array_equal(got, fmt["f2h"])


def test_dequant_and_row_dots(fmt, weights_path, weights_digest_ok):
    from moss_b200 import mossfile
    L = lib()
    data, ents = mossfile.read_moss(weights_path)
    t = ents["g0.attn.w"]
    blob = np.frombuffer(data, np.uint8, t.nbytes, t.offset)
    nb = t.cols // 32
    for i, r in enumerate(fmt["deq_rows"]):
        grp = np.ascontiguousarray(blob[(r // 4) * nb * 136:(r // 4 + 1) * nb * 136])
        out = np.empty(t.cols, np.float32)
        L.or_dequant_row_q8x4(grp, nb, int(r) % 4, out)
        assert np.array_equal(out, fmt["deq"][i])
        # the numpy unpack used by the GPU tests agrees with the C dequant
        assert np.array_equal(mossfile.dequant_q8x4(blob, t.rows, t.cols)[r], out)
    t2 = ents["g0.fc_out.w"]
    blob2 = np.frombuffer(data, np.uint8, t2.nbytes, t2.offset)
    nb2 = t2.cols // 32
    x = fmt["dot_x"]
    qa = np.empty(t2.cols, np.int8)
    qs = np.empty(nb2, np.float32)
    L.or_quantize_act(x, t2.cols, qa, qs)
    assert np.array_equal(qa, fmt["qa"]) and np.array_equal(qs, fmt["qs"])
    for i, r in enumerate(fmt["dot_rows"]):
        grp = np.ascontiguousarray(blob2[(r // 4) * nb2 * 136:(r // 4 + 1) * nb2 * 136])
        assert L.or_row_dot_a16(grp, nb2, int(r) % 4, x) == fmt["dot_a16"][i]
        assert L.or_row_dot_a8(grp, nb2, int(r) % 4, qa, qs) == fmt["dot_a8"][i]


def test_global_step_bitexact(dec, weights_path, weights_digest_ok):
    o = Oracle(weights_path, max_ctx=512)
    k, v, h0, x = global_state(128)
    assert sha(k) + sha(v) + sha(h0) + sha(x) == str(dec["gs_inputs_sha"])
    o.set_state(k, v, h0)
    assert np.array_equal(o.global_step_embed(x), dec["gs_hidden1"])
    for layer in (0, 5, 11):
        kk, vv = o.kv(layer, 128, 1)
        assert np.array_equal(kk[0], dec[f"gs_k{layer}"]) and np.array_equal(vv[0], dec[f"gs_v{layer}"])
    assert np.array_equal(o.embed_row(dec["gs_row"]), dec["gs_embed_row"])
    h = o.global_step_row(dec["gs_row"])
    assert np.array_equal(h, dec["gs_hidden2"])
    assert o.position == 130
    l0 = o.local_step(0, h)
    assert np.array_equal(l0, dec["lc_out0"])
    assert np.array_equal(o.gate(l0), dec["lc_gate"])
    assert np.array_equal(o.audio_logits(0, o.local_step(1, dec["gs_embed_row"])), dec["lc_logits0"])


def test_long_context_global_step_bitexact(weights_path, weights_digest_ok):
    """L = 4000 injected positions: RoPE rows near the end of the context and a 4001-position
    attention, then a row step (the long-form configs' lengths)."""
    g = np.load(G / "long_ctx.npz")
    o = Oracle(weights_path, max_ctx=LONG_CTX + 8)
    k, v, h0, x = global_state(LONG_CTX, seed=11)
    assert sha(k) + sha(v) + sha(h0) + sha(x) == str(g["inputs_sha"])
    o.set_state(k, v, h0)
    del k, v
    assert np.array_equal(o.global_step_embed(x), g["hidden1"])
    for layer in (0, 11):
        kk, vv = o.kv(layer, LONG_CTX, 1)
        assert np.array_equal(kk[0], g[f"k{layer}"]) and np.array_equal(vv[0], g[f"v{layer}"])
    assert np.array_equal(o.global_step_row(g["row"]), g["hidden2"])
    assert o.position == int(g["position"]) == LONG_CTX + 2


def test_teacher_forced_generate_bitexact(dec, weights_path, weights_digest_ok):
    o = Oracle(weights_path, max_ctx=512)
    rows = prompt_rows(40, seed=3)
    assert np.array_equal(rows, dec["tf_rows"])
    o.prefill_rows(rows)
    assert np.array_equal(o.hidden(), dec["tf_prefill_hidden"])
    forced = forced_codes(6, seed=4)
    codes, logits, _ = o.generate(6, sample_params(greedy=True, rep=1.2, min_frames=99), forced=forced,
                                  want_logits=True)
    assert np.array_equal(codes, dec["tf_codes"])
    assert np.array_equal(logits[:3], dec["tf_logits"])
    assert np.array_equal(logits.argmax(-1), dec["tf_argmax"])
    assert o.position == int(dec["tf_position"])


def test_free_and_sampled_generate(dec, weights_path, weights_digest_ok):
    rows = prompt_rows(40, seed=3)
    o = Oracle(weights_path, max_ctx=512)
    o.prefill_rows(rows)
    codes, _, _ = o.generate(8, sample_params(greedy=True, rep=1.2, min_frames=3))
    assert np.array_equal(codes, dec["fg_codes"])
    o2 = Oracle(weights_path, max_ctx=512)
    o2.prefill_rows(rows)
    codes, _, _ = o2.generate(8, sample_params(greedy=False, min_frames=99), seed=7)
    assert np.array_equal(codes, dec["sg_codes"])


def test_sampler_cases(dec):
    L = lib()
    for case in range(6):
        logits, prev, greedy, seed = sampler_case(case)
        rng = np.zeros(4, np.uint32)
        L.or_rng_seed(rng, seed)
        p = sample_params(greedy=bool(greedy))
        got = L.or_sample_token(logits, logits.size, C.byref(p), prev.ctypes.data_as(C.c_void_p), prev.size, rng)
        assert got == dec["sampler_picks"][case]


def test_prefill_continuation_and_context_clamp(weights_path, weights_digest_ok):
    """prefill(rows, start) after an earlier prefill, and rows past the context limit, which the
    reference clamps to kMaxCtx - start (llm.cpp:329-331), in the product (W8A8) prefill mode."""
    g = np.load(G / "prefill_continue.npz")
    o = Oracle(weights_path, max_ctx=64)
    o.prefill_rows(prompt_rows(10, seed=41))
    o.prefill_rows(prompt_rows(7, seed=42), start=10)
    assert o.position == int(g["cont_position"]) == 17
    assert np.array_equal(o.hidden(), g["cont_hidden"])
    for layer in (0, 11):
        kk, vv = o.kv(layer, 10, 7)
        assert np.array_equal(kk, g[f"cont_k{layer}"]) and np.array_equal(vv, g[f"cont_v{layer}"])
    max_ctx = int(g["clamp_max_ctx"])
    o = Oracle(weights_path, max_ctx=max_ctx)
    k, v, h0, _ = global_state(max_ctx - 8, seed=43)
    o.set_state(k, v, h0)
    del k, v
    o.prefill_rows(prompt_rows(20, seed=44), start=max_ctx - 8)
    assert o.position == int(g["clamp_position"]) == max_ctx
    assert np.array_equal(o.hidden(), g["clamp_hidden"])
    kk, vv = o.kv(11, max_ctx - 8, 8)
    assert np.array_equal(kk, g["clamp_k11"]) and np.array_equal(vv, g["clamp_v11"])


def test_sampled_end_decision_and_greedy_frames(weights_path, weights_digest_ok):
    """end_greedy = 0 (one draw per frame against p(slot), llm.cpp:30-35) for three seeds, and
    greedy_frames = 3 ahead of sampled codes, after the 40-row prompt: the same frames as the
    reference's generate()."""
    g = np.load(G / "end_decision.npz")
    rows = prompt_rows(40, seed=3)
    for seed in END_SEEDS:
        o = Oracle(weights_path, max_ctx=256)
        o.prefill_rows(rows)
        codes, _, _ = o.generate(24, sample_params(greedy=True, rep=1.2, end_greedy=False, min_frames=1), seed=seed)
        want = g[f"se_codes_{seed}"]
        assert codes.shape == want.shape and np.array_equal(codes, want), seed
    o = Oracle(weights_path, max_ctx=256)
    o.prefill_rows(rows)
    codes, _, _ = o.generate(8, sample_params(greedy=False, temperature=0.8, top_k=25, top_p=0.95, rep=1.2,
                                              min_frames=99, greedy_frames=3), seed=5)
    assert np.array_equal(codes, g["gf_codes"])


def test_sampler_over_its_parameter_space():
    """400 seeded cases (temperature 0-1.5, top-k none..above the codebook, top-p 0..1,
    penalties 0.9-1.2, histories of 0-299 codes, peaked to flat logits) against the
    reference's sample_token.  The logits are random, so no two candidates tie: with exact
    ties the reference orders candidates by its standard library's unstable sort, which the
    restatement does not reproduce (it orders ties by index)."""
    picks = np.load(G / "sampler_sweep.npz")["picks"]
    assert picks.size == SAMPLER_SWEEP
    L = lib()
    for case in range(SAMPLER_SWEEP):
        logits, prev, greedy, t, k, p, rep, seed = sampler_sweep_case(case)
        rng = np.zeros(4, np.uint32)
        L.or_rng_seed(rng, seed)
        sp = sample_params(greedy=bool(greedy), temperature=t, top_k=k, top_p=p, rep=rep)
        got = L.or_sample_token(logits, logits.size, C.byref(sp), prev.ctypes.data_as(C.c_void_p), prev.size, rng)
        assert got == picks[case], case


def test_prefill_a16_bitexact(weights_path, weights_digest_ok):
    g = np.load(G / "prefill_a16.npz")
    o = Oracle(weights_path, max_ctx=512, a16_prefill=True)
    rows = prompt_rows(64, seed=5)
    assert np.array_equal(rows, g["rows"])
    o.prefill_rows(rows)
    assert np.array_equal(o.hidden(), g["hidden"])
    for layer in (0, 11):
        kk, vv = o.kv(layer, 0, 64)
        assert np.array_equal(kk[[0, 31, 63]], g[f"k{layer}"]) and np.array_equal(vv[[0, 31, 63]], g[f"v{layer}"])
