"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in the build container (where the reference checkout and oracle/_ref/libmossref.so
exist); the fixtures are committed so the GPU box, which has neither, can use them.

    make -C oracle ref && python tests/golden/make_golden.py

Every output comes from the reference's own code: its numpy writer
(tools/export_weights.py: pack_q8_4x4, write_moss) for the byte layout, and its C++
LlmModel (compiled from its sources into oracle/_ref/libmossref.so) for the numerics.
Inputs are seeded; the fixtures record a sha256 of every large input so a test that
regenerates them can tell when the generator changed.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))

from golden_inputs import (END_SEEDS, LONG_CTX, PREFIX_FILE_ROWS, SAMPLER_SWEEP, WEIGHTS_SEED, global_state, prompt_rows,  # noqa: E402
                           forced_codes, sampler_case, sampler_sweep_case, sha, CODEC_CASES, CODEC_DECODER_SEED,
                           CODEC_STRIDE, codec_codes, codec_frame_energy)

# the reference checkout: REF_ROOT, else a directory named `reference` beside this repository
REF_ROOT = Path(os.environ.get("REF_ROOT", Path(__file__).resolve().parents[3] / "reference"))


def load_pkg():
    spec = importlib.util.spec_from_file_location(
        "moss_b200", ROOT / "dsh-moss-tts_b200" / "__init__.py",
        submodule_search_locations=[str(ROOT / "dsh-moss-tts_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moss_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def reference_export_module():
    spec = importlib.util.spec_from_file_location("ref_export_weights", REF_ROOT / "tools" / "export_weights.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_export_weights"] = mod
    spec.loader.exec_module(mod)
    return mod


def format_fixture(weights: Path):
    ex = reference_export_module()
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((8, 64)) * 0.05).astype(np.float32)
    w[1, :32] = 0.0  # an all-zero block (d = 0)
    packed = ex.pack_q8_4x4(w)
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "tiny.moss"
        ex.write_moss(p, [("m", 4, (8, 64), packed.tobytes()),
                          ("v", 3, (1, 5), np.arange(5, dtype=np.float32).tobytes())])
        container = np.frombuffer(p.read_bytes(), np.uint8)
    from oracle_py import RefModel
    lib = RefModel.lib("decode")
    halves = np.arange(65536, dtype=np.uint16)
    h2f = np.empty(65536, np.float32)
    lib.ref_half_to_float_n(halves, 65536, h2f)
    fl = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
                         np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 6e-8, np.inf, -np.inf], np.float32)]).astype(np.float32)
    f2h = np.empty(fl.size, np.uint16)
    lib.ref_float_to_half_n(fl, fl.size, f2h)
    # dequant of real rows of the synthetic weights (g0.attn.w, rows 0..7 and 2300..2303)
    pkg = load_pkg()
    from moss_b200 import mossfile
    data, ents = mossfile.read_moss(weights)
    t = ents["g0.attn.w"]
    blob = np.frombuffer(data, np.uint8, t.nbytes, t.offset)
    nb = t.cols // 32
    rows = [0, 1, 2, 3, 5, 2300, 2303]
    deq = np.empty((len(rows), t.cols), np.float32)
    for i, r in enumerate(rows):
        grp = np.ascontiguousarray(blob[(r // 4) * nb * 136:(r // 4 + 1) * nb * 136])
        lib.ref_dequant_row_q8x4(grp, nb, r % 4, deq[i])
    # row dots (A16, A8) on g0.fc_out.w (K = 3072)
    t2 = ents["g0.fc_out.w"]
    blob2 = np.frombuffer(data, np.uint8, t2.nbytes, t2.offset)
    nb2 = t2.cols // 32
    x = rng.standard_normal(t2.cols).astype(np.float32)
    drows = np.array([0, 7, 100, 767], np.int32)
    a16 = np.empty(len(drows), np.float32)
    a8 = np.empty(len(drows), np.float32)
    for i, r in enumerate(drows):
        grp = np.ascontiguousarray(blob2[(r // 4) * nb2 * 136:(r // 4 + 1) * nb2 * 136])
        a16[i] = lib.ref_row_dot_a16(grp, nb2, int(r) % 4, x)
        a8[i] = lib.ref_row_dot_a8(grp, nb2, int(r) % 4, x, t2.cols)
    qa = np.empty(t2.cols, np.int8)
    qs = np.empty(t2.cols // 32, np.float32)
    lib.ref_quantize_act(x, t2.cols, qa, qs)
    np.savez_compressed(OUT / "format.npz", w=w, packed=packed, container=container, h2f_sha=sha(h2f),
                        h2f_sample=h2f[::97], f2h_in=fl, f2h=f2h, deq_rows=np.array(rows, np.int32), deq=deq,
                        dot_x=x, dot_rows=drows, dot_a16=a16, dot_a8=a8, qa=qa, qs=qs)


def decode_fixture(weights: Path):
    from oracle_py import RefModel
    ref = RefModel(weights, threads=4, a16_mode="decode")
    out = {}
    # config-1 shaped global step: injected L=128 fp16 N(0,1) KV, fp16 N(0,1) embedding
    k, v, h0, x = global_state(128)
    out["gs_inputs_sha"] = sha(k) + sha(v) + sha(h0) + sha(x)
    ref.set_state(k, v, h0)
    out["gs_hidden1"] = ref.global_step_embed(x)
    for layer in (0, 5, 11):
        kk, vv = ref.kv(layer, 128, 1)
        out[f"gs_k{layer}"], out[f"gs_v{layer}"] = kk[0], vv[0]
    row = np.array([9] + list(range(100, 1700, 100)), np.int32)
    row[5] = 1024  # pad code: skipped by embed_row
    out["gs_row"] = row
    out["gs_hidden2"] = ref.global_step_row(row)
    out["gs_embed_row"] = ref.embed_row(row)
    # local decoder pieces on the step output
    h = out["gs_hidden2"]
    l0 = ref.local_step(0, h)
    out["lc_out0"] = l0
    out["lc_gate"] = ref.gate(l0)
    out["lc_logits0"] = ref.audio_logits(0, ref.local_step(1, out["gs_embed_row"]))
    # teacher-forced generation after a 40-row prompt (W8A8 prefill: the product default)
    rows = prompt_rows(40, seed=3)
    forced = forced_codes(6, seed=4)
    ref2 = RefModel(weights, threads=4, a16_mode="decode")
    ref2.prefill_rows(rows)
    out["tf_rows"] = rows
    out["tf_prefill_hidden"] = ref2.hidden()
    out["tf_forced"] = forced
    codes, logits = ref2.generate(6, greedy=True, rep=1.2, min_frames=99, forced=forced, want_logits=True)
    out["tf_codes"] = codes
    out["tf_logits"] = logits[:3]
    out["tf_argmax"] = logits.argmax(-1).astype(np.int32)
    out["tf_position"] = np.int32(ref2.position)
    # free greedy generation from the same prompt, stopping on the gate
    ref3 = RefModel(weights, threads=4, a16_mode="decode")
    ref3.prefill_rows(rows)
    codes, _ = ref3.generate(8, greedy=True, rep=1.2, min_frames=3)
    out["fg_codes"] = codes
    ref4 = RefModel(weights, threads=4, a16_mode="decode")
    ref4.prefill_rows(rows)
    codes, _ = ref4.generate(8, greedy=False, temperature=0.8, top_k=25, top_p=0.95, rep=1.2, min_frames=99, seed=7)
    out["sg_codes"] = codes
    # sampler cases
    lib = RefModel.lib()
    picks = []
    for case in range(6):
        logits, prev, greedy, seed = sampler_case(case)
        picks.append(lib.ref_sample_token(logits, logits.size, greedy, 0.8, 25, 0.95, 1.2,
                                          prev.ctypes.data_as(__import__("ctypes").c_void_p), prev.size, seed))
    out["sampler_picks"] = np.array(picks, np.int32)
    np.savez_compressed(OUT / "decode.npz", **out)


def long_ctx_fixture(weights: Path):
    """One global step at L = 4000 injected positions (RoPE rows near the end of a 4608
    context, a 4001-position attention), then one row step: the long-form configs' lengths."""
    from oracle_py import RefModel
    ref = RefModel(weights, threads=4, a16_mode="decode")
    k, v, h0, x = global_state(LONG_CTX, seed=11)
    out = {"inputs_sha": sha(k) + sha(v) + sha(h0) + sha(x)}
    ref.set_state(k, v, h0)
    out["hidden1"] = ref.global_step_embed(x)
    for layer in (0, 11):
        kk, vv = ref.kv(layer, LONG_CTX, 1)
        out[f"k{layer}"], out[f"v{layer}"] = kk[0], vv[0]
    row = np.array([9] + list(range(7, 1024, 64)), np.int32)
    out["row"] = row
    out["hidden2"] = ref.global_step_row(row)
    out["position"] = np.int32(ref.position)
    np.savez_compressed(OUT / "long_ctx.npz", **out)


def end_decision_fixture(weights: Path):
    """generate() with the sampled end decision (end_greedy = 0: one draw per frame against
    p(slot), llm.cpp:30-35) for three seeds, and with greedy_frames = 3 (the first frames
    greedy, then sampled codes, llm.cpp:682-684), after the 40-row prompt."""
    from oracle_py import RefModel
    rows = prompt_rows(40, seed=3)
    out = {}
    for seed in END_SEEDS:
        ref = RefModel(weights, threads=4, a16_mode="decode")
        ref.prefill_rows(rows)
        codes, _ = ref.generate(24, greedy=True, rep=1.2, end_greedy=False, min_frames=1, seed=seed)
        out[f"se_codes_{seed}"] = codes
    ref = RefModel(weights, threads=4, a16_mode="decode")
    ref.prefill_rows(rows)
    codes, _ = ref.generate(8, greedy=False, temperature=0.8, top_k=25, top_p=0.95, rep=1.2, min_frames=99,
                            greedy_frames=3, seed=5)
    out["gf_codes"] = codes
    np.savez_compressed(OUT / "end_decision.npz", **out)


def prefix_file_fixture(weights: Path):
    """The reference's .mosskv prefix file (save_prefix, llm.cpp:485-509) after a 3-row prompt:
    its 40-byte header, the sha256 of its K/V payload, and the weights fingerprint input.  The
    payload itself is not stored (216 KB): the oracle's prefill reproduces it."""
    import hashlib
    from oracle_py import RefModel
    rows = prompt_rows(PREFIX_FILE_ROWS, seed=61)
    ref = RefModel(weights, threads=4, a16_mode="decode")
    ref.prefill_rows(rows)
    path = Path(tempfile.gettempdir()) / "moss_golden_prefix.mosskv"
    ref.save_prefix(path, rows)
    data = path.read_bytes()
    ref.save_state(path, rows)  # the debug state file: the same header and payload, then hidden
    state = path.read_bytes()
    path.unlink()
    np.savez_compressed(OUT / "prefix_file.npz", header=np.frombuffer(data[:40], np.uint8),
                        payload_sha=np.array(hashlib.sha256(data[40:]).hexdigest()),
                        size=np.int64(len(data)), state_header=np.frombuffer(state[:40], np.uint8),
                        state_payload_sha=np.array(hashlib.sha256(state[40:]).hexdigest()),
                        state_size=np.int64(len(state)))


def prefill_continue_fixture(weights: Path):
    """prefill(rows, start) (llm.cpp:327-401) in the product mode: 10 rows, then 7 more at
    start = 10; and rows past the context limit, which prefill clamps to kMaxCtx - start
    (llm.cpp:329-331): 20 rows at start = kMaxCtx - 8 after an injected state."""
    from oracle_py import RefModel
    out = {}
    a, b = prompt_rows(10, seed=41), prompt_rows(7, seed=42)
    ref = RefModel(weights, threads=4, a16_mode="decode")
    ref.prefill_rows(a)
    ref.prefill_rows(b, start=10)
    out["cont_hidden"] = ref.hidden()
    out["cont_position"] = np.int32(ref.position)
    for layer in (0, 11):
        kk, vv = ref.kv(layer, 10, 7)
        out[f"cont_k{layer}"], out[f"cont_v{layer}"] = kk, vv
    ref2 = RefModel(weights, threads=4, a16_mode="decode")
    L = ref2.max_ctx - 8
    k, v, h0, _ = global_state(L, seed=43)
    ref2.set_state(k, v, h0)
    del k, v
    ref2.prefill_rows(prompt_rows(20, seed=44), start=L)
    out["clamp_max_ctx"] = np.int32(ref2.max_ctx)
    out["clamp_position"] = np.int32(ref2.position)
    out["clamp_hidden"] = ref2.hidden()
    kk, vv = ref2.kv(11, L, 8)
    out["clamp_k11"], out["clamp_v11"] = kk, vv
    np.savez_compressed(OUT / "prefill_continue.npz", **out)


def sampler_sweep_fixture():
    """The reference's sample_token (sampler.cpp:9-77) over SAMPLER_SWEEP seeded cases of its
    parameter space (golden_inputs.sampler_sweep_case); only the picks are stored."""
    import ctypes
    from oracle_py import RefModel
    lib = RefModel.lib("decode")
    picks = []
    for case in range(SAMPLER_SWEEP):
        logits, prev, greedy, t, k, p, rep, seed = sampler_sweep_case(case)
        picks.append(lib.ref_sample_token(logits, logits.size, greedy, t, k, p, rep,
                                          prev.ctypes.data_as(ctypes.c_void_p), prev.size, seed))
    np.savez_compressed(OUT / "sampler_sweep.npz", picks=np.array(picks, np.int32))


def prefill_a16_fixture(weights: Path):
    """MOSS_A16=all is read once per process, so this runs in its own interpreter."""
    from oracle_py import RefModel
    ref = RefModel(weights, threads=4, a16_mode="all")
    rows = prompt_rows(64, seed=5)
    ref.prefill_rows(rows)
    out = {"rows": rows, "hidden": ref.hidden(), "position": np.int32(ref.position)}
    for layer in (0, 11):
        kk, vv = ref.kv(layer, 0, 64)
        out[f"k{layer}"], out[f"v{layer}"] = kk[[0, 31, 63]], vv[[0, 31, 63]]
    np.savez_compressed(OUT / "prefill_a16.npz", **out)


def codec_fixture():
    """The reference's AudioDecoder (decoder.cpp, compiled into oracle/_ref/libmossref.so) on
    the seeded synthetic decoder file: decode() of 12 frames, and two streaming runs through
    decode_chunk from reset_stream -- chunks of 4, 8, 8, 3 frames, and 160 frames in the
    engine's chunking (4, then 8s; engine.cpp:482-486), long enough that every stage's ring
    (500 / 800 / 1200 / 1600 rows = 125 / 100 / 75 / 50 frames) wraps."""
    from oracle_py import RefCodec
    from moss_b200 import codecfile
    path = Path(tempfile.gettempdir()) / "moss_golden_dec1.moss"
    digest = codecfile.synth_decoder(path, CODEC_DECODER_SEED)
    ref = RefCodec(path, threads=8)
    out = {"decoder_sha256": np.array(digest), "decoder_bytes": np.int64(path.stat().st_size)}
    for name, seed, chunks in CODEC_CASES:
        codes = codec_codes(sum(chunks), seed)
        if name == "whole":
            pcm = ref.decode(codes)
        else:
            ref.reset()
            parts, f0 = [], 0
            for k in chunks:
                parts.append(ref.decode_chunk(codes[:, f0:f0 + k]))
                f0 += k
            pcm = np.concatenate(parts)
        assert pcm.size == sum(chunks) * 7680
        out[f"{name}_codes_sha"] = np.array(sha(codes))
        out[f"{name}_sub"] = pcm[::CODEC_STRIDE].copy()
        out[f"{name}_energy"] = codec_frame_energy(pcm)
    np.savez_compressed(OUT / "codec.npz", **out)


def main():
    weights = Path(tempfile.gettempdir()) / "moss_golden_w0.moss"
    load_pkg()
    from moss_b200 import mossfile
    digest = mossfile.synth_weights(weights, WEIGHTS_SEED)
    if len(sys.argv) > 1 and sys.argv[1] == "--a16-prefill":
        prefill_a16_fixture(weights)
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--sampler-sweep":
        sampler_sweep_fixture()
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--long-ctx":
        long_ctx_fixture(weights)
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--end-decision":
        end_decision_fixture(weights)
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--prefix-file":
        prefix_file_fixture(weights)
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--prefill-continue":
        prefill_continue_fixture(weights)
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--codec":
        codec_fixture()
        return
    ex = reference_export_module()
    # the synthetic-weight writer must produce the reference writer's bytes
    rng = np.random.default_rng(0)
    w = rng.standard_normal((2304, 768), dtype=np.float32) * np.float32(0.02)
    assert np.array_equal(ex.pack_q8_4x4(w), mossfile.pack_q8x4(w)), "pack_q8x4 != reference pack_q8_4x4"
    (OUT / "weights.json").write_text(json.dumps({"seed": WEIGHTS_SEED, "bytes": weights.stat().st_size,
                                                   "sha256": digest}, indent=1) + "\n")
    format_fixture(weights)
    decode_fixture(weights)
    sampler_sweep_fixture()
    long_ctx_fixture(weights)
    end_decision_fixture(weights)
    prefix_file_fixture(weights)
    prefill_continue_fixture(weights)
    codec_fixture()
    subprocess.run([sys.executable, __file__, "--a16-prefill"], check=True)
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
