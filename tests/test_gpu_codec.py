"""The GPU audio codec decoder (csrc/codec.cu, mossgpu_codec_*) against the reference's own
AudioDecoder: the golden fixtures (tests/golden/codec.npz, made by the reference) for the
whole-utterance decode, chunked streaming and 160 frames of streaming that wrap every stage's
ring, then the batched entry points against per-stream decoding by the reference (or the
numpy restatement where oracle/_ref is not built), and the error behaviour.

Tolerance: samples within 5e-4 absolute (outputs reach about 20), per-frame energies within
1e-5 relative: the GPU's products use fp16 hi + lo splits of the fp32 operands (about 22
significant bits) with fp32 accumulation in another order than the reference's."""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import CODEC_CASES, CODEC_STRIDE, codec_codes, codec_frame_energy, sha
from oracle_py import REF_SO

pytestmark = pytest.mark.gpu
ATOL = 5e-4
ENERGY_RTOL = 1e-5
SPF = 7680


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


@pytest.fixture(scope="module")
def golden(golden_dir):
    return dict(np.load(golden_dir / "codec.npz"))


def checker(path):
    """The reference decoder when oracle/_ref is built, else the numpy restatement."""
    if REF_SO.exists():
        from oracle_py import RefCodec
        return RefCodec(path, threads=8)
    from codec_oracle import CodecOracle
    return CodecOracle(path)


def close_enough(got, want):
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() <= ATOL, np.abs(got - want).max()


@pytest.mark.parametrize("case", CODEC_CASES, ids=[c[0] for c in CODEC_CASES])
def test_codec_matches_reference_fixtures(pkg, decoder_file, golden, case):
    name, seed, chunks = case
    codes = codec_codes(sum(chunks), seed)
    assert sha(codes) == str(golden[f"{name}_codes_sha"])
    codec = pkg.Codec(decoder_file, device=0, max_streams=2, max_batch_frames=16)
    try:
        if name == "whole":
            pcm = codec.decode(codes)
        else:
            sid = codec.open()
            parts, f0 = [], 0
            for k in chunks:
                parts.append(codec.decode_chunk(sid, codes[:, f0:f0 + k]))
                f0 += k
            pcm = np.concatenate(parts)
        assert pcm.size == sum(chunks) * SPF
        close_enough(pcm[::CODEC_STRIDE], golden[f"{name}_sub"])
        np.testing.assert_allclose(codec_frame_energy(pcm), golden[f"{name}_energy"], rtol=ENERGY_RTOL)
    finally:
        codec.close()


def test_whole_decode_longer_than_one_call(pkg, decoder_file, golden):
    """decode() of 12 frames through calls of at most 5 frames: the streaming pieces compute
    the same rows as one pass (decoder.cpp decode == decode_chunk from reset)."""
    name, seed, chunks = CODEC_CASES[0]
    codec = pkg.Codec(decoder_file, device=0, max_streams=1, max_batch_frames=5)
    try:
        pcm = codec.decode(codec_codes(sum(chunks), seed))
        close_enough(pcm[::CODEC_STRIDE], golden[f"{name}_sub"])
    finally:
        codec.close()


def test_one_call_longer_than_every_window(pkg, decoder_file):
    """decode() of 200 frames in one call: 800 rows at stage 0 against its 500-row window and
    6,400 rows at stage 3 against 1,600, so rows of the chunk see only the chunk's own last
    window of keys and only the last `context` rows of a chunk reach the ring.  Against the
    reference's decode() of the same utterance, and the next chunk against its decode_chunk."""
    codes = codec_codes(200, seed=31)
    nxt = codec_codes(8, seed=32)
    codec = pkg.Codec(decoder_file, device=0, max_streams=1, max_batch_frames=200)
    ref = checker(decoder_file)
    try:
        close_enough(codec.decode(codes)[::7], ref.decode(codes)[::7])
        sid = codec.open()
        codec.decode_chunk(sid, codes)  # the same 200 frames as one streaming chunk, then 8 more
        ref.reset()
        ref.decode_chunk(codes)
        close_enough(codec.decode_chunk(sid, nxt), ref.decode_chunk(nxt))
    finally:
        codec.close()


def test_batched_streams_with_different_histories(pkg, decoder_file):
    """Seven streams with 0..6 earlier chunks of different lengths (ring fill and RoPE offsets
    differ per stream) decode one 8-frame chunk in one batched call, in a scrambled stream
    order; each equals the reference decoding that stream alone."""
    n = 7
    codec = pkg.Codec(decoder_file, device=0, max_streams=n + 2, max_batch_frames=64)
    ref = checker(decoder_file)
    try:
        sids = [codec.open() for _ in range(n)]
        hist = {}
        for b, sid in enumerate(sids):
            hist[sid] = [codec_codes(k, seed=100 + 10 * b + j) for j, k in enumerate([3, 8, 5, 8, 8, 2][:b])]
            for c in hist[sid]:
                codec.decode_chunk(sid, c)
        order = [sids[i] for i in (4, 0, 6, 2, 5, 1, 3)]
        new = np.stack([codec_codes(8, seed=500 + s) for s in order])
        got = codec.decode_batch(order, new)
        for b, sid in enumerate(order):
            if sid not in (order[0], order[2], order[6]):  # three streams checked against the reference
                continue
            ref.reset()
            for c in hist[sid]:
                ref.decode_chunk(c)
            close_enough(got[b], ref.decode_chunk(new[b]))
    finally:
        codec.close()


def test_full_batch_and_device_entry_point(pkg, decoder_file):
    """64 streams x 8 frames (the benchmark's chunk shape) after a 4-frame first chunk: the
    device-pointer entry point equals the host one bit for bit, and sampled streams equal the
    reference."""
    import torch
    n = 64
    first = np.stack([codec_codes(4, seed=900 + b) for b in range(n)])
    second = np.stack([codec_codes(8, seed=1900 + b) for b in range(n)])
    outs = []
    for device_path in (False, True):
        codec = pkg.Codec(decoder_file, device=0, max_streams=n, max_batch_frames=n * 8)
        try:
            sids = [codec.open() for _ in range(n)]
            codec.decode_batch(sids, first)
            if device_path:
                stream = torch.cuda.current_stream()
                codec.set_cuda_stream(stream.cuda_stream)
                dcodes = torch.from_numpy(second).cuda()
                dout = torch.empty((n, 8 * SPF), dtype=torch.float32, device="cuda")
                codec.decode_batch_device(sids, dcodes.data_ptr(), 8, dout.data_ptr())
                stream.synchronize()
                outs.append(dout.cpu().numpy())
            else:
                outs.append(codec.decode_batch(sids, second))
        finally:
            codec.close()
    assert np.array_equal(outs[0], outs[1])
    ref = checker(decoder_file)
    for b in (0, 37, 63):
        ref.reset()
        ref.decode_chunk(first[b])
        close_enough(outs[0][b], ref.decode_chunk(second[b]))


def test_reset_close_and_decode_leave_other_state_alone(pkg, decoder_file):
    codec = pkg.Codec(decoder_file, device=0, max_streams=2, max_batch_frames=16)
    try:
        a, b = codec.open(), codec.open()
        c1, c2 = codec_codes(3, seed=1), codec_codes(3, seed=2)
        fresh = codec.decode_chunk(a, c1)
        codec.decode_chunk(b, c1)
        mid = codec.decode_chunk(b, c2)  # stream b continues after c1
        whole = codec.decode(codec_codes(6, seed=3))  # stateless: touches neither stream
        assert whole.size == 6 * SPF
        codec.reset(a)
        assert np.array_equal(codec.decode_chunk(a, c1), fresh)
        codec.reset(b)
        codec.decode_chunk(b, c1)
        assert np.array_equal(codec.decode_chunk(b, c2), mid)
        codec.close_stream(a)
        assert codec.open() == a
    finally:
        codec.close()


def test_codec_errors(pkg, decoder_file, tmp_path):
    codec = pkg.Codec(decoder_file, device=0, max_streams=2, max_batch_frames=8)
    try:
        sid = codec.open()
        assert codec.decode_chunk(sid, np.zeros((16, 0), np.int32)).size == 0
        bad = codec_codes(2, seed=4)
        bad[5, 1] = 1024
        with pytest.raises(pkg.MossGpuError, match="outside"):
            codec.decode_chunk(sid, bad)
        with pytest.raises(pkg.MossGpuError, match="max_batch_frames"):
            codec.decode_chunk(sid, codec_codes(9, seed=5))
        with pytest.raises(pkg.MossGpuError, match="repeats"):
            codec.decode_batch([sid, sid], np.stack([codec_codes(2, seed=6)] * 2))
        with pytest.raises(pkg.MossGpuError, match="not open"):
            codec.decode_chunk(1, codec_codes(2, seed=6))
        codec.open()
        with pytest.raises(pkg.MossGpuError, match="all 2 codec streams"):
            codec.open()
        # a failed call leaves the stream where it was: the next chunk is the first one
        ok = codec.decode_chunk(sid, codec_codes(2, seed=7))
        codec.reset(sid)
        assert np.array_equal(codec.decode_chunk(sid, codec_codes(2, seed=7)), ok)
    finally:
        codec.close()
    with pytest.raises(pkg.MossGpuError, match="cannot open"):
        pkg.Codec(str(tmp_path / "missing.moss"))
    (tmp_path / "junk.moss").write_bytes(b"NOTMOSS" + bytes(64))
    with pytest.raises(pkg.MossGpuError, match="magic"):
        pkg.Codec(str(tmp_path / "junk.moss"))


def test_audio_decoder_interface(pkg, decoder_file, golden):
    """moss::AudioDecoder's methods (decoder.h:16-33): load -> (ok, err), decode,
    reset_stream, decode_chunk (a chunk longer than one call is split)."""
    dec = pkg.AudioDecoder(threads=4, max_chunk_frames=5)
    ok, err = dec.load(decoder_file)
    assert ok, err
    name, seed, chunks = CODEC_CASES[1]
    codes = codec_codes(sum(chunks), seed)
    dec.reset_stream()
    pcm = np.concatenate([dec.decode_chunk(codes[:, :12], 12), dec.decode_chunk(codes[:, 12:], sum(chunks) - 12)])
    close_enough(pcm[::CODEC_STRIDE], golden[f"{name}_sub"])
    bad = pkg.AudioDecoder()
    ok, err = bad.load("/nonexistent/decoder.moss")
    assert not ok and "cannot open" in err


def test_activation_outside_fp16_range_is_reported(pkg, tmp_path):
    """The tensor-core split needs activations below 65504 in magnitude: a decoder whose q.out
    bias is 1e5 overflows it, the host entry point fails with the reason, the device entry point
    reports it through mossgpu_codec_status, and a normal call afterwards succeeds."""
    import torch
    from moss_b200 import codecfile
    path = tmp_path / "big.moss"
    codecfile.synth_decoder(path, 1, add={"q.out.b": 1e5})
    codec = pkg.Codec(str(path), device=0, max_streams=2, max_batch_frames=8)
    try:
        sid = codec.open()
        with pytest.raises(pkg.MossGpuError, match="fp16 range"):
            codec.decode_chunk(sid, codec_codes(2, seed=8))
        assert codec.status() == 0  # the failed call's flag was read and cleared
        dcodes = torch.from_numpy(codec_codes(2, seed=9)[None]).cuda()
        dout = torch.empty((1, 2 * SPF), dtype=torch.float32, device="cuda")
        codec.reset(sid)
        codec.decode_batch_device([sid], dcodes.data_ptr(), 2, dout.data_ptr())
        assert codec.status() == 1
        assert codec.status() == 0
    finally:
        codec.close()
