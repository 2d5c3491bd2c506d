"""The audio codec decoder's checkers, pinned on the CPU: the synthetic decoder writer
(codecfile.synth_decoder) reproduces the file the fixtures were made from, the reference's
own AudioDecoder (oracle/_ref) reproduces tests/golden/codec.npz bit for bit, and the numpy
restatement (oracle/codec_oracle.py) agrees with it within 2e-4 absolute (outputs reach about
20; the two differ only in fp32 summation order)."""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import CODEC_CASES, CODEC_DECODER_SEED, CODEC_STRIDE, codec_codes, codec_frame_energy, sha
from oracle_py import REF_SO

ATOL = 2e-4
ENERGY_RTOL = 1e-5


@pytest.fixture(scope="module")
def golden(golden_dir):
    return dict(np.load(golden_dir / "codec.npz"))


@pytest.fixture(scope="module")
def decoder_path(tmp_path_factory):
    import moss_b200.codecfile as cf
    path = tmp_path_factory.mktemp("codec") / "dec1.moss"
    digest = cf.synth_decoder(path, CODEC_DECODER_SEED)
    return path, digest


def run_case(dec, name, seed, chunks):
    codes = codec_codes(sum(chunks), seed)
    if name == "whole":
        return codes, dec.decode(codes)
    dec.reset()
    parts, f0 = [], 0
    for k in chunks:
        parts.append(dec.decode_chunk(codes[:, f0:f0 + k]))
        f0 += k
    return codes, np.concatenate(parts)


def test_synthetic_decoder_file_is_the_fixture_file(decoder_path, golden):
    path, digest = decoder_path
    assert digest == str(golden["decoder_sha256"])
    assert path.stat().st_size == int(golden["decoder_bytes"])


@pytest.mark.skipif(not REF_SO.exists(), reason="oracle/_ref not built (needs the reference checkout)")
def test_reference_decoder_reproduces_the_fixture(decoder_path, golden):
    from oracle_py import RefCodec
    ref = RefCodec(decoder_path[0], threads=4)
    for name, seed, chunks in CODEC_CASES[:2]:
        codes, pcm = run_case(ref, name, seed, chunks)
        assert str(golden[f"{name}_codes_sha"]) == sha(codes)
        assert np.array_equal(pcm[::CODEC_STRIDE], golden[f"{name}_sub"]), name
    ref.close()


@pytest.mark.parametrize("case", CODEC_CASES[:2], ids=[c[0] for c in CODEC_CASES[:2]])
def test_numpy_restatement_matches_the_reference(decoder_path, golden, case):
    from codec_oracle import CodecOracle
    name, seed, chunks = case
    _, pcm = run_case(CodecOracle(str(decoder_path[0])), name, seed, chunks)
    assert np.abs(pcm[::CODEC_STRIDE] - golden[f"{name}_sub"]).max() <= ATOL
    np.testing.assert_allclose(codec_frame_energy(pcm), golden[f"{name}_energy"], rtol=ENERGY_RTOL)


def test_numpy_restatement_decode_is_stateless_and_equals_streaming(decoder_path):
    """decode() from a clean state equals decode_chunk() from reset (decoder.cpp:211-280), and
    leaves the streaming state alone; a reset stream starts over."""
    from codec_oracle import CodecOracle
    dec = CodecOracle(str(decoder_path[0]))
    codes = codec_codes(5, seed=7)
    first = dec.decode_chunk(codes[:, :2])
    whole = dec.decode(codes)
    assert np.abs(whole[:first.size] - first).max() == 0.0
    rest = dec.decode_chunk(codes[:, 2:])
    assert np.abs(np.concatenate([first, rest]) - whole).max() <= 1e-5
    dec.reset()
    assert np.array_equal(dec.decode_chunk(codes[:, :2]), first)
