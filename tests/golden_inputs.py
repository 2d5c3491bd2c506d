"""Seeded inputs shared by the golden-fixture generator and the tests.

Shapes and value distributions follow the benchmark configs: KV caches and embeddings are
N(0,1) rounded to fp16 (then widened to fp32 for the CPU checkers), prompt rows mix text
rows (audio codes = pad 1024) with voice-frame rows (16 codes each), codes are uniform in
[0, 1024).
"""
from __future__ import annotations

import hashlib

import numpy as np

WEIGHTS_SEED = 0
HIDDEN, NVQ, CODEBOOK, LAYERS = 768, 16, 1024, 12


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def fp16_normal(rng, shape) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32).astype(np.float16).astype(np.float32)


def global_state(L: int, seed: int = 1):
    """KV [12][L][768] x2, a last hidden [768], and the next embedding [768]."""
    rng = np.random.default_rng(seed)
    k = fp16_normal(rng, (LAYERS, L, HIDDEN))
    v = fp16_normal(rng, (LAYERS, L, HIDDEN))
    h0 = rng.standard_normal(HIDDEN, dtype=np.float32)
    x = fp16_normal(rng, HIDDEN)
    return k, v, h0, x


def prompt_rows(n: int, seed: int) -> np.ndarray:
    """[n][17] int32: text rows with a voice-frame block in the middle third."""
    rng = np.random.default_rng(seed)
    rows = np.full((n, NVQ + 1), 1024, np.int32)
    rows[:, 0] = rng.integers(0, 16384, n)
    a, b = n // 3, 2 * n // 3
    rows[a:b, 0] = 8  # user-slot text id of a voice-frame row (prompt.h:14)
    rows[a:b, 1:] = rng.integers(0, CODEBOOK, (b - a, NVQ))
    return rows


def forced_codes(frames: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, CODEBOOK, (frames, NVQ)).astype(np.int32)


def sampler_case(case: int):
    """(logits[1024], history, greedy, seed) for the sampler fixture."""
    rng = np.random.default_rng(100 + case)
    logits = (rng.standard_normal(CODEBOOK, dtype=np.float32) * 2.0).astype(np.float32)
    top = int(np.argmax(logits))
    prev = np.concatenate([rng.integers(0, CODEBOOK, 12), [top, top, top]]).astype(np.int32)
    greedy = int(case % 2 == 0)
    return logits, prev, greedy, 1000 + case


SAMPLER_SWEEP = 400
LONG_CTX = 4000  # injected positions of the long-context global-step fixture
END_SEEDS = (3, 17, 99)  # generator seeds of the sampled-end-decision fixture
PREFIX_FILE_ROWS = 3  # prompt rows of the .mosskv interchange fixture


def sampler_sweep_case(case: int):
    """(logits[1024], history, greedy, temperature, top_k, top_p, penalty, seed): the sampler
    over its parameter space -- peaked to near-uniform logits, histories of 0-299 codes,
    temperature 0 (no scaling) to 1.5, top-k none / 1 / 5 / 25 / all / above the codebook,
    top-p 0 (keep one) to 1 (no cut), penalties below, at and above 1.  Random logits, so no
    two candidates tie."""
    rng = np.random.default_rng(2000 + case)
    scale = (0.01, 0.5, 2.0, 8.0, 30.0)[case % 5]
    logits = (rng.standard_normal(CODEBOOK) * scale).astype(np.float32)
    prev = rng.integers(0, CODEBOOK, int(rng.integers(0, 300))).astype(np.int32)
    greedy = int(rng.random() < 0.2)
    temperature = (0.5, 0.8, 1.0, 1.5, 0.0)[int(rng.integers(0, 5))]
    top_k = (0, 1, 5, 25, 1024, 5000)[int(rng.integers(0, 6))]
    top_p = (0.0, 0.3, 0.95, 1.0)[int(rng.integers(0, 4))]
    penalty = (1.0, 1.2, 0.9)[int(rng.integers(0, 3))]
    return logits, prev, greedy, temperature, top_k, top_p, penalty, 5000 + case


# The audio codec decoder: the seeded synthetic decoder file (codecfile.synth_decoder) and
# three streaming cases -- (name, codes seed, chunk sizes); "whole" is one decode() call.
CODEC_DECODER_SEED = 1
CODEC_CASES = (("whole", 21, (12,)), ("chunks", 22, (4, 8, 8, 3)), ("long", 23, (4,) + (8,) * 19 + (4,)))
CODEC_STRIDE = 53  # the fixtures keep samples [::53] plus per-frame sums of squares


def codec_codes(frames: int, seed: int) -> np.ndarray:
    """[16][frames] int32 codes, uniform in [0, 1024)."""
    return np.random.default_rng(seed).integers(0, CODEBOOK, (NVQ, frames)).astype(np.int32)


def codec_frame_energy(pcm: np.ndarray) -> np.ndarray:
    """Per-frame sum of squares (float64) of samples [frames * 7680]."""
    return (pcm.astype(np.float64).reshape(-1, 7680) ** 2).sum(axis=1)
