"""A numpy restatement of the reference's audio codec decoder (streaming form).

TEST INFRASTRUCTURE ONLY: used by tests/ and bench.py's CPU baseline as a checker, never by
the product.  It restates csrc/src/decoder.cpp and csrc/src/audio_layer.cpp of the reference
step by step, in fp32, with the reference's [T][C] activation layout:

* quantize_front (decoder.cpp:226-253): z[t] = sum_i (out_b_i + out_w_i @ cb_i[code_i[t]]),
  then x = q.out.w @ z + q.out.b;
* per stage (decoder.cpp:198-209): patch (decoder.cpp:73-87), in.w, the layers, out.w;
* per layer (decoder.cpp:116-196): LN1 (audio_layer.cpp:17-29), qkv, RoPE on q and k at
  position offset + i (audio_layer.cpp:31-44), causal attention over the ring of the last
  `context` rows plus the chunk (attn_scalar.cpp:165-203), proj, x += ls1 * r, LN2, f1,
  erf GELU (audio_layer.cpp:46), f2, x += ls2 * r; the ring keeps the last `context` K/V rows;
* the final patch of 240 flattens [t][240] into the samples (decoder.cpp:221).

Matrix products use numpy's fp32 matmul, so results agree with the reference to float
rounding (summation order), not bit for bit; the tests pin this restatement against the
reference's own outputs (tests/golden/codec.npz) within a stated tolerance.
"""
from __future__ import annotations

import math

import numpy as np

D_MODEL, HEADS, HEAD_DIM = 256, 4, 64
PATCHES, CONTEXTS, STAGE_IDS, LAYER_COUNTS = (4, 2, 2, 2), (500, 800, 1200, 1600), (1, 3, 5, 7), (4, 2, 2, 4)


def read_tensors(path: str) -> dict[str, np.ndarray]:
    """The .moss table (weights.cpp:27-126): 16-byte header, 80-byte entries, f32 (3) and
    f16 (0) payloads; returns fp32 arrays [rows][cols]."""
    raw = np.fromfile(path, np.uint8)
    assert raw[:4].tobytes() == b"MOSW", "not a .moss file"
    n = int(raw[8:12].view(np.uint32)[0])
    out = {}
    for i in range(n):
        e = raw[16 + 80 * i:16 + 80 * (i + 1)]
        name = e[:48].tobytes().split(b"\0", 1)[0].decode()
        dtype = int(e[48])
        rows, cols = (int(v) for v in e[52:60].view(np.uint32))
        off, nbytes = (int(v) for v in e[64:80].view(np.uint64))
        blob = raw[off:off + nbytes]
        if dtype == 0:
            a = blob.view(np.float16).astype(np.float32)
        elif dtype == 3:
            a = blob.view(np.float32).copy()
        else:
            raise ValueError(f"{name}: dtype {dtype} is not f16/f32")
        out[name] = a.reshape(rows, cols)
    return out


def layernorm(x, w, b):
    mean = x.mean(axis=1, keepdims=True, dtype=np.float32)
    var = ((x - mean) ** 2).mean(axis=1, keepdims=True, dtype=np.float32)
    return ((x - mean) * (np.float32(1.0) / np.sqrt(var + np.float32(1e-5))) * w + b).astype(np.float32)


def rope(v, positions):
    """v [t][heads * 64] in place; pairs (2i, 2i+1) rotated by pos * exp(-ln(1e4) 2i / 64)."""
    i = np.arange(HEAD_DIM // 2, dtype=np.float32)
    freq = np.exp(np.float32(-math.log(10000.0)) * np.float32(2.0) * i / np.float32(HEAD_DIM)).astype(np.float32)
    ang = positions.astype(np.float32)[:, None] * freq[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    h = v.reshape(v.shape[0], HEADS, HEAD_DIM // 2, 2)
    x0, x1 = h[..., 0].copy(), h[..., 1].copy()
    h[..., 0] = x0 * c - x1 * s
    h[..., 1] = x0 * s + x1 * c


def gelu(v):
    from scipy.special import erf  # noqa: PLC0415
    return (np.float32(0.5) * v * (np.float32(1.0) + erf(v * np.float32(0.7071067811865476)).astype(np.float32))
            ).astype(np.float32)


class CodecOracle:
    """AudioDecoder's streaming state and decode_chunk / reset_stream / decode."""

    def __init__(self, path: str):
        self.w = read_tensors(path)
        self.reset()

    def reset(self):
        self.offset = [0] * 4
        self.kv = [[(np.zeros((0, D_MODEL), np.float32), np.zeros((0, D_MODEL), np.float32))
                    for _ in range(LAYER_COUNTS[s])] for s in range(4)]

    def front(self, codes):
        w = self.w
        t = codes.shape[1]
        z = np.zeros((t, 512), np.float32)
        for i in range(16):
            emb = w[f"q{i}.cb"][codes[i]]  # [t][8]
            z += emb @ w[f"q{i}.out.w"].T + w[f"q{i}.out.b"][0]
        return (z @ w["q.out.w"].T + w["q.out.b"][0]).astype(np.float32)

    def attention(self, qkv, ck, cv, window):
        t = qkv.shape[0]
        n = ck.shape[0]
        q = qkv[:, :D_MODEL]
        keys = np.concatenate([ck, qkv[:, D_MODEL:2 * D_MODEL]])
        vals = np.concatenate([cv, qkv[:, 2 * D_MODEL:]])
        out = np.empty((t, D_MODEL), np.float32)
        scale = np.float32(1.0 / math.sqrt(HEAD_DIM))
        for i in range(t):
            lo, hi = max(0, i + n - window + 1), i + n
            k = keys[lo:hi + 1].reshape(-1, HEADS, HEAD_DIM)
            s = np.einsum("uhd,hd->hu", k, q[i].reshape(HEADS, HEAD_DIM)) * scale  # [heads][keys]
            e = np.exp(s - s.max(axis=1, keepdims=True))
            wgt = e / e.sum(axis=1, keepdims=True)
            out[i] = np.einsum("hu,uhd->hd", wgt, vals[lo:hi + 1].reshape(-1, HEADS, HEAD_DIM)).reshape(-1)
        return out

    def layer(self, s, li, x, offset):
        w, p = self.w, f"d{STAGE_IDS[s]}.l{li}."
        t = x.shape[0]
        qkv = layernorm(x, w[p + "n1.w"][0], w[p + "n1.b"][0]) @ w[p + "attn.w"].T
        pos = np.arange(offset, offset + t)
        rope(qkv[:, :D_MODEL], pos)
        rope(qkv[:, D_MODEL:2 * D_MODEL], pos)
        ck, cv = self.kv[s][li]
        att = self.attention(qkv, ck, cv, CONTEXTS[s])
        ck = np.concatenate([ck, qkv[:, D_MODEL:2 * D_MODEL]])[-CONTEXTS[s]:]
        cv = np.concatenate([cv, qkv[:, 2 * D_MODEL:]])[-CONTEXTS[s]:]
        self.kv[s][li] = (ck.copy(), cv.copy())
        x = x + w[p + "ls1"][0] * (att @ w[p + "proj.w"].T)
        f = gelu(layernorm(x, w[p + "n2.w"][0], w[p + "n2.b"][0]) @ w[p + "f1.w"].T)
        return (x + w[p + "ls2"][0] * (f @ w[p + "f2.w"].T)).astype(np.float32)

    def decode_chunk(self, codes) -> np.ndarray:
        """codes [16][frames] -> samples [frames * 7680]."""
        codes = np.asarray(codes, np.int64)
        x = self.front(codes)
        for s in range(4):
            p = PATCHES[s]
            t, c = x.shape
            x = x.reshape(t, c // p, p).transpose(0, 2, 1).reshape(t * p, c // p)  # out[t p + j][ci] = x[t][ci p + j]
            y = x @ self.w[f"d{STAGE_IDS[s]}.in.w"].T
            for li in range(LAYER_COUNTS[s]):
                y = self.layer(s, li, y, self.offset[s])
            self.offset[s] += y.shape[0]
            x = (y @ self.w[f"d{STAGE_IDS[s]}.out.w"].T).astype(np.float32)
        return x.reshape(-1)

    def decode(self, codes) -> np.ndarray:
        saved = (self.offset, self.kv)
        self.reset()
        try:
            return self.decode_chunk(codes)
        finally:
            self.offset, self.kv = saved
