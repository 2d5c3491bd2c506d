"""ctypes bindings for the two CPU checkers.

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline.  `Oracle` wraps liboracle.so (the C restatement, moss_oracle.c); `RefModel` wraps
oracle/_ref/libmossref.so (the reference's own sources + ref_harness.cpp), which exists
only where the reference checkout was available to compile it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libmossref.so"
HIDDEN, NVQ, CODEBOOK, LAYERS = 768, 16, 1024, 12

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build_oracle() -> Path:
    """Compile liboracle.so (gcc, a few seconds) when it is missing or stale."""
    src = HERE / "moss_oracle.c"
    if not ORACLE_SO.exists() or ORACLE_SO.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True, capture_output=True)
    return ORACLE_SO


class SampleParams(C.Structure):
    _fields_ = [("greedy", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int),
                ("top_p", C.c_float), ("repetition_penalty", C.c_float), ("end_greedy", C.c_int),
                ("min_frames", C.c_int), ("greedy_frames", C.c_int)]


def sample_params(greedy=True, temperature=0.8, top_k=25, top_p=0.95, rep=1.2, end_greedy=True,
                  min_frames=0, greedy_frames=0) -> SampleParams:
    return SampleParams(int(greedy), temperature, top_k, top_p, rep, int(end_greedy), min_frames,
                        greedy_frames)


def _lib() -> C.CDLL:
    lib = C.CDLL(str(build_oracle()))
    lib.or_create.restype = C.c_void_p
    lib.or_create.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_int]
    lib.or_destroy.argtypes = [C.c_void_p]
    lib.or_set_modes.argtypes = [C.c_void_p, C.c_int, C.c_int]
    lib.or_reset.argtypes = [C.c_void_p]
    lib.or_position.argtypes = [C.c_void_p]
    lib.or_get_hidden.argtypes = [C.c_void_p, _f32p]
    lib.or_set_state.argtypes = [C.c_void_p, _f32p, _f32p, C.c_int, _f32p]
    lib.or_get_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
    lib.or_embed_row.argtypes = [C.c_void_p, _i32p, _f32p]
    lib.or_global_step_embed.argtypes = [C.c_void_p, _f32p, _f32p]
    lib.or_global_step_row.argtypes = [C.c_void_p, _i32p, _f32p]
    lib.or_prefill_rows.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int]
    lib.or_prefill_embeds.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int]
    lib.or_local_step.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
    lib.or_audio_logits.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
    lib.or_assistant_logits.argtypes = [C.c_void_p, _f32p, _f32p]
    lib.or_generate.restype = C.c_int
    lib.or_generate.argtypes = [C.c_void_p, C.c_int, C.POINTER(SampleParams), C.c_uint64, C.c_void_p,
                                _i32p, C.c_void_p, C.c_void_p]
    lib.or_half_to_float.restype = C.c_float
    lib.or_half_to_float.argtypes = [C.c_uint16]
    lib.or_float_to_half.restype = C.c_uint16
    lib.or_float_to_half.argtypes = [C.c_float]
    lib.or_half_to_float_n.argtypes = [np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int, _f32p]
    lib.or_float_to_half_n.argtypes = [_f32p, C.c_int, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")]
    lib.or_dequant_row_q8x4.argtypes = [_u8p, C.c_int, C.c_int, _f32p]
    lib.or_row_dot_a16.restype = C.c_float
    lib.or_row_dot_a16.argtypes = [_u8p, C.c_int, C.c_int, _f32p]
    lib.or_quantize_act.argtypes = [_f32p, C.c_int, _i8p, _f32p]
    lib.or_row_dot_a8.restype = C.c_float
    lib.or_row_dot_a8.argtypes = [_u8p, C.c_int, C.c_int, _i8p, _f32p]
    lib.or_gemv.argtypes = [_u8p, C.c_int, C.c_int, _f32p, _f32p, C.c_int]
    lib.or_sample_token.restype = C.c_int
    lib.or_sample_token.argtypes = [_f32p, C.c_int, C.POINTER(SampleParams), C.c_void_p, C.c_int,
                                    np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")]
    lib.or_rng_seed.argtypes = [np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS"), C.c_uint64]
    return lib


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _lib()
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Oracle:
    """The C restatement of LlmModel (moss_oracle.c)."""

    def __init__(self, weights: str, max_ctx: int = 4608, a16_decode: bool = True, a16_prefill: bool = False):
        self.lib = lib()
        err = C.create_string_buffer(512)
        self.h = self.lib.or_create(str(weights).encode(), max_ctx, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        self.max_ctx = max_ctx
        self.lib.or_set_modes(self.h, int(a16_decode), int(a16_prefill))

    def close(self):
        if self.h:
            self.lib.or_destroy(self.h)
            self.h = None

    __del__ = close

    @property
    def position(self) -> int:
        return self.lib.or_position(self.h)

    def hidden(self) -> np.ndarray:
        out = np.empty(HIDDEN, np.float32)
        self.lib.or_get_hidden(self.h, out)
        return out

    def set_state(self, k, v, hidden):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        n = k.shape[1]
        if not self.lib.or_set_state(self.h, k, v, n, np.ascontiguousarray(hidden, np.float32)):
            raise ValueError("bad state length")

    def kv(self, layer, p0, n):
        k = np.empty((n, HIDDEN), np.float32)
        v = np.empty((n, HIDDEN), np.float32)
        self.lib.or_get_kv(self.h, layer, p0, n, k, v)
        return k, v

    def embed_row(self, row):
        out = np.empty(HIDDEN, np.float32)
        self.lib.or_embed_row(self.h, np.ascontiguousarray(row, np.int32), out)
        return out

    def global_step_embed(self, x):
        out = np.empty(HIDDEN, np.float32)
        self.lib.or_global_step_embed(self.h, np.ascontiguousarray(x, np.float32), out)
        return out

    def global_step_row(self, row):
        out = np.empty(HIDDEN, np.float32)
        self.lib.or_global_step_row(self.h, np.ascontiguousarray(row, np.int32), out)
        return out

    def prefill_rows(self, rows, start=0):
        rows = np.ascontiguousarray(rows, np.int32)
        self.lib.or_prefill_rows(self.h, rows, rows.shape[0], start)

    def prefill_embeds(self, x, start=0):
        x = np.ascontiguousarray(x, np.float32)
        self.lib.or_prefill_embeds(self.h, x, x.shape[0], start)

    def local_step(self, lpos, x):
        out = np.empty(HIDDEN, np.float32)
        self.lib.or_local_step(self.h, lpos, np.ascontiguousarray(x, np.float32), out)
        return out

    def audio_logits(self, ch, h):
        out = np.empty(CODEBOOK, np.float32)
        self.lib.or_audio_logits(self.h, ch, np.ascontiguousarray(h, np.float32), out)
        return out

    def gate(self, h):
        out = np.empty(2, np.float32)
        self.lib.or_assistant_logits(self.h, np.ascontiguousarray(h, np.float32), out)
        return out

    def generate(self, frames, params=None, seed=0, forced=None, want_logits=False):
        params = params or sample_params()
        codes = np.zeros((frames, NVQ), np.int32)
        logits = np.zeros((frames, NVQ, CODEBOOK), np.float32) if want_logits else None
        gate = np.zeros((frames, 2), np.float32)
        f = None if forced is None else np.ascontiguousarray(forced, np.int32)
        n = self.lib.or_generate(self.h, frames, C.byref(params), seed, _ptr(f), codes, _ptr(logits), _ptr(gate))
        return codes[:n], (logits[:n] if want_logits else None), gate[:n]


class RefModel:
    """The reference's own LlmModel (oracle/_ref/libmossref.so)."""

    _lib = None

    @classmethod
    def available(cls) -> bool:
        return REF_SO.exists()

    @classmethod
    def lib(cls, a16_mode: str = "decode") -> C.CDLL:
        if cls._lib is None:
            lib = C.CDLL(str(REF_SO))
            lib.ref_set_a16_env.argtypes = [C.c_char_p]
            lib.ref_set_a16_env(a16_mode.encode())
            lib.ref_create.restype = C.c_void_p
            lib.ref_create.argtypes = [C.c_char_p, C.c_int]
            lib.ref_destroy.argtypes = [C.c_void_p]
            lib.ref_position.argtypes = [C.c_void_p]
            lib.ref_hidden.argtypes = [C.c_void_p, _f32p]
            lib.ref_prefill_rows.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int]
            lib.ref_set_state.argtypes = [C.c_void_p, _f32p, _f32p, C.c_int, _f32p]
            lib.ref_get_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
            lib.ref_global_step_embed.argtypes = [C.c_void_p, _f32p, _f32p]
            lib.ref_global_step_row.argtypes = [C.c_void_p, _i32p, _f32p]
            lib.ref_embed_row.argtypes = [C.c_void_p, _i32p, _f32p]
            lib.ref_local_step.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
            lib.ref_audio_logits.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
            lib.ref_assistant_logits.argtypes = [C.c_void_p, _f32p, _f32p]
            lib.ref_generate.restype = C.c_int
            lib.ref_generate.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float,
                                         C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_void_p, _i32p, C.c_void_p,
                                         C.c_char_p]
            lib.ref_max_ctx.restype = C.c_int
            lib.ref_dequant_row_q8x4.argtypes = [_u8p, C.c_int, C.c_int, _f32p]
            lib.ref_row_dot_a16.restype = C.c_float
            lib.ref_row_dot_a16.argtypes = [_u8p, C.c_int, C.c_int, _f32p]
            lib.ref_row_dot_a8.restype = C.c_float
            lib.ref_row_dot_a8.argtypes = [_u8p, C.c_int, C.c_int, _f32p, C.c_int]
            lib.ref_quantize_act.argtypes = [_f32p, C.c_int, _i8p, _f32p]
            lib.ref_half_to_float_n.argtypes = [np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int, _f32p]
            lib.ref_float_to_half_n.argtypes = [_f32p, C.c_int, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")]
            lib.ref_save_prefix.restype = C.c_int
            lib.ref_save_prefix.argtypes = [C.c_void_p, C.c_char_p, _i32p, C.c_int]
            lib.ref_save_state.restype = C.c_int
            lib.ref_save_state.argtypes = [C.c_void_p, C.c_char_p, _i32p, C.c_int]
            lib.ref_sample_token.restype = C.c_int
            lib.ref_sample_token.argtypes = [_f32p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float,
                                             C.c_void_p, C.c_int, C.c_uint64]
            cls._lib = lib
        return cls._lib

    def __init__(self, weights: str, threads: int = 1, a16_mode: str = "decode"):
        self.lib = self.lib(a16_mode)
        self.h = self.lib.ref_create(str(weights).encode(), threads)
        if not self.h:
            raise RuntimeError("reference failed to load weights")
        self.max_ctx = self.lib.ref_max_ctx()

    def close(self):
        if self.h:
            self.lib.ref_destroy(self.h)
            self.h = None

    __del__ = close

    @property
    def position(self):
        return self.lib.ref_position(self.h)

    def hidden(self):
        out = np.empty(HIDDEN, np.float32)
        self.lib.ref_hidden(self.h, out)
        return out

    def set_state(self, k, v, hidden):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        if not self.lib.ref_set_state(self.h, k, v, k.shape[1], np.ascontiguousarray(hidden, np.float32)):
            raise ValueError("bad state length")

    def kv(self, layer, p0, n):
        k = np.empty((n, HIDDEN), np.float32)
        v = np.empty((n, HIDDEN), np.float32)
        self.lib.ref_get_kv(self.h, layer, p0, n, k, v)
        return k, v

    def embed_row(self, row):
        out = np.empty(HIDDEN, np.float32)
        self.lib.ref_embed_row(self.h, np.ascontiguousarray(row, np.int32), out)
        return out

    def global_step_embed(self, x):
        out = np.empty(HIDDEN, np.float32)
        self.lib.ref_global_step_embed(self.h, np.ascontiguousarray(x, np.float32), out)
        return out

    def global_step_row(self, row):
        out = np.empty(HIDDEN, np.float32)
        self.lib.ref_global_step_row(self.h, np.ascontiguousarray(row, np.int32), out)
        return out

    def prefill_rows(self, rows, start=0):
        rows = np.ascontiguousarray(rows, np.int32)
        self.lib.ref_prefill_rows(self.h, rows, rows.shape[0], start)

    def save_prefix(self, path, rows):
        """LlmModel::save_prefix (llm.cpp:485-509): the reference's .mosskv file."""
        rows = np.ascontiguousarray(rows, np.int32)
        if not self.lib.ref_save_prefix(self.h, str(path).encode(), rows, rows.shape[0]):
            raise RuntimeError("reference save_prefix failed")

    def save_state(self, path, rows):
        """LlmModel::save_state (llm.cpp:561-587): header, K/V layer by layer, then hidden."""
        rows = np.ascontiguousarray(rows, np.int32)
        if not self.lib.ref_save_state(self.h, str(path).encode(), rows, rows.shape[0]):
            raise RuntimeError("reference save_state failed")

    def local_step(self, lpos, x):
        out = np.empty(HIDDEN, np.float32)
        self.lib.ref_local_step(self.h, lpos, np.ascontiguousarray(x, np.float32), out)
        return out

    def audio_logits(self, ch, h):
        out = np.empty(CODEBOOK, np.float32)
        self.lib.ref_audio_logits(self.h, ch, np.ascontiguousarray(h, np.float32), out)
        return out

    def gate(self, h):
        out = np.empty(2, np.float32)
        self.lib.ref_assistant_logits(self.h, np.ascontiguousarray(h, np.float32), out)
        return out

    def generate(self, frames, greedy=True, temperature=0.8, top_k=25, top_p=0.95, rep=1.2, end_greedy=True,
                 min_frames=0, greedy_frames=0, seed=0, forced=None, want_logits=False, tmp_path=None):
        codes = np.zeros((frames, NVQ), np.int32)
        logits = np.zeros((frames, NVQ, CODEBOOK), np.float32) if want_logits else None
        f = None if forced is None else np.ascontiguousarray(forced, np.int32)
        tmp = (tmp_path or f"/tmp/ref_logits_{os.getpid()}.bin").encode() if want_logits else None
        n = self.lib.ref_generate(self.h, frames, int(greedy), temperature, top_k, top_p, rep, int(end_greedy),
                                  min_frames, greedy_frames, seed, _ptr(f), codes, _ptr(logits), tmp)
        return codes[:n], (logits[:n] if want_logits else None)


class RefCodec:
    """The reference's own AudioDecoder (decoder.cpp) in oracle/_ref/libmossref.so: streaming
    decode_chunk / reset_stream and the whole-utterance decode."""

    def __init__(self, weights: str, threads: int = 1):
        self.lib = RefModel.lib()
        L = self.lib
        L.ref_codec_create.restype = C.c_void_p
        L.ref_codec_create.argtypes = [C.c_char_p, C.c_int]
        L.ref_codec_destroy.argtypes = [C.c_void_p]
        L.ref_codec_reset.argtypes = [C.c_void_p]
        L.ref_codec_decode_chunk.restype = C.c_int
        L.ref_codec_decode_chunk.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p, C.c_int]
        L.ref_codec_decode.restype = C.c_int
        L.ref_codec_decode.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p, C.c_int]
        self.h = L.ref_codec_create(str(weights).encode(), threads)
        if not self.h:
            raise RuntimeError("reference failed to load the decoder")

    def close(self):
        if self.h:
            self.lib.ref_codec_destroy(self.h)
            self.h = None

    __del__ = close

    def reset(self):
        self.lib.ref_codec_reset(self.h)

    def _run(self, fn, codes):
        codes = np.ascontiguousarray(codes, np.int32)  # [16][frames]
        frames = codes.shape[1]
        out = np.empty(frames * 7680 + 16, np.float32)
        n = fn(self.h, codes, frames, out, out.size)
        if n < 0:
            raise RuntimeError("output buffer too small")
        return out[:n].copy()

    def decode_chunk(self, codes):
        return self._run(self.lib.ref_codec_decode_chunk, codes)

    def decode(self, codes):
        return self._run(self.lib.ref_codec_decode, codes)

