"""moss_b200 -- B200-native engine for MOSS-TTS-Nano's per-frame LLM step.

The product is libmossgpu.so (C ABI: include/mossgpu.h; CUDA kernels for sm_100a in
csrc/).  This module is the Python host side over that ABI:

* `Engine`   -- the batched engine: stream slots, prefill, one-frame steps over many
                streams, state access.  One instance per GPU.
* `LlmModel` -- the reference's single-stream `moss::LlmModel` interface
                (csrc/include/moss/llm.h:39-90 in the reference) on top of one Engine
                stream, with the same method names, argument meaning and error behaviour
                (load() returns (ok, err); generate() stops on the end gate, honours
                teacher forcing, the cancel flag and the logits dump).
* `Codec`    -- the batched audio codec decoder (mossgpu_codec_*): codec streams, chunked
                decode of many streams per call, whole-utterance decode.
* `AudioDecoder` -- the reference's `moss::AudioDecoder` interface (decoder.h:16-33) over one
                Codec stream: load, decode, reset_stream, decode_chunk.

There is no CPU fallback: constructing an Engine without the built library or without a
CUDA device raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from dataclasses import dataclass
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
# MOSSGPU_LIB_VARIANT=stamps loads (and builds) the profiling build with phase stamps instead
LIB_VARIANT = os.environ.get("MOSSGPU_LIB_VARIANT", "")
LIB_PATH = PKG / ("libmossgpu_stamps.so" if LIB_VARIANT == "stamps" else "libmossgpu.so")

HIDDEN, HEADS, HEAD_DIM, FF, VOCAB = 768, 12, 64, 3072, 16384
NVQ, CODEBOOK, AUDIO_PAD, SLOT_TOKEN, END_TOKEN, LOCAL_LEN, LAYERS = 16, 1024, 1024, 9, 7, 17, 12

# Every symbol include/mossgpu.h declares (checked by the tests).
EXPORTS = [
    "mossgpu_create", "mossgpu_destroy", "mossgpu_last_error", "mossgpu_version", "mossgpu_set_cuda_stream",
    "mossgpu_stream_open", "mossgpu_stream_close", "mossgpu_stream_reset", "mossgpu_stream_position",
    "mossgpu_prefill", "mossgpu_prefill_embeds", "mossgpu_generate_begin", "mossgpu_step",
    "mossgpu_global_step_embed", "mossgpu_set_state", "mossgpu_get_kv", "mossgpu_get_hidden",
    "mossgpu_debug_matrix_bytes", "mossgpu_last_launch_count", "mossgpu_fill_state_random", "mossgpu_set_graphs",
    "mossgpu_kernel_profile", "mossgpu_kernel_profile_read", "mossgpu_kernel_name", "mossgpu_step_frames",
    "mossgpu_attention_workspace_bytes", "mossgpu_attention_decode_paged", "mossgpu_op_last_error",
    "mossgpu_attention_decode_paged_noalloc", "mossgpu_set_gemm_path", "mossgpu_debug_matrix_tile_bytes",
    "mossgpu_stream_fork", "mossgpu_create_rows", "mossgpu_prefill_batch", "mossgpu_prefill_embeds_batch",
    "mossgpu_set_tc_policy", "mossgpu_op_device_status", "mossgpu_debug_inject_wait_timeout", "mossgpu_set_local_path",
    "mossgpu_set_small_layers", "mossgpu_debug_small_layer_stamps",
    "mossgpu_codec_create", "mossgpu_codec_destroy", "mossgpu_codec_last_error", "mossgpu_codec_samples_per_frame",
    "mossgpu_codec_launches_per_call", "mossgpu_codec_device_bytes", "mossgpu_codec_set_cuda_stream",
    "mossgpu_codec_open", "mossgpu_codec_close", "mossgpu_codec_reset", "mossgpu_codec_decode_chunk",
    "mossgpu_codec_decode_batch", "mossgpu_codec_decode_batch_device", "mossgpu_codec_decode",
    "mossgpu_codec_profile", "mossgpu_codec_profile_read", "mossgpu_codec_kernel_name", "mossgpu_codec_status",
]


class MossGpuError(RuntimeError):
    pass


class SampleParams(C.Structure):
    """moss::SampleParams (reference csrc/include/moss/sampler.h:8-22)."""
    _fields_ = [("greedy", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("end_greedy", C.c_int), ("min_frames", C.c_int),
                ("greedy_frames", C.c_int)]

    @classmethod
    def make(cls, greedy=True, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, end_greedy=True,
             min_frames=0, greedy_frames=0) -> "SampleParams":
        return cls(int(greedy), temperature, top_k, top_p, repetition_penalty, int(end_greedy), min_frames,
                   greedy_frames)


_f32 = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32 = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_LIB = None
_LIB_LOCK = threading.Lock()


def build(force: bool = False) -> Path:
    from . import buildlib as _b  # noqa: PLC0415
    return _b.build(force=force, variant=LIB_VARIANT)


def lib() -> C.CDLL:
    """Load libmossgpu.so; raises if it has not been built (no fallback)."""
    global _LIB
    with _LIB_LOCK:
        if _LIB is not None:
            return _LIB
        if not LIB_PATH.exists():
            raise MossGpuError(f"{LIB_PATH} is missing: build it with moss_b200.build() (nvcc, sm_100a)")
        L = C.CDLL(str(LIB_PATH))
        L.mossgpu_create.restype = C.c_void_p
        L.mossgpu_create.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
        L.mossgpu_create_rows.restype = C.c_void_p
        L.mossgpu_create_rows.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
        L.mossgpu_prefill_batch.argtypes = [C.c_void_p, C.c_int, _i32, _i32, _i32, _i32]
        L.mossgpu_prefill_embeds_batch.argtypes = [C.c_void_p, C.c_int, _i32, _i32, _i32, _f32]
        L.mossgpu_set_tc_policy.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.mossgpu_destroy.argtypes = [C.c_void_p]
        L.mossgpu_last_error.restype = C.c_char_p
        L.mossgpu_last_error.argtypes = [C.c_void_p]
        L.mossgpu_version.restype = C.c_char_p
        L.mossgpu_set_cuda_stream.argtypes = [C.c_void_p, C.c_void_p]
        L.mossgpu_stream_open.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        L.mossgpu_stream_close.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_stream_reset.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_stream_position.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_int)]
        L.mossgpu_stream_fork.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]
        L.mossgpu_prefill.argtypes = [C.c_void_p, C.c_int, _i32, C.c_int, C.c_int]
        L.mossgpu_prefill_embeds.argtypes = [C.c_void_p, C.c_int, _f32, C.c_int, C.c_int]
        L.mossgpu_generate_begin.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
        L.mossgpu_step.argtypes = [C.c_void_p, _i32, C.c_int, C.POINTER(SampleParams), C.c_void_p, _i32, C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_int]
        L.mossgpu_global_step_embed.argtypes = [C.c_void_p, _i32, C.c_int, _f32, C.c_void_p]
        L.mossgpu_set_state.argtypes = [C.c_void_p, C.c_int, _f32, _f32, C.c_int, C.c_void_p]
        L.mossgpu_get_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.mossgpu_get_hidden.argtypes = [C.c_void_p, C.c_int, _f32]
        L.mossgpu_debug_matrix_bytes.argtypes = [C.c_void_p, C.c_char_p,
                                                 np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS"), C.c_size_t]
        L.mossgpu_last_launch_count.argtypes = [C.c_void_p]
        L.mossgpu_fill_state_random.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_uint64]
        L.mossgpu_step_frames.argtypes = [C.c_void_p, _i32, C.c_int, C.POINTER(SampleParams), C.c_int, C.c_void_p,
                                          C.c_void_p]
        L.mossgpu_set_graphs.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_set_gemm_path.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_debug_matrix_tile_bytes.argtypes = [C.c_void_p, C.c_char_p,
                                                      np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS"), C.c_size_t]
        L.mossgpu_kernel_profile.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_kernel_profile_read.argtypes = [C.c_void_p, _f32, np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"),
                                                  C.c_int, C.POINTER(C.c_int)]
        L.mossgpu_kernel_name.restype = C.c_char_p
        L.mossgpu_kernel_name.argtypes = [C.c_int]
        L.mossgpu_attention_workspace_bytes.restype = C.c_size_t
        L.mossgpu_attention_workspace_bytes.argtypes = [C.c_int]
        L.mossgpu_attention_decode_paged.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                                     C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t,
                                                     C.c_void_p]
        L.mossgpu_op_last_error.restype = C.c_char_p
        L.mossgpu_op_device_status.argtypes = [C.POINTER(C.c_int)]
        L.mossgpu_debug_inject_wait_timeout.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_set_local_path.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_set_small_layers.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_debug_small_layer_stamps.argtypes = [C.c_void_p, C.POINTER(C.c_ulonglong), C.c_size_t]
        L.mossgpu_attention_decode_paged_noalloc.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                                             C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.mossgpu_codec_create.restype = C.c_void_p
        L.mossgpu_codec_create.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
        L.mossgpu_codec_destroy.argtypes = [C.c_void_p]
        L.mossgpu_codec_last_error.restype = C.c_char_p
        L.mossgpu_codec_last_error.argtypes = [C.c_void_p]
        L.mossgpu_codec_samples_per_frame.argtypes = [C.c_void_p]
        L.mossgpu_codec_launches_per_call.argtypes = [C.c_void_p]
        L.mossgpu_codec_device_bytes.restype = C.c_size_t
        L.mossgpu_codec_device_bytes.argtypes = [C.c_void_p]
        L.mossgpu_codec_set_cuda_stream.argtypes = [C.c_void_p, C.c_void_p]
        L.mossgpu_codec_open.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        L.mossgpu_codec_close.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_codec_reset.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_codec_decode_chunk.argtypes = [C.c_void_p, C.c_int, _i32, C.c_int, _f32, C.c_size_t,
                                                 C.POINTER(C.c_int)]
        L.mossgpu_codec_decode_batch.argtypes = [C.c_void_p, _i32, C.c_int, _i32, C.c_int, _f32, C.c_size_t]
        L.mossgpu_codec_decode_batch_device.argtypes = [C.c_void_p, _i32, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
        L.mossgpu_codec_decode.argtypes = [C.c_void_p, _i32, C.c_int, _f32, C.c_size_t, C.POINTER(C.c_int)]
        L.mossgpu_codec_profile.argtypes = [C.c_void_p, C.c_int]
        L.mossgpu_codec_profile_read.argtypes = [C.c_void_p, _f32, _i32, C.c_int, C.POINTER(C.c_int)]
        L.mossgpu_codec_kernel_name.restype = C.c_char_p
        L.mossgpu_codec_kernel_name.argtypes = [C.c_int]
        L.mossgpu_codec_status.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        _LIB = L
        return L


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Engine:
    """One GPU's batched engine (mossgpu_create)."""

    def __init__(self, weights: str, device: int = 0, max_streams: int = 64, max_ctx: int = 4608, kv_pages: int = 0,
                 max_rows: int = 0):
        self.lib = lib()
        err = C.create_string_buffer(1024)
        self.h = self.lib.mossgpu_create_rows(str(weights).encode(), device, max_streams, max_ctx, kv_pages, max_rows,
                                              err, 1024)
        if not self.h:
            raise MossGpuError(err.value.decode(errors="replace"))
        self.max_streams, self.max_ctx = max_streams, max_ctx

    def _check(self, rc: int):
        if rc != 0:
            raise MossGpuError(self.lib.mossgpu_last_error(self.h).decode(errors="replace"))

    def close(self):
        if getattr(self, "h", None):
            self.lib.mossgpu_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def set_cuda_stream(self, stream_handle: int | None):
        self._check(self.lib.mossgpu_set_cuda_stream(self.h, C.c_void_p(stream_handle or 0)))

    def open(self) -> int:
        sid = C.c_int()
        self._check(self.lib.mossgpu_stream_open(self.h, C.byref(sid)))
        return sid.value

    def close_stream(self, sid: int):
        self._check(self.lib.mossgpu_stream_close(self.h, sid))

    def reset(self, sid: int):
        self._check(self.lib.mossgpu_stream_reset(self.h, sid))

    def fork(self, src: int, n_pos: int) -> int:
        """A new stream sharing src's first n_pos KV positions (see mossgpu_stream_fork)."""
        out = C.c_int(-1)
        self._check(self.lib.mossgpu_stream_fork(self.h, src, n_pos, C.byref(out)))
        return out.value

    def position(self, sid: int) -> int:
        p = C.c_int()
        self._check(self.lib.mossgpu_stream_position(self.h, sid, C.byref(p)))
        return p.value

    def prefill(self, sid: int, rows, start: int = 0):
        rows = np.ascontiguousarray(rows, np.int32).reshape(-1, NVQ + 1)
        self._check(self.lib.mossgpu_prefill(self.h, sid, rows, rows.shape[0], start))

    def prefill_embeds(self, sid: int, x, start: int = 0):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, HIDDEN)
        self._check(self.lib.mossgpu_prefill_embeds(self.h, sid, x, x.shape[0], start))

    @staticmethod
    def _batch(sids, parts, starts, m, width, dtype):
        sids = np.ascontiguousarray(sids, np.int32)
        if m is None:  # a list of per-stream arrays
            arrs = [np.ascontiguousarray(p, dtype).reshape(-1, width) for p in parts]
            m = np.array([a.shape[0] for a in arrs], np.int32)
            flat = np.concatenate(arrs) if arrs else np.zeros((0, width), dtype)
        else:  # one array holding the streams' rows one after the other, m[i] rows each
            m = np.ascontiguousarray(m, np.int32)
            flat = np.ascontiguousarray(parts, dtype).reshape(-1, width)
            if flat.shape[0] < int(m.sum()):
                raise ValueError("fewer rows than sum(m)")
        if flat.shape[0] == 0:
            flat = np.zeros((1, width), dtype)
        st = np.zeros(len(sids), np.int32) if starts is None else np.ascontiguousarray(starts, np.int32)
        if not (len(sids) == len(m) == len(st)):
            raise ValueError("stream ids, row counts and starts differ in length")
        return sids, m, st, flat

    def prefill_batch(self, sids, rows, starts=None, m=None):
        """Several streams' prompts in shared passes: rows = a list of [m_i][17] arrays (one per
        stream of sids), or one [sum m][17] array with the row counts in m."""
        s, m, st, flat = self._batch(sids, rows, starts, m, NVQ + 1, np.int32)
        self._check(self.lib.mossgpu_prefill_batch(self.h, len(s), s, m, st, flat))

    def prefill_embeds_batch(self, sids, x, starts=None, m=None):
        s, m, st, flat = self._batch(sids, x, starts, m, HIDDEN, np.float32)
        self._check(self.lib.mossgpu_prefill_embeds_batch(self.h, len(s), s, m, st, flat))

    def set_tc_policy(self, direct_min_rows: int = 256, direct_rows: int = 0):
        self._check(self.lib.mossgpu_set_tc_policy(self.h, direct_min_rows, direct_rows))

    def generate_begin(self, sid: int, seed: int = 0):
        self._check(self.lib.mossgpu_generate_begin(self.h, sid, seed))

    def step(self, sids, params: SampleParams, forced=None, want_logits=False, run_global=True):
        """One frame for every stream in `sids`.  Returns (codes[n][16], stop[n], gate[n][2], logits)."""
        sids = np.ascontiguousarray(sids, np.int32).reshape(-1)
        n = sids.size
        codes = np.zeros((n, NVQ), np.int32)
        stop = np.zeros(n, np.uint8)
        gate = np.zeros((n, 2), np.float32)
        logits = np.zeros((n, NVQ, CODEBOOK), np.float32) if want_logits else None
        f = None if forced is None else np.ascontiguousarray(forced, np.int32).reshape(n, NVQ)
        self._check(self.lib.mossgpu_step(self.h, sids, n, C.byref(params), _ptr(f), codes, _ptr(stop), _ptr(logits),
                                          _ptr(gate), int(run_global)))
        return codes, stop.astype(bool), gate, logits

    def step_frames(self, sids, params: SampleParams, n_frames: int, want_codes=True):
        """n_frames free-running frames on the device.  Returns (codes[n_frames][n][16], frames_done[n])."""
        sids = np.ascontiguousarray(sids, np.int32).reshape(-1)
        codes = np.zeros((n_frames, sids.size, NVQ), np.int32) if want_codes else None
        done = np.zeros(sids.size, np.int32)
        self._check(self.lib.mossgpu_step_frames(self.h, sids, sids.size, C.byref(params), n_frames, _ptr(codes),
                                                 _ptr(done)))
        return codes, done

    def global_step_embed(self, sids, x, want_hidden=True):
        sids = np.ascontiguousarray(sids, np.int32).reshape(-1)
        x = np.ascontiguousarray(x, np.float32).reshape(sids.size, HIDDEN)
        out = np.zeros((sids.size, HIDDEN), np.float32) if want_hidden else None
        self._check(self.lib.mossgpu_global_step_embed(self.h, sids, sids.size, x, _ptr(out)))
        return out

    def set_state(self, sid: int, k, v, hidden=None):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        h = None if hidden is None else np.ascontiguousarray(hidden, np.float32)
        self._check(self.lib.mossgpu_set_state(self.h, sid, k, v, k.shape[1], _ptr(h)))

    def kv(self, sid: int, layer: int, p0: int, n: int):
        k = np.zeros((n, HIDDEN), np.float32)
        v = np.zeros((n, HIDDEN), np.float32)
        self._check(self.lib.mossgpu_get_kv(self.h, sid, layer, p0, n, _ptr(k), _ptr(v)))
        return k, v

    def hidden(self, sid: int) -> np.ndarray:
        out = np.zeros(HIDDEN, np.float32)
        self._check(self.lib.mossgpu_get_hidden(self.h, sid, out))
        return out

    def matrix_bytes(self, name: str, rows: int, cols: int) -> np.ndarray:
        out = np.zeros((rows // 4) * (cols // 32) * 136, np.uint8)
        self._check(self.lib.mossgpu_debug_matrix_bytes(self.h, name.encode(), out, out.size))
        return out

    def last_launch_count(self) -> int:
        return self.lib.mossgpu_last_launch_count(self.h)

    def fill_state_random(self, sid: int, n_pos: int, seed: int = 0):
        self._check(self.lib.mossgpu_fill_state_random(self.h, sid, n_pos, seed))

    def debug_inject_wait_timeout(self, enable: bool):
        """Test hook: make the next frames' first split-K attention wait run out (see mossgpu.h)."""
        self._check(self.lib.mossgpu_debug_inject_wait_timeout(self.h, int(enable)))

    def set_local_path(self, mode: int):
        """0 = fused local decoder for greedy frames, 1 = per-step kernels for every frame (default)."""
        self._check(self.lib.mossgpu_set_local_path(self.h, mode))

    def set_small_layers(self, mode: int):
        """Global layers of <= 8-row decode batches: 1 = two launches a layer (default), 0 = five."""
        self._check(self.lib.mossgpu_set_small_layers(self.h, mode))

    def small_layer_stamps(self) -> np.ndarray:
        """[24 launches][96 CTAs][12 phases] %globaltimer stamps (ns) of the last small-layer step;
        only in a library built with phase stamps (MOSSGPU_LIB_VARIANT=stamps)."""
        out = np.zeros((24, 96, 12), dtype=np.uint64)
        self._check(self.lib.mossgpu_debug_small_layer_stamps(
            self.h, out.ctypes.data_as(C.POINTER(C.c_ulonglong)), out.size))
        return out

    def set_graphs(self, enable: bool):
        self._check(self.lib.mossgpu_set_graphs(self.h, int(enable)))

    def set_gemm_path(self, mode: int):
        """0 = automatic, 1 = CUDA-core GEMV, 2 = tcgen05 tensor cores, 3 = tensor cores with single fp16 operands."""
        self._check(self.lib.mossgpu_set_gemm_path(self.h, mode))

    def matrix_tile_bytes(self, name: str, rows: int, cols: int) -> np.ndarray:
        out = np.zeros((rows // 4) * (cols // 32) * 136, np.uint8)
        self._check(self.lib.mossgpu_debug_matrix_tile_bytes(self.h, name.encode(), out, out.size))
        return out

    def kernel_profile(self, enable: bool):
        self._check(self.lib.mossgpu_kernel_profile(self.h, int(enable)))

    def kernel_profile_read(self) -> dict[str, tuple[float, int]]:
        """{kernel class: (summed ms, launches)} since kernel_profile(True)."""
        ms = np.zeros(64, np.float32)
        n = np.zeros(64, np.int32)
        k = C.c_int()
        self._check(self.lib.mossgpu_kernel_profile_read(self.h, ms, n, 64, C.byref(k)))
        return {self.lib.mossgpu_kernel_name(i).decode(): (float(ms[i]), int(n[i])) for i in range(k.value)}


@dataclass
class FrameTiming:
    """moss::FrameTiming (llm.h:34-37)."""
    global_ms: float = 0.0
    local_ms: float = 0.0


class LlmModel:
    """The reference's moss::LlmModel interface (llm.h:39-90) over one Engine stream."""

    def __init__(self, device: int = 0, max_ctx: int = 4608, engine: Engine | None = None):
        self._device, self._max_ctx = device, max_ctx
        self._engine = engine
        self._sid = None
        self._prefix_pos = 0
        self._prefix_kv = None
        self._logits_dump_path = ""
        self._gate_dump_path = ""
        self._cancel = None

    # llm.h:46 -- bool load(path, std::string* err)
    def load(self, weights_path: str) -> tuple[bool, str]:
        try:
            if self._engine is None:
                self._engine = Engine(weights_path, self._device, max_streams=1, max_ctx=self._max_ctx)
            self._sid = self._engine.open()
        except (MossGpuError, OSError) as e:
            return False, str(e)
        return True, ""

    def reset(self):  # llm.h:49
        self._engine.reset(self._sid)

    def prefill(self, rows, start: int = 0):  # llm.h:53
        self._engine.prefill(self._sid, rows, start)

    def snapshot_prefix(self):  # llm.h:57, llm.cpp:455-467
        self._prefix_pos = self.position()
        if self._prefix_pos > 0:
            self._prefix_kv = [self._engine.kv(self._sid, l, 0, self._prefix_pos) for l in range(LAYERS)]

    def restore_prefix(self):  # llm.h:59, llm.cpp:469-483
        if self._prefix_pos <= 0:
            self._engine.reset(self._sid)
            return
        k = np.stack([kv[0] for kv in self._prefix_kv])
        v = np.stack([kv[1] for kv in self._prefix_kv])
        self._engine.set_state(self._sid, k, v, None)

    def prefix_pos(self) -> int:
        return self._prefix_pos

    def set_logits_dump(self, path: str):  # llm.h:76
        self._logits_dump_path = path

    def set_gate_dump(self, path: str):  # llm.h:79
        self._gate_dump_path = path

    def set_cancel_flag(self, flag):  # llm.h:83: any object with is_set() (threading.Event)
        self._cancel = flag

    def hidden(self) -> np.ndarray:
        return self._engine.hidden(self._sid)

    def position(self) -> int:
        return self._engine.position(self._sid)

    def generate(self, max_frames: int, params: SampleParams, seed: int = 0, timing: list | None = None,
                 forced=None, on_frame=None) -> list[list[int]]:
        """llm.cpp:634-733.  Returns rows [0, code0..code15] like moss::Row (text slot 0)."""
        import time
        frames = []
        logits_dump = [] if self._logits_dump_path else None
        gate_dump = [] if self._gate_dump_path else None
        self._engine.generate_begin(self._sid, seed)
        forced = None if forced is None else np.asarray(forced, np.int32).reshape(-1, NVQ)
        for f in range(max_frames):
            if self.position() >= self._max_ctx:
                break
            if self._cancel is not None and self._cancel.is_set():
                break
            t0 = time.perf_counter()
            last = not (f + 1 < max_frames)
            fr = None if forced is None else forced[f]
            codes, stop, gate, logits = self._engine.step([self._sid], params, forced=fr,
                                                          want_logits=logits_dump is not None, run_global=not last)
            dt = (time.perf_counter() - t0) * 1e3
            if gate_dump is not None:
                gate_dump.append((f, float(gate[0, 1] - gate[0, 0])))
            if stop[0]:
                break
            if logits_dump is not None:
                logits_dump.append(logits[0])
            row = [0] + [int(c) for c in codes[0]]
            frames.append(row)
            if timing is not None:
                timing.append(FrameTiming(global_ms=0.0 if last else dt, local_ms=0.0))
            if on_frame is not None:
                on_frame(f, row)
        if logits_dump is not None:
            np.asarray(logits_dump, np.float32).tofile(self._logits_dump_path)
        if gate_dump is not None:
            with open(self._gate_dump_path, "w") as fh:
                fh.write("frame,slot_minus_end\n")
                for f, m in gate_dump:
                    fh.write(f"{f},{m:.4f}\n")
        return frames


class Codec:
    """One GPU's batched audio codec decoder (mossgpu_codec_create)."""

    def __init__(self, decoder_path: str, device: int = 0, max_streams: int = 8, max_batch_frames: int = 64):
        self.lib = lib()
        err = C.create_string_buffer(1024)
        self.h = self.lib.mossgpu_codec_create(str(decoder_path).encode(), device, max_streams, max_batch_frames,
                                               err, 1024)
        if not self.h:
            raise MossGpuError(err.value.decode(errors="replace"))
        self.max_streams, self.max_batch_frames = max_streams, max_batch_frames
        self.samples_per_frame = self.lib.mossgpu_codec_samples_per_frame(self.h)

    def _check(self, rc: int):
        if rc != 0:
            raise MossGpuError(self.lib.mossgpu_codec_last_error(self.h).decode(errors="replace"))

    def close(self):
        if getattr(self, "h", None):
            self.lib.mossgpu_codec_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def set_cuda_stream(self, stream_handle: int | None):
        self._check(self.lib.mossgpu_codec_set_cuda_stream(self.h, C.c_void_p(stream_handle or 0)))

    def launches_per_call(self) -> int:
        return self.lib.mossgpu_codec_launches_per_call(self.h)

    def profile(self, enable: bool):
        self._check(self.lib.mossgpu_codec_profile(self.h, int(enable)))

    def profile_read(self) -> dict:
        """{kernel class: (device ms, launches)} since the last read (synchronises)."""
        ms = np.zeros(16, np.float32)
        n = np.zeros(16, np.int32)
        k = C.c_int()
        self._check(self.lib.mossgpu_codec_profile_read(self.h, ms, n, 16, C.byref(k)))
        return {self.lib.mossgpu_codec_kernel_name(i).decode(): (float(ms[i]), int(n[i])) for i in range(k.value)}

    def device_bytes(self) -> int:
        return self.lib.mossgpu_codec_device_bytes(self.h)

    def open(self) -> int:
        sid = C.c_int(-1)
        self._check(self.lib.mossgpu_codec_open(self.h, C.byref(sid)))
        return sid.value

    def close_stream(self, sid: int):
        self._check(self.lib.mossgpu_codec_close(self.h, sid))

    def reset(self, sid: int):
        self._check(self.lib.mossgpu_codec_reset(self.h, sid))

    def decode_chunk(self, sid: int, codes) -> np.ndarray:
        """codes [16][frames] -> samples [frames * samples_per_frame]."""
        codes = np.ascontiguousarray(codes, np.int32).reshape(NVQ, -1)
        frames = codes.shape[1]
        out = np.empty(frames * self.samples_per_frame, np.float32)
        n = C.c_int(0)
        self._check(self.lib.mossgpu_codec_decode_chunk(self.h, sid, codes, frames, out, out.size, C.byref(n)))
        return out[:n.value]

    def decode_batch(self, sids, codes) -> np.ndarray:
        """codes [n][16][frames] -> samples [n][frames * samples_per_frame]."""
        sids = np.ascontiguousarray(sids, np.int32).reshape(-1)
        codes = np.ascontiguousarray(codes, np.int32).reshape(sids.size, NVQ, -1)
        frames = codes.shape[2]
        out = np.empty((sids.size, frames * self.samples_per_frame), np.float32)
        self._check(self.lib.mossgpu_codec_decode_batch(self.h, sids, sids.size, codes, frames, out, out.size))
        return out

    def decode_batch_device(self, sids, codes_ptr: int, frames: int, out_ptr: int):
        """Enqueue a batch with device codes [n][16][frames] (int32) and output (fp32)."""
        sids = np.ascontiguousarray(sids, np.int32).reshape(-1)
        self._check(self.lib.mossgpu_codec_decode_batch_device(self.h, sids, sids.size, C.c_void_p(codes_ptr),
                                                               frames, C.c_void_p(out_ptr)))

    def status(self) -> int:
        """1 when an activation since the last read left the fp16 range (synchronises)."""
        code = C.c_int(0)
        self._check(self.lib.mossgpu_codec_status(self.h, C.byref(code)))
        return code.value

    def decode(self, codes) -> np.ndarray:
        """A whole utterance, codes [16][frames], from a clean state."""
        codes = np.ascontiguousarray(codes, np.int32).reshape(NVQ, -1)
        frames = codes.shape[1]
        out = np.empty(frames * self.samples_per_frame, np.float32)
        n = C.c_int(0)
        self._check(self.lib.mossgpu_codec_decode(self.h, codes, frames, out, out.size, C.byref(n)))
        return out[:n.value]


class AudioDecoder:
    """The reference's moss::AudioDecoder interface (decoder.h:16-33) over one Codec stream.

    `threads` is accepted for the signature and ignored (the work runs on the GPU)."""

    def __init__(self, threads: int = 1, device: int = 0, max_chunk_frames: int = 64):
        self._device, self._max_chunk = device, max_chunk_frames
        self._codec = None
        self._sid = None
        self._info = ""

    def load(self, path: str) -> tuple[bool, str]:  # decoder.h:21
        try:
            self._codec = Codec(path, self._device, max_streams=1, max_batch_frames=self._max_chunk)
            self._sid = self._codec.open()
        except (MossGpuError, OSError) as e:
            return False, str(e)
        self._info = f"decoder weights={path} device={self._device}"
        return True, ""

    def decode(self, codes, frames: int) -> np.ndarray:  # decoder.h:24
        return self._codec.decode(np.asarray(codes, np.int32).reshape(NVQ, frames))

    def reset_stream(self):  # decoder.h:27
        self._codec.reset(self._sid)

    def decode_chunk(self, codes, frames: int) -> np.ndarray:  # decoder.h:29
        codes = np.asarray(codes, np.int32).reshape(NVQ, frames)
        if frames <= self._max_chunk:
            return self._codec.decode_chunk(self._sid, codes)
        return np.concatenate([self._codec.decode_chunk(self._sid, codes[:, f:f + self._max_chunk])
                               for f in range(0, frames, self._max_chunk)])

    def info(self) -> str:
        return self._info
