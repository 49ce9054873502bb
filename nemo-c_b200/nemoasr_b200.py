"""ctypes bindings for libnemoasr_b200.so (include/nemoasr.h and include/nemo_gpu.h).

The library is the product: host C (API, streaming bookkeeping, front end) over sm_100a CUDA
kernels. This module only marshals arguments; it has no compute of its own.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnemoasr_b200.so")

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int)
u16p = C.POINTER(C.c_uint16)
_lib = None


class SynthSpec(C.Structure):  # nemoasr_synth_spec_t
    _fields_ = [("seed", C.c_uint64), ("n_layers", C.c_int), ("d_model", C.c_int), ("ff_factor", C.c_int),
                ("sub_channels", C.c_int), ("num_prompts", C.c_int), ("prompt_hidden", C.c_int),
                ("pred_hidden", C.c_int), ("joint_hidden", C.c_int), ("vocab_size", C.c_int), ("att_left", C.c_int),
                ("weight_std", C.c_float), ("blank_bias", C.c_float)]


class Stats(C.Structure):  # nemoasr_stats_t
    _fields_ = [("audio_seconds", C.c_double), ("chunks", C.c_size_t), ("tokens", C.c_size_t),
                ("encoder_ms", C.c_double), ("decoder_ms", C.c_double)]


class GemmArgs(C.Structure):  # nemo_gemm_args_t
    _fields_ = [("A", C.c_void_p), ("lda", C.c_int64), ("a_plane", C.c_int64), ("a_fmt", C.c_int),
                ("W", C.c_void_p), ("ldw", C.c_int64), ("bias", C.c_void_p), ("bias_gstride", C.c_int64),
                ("C", C.c_void_p), ("ldc", C.c_int64), ("c_plane", C.c_int64), ("c_fmt", C.c_int),
                ("rpg", C.c_int), ("gstride", C.c_int64), ("rowoff", C.c_void_p), ("dynM", C.c_void_p),
                ("M", C.c_int), ("N", C.c_int), ("K", C.c_int), ("act", C.c_int), ("accumulate", C.c_int),
                ("alpha", C.c_float), ("c32", C.c_void_p), ("ldc32", C.c_int64)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C nemo-c_b200` (needs nvcc)")
        L = C.CDLL(LIB_PATH)
        L.nemoasr_synth_default.argtypes = [C.POINTER(SynthSpec)]
        L.nemoasr_synth_write.argtypes = [C.c_char_p, C.POINTER(SynthSpec), C.c_char_p, C.c_size_t]
        L.nemoasr_synth_audio.argtypes = [C.c_uint64, C.c_int, C.c_size_t, C.c_int, f32p]
        _lib = L
    return _lib


def synth_default(**kw):
    s = SynthSpec()
    lib().nemoasr_synth_default(C.byref(s))
    for k, v in kw.items():
        setattr(s, k, v)
    return s


def synth_tiny(**kw):
    """Small architecture of the same structure (fast CPU oracle runs). Larger weights and a
    blank offset chosen so ~35% of frames emit on the test audio, like the full model."""
    base = dict(n_layers=2, d_model=256, ff_factor=4, sub_channels=64, num_prompts=8, prompt_hidden=256,
                pred_hidden=128, joint_hidden=128, vocab_size=64, weight_std=0.1, blank_bias=1.9)
    base.update(kw)
    return synth_default(**base)


def synth_write(d, spec):
    err = C.create_string_buffer(512)
    if lib().nemoasr_synth_write(d.encode(), C.byref(spec), err, 512):
        raise RuntimeError(err.value.decode())
    return d


def synth_audio(seed, rate, seconds=None, n=None, pauses=False):
    n = int(round(seconds * rate)) if n is None else n
    out = np.zeros(n, np.float32)
    lib().nemoasr_synth_audio(seed, rate, n, int(pauses), out.ctypes.data_as(f32p))
    return out


def _setup_api(L):
    L.nemoasr_open.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_open.restype = C.c_void_p
    L.nemoasr_open_synthetic.argtypes = [C.POINTER(SynthSpec), C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_open_synthetic.restype = C.c_void_p
    L.nemoasr_close.argtypes = [C.c_void_p]
    L.nemoasr_feed.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_feed.restype = C.c_void_p
    L.nemoasr_free.argtypes = [C.c_void_p]
    L.nemoasr_feed_tokens.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, i32p, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_reset.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_prepare_latency.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_load_ms.argtypes = [C.c_void_p]
    L.nemoasr_load_ms.restype = C.c_double
    L.nemoasr_gpu_name.argtypes = [C.c_void_p]
    L.nemoasr_gpu_name.restype = C.c_char_p
    L.nemoasr_latency_ms.argtypes = [C.c_void_p]
    L.nemoasr_stats.argtypes = [C.c_void_p, C.POINTER(Stats)]
    L.nemoasr_set_taps.argtypes = [C.c_void_p, f32p, f32p, C.c_size_t, i32p, C.c_size_t]
    L.nemoasr_tap_counts.argtypes = [C.c_void_p, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
    L.nemoasr_batch_open.argtypes = [C.c_char_p, C.POINTER(SynthSpec), C.c_int, C.POINTER(C.c_char_p), C.c_int, C.c_int, C.c_char_p, C.c_size_t]
    L.nemoasr_batch_open.restype = C.c_void_p
    L.nemoasr_batch_close.argtypes = [C.c_void_p]
    L.nemoasr_batch_feed.argtypes = [C.c_void_p, C.POINTER(f32p), C.c_size_t, C.c_int, i32p, C.c_int, i32p, C.c_char_p, C.c_size_t]
    L.nemoasr_batch_reset.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    L.nemoasr_batch_stats.argtypes = [C.c_void_p, C.POINTER(Stats)]
    L.nemoasr_batch_set_taps.argtypes = [C.c_void_p, f32p, f32p, C.c_size_t, i32p, C.c_size_t]
    L.nemoasr_batch_attach_mel.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_size_t, C.c_char_p, C.c_size_t]
    L.nemoasr_batch_step.argtypes = [C.c_void_p, C.c_int, i32p, C.c_int, i32p, i32p, C.c_char_p, C.c_size_t]
    L.nemoasr_batch_decode_counts.argtypes = [C.c_void_p, C.POINTER(C.c_longlong), C.c_char_p, C.c_size_t]
    L.nemoasr_graphs_captured.argtypes = [C.c_void_p]
    L.nemo_gpu_wait_selftest.argtypes = [C.c_int, C.c_longlong, C.c_void_p]
    L.nemo_gemm_noalloc.argtypes = [C.POINTER(GemmArgs), C.c_void_p]
    L.nemoasr_batch_gpu_ms.argtypes = [C.c_void_p]
    L.nemoasr_batch_gpu_ms.restype = C.c_double
    L.nemo_gemm.argtypes = [C.POINTER(GemmArgs), C.c_void_p]
    L.nemo_gemm_forced.argtypes = [C.POINTER(GemmArgs), C.c_int, C.c_void_p]
    vp, i64 = C.c_void_p, C.c_int64
    L.nemo_layernorm.argtypes = [vp, vp, vp, vp, C.c_int, i64, C.c_int, C.c_int, C.c_float, vp]
    L.nemo_layernorm2.argtypes = [vp, vp, vp, vp, vp, vp, vp, C.c_int, i64, C.c_int, C.c_int, C.c_float, vp]
    L.nemo_attention_rel.argtypes = [vp, i64, i64, vp, vp, i64, i64, vp, vp, vp, vp, vp, vp, C.c_int, i64, i64] + [C.c_int] * 6 + [C.c_float, vp]
    L.nemo_dwconv_ln_silu.argtypes = [vp, i64, vp, vp, vp, vp, vp, C.c_int, i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp]
    L.nemo_conv2d_c1_s2_relu.argtypes = [vp, i64, vp, vp, vp] + [C.c_int] * 6 + [vp]
    L.nemo_dwconv2d_s2.argtypes = [vp, vp, vp, vp] + [C.c_int] * 6 + [vp]
    L.nemo_subsample_front.argtypes = [vp, i64, vp, vp, vp, vp, vp, C.c_int, i64] + [C.c_int] * 4 + [vp]
    L.nemo_flatten_rows.argtypes = [vp, vp, vp] + [C.c_int] * 5 + [vp]
    L.nemo_lstm_cell.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, vp]
    L.nemo_joint_argmax.argtypes = [vp, i64, vp, i64, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]
    L.nemo_gpu_last_error.restype = C.c_char_p
    L.nemo_gpu_launch_count.restype = C.c_uint64
    L.nemoasr_mel_create.restype = C.c_void_p
    L.nemoasr_mel_destroy.argtypes = [C.c_void_p]
    L.nemoasr_mel_push.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, f32p, C.c_size_t]
    L.nemoasr_mel_push.restype = C.c_size_t
    L.nemoasr_resampler_create.argtypes = [C.c_int, C.c_int]
    L.nemoasr_resampler_create.restype = C.c_void_p
    L.nemoasr_resampler_destroy.argtypes = [C.c_void_p]
    L.nemoasr_resampler_process.argtypes = [C.c_void_p, f32p, C.c_size_t, f32p, C.c_size_t]
    L.nemoasr_resampler_process.restype = C.c_size_t
    L.nemoasr_resampler_flush.argtypes = [C.c_void_p, f32p, C.c_size_t]
    L.nemoasr_resampler_flush.restype = C.c_size_t


def api():
    L = lib()
    if not getattr(L, "_api_ready", False):
        _setup_api(L)
        L._api_ready = True
    return L


def check(rc, what="call"):
    if rc != 0:
        raise RuntimeError(f"{what}: {api().nemo_gpu_last_error().decode()}")


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


class Session:
    """One stream through the public API (include/nemoasr.h)."""

    def __init__(self, model_dir=None, spec=None, language="auto", latency_ms=560, rate=16000):
        L = api()
        err = C.create_string_buffer(1024)
        if spec is not None:
            self.h = L.nemoasr_open_synthetic(C.byref(spec), language.encode(), latency_ms, rate, err, 1024)
        else:
            self.h = L.nemoasr_open(model_dir.encode(), language.encode(), latency_ms, rate, err, 1024)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def feed(self, samples, final=False):
        x = _f32(samples)
        err = C.create_string_buffer(1024)
        t = api().nemoasr_feed(self.h, x.ctypes.data_as(f32p), x.size, int(final), err, 1024)
        if err.value:
            raise RuntimeError(err.value.decode())
        if not t:
            return ""
        s = C.string_at(t).decode()
        api().nemoasr_free(t)
        return s

    def feed_tokens(self, samples, final=False, max_tokens=1 << 16):
        x = _f32(samples)
        out = np.zeros(max_tokens, np.int32)
        err = C.create_string_buffer(1024)
        n = api().nemoasr_feed_tokens(self.h, x.ctypes.data_as(f32p), x.size, int(final), out.ctypes.data_as(i32p), max_tokens, err, 1024)
        if n < 0:
            raise RuntimeError(err.value.decode())
        return out[:n].tolist()

    def set_taps(self, rows, d_model, joint_hidden):
        self.tp = np.zeros((rows, d_model), np.float32)
        self.tj = np.zeros((rows, joint_hidden), np.float32)
        self.tc = np.zeros(rows, np.int32)
        api().nemoasr_set_taps(self.h, self.tp.ctypes.data_as(f32p), self.tj.ctypes.data_as(f32p), rows, self.tc.ctypes.data_as(i32p), rows)

    def taps(self):
        r, c = C.c_size_t(), C.c_size_t()
        api().nemoasr_tap_counts(self.h, C.byref(r), C.byref(c))
        return dict(prompted=self.tp[:r.value].copy(), joint=self.tj[:r.value].copy(), chunk_rows=self.tc[:c.value].copy())

    def reset(self, language=None, latency_ms=560):
        err = C.create_string_buffer(1024)
        if api().nemoasr_reset(self.h, language.encode() if language else None, latency_ms, err, 1024):
            raise RuntimeError(err.value.decode())

    def stats(self):
        s = Stats()
        api().nemoasr_stats(self.h, C.byref(s))
        return dict(audio_seconds=s.audio_seconds, chunks=s.chunks, tokens=s.tokens, encoder_ms=s.encoder_ms, decoder_ms=s.decoder_ms)

    def gpu_name(self):
        return api().nemoasr_gpu_name(self.h).decode()

    def close(self):
        if getattr(self, "h", None):
            api().nemoasr_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: the module's globals are already gone
            pass


def _token_lists(tok, cnt):
    """Row s of tok holds cnt[s] token ids: one list per row, converted in one pass over the
    tokens actually written."""
    m = int(cnt.max()) if len(cnt) else 0
    if m == 0:
        return [[] for _ in range(len(cnt))]
    flat = tok[:, :m][np.arange(m)[None, :] < cnt[:, None]].tolist()
    out, s = [], 0
    for e in np.cumsum(cnt).tolist():
        out.append(flat[s:e])
        s = e
    return out


class Batch:
    """B lockstep streams on the current GPU (nemoasr_batch_*)."""

    def __init__(self, n_streams, model_dir=None, spec=None, languages=None, latency_ms=560, rate=16000):
        L = api()
        err = C.create_string_buffer(1024)
        self.B = n_streams
        langs = None
        if languages is not None:
            langs = (C.c_char_p * n_streams)(*[s.encode() for s in languages])
        self.h = L.nemoasr_batch_open(model_dir.encode() if model_dir else None, C.byref(spec) if spec is not None else None, n_streams,
                                      langs, latency_ms, rate, err, 1024)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def feed(self, samples, final=False, max_tokens=4096):
        """samples: [B][n] float32 (host). Returns a list of token-id lists, one per stream."""
        x = samples if isinstance(samples, np.ndarray) and samples.dtype == np.float32 and samples.ndim == 2 and samples.strides[1] == 4 else _f32(samples)
        assert x.shape[0] == self.B
        # one pointer per stream: rows need not be adjacent (a column slice of a larger array is read in place)
        addr = np.uint64(x.ctypes.data) + np.arange(self.B, dtype=np.uint64) * np.uint64(x.strides[0])
        ptrs = addr.ctypes.data_as(C.POINTER(f32p))
        tok = getattr(self, "_tok", None)
        if tok is None or tok.shape[1] != max_tokens:
            tok = self._tok = np.empty((self.B, max_tokens), np.int32)
        cnt = np.zeros(self.B, np.int32)
        err = C.create_string_buffer(1024)
        rc = api().nemoasr_batch_feed(self.h, ptrs, x.shape[1], int(final), tok.ctypes.data_as(i32p), max_tokens, cnt.ctypes.data_as(i32p), err, 1024)
        if rc:
            raise RuntimeError(err.value.decode())
        return _token_lists(tok, cnt)

    def set_taps(self, rows, d_model, joint_hidden):
        self.tp = np.zeros((rows, d_model), np.float32)
        self.tj = np.zeros((rows, joint_hidden), np.float32)
        self.tc = np.zeros(rows, np.int32)
        api().nemoasr_batch_set_taps(self.h, self.tp.ctypes.data_as(f32p), self.tj.ctypes.data_as(f32p), rows, self.tc.ctypes.data_as(i32p), rows)

    def decode_counts(self):
        """Greedy-decoder counts since open/reset: stream-frames, frames that emitted, decisions,
        loop iterations."""
        out = (C.c_longlong * 4)()
        err = C.create_string_buffer(1024)
        if api().nemoasr_batch_decode_counts(self.h, out, err, 1024):
            raise RuntimeError(err.value.decode())
        return dict(frames=out[0], emitting_frames=out[1], decisions=out[2], iterations=out[3])

    def stats(self):
        s = Stats()
        api().nemoasr_batch_stats(self.h, C.byref(s))
        return dict(audio_seconds=s.audio_seconds, chunks=s.chunks, tokens=s.tokens, encoder_ms=s.encoder_ms, decoder_ms=s.decoder_ms)

    def reset(self):
        err = C.create_string_buffer(1024)
        if api().nemoasr_batch_reset(self.h, err, 1024):
            raise RuntimeError(err.value.decode())

    def attach_mel(self, d_mel_ptr, stream_stride, frames):
        """Read log-mel frames from device memory (stream s at d_mel + s*stream_stride floats)."""
        err = C.create_string_buffer(1024)
        if api().nemoasr_batch_attach_mel(self.h, C.c_void_p(d_mel_ptr), stream_stride, frames, err, 1024):
            raise RuntimeError(err.value.decode())

    def step(self, final=False, max_tokens=256):
        """One chunk step of every stream; returns (status, rows, token lists)."""
        tok = np.zeros((self.B, max_tokens), np.int32)
        cnt = np.zeros(self.B, np.int32)
        rows = C.c_int(0)
        err = C.create_string_buffer(1024)
        rc = api().nemoasr_batch_step(self.h, int(final), tok.ctypes.data_as(i32p), max_tokens, cnt.ctypes.data_as(i32p), C.byref(rows), err, 1024)
        if rc < 0:
            raise RuntimeError(err.value.decode())
        return rc, rows.value, [tok[i, :cnt[i]].tolist() for i in range(self.B)]

    def gpu_ms(self):
        return api().nemoasr_batch_gpu_ms(self.h)

    def close(self):
        if getattr(self, "h", None):
            api().nemoasr_batch_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: the module's globals are already gone
            pass


def mel(samples, blocks=None):
    """Host log-mel front end of the library (same streaming behaviour as the reference)."""
    L = api()
    m = L.nemoasr_mel_create()
    samples = _f32(samples)
    blocks = blocks or [len(samples)]
    out, p = [], 0
    for i, b in enumerate(blocks):
        x = samples[p:p + b]
        p += b
        cap = p // 160 + 4
        buf = np.zeros((cap, 128), np.float32)
        n = L.nemoasr_mel_push(m, x.ctypes.data_as(f32p), x.size, int(i == len(blocks) - 1), buf.ctypes.data_as(f32p), cap)
        out.append(buf[:n])
    L.nemoasr_mel_destroy(m)
    return np.concatenate(out) if out else np.zeros((0, 128), np.float32)


def resample(samples, in_rate, out_rate, block=None):
    L = api()
    r = L.nemoasr_resampler_create(in_rate, out_rate)
    samples = _f32(samples)
    block = block or len(samples)
    out = []
    for p in range(0, len(samples), block):
        x = samples[p:p + block]
        cap = int(len(x) * out_rate / in_rate) + 4096
        buf = np.zeros(cap, np.float32)
        n = L.nemoasr_resampler_process(r, x.ctypes.data_as(f32p), x.size, buf.ctypes.data_as(f32p), cap)
        out.append(buf[:n])
    buf = np.zeros(8192, np.float32)
    n = L.nemoasr_resampler_flush(r, buf.ctypes.data_as(f32p), buf.size)
    out.append(buf[:n])
    L.nemoasr_resampler_destroy(r)
    return np.concatenate(out)
