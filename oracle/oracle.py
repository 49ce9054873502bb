"""ORACLE — TEST INFRASTRUCTURE ONLY.

ctypes bindings for the C restatement (liboracle.so, see oracle.h) and for the reference's own host
code built on the CPU (_ref/libnemoref.so, see ref_gpu_cpu.c). Only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline / reference arm import this module, as the checker
or the timed CPU baseline; the product never does.
"""
import ctypes as C
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libnemoref.so")

_lib = None
_ref = None

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int)
u16p = C.POINTER(C.c_uint16)


def _ptr(a, t=f32p):
    return a.ctypes.data_as(t) if a is not None else None


class OrConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "n_layers", "d_model", "n_heads", "d_ff", "sub_channels", "feat_in", "num_prompts", "prompt_hidden",
        "pred_hidden", "vocab_size", "joint_hidden", "max_symbols", "att_left", "max_right")]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `make -C oracle`")
        L = C.CDLL(LIB_PATH)
        L.or_gemm.argtypes = [f32p, C.c_int, u16p, C.c_int, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.or_layernorm.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_float]
        L.or_layernorm2.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_float]
        L.or_attention_rel.argtypes = [f32p, C.c_int, f32p, f32p, C.c_int, f32p, f32p, f32p, f32p] + [C.c_int] * 6 + [C.c_float]
        L.or_dwconv_ln_silu.argtypes = [f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_float]
        L.or_conv2d_c1_s2_relu.argtypes = [f32p, f32p, f32p, f32p] + [C.c_int] * 5
        L.or_dwconv2d_s2.argtypes = [f32p, f32p, f32p, f32p] + [C.c_int] * 5
        L.or_flatten_cf.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_int]
        L.or_lstm_cell.argtypes = [f32p, f32p, f32p, f32p, C.c_int]
        L.or_joint_argmax.argtypes = [f32p, C.c_int, f32p, u16p, f32p, C.c_int, C.c_int, C.c_int, i32p, f32p, f32p]
        L.or_model_create.argtypes = [C.POINTER(OrConfig), C.c_int, C.POINTER(C.c_char_p), C.POINTER(u16p),
                                      C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t]
        L.or_model_create.restype = C.c_void_p
        L.or_model_set_language.argtypes = [C.c_void_p, C.c_int]
        L.or_model_free.argtypes = [C.c_void_p]
        L.or_model_ptab.argtypes = [C.c_void_p, C.c_int]
        L.or_model_ptab.restype = f32p
        L.or_model_prompt_bias.argtypes = [C.c_void_p]
        L.or_model_prompt_bias.restype = f32p
        L.or_open.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
        L.or_open.restype = C.c_void_p
        L.or_close.argtypes = [C.c_void_p]
        L.or_feed.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, i32p, C.c_int, C.c_char_p, C.c_size_t]
        L.or_set_taps.argtypes = [C.c_void_p, f32p, f32p, C.c_size_t, i32p, C.c_size_t, i32p, i32p, f32p, C.c_size_t]
        L.or_tap_counts.argtypes = [C.c_void_p, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        L.or_mel_create.restype = C.c_void_p
        L.or_mel_destroy.argtypes = [C.c_void_p]
        L.or_mel_push.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, f32p, C.c_size_t]
        L.or_mel_push.restype = C.c_size_t
        L.or_resampler_create.argtypes = [C.c_int, C.c_int]
        L.or_resampler_create.restype = C.c_void_p
        L.or_resampler_destroy.argtypes = [C.c_void_p]
        L.or_resampler_process.argtypes = [C.c_void_p, f32p, C.c_size_t, f32p, C.c_size_t]
        L.or_resampler_process.restype = C.c_size_t
        L.or_resampler_flush.argtypes = [C.c_void_p, f32p, C.c_size_t]
        L.or_resampler_flush.restype = C.c_size_t
        L.or_num_threads.restype = C.c_int
        _lib = L
    return _lib


# ---------------------------------------------------------------------------------------------
# checkpoint reading (safetensors + config.json in the reference's layout)

def read_checkpoint(d):
    """Returns (config dict, {name: np.uint16 array}) with the tensors memory-mapped."""
    cfg = json.load(open(os.path.join(d, "config.json")))
    path = os.path.join(d, "model.safetensors")
    with open(path, "rb") as f:
        hl = int.from_bytes(f.read(8), "little")
        hdr = json.loads(f.read(hl))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    tensors = {}
    for k, v in hdr.items():
        if k == "__metadata__":
            continue
        assert v["dtype"] == "BF16", k
        a, b = v["data_offsets"]
        tensors[k] = mm[8 + hl + a: 8 + hl + b].view(np.uint16)
    return cfg, tensors


def or_config(cfg):
    enc, pr, dec, jo = cfg["encoder"], cfg["prompt"], cfg["decoder"], cfg["joint"]
    rights = [p[1] for p in enc["att_context_size"]]
    return OrConfig(enc["n_layers"], enc["d_model"], enc["n_heads"], enc["d_model"] * enc["ff_expansion_factor"],
                    enc["subsampling_conv_channels"], enc["feat_in"], pr["num_prompts"], pr["prompt_hidden"],
                    dec["pred_hidden"], dec["vocab_size"], jo["joint_hidden"], cfg.get("max_symbols", 10),
                    enc["att_context_size"][-1][0], max(rights))


class Model:
    def __init__(self, ckpt_dir):
        L = lib()
        self.cfg, t = read_checkpoint(ckpt_dir)
        self.oc = or_config(self.cfg)
        names = list(t.keys())
        arrs = [np.ascontiguousarray(t[n]) for n in names]
        cn = (C.c_char_p * len(names))(*[n.encode() for n in names])
        cp = (u16p * len(names))(*[_ptr(a, u16p) for a in arrs])
        cnum = (C.c_size_t * len(names))(*[a.size for a in arrs])
        err = C.create_string_buffer(512)
        self.h = L.or_model_create(C.byref(self.oc), len(names), cn, cp, cnum, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        self.prompt_dict = self.cfg["prompt"]["prompt_dictionary"]

    def set_language(self, lang):
        idx = self.prompt_dict[lang] if isinstance(lang, str) else int(lang)
        if lib().or_model_set_language(self.h, idx):
            raise ValueError(lang)

    def ptab(self, layer):
        P = 2 * (self.oc.att_left + self.oc.max_right + 3) - 1
        return np.ctypeslib.as_array(lib().or_model_ptab(self.h, layer), shape=(P * self.oc.d_model,)).reshape(P, -1).copy()

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.or_model_free(self.h)
            self.h = None


class Session:
    """Restated nemoasr session: feed() returns token ids; taps record encoder rows."""

    def __init__(self, model, latency_ms, input_rate, tap_rows=0, tap_decisions=0):
        L = lib()
        err = C.create_string_buffer(512)
        self.model = model
        self.h = L.or_open(model.h, latency_ms, input_rate, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        self.tap_rows = tap_rows
        if tap_rows:
            D, JH = model.oc.d_model, model.oc.joint_hidden
            self.prompted = np.zeros((tap_rows, D), np.float32)
            self.joint = np.zeros((tap_rows, JH), np.float32)
            self.chunk_rows = np.zeros(tap_rows, np.int32)
            nd = max(tap_decisions, 1)
            self.dec_frame = np.zeros(nd, np.int32)
            self.dec_token = np.zeros(nd, np.int32)
            self.dec_margin = np.zeros(nd, np.float32)
            L.or_set_taps(self.h, _ptr(self.prompted), _ptr(self.joint), tap_rows, _ptr(self.chunk_rows, i32p), tap_rows,
                          _ptr(self.dec_frame, i32p), _ptr(self.dec_token, i32p), _ptr(self.dec_margin), nd)

    def feed(self, samples, final=False, max_tokens=1 << 16):
        samples = np.ascontiguousarray(samples, np.float32)
        out = np.zeros(max_tokens, np.int32)
        err = C.create_string_buffer(512)
        n = lib().or_feed(self.h, _ptr(samples), samples.size, int(final), _ptr(out, i32p), max_tokens, err, 512)
        if n < 0:
            raise RuntimeError(err.value.decode())
        return out[:n].tolist()

    def taps(self):
        r, c, d = C.c_size_t(), C.c_size_t(), C.c_size_t()
        lib().or_tap_counts(self.h, C.byref(r), C.byref(c), C.byref(d))
        r, c, d = r.value, c.value, d.value
        nd = min(d, self.dec_frame.size)
        return dict(prompted=self.prompted[:r].copy(), joint=self.joint[:r].copy(), chunk_rows=self.chunk_rows[:c].copy(),
                    dec_frame=self.dec_frame[:nd].copy(), dec_token=self.dec_token[:nd].copy(),
                    dec_margin=self.dec_margin[:nd].copy(), decisions=d)

    def close(self):
        if self.h:
            lib().or_close(self.h)
            self.h = None

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            self.close()


def run_stream(model, audio, rate, latency_ms, language="auto", block=None, tap_rows=4096, tap_decisions=1 << 16):
    """Feed audio in blocks (default 100 ms, like tools/libtest.c:21-26) with a final flush."""
    model.set_language(language)
    s = Session(model, latency_ms, rate, tap_rows=tap_rows, tap_decisions=tap_decisions)
    block = block or rate // 10
    toks = []
    for p in range(0, len(audio), block):
        toks += s.feed(audio[p:p + block], final=p + block >= len(audio))
    if len(audio) == 0:
        toks += s.feed(np.zeros(0, np.float32), final=True)
    t = s.taps()
    s.close()
    t["tokens"] = toks
    return t


def mel(samples, blocks=None):
    """Streaming log-mel of samples (16 kHz); blocks = list of block lengths (default one block)."""
    L = lib()
    m = L.or_mel_create()
    samples = np.ascontiguousarray(samples, np.float32)
    blocks = blocks or [len(samples)]
    out = []
    p = 0
    for i, b in enumerate(blocks):
        x = samples[p:p + b]
        p += b
        cap = (p // 160) + 4
        buf = np.zeros((cap, 128), np.float32)
        n = L.or_mel_push(m, _ptr(x), x.size, int(i == len(blocks) - 1), _ptr(buf), cap)
        out.append(buf[:n])
    L.or_mel_destroy(m)
    return np.concatenate(out) if out else np.zeros((0, 128), np.float32)


def resample(samples, in_rate, out_rate, block=None):
    L = lib()
    r = L.or_resampler_create(in_rate, out_rate)
    samples = np.ascontiguousarray(samples, np.float32)
    block = block or len(samples)
    out = []
    for p in range(0, len(samples), block):
        x = samples[p:p + block]
        cap = int(len(x) * out_rate / in_rate) + 4096
        buf = np.zeros(cap, np.float32)
        n = L.or_resampler_process(r, _ptr(x), x.size, _ptr(buf), cap)
        out.append(buf[:n])
    buf = np.zeros(8192, np.float32)
    n = L.or_resampler_flush(r, _ptr(buf), buf.size)
    out.append(buf[:n])
    L.or_resampler_destroy(r)
    return np.concatenate(out)


# ---------------------------------------------------------------------------------------------
# kernels (numpy in, numpy out)

def gemm(A, W, bias=None, C0=None, act=0, accumulate=False, alpha=1.0):
    A = np.ascontiguousarray(A, np.float32)
    W = np.ascontiguousarray(W, np.uint16)
    M, K = A.shape
    N = W.shape[0]
    nout = N // 2 if act == 3 else N
    Cm = np.zeros((M, nout), np.float32) if C0 is None else np.array(C0, np.float32, copy=True)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().or_gemm(_ptr(A), K, _ptr(W, u16p), W.shape[1], _ptr(b), _ptr(Cm), nout, M, N, K, act, int(accumulate), alpha)
    return Cm


def layernorm(X, g, b, eps=1e-5):
    X = np.ascontiguousarray(X, np.float32)
    Y = np.zeros_like(X)
    lib().or_layernorm(_ptr(X), _ptr(np.ascontiguousarray(g, np.float32)), _ptr(np.ascontiguousarray(b, np.float32)), _ptr(Y),
                       X.shape[0], X.shape[1], eps)
    return Y


def layernorm2(X, g1, b1, g2, b2, eps=1e-5):
    X = np.ascontiguousarray(X, np.float32)
    Y1, Y2 = np.zeros_like(X), np.zeros_like(X)
    c = lambda a: _ptr(np.ascontiguousarray(a, np.float32))
    lib().or_layernorm2(_ptr(X), c(g1), c(b1), c(g2), c(b2), _ptr(Y1), _ptr(Y2), X.shape[0], X.shape[1], eps)
    return Y1, Y2


def attention_rel(Q, K, V, P, bu, bv, c, L, Lmax, H, dh):
    """Q [c][ldq], K/V [L][ldk] (views with row strides), P [2Lmax-1][D]."""
    D = H * dh
    O = np.zeros((c, D), np.float32)
    Qc, Kc, Vc = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V))
    lib().or_attention_rel(_ptr(Qc), Qc.shape[1], _ptr(Kc), _ptr(Vc), Kc.shape[1], _ptr(np.ascontiguousarray(P, np.float32)),
                           _ptr(np.ascontiguousarray(bu, np.float32)), _ptr(np.ascontiguousarray(bv, np.float32)), _ptr(O),
                           c, L, Lmax, H, dh, D, 1.0 / np.sqrt(np.float32(dh)))
    return O


def dwconv_ln_silu(din, W, g, b, c, taps=9, eps=1e-5):
    din = np.ascontiguousarray(din, np.float32)
    D = din.shape[1]
    Y = np.zeros((c, D), np.float32)
    c_ = lambda a: _ptr(np.ascontiguousarray(a, np.float32))
    lib().or_dwconv_ln_silu(_ptr(din), c_(W), c_(g), c_(b), _ptr(Y), c, D, taps, eps)
    return Y


def conv2d_c1_s2_relu(X, W, b):
    X = np.ascontiguousarray(X, np.float32)
    T, F = X.shape
    CH = b.size
    T1, F1 = T // 2 + 1, F // 2 + 1
    Y = np.zeros((T1, F1, CH), np.float32)
    lib().or_conv2d_c1_s2_relu(_ptr(X), _ptr(np.ascontiguousarray(W, np.float32)), _ptr(np.ascontiguousarray(b, np.float32)),
                               _ptr(Y), T, F, T1, F1, CH)
    return Y


def dwconv2d_s2(X, W, b):
    X = np.ascontiguousarray(X, np.float32)
    T, F, CH = X.shape
    T1, F1 = T // 2 + 1, F // 2 + 1
    Y = np.zeros((T1, F1, CH), np.float32)
    lib().or_dwconv2d_s2(_ptr(X), _ptr(np.ascontiguousarray(W, np.float32)), _ptr(np.ascontiguousarray(b, np.float32)),
                         _ptr(Y), T, F, T1, F1, CH)
    return Y


def flatten_cf(X):
    X = np.ascontiguousarray(X, np.float32)
    T, F, CH = X.shape
    Y = np.zeros((T, CH * F), np.float32)
    lib().or_flatten_cf(_ptr(X), _ptr(Y), T, F, CH)
    return Y


def lstm_cell(gates, c_in):
    H = c_in.size
    c_out, h_out = np.zeros(H, np.float32), np.zeros(H, np.float32)
    lib().or_lstm_cell(_ptr(np.ascontiguousarray(gates, np.float32)), _ptr(np.ascontiguousarray(c_in, np.float32)),
                       _ptr(c_out), _ptr(h_out), H)
    return c_out, h_out


def joint_argmax(enc, pred, W, bias):
    enc = np.ascontiguousarray(enc, np.float32)
    rows, H = enc.shape
    V = W.shape[0]
    idx = np.zeros(rows, np.int32)
    val = np.zeros(rows, np.float32)
    mar = np.zeros(rows, np.float32)
    lib().or_joint_argmax(_ptr(enc), H, _ptr(np.ascontiguousarray(pred, np.float32)), _ptr(np.ascontiguousarray(W, np.uint16), u16p),
                          _ptr(np.ascontiguousarray(bias, np.float32)), V, H, rows, _ptr(idx, i32p), _ptr(val), _ptr(mar))
    return idx, val, mar


def num_threads():
    return lib().or_num_threads()


# ---------------------------------------------------------------------------------------------
# the benchmark's synthetic workload, generated without the product library (oracle_synth.c)

class SynthSpec(C.Structure):  # or_synth_spec_t (the layout of nemoasr_synth_spec_t)
    _fields_ = [("seed", C.c_uint64), ("n_layers", C.c_int), ("d_model", C.c_int), ("ff_factor", C.c_int),
                ("sub_channels", C.c_int), ("num_prompts", C.c_int), ("prompt_hidden", C.c_int),
                ("pred_hidden", C.c_int), ("joint_hidden", C.c_int), ("vocab_size", C.c_int), ("att_left", C.c_int),
                ("weight_std", C.c_float), ("blank_bias", C.c_float)]


def synth_default(**kw):
    s = SynthSpec()
    lib().or_synth_default(C.byref(s))
    for k, v in kw.items():
        setattr(s, k, v)
    return s


def synth_write(d, spec):
    L = lib()
    L.or_synth_write.argtypes = [C.c_char_p, C.POINTER(SynthSpec), C.c_char_p, C.c_size_t]
    err = C.create_string_buffer(512)
    if L.or_synth_write(d.encode(), C.byref(spec), err, 512):
        raise RuntimeError(err.value.decode())
    return d


def synth_audio(seed, rate, seconds=None, n=None, pauses=False):
    L = lib()
    L.or_synth_audio.argtypes = [C.c_uint64, C.c_int, C.c_size_t, C.c_int, f32p]
    n = int(round(seconds * rate)) if n is None else n
    out = np.zeros(n, np.float32)
    L.or_synth_audio(seed, rate, n, int(pauses), _ptr(out))
    return out


# ---------------------------------------------------------------------------------------------
# the reference's own host code on CPU (built only where the reference sources are present)

def ref_available():
    return os.path.exists(REF_PATH)


def ref():
    global _ref
    if _ref is None:
        R = C.CDLL(REF_PATH)
        R.nemoasr_open.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
        R.nemoasr_open.restype = C.c_void_p
        R.nemoasr_feed.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
        R.nemoasr_feed.restype = C.c_void_p
        R.nemoasr_free.argtypes = [C.c_void_p]
        R.nemoasr_close.argtypes = [C.c_void_p]
        R.model_load.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
        R.model_load.restype = C.c_void_p
        R.model_set_language.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_size_t]
        R.model_free.argtypes = [C.c_void_p]
        R.encoder_create.argtypes = [C.c_void_p, C.c_int]
        R.encoder_create.restype = C.c_void_p
        R.encoder_destroy.argtypes = [C.c_void_p]
        R.encoder_push.argtypes = [C.c_void_p, f32p, C.c_size_t]
        R.encoder_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]
        R.decoder_create.argtypes = [C.c_void_p]
        R.decoder_create.restype = C.c_void_p
        R.decoder_destroy.argtypes = [C.c_void_p]
        R.decoder_run.argtypes = [C.c_void_p, C.c_void_p, C.c_int, i32p, C.c_int, C.c_char_p, C.c_size_t]
        R.gpu_buf_ptr.argtypes = [C.c_void_p]
        R.gpu_buf_ptr.restype = C.c_void_p
        R.mel_create.restype = C.c_void_p
        R.mel_destroy.argtypes = [C.c_void_p]
        R.mel_push.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, C.POINTER(f32p), C.POINTER(C.c_size_t)]
        R.resampler_create.argtypes = [C.c_int, C.c_int]
        R.resampler_create.restype = C.c_void_p
        R.resampler_destroy.argtypes = [C.c_void_p]
        R.resampler_process.argtypes = [C.c_void_p, f32p, C.c_size_t, f32p, C.c_size_t]
        R.resampler_process.restype = C.c_size_t
        R.resampler_flush.argtypes = [C.c_void_p, f32p, C.c_size_t]
        R.resampler_flush.restype = C.c_size_t
        _ref = R
    return _ref


class _EncOut(C.Structure):  # src/encoder.h:9-14
    _fields_ = [("frames", C.c_int), ("prompted", C.c_void_p), ("joint_enc", C.c_void_p), ("gpu_ms", C.c_double), ("wall_ms", C.c_double)]


def ref_run_stream(ckpt_dir, audio, latency_ms, language="auto", block=1600):
    """Run the reference's own encoder_step / decoder_run loop (src/nemoasr.c:112-160 with the
    mel front end, 16 kHz input) and return per-row encoder outputs and tokens."""
    R = ref()
    err = C.create_string_buffer(512)
    m = R.model_load(ckpt_dir.encode(), err, 512)
    if not m:
        raise RuntimeError(err.value.decode())
    if R.model_set_language(m, language.encode(), err, 512):
        raise RuntimeError(err.value.decode())
    right = {80: 0, 160: 1, 320: 3, 560: 6, 1120: 13}[latency_ms]
    e, d, ms = R.encoder_create(m, right), R.decoder_create(m), R.mel_create()
    cfg = json.load(open(os.path.join(ckpt_dir, "config.json")))
    D, JH = cfg["encoder"]["d_model"], cfg["joint"]["joint_hidden"]
    prompted, joint, rows, toks = [], [], [], []
    audio = np.ascontiguousarray(audio, np.float32)
    nblk = max(1, (len(audio) + block - 1) // block)
    tokbuf = np.zeros(4096, np.int32)
    for i in range(nblk):
        x = audio[i * block:(i + 1) * block]
        final = int(i == nblk - 1)
        fr, nf = f32p(), C.c_size_t()
        R.mel_push(ms, _ptr(x), x.size, final, C.byref(fr), C.byref(nf))
        if nf.value:
            R.encoder_push(e, fr, nf.value)
        out = _EncOut()
        while True:
            rc = R.encoder_step(e, final, C.byref(out), err, 512)
            if rc < 0:
                raise RuntimeError(err.value.decode())
            if rc != 1:
                break
            if out.frames <= 0:
                continue
            pp = np.ctypeslib.as_array(C.cast(R.gpu_buf_ptr(out.prompted), f32p), shape=(out.frames * D,))
            jj = np.ctypeslib.as_array(C.cast(R.gpu_buf_ptr(out.joint_enc), f32p), shape=(out.frames * JH,))
            prompted.append(pp.reshape(out.frames, D).copy())
            joint.append(jj.reshape(out.frames, JH).copy())
            rows.append(out.frames)
            n = R.decoder_run(d, out.joint_enc, out.frames, _ptr(tokbuf, i32p), 4096, err, 512)
            if n < 0:
                raise RuntimeError(err.value.decode())
            toks += tokbuf[:n].tolist()
    R.mel_destroy(ms)
    R.decoder_destroy(d)
    R.encoder_destroy(e)
    R.model_free(m)
    cat = lambda xs, w: np.concatenate(xs) if xs else np.zeros((0, w), np.float32)
    return dict(prompted=cat(prompted, D), joint=cat(joint, JH), chunk_rows=np.array(rows, np.int32), tokens=toks)


def ref_feed_text(ckpt_dir, audio, rate, latency_ms, language="auto", block=None):
    """The reference's public API end to end (src/nemoasr.h): returns the concatenated text."""
    R = ref()
    err = C.create_string_buffer(512)
    s = R.nemoasr_open(ckpt_dir.encode(), language.encode(), latency_ms, rate, err, 512)
    if not s:
        raise RuntimeError(err.value.decode())
    audio = np.ascontiguousarray(audio, np.float32)
    block = block or rate // 10
    text = b""
    for p in range(0, len(audio), block):
        x = audio[p:p + block]
        t = R.nemoasr_feed(s, _ptr(x), x.size, int(p + block >= len(audio)), err, 512)
        if err.value:
            raise RuntimeError(err.value.decode())
        if t:
            text += C.string_at(t)
            R.nemoasr_free(t)
    R.nemoasr_close(s)
    return text.decode()


def ref_mel(samples, blocks=None):
    R = ref()
    m = R.mel_create()
    samples = np.ascontiguousarray(samples, np.float32)
    blocks = blocks or [len(samples)]
    out, p = [], 0
    for i, b in enumerate(blocks):
        x = samples[p:p + b]
        p += b
        fr, nf = f32p(), C.c_size_t()
        R.mel_push(m, _ptr(x), x.size, int(i == len(blocks) - 1), C.byref(fr), C.byref(nf))
        if nf.value:
            out.append(np.ctypeslib.as_array(fr, shape=(nf.value * 128,)).reshape(-1, 128).copy())
    R.mel_destroy(m)
    return np.concatenate(out) if out else np.zeros((0, 128), np.float32)


def ref_resample(samples, in_rate, out_rate, block=None):
    R = ref()
    r = R.resampler_create(in_rate, out_rate)
    samples = np.ascontiguousarray(samples, np.float32)
    block = block or len(samples)
    out = []
    for p in range(0, len(samples), block):
        x = samples[p:p + block]
        cap = int(len(x) * out_rate / in_rate) + 4096
        buf = np.zeros(cap, np.float32)
        n = R.resampler_process(r, _ptr(x), x.size, _ptr(buf), cap)
        out.append(buf[:n])
    buf = np.zeros(8192, np.float32)
    n = R.resampler_flush(r, _ptr(buf), buf.size)
    out.append(buf[:n])
    R.resampler_destroy(r)
    return np.concatenate(out)
