"""Host staging of the GPU log-mel (nb_mel_stage): the span handed to the GPU for each call holds
the pre-emphasised samples its new frames read, reflected at the stream edges, as src/mel.c
defines them (pre-emphasis x[i] - 0.97 x[i-1] with the first sample kept, centred 512-sample
frames every 160 samples, reflection without repeating the edge sample). Checked bit-exactly on
the CPU against a numpy restatement, for feeds split at random points, with and without a final
call."""
import ctypes as C

import numpy as np
import pytest

import nemoasr_b200 as nb

f32p = C.POINTER(C.c_float)
HOP, NFFT = 160, 512


def lib():
    L = nb.api()
    L.nb_mel_create.restype = C.c_void_p
    L.nb_mel_destroy.argtypes = [C.c_void_p]
    L.nb_mel_stage.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, f32p, C.c_size_t]
    L.nb_mel_stage.restype = C.c_size_t
    return L


def preemph(x):
    """y[0] = x[0], y[i] = x[i] - 0.97f * x[i-1] rounded once (a fused multiply-add): the product
    of two floats is exact in double precision; the difference is exact there for these samples
    (similar magnitudes) and is rounded once to float."""
    x = np.asarray(x, np.float32)
    y = x.copy()
    y[1:] = (x[1:].astype(np.float64) - np.float64(np.float32(0.97)) * x[:-1].astype(np.float64)).astype(np.float32)
    return y


def expected_span(y, N, t0, count):
    g = np.arange(t0 * HOP - NFFT // 2, t0 * HOP - NFFT // 2 + (count - 1) * HOP + NFFT)
    g = np.where(g < 0, -g, g)
    g = np.where(g >= N, 2 * N - 2 - g, g)
    ok = (g >= 0) & (g < N)
    return np.where(ok, y[np.clip(g, 0, max(N - 1, 0))], np.float32(0)).astype(np.float32)


@pytest.mark.parametrize("seed,final", [(1, True), (2, True), (3, False), (4, True)])
def test_staged_spans_match_restatement(seed, final):
    L = lib()
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(int(16000 * 2.3)) * 0.1 + 0.3 * np.sin(np.arange(int(16000 * 2.3)) * 0.01)).astype(np.float32)
    cuts = np.sort(rng.choice(np.arange(1, len(x)), size=9, replace=False))
    pieces = np.split(x, cuts)
    pieces.insert(3, x[:0])
    if seed == 4:
        pieces = [x[:100], x[100:300]] + [x[300:]]  # the first frames reflect at the start
    y = preemph(x)
    m = lib().nb_mel_create()
    span = np.zeros(1 << 20, np.float32)
    t0, seen = 0, 0
    for k, p in enumerate(pieces):
        last = final and k == len(pieces) - 1
        p = np.ascontiguousarray(p)
        seen += len(p)
        n = L.nb_mel_stage(m, p.ctypes.data_as(f32p), p.size, int(last), span.ctypes.data_as(f32p), span.size)
        assert n != C.c_size_t(-1).value
        if n:
            want = expected_span(y[:seen], seen, t0, n)
            np.testing.assert_array_equal(span[:len(want)], want, err_msg=f"piece {k}")
        t0 += n
    L.nb_mel_destroy(m)
    # every frame of the stream was staged exactly once: centred frames, one per hop
    assert t0 == (len(x) // HOP + 1 if final else (len(x) - NFFT // 2) // HOP + 1)


def test_short_final_stream_reflects_both_edges():
    """A stream shorter than one frame: every sample of its only frames reflects."""
    L = lib()
    x = np.ascontiguousarray((np.random.default_rng(9).standard_normal(300) * 0.1).astype(np.float32))
    m = L.nb_mel_create()
    span = np.zeros(1 << 16, np.float32)
    n = L.nb_mel_stage(m, x.ctypes.data_as(f32p), x.size, 1, span.ctypes.data_as(f32p), span.size)
    L.nb_mel_destroy(m)
    assert n == 300 // HOP + 1
    want = expected_span(preemph(x), 300, 0, n)
    np.testing.assert_array_equal(span[:len(want)], want)
