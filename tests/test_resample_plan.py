"""Host half of the GPU resampler: nb_resampler_plan / nb_resampler_commit hand the GPU the same
outputs that process (+ flush) computes on the host, which is bit-exact with the reference's
src/resample.c (test_oracle_golden.py). Checked on the CPU: the output counts of every feed
call, and the sums of src/resample.c:52-71 evaluated in numpy over the planned window (the
inputs the kernel sees) against the host's outputs."""
import ctypes as C

import numpy as np
import pytest

import nemoasr_b200 as nb

f32p = C.POINTER(C.c_float)


class Job(C.Structure):
    _fields_ = [("win", C.c_void_p), ("start", C.c_longlong), ("len", C.c_size_t), ("nin", C.c_ulonglong), ("out0", C.c_ulonglong),
                ("count", C.c_size_t), ("in_rate", C.c_int), ("out_rate", C.c_int)]


def lib():
    L = nb.api()
    L.nb_resampler_create.argtypes = [C.c_int, C.c_int]
    L.nb_resampler_create.restype = C.c_void_p
    L.nb_resampler_destroy.argtypes = [C.c_void_p]
    L.nb_resampler_plan.argtypes = [C.c_void_p, f32p, C.c_size_t, C.c_int, C.POINTER(Job)]
    L.nb_resampler_commit.argtypes = [C.c_void_p, C.c_size_t]
    return L


def sums(job):
    """Outputs [out0, out0 + count) of the planned job: the kernel's formula in numpy."""
    ratio = job.in_rate / job.out_rate
    half = 16.0 * max(ratio, 1.0)
    fc2 = min(1.0, 1.0 / ratio)
    win = np.ctypeslib.as_array(C.cast(job.win, f32p), shape=(job.len,)).astype(np.float64) if job.len else np.zeros(0)
    out = np.zeros(job.count, np.float32)
    for q in range(job.count):
        t = float(job.out0 + q) * ratio
        a, b = int(np.ceil(t - half)), int(np.floor(t + half))
        i = np.arange(a, b + 1)
        u = i.astype(np.float64) - t
        x = u / half
        bl = 0.42 + 0.5 * np.cos(np.pi * x) + 0.08 * np.cos(2.0 * np.pi * x)
        ang = np.pi * fc2 * u
        with np.errstate(invalid="ignore", divide="ignore"):
            sinc = np.where(np.abs(ang) < 1e-9, 1.0, np.sin(ang) / ang)
        h = np.where((x <= -1.0) | (x >= 1.0), 0.0, fc2 * sinc * bl)
        ok = (i >= 0) & (i < job.nin) & (i >= job.start) & (i < job.start + job.len)
        xs = np.where(ok, win[np.clip(i - job.start, 0, max(job.len - 1, 0))] if job.len else 0.0, 0.0)
        ws = h.sum()
        out[q] = np.float32(np.dot(h, xs) / ws) if ws > 0 else 0.0
    return out


@pytest.mark.parametrize("rate", [48000, 44100, 22050, 8000, 96000])
def test_plan_commit_reproduces_process_flush(rate):
    L = lib()
    audio = nb.synth_audio(7, rate, seconds=0.4, pauses=True)
    rng = np.random.default_rng(rate)
    cuts = np.sort(rng.choice(np.arange(1, len(audio)), size=5, replace=False))
    blocks = np.split(audio, cuts)
    blocks.insert(2, audio[:0])  # an empty feed in the middle
    ref = nb.resample(audio, rate, 16000, block=None)  # one process + flush
    host = []
    r_host = L.nemoasr_resampler_create(rate, 16000)
    r_plan = L.nb_resampler_create(rate, 16000)
    got = []
    for k, x in enumerate(blocks):
        final = k == len(blocks) - 1
        x = np.ascontiguousarray(x, np.float32)
        cap = len(x) + 8192
        buf = np.zeros(cap, np.float32)
        n = L.nemoasr_resampler_process(r_host, x.ctypes.data_as(f32p), x.size, buf.ctypes.data_as(f32p), cap) if x.size else 0
        if final:
            n += L.nemoasr_resampler_flush(r_host, buf[n:].ctypes.data_as(f32p), cap - n)
        host.append(buf[:n].copy())
        job = Job()
        L.nb_resampler_plan(r_plan, x.ctypes.data_as(f32p), x.size, int(final), C.byref(job))
        assert job.count == n, f"block {k}: planned {job.count} outputs, host produced {n}"
        assert job.start + job.len == job.nin
        got.append(sums(job))
        L.nb_resampler_commit(r_plan, job.count)
    L.nemoasr_resampler_destroy(r_host)
    L.nb_resampler_destroy(r_plan)
    host = np.concatenate(host)
    got = np.concatenate(got)
    np.testing.assert_array_equal(host, ref)
    assert got.shape == host.shape
    assert np.max(np.abs(got - host)) <= 1e-6


def test_plan_final_only_short_input():
    """A stream shorter than the kernel's half width, fed once with final=1: like the host (and
    the reference), outputs before the first that starts inside the input are not produced."""
    L = lib()
    x = np.ascontiguousarray(nb.synth_audio(3, 48000, seconds=0.0005), np.float32)
    r = L.nb_resampler_create(48000, 16000)
    job = Job()
    L.nb_resampler_plan(r, x.ctypes.data_as(f32p), x.size, 1, C.byref(job))
    h = L.nemoasr_resampler_create(48000, 16000)
    buf = np.zeros(8192, np.float32)
    n = L.nemoasr_resampler_process(h, x.ctypes.data_as(f32p), x.size, buf.ctypes.data_as(f32p), buf.size)
    n += L.nemoasr_resampler_flush(h, buf[n:].ctypes.data_as(f32p), buf.size - n)
    assert job.count == n
    L.nb_resampler_destroy(r)
    L.nemoasr_resampler_destroy(h)


def test_plan_counts_match_host_across_rates():
    """Output counts of planned feeds against the host's process + flush, for down- and
    upsampling rates (including ones that share no factor with 16 kHz), random splits, with and
    without a final call."""
    L = lib()
    rng = np.random.default_rng(11)
    for trial in range(60):
        rate = int(rng.choice([7999, 8000, 11025, 12345, 22050, 44100, 48000, 96000, 15999, 16001]))
        n = int(rng.integers(0, 20000))
        x = rng.standard_normal(n).astype(np.float32)
        pieces = np.split(x, np.sort(rng.integers(0, n + 1, size=int(rng.integers(0, 6))))) if n else [x]
        final = bool(rng.integers(0, 2))
        rh, rp = L.nemoasr_resampler_create(rate, 16000), L.nb_resampler_create(rate, 16000)
        for i, p in enumerate(pieces):
            last = final and i == len(pieces) - 1
            p = np.ascontiguousarray(p, np.float32)
            cap = int(p.size * 16000 / rate) + 8192
            buf = np.zeros(cap, np.float32)
            c = L.nemoasr_resampler_process(rh, p.ctypes.data_as(f32p), p.size, buf.ctypes.data_as(f32p), cap) if p.size else 0
            if last:
                c += L.nemoasr_resampler_flush(rh, buf[c:].ctypes.data_as(f32p), cap - c)
            job = Job()
            L.nb_resampler_plan(rp, p.ctypes.data_as(f32p), p.size, int(last), C.byref(job))
            assert job.count == c, f"rate {rate}, {n} samples, piece {i}: planned {job.count}, host {c}"
            L.nb_resampler_commit(rp, job.count)
        L.nemoasr_resampler_destroy(rh)
        L.nb_resampler_destroy(rp)
