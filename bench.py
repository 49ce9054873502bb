"""Throughput benchmark: batched streaming ASR (encoder chunk step + greedy RNNT) on B200s.

Workload (BASELINE config #4): 256 independent streams per GPU at 560 ms latency, 30 s of seeded
synthetic audio each (three 100->4000 Hz chirps + noise, random 200-600 ms pauses, per-stream
seed), a random language prompt per stream among 128, full Nemotron-ASR-streaming-0.6B shape
with random-init bf16 weights (the checkpoint is not used). One step = one 560 ms chunk of every
stream: subsampling, 24 conformer blocks, prompt, joint projection and the greedy decode.

  value : audio-sec/sec over all GPUs with the log-mel features already in HBM (CUDA-event time
          on the engine's stream, max over ranks);
  e2e   : the same metric through the public API (nemoasr_batch_feed) from host audio: host
          pre-emphasis and frame bookkeeping, H2D sample spans, GPU log-mel and the step, D2H token
          reads inside the timed region.

Streams shard across GPUs with no collective (one process per GPU); torch.distributed is used
only for the start barrier and the max-over-ranks of the timings. Under torchrun every rank gets
an equal share of the host's cores for its OpenMP and thread-pool work.

The same line carries the other BASELINE configs measured in the run: `single_stream` (config
#1: one stream, 4.0 s, 560 ms chunks), `config5` (1024 streams per GPU at 1120 ms with the blank
bias calibrated for ~35 % emitting frames); `--sweep` prints config #2 (the GEMM sweep) and
`--session48k` config #3, one line each.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nemo-c_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def host_threads():
    """Host threads this rank may use: all cores alone, an equal share under torchrun."""
    per_node = max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
    return max(1, (os.cpu_count() or 8) // per_node)


# OpenMP in the product library and the oracle reads this when the library loads
if int(os.environ.get("LOCAL_WORLD_SIZE", "1")) > 1:
    os.environ["OMP_NUM_THREADS"] = str(host_threads())

METRIC = "audio-sec/sec (RTFx) at N streams on 1/2/4/8 B200"
# DRAM bytes of one FF-in launch at 1792 rows (8.39 MB weights + 7.34 MB activation planes
# algorithmic), measured by ncu on the 208-row tiles: 15,807,232 B read + 4,096 B written
FFIN_TRAFFIC = 15811328
UNIT = "audio-sec/sec"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--streams", type=int, default=256)
    ap.add_argument("--latency", type=int, default=560)
    ap.add_argument("--seconds", type=float, default=30.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-single", action="store_true", help="skip the single-stream (config #1) chunk latency")
    ap.add_argument("--kernel-only", action="store_true", help="time only the dominant GEMM (small device footprint, for ncu captures)")
    ap.add_argument("--attention-only", action="store_true", help="time only the attention launch at the step's shape (1.6 GB on the device, for ncu captures)")
    ap.add_argument("--session48k", type=float, default=0, metavar="SECONDS",
                    help="BASELINE config #3 only: one stream, 80 ms chunks, SECONDS of 48 kHz audio through the public API, GPU vs host resampler")
    ap.add_argument("--resample-only", type=int, default=0, metavar="RATE",
                    help="time only the GPU resampler: one chunk of every stream arriving at RATE Hz (small device footprint, for ncu captures)")
    ap.add_argument("--no-config5", action="store_true", help="skip the nested BASELINE config #5 measurement")
    ap.add_argument("--single-only", action="store_true", help="BASELINE config #1 only: one stream, 560 ms chunks, 4.0 s (small device footprint, for ncu captures)")
    ap.add_argument("--config5-streams", type=int, default=1024)
    ap.add_argument("--config5-steps", type=int, default=5)
    ap.add_argument("--sweep", action="store_true", help="BASELINE config #2 only: the GEMM sweep, one JSON line per case")
    ap.add_argument("--calibrate", action="store_true", help="find the config #5 blank bias (~35 %% of stream-frames emit) and print it")
    return ap.parse_args()


def config_dict(a, world):
    return {"workload": f"BASELINE config #4: {a.streams} streams/GPU, {a.latency} ms chunks, {a.seconds:g} s synthetic audio per stream",
            "streams_per_gpu": a.streams, "latency_ms": a.latency, "audio_s_per_stream": a.seconds, "parallelism": f"streams sharded over {world} GPU(s), no collective",
            "l2": "inputs > L2: 1.2 GB of weights streamed per step (126 MB L2)", "model": "nemotron-asr-streaming-0.6b shape, random-init bf16"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index):
        self.index, self.lines, self.p = index, [], None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "-i", str(self.index), "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=lambda: [self.lines.append(l.strip()) for l in self.p.stdout], daemon=True).start()
            # nvidia-smi takes a moment to print its first line: wait for it (bounded) so that the
            # samples from here on fall into the timed region, which may last only ~0.1 s
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0 and self.p.poll() is None:
                time.sleep(0.01)
            self.n0 = len(self.lines)
        except OSError:
            self.p = None

    def stop(self):
        if self.p:
            # at least one sample taken after the timed region began (bounded wait)
            t0 = time.time()
            while len(self.lines) <= getattr(self, "n0", 0) and time.time() - t0 < 1.0 and self.p.poll() is None:
                time.sleep(0.01)
            self.lines = self.lines[getattr(self, "n0", 0):] or self.lines
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        rows = []
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) >= 8:
                try:
                    rows.append((float(f[0]), float(f[1]), f[4:8]))
                except ValueError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, fl in rows for i, v in enumerate(fl) if v.lower() == "active"})
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons, "samples": len(rows)}


def make_inputs(nb, a, rank):
    """Per-stream audio (host) and its log-mel features, generated in parallel threads."""
    from concurrent.futures import ThreadPoolExecutor
    n = int(round(a.seconds * 16000))
    audio = np.zeros((a.streams, n), np.float32)
    seeds = stream_seeds(a, rank)
    with ThreadPoolExecutor(min(32, host_threads())) as ex:
        for s, x in enumerate(ex.map(lambda sd: nb.synth_audio(sd, 16000, n=n, pauses=True), seeds)):
            audio[s] = x
        mels = list(ex.map(lambda s: nb.mel(audio[s]), range(a.streams)))
    T = min(m.shape[0] for m in mels)
    mel = np.stack([m[:T] for m in mels])
    return audio, mel


def stream_seeds(a, rank):
    """Audio seeds of this rank's streams: every rank owns a disjoint set of streams (weak scaling;
    nothing is exchanged between ranks)."""
    return [100000 * (rank + 1) + s for s in range(a.streams)]


def max_over_ranks(dist, x, device):
    """Max of a host float over ranks (the step time of the slowest GPU); x itself when alone."""
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def languages(a, rank):
    rng = np.random.default_rng(777 + rank)
    keys = ["auto", "en-US"] + [f"lang{i}" for i in range(2, 128)]
    return [keys[i] for i in rng.integers(0, 128, size=a.streams)]


def dominant_gemm(nb, torch, a, B, c):
    """CUDA-event time of the FF-in GEMM of one step (M = streams x rows, N = 4096, K = 1024),
    launched through the C-ABI on a torch stream, averaged over 20 launches of 24 distinct weights
    (more than L2 holds)."""
    import ctypes as C
    M, N, K = B * c, 4096, 1024
    A = torch.randn(2 * M, K, device="cuda", dtype=torch.float32).to(torch.bfloat16)  # hi and lo planes
    Ws = [torch.randint(0, 1 << 15, (N, K), device="cuda", dtype=torch.int16) & 0x3C7F for _ in range(24)]
    Cm = torch.empty(M, N, device="cuda", dtype=torch.float32)
    args = nb.GemmArgs()
    args.A, args.lda, args.a_fmt, args.a_plane = A.data_ptr(), K, 1, M * K
    args.ldw, args.C, args.ldc, args.M, args.N, args.K, args.act, args.alpha = K, Cm.data_ptr(), N, M, N, K, 1, 1.0
    st = torch.cuda.current_stream()
    for w in Ws[:3]:
        args.W = w.data_ptr()
        nb.check(nb.api().nemo_gemm(C.byref(args), C.c_void_p(st.cuda_stream)))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(20):
        args.W = Ws[i % 24].data_ptr()
        nb.check(nb.api().nemo_gemm(C.byref(args), C.c_void_p(st.cuda_stream)))
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    return ms, 2.0 * M * N * K


def attention_kernel(nb, torch, peaks, B, c):
    """CUDA-event time of one nemo_attention_rel launch at the step's shape (B streams, c rows,
    full cache of att_left rows, the synthetic model's window bound att_left + 16), averaged over
    40 launches that rotate over 4 K/V caches (1.6 GB: the window rows come from HBM, as in the
    step), with the HBM bytes it must move: the window's K and V rows of every head plus the
    query rows and the output."""
    import ctypes as C
    H, D, dh = 8, 1024, 128
    left = nb.synth_default().att_left
    Lmax, L, cap = left + 16, left + c, 128
    pos = left + 8
    kvs = [torch.randn(B, cap, 3 * D, device="cuda") for _ in range(4)]
    P = torch.randn(2 * Lmax - 1, D, device="cuda")
    bu, bv = torch.randn(D, device="cuda") * 0.1, torch.randn(D, device="cuda") * 0.1
    dpos, dcl = torch.tensor([pos], dtype=torch.int32, device="cuda"), torch.tensor([left], dtype=torch.int32, device="cuda")
    O = torch.empty(B * c, D, device="cuda")
    st = torch.cuda.current_stream()
    f = nb.api().nemo_attention_rel
    f.restype = C.c_int

    def run(kv):
        b = kv.data_ptr()
        nb.check(f(C.c_void_p(b), C.c_int64(3 * D), C.c_int64(cap * 3 * D), C.c_void_p(b + 4 * D), C.c_void_p(b + 8 * D), C.c_int64(3 * D),
                   C.c_int64(cap * 3 * D), C.c_void_p(dpos.data_ptr()), C.c_void_p(dcl.data_ptr()), C.c_void_p(P.data_ptr()), C.c_void_p(bu.data_ptr()),
                   C.c_void_p(bv.data_ptr()), C.c_void_p(O.data_ptr()), 0, C.c_int64(0), C.c_int64(c * D), B, c, Lmax, H, dh, D,
                   C.c_float(dh ** -0.5), C.c_void_p(st.cuda_stream)))
    for i in range(4):
        run(kvs[i])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(40):
        run(kvs[i % 4])
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / 40 * 1e3
    nbytes = B * (2 * L * D + 2 * c * D) * 4
    peak = peaks.get("hbm_gbs", 6650.0)
    del kvs
    return {"kernel": "nemo_attention_rel (streams=%d, rows=%d, keys=%d, heads=%d)" % (B, c, L, H), "us_per_launch": us, "hbm_bytes": nbytes,
            "achieved_gbs": nbytes / (us * 1e-6) / 1e9, "peak_gbs": peak, "frac": nbytes / (us * 1e-6) / 1e9 / peak}


def resample_kernel(nb, torch, a, rate):
    """CUDA-event time of nemo_resample over one chunk of every stream (the outputs of one
    latency-long chunk, from the inputs they reach), averaged over 20 launches; beside it the
    host resampler's time for the same chunk of one stream on one thread."""
    import ctypes as C
    L = nb.api()
    L.nemo_resample.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int64,
                                C.c_int, C.c_void_p]
    B, count = a.streams, a.latency * 16
    ratio = rate / 16000
    out0 = 1000
    start = int(np.ceil(out0 * ratio - 16.0 * max(ratio, 1.0)))
    nin = int(np.floor((out0 + count - 1) * ratio + 16.0 * max(ratio, 1.0))) + 1
    x = torch.randn(B, nin - start, device="cuda") * 0.1
    y = torch.empty(B, count, device="cuda")
    st = torch.cuda.current_stream()

    def run():
        if L.nemo_resample(x.data_ptr(), nin - start, start, nin - start, nin, out0, count, rate, 16000, y.data_ptr(), count, B, st.cuda_stream):
            raise RuntimeError(L.nemo_gpu_last_error().decode())
    for _ in range(3):
        run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(20):
        run()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    audio = np.ascontiguousarray(nb.synth_audio(1, rate, seconds=a.latency / 1000 * 4), np.float32)
    t0 = time.perf_counter()
    nb.resample(audio, rate, 16000, block=rate * a.latency // 1000)
    host_ms = (time.perf_counter() - t0) / 4 * 1e3
    return {"kernel": "nemo_resample", "rate": rate, "streams": B, "outputs_per_stream": count, "inputs_per_stream": nin - start, "us": ms * 1e3,
            "outputs_per_s": B * count / (ms / 1e3), "host_ms_per_stream_chunk_1_thread": host_ms}


def session_48k(nb, seconds, latency=80, rate=48000, peaks=None):
    """BASELINE config #3: one stream of the full model, 80 ms chunks, 48 kHz audio resampled
    internally, fed in 80 ms blocks through the public API (nemoasr_feed_tokens), host buffers in,
    tokens out. Per chunk (one graph launch of the step: encoder graph + persistent decoder) the
    device time from the engine's CUDA events (nemoasr_stats encoder_ms + decoder_ms, read after
    each feed, every steady feed makes exactly one chunk), p50 / p99 and the HBM fraction of its
    1.1765 GB of weights; beside it the wall time of every feed (resampling, log-mel, the step and
    the token read). GPU resampler, then the host resampler (NEMO_GPU_RESAMPLE=0). The session
    first runs nemoasr_prepare_latency, so no chunk captures a graph."""
    import ctypes as C
    peaks = peaks or {}
    audio = nb.synth_audio(3, rate, seconds=seconds, pauses=True)
    s = nb.Session(spec=nb.synth_default(), latency_ms=latency, rate=rate)
    err = C.create_string_buffer(1024)
    if nb.api().nemoasr_prepare_latency(s.h, latency, err, 1024):
        raise RuntimeError(err.value.decode())
    block = rate * latency // 1000
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = {}
    old = os.environ.get("NEMO_GPU_RESAMPLE")
    try:
        for mode in ("warm-up", "gpu", "host"):
            os.environ["NEMO_GPU_RESAMPLE"] = "0" if mode == "host" else "1"
            s.reset(latency_ms=latency)
            x = audio[: 2 * rate] if mode == "warm-up" else audio
            ts, dev, toks, c0 = [], [], 0, s.stats()["chunks"]  # stats run on across resets
            t_all = time.perf_counter()
            for q in range(0, len(x), block):
                st0 = s.stats()
                t0 = time.perf_counter()
                toks += len(s.feed_tokens(x[q:q + block], final=q + block >= len(x)))
                ts.append(time.perf_counter() - t0)
                st1 = s.stats()
                if st1["chunks"] - st0["chunks"] == 1:
                    dev.append(st1["encoder_ms"] + st1["decoder_ms"] - st0["encoder_ms"] - st0["decoder_ms"])
            wall = time.perf_counter() - t_all
            if mode != "warm-up":
                st = s.stats()
                p50 = float(np.median(dev))
                out[mode] = {"rtfx": len(x) / rate / wall, "p50_feed_ms": float(np.median(ts)) * 1e3, "p99_feed_ms": float(np.percentile(ts, 99)) * 1e3,
                             "p50_chunk_device_ms": p50, "p99_chunk_device_ms": float(np.percentile(dev, 99)), "chunks_timed": len(dev),
                             "hbm_frac_of_measured": 1.1765e9 / (p50 / 1e3) / 1e9 / hbm, "chunks": st["chunks"] - c0, "tokens": toks}
    finally:
        if old is None:
            os.environ.pop("NEMO_GPU_RESAMPLE", None)
        else:
            os.environ["NEMO_GPU_RESAMPLE"] = old
    s.close()
    return {"workload": f"BASELINE config #3: 1 stream, {latency} ms chunks, {seconds:g} s of 48 kHz audio in {latency} ms feeds, public API",
            "gpu_resampler": out["gpu"], "host_resampler": out["host"], "graphs_captured_after_warmup": 0}


def single_stream(nb, torch, peaks, seconds=4.0, latency=560, passes=6):
    """BASELINE config #1: one stream, full model, 560 ms chunks, 4.0 s of audio (7 whole chunks and
    the final one), the mel frames in HBM. The clip runs `passes` times (reset between); the first
    pass captures the graphs and is not counted. Per-chunk device time from CUDA events around
    each chunk's step; HBM fraction = the chunk's 1.1765 GB of encoder weights / p50 / measured
    copy bandwidth."""
    b = nb.Batch(1, spec=nb.synth_default(), latency_ms=latency)
    mel = nb.mel(nb.synth_audio(1, 16000, seconds=seconds))[None]
    d = torch.from_numpy(np.ascontiguousarray(mel)).cuda()
    ts, enc, dec = [], [], []
    for p in range(passes):
        b.reset()
        b.attach_mel(d.data_ptr(), mel.shape[1] * 128, mel.shape[1])
        while True:
            st0, g0 = b.stats(), b.gpu_ms()
            rc, rows, _ = b.step(final=True)
            if rc != 1:
                break
            if rows and p:
                st1 = b.stats()
                ts.append(b.gpu_ms() - g0)
                enc.append(st1["encoder_ms"] - st0["encoder_ms"])
                dec.append(st1["decoder_ms"] - st0["decoder_ms"])
    b.close()
    ts = np.array(ts)
    p50 = float(np.median(ts))
    hbm = peaks.get("hbm_gbs", 6650.0)
    return {"workload": f"BASELINE config #1: 1 stream, {latency} ms chunks, {seconds:g} s audio ({passes - 1} timed passes), mel in HBM",
            "chunks": int(len(ts)), "p50_chunk_ms": p50, "p99_chunk_ms": float(np.percentile(ts, 99)),
            "p50_encoder_ms": float(np.median(enc)), "p50_decoder_ms": float(np.median(dec)), "weight_bytes_per_chunk": 1.1765e9,
            "achieved_gbs": 1.1765e9 / (p50 / 1e3) / 1e9, "hbm_peak_gbs": hbm, "hbm_frac": 1.1765e9 / (p50 / 1e3) / 1e9 / hbm,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback 6.65 TB/s"}


# Blank-joint-bias offset of the config #5 model: about 35 % of stream-frames emit a token over the
# chunks config #5 times (its 1024 streams, chunks 3..7: per-stream seeds, pauses, random
# languages). Found by `python bench.py --calibrate` (bisection down to adjacent bf16-representable
# offsets): 0.390625 -> 38.4 % of the stream-frames emit; the next offset up (0.3916015625) gives
# 30.1 %. The rate is a steep function of the offset with these random-init weights.
CONFIG5_BLANK_BIAS = 0.390625


def emission(nb, batch, before=None):
    """Emitting fraction of the stream-frames decoded since `before` (decode_counts)."""
    c = batch.decode_counts()
    if before:
        c = {k: c[k] - before[k] for k in c}
    return c


def config5_inputs(nb, B, seconds, rank):
    from concurrent.futures import ThreadPoolExecutor
    n = int(round(seconds * 16000))
    audio = np.zeros((B, n), np.float32)
    seeds = [500000 * (rank + 1) + s for s in range(B)]
    with ThreadPoolExecutor(min(32, host_threads())) as ex:
        for s, x in enumerate(ex.map(lambda sd: nb.synth_audio(sd, 16000, n=n, pauses=True), seeds)):
            audio[s] = x
    rng = np.random.default_rng(9000 + rank)
    keys = ["auto", "en-US"] + [f"lang{i}" for i in range(2, 128)]
    return audio, [keys[i] for i in rng.integers(0, 128, size=B)]


def calibrate(nb, B=1024, latency=1120, warm=2, chunks=5, target=0.35):
    """Bisection on the joint blank bias for `target` emitting stream-frames, counted over the chunks
    config #5 times (chunks warm + 1 .. warm + chunks of its 1024 streams)."""
    blk = latency * 16
    audio, langs = config5_inputs(nb, B, (warm + chunks + 1) * latency / 1000, 0)

    def rate(bias):
        b = nb.Batch(B, spec=nb.synth_default(blank_bias=bias), languages=langs, latency_ms=latency)
        for i in range(warm):
            b.feed(audio[:, i * blk:(i + 1) * blk])
        c0 = b.decode_counts()
        for i in range(warm, warm + chunks):
            b.feed(audio[:, i * blk:(i + 1) * blk])
        c = b.decode_counts()
        b.close()
        r = (c["emitting_frames"] - c0["emitting_frames"]) / (c["frames"] - c0["frames"])
        print(json.dumps({"blank_bias": bias, "emitting_frames": r}), flush=True)
        return r
    # the offset lands in a bf16 bias (steps of ~0.002 near 0.4) and the rate jumps between steps:
    # bisect down to adjacent representable offsets, then keep the one nearer the target
    lo, hi = -2.0, 6.0
    rates = {lo: rate(lo), hi: rate(hi)}
    for _ in range(16):
        mid = 0.5 * (lo + hi)
        rates[mid] = rate(mid)
        if abs(rates[mid] - target) < 0.01:
            lo = hi = mid
            break
        if rates[mid] > target:
            lo = mid
        else:
            hi = mid
        if hi - lo < 1e-3:
            break
    bias = min((lo, hi), key=lambda x: abs(rates[x] - target))
    print(json.dumps({"calibrated_blank_bias": bias, "emitting_frames": rates[bias], "streams": B, "latency_ms": latency,
                      "counted_chunks": [warm + 1, warm + chunks], "neighbours": {str(lo): rates[lo], str(hi): rates[hi]}}), flush=True)


def config5(nb, torch, a, rank, world, dist, barrier):
    """BASELINE config #5: 1024 streams per GPU at 1120 ms (14 rows per stream, 14336 rows per
    GEMM), the blank bias offset so ~35 % of stream-frames emit. Audio through the public batch
    API (GPU log-mel), one 1120 ms feed per step. value = audio-s/s from the engine's device
    time of the timed steps (max over ranks); e2e = the same from wall time of the feeds."""
    B, lat = a.config5_streams, 1120
    blk = lat * 16
    W, K = 2, a.config5_steps
    audio, langs = config5_inputs(nb, B, (W + K + 1) * lat / 1000, rank)
    bias = CONFIG5_BLANK_BIAS if CONFIG5_BLANK_BIAS is not None else nb.synth_default().blank_bias
    b = nb.Batch(B, spec=nb.synth_default(blank_bias=bias), languages=langs, latency_ms=lat)
    for i in range(W):
        b.feed(audio[:, i * blk:(i + 1) * blk])
    torch.cuda.synchronize()
    barrier()
    c0, st0, g0 = b.decode_counts(), b.stats(), b.gpu_ms()
    t0 = time.perf_counter()
    for i in range(W, W + K):
        b.feed(audio[:, i * blk:(i + 1) * blk])
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    st1, gpu_ms = b.stats(), b.gpu_ms() - g0
    c = emission(nb, b, c0)
    b.close()
    gpu_ms_max = max_over_ranks(dist, gpu_ms, "cuda")
    wall_max = max_over_ranks(dist, wall, "cuda")
    enc, dec = st1["encoder_ms"] - st0["encoder_ms"], st1["decoder_ms"] - st0["decoder_ms"]
    audio_s = K * lat / 1000 * B * world
    return {"workload": f"BASELINE config #5: {B} streams/GPU, {lat} ms chunks (timed chunks {W + 1}..{W + K} of each stream's 60 s), "
                        "public batch API with GPU log-mel",
            "value": audio_s / (gpu_ms_max / 1e3), "e2e": audio_s / wall_max, "unit": UNIT, "ms_per_step": gpu_ms_max / K,
            "blank_bias": bias, "blank_bias_source": "CONFIG5_BLANK_BIAS (bench.py --calibrate)" if CONFIG5_BLANK_BIAS is not None else "uncalibrated default",
            "emission_rate": c["emitting_frames"] / max(c["frames"], 1), "tokens_per_frame": (c["decisions"] - c["frames"]) / max(c["frames"], 1),
            "greedy_iterations_per_chunk": c["iterations"] / K, "decoder_share": dec / max(enc + dec, 1e-9),
            "encoder_ms_per_step": enc / K, "decoder_ms_per_step": dec / K}


def cpu_baseline(nb, a, audio0, budget_s=25.0):
    """The oracle (plain-C fp32 restatement, OpenMP) on one stream of this workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    with tempfile.TemporaryDirectory() as d:
        orc.synth_write(d, orc.synth_default())
        m = orc.Model(d)
        secs = 4.0
        t0 = time.time()
        orc.run_stream(m, audio0[: int(secs * 16000)], 16000, a.latency)
        dt = time.time() - t0
        more = min(a.seconds, max(secs, secs * budget_s / max(dt, 1e-3) * 0.5))
        if more > secs:
            t0 = time.time()
            orc.run_stream(m, audio0[: int(more * 16000)], 16000, a.latency)
            dt, secs = time.time() - t0, more
        del m
    return {"value": secs / dt, "unit": UNIT, "cores": orc.num_threads(), "kind": "port",
            "sample": f"1 stream x {secs:.1f} s of the config #4 audio through the oracle (full model, {a.latency} ms chunks)"}


def run_reference(a):
    """The reference's own host C (oracle/_ref/libnemoref.so: src/nemoasr.c, encoder.c, decoder.c,
    ... over the restated CPU kernels), else the oracle port, on one stream of the workload. The
    checkpoint and audio come from the oracle's copy of the workload generator: this process
    loads no product library."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    audio = orc.synth_audio(100001, 16000, seconds=max(a.seconds, (a.warmup + a.steps + 2) * a.latency / 1000))
    block = a.latency * 16
    times = []
    with tempfile.TemporaryDirectory() as d:
        orc.synth_write(d, orc.synth_default())
        if orc.ref_available():
            import ctypes as C
            R = orc.ref()
            err = C.create_string_buffer(512)
            s = R.nemoasr_open(d.encode(), b"auto", a.latency, 16000, err, 512)
            if not s:
                raise RuntimeError(err.value.decode())
            kind = "reference"
            for i in range(a.warmup + a.steps):
                x = np.ascontiguousarray(audio[i * block:(i + 1) * block])
                t0 = time.perf_counter()
                t = R.nemoasr_feed(s, x.ctypes.data_as(orc.f32p), x.size, 0, err, 512)
                dt = time.perf_counter() - t0
                if t:
                    R.nemoasr_free(t)
                if i >= a.warmup:
                    times.append(dt)
            R.nemoasr_close(s)
        else:
            kind = "port"
            m = orc.Model(d)
            sess = orc.Session(m, a.latency, 16000)
            for i in range(a.warmup + a.steps):
                t0 = time.perf_counter()
                sess.feed(audio[i * block:(i + 1) * block])
                if i >= a.warmup:
                    times.append(time.perf_counter() - t0)
            sess.close()
    # each feed of one chunk of audio yields one step
    ms = float(np.mean(times)) * 1000
    val = (a.latency / 1000) / (ms / 1000)
    threads = orc.num_threads()
    loaded = sorted({l.split()[-1] for l in open("/proc/self/maps") if l.rstrip().endswith(".so") and ROOT in l})
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(a, a.gpus),
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": f"1 stream, {a.steps} chunks of {a.latency} ms through the reference's own host C (nemoasr_feed) "
                                       f"with the restated CPU kernels, {threads} threads"},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "libraries_from_repo": [os.path.relpath(x, ROOT) for x in loaded]}
    print(json.dumps(line), flush=True)


SWEEP_M = [1, 2, 4, 7, 14, 16, 56, 112, 448, 1792]
SWEEP_NK = [(3072, 1024), (4096, 1024), (1024, 4096), (2048, 1024), (1024, 1024)]
SWEEP_EPI = {"bias": (0, 0, 1.0), "bias+silu": (1, 0, 1.0), "glu": (3, 0, 1.0), "0.5x_residual_acc": (0, 1, 0.5)}


def sweep(nb, torch, peaks):
    """BASELINE config #2 (tools/kbench.c:162-195): nemo_gemm over M x (N, K) x epilogue, 24
    distinct seeded bf16 weight matrices N(0, 0.02) per shape cycled so the weights stream from
    HBM (24 x N x K x 2 B > 126 MB L2), activations N(0,1) fp32 carried as bf16 hi/lo planes.
    CUDA-event time over 48 launches after 3 warm-up launches. HBM GB/s of the weight bytes for
    M <= 16, TFLOP/s above; each case with M in {1, 7, 16, 112} also checked against the oracle
    GEMM on one weight matrix (max|d| / max|ref| <= 2e-4)."""
    import ctypes as C
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    from parity import rel_err
    L = nb.api()
    st = torch.cuda.current_stream()
    hbm, tc = peaks.get("hbm_gbs", 6650.0), peaks.get("bf16_tflops", 1590.0)
    g = torch.Generator(device="cuda")
    g.manual_seed(2024)
    for N, K in SWEEP_NK:
        Ws = [(torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for _ in range(24)]
        bias = torch.randn(N, device="cuda", generator=g) * 0.1
        for M in SWEEP_M:
            A = torch.randn(M, K, device="cuda", generator=g)
            hi = A.to(torch.bfloat16)
            planes = torch.cat([hi.reshape(-1), (A - hi.float()).to(torch.bfloat16).reshape(-1)])
            for name, (act, acc, alpha) in SWEEP_EPI.items():
                nout = N // 2 if act == 3 else N
                C0 = torch.randn(M, nout, device="cuda", generator=g)
                Cm = C0.clone()
                args = nb.GemmArgs()
                args.A, args.lda, args.a_fmt, args.a_plane = planes.data_ptr(), K, 1, M * K
                args.ldw, args.bias, args.C, args.ldc = K, bias.data_ptr(), Cm.data_ptr(), nout
                args.M, args.N, args.K, args.act, args.accumulate, args.alpha = M, N, K, act, acc, alpha

                def launch(w):
                    args.W = w.data_ptr()
                    nb.check(L.nemo_gemm(C.byref(args), C.c_void_p(st.cuda_stream)), "nemo_gemm")
                ok = None
                if M in (1, 7, 16, 112):
                    Cm.copy_(C0)
                    launch(Ws[0])
                    torch.cuda.synchronize()
                    want = orc.gemm(A.cpu().numpy(), Ws[0].view(torch.int16).cpu().numpy().view(np.uint16), bias.cpu().numpy(), C0=C0.cpu().numpy(),
                                    act=act, accumulate=bool(acc), alpha=alpha)
                    err = rel_err(Cm.cpu().numpy(), want)
                    ok = {"rel_err": err, "pass": bool(err <= 2e-4)}
                for i in range(3):
                    launch(Ws[i])
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record(st)
                for i in range(48):
                    launch(Ws[i % 24])
                e1.record(st)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) / 48 * 1e3
                line = {"config": "BASELINE config #2", "kernel": "nemo_gemm", "M": M, "N": N, "K": K, "epilogue": name, "us": us}
                if M <= 16:
                    gbs = N * K * 2 / (us * 1e-6) / 1e9
                    line.update({"hbm_gbs": gbs, "hbm_frac_of_measured": gbs / hbm})
                else:
                    tf = 2.0 * M * N * K / (us * 1e-6) / 1e12
                    line.update({"tflops": tf, "tensor_frac_of_measured_burst": tf / tc, "issued_mma_factor": 2})
                if ok is not None:
                    line["oracle"] = ok
                print(json.dumps(line), flush=True)
        del Ws


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    if a.kernel_only:
        import torch
        import nemoasr_b200 as nb
        c = a.latency // 80
        ms, flops = dominant_gemm(nb, torch, a, a.streams, c)
        print(json.dumps({"kernel": "nemo_gemm FF-in", "M": a.streams * c, "N": 4096, "K": 1024, "us": ms * 1e3, "tflops": flops / ms / 1e9}))
        return
    if a.attention_only:
        import torch
        import nemoasr_b200 as nb
        print(json.dumps(attention_kernel(nb, torch, peaks, a.streams, a.latency // 80)))
        return
    if a.session48k:
        import torch  # noqa: F401 (CUDA context as in the other modes)
        import nemoasr_b200 as nb
        print(json.dumps(session_48k(nb, a.session48k, peaks=peaks)))
        return
    if a.resample_only:
        import torch
        import nemoasr_b200 as nb
        print(json.dumps(resample_kernel(nb, torch, a, a.resample_only)))
        return
    if a.sweep:
        import torch
        import nemoasr_b200 as nb
        sweep(nb, torch, peaks)
        return
    if a.single_only:
        import torch
        import nemoasr_b200 as nb
        print(json.dumps(single_stream(nb, torch, peaks)))
        return
    if a.calibrate:
        import torch  # noqa: F401
        import nemoasr_b200 as nb
        calibrate(nb)
        return
    a.seconds = max(a.seconds, (a.warmup + a.steps + 3) * a.latency / 1000.0)
    import torch
    import nemoasr_b200 as nb
    rank, world, local = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    audio, mel = make_inputs(nb, a, rank)
    B, T = a.streams, mel.shape[1]
    chunk_s = a.latency / 1000.0
    batch = nb.Batch(B, spec=nb.synth_default(), languages=languages(a, rank), latency_ms=a.latency)

    # ---- value: features resident in HBM --------------------------------------------------
    d_mel = torch.from_numpy(mel).cuda()
    batch.attach_mel(d_mel.data_ptr(), T * 128, T)
    for _ in range(a.warmup):
        batch.step()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    c0, st0 = batch.decode_counts(), batch.stats()
    g0, l0 = batch.gpu_ms(), nb.api().nemo_gpu_launch_count()
    toks = 0
    for _ in range(a.steps):
        rc, rows, out = batch.step()
        if rc != 1 or rows == 0:
            raise RuntimeError("stream ran out of audio inside the timed region")
        toks += sum(len(t) for t in out)
    torch.cuda.synchronize()
    gpu_ms = batch.gpu_ms() - g0
    launches = nb.api().nemo_gpu_launch_count() - l0
    clk = clocks.stop()
    dc, st1 = emission(nb, batch, c0), batch.stats()
    enc_ms, dec_ms = st1["encoder_ms"] - st0["encoder_ms"], st1["decoder_ms"] - st0["decoder_ms"]
    decode = {"emission_rate": dc["emitting_frames"] / max(dc["frames"], 1), "tokens_per_frame": toks / max(dc["frames"], 1),
              "greedy_iterations_per_chunk": dc["iterations"] / a.steps, "decoder_share": dec_ms / max(enc_ms + dec_ms, 1e-9),
              "encoder_ms_per_step": enc_ms / a.steps, "decoder_ms_per_step": dec_ms / a.steps,
              "model_blank_bias": nb.synth_default().blank_bias}
    gpu_ms = max_over_ranks(dist, gpu_ms, "cuda")
    value = a.steps * chunk_s * B * world / (gpu_ms / 1000.0)

    # ---- e2e: host audio through nemoasr_batch_feed -----------------------------------------
    e2e = None
    if not a.no_e2e:
        batch.reset()
        blk = int(a.latency * 16)
        for i in range(a.warmup + 1):
            batch.feed(audio[:, i * blk:(i + 1) * blk])
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for i in range(a.warmup + 1, a.warmup + 1 + a.steps):
            batch.feed(audio[:, i * blk:(i + 1) * blk])
        torch.cuda.synchronize()
        wall = max_over_ranks(dist, time.perf_counter() - t0, "cuda")
        frames = a.latency // 10  # log-mel frames per step and stream
        e2e = {"value": a.steps * chunk_s * B * world / wall, "unit": UNIT,
               "h2d_bytes_per_step": B * ((frames - 1) * 160 + 512) * 4 + 12,
               "d2h_bytes_per_step": B * 4 + B * 16 * 10 * 4,
               "note": "host audio -> host pre-emphasis and frame bookkeeping -> H2D sample spans -> GPU log-mel + step -> D2H tokens, wall clock"}
    batch.close()
    del d_mel

    # ---- dominant kernel roofline ------------------------------------------------------------
    c = a.latency // 80
    ms, flops = dominant_gemm(nb, torch, a, B, c)
    att = attention_kernel(nb, torch, peaks, B, c) if c <= 16 else None
    single = None if a.no_single or rank != 0 else single_stream(nb, torch, peaks)
    cfg5 = None if a.no_config5 else config5(nb, torch, a, rank, world, dist, barrier)
    peak = peaks.get("bf16_tflops", 1590.0)
    ach = flops / (ms / 1e3) / 1e12
    roof = {"bound": "tensor", "kernel": "nemo_gemm FF-in (M=%d N=4096 K=1024, SiLU)" % (B * c), "achieved": ach, "peak": peak, "unit": "TFLOP/s",
            "frac": ach / peak, "traffic": FFIN_TRAFFIC if B * c == 1792 else None,
            "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of this launch shape",
            "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst)" if peaks else "fallback 1.59 PFLOP/s",
            "issued_mma_factor": 2, "note": "each product is issued as two bf16 MMAs (activation hi and lo planes) on the algorithmic FLOPs counted here"}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        cpu = cpu_baseline(nb, a, audio[0])

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": gpu_ms / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "operands": "bf16 weights x bf16 hi/lo activation planes (16 significant bits), fp32 accumulate and fp32 elsewhere",
                "data": "synthetic (seeded chirps + noise + pauses; random-init bf16 weights of the published shape)",
                "config": config_dict(a, world), "e2e": e2e, "gpu_launches": int(launches), "tokens_in_timed_region": toks, "decode": decode,
                "roofline": roof, "attention": att, "cpu_baseline": cpu, "clocks": clk, "single_stream": single, "config5": cfg5}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
