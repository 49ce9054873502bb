"""GPU log-mel (nemo_logmel_frames) against the host front end, which is bit-exact with the
reference's src/mel.c (test_oracle_golden.py): every frame within 1e-5, including the frames
whose windows reflect at both stream edges; and the streaming engine fed through the GPU
transform against the host transform (NEMO_HOST_MEL=1)."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import nemoasr_b200 as nb
import oracle as orc
from parity import REL_TOL, per_chunk_rel, tokens_match
from test_gpu_stream import run_session, tiny_oracle  # noqa: F401 (fixture)

pytestmark = pytest.mark.gpu
MEL_TOL = 1e-5


def spans_of(audio):
    """Pre-emphasised samples each frame of a whole (final) stream reads, reflected at the edges
    like the host front end: frame t covers span[t * 160 .. t * 160 + 512)."""
    x = np.asarray(audio, np.float32)
    y = x.copy()
    # x - 0.97f * x_prev with one rounding, as the host's fused multiply-add computes it (a one-ulp
    # difference in the samples moves low-energy log-mel bins by ~6e-5)
    y[1:] = (x[1:].astype(np.float64) - np.float64(np.float32(0.97)) * x[:-1].astype(np.float64)).astype(np.float32)
    n = len(y)
    frames = n // 160 + 1
    g = np.arange((frames - 1) * 160 + 512) - 256
    g = np.where(g < 0, -g, g)
    g = np.where(g >= n, 2 * n - 2 - g, g)
    ok = (g >= 0) & (g < n)
    return np.where(ok, y[np.clip(g, 0, n - 1)], 0.0).astype(np.float32), frames


@pytest.mark.parametrize("seconds", [0.05, 1.3, 4.0])
def test_logmel_gpu_matches_host_transform(seconds):
    L = nb.api()
    L.nemo_logmel_frames.argtypes = [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_int64, C.c_void_p]
    audios = [nb.synth_audio(seed, 16000, seconds=seconds) for seed in (3, 4)]
    refs = [nb.mel(a) for a in audios]
    spans = [spans_of(a) for a in audios]
    T = spans[0][1]
    assert all(r.shape[0] == T for r in refs)
    width = len(spans[0][0])
    d_span = torch.from_numpy(np.stack([s for s, _ in spans])).cuda()
    d_out = torch.zeros((2, T, 128), device="cuda")
    assert L.nemo_logmel_frames(d_span.data_ptr(), width, 2, T, d_out.data_ptr(), T * 128, None) == 0
    got = d_out.cpu().numpy()
    for s in range(2):
        assert np.max(np.abs(got[s] - refs[s])) <= MEL_TOL


def _session(host_mel, **kw):
    old = os.environ.get("NEMO_HOST_MEL")
    os.environ["NEMO_HOST_MEL"] = "1" if host_mel else "0"
    try:
        return nb.Session(**kw)
    finally:
        if old is None:
            os.environ.pop("NEMO_HOST_MEL", None)
        else:
            os.environ["NEMO_HOST_MEL"] = old


@pytest.mark.parametrize("lat,block", [(560, 1600), (80, 4000), (1120, 23456)])
def test_stream_with_gpu_mel_matches_host_mel(tiny_ckpt, lat, block):
    audio = nb.synth_audio(77, 16000, seconds=6.0, pauses=True)
    out = []
    for host in (False, True):
        s = _session(host, model_dir=tiny_ckpt, latency_ms=lat)
        out.append(run_session(s, audio, 16000, 4096, 256, 128, block=block))
        s.close()
    a, b = out
    np.testing.assert_array_equal(a["chunk_rows"], b["chunk_rows"])
    assert max(per_chunk_rel(a["prompted"], b["prompted"], a["chunk_rows"])) < REL_TOL
    assert a["tokens"] == b["tokens"]


def _batch(host_mel, B, ckpt, lat):
    old = os.environ.get("NEMO_HOST_MEL")
    os.environ["NEMO_HOST_MEL"] = "1" if host_mel else "0"
    try:
        return nb.Batch(B, model_dir=ckpt, latency_ms=lat)
    finally:
        if old is None:
            os.environ.pop("NEMO_HOST_MEL", None)
        else:
            os.environ["NEMO_HOST_MEL"] = old


def test_batch_gpu_mel_grouped_staging_matches_host_mel(tiny_ckpt, tiny_oracle):
    # 64 streams: the spans are staged and uploaded in groups. The GPU log-mel agrees with the host
    # transform to MEL_TOL (not bit for bit), so the two runs' encoder outputs must agree per chunk
    # within REL_TOL, and their tokens must be identical except in a stream whose decisions meet a
    # near-tie: where a stream's tokens differ, both runs must match the oracle's under the
    # near-tie rule.
    B, lat, block = 64, 560, 8960
    audio = np.stack([nb.synth_audio(300 + i, 16000, seconds=3.0, pauses=True) for i in range(B)])
    out, taps = [], []
    for host in (False, True):
        b = _batch(host, B, tiny_ckpt, lat)
        b.set_taps(B * 64, 256, 128)
        toks = [[] for _ in range(B)]
        for q in range(0, audio.shape[1], block):
            o = b.feed(audio[:, q:q + block], final=q + block >= audio.shape[1])
            for i in range(B):
                toks[i] += o[i]
        taps.append((b.tc[:np.count_nonzero(b.tc)].copy(), b.tp.copy()))
        b.close()
        out.append(toks)
    assert sum(len(t) for t in out[0]) > 0
    rows = taps[0][0]
    np.testing.assert_array_equal(rows, taps[1][0])
    n = int(rows.sum()) * B  # taps are [chunk][stream][row]
    assert max(per_chunk_rel(taps[0][1][:n], taps[1][1][:n], rows * B)) < REL_TOL
    for i in range(B):
        if out[0][i] != out[1][i]:
            o = orc.run_stream(tiny_oracle, audio[i], 16000, lat, block=block)
            for k in range(2):
                ok, note = tokens_match(out[k][i], o["tokens"], o["dec_token"], o["dec_margin"], blank=64)
                assert ok, f"stream {i}, {'host' if k else 'GPU'} log-mel: {note}"
