"""GPU resampler (nemo_resample) against the oracle's restatement of src/resample.c, which is pinned
bit-exact to the reference's golden vectors (test_oracle_golden.py): every output within 1e-5,
for several rates, more streams than one block takes, and a window that starts inside a stream;
and the streaming API fed at 48 kHz through the GPU resampler against the host resampler
(NEMO_GPU_RESAMPLE=0)."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import nemoasr_b200 as nb
import oracle as orc
from parity import tokens_match
from test_gpu_stream import tiny_oracle  # noqa: F401 (fixture)

pytestmark = pytest.mark.gpu
RS_TOL = 1e-5


def _kernel():
    L = nb.api()
    L.nemo_resample.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int64,
                                C.c_int, C.c_void_p]
    return L


@pytest.mark.parametrize("rate,streams", [(48000, 3), (44100, 70), (22050, 2), (8000, 2), (96000, 2), (11025, 1)])
def test_resample_kernel_matches_oracle(rate, streams):
    L = _kernel()
    secs = 0.25 if streams > 8 else 0.6
    audio = np.stack([nb.synth_audio(40 + s, rate, seconds=secs, pauses=True) for s in range(streams)])
    refs = [orc.resample(a, rate, 16000) for a in audio]
    n_out = len(refs[0])
    assert all(len(r) == n_out for r in refs) and n_out > 0
    nin = audio.shape[1]
    d_in = torch.from_numpy(audio).cuda()
    d_out = torch.full((streams, n_out + 5), 7.0, device="cuda")
    assert L.nemo_resample(d_in.data_ptr(), nin, 0, nin, nin, 0, n_out, rate, 16000, d_out.data_ptr(), n_out + 5, streams, None) == 0, \
        L.nemo_gpu_last_error()
    got = d_out.cpu().numpy()
    for s in range(streams):
        assert np.max(np.abs(got[s, :n_out] - refs[s])) <= RS_TOL
        assert np.all(got[s, n_out:] == 7.0)  # nothing written past the outputs asked for


def test_resample_kernel_window_inside_stream():
    """Outputs [out0, out0 + count) from a window that holds only the inputs they reach."""
    L = _kernel()
    rate = 44100
    audio = nb.synth_audio(61, rate, seconds=1.0, pauses=True)
    ref = orc.resample(audio, rate, 16000)
    ratio, half = rate / 16000, 16.0 * rate / 16000
    out0, count = 5001, 3000
    start = int(np.ceil(out0 * ratio - half)) - 3
    nin = int(np.floor((out0 + count - 1) * ratio + half)) + 1  # the last output's taps have all arrived
    win = np.ascontiguousarray(audio[start:nin])
    d_in = torch.from_numpy(win).cuda()
    d_out = torch.zeros(count, device="cuda")
    assert L.nemo_resample(d_in.data_ptr(), len(win), start, len(win), nin, out0, count, rate, 16000, d_out.data_ptr(), count, 1, None) == 0, \
        L.nemo_gpu_last_error()
    assert np.max(np.abs(d_out.cpu().numpy() - ref[out0:out0 + count])) <= RS_TOL


def test_resample_kernel_rejects_bad_window():
    L = _kernel()
    d = torch.zeros(64, device="cuda")
    # a window that ends past the samples seen: refused on the host, nothing launched
    assert L.nemo_resample(d.data_ptr(), 64, 10, 64, 32, 0, 8, 48000, 16000, d.data_ptr(), 64, 1, None) != 0


def _batch(gpu_rs, B, ckpt, langs, rate):
    old = os.environ.get("NEMO_GPU_RESAMPLE")
    os.environ["NEMO_GPU_RESAMPLE"] = "1" if gpu_rs else "0"
    try:
        return nb.Batch(B, model_dir=ckpt, languages=langs, latency_ms=560, rate=rate)
    finally:
        if old is None:
            os.environ.pop("NEMO_GPU_RESAMPLE", None)
        else:
            os.environ["NEMO_GPU_RESAMPLE"] = old


# the last case feeds each stream's 3 s in one call: three one-second resampler passes on the GPU side
@pytest.mark.parametrize("rate,block", [(48000, 4800), (44100, 7777), (48000, 1 << 30)])
def test_batch_gpu_resampler_matches_host_resampler(tiny_ckpt, tiny_oracle, rate, block):
    B = 6
    langs = ["auto", "en-US"] * (B // 2)
    audio = np.stack([nb.synth_audio(500 + i, rate, seconds=3.0, pauses=True) for i in range(B)])
    out = []
    for gpu_rs in (True, False):
        b = _batch(gpu_rs, B, tiny_ckpt, langs, rate)
        toks = [[] for _ in range(B)]
        for q in range(0, audio.shape[1], block):
            o = b.feed(audio[:, q:q + block], final=q + block >= audio.shape[1])
            for i in range(B):
                toks[i] += o[i]
        secs = b.stats()["audio_seconds"]
        b.close()
        out.append(toks)
        assert abs(secs - 3.0 * B) < 0.01 * B
    assert sum(len(t) for t in out[0]) > 0
    for i in range(B):
        if out[0][i] != out[1][i]:
            o = orc.run_stream(tiny_oracle, audio[i], rate, 560, language=langs[i], block=1600)
            ok, note = tokens_match(out[0][i], o["tokens"], o["dec_token"], o["dec_margin"], blank=64)
            assert ok, f"stream {i}: {note}"
