"""Edge cases of the streaming API, as the reference's bookkeeping defines them: a stream closed
with no samples at all, a 48 kHz stream too short for the resampler to produce any output (its
first output needs input at and before time zero), and feeds after the final one. Each against
the oracle, which follows the reference's src/nemoasr.c, src/resample.c and src/mel.c; none of
these cases launches encoder work."""
import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from test_gpu_stream import tiny_oracle  # noqa: F401 (fixture)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rate,n", [(16000, 0), (48000, 0), (48000, 10)])
def test_session_closed_with_almost_no_audio(tiny_ckpt, tiny_oracle, rate, n):
    audio = nb.synth_audio(5, rate, seconds=1.0)[:n]
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=560, rate=rate)
    toks = s.feed_tokens(audio, final=True)
    assert s.feed_tokens(nb.synth_audio(6, rate, seconds=0.2), final=True) == []  # after the final feed: nothing
    st = s.stats()
    s.close()
    o = orc.run_stream(tiny_oracle, audio, rate, 560)
    assert toks == o["tokens"] == []
    assert st["chunks"] == 0


@pytest.mark.parametrize("rate", [16000, 48000])
def test_batch_closed_with_no_audio(tiny_ckpt, rate):
    b = nb.Batch(3, model_dir=tiny_ckpt, latency_ms=560, rate=rate)
    out = b.feed(np.zeros((3, 0), np.float32), final=True)
    again = b.feed(np.zeros((3, 1600), np.float32), final=True)
    st = b.stats()
    b.close()
    assert out == [[], [], []] and again == [[], [], []]
    assert st["chunks"] == 0 and st["audio_seconds"] == 0.0
