"""nemoasr_prepare_latency (src/nemoasr.h:49, src/warmup.c:23-42): the warm-up captures the graph
of every chunk shape a latency can produce, so a stream after a reset to that latency captures
none, and its results are those of the oracle."""
import ctypes as C

import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from parity import REL_TOL, per_chunk_rel, tokens_match
from test_gpu_stream import run_session, tiny_oracle  # noqa: F401 (fixture)

pytestmark = pytest.mark.gpu


def _graphs(s):
    L = nb.api()
    L.nemoasr_graphs_captured.argtypes = [C.c_void_p]
    return L.nemoasr_graphs_captured(s.h)


def _prepare(s, lat):
    err = C.create_string_buffer(1024)
    if nb.api().nemoasr_prepare_latency(s.h, lat, err, 1024):
        raise RuntimeError(err.value.decode())


@pytest.mark.parametrize("lat,secs", [(560, 2.37), (80, 1.13), (1120, 3.05)])
def test_prepare_then_reset_captures_nothing_and_matches_oracle(tiny_ckpt, tiny_oracle, lat, secs):
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=320, language="en-US")
    _prepare(s, lat)                       # another latency: warms an engine kept for it
    s.reset(latency_ms=lat)                # takes that engine over (language kept)
    n0 = _graphs(s)
    assert n0 > 0
    audio = nb.synth_audio(61, 16000, seconds=secs, pauses=True)
    g = run_session(s, audio, 16000, 512, 256, 128, block=1600)
    assert _graphs(s) == n0, "a chunk captured a graph after the warm-up"
    # the session's own latency: warming it again adds nothing
    _prepare(s, lat)
    assert _graphs(s) == n0
    s.close()
    o = orc.run_stream(tiny_oracle, audio, 16000, lat, language="en-US", block=1600)
    np.testing.assert_array_equal(g["chunk_rows"], o["chunk_rows"])
    assert max(per_chunk_rel(g["prompted"], o["prompted"], o["chunk_rows"])) < REL_TOL
    ok, note = tokens_match(g["tokens"], o["tokens"], o["dec_token"], o["dec_margin"], blank=64)
    assert ok, note


def test_stream_lengths_all_covered_by_the_warm_up(tiny_ckpt):
    """Every final-chunk length: streams of 1..chunk frames beyond 0, 1 and 2 whole chunks."""
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=560)
    _prepare(s, 560)
    n0 = _graphs(s)
    for whole in (0, 1, 2):
        for extra in range(1, 57, 5):
            s.reset(latency_ms=560)
            n = (whole * 56 + extra) * 160
            s.feed_tokens(nb.synth_audio(5 + extra, 16000, n=n), final=True)
    assert _graphs(s) == n0
    s.close()


def test_prepare_rejects_bad_latency(tiny_ckpt):
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=560)
    with pytest.raises(RuntimeError, match="80, 160, 320, 560, 1120"):
        _prepare(s, 100)
    s.close()
