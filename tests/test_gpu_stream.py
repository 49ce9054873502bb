"""End-to-end parity of the GPU streaming engine through the public API (include/nemoasr.h):
per-chunk encoder outputs within 1e-3 relative of the reference/oracle and token ids identical
up to oracle near-ties (tests/parity.py)."""
import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from parity import per_chunk_rel, REL_TOL, tokens_match

pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CASES = {"s560": (560, 2.0), "s80": (80, 1.0), "s1120": (1120, 3.1), "s560_long": (560, 15.0), "s320_short": (320, 0.21)}


def run_session(sess, audio, rate, rows, D, JH, block=None):
    sess.set_taps(rows, D, JH)
    block = block or rate // 10
    toks = []
    for q in range(0, len(audio), block):
        toks += sess.feed_tokens(audio[q:q + block], final=q + block >= len(audio))
    t = sess.taps()
    t["tokens"] = toks
    return t


@pytest.fixture(scope="module")
def tiny_oracle(tiny_ckpt):
    return orc.Model(tiny_ckpt)


@pytest.mark.parametrize("case", list(CASES))
def test_tiny_stream_matches_reference_fixtures(tiny_ckpt, tiny_oracle, golden, case):
    lat, secs = CASES[case]
    seed, pauses = golden[f"{case}_audio_seed"]
    audio = nb.synth_audio(int(seed), 16000, seconds=secs, pauses=bool(pauses))
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=lat)
    g = run_session(s, audio, 16000, 512, 256, 128, block=1600)
    s.close()
    rows = golden[f"{case}_chunk_rows"]
    np.testing.assert_array_equal(g["chunk_rows"], rows)
    assert max(per_chunk_rel(g["prompted"], golden[f"{case}_prompted"], rows)) < REL_TOL
    assert max(per_chunk_rel(g["joint"], golden[f"{case}_joint"], rows)) < REL_TOL
    o = orc.run_stream(tiny_oracle, audio, 16000, lat, block=1600)
    ok, note = tokens_match(g["tokens"], golden[f"{case}_tokens"], o["dec_token"], o["dec_margin"], blank=64)
    assert ok, note


def test_tiny_api_text_48k(tiny_ckpt, golden):
    a48 = nb.synth_audio(21, 48000, seconds=2.5)
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=560, rate=48000, language="en-US")
    text = ""
    for q in range(0, len(a48), 4800):
        text += s.feed(a48[q:q + 4800], final=q + 4800 >= len(a48))
    st = s.stats()
    s.close()
    assert text == str(golden["api48_text"])
    assert st["chunks"] > 0 and abs(st["audio_seconds"] - 2.5) < 0.01


def test_reset_and_reuse(tiny_ckpt, golden):
    audio = nb.synth_audio(11, 16000, seconds=2.0)
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=560)
    a = run_session(s, audio, 16000, 64, 256, 128, block=1600)
    s.reset(language="auto", latency_ms=560)
    b = run_session(s, audio, 16000, 64, 256, 128, block=1600)
    s.reset(latency_ms=80)
    s.close()
    np.testing.assert_array_equal(a["prompted"], b["prompted"])
    assert a["tokens"] == b["tokens"]


@pytest.fixture(scope="module")
def full_ckpt(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("ckpt_full"))
    nb.synth_write(d, nb.synth_default())
    return d


@pytest.fixture(scope="module")
def full_oracle(full_ckpt):
    return orc.Model(full_ckpt)


@pytest.mark.parametrize("lat,secs", [(560, 4.0), (80, 1.2), (1120, 2.5)])
def test_full_model_stream_matches_oracle(full_ckpt, full_oracle, lat, secs):
    audio = nb.synth_audio(1, 16000, seconds=secs)
    o = orc.run_stream(full_oracle, audio, 16000, lat)
    s = nb.Session(model_dir=full_ckpt, latency_ms=lat)
    g = run_session(s, audio, 16000, 512, 1024, 640)
    s.close()
    np.testing.assert_array_equal(g["chunk_rows"], o["chunk_rows"])
    rel_p = per_chunk_rel(g["prompted"], o["prompted"], o["chunk_rows"])
    rel_j = per_chunk_rel(g["joint"], o["joint"], o["chunk_rows"])
    print(f"latency {lat}: max per-chunk rel err prompted {max(rel_p):.2e} joint {max(rel_j):.2e}")
    assert max(rel_p) < REL_TOL and max(rel_j) < REL_TOL
    ok, note = tokens_match(g["tokens"], o["tokens"], o["dec_token"], o["dec_margin"], blank=1024)
    print("tokens:", note)
    assert ok, note


def test_batched_streams_match_single_stream_oracle(tiny_ckpt, tiny_oracle):
    B, secs, lat = 5, 3.0, 560
    langs = ["auto", "en-US", "lang2", "lang5", "auto"]
    audio = np.stack([nb.synth_audio(40 + i, 16000, seconds=secs, pauses=True) for i in range(B)])
    b = nb.Batch(B, model_dir=tiny_ckpt, languages=langs, latency_ms=lat)
    b.set_taps(B * 64, 256, 128)
    toks = [[] for _ in range(B)]
    for q in range(0, audio.shape[1], 1600):
        out = b.feed(audio[:, q:q + 1600], final=q + 1600 >= audio.shape[1])
        for i in range(B):
            toks[i] += out[i]
    rows = b.tc[:np.count_nonzero(b.tc)]
    prompted = b.tp
    b.close()
    for i in range(B):
        o = orc.run_stream(tiny_oracle, audio[i], 16000, lat, language=langs[i], block=1600)
        np.testing.assert_array_equal(rows, o["chunk_rows"])
        # taps are [chunk][stream][row] -> this stream's rows
        mine, r0 = [], 0
        for c in rows:
            mine.append(prompted[r0 + i * c: r0 + (i + 1) * c])
            r0 += B * c
        mine = np.concatenate(mine)
        assert max(per_chunk_rel(mine, o["prompted"], rows)) < REL_TOL
        ok, note = tokens_match(toks[i], o["tokens"], o["dec_token"], o["dec_margin"], blank=64)
        assert ok, f"stream {i}: {note}"
