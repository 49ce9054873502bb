"""Per-chunk oracle parity of the batched full-size model at the shapes the benchmark times.

BASELINE config #4 shape: 256 streams x 560 ms chunks (1792-row activation-major tensor-core
tiles, per-stream language prompts, pauses), run through the public batch API from host audio
past one cache compaction epoch (>= 20 chunks). Config #5's tile shapes: 64 streams x 1120 ms
(896 rows per GEMM). A seeded sample of 4 streams per batch is run through the oracle
(src/encoder.c:213-267 feeding src/decoder.c:92-127): per chunk, the post-prompt encoder rows and
the joint encoder rows within max|d|/max|ref| <= 1e-3 (tools/compare.py:30); tokens identical
except at logged oracle near-ties."""
import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from parity import REL_TOL, per_chunk_rel, tokens_match
from test_gpu_stream import full_ckpt, full_oracle  # noqa: F401 (fixtures)

pytestmark = pytest.mark.gpu


def _languages(B, seed, prompts=128):
    rng = np.random.default_rng(seed)
    keys = ["auto", "en-US"] + [f"lang{i}" for i in range(2, prompts)]
    return [keys[i] for i in rng.integers(0, prompts, size=B)]


def _run_batch(ckpt, B, lat, secs, seed0, block=1600):
    langs = _languages(B, seed0)
    n = int(round(secs * 16000))
    audio = np.stack([nb.synth_audio(seed0 + s, 16000, n=n, pauses=True) for s in range(B)])
    b = nb.Batch(B, model_dir=ckpt, languages=langs, latency_ms=lat)
    c = lat // 80
    chunks = n // (lat * 16) + 3
    b.set_taps(B * c * chunks, 1024, 640)
    toks = [[] for _ in range(B)]
    for q in range(0, n, block):
        out = b.feed(audio[:, q:q + block], final=q + block >= n)
        for i in range(B):
            toks[i] += out[i]
    rows = b.tc[:np.count_nonzero(b.tc)].copy()
    prompted, joint = b.tp, b.tj
    b.close()
    return audio, langs, rows, prompted, joint, toks


def _stream_rows(taps, rows, B, i):
    """Rows of stream i out of the batch taps ([chunk][stream][row])."""
    out, r0 = [], 0
    for c in rows:
        out.append(taps[r0 + i * c: r0 + (i + 1) * c])
        r0 += B * c
    return np.concatenate(out)


def _check(ckpt, oracle_model, B, lat, secs, seed0, min_chunks):
    audio, langs, rows, prompted, joint, toks = _run_batch(ckpt, B, lat, secs, seed0)
    assert len(rows) >= min_chunks, f"{len(rows)} chunks"
    sample = sorted(np.random.default_rng(seed0).choice(B, size=4, replace=False).tolist())
    worst_p = worst_j = 0.0
    notes = []
    for i in sample:
        o = orc.run_stream(oracle_model, audio[i], 16000, lat, language=langs[i], block=1600)
        np.testing.assert_array_equal(rows, o["chunk_rows"])
        rp = per_chunk_rel(_stream_rows(prompted, rows, B, i), o["prompted"], rows)
        rj = per_chunk_rel(_stream_rows(joint, rows, B, i), o["joint"], rows)
        worst_p, worst_j = max(worst_p, max(rp)), max(worst_j, max(rj))
        assert max(rp) < REL_TOL, f"stream {i}: prompted rel err {max(rp):.2e} at chunk {int(np.argmax(rp))}"
        assert max(rj) < REL_TOL, f"stream {i}: joint rel err {max(rj):.2e} at chunk {int(np.argmax(rj))}"
        ok, note = tokens_match(toks[i], o["tokens"], o["dec_token"], o["dec_margin"], blank=1024)
        notes.append(f"stream {i} ({len(o['tokens'])} tokens): {note}")
        assert ok, notes[-1]
    print(f"{B} streams x {lat} ms, {len(rows)} chunks: worst per-chunk rel err prompted {worst_p:.2e} joint {worst_j:.2e}; " + "; ".join(notes))


def test_batch_config4_shape_matches_oracle(full_ckpt, full_oracle):
    # 21 chunks of 7 rows: the 18-chunk compaction epoch is crossed once
    _check(full_ckpt, full_oracle, 256, 560, 12.0, 100001, 20)


def test_batch_1120ms_896_rows_matches_oracle(full_ckpt, full_oracle):
    # 12 chunks of 14 rows: the 9-chunk compaction epoch is crossed once
    _check(full_ckpt, full_oracle, 64, 1120, 14.0, 300001, 12)
