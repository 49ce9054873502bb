"""The fused batched greedy iteration (LSTM cells and the joint input computed in the tensor-core
GEMM epilogues, the input half of LSTM layer 0 read from a per-token gate table, one step kernel
per iteration) against the kernel-by-kernel iteration (NEMO_DEC_FUSED=0), and against the oracle
for two fixed streams of every batch plus any stream whose tokens differ between the two: token
ids identical up to oracle near-ties. 40 streams of the full-size model (activation-major tiles,
several compaction epochs) and 5 of the tiny one."""
import os

import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from parity import tokens_match
from test_gpu_stream import full_ckpt, full_oracle, tiny_oracle  # noqa: F401 (fixtures)

pytestmark = pytest.mark.gpu


def _batch_tokens(fused, B, ckpt, langs, audio, lat, block=1600):
    old = os.environ.get("NEMO_DEC_FUSED")
    if fused:
        os.environ.pop("NEMO_DEC_FUSED", None)
    else:
        os.environ["NEMO_DEC_FUSED"] = "0"
    try:
        b = nb.Batch(B, model_dir=ckpt, languages=langs, latency_ms=lat)
    finally:
        if old is None:
            os.environ.pop("NEMO_DEC_FUSED", None)
        else:
            os.environ["NEMO_DEC_FUSED"] = old
    toks = [[] for _ in range(B)]
    for q in range(0, audio.shape[1], block):
        out = b.feed(audio[:, q:q + block], final=q + block >= audio.shape[1])
        for i in range(B):
            toks[i] += out[i]
    b.close()
    return toks


def _check(B, ckpt, oracle_model, lat, secs, blank, seed0, prompts=128):
    rng = np.random.default_rng(seed0)
    keys = ["auto", "en-US"] + [f"lang{i}" for i in range(2, prompts)]
    langs = [keys[i] for i in rng.integers(0, prompts, size=B)]
    audio = np.stack([nb.synth_audio(seed0 + i, 16000, seconds=secs, pauses=True) for i in range(B)])
    fused = _batch_tokens(True, B, ckpt, langs, audio, lat)
    plain = _batch_tokens(False, B, ckpt, langs, audio, lat)
    assert sum(len(t) for t in fused) > 0
    differ = [i for i in range(B) if fused[i] != plain[i]]
    print(f"{B} streams: {sum(len(t) for t in fused)} tokens, {len(differ)} streams differ")
    for i in sorted(set(differ) | {0, B - 1}):
        o = orc.run_stream(oracle_model, audio[i], 16000, lat, language=langs[i], block=1600)
        for t in (fused[i], plain[i]):
            ok, note = tokens_match(t, o["tokens"], o["dec_token"], o["dec_margin"], blank=blank)
            assert ok, f"stream {i}: {note}"


def test_fused_decoder_full_model_40_streams(full_ckpt, full_oracle):
    _check(40, full_ckpt, full_oracle, 560, 6.0, 1024, 500)


def test_fused_decoder_full_model_80ms(full_ckpt, full_oracle):
    _check(36, full_ckpt, full_oracle, 80, 1.5, 1024, 700)


def test_fused_decoder_tiny_model(tiny_ckpt, tiny_oracle):
    _check(5, tiny_ckpt, tiny_oracle, 560, 3.0, 64, 900, prompts=6)
