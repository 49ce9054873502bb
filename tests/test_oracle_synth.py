"""The oracle's copy of the benchmark's synthetic workload generator (oracle/oracle_synth.c, used by
bench.py's CPU reference arm so that arm never loads the product library) writes the same bytes as
the product's generator: checkpoint files and audio samples, bit for bit."""
import hashlib
import os

import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc


def _digest(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 22), b""):
            h.update(blk)
    return h.hexdigest()


@pytest.mark.parametrize("kw", [dict(n_layers=2, d_model=256, sub_channels=64, num_prompts=8, prompt_hidden=256, pred_hidden=128,
                                     joint_hidden=128, vocab_size=64, weight_std=0.1, blank_bias=1.9, seed=7),
                                dict(n_layers=1, blank_bias=-0.25, seed=99)])
def test_checkpoint_bytes_identical(tmp_path, kw):
    a, b = str(tmp_path / "product"), str(tmp_path / "oracle")
    nb.synth_write(a, nb.synth_default(**kw))
    orc.synth_write(b, orc.synth_default(**kw))
    for f in ("config.json", "model.safetensors"):
        assert _digest(os.path.join(a, f)) == _digest(os.path.join(b, f)), f


def test_default_spec_identical():
    p, o = nb.synth_default(), orc.synth_default()
    for name, _ in nb.SynthSpec._fields_:
        assert getattr(p, name) == getattr(o, name), name


@pytest.mark.parametrize("seed,rate,secs,pauses", [(1, 16000, 4.0, False), (100001, 16000, 12.0, True), (3, 48000, 2.5, True)])
def test_audio_identical(seed, rate, secs, pauses):
    x = nb.synth_audio(seed, rate, seconds=secs, pauses=pauses)
    y = orc.synth_audio(seed, rate, seconds=secs, pauses=pauses)
    assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
