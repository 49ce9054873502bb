"""Generate tests/golden/golden_tiny.npz from the reference's own host code.

The reference (nemoasr-c) cannot run its Metal kernels here, so oracle/Makefile compiles its host C
sources (src/encoder.c, decoder.c, model.c, nemoasr.c, mel.c, resample.c, ...) unmodified, linked
with oracle/ref_gpu_cpu.c, a CPU stand-in for its GPU layer that executes each kernel dispatch
with the restated kernels. The fixtures below are what that build produces on a small seeded
random-init checkpoint of the same architecture. Run from the repository root after
`NEMO_REFERENCE_SRC=<reference checkout> python -c "import __graft_entry__ as g; g.build()"`:

    python tests/golden/make_golden.py
"""
import hashlib
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "nemo-c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import nemoasr_b200 as nb  # noqa: E402
import oracle as orc  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_tiny.npz")

# (name, latency ms, seconds of 16 kHz audio, audio seed, pauses)
STREAM_CASES = [
    ("s560", 560, 2.0, 11, False),
    ("s80", 80, 1.0, 12, False),
    ("s1120", 1120, 3.1, 13, False),
    ("s560_long", 560, 15.0, 14, True),   # crosses a cache compaction epoch
    ("s320_short", 320, 0.21, 15, False), # shorter than one chunk: only the final boundary window
]


def spec_tiny():
    return nb.synth_tiny(seed=7)


def checkpoint_sha(d):
    h = hashlib.sha256()
    for f in ("config.json", "model.safetensors"):
        h.update(open(os.path.join(d, f), "rb").read())
    return h.hexdigest()


def main():
    if not orc.ref_available():
        sys.exit("oracle/_ref/libnemoref.so is missing (needs the reference sources to build)")
    out = {}
    with tempfile.TemporaryDirectory() as d:
        nb.synth_write(d, spec_tiny())
        out["ckpt_sha256"] = np.array(checkpoint_sha(d))
        for name, lat, secs, seed, pauses in STREAM_CASES:
            audio = nb.synth_audio(seed, 16000, seconds=secs, pauses=pauses)
            r = orc.ref_run_stream(d, audio, lat)
            out[f"{name}_audio_seed"] = np.array([seed, int(pauses)])
            out[f"{name}_prompted"] = r["prompted"]
            out[f"{name}_joint"] = r["joint"]
            out[f"{name}_chunk_rows"] = r["chunk_rows"]
            out[f"{name}_tokens"] = np.array(r["tokens"], np.int32)
        # public API end to end, 48 kHz input through the resampler, 100 ms blocks
        a48 = nb.synth_audio(21, 48000, seconds=2.5)
        out["api48_text"] = np.array(orc.ref_feed_text(d, a48, 48000, 560, language="en-US"))
    # front end
    a = nb.synth_audio(31, 16000, seconds=1.37)
    blocks = [1000, 1600, 37, 5000, 160, len(a) - 7797]
    out["mel_blocks"] = np.array(blocks)
    out["mel"] = orc.ref_mel(a, blocks)
    a48 = nb.synth_audio(32, 48000, seconds=0.7)
    out["rs48"] = orc.ref_resample(a48, 48000, 16000, block=4800)
    a441 = nb.synth_audio(33, 44100, seconds=0.7)
    out["rs441"] = orc.ref_resample(a441, 44100, 16000, block=4410)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
