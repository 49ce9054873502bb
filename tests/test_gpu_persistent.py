"""One stream through the persistent single-stream kernels (the conformer blocks of a chunk in one
launch, the greedy loop of a chunk in one launch) against the same stream through the
kernel-by-kernel path (NEMO_PERSISTENT=0): encoder rows within the parity tolerance, token ids
identical up to oracle near-ties, on the full-size model at three chunk sizes and across
several compaction epochs."""
import os

import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from parity import REL_TOL, per_chunk_rel, tokens_match
from test_gpu_stream import full_ckpt, full_oracle, run_session  # noqa: F401 (fixtures)

pytestmark = pytest.mark.gpu


def _session(path_off, **kw):
    old = os.environ.get("NEMO_PERSISTENT")
    if path_off:
        os.environ["NEMO_PERSISTENT"] = "0"
    else:
        os.environ.pop("NEMO_PERSISTENT", None)
    try:
        return nb.Session(**kw)
    finally:
        if old is None:
            os.environ.pop("NEMO_PERSISTENT", None)
        else:
            os.environ["NEMO_PERSISTENT"] = old


@pytest.mark.parametrize("lat,secs", [(560, 9.0), (80, 2.0), (1120, 6.0)])
def test_persistent_matches_kernel_by_kernel(full_ckpt, full_oracle, lat, secs):
    audio = nb.synth_audio(1000 + lat, 16000, seconds=secs, pauses=True)
    out = []
    for off in (False, True):
        s = _session(off, model_dir=full_ckpt, latency_ms=lat)
        out.append(run_session(s, audio, 16000, 4096, 1024, 640, block=1600))
        s.close()
    a, b = out
    np.testing.assert_array_equal(a["chunk_rows"], b["chunk_rows"])
    assert max(per_chunk_rel(a["prompted"], b["prompted"], a["chunk_rows"])) < REL_TOL
    assert max(per_chunk_rel(a["joint"], b["joint"], a["chunk_rows"])) < REL_TOL
    if a["tokens"] != b["tokens"]:
        # both follow the same greedy rule: each must match the oracle up to its near-ties
        o = orc.run_stream(full_oracle, audio, 16000, lat, block=1600)
        for t in (a["tokens"], b["tokens"]):
            ok, note = tokens_match(t, o["tokens"], o["dec_token"], o["dec_margin"], blank=1024)
            assert ok, note
