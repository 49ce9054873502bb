"""The oracle (CPU restatement) pinned against fixtures produced by the reference's own host code
(tests/golden/make_golden.py), plus checks of the oracle's kernel math against numpy."""
import hashlib
import os

import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc

CASES = ["s560", "s80", "s1120", "s560_long", "s320_short"]
LAT = {"s560": 560, "s80": 80, "s1120": 1120, "s560_long": 560, "s320_short": 320}
SECS = {"s560": 2.0, "s80": 1.0, "s1120": 3.1, "s560_long": 15.0, "s320_short": 0.21}


def test_checkpoint_generator_is_pinned(tiny_ckpt, golden):
    h = hashlib.sha256()
    for f in ("config.json", "model.safetensors"):
        h.update(open(os.path.join(tiny_ckpt, f), "rb").read())
    assert h.hexdigest() == str(golden["ckpt_sha256"])


@pytest.fixture(scope="module")
def tiny_model(tiny_ckpt):
    return orc.Model(tiny_ckpt)


@pytest.mark.parametrize("case", CASES)
def test_oracle_stream_matches_reference(tiny_model, golden, case):
    seed, pauses = golden[f"{case}_audio_seed"]
    audio = nb.synth_audio(int(seed), 16000, seconds=SECS[case], pauses=bool(pauses))
    o = orc.run_stream(tiny_model, audio, 16000, LAT[case], block=1600)
    np.testing.assert_array_equal(o["chunk_rows"], golden[f"{case}_chunk_rows"])
    # same kernels, same order of operations: the restated bookkeeping reproduces the
    # reference's own host code exactly
    np.testing.assert_array_equal(o["prompted"], golden[f"{case}_prompted"])
    np.testing.assert_array_equal(o["joint"], golden[f"{case}_joint"])
    assert o["tokens"] == golden[f"{case}_tokens"].tolist()


def _text(tokens, cfg):
    voc = cfg["vocabulary"]
    out = ""
    for t in tokens:
        p = voc[t] if 0 <= t < len(voc) else ""
        if p in ("<unk>", "<pad>", "<s>", "</s>"):
            continue
        s = p.replace("▁", " ")
        if not out:
            s = s.lstrip(" ")
        out += s
    return out


def test_oracle_api_48k_matches_reference_text(tiny_model, golden):
    a48 = nb.synth_audio(21, 48000, seconds=2.5)
    o = orc.run_stream(tiny_model, a48, 48000, 560, language="en-US")
    assert _text(o["tokens"], tiny_model.cfg) == str(golden["api48_text"])


def test_oracle_frontend_matches_reference(golden):
    a = nb.synth_audio(31, 16000, seconds=1.37)
    np.testing.assert_array_equal(orc.mel(a, golden["mel_blocks"].tolist()), golden["mel"])
    np.testing.assert_array_equal(orc.resample(nb.synth_audio(32, 48000, seconds=0.7), 48000, 16000, block=4800), golden["rs48"])
    np.testing.assert_array_equal(orc.resample(nb.synth_audio(33, 44100, seconds=0.7), 44100, 16000, block=4410), golden["rs441"])


def test_product_host_frontend_matches_reference(golden):
    """The library's host front end (nemoasr_mel_*, nemoasr_resampler_*) needs no GPU."""
    a = nb.synth_audio(31, 16000, seconds=1.37)
    np.testing.assert_array_equal(nb.mel(a, golden["mel_blocks"].tolist()), golden["mel"])
    np.testing.assert_array_equal(nb.resample(nb.synth_audio(32, 48000, seconds=0.7), 48000, 16000, block=4800), golden["rs48"])
    np.testing.assert_array_equal(nb.resample(nb.synth_audio(33, 44100, seconds=0.7), 44100, 16000, block=4410), golden["rs441"])


@pytest.mark.skipif(not orc.ref_available(), reason="reference host build not present (built only where its sources are)")
@pytest.mark.parametrize("lat,secs,seed", [(560, 3.3, 101), (160, 1.7, 102), (1120, 1.0, 103)])
def test_oracle_matches_reference_live(tiny_ckpt, tiny_model, lat, secs, seed):
    audio = nb.synth_audio(seed, 16000, seconds=secs, pauses=True)
    r = orc.ref_run_stream(tiny_ckpt, audio, lat)
    o = orc.run_stream(tiny_model, audio, 16000, lat, block=1600)
    np.testing.assert_array_equal(o["prompted"], r["prompted"])
    assert o["tokens"] == r["tokens"]


# ---- the oracle's kernels against an independent float64 numpy statement ------------------
def _bf16(rng, shape, std=0.05):
    f = (rng.standard_normal(shape) * std).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def _w(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_oracle_gemm_epilogues(act):
    rng = np.random.default_rng(act)
    M, N, K = 5, 64, 96
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = _bf16(rng, (N, K))
    b = rng.standard_normal(N).astype(np.float32)
    C0 = rng.standard_normal((M, N // 2 if act == 3 else N)).astype(np.float32)
    got = orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)
    z = A.astype(np.float64) @ _w(W).T + b
    if act == 3:
        ref = z[:, :N // 2] / (1 + np.exp(-z[:, N // 2:]))
    elif act == 1:
        ref = z / (1 + np.exp(-z))
    elif act == 2:
        ref = np.maximum(z, 0)
    else:
        ref = z
    np.testing.assert_allclose(got, C0 + 0.5 * ref, rtol=1e-5, atol=1e-5)


def test_oracle_attention_rel():
    rng = np.random.default_rng(5)
    H, dh, c, L, Lmax = 2, 128, 3, 9, 12
    D = H * dh
    Q = rng.standard_normal((c, D)).astype(np.float32)
    K = rng.standard_normal((L, D)).astype(np.float32)
    V = rng.standard_normal((L, D)).astype(np.float32)
    P = rng.standard_normal((2 * Lmax - 1, D)).astype(np.float32)
    bu, bv = rng.standard_normal(D).astype(np.float32), rng.standard_normal(D).astype(np.float32)
    got = orc.attention_rel(Q, K, V, P, bu, bv, c, L, Lmax, H, dh)
    ref = np.zeros((c, D))
    for h in range(H):
        sl = slice(h * dh, (h + 1) * dh)
        for i in range(c):
            s = np.array([((Q[i, sl] + bu[sl]) @ K[j, sl] + (Q[i, sl] + bv[sl]) @ P[(Lmax - L) + (c - 1 - i + j), sl]) / np.sqrt(dh)
                          for j in range(L)], np.float64)
            p = np.exp(s - s.max())
            ref[i, sl] = (p / p.sum()) @ V[:, sl]
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_oracle_joint_argmax_tie_takes_lowest_index():
    rng = np.random.default_rng(3)
    H, V = 32, 10
    W = np.zeros((V, H), np.uint16)
    bias = np.zeros(V, np.float32)
    bias[[3, 7]] = 1.0
    enc = rng.standard_normal((2, H)).astype(np.float32)
    idx, val, mar = orc.joint_argmax(enc, np.zeros(H, np.float32), W, bias)
    assert idx.tolist() == [3, 3] and np.all(mar == 0)
