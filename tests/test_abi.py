"""The C-ABI library loads and exports every entry point its headers declare; host-only logic
(synthetic checkpoint IO, config checks, error paths) works without a GPU."""
import ctypes as C
import json
import os
import re

import numpy as np
import pytest

import nemoasr_b200 as nb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("nemoasr.h", "nemo_gpu.h"):
        txt = open(os.path.join(ROOT, "include", h)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b((?:nemoasr|nemo)_\w+)\s*\(", txt, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_entry_points():
    names = declared_functions()
    assert "nemoasr_open" in names and "nemo_gemm" in names and len(names) > 30


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports(name):
    lib = nb.lib()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_synthetic_checkpoint_roundtrip(tmp_path):
    spec = nb.synth_tiny(seed=3)
    nb.synth_write(str(tmp_path), spec)
    cfg = json.load(open(tmp_path / "config.json"))
    assert cfg["encoder"]["d_model"] == 256 and cfg["decoder"]["vocab_size"] == 64
    with open(tmp_path / "model.safetensors", "rb") as f:
        hl = int.from_bytes(f.read(8), "little")
        hdr = json.loads(f.read(hl))
    assert hdr["joint.joint_net.2.weight"]["shape"] == [65, 128]
    assert all(v["dtype"] == "BF16" for k, v in hdr.items() if k != "__metadata__")
    # deterministic: the same spec writes the same bytes
    d2 = tmp_path / "again"
    nb.synth_write(str(d2), spec)
    assert (tmp_path / "model.safetensors").read_bytes() == (d2 / "model.safetensors").read_bytes()


def test_synthetic_audio_is_seeded():
    a = nb.synth_audio(5, 16000, seconds=0.5)
    b = nb.synth_audio(5, 16000, seconds=0.5)
    c = nb.synth_audio(6, 16000, seconds=0.5)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert 0.1 < np.abs(a).max() < 1.0
    p = nb.synth_audio(5, 16000, seconds=8.0, pauses=True)
    # pauses mute the chirps: some 100 ms windows carry only the 0.05 noise
    w = np.abs(p[: 8 * 16000].reshape(80, 1600)).max(axis=1)
    assert (w < 0.3).any() and (w > 0.3).any()


def _gpu_present():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_gpu_present(), reason="checks the no-GPU error path")
def test_open_fails_loudly_without_gpu(tiny_ckpt):
    with pytest.raises(RuntimeError, match="CUDA device"):
        nb.Session(model_dir=tiny_ckpt)


def test_open_rejects_bad_arguments(tiny_ckpt):
    with pytest.raises(RuntimeError, match="latency"):
        nb.Session(model_dir=tiny_ckpt, latency_ms=100)
    with pytest.raises(RuntimeError, match="input_rate"):
        nb.Session(model_dir=tiny_ckpt, rate=0)
    with pytest.raises(RuntimeError, match="cannot read"):
        nb.Session(model_dir="/nonexistent-dir")


def test_gemm_rejects_bad_shapes():
    lib = nb.api()
    a = nb.GemmArgs()
    assert lib.nemo_gemm(C.byref(a), None) == -1
    assert b"null pointer" in lib.nemo_gpu_last_error()


def test_resample_rejects_bad_arguments():
    """Checked on the host before any launch: rates, a window past the samples seen, an output
    row shorter than the outputs asked for, and rates whose weight rows exceed shared memory."""
    lib = nb.api()
    lib.nemo_resample.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int64,
                                  C.c_int, C.c_void_p]
    assert lib.nemo_resample(None, 64, 0, 64, 64, 0, 8, 0, 16000, None, 64, 1, None) == -1
    assert b"rates" in lib.nemo_gpu_last_error()
    assert lib.nemo_resample(None, 64, 10, 64, 32, 0, 8, 48000, 16000, None, 64, 1, None) == -1
    assert b"window" in lib.nemo_gpu_last_error()
    assert lib.nemo_resample(None, 64, 0, 64, 64, 0, 80, 48000, 16000, None, 64, 1, None) == -1
    assert lib.nemo_resample(None, 1 << 20, 0, 1 << 20, 1 << 20, 0, 8, 1000000, 16000, None, 64, 1, None) == -1
    assert b"shared memory" in lib.nemo_gpu_last_error()
    assert lib.nemo_resample(None, 64, 0, 64, 64, 0, 0, 48000, 16000, None, 64, 1, None) == 0  # nothing to do


def test_decoder_joint_partials():
    """Argmax partials per stream of the joint GEMM (two per column tile): 80-column tiles while
    the partials fit the step kernel's one-warp reduction, else 128-column tiles."""
    f = nb.api().nb_dec_joint_parts
    f.argtypes, f.restype = [C.c_int], C.c_int
    assert f(1025) == 26  # the vocabulary + blank of the published model: 13 tiles of 80
    assert f(65) == 2
    assert f(1280) == 32
    assert f(1281) == 22  # 17 tiles of 80 would be 34 partials: 11 tiles of 128
    assert f(2048) == 32
    assert f(2049) == 34  # over 32: the engine then keeps the separate argmax kernel


def test_attention_rejects_bad_arguments():
    """Checked on the host before any launch: head dim, chunk rows, window, 16-byte alignment."""
    lib = nb.api()
    f = lib.nemo_attention_rel
    p, i64 = C.c_void_p, C.c_int64
    f.argtypes = [p, i64, i64, p, p, i64, i64, p, p, p, p, p, p, C.c_int, i64, i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, p]
    f.restype = C.c_int
    A = 0x10000  # never dereferenced: every case below returns before a launch

    def call(dh=128, c=7, Lmax=72, bias=A, ldk=3072):
        return f(A, 3072, 3072 * 128, A, A, ldk, 3072 * 128, A, A, A, bias, A, A, 0, 0, c * 1024, 2, c, Lmax, 8, dh, 1024, 0.088, None)
    assert call(dh=64) == -1 and b"head dim" in lib.nemo_gpu_last_error()
    assert call(c=17) == -1 and b"too large" in lib.nemo_gpu_last_error()
    assert call(Lmax=97) == -1 and b"too large" in lib.nemo_gpu_last_error()
    assert call(bias=A + 8) == -1 and b"16-byte aligned" in lib.nemo_gpu_last_error()
    assert call(ldk=3070) == -1 and b"16-byte aligned" in lib.nemo_gpu_last_error()
    assert call(c=0) == 0  # nothing to do
