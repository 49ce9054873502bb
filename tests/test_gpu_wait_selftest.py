"""Bounded device waits run out into an error status, not a hang or a trap (the reference surfaces
command-buffer errors through err/errlen, src/gpu.m:131-134). nemo_gpu_wait_selftest waits on an
mbarrier nothing arrives on (the tensor-core kernels' wait) or a grid barrier one arrival short
(the persistent kernels' barrier), with a limit of about a millisecond; the kernel returns, the
context stays usable, nemo_gpu_check_device_errors reports the failure once, and a session's next
feed reports it through err."""
import ctypes as C

import pytest
import torch

import nemoasr_b200 as nb

pytestmark = pytest.mark.gpu

LIMIT = 2_000_000  # clock cycles, ~1 ms


def _selftest(kind):
    L = nb.api()
    L.nemo_gpu_wait_selftest.argtypes = [C.c_int, C.c_longlong, C.c_void_p]
    return L.nemo_gpu_wait_selftest(kind, LIMIT, None)


@pytest.mark.parametrize("kind,code", [(0, 9), (1, 10)])
def test_wait_runs_out_into_an_error_status(kind, code):
    L = nb.api()
    assert L.nemo_gpu_check_device_errors() == 0, L.nemo_gpu_last_error().decode()
    assert _selftest(kind) == 0, L.nemo_gpu_last_error().decode()
    torch.cuda.synchronize()  # the kernel returned: the wait gave up instead of hanging
    assert L.nemo_gpu_check_device_errors() != 0
    msg = L.nemo_gpu_last_error().decode()
    assert "bounded device wait gave up" in msg and f"code {code}" in msg, msg
    assert L.nemo_gpu_check_device_errors() == 0  # reported once
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2  # the context still runs work


def test_device_error_reaches_session_err(tiny_ckpt):
    s = nb.Session(model_dir=tiny_ckpt, latency_ms=560)
    audio = nb.synth_audio(3, 16000, seconds=1.2)
    s.feed_tokens(audio[:9000])
    assert _selftest(0) == 0
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="bounded device wait gave up"):
        s.feed_tokens(audio[9000:])
    s.close()
    assert nb.api().nemo_gpu_check_device_errors() == 0
