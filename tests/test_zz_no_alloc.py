"""nemo_gemm_noalloc (the allocation-free tensor-core GEMM) against nemo_gemm through the C ABI,
and against the oracle GEMM (src/kernels.metal:120-208 restated in oracle/).

Both entry points run the same kernel with the same split-K plan, so results should agree to the
bit; NOALLOC_TOL (max|d| / max|ref|) only allows for that changing. Against the oracle the bar is
the tensor-core GEMM's own (activations carried as bf16 hi/lo planes). Each case calls the new
entry twice in a row into fresh outputs, so a counter or partial tile left over by the first call
would show up in the second."""
import ctypes as C

import numpy as np
import pytest
import torch

import nemoasr_b200 as nb
import oracle as orc
from parity import rel_err

pytestmark = pytest.mark.gpu

NOALLOC_TOL = 1e-6
ORACLE_TOL = 2e-4  # bf16 hi/lo activation planes (16-bit mantissa) into the tensor cores


def _lib():
    L = nb.api()
    L.nemo_gemm_noalloc.argtypes = [C.POINTER(nb.GemmArgs), C.c_void_p]
    L.nemo_gemm_noalloc.restype = C.c_int
    return L


def _err():
    return nb.api().nemo_gpu_last_error().decode()


def _planes(A):
    hi = torch.from_numpy(A).to(torch.bfloat16)
    lo = (torch.from_numpy(A) - hi.float()).to(torch.bfloat16)
    return torch.cat([hi.reshape(-1), lo.reshape(-1)]).cuda()


def _args(dA, dW, db, dC, M, N, K, act, acc, alpha):
    a = nb.GemmArgs()
    a.A, a.lda, a.a_fmt, a.a_plane = dA.data_ptr(), K, 1, M * K
    a.W, a.ldw = dW.data_ptr(), K
    a.bias = db.data_ptr() if db is not None else None
    a.C, a.ldc, a.c_fmt = dC.data_ptr(), (N // 2 if act == 3 else N), 0
    a.M, a.N, a.K, a.act, a.accumulate, a.alpha = M, N, K, act, acc, alpha
    return a


# (M, N, K, act, accumulate): single-stream encoder shapes (FF in/out, GLU pointwise conv),
# one row, and the 32-row maximum
CASES = [(7, 4096, 1024, 1, 0), (14, 1024, 4096, 0, 1), (7, 2048, 1024, 3, 0), (1, 1024, 1024, 2, 1), (32, 3072, 1024, 0, 0)]


@pytest.mark.parametrize("M,N,K,act,acc", CASES)
def test_noalloc_matches_nemo_gemm(M, N, K, act, acc):
    L = _lib()
    rng = np.random.default_rng(4242 + M + N + act)
    A = rng.standard_normal((M, K)).astype(np.float32)
    dA = _planes(A)
    dW = (torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)) * 0.02).to(torch.bfloat16).cuda()
    db = torch.from_numpy((rng.standard_normal(N) * 0.1).astype(np.float32)).cuda()
    nout = N // 2 if act == 3 else N
    C0 = torch.from_numpy(rng.standard_normal((M, nout)).astype(np.float32)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):  # the allocation-free entry first (alone in a process, it does its own set-up)
        dC = C0.clone()
        rc = L.nemo_gemm_noalloc(C.byref(_args(dA, dW, db, dC, M, N, K, act, acc, 0.5)), C.c_void_p(st))
        assert rc == 0, _err()
        outs.append(dC)
    dR = C0.clone()
    nb.check(L.nemo_gemm(C.byref(_args(dA, dW, db, dR, M, N, K, act, acc, 0.5)), C.c_void_p(st)), "nemo_gemm")
    torch.cuda.synchronize()
    assert L.nemo_gpu_check_device_errors() == 0, _err()
    ref = dR.cpu().numpy()
    Wh = dW.view(torch.int16).cpu().numpy().view(np.uint16)
    want = orc.gemm(A, Wh, db.cpu().numpy(), C0=C0.cpu().numpy(), act=act, accumulate=bool(acc), alpha=0.5)
    for o in outs:
        assert rel_err(o.cpu().numpy(), ref) <= NOALLOC_TOL
        assert rel_err(o.cpu().numpy(), want) <= ORACLE_TOL


def test_noalloc_rejects_beyond_its_limits():
    L = _lib()
    M, N, K = 33, 256, 256
    dA = _planes(np.zeros((M, K), np.float32))
    dW = torch.zeros((N, K), dtype=torch.bfloat16, device="cuda")
    dC = torch.zeros((M, N), device="cuda")
    a = _args(dA, dW, None, dC, M, N, K, 0, 0, 1.0)
    assert L.nemo_gemm_noalloc(C.byref(a), None) != 0
    assert "rows" in _err()
    a.M, a.a_fmt = 8, 0
    assert L.nemo_gemm_noalloc(C.byref(a), None) != 0
    assert "BF16X2" in _err()
    # the checks nemo_gemm makes, all on the host before any launch
    a = _args(dA, dW, None, dC, 8, N, K, 0, 0, 1.0)
    a.C = None
    assert L.nemo_gemm_noalloc(C.byref(a), None) != 0
    assert "null pointer" in _err()
    a = _args(dA, dW, None, dC, 8, N, K, 0, 1, 1.0)
    a.c_fmt = 1
    assert L.nemo_gemm_noalloc(C.byref(a), None) != 0
    assert "accumulate" in _err()
    a = _args(dA, dW, None, dC, 8, 129, K, 3, 0, 1.0)
    assert L.nemo_gemm_noalloc(C.byref(a), None) != 0
    assert "even N" in _err()
    a = _args(dA, dW, None, dC, 0, N, K, 0, 0, 1.0)
    assert L.nemo_gemm_noalloc(C.byref(a), None) == 0  # no rows: nothing to do, as nemo_gemm
