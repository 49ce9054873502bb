"""Each C-ABI kernel (include/nemo_gpu.h) against the oracle's restatement of the Metal kernel it
replaces, on seeded inputs, through the library's own entry points (device memory from torch)."""
import ctypes as C

import numpy as np
import pytest

import nemoasr_b200 as nb
import oracle as orc
from parity import rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FP32_TOL = 2e-5   # fp32 math, different summation order
BF16X2_TOL = 2e-4  # activations carried as bf16 hi/lo planes (16-bit mantissa) into tensor cores


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


_keep = []


def p(t):
    """Device pointer of t; t stays referenced until the test ends (a temporary tensor would be
    freed, and its memory reused, before the kernel runs)."""
    if t is None:
        return None
    _keep.append(t)
    return C.c_void_p(t.data_ptr())


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    torch.cuda.synchronize()
    _keep.clear()


def bf16(rng, shape, std=0.05):
    f = (rng.standard_normal(shape) * std).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def split_bf16x2(x):
    """fp32 -> (hi, lo) bf16 planes as the producers write them (round to nearest even)."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    hi = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r = (x - (hi.astype(np.uint32) << 16).view(np.float32)).astype(np.float32)
    ur = r.view(np.uint32).astype(np.uint64)
    lo = ((ur + 0x7FFF + ((ur >> 16) & 1)) >> 16).astype(np.uint16)
    return hi, lo


def run_gemm(A, W, bias=None, C0=None, act=0, acc=0, alpha=1.0, kind=0, a_fmt=0, rpg=0, gstride=0, rowoff=None, ldc=None,
             crows=None, dynM=None, bias_gstride=0):
    M, K = A.shape
    N = W.shape[0]
    nout = N // 2 if act == 3 else N
    if a_fmt == 1:
        hi, lo = split_bf16x2(A)
        dA = dev(np.concatenate([hi.ravel(), lo.ravel()]))
    else:
        dA = dev(A)
    dW = dev(W)
    db = dev(bias) if bias is not None else None
    ldc = ldc or nout
    dC = dev(C0 if C0 is not None else np.zeros((crows or M, ldc), np.float32))
    a = nb.GemmArgs()
    a.A, a.lda, a.a_fmt, a.a_plane = dA.data_ptr(), K, a_fmt, M * K
    a.W, a.ldw = dW.data_ptr(), K
    a.bias = db.data_ptr() if db is not None else None
    a.bias_gstride = bias_gstride
    a.C, a.ldc, a.c_fmt = dC.data_ptr(), ldc, 0
    a.M, a.N, a.K, a.act, a.accumulate, a.alpha = M, N, K, act, acc, alpha
    a.rpg, a.gstride = rpg, gstride
    keep = []
    if rowoff is not None:
        r = dev(np.array([rowoff], np.int32)); keep.append(r); a.rowoff = r.data_ptr()
    if dynM is not None:
        r = dev(np.array([dynM], np.int32)); keep.append(r); a.dynM = r.data_ptr()
    nb.check(nb.api().nemo_gemm_forced(C.byref(a), kind, None), "nemo_gemm")
    return host(dC)


@pytest.mark.parametrize("M", [1, 2, 7, 14, 16])
@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_gemm_streaming_matches_oracle(M, act):
    rng = np.random.default_rng(M * 10 + act)
    N, K = 512, 1024
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    C0 = rng.standard_normal((M, N // 2 if act == 3 else N)).astype(np.float32)
    got = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=1)
    ref = orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)
    assert rel_err(got, ref) < FP32_TOL


@pytest.mark.parametrize("shape", [(3072, 1024), (4096, 1024), (1024, 4096), (2048, 1024), (1024, 1024), (1024, 4352), (2560, 1280)])
def test_gemm_streaming_baseline_shapes(shape):
    rng = np.random.default_rng(sum(shape))
    N, K = shape
    A = rng.standard_normal((7, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.02)
    got = run_gemm(A, W, kind=1)
    assert rel_err(got, orc.gemm(A, W)) < FP32_TOL


@pytest.mark.parametrize("M", [17, 64, 200])
@pytest.mark.parametrize("act", [0, 2, 3])
def test_gemm_many_rows_fp32(M, act):
    rng = np.random.default_rng(M + act)
    N, K = 256, 320
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    b = rng.standard_normal(N).astype(np.float32)
    got = run_gemm(A, W, b, act=act, kind=3)
    assert rel_err(got, orc.gemm(A, W, b, act=act)) < FP32_TOL


def test_gemm_row_mapping_and_dynamic_rows():
    """Rows grouped per stream, written at a device row offset inside each stream's cache (the
    q|k|v append of src/encoder.c:160), per-stream bias, and a device-side row count."""
    rng = np.random.default_rng(9)
    streams, c, N, K, cap, off = 3, 5, 128, 256, 20, 7
    A = rng.standard_normal((streams * c, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    bias = rng.standard_normal((streams, N)).astype(np.float32)
    got = run_gemm(A, W, bias.ravel(), act=0, kind=0, rpg=c, gstride=cap * N, rowoff=off, crows=streams * cap, bias_gstride=N)
    got = got.reshape(streams, cap, N)
    for s in range(streams):
        ref = orc.gemm(A[s * c:(s + 1) * c], W, bias[s])
        assert rel_err(got[s, off:off + c], ref) < FP32_TOL
        assert np.all(got[s, :off] == 0) and np.all(got[s, off + c:] == 0)
    got = run_gemm(A[:9], W, dynM=4, kind=1)
    assert rel_err(got[:4], orc.gemm(A[:4], W)) < FP32_TOL and np.all(got[4:] == 0)


@pytest.mark.parametrize("D,M", [(256, 9), (1024, 9), (1024, 1795)])
def test_layernorms(D, M):
    # M = 1795: a batch-sized row count (one block per row)
    rng = np.random.default_rng(D + M)
    X = (rng.standard_normal((M, D)) * 3 + 1).astype(np.float32)
    g1, b1, g2, b2 = (rng.standard_normal(D).astype(np.float32) for _ in range(4))
    dX, dY1, dY2 = dev(X), dev(np.zeros_like(X)), dev(np.zeros_like(X))
    L = nb.api()
    nb.check(L.nemo_layernorm(p(dX), p(dev(g1)), p(dev(b1)), p(dY1), 0, 0, M, D, C.c_float(1e-5), None))
    assert rel_err(host(dY1), orc.layernorm(X, g1, b1)) < FP32_TOL
    nb.check(L.nemo_layernorm2(p(dX), p(dev(g1)), p(dev(b1)), p(dev(g2)), p(dev(b2)), p(dY1), p(dY2), 0, 0, M, D, C.c_float(1e-5), None))
    r1, r2 = orc.layernorm2(X, g1, b1, g2, b2)
    assert rel_err(host(dY1), r1) < FP32_TOL and rel_err(host(dY2), r2) < FP32_TOL


# c <= 8: keys as the MMA's 16-row side (attention8_kernel); c > 8: queries as the 16-row side.
# (8, 64, 72): the window fills Lmax (position rows from 0); (8, 88, 96) and (16, 80, 96): the
# largest window (96 keys; 103 position rows, so the key warps also form position tiles 4-6)
@pytest.mark.parametrize("c,cache_len,Lmax", [(7, 56, 72), (1, 0, 72), (14, 40, 72), (16, 56, 72), (3, 5, 72), (8, 64, 72), (8, 88, 96), (16, 80, 96)])
def test_attention_over_cache(c, cache_len, Lmax):
    rng = np.random.default_rng(c * 100 + cache_len)
    H, dh, streams = 8, 128, 2
    D = H * dh
    cap, pos = 120, cache_len + 11
    kv = rng.standard_normal((streams, cap, 3 * D)).astype(np.float32)
    P = rng.standard_normal((2 * Lmax - 1, D)).astype(np.float32)
    bu, bv = rng.standard_normal(D).astype(np.float32) * 0.1, rng.standard_normal(D).astype(np.float32) * 0.1
    dkv = dev(kv)
    O = dev(np.zeros((streams * c, D), np.float32))
    dpos, dcl = dev(np.array([pos], np.int32)), dev(np.array([cache_len], np.int32))
    base = dkv.data_ptr()
    nb.check(nb.api().nemo_attention_rel(C.c_void_p(base), 3 * D, cap * 3 * D, C.c_void_p(base + 4 * D), C.c_void_p(base + 8 * D), 3 * D,
                                         cap * 3 * D, p(dpos), p(dcl), p(dev(P)), p(dev(bu)), p(dev(bv)), p(O), 0, 0, c * D, streams, c, Lmax,
                                         H, dh, D, C.c_float(1 / np.sqrt(128.0)), None))
    got = host(O).reshape(streams, c, D)
    L = cache_len + c
    for s in range(streams):
        win = kv[s, pos - cache_len:pos + c]
        ref = orc.attention_rel(kv[s, pos:pos + c, :D], win[:, D:2 * D], win[:, 2 * D:], P, bu, bv, c, L, Lmax, H, dh)
        # score and value products on the tensor cores with both operands split into bf16 hi + lo
        assert rel_err(got[s], ref) < BF16X2_TOL


@pytest.mark.parametrize("c", [1, 7, 8, 14])  # c <= 8: one block per stream; 14: one block per row
def test_dwconv_ln_silu(c):
    rng = np.random.default_rng(4 + c)
    streams, D, cap, pos = 3, 1024, 40, 20
    din = rng.standard_normal((streams, cap, D)).astype(np.float32)
    W = rng.standard_normal((D, 9)).astype(np.float32) * 0.3
    g, b = rng.standard_normal(D).astype(np.float32), rng.standard_normal(D).astype(np.float32)
    Y = dev(np.zeros((streams * c, D), np.float32))
    nb.check(nb.api().nemo_dwconv_ln_silu(p(dev(din)), cap * D, p(dev(np.array([pos], np.int32))), p(dev(W)), p(dev(g)), p(dev(b)), p(Y), 0, 0,
                                          streams, c, D, 9, C.c_float(1e-5), None))
    got = host(Y).reshape(streams, c, D)
    for s in range(streams):
        assert rel_err(got[s], orc.dwconv_ln_silu(din[s, pos - 8:pos + c], W, g, b, c)) < FP32_TOL


def test_subsampling_convs_and_flatten():
    rng = np.random.default_rng(6)
    streams, T, F, CH = 2, 72, 128, 64
    X = rng.standard_normal((streams, T, F)).astype(np.float32)
    W0, b0 = rng.standard_normal(CH * 9).astype(np.float32), rng.standard_normal(CH).astype(np.float32)
    W2, b2 = rng.standard_normal(CH * 9).astype(np.float32), rng.standard_normal(CH).astype(np.float32)
    T1, F1 = T // 2 + 1, F // 2 + 1
    T2, F2 = T1 // 2 + 1, F1 // 2 + 1
    Y0 = dev(np.zeros((streams, T1, F1, CH), np.float32))
    L = nb.api()
    nb.check(L.nemo_conv2d_c1_s2_relu(p(dev(X)), T * F, p(dev(W0)), p(dev(b0)), p(Y0), streams, T, F, T1, F1, CH, None))
    y0 = host(Y0)
    Y1 = dev(np.zeros((streams, T2, F2, CH), np.float32))
    nb.check(L.nemo_dwconv2d_s2(p(Y0), p(dev(W2)), p(dev(b2)), p(Y1), streams, T1, F1, T2, F2, CH, None))
    y1 = host(Y1)
    lo, c = 2, 7
    Z = dev(np.zeros((streams * c, CH * F2), np.float32))
    nb.check(L.nemo_flatten_rows(p(Y1), p(Z), p(dev(np.array([lo], np.int32))), streams, T2, F2, CH, c, None))
    z = host(Z)
    for s in range(streams):
        r0 = orc.conv2d_c1_s2_relu(X[s], W0, b0)
        assert rel_err(y0[s], r0) < FP32_TOL
        r1 = orc.dwconv2d_s2(r0, W2, b2)
        assert rel_err(y1[s], r1) < FP32_TOL
        assert rel_err(z[s * c:(s + 1) * c], orc.flatten_cf(r1)[lo:lo + c]) < FP32_TOL


def test_lstm_cell_and_joint_argmax():
    rng = np.random.default_rng(8)
    H = 640
    gates = rng.standard_normal((3, 4 * H)).astype(np.float32)
    c_in = rng.standard_normal((3, H)).astype(np.float32)
    dco, dho = dev(np.zeros((3, H), np.float32)), dev(np.zeros((3, H), np.float32))
    nb.check(nb.api().nemo_lstm_cell(p(dev(gates)), p(dev(c_in)), p(dco), p(dho), 3, H, None))
    for r in range(3):
        co, ho = orc.lstm_cell(gates[r], c_in[r])
        assert rel_err(host(dco)[r], co) < 1e-6 and rel_err(host(dho)[r], ho) < 1e-6
    V, JH, rows = 1025, 640, 5
    W = bf16(rng, (V, JH), 0.02)
    bias = (rng.standard_normal(V) * 0.02).astype(np.float32)
    enc = rng.standard_normal((rows, JH)).astype(np.float32)
    pred = rng.standard_normal(JH).astype(np.float32)
    di, dv = dev(np.zeros(rows, np.int32)), dev(np.zeros(rows, np.float32))
    nb.check(nb.api().nemo_joint_argmax(p(dev(enc)), JH, p(dev(pred)), 0, p(dev(W)), p(dev(bias)), V, JH, rows, p(di), p(dv), None))
    ri, rv, rm = orc.joint_argmax(enc, pred, W, bias)
    gi, gv = host(di), host(dv)
    for r in range(rows):
        assert gi[r] == ri[r] or rm[r] < 1e-3
        assert abs(gv[r] - rv[r]) < 1e-4 * max(1.0, abs(rv[r]))


@pytest.mark.parametrize("T,C", [(72, 64), (56, 256), (17, 32)])
def test_subsample_front_fused(T, C):
    rng = np.random.default_rng(T + C)
    streams, F = 2, 128
    X = rng.standard_normal((streams, T + 3, F)).astype(np.float32)  # padded stride like the engine window
    W0, b0 = rng.standard_normal(C * 9).astype(np.float32), rng.standard_normal(C).astype(np.float32)
    W2, b2 = rng.standard_normal(C * 9).astype(np.float32), rng.standard_normal(C).astype(np.float32)
    T1, F1 = T // 2 + 1, F // 2 + 1
    T2, F2 = T1 // 2 + 1, F1 // 2 + 1
    Y = dev(np.zeros((streams, T2, F2, C), np.float32))
    nb.check(nb.api().nemo_subsample_front(p(dev(X)), (T + 3) * F, p(dev(W0)), p(dev(b0)), p(dev(W2)), p(dev(b2)), p(Y), 0, 0, streams, T, F, C,
                                           None))
    y = host(Y)
    for s in range(streams):
        ref = orc.dwconv2d_s2(orc.conv2d_c1_s2_relu(X[s, :T], W0, b0), W2, b2)
        assert rel_err(y[s], ref) < FP32_TOL
