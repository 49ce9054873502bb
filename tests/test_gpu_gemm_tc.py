"""The tcgen05 tensor-core GEMM (activations as bf16 hi/lo planes) against the oracle GEMM, for
row counts from a single stream (split-K weight streaming) to large batches, every epilogue."""
import numpy as np
import pytest

import oracle as orc
from parity import rel_err
from test_gpu_kernels import BF16X2_TOL, bf16, run_gemm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M", [1, 7, 16, 17, 40, 64, 100, 128, 200, 600])
@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_tc_gemm_epilogues(M, act):
    rng = np.random.default_rng(1000 + M * 4 + act)
    N, K = 256, 320
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    C0 = rng.standard_normal((M, N // 2 if act == 3 else N)).astype(np.float32)
    got = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=2, a_fmt=1)
    ref = orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)
    assert rel_err(got, ref) < BF16X2_TOL


@pytest.mark.parametrize("M", [7, 14, 1792])
@pytest.mark.parametrize("shape", [(3072, 1024), (4096, 1024), (1024, 4096), (2048, 1024), (640, 1024), (2560, 1280), (1024, 4352)])
def test_tc_gemm_model_shapes(M, shape):
    rng = np.random.default_rng(M + sum(shape))
    N, K = shape
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.02)
    got = run_gemm(A, W, kind=2, a_fmt=1)
    assert rel_err(got, orc.gemm(A, W)) < BF16X2_TOL


def test_tc_gemm_glu_model_shape():
    rng = np.random.default_rng(77)
    A = rng.standard_normal((7, 1024)).astype(np.float32)
    W = bf16(rng, (2048, 1024), 0.02)
    got = run_gemm(A, W, act=3, kind=2, a_fmt=1)
    assert rel_err(got, orc.gemm(A, W, act=3)) < BF16X2_TOL


def test_tc_gemm_row_mapping_dynamic_rows():
    rng = np.random.default_rng(19)
    streams, c, N, K, cap, off = 6, 7, 256, 256, 30, 9
    A = rng.standard_normal((streams * c, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    bias = rng.standard_normal((streams, N)).astype(np.float32)
    got = run_gemm(A, W, bias.ravel(), kind=2, a_fmt=1, rpg=c, gstride=cap * N, rowoff=off, crows=streams * cap, bias_gstride=N)
    got = got.reshape(streams, cap, N)
    for s in range(streams):
        assert rel_err(got[s, off:off + c], orc.gemm(A[s * c:(s + 1) * c], W, bias[s])) < BF16X2_TOL
        assert np.all(got[s, :off] == 0) and np.all(got[s, off + c:] == 0)
    got = run_gemm(A[:20], W, kind=2, a_fmt=1, dynM=5)
    assert rel_err(got[:5], orc.gemm(A[:5], W)) < BF16X2_TOL and np.all(got[5:] == 0)


def test_tc_gemm_is_deterministic():
    rng = np.random.default_rng(5)
    A = rng.standard_normal((7, 4096)).astype(np.float32)
    W = bf16(rng, (1024, 4096), 0.02)
    a = run_gemm(A, W, kind=2, a_fmt=1)
    b = run_gemm(A, W, kind=2, a_fmt=1)
    assert np.array_equal(a, b)


# ---- activation-major tiles (kind 5): 128 activation rows x 128/256 weight rows per tile ----

@pytest.mark.parametrize("M", [128, 200, 600, 1792])
@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_tcr_gemm_epilogues(M, act):
    rng = np.random.default_rng(3000 + M * 4 + act)
    N, K = 512, 320
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    C0 = rng.standard_normal((M, N // 2 if act == 3 else N)).astype(np.float32)
    got = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=5, a_fmt=1)
    ref = orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)
    assert rel_err(got, ref) < BF16X2_TOL


@pytest.mark.parametrize("N", [4096, 3072, 1024])
@pytest.mark.parametrize("act", [0, 1, 2])
def test_tcr_gemm_odd_width_tiles(N, act):
    # at 1792 rows the planner takes 208-row weight tiles for N = 4096 (280 tiles: 1.9 rounds of
    # 148 SMs; the last tile holds 144 real rows), 160-row tiles for N = 3072 (280 tiles) and
    # 112-row tiles for N = 1024 (140 tiles, epilogue halves of 64 + 48 columns); bias,
    # activation, alpha and accumulation on every chunk
    rng = np.random.default_rng(51 + act + N)
    M, K = 1792, 320
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    got = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=5, a_fmt=1)
    ref = orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)
    assert rel_err(got, ref) < BF16X2_TOL


@pytest.mark.parametrize("shape", [(3072, 1024), (4096, 1024), (1024, 4096), (2048, 1024), (640, 1024), (1025, 640), (1024, 4352)])
def test_tcr_gemm_model_shapes(shape):
    rng = np.random.default_rng(11 + sum(shape))
    N, K = shape
    A = rng.standard_normal((1792, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.02)
    got = run_gemm(A, W, kind=5, a_fmt=1)
    assert rel_err(got, orc.gemm(A, W)) < BF16X2_TOL


@pytest.mark.parametrize("act", [0, 3])
def test_tcr_gemm_split_k(act):
    # one or two tiles: the k-blocks are split over many CTAs and reduced in a fixed order
    rng = np.random.default_rng(23 + act)
    M, N, K = 130, 256, 4096
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.02)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    C0 = rng.standard_normal((M, N // 2 if act == 3 else N)).astype(np.float32)
    got = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=5, a_fmt=1)
    assert rel_err(got, orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)) < BF16X2_TOL
    again = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=5, a_fmt=1)
    assert np.array_equal(got, again)


def test_tcr_gemm_row_mapping_dynamic_rows():
    rng = np.random.default_rng(29)
    streams, c, N, K, cap, off = 40, 7, 256, 256, 30, 9
    A = rng.standard_normal((streams * c, K)).astype(np.float32)
    W = bf16(rng, (N, K))
    bias = rng.standard_normal((streams, N)).astype(np.float32)
    got = run_gemm(A, W, bias.ravel(), kind=5, a_fmt=1, rpg=c, gstride=cap * N, rowoff=off, crows=streams * cap, bias_gstride=N)
    got = got.reshape(streams, cap, N)
    for s in range(streams):
        assert rel_err(got[s, off:off + c], orc.gemm(A[s * c:(s + 1) * c], W, bias[s])) < BF16X2_TOL
        assert np.all(got[s, :off] == 0) and np.all(got[s, off + c:] == 0)
    got = run_gemm(A, W, kind=5, a_fmt=1, dynM=150)
    assert rel_err(got[:150], orc.gemm(A[:150], W)) < BF16X2_TOL and np.all(got[150:] == 0)


def test_tcr_matches_weight_major_tiles():
    rng = np.random.default_rng(31)
    A = rng.standard_normal((448, 1024)).astype(np.float32)
    W = bf16(rng, (2048, 1024), 0.02)
    for act in (1, 3):
        a = run_gemm(A, W, act=act, kind=4, a_fmt=1)
        b = run_gemm(A, W, act=act, kind=5, a_fmt=1)
        assert rel_err(b, a) < 1e-5  # same products, fp32 sums in a different order (k-splits differ)


# ---- stream-K schedule (kind 6): every CTA an equal share of all tiles' k-blocks ----

@pytest.mark.parametrize("M", [128, 200, 600, 1792])
@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_tcr_stream_k_epilogues(M, act):
    rng = np.random.default_rng(5000 + M * 4 + act)
    N, K = 512, 1280
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.03)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    C0 = rng.standard_normal((M, N // 2 if act == 3 else N)).astype(np.float32)
    got = run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=6, a_fmt=1)
    ref = orc.gemm(A, W, b, C0=C0, act=act, accumulate=True, alpha=0.5)
    assert rel_err(got, ref) < BF16X2_TOL
    # pieces are summed in slot order: the result does not depend on which piece finishes last
    assert np.array_equal(got, run_gemm(A, W, b, C0, act=act, acc=1, alpha=0.5, kind=6, a_fmt=1))


@pytest.mark.parametrize("shape", [(3072, 1024), (4096, 1024), (1024, 4096), (2048, 1024), (1024, 1024), (1025, 640)])
def test_tcr_stream_k_model_shapes(shape):
    rng = np.random.default_rng(17 + sum(shape))
    N, K = shape
    A = rng.standard_normal((1792, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.02)
    got = run_gemm(A, W, kind=6, a_fmt=1)
    assert rel_err(got, orc.gemm(A, W)) < BF16X2_TOL
    assert rel_err(got, run_gemm(A, W, kind=5, a_fmt=1)) < 1e-5


def test_tcr_stream_k_row_mapping():
    rng = np.random.default_rng(37)
    streams, c, N, K, cap, off = 40, 7, 256, 1024, 30, 9
    A = rng.standard_normal((streams * c, K)).astype(np.float32)
    W = bf16(rng, (N, K), 0.03)
    bias = rng.standard_normal((streams, N)).astype(np.float32)
    got = run_gemm(A, W, bias.ravel(), kind=6, a_fmt=1, rpg=c, gstride=cap * N, rowoff=off, crows=streams * cap, bias_gstride=N)
    got = got.reshape(streams, cap, N)
    for s in range(streams):
        assert rel_err(got[s, off:off + c], orc.gemm(A[s * c:(s + 1) * c], W, bias[s])) < BF16X2_TOL
        assert np.all(got[s, :off] == 0) and np.all(got[s, off + c:] == 0)
