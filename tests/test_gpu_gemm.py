"""Tensor-core Q4_0 x f16 GEMM (pb_q4_gemm, the batched configuration), both
the fused-dequant kernel (M < 512) and the TMA-fed kernel over f16 copies.

Two references: the same f16-rounded operands summed in f64 (the only
difference left is the f32 accumulation order on the tensor cores: rtol 2e-5
of the output scale), and the reference's exact f32 arithmetic from the
oracle (the per-row WASM matvec; f16 operand rounding: rtol 4e-3).  The
three-term form (pb_q4_gemm_ex, pb_q4_gemm_hl: hi/lo operand pairs) meets
the reference within the accumulation bound alone."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
f32 = np.float32
RTOL_SAME_OPERANDS = 2e-5
RTOL_VS_REFERENCE = 4e-3


def rand_q4_0(rng, N, K):
    raw = rng.integers(0, 256, N * (K // 32) * 18, dtype=np.uint8)
    d = (rng.standard_normal(N * (K // 32)) * 0.01).astype(np.float16).view(np.uint8).reshape(-1, 2)
    raw.reshape(-1, 18)[:, :2] = d
    return raw


def wasm_scales(blk):
    """The block scales decoded as the reference decodes them (wasm-q4.js:88-109):
    a zero exponent (zero or subnormal) is +0."""
    bits = blk[:, :, :2].copy().view(np.uint16)[:, :, 0]
    d = bits.view(np.float16).astype(np.float64)
    return np.where((bits & 0x7C00) == 0, 0.0, d)


def dequant_f16(raw, N, K):
    blk = raw.reshape(N, K // 32, 18)
    d = wasm_scales(blk).astype(np.float32)
    q = blk[:, :, 2:]
    lo = (q & 15).astype(np.int32) - 8
    hi = (q >> 4).astype(np.int32) - 8
    w = np.concatenate([lo, hi], axis=2).astype(np.float32) * d[:, :, None]
    return w.reshape(N, K).astype(np.float16).astype(np.float64)


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (37, 200, 2048), (128, 256, 128), (300, 1000, 576),
                                   (64, 3072, 2048), (256, 2048, 8192), (130, 16384, 2048),
                                   # M >= 512: f16 copies + TMA-fed pipeline (K % 64 == 0)
                                   (512, 256, 2048), (1000, 3072, 2048), (600, 2048, 8192), (4096, 384, 576),
                                   (513, 300, 1056)])
def test_q4_gemm(native, ctx, oracle, M, N, K):
    rng = np.random.default_rng(M * 131 + N + K)
    raw = rand_q4_0(rng, N, K)
    X = rng.standard_normal((M, K)).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx = ctx.to_device(X)
    dc = ctx.alloc(M * N * 4)
    ctx._check(native.lib().pb_q4_gemm(ctx.h, m.h, dx.ptr, M, K, dc.ptr, N))
    ctx.sync()
    assert ctx.device_error() == 0
    C = dc.download(count=M * N).reshape(M, N)
    ref16 = X.astype(np.float16).astype(np.float64) @ dequant_f16(raw, N, K).T
    scale = np.max(np.abs(ref16))
    assert np.max(np.abs(C - ref16)) <= RTOL_SAME_OPERANDS * scale
    rows = [0, M // 2, M - 1]
    exact = np.stack([oracle.q4_0_matvec(X[i], raw, N, K) for i in rows])
    assert np.max(np.abs(C[rows] - exact)) <= RTOL_VS_REFERENCE * np.max(np.abs(exact))


@pytest.mark.parametrize("M", [8, 600])
def test_q4_gemm_table_layout(native, ctx, M):
    """The batched LM head runs the GEMM over the head-table layout: same bits as the row layout."""
    rng = np.random.default_rng(M)
    N, K = 1000, 256
    raw = rand_q4_0(rng, N, K)
    X = rng.standard_normal((M, K)).astype(f32)
    L = native.lib()
    dx = ctx.to_device(X)
    outs = []
    for t in (native.TYPE_Q4_0, native.TYPE_Q4_0 | native.QMAT_TABLE):
        m = native.QMat(ctx, t, raw, N, K)
        dc = ctx.alloc(M * N * 4)
        ctx._check(L.pb_q4_gemm(ctx.h, m.h, dx.ptr, M, K, dc.ptr, N))
        ctx.sync()
        outs.append(dc.download(count=M * N))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_q4_gemm_rejects(native, ctx):
    rng = np.random.default_rng(1)
    raw = rand_q4_0(rng, 64, 64)
    L = native.lib()
    dx, dc = ctx.alloc(64 * 64 * 4), ctx.alloc(64 * 64 * 4)
    rows = native.QMat(ctx, native.TYPE_Q4_0, raw, 64, 64)
    assert L.pb_q4_gemm(ctx.h, rows.h, dx.ptr, 4, 63, dc.ptr, 64) == native.PB_ERR_ARG  # ldx < K
    q8 = native.QMat(ctx, native.TYPE_Q8_0, np.zeros(64 * 2 * 34, np.uint8), 64, 64)
    assert L.pb_q4_gemm(ctx.h, q8.h, dx.ptr, 4, 64, dc.ptr, 64) == native.PB_ERR_ARG  # Q4_0 only


@pytest.mark.parametrize("M,N,K,table", [(1, 128, 64, False), (3, 200, 2048, False), (64, 3072, 2048, False),
                                         (17, 16384, 2048, False), (64, 2048, 8192, False), (40, 1000, 256, True),
                                         (64, 4104, 2048, True)])
def test_q4_gemm_f16_decode_size_same_bits(native, ctx, M, N, K, table):
    """pb_q4_gemm_f16 at M <= 64 (the warp-specialised kernel: TMA-fed payload
    and activations, half-precision dequant) gives the same bits as
    pb_q4_gemm (the fused kernel) on activations already rounded to f16: the
    same weight values, the same K-step order.  Both layouts."""
    rng = np.random.default_rng(M * 7 + N + K)
    raw = rand_q4_0(rng, N, K)
    X = rng.standard_normal((M, K)).astype(np.float16)
    L = native.lib()
    m = native.QMat(ctx, native.TYPE_Q4_0 | (native.QMAT_TABLE if table else 0), raw, N, K)
    dx32 = ctx.to_device(X.astype(f32))
    dx16 = ctx.to_device(X)
    c32, c16 = ctx.alloc(M * N * 4), ctx.alloc(M * N * 4)
    ctx._check(L.pb_q4_gemm(ctx.h, m.h, dx32.ptr, M, K, c32.ptr, N))
    ctx._check(L.pb_q4_gemm_f16(ctx.h, m.h, dx16.ptr, M, c16.ptr, N))
    ctx.sync()
    assert ctx.device_error() == 0
    a, b = c32.download(count=M * N), c16.download(count=M * N)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"max abs diff {np.max(np.abs(a - b)):.3e}"
    ref16 = X.astype(np.float64) @ dequant_f16(raw, N, K).T
    assert np.max(np.abs(b.reshape(M, N) - ref16)) <= RTOL_SAME_OPERANDS * np.max(np.abs(ref16))


def exact_w(raw, N, K):
    """The dequantized weights exactly ((q - 8) * d in f64, d decoded the reference's way)."""
    blk = raw.reshape(N, K // 32, 18)
    d = wasm_scales(blk)
    q = blk[:, :, 2:]
    lo = (q & 15).astype(np.float64) - 8
    hi = (q >> 4).astype(np.float64) - 8
    return (np.concatenate([lo, hi], axis=2) * d[:, :, None]).reshape(N, K)


def hl_rows(X):
    """Rows of K f32 values as 2K halves: per 64-wide group its hi halves, then its lo halves."""
    M, K = X.shape
    hi = X.astype(np.float16)
    lo = (X - hi.astype(f32)).astype(np.float16)
    return np.stack([hi.reshape(M, K // 64, 64), lo.reshape(M, K // 64, 64)], axis=2).reshape(M, 2 * K)


# three-term products: the operands carry about 22 bits, so what is left is
# the tensor cores' f32 accumulation, three MMAs per 16-wide K slice; its
# error grows about linearly with K (measured 7e-6 of the output scale at
# K = 2048, 3.2e-5 at K = 8192)
RTOL_THREE_TERMS = 5e-5


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (37, 200, 2048), (64, 3072, 2048), (256, 2048, 8192),
                                   (130, 16384, 2048), (512, 256, 2048), (1000, 3072, 2048), (600, 2048, 8192),
                                   (513, 300, 1088)])
def test_q4_gemm_three_terms(native, ctx, oracle, M, N, K):
    """pb_q4_gemm_ex(terms = 3) against the exact product of the f32
    activations and the exact weight values, and against the reference's
    f32 matvec (the oracle) on three rows."""
    rng = np.random.default_rng(M * 13 + N + K)
    raw = rand_q4_0(rng, N, K)
    X = rng.standard_normal((M, K)).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx = ctx.to_device(X)
    dc = ctx.alloc(M * N * 4)
    ctx._check(native.lib().pb_q4_gemm_ex(ctx.h, m.h, dx.ptr, M, K, dc.ptr, N, 3))
    ctx.sync()
    assert ctx.device_error() == 0
    C = dc.download(count=M * N).reshape(M, N)
    ref = X.astype(np.float64) @ exact_w(raw, N, K).T
    scale = np.max(np.abs(ref))
    err = np.max(np.abs(C - ref)) / scale
    rows = [0, M // 2, M - 1]
    exact = np.stack([oracle.q4_0_matvec(X[i], raw, N, K) for i in rows])
    err_ref = np.max(np.abs(C[rows] - exact)) / np.max(np.abs(exact))
    print(f"[three-term] M={M} N={N} K={K}: vs exact {err:.3e}, vs reference {err_ref:.3e}")
    assert err <= RTOL_THREE_TERMS
    assert err_ref <= RTOL_THREE_TERMS


@pytest.mark.parametrize("M,N,K,table", [(3, 200, 2048, False), (64, 3072, 2048, False), (64, 2048, 8192, False),
                                         (40, 1000, 256, True), (600, 2048, 2048, False), (513, 300, 1088, False)])
def test_q4_gemm_hl_same_bits(native, ctx, M, N, K, table):
    """Activations given as hi/lo pairs (the batched producers' layout) give
    the same bits as the three-term product of the f32 activations: at
    M <= 64 the warp-specialised kernel against the fused one, at M >= 512
    the TMA kernel against itself after the device-side split."""
    rng = np.random.default_rng(M * 5 + N + K)
    raw = rand_q4_0(rng, N, K)
    X = rng.standard_normal((M, K)).astype(f32)
    L = native.lib()
    m = native.QMat(ctx, native.TYPE_Q4_0 | (native.QMAT_TABLE if table else 0), raw, N, K)
    dx32 = ctx.to_device(X)
    dxhl = ctx.to_device(hl_rows(X))
    c32, chl = ctx.alloc(M * N * 4), ctx.alloc(M * N * 4)
    ctx._check(L.pb_q4_gemm_ex(ctx.h, m.h, dx32.ptr, M, K, c32.ptr, N, 3))
    ctx._check(L.pb_q4_gemm_hl(ctx.h, m.h, dxhl.ptr, M, chl.ptr, N))
    ctx.sync()
    assert ctx.device_error() == 0
    a, b = c32.download(count=M * N), chl.download(count=M * N)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"max abs diff {np.max(np.abs(a - b)):.3e}"


def test_q4_gemm_ex_rejects(native, ctx):
    rng = np.random.default_rng(3)
    m = native.QMat(ctx, native.TYPE_Q4_0, rand_q4_0(rng, 64, 64), 64, 64)
    dx, dc = ctx.alloc(100 * 64 * 4), ctx.alloc(100 * 64 * 4)
    L = native.lib()
    assert L.pb_q4_gemm_ex(ctx.h, m.h, dx.ptr, 4, 64, dc.ptr, 64, 2) == native.PB_ERR_ARG  # terms 1 or 3
    assert L.pb_q4_gemm_hl(ctx.h, m.h, dx.ptr, 100, dc.ptr, 64) == native.PB_ERR_ARG  # 64 < M < 512


def test_q4_gemm_f16_rejects(native, ctx):
    rng = np.random.default_rng(2)
    m = native.QMat(ctx, native.TYPE_Q4_0, rand_q4_0(rng, 64, 64), 64, 64)
    dx, dc = ctx.alloc(100 * 64 * 2), ctx.alloc(100 * 64 * 4)
    assert native.lib().pb_q4_gemm_f16(ctx.h, m.h, dx.ptr, 100, dc.ptr, 64) == native.PB_ERR_ARG  # 64 < M < 512
