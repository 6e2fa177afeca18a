"""GPU parity of every kernel against the CPU oracle, through the C ABI.

Bit-exact (`bits_equal`) where the kernel reproduces the reference's exact
operation order (Q4 matvecs, heads, f32 / Q8 matmuls, quantizers, RoPE,
decoders); within a stated relative tolerance where the reference sums many
doubles left to right and the kernel uses a tree (norms, softmax, attention).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
f32 = np.float32
# float outputs of double-precision reductions: the tree sum and the
# reference's left-to-right sum differ in the last double bits, which moves
# an f32 result by at most an ulp or two
RTOL_REDUCE = 2e-6


def bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def close(a, b, rtol=RTOL_REDUCE):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = max(np.max(np.abs(b)), 1e-30)
    return np.max(np.abs(a - b)) <= rtol * scale


def dev(ctx, arr):
    return ctx.to_device(np.ascontiguousarray(arr))


def out(ctx, n, dtype=np.float32):
    return ctx.alloc(max(np.dtype(dtype).itemsize * n, 16))


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def rand_q4_0(rng, N, K):
    raw = rng.integers(0, 256, N * (K // 32) * 18, dtype=np.uint8)
    d = (rng.standard_normal(N * (K // 32)) * 0.01).astype(np.float16).view(np.uint8).reshape(-1, 2)
    raw.reshape(-1, 18)[:, :2] = d
    return raw


# ---------------------------------------------------------------------------
# Q4 matvec (wasm-q4.js:118-267), bit-exact
# ---------------------------------------------------------------------------

def test_selftest_kat(native, ctx):
    from purebee_b200 import wasm_q4
    assert wasm_q4.init()
    raw = np.zeros(36, np.uint8)
    raw[1], raw[2:18], raw[19], raw[20:36] = 0x3C, 0x99, 0x40, 0xAA
    assert wasm_q4.q4_0_matvec(np.ones(32, f32), raw, 2, 32).tolist() == [32.0, 128.0]


def test_q4_0_matvec_golden(native, ctx, golden):
    from purebee_b200 import wasm_q4
    for tag in "abc":
        N, K = (int(v) for v in golden[f"q4_0_{tag}_shape"])
        y = wasm_q4.q4_0_matvec(golden[f"q4_0_{tag}_x"], golden[f"q4_0_{tag}_raw"], N, K)
        assert bits_equal(y, golden[f"q4_0_{tag}_y"]), tag


def test_q4_1_matvec_golden(native, ctx, golden):
    from purebee_b200 import wasm_q4
    N, K = (int(v) for v in golden["q4_1_shape"])
    assert bits_equal(wasm_q4.q4_1_matvec(golden["q4_1_x"], golden["q4_1_raw"], N, K), golden["q4_1_y"])


@pytest.mark.parametrize("N,K", [(1, 32), (31, 64), (100, 320), (512, 2048), (2048, 2048), (3072, 2048),
                                 (2048, 8192), (16384, 2048), (576, 576), (192, 576), (576, 1536)])
def test_q4_0_matvec_shapes(native, ctx, oracle, N, K):
    rng = np.random.default_rng(N * 7 + K)
    x = rng.standard_normal(K).astype(f32)
    raw = rand_q4_0(rng, N, K)
    from purebee_b200 import wasm_q4
    assert bits_equal(wasm_q4.q4_0_matvec(x, raw, N, K), oracle.q4_0_matvec(x, raw, N, K))


def test_q4_0_matvec_special_scales(native, ctx, oracle):
    """Zero, negative zero, subnormal (flushed by the WASM decode) and exponent-31 scales."""
    rng = np.random.default_rng(11)
    N, K = 64, 256
    raw = rand_q4_0(rng, N, K)
    flat = raw.reshape(-1, 18)
    flat[0::5, 0:2] = [0x00, 0x00]
    flat[1::5, 0:2] = [0x00, 0x80]
    flat[2::5, 0:2] = [0x37, 0x02]
    flat[3::7, 0:2] = [0x00, 0x7C]
    x = rng.standard_normal(K).astype(f32)
    from purebee_b200 import wasm_q4
    assert bits_equal(wasm_q4.q4_0_matvec(x, raw, N, K), oracle.q4_0_matvec(x, raw, N, K))


@pytest.fixture
def exact_mode(native, ctx):
    """The resident matvec in the reference's exact lane order for one test."""
    ctx.set_matvec_mode(native.MATVEC_EXACT)
    yield
    ctx.set_matvec_mode(native.MATVEC_FAST)


def test_resident_matvec_row_split(native, ctx, oracle, exact_mode):
    """Rows split like thread-pool.js:174-203 give the same bits as one call,
    and in the exact mode the reference's bits."""
    rng = np.random.default_rng(12)
    N, K = 1024, 2048
    raw = rand_q4_0(rng, N, K)
    x = rng.standard_normal(K).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx, dy = dev(ctx, x), out(ctx, N)
    L = native.lib()
    for r0, rows in [(0, 256), (256, 504), (760, 8), (768, 256)]:
        ctx._check(L.pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, r0, rows))
    ctx.sync()
    assert bits_equal(dy.download(count=N), oracle.q4_0_matvec(x, raw, N, K))
    assert bits_equal(m.gguf_bytes(), raw)  # device layout round trip


# the fast resident matvec: exact (q - 8) * x products summed with one FMA
# per weight in another order; per-op bar of the north star is an f32
# relative tolerance, this is far inside it
RTOL_MATVEC_FAST = 2e-6
# the fast mode's decode attention: f32 dots, exponentials and sums where the
# reference uses double
RTOL_ATTN_FAST = 5e-6


@pytest.fixture(params=["f32", "int8", "tcgen05"])
def fast_kernel(request, native, ctx):
    """Each fast-mode Q4_0 kernel in turn: the f32 one, the mma.sync int8
    one (taken for every matrix size for the test), and the tcgen05 int8 one
    (off by default; it takes K % 128 == 0, K <= 16384, other shapes fall
    back to the f32 kernel).  The test's matrices are uploaded after the
    switch, so they carry the tcgen05 kernel's copy."""
    ctx.set_mvt(request.param == "tcgen05")
    ctx.set_mvi_min_rows(1 << 30 if request.param != "int8" else 0)
    yield request.param
    ctx.set_mvi_min_rows(32768)
    ctx.set_mvt(False)


@pytest.mark.parametrize("N,K", [(64, 64), (136, 576), (512, 1536), (3072, 2048), (2048, 8192), (16384, 2048),
                                 (1000, 4096), (40, 16384)])
def test_fast_matvec_shapes(native, ctx, oracle, fast_kernel, N, K):
    """Every decode shape of configs[2]/[3] and ragged ones (N not a multiple
    of 8, K with a partial last 32-block chunk): within RTOL_MATVEC_FAST of
    the reference's lane order, and row splits give the same bits as one call."""
    assert ctx.matvec_mode == native.MATVEC_FAST
    rng = np.random.default_rng(N * 7 + K)
    raw = rand_q4_0(rng, N, K)
    x = rng.standard_normal(K).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx, dy, dz = dev(ctx, x), out(ctx, N), out(ctx, N)
    L = native.lib()
    ctx._check(L.pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, 0, 0))
    y = dy.download(count=N)
    assert close(y, oracle.q4_0_matvec(x, raw, N, K), RTOL_MATVEC_FAST)
    step = max(8, (N // 3) // 8 * 8)
    for r0 in range(0, N, step):
        ctx._check(L.pb_qmat_matvec(ctx.h, m.h, dx.ptr, dz.ptr, r0, min(step, N - r0)))
    assert bits_equal(dz.download(count=N), y)


def test_fast_matvec_special_scales(native, ctx, oracle, fast_kernel):
    """Zero, -0, subnormal (decoded as 0 the WASM way) and exponent-31 scales."""
    rng = np.random.default_rng(14)
    N, K = 64, 512
    raw = rand_q4_0(rng, N, K)
    blk = raw.reshape(-1, 18)
    for i, bits in enumerate([0x0000, 0x8000, 0x0001, 0x83FF, 0x7C00, 0xFBFF]):
        blk[i * 7, 0], blk[i * 7, 1] = bits & 0xFF, bits >> 8
    x = rng.standard_normal(K).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx, dy = dev(ctx, x), out(ctx, N)
    ctx._check(native.lib().pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, 0, 0))
    assert close(dy.download(count=N), oracle.q4_0_matvec(x, raw, N, K), RTOL_MATVEC_FAST)


def test_matvec_mode_switch(native, ctx, oracle):
    rng = np.random.default_rng(15)
    N, K = 256, 2048
    raw = rand_q4_0(rng, N, K)
    x = rng.standard_normal(K).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx, dy = dev(ctx, x), out(ctx, N)
    L = native.lib()
    want = oracle.q4_0_matvec(x, raw, N, K)
    for mode in (native.MATVEC_EXACT, native.MATVEC_FAST, native.MATVEC_EXACT):
        ctx.set_matvec_mode(mode)
        ctx._check(L.pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, 0, 0))
        got = dy.download(count=N)
        assert bits_equal(got, want) if mode == native.MATVEC_EXACT else close(got, want, RTOL_MATVEC_FAST)
    ctx.set_matvec_mode(native.MATVEC_FAST)
    assert L.pb_set_matvec_mode(ctx.h, 7) == native.PB_ERR_ARG


def test_matvec_rejects_bad_rows(native, ctx):
    rng = np.random.default_rng(13)
    m = native.QMat(ctx, native.TYPE_Q4_0, rand_q4_0(rng, 64, 64), 64, 64)
    dx, dy = out(ctx, 64), out(ctx, 64)
    rc = native.lib().pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, 12, 32)  # start not a multiple of 8
    assert rc == native.PB_ERR_ARG
    hx, hraw, hy = np.zeros(33, f32), np.zeros(64, np.uint8), np.zeros(4, f32)
    rc = native.lib().pb_q4_0_matvec(ctx.h, native.ptr(hx), native.ptr(hraw), 4, 33, native.ptr(hy))
    assert rc == native.PB_ERR_ARG  # K must be a multiple of 32


# ---------------------------------------------------------------------------
# heads (wasm-q4.js:447-566 batch_dot), bit-exact, with argmax
# ---------------------------------------------------------------------------

def test_lm_head_f32_golden(native, ctx, golden):
    from purebee_b200 import wasm_q4
    assert bits_equal(wasm_q4.lmHead(golden["bd_x"], golden["bd_W"], 37, 70), golden["bd_y"])


@pytest.mark.parametrize("typ,V,D", [("q4_0", 1000, 64), ("q4_0", 128256, 2048), ("q8_0", 4000, 576),
                                     ("q8_0", 49152, 576)])
def test_resident_head(native, ctx, oracle, typ, V, D):
    rng = np.random.default_rng(V + D)
    w = rng.standard_normal(V * D, dtype=np.float32) * np.float32(0.02)
    if typ == "q4_0":
        raw, t = oracle.quantize_gguf_q4_0(w), native.TYPE_Q4_0
        table = oracle.dequant_q4_0(raw, V * D)
    else:
        raw, t = oracle.quantize_gguf_q8_0(w), native.TYPE_Q8_0
        table = oracle.dequant_q8_0(raw, V * D)
    h = rng.standard_normal(D).astype(f32)
    want = oracle.batch_dot(h, table, V, D)
    m = native.QMat(ctx, t | native.QMAT_TABLE, raw, V, D)
    assert bits_equal(m.gguf_bytes(), raw)  # table layout round trip
    dh, dl, di = dev(ctx, h), out(ctx, V), out(ctx, 4, np.int32)
    ctx._check(native.lib().pb_qmat_head(ctx.h, m.h, dh.ptr, dl.ptr, di.ptr))
    ctx.sync()
    assert bits_equal(dl.download(count=V), want)
    assert int(di.download(np.int32, 1)[0]) == oracle.argmax(want)


def test_layouts_are_checked(native, ctx):
    """A matvec matrix is not a head table and vice versa: clean PB_ERR_ARG."""
    rng = np.random.default_rng(14)
    raw = rand_q4_0(rng, 64, 64)
    L = native.lib()
    rows = native.QMat(ctx, native.TYPE_Q4_0, raw, 64, 64)
    table = native.QMat(ctx, native.TYPE_Q4_0 | native.QMAT_TABLE, raw, 64, 64)
    dx, dy = out(ctx, 64), out(ctx, 64)
    assert L.pb_qmat_head(ctx.h, rows.h, dx.ptr, dy.ptr, None) == native.PB_ERR_ARG
    assert L.pb_qmat_matvec(ctx.h, table.h, dx.ptr, dy.ptr, 0, 0) == native.PB_ERR_ARG
    assert bits_equal(rows.gguf_bytes(), table.gguf_bytes())


def test_argmax_ties_nan(native, ctx):
    v = np.array([1.0, np.nan, 3.0, 3.0, -np.inf, 2.0], f32)
    dv, di = dev(ctx, v), out(ctx, 4, np.int32)
    ctx._check(native.lib().pb_argmax(ctx.h, dv.ptr, v.size, di.ptr))
    ctx.sync()
    assert int(di.download(np.int32, 1)[0]) == 2
    v = np.full(7, -np.inf, f32)
    dv = dev(ctx, v)
    ctx._check(native.lib().pb_argmax(ctx.h, dv.ptr, v.size, di.ptr))
    ctx.sync()
    assert int(di.download(np.int32, 1)[0]) == 0


# ---------------------------------------------------------------------------
# quantizers / decoders, bit-exact
# ---------------------------------------------------------------------------

def test_quantizers_golden(native, ctx, golden):
    L = native.lib()
    data = golden["qa_data"]
    n = data.size
    nb = (n + 31) // 32
    dd = dev(ctx, data)
    s, q = out(ctx, nb), out(ctx, nb * 32, np.int8)
    ctx._check(L.pb_quantize_q8a(ctx.h, dd.ptr, n, s.ptr, q.ptr))
    ctx.sync()
    assert bits_equal(s.download(count=nb), golden["q8a_scales"])
    assert bits_equal(q.download(np.int8, nb * 32), golden["q8a_q"])
    deq = out(ctx, n)
    ctx._check(L.pb_dequantize_q8a(ctx.h, s.ptr, q.ptr, n, deq.ptr))
    ctx.sync()
    assert bits_equal(deq.download(count=n), golden["q8a_deq"])
    s4, q4 = out(ctx, nb), out(ctx, nb * 16, np.uint8)
    ctx._check(L.pb_quantize_q4a(ctx.h, dd.ptr, n, s4.ptr, q4.ptr))
    ctx.sync()
    assert bits_equal(s4.download(count=nb), golden["q4a_scales"])
    assert bits_equal(q4.download(np.uint8, nb * 16), golden["q4a_q"])
    ctx._check(L.pb_dequantize_q4a(ctx.h, s4.ptr, q4.ptr, n, deq.ptr))
    ctx.sync()
    assert bits_equal(deq.download(count=n), golden["q4a_deq"])


def test_gguf_encoders_and_decoders(native, ctx, oracle, golden):
    L = native.lib()
    rng = np.random.default_rng(21)
    x = np.concatenate([golden["gg_x"], (rng.standard_normal(32 * 300) * 0.02).astype(f32)])
    x[300:310] = 0.0
    dx = dev(ctx, x)
    for typ, bb, enc, dec in [(native.TYPE_Q4_0, 18, oracle.quantize_gguf_q4_0, oracle.dequant_q4_0),
                              (native.TYPE_Q8_0, 34, oracle.quantize_gguf_q8_0, oracle.dequant_q8_0)]:
        raw = out(ctx, x.size // 32 * bb, np.uint8)
        ctx._check(L.pb_gguf_quantize(ctx.h, typ, dx.ptr, x.size, raw.ptr))
        ctx.sync()
        got = raw.download(np.uint8, x.size // 32 * bb)
        assert bits_equal(got, enc(x))
        deq = out(ctx, x.size)
        ctx._check(L.pb_gguf_dequant(ctx.h, typ, raw.ptr, x.size, deq.ptr))
        ctx.sync()
        assert bits_equal(deq.download(count=x.size), dec(got, x.size))
    raw1 = rng.integers(0, 256, 64 * 20, dtype=np.uint8)
    blk = raw1.reshape(64, 20)
    blk[:, 1] &= 0xBF  # finite f16 scale and min (NaN payloads are not part of the format)
    blk[:, 3] &= 0xBF
    r1 = dev(ctx, raw1)
    deq = out(ctx, 64 * 32)
    ctx._check(L.pb_gguf_dequant(ctx.h, native.TYPE_Q4_1, r1.ptr, 64 * 32, deq.ptr))
    ctx.sync()
    assert bits_equal(deq.download(count=64 * 32), oracle.dequant_q4_1(raw1, 64 * 32))


def test_gguf_q6_k_decode(native, ctx, oracle):
    """gguf.js:317-355 Q6_K on the device: bit for bit with the oracle,
    including zero and subnormal scales and a partial last block."""
    L = native.lib()
    rng = np.random.default_rng(66)
    nblk = 40
    raw = rng.integers(0, 256, nblk * 210, dtype=np.uint8)
    d = (rng.standard_normal(nblk) * 0.02).astype(np.float16)
    d[3], d[4] = np.float16(0.0), np.float16(-6e-8)
    raw.reshape(nblk, 210)[:, 208:210] = d.view(np.uint8).reshape(nblk, 2)
    for n in (nblk * 256, nblk * 256 - 77):
        r = dev(ctx, raw)
        deq = out(ctx, n)
        ctx._check(L.pb_gguf_dequant(ctx.h, 14, r.ptr, n, deq.ptr))
        ctx.sync()
        assert bits_equal(deq.download(count=n), oracle.dequant_q6_k(raw, n))


def test_synth_device_equals_host(native, ctx, oracle):
    L = native.lib()
    n = 300001
    d = out(ctx, n)
    ctx._check(L.pb_synth_weights(ctx.h, d.ptr, n, 1234, 5, 0.02))
    ctx.sync()
    assert bits_equal(d.download(count=n), oracle.synth_weights(n, 1234, 5, 0.02))
    ctx._check(L.pb_synth_activation(ctx.h, d.ptr, n, 99, 3))
    ctx.sync()
    assert bits_equal(d.download(count=n), oracle.synth_activation(n, 99, 3))


# ---------------------------------------------------------------------------
# engine ops
# ---------------------------------------------------------------------------

def test_matmul_f32_and_q8a(native, ctx, oracle, golden):
    L = native.lib()
    A, B, bias = golden["mm_A"], golden["mm_B"], golden["mm_bias"]
    C = out(ctx, 21)
    dA, dB, db = dev(ctx, A), dev(ctx, B), dev(ctx, bias)
    ctx._check(L.pb_matmul_f32(ctx.h, dA.ptr, 3, 5, dB.ptr, 7, db.ptr, C.ptr))
    ctx.sync()
    assert bits_equal(C.download(count=21), golden["mm_C"])
    a, s, q = golden["mq_a"], golden["mq_scales"], golden["mq_q"]
    o = out(ctx, 80)
    da, ds, dq = dev(ctx, a), dev(ctx, s), dev(ctx, q)
    ctx._check(L.pb_matmul_q8a(ctx.h, da.ptr, 2, 40, ds.ptr, dq.ptr, 40, None, o.ptr))
    ctx.sync()
    assert bits_equal(o.download(count=80), golden["mq_out"])
    # larger: stories15M shapes
    rng = np.random.default_rng(31)
    for M, K, N in [(1, 288, 768), (16, 768, 288)]:
        a = rng.standard_normal(M * K).astype(f32)
        w = (rng.standard_normal(K * N) * 0.02).astype(f32)
        s, q = oracle.quantize_q8a(w)
        o = out(ctx, M * N)
        da, ds, dq = dev(ctx, a), dev(ctx, s), dev(ctx, q)
        ctx._check(L.pb_matmul_q8a(ctx.h, da.ptr, M, K, ds.ptr, dq.ptr, N, None, o.ptr))
        ctx.sync()
        assert bits_equal(o.download(count=M * N), oracle.matmul_q8(a, M, K, s, q, N))


def test_norms_softmax_activations(native, ctx, oracle, golden):
    L = native.lib()
    x, w, b = golden["op_x"], golden["op_w"], golden["op_b"]
    dx, dw, db, o = dev(ctx, x), dev(ctx, w), dev(ctx, b), out(ctx, x.size)
    ctx._check(L.pb_rmsnorm(ctx.h, dx.ptr, 3, 48, dw.ptr, 1e-5, o.ptr)); ctx.sync()
    assert close(o.download(count=x.size), golden["op_rmsnorm"])
    ctx._check(L.pb_softmax(ctx.h, dx.ptr, 3, 48, o.ptr)); ctx.sync()
    assert close(o.download(count=x.size), golden["op_softmax"])
    ctx._check(L.pb_layernorm(ctx.h, dx.ptr, 3, 48, dw.ptr, db.ptr, 1e-5, o.ptr)); ctx.sync()
    assert close(o.download(count=x.size), golden["op_layernorm"])
    ctx._check(L.pb_gelu(ctx.h, dx.ptr, x.size, o.ptr)); ctx.sync()
    assert close(o.download(count=x.size), golden["op_gelu"], 1e-6)
    ctx._check(L.pb_silu(ctx.h, dx.ptr, x.size, o.ptr)); ctx.sync()
    assert close(o.download(count=x.size), golden["op_silu"], 1e-6)
    y = (x * 0.5).astype(f32)
    dy = dev(ctx, y)
    ctx._check(L.pb_tensoradd(ctx.h, dx.ptr, dy.ptr, x.size, o.ptr)); ctx.sync()
    assert bits_equal(o.download(count=x.size).reshape(x.shape), oracle.tensoradd(x, y).reshape(x.shape))
    ctx._check(L.pb_elementmul(ctx.h, dx.ptr, dy.ptr, x.size, o.ptr)); ctx.sync()
    assert bits_equal(o.download(count=x.size).reshape(x.shape), oracle.elementmul(x, y).reshape(x.shape))
    ctx._check(L.pb_swiglu(ctx.h, dx.ptr, dy.ptr, x.size, o.ptr)); ctx.sync()
    assert close(o.download(count=x.size), oracle.swiglu_fused(x, y), 1e-6)
    # a Llama-size row
    rng = np.random.default_rng(41)
    x2 = rng.standard_normal((4, 2048)).astype(f32)
    w2 = rng.standard_normal(2048).astype(f32)
    d2, dw2, o2 = dev(ctx, x2), dev(ctx, w2), out(ctx, x2.size)
    ctx._check(L.pb_rmsnorm(ctx.h, d2.ptr, 4, 2048, dw2.ptr, 1e-5, o2.ptr)); ctx.sync()
    assert close(o2.download(count=x2.size), oracle.rmsnorm(x2, 4, 2048, w2))


def test_rope_bit_exact(native, ctx, golden):
    L = native.lib()
    q, k = golden["rope_q"].copy(), golden["rope_k"].copy()
    dq, dk = dev(ctx, q), dev(ctx, k)
    ctx._check(L.pb_rope(ctx.h, dq.ptr, dk.ptr, 3, 5, 4, 2, 16, 500000.0))
    ctx.sync()
    assert bits_equal(dq.download(count=q.size), golden["rope_qr"])
    assert bits_equal(dk.download(count=k.size), golden["rope_kr"])


def test_attention_cached_and_generic(native, ctx, oracle, golden):
    L = native.lib()
    q, kc, vc = golden["att_q"], golden["att_kc"], golden["att_vc"]
    dq, dkc, dvc, o = dev(ctx, q), dev(ctx, kc), dev(ctx, vc), out(ctx, 3 * 64)
    ctx._check(L.pb_attn_cached(ctx.h, dq.ptr, dkc.ptr, dvc.ptr, 3, 5, 4, 2, 16, o.ptr))
    ctx.sync()
    assert close(o.download(count=3 * 64), golden["att_out"])
    # decode shape: Llama-3.2-1B heads at 640 cached positions
    rng = np.random.default_rng(51)
    nh, nkv, hd, pos = 32, 8, 64, 639
    qq = rng.standard_normal(nh * hd).astype(f32)
    kk = rng.standard_normal(((pos + 1), nkv * hd)).astype(f32)
    vv = rng.standard_normal(((pos + 1), nkv * hd)).astype(f32)
    dq, dkc, dvc, o = dev(ctx, qq), dev(ctx, kk), dev(ctx, vv), out(ctx, nh * hd)
    ctx._check(L.pb_attn_cached(ctx.h, dq.ptr, dkc.ptr, dvc.ptr, 1, pos, nh, nkv, hd, o.ptr))
    ctx.sync()
    assert close(o.download(count=nh * hd), oracle.attn_cached(qq, kk, vv, 1, pos, nh * hd, nh, nkv, hd))
    # engine.js attention (causal)
    Q = rng.standard_normal((5, 8)).astype(f32)
    K = rng.standard_normal((5, 8)).astype(f32)
    V = rng.standard_normal((5, 6)).astype(f32)
    dQ, dK, dV, o = dev(ctx, Q), dev(ctx, K), dev(ctx, V), out(ctx, 30)
    ctx._check(L.pb_attention(ctx.h, dQ.ptr, dK.ptr, dV.ptr, 5, 5, 8, 6, 1, o.ptr))
    ctx.sync()
    assert close(o.download(count=30), oracle.attention(Q, K, V, 5, 5, 8, 6, True))


@pytest.mark.parametrize("nh,nkv,hd,max_len,positions", [
    (32, 8, 64, 2048, (0, 5, 128, 384, 639, 2047)),  # configs[3]: Llama-3.2-1B heads
    (9, 3, 64, 512, (31, 287)),                       # configs[2]: SmolLM2-135M
    (6, 6, 48, 256, (15, 143)),                       # configs[0]: stories15M
])
@pytest.mark.parametrize("mode", ["fast", "exact"])
def test_split_decode_attention(native, ctx, oracle, nh, nkv, hd, max_len, positions, mode):
    """The decode step's position-split attention (pb_attn_decode) against
    the oracle's llama-streaming.js:543-573 at cache lengths from 1 to the
    maximum, within the reduction tolerance (the fast mode's f32 form within
    RTOL_ATTN_FAST); a second call on the same buffers gives the same bits
    (the split counters are left at zero)."""
    L = native.lib()
    ctx.set_matvec_mode(native.MATVEC_FAST if mode == "fast" else native.MATVEC_EXACT)
    rtol = RTOL_ATTN_FAST if mode == "fast" else RTOL_REDUCE
    worst = 0.0
    rng = np.random.default_rng(52 + hd)
    kv = nkv * hd
    kk = rng.standard_normal((max_len, kv)).astype(f32)
    vv = rng.standard_normal((max_len, kv)).astype(f32)
    dkc, dvc = dev(ctx, kk), dev(ctx, vv)
    for pos in positions:
        qq = (rng.standard_normal(nh * hd) * 0.5).astype(f32)
        dq, o = dev(ctx, qq), out(ctx, nh * hd)
        ctx._check(L.pb_attn_decode(ctx.h, dq.ptr, dkc.ptr, dvc.ptr, pos, nh, nkv, hd, max_len, o.ptr))
        got = o.download(count=nh * hd)
        want = oracle.attn_cached(qq, kk[:pos + 1], vv[:pos + 1], 1, pos, nh * hd, nh, nkv, hd)
        worst = max(worst, np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))
        assert close(got, want, rtol), pos
        ctx._check(L.pb_attn_decode(ctx.h, dq.ptr, dkc.ptr, dvc.ptr, pos, nh, nkv, hd, max_len, o.ptr))
        assert bits_equal(o.download(count=nh * hd), got), pos
    print(f"[decode attention] {mode} {nh}/{nkv}x{hd} max_len {max_len}: worst rel err {worst:.3e}")
    with pytest.raises(native.PureBeeError):
        ctx._check(L.pb_attn_decode(ctx.h, dq.ptr, dkc.ptr, dvc.ptr, max_len, nh, nkv, hd, max_len, o.ptr))
    ctx.set_matvec_mode(native.MATVEC_FAST)


def test_capture_replay(native, ctx, oracle):
    """pb_capture_begin/end record device-pointer calls; a replay gives the same bits."""
    rng = np.random.default_rng(31)
    N, K = 512, 2048
    raw = rand_q4_0(rng, N, K)
    x = rng.standard_normal(K).astype(f32)
    m = native.QMat(ctx, native.TYPE_Q4_0, raw, N, K)
    dx, dy = dev(ctx, x), out(ctx, N)
    L = native.lib()
    ctx.sync()
    ctx._check(L.pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, 0, 0))
    direct = dy.download(count=N)
    g = ctx.capture(lambda: ctx._check(L.pb_qmat_matvec(ctx.h, m.h, dx.ptr, dy.ptr, 0, 0)))
    ctx._check(L.pb_memset(ctx.h, dy.ptr, 0, N * 4))
    g.launch()
    g.launch()
    ctx.sync()
    assert bits_equal(dy.download(count=N), direct)
    assert close(direct, oracle.q4_0_matvec(x, raw, N, K), 2e-6)
    g.free()
    # a blocking call while recording is refused, and the context stays usable
    ctx._check(L.pb_capture_begin(ctx.h))
    rc = L.pb_sync(ctx.h)
    gh = native.V()
    L.pb_capture_end(ctx.h, native.ctypes.byref(gh))
    if gh.value:
        L.pb_graph_free(gh.value)
    assert rc != native.PB_OK
    ctx.sync()
