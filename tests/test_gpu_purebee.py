"""The PureBee instruction set (purebee.js) on the device: the reference's
main.js known-answer tests, LINEAR's QuantizedTensor dispatch, and parity of
each instruction with the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
f32 = np.float32


@pytest.fixture(scope="module")
def gpu(native, ctx):
    from purebee_b200.purebee import PureBee
    return PureBee(ctx=ctx)


def test_main_js_kats(gpu):
    """main.js:65-118: TENSOR_MUL, SOFTMAX, LAYER_NORM, the instruction pipeline."""
    gpu.GRID_WRITE("mat_a", [2, 3], np.array([1, 2, 3, 4, 5, 6], f32))
    gpu.GRID_WRITE("mat_b", [3, 2], np.array([7, 8, 9, 10, 11, 12], f32))
    assert gpu.TENSOR_MUL("mat_a", "mat_b", "mat_c").data.tolist() == [58, 64, 139, 154]
    gpu.GRID_WRITE("v", [1, 4], np.array([1, 2, 3, 4], f32))
    p = gpu.SOFTMAX("v", "v_probs").data
    assert abs(float(p.astype(np.float64).sum()) - 1.0) < 1e-5
    gpu.GELU("v", "v_gelu")
    gpu.GRID_WRITE("xn", [2, 4], np.arange(1, 9, dtype=f32))
    gpu.GRID_WRITE("wn", [4], np.ones(4, f32))
    gpu.GRID_WRITE("bn", [4], np.zeros(4, f32))
    ln = gpu.LAYER_NORM("xn", "wn", "bn", "normed").data
    assert abs(float(ln[:4].astype(np.float64).mean())) < 1e-4
    assert gpu.SYNC() is True
    assert gpu.stats()["ops"] > 0


def test_linear_dispatch_q8_and_f32(gpu, oracle):
    """purebee.js:74-88: a QuantizedTensor weight takes matmul_q8 (quantize.js:224-266)."""
    from purebee_b200.purebee import quantize_q8, dequantize
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 64)).astype(f32)
    w = (rng.standard_normal(64 * 96) * 0.05).astype(f32)
    gpu.GRID_WRITE("x", [4, 64], x)
    qt = quantize_q8(gpu.ctx, "w_q", [64, 96], w)
    s, q = qt.host()
    s_o, q_o = oracle.quantize_q8a(w)
    assert np.array_equal(s, s_o) and np.array_equal(q, q_o)
    assert np.array_equal(dequantize(qt), oracle.dequantize_q8a(s_o, q_o, w.size))
    gpu.GRID_WRITE_RAW("w_q", qt)
    y = gpu.LINEAR("x", "w_q", None, "y").data
    assert np.array_equal(y.view(np.uint32), oracle.matmul_q8(x, 4, 64, s_o, q_o, 96).view(np.uint32))
    gpu.GRID_WRITE("w_f", [64, 96], w)
    gpu.GRID_WRITE("b", [96], np.ones(96, f32))
    y = gpu.LINEAR("x", "w_f", "b", "y2").data
    assert np.array_equal(y.view(np.uint32), oracle.matmul_wasm(x, 4, 64, w, 96, np.ones(96, f32)).view(np.uint32))


def test_instructions_match_oracle(gpu, oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 40)).astype(f32)
    w = rng.standard_normal(40).astype(f32)
    gpu.GRID_WRITE("x", [3, 40], x)
    gpu.GRID_WRITE("w", [40], w)
    tol = lambda a, b, r: np.max(np.abs(a.astype(np.float64) - b)) <= r * np.max(np.abs(b))
    assert tol(gpu.RMS_NORM("x", "w", "r").data, oracle.rmsnorm(x, 3, 40, w), 2e-6)
    assert tol(gpu.SILU("x", "s").data, oracle.silu(x), 1e-6)
    assert np.array_equal(gpu.TENSOR_ADD("x", "x", "a").data, oracle.tensoradd(x, x))
    assert np.array_equal(gpu.ELEMENT_MUL("x", "x", "m").data, oracle.elementmul(x, x))
    Q = rng.standard_normal((6, 8)).astype(f32)
    gpu.GRID_WRITE("Q", [6, 8], Q)
    gpu.GRID_WRITE("V", [6, 5], rng.standard_normal((6, 5)).astype(f32))
    a = gpu.ATTENTION("Q", "Q", "V", "att", True).data
    assert tol(a, oracle.attention(Q, Q, gpu.GRID_READ("V").data, 6, 6, 8, 5, True), 2e-6)
    with pytest.raises(KeyError):
        gpu.GRID_READ("missing")
    with pytest.raises(ValueError):
        gpu.GRID_WRITE("z", [5], np.zeros(5, f32))
        gpu.TENSOR_ADD("x", "z", "bad")
    with pytest.raises(NotImplementedError):
        gpu.PARALLEL_MAP("x", lambda v, i: v, "y")
