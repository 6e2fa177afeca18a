"""Llama-3 RoPE frequency scaling: an opt-in flag, off by default.

The reference rotates by pos / theta^(i/hd) with no scaling
(llama-streaming.js:316-336; gguf.js:378-410 never maps rope_freqs.weight), so
parity runs keep the flag off.  The scaled frequencies are checked on the CPU
against a restatement of the published Llama 3.1 / 3.2 rule, and on the GPU
through the K rows a model writes into its cache.
"""
import math

import numpy as np
import pytest


def llama3_freqs(theta, hd, factor, low, high, ctx_len):
    """The published rule, restated: wavelengths shorter than ctx/high keep
    their frequency, longer than ctx/low are divided by factor, and the band
    between is blended linearly in ctx / wavelength."""
    out = []
    for i in range(0, hd, 2):
        f = 1.0 / math.pow(theta, i / hd)
        w = 2 * math.pi / f
        if w < ctx_len / high:
            out.append(f)
        elif w > ctx_len / low:
            out.append(f / factor)
        else:
            s = (ctx_len / w - low) / (high - low)
            out.append((1 - s) * f / factor + s * f)
    return np.array(out)


def _freqs(native, theta, hd, factor, low=1.0, high=4.0, ctx_len=8192):
    out = np.zeros(hd // 2, np.float64)
    rc = native.lib().pb_rope_freqs(theta, hd, factor, low, high, ctx_len, native.ptr(out))
    return rc, out


@pytest.fixture(scope="module")
def lib_only():
    from purebee_b200 import _native
    _native.lib()
    return _native


def test_unscaled_is_the_reference_frequency(lib_only):
    for theta, hd in ((10000.0, 48), (500000.0, 64), (10000.0, 64)):
        rc, f = _freqs(lib_only, theta, hd, 0.0)
        assert rc == 0
        want = np.array([1.0 / math.pow(theta, i / hd) for i in range(0, hd, 2)])
        assert np.array_equal(f, want)


def test_llama32_1b_scaled_frequencies(lib_only):
    rc, f = _freqs(lib_only, 500000.0, 64, 32.0, 1.0, 4.0, 8192)
    assert rc == 0
    want = llama3_freqs(500000.0, 64, 32.0, 1.0, 4.0, 8192)
    np.testing.assert_allclose(f, want, rtol=1e-14, atol=0)
    base = llama3_freqs(500000.0, 64, 1.0, 1.0, 4.0, 8192)  # factor 1: nothing changes
    assert np.all(f <= base)
    assert f[0] == base[0]  # the highest frequency is kept
    assert f[-1] == pytest.approx(base[-1] / 32.0, rel=1e-15)  # the lowest is divided by the factor
    blended = (f != base) & (np.abs(f - base / 32.0) > 1e-18 * base)
    assert blended.any()  # some pairs fall in the blended band


def test_scaling_argument_errors(lib_only):
    assert _freqs(lib_only, 500000.0, 64, 32.0, 4.0, 1.0)[0] == lib_only.PB_ERR_ARG  # low >= high
    assert _freqs(lib_only, 500000.0, 64, 32.0, 1.0, 4.0, 0)[0] == lib_only.PB_ERR_ARG
    assert _freqs(lib_only, 500000.0, 63, 0.0)[0] == lib_only.PB_ERR_ARG  # odd head size
    assert _freqs(lib_only, -1.0, 64, 0.0)[0] == lib_only.PB_ERR_ARG


@pytest.mark.gpu
def test_scaled_rotation_in_the_kv_cache(native, ctx, oracle):
    """Layer 0's K row at position p depends only on the token and wk, so the
    unrotated k can be recovered from the oracle's (unscaled) row and rotated
    by the scaled angles; the device's row must match it.  Turning the flag
    off again restores the reference's bits."""
    import sys
    import os
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_golden as mg
    from purebee_b200.runtime import StreamingLlamaRuntime
    from test_gpu_model import cfg_objects
    kw = dict(mg.TINY_STREAMING, rope_theta=500000.0, seq_len=64)
    oc, lc = cfg_objects(kw)
    rt = StreamingLlamaRuntime(lc, ctx=ctx, emb_type=kw["emb_type"])
    rt.loadSynthetic(11)
    om = oracle.Model(oc)
    om.init_synthetic(11)
    toks = [5, 17, 33, 42, 7, 9, 60, 61]
    hd, kvd = kw["head_dim"], kw["n_kv_heads"] * kw["head_dim"]
    # small context so that positions < 64 reach the scaled bands
    factor, low, high, ctx_len = 8.0, 1.0, 4.0, 64
    rt.model.set_rope_scaling(factor, low, high, ctx_len)
    assert rt.model.rope_scaling_factor == factor
    rt.forward(toks, 0)
    k_dev = rt.model.kv(0, 0)[:len(toks)].astype(np.float64)
    om.forward(toks, 0)
    k_orc = om.kv(0, 0)[:len(toks)].astype(np.float64)
    f0 = np.array([1.0 / math.pow(500000.0, i / hd) for i in range(0, hd, 2)])
    f1 = llama3_freqs(500000.0, hd, factor, low, high, ctx_len)
    assert np.any(f0 != f1)
    for p in range(len(toks)):
        for h in range(kvd // hd):
            row = k_orc[p, h * hd:(h + 1) * hd]
            x0, x1 = row[0::2], row[1::2]
            a0, a1 = p * f0, p * f1
            # undo the unscaled rotation, apply the scaled one
            u0 = x0 * np.cos(a0) + x1 * np.sin(a0)
            u1 = -x0 * np.sin(a0) + x1 * np.cos(a0)
            want = np.empty(hd)
            want[0::2] = u0 * np.cos(a1) - u1 * np.sin(a1)
            want[1::2] = u0 * np.sin(a1) + u1 * np.cos(a1)
            got = k_dev[p, h * hd:(h + 1) * hd]
            assert np.max(np.abs(got - want)) <= 1e-5 * max(1.0, np.max(np.abs(want))), (p, h)
    # off again: the reference's table, the oracle's bits
    rt.model.set_rope_scaling(0.0)
    assert rt.model.rope_scaling_factor == 0.0
    rt.resetCache()
    rt.forward(toks, 0)
    k_off, k_ref = rt.model.kv(0, 0)[:len(toks)], om.kv(0, 0)[:len(toks)]
    assert np.max(np.abs(k_off - k_ref)) <= 2e-6 * np.max(np.abs(k_ref))  # the RMSNorm's reduction order
    rt.shutdown()
