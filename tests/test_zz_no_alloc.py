"""pb_attention_noalloc (scores in a fixed per-device array) against
pb_attention (scores in the context scratch): the same bits, on two calls in
a row, and a clean PB_ERR_ARG past the array's size.  Collected last so it
also runs after every other GPU test has used the context."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
f32 = np.float32


def _attn(native, ctx, fn, bufs, sq, sk, dk, dv, causal):
    Q, K, V, out = bufs
    ctx._check(getattr(native.lib(), fn)(ctx.h, Q.ptr, K.ptr, V.ptr, sq, sk, dk, dv, causal, out.ptr))


def _inputs(ctx, rng, sq, sk, dk, dv):
    Q = ctx.to_device(rng.standard_normal((sq, dk)).astype(f32))
    K = ctx.to_device(rng.standard_normal((sk, dk)).astype(f32))
    V = ctx.to_device(rng.standard_normal((sk, dv)).astype(f32))
    return Q, K, V


def test_noalloc_attention_equals_scratch_path(native, ctx):
    rng = np.random.default_rng(2026)
    cases = [(48, 300, 64, 32, 1), (5, 1000, 16, 8, 0)]  # the second call is a different shape
    bufs = []
    for sq, sk, dk, dv, causal in cases:
        Q, K, V = _inputs(ctx, rng, sq, sk, dk, dv)
        bufs.append((Q, K, V, ctx.alloc(sq * dv * 4), ctx.alloc(sq * dv * 4)))
    # two no-alloc calls back to back on the stream, then the scratch path
    for (Q, K, V, o_na, _), c in zip(bufs, cases):
        _attn(native, ctx, "pb_attention_noalloc", (Q, K, V, o_na), *c)
    for (Q, K, V, _, o_ref), c in zip(bufs, cases):
        _attn(native, ctx, "pb_attention", (Q, K, V, o_ref), *c)
    ctx.sync()
    for (_, _, _, o_na, o_ref), (sq, _, _, dv, _) in zip(bufs, cases):
        a = o_na.download(count=sq * dv)
        b = o_ref.download(count=sq * dv)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.all(np.isfinite(a))


def test_noalloc_attention_rejects_oversize(native, ctx):
    rng = np.random.default_rng(7)
    sq, sk = 512, 1025  # 2 * 4 * 512 * 1025 bytes > 4 MiB
    Q, K, V = _inputs(ctx, rng, sq, sk, 8, 8)
    out = ctx.alloc(sq * 8 * 4)
    launches = ctx.launches
    rc = native.lib().pb_attention_noalloc(ctx.h, Q.ptr, K.ptr, V.ptr, sq, sk, 8, 8, 0, out.ptr)
    assert rc == native.PB_ERR_ARG
    assert b"fixed array" in native.lib().pb_last_error(ctx.h)
    assert ctx.launches == launches  # rejected before any launch
    # more queries than one grid dimension holds, although the scores fit:
    # rejected by both entry points, again before any launch (buffers sized
    # for the call all the same)
    sq_big, sk_small = 65536, 1
    Qb, Kb, Vb = _inputs(ctx, rng, sq_big, sk_small, 8, 8)
    ob = ctx.alloc(sq_big * 8 * 4)
    for fn in ("pb_attention_noalloc", "pb_attention"):
        rc = getattr(native.lib(), fn)(ctx.h, Qb.ptr, Kb.ptr, Vb.ptr, sq_big, sk_small, 8, 8, 0, ob.ptr)
        assert rc == native.PB_ERR_ARG, fn
        assert b"65535" in native.lib().pb_last_error(ctx.h)
    assert ctx.launches == launches
    # the largest case that fits (seqQ * seqK = 524288) still runs and matches
    sk = 1024
    Q, K, V = _inputs(ctx, rng, sq, sk, 8, 8)
    o_na, o_ref = ctx.alloc(sq * 8 * 4), ctx.alloc(sq * 8 * 4)
    _attn(native, ctx, "pb_attention_noalloc", (Q, K, V, o_na), sq, sk, 8, 8, 1)
    _attn(native, ctx, "pb_attention", (Q, K, V, o_ref), sq, sk, 8, 8, 1)
    ctx.sync()
    assert np.array_equal(o_na.download(count=sq * 8).view(np.uint32), o_ref.download(count=sq * 8).view(np.uint32))
