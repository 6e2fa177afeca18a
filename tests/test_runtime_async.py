"""The reference's async entry points of StreamingLlamaRuntime
(llama-streaming.js:230-244, 821-823, 976-978) on CPU: forwardAsync and
generateAsync resolve to forward() and generate() with the same arguments,
and initThreadPool resolves false (no host worker pool: the matvecs run on the
device).  The runtime is built without a device model; forward and generate
are stand-ins that record their arguments."""
import asyncio

from purebee_b200.runtime import LlamaRuntime, StreamingLlamaRuntime


def bare(cls):
    rt = object.__new__(cls)
    rt.calls = []
    rt.forward = lambda *a: rt.calls.append(("forward", a)) or {"logits": [0.0, 1.0], "layersUsed": 2}
    rt.generate = lambda *a: rt.calls.append(("generate", a)) or {"tokens": [1, 2, 3], "generated": 1}
    return rt


def test_forward_async_wraps_forward():
    for cls in (StreamingLlamaRuntime, LlamaRuntime):
        rt = bare(cls)
        out = asyncio.run(rt.forwardAsync([5, 6], 3, {"maxLayers": 2}))
        assert out == {"logits": [0.0, 1.0], "layersUsed": 2}
        assert rt.calls == [("forward", ([5, 6], 3, {"maxLayers": 2}))]
        rt.calls.clear()
        asyncio.run(rt.forwardAsync([7]))
        assert rt.calls == [("forward", ([7], 0, None))]


def test_generate_async_wraps_generate():
    rt = bare(StreamingLlamaRuntime)
    out = asyncio.run(rt.generateAsync([1, 2], 4, {"greedy": True}))
    assert out["tokens"] == [1, 2, 3]
    assert rt.calls == [("generate", ([1, 2], 4, {"greedy": True}))]
    rt.calls.clear()
    asyncio.run(rt.generateAsync([9]))
    assert rt.calls == [("generate", ([9], 50, None))]


def test_init_thread_pool_resolves_false():
    rt = bare(StreamingLlamaRuntime)
    assert asyncio.run(rt.initThreadPool()) is False
    assert asyncio.run(rt.initThreadPool(8)) is False
    assert rt.calls == []
