"""The SDK / worker protocol (src/sdk.ts:6-49 and src/worker.ts:6-25 of the reference) without a
GPU: the worker's engine is replaced by a fake, as the reference's own tests replace engine
internals. One request at a time ("The runtime is busy."), progress and token streaming, errors
with their messages, cancellation as AbortError, and disposal."""
import threading
import time

import pytest

import webgpu_b200.sdk as sdk
from webgpu_b200.engine import AbortError


class FakeEngine:
    instances = []

    def __init__(self, progress=None):
        self.progress = progress or (lambda p: None)
        self.cancelled = self.disposed = self.was_reset = False
        FakeEngine.instances.append(self)

    def load(self, src, options=None, signal=None):
        self.progress({"phase": "loading", "fraction": 0.5})
        if src == "bad":
            raise ValueError("Invalid model file size.")
        return {"name": src}

    def generate_ids(self, ids, options=None, signal=None):
        for t in ids:
            if (options or {}).get("slow"):
                time.sleep(0.05)
            if signal is not None and signal.is_set():
                raise AbortError("Stopped by user")
            yield {"token": t}

    def generate(self, messages, options=None, signal=None):
        yield from self.generate_ids([7, 8, 9], options, signal)

    def reset(self):
        self.was_reset = True

    def cancel(self):
        self.cancelled = True

    def dispose(self):
        self.disposed = True


@pytest.fixture
def rt(monkeypatch):
    FakeEngine.instances.clear()
    monkeypatch.setattr(sdk, "PagedEngine", FakeEngine)
    r = sdk.WebGPU()
    yield r
    r.dispose()


def test_load_reports_progress_and_info(rt):
    seen = []
    rt.on_progress = seen.append
    assert rt.load("model.gguf") == {"name": "model.gguf"}
    assert seen == [{"phase": "loading", "fraction": 0.5}]


def test_load_error_keeps_its_message_and_is_not_an_abort(rt):
    with pytest.raises(RuntimeError, match="Invalid model file size") as e:
        rt.load("bad")
    assert not isinstance(e.value, AbortError)
    assert rt.load("good.gguf") == {"name": "good.gguf"}  # the runtime is usable again


def test_generate_needs_a_model_then_streams_tokens_in_order(rt):
    with pytest.raises(RuntimeError, match="Load a model first"):
        list(rt.generate(ids=[1, 2]))
    rt.load("m.gguf")
    assert [t["token"] for t in rt.generate(ids=[3, 1, 2])] == [3, 1, 2]
    assert [t["token"] for t in rt.generate([{"role": "user", "content": "hello"}])] == [7, 8, 9]


def test_one_request_at_a_time(rt):
    rt.load("m.gguf")
    gen = rt.generate(ids=list(range(20)), options={"slow": True})
    assert next(gen)["token"] == 0  # the generate request is running
    with pytest.raises(RuntimeError, match="The runtime is busy"):
        rt.load("other.gguf")
    with pytest.raises(RuntimeError, match="The runtime is busy"):
        rt.reset()
    gen.close()  # leaving the loop early stops the request
    rt.reset()
    assert FakeEngine.instances[-1].was_reset


def test_stop_cancels_a_running_generation_with_abort_error(rt):
    rt.load("m.gguf")
    got = []

    def consume():
        try:
            for t in rt.generate(ids=list(range(100)), options={"slow": True}):
                got.append(t["token"])
        except AbortError as e:
            got.append(str(e))

    th = threading.Thread(target=consume)
    th.start()
    while not got:
        time.sleep(0.01)
    rt.stop()
    th.join(timeout=10)
    assert not th.is_alive()
    assert got[-1] == "Stopped by user" and len(got) < 100
    assert FakeEngine.instances[-1].cancelled


def test_dispose_frees_the_engine_and_refuses_further_calls(monkeypatch):
    FakeEngine.instances.clear()
    monkeypatch.setattr(sdk, "PagedEngine", FakeEngine)
    r = sdk.WebGPU()
    r.load("m.gguf")
    r.dispose()
    assert FakeEngine.instances[-1].disposed
    with pytest.raises(RuntimeError, match="This runtime was disposed"):
        r.load("m.gguf")


def test_dispose_fails_a_pending_request(monkeypatch):
    class SlowLoad(FakeEngine):
        def load(self, src, options=None, signal=None):
            for _ in range(500):
                if signal is not None and signal.is_set():
                    raise AbortError("Stopped by user")
                time.sleep(0.01)
            return {"name": src}

    monkeypatch.setattr(sdk, "PagedEngine", SlowLoad)
    r = sdk.WebGPU()
    out = []

    def load():
        try:
            out.append(r.load("m.gguf"))
        except RuntimeError as e:
            out.append(str(e))

    th = threading.Thread(target=load)
    th.start()
    time.sleep(0.1)
    r.dispose()
    th.join(timeout=10)
    assert out == ["Runtime disposed."]
