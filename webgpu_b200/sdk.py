"""The public SDK: `WebGPU` with load / generate / stop / reset / dispose and an
on_progress callback, over a worker thread that owns the engine.

Mirrors the reference's SDK and worker protocol (src/sdk.ts:6-49,
src/worker.ts:6-25 of ahpah-dev/WebGPU 0.9.0): requests {id, action:
load|generate|reset|cancel}; replies {id, type: progress|token|done|error,
value | error, aborted}; one request at a time ("The runtime is busy."); a
cancelled request fails with AbortError. The browser Worker becomes a Python
thread; the worker owns every GPU resource.
"""
from __future__ import annotations

import queue
import threading

from .engine import AbortError, PagedEngine


class _Worker(threading.Thread):
    """worker.ts:6-25."""

    def __init__(self):
        super().__init__(daemon=True)
        self.inbox: queue.Queue = queue.Queue()
        self.listeners = []
        self.engine: PagedEngine | None = None
        self.current: threading.Event | None = None
        self.active_id = 0
        self.start()

    def post(self, msg):
        for fn in list(self.listeners):
            fn(msg)

    def run(self):
        while True:
            data = self.inbox.get()
            if data is None:
                if self.engine:
                    self.engine.dispose()
                return
            self.handle(data)

    def handle(self, data):
        mid, action = data.get("id"), data.get("action")
        if self.current is not None:
            self.post({"id": mid, "type": "error", "error": "The runtime is busy."})
            return
        self.active_id = mid
        self.current = threading.Event()
        signal = self.current
        try:
            if action == "load":
                if self.engine:
                    self.engine.dispose()
                self.engine = PagedEngine(lambda p: self.post({"id": self.active_id, "type": "progress", "value": p}))
                info = self.engine.load(data["source"], data.get("options"), signal)
                self.post({"id": mid, "type": "done", "value": info})
            elif action == "generate":
                if not self.engine:
                    raise RuntimeError("Load a model first.")
                gen = (self.engine.generate_ids(data["ids"], data.get("options"), signal) if data.get("ids") is not None
                       else self.engine.generate(data["messages"], data.get("options"), signal))
                for token in gen:
                    self.post({"id": mid, "type": "token", "value": token})
                self.post({"id": mid, "type": "done"})
            elif action == "reset":
                if self.engine:
                    self.engine.reset()
                self.post({"id": mid, "type": "done"})
            else:
                raise RuntimeError("Unknown runtime action.")
        except BaseException as e:  # noqa: BLE001 - reported to the caller
            self.post({"id": mid, "type": "error", "error": str(e), "aborted": signal.is_set() or isinstance(e, AbortError)})
        finally:
            self.current = None


class WebGPU:
    """sdk.ts:6-49 — the runtime handle. (The class keeps the reference's name so
    SDK callers switch without edits; the device underneath is a B200.)"""

    def __init__(self):
        self._worker = _Worker()
        self._sequence = 0
        self._busy = False
        self._disposed = False
        self.on_progress = None

    def _request(self, action: str, payload: dict, on_token=None):
        if self._disposed:
            raise RuntimeError("This runtime was disposed. Create a new WebGPU instance.")
        if self._busy:
            raise RuntimeError("The runtime is busy.")
        self._busy = True
        self._sequence += 1
        mid = self._sequence
        done = threading.Event()
        result = {}

        def listener(m):
            if m.get("id") != mid:
                return
            t = m["type"]
            if t == "progress" and self.on_progress:
                self.on_progress(m["value"])
            elif t == "token" and on_token:
                on_token(m["value"])
            elif t in ("done", "error"):
                result.update(m)
                done.set()

        self._worker.listeners.append(listener)
        self._worker.inbox.put({"id": mid, "action": action, **payload})
        return mid, done, result, listener

    def _finish(self, listener):
        self._busy = False
        if listener in self._worker.listeners:
            self._worker.listeners.remove(listener)

    @staticmethod
    def _raise(result):
        err = result.get("error", "unknown error")
        if result.get("aborted"):
            raise AbortError(err)
        raise RuntimeError(err)

    def _settle(self, result):
        # sdk.ts:48: a request still pending when the runtime is disposed fails with this message
        if self._disposed:
            raise RuntimeError("Runtime disposed.")
        if result.get("type") == "error":
            self._raise(result)

    def load(self, source, options: dict | None = None):
        _, done, result, listener = self._request("load", {"source": source, "options": options or {}})
        done.wait()
        self._finish(listener)
        self._settle(result)
        return result.get("value")

    def generate(self, messages=None, options: dict | None = None, ids=None):
        """Streams TokenEvents; `ids` drives token ids directly instead of chat messages."""
        tokens: queue.Queue = queue.Queue()
        _, done, result, listener = self._request("generate", {"messages": messages, "ids": ids, "options": options or {}},
                                                  on_token=tokens.put)
        finished = False
        try:
            while True:
                try:
                    yield tokens.get(timeout=0.05)
                    continue
                except queue.Empty:
                    pass
                if done.is_set() and tokens.empty():
                    break
            finished = True
        finally:
            if not finished:
                self.stop()
                done.wait()
            self._finish(listener)
        self._settle(result)

    def stop(self):
        """sdk.ts:46 — cancel the running request (worker.ts:8)."""
        cur = self._worker.current
        if cur is not None:
            cur.set()
        if self._worker.engine:
            self._worker.engine.cancel()

    def reset(self):
        _, done, result, listener = self._request("reset", {})
        done.wait()
        self._finish(listener)
        self._settle(result)

    def dispose(self):
        """sdk.ts:48 — ends the worker and frees the device; a pending request is cancelled and
        fails with "Runtime disposed."."""
        self._disposed = True
        if self._busy:
            self.stop()
        self._worker.inbox.put(None)
        self._worker.join(timeout=60)
        self._busy = False
