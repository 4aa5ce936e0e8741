"""Random-access byte sources; a mirror of the reference's ByteSource
(src/core/source.ts:2-36). A Node host reads files with fs.read; here a file
path stands in for the browser File, an in-memory GGUF image for a synthetic
model, and a {url, size, name} descriptor reads HTTP byte ranges exactly as the
reference's URL source does."""
from __future__ import annotations

import os
import urllib.error
import urllib.request

import numpy as np

MAX_READ = 64 * 1024 ** 2


class ByteSource:
    name: str
    size: int

    def read(self, offset: int, length: int):  # pragma: no cover - interface
        raise NotImplementedError

    def view(self):
        """A zero-copy uint8 view of the whole source when it is memory-resident, else None."""
        return None


def _check(offset: int, length: int, size: int) -> None:
    # source.ts:17-18
    if offset < 0 or length < 1 or offset + length > size or length > MAX_READ:
        raise ValueError("Invalid model byte range (maximum read: 64 MiB).")


class FileSource(ByteSource):
    def __init__(self, path: str):
        self.path = path
        self.name = os.path.basename(path)
        self.size = os.path.getsize(path)
        if self.size < 24:
            raise ValueError("Invalid model file size.")
        self._mm = None

    def read(self, offset: int, length: int):
        _check(offset, length, self.size)
        with open(self.path, "rb") as f:
            f.seek(offset)
            data = f.read(length)
        if len(data) != length:
            raise ValueError("The local file changed or could not be read.")
        return data

    def view(self):
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        return self._mm


class MemorySource(ByteSource):
    """A GGUF image already in host memory (e.g. a synthetic model)."""

    def __init__(self, image: np.ndarray, name: str = "memory.gguf"):
        self.image = np.ascontiguousarray(image, dtype=np.uint8).reshape(-1)
        self.name = name
        self.size = int(self.image.nbytes)
        if self.size < 24:
            raise ValueError("Invalid model file size.")

    def read(self, offset: int, length: int):
        _check(offset, length, self.size)
        return memoryview(self.image[offset:offset + length])

    def view(self):
        return self.image


class UrlSource(ByteSource):
    """The reference's URL source (source.ts:7-35): every read is one HTTP GET with an exact
    `Range: bytes=a-b` header; anything but a 206 whose Content-Range names exactly that range of
    a file of `size` bytes is refused (the server would otherwise send the whole model), a 404 means
    the served file went away, and a short body is a truncated range. `opener(request)` returns a
    response with `.status`, `.headers.get()`, `.read()` and `.close()` (urllib's urlopen by default;
    tests pass a fake)."""

    def __init__(self, url: str, size: int, name: str | None = None, opener=None):
        if not isinstance(size, int) or isinstance(size, bool) or size < 24:
            raise ValueError("Invalid model file size.")
        self.url = url
        self.size = size
        self.name = name or "local-model.gguf"
        self._open = opener or (lambda req: urllib.request.urlopen(req, timeout=120))  # a stalled server fails the read

    def read(self, offset: int, length: int):
        _check(offset, length, self.size)
        last = offset + length - 1
        req = urllib.request.Request(self.url, headers={"Range": f"bytes={offset}-{last}"})
        try:
            resp = self._open(req)
        except urllib.error.HTTPError as e:  # urlopen raises for 4xx/5xx
            resp = e
        try:
            status = getattr(resp, "status", None) or getattr(resp, "code", None)
            if status != 206 or resp.headers.get("Content-Range") != f"bytes {offset}-{last}/{self.size}":
                if status == 404:
                    raise ValueError("The selected model file is no longer available. Reopen it from your model library "
                                     "or select the local GGUF file.")
                raise ValueError("The file server must support exact HTTP Range requests. Select the local GGUF file instead.")
            data = resp.read()
        finally:
            resp.close()
        if len(data) != length:
            raise ValueError("Truncated model range.")
        return data


def make_source(src) -> ByteSource:
    """source.ts:8 — accepts a path, an existing ByteSource, a uint8 array, or a
    {url, size, name} descriptor (HTTP range reads)."""
    if isinstance(src, ByteSource):
        return src
    if isinstance(src, (str, os.PathLike)):
        return FileSource(os.fspath(src))
    if isinstance(src, np.ndarray):
        return MemorySource(src)
    if isinstance(src, dict) and "url" in src:
        return UrlSource(src["url"], src.get("size"), src.get("name"))
    raise TypeError("model source must be a path, a ByteSource, a uint8 array or a {url, size, name} descriptor")
