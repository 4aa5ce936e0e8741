"""Random-access byte sources; a mirror of the reference's ByteSource
(src/core/source.ts:2-36). A Node host reads files with fs.read; here a file
path, or an in-memory GGUF image, stands in for the browser File / HTTP range."""
from __future__ import annotations

import os

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
    # source.ts:59-60
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


def make_source(src) -> ByteSource:
    """source.ts:8 — accepts a path, an existing ByteSource or a uint8 array."""
    if isinstance(src, ByteSource):
        return src
    if isinstance(src, (str, os.PathLike)):
        return FileSource(os.fspath(src))
    if isinstance(src, np.ndarray):
        return MemorySource(src)
    raise TypeError("model source must be a path, a ByteSource or a uint8 array")
