"""Byte sources (source.ts of the reference), restating the cases of its tests/source.test.ts:
a file source reads exactly the requested range and rejects bad ranges; the HTTP source
refuses a server that ignores Range (and does not read its body), rejects a wrong
Content-Range and a truncated body, and reports a 404 as a file that went away."""
import numpy as np
import pytest

from webgpu_b200.source import FileSource, MemorySource, UrlSource, make_source


class FakeResponse:
    def __init__(self, status, body=b"", content_range=None):
        self.status = status
        self.headers = {"Content-Range": content_range} if content_range else {}
        self._body = body
        self.read_called = False
        self.closed = False

    def read(self):
        self.read_called = True
        return self._body

    def close(self):
        self.closed = True


def _opener(resp, seen=None):
    def open_(req):
        if seen is not None:
            seen.append(req.get_header("Range"))
        return resp
    return open_


def test_file_source_reads_only_the_selected_range(tmp_path):
    p = tmp_path / "fixture.gguf"
    p.write_bytes(bytes(range(100)))
    src = make_source(str(p))
    assert isinstance(src, FileSource) and src.name == "fixture.gguf" and src.size == 100
    assert list(src.read(75, 5)) == [75, 76, 77, 78, 79]
    for off, n in ((99, 2), (0, 0), (-1, 1)):
        with pytest.raises(ValueError, match="Invalid model byte range"):
            src.read(off, n)


def test_memory_source_range_rules():
    src = make_source(np.arange(100, dtype=np.uint8))
    assert isinstance(src, MemorySource)
    assert bytes(src.read(10, 3)) == bytes([10, 11, 12])
    with pytest.raises(ValueError, match="Invalid model byte range"):
        src.read(0, 64 * 1024 ** 2 + 1)


def test_http_source_sends_exact_range_and_accepts_exact_answer():
    seen = []
    resp = FakeResponse(206, bytes(range(16, 21)), "bytes 16-20/100")
    src = UrlSource("http://localhost/test.gguf", 100, opener=_opener(resp, seen))
    assert src.name == "local-model.gguf"
    assert list(src.read(16, 5)) == [16, 17, 18, 19, 20]
    assert seen == ["bytes=16-20"] and resp.closed


def test_http_source_refuses_servers_that_would_download_the_entire_model():
    resp = FakeResponse(200, b"x" * 100)
    src = UrlSource("http://localhost/test.gguf", 100, opener=_opener(resp))
    with pytest.raises(ValueError, match="Range"):
        src.read(0, 16)
    assert resp.closed and not resp.read_called


def test_http_source_detects_incorrect_content_range_and_truncated_responses():
    src = UrlSource("http://localhost/test.gguf", 100, opener=_opener(FakeResponse(206, bytes(4), "bytes 0-4/100")))
    with pytest.raises(ValueError, match="Truncated"):
        src.read(0, 5)
    src = UrlSource("http://localhost/test.gguf", 100, opener=_opener(FakeResponse(206, bytes(5), "bytes 1-5/100")))
    with pytest.raises(ValueError, match="Range"):
        src.read(0, 5)


def test_removed_model_reports_unavailable_file_instead_of_range_error():
    src = UrlSource("http://localhost/test.gguf", 100, opener=_opener(FakeResponse(404)))
    with pytest.raises(ValueError, match="model file is no longer available"):
        src.read(0, 16)


def test_descriptor_sizes_and_make_source():
    src = make_source({"url": "http://localhost/m.gguf", "size": 1000, "name": "m.gguf"})
    assert isinstance(src, UrlSource) and src.name == "m.gguf" and src.size == 1000
    for bad in (0, 23, 1.5, None):
        with pytest.raises(ValueError, match="Invalid model file size"):
            UrlSource("http://localhost/m.gguf", bad)
    with pytest.raises(TypeError):
        make_source(42)


def test_gguf_directory_read_over_a_real_http_range_server():
    """A local HTTP server that honours Range serves a synthetic GGUF; the directory read through
    UrlSource (urllib, real sockets) equals the one read from memory."""
    import http.server
    import threading

    from webgpu_b200 import synth
    from webgpu_b200.gguf import model_config, read_gguf

    image = synth.build_gguf(synth.baseline_spec(0)).tobytes()

    class RangeHandler(http.server.BaseHTTPRequestHandler):
        def do_GET(self):
            a, b = (int(v) for v in self.headers["Range"].removeprefix("bytes=").split("-"))
            body = image[a:b + 1]
            self.send_response(206)
            self.send_header("Content-Range", f"bytes {a}-{b}/{len(image)}")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def log_message(self, *args):
            pass

    server = http.server.ThreadingHTTPServer(("127.0.0.1", 0), RangeHandler)
    t = threading.Thread(target=server.serve_forever, daemon=True)
    t.start()
    try:
        src = make_source({"url": f"http://127.0.0.1:{server.server_address[1]}/tiny.gguf", "size": len(image)})
        g_http = read_gguf(src)
        g_mem = read_gguf(MemorySource(np.frombuffer(image, np.uint8)))
        assert list(g_http.tensors) == list(g_mem.tensors)
        assert model_config(g_http) == model_config(g_mem)
        t0 = next(iter(g_http.tensors.values()))
        assert bytes(src.read(t0.offset, 64)) == image[t0.offset:t0.offset + 64]
    finally:
        server.shutdown()
        server.server_close()
