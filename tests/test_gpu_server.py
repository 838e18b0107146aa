"""The protocol server (bin/nelisp-cuserver) end to end, driven by the
restated Elisp client: the reference's upload-file test, compiled batches,
and the error conventions of host/vkserver.c."""
import os
import struct
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture()
def server():
    from nelisp_cuda.server import Server
    s = Server()
    yield s
    s.stop()


def readback(server, h, n):
    """uft-readback (test/upload-file-test.el:21-27): copy through add2."""
    return server.batch([("res", h, n), ("in", np.zeros(n)), ("out", n)],
                        [("add2", [0, 1, 2], [n], (n + 63) // 64)])[0]


def test_upload_file_region_is_exact(server, tmp_path):
    # test/upload-file-test.el:29-104
    n, pad = 4096, 12
    vec = np.array([3.0 * i - 5000 for i in range(n)])
    path = str(tmp_path / "uft.bin")
    with open(path, "wb") as f:
        f.write(b"\0" * (pad * 4) + vec.astype("<f4").tobytes())
    h = server.upload_file(path, pad * 4, n * 4)
    got = readback(server, h, n)
    assert np.array_equal(got, vec) and np.any(got != 0.0)
    h2 = server.upload_file(path, (pad + 1) * 4, (n - 1) * 4)
    g2 = readback(server, h2, n - 1)
    assert not np.array_equal(g2, vec[:n - 1])          # control: the offset is honoured
    assert np.array_equal(g2, vec[1:])
    server.free(h2)
    raw = open(path, "rb").read()[pad * 4:]
    h3 = server.upload_bytes(raw)
    assert np.array_equal(readback(server, h3, n), got)  # both upload paths agree
    server.free(h3)
    half = n // 2
    h4 = server.upload_file(path, (pad + half) * 4, half * 4)
    assert np.array_equal(readback(server, h4, half), vec[half:])
    server.free(h4)
    server.free(h)


def test_upload_file_failures(server, tmp_path):
    path = str(tmp_path / "short.bin")
    open(path, "wb").write(b"\1" * 40)
    with pytest.raises(RuntimeError, match="upload-file error"):
        server.upload_file(path, 0, 80)                  # short read
    with pytest.raises(RuntimeError, match="upload-file error"):
        server.upload_file(str(tmp_path / "missing.bin"), 0, 4)
    h = server.upload([1.0, 2.0])                        # the server is still usable
    assert list(server.read_resident(h, 2)) == [1.0, 2.0]


def test_compile_run_compiled_write_resident(server):
    n = 300
    a = np.linspace(-1, 1, n)
    h = server.upload(a)
    hc, outs = server.compile([("res", h, n), ("in", np.ones(n)), ("tmp", n), ("out", n)],
                              [("add2", [0, 1, 2], [n], 5), ("silu-mul", [2, 1, 3], [n], 5)])
    r1 = server.run_compiled(hc, outs)[0]
    x = a.astype(np.float32) + 1.0
    assert np.allclose(r1, x / (1 + np.exp(-x.astype(np.float64))), rtol=1e-5)
    server.write_resident(h, 2 * a)
    r2 = server.run_compiled(hc, outs)[0]
    x2 = (2 * a).astype(np.float32) + 1.0
    assert np.allclose(r2, x2 / (1 + np.exp(-x2.astype(np.float64))), rtol=1e-5)
    server.free_compiled(hc)
    with pytest.raises(RuntimeError, match="write-resident"):
        server.write_resident(999, [1.0])


def test_run_errors_keep_the_stream_in_sync(server):
    with pytest.raises(RuntimeError, match="run error"):
        server.run2("no-such-kernel", [("out", 5)], [5], 1)
    with pytest.raises(RuntimeError, match="batch error"):
        server.batch([("res", 77, 4), ("out", 4)], [("scale", [0, 0, 1], [4], 1)])
    # the next request is answered correctly
    out = server.run("add2", [[1.0, 2.0], [3.0, 4.0], [0.0, 0.0]], [2], 1)
    assert list(out[2]) == [4.0, 6.0]


def test_exit_codes():
    from nelisp_cuda.server import SERVER_BIN
    r = subprocess.run([SERVER_BIN, "/tmp"], input=b"", capture_output=True, timeout=120)
    assert r.returncode == 0                             # EOF exits 0
    r = subprocess.run([SERVER_BIN, "/tmp"], input=struct.pack("<I", 42),
                       capture_output=True, timeout=120)
    assert r.returncode == 2 and b"bad opcode" in r.stderr
    r = subprocess.run([SERVER_BIN, "/tmp"], input=struct.pack("<II", 0, 64),
                       capture_output=True, timeout=120)
    assert r.returncode == 2                             # name too long
    # RUN_COMPILED on a bad handle: a bare status 1 (host/vkserver.c:593)
    r = subprocess.run([SERVER_BIN, "/tmp"], input=struct.pack("<II", 5, 3),
                       capture_output=True, timeout=120)
    assert r.returncode == 0 and r.stdout == struct.pack("<I", 1)


def test_cli_vkmatmul_vksoftmax_vkrun(tmp_path):
    from nelisp_cuda._lib import BIN_DIR
    for mode in ["naive", "tiled", "reg"]:
        r = subprocess.run([os.path.join(BIN_DIR, "vkmatmul"), "kernels/matmul.spv", "256",
                            "256", "256", mode, "5"], capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, r.stderr
        assert "matmul 256x256 x 256x256" in r.stdout and r.stdout.strip().endswith("PASS")
    r = subprocess.run([os.path.join(BIN_DIR, "vksoftmax"), "kernels/softmax.spv", "64", "256"],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "row0_sum=1.00000" in r.stdout and "PASS" in r.stdout
    # vkrun: every buffer in, every buffer back
    M, N = 4, 8
    A = np.arange(M * N, dtype=np.float32) * 0.1
    inp, outp = tmp_path / "in.bin", tmp_path / "out.bin"
    inp.write_bytes(np.concatenate([A, np.zeros(M * N, np.float32)]).tobytes())
    r = subprocess.run([os.path.join(BIN_DIR, "vkrun"), "/x/softmax.spv", str(inp), str(outp),
                        "64", "1", f"{M},{N}", f"{M * N},{M * N}"], capture_output=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.frombuffer(outp.read_bytes(), np.float32)
    import oracle as nlo
    assert np.array_equal(got[:M * N], A)
    assert nlo.tk_err(got[M * N:], nlo.softmax(A, M, N)) < 1e-4
    r = subprocess.run([os.path.join(BIN_DIR, "vkrun"), "/tmp/nlgpu123.spv", str(inp), str(outp),
                        "64", "1", "-", "4"], capture_output=True, timeout=120)
    assert r.returncode == 2                             # unknown kernel name


def test_bounded_wait_timeout_is_reported():
    """A kernel wait that can never complete gives up after its bound, sets the
    host-mapped flag, and the host reads it as an error; the context stays
    usable and the flag is cleared by the report."""
    from nelisp_cuda import _lib as L
    lib = L.load()
    L.check(lib.nl_init(-1))
    assert lib.nl_wait_status() == L.NL_OK
    assert lib.nl_selftest_wait_timeout() == L.NL_ERROR
    assert b"timed out" in lib.nl_last_error()
    assert lib.nl_wait_status() == L.NL_OK          # cleared
    from nelisp_cuda.host import Host
    h = Host()
    got = h.run2("add2", [("in", [1.0, 2.0]), ("in", [3.0, 4.0]), ("out", 2)], [2], 1)[0]
    assert list(got) == [4.0, 6.0]
