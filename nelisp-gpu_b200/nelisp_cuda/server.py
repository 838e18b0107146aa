"""Subprocess client of nelisp-cuserver, mirroring lisp/nelisp-gpu-server.el.

The function names and argument meaning are the Elisp client's
(`nelisp-gpu-server-start', `-upload', `-upload-bytes', `-upload-file',
`-free', `-write-resident', `-read-resident', `-run2', `-run', `-batch',
`-compile', `-run-compiled', `-free-compiled'), so the parity tests read
like the reference's own tests.  Errors raise RuntimeError with the
reference's messages ("vkserver upload error", "vkserver died", ...).
"""
from __future__ import annotations

import os
import subprocess
import tempfile

import numpy as np

from . import protocol as P
from ._lib import BIN_DIR
from .f32codec import decode_words

SERVER_BIN = os.path.join(BIN_DIR, "nelisp-cuserver")


class Server:
    def __init__(self, binary: str = SERVER_BIN, env=None):
        if not os.path.exists(binary):
            raise FileNotFoundError(f"{binary} is not built")
        self._kdir = tempfile.mkdtemp(prefix="nlgpu-k")
        self.proc = subprocess.Popen([binary, self._kdir], stdin=subprocess.PIPE,
                                     stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                     env=env)
        self._resident = {}

    # -- transport: `nelisp-gpu--server-xfer' (server.el:112-119)
    def xfer(self, req: bytes, expected: int) -> bytes:
        if self.proc.poll() is not None:
            raise RuntimeError("vkserver died")
        try:
            self.proc.stdin.write(req)
            self.proc.stdin.flush()
        except BrokenPipeError:
            raise RuntimeError("vkserver died")
        buf = b""
        while len(buf) < expected:
            chunk = self.proc.stdout.read(expected - len(buf))
            if not chunk:
                raise RuntimeError("vkserver died")
            buf += chunk
        return buf

    @staticmethod
    def _u32(buf, i):
        return int.from_bytes(buf[4 * i:4 * i + 4], "little")

    def stop(self):
        if self.proc.poll() is None:
            try:
                self.proc.stdin.close()
            except OSError:
                pass
            try:
                self.proc.wait(timeout=30)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self._resident = {}

    def stderr_text(self) -> str:
        return self.proc.stderr.read().decode(errors="replace") if self.proc.stderr else ""

    # -- resident buffers
    def upload(self, vec) -> int:
        buf = self.xfer(P.encode_upload(vec), 8)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver upload error")
        return self._u32(buf, 1)

    def upload_u32(self, words) -> int:
        buf = self.xfer(P.encode_upload_words(words), 8)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver upload-u32 error")
        return self._u32(buf, 1)

    def upload_bytes(self, raw: bytes) -> int:
        buf = self.xfer(P.encode_upload_bytes(raw), 8)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver upload-bytes error")
        return self._u32(buf, 1)

    def upload_file(self, path: str, offset: int, nbytes: int) -> int:
        buf = self.xfer(P.encode_upload_file(os.path.abspath(path), offset, nbytes), 8)
        if self._u32(buf, 0):
            raise RuntimeError(f"vkserver upload-file error ({path} +{offset}, {nbytes} bytes)")
        return self._u32(buf, 1)

    def free(self, h: int) -> None:
        buf = self.xfer(P.encode_free(h), 4)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver free error")

    def write_resident(self, h: int, vec) -> None:
        buf = self.xfer(P.encode_write_resident(h, vec), 4)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver write-resident error")

    def read_resident(self, h: int, n: int) -> np.ndarray:
        """Through the `scale'-by-1 kernel, as server.el:211-217."""
        return self.run2("scale", [("res", h, n), ("in", [1.0]), ("out", n)],
                         [n], (n + 63) // 64)[0]

    def resident(self, vec) -> int:
        key = id(vec)
        if key not in self._resident:
            self._resident[key] = (vec, self.upload(vec))
        return self._resident[key][1]

    # -- dispatch
    def run2(self, name, descs, push, groups):
        req, outsizes = P.encode_run(name, descs, push, groups)
        buf = self.xfer(req, 4 + 4 * sum(outsizes))
        if self._u32(buf, 0):
            raise RuntimeError("vkserver run error")
        return self._decode(buf, outsizes)

    def run(self, name, buffers, push, groups):
        return self.run2(name, [("inout", b) for b in buffers], push, groups)

    def batch(self, slots, disps):
        body, outsizes = P.encode_batch_body(slots, disps)
        buf = self.xfer(P.u32_bytes(P.OP_BATCH) + body, 4 + 4 * sum(outsizes))
        if self._u32(buf, 0):
            raise RuntimeError("vkserver batch error")
        return self._decode(buf, outsizes)

    def compile(self, slots, disps):
        body, outsizes = P.encode_batch_body(slots, disps)
        buf = self.xfer(P.u32_bytes(P.OP_COMPILE) + body, 8)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver compile error")
        return self._u32(buf, 1), outsizes

    def run_compiled(self, h, outsizes):
        buf = self.xfer(P.encode_run_compiled(h), 4 + 4 * sum(outsizes))
        if self._u32(buf, 0):
            raise RuntimeError("vkserver run-compiled error")
        return self._decode(buf, outsizes)

    def free_compiled(self, h):
        buf = self.xfer(P.encode_free_compiled(h), 4)
        if self._u32(buf, 0):
            raise RuntimeError("vkserver free-compiled error")

    @staticmethod
    def _decode(buf, outsizes):
        res, off = [], 1
        for s in outsizes:
            res.append(decode_words(buf, off, s))
            off += s
        return res

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.stop()


def start(**kw) -> Server:
    """`nelisp-gpu-server-start'."""
    return Server(**kw)
