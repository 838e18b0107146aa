"""In-process host API over the C ABI, with the server client's call shapes.

`Host` exposes the operations of lisp/nelisp-gpu-server.el -- upload,
upload_file, free, write_resident, read_resident, run2, run, batch, compile,
run_compiled, free_compiled -- as direct calls into libnelisp_cuda (no
process boundary).  Vectors are float values (encoded with the reference's
f32 codec) or, with ``words=True``/uint32 arrays, raw 32-bit words.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .f32codec import bits_f32, f32_bits


def _as_words(vec) -> np.ndarray:
    a = np.asarray(vec)
    if a.dtype == np.uint32:
        return np.ascontiguousarray(a)
    if a.dtype == np.float32:
        return np.ascontiguousarray(a).view(np.uint32)
    return f32_bits(a)


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a.size else None


class Host:
    def __init__(self, device: int = -1):
        self.lib = L.load()
        L.check(self.lib.nl_init(device))

    @property
    def device_name(self) -> str:
        return self.lib.nl_device_name().decode()

    def kernels(self):
        return [self.lib.nl_kernel_name(i).decode() for i in range(self.lib.nl_kernel_count())]

    # -- resident buffers
    def upload(self, vec) -> int:
        w = _as_words(vec)
        h = ctypes.c_uint32()
        L.check(self.lib.nl_upload(_ptr(w), w.size, ctypes.byref(h)))
        return h.value

    def upload_file(self, path: str, offset: int, nbytes: int) -> int:
        if nbytes % 4:
            raise ValueError("upload-file: not a whole number of uint32 words")
        h = ctypes.c_uint32()
        L.check(self.lib.nl_upload_file(path.encode(), offset, nbytes // 4, ctypes.byref(h)))
        return h.value

    def free(self, h: int) -> None:
        L.check(self.lib.nl_free(h))

    def write_resident(self, h: int, vec) -> None:
        w = _as_words(vec)
        L.check(self.lib.nl_write_resident(h, _ptr(w), w.size))

    def read_words(self, h: int, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), np.uint32)
        L.check(self.lib.nl_read_resident(h, _ptr(out), n))
        return out[:n]

    def read_resident(self, h: int, n: int) -> np.ndarray:
        return bits_f32(self.read_words(h, n))

    def resident_ptr(self, h: int):
        p, n = ctypes.c_void_p(), ctypes.c_uint32()
        L.check(self.lib.nl_resident_info(h, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    # -- dispatch
    def run2(self, name, descs, push, groups, words=False):
        bufs = (L.RunBuffer * max(len(descs), 1))()
        inline, outsizes = [], []
        for i, d in enumerate(descs):
            k = d[0]
            if k == "in":
                w = _as_words(d[1]); inline.append(w)
                bufs[i] = L.RunBuffer(w.size, L.RUN_IN, 0)
            elif k == "res":
                bufs[i] = L.RunBuffer(int(d[2]), L.RUN_RESIDENT, int(d[1]))
            elif k == "out":
                bufs[i] = L.RunBuffer(int(d[1]), L.RUN_OUT, 0); outsizes.append(int(d[1]))
            elif k == "inout":
                w = _as_words(d[1]); inline.append(w)
                bufs[i] = L.RunBuffer(w.size, L.RUN_INOUT, 0); outsizes.append(w.size)
            else:
                raise ValueError(f"bad descriptor kind {k!r}")
        inl = np.concatenate(inline) if inline else np.zeros(0, np.uint32)
        out = np.zeros(max(sum(outsizes), 1), np.uint32)
        pushv = L.u32_array(push)
        L.check(self.lib.nl_run(str(name).encode(), len(descs), bufs, len(push), pushv, groups,
                                _ptr(inl), _ptr(out)))
        return self._split(out, outsizes, words)

    def run(self, name, buffers, push, groups, words=False):
        return self.run2(name, [("inout", b) for b in buffers], push, groups, words)

    def _batch_args(self, slots, disps):
        S = (L.Slot * max(len(slots), 1))()
        inline, outsizes = [], []
        for i, s in enumerate(slots):
            k = s[0]
            if k == "in":
                w = _as_words(s[1]); inline.append(w); S[i] = L.Slot(L.SLOT_IN, w.size, 0)
            elif k == "res":
                S[i] = L.Slot(L.SLOT_RESIDENT, int(s[2]), int(s[1]))
            elif k == "tmp":
                S[i] = L.Slot(L.SLOT_TMP, int(s[1]), 0)
            elif k == "out":
                S[i] = L.Slot(L.SLOT_OUT, int(s[1]), 0); outsizes.append(int(s[1]))
            else:
                raise ValueError(f"bad slot kind {k!r}")
        D = (L.Dispatch * max(len(disps), 1))()
        for i, (name, idx, push, groups) in enumerate(disps):
            d = D[i]
            d.name = str(name).encode()
            d.nbuf = len(idx)
            for j, v in enumerate(idx):
                d.slot[j] = v
            d.npush = len(push)
            for j, v in enumerate(push):
                d.push[j] = v
            d.groups = groups
        inl = np.concatenate(inline) if inline else np.zeros(0, np.uint32)
        return S, D, inl, outsizes

    def batch(self, slots, disps, words=False):
        S, D, inl, outsizes = self._batch_args(slots, disps)
        out = np.zeros(max(sum(outsizes), 1), np.uint32)
        L.check(self.lib.nl_batch(len(slots), S, len(disps), D, _ptr(inl), _ptr(out)))
        return self._split(out, outsizes, words)

    def compile(self, slots, disps):
        S, D, inl, outsizes = self._batch_args(slots, disps)
        h = ctypes.c_uint32()
        L.check(self.lib.nl_compile(len(slots), S, len(disps), D, _ptr(inl), ctypes.byref(h)))
        return h.value, outsizes

    def run_compiled(self, h, outsizes, words=False):
        out = np.zeros(max(sum(outsizes), 1), np.uint32)
        L.check(self.lib.nl_run_compiled(h, _ptr(out)))
        return self._split(out, outsizes, words)

    def time_compiled(self, h, reps=1) -> float:
        ms = ctypes.c_double()
        L.check(self.lib.nl_time_compiled(h, reps, ctypes.byref(ms)))
        return ms.value

    def free_compiled(self, h):
        L.check(self.lib.nl_free_compiled(h))

    @staticmethod
    def _split(out, sizes, words):
        res, off = [], 0
        for s in sizes:
            w = out[off:off + s]
            res.append(w.copy() if words else bits_f32(w))
            off += s
        return res
