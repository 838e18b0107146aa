"""Request encoders of the reference's server protocol.

A restatement of the byte layout lisp/nelisp-gpu-server.el builds (the Emacs
client cannot run here), shared by the subprocess client (server.py) and the
tests.  Buffer descriptors follow the Elisp forms:

  run2 descs  : ("in", vec) | ("res", handle, size) | ("out", size) | ("inout", vec)
  batch slots : ("in", vec) | ("res", handle, size) | ("tmp", size) | ("out", size)
  dispatches  : (name, [slot indices], [push constants], groups)
"""
from __future__ import annotations

from .f32codec import floats_bytes, u32_bytes

OP_RUN, OP_UPLOAD, OP_FREE, OP_BATCH, OP_COMPILE = 0, 1, 2, 3, 4
OP_RUN_COMPILED, OP_FREE_COMPILED, OP_WRITE_RESIDENT, OP_UPLOAD_FILE = 5, 6, 7, 8


def _name(name) -> bytes:
    s = name if isinstance(name, str) else str(name)
    return s.encode("utf-8")


def encode_run(name, descs, push, groups):
    """`nelisp-gpu-server-run2' (server.el:240-289).  Returns (request bytes,
    output sizes in binding order)."""
    nm = _name(name)
    parts = [u32_bytes(OP_RUN), u32_bytes(len(nm)), nm, u32_bytes(len(descs))]
    inline, outsizes = [], []
    for d in descs:
        kind = d[0]
        if kind == "in":
            parts += [u32_bytes(len(d[1])), u32_bytes(0)]
            inline.append(d[1])
        elif kind == "res":
            parts += [u32_bytes(d[2]), u32_bytes(1), u32_bytes(d[1])]
        elif kind == "out":
            parts += [u32_bytes(d[1]), u32_bytes(2)]
            outsizes.append(int(d[1]))
        elif kind == "inout":
            parts += [u32_bytes(len(d[1])), u32_bytes(3)]
            inline.append(d[1])
            outsizes.append(len(d[1]))
        else:
            raise ValueError(f"bad descriptor kind {kind!r}")
    parts.append(u32_bytes(len(push)))
    parts += [u32_bytes(p) for p in push]
    parts.append(u32_bytes(groups))
    parts.append(floats_bytes(*inline))
    return b"".join(parts), outsizes


def encode_batch_body(slots, disps):
    """`nelisp-gpu--batch-body' (server.el:300-331): the body after the
    opcode.  Returns (body bytes, output sizes in slot order)."""
    parts = [u32_bytes(len(slots))]
    inline, outsizes = [], []
    for s in slots:
        kind = s[0]
        if kind == "in":
            parts += [u32_bytes(0), u32_bytes(len(s[1]))]
            inline.append(s[1])
        elif kind == "res":
            parts += [u32_bytes(1), u32_bytes(s[2]), u32_bytes(s[1])]
        elif kind == "tmp":
            parts += [u32_bytes(2), u32_bytes(s[1])]
        elif kind == "out":
            parts += [u32_bytes(3), u32_bytes(s[1])]
            outsizes.append(int(s[1]))
        else:
            raise ValueError(f"bad slot kind {kind!r}")
    parts.append(u32_bytes(len(disps)))
    for name, slotidx, pushv, grp in disps:
        nm = _name(name)
        parts += [u32_bytes(len(nm)), nm, u32_bytes(len(slotidx))]
        parts += [u32_bytes(i) for i in slotidx]
        parts.append(u32_bytes(len(pushv)))
        parts += [u32_bytes(p) for p in pushv]
        parts.append(u32_bytes(grp))
    parts.append(floats_bytes(*inline))
    return b"".join(parts), outsizes


def encode_upload(vec) -> bytes:
    return u32_bytes(OP_UPLOAD) + u32_bytes(len(vec)) + floats_bytes(vec)


def encode_upload_words(words) -> bytes:
    import numpy as np
    w = np.asarray(words, dtype="<u4")
    return u32_bytes(OP_UPLOAD) + u32_bytes(w.size) + w.tobytes()


def encode_upload_bytes(raw: bytes) -> bytes:
    if len(raw) % 4:
        raise ValueError(f"upload-bytes: {len(raw)} bytes is not a whole number of uint32 words")
    return u32_bytes(OP_UPLOAD) + u32_bytes(len(raw) // 4) + raw


def encode_upload_file(path: str, offset: int, nbytes: int) -> bytes:
    if nbytes % 4:
        raise ValueError(f"upload-file: {nbytes} bytes is not a whole number of uint32 words")
    full = path.encode("utf-8")
    return (u32_bytes(OP_UPLOAD_FILE) + u32_bytes(len(full)) + full +
            u32_bytes(offset & 0xFFFFFFFF) + u32_bytes(offset >> 32) + u32_bytes(nbytes // 4))


def encode_free(h) -> bytes:
    return u32_bytes(OP_FREE) + u32_bytes(h)


def encode_write_resident(h, vec) -> bytes:
    return u32_bytes(OP_WRITE_RESIDENT) + u32_bytes(h) + u32_bytes(len(vec)) + floats_bytes(vec)


def encode_run_compiled(h) -> bytes:
    return u32_bytes(OP_RUN_COMPILED) + u32_bytes(h)


def encode_free_compiled(h) -> bytes:
    return u32_bytes(OP_FREE_COMPILED) + u32_bytes(h)
