"""Request encoders against the byte layout of lisp/nelisp-gpu-server.el
(run2 :240-289, batch body :300-331, upload-file :168-195)."""
import struct

from nelisp_cuda import protocol as P


def words(b):
    return list(struct.unpack(f"<{len(b) // 4}I", b))


def test_run_layout():
    req, outs = P.encode_run("add2", [("in", [1.0, 2.0]), ("res", 7, 2), ("out", 2)], [2], 1)
    w = words(req[:12])
    assert w == [0, 4, int.from_bytes(b"add2", "little")]
    rest = words(req[12:])
    # nbuf; (size kind) (size kind handle) (size kind); npush push; groups; inline
    assert rest == [3, 2, 0, 2, 1, 7, 2, 2, 1, 2, 1, 0x3F800000, 0x40000000]
    assert outs == [2]


def test_inout_is_returned_and_sent():
    req, outs = P.encode_run("scale", [("inout", [0.5])], [], 1)
    assert outs == [1] and words(req[-4:]) == [0x3F000000]


def test_batch_layout_and_kind_numbering():
    body, outs = P.encode_batch_body(
        [("in", [1.0]), ("res", 3, 4), ("tmp", 5), ("out", 6)],
        [("softmax", [0, 3], [1, 6], 1)])
    w = words(body[:4 * 12])
    # slots: kind size [handle] -- kind/size order differs from RUN's size/kind
    assert w[:11] == [4, 0, 1, 1, 4, 3, 2, 5, 3, 6, 1]
    assert w[11] == 7                      # name length of "softmax"
    assert outs == [6]


def test_upload_file_layout():
    req = P.encode_upload_file("/tmp/x.bin", (5 << 32) + 48, 4096)
    w = words(req[:8])
    assert w == [8, len("/tmp/x.bin")]
    tail = words(req[8 + len("/tmp/x.bin"):])
    assert tail == [48, 5, 1024]
