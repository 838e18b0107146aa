"""Typed entry points on device tensors (torch is only the allocator here).

Each function passes raw device pointers and the current CUDA stream to the
C ABI; the arithmetic is libnelisp_cuda's.  Tensors must be contiguous CUDA
tensors of the stated dtype.
"""
from __future__ import annotations

import ctypes

from . import _lib as L


_ready = False


def _lib():
    """The library, with its context on the current torch device."""
    global _ready
    lib = L.load()
    if not _ready:
        import torch
        L.check(lib.nl_init(torch.cuda.current_device()))
        _ready = True
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _check_tensor(t, dtype_name):
    if t is None:
        return
    if not t.is_cuda or not t.is_contiguous() or str(t.dtype) != dtype_name:
        raise ValueError(f"expected a contiguous CUDA {dtype_name} tensor")


def dispatch(name, bufs, push, groups, stream=None):
    """Any registry kernel (a reference DSL name) on device tensors; the
    32-bit word count of each tensor is its bounds for the checks."""
    lib = _lib()
    n = len(bufs)
    ptrs = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in bufs])
    words = (ctypes.c_uint32 * max(n, 1))(*[t.numel() * t.element_size() // 4 for t in bufs])
    L.check(lib.nl_dispatch_dev(name.encode(), n, ptrs, words, len(push), L.u32_array(push),
                                groups, _stream(stream)))


def ternary_workspace_bytes(seq: int, cols: int) -> int:
    return int(_lib().nl_ternary_workspace_bytes(seq, cols))


def ternary_rows(X, WP, BIAS, BETA, Y, seq, out, cols, nblk, wng, workspace=None, stream=None):
    _check_tensor(X, "torch.float32"); _check_tensor(Y, "torch.float32")
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    L.check(_lib().nl_ternary_rows_dev(_p(X), _p(WP), _p(BIAS), _p(BETA), _p(Y), seq, out,
                                         cols, nblk, wng, _p(workspace), ws_bytes,
                                         _stream(stream)))


def ternary_gemv(X, WP, S, Y, seq, out, cols, bias=None, workspace=None, stream=None):
    """Y = diag(S) (W X) (+ bias): per-row scales."""
    _check_tensor(X, "torch.float32"); _check_tensor(Y, "torch.float32")
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    L.check(_lib().nl_ternary_gemv_dev(_p(X), _p(WP), _p(S), _p(bias), _p(Y), seq, out, cols,
                                         _p(workspace), ws_bytes, _stream(stream)))


def ternary_gemv_batched(count, X, x_stride, WP, w_stride, S, s_stride, Y, y_stride, seq, out,
                         cols, workspace=None, stream=None):
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    L.check(_lib().nl_ternary_gemv_batched_dev(count, _p(X), x_stride, _p(WP), w_stride, _p(S),
                                                 s_stride, _p(Y), y_stride, seq, out, cols,
                                                 _p(workspace), ws_bytes, _stream(stream)))


def decode_attn_rope(QKV, CK, CV, POS, C, batch, heads, kv_heads, head_dim, max_seq,
                     rope_base=10000.0, stream=None):
    """One decode position: RoPE of q and the new key at POS[0] (int32 on the
    device), the cache append of key and value, attention over 0..POS[0]."""
    for t in (QKV, CK, CV, C):
        _check_tensor(t, "torch.float32")
    _check_tensor(POS, "torch.int32")
    L.check(_lib().nl_decode_attn_rope_dev(_p(QKV), _p(CK), _p(CV), _p(POS), _p(C), batch, heads,
                                             kv_heads, head_dim, max_seq, rope_base,
                                             _stream(stream)))


def launch_count() -> int:
    return int(L.load().nl_launch_count())
