"""ctypes binding of libnelisp_cuda's C ABI (include/nelisp_cuda.h).

This is the reference-side binding a Python caller would write for the
library: every entry point of the header, with argument types, and an
exception for a non-zero status carrying nl_last_error().  Loading fails
loudly when the shared library has not been built; there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libnelisp_cuda.so")
BIN_DIR = os.path.join(PKG_DIR, "bin")

NL_OK, NL_ERROR, NL_FATAL = 0, 1, 2
RUN_IN, RUN_RESIDENT, RUN_OUT, RUN_INOUT = 0, 1, 2, 3
SLOT_IN, SLOT_RESIDENT, SLOT_TMP, SLOT_OUT = 0, 1, 2, 3
MAX_BUFS, MAX_PUSH, MAX_NAME = 16, 16, 63

_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t


class RunBuffer(ctypes.Structure):
    _fields_ = [("size", _u32), ("kind", _u32), ("handle", _u32)]


class Slot(ctypes.Structure):
    _fields_ = [("kind", _u32), ("size", _u32), ("handle", _u32)]


class Dispatch(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * (MAX_NAME + 1)), ("nbuf", _u32),
                ("slot", _u32 * MAX_BUFS), ("npush", _u32),
                ("push", _u32 * MAX_PUSH), ("groups", _u32)]


class NlError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libnelisp_cuda status {code}: {msg}")
        self.code = code


# name -> (restype, argtypes)
SIGNATURES = {
    "nl_init": (_i, [_i]),
    "nl_shutdown": (None, []),
    "nl_last_error": (ctypes.c_char_p, []),
    "nl_version": (ctypes.c_char_p, []),
    "nl_device": (_i, []),
    "nl_device_name": (ctypes.c_char_p, []),
    "nl_kernel_count": (_i, []),
    "nl_kernel_name": (ctypes.c_char_p, [_i]),
    "nl_kernel_arity": (_i, [ctypes.c_char_p, ctypes.POINTER(_u32), ctypes.POINTER(_u32)]),
    "nl_upload": (_i, [_vp, _u32, ctypes.POINTER(_u32)]),
    "nl_upload_file": (_i, [ctypes.c_char_p, _u64, _u32, ctypes.POINTER(_u32)]),
    "nl_write_resident": (_i, [_u32, _vp, _u32]),
    "nl_read_resident": (_i, [_u32, _vp, _u32]),
    "nl_free": (_i, [_u32]),
    "nl_resident_info": (_i, [_u32, ctypes.POINTER(_vp), ctypes.POINTER(_u32)]),
    "nl_run": (_i, [ctypes.c_char_p, _u32, ctypes.POINTER(RunBuffer), _u32,
                    ctypes.POINTER(_u32), _u32, _vp, _vp]),
    "nl_batch": (_i, [_u32, ctypes.POINTER(Slot), _u32, ctypes.POINTER(Dispatch), _vp, _vp]),
    "nl_compile": (_i, [_u32, ctypes.POINTER(Slot), _u32, ctypes.POINTER(Dispatch), _vp,
                        ctypes.POINTER(_u32)]),
    "nl_run_compiled": (_i, [_u32, _vp]),
    "nl_free_compiled": (_i, [_u32]),
    "nl_compiled_out_words": (_i, [_u32, ctypes.POINTER(_u64)]),
    "nl_time_compiled": (_i, [_u32, _u32, ctypes.POINTER(ctypes.c_double)]),
    "nl_dispatch_dev": (_i, [ctypes.c_char_p, _u32, ctypes.POINTER(_vp), ctypes.POINTER(_u32),
                             _u32, ctypes.POINTER(_u32), _u32, _vp]),
    "nl_ternary_workspace_bytes": (_sz, [_u32, _u32]),
    "nl_ternary_rows_dev": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32,
                                 _vp, _sz, _vp]),
    "nl_ternary_gemv_dev": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _sz, _vp]),
    "nl_ternary_gemv_batched_dev": (_i, [_u32, _vp, _u64, _vp, _u64, _vp, _u64, _vp, _u64,
                                         _u32, _u32, _u32, _vp, _sz, _vp]),
    "nl_ternary_gemv_static_dev": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "nl_decode_attn_rope_dev": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32,
                                     ctypes.c_float, _vp]),
    "nl_wait_status": (_i, []),
    "nl_upload_file_ternary": (_i, [ctypes.c_char_p, _u64, _u32, _u32, ctypes.c_int,
                                    ctypes.POINTER(_u32), ctypes.POINTER(_u32)]),
    "nl_selftest_wait_timeout": (_i, []),
    "nl_ternary_gemv_batched_host": (_i, [_u32, _vp, _u64, _vp, _u64, _vp, _u64, _vp, _u64,
                                          _u32, _u32, _u32]),
    "nl_ternary_gemv_host_submit": (_i, [_u32, _vp, _u64, _vp, _u64, _vp, _u64, _vp, _u64,
                                         _u32, _u32, _u32, ctypes.POINTER(_u64)]),
    "nl_host_wait": (_i, [_u64]),
    "nl_launch_count": (_u64, []),
    # decoder (nelisp_cuda.decoder rebinds these with the config struct)
    "nl_nccl_unique_id": (_i, [_vp]),
    "nl_decoder_create": (_i, [_vp, _i, _i, _vp, _i, ctypes.POINTER(_vp)]),
    "nl_decoder_create_from_weights": (_i, [_vp, _vp, _i, _i, _vp, _i, ctypes.POINTER(_vp)]),
    "nl_decoder_generate": (_i, [_vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp]),
    "nl_decoder_logits": (_i, [_vp, _vp, _u64]),
    "nl_decoder_info": (_i, [_vp, _vp, _vp, _vp]),
    "nl_decoder_shard": (_i, [_vp, _i, _i, _vp]),
    "nl_decoder_destroy": (None, [_vp]),
}

_lib = None


def _prefer_bundled_nccl() -> None:
    """Point the decoder's NCCL loader at the NCCL that ships with PyTorch
    (the `nvidia-nccl` wheel) when there is one.  The dynamic linker matches a
    dependency by soname against libraries already in the process, so an
    older system libnccl.so.2 opened first would be handed to libtorch_cuda
    later and fail its symbol lookups."""
    if os.environ.get("NELISP_NCCL_LIB"):
        return
    import importlib.util
    try:
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for d in (spec.submodule_search_locations or []) if spec else []:
        cand = os.path.join(d, "lib", "libnccl.so.2")
        if os.path.exists(cand):
            os.environ["NELISP_NCCL_LIB"] = cand
            return


def load(path: str = LIB_PATH):
    """Load libnelisp_cuda; raises if it is missing (no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"libnelisp_cuda is not built ({path} missing); run "
            "`python -c 'import __graft_entry__ as g; g.build()'` or `make -C nelisp-gpu_b200`")
    _prefer_bundled_nccl()
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != NL_OK:
        raise NlError(rc, load().nl_last_error().decode(errors="replace"))


def u32_array(values):
    vals = list(values)
    return (_u32 * max(len(vals), 1))(*vals)
