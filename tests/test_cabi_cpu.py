"""The C-ABI library on a machine without a GPU: it loads, exports every
function include/nelisp_cuda.h declares, answers registry queries, and fails
cleanly (status, message) where a device is needed."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "nelisp_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nl_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from nelisp_cuda import _lib
    if not os.path.exists(_lib.LIB_PATH):
        _lib_build()
    return _lib.load()


def _lib_build():
    from nelisp_cuda.build import build
    build()


def test_header_declares_the_opcode_surface():
    fns = declared_functions()
    for name in ["nl_init", "nl_upload", "nl_upload_file", "nl_write_resident", "nl_free",
                 "nl_run", "nl_batch", "nl_compile", "nl_run_compiled", "nl_free_compiled",
                 "nl_ternary_gemv_dev", "nl_dispatch_dev"]:
        assert name in fns


def test_library_exports_every_declared_symbol(lib):
    from nelisp_cuda import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (nl_[a-z0-9_]+)$", out, flags=re.M))
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, missing
    # and the ctypes binding covers the header
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_registry_names_the_reference_kernels(lib):
    names = {lib.nl_kernel_name(i).decode() for i in range(lib.nl_kernel_count())}
    hot = {"ternary-rows", "ternary-rows-t", "bitlinear-packed", "bitlinear-packed-v",
           "pack-act-rows", "bitlinear-dp4a-rows", "bitlinear-dp4a-1f", "matmul",
           "matmul-tiled", "matmul-reg", "linear", "softmax", "silu-mul", "add2",
           "rmsnorm-istd", "rmsnorm-fwd", "rope-half", "decode-rope", "decode-rope-b",
           "cache-append", "cache-append-b", "decode-attn", "decode-attn-b", "attn-causal-gqa",
           "embed-gather", "scale",
           # paged / streaming KV caches
           "cache-append-ring", "decode-attn-stream", "qkv-append", "attn-stream-entries",
           "cache-append-paged", "decode-attn-paged", "block-copy", "decode-rope-b-v",
           "cache-append-paged-v", "decode-attn-paged-v",
           # unfused prefill attention, QK-norm, RoPE, DP4A spikes, backward GEMMs
           "matmul-at", "causal-mask", "attn-scores", "attn-context", "dp4a-dot",
           "bitlinear-dp4a", "dp4a-rows-t", "rmsnorm-heads", "rope-apply", "silu", "scale-rows",
           # BitNet quantization family
           "sumsq-acc", "clip-scale", "absmean-acc", "quant-act", "quant-w",
           # training-side operators
           "transpose", "slice-cols", "set-cols", "silu-mul-bwd", "silu-bwd", "gelu-bwd",
           "sub-scale", "sgd", "adam", "colsum", "rmsnorm-dgamma", "rmsnorm-dx", "softmax-bwd",
           "rowdot", "ce-grad", "ce-grad-idx", "topk-mask", "embed-bwd", "gather-spike",
           "scatter-spike", "gdn-step", "tree-attn", "attn-sc-dq", "attn-sc-dk", "attn-ctx-dp",
           "attn-ctx-dv"}
    assert hot <= names
    nb, npush = ctypes.c_uint32(), ctypes.c_uint32()
    assert lib.nl_kernel_arity(b"ternary-rows", ctypes.byref(nb), ctypes.byref(npush)) == 0
    assert (nb.value, npush.value) == (5, 5)      # (X WP BIAS BETA Y) (seq out cols nblk wng)
    assert lib.nl_kernel_arity(b"decode-attn-b", ctypes.byref(nb), ctypes.byref(npush)) == 0
    assert (nb.value, npush.value) == (5, 5)
    for name, arity in [(b"bitlinear-dp4a", (8, 3)), (b"dp4a-rows-t", (4, 4)),
                        (b"attn-scores", (3, 4)), (b"rope-apply", (5, 3))]:
        assert lib.nl_kernel_arity(name, ctypes.byref(nb), ctypes.byref(npush)) == 0
        assert (nb.value, npush.value) == arity, name
    assert lib.nl_kernel_arity(b"no-such-kernel", None, None) == 1


def test_no_device_is_a_clean_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc = lib.nl_init(-1)
    assert rc == 2 and b"CUDA" in lib.nl_last_error()


def test_binaries_are_built():
    from nelisp_cuda import _lib
    for b in ["nelisp-cuserver", "vkrun", "vkmatmul", "vksoftmax"]:
        assert os.access(os.path.join(_lib.BIN_DIR, b), os.X_OK), b


def test_server_usage_without_dir():
    from nelisp_cuda import _lib
    r = subprocess.run([os.path.join(_lib.BIN_DIR, "nelisp-cuserver")], capture_output=True)
    assert r.returncode == 1 and b"usage" in r.stderr
