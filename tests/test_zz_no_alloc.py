"""nl_ternary_gemv_static_dev: the ternary GEMV on the library's file-scope
device workspace, for callers that cannot let a library allocate (an
allocator-owning host runtime, a real-time loop).  Called through the C ABI
against nl_ternary_gemv_dev with a caller-provided workspace on the same
inputs, two calls in a row: the two run the same kernels, so the outputs must
be the same bits, and both within tk-err 1e-5 (the bar of the ternary tests)
of the CPU oracle.  Also its size limit, and its refusal to run before
nl_init in a fresh process (the library would otherwise have to allocate its
wait flag).

Collected last (file name) so that it also runs after every other GPU test in
the same process; it needs nothing from them and passes alone as well.
"""
import ctypes

import numpy as np
import pytest

import oracle as nlo

pytestmark = pytest.mark.gpu
TOL = 1e-5
STATIC_MAX = 2 << 20   # NL_TERNARY_STATIC_WS_BYTES


def _pack(t):
    out, cols = t.shape
    codes = np.where(t == 1, 1, np.where(t == -1, 3, 0)).astype(np.uint32)
    w = np.zeros((out, cols // 16), np.uint32)
    for f in range(16):
        w |= codes[:, f::16] << np.uint32(2 * f)
    return w.ravel()


def _problem(rng, seq, out, cols):
    import torch
    t = rng.integers(-1, 2, size=(out, cols))
    X = rng.standard_normal((seq, cols)).astype(np.float32)
    S = rng.uniform(0.5, 1.5, size=out).astype(np.float32)
    B = rng.uniform(-0.2, 0.2, size=out).astype(np.float32)
    dev = torch.device("cuda", torch.cuda.current_device())
    WP = torch.from_numpy(_pack(t).view(np.int32)).to(dev)
    return (torch.from_numpy(X).to(dev), WP, torch.from_numpy(S).to(dev),
            torch.from_numpy(B).to(dev))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    from nelisp_cuda import dev
    return dev._lib()   # the library, initialised on the current torch device


def test_static_workspace_matches_caller_workspace(lib):
    import torch
    from nelisp_cuda import _lib as L
    rng = np.random.default_rng(20261201)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # decode shapes, the tcgen05 GEMV (6-16 rows), a ragged row count, and
    # more than 16 rows (the tcgen05 GEMM, whose workspace must also fit)
    cases = [(1, 4096, 4096), (5, 2560, 6912), (16, 1024, 2560), (3, 700, 4096),
             (40, 1024, 2560)]
    probs = [_problem(rng, *c) for c in cases]
    ws = torch.empty(max(int(lib.nl_ternary_workspace_bytes(s, c)) for s, _, c in cases),
                     dtype=torch.uint8, device=probs[0][0].device)
    outs = [(torch.empty(s, o, device=ws.device), torch.empty(s, o, device=ws.device))
            for s, o, _ in cases]
    free0 = None
    for rep in range(2):                     # two calls in a row per shape
        if rep == 1:
            # Every kernel involved has run once (and been loaded); the second
            # round of calls must leave the device's free memory where it was.
            torch.cuda.synchronize()
            free0, _ = torch.cuda.mem_get_info()
        for (seq, out, cols), (X, WP, S, B), (ys, yr) in zip(cases, probs, outs):
            ys.fill_(float("nan"))
            yr.fill_(float("nan"))
            L.check(lib.nl_ternary_gemv_static_dev(_p(X), _p(WP), _p(S), _p(B), _p(ys), seq,
                                                   out, cols, stream))
            L.check(lib.nl_ternary_gemv_dev(_p(X), _p(WP), _p(S), _p(B), _p(yr), seq, out,
                                            cols, _p(ws), ws.numel(), stream))
            torch.cuda.synchronize()
            a, r = ys.cpu().numpy(), yr.cpu().numpy()
            assert np.isfinite(a).all()
            assert np.array_equal(a.view(np.uint32), r.view(np.uint32)), (rep, seq, out, cols)
            if rep == 0:
                # ternary-rows with the row scale in each of its 128-column blocks
                nblk = (cols + 127) // 128
                want = nlo.ternary_rows(X.cpu().numpy().ravel(),
                                        WP.cpu().numpy().view(np.uint32), B.cpu().numpy(),
                                        np.repeat(S.cpu().numpy(), nblk), seq, out, cols, nblk,
                                        cols // 16)
                err = nlo.tk_err(a.ravel(), want.ravel())
                assert err < TOL, (seq, out, cols, err)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 >= free0


def test_static_workspace_rejects_oversize(lib):
    import torch
    from nelisp_cuda import _lib as L
    # seq 16 needs 48 bytes per column plus a 1280-byte tail (row scales,
    # flags and offset sums): 43664 columns is the widest row that fits
    cols = 43664 + 16
    assert lib.nl_ternary_workspace_bytes(16, cols) > STATIC_MAX
    assert lib.nl_ternary_workspace_bytes(16, 43664) <= STATIC_MAX
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.nl_ternary_gemv_static_dev(None, None, None, None, None, 16, 8, cols, stream)
    assert rc == L.NL_ERROR
    msg = lib.nl_last_error().decode()
    assert "static maximum" in msg and str(STATIC_MAX) in msg
    # a prefill-sized request: the tcgen05 GEMM's limb matrix does not fit
    assert lib.nl_ternary_workspace_bytes(512, 2560) > STATIC_MAX
    rc = lib.nl_ternary_gemv_static_dev(None, None, None, None, None, 512, 8, 2560, stream)
    assert rc == L.NL_ERROR
    assert "static maximum" in lib.nl_last_error().decode()


_FRESH = r"""
import sys
sys.path[:0] = [{root!r}, {pkg!r}]
from nelisp_cuda import _lib as L
lib = L.load()
rc = lib.nl_ternary_gemv_static_dev(None, None, None, None, None, 1, 16, 128, None)
msg = lib.nl_last_error().decode()
assert rc == L.NL_ERROR and "nl_init" in msg, (rc, msg)
L.check(lib.nl_init(0))
print("FRESH_OK")
"""


def test_static_refused_before_init():
    """In a fresh process, before nl_init: refused with a message, nothing
    launched and nothing allocated."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = _FRESH.format(root=root, pkg=os.path.join(root, "nelisp-gpu_b200"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "FRESH_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
