"""OP_UPLOAD_FILE at streaming speed and the on-device repacking of an f32
weight matrix into the two-bit GEMV format (nl_upload_file_ternary), plus the
reference's quantization operators (lisp/nelisp-gpu-kernels.el:496-561),
against the oracle (oracle/nl_oracle_misc.c).  File regions are exact; the
elementwise quantizers are bit-exact; the serial f32 accumulators of the
reference are matched within f32 rounding."""
import ctypes

import numpy as np
import pytest

import oracle as nlo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def host():
    from nelisp_cuda.host import Host
    return Host()


def g64(n):
    return max(1, (n + 63) // 64)


@pytest.mark.parametrize("offset,nwords", [(0, 10_000_003), (12, 10_000_000), (4096 * 3 + 36, 777),
                                           (5, 1000)])
def test_upload_file_region_exact(host, tmp_path, offset, nwords):
    """Regions spanning several 16 MiB staging slots, at offsets that are and
    are not 4 KiB aligned (the O_DIRECT path reads from the aligned start and
    skips the leading bytes)."""
    rng = np.random.default_rng(offset + nwords)
    data = rng.integers(0, 2 ** 32, size=10_000_050, dtype=np.uint64).astype(np.uint32)
    path = tmp_path / "w.bin"
    raw = data.tobytes()
    path.write_bytes(raw)
    h = host.upload_file(str(path), offset, nwords * 4)
    got = host.read_words(h, nwords)
    want = np.frombuffer(raw[offset:offset + nwords * 4], dtype=np.uint32)
    assert np.array_equal(got, want)
    host.free(h)


def test_upload_file_short_file_is_an_error(host, tmp_path):
    from nelisp_cuda import NlError
    path = tmp_path / "short.bin"
    path.write_bytes(np.arange(1000, dtype=np.uint32).tobytes())
    h0 = host.upload(np.zeros(4, np.uint32))
    host.free(h0)
    with pytest.raises(NlError) as e:
        host.upload_file(str(path), 8, 1000 * 4)
    assert "short read" in str(e.value)
    with pytest.raises(NlError):
        host.upload_file(str(tmp_path / "missing.bin"), 0, 16)
    assert host.upload(np.zeros(4, np.uint32)) == h0       # no handle leaked


def _ternary_upload(host, path, offset, rows, cols, per_row):
    from nelisp_cuda import _lib as L
    hw, hs = ctypes.c_uint32(), ctypes.c_uint32()
    L.check(host.lib.nl_upload_file_ternary(str(path).encode(), offset, rows, cols, int(per_row),
                                            ctypes.byref(hw), ctypes.byref(hs)))
    wng = (cols + 15) // 16
    return hw.value, hs.value, host.read_words(hw.value, rows * wng), \
        host.read_words(hs.value, rows).view(np.float32)


@pytest.mark.parametrize("per_row", [False, True])
@pytest.mark.parametrize("rows,cols,offset", [(2560, 2560, 0), (300, 1000, 44), (7, 9, 4)])
def test_upload_file_ternary_matches_oracle(host, tmp_path, per_row, rows, cols, offset):
    rng = np.random.default_rng(rows + cols + per_row)
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    path = tmp_path / "w32.bin"
    path.write_bytes(b"\0" * offset + W.tobytes())
    hw, hs, WP, S = _ternary_upload(host, path, offset, rows, cols, per_row)
    WPo, So = nlo.quant_w_pack(W.ravel(), rows, cols, per_row)
    # both sum |W| in f64, in different orders: the scales agree to a few ulp
    assert np.allclose(S, So, rtol=4e-7, atol=0)
    if np.array_equal(S, So):
        assert np.array_equal(WP, WPo)
    else:   # a trit may only differ where W / beta sits on a threshold
        wng = (cols + 15) // 16
        diff = (WP != WPo).reshape(rows, wng)
        for o, wi in zip(*np.nonzero(diff)):
            c = np.arange(16 * wi, min(16 * wi + 16, cols))
            q = np.abs(W[o, c] / So[o])
            assert np.min(np.abs(q - 0.5)) < 1e-5
    host.free(hw)
    host.free(hs)


def test_upload_file_ternary_gemv_equals_fake_quant_matmul(host, tmp_path):
    """The repacked weights through the ternary GEMV reproduce quant-w's
    fake-quantized f32 weights times x (per-row scales)."""
    import torch
    from nelisp_cuda import dev
    rng = np.random.default_rng(5)
    rows, cols, seq = 1024, 2048, 3
    W = rng.standard_normal((rows, cols)).astype(np.float32)
    path = tmp_path / "w.bin"
    path.write_bytes(W.tobytes())
    hw, hs, WP, S = _ternary_upload(host, path, 0, rows, cols, True)
    X = rng.standard_normal((seq, cols)).astype(np.float32)
    d = torch.device("cuda")
    tY = torch.empty(seq * rows, dtype=torch.float32, device=d)
    dev.ternary_gemv(torch.from_numpy(X.ravel()).to(d), torch.from_numpy(WP.view(np.int32)).to(d),
                     torch.from_numpy(S).to(d), tY, seq, rows, cols)
    torch.cuda.synchronize()
    WQ = np.stack([nlo.quant_w(W[o], np.float32(S[o]) * np.float32(cols), cols) for o in range(rows)])
    want = (X.astype(np.float64) @ WQ.astype(np.float64).T).ravel()
    assert nlo.tk_err(tY.cpu().numpy(), want) < 1e-5
    host.free(hw)
    host.free(hs)


def test_quant_w_and_quant_act_ops(host):
    rng = np.random.default_rng(6)
    n = 5000
    W = rng.standard_normal(n).astype(np.float32)
    S0 = float(np.abs(W).sum())
    got = host.run2("quant-w", [("in", W), ("in", [S0]), ("out", n)], [n], g64(n))[0]
    assert np.array_equal(got, nlo.quant_w(W, np.float32(S0), n))
    seq, cols = 5, 3000
    X = (rng.standard_normal(seq * cols) * 2).astype(np.float32)
    got = host.run2("quant-act", [("in", X), ("out", seq * cols)], [seq, cols], 1)[0]
    assert np.array_equal(got, nlo.quant_act(X, seq, cols))


def test_accumulator_and_clip_ops(host):
    rng = np.random.default_rng(7)
    n = 100_000
    G = rng.standard_normal(n).astype(np.float32)
    # The device sums in f64 and rounds once; the reference's single thread
    # sums serially in f32.  Both are checked against the exact sum: ours to
    # f32 rounding, the reference's (the oracle) to its serial bound n * 2^-24.
    G64 = G.astype(np.float64)
    for name, acc0, exact, ref in [
            ("absmean-acc", 3.0, 3.0 + np.abs(G64).sum(), nlo.absmean_acc(G, 3.0, n)),
            ("sumsq-acc", 0.5, 0.5 + (G64 ** 2).sum(), nlo.sumsq_acc(G, 0.5, n))]:
        got = host.run2(name, [("in", G), ("inout", [acc0])], [n], 1)[0][0]
        assert abs(got - exact) <= 2.0 ** -22 * exact, name
        assert abs(ref - exact) <= n * 2.0 ** -24 * exact, name
    for gsq, cfg in [(9.0, 1.0), (0.01, 1.0), (0.0, 0.5)]:
        got = host.run2("clip-scale", [("in", [gsq]), ("in", [cfg]), ("out", 1)], [1], 1)[0][0]
        assert got == nlo.clip_scale(gsq, cfg)
