"""Pin the CPU restatements of the remaining reference operators
(oracle/nl_oracle_misc.c) against independent numpy transcriptions of the
reference formulas (lisp/nelisp-gpu-kernels.el, lines cited per test) and
against test/verify.el's causal-mask known answer."""
import numpy as np
import pytest

import oracle as nlo


def test_causal_mask_verify_el():
    # test/verify.el:110-117: S = 1..36 (6x6), j > i -> -1e30
    n = 6
    S = np.arange(1, n * n + 1, dtype=np.float32)
    got = nlo.causal_mask(S, n).reshape(n, n)
    want = S.reshape(n, n).copy()
    want[np.triu_indices(n, 1)] = -1.0e30
    assert np.array_equal(got, want)


def test_matmul_at():
    # :177-186, C[m,n] = sum_k A[k,m] B[k,n]
    rng = np.random.default_rng(1)
    M, K, N = 13, 29, 7
    A = rng.standard_normal((K, M)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    got = nlo.matmul_at(A.ravel(), B.ravel(), M, K, N)
    assert nlo.tk_err(got, (A.astype(np.float64).T @ B).ravel()) < 1e-6


@pytest.mark.parametrize("heads,kvheads", [(4, 4), (4, 2), (6, 1)])
def test_attn_scores_and_context(heads, kvheads):
    # :208-235
    rng = np.random.default_rng(heads + kvheads)
    seq, hd = 9, 8
    dim, kvdim, grp = heads * hd, kvheads * hd, heads // kvheads
    Q = rng.standard_normal((seq, dim)).astype(np.float32)
    K = rng.standard_normal((seq, kvdim)).astype(np.float32)
    V = rng.standard_normal((seq, kvdim)).astype(np.float32)
    S = nlo.attn_scores(Q.ravel(), K.ravel(), seq, dim, heads, kvheads).reshape(heads, seq, seq)
    P = rng.random((heads, seq, seq)).astype(np.float32)
    C = nlo.attn_context(P.ravel(), V.ravel(), seq, dim, heads, kvheads).reshape(seq, dim)
    for h in range(heads):
        kv = h // grp
        q = Q[:, h * hd:(h + 1) * hd].astype(np.float64)
        k = K[:, kv * hd:(kv + 1) * hd].astype(np.float64)
        ws = q @ k.T / np.sqrt(hd)
        mask = np.triu(np.ones((seq, seq), bool), 1)
        assert np.all(S[h][mask] == np.float32(-1.0e30))
        assert np.max(np.abs(S[h][~mask] - ws[~mask])) < 1e-5
        wc = P[h].astype(np.float64) @ V[:, kv * hd:(kv + 1) * hd]
        assert np.max(np.abs(C[:, h * hd:(h + 1) * hd] - wc)) < 1e-5


def _halves(words):
    w = np.asarray(words, np.uint32)
    return (w & 0xFFFF).astype(np.float32), (w >> 16).astype(np.float32)


def _lanes(words):
    return np.asarray(words, np.uint32).view(np.uint8).view(np.int8).astype(np.int64).reshape(-1, 4)


def test_dp4a_dot_and_bitlinear():
    # :592-620: words rebuilt as lo + hi * 65536; signed 4x8 dot in int32
    rng = np.random.default_rng(3)
    n = 257
    a = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    b = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    got = nlo.dp4a_dot(*_halves(a), *_halves(b), n)
    assert np.array_equal(got, (_lanes(a) * _lanes(b)).sum(1).astype(np.float32))
    seq, out, ng = 3, 5, 11
    A = rng.integers(0, 2 ** 32, seq * ng, dtype=np.uint64).astype(np.uint32)
    W = rng.integers(0, 2 ** 32, out * ng, dtype=np.uint64).astype(np.uint32)
    bias = rng.standard_normal(out).astype(np.float32)
    beta = np.array([0.75], np.float32)
    gamma = rng.random(seq).astype(np.float32)
    Y = nlo.bitlinear_dp4a(*_halves(A), *_halves(W), bias, beta, gamma, seq, out, ng)
    acc = _lanes(A).reshape(seq, ng * 4) @ _lanes(W).reshape(out, ng * 4).T
    want = bias[None, :] + (beta[0] * gamma[:, None]) * acc.astype(np.float32)
    assert np.array_equal(Y.reshape(seq, out), want.astype(np.float32))


def test_dp4a_rows_t():
    # :792-810: X[p, i] = sum_o sv(o, i) * (BETA[o] * G[p, o])
    rng = np.random.default_rng(4)
    out, cols, seq = 9, 22, 3
    ng = (cols + 3) // 4
    WP = rng.integers(0, 2 ** 32, out * ng, dtype=np.uint64).astype(np.uint32)
    beta = rng.random(out).astype(np.float32)
    G = rng.standard_normal((seq, out)).astype(np.float32)
    X = nlo.dp4a_rows_t(WP, beta, G.ravel(), out, cols, ng, seq).reshape(seq, cols)
    sv = _lanes(WP).reshape(out, ng * 4)[:, :cols].astype(np.float64)
    want = (G.astype(np.float64) * beta[None, :]) @ sv
    assert np.max(np.abs(X - want)) < 1e-4


def test_rmsnorm_heads_rope_silu_scale_rows():
    rng = np.random.default_rng(5)
    seq, heads, hd = 4, 3, 16
    X = rng.standard_normal((seq, heads, hd)).astype(np.float32)
    G = rng.random(hd).astype(np.float32)
    # :828-845, eps 1e-6
    Y = nlo.rmsnorm_heads(X.ravel(), G, seq, heads, hd).reshape(seq, heads, hd)
    x64 = X.astype(np.float64)
    want = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * G
    assert np.max(np.abs(Y - want)) < 1e-5
    # :1290-1303, adjacent pairs, SG = -1 inverts SG = +1
    dim, half = heads * hd, hd // 2
    ang = rng.uniform(0, 6.3, (seq, half))
    co, si = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    R = nlo.rope_apply(X.ravel(), co.ravel(), si.ravel(), [1.0], seq, dim, heads)
    back = nlo.rope_apply(R, co.ravel(), si.ravel(), [-1.0], seq, dim, heads)
    assert np.max(np.abs(back - X.ravel())) < 1e-5
    a0, a1 = x64[..., 0::2], x64[..., 1::2]
    c, s = co[:, None, :], si[:, None, :]
    r = R.reshape(seq, heads, hd)
    assert np.max(np.abs(r[..., 0::2] - (a0 * c - a1 * s))) < 1e-5
    assert np.max(np.abs(r[..., 1::2] - (a0 * s + a1 * c))) < 1e-5
    # :1306-1312, :1365-1372
    v = rng.standard_normal(100).astype(np.float32) * 4
    assert np.max(np.abs(nlo.silu(v, 100) - v / (1 + np.exp(-v.astype(np.float64))))) < 1e-5
    Yr = rng.standard_normal((7, 5)).astype(np.float32)
    S = rng.standard_normal(7).astype(np.float32)
    assert np.array_equal(nlo.scale_rows(Yr.ravel(), S, 7, 5).reshape(7, 5), Yr * S[:, None])


def test_quantization_family_restatements():
    rng = np.random.default_rng(11)
    # :550-561 quant-w, beta = S[0] / n, thresholds at +-0.5
    W = rng.standard_normal(200).astype(np.float32)
    S0 = np.float32(np.abs(W).sum())
    WQ = nlo.quant_w(W, S0, 200)
    beta = np.float32(S0 / np.float32(200))
    q = W / beta
    want = beta * np.where(q >= 0.5, 1.0, np.where(q <= -0.5, -1.0, 0.0)).astype(np.float32)
    assert np.array_equal(WQ, want.astype(np.float32))
    assert not nlo.quant_w(W, 0.0, 200).any()                 # beta 0: all zero
    # :529-548 quant-act: gamma = max|x|/127, round by truncating |q| + 0.5
    X = (rng.standard_normal((3, 50)) * 3).astype(np.float32)
    XQ = nlo.quant_act(X.ravel(), 3, 50).reshape(3, 50)
    for r in range(3):
        g = np.float32(np.abs(X[r]).max() / np.float32(127.0))
        qq = X[r] / g
        rf = np.minimum(np.floor(np.abs(qq) + np.float32(0.5)), 127).astype(np.float32)
        assert np.array_equal(XQ[r], (g * (np.sign(qq) * rf)).astype(np.float32))
    # :505-512 clip-scale and the accumulators
    assert nlo.clip_scale(4.0, 1.0) == np.float32(1.0) / np.sqrt(np.float32(4.0) + np.float32(1e-12))
    assert nlo.clip_scale(0.25, 1.0) == 1.0
    G = rng.standard_normal(1000).astype(np.float32)
    assert abs(nlo.absmean_acc(G, 2.0, 1000) - (2.0 + np.abs(G.astype(np.float64)).sum())) < 1e-3
    assert abs(nlo.sumsq_acc(G, 0.0, 1000) - (G.astype(np.float64) ** 2).sum()) < 1e-2


@pytest.mark.parametrize("per_row", [False, True])
def test_quant_w_pack_decodes_to_quant_w(per_row):
    """The repacked weights decode (two-bit codes x row scale) to quant-w's
    fake-quantized values with beta = mean |W| of the tensor or the row."""
    rng = np.random.default_rng(12 + per_row)
    rows, cols = 9, 37
    W = rng.standard_normal((rows, cols)).astype(np.float32)
    WP, S = nlo.quant_w_pack(W.ravel(), rows, cols, per_row)
    wng = (cols + 15) // 16
    codes = np.zeros((rows, wng * 16), np.int64)
    w = WP.reshape(rows, wng)
    for f in range(16):
        c = (w >> np.uint32(2 * f)) & 3
        codes[:, f::16] = np.where(c == 1, 1, np.where(c == 3, -1, 0))
    assert not codes[:, cols:].any()
    dec = codes[:, :cols] * S[:, None]
    for o in range(rows):
        n = cols if per_row else rows * cols
        S0 = np.abs(W[o] if per_row else W).astype(np.float64).sum()
        want = nlo.quant_w(W[o], np.float32(S0), n) if per_row else None
        if per_row:
            # beta rounds the f64 mean once; quant-w divides two f32 values:
            # the scales may differ in the last bit, the trits may not
            assert abs(S[o] - np.float32(S0 / n)) <= 1e-6 * S[o]
            assert np.array_equal(codes[o, :cols], np.sign(want).astype(np.int64))
        else:
            assert S[o] == S[0]
    if not per_row:
        assert abs(S[0] - np.abs(W.astype(np.float64)).mean()) <= 1e-6 * S[0]


def test_decoder_tensor_export_shapes_and_values():
    """The CPU model's weights exported per tensor: packed trits decode to
    {-1, 0, +1} in about equal shares, scales lie in [0.5, 1.5) / sqrt(2K/3)."""
    cfg = dict(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=300,
               rms_eps=1e-5, rope_base=10000.0, seed=5, max_batch=1, max_seq=4)
    w = nlo.decoder_tensor(cfg, 1, "wgate")
    assert w.dtype == np.uint32 and w.size == 512 * 256 // 16
    codes = (w[:, None] >> (2 * np.arange(16, dtype=np.uint32))) & 3
    share = [(codes == c).mean() for c in (0, 1, 3)]
    assert (codes != 2).all() and all(0.3 < x < 0.37 for x in share)
    s = nlo.decoder_tensor(cfg, 0, "sdown")
    rs = 1.0 / np.sqrt(2.0 * 512 / 3.0)
    assert s.size == 256 and (s >= 0.5 * rs * 0.999).all() and (s < 1.5 * rs * 1.001).all()
    assert nlo.decoder_tensor(cfg, 0, "embed").size == 300 * 256
