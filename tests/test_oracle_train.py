"""Pin the CPU restatements of the reference's training-side operators
(oracle/nl_oracle_misc.c) against test/verify.el's known answers (transpose,
slice-cols, set-cols) and against independent numpy transcriptions of the
reference formulas (lisp/nelisp-gpu-kernels.el, cited per operator)."""
import numpy as np
import pytest

import oracle as nlo

f32 = np.float32


def test_glue_ops_verify_el():
    # test/verify.el: transpose (5x7) of A[i] = i; slice-cols / set-cols (4x8), cols [2,5)
    R, Co = 5, 7
    A = np.arange(R * Co, dtype=f32)
    C = np.zeros(R * Co, f32)
    nlo.call("transpose", A, C, R, Co)
    assert np.array_equal(C, A.reshape(R, Co).T.ravel())
    seq, dim, hd, c0 = 4, 8, 3, 2
    A = np.arange(seq * dim, dtype=f32)
    C = np.zeros(seq * hd, f32)
    nlo.call("slice_cols", A, C, seq, dim, hd, c0)
    assert np.array_equal(C, A.reshape(seq, dim)[:, c0:c0 + hd].ravel())
    D = (10 * np.arange(seq * dim)).astype(f32)
    Sx = (-np.arange(seq * hd)).astype(f32)
    ref = D.reshape(seq, dim).copy()
    ref[:, c0:c0 + hd] = Sx.reshape(seq, hd)
    nlo.call("set_cols", D, Sx, seq, dim, hd, c0)
    assert np.array_equal(D, ref.ravel())


def _silu(x):
    return x / (1 + np.exp(-x))


def _gelu_tanh(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def test_elementwise_gradients_are_derivatives():
    rng = np.random.default_rng(1)
    n = 500
    x = rng.standard_normal(n).astype(f32) * 3
    b = rng.standard_normal(n).astype(f32)
    g = rng.standard_normal(n).astype(f32)
    x64, eps = x.astype(np.float64), 1e-4
    # :1314-1320 silu-bwd = g * silu'(x); :195-204 silu-mul-bwd
    D = np.zeros(n, f32)
    nlo.call("silu_bwd", g, x, D, n)
    num = (_silu(x64 + eps) - _silu(x64 - eps)) / (2 * eps)
    assert np.max(np.abs(D - g * num)) < 1e-4
    DA, DB = np.zeros(n, f32), np.zeros(n, f32)
    nlo.call("silu_mul_bwd", g, x, b, DA, DB, n)
    assert np.max(np.abs(DA - g * b * num)) < 1e-4
    assert np.max(np.abs(DB - g * _silu(x64))) < 1e-4
    # :473-485 gelu-bwd (tanh form)
    nlo.call("gelu_bwd", g, x, D, n)
    num = (_gelu_tanh(x64 + eps) - _gelu_tanh(x64 - eps)) / (2 * eps)
    assert np.max(np.abs(D - g * num)) < 2e-4


def test_optimizers():
    rng = np.random.default_rng(2)
    n = 300
    W0 = rng.standard_normal(n).astype(f32)
    G = rng.standard_normal(n).astype(f32)
    # :488-493 sgd
    W = W0.copy()
    nlo.call("sgd", W, G, np.array([0.1], f32), np.array([0.5], f32), n)
    assert np.array_equal(W, W0 - f32(f32(0.1) * f32(0.5)) * G)
    # :1338-1351 adam
    W, M, V = W0.copy(), np.zeros(n, f32), np.zeros(n, f32)
    H = np.array([1e-3, 0.9, 0.999, 1e-8], f32)
    nlo.call("adam", W, G, M, V, H, np.array([1.0], f32), n)
    m = (1 - np.float64(f32(0.9))) * G.astype(np.float64)      # b1, b2 as the f32 values
    v = (1 - np.float64(f32(0.999))) * G.astype(np.float64) ** 2
    assert np.allclose(M, m, rtol=1e-6) and np.allclose(V, v, rtol=1e-5)
    assert np.allclose(W, W0 - 1e-3 * m / (np.sqrt(v) + 1e-8), rtol=1e-5, atol=1e-7)
    # :455-460 sub-scale
    C = np.zeros(n, f32)
    nlo.call("sub_scale", W0, G, np.array([0.25], f32), C, n)
    assert np.array_equal(C, (W0 - G) * f32(0.25))


def test_reductions():
    rng = np.random.default_rng(3)
    M, N = 7, 33
    DY, X, G = (rng.standard_normal((M, N)).astype(f32) for _ in range(3))
    S = rng.random(M).astype(f32) + 0.5
    gam = rng.random(N).astype(f32) + 0.5
    D = np.zeros(N, f32)
    nlo.call("colsum", G.ravel(), D, M, N)
    assert np.allclose(D, G.sum(0), atol=1e-5)
    nlo.call("rmsnorm_dgamma", DY.ravel(), X.ravel(), S, D, M, N)
    assert np.allclose(D, (DY * X * S[:, None]).sum(0), atol=1e-5)
    # :1267-1278 rmsnorm-dx, the gradient of x * s(x) * g with s = 1/rms
    DX = np.zeros(M * N, f32)
    nlo.call("rmsnorm_dx", DY.ravel(), X.ravel(), S, gam, DX, M, N)
    a = (DY * gam * X).sum(1, keepdims=True)
    want = S[:, None] * DY * gam - (S[:, None] ** 3) * X * a / N
    assert np.allclose(DX.reshape(M, N), want, atol=1e-5)
    # :1327-1335 softmax-bwd, :1373-1381 rowdot
    P = np.exp(X) / np.exp(X).sum(1, keepdims=True)
    P = P.astype(f32)
    DS = np.zeros(M * N, f32)
    nlo.call("softmax_bwd", P.ravel(), G.ravel(), DS, M, N)
    assert np.allclose(DS.reshape(M, N), P * (G - (P * G).sum(1, keepdims=True)), atol=1e-6)
    Dr = np.zeros(M, f32)
    nlo.call("rowdot", G.ravel(), DY.ravel(), Dr, M, N)
    assert np.allclose(Dr, (G * DY).sum(1), atol=1e-5)
    # :1407-1439 ce-grad(-idx): (softmax - target) / M
    LG = X
    tg = rng.integers(0, N, M)
    oh = np.zeros((M, N), f32)
    oh[np.arange(M), tg] = 1
    sm = np.exp(LG - LG.max(1, keepdims=True))
    sm /= sm.sum(1, keepdims=True)
    for idx, T in ((1, tg.astype(f32)), (0, oh.ravel())):
        Gr = np.zeros(M * N, f32)
        nlo.call("ce_grad", LG.ravel(), T, Gr, M, N, idx)
        assert np.allclose(Gr.reshape(M, N), (sm - oh) / M, atol=1e-7)


def test_topk_embed_spikes_gdn():
    rng = np.random.default_rng(4)
    M, E, K = 5, 9, 3
    LG = rng.standard_normal((M, E)).astype(f32)
    MK = np.zeros(M * E, f32)
    nlo.call("topk_mask", LG.ravel(), MK, M, E, K)
    top = np.argsort(-LG, 1)[:, :K]
    want = np.full((M, E), -1e30, f32)
    want[np.arange(M)[:, None], top] = 0
    assert np.array_equal(MK.reshape(M, E), want)
    # :1395-1405 embed-bwd
    seq, dim, vocab = 6, 4, 5
    tok = rng.integers(0, vocab, seq)
    GX = rng.standard_normal((seq, dim)).astype(f32)
    DW = np.zeros(vocab * dim, f32)
    nlo.call("embed_bwd", tok.astype(f32), GX.ravel(), DW, seq, dim, vocab)
    want = np.zeros((vocab, dim))
    np.add.at(want, tok, GX)
    assert np.allclose(DW.reshape(vocab, dim), want, atol=1e-6)
    # :569-585 gather / scatter through a table
    n, bs = 3, 4
    table = np.array([2, 0, 1], f32)
    pool = np.arange(12, dtype=f32)
    out = np.zeros(12, f32)
    nlo.call("gather_spike", table, pool, out, n, bs, 12)
    assert np.array_equal(out, np.concatenate([pool[8:12], pool[0:4], pool[4:8]]))
    pool2 = np.zeros(12, f32)
    nlo.call("scatter_spike", table, out, pool2, n, bs, 12)
    assert np.array_equal(pool2, pool)
    # :673-698 gdn-step: S <- g S; S <- S + k (b (v - k.S)); o = q.S
    nv, dk, dv, t = 2, 3, 4, 1
    S0 = rng.standard_normal((nv, dk, dv)).astype(f32)
    Q, Kk = (rng.standard_normal((t + 1, nv, dk)).astype(f32) for _ in range(2))
    V = rng.standard_normal((t + 1, nv, dv)).astype(f32)
    Gg, Bb = (rng.random((t + 1, nv)).astype(f32) for _ in range(2))
    S = S0.copy().ravel()
    OUT = np.zeros((t + 1) * nv * dv, f32)
    nlo.call("gdn_step", S, Q.ravel(), Kk.ravel(), V.ravel(), Gg.ravel(), Bb.ravel(), OUT, nv, dk,
             dv, t)
    for h in range(nv):
        s = S0[h].astype(np.float64) * Gg[t, h]
        k = Kk[t, h].astype(np.float64)
        d = Bb[t, h] * (V[t, h] - k @ s)
        s = s + np.outer(k, d)
        assert np.allclose(S.reshape(nv, dk, dv)[h], s, atol=1e-5)
        assert np.allclose(OUT.reshape(t + 1, nv, dv)[t, h], Q[t, h] @ s, atol=1e-5)


@pytest.mark.parametrize("heads,kvheads", [(4, 4), (4, 2)])
def test_attention_backward(heads, kvheads):
    rng = np.random.default_rng(heads + kvheads)
    seq, hd = 6, 8
    dim, kvdim, grp = heads * hd, kvheads * hd, heads // kvheads
    DS, P = (rng.standard_normal((heads, seq, seq)).astype(f32) for _ in range(2))
    Q, DC = (rng.standard_normal((seq, dim)).astype(f32) for _ in range(2))
    Kk, V = (rng.standard_normal((seq, kvdim)).astype(f32) for _ in range(2))
    DQ, DK = np.zeros(seq * dim, f32), np.zeros(seq * kvdim, f32)
    DP, DV = np.zeros(heads * seq * seq, f32), np.zeros(seq * kvdim, f32)
    nlo.call("attn_sc_dq", DS.ravel(), Kk.ravel(), DQ, seq, dim, heads, kvheads)
    nlo.call("attn_sc_dk", DS.ravel(), Q.ravel(), DK, seq, dim, heads, kvheads)
    nlo.call("attn_ctx_dp", DC.ravel(), V.ravel(), DP, seq, dim, heads, kvheads)
    nlo.call("attn_ctx_dv", DC.ravel(), P.ravel(), DV, seq, dim, heads, kvheads)
    sc = 1 / np.sqrt(hd)
    wdk = np.zeros((seq, kvdim))
    wdv = np.zeros((seq, kvdim))
    for h in range(heads):
        kv = h // grp
        ks, qs = slice(kv * hd, (kv + 1) * hd), slice(h * hd, (h + 1) * hd)
        assert np.allclose(DQ.reshape(seq, dim)[:, qs], sc * DS[h] @ Kk[:, ks], atol=1e-5)
        assert np.allclose(DP.reshape(heads, seq, seq)[h], DC[:, qs] @ V[:, ks].T, atol=1e-5)
        wdk[:, ks] += sc * DS[h].T @ Q[:, qs]
        wdv[:, ks] += P[h].T @ DC[:, qs]
    assert np.allclose(DK.reshape(seq, kvdim), wdk, atol=1e-5)
    assert np.allclose(DV.reshape(seq, kvdim), wdv, atol=1e-5)


def test_tree_attention():
    # :1144-1180: row i attends to the L cached keys and to its tree ancestors
    rng = np.random.default_rng(9)
    M, heads, hd, L, depth = 5, 2, 4, 3, 3
    dim = heads * hd
    Q, NK, NV = (rng.standard_normal((M, dim)).astype(f32) for _ in range(3))
    CK, CV = (rng.standard_normal((L, dim)).astype(f32) for _ in range(2))
    par = np.array([99, 0, 0, 1, 3], f32)          # a parent >= M ends the walk
    C = np.zeros(M * dim, f32)
    nlo.call("tree_attn", Q.ravel(), CK.ravel(), CV.ravel(), NK.ravel(), NV.ravel(), par,
             np.array([L], f32), C, M, dim, heads, heads, depth)
    for i in range(M):
        anc, cur = [], i
        for _ in range(depth):
            if cur >= M:
                break
            anc.append(cur)
            cur = int(par[cur])
        for h in range(heads):
            sl = slice(h * hd, (h + 1) * hd)
            keys = np.concatenate([CK[:, sl], NK[anc, sl]])
            vals = np.concatenate([CV[:, sl], NV[anc, sl]])
            s = keys @ Q[i, sl] / np.sqrt(hd)
            p = np.exp(s - s.max())
            assert np.allclose(C.reshape(M, dim)[i, sl], p @ vals / p.sum(), atol=1e-5)
