"""The reference's training-side operators on the GPU against the oracle
(oracle/nl_oracle_misc.c): glue copies, gradients, optimizers, the MoE top-k
mask, embedding backward, the paged gather / scatter spikes, the gated
delta-net step, tree attention and the attention backward products
(lisp/nelisp-gpu-kernels.el).  Copies and the products without a
transcendental are bit-exact where the order of the reference is kept;
expf-bearing and reordered sums are within 1e-5 (tk-err)."""
import numpy as np
import pytest

import oracle as nlo

pytestmark = pytest.mark.gpu
f32 = np.float32


@pytest.fixture(scope="module")
def host():
    from nelisp_cuda.host import Host
    return Host()


def g64(n):
    return max(1, (n + 63) // 64)


def rnd(rng, *shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(f32)


def test_glue(host):
    rng = np.random.default_rng(1)
    R, Co = 37, 53
    A = rnd(rng, R * Co)
    C = np.zeros(R * Co, f32)
    nlo.call("transpose", A, C, R, Co)
    got = host.run2("transpose", [("in", A), ("out", R * Co)], [R, Co], g64(R * Co))[0]
    assert np.array_equal(got, C)
    seq, dim, hd, c0 = 9, 40, 13, 21
    A = rnd(rng, seq * dim)
    C = np.zeros(seq * hd, f32)
    nlo.call("slice_cols", A, C, seq, dim, hd, c0)
    got = host.run2("slice-cols", [("in", A), ("out", seq * hd)], [seq, dim, hd, c0],
                    g64(seq * hd))[0]
    assert np.array_equal(got, C)
    D = rnd(rng, seq * dim)
    want = D.copy()
    nlo.call("set_cols", want, C, seq, dim, hd, c0)
    got = host.run2("set-cols", [("inout", D), ("in", C)], [seq, dim, hd, c0], g64(seq * hd))[0]
    assert np.array_equal(got, want)


def test_elementwise(host):
    rng = np.random.default_rng(2)
    n = 20000
    G, A, B = rnd(rng, n), rnd(rng, n, scale=3), rnd(rng, n)
    DA, DB, D = np.zeros(n, f32), np.zeros(n, f32), np.zeros(n, f32)
    nlo.call("silu_mul_bwd", G, A, B, DA, DB, n)
    got = host.run2("silu-mul-bwd", [("in", G), ("in", A), ("in", B), ("out", n), ("out", n)], [n],
                    g64(n))
    assert nlo.tk_err(got[0], DA) < 1e-6 and nlo.tk_err(got[1], DB) < 1e-6
    for name in ("silu_bwd", "gelu_bwd"):
        nlo.call(name, G, A, D, n)
        got = host.run2(name.replace("_", "-"), [("in", G), ("in", A), ("out", n)], [n], g64(n))[0]
        # the reference's gelu-bwd gives (inf - 1) / (inf + 1) = NaN once exp
        # overflows (|x| above ~9): the same positions must be NaN here
        nan = np.isnan(D)
        assert np.array_equal(np.isnan(got), nan), name
        assert nlo.tk_err(got[~nan], D[~nan]) < 1e-5, name   # expf differs from glibc
    S = np.array([0.37], f32)
    nlo.call("sub_scale", A, B, S, D, n)
    got = host.run2("sub-scale", [("in", A), ("in", B), ("in", S), ("out", n)], [n], g64(n))[0]
    assert np.array_equal(got, D)


def test_optimizers(host):
    rng = np.random.default_rng(3)
    n = 10000
    W, G = rnd(rng, n), rnd(rng, n)
    L, S = np.array([0.05], f32), np.array([0.8], f32)
    want = W.copy()
    nlo.call("sgd", want, G, L, S, n)
    got = host.run2("sgd", [("inout", W), ("in", G), ("in", L), ("in", S)], [n], g64(n))[0]
    assert np.array_equal(got, want)
    M, V = rnd(rng, n, scale=0.1), np.abs(rnd(rng, n, scale=0.1))
    H = np.array([1e-3, 0.9, 0.999, 1e-8], f32)
    wW, wM, wV = W.copy(), M.copy(), V.copy()
    nlo.call("adam", wW, G, wM, wV, H, S, n)
    got = host.run2("adam", [("inout", W), ("in", G), ("inout", M), ("inout", V), ("in", H),
                             ("in", S)], [n], g64(n))
    assert np.array_equal(got[1], wM) and np.array_equal(got[2], wV)
    assert np.max(np.abs(got[0] - wW)) <= 1e-6      # sqrtf and division: correctly rounded both


def test_reductions(host):
    rng = np.random.default_rng(4)
    M, N = 97, 515
    DY, X, G = rnd(rng, M * N), rnd(rng, M * N), rnd(rng, M * N)
    S = (rng.random(M) + 0.5).astype(f32)
    gam = (rng.random(N) + 0.5).astype(f32)
    D = np.zeros(N, f32)
    nlo.call("colsum", G, D, M, N)
    got = host.run2("colsum", [("in", G), ("out", N)], [M, N], g64(N))[0]
    assert np.array_equal(got, D)
    nlo.call("rmsnorm_dgamma", DY, X, S, D, M, N)
    got = host.run2("rmsnorm-dgamma", [("in", DY), ("in", X), ("in", S), ("out", N)], [M, N],
                    g64(N))[0]
    assert np.array_equal(got, D)
    DX = np.zeros(M * N, f32)
    nlo.call("rmsnorm_dx", DY, X, S, gam, DX, M, N)
    got = host.run2("rmsnorm-dx", [("in", DY), ("in", X), ("in", S), ("in", gam), ("out", M * N)],
                    [M, N], g64(M))[0]
    assert nlo.tk_err(got, DX) < 1e-5
    P = (rng.random(M * N)).astype(f32)
    DS = np.zeros(M * N, f32)
    nlo.call("softmax_bwd", P, G, DS, M, N)
    got = host.run2("softmax-bwd", [("in", P), ("in", G), ("out", M * N)], [M, N], g64(M))[0]
    assert nlo.tk_err(got, DS) < 1e-5
    Dr = np.zeros(M, f32)
    nlo.call("rowdot", G, DY, Dr, M, N)
    got = host.run2("rowdot", [("in", G), ("in", DY), ("out", M)], [M, N], g64(M))[0]
    assert nlo.tk_err(got, Dr) < 1e-5
    LG = rnd(rng, M * N, scale=2)
    tg = rng.integers(0, N, M).astype(f32)
    oh = np.zeros((M, N), f32)
    oh[np.arange(M), tg.astype(int)] = 1
    for name, idx, T in (("ce-grad-idx", 1, tg), ("ce-grad", 0, oh.ravel())):
        want = np.zeros(M * N, f32)
        nlo.call("ce_grad", LG, T, want, M, N, idx)
        got = host.run2(name, [("in", LG), ("in", T), ("out", M * N)], [M, N], g64(M))[0]
        assert nlo.tk_err(got, want) < 1e-5, name


def test_topk_embed_spikes(host):
    rng = np.random.default_rng(5)
    M, E, K = 64, 16, 4
    LG = rnd(rng, M * E)
    want = np.zeros(M * E, f32)
    nlo.call("topk_mask", LG, want, M, E, K)
    got = host.run2("topk-mask", [("in", LG), ("out", M * E)], [M, E, K], g64(M * E))[0]
    assert np.array_equal(got, want)
    seq, dim, vocab = 50, 64, 40
    tok = rng.integers(0, vocab, seq).astype(f32)
    GX = rnd(rng, seq * dim)
    want = np.zeros(vocab * dim, f32)
    nlo.call("embed_bwd", tok, GX, want, seq, dim, vocab)
    got = host.run2("embed-bwd", [("in", tok), ("in", GX), ("out", vocab * dim)], [seq, dim, vocab],
                    g64(vocab * dim))[0]
    assert np.array_equal(got, want)
    n, bs, nblocks = 6, 32, 10
    table = np.array([3, 9, 0, 1, 500, 7], f32)          # 500: past the pool, skipped
    pool = rnd(rng, nblocks * bs)
    out = np.zeros(n * bs, f32)
    nlo.call("gather_spike", table, pool, out, n, bs, nblocks * bs)
    got = host.run2("gather-spike", [("in", table), ("in", pool), ("out", n * bs)], [n, bs],
                    g64(n * bs))[0]
    assert np.array_equal(got, out)
    src = rnd(rng, n * bs)
    want = pool.copy()
    nlo.call("scatter_spike", table, src, want, n, bs, nblocks * bs)
    got = host.run2("scatter-spike", [("in", table), ("in", src), ("inout", pool)], [n, bs],
                    g64(n * bs))[0]
    assert np.array_equal(got, want)


def test_gdn_step(host):
    rng = np.random.default_rng(6)
    nv, dk, dv, t = 4, 32, 48, 2
    S = rnd(rng, nv * dk * dv, scale=0.1)
    Q, K = rnd(rng, (t + 1) * nv * dk), rnd(rng, (t + 1) * nv * dk)
    V = rnd(rng, (t + 1) * nv * dv)
    G, B = (rng.random((t + 1) * nv).astype(f32) for _ in range(2))
    wS, wO = S.copy(), np.zeros((t + 1) * nv * dv, f32)
    nlo.call("gdn_step", wS, Q, K, V, G, B, wO, nv, dk, dv, t)
    got = host.run2("gdn-step", [("inout", S), ("in", Q), ("in", K), ("in", V), ("in", G),
                                 ("in", B), ("out", (t + 1) * nv * dv)], [nv, dk, dv, t],
                    g64(nv * dv))
    assert np.array_equal(got[0], wS)
    assert np.array_equal(got[1], wO)


@pytest.mark.parametrize("seq,heads,kvheads,hd", [(9, 4, 2, 8), (70, 8, 2, 64)])
def test_attention_backward(host, seq, heads, kvheads, hd):
    rng = np.random.default_rng(seq + hd)
    dim, kvdim = heads * hd, kvheads * hd
    DS, P = rnd(rng, heads * seq * seq), rnd(rng, heads * seq * seq)
    Q, DC = rnd(rng, seq * dim), rnd(rng, seq * dim)
    K, V = rnd(rng, seq * kvdim), rnd(rng, seq * kvdim)
    push = [seq, dim, heads, kvheads]
    cases = [("attn-sc-dq", "attn_sc_dq", DS, K, seq * dim, False),
             ("attn-sc-dk", "attn_sc_dk", DS, Q, seq * kvdim, True),
             ("attn-ctx-dp", "attn_ctx_dp", DC, V, heads * seq * seq, False),
             ("attn-ctx-dv", "attn_ctx_dv", DC, P, seq * kvdim, True)]
    for name, oname, a, b, n, exact in cases:
        want = np.zeros(n, f32)
        nlo.call(oname, a, b, want, *push)
        got = host.run2(name, [("in", a), ("in", b), ("out", n)], push, g64(n))[0]
        if exact:
            assert np.array_equal(got, want), name
        else:
            assert nlo.tk_err(got, want) < 1e-5, name


def test_tree_attention(host):
    rng = np.random.default_rng(7)
    M, heads, kvheads, hd, L, depth = 12, 4, 2, 32, 20, 4
    dim, kvdim = heads * hd, kvheads * hd
    Q, NK, NV = rnd(rng, M * dim), rnd(rng, M * kvdim), rnd(rng, M * kvdim)
    CK, CV = rnd(rng, L * kvdim), rnd(rng, L * kvdim)
    par = np.array([99, 0, 0, 1, 3, 4, 2, 6, 7, 5, 9, 10], f32)
    want = np.zeros(M * dim, f32)
    args = [Q, CK, CV, NK, NV, par, np.array([L], f32)]
    nlo.call("tree_attn", *args, want, M, dim, heads, kvheads, depth)
    got = host.run2("tree-attn", [("in", x) for x in args] + [("out", M * dim)],
                    [M, dim, heads, kvheads, depth], g64(M * dim))[0]
    assert nlo.tk_err(got, want) < 1e-5
