"""The remaining reference operators on the GPU against the oracle
(oracle/nl_oracle_misc.c): matmul-at, causal-mask, attn-scores, attn-context,
dp4a-dot, bitlinear-dp4a, dp4a-rows-t, rmsnorm-heads, rope-apply, silu and
scale-rows (lisp/nelisp-gpu-kernels.el).  Integer sums and the elementwise
copies are bit-exact; f32 sums whose order the GPU changes are within 1e-5
(tk-err), the bar of the reference's own matmul and attention checks being
1e-4 and 1e-3."""
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


def rand_words(rng, n):
    return rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)


def halves(w):
    return (w & 0xFFFF).astype(np.float32), (w >> 16).astype(np.float32)


@pytest.mark.parametrize("mkn", [(256, 256, 256), (13, 29, 7), (70, 300, 33), (1, 5, 1)])
def test_matmul_at(host, mkn):
    M, K, N = mkn
    rng = np.random.default_rng(M + K + N)
    A = rng.uniform(-1, 1, K * M).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    got = host.run2("matmul-at", [("in", A), ("in", B), ("out", M * N)], [M, K, N], g64(M * N))[0]
    assert nlo.tk_err(got, nlo.matmul_at(A, B, M, K, N)) < 1e-5


def test_causal_mask(host):
    for n in (6, 100):
        S = np.arange(1, n * n + 1, dtype=np.float32)
        got = host.run2("causal-mask", [("inout", S)], [n], g64(n * n))[0]
        assert np.array_equal(got, nlo.causal_mask(S, n))
    # short grid: invocations past groups*64 leave S untouched
    n = 20
    S = np.arange(n * n, dtype=np.float32)
    got = host.run2("causal-mask", [("inout", S)], [n], 2)[0]
    want = nlo.causal_mask(S, n)
    want[128:] = S[128:]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("seq,heads,kvheads,hd", [(9, 4, 2, 8), (64, 8, 8, 128),
                                                  (100, 6, 2, 64), (33, 4, 1, 40)])
def test_attn_scores_context(host, seq, heads, kvheads, hd):
    dim, kvdim = heads * hd, kvheads * hd
    rng = np.random.default_rng(seq + hd)
    Q = rng.standard_normal(seq * dim).astype(np.float32)
    K = rng.standard_normal(seq * kvdim).astype(np.float32)
    V = rng.standard_normal(seq * kvdim).astype(np.float32)
    push = [seq, dim, heads, kvheads]
    S = host.run2("attn-scores", [("in", Q), ("in", K), ("out", heads * seq * seq)], push,
                  g64(heads * seq * seq))[0]
    want = nlo.attn_scores(Q, K, *push)
    masked = want == np.float32(-1.0e30)
    assert np.array_equal(S[masked], want[masked])
    assert nlo.tk_err(S[~masked], want[~masked]) < 1e-5
    P = rng.random(heads * seq * seq).astype(np.float32)
    C = host.run2("attn-context", [("in", P), ("in", V), ("out", seq * dim)], push,
                  g64(seq * dim))[0]
    assert nlo.tk_err(C, nlo.attn_context(P, V, *push)) < 1e-5


def test_attn_scores_short_grid(host):
    seq, heads, hd = 40, 2, 16
    dim = heads * hd
    rng = np.random.default_rng(9)
    Q = rng.standard_normal(seq * dim).astype(np.float32)
    K = rng.standard_normal(seq * dim).astype(np.float32)
    S = host.run2("attn-scores", [("in", Q), ("in", K), ("out", heads * seq * seq)],
                  [seq, dim, heads, heads], 30)[0]
    want = nlo.attn_scores(Q, K, seq, dim, heads, heads)
    lim = 30 * 64
    assert np.all(S[lim:] == 0.0)
    assert nlo.tk_err(S[:lim], want[:lim]) < 1e-5


def test_dp4a_dot(host):
    rng = np.random.default_rng(1)
    n = 1000
    a, b = rand_words(rng, n), rand_words(rng, n)
    bufs = [("in", x) for x in (*halves(a), *halves(b))] + [("out", n)]
    got = host.run2("dp4a-dot", bufs, [n], g64(n))[0]
    assert np.array_equal(got, nlo.dp4a_dot(*halves(a), *halves(b), n))


@pytest.mark.parametrize("seq,out,ng", [(3, 5, 11), (16, 640, 64), (1, 2560, 640)])
def test_bitlinear_dp4a(host, seq, out, ng):
    rng = np.random.default_rng(seq * out)
    A, W = rand_words(rng, seq * ng), rand_words(rng, out * ng)
    bias = rng.standard_normal(out).astype(np.float32)
    beta = np.array([0.01], np.float32)
    gamma = rng.random(seq).astype(np.float32)
    ins = [*halves(A), *halves(W), bias, beta, gamma]
    got = host.run2("bitlinear-dp4a", [("in", x) for x in ins] + [("out", seq * out)],
                    [seq, out, ng], g64(seq * out))[0]
    assert np.array_equal(got, nlo.bitlinear_dp4a(*ins, seq, out, ng))


@pytest.mark.parametrize("out,cols,seq", [(9, 22, 3), (256, 512, 4), (2560, 128, 1)])
def test_dp4a_rows_t(host, out, cols, seq):
    rng = np.random.default_rng(out + cols)
    ng = (cols + 3) // 4
    WP = rand_words(rng, out * ng)
    beta = rng.random(out).astype(np.float32)
    G = rng.standard_normal(seq * out).astype(np.float32)
    got = host.run2("dp4a-rows-t", [("in", WP.view(np.float32)), ("in", beta), ("in", G),
                                    ("out", seq * cols)], [out, cols, ng, seq], g64(seq * cols))[0]
    assert np.array_equal(got, nlo.dp4a_rows_t(WP, beta, G, out, cols, ng, seq))


@pytest.mark.parametrize("seq,heads,hd", [(4, 3, 16), (7, 16, 128), (1, 8, 64)])
def test_rmsnorm_heads(host, seq, heads, hd):
    rng = np.random.default_rng(hd)
    X = rng.standard_normal(seq * heads * hd).astype(np.float32)
    G = rng.random(hd).astype(np.float32)
    n = seq * heads * hd
    got = host.run2("rmsnorm-heads", [("in", X), ("in", G), ("out", n)], [seq, heads, hd],
                    g64(seq * heads))[0]
    assert nlo.tk_err(got, nlo.rmsnorm_heads(X, G, seq, heads, hd)) < 1e-5


@pytest.mark.parametrize("sg", [1.0, -1.0])
def test_rope_apply(host, sg):
    seq, heads, hd = 33, 4, 64
    dim, half = heads * hd, hd // 2
    rng = np.random.default_rng(int(sg + 5))
    X = rng.standard_normal(seq * dim).astype(np.float32)
    ang = rng.uniform(0, 6.3, seq * half)
    co, si = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    got = host.run2("rope-apply", [("in", X), ("in", co), ("in", si), ("in", [sg]),
                                   ("out", seq * dim)], [seq, dim, heads], g64(seq * dim // 2))[0]
    assert np.max(np.abs(got - nlo.rope_apply(X, co, si, [sg], seq, dim, heads))) < 1e-5


def test_silu_scale_rows(host):
    rng = np.random.default_rng(8)
    n = 11008 * 3
    X = (rng.standard_normal(n) * 4).astype(np.float32)
    got = host.run2("silu", [("in", X), ("out", n)], [n], g64(n))[0]
    assert nlo.tk_err(got, nlo.silu(X, n)) < 1e-6
    M, N = 37, 300
    Y = rng.standard_normal(M * N).astype(np.float32)
    S = rng.standard_normal(M).astype(np.float32)
    got = host.run2("scale-rows", [("in", Y), ("in", S), ("out", M * N)], [M, N], g64(M * N))[0]
    assert np.array_equal(got, nlo.scale_rows(Y, S, M, N))
    # short grid: the tail stays zero
    got = host.run2("scale-rows", [("in", Y), ("in", S), ("out", M * N)], [M, N], 3)[0]
    assert np.array_equal(got[:192], nlo.scale_rows(Y, S, M, N)[:192]) and not got[192:].any()


def test_misc_rejects_bad_shapes(host):
    from nelisp_cuda import NlError
    with pytest.raises(NlError):     # dim not divisible by heads
        host.run2("attn-scores", [("in", np.zeros(10)), ("in", np.zeros(10)), ("out", 10)],
                  [1, 10, 3, 3], 1)
    with pytest.raises(NlError):     # odd head size
        host.run2("rope-apply", [("in", np.zeros(6)), ("in", np.zeros(3)), ("in", np.zeros(3)),
                                 ("in", [1.0]), ("out", 6)], [1, 6, 2], 1)
