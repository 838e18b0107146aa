"""Pin the CPU oracle against the reference's own tests and known answers.

The oracle (oracle/nl_oracle.c) is the checker for every CUDA parity test, so
it is checked first, on the CPU, against what the reference's tests assert:

* test/ternary-kernel-test.el -- the seed-20260921 fixture at tk-err < 1e-5
  against the double-precision `tk-cpu-forward', the transpose, the adjoint
  identity <W.x, g> = <x, W'.g>, and both negative controls (non-zero output;
  tripling one block scale moves exactly that row);
* host/vkmatmul.c -- A[i]=i%4, B[i]=i%3 with EXACT equality on a 7x7 sample;
* host/vksoftmax.c -- A[i]=(i%7)*0.3f within 1e-3 of a double softmax, row
  sum 1;
* test/verify.el -- matmul, softmax, linear, matmul-tiled, matmul-reg and
  scale on its modular generators within verify.el's tolerances.
"""
import numpy as np
import pytest

import oracle as nlo

pytestmark = pytest.mark.filterwarnings("ignore")


def _unpack_dsl(wp, out, cols, wng):
    """The DSL's unpack, (int(w << (30-2f)) >> 30), in numpy."""
    w = np.asarray(wp, np.uint32).reshape(out, wng)
    t = np.zeros((out, wng * 16), np.int32)
    for f in range(16):
        t[:, f::16] = ((w << np.uint32(30 - 2 * f)).astype(np.uint32)
                       .view(np.int32) >> 30)
    return t[:, :cols]


def test_tk_pack_layout_roundtrips(tk_fixture):
    d = tk_fixture
    t = _unpack_dsl(d["wp"], int(d["out"]), int(d["cols"]), int(d["wng"]))
    assert np.array_equal(t.ravel(), d["trits"].astype(np.int32))


def test_code_10_decodes_to_minus_two():
    # kernels.el:736-743: the arithmetic shift sign-extends, so 10 -> -2.
    w = np.array([0b10 | (0b01 << 2) | (0b11 << 4)], np.uint32)
    t = _unpack_dsl(w, 1, 16, 1)[0, :3]
    assert list(t) == [-2, 1, -1]
    y = nlo.ternary_rows(np.r_[np.ones(3), np.zeros(13)], w, [0.0], [1.0],
                         1, 1, 16, 1, 1)
    assert y[0] == -2.0 + 1.0 - 1.0


def _tk_run(d, beta=None, bias=None):
    seq, out, cols, nblk, wng = (int(d[k]) for k in ("seq", "out", "cols", "nblk", "wng"))
    b = d["beta"] if beta is None else beta
    bi = d["bias"] if bias is None else bias
    return nlo.ternary_rows(d["x"], d["wp"], bi, b, seq, out, cols, nblk, wng)


def test_tk_forward_matches_double_reference(tk_fixture):
    y = _tk_run(tk_fixture)
    assert nlo.tk_err(y, tk_fixture["y_want"]) < 1e-5
    assert np.any(y != 0.0)                     # control: not all zero


def test_tk_transpose_and_adjoint(tk_fixture):
    d = tk_fixture
    seq, out, cols, nblk, wng = (int(d[k]) for k in ("seq", "out", "cols", "nblk", "wng"))
    xt = nlo.ternary_rows_t(d["wp"], d["beta"], d["g"], out, cols, nblk, wng, seq)
    assert nlo.tk_err(xt, d["xt_want"]) < 1e-5
    y = _tk_run(d, bias=np.zeros(out))
    l = float(np.dot(y.astype(np.float64), d["g"]))
    r = float(np.dot(d["x"], xt.astype(np.float64)))
    assert abs(l - r) / max(1e-6, abs(l)) < 1e-5


def test_tk_block_scale_control(tk_fixture):
    d = tk_fixture
    seq, out = int(d["seq"]), int(d["out"])
    b2 = d["beta"].copy()
    b2[1] *= 3.0                                 # row 0, second block only
    y0, y1 = _tk_run(d), _tk_run(d, beta=b2)
    moved = sum(y0[s * out] != y1[s * out] for s in range(seq))
    spilled = sum(y0[s * out + o] != y1[s * out + o]
                  for s in range(seq) for o in range(1, out))
    assert moved == seq and spilled == 0


@pytest.mark.parametrize("mkn", [(128, 128, 128), (256, 256, 256), (64, 48, 80)])
def test_vkmatmul_exact_sample(mkn):
    M, K, N = mkn
    A = (np.arange(M * K) % 4).astype(np.float32)
    B = (np.arange(K * N) % 3).astype(np.float32)
    C = nlo.matmul(A, B, M, K, N)
    rs = range(0, M, max(M // 7, 1))
    cs = range(0, N, max(N // 7, 1))
    for r in rs:
        for c in cs:
            assert float(C[r * N + c]) == nlo.matmul_sample_ref(r, c, K, N)


def test_vksoftmax_check():
    M, N = 64, 256
    i = np.arange(M * N)
    A = (i % 7).astype(np.float32) * np.float32(0.3)
    C = nlo.softmax(A, M, N)
    ref = nlo.softmax_ref_f64((i % 7) * 0.3, M, N)
    assert np.max(np.abs(C - ref)) <= 1e-3
    assert abs(float(np.sum(C[:N], dtype=np.float64)) - 1.0) < 1e-5


def test_verify_el_generators(verify_fixture):
    d = verify_fixture
    got = nlo.matmul(d["matmul_A"], d["matmul_B"], 32, 24, 16)
    assert np.max(np.abs(got - d["matmul_C"])) < 1e-3
    got = nlo.softmax(d["softmax_A"], 24, 40)
    assert np.max(np.abs(got - d["softmax_C"])) < 1e-4
    got = nlo.linear(d["linear_X"], d["linear_W"], d["linear_B"], 20, 12, 16)
    assert np.max(np.abs(got - d["linear_C"])) < 1e-3
    got = nlo.matmul_tiled(d["tiled_A"], d["tiled_B"], 20, 24, 12)
    assert np.max(np.abs(got - d["tiled_C"])) < 1e-3
    got = nlo.matmul_reg(d["tiled_A"], d["tiled_B"], 20, 24, 12)
    assert np.max(np.abs(got - d["tiled_C"])) < 1e-3
    got = nlo.scale(d["scale_A"], d["scale_k"], 50)
    assert np.max(np.abs(got - d["scale_C"])) < 1e-5


def test_pack_act_rows_known_answers():
    # gamma = amax/127; lanes are round-half-up magnitudes, two's complement.
    X = np.array([127.0, -63.5, 0.2, -0.7, 1.0], np.float32)
    XQ, G = nlo.pack_act_rows(X, 1, 5, 2)
    assert G[0] == np.float32(127.0) / np.float32(127.0)
    lanes = [(int(XQ[0]) >> (8 * k)) & 0xFF for k in range(4)] + [int(XQ[1]) & 0xFF]
    assert lanes == [127, (256 - 64) % 256, 0, (256 - 1) % 256, 1]
    assert (int(XQ[1]) >> 8) == 0                # lanes past cols are zero
    XQ0, G0 = nlo.pack_act_rows(np.zeros(8, np.float32), 1, 8, 2)
    assert G0[0] == 0.0 and not XQ0.any()        # gamma 0 gives zeros


def test_dp4a_rows_integer_sum_is_exact():
    rng = np.random.default_rng(7)
    seq, out, ng = 3, 5, 40
    a = rng.integers(-128, 128, size=(seq, ng * 4), dtype=np.int8)
    w = rng.integers(-1, 2, size=(out, ng * 4), dtype=np.int8)
    AP, WP = a.view(np.uint32).ravel(), w.view(np.uint32).ravel()
    ones = np.ones(out, np.float32)
    Y = nlo.dp4a_rows(AP, WP, np.zeros(out), ones, np.ones(seq), seq, out, ng, 1)
    want = (a.astype(np.int64) @ w.astype(np.int64).T).ravel()
    assert np.array_equal(Y.astype(np.int64), want)


def test_decode_attn_b_against_numpy():
    rng = np.random.default_rng(3)
    B, heads, kvheads, hd, maxseq, pos = 2, 4, 2, 16, 9, 6
    dim, kvdim = heads * hd, kvheads * hd
    Q = rng.standard_normal(B * dim).astype(np.float32)
    CK = rng.standard_normal(B * maxseq * kvdim).astype(np.float32)
    CV = rng.standard_normal(B * maxseq * kvdim).astype(np.float32)
    C = nlo.decode_attn_b(Q, CK, CV, [float(pos)], B, dim, heads, kvheads, maxseq)
    q = Q.reshape(B, heads, hd).astype(np.float64)
    k = CK.reshape(B, maxseq, kvheads, hd)[:, :pos + 1].astype(np.float64)
    v = CV.reshape(B, maxseq, kvheads, hd)[:, :pos + 1].astype(np.float64)
    grp = heads // kvheads
    want = np.zeros((B, heads, hd))
    for b in range(B):
        for h in range(heads):
            s = k[b, :, h // grp] @ q[b, h] / np.sqrt(hd)
            p = np.exp(s - s.max())
            want[b, h] = (p / p.sum()) @ v[b, :, h // grp]
    assert nlo.tk_err(C, want.ravel()) < 1e-5


def test_rope_half_against_numpy():
    rng = np.random.default_rng(5)
    seq, nh, hd = 5, 3, 8
    X = rng.standard_normal(seq * nh * hd).astype(np.float32)
    rbase = np.array([10000.0], np.float32).view(np.uint32)[0]
    one = np.array([1.0], np.float32).view(np.uint32)[0]
    Y = nlo.rope_half(X, seq, nh, hd, int(rbase), int(one)).reshape(seq, nh, hd)
    x = X.reshape(seq, nh, hd).astype(np.float64)
    half = hd // 2
    th = np.arange(seq)[:, None] / (10000.0 ** (2.0 * np.arange(half) / hd))[None]
    c, s = np.cos(th)[:, None], np.sin(th)[:, None]
    want = np.concatenate([x[..., :half] * c - x[..., half:] * s,
                           x[..., half:] * c + x[..., :half] * s], axis=-1)
    assert np.max(np.abs(Y - want)) < 1e-5


def test_oracle_attn_causal_gqa_follows_the_reference_loop():
    """nlo_attn_causal_gqa against a direct Python transcription of
    kernels.el:949-990 (three passes per (head, row), f32 arithmetic)."""
    rng = np.random.default_rng(11)
    seq, heads, kvh, hd = 6, 4, 2, 8
    Q = rng.standard_normal(seq * heads * hd).astype(np.float32)
    K = rng.standard_normal(seq * kvh * hd).astype(np.float32)
    V = rng.standard_normal(seq * kvh * hd).astype(np.float32)
    got = nlo.attn_causal_gqa(Q, K, V, seq, heads, kvh, hd)
    f = np.float32
    want = np.zeros(seq * heads * hd, np.float32)
    qdim, kvdim, grp, scale = heads * hd, kvh * hd, heads // kvh, f(1.0) / np.sqrt(f(hd))
    for idx in range(heads * seq):
        h, i = idx // seq, idx % seq
        qb, kc = i * qdim + h * hd, (h // grp) * hd

        def score(j):
            acc = f(0.0)
            for t in range(hd):
                acc = f(acc + f(Q[qb + t] * K[j * kvdim + kc + t]))
            return f(acc * scale)
        mx = f(-1.0e30)
        for j in range(i + 1):
            mx = max(mx, score(j))
        sm = f(0.0)
        for j in range(i + 1):
            sm = f(sm + f(np.exp(f(score(j) - mx))))
        for j in range(i + 1):
            pj = f(f(np.exp(f(score(j) - mx))) / sm)
            for t in range(hd):
                want[qb + t] = f(want[qb + t] + f(pj * V[j * kvdim + kc + t]))
    assert np.max(np.abs(got - want)) < 2e-6
