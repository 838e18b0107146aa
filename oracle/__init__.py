"""CPU oracle for the nelisp-gpu hot path -- TEST INFRASTRUCTURE ONLY.

A numpy-facing ctypes binding of ``oracle/_build/libnl_oracle.so``, the C
restatement of the reference's DSL kernels (lisp/nelisp-gpu-kernels.el in
zawatton/nelisp-gpu, cited per function in nl_oracle.c).  It is the parity
checker for the CUDA path and the timed CPU baseline.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import
it; the product library never calls it.

Parity of this restatement is pinned by ``tests/test_oracle_golden.py``
against the reference's own test generators and known answers (the tk LCG
fixture of test/ternary-kernel-test.el, host/vkmatmul.c's exact integer
sums, host/vksoftmax.c's double softmax and test/verify.el's generators).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libnl_oracle.so")
_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_U = ctypes.POINTER(ctypes.c_uint32)
_D = ctypes.POINTER(ctypes.c_double)
_u32 = ctypes.c_uint32


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    sigs = {
        "nlo_ternary_rows": [_F, _U, _F, _F, _F] + [_u32] * 5,
        "nlo_ternary_rows_t": [_U, _F, _F, _F] + [_u32] * 5,
        "nlo_ternary_gemv_rows": [_F, _U, _F, _F] + [_u32] * 3,
        "nlo_bitlinear_packed": [_F, _F, _F, _F, _F] + [_u32] * 5 + [ctypes.c_int],
        "nlo_pack_act_rows": [_F, _U, _F] + [_u32] * 3,
        "nlo_dp4a_rows": [_U, _U, _F, _F, _F, _F] + [_u32] * 3 + [ctypes.c_int],
        "nlo_matmul": [_F, _F, _F] + [_u32] * 3,
        "nlo_matmul_tiled": [_F, _F, _F] + [_u32] * 3,
        "nlo_matmul_reg": [_F, _F, _F] + [_u32] * 3,
        "nlo_linear": [_F, _F, _F, _F] + [_u32] * 3,
        "nlo_softmax": [_F, _F] + [_u32] * 2,
        "nlo_silu_mul": [_F, _F, _F, _u32],
        "nlo_add2": [_F, _F, _F, _u32],
        "nlo_scale": [_F, _F, _F, _u32],
        "nlo_rmsnorm_istd": [_F, _F, _u32, _u32],
        "nlo_rmsnorm_fwd": [_F, _F, _F, _F, _u32, _u32],
        "nlo_rope_half": [_F, _F] + [_u32] * 5,
        "nlo_decode_rope_b": [_F] * 6 + [_u32] * 3,
        "nlo_cache_append_b": [_F, _F, _F] + [_u32] * 3,
        "nlo_decode_attn_b": [_F] * 5 + [_u32] * 5,
        "nlo_attn_causal_gqa": [_F] * 4 + [_u32] * 4,
        "nlo_cache_append_ring": [_F] * 3 + [_u32] * 3,
        "nlo_qkv_append": [_F] * 3 + [_u32] * 3,
        "nlo_cache_append_paged": [_F] * 5 + [_u32] * 4,
        "nlo_block_copy": [_F] + [_u32] * 4,
        "nlo_decode_rope_b_v": [_F] * 6 + [_u32] * 3,
        "nlo_decode_attn_stream": [_F] * 7 + [_u32] * 5,
        "nlo_attn_stream_entries": [_F] * 7 + [_u32] * 5,
        "nlo_decode_attn_paged": [_F] * 7 + [_u32] * 6,
        "nlo_embed_gather": [_F, _F, _F, _u32, _u32],
        "nlo_matmul_at": [_F, _F, _F] + [_u32] * 3,
        "nlo_causal_mask": [_F, _u32],
        "nlo_attn_scores": [_F] * 3 + [_u32] * 4,
        "nlo_attn_context": [_F] * 3 + [_u32] * 4,
        "nlo_dp4a_dot": [_F] * 5 + [_u32],
        "nlo_bitlinear_dp4a": [_F] * 8 + [_u32] * 3,
        "nlo_dp4a_rows_t": [_F] * 4 + [_u32] * 4,
        "nlo_rmsnorm_heads": [_F] * 3 + [_u32] * 3,
        "nlo_rope_apply": [_F] * 5 + [_u32] * 3,
        "nlo_silu": [_F, _F, _u32],
        "nlo_scale_rows": [_F] * 3 + [_u32] * 2,
        "nlo_sumsq_acc": [_F, _F, _u32],
        "nlo_absmean_acc": [_F, _F, _u32],
        "nlo_clip_scale": [_F, _F, _F],
        "nlo_quant_act": [_F, _F, _u32, _u32],
        "nlo_quant_w": [_F, _F, _F, _u32],
        "nlo_quant_w_pack": [_F, _u32, _u32, ctypes.c_int, _U, _F],
        "nlo_transpose": [_F, _F, _u32, _u32],
        "nlo_slice_cols": [_F, _F] + [_u32] * 4,
        "nlo_set_cols": [_F, _F] + [_u32] * 4,
        "nlo_silu_mul_bwd": [_F] * 5 + [_u32],
        "nlo_silu_bwd": [_F] * 3 + [_u32],
        "nlo_gelu_bwd": [_F] * 3 + [_u32],
        "nlo_sub_scale": [_F] * 4 + [_u32],
        "nlo_sgd": [_F] * 4 + [_u32],
        "nlo_adam": [_F] * 6 + [_u32],
        "nlo_colsum": [_F, _F, _u32, _u32],
        "nlo_rmsnorm_dgamma": [_F] * 4 + [_u32, _u32],
        "nlo_rmsnorm_dx": [_F] * 5 + [_u32, _u32],
        "nlo_softmax_bwd": [_F] * 3 + [_u32, _u32],
        "nlo_rowdot": [_F] * 3 + [_u32, _u32],
        "nlo_ce_grad": [_F] * 3 + [_u32, _u32, ctypes.c_int],
        "nlo_topk_mask": [_F, _F] + [_u32] * 3,
        "nlo_embed_bwd": [_F] * 3 + [_u32] * 3,
        "nlo_gather_spike": [_F] * 3 + [_u32, _u32, ctypes.c_uint64],
        "nlo_scatter_spike": [_F] * 3 + [_u32, _u32, ctypes.c_uint64],
        "nlo_gdn_step": [_F] * 7 + [_u32] * 4,
        "nlo_attn_sc_dq": [_F] * 3 + [_u32] * 4,
        "nlo_attn_sc_dk": [_F] * 3 + [_u32] * 4,
        "nlo_attn_ctx_dp": [_F] * 3 + [_u32] * 4,
        "nlo_attn_ctx_dv": [_F] * 3 + [_u32] * 4,
        "nlo_tree_attn": [_F] * 8 + [_u32] * 5,
        "nlo_matmul_sample_ref": [_u32] * 4,
        "nlo_softmax_ref_f64": [_D, _D, _u32, _u32],
        "nlo_set_threads": [ctypes.c_int],
        "nlo_decoder_generate": [ctypes.c_void_p, _u32, _u32, ctypes.POINTER(ctypes.c_int32), _u32,
                                 ctypes.POINTER(ctypes.c_int32), _F],
        "nlo_threads": [],
        "nlo_decoder_time_positions": [ctypes.c_void_p, _u32, _u32, _u32],
        "nlo_decoder_tensor": [ctypes.c_void_p, _u32, _u32, ctypes.c_void_p],
    }
    for name, argt in sigs.items():
        fn = getattr(L, name)
        fn.argtypes = argt
        fn.restype = None
    L.nlo_matmul_sample_ref.restype = ctypes.c_double
    L.nlo_threads.restype = ctypes.c_int
    L.nlo_decoder_generate.restype = ctypes.c_int
    L.nlo_decoder_time_positions.restype = ctypes.c_double
    L.nlo_decoder_tensor.restype = ctypes.c_uint64


def _f(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def _u(a):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_U)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def threads() -> int:
    return lib().nlo_threads()


def set_threads(n: int) -> None:
    lib().nlo_set_threads(int(n))


# ---- kernels -------------------------------------------------------------

def ternary_rows(X, WP, BIAS, BETA, seq, out, cols, nblk, wng):
    X, WP, BIAS, BETA = f32(X), u32(WP), f32(BIAS), f32(BETA)
    Y = np.zeros(seq * out, np.float32)
    lib().nlo_ternary_rows(_f(X), _u(WP), _f(BIAS), _f(BETA), _f(Y),
                           seq, out, cols, nblk, wng)
    return Y


def ternary_rows_t(WP, BETA, G, out, cols, nblk, wng, seq):
    WP, BETA, G = u32(WP), f32(BETA), f32(G)
    X = np.zeros(seq * cols, np.float32)
    lib().nlo_ternary_rows_t(_u(WP), _f(BETA), _f(G), _f(X),
                             out, cols, nblk, wng, seq)
    return X


def ternary_gemv_rows(X, WP, S, seq, out, cols):
    X, WP, S = f32(X), u32(WP), f32(S)
    Y = np.zeros(seq * out, np.float32)
    lib().nlo_ternary_gemv_rows(_f(X), _u(WP), _f(S), _f(Y), seq, out, cols)
    return Y


def bitlinear_packed(X, WPK, BIAS, BETA, seq, inn, out, pk, fcount, per_row):
    X, WPK, BIAS, BETA = f32(X), f32(WPK), f32(BIAS), f32(BETA)
    Y = np.zeros(seq * out, np.float32)
    lib().nlo_bitlinear_packed(_f(X), _f(WPK), _f(BIAS), _f(BETA), _f(Y),
                               seq, inn, out, pk, fcount, int(per_row))
    return Y


def pack_act_rows(X, seq, cols, ng):
    X = f32(X)
    XQ = np.zeros(seq * ng, np.uint32)
    G = np.zeros(seq, np.float32)
    lib().nlo_pack_act_rows(_f(X), _u(XQ), _f(G), seq, cols, ng)
    return XQ, G


def dp4a_rows(AP, WP, BIAS, BETA, GAMMA, seq, out, ng, per_row):
    AP, WP, BIAS, BETA, GAMMA = u32(AP), u32(WP), f32(BIAS), f32(BETA), f32(GAMMA)
    Y = np.zeros(seq * out, np.float32)
    lib().nlo_dp4a_rows(_u(AP), _u(WP), _f(BIAS), _f(BETA), _f(GAMMA), _f(Y),
                        seq, out, ng, int(per_row))
    return Y


def _mm(fn, A, B, M, K, N):
    A, B = f32(A), f32(B)
    C = np.zeros(M * N, np.float32)
    fn(_f(A), _f(B), _f(C), M, K, N)
    return C


def matmul(A, B, M, K, N):
    return _mm(lib().nlo_matmul, A, B, M, K, N)


def matmul_tiled(A, B, M, K, N):
    return _mm(lib().nlo_matmul_tiled, A, B, M, K, N)


def matmul_reg(A, B, M, K, N):
    return _mm(lib().nlo_matmul_reg, A, B, M, K, N)


def linear(X, W, B, M, IN, OUT):
    X, W, B = f32(X), f32(W), f32(B)
    C = np.zeros(M * OUT, np.float32)
    lib().nlo_linear(_f(X), _f(W), _f(B), _f(C), M, IN, OUT)
    return C


def softmax(A, M, N):
    A = f32(A)
    C = np.zeros(M * N, np.float32)
    lib().nlo_softmax(_f(A), _f(C), M, N)
    return C


def _ew(fn, A, B, n):
    A, B = f32(A), f32(B)
    C = np.zeros(n, np.float32)
    fn(_f(A), _f(B), _f(C), n)
    return C


def silu_mul(A, B, n):
    return _ew(lib().nlo_silu_mul, A, B, n)


def add2(A, B, n):
    return _ew(lib().nlo_add2, A, B, n)


def scale(A, S, n):
    return _ew(lib().nlo_scale, A, S, n)


def rmsnorm_istd(X, M, N):
    X = f32(X)
    S = np.zeros(M, np.float32)
    lib().nlo_rmsnorm_istd(_f(X), _f(S), M, N)
    return S


def rmsnorm_fwd(X, S, G, M, N):
    X, S, G = f32(X), f32(S), f32(G)
    C = np.zeros(M * N, np.float32)
    lib().nlo_rmsnorm_fwd(_f(X), _f(S), _f(G), _f(C), M, N)
    return C


def rope_half(X, seq, nheads, hd, rbase_bits, sgn_bits):
    X = f32(X)
    Y = np.zeros(seq * nheads * hd, np.float32)
    lib().nlo_rope_half(_f(X), _f(Y), seq, nheads, hd, rbase_bits, sgn_bits)
    return Y


def decode_rope_b(X, CO, SI, SG, POS, B, cols, heads):
    X, CO, SI, SG, POS = f32(X), f32(CO), f32(SI), f32(SG), f32(POS)
    C = np.zeros(B * cols, np.float32)
    lib().nlo_decode_rope_b(_f(X), _f(CO), _f(SI), _f(SG), _f(POS), _f(C),
                            B, cols, heads)
    return C


def cache_append_b(SRC, POS, CACHE, B, kvdim, maxseq):
    SRC, POS = f32(SRC), f32(POS)
    CACHE = f32(CACHE).copy()
    lib().nlo_cache_append_b(_f(SRC), _f(POS), _f(CACHE), B, kvdim, maxseq)
    return CACHE


def decode_attn_b(Q, CK, CV, POS, B, dim, heads, kvheads, maxseq):
    Q, CK, CV, POS = f32(Q), f32(CK), f32(CV), f32(POS)
    C = np.zeros(B * dim, np.float32)
    lib().nlo_decode_attn_b(_f(Q), _f(CK), _f(CV), _f(POS), _f(C),
                            B, dim, heads, kvheads, maxseq)
    return C


def attn_causal_gqa(Q, K, V, seq, heads, kvheads, hd):
    """attn-causal-gqa (lisp/nelisp-gpu-kernels.el:949-990): CTX [seq x heads*hd]."""
    Q, K, V = f32(Q), f32(K), f32(V)
    CTX = np.zeros(seq * heads * hd, np.float32)
    lib().nlo_attn_causal_gqa(_f(Q), _f(K), _f(V), _f(CTX), seq, heads, kvheads, hd)
    return CTX


def _fz(a):
    return _f(a) if a is not None else None


def cache_append_ring(SRC, POS, CACHE, kvdim, nsink, win):
    out = f32(CACHE).copy()
    lib().nlo_cache_append_ring(_f(f32(SRC)), _f(f32(POS)), _f(out), kvdim, nsink, win)
    return out


def qkv_append(QKV, CK, CV, dim, kvdim, wbase):
    ck, cv = f32(CK).copy(), f32(CV).copy()
    lib().nlo_qkv_append(_f(f32(QKV)), _f(ck), _f(cv), dim, kvdim, wbase)
    return ck, cv


def cache_append_paged(SRC, POS, LENS, TABLE, POOL, B, kvdim, bs, mbps):
    out = f32(POOL).copy()
    lib().nlo_cache_append_paged(_f(f32(SRC)), _fz(None if POS is None else f32(POS)),
                                 _fz(None if LENS is None else f32(LENS)), _f(f32(TABLE)),
                                 _f(out), B, kvdim, bs, mbps)
    return out


def block_copy(POOL, bs, kvdim, src, dst):
    out = f32(POOL).copy()
    lib().nlo_block_copy(_f(out), bs, kvdim, src, dst)
    return out


def decode_rope_b_v(X, CO, SI, SG, LENS, B, cols, heads):
    C = np.zeros(B * cols, np.float32)
    lib().nlo_decode_rope_b_v(_f(f32(X)), _f(f32(CO)), _f(f32(SI)), _f(f32(SG)), _f(f32(LENS)),
                              _f(C), B, cols, heads)
    return C


def decode_attn_stream(Q, CK, CV, POS, CO, SI, dim, heads, kvheads, nsink, win):
    C = np.zeros(dim, np.float32)
    lib().nlo_decode_attn_stream(_f(f32(Q)), _f(f32(CK)), _f(f32(CV)), _f(f32(POS)), _f(f32(CO)),
                                 _f(f32(SI)), _f(C), dim, heads, kvheads, nsink, win)
    return C


def attn_stream_entries(Q, CK, CV, ENT, CO, SI, dim, heads, kvheads, ne, qcrel):
    C = np.zeros(dim, np.float32)
    lib().nlo_attn_stream_entries(_f(f32(Q)), _f(f32(CK)), _f(f32(CV)), _f(f32(ENT)),
                                  _f(f32(CO)), _f(f32(SI)), _f(C), dim, heads, kvheads, ne, qcrel)
    return C


def decode_attn_paged(Q, CK, CV, POS, LENS, TABLE, B, dim, heads, kvheads, bs, mbps):
    C = np.zeros(B * dim, np.float32)
    lib().nlo_decode_attn_paged(_f(f32(Q)), _f(f32(CK)), _f(f32(CV)),
                                _fz(None if POS is None else f32(POS)),
                                _fz(None if LENS is None else f32(LENS)), _f(f32(TABLE)), _f(C),
                                B, dim, heads, kvheads, bs, mbps)
    return C


def embed_gather(TOK, WTE, seq, dim):
    TOK, WTE = f32(TOK), f32(WTE)
    C = np.zeros(seq * dim, np.float32)
    lib().nlo_embed_gather(_f(TOK), _f(WTE), _f(C), seq, dim)
    return C


def matmul_at(A, B, M, K, N):
    return _mm(lib().nlo_matmul_at, A, B, M, K, N)


def causal_mask(S, n):
    S = f32(S).copy()
    lib().nlo_causal_mask(_f(S), n)
    return S


def attn_scores(Q, K, seq, dim, heads, kvheads):
    Q, K = f32(Q), f32(K)
    S = np.zeros(heads * seq * seq, np.float32)
    lib().nlo_attn_scores(_f(Q), _f(K), _f(S), seq, dim, heads, kvheads)
    return S


def attn_context(P, V, seq, dim, heads, kvheads):
    P, V = f32(P), f32(V)
    C = np.zeros(seq * dim, np.float32)
    lib().nlo_attn_context(_f(P), _f(V), _f(C), seq, dim, heads, kvheads)
    return C


def dp4a_dot(ALO, AHI, BLO, BHI, n):
    a = [f32(x) for x in (ALO, AHI, BLO, BHI)]
    out = np.zeros(n, np.float32)
    lib().nlo_dp4a_dot(*[_f(x) for x in a], _f(out), n)
    return out


def bitlinear_dp4a(ALO, AHI, WLO, WHI, BIAS, BETA, GAMMA, seq, out, ng):
    a = [f32(x) for x in (ALO, AHI, WLO, WHI, BIAS, BETA, GAMMA)]
    Y = np.zeros(seq * out, np.float32)
    lib().nlo_bitlinear_dp4a(*[_f(x) for x in a], _f(Y), seq, out, ng)
    return Y


def dp4a_rows_t(WP, BETA, G, out, cols, ng, seq):
    """WP: the packed int8 words (uint32) or their f32 bit-casts."""
    WP = np.ascontiguousarray(WP)
    if WP.dtype != np.float32:
        WP = np.ascontiguousarray(WP, np.uint32).view(np.float32)
    BETA, G = f32(BETA), f32(G)
    X = np.zeros(seq * cols, np.float32)
    lib().nlo_dp4a_rows_t(_f(WP), _f(BETA), _f(G), _f(X), out, cols, ng, seq)
    return X


def rmsnorm_heads(X, G, seq, nheads, hd):
    X, G = f32(X), f32(G)
    Y = np.zeros(seq * nheads * hd, np.float32)
    lib().nlo_rmsnorm_heads(_f(X), _f(G), _f(Y), seq, nheads, hd)
    return Y


def rope_apply(X, CO, SI, SG, seq, dim, heads):
    X, CO, SI, SG = f32(X), f32(CO), f32(SI), f32(SG)
    C = np.zeros(seq * dim, np.float32)
    lib().nlo_rope_apply(_f(X), _f(CO), _f(SI), _f(SG), _f(C), seq, dim, heads)
    return C


def silu(X, n):
    X = f32(X)
    C = np.zeros(n, np.float32)
    lib().nlo_silu(_f(X), _f(C), n)
    return C


def scale_rows(Y, S, M, N):
    Y, S = f32(Y), f32(S)
    C = np.zeros(M * N, np.float32)
    lib().nlo_scale_rows(_f(Y), _f(S), _f(C), M, N)
    return C


def sumsq_acc(G, acc0, n):
    G, A = f32(G), np.array([acc0], np.float32)
    lib().nlo_sumsq_acc(_f(G), _f(A), n)
    return A[0]


def absmean_acc(G, acc0, n):
    G, A = f32(G), np.array([acc0], np.float32)
    lib().nlo_absmean_acc(_f(G), _f(A), n)
    return A[0]


def clip_scale(gsq, cfg):
    G, C, S = (np.array([v], np.float32) for v in (gsq, cfg, 0.0))
    lib().nlo_clip_scale(_f(G), _f(C), _f(S))
    return S[0]


def quant_act(X, seq, cols):
    X = f32(X)
    XQ = np.zeros(seq * cols, np.float32)
    lib().nlo_quant_act(_f(X), _f(XQ), seq, cols)
    return XQ


def quant_w(W, S0, n):
    W, S = f32(W), np.array([S0], np.float32)
    WQ = np.zeros(n, np.float32)
    lib().nlo_quant_w(_f(W), _f(S), _f(WQ), n)
    return WQ


def quant_w_pack(W, rows, cols, per_row):
    W = f32(W)
    wng = (cols + 15) // 16
    WP = np.zeros(rows * wng, np.uint32)
    S = np.zeros(rows, np.float32)
    lib().nlo_quant_w_pack(_f(W), rows, cols, int(per_row), _u(WP), _f(S))
    return WP, S


def call(name, *args):
    """Call oracle function nlo_NAME: float32 arrays go as pointers (modified
    in place where the function writes them), everything else as integers."""
    conv = []
    for a in args:
        if isinstance(a, np.ndarray):
            conv.append(_f(a))
        else:
            conv.append(int(a))
    getattr(lib(), "nlo_" + name)(*conv)


def matmul_sample_ref(r, c, K, N) -> float:
    return lib().nlo_matmul_sample_ref(r, c, K, N)


def softmax_ref_f64(A, M, N):
    A = np.ascontiguousarray(A, np.float64)
    C = np.zeros(M * N, np.float64)
    lib().nlo_softmax_ref_f64(A.ctypes.data_as(_D), C.ctypes.data_as(_D), M, N)
    return C


# ---- decoder --------------------------------------------------------------

class DecoderConfig(ctypes.Structure):
    """Field layout of nl_decoder_config (include/nelisp_cuda.h)."""
    _fields_ = [("hidden", _u32), ("layers", _u32), ("heads", _u32), ("kv_heads", _u32),
                ("head_dim", _u32), ("ffn", _u32), ("vocab", _u32), ("max_batch", _u32),
                ("max_seq", _u32), ("rms_eps", ctypes.c_float), ("rope_base", ctypes.c_float),
                ("seed", ctypes.c_uint64)]


def decoder_generate(cfg: dict, prompt, steps: int, keep_logits: bool = False):
    """Greedy generation by the CPU model (nl_oracle_decoder.c).  PROMPT is
    [batch x prompt_len] int; returns (tokens [batch x steps], logits
    [positions x batch x vocab] or None)."""
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    B, P = prompt.shape
    c = DecoderConfig(**cfg)
    out = np.zeros((B, steps), np.int32)
    npos = P + steps - 1
    lg = np.zeros((npos, B, cfg["vocab"]), np.float32) if keep_logits else None
    rc = lib().nlo_decoder_generate(ctypes.byref(c), B, P,
                                    prompt.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), steps,
                                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                    lg.ctypes.data_as(_F) if lg is not None else None)
    if rc != 0:
        raise RuntimeError(f"nlo_decoder_generate: {rc}")
    return out, lg


def decoder_time_positions(cfg: dict, batch: int, ctx: int, steps: int) -> float:
    """Seconds the CPU model takes for STEPS greedy decode positions at
    context CTX .. CTX+STEPS-1 (KV cache rows below CTX filled with seeded
    values; weight generation not timed)."""
    c = DecoderConfig(**cfg)
    sec = lib().nlo_decoder_time_positions(ctypes.byref(c), batch, ctx, steps)
    if sec < 0:
        raise RuntimeError("nlo_decoder_time_positions: bad arguments")
    return sec


DECODER_TENSORS = ["wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "sq", "sk", "sv", "so",
                   "sgate", "sup", "sdown", "attn_norm", "ffn_norm"]


def decoder_tensor(cfg: dict, layer: int, name: str) -> np.ndarray:
    """One tensor of the CPU model's synthetic weights (the same values the
    library generates from the seed): packed two-bit rows as uint32 for the
    ternary matrices, float32 for scales, gains ('embed', 'final_norm' with
    layer 0)."""
    which = {"embed": 16, "final_norm": 17}.get(name)
    if which is None:
        which = DECODER_TENSORS.index(name)
    H, hd, F = cfg["hidden"], cfg["head_dim"], cfg["ffn"]
    qd, kvd = cfg["heads"] * hd, cfg["kv_heads"] * hd
    words = {"wq": qd * H // 16, "wk": kvd * H // 16, "wv": kvd * H // 16, "wo": H * qd // 16,
             "wgate": F * H // 16, "wup": F * H // 16, "wdown": H * F // 16, "sq": qd,
             "sk": kvd, "sv": kvd, "so": H, "sgate": F, "sup": F, "sdown": H, "attn_norm": H,
             "ffn_norm": H, "embed": cfg["vocab"] * H, "final_norm": H}[name]
    out = np.zeros(words, np.uint32 if name.startswith("w") else np.float32)
    c = DecoderConfig(**{k: v for k, v in cfg.items() if k in [f[0] for f in DecoderConfig._fields_]})
    n = lib().nlo_decoder_tensor(ctypes.byref(c), layer, which, out.ctypes.data_as(ctypes.c_void_p))
    if n != words:
        raise RuntimeError(f"nlo_decoder_tensor({name}): {n} words, expected {words}")
    return out


# ---- metrics -------------------------------------------------------------

def tk_err(got, want) -> float:
    """max|got - want| / max|want| -- test/ternary-kernel-test.el:23-34."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if want.size == 0:
        return 0.0
    scale = max(float(np.max(np.abs(want))), 1.0e-12)
    return float(np.max(np.abs(got - want))) / scale
