"""Generate the golden fixtures under tests/golden/ from the reference's tests.

The reference (zawatton/nelisp-gpu) tests its kernels from Emacs, which is not
installed here, so its expected values cannot be produced by running it.  Each
fixture below instead restates one of the reference tests' deterministic
generators and its CPU reference arithmetic, in double precision as Emacs
floats are, and stores inputs and expected outputs:

* ``ternary_tk.npz`` -- test/ternary-kernel-test.el:17-99: the LCG
  x <- (x*1103515245 + 12345) mod 2^31 from seed 20260921 (:17, :36-38), the
  draw order of `tk-run' (:53-66), the two-bit packer `tk-pack' (:40-50) and
  the double sums of `tk-cpu-forward' (:79-89) and of the transpose check
  (:119-127).
* ``verify_el.npz`` -- test/verify.el:22-151: the modular generators for
  matmul 32x24x16, softmax 24x40, linear 20x12->16 (:65-77), matmul-tiled and
  matmul-reg 20x24x12 and scale n=50 (:101-108), with float64 expected outputs (the
  photon-tensor oracle that verify.el compares with is absent; its results
  are the same float64 arithmetic).
* ``f32_codec.npz`` -- test/f32-test.el:36-108: the encoder boundary cases.

Run:  python tests/golden/make_golden.py   (writes next to this file)
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


# ---- test/ternary-kernel-test.el ------------------------------------------

class TkRng:
    """`tk-rnd' (test/ternary-kernel-test.el:36-38)."""

    def __init__(self, seed: int = 20260921):
        self.seed = seed

    def __call__(self) -> float:
        self.seed = (self.seed * 1103515245 + 12345) % 2147483648
        return self.seed / 2147483648.0


def tk_pack(trits: np.ndarray, out: int, cols: int, wng: int) -> np.ndarray:
    """`tk-pack' (:40-50): code +1 -> 01, -1 -> 11, 0 -> 00; field i of a row
    at byte i/4, bits 2*(i%4); returned as little-endian uint32 words."""
    by = np.zeros(out * wng * 4, np.uint8)
    for o in range(out):
        for i in range(cols):
            v = int(trits[o * cols + i])
            code = 1 if v == 1 else (3 if v == -1 else 0)
            idx = o * wng * 4 + (i >> 2)
            by[idx] |= code << (2 * (i & 3))
    return by.view("<u4").astype(np.uint32)


def make_tk() -> dict:
    seq, out, cols, bsize = 3, 6, 256, 128
    nblk, wng = cols // bsize, cols // 16
    rnd = TkRng()
    trits = np.zeros(out * cols, np.int8)
    beta = np.zeros(out * nblk, np.float64)
    bias = np.zeros(out, np.float64)
    x = np.zeros(seq * cols, np.float64)
    g = np.zeros(seq * out, np.float64)
    for o in range(out):
        bias[o] = 0.4 * rnd() - 0.2
        for b in range(nblk):
            beta[o * nblk + b] = 0.01 + 0.05 * rnd()
        for i in range(cols):
            trits[o * cols + i] = int(3.0 * rnd()) - 1     # truncate toward 0
    for i in range(seq * cols):
        x[i] = 2.0 * rnd() - 1.0
    for i in range(seq * out):
        g[i] = 2.0 * rnd() - 1.0
    wp = tk_pack(trits, out, cols, wng)
    # tk-cpu-forward (:79-89): acc += trit*beta*x, left to right; y = bias + acc
    y = np.zeros(seq * out, np.float64)
    for s in range(seq):
        for o in range(out):
            acc = 0.0
            for i in range(cols):
                acc += (float(trits[o * cols + i]) * beta[o * nblk + i // bsize]) * x[s * cols + i]
            y[s * out + o] = bias[o] + acc
    # transpose reference (:119-127): acc += trit*beta*g over o
    xt = np.zeros(seq * cols, np.float64)
    for s in range(seq):
        for i in range(cols):
            acc = 0.0
            for o in range(out):
                acc += (float(trits[o * cols + i]) * beta[o * nblk + i // 128]) * g[s * out + o]
            xt[s * cols + i] = acc
    return dict(seq=seq, out=out, cols=cols, nblk=nblk, wng=wng,
                trits=trits, wp=wp, beta=beta, bias=bias, x=x, g=g,
                y_want=y, xt_want=xt)


# ---- test/verify.el -------------------------------------------------------

def gen(n, fn) -> np.ndarray:
    """`nelisp-gpu-gen' (lisp/nelisp-gpu-run.el:99-103) in float64."""
    return np.array([float(fn(i)) for i in range(n)], np.float64)


def make_verify() -> dict:
    d = {}
    # matmul (32x24)*(24x16), verify.el:22-32
    M, K, N = 32, 24, 16
    A = gen(M * K, lambda i: 0.1 * ((i % 7) - 3))
    B = gen(K * N, lambda i: 0.1 * ((i % 5) - 2))
    d["matmul_A"], d["matmul_B"] = A, B
    d["matmul_C"] = (A.reshape(M, K) @ B.reshape(K, N)).ravel()
    # softmax (24x40), verify.el:34-42
    M2, N2 = 24, 40
    S = gen(M2 * N2, lambda i: 0.2 * ((i % 11) - 5)).reshape(M2, N2)
    e = np.exp(S - S.max(axis=1, keepdims=True))
    d["softmax_A"] = S.ravel()
    d["softmax_C"] = (e / e.sum(axis=1, keepdims=True)).ravel()
    # linear X(20x12) W(16x12)^T + B(16), verify.el:65-77
    Mx, IN, OUT = 20, 12, 16
    X = gen(Mx * IN, lambda i: 0.1 * ((i % 7) - 3))
    W = gen(OUT * IN, lambda i: 0.1 * ((i % 5) - 2))
    Bv = gen(OUT, lambda i: 0.05 * ((i % 3) - 1))
    d["linear_X"], d["linear_W"], d["linear_B"] = X, W, Bv
    d["linear_C"] = (X.reshape(Mx, IN) @ W.reshape(OUT, IN).T + Bv).ravel()
    # matmul-tiled / matmul-reg (20x24)*(24x12), verify.el:79-89, :139-151
    Mt, Kt, Nt = 20, 24, 12
    At = gen(Mt * Kt, lambda i: 0.1 * ((i % 7) - 3))
    Bt = gen(Kt * Nt, lambda i: 0.1 * ((i % 5) - 2))
    d["tiled_A"], d["tiled_B"] = At, Bt
    d["tiled_C"] = (At.reshape(Mt, Kt) @ Bt.reshape(Kt, Nt)).ravel()
    # scale n=50, k=0.3, verify.el:101-108
    A5 = gen(50, lambda i: 0.1 * (i - 25))
    d["scale_A"], d["scale_k"] = A5, np.array([0.3])
    d["scale_C"] = A5 * 0.3
    return d


# ---- test/f32-test.el -----------------------------------------------------

def make_f32() -> dict:
    return dict(
        normals=np.array([1.0, 0.5, -3.25, 3.14159265358979, 1.0e-10, -2.5e7,
                          6.02e23, 1.0e-30]),
        subnormals=np.array([1.0e-38, 1.0e-39, 1.0e-40, 3.7e-44, -3.7e-44,
                             1.0e-45, -1.0e-41]),
        small=np.array([1.0e-39, 1.0e-40, 1.0e-42, 3.7e-44, 1.0e-45, 1.0e-60,
                        1.0e-300]),
        flush=np.array([1.0e-60, 5.0e-46]),
        overflow=np.array([1.0e300, -1.0e39]),
        flt_max=np.array([3.4028234663852886e38]),
        softmax_tail=np.exp(-0.05 * np.arange(4096, dtype=np.float64)),
    )


def main() -> None:
    np.savez_compressed(os.path.join(HERE, "ternary_tk.npz"), **make_tk())
    np.savez_compressed(os.path.join(HERE, "verify_el.npz"), **make_verify())
    np.savez_compressed(os.path.join(HERE, "f32_codec.npz"), **make_f32())
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
