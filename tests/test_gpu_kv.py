"""Paged, ring (attention sink + rolling window) and entry-list KV caches on
the GPU against the oracle (oracle/nl_oracle.c, restating
lisp/nelisp-gpu-kernels.el:396-451 and :1044-1246).  Copies are exact;
attention is within 1e-4 (tk-err) as the other attention operators."""
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


def rope_tables(rows, half, rng):
    ang = rng.uniform(0, 6.3, size=(rows, half)).astype(np.float32)
    return np.cos(ang).astype(np.float32).ravel(), np.sin(ang).astype(np.float32).ravel()


@pytest.mark.parametrize("pos", [1, 3, 4, 9, 13])
def test_cache_append_ring(host, pos):
    kvdim, nsink, win = 96, 3, 5
    rng = np.random.default_rng(pos)
    src = rng.standard_normal(kvdim).astype(np.float32)
    cache = rng.standard_normal((nsink + win) * kvdim).astype(np.float32)
    got = host.run2("cache-append-ring", [("in", src), ("in", [float(pos)]), ("inout", cache)],
                    [kvdim, nsink, win], g64(kvdim))[0]
    want = nlo.cache_append_ring(src, [float(pos)], cache, kvdim, nsink, win)
    assert np.array_equal(got, want)


def test_qkv_append(host):
    dim, kvdim, wbase = 256, 128, 3 * 128
    rng = np.random.default_rng(2)
    qkv = rng.standard_normal(dim + 2 * kvdim).astype(np.float32)
    ck = rng.standard_normal(6 * kvdim).astype(np.float32)
    cv = rng.standard_normal(6 * kvdim).astype(np.float32)
    got = host.run2("qkv-append", [("in", qkv), ("inout", ck), ("inout", cv)], [dim, kvdim, wbase],
                    g64(kvdim))
    wk, wv = nlo.qkv_append(qkv, ck, cv, dim, kvdim, wbase)
    assert np.array_equal(got[0], wk) and np.array_equal(got[1], wv)


def paged_pool(rng, B, mbps, bs, kvdim, nblocks):
    table = np.stack([rng.permutation(nblocks)[:mbps] for _ in range(B)]).astype(np.float32)
    pool = rng.standard_normal(nblocks * bs * kvdim).astype(np.float32)
    return table.ravel(), pool


@pytest.mark.parametrize("var", [False, True])
def test_cache_append_paged(host, var):
    B, kvdim, bs, mbps, nblocks = 3, 64, 4, 5, 20
    rng = np.random.default_rng(7 + var)
    table, pool = paged_pool(rng, B, mbps, bs, kvdim, nblocks)
    src = rng.standard_normal(B * kvdim).astype(np.float32)
    if var:
        lens = np.array([2, 9, 17], np.float32)
        got = host.run2("cache-append-paged-v", [("in", src), ("in", lens), ("in", table),
                                                 ("inout", pool)], [B, kvdim, bs, mbps],
                        g64(B * kvdim))[0]
        want = nlo.cache_append_paged(src, None, lens, table, pool, B, kvdim, bs, mbps)
    else:
        got = host.run2("cache-append-paged", [("in", src), ("in", [11.0]), ("in", table),
                                               ("inout", pool)], [B, kvdim, bs, mbps],
                        g64(B * kvdim))[0]
        want = nlo.cache_append_paged(src, [11.0], None, table, pool, B, kvdim, bs, mbps)
    assert np.array_equal(got, want)


def test_block_copy(host):
    bs, kvdim = 4, 32
    rng = np.random.default_rng(5)
    pool = rng.standard_normal(6 * bs * kvdim).astype(np.float32)
    got = host.run2("block-copy", [("inout", pool)], [bs, kvdim, 1, 4], g64(bs * kvdim))[0]
    assert np.array_equal(got, nlo.block_copy(pool, bs, kvdim, 1, 4))


def test_decode_rope_b_v(host):
    B, heads, hd, rows = 3, 4, 64, 40
    cols = heads * hd
    rng = np.random.default_rng(6)
    X = rng.standard_normal(B * cols).astype(np.float32)
    co, si = rope_tables(rows, hd // 2, rng)
    lens = np.array([0, 17, 39], np.float32)
    got = host.run2("decode-rope-b-v", [("in", X), ("in", co), ("in", si), ("in", [-1.0]),
                                        ("in", lens), ("out", B * cols)], [B, cols, heads],
                    g64(B * heads * hd // 2))[0]
    want = nlo.decode_rope_b_v(X, co, si, [-1.0], lens, B, cols, heads)
    assert np.max(np.abs(got - want)) < 1e-6


@pytest.mark.parametrize("var", [False, True])
@pytest.mark.parametrize("heads,kvheads,hd", [(8, 8, 128), (8, 2, 64), (4, 2, 32)])
def test_decode_attn_paged(host, var, heads, kvheads, hd):
    B, bs, mbps, nblocks = 3, 16, 6, 24
    dim, kvdim = heads * hd, kvheads * hd
    rng = np.random.default_rng(heads * 10 + hd + var)
    table, _ = paged_pool(rng, B, mbps, bs, kvdim, nblocks)
    ck = rng.standard_normal(nblocks * bs * kvdim).astype(np.float32)
    cv = rng.standard_normal(nblocks * bs * kvdim).astype(np.float32)
    Q = rng.standard_normal(B * dim).astype(np.float32)
    if var:
        lens = np.array([0, 40, 95], np.float32)
        got = host.run2("decode-attn-paged-v", [("in", Q), ("in", ck), ("in", cv), ("in", lens),
                                                ("in", table), ("out", B * dim)],
                        [B, dim, heads, kvheads, bs, mbps], g64(B * dim))[0]
        want = nlo.decode_attn_paged(Q, ck, cv, None, lens, table, B, dim, heads, kvheads, bs,
                                     mbps)
    else:
        got = host.run2("decode-attn-paged", [("in", Q), ("in", ck), ("in", cv), ("in", [70.0]),
                                              ("in", table), ("out", B * dim)],
                        [B, dim, heads, kvheads, bs, mbps], g64(B * dim))[0]
        want = nlo.decode_attn_paged(Q, ck, cv, [70.0], None, table, B, dim, heads, kvheads, bs,
                                     mbps)
    assert nlo.tk_err(got, want) < 1e-4


@pytest.mark.parametrize("pos", [5, 30, 77])
@pytest.mark.parametrize("hd", [128, 64])
def test_decode_attn_stream(host, pos, hd):
    heads, kvheads, nsink, win = 8, 4, 4, 28
    dim, kvdim, cap = heads * hd, kvheads * hd, nsink + win
    rng = np.random.default_rng(pos + hd)
    Q = rng.standard_normal(dim).astype(np.float32)
    ck = rng.standard_normal(cap * kvdim).astype(np.float32)
    cv = rng.standard_normal(cap * kvdim).astype(np.float32)
    co, si = rope_tables(cap, hd // 2, rng)
    got = host.run2("decode-attn-stream", [("in", Q), ("in", ck), ("in", cv), ("in", [float(pos)]),
                                           ("in", co), ("in", si), ("out", dim)],
                    [dim, heads, kvheads, nsink, win], g64(dim))[0]
    want = nlo.decode_attn_stream(Q, ck, cv, [float(pos)], co, si, dim, heads, kvheads, nsink, win)
    assert nlo.tk_err(got, want) < 1e-4


@pytest.mark.parametrize("hd", [128, 32])
def test_attn_stream_entries(host, hd):
    heads, kvheads, ne, rows = 4, 2, 37, 64
    dim, kvdim = heads * hd, kvheads * hd
    rng = np.random.default_rng(hd)
    ck = rng.standard_normal(rows * kvdim).astype(np.float32)
    cv = rng.standard_normal(rows * kvdim).astype(np.float32)
    ent = np.stack([rng.permutation(rows)[:ne] * kvdim, rng.integers(0, rows, ne)], 1)
    ent = ent.astype(np.float32).ravel()
    Q = rng.standard_normal(dim).astype(np.float32)
    co, si = rope_tables(rows, hd // 2, rng)
    got = host.run2("attn-stream-entries", [("in", Q), ("in", ck), ("in", cv), ("in", ent),
                                            ("in", co), ("in", si), ("out", dim)],
                    [dim, heads, kvheads, ne, 21], g64(dim))[0]
    want = nlo.attn_stream_entries(Q, ck, cv, ent, co, si, dim, heads, kvheads, ne, 21)
    assert nlo.tk_err(got, want) < 1e-4


def test_paged_table_out_of_range_is_skipped(host):
    # a block id past the pool: the key is skipped (the reference would read
    # past the buffer); the call neither faults nor fails
    B, heads, hd, bs, mbps = 1, 2, 128, 16, 2
    dim = heads * hd
    ck = np.ones(bs * dim, np.float32)
    cv = np.ones(bs * dim, np.float32)
    table = np.array([0.0, 1000.0], np.float32)
    got = host.run2("decode-attn-paged", [("in", np.ones(dim, np.float32)), ("in", ck), ("in", cv),
                                          ("in", [20.0]), ("in", table), ("out", dim)],
                    [B, dim, heads, heads, bs, mbps], g64(dim))[0]
    assert np.allclose(got, 1.0)
