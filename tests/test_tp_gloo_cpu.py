"""The tensor-parallel decoder's partition and recombination, on CPU.

nl_decoder_shard (host arithmetic, the function the decoder's constructors
use) gives each rank its KV heads, FFN rows and vocabulary rows.  Two gloo
ranks then take their parts of one layer's products with the CPU model's
ternary GEMV (oracle/nl_oracle.c, the reference's ternary-rows) and put them
back together the way the decoder does on the GPU:

- Q|K|V and gate|up are split by output rows: the ranks' rows, concatenated
  in rank order, equal the unsharded product bit for bit;
- O and down are split by input columns: each rank applies the per-row scale
  to its partial product, and the sum over ranks (the decoder's all-reduce)
  matches the unsharded product within 1e-6 of its largest magnitude (only
  the order of the float additions differs);
- the LM head is split by vocabulary rows: each rank's best (logit, index)
  key, all-gathered and maximised, gives the global greedy token with the
  lowest index winning a tie, inside one rank and across two.

The same checks also run at three ranks (the row-split sums then within the
tolerance only: gloo does not fix the order of three addends).  Each check
has a control that must fail: the parts in the wrong rank order, one rank's
partial product without the sum, and a tie-break that favours the higher
index.
"""
import datetime
import multiprocessing as mp
import socket
import traceback

import numpy as np
import pytest

import oracle as nlo

CFG = dict(hidden=256, layers=1, heads=6, kv_heads=3, head_dim=64, ffn=384, vocab=1001,
           rms_eps=1e-5, rope_base=10000.0, seed=5, max_batch=3, max_seq=8)
ROW_SPLIT_TOL = 1e-6


def _shard(cfg, rank, size):
    from nelisp_cuda.decoder import shard
    return shard(cfg, rank, size)


# ---- the partition (single process) ----------------------------------------------

def _check_cover(cfg, size):
    parts = [_shard(cfg, r, size) for r in range(size)]
    for key, total in (("kv_head", cfg["kv_heads"]), ("ffn", cfg["ffn"]),
                       ("vocab", cfg["vocab"])):
        begin = "kv_head_begin" if key == "kv_head" else key + "_begin"
        count = "kv_heads" if key == "kv_head" else key
        at = 0
        for p in parts:                      # contiguous, in rank order, no gap or overlap
            assert p[begin] == at, (key, size, parts)
            assert p[count] > 0
            at += p[count]
        assert at == total, (key, size)
        counts = [p[count] for p in parts]
        assert max(counts) - min(counts) <= (128 if key == "ffn" else 1)
        assert counts == sorted(counts, reverse=True)      # the longer ranges first
    assert all(p["ffn_begin"] % 128 == 0 and p["ffn"] % 128 == 0 for p in parts)
    return parts


def test_shard_partition_bitnet_shapes():
    from nelisp_cuda.decoder import BITNET_2B
    for size in (1, 2, 3, 4, 5, 8):
        _check_cover(BITNET_2B, size)
    parts = _check_cover(BITNET_2B, 8)
    assert [p["kv_heads"] for p in parts] == [3, 3, 3, 3, 2, 2, 2, 2]
    assert [p["ffn"] for p in parts] == [896] * 6 + [768] * 2
    assert [p["vocab"] for p in parts] == [16032] * 8
    assert _shard(BITNET_2B, 0, 1) == dict(kv_head_begin=0, kv_heads=20, ffn_begin=0,
                                           ffn=6912, vocab_begin=0, vocab=128256)


def test_shard_partition_gqa_and_refusals():
    from nelisp_cuda import NlError
    gqa = dict(CFG, heads=16, kv_heads=4, head_dim=128, hidden=512, ffn=1024, vocab=5003)
    for size in (1, 2, 3, 4):
        _check_cover(gqa, size)
    with pytest.raises(NlError, match="without heads"):
        _shard(gqa, 4, 5)                    # 5 ranks over 4 KV heads
    with pytest.raises(NlError, match="rank"):
        _shard(gqa, 2, 2)
    with pytest.raises(NlError, match="rank"):
        _shard(gqa, 0, 0)
    with pytest.raises(NlError, match="decoder config"):
        _shard(dict(gqa, heads=6), 0, 1)     # heads not a multiple of kv_heads


# ---- recombination over two gloo ranks -------------------------------------------

def argmax_keys(logits, index0):
    """The decoder's order-preserving argmax key per row of LOGITS
    [rows x n] (columns are vocabulary rows INDEX0, INDEX0+1, ...): the float's
    bits made to sort as unsigned integers (a NaN scores lowest) in the high
    word, 0xFFFFFFFF - index in the low word, so that the largest key is the
    largest logit and, among equal logits, the lowest index.  Returns each
    row's largest key (uint64)."""
    v = np.ascontiguousarray(logits, np.float32)
    u = v.view(np.uint32)
    u = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000))
    u = np.where(np.isnan(v), np.uint32(0), u).astype(np.uint64)
    idx = (np.arange(v.shape[1], dtype=np.uint64) + np.uint64(index0))[None, :]
    keys = (u << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - idx)
    return keys.max(axis=1)


def _rows(wp, cols, r0, n):
    """Rows R0 .. R0+N-1 of a packed ternary matrix of COLS columns."""
    return np.ascontiguousarray(wp.reshape(-1, cols // 16)[r0:r0 + n])


def _cols(wp, cols, c0, n):
    """Columns C0 .. C0+N-1 (multiples of 16) of a packed ternary matrix."""
    return np.ascontiguousarray(wp.reshape(-1, cols // 16)[:, c0 // 16:(c0 + n) // 16])


def _lm_problem(cfg):
    """LM-head inputs with planted ties: sequence 0's best rows are 100 and 700
    (equal logits, on different ranks at TP = 2), sequence 1's are 800 and
    900 (equal, both on rank 1); sequence 2 is left to chance."""
    H = cfg["hidden"]
    rng = np.random.default_rng(31)
    E = nlo.decoder_tensor(cfg, 0, "embed").reshape(cfg["vocab"], H).copy()
    h = rng.standard_normal((3, H)).astype(np.float32)
    E[100] = E[700] = np.sign(h[0])
    E[800] = E[900] = 2.0 * np.sign(h[1])
    return E, h


def _lm_logits(E, h):
    # each row summed on its own (float64 pairwise), so slices give the same bits
    return np.stack([(E.astype(np.float64) * hb.astype(np.float64)).sum(axis=1)
                     for hb in h]).astype(np.float32)


def _rank_main(rank, size, port, errors):
    try:
        import torch
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=size, timeout=datetime.timedelta(seconds=60))
        try:
            _rank_checks(rank, size, dist, torch)
        finally:
            dist.destroy_process_group()
    except BaseException:                    # reported to the parent, which fails the test
        errors.put((rank, traceback.format_exc()))


def _gather(dist, a):
    """Every rank's array A in rank order (the shards differ in size, which
    gloo's tensor all_gather does not take; the arrays travel pickled, bits
    unchanged)."""
    outs = [None] * dist.get_world_size()
    dist.all_gather_object(outs, np.ascontiguousarray(a))
    return outs


def _rank_checks(rank, size, dist, torch):
    nlo.set_threads(1)
    cfg = CFG
    H, hd, F = cfg["hidden"], cfg["head_dim"], cfg["ffn"]
    grp = cfg["heads"] // cfg["kv_heads"]
    qd, kvd = cfg["heads"] * hd, cfg["kv_heads"] * hd
    me = _shard(cfg, rank, size)
    T = {n: nlo.decoder_tensor(cfg, 0, n) for n in nlo.DECODER_TENSORS}
    rng = np.random.default_rng(17)          # the same inputs on every rank
    B = 3
    x = rng.standard_normal((B, H)).astype(np.float32)
    ctx = rng.standard_normal((B, qd)).astype(np.float32)
    act = rng.standard_normal((B, F)).astype(np.float32)

    # split by output rows: Q, K, V (by KV head with its query heads), gate and up
    h0, hr = me["kv_head_begin"] * grp * hd, me["kv_heads"] * grp * hd
    k0, kr = me["kv_head_begin"] * hd, me["kv_heads"] * hd
    f0, fr = me["ffn_begin"], me["ffn"]
    for w, s, full_rows, r0, n in (("wq", "sq", qd, h0, hr), ("wk", "sk", kvd, k0, kr),
                                   ("wv", "sv", kvd, k0, kr), ("wgate", "sgate", F, f0, fr),
                                   ("wup", "sup", F, f0, fr)):
        part = nlo.ternary_gemv_rows(x, _rows(T[w], H, r0, n), T[s][r0:r0 + n], B, n, H)
        got = np.concatenate([p.reshape(B, -1) for p in _gather(dist, part.reshape(B, n))],
                             axis=1)
        want = nlo.ternary_gemv_rows(x, T[w], T[s], B, full_rows, H).reshape(B, full_rows)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), w
        # control: the same parts in the wrong rank order do not give the product
        parts = _gather(dist, part.reshape(B, n))
        swapped = np.concatenate([p.reshape(B, -1) for p in parts[1:] + parts[:1]], axis=1)
        assert not np.array_equal(swapped, want), w

    # split by input columns: O (the rank's query heads), down (its FFN rows)
    for w, s, a, cols, c0, n in (("wo", "so", ctx, qd, h0, hr), ("wdown", "sdown", act, F, f0, fr)):
        part = nlo.ternary_gemv_rows(np.ascontiguousarray(a[:, c0:c0 + n]), _cols(T[w], cols, c0, n),
                                     T[s], B, H, n).reshape(B, H)
        parts = _gather(dist, part)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        summed = t.numpy()
        in_order = parts[0].copy()
        for p in parts[1:]:
            in_order = (in_order + p).astype(np.float32)
        if size == 2:                        # two addends: the order cannot matter
            assert np.array_equal(summed.view(np.uint32), in_order.view(np.uint32)), w
        want = nlo.ternary_gemv_rows(a, T[w], T[s], B, H, cols).reshape(B, H)
        assert nlo.tk_err(summed, want) < ROW_SPLIT_TOL, (w, nlo.tk_err(summed, want))
        # control: one rank's partial product without the all-reduce is far off
        assert nlo.tk_err(parts[0], want) > 1e-2, w

    # LM head split by vocabulary rows: the best key of each rank, all-gathered
    E, h = _lm_problem(cfg)
    v0, vr = me["vocab_begin"], me["vocab"]
    mine = argmax_keys(_lm_logits(E[v0:v0 + vr], h), v0)
    keys = np.stack([k.view(np.uint64) for k in _gather(dist, mine.view(np.int64))])
    best = keys.max(axis=0)
    token = (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64)
    full = _lm_logits(E, h)
    assert token.tolist() == np.argmax(full, axis=1).tolist()
    assert token[0] == 100 and token[1] == 800
    # control: a key whose low word favoured the higher index breaks the tie
    # inside rank order the other way (row 1: 900, not 800)
    v = np.ascontiguousarray(_lm_logits(E[v0:v0 + vr], h))
    hi = [(float(r.max()), v0 + int(np.flatnonzero(r == r.max())[-1])) for r in v]
    hi_all = [None] * size
    dist.all_gather_object(hi_all, hi)
    wrong = [max(q[b] for q in hi_all)[1] for b in range(len(hi))]
    assert wrong[1] == 900 and wrong[0] == 700


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("size", [2, 3])
def test_tp_layer_recombines_over_gloo_ranks(size):
    """Two ranks (KV heads 2/1, FFN blocks 2/1, vocabulary 501/500) and three
    (one KV head and one FFN block each, vocabulary 334/334/333)."""
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, size, port, errors)) for r in range(size)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    hung = [p for p in procs if p.is_alive()]
    for p in hung:
        p.kill()
        p.join()
    reports = []
    while not errors.empty():
        reports.append(errors.get())
    assert not hung, "a gloo rank did not finish"
    assert not reports, "\n".join(f"rank {r}:\n{t}" for r, t in reports)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_argmax_key_order():
    """Larger logit first, lower index on ties, negative values below positive
    ones, a NaN never chosen."""
    v = np.array([[-3.0, -1.0, -1.0, np.nan, -2.0]], np.float32)
    k = argmax_keys(v, 10)
    assert int(np.uint64(0xFFFFFFFF) - (k[0] & np.uint64(0xFFFFFFFF))) == 11
    v = np.array([[0.5, 2.0, 2.0, -7.0]], np.float32)
    k = argmax_keys(v, 0)
    assert int(np.uint64(0xFFFFFFFF) - (k[0] & np.uint64(0xFFFFFFFF))) == 1
