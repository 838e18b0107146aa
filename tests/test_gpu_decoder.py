"""The ternary decoder on the GPU against its CPU model (oracle/nl_oracle_decoder.c).

No reference decoder exists to pin against (the reference repository holds
the kernels, not the model), so parity is with the composition of the
restated kernels: every step's logits within tk-err 1e-4, and the greedy
tokens identical wherever the CPU model's top two logits are not a near tie.
"""
import numpy as np
import pytest

import oracle as nlo

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=256, layers=2, heads=4, kv_heads=4, head_dim=64, ffn=512, vocab=1000,
             rms_eps=1e-5, rope_base=10000.0, seed=7)


def check_against_cpu(cfg, prompt, steps, max_seq):
    from nelisp_cuda.decoder import Decoder
    B, P = prompt.shape
    dec = Decoder(cfg, max_batch=B, max_seq=max_seq, keep_logits=True)
    toks, pf, dc = dec.generate(prompt, steps)
    lg = dec.logits()
    dec.close()
    want_t, want_lg = nlo.decoder_generate(dict(cfg, max_batch=B, max_seq=max_seq), prompt, steps,
                                           keep_logits=True)
    npos = P + steps - 1
    for p in range(npos):
        for b in range(B):
            err = nlo.tk_err(lg[p, b], want_lg[p, b])
            assert err < 1e-4, (p, b, err)
    # tokens: equal up to the first step whose top-2 margin is a near tie
    for b in range(B):
        for i in range(steps):
            row = want_lg[P - 1 + i, b]
            top2 = np.sort(row)[-2:]
            if top2[1] - top2[0] < 1e-3 * max(1.0, abs(top2[1])):
                break
            assert toks[b, i] == want_t[b, i], (b, i)
    assert pf >= 0 and dc > 0


def test_decoder_matches_cpu_model_mha():
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, SMALL["vocab"], size=(2, 5))
    check_against_cpu(SMALL, prompt, steps=6, max_seq=16)


def test_decoder_matches_cpu_model_gqa_batch3():
    cfg = dict(SMALL, heads=8, kv_heads=2, head_dim=32, hidden=256, seed=11)
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, cfg["vocab"], size=(3, 4))
    check_against_cpu(cfg, prompt, steps=5, max_seq=12)


def test_decoder_long_cache_many_splits():
    # max_seq 1100 over 4 KV heads at batch 1: 35 attention splits of 32 keys,
    # more than the merge loads in one round trip (its batched two-pass form)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, SMALL["vocab"], size=(1, 5))
    check_against_cpu(SMALL, prompt, steps=4, max_seq=1100)


def test_decoder_bitnet_shapes_one_layer():
    # the benchmark's layer shapes (hidden 2560, 20 heads of 128, FFN 6912)
    cfg = dict(hidden=2560, layers=1, heads=20, kv_heads=20, head_dim=128, ffn=6912,
               vocab=2048, rms_eps=1e-5, rope_base=10000.0, seed=3)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, cfg["vocab"], size=(2, 3))
    check_against_cpu(cfg, prompt, steps=3, max_seq=8)


def test_decoder_rejects_bad_requests():
    from nelisp_cuda import NlError
    from nelisp_cuda.decoder import Decoder
    dec = Decoder(SMALL, max_batch=2, max_seq=8)
    with pytest.raises(NlError):
        dec.generate(np.zeros((3, 2), np.int32), 2)          # batch > max_batch
    with pytest.raises(NlError):
        dec.generate(np.zeros((1, 6), np.int32), 4)          # past max_seq
    with pytest.raises(NlError):
        dec.generate(np.full((1, 2), SMALL["vocab"]), 2)     # token out of range
    dec.close()


def test_decoder_batched_prefill_matches_cpu_model():
    """Prompts of more than 16 rows in all take the batched prefill (tcgen05
    GEMMs, causal attention over the prompt); the generated tokens and the
    logits from the last prompt position on match the CPU model, which steps
    through the prompt one position at a time."""
    from nelisp_cuda.decoder import Decoder
    cfg = dict(SMALL, heads=8, kv_heads=4, head_dim=64, hidden=512, ffn=1024, seed=23)
    rng = np.random.default_rng(9)
    B, P, steps, max_seq = 3, 40, 5, 48
    prompt = rng.integers(0, cfg["vocab"], size=(B, P))
    dec = Decoder(cfg, max_batch=B, max_seq=max_seq, keep_logits=True)
    toks, pf, dc = dec.generate(prompt, steps)
    lg = dec.logits()
    dec.close()
    want_t, want_lg = nlo.decoder_generate(dict(cfg, max_batch=B, max_seq=max_seq), prompt, steps,
                                           keep_logits=True)
    for p in range(P - 1, P + steps - 1):
        for b in range(B):
            err = nlo.tk_err(lg[p, b], want_lg[p, b])
            assert err < 1e-4, (p, b, err)
    for b in range(B):
        for i in range(steps):
            row = want_lg[P - 1 + i, b]
            top2 = np.sort(row)[-2:]
            if top2[1] - top2[0] < 1e-3 * max(1.0, abs(top2[1])):
                break
            assert toks[b, i] == want_t[b, i], (b, i)


def test_decoder_from_uploaded_weights_matches_synthetic():
    """nl_decoder_create_from_weights on resident buffers (nl_upload) holding
    the very tensors the seed generates: the same logits, bit for bit, as the
    synthetic decoder; the handles are freed right after the constructor,
    which copies what it needs."""
    import ctypes

    from nelisp_cuda import _lib as L
    from nelisp_cuda.decoder import LAYER_TENSORS, Decoder
    cfg = dict(SMALL, heads=8, kv_heads=4, hidden=512, ffn=1024, seed=41)
    lib = L.load()
    rng = np.random.default_rng(8)
    B, P, steps, max_seq = 2, 4, 4, 12
    prompt = rng.integers(0, cfg["vocab"], size=(B, P))
    handles = []

    def up(a):
        h = ctypes.c_uint32()
        a = np.ascontiguousarray(a)
        L.check(lib.nl_upload(a.ctypes.data, a.size, ctypes.byref(h)))
        handles.append(h.value)
        return h.value

    full = dict(cfg, max_batch=B, max_seq=max_seq)
    w = {n: [up(nlo.decoder_tensor(full, l, n)) for l in range(cfg["layers"])]
         for n in LAYER_TENSORS}
    w["embed"] = up(nlo.decoder_tensor(full, 0, "embed"))
    w["final_norm"] = up(nlo.decoder_tensor(full, 0, "final_norm"))
    dec = Decoder(cfg, max_batch=B, max_seq=max_seq, keep_logits=True, weights=w)
    for h in handles:
        lib.nl_free(h)
    t1, _, _ = dec.generate(prompt, steps)
    lg1 = dec.logits()
    dec.close()
    dec = Decoder(cfg, max_batch=B, max_seq=max_seq, keep_logits=True)
    t0, _, _ = dec.generate(prompt, steps)
    lg0 = dec.logits()
    dec.close()
    assert np.array_equal(t1, t0)
    npos = P + steps - 1
    assert np.array_equal(lg1[:npos].view(np.uint32), lg0[:npos].view(np.uint32))


def test_decoder_from_weights_rejects_wrong_shapes():
    import ctypes

    from nelisp_cuda import NlError
    from nelisp_cuda import _lib as L
    from nelisp_cuda.decoder import LAYER_TENSORS, Decoder
    lib = L.load()
    h = ctypes.c_uint32()
    a = np.zeros(7, np.uint32)
    L.check(lib.nl_upload(a.ctypes.data, a.size, ctypes.byref(h)))
    w = {n: [h.value] * SMALL["layers"] for n in LAYER_TENSORS}
    w["embed"] = w["final_norm"] = h.value
    with pytest.raises(NlError) as e:
        Decoder(SMALL, max_batch=1, max_seq=8, weights=w)
    assert "holds 7 words" in str(e.value)
    lib.nl_free(h.value)
