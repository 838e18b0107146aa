"""The decode step as one persistent kernel (nl_step.cu: tensor parallelism 1,
batch <= 8; NELISP_DECODER_STEP=kernel) against the decoder's separate
kernels (NELISP_DECODER_STEP=kernels) and against the CPU model.

The GEMVs, the attention and the SwiGLU of the two paths are the same
arithmetic; the RMSNorm sums of squares are reduced in different orders, so
the logits agree to within a few f32 ulps of their rows (tk-err 1e-5), and
both paths stay within the decoder tests' 1e-4 of the CPU model.
"""
import os

import numpy as np
import pytest

import oracle as nlo

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=256, layers=2, heads=4, kv_heads=4, head_dim=64, ffn=512, vocab=1000,
             rms_eps=1e-5, rope_base=10000.0, seed=7)
GQA = dict(SMALL, hidden=512, heads=8, kv_heads=4, ffn=1024, seed=23)
# the benchmark's layer shapes; FFN 6912 splits the down GEMV into three K chunks
BITNET1 = dict(hidden=2560, layers=1, heads=20, kv_heads=20, head_dim=128, ffn=6912,
               vocab=2048, rms_eps=1e-5, rope_base=10000.0, seed=3)


def _run(cfg, prompt, steps, max_seq, mode):
    from nelisp_cuda.decoder import Decoder
    old = os.environ.get("NELISP_DECODER_STEP")
    if mode:
        os.environ["NELISP_DECODER_STEP"] = mode
    else:
        os.environ.pop("NELISP_DECODER_STEP", None)
    try:
        B = prompt.shape[0]
        dec = Decoder(cfg, max_batch=B, max_seq=max_seq, keep_logits=True)
        toks, _, _ = dec.generate(prompt, steps)
        lg = dec.logits()
        kps = dec.info()["kernels_per_step"]
        dec.close()
    finally:
        if old is None:
            os.environ.pop("NELISP_DECODER_STEP", None)
        else:
            os.environ["NELISP_DECODER_STEP"] = old
    return toks, lg, kps


@pytest.mark.parametrize("name,cfg,B,P,steps", [
    ("small_b1", SMALL, 1, 4, 5),
    ("small_b8", SMALL, 8, 2, 4),
    ("gqa_b3", GQA, 3, 3, 4),
    ("bitnet_b1", BITNET1, 1, 3, 3),
    ("bitnet_b8", BITNET1, 8, 2, 3),
    ("gqa_prefill_b2", GQA, 2, 20, 4),      # 38 prompt rows: the batched prefill first
])
def test_step_kernel_matches_separate_kernels_and_cpu(name, cfg, B, P, steps):
    rng = np.random.default_rng(sum(map(ord, name)))
    prompt = rng.integers(0, cfg["vocab"], size=(B, P))
    max_seq = P + steps + 2
    t1, lg1, kps1 = _run(cfg, prompt, steps, max_seq, "kernel")
    t0, lg0, kps0 = _run(cfg, prompt, steps, max_seq, "kernels")
    assert kps1 == 3, kps1                 # the step kernel, the LM head, the next token
    assert kps0 > 3 * cfg["layers"], kps0
    want_t, want_lg = nlo.decoder_generate(dict(cfg, max_batch=B, max_seq=max_seq), prompt,
                                           steps, keep_logits=True)
    first = P - 1 if B * (P - 1) > 16 else 0
    for p in range(first, P + steps - 1):
        for b in range(B):
            assert nlo.tk_err(lg1[p, b], lg0[p, b]) < 1e-5, (p, b)
            assert nlo.tk_err(lg1[p, b], want_lg[p, b]) < 1e-4, (p, b)
    assert np.array_equal(t1, t0)
