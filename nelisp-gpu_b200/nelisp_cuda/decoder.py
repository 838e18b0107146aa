"""The ternary decoder of libnelisp_cuda (nl_decoder_* in include/nelisp_cuda.h).

    dec = Decoder(config, tp_rank=0, tp_size=1)         # weights generated on the GPU
    tokens, prefill_ms, decode_ms = dec.generate(prompt, steps)

For tensor parallelism run one process per GPU: rank 0 calls nccl_unique_id()
and broadcasts the 128 bytes (e.g. with torch.distributed) before every rank
constructs its Decoder with the same id.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L

BITNET_2B = dict(hidden=2560, layers=30, heads=20, kv_heads=20, head_dim=128, ffn=6912,
                 vocab=128256, rms_eps=1e-5, rope_base=10000.0, seed=20261201)


class Config(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_uint32), ("layers", ctypes.c_uint32),
                ("heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
                ("vocab", ctypes.c_uint32), ("max_batch", ctypes.c_uint32),
                ("max_seq", ctypes.c_uint32), ("rms_eps", ctypes.c_float),
                ("rope_base", ctypes.c_float), ("seed", ctypes.c_uint64)]


_U32P = ctypes.POINTER(ctypes.c_uint32)


class Weights(ctypes.Structure):
    """nl_decoder_weights: resident-buffer handles of a decoder's tensors."""
    _P = _U32P
    _fields_ = [("embed", ctypes.c_uint32), ("final_norm", ctypes.c_uint32)] + \
        [(n, _U32P) for n in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "sq", "sk", "sv",
                           "so", "sgate", "sup", "sdown", "attn_norm", "ffn_norm")]


LAYER_TENSORS = ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "sq", "sk", "sv", "so",
                 "sgate", "sup", "sdown", "attn_norm", "ffn_norm")


def _bind(lib):
    if getattr(lib, "_nl_decoder_bound", False):
        return lib
    lib.nl_nccl_unique_id.argtypes = [ctypes.c_void_p]
    lib.nl_nccl_unique_id.restype = ctypes.c_int
    lib.nl_decoder_create.argtypes = [ctypes.POINTER(Config), ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_void_p)]
    lib.nl_decoder_create.restype = ctypes.c_int
    lib.nl_decoder_create_from_weights.argtypes = [ctypes.POINTER(Config), ctypes.POINTER(Weights),
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                                   ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
    lib.nl_decoder_create_from_weights.restype = ctypes.c_int
    lib.nl_decoder_generate.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32,
                                        ctypes.POINTER(ctypes.c_int32),
                                        ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_double)]
    lib.nl_decoder_generate.restype = ctypes.c_int
    lib.nl_decoder_logits.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_float),
                                      ctypes.c_uint64]
    lib.nl_decoder_logits.restype = ctypes.c_int
    lib.nl_decoder_info.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32),
                                    ctypes.POINTER(ctypes.c_uint64),
                                    ctypes.POINTER(ctypes.c_uint64)]
    lib.nl_decoder_info.restype = ctypes.c_int
    lib.nl_decoder_shard.argtypes = [ctypes.POINTER(Config), ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_uint32)]
    lib.nl_decoder_shard.restype = ctypes.c_int
    lib.nl_decoder_destroy.argtypes = [ctypes.c_void_p]
    lib.nl_decoder_destroy.restype = None
    lib._nl_decoder_bound = True
    return lib


def nccl_unique_id() -> bytes:
    lib = _bind(L.load())
    buf = ctypes.create_string_buffer(128)
    L.check(lib.nl_nccl_unique_id(buf))
    return buf.raw


SHARD_KEYS = ("kv_head_begin", "kv_heads", "ffn_begin", "ffn", "vocab_begin", "vocab")


def _config(cfg: dict) -> Config:
    return Config(**{k: v for k, v in cfg.items() if k in [f[0] for f in Config._fields_]})


def shard(config: dict, tp_rank: int, tp_size: int) -> dict:
    """Rank TP_RANK's part of a TP_SIZE-way decoder of CONFIG (the keys of
    Decoder.info()'s shard), computed on the host by nl_decoder_shard: no GPU
    or decoder needed.  Raises NlError where the constructors would refuse."""
    lib = _bind(L.load())
    c = _config(dict(dict(max_batch=1, max_seq=1), **config))
    out = (ctypes.c_uint32 * 6)()
    L.check(lib.nl_decoder_shard(ctypes.byref(c), tp_rank, tp_size, out))
    return dict(zip(SHARD_KEYS, list(out)))


class Decoder:
    def __init__(self, config: dict, max_batch: int, max_seq: int, tp_rank: int = 0,
                 tp_size: int = 1, nccl_id: bytes | None = None, keep_logits: bool = False,
                 device: int | None = None, weights: dict | None = None):
        """WEIGHTS (optional): resident-buffer handles (nl_upload ...) of the
        full tensors -- 'embed' and 'final_norm' handles, and for each name in
        LAYER_TENSORS a list of one handle per layer; without it the weights
        are generated from the config's seed."""
        self.lib = _bind(L.load())
        if device is not None:
            L.check(self.lib.nl_init(device))
        self.cfg = dict(config, max_batch=max_batch, max_seq=max_seq)
        c = _config(self.cfg)
        h = ctypes.c_void_p()
        idbuf = ctypes.create_string_buffer(nccl_id, 128) if nccl_id else None
        if weights is None:
            L.check(self.lib.nl_decoder_create(ctypes.byref(c), tp_rank, tp_size, idbuf,
                                               1 if keep_logits else 0, ctypes.byref(h)))
        else:
            arrays = {n: (ctypes.c_uint32 * len(weights[n]))(*weights[n]) for n in LAYER_TENSORS}
            w = Weights(embed=weights["embed"], final_norm=weights["final_norm"],
                        **{n: ctypes.cast(a, Weights._P) for n, a in arrays.items()})
            L.check(self.lib.nl_decoder_create_from_weights(ctypes.byref(c), ctypes.byref(w),
                                                            tp_rank, tp_size, idbuf,
                                                            1 if keep_logits else 0,
                                                            ctypes.byref(h)))
        self.h = h
        self.tp_rank, self.tp_size = tp_rank, tp_size

    def generate(self, prompt, steps: int):
        """Greedy decode STEPS tokens after PROMPT ([batch x prompt_len] ints).
        Returns (tokens [batch x steps], prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        B, P = p.shape
        out = np.zeros((B, steps), np.int32)
        pf, dc = ctypes.c_double(), ctypes.c_double()
        L.check(self.lib.nl_decoder_generate(self.h, B, P,
                                             p.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                             steps,
                                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                             ctypes.byref(pf), ctypes.byref(dc)))
        return out, pf.value, dc.value

    def info(self):
        shard = (ctypes.c_uint32 * 6)()
        wb, kps = ctypes.c_uint64(), ctypes.c_uint64()
        L.check(self.lib.nl_decoder_info(self.h, shard, ctypes.byref(wb), ctypes.byref(kps)))
        return dict(zip(SHARD_KEYS, list(shard)), weight_bytes=wb.value,
                    kernels_per_step=kps.value)

    def logits(self):
        """[max_seq, max_batch, vocab rows of this rank] of the last generate."""
        info = self.info()
        n = self.cfg["max_seq"] * self.cfg["max_batch"] * info["vocab"]
        out = np.zeros(n, np.float32)
        L.check(self.lib.nl_decoder_logits(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                           n))
        return out.reshape(self.cfg["max_seq"], self.cfg["max_batch"], info["vocab"])

    def close(self):
        if self.h:
            self.lib.nl_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
