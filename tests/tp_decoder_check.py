"""One rank of the tensor-parallel decoder parity check (run by torchrun from
tests/test_gpu_decoder_tp.py).  Every rank builds its shard of the same
synthetic decoder, the ranks decode together over NCCL, and rank 0 checks
the tokens and the gathered logits against the CPU model
(oracle/nl_oracle_decoder.c) with the bars of the single-GPU decoder tests."""
import datetime
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(ROOT, "nelisp-gpu_b200")]

CFG = dict(hidden=512, layers=2, heads=8, kv_heads=4, head_dim=64, ffn=1024, vocab=1001,
           rms_eps=1e-5, rope_base=10000.0, seed=29)
# The BitNet-2B layer shapes on 2 layers: at 4 and 8 ranks the 20 KV heads,
# the 54 FFN blocks of 128 and the 5003 vocabulary rows split unevenly
# (TP 8: heads 3,3,3,3,2,2,2,2; FFN 896 on rank 0).
CFG20 = dict(hidden=2560, layers=2, heads=20, kv_heads=20, head_dim=128, ffn=6912, vocab=5003,
             rms_eps=1e-5, rope_base=10000.0, seed=31)
# Five heads of 128 and 11 FFN blocks: at 2 ranks heads 3,2 and FFN 768,640,
# the uneven split of 8 ranks on the 20-head model, on two GPUs.
CFG5 = dict(hidden=640, layers=2, heads=5, kv_heads=5, head_dim=128, ffn=1408, vocab=1003,
            rms_eps=1e-5, rope_base=10000.0, seed=37)


def peer_timeout(ws, rank, local):
    """Rank 1 decodes 2 steps, rank 0 asks for 6: rank 0's peer waits for the
    steps rank 1 never runs give up (bounded, about 0.4 s), its generate
    reports the error, and its context stays usable."""
    import torch
    import torch.distributed as dist
    from nelisp_cuda import NlError, dev
    from nelisp_cuda.decoder import Decoder, nccl_unique_id
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    prompt = np.array([[3, 14, 15]])
    dec = Decoder(CFG, max_batch=1, max_seq=16, tp_rank=rank, tp_size=ws, nccl_id=obj[0],
                  device=local)
    dec.generate(prompt, 2)                      # both ranks: a complete generation
    ok = True
    try:
        dec.generate(prompt, 6 if rank == 0 else 2)
        if rank == 0:
            print("no error reported", flush=True)
            ok = False
    except NlError as e:
        if rank != 0 or "timed out" not in str(e):
            print("unexpected error", rank, e, flush=True)
            ok = False
    dec.close()
    # the context still works: one small GEMV against the oracle
    import oracle as nlo
    rng = np.random.default_rng(1)
    out, cols = 64, 256
    t = rng.integers(-1, 2, size=(out, cols))
    codes = np.where(t == 1, 1, np.where(t == -1, 3, 0)).astype(np.uint32)
    wp = np.zeros((out, cols // 16), np.uint32)
    for f in range(16):
        wp |= codes[:, f::16] << np.uint32(2 * f)
    x = rng.standard_normal(cols).astype(np.float32)
    s = rng.uniform(0.5, 1.5, out).astype(np.float32)
    d = torch.device("cuda", local)
    ty = torch.empty(out, device=d)
    dev.ternary_gemv(torch.from_numpy(x).to(d), torch.from_numpy(wp.ravel().view(np.int32)).to(d),
                     torch.from_numpy(s).to(d), ty, 1, out, cols)
    torch.cuda.synchronize()
    if not nlo.tk_err(ty.cpu().numpy(), nlo.ternary_gemv_rows(x, wp.ravel(), s, 1, out, cols)) < 1e-5:
        print("context unusable after the timeout", rank, flush=True)
        ok = False
    flags = [None] * ws
    dist.all_gather_object(flags, ok)
    if rank == 0:
        print("TIMEOUT_OK" if all(flags) else "TIMEOUT_FAIL", ws, flush=True)
    dist.destroy_process_group()
    return 0 if all(flags) else 1


def main():
    import torch
    import torch.distributed as dist
    ws, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    if "--peer-timeout" in sys.argv:
        return peer_timeout(ws, rank, local)
    from nelisp_cuda.decoder import Decoder, nccl_unique_id
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    cfg = CFG5 if "--uneven" in sys.argv else (CFG if ws <= 2 else CFG20)
    rng = np.random.default_rng(5)
    B, P, steps, max_seq = 2, 5, 6, 16
    prompt = rng.integers(0, cfg["vocab"], size=(B, P))
    dec = Decoder(cfg, max_batch=B, max_seq=max_seq, tp_rank=rank, tp_size=ws,
                  nccl_id=obj[0], keep_logits=True, device=local)
    toks, _, _ = dec.generate(prompt, steps)
    info = dec.info()
    lg = dec.logits()
    dec.close()
    # The same decoder built from uploaded full tensors (each rank copies its
    # shard out of them): this rank's logits must be the same bits.
    import ctypes

    import oracle as nlo
    from nelisp_cuda import _lib as L
    from nelisp_cuda.decoder import LAYER_TENSORS
    lib = L.load()
    full_cfg = dict(cfg, max_batch=B, max_seq=max_seq)
    handles = []

    def up(a):
        h = ctypes.c_uint32()
        a = np.ascontiguousarray(a)
        L.check(lib.nl_upload(a.ctypes.data, a.size, ctypes.byref(h)))
        handles.append(h.value)
        return h.value

    w = {n: [up(nlo.decoder_tensor(full_cfg, l, n)) for l in range(cfg["layers"])]
         for n in LAYER_TENSORS}
    w["embed"] = up(nlo.decoder_tensor(full_cfg, 0, "embed"))
    w["final_norm"] = up(nlo.decoder_tensor(full_cfg, 0, "final_norm"))
    # a communicator of its own: an NCCL unique id serves one initialisation
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    dec = Decoder(cfg, max_batch=B, max_seq=max_seq, tp_rank=rank, tp_size=ws,
                  nccl_id=obj[0], keep_logits=True, device=local, weights=w)
    for h in handles:
        lib.nl_free(h)
    toks_w, _, _ = dec.generate(prompt, steps)
    lg_w = dec.logits()
    dec.close()
    same_w = bool(np.array_equal(toks_w, toks) and
                  np.array_equal(lg_w[:P + steps - 1].view(np.uint32),
                                 lg[:P + steps - 1].view(np.uint32)))
    parts = [None] * ws
    dist.all_gather_object(parts, (info["vocab_begin"], lg, toks, same_w))
    ok = True
    if rank == 0:
        if not all(p[3] for p in parts):
            print("decoder from uploaded weights differs", [p[3] for p in parts], flush=True)
            ok = False
        want_t, want_lg = nlo.decoder_generate(dict(cfg, max_batch=B, max_seq=max_seq), prompt,
                                               steps, keep_logits=True)
        parts.sort(key=lambda p: p[0])
        full = np.concatenate([p[1] for p in parts], axis=2)
        for p in range(P + steps - 1):
            for b in range(B):
                err = nlo.tk_err(full[p, b], want_lg[p, b])
                if not err < 1e-4:
                    print("logits", p, b, err, flush=True)
                    ok = False
        for r in range(ws):
            if not np.array_equal(parts[r][2], parts[0][2]):
                print("ranks disagree on tokens", r, flush=True)
                ok = False
        for b in range(B):
            for i in range(steps):
                row = want_lg[P - 1 + i, b]
                top2 = np.sort(row)[-2:]
                if top2[1] - top2[0] < 1e-3 * max(1.0, abs(top2[1])):
                    break
                if toks[b, i] != want_t[b, i]:
                    print("token", b, i, toks[b, i], want_t[b, i], flush=True)
                    ok = False
        print("TP_OK" if ok else "TP_FAIL", ws, flush=True)
    flag = torch.tensor([1 if ok else 0], device=torch.device("cuda", local))
    dist.broadcast(flag, src=0)
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
