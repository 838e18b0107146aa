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


def main():
    import torch
    import torch.distributed as dist
    ws, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    from nelisp_cuda.decoder import Decoder, nccl_unique_id
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    rng = np.random.default_rng(5)
    B, P, steps, max_seq = 2, 5, 6, 16
    prompt = rng.integers(0, CFG["vocab"], size=(B, P))
    dec = Decoder(CFG, max_batch=B, max_seq=max_seq, tp_rank=rank, tp_size=ws,
                  nccl_id=obj[0], keep_logits=True, device=local)
    toks, _, _ = dec.generate(prompt, steps)
    info = dec.info()
    lg = dec.logits()
    dec.close()
    parts = [None] * ws
    dist.all_gather_object(parts, (info["vocab_begin"], lg, toks))
    ok = True
    if rank == 0:
        import oracle as nlo
        want_t, want_lg = nlo.decoder_generate(dict(CFG, max_batch=B, max_seq=max_seq), prompt,
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
