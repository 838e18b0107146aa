#!/usr/bin/env python
"""Benchmark of the ternary GEMV hot path.

Workload (one step): 64 independent ternary GEMVs y = diag(s) (W x) with
W 4096x4096 (trits -1/0/+1 each p=1/3, two bits per weight, four per byte,
row-major), s ~ U[0.5, 1.5] per row, x ~ N(0, 1), batch 1 -- 64 distinct
weight copies (271 MB per step, more than the 126 MB L2) so every step
streams its weights from HBM.  All inputs are seeded synthetic data.

Metric: GB/s of algorithmic bytes (packed weights + scales + x + y per GEMV,
4,243,456 B at batch 1), whole job, as a fraction of the measured HBM peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own arithmetic on the host cores: the
C restatement of `ternary-rows' under oracle/ (the reference's own path is
Elisp/SPIR-V/Vulkan and cannot run here), all host threads, bounded samples.
Under torchrun with N>1 each rank runs its own 64 copies (weak scaling; the
path has no exchange step) and the time is the max over ranks; the reference
arm runs on rank 0 only.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "nelisp-gpu_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

BASE = json.load(open(os.path.join(ROOT, "BASELINE.json")))
METRIC = BASE["metric"]
OUT = COLS = 4096
COPIES = 64
# requests in flight beyond the one being waited for in the e2e serving loop
# (measured on B200: depth 3 >= depth 2 > depth 1)
E2E_DEPTH = 3
FALLBACK_HBM_GBS = 6650.0


def gemv_bytes(out, cols, batch):
    """Algorithmic bytes of one GEMV: packed W, per-row s, x and y."""
    return out * cols // 4 + out * 4 + cols * 4 * batch + out * 4 * batch


def gemv_config(batch):
    """The workload description both arms report (so the two lines name the
    same configuration)."""
    return {"workload": "ternary GEMV y=diag(s)(W x), W 4096x4096 2-bit packed, "
                        f"batch {batch}, {COPIES} distinct weight copies per step",
            "out": OUT, "cols": COLS, "batch": batch, "copies_per_step": COPIES,
            "bytes_per_gemv": gemv_bytes(OUT, COLS, batch),
            "l2": "inputs larger than L2 (271 MB of weights per step per GPU)",
            "parallelism": "weak: every rank runs its own copies, no collective"}


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_summary():
    """Per-launch DRAM bytes of the main GEMV kernel from the committed ncu
    summary, if there is one."""
    p = os.path.join(ROOT, "profiles", "ternary_gemv_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except (OSError, ValueError):
            return None
    return None


# ---- distributed plumbing -----------------------------------------------------------

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws):
    if ws <= 1:
        return None
    import datetime

    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return dist


# ---- clocks -------------------------------------------------------------------------

CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        items = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(items) and items[local_rank].isdigit():
            return int(items[local_rank])
    return local_rank


# ---- problem generation (on the device, seeded) ----------------------------------------

def make_weights(torch, copies, out, cols, seed, device):
    """Packed trits, codes 00 (0), 01 (+1), 11 (-1) each with p = 1/3."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    lut = torch.tensor([0, 1, 3], dtype=torch.int64, device=device)
    shifts = (2 * torch.arange(16, device=device, dtype=torch.int64))
    W = torch.empty(copies, out * cols // 16, dtype=torch.int32, device=device)
    for z in range(copies):
        r = torch.randint(0, 3, (out, cols // 16, 16), generator=g, device=device)
        w = (lut[r] << shifts).sum(-1)
        w = torch.where(w >= 2 ** 31, w - 2 ** 32, w)
        W[z] = w.reshape(-1).to(torch.int32)
    S = torch.rand(copies, out, generator=g, device=device) + 0.5
    return W, S


# ---- the GPU arm -------------------------------------------------------------------------

def run_gpu(args):
    import numpy as np
    import torch

    from nelisp_cuda import dev, load
    ws, rank, local = dist_env()
    dist = init_dist(ws)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    lib = load()
    from nelisp_cuda import _lib as L0
    L0.check(lib.nl_init(local))          # the library's context on this rank's GPU
    batch = args.batch
    W, S = make_weights(torch, COPIES, OUT, COLS, 1234 + rank, device)
    g = torch.Generator(device=device)
    g.manual_seed(99 + rank)
    X = torch.randn(COPIES, batch, COLS, generator=g, device=device)
    Y = torch.empty(COPIES, batch, OUT, device=device)
    wsb = COPIES * dev.ternary_workspace_bytes(batch, COLS)
    WS = torch.empty(wsb, dtype=torch.uint8, device=device)

    def step():
        dev.ternary_gemv_batched(COPIES, X, batch * COLS, W, OUT * COLS // 16, S, OUT, Y,
                                 batch * OUT, batch, OUT, COLS, workspace=WS)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def load_for(seconds):
        t_end = time.time() + seconds
        while time.time() < t_end:
            for _ in range(50):
                step()
            torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    if args.profile_run:
        # the capture case for ncu: the same launches, nothing else
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        if rank == 0:
            emit({"profile_run": True, "steps": args.steps})
        return
    # the clock record covers load only: 0.5 s before the timed region, the
    # region itself and 1 s after it, all running this same step
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    load_for(0.5)
    n0 = dev.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    barrier()
    n1 = dev.launch_count()
    ms = e0.elapsed_time(e1) / args.steps
    load_for(1.0)
    clocks = sampler.stop()
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    per_gemv = gemv_bytes(OUT, COLS, batch)
    step_bytes = COPIES * per_gemv
    value = ws * step_bytes / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9        # this rank's launches, prep included

    # single-GEMV device time: 50 launches on one copy captured in a CUDA graph
    # and replayed, so host submission does not enter (the 4 MB of weights
    # stay in L2: a latency figure, not the bandwidth headline)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            dev.ternary_gemv(X[0].reshape(-1), W[0], S[0], Y[0].reshape(-1), batch, OUT, COLS,
                             workspace=WS)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        for _ in range(50):
            dev.ternary_gemv(X[0].reshape(-1), W[0], S[0], Y[0].reshape(-1), batch, OUT, COLS,
                             workspace=WS)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    single_us = 1e3 * a.elapsed_time(b) / 50
    del graph

    # other batch sizes of the config, same 64 copies
    batches = {}
    for bb in ([4, 16] if batch == 1 else []):
        Xb = torch.randn(COPIES, bb, COLS, generator=g, device=device)
        Yb = torch.empty(COPIES, bb, OUT, device=device)
        WSb = torch.empty(COPIES * dev.ternary_workspace_bytes(bb, COLS), dtype=torch.uint8,
                          device=device)

        def stepb():
            dev.ternary_gemv_batched(COPIES, Xb, bb * COLS, W, OUT * COLS // 16, S, OUT, Yb,
                                     bb * OUT, bb, OUT, COLS, workspace=WSb)
        for _ in range(3):
            stepb()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            stepb()
        b.record()
        torch.cuda.synchronize()
        msb = a.elapsed_time(b) / args.steps
        gbs = COPIES * gemv_bytes(OUT, COLS, bb) / (msb * 1e-3) / 1e9
        batches[str(bb)] = {"GB/s": round(gbs, 1), "frac": round(gbs / peak, 4),
                            "ms_per_step": round(msb, 4)}
        del Xb, Yb, WSb

    # e2e: through the C ABI with host buffers -- weights resident (uploaded
    # once, as a client of the server uploads them), every step copies its
    # own activations in from pinned memory and reads its outputs back.  A
    # serving loop: E2E_DEPTH + 1 host buffer pairs, request i waited for
    # after request i + E2E_DEPTH is submitted, so the steps' copies overlap
    # the other steps' kernels; the serial form (submit, wait) is reported
    # beside it.
    import ctypes
    from nelisp_cuda import _lib as L
    hw, hs = ctypes.c_uint32(), ctypes.c_uint32()
    Wh = W.cpu().numpy().view(np.uint32)
    Sh = S.cpu().numpy()
    L.check(lib.nl_upload(Wh.ctypes.data, Wh.size, ctypes.byref(hw)))
    L.check(lib.nl_upload(Sh.ctypes.data, Sh.size, ctypes.byref(hs)))
    ptr = {}
    for name, h in (("w", hw), ("s", hs)):
        p, n = ctypes.c_void_p(), ctypes.c_uint32()
        L.check(lib.nl_resident_info(h.value, ctypes.byref(p), ctypes.byref(n)))
        ptr[name] = p.value
    nx, ny = COPIES * batch * COLS, COPIES * batch * OUT
    Xps = [X.cpu().pin_memory() for _ in range(E2E_DEPTH + 1)]
    Yps = [torch.full((ny,), float("nan"), dtype=torch.float32).pin_memory()
           for _ in range(E2E_DEPTH + 1)]

    def submit(i):
        t = ctypes.c_uint64()
        L.check(lib.nl_ternary_gemv_host_submit(
            COPIES, Xps[i % len(Xps)].data_ptr(), batch * COLS, ptr["w"], OUT * COLS // 16,
            ptr["s"], OUT, Yps[i % len(Yps)].data_ptr(), batch * OUT, batch, OUT, COLS,
            ctypes.byref(t)))
        return t.value

    def e2e_run(steps, overlap):
        depth = E2E_DEPTH if overlap else 0
        pending = []
        for i in range(steps):
            pending.append(submit(i))
            if len(pending) > depth:
                L.check(lib.nl_host_wait(pending.pop(0)))
        for t in pending:
            L.check(lib.nl_host_wait(t))

    # host-timed: enough steps that a few microseconds of host jitter per
    # call average out (the device-timed region above uses --steps)
    E2E_STEPS = max(args.steps, 200)

    def e2e_time(overlap):
        e2e_run(max(args.warmup, 10), overlap)     # allocates all 8 staging slots
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        e2e_run(E2E_STEPS, overlap)
        sec = (time.perf_counter() - t0) / E2E_STEPS
        if dist:
            t = torch.tensor([sec], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t.item())
        return sec

    e2e_serial_s = e2e_time(False)
    e2e_s = e2e_time(True)
    e2e_value = ws * step_bytes / e2e_s / 1e9
    e2e_serial = ws * step_bytes / e2e_serial_s / 1e9
    y_dev = Y.reshape(-1).cpu().numpy()
    e2e_ok = all(np.array_equal(Yp.numpy().view(np.uint32), y_dev.view(np.uint32))
                 for Yp in Yps)
    for h in (hw, hs):
        lib.nl_free(h.value)

    # CPU baseline: the oracle port on this box's host cores (rank 0, N = 1)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_baseline(batch, seconds=args.cpu_seconds)

    kernels = None
    if not args.no_kernels:
        kernels = run_kernel_rows(device, peak, rank == 0 and ws == 1 and not args.no_cpu,
                                  with_upload=rank == 0)

    tp_parity = None
    if not args.no_decode:
        tp_parity = tp_parity_check(dist, ws, rank, local)
    decode = None
    if not args.no_decode:
        decode = run_decoder(dist, ws, rank, local, peak)
        decode = {"metric": "ternary-LM decode tok/s (BitNet-b1.58-2B shape, greedy)",
                  "tp": ws, "prompt": PROMPT_LEN, "generated": GEN_STEPS,
                  "data": "synthetic seeded weights and prompt ids", **decode}
        if rank == 0 and ws == 1 and not args.no_cpu:
            decode["cpu_baseline"] = cpu_decode_baseline()

    tr = traffic_summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xint8->int32 (exact ternary x int8-limb activations) + f32 epilogue",
            "data": "synthetic (seeded; trits p=1/3, s~U[0.5,1.5], x~N(0,1))",
            "config": gemv_config(batch),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6650 GB/s",
                         "traffic": (tr or {}).get("bytes_per_launch"),
                         "note": "achieved = algorithmic bytes per step / device time of the "
                                 "step's two launches (prep + tensor-core GEMV)"},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": nx * 4, "d2h_bytes_per_step": ny * 4,
                    "path": "C ABI: nl_ternary_gemv_host_submit + nl_host_wait per step "
                            "(pinned host x in, GEMVs on resident weights, y out; step i "
                            f"waited for after step i+{E2E_DEPTH} is submitted), wall clock",
                    "serial_value": round(e2e_serial, 1),
                    "serial_path": "nl_ternary_gemv_batched_host per step (copy in, GEMVs, "
                                   "copy out, then return)",
                    "matches_device_run": e2e_ok},
            "gpu_launches": int(n1 - n0),
            "clocks": clocks,
            "single_gemv_us": round(single_us, 2),
            "batches": batches,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        if kernels:
            line["kernels"] = kernels
        if decode:
            line["decode"] = decode
        if tp_parity:
            line["tp_parity"] = tp_parity       # last: it stays in a tail of the output
        emit(line)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


PROMPT_LEN, GEN_STEPS = 512, 256


def decode_step_bytes(info, cfg, batch, prompt_len, steps):
    """Bytes one rank streams per decode step, averaged over the STEPS steps:
    its ternary weights and scales, its LM-head rows, and the KV cache read
    by attention (positions 0..p for the step at position p)."""
    H, L, hd = cfg["hidden"], cfg["layers"], cfg["head_dim"]
    avg_ctx = prompt_len + (steps - 1) / 2.0
    kv = 2 * L * batch * avg_ctx * info["kv_heads"] * hd * 4
    return info["weight_bytes"] + kv + batch * H * 4 * 2


def run_decoder(dist, ws, rank, local, peak):
    """ternary-LM decode tok/s at tensor parallelism = ws."""
    import numpy as np
    import torch

    from nelisp_cuda.decoder import BITNET_2B, Decoder, nccl_unique_id
    nid = None
    if ws > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    dec = Decoder(BITNET_2B, max_batch=8, max_seq=PROMPT_LEN + GEN_STEPS, tp_rank=rank,
                  tp_size=ws, nccl_id=nid)
    info = dec.info()
    res = {}
    rng = np.random.default_rng(512)
    for batch in (1, 8):
        prompt = rng.integers(0, BITNET_2B["vocab"], size=(batch, PROMPT_LEN))
        # warm-up at the timed prompt length: the step graph for this prompt,
        # the batched prefill's buffers and its collectives' first use
        dec.generate(prompt, 2)
        toks, pf, dc = dec.generate(prompt, GEN_STEPS)
        t = torch.tensor([pf, dc], device=torch.device("cuda", local))
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pf, dc = float(t[0]), float(t[1])
        step_ms = dc / GEN_STEPS
        nbytes = decode_step_bytes(info, BITNET_2B, batch, PROMPT_LEN, GEN_STEPS)
        gbs = nbytes / (step_ms * 1e-3) / 1e9
        res[f"batch{batch}"] = {
            "tok_s": round(batch * GEN_STEPS / (dc * 1e-3), 1),
            "ms_per_step": round(step_ms, 4),
            "prefill_ms": round(pf, 1),
            "prefill_tok_s": round(batch * (PROMPT_LEN - 1) / (pf * 1e-3), 1),
            "bytes_per_step_per_gpu": int(nbytes),
            "achieved_GBs_per_gpu": round(gbs, 1),
            "frac_of_hbm": round(gbs / peak, 4),
            "tokens_sha256_16": hashlib.sha256(
                np.ascontiguousarray(toks, dtype="<i4").tobytes()).hexdigest()[:16],
        }
    res["kernels_per_step"] = dec.info()["kernels_per_step"]
    res["shard_rank0"] = {k: info[k] for k in ("kv_heads", "ffn", "vocab")}
    dec.close()
    return res


# Tensor-parallel parity: the BitNet-2B layer shapes (20 heads over 20 KV
# heads of 128, FFN 6912) on 2 layers with an odd vocabulary, so that every
# TP size splits heads, FFN blocks and vocabulary rows unevenly where they do
# not divide (TP = 8: heads 3,3,3,3,2,2,2,2; FFN blocks 7 x 6 + 6 x 2).
TP_CHECK_CFG = dict(hidden=2560, layers=2, heads=20, kv_heads=20, head_dim=128, ffn=6912,
                    vocab=5003, rms_eps=1e-5, rope_base=10000.0, seed=29)
TP_TOL = 1e-4        # logits, tk-err per (position, sequence): the decoder tests' bar


def tp_parity_check(dist, ws, rank, local):
    """Every rank builds its shard of the TP_CHECK_CFG decoder; the ranks
    decode together (two runs: a short prompt stepped through the decode
    graph, and a 12-token prompt through the batched prefill), the logits of
    every rank's vocabulary rows are gathered, and rank 0 compares them with
    the CPU model (oracle/nl_oracle_decoder.c) at every position both have.
    Returns the summary on rank 0 (None elsewhere)."""
    import numpy as np

    from nelisp_cuda.decoder import Decoder, nccl_unique_id
    nid = None
    if ws > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    runs = [(2, 5, 6), (3, 12, 4)]            # (batch, prompt, steps)
    max_seq = 16
    rng = np.random.default_rng(77)
    prompts = [rng.integers(0, TP_CHECK_CFG["vocab"], size=(b, p)) for b, p, _ in runs]
    dec = Decoder(TP_CHECK_CFG, max_batch=3, max_seq=max_seq, tp_rank=rank, tp_size=ws,
                  nccl_id=nid, keep_logits=True, device=local)
    info = dec.info()
    mine = []
    for (b, p, steps), prompt in zip(runs, prompts):
        toks, _, _ = dec.generate(prompt, steps)
        mine.append((toks, dec.logits()[:, :b].copy()))
    dec.close()
    parts = [None] * ws
    if dist:
        dist.all_gather_object(parts, (info["vocab_begin"], info["kv_heads"], info["ffn"], mine))
    else:
        parts = [(info["vocab_begin"], info["kv_heads"], info["ffn"], mine)]
    if rank != 0:
        return None
    import oracle as nlo
    nlo.set_threads(host_cores())
    parts.sort(key=lambda q: q[0])
    worst, tokens_equal, ranks_agree, checksum, hashes = 0.0, True, True, 0.0, []
    for i, ((b, p, steps), prompt) in enumerate(zip(runs, prompts)):
        full = np.concatenate([q[3][i][1] for q in parts], axis=2)       # [max_seq, b, vocab]
        toks = parts[0][3][i][0]
        ranks_agree &= all(np.array_equal(q[3][i][0], toks) for q in parts)
        want_t, want_lg = nlo.decoder_generate(dict(TP_CHECK_CFG, max_batch=b, max_seq=max_seq),
                                               prompt, steps, keep_logits=True)
        batched = b * (p - 1) > 16          # positions 0..p-2 ran in the batched prefill
        first = p - 1 if batched else 0
        for pos in range(first, p + steps - 1):
            for bb in range(b):
                worst = max(worst, nlo.tk_err(full[pos, bb], want_lg[pos, bb]))
        checksum += float(np.abs(full[first:p + steps - 1].astype(np.float64)).sum())
        for bb in range(b):
            for j in range(steps):
                top2 = np.sort(want_lg[p - 1 + j, bb])[-2:]
                if top2[1] - top2[0] < 1e-3 * max(1.0, abs(float(top2[1]))):
                    break                    # a near tie: later tokens may differ legitimately
                tokens_equal &= bool(toks[bb, j] == want_t[bb, j])
        hashes.append(hashlib.sha256(np.ascontiguousarray(toks, "<i4").tobytes()).hexdigest()[:16])
    return {"config": "hidden 2560, 2 layers, 20 heads / 20 kv heads x 128, ffn 6912, "
                      "vocab 5003; runs (batch, prompt, steps) = " + str(runs),
            "tp": ws,
            "shards": [{"kv_heads": q[1], "ffn": q[2]} for q in parts],
            "max_tk_err": float(f"{worst:.3e}"), "tol": TP_TOL,
            "tokens_equal": bool(tokens_equal), "ranks_agree": bool(ranks_agree),
            "logits_abs_sum": float(f"{checksum:.9e}"), "tokens_sha256_16": hashes,
            "ok": bool(worst < TP_TOL and tokens_equal and ranks_agree)}


def run_kernel_rows(device, peak, with_cpu, with_upload=True):
    """The other hot-path kernels at BASELINE.json's configs (0, 2, 3):
    f32 matmul 256^3, row softmax 4096x4096 ~ N(0, 4), SwiGLU 16x11008 and
    decode attention (B 8, 32 heads x 128, context 4096), each through the
    registry (nl_dispatch_dev, the reference's kernel names and push
    constants) on device tensors.  Every timed launch is bracketed by its own
    CUDA events after a 256 MB L2 flush (a read, so that no dirty flush data
    is written back during the timed launch), so each reads its inputs from HBM
    (SwiGLU's 2 MB stay L2-sized: reported as such)."""
    import numpy as np
    import torch

    from nelisp_cuda import dev
    g = torch.Generator(device=device)
    g.manual_seed(2026)
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=device)

    def timed(fn, iters=20):
        for _ in range(3):
            fn()
        tot = 0.0
        for _ in range(iters):
            flush.sum()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / iters * 1e-3          # seconds per launch

    def g64(n):
        return (n + 63) // 64

    def cpu_time(fn, reps=1):
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    rows = {}
    if with_cpu:
        import oracle as nlo
        nlo.lib()
    # f32 matmul 256^3; FFMA-bound, latency-bound at this size
    M = K = N = 256
    A = torch.rand(M * K, generator=g, device=device) * 2 - 1
    B = torch.rand(K * N, generator=g, device=device) * 2 - 1
    C = torch.empty(M * N, device=device)
    for name, groups in (("matmul", g64(M * N)), ("matmul-tiled", (M // 16) * (N // 16)),
                         ("matmul-reg", g64(M * N // 16))):
        t = timed(lambda: dev.dispatch(name, [A, B, C], [M, K, N], groups))
        flops = 2.0 * M * N * K
        rows[name + " 256^3"] = {"us": round(t * 1e6, 2), "GFLOP/s": round(flops / t / 1e9, 1),
                                 "bound": "ffma (latency at this size)"}
    ffma_peak = 148 * 128 * 2 * 1.965e9 / 1e9
    rows["matmul 256^3"]["peak_GFLOP/s_nominal"] = round(ffma_peak, 1)
    if with_cpu:
        Ah, Bh = A.cpu().numpy(), B.cpu().numpy()
        tc = cpu_time(lambda: nlo.matmul(Ah, Bh, M, K, N), 3)
        rows["matmul 256^3"]["cpu_GFLOP/s"] = round(2.0 * M * N * K / tc / 1e9, 2)
    del A, B, C
    # row softmax 4096 x 4096, x ~ N(0, 4)
    M = N = 4096
    X = torch.randn(M * N, generator=g, device=device) * 2.0
    Y = torch.empty(M * N, device=device)
    t = timed(lambda: dev.dispatch("softmax", [X, Y], [M, N], g64(M)))
    nbytes = 8 * M * N
    rows["softmax 4096x4096"] = {"us": round(t * 1e6, 2), "GB/s": round(nbytes / t / 1e9, 1),
                                 "frac_of_hbm": round(nbytes / t / 1e9 / peak, 4),
                                 "bytes": nbytes, "bound": "hbm"}
    # back to back over four distinct 64 MB rows sets (512 MB: every launch
    # reads HBM), so one launch's start-up is not charged to each row set
    Xs = [torch.randn(M * N, generator=g, device=device) * 2.0 for _ in range(3)] + [X]
    Ys = [torch.empty(M * N, device=device) for _ in range(3)] + [Y]
    for i in range(4):
        dev.dispatch("softmax", [Xs[i], Ys[i]], [M, N], g64(M))
    torch.cuda.synchronize()
    reps = 40
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(reps):
        dev.dispatch("softmax", [Xs[i % 4], Ys[i % 4]], [M, N], g64(M))
    b.record()
    torch.cuda.synchronize()
    ts = a.elapsed_time(b) * 1e-3 / reps
    rows["softmax 4096x4096"].update({
        "us_stream": round(ts * 1e6, 2), "GB/s_stream": round(nbytes / ts / 1e9, 1),
        "frac_of_hbm_stream": round(nbytes / ts / 1e9 / peak, 4),
        "note": "us: one launch after an L2 flush, launch start-up included; us_stream: "
                "launches back to back over 4 distinct 64 MB inputs"})
    if with_cpu:
        Xh = X.cpu().numpy()
        tc = cpu_time(lambda: nlo.softmax(Xh, M, N))
        rows["softmax 4096x4096"]["cpu_GB/s"] = round(nbytes / tc / 1e9, 2)
    del X, Y, Xs, Ys
    # SwiGLU silu(g) * u on 16 x 11008
    n = 16 * 11008
    Gt, U, O = (torch.randn(n, generator=g, device=device), torch.randn(n, generator=g,
                device=device), torch.empty(n, device=device))
    t = timed(lambda: dev.dispatch("silu-mul", [Gt, U, O], [n], g64(n)))
    nbytes = 12 * n
    rows["silu-mul 16x11008"] = {"us": round(t * 1e6, 2), "GB/s": round(nbytes / t / 1e9, 1),
                                 "bytes": nbytes,
                                 "bound": "latency (2.1 MB: one wave, L2-sized)"}
    if with_cpu:
        gh, uh = Gt.cpu().numpy(), U.cpu().numpy()
        tc = cpu_time(lambda: nlo.silu_mul(gh, uh, n), 5)
        rows["silu-mul 16x11008"]["cpu_GB/s"] = round(nbytes / tc / 1e9, 2)
    del Gt, U, O
    # decode attention: B 8, 32 heads x 128, context 4096 as the
    # configuration states it: RoPE (base 10000) of q and of the new key at
    # position 4095, the append of key and value, softmax attention over the
    # 4096 positions (scale 1/sqrt(128)) -- nl_decode_attn_rope_dev, one
    # pass; the cache holds the earlier keys already rotated
    Bn, H, hd, ctx = 8, 32, 128, 4096
    dim = H * hd
    QKV = torch.randn(Bn * 3 * dim, generator=g, device=device)
    CK = torch.randn(Bn * ctx * dim, generator=g, device=device)
    CV = torch.randn(Bn * ctx * dim, generator=g, device=device)
    POSi = torch.tensor([ctx - 1], dtype=torch.int32, device=device)
    Cq = torch.empty(Bn * dim, device=device)
    t = timed(lambda: dev.decode_attn_rope(QKV, CK, CV, POSi, Cq, Bn, H, H, hd, ctx, 10000.0))
    nbytes = (2 * Bn * (ctx - 1) * dim * 4 + 2 * Bn * dim * 4      # cached K, V read; new row written
              + Bn * 3 * dim * 4 + Bn * dim * 4)                   # q|k|v in, context out
    rows["decode-attn B8 H32 ctx4096 (RoPE q/k + append + attention)"] = {
        "us": round(t * 1e6, 2), "GB/s": round(nbytes / t / 1e9, 1),
        "frac_of_hbm": round(nbytes / t / 1e9 / peak, 4), "bytes": nbytes, "bound": "hbm",
        "entry": "nl_decode_attn_rope_dev"}
    # the registry's decode-attn-b on the same cache (q taken as given)
    POS = torch.tensor([float(ctx - 1)], device=device)
    Q = QKV[:Bn * dim].contiguous()
    t = timed(lambda: dev.dispatch("decode-attn-b", [Q, CK, CV, POS, Cq], [Bn, dim, H, H, ctx],
                                   g64(Bn * dim)))
    nbytes = 2 * Bn * ctx * dim * 4 + 2 * Bn * dim * 4
    rows["decode-attn-b B8 H32 ctx4096"] = {
        "us": round(t * 1e6, 2), "GB/s": round(nbytes / t / 1e9, 1),
        "frac_of_hbm": round(nbytes / t / 1e9 / peak, 4), "bytes": nbytes, "bound": "hbm",
        "entry": "nl_dispatch_dev decode-attn-b (registry op; no RoPE)"}
    if with_cpu:
        Qh, Kh, Vh = Q.cpu().numpy(), CK.cpu().numpy(), CV.cpu().numpy()
        tc = cpu_time(lambda: nlo.decode_attn_b(Qh, Kh, Vh, [float(ctx - 1)], Bn, dim, H, H,
                                                ctx))
        rows["decode-attn-b B8 H32 ctx4096"]["cpu_GB/s"] = round(nbytes / tc / 1e9, 2)
    del Q, QKV, CK, CV, Cq
    # causal prefill attention at the decoder's prefill shape: 512 rows,
    # 20 heads x 128 (f32 on the CUDA cores; FFMA-bound)
    seq, H, hd = PROMPT_LEN, 20, 128
    Qp = torch.randn(seq * H * hd, generator=g, device=device)
    Kp = torch.randn(seq * H * hd, generator=g, device=device)
    Vp = torch.randn(seq * H * hd, generator=g, device=device)
    Cp = torch.empty(seq * H * hd, device=device)
    t = timed(lambda: dev.dispatch("attn-causal-gqa", [Qp, Kp, Vp, Cp], [seq, H, H, hd],
                                   g64(H * seq)))
    flops = 4.0 * hd * H * seq * (seq + 1) / 2
    rows["attn-causal-gqa 512x20x128"] = {
        "us": round(t * 1e6, 2), "TFLOP/s": round(flops / t / 1e12, 2),
        "frac_of_ffma_nominal": round(flops / t / 1e9 / ffma_peak, 4),
        "bound": "ffma (f32, 1e-4 bar)"}
    if with_cpu:
        Qh, Kh, Vh = Qp.cpu().numpy(), Kp.cpu().numpy(), Vp.cpu().numpy()
        tc = cpu_time(lambda: nlo.attn_causal_gqa(Qh, Kh, Vh, seq, H, H, hd))
        rows["attn-causal-gqa 512x20x128"]["cpu_GFLOP/s"] = round(flops / tc / 1e9, 2)
    del Qp, Kp, Vp, Cp, flush
    torch.cuda.empty_cache()
    if with_upload:            # one process reads the disk; the other ranks skip it
        rows.update(upload_rows())
    return rows


def upload_rows():
    """OP_UPLOAD_FILE of a 1 GiB file (the pipelined reader: parallel preads,
    O_DIRECT where the file system takes it, copies overlapping reads) and the
    f32 -> two-bit repacking of a 6912 x 2560 weight matrix from a file."""
    import ctypes
    import os
    import tempfile

    import numpy as np

    from nelisp_cuda import _lib as L
    lib = L.load()
    rows = {}
    d = tempfile.mkdtemp(prefix="nl_upload_")
    try:
        path = os.path.join(d, "weights.bin")
        nbytes = 1 << 30
        blk = np.random.default_rng(3).integers(0, 2 ** 32, size=(16 << 20) // 4,
                                                 dtype=np.uint64).astype(np.uint32).tobytes()
        with open(path, "wb") as f:
            for _ in range(nbytes // len(blk)):
                f.write(blk)
            f.flush()
            os.fsync(f.fileno())
        try:
            fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
            os.close(fd)
            direct = True
        except (OSError, AttributeError):
            direct = False
        h = ctypes.c_uint32()
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            L.check(lib.nl_upload_file(path.encode(), 0, nbytes // 4, ctypes.byref(h)))
            times.append(time.perf_counter() - t0)
            lib.nl_free(h.value)
        t = min(times)
        rows["upload-file 1 GiB"] = {
            "ms": round(t * 1e3, 1), "GB/s": round(nbytes / t / 1e9, 2),
            "o_direct": direct,
            "note": "file -> device through 4 x 16 MiB pinned slots, 4 parallel preads per slot; "
                    "with O_DIRECT the reads bypass the page cache and come from the disk"}
        rws, cls = 6912, 2560
        w = (np.random.default_rng(4).standard_normal((rws, cls)) * 0.02).astype(np.float32)
        wpath = os.path.join(d, "ffn_f32.bin")
        with open(wpath, "wb") as f:
            f.write(w.tobytes())
            os.fsync(f.fileno())
        hw, hs = ctypes.c_uint32(), ctypes.c_uint32()
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            L.check(lib.nl_upload_file_ternary(wpath.encode(), 0, rws, cls, 1, ctypes.byref(hw),
                                               ctypes.byref(hs)))
            times.append(time.perf_counter() - t0)
            lib.nl_free(hw.value)
            lib.nl_free(hs.value)
        t = min(times)
        rows["upload-file-ternary 6912x2560 f32"] = {
            "ms": round(t * 1e3, 2), "GB/s_f32_read": round(w.nbytes / t / 1e9, 2),
            "note": "read the f32 matrix, per-row absmean, quant-w thresholds, pack to 2 bits "
                    "(70.8 MB in, 4.4 MB packed + scales out)"}
    finally:
        for fn in os.listdir(d):
            os.remove(os.path.join(d, fn))
        os.rmdir(d)
    return rows


def cpu_gemv_problems(batch, n_mats=8, seed=1234):
    """N_MATS distinct seeded 4096x4096 problems for the CPU legs (cycled, so
    the weights do not all stay in one core's cache)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    Ws, Ss, Xs = [], [], []
    for _ in range(n_mats):
        t = rng.integers(0, 3, size=(OUT, COLS // 16, 16))
        codes = np.array([0, 1, 3], np.uint32)[t]
        Ws.append((codes << (2 * np.arange(16, dtype=np.uint32))).sum(-1).astype(np.uint32).ravel())
        Ss.append(rng.uniform(0.5, 1.5, OUT).astype(np.float32))
        Xs.append(rng.standard_normal(batch * COLS).astype(np.float32))
    return Ws, Ss, Xs


def cpu_gemv_step(nlo, probs, batch, n_gemv):
    Ws, Ss, Xs = probs
    for i in range(n_gemv):
        z = i % len(Ws)
        nlo.ternary_gemv_rows(Xs[z], Ws[z], Ss[z], batch, OUT, COLS)


def cpu_gemv_calibrate(nlo, probs, batch, step_s=0.25):
    """GEMVs per CPU step for about STEP_S seconds of work (4 .. 64)."""
    t0 = time.perf_counter()
    cpu_gemv_step(nlo, probs, batch, len(probs[0]))
    per = (time.perf_counter() - t0) / len(probs[0])
    return int(min(COPIES, max(4, round(step_s / max(per, 1e-6)))))


def cpu_baseline(batch, seconds=10.0):
    """The oracle's ternary GEMV (restated `ternary-rows' with the row scale
    in every block) on all host threads, over a bounded sample: the same
    steps as the reference arm, repeated for about SECONDS."""
    import oracle as nlo
    nlo.lib()
    nlo.set_threads(host_cores())
    probs = cpu_gemv_problems(batch)
    n_gemv = cpu_gemv_calibrate(nlo, probs, batch)
    cpu_gemv_step(nlo, probs, batch, n_gemv)           # warm-up
    n = 0
    t0 = time.perf_counter()
    while True:
        cpu_gemv_step(nlo, probs, batch, n_gemv)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    per = el / (n * n_gemv)
    return {"value": round(gemv_bytes(OUT, COLS, batch) / per / 1e9, 3), "unit": "GB/s",
            "cores": nlo.threads(), "kind": "port",
            "sample": f"{n * n_gemv} GEMVs 4096x4096 batch {batch} ({n} steps of {n_gemv}) in "
                      f"{el:.1f} s (oracle/nl_oracle.c ternary-rows restatement, OpenMP)"}


def run_decode_profile(args):
    import numpy as np
    import torch

    from nelisp_cuda.decoder import BITNET_2B, Decoder
    torch.cuda.set_device(0)
    dec = Decoder(BITNET_2B, max_batch=8, max_seq=args.prompt + 8, device=0)
    prompt = np.random.default_rng(5).integers(0, BITNET_2B["vocab"],
                                               size=(args.batch, args.prompt))
    toks, pf, dc = dec.generate(prompt, 4)
    emit({"decode_profile": True, "batch": args.batch, "ms_per_step": dc / 4,
                      "kernels_per_step": dec.info()["kernels_per_step"]})
    dec.close()


def run_attn_profile(args):
    """Only the causal prefill attention at the decoder's prefill shape
    (512 rows, 20 heads x 128), warm-up then timed launches: the case ncu
    captures for that kernel."""
    import torch

    from nelisp_cuda import dev, load
    torch.cuda.set_device(0)
    load()
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(7)
    seq, H, hd = PROMPT_LEN, 20, 128
    Q, K, V = (torch.randn(seq * H * hd, generator=g, device=device) for _ in range(3))
    C = torch.empty(seq * H * hd, device=device)
    for _ in range(args.warmup + args.steps):
        dev.dispatch("attn-causal-gqa", [Q, K, V, C], [seq, H, H, hd], (H * seq + 63) // 64)
    torch.cuda.synchronize()
    emit({"attn_profile": True, "launches": args.warmup + args.steps})


def run_softmax_profile(args):
    """Only row-softmax launches at the benchmark's shape (4096 x 4096, x ~
    N(0, 4)), warm-up then timed: the case ncu captures for that kernel."""
    import torch

    from nelisp_cuda import dev, load
    torch.cuda.set_device(0)
    load()
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(11)
    M = N = 4096
    X = torch.randn(M * N, generator=g, device=device) * 2.0
    Y = torch.empty(M * N, device=device)
    for _ in range(args.warmup + args.steps):
        dev.dispatch("softmax", [X, Y], [M, N], (M + 63) // 64)
    torch.cuda.synchronize()
    emit({"softmax_profile": True, "launches": args.warmup + args.steps})


def run_dattn_profile(args):
    """Only the fused decode attention (RoPE of q and k, cache append,
    split-K attention) at the benchmark's shape: batch 8, 32 heads x 128,
    context 4096 -- the case ncu captures for those kernels."""
    import torch

    from nelisp_cuda import dev, load
    torch.cuda.set_device(0)
    load()
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(12)
    Bn, H, hd, ctx = 8, 32, 128, 4096
    dim = H * hd
    QKV = torch.randn(Bn * 3 * dim, generator=g, device=device)
    CK = torch.randn(Bn * ctx * dim, generator=g, device=device)
    CV = torch.randn(Bn * ctx * dim, generator=g, device=device)
    POS = torch.tensor([ctx - 1], dtype=torch.int32, device=device)
    C = torch.empty(Bn * dim, device=device)
    for _ in range(args.warmup + args.steps):
        dev.decode_attn_rope(QKV, CK, CV, POS, C, Bn, H, H, hd, ctx, 10000.0)
    torch.cuda.synchronize()
    emit({"dattn_profile": True, "launches": args.warmup + args.steps})


def run_gemm_profile(args):
    """Only the prefill ternary GEMM (512 rows x 2560 -> 6912, the tcgen05
    path for more than 16 rows), warm-up then timed launches: the case ncu
    captures for that kernel."""
    import torch

    from nelisp_cuda import dev, load
    torch.cuda.set_device(0)
    load()
    device = torch.device("cuda", 0)
    seq, out, cols = PROMPT_LEN, 6912, 2560
    W, S = make_weights(torch, 1, out, cols, 77, device)
    g = torch.Generator(device=device)
    g.manual_seed(8)
    X = torch.randn(seq * cols, generator=g, device=device)
    Y = torch.empty(seq * out, device=device)
    for _ in range(args.warmup + args.steps):
        dev.ternary_gemv(X, W[0], S[0], Y, seq, out, cols)   # library workspace
    torch.cuda.synchronize()
    emit({"gemm_profile": True, "launches": args.warmup + args.steps})


DECODE_CPU_CTX = PROMPT_LEN + GEN_STEPS // 2     # the average context of the 256 steps


def cpu_decode_baseline():
    """The CPU model of the decoder (oracle/nl_oracle_decoder.c) on the full
    configuration at the benchmark's context: batch 1, two greedy positions
    at context 640 (the average over the 256 generated tokens after the
    512-token prompt), the KV cache rows below it filled with seeded values.
    Weight generation is not timed; all host threads."""
    import oracle as nlo
    from nelisp_cuda.decoder import BITNET_2B
    nlo.set_threads(host_cores())
    steps = 2
    cfg = dict(BITNET_2B, max_batch=1, max_seq=DECODE_CPU_CTX + steps)
    sec = nlo.decoder_time_positions(cfg, 1, DECODE_CPU_CTX, steps)
    return {"value": round(steps / sec, 4), "unit": "tok/s", "cores": nlo.threads(),
            "kind": "port",
            "sample": f"batch 1, {steps} decode positions at context {DECODE_CPU_CTX} "
                      f"({sec:.1f} s; the reference's per-output-lane decode-attn-b and "
                      "ternary-rows restated, OpenMP)"}


# ---- the reference arm ----------------------------------------------------------------------

def run_reference(args):
    """The reference's arithmetic for the headline path on the host cores:
    the C restatement of `ternary-rows' (oracle/nl_oracle.c) with the row
    scale in every block, on all the host threads this process may use (set
    explicitly: torchrun exports OMP_NUM_THREADS=1).  A step is a bounded
    sample of the 64-GEMV step, sized to about 0.25 s; rank 0 alone runs."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle as nlo
    nlo.lib()
    nlo.set_threads(host_cores())
    batch = args.batch
    probs = cpu_gemv_problems(batch)
    n_gemv = cpu_gemv_calibrate(nlo, probs, batch)

    def step():
        cpu_gemv_step(nlo, probs, batch, n_gemv)

    for _ in range(args.warmup):
        step()
    # at least the asked-for steps and at least 2 s of work
    t0 = time.perf_counter()
    done = 0
    while done < args.steps or time.perf_counter() - t0 < 2.0:
        step()
        done += 1
    el = time.perf_counter() - t0
    per = el / done
    value = n_gemv * gemv_bytes(OUT, COLS, batch) / per / 1e9
    sample = (f"{n_gemv} of the step's {COPIES} GEMVs per step (4096x4096, batch {batch}), "
              f"{done} steps timed in {el:.1f} s; oracle/nl_oracle.c restatement of "
              "ternary-rows, OpenMP")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": gemv_config(batch),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": nlo.threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's own path (Elisp DSL -> SPIR-V -> Vulkan) cannot run: no "
                "Emacs, no Vulkan loader or ICD (unavailable on this box); this arm times its "
                "algorithm restated in C on the host cores, rank 0 only",
    }
    emit(line)


_RESULT_OUT = None


def emit(obj):
    """The result line: the only thing this program writes to standard output."""
    out = _RESULT_OUT or sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def main():
    global _RESULT_OUT
    # Libraries write to file descriptor 1 too (NCCL's version banner, for
    # one); keep the real standard output for the result line and send
    # everything else to standard error.
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-decode", action="store_true", help="skip the decoder section")
    ap.add_argument("--no-kernels", action="store_true",
                    help="skip the matmul / softmax / SwiGLU / attention rows")
    ap.add_argument("--decode-profile", action="store_true",
                    help="only a short decoder run, batch --batch (the case ncu lists)")
    ap.add_argument("--prompt", type=int, default=4,
                    help="prompt length of --decode-profile (the decode steps' context)")
    ap.add_argument("--profile-run", action="store_true",
                    help="only warm-up and timed steps (the case ncu captures)")
    ap.add_argument("--attn-profile", action="store_true",
                    help="only causal prefill attention launches (the case ncu captures)")
    ap.add_argument("--gemm-profile", action="store_true",
                    help="only prefill ternary GEMM launches (the case ncu captures)")
    ap.add_argument("--softmax-profile", action="store_true",
                    help="only softmax 4096x4096 launches (the case ncu captures)")
    ap.add_argument("--dattn-profile", action="store_true",
                    help="only fused decode-attention launches (the case ncu captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    elif args.decode_profile:
        run_decode_profile(args)
    elif args.attn_profile:
        run_attn_profile(args)
    elif args.gemm_profile:
        run_gemm_profile(args)
    elif args.softmax_profile:
        run_softmax_profile(args)
    elif args.dattn_profile:
        run_dattn_profile(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
