#!/usr/bin/env python
"""Decode throughput of the paged-KV Qwen3-0.6B decoder on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N)

Workload (one step): one greedy decode step of the full 28-layer Qwen3-0.6B decoder
(Q8_0 weights, paged f16 KV cache) for 128 sequences that sit at a 2048-token context
(growing by one token per step): embedding gather, per layer RMSNorm, QKV GEMM,
QK-norm + RoPE + paged append, paged GQA attention, o_proj, SwiGLU MLP, then the
final norm, lm_head with fused argmax and the feedback of the argmax as next input.
Every GPU runs its own 128 streams (independent replicas, weak scaling, no collectives).

Prints one JSON line. `value` = whole-job decode tokens/s timed on the device (CUDA
events around exactly K steps, inputs resident in HBM, max over ranks); `e2e` = the same
through fa_decode_step with host token ids in and next ids out every step.
The KV cache read per step is ~30 GB, far larger than L2, so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "funasr-ggml_b200"))

import fa_multi  # noqa: E402
import fa_synth  # noqa: E402

METRIC = "decode tokens/s per GPU (bs128, 2k ctx) at 1/2/4/8 B200; paged-attn HBM GB/s"
KV_BYTES_PER_TOKEN_LAYER = 8 * 2 * 128 * 2     # K+V of 8 heads x 128 dims, f16


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--e2e-steps", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--no-pdl", action="store_true", help="plain stream order between kernels")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "attention", "gemm", "prefill", "serve", "pipeline", "append"],
                    help="attention: kernel (2) alone over one layer's pages at the same batch and context; "
                         "gemm: the decode step's weight GEMMs alone; prefill: batched chunked prefill of "
                         "16 utterances then 64 greedy tokens each; serve: continuous batching of --streams "
                         "streams with Poisson arrivals; pipeline: one 5 s utterance through the encoder, "
                         "adaptor, prefill and 32 greedy tokens; append: the paged KV append + gather of "
                         "32 sequences over 28 layers")
    ap.add_argument("--append-layers", type=int, default=28,
                    help="append: layers in the pool (28 is the workload; fewer only for small profiler captures)")
    ap.add_argument("--streams", type=int, default=1024, help="serve: streams over all GPUs")
    ap.add_argument("--arrival-rate", type=float, default=100.0, help="serve: streams per second (Poisson)")
    ap.add_argument("--kv-gb", type=float, default=160.0, help="serve: page pool per GPU, GB")
    ap.add_argument("--serve-seconds", type=float, default=60.0, help="serve: wall-clock budget of the timed run")
    ap.add_argument("--serve-rows", type=int, default=4096,
                    help="serve: rows per forward (decode rows + prompt chunks); 1024 / 2048 / 4096 gave 10.4 / "
                         "12.0 / 12.7 k generated tokens/s")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- CPU baseline --
def cpu_oracle_sample(cfg, w, ctx, budget_s, rows=2, seed=0, max_new=1024):
    """Oracle decode steps (ggml-CPU arithmetic: Q8_0 activations) for `rows` sequences
    at `ctx` tokens of synthetic cache, repeated for about budget_s seconds (at most
    max_new tokens per sequence)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    # all host threads (torchrun sets OMP_NUM_THREADS=1 for its workers)
    oracle.set_num_threads(len(os.sched_getaffinity(0)))
    pages = (ctx + max_new + 15) // 16
    od = oracle.OracleDecoder(cfg, w, n_pages=rows * pages, max_seqs=rows, max_pages_per_seq=pages,
                              max_pos=ctx + max_new, mode=oracle.MODE_GGML_CPU)
    rng = np.random.default_rng(seed)
    for s in range(rows):
        od.seq_open(s)
        od._reserve(s, ctx)
        od.seq_len[s] = ctx
    L = od.pool.shape[0]
    for l in range(L):
        od.pool[l] = oracle.f32_to_f16_bits(rng.uniform(-2, 2, od.pool.shape[1:]).astype(np.float32))
    toks = rng.integers(0, cfg["vocab"], rows)
    n_tok, t0 = 0, time.perf_counter()
    while True:
        _, nxt = od.forward(list(range(rows)), tokens=toks, want_logits=False)
        toks = nxt
        n_tok += rows
        el = time.perf_counter() - t0
        if el >= budget_s or od.seq_len[0] >= ctx + max_new - 1:
            break
    return n_tok / el, oracle.num_threads(), n_tok, el


# ------------------------------------------------------------------- ours --
def run_ours(a):
    rank, local, world = fa_multi.init("nccl")
    import torch
    torch.cuda.set_device(local)
    import fa_dec

    cfg = fa_synth.QWEN3_06B
    B, ctx, K, W, E = a.batch, a.ctx, a.steps, a.warmup, a.e2e_steps
    w = fa_synth.make_weights(cfg, seed=1)
    total_new = W + K + 2 + E + 1
    max_ctx = (ctx + total_new + 31) // 16 * 16
    pages_per_seq = max_ctx // 16
    dec = fa_dec.Decoder(local, **fa_synth.decoder_desc(cfg, max_ctx=max_ctx, n_pages=B * pages_per_seq + 16,
                                                        max_seqs=B, max_rows=B))
    dec.load_weights(w)
    if a.no_pdl:
        dec.set_pdl(False)
    sids = [dec.seq_open(max_ctx) for _ in range(B)]
    for i, s in enumerate(sids):
        dec.kv_fill_synthetic(s, ctx, seed=rank * 100003 + i)
    rng = np.random.default_rng(rank)
    toks = rng.integers(0, cfg["vocab"], B)

    dec.profile(True)
    ids, _ = dec.generate(sids, toks, W)
    toks = ids[-1]
    sampler = ClockSampler(local)
    torch.cuda.synchronize()
    fa_multi.barrier()
    sampler.start()
    ids, dev_ms = dec.generate(sids, toks, K)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    fa_multi.barrier()
    attn_ms, n_att = dec.profile_attention()
    row_ms = dec.profile_row_step()
    launches = dec.step_launches()
    dec.profile(False)
    max_ms = fa_multi.reduce(dev_ms, "max")
    value = B * K * world / (max_ms / 1e3)

    # attention roofline of the last timed step: every row at ctx + W + K tokens
    n_kv_last = ctx + W + K
    att_bytes = B * n_kv_last * KV_BYTES_PER_TOKEN_LAYER
    att_launch_ms = attn_ms / max(n_att, 1)
    achieved = att_bytes / (att_launch_ms / 1e3) / 1e9 if att_launch_ms > 0 else None
    peak, peak_kind = measured_peaks()
    traffic = None
    tf = os.path.join(ROOT, "profiles", "attention_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            t = json.load(f)
        # bytes scale with the (row, token) pairs read per launch
        traffic = t["dram_bytes_per_launch"] * (B * n_kv_last) / (t["rows"] * t["n_kv"])

    kernel, bytes_per_launch, ms_per_launch = "paged_attn_kernel (+ split merge)", att_bytes, att_launch_ms
    # what one step reads: every layer's Q8_0 weights (q and scale planes, 34 B per 32
    # weights), the lm_head, and the rows' K/V
    wq = sum(n * k for n, k in ((4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072)))
    step_bytes = (cfg["n_layers"] * (wq * 34 // 32 + B * (ctx + W) * KV_BYTES_PER_TOKEN_LAYER)
                  + cfg["vocab"] * cfg["hidden"] * 34 // 32)
    if row_ms > 0:
        # one row: the persistent step kernel is the step; its algorithmic bytes are every
        # layer's Q8_0 weights (q and row-major scale planes, 34 B per 32 weights) and the
        # row's K/V pages, each read once
        bytes_per_launch = cfg["n_layers"] * (wq * 34 // 32 + B * n_kv_last * KV_BYTES_PER_TOKEN_LAYER)
        kernel = "row_step_kernel (one-row step: 28 layers, persistent)"
        if launches == 1:   # the lm_head runs in the kernel too
            bytes_per_launch += cfg["vocab"] * cfg["hidden"] * 34 // 32
            kernel = "row_step_kernel (one-row step: 28 layers + lm_head + argmax, persistent)"
        ms_per_launch = row_ms
        achieved = bytes_per_launch / (row_ms / 1e3) / 1e9
        traffic = None
        tf = os.path.join(ROOT, "profiles", "row_step_traffic.json")
        if os.path.exists(tf):
            with open(tf) as f:
                traffic = json.load(f)["dram_bytes_per_launch"]

    # e2e through the public step call, host ids in and out every step
    toks = ids[-1]
    for _ in range(2):
        toks, _ = dec.decode_step(sids, toks)
    torch.cuda.synchronize()
    fa_multi.barrier()
    t0 = time.perf_counter()
    for _ in range(E):
        toks, _ = dec.decode_step(sids, toks)
    e2e_s = time.perf_counter() - t0
    fa_multi.barrier()
    e2e_s = fa_multi.reduce(e2e_s, "max")
    e2e_value = B * E * world / e2e_s
    all_clocks = fa_multi.gather(clocks)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        v, cores, n_tok, el = cpu_oracle_sample(cfg, w, ctx, a.cpu_budget_s)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{n_tok} decode tokens (2 sequences at {ctx}-token synthetic context, full 28-layer "
                         f"model, ggml-CPU arithmetic) in {el:.1f} s; CPU restatement of the reference "
                         f"(ggml unavailable)"}
    dec.close()
    if rank == 0:
        c0 = all_clocks[0]
        reasons = sorted(set(r for c in all_clocks for r in c.get("reasons", [])))
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": max_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic: seeded random-init Q8_0 Qwen3-0.6B weights, synthetic f16 KV cache, random first tokens",
            "config": {"workload": f"steady-state paged GQA decode, {B} sequences per GPU at {ctx}-token context "
                                   f"(grows to {ctx + W + K}), Qwen3-0.6B 28 layers 16q/8kv x 128, Q8_0 weights, f16 KV",
                       "batch_per_gpu": B, "ctx": ctx, "page_tokens": 16,
                       "l2": f"no flush: each step reads {step_bytes / 1e9:.2f} GB (weights, lm_head, K/V), "
                             f"above the 126 MB L2",
                       "parallelism": f"independent replicas x{world}, no collectives"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak if achieved else None, "traffic": traffic,
                         "kernel": kernel, "peak_kind": peak_kind,
                         "bytes_per_launch": bytes_per_launch, "ms_per_launch": ms_per_launch},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": B * 12,
                    "d2h_bytes_per_step": B * 4 + 4, "steps": E},
            "gpu_launches": launches * K,
            "clocks": {"sm_mhz": c0.get("sm_mhz"), "sm_max_mhz": c0.get("sm_max_mhz"), "reasons": reasons},
        }
        print(json.dumps(line), flush=True)
    fa_multi.shutdown()


# ------------------------------------------------------ attention alone --
def run_attention(a):
    """Paged GQA decode attention (plus its split combine) of one layer on its own:
    B rows at `ctx` tokens, two page pools used alternately (each ~1 GB at B=128,
    ctx 2048, so nothing stays in L2 between launches), the decoder's split choice,
    f16 hi/lo output as the decoder writes it. Prints the achieved HBM GB/s."""
    import torch
    import fa_dec

    rank, local, world = fa_multi.init("nccl")
    torch.cuda.set_device(local)
    B, ctx, K, W = a.batch, a.ctx, a.steps, a.warmup
    n_kv = np.full(B, ctx, np.int32)
    pages = (ctx + 15) // 16
    n_pages = B * pages
    rng = np.random.default_rng(rank)
    dev = torch.device("cuda", local)
    pools = [torch.randn(n_pages * 8 * 2 * 16 * 128, dtype=torch.float16, device=dev).view(torch.int16)
             for _ in range(2)]
    bts = [torch.from_numpy(rng.permutation(n_pages).reshape(B, pages).astype(np.int32)).to(dev) for _ in range(2)]
    q = (torch.randn(B, 16, 128, device=dev) * 0.3).contiguous()
    pos = torch.from_numpy(n_kv - 1).to(dev)
    slot = torch.arange(B, dtype=torch.int32, device=dev)
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    pps, n_splits = fa_dec.op_attention_plan(n_kv, n_sm)
    scratch = torch.empty(max(fa_dec.op_attention_scratch_bytes(B, n_splits), 16), dtype=torch.uint8, device=dev)
    out16 = torch.empty(B, 2048, dtype=torch.int16, device=dev)
    out_lo = torch.empty_like(out16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def launch(i):
        fa_dec.op_paged_attention(q.data_ptr(), B, pos.data_ptr(), slot.data_ptr(), bts[i % 2].data_ptr(), pages,
                                  n_pages, pools[i % 2].data_ptr(), pps, n_splits, scratch.data_ptr(),
                                  out16=out16.data_ptr(), out16_lo=out_lo.data_ptr(), err=err.data_ptr(),
                                  stream=stream)

    for i in range(W):
        launch(i)
    torch.cuda.synchronize()
    fa_multi.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        launch(i)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    fa_multi.barrier()
    assert int(err.item()) == 0, "attention reported a device error"
    ms = fa_multi.reduce(e0.elapsed_time(e1), "max")
    bytes_per_launch = B * ctx * KV_BYTES_PER_TOKEN_LAYER
    gbs = bytes_per_launch * K * world / (ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    all_clocks = fa_multi.gather(clocks)
    if rank == 0:
        reasons = sorted(set(r for c in all_clocks for r in c.get("reasons", [])))
        print(json.dumps({
            "metric": "paged-attn HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic: N(0,1) f16 pages, random block tables",
            "config": {"workload": f"paged GQA decode attention of one layer, {B} rows at {ctx} tokens, "
                                   f"16q/8kv x 128, f16 pages of 16 tokens", "batch_per_gpu": B, "ctx": ctx,
                       "pages_per_split": pps, "n_splits": n_splits,
                       "l2": "no flush: two ~1 GB page pools used alternately"},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak, "peak_kind": peak_kind, "bytes_per_launch": bytes_per_launch},
            "gpu_launches": K * (2 if n_splits > 1 else 1),
            "clocks": {"sm_mhz": all_clocks[0].get("sm_mhz"), "sm_max_mhz": all_clocks[0].get("sm_max_mhz"),
                       "reasons": reasons},
        }), flush=True)
    fa_multi.shutdown()


# ---------------------------------------------------------- GEMMs alone --
def run_gemm(a):
    """The weight GEMMs of one decode step on their own: for each of the 28 layers the
    QKV (4096 x 1024), o_proj (1024 x 2048), gate/up (6144 x 1024) and down (1024 x 3072)
    GEMMs, then lm_head (151936 x 1024) with its argmax, all at M = batch rows, with
    each layer's own Q8_0 weights in the decoder's plane form (0.633 GB of q and scales
    read per step, so weights come from HBM as in the decoder) and the decoder's split-K
    choice. Prints the weight-read GB/s (algorithmic: 34 B per 32 weights)."""
    import torch
    import fa_dec

    rank, local, world = fa_multi.init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = fa_synth.QWEN3_06B
    M, K, W = a.batch, a.steps, a.warmup
    H, F, V, L = cfg["hidden"], cfg["ffn"], cfg["vocab"], cfg["n_layers"]
    shapes = [("qkv", 4096, H), ("o", H, 2048), ("gate_up", 2 * F, H), ("down", H, F)]
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    splits = {nm: fa_dec.op_gemm_plan(M, n, k, 0, n_sm) for nm, n, k in shapes}
    def planes(n, k):
        """Q8_0 planes: q int8 [n][k], scales f16 [k/32][n] and [n][k/32] ~U(0.001, 0.02)."""
        buf = torch.empty(fa_dec.op_q8_planes_bytes(n, k), dtype=torch.uint8, device=dev)
        buf[:n * k].view(torch.int8).copy_(torch.randint(-127, 128, (n * k,), dtype=torch.int8, device=dev))
        d = (torch.rand(k // 32, n, device=dev) * 0.019 + 0.001).half()
        nd = n * k // 32
        buf[n * k:n * k + 2 * nd].view(torch.float16).copy_(d.reshape(-1))
        buf[n * k + 2 * nd:].view(torch.float16).copy_(d.t().contiguous().reshape(-1))
        return buf

    weights = [{nm: planes(n, k) for nm, n, k in shapes} for _ in range(L)]
    lm = planes(V, H)
    a_hi = (torch.randn(M, max(F, 2048), device=dev)).half()
    a_lo = (torch.randn(M, max(F, 2048), device=dev) * 1e-4).half()
    part = torch.empty(max(splits.values()) * M * 2 * F, dtype=torch.float32, device=dev)
    am_scr = torch.zeros(fa_dec.op_argmax_scratch_bytes(M, V), dtype=torch.uint8, device=dev)
    nxt = torch.empty(M, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def step():
        for l in range(L):
            for nm, n, k in shapes:
                fa_dec.op_q8p_gemm(a_hi.data_ptr(), a_lo.data_ptr(), M, k, weights[l][nm].data_ptr(), n,
                                   splits[nm], part.data_ptr(), 0, stream)
        fa_dec.op_q8p_gemm_argmax(a_hi.data_ptr(), a_lo.data_ptr(), M, H, lm.data_ptr(), V, am_scr.data_ptr(),
                                  nxt.data_ptr(), 0, 0, stream)

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    fa_multi.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = fa_multi.reduce(e0.elapsed_time(e1), "max") / K
    wbytes = (sum(n * k for _, n, k in shapes) * L + V * H) * 34 // 32
    gbs = wbytes / (ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "decode-step weight GEMMs, weight-read GB/s", "value": gbs * world, "unit": "GB/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 x f16 pair (exact d*q, fp32 sums)",
            "data": "synthetic: random Q8_0 weights (scales U(0.001, 0.02)) and activations",
            "config": {"workload": f"{L} layers x (QKV, o_proj, gate/up, down) + lm_head with argmax at M={M}",
                       "splits": splits, "weight_bytes": wbytes,
                       "l2": "no flush: 0.63 GB of distinct Q8_0 weights per step"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "peak_kind": peak_kind},
            "gpu_launches": K * (4 * L + 2),
            "clocks": clocks,
        }), flush=True)
    fa_multi.shutdown()


# ------------------------------------------------------ batched prefill --
def run_prefill(a):
    """Batched chunked prefill (16 utterances of 3-15 s): the utterances' LFR frames
    (49-249 each, stand-in values) go through the SANM encoder and adaptor in batches of
    <= 1024 frames, each utterance's embeddings are prefixed with 30 prompt-token
    embeddings, the rows are packed into forward calls of at most 512 rows, then 64
    greedy decode tokens per stream. Times the whole job on the host clock, after an
    identical warm-up job on other sequences (so every step shape has its graph)."""
    import torch
    import fa_dec

    rank, local, world = fa_multi.init("nccl")
    torch.cuda.set_device(local)
    cfg = fa_synth.QWEN3_06B
    w = fa_synth.make_weights(cfg, seed=1)
    H = cfg["hidden"]
    emb_table = w["llm.model.embed_tokens.weight"][2].reshape(cfg["vocab"], H)
    rng = np.random.default_rng(100 + rank)
    prompts, lfrs = [], []
    for _ in range(16):
        frames = int(rng.uniform(3.0, 15.0) * 100) - 2
        T = (frames + 5) // 6
        ids = rng.integers(0, cfg["vocab"], 30)
        prompts.append((emb_table[ids].astype(np.uint32) << 16).view(np.float32))
        lfrs.append(fa_synth.lfr_features(rng, T))
    enc = fa_dec.Encoder(local, max_frames=1024)
    enc.load_weights(fa_synth.make_encoder_weights(seed=2))
    streams = []

    def encode():
        audio, group, n = [], [], 0
        for x in lfrs:
            if n + len(x) > 1024:
                audio += enc.forward_batch(group)
                group, n = [], 0
            group.append(x)
            n += len(x)
        audio += enc.forward_batch(group)
        return [np.ascontiguousarray(np.concatenate([p, au]), np.float32) for p, au in zip(prompts, audio)]
    chunk, n_new = 512, 64
    max_ctx = 512 + n_new + 16
    dec = fa_dec.Decoder(local, **fa_synth.decoder_desc(cfg, max_ctx=max_ctx, n_pages=2 * 16 * (max_ctx // 16 + 1),
                                                        max_seqs=32, max_rows=chunk))
    dec.load_weights(w)

    timing = {}

    def job():
        torch.cuda.synchronize()
        te = time.perf_counter()
        streams[:] = encode()
        timing["encoder_ms"] = (time.perf_counter() - te) * 1e3
        sids = [dec.seq_open(max_ctx) for _ in streams]
        calls, rows, embs, firsts = [], [], [], {}
        for s, e in zip(sids, streams):
            if len(rows) + len(e) > chunk:
                calls.append((rows, np.concatenate(embs)))
                rows, embs = [], []
            rows = rows + [s] * len(e)
            embs.append(e)
        calls.append((rows, np.concatenate(embs)))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for rows, e in calls:
            ends = {}
            for i, s in enumerate(rows):
                ends[s] = i
            # only each stream's last row goes through lm_head
            nxt, _ = dec.forward_rows(rows, list(ends.values()), embeds=e)
            for s, v in zip(ends.keys(), nxt):
                firsts[s] = int(v)
        t1 = time.perf_counter()
        ids, dev_ms = dec.generate(sids, [firsts[s] for s in sids], n_new)
        t2 = time.perf_counter()
        for s in sids:
            dec.seq_close(s)
        return t1 - t0, t2 - t1, dev_ms, len(calls)

    job()
    torch.cuda.synchronize()
    fa_multi.barrier()
    pre_s, gen_s, gen_dev_ms, n_calls = job()
    enc_s = timing["encoder_ms"] / 1e3
    total = enc_s + pre_s + gen_s
    total = fa_multi.reduce(total, "max")
    n_pre = sum(len(e) for e in streams)
    peak, peak_kind = measured_peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "16 utterances: encoder + batched chunked prefill + 64-token decode, tokens/s",
            "value": (n_pre + 16 * n_new) * world / total,
            "unit": "tokens/s", "n_gpus": world, "steps": 1, "warmup": 1, "ms_per_step": total * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic: seeded random-init Q8_0 encoder, adaptor and decoder weights; stand-in LFR frames",
            "config": {"workload": "16 utterances (49-249 LFR frames through the encoder and adaptor, 30 prompt "
                                   "tokens), prefill in calls of <= 512 rows, then 64 greedy tokens each",
                       "encoder_ms": enc_s * 1e3,
                       "prefill_rows": n_pre, "prefill_calls": n_calls, "prefill_ms": pre_s * 1e3,
                       "prefill_tokens_per_s": n_pre / pre_s, "decode_ms": gen_s * 1e3,
                       "decode_device_ms": gen_dev_ms, "decode_tokens_per_s": 16 * n_new / gen_s},
            "gpu_launches": None,
        }), flush=True)
    dec.close()
    enc.close()
    fa_multi.shutdown()


# --------------------------------------------------- continuous batching --
def run_serve(a):
    """Continuous batching (fa_sched_*): --streams streams over all GPUs, each given at
    its arrival to the rank with the fewest outstanding KV pages (no collectives); prompt lengths log-uniform in [200, 6000] tokens,
    output lengths uniform in [16, 512] (EOS ignored), Poisson arrivals at
    --arrival-rate streams/s over all GPUs, a --kv-gb page pool per GPU. Each step
    runs one forward over every running stream's next token plus prompt chunks of up to
    512 rows per stream, within --serve-rows rows per forward.
    Reports generated and processed tokens/s over the run (wall clock, max over ranks;
    the run stops after --serve-seconds even with streams left), time to first token
    and the peak number of concurrent streams."""
    import torch
    import fa_dec

    rank, local, world = fa_multi.init("nccl")
    torch.cuda.set_device(local)
    cfg = fa_synth.QWEN3_06B
    w = fa_synth.make_weights(cfg, seed=1)
    rng = np.random.default_rng(2024)
    n = a.streams
    plen = np.exp(rng.uniform(np.log(200), np.log(6000), n)).astype(np.int64)
    olen = rng.integers(16, 513, n)
    arrive = np.cumsum(rng.exponential(1.0 / a.arrival_rate, n))
    # streams go to the rank with the fewest outstanding KV pages at their arrival
    owner = fa_multi.dispatch_by_pages(arrive, plen, olen, world)
    mine = [int(i) for i in np.flatnonzero(owner == rank)]
    page_bytes = 28 * 8 * 2 * 16 * 128 * 2
    n_pages = int(a.kv_gb * 1e9 // page_bytes)
    max_ctx = int((plen.max() + olen.max() + 31) // 16 * 16)
    dec = fa_dec.Decoder(local, **fa_synth.decoder_desc(cfg, max_ctx=max_ctx, n_pages=n_pages,
                                                        max_seqs=max(len(mine), 1), max_rows=a.serve_rows))
    dec.load_weights(w)
    dec.set_graphs(False)          # every step has its own shape
    prompts = {i: rng.integers(0, cfg["vocab"], int(plen[i])).astype(np.int32) for i in mine}

    # warm-up: a few short streams through the same path
    sch = fa_dec.Scheduler(dec, max_batch_rows=a.serve_rows, prefill_chunk=512, max_running=1024, eos_id=-1)
    for k in range(4):
        sch.submit(-1 - k, 8, ids=rng.integers(0, cfg["vocab"], 300).astype(np.int32))
    while not sch.idle():
        sch.step()
    sch.close()

    sch = fa_dec.Scheduler(dec, max_batch_rows=a.serve_rows, prefill_chunk=512, max_running=1024, eos_id=-1)
    torch.cuda.synchronize()
    fa_multi.barrier()
    t0 = time.perf_counter()
    nxt, first, gen, peak_run = 0, {}, 0, 0
    order = sorted(mine, key=lambda i: arrive[i])
    while (nxt < len(order) or not sch.idle()) and time.perf_counter() - t0 < a.serve_seconds:
        now = time.perf_counter() - t0
        while nxt < len(order) and arrive[order[nxt]] <= now:
            i = order[nxt]
            sch.submit(i, int(olen[i]), ids=prompts[i])
            nxt += 1
        if sch.idle():
            time.sleep(max(0.0, min(0.01, arrive[order[nxt]] - now)))
            continue
        for tag, tok, fin in sch.step():
            gen += 1
            if tag not in first:
                first[tag] = time.perf_counter() - t0 - arrive[tag]
        peak_run = max(peak_run, sch.stats()["running"])
    el = time.perf_counter() - t0
    st = sch.stats()
    sch.close()
    dec.close()
    el_max = fa_multi.reduce(el, "max")
    gen_all = fa_multi.reduce(gen, "sum")
    rows_all = fa_multi.reduce(st["rows"], "sum")
    ttft = np.array(list(first.values())) if first else np.zeros(1)
    if rank == 0:
        print(json.dumps({
            "metric": "continuous-batching generated tokens/s", "value": gen_all / el_max, "unit": "tokens/s",
            "n_gpus": world, "steps": int(st["steps"]), "warmup": 1, "ms_per_step": el * 1e3 / max(st["steps"], 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic: seeded random-init Q8_0 weights, random prompt token ids",
            "config": {"workload": f"{n} streams, prompts log-U[200,6000], outputs U[16,512], Poisson "
                                   f"{a.arrival_rate}/s, {a.kv_gb} GB pages per GPU, <= {a.serve_rows} rows per step",
                       "streams": n, "finished_streams_rank0": int(st["finished"]),
                       "processed_tokens_per_s": rows_all / el_max, "elapsed_s": el_max,
                       "ttft_p50_s": float(np.percentile(ttft, 50)), "ttft_p99_s": float(np.percentile(ttft, 99)),
                       "peak_running_rank0": peak_run, "pages_per_gpu": n_pages},
            "gpu_launches": None,
        }), flush=True)
    fa_multi.shutdown()


# --------------------------------------------------------- one utterance --
def run_pipeline(a):
    """One utterance end to end on the GPU (the front end excluded): 5 s of audio as 82
    LFR frames of 560 features (stand-in values), the full SANM encoder (50 + 20
    layers) and adaptor, a prefill of 16 prompt tokens + 82 audio frames + 14 prompt
    tokens, then exactly 32 greedy tokens (EOS ignored), batch 1, random-init Q8_0
    weights everywhere. Reports the latency per utterance and the real-time factor;
    the CPU restatement of the same work runs beside it on the host cores."""
    import torch
    import fa_dec

    rank, local, world = fa_multi.init("nccl")
    torch.cuda.set_device(local)
    cfg = fa_synth.QWEN3_06B
    w = fa_synth.make_weights(cfg, seed=1)
    we = fa_synth.make_encoder_weights(seed=2)
    rng = np.random.default_rng(rank)
    T, n_new = 82, 32
    lfr = fa_synth.lfr_features(rng, T)
    table = w["llm.model.embed_tokens.weight"][2].reshape(cfg["vocab"], cfg["hidden"])
    pre, suf = rng.integers(0, cfg["vocab"], 16), rng.integers(0, cfg["vocab"], 14)
    emb_pre = (table[pre].astype(np.uint32) << 16).view(np.float32)
    emb_suf = (table[suf].astype(np.uint32) << 16).view(np.float32)
    enc = fa_dec.Encoder(local, max_frames=256)
    enc.load_weights(we)
    dec = fa_dec.Decoder(local, **fa_synth.decoder_desc(cfg, max_ctx=512, n_pages=64, max_seqs=2, max_rows=256))
    dec.load_weights(w)

    parts = {"encoder_ms": 0.0, "prefill_ms": 0.0, "decode_ms": 0.0}

    def utterance():
        t0 = time.perf_counter()
        audio = enc.forward(lfr)
        t1 = time.perf_counter()
        rows = np.concatenate([emb_pre, audio, emb_suf]).astype(np.float32)
        s = dec.seq_open(512)
        first, _ = dec.prefill(s, rows)
        t2 = time.perf_counter()
        toks = [first]
        for _ in range(n_new - 1):
            nx, _ = dec.decode_step([s], [toks[-1]])
            toks.append(int(nx[0]))
        dec.seq_close(s)
        t3 = time.perf_counter()
        parts["encoder_ms"] += (t1 - t0) * 1e3
        parts["prefill_ms"] += (t2 - t1) * 1e3
        parts["decode_ms"] += (t3 - t2) * 1e3
        return toks

    for _ in range(max(a.warmup, 1)):
        utterance()
    torch.cuda.synchronize()
    fa_multi.barrier()
    K = max(a.steps, 1)
    for k in parts:
        parts[k] = 0.0
    t0 = time.perf_counter()
    for _ in range(K):
        toks = utterance()
    ms = (time.perf_counter() - t0) * 1e3 / K
    ms = fa_multi.reduce(ms, "max")
    cpu = None
    if rank == 0 and not a.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        import encoder as enc_oracle
        oracle.build()
        oracle.set_num_threads(len(os.sched_getaffinity(0)))
        t1 = time.perf_counter()
        audio = enc_oracle.adaptor_forward(we, enc_oracle.encoder_forward(we, lfr))
        rows = np.concatenate([emb_pre, audio, emb_suf]).astype(np.float32)
        od = oracle.OracleDecoder(cfg, w, n_pages=16, max_seqs=1, max_pages_per_seq=16, max_pos=256,
                                  mode=oracle.MODE_GGML_CPU)
        od.seq_open(0)
        _, nx = od.forward([0] * len(rows), embeds=rows, want_logits=False)
        tok = int(nx[-1])
        for _ in range(n_new - 1):
            _, nx = od.forward([0], tokens=[tok], want_logits=False)
            tok = int(nx[0])
        cpu_ms = (time.perf_counter() - t1) * 1e3
        cpu = {"value": cpu_ms, "unit": "ms per utterance", "cores": oracle.num_threads(), "kind": "port",
               "sample": "one utterance: encoder + adaptor in numpy float64, decoder prefill + 32 tokens in the "
                         "C++ oracle (ggml-CPU arithmetic); CPU restatement of the reference (ggml unavailable)"}
    if rank == 0:
        print(json.dumps({
            "metric": "utterance latency, encoder + adaptor + prefill + 32 greedy tokens", "value": ms,
            "unit": "ms", "n_gpus": world, "steps": K, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic: random-init Q8_0 encoder, adaptor and decoder; stand-in LFR frames",
            "config": {"workload": "5 s utterance: 82 LFR frames x 560, SANM 50+20 layers, adaptor, 112-row "
                                   "prefill, 32 greedy tokens, batch 1",
                       "rtf": ms / 5000.0, **{k: v / K for k, v in parts.items()}},
            "cpu_baseline": cpu, "gpu_launches": None,
        }), flush=True)
    enc.close()
    dec.close()
    fa_multi.shutdown()


# ------------------------------------------------- KV append + gather --
APPEND_METRIC = "KV append + gather GB/s (32 sequences, 28 layers, f16 pages of 16 tokens)"


def _append_case(rank, steps_total, L=28):
    """The append + gather workload: 32 sequences with contexts ~U[64, 1024], block tables
    cut from a random permutation of a 4096-page pool, positions, lengths and slab row
    offsets of every step."""
    rng = np.random.default_rng(2024 + rank)
    n_pages, n_seq = 4096, 32
    ctx0 = rng.integers(64, 1025, n_seq).astype(np.int32)
    bt_stride = (1024 + steps_total + 15) // 16
    if n_seq * bt_stride > n_pages:
        raise SystemExit(f"append workload: warmup + steps must stay below {n_pages // n_seq * 16 - 1039}")
    bt = rng.permutation(n_pages)[: n_seq * bt_stride].reshape(n_seq, bt_stride).astype(np.int32)
    s = np.arange(steps_total, dtype=np.int32)[:, None]
    pos = ctx0[None, :] + s                              # token written at step s
    n_kv = pos + 1                                       # tokens gathered after it
    row0 = np.concatenate([np.zeros((steps_total, 1), np.int64), np.cumsum(n_kv, 1)[:, :-1]], 1).astype(np.int32)
    return L, n_pages, n_seq, ctx0, bt, bt_stride, pos.astype(np.int32), n_kv.astype(np.int32), row0


def _append_bytes(n_seq, n_kv_step, L=28):
    """Algorithmic bytes of one step: the appended K/V read and written once, every
    gathered token read from its page and written to the slabs once."""
    return 2 * n_seq * L * KV_BYTES_PER_TOKEN_LAYER + 2 * int(n_kv_step.sum()) * L * KV_BYTES_PER_TOKEN_LAYER


def cpu_append_sample(budget_s, n_steps_max=256):
    """The oracle's append (C) and gather (numpy) on the same workload, one host thread,
    for about budget_s seconds. Returns GB/s, steps done, seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    L, n_pages, n_seq, ctx0, bt, bt_stride, pos, n_kv, row0 = _append_case(0, n_steps_max)
    pool = np.zeros((L, n_pages, 8 * 2 * 16 * 128), np.uint16)
    rng = np.random.default_rng(5)
    slots = np.arange(n_seq, dtype=np.int32)
    done, nbytes, el = 0, 0, 0.0          # el counts append + gather only, not input generation
    while done < n_steps_max and el < budget_s:
        k = oracle.f32_to_f16_bits(rng.standard_normal((n_seq, L, 8, 128)).astype(np.float32))
        v = oracle.f32_to_f16_bits(rng.standard_normal((n_seq, L, 8, 128)).astype(np.float32))
        t1 = time.perf_counter()
        oracle.kv_append_raw(k, v, slots, pos[done], bt, pool, L, n_pages)
        oracle.kv_gather(pool, bt, slots, n_kv[done], row0[done], int(n_kv[done].sum()))
        el += time.perf_counter() - t1
        nbytes += _append_bytes(n_seq, n_kv[done])
        done += 1
    return nbytes / el / 1e9, done, el


def run_append(a):
    """Paged KV append + gather on its own: each step appends one token per sequence in
    all 28 layers (K/V ~N(0,1) f16, through fa_op_kv_append) and then gathers every
    sequence's K/V over its whole length into head-major slabs [28][8][rows][128]
    (fa_op_kv_gather), the layout the reference's attention reads. Prints GB/s of
    algorithmic bytes."""
    import torch
    import fa_dec

    rank, local, world = fa_multi.init("nccl")
    torch.cuda.set_device(local)
    K, W = a.steps, a.warmup
    E = a.e2e_steps
    steps_total = W + K + E
    L, n_pages, n_seq, ctx0, bt, bt_stride, pos, n_kv, row0 = _append_case(rank, steps_total, a.append_layers)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(rank)
    pool = torch.empty((L, n_pages, 8 * 2 * 16 * 128), dtype=torch.float16, device=dev)
    for l in range(L):
        pool[l].normal_(generator=g)
    pool = pool.view(torch.int16)
    kv_shape = (W + K, n_seq, L, 8, 128)
    k_in = torch.randn(kv_shape, dtype=torch.float16, device=dev, generator=g).view(torch.int16)
    v_in = torch.randn(kv_shape, dtype=torch.float16, device=dev, generator=g).view(torch.int16)
    max_rows = int(n_kv.sum(1).max())
    k_out = torch.empty((L, 8, max_rows, 128), dtype=torch.int16, device=dev)
    v_out = torch.empty_like(k_out)
    d_bt = torch.from_numpy(bt).to(dev)
    d_pos, d_nkv, d_row0 = (torch.from_numpy(x).to(dev) for x in (pos, n_kv, row0))
    slot = torch.arange(n_seq, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def append(i, kp, vp):
        fa_dec.op_kv_append(kp, vp, n_seq, L, d_pos[i].data_ptr(), slot.data_ptr(), d_bt.data_ptr(), bt_stride,
                            n_pages, pool.data_ptr(), err.data_ptr(), stream)

    def gather(i):
        fa_dec.op_kv_gather(pool.data_ptr(), L, n_pages, d_bt.data_ptr(), bt_stride, slot.data_ptr(),
                            d_nkv[i].data_ptr(), d_row0[i].data_ptr(), n_seq, bt_stride, max_rows,
                            k_out.data_ptr(), v_out.data_ptr(), err.data_ptr(), stream)

    for i in range(W):
        append(i, k_in[i].data_ptr(), v_in[i].data_ptr())
        gather(i)
    torch.cuda.synchronize()
    fa_multi.barrier()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    sampler = ClockSampler(local)
    sampler.start()
    for j in range(K):
        i = W + j
        ev[j][0].record()
        append(i, k_in[i].data_ptr(), v_in[i].data_ptr())
        ev[j][1].record()
        gather(i)
        ev[j][2].record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    fa_multi.barrier()
    assert int(err.item()) == 0, "append or gather reported a device error"
    ms = fa_multi.reduce(ev[0][0].elapsed_time(ev[-1][2]), "max")
    step_bytes = [_append_bytes(n_seq, n_kv[W + j], L) for j in range(K)]
    value = sum(step_bytes) * world / (ms / 1e3) / 1e9
    gather_ms = sum(ev[j][1].elapsed_time(ev[j][2]) for j in range(K))
    append_ms = sum(ev[j][0].elapsed_time(ev[j][1]) for j in range(K))
    gather_bytes = sum(2 * int(n_kv[W + j].sum()) * L * KV_BYTES_PER_TOKEN_LAYER for j in range(K))
    achieved = gather_bytes / (gather_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    traffic = None
    tf = os.path.join(ROOT, "profiles", "gather_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            t = json.load(f)
        # DRAM bytes scale with the algorithmic bytes (layers x tokens gathered)
        traffic = t["dram_bytes_per_launch"] * (gather_bytes / K) / t["algorithmic_bytes_per_launch"]

    # e2e: the step's K/V come from pinned host memory each step, the error word goes back
    k_host = torch.randn((E, n_seq, L, 8, 128), dtype=torch.float16).view(torch.int16).pin_memory()
    v_host = torch.randn((E, n_seq, L, 8, 128), dtype=torch.float16).view(torch.int16).pin_memory()
    k_dev = torch.empty((n_seq, L, 8, 128), dtype=torch.int16, device=dev)
    v_dev = torch.empty_like(k_dev)
    err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize()
    fa_multi.barrier()
    t0 = time.perf_counter()
    e2e_bytes = 0
    for j in range(E):
        i = W + K + j
        k_dev.copy_(k_host[j], non_blocking=True)
        v_dev.copy_(v_host[j], non_blocking=True)
        append(i, k_dev.data_ptr(), v_dev.data_ptr())
        gather(i)
        err_host.copy_(err, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        if int(err_host.item()) != 0:
            raise RuntimeError("append or gather reported a device error")
        e2e_bytes += _append_bytes(n_seq, n_kv[i], L)
    e2e_s = fa_multi.reduce(time.perf_counter() - t0, "max")
    e2e_value = e2e_bytes * world / e2e_s / 1e9
    all_clocks = fa_multi.gather(clocks)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline and L == 28:
        del pool, k_in, v_in
        v, n_done, el = cpu_append_sample(a.cpu_budget_s)
        cpu = {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"the first {n_done} steps of the same workload (32 sequences, 28 layers) through the "
                         f"oracle's append and gather in {el:.1f} s, one thread"}
    if rank == 0:
        reasons = sorted(set(r for c in all_clocks for r in c.get("reasons", [])))
        print(json.dumps({
            "metric": APPEND_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic: N(0,1) f16 K/V and pages, seeded contexts and block tables",
            "config": {"workload": f"isolated paged KV append + gather: 32 sequences at contexts ~U[64,1024], {L} "
                                   "layers x 8 KV heads x 128 f16, pages of 16 tokens, block tables from a random "
                                   "permutation of a 4096-page pool, 1 token appended per sequence per step, every "
                                   "sequence gathered over its whole length each step",
                       "append_ms_per_step": append_ms / K, "gather_ms_per_step": gather_ms / K,
                       "layers": L, "l2": "no flush: each step reads 67-100 MB of pages per layer (1.9-2.8 GB at 28 "
                                          "layers) out of a 268 MB-per-layer pool and writes as much, far above L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "kernel": "kv_gather_kernel", "peak_kind": peak_kind,
                         "bytes_per_launch": gather_bytes / K, "ms_per_launch": gather_ms / K},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": 2 * n_seq * L * 8 * 128 * 2,
                    "d2h_bytes_per_step": 4, "steps": E},
            "gpu_launches": 2 * K,
            "clocks": {"sm_mhz": all_clocks[0].get("sm_mhz"), "sm_max_mhz": all_clocks[0].get("sm_max_mhz"),
                       "reasons": reasons},
        }), flush=True)
    fa_multi.shutdown()


# -------------------------------------------------------------- reference --
def run_append_reference(a):
    """The append + gather workload through the oracle on the host cores (the reference's
    ggml CPU path cannot be built here), about --cpu-budget-s seconds of steps."""
    v, n_done, el = cpu_append_sample(a.cpu_budget_s, n_steps_max=max(a.steps, 1))
    print(json.dumps({
        "impl": "reference", "metric": APPEND_METRIC, "value": v, "unit": "GB/s", "n_gpus": a.gpus,
        "steps": n_done, "warmup": 0, "ms_per_step": el * 1e3 / n_done, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: N(0,1) f16 K/V, seeded contexts and block tables",
        "config": {"workload": "isolated paged KV append + gather: 32 sequences at contexts ~U[64,1024], 28 layers "
                               "x 8 KV heads x 128 f16, pages of 16 tokens, 1 token appended per sequence per step, "
                               "every sequence gathered over its whole length each step"},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
                         "sample": f"the first {n_done} steps in {el:.1f} s through the oracle's append and gather"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference(a):
    """The reference's CPU path (ggml) cannot be built here, so its restatement (the
    oracle, ggml-CPU arithmetic, all host threads) is timed on the same config: each
    step is one decode step of a 2-sequence sample at the 2048-token context."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    if a.workload == "append":
        return run_append_reference(a)
    cfg = fa_synth.QWEN3_06B
    w = fa_synth.make_weights(cfg, seed=1)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    oracle.set_num_threads(len(os.sched_getaffinity(0)))   # torchrun sets OMP_NUM_THREADS=1
    rows = 2
    ctx = a.ctx
    n_steps = a.warmup + a.steps
    pages = (ctx + n_steps + 32) // 16
    od = oracle.OracleDecoder(cfg, w, n_pages=rows * pages, max_seqs=rows, max_pages_per_seq=pages,
                              max_pos=ctx + n_steps + 32, mode=oracle.MODE_GGML_CPU)
    rng = np.random.default_rng(0)
    for s in range(rows):
        od.seq_open(s)
        od._reserve(s, ctx)
        od.seq_len[s] = ctx
    for l in range(od.pool.shape[0]):
        od.pool[l] = oracle.f32_to_f16_bits(rng.uniform(-2, 2, od.pool.shape[1:]).astype(np.float32))
    toks = rng.integers(0, cfg["vocab"], rows)
    for _ in range(a.warmup):
        _, toks = od.forward([0, 1], tokens=toks, want_logits=False)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        _, toks = od.forward([0, 1], tokens=toks, want_logits=False)
    el = time.perf_counter() - t0
    v = rows * a.steps / el
    cores = oracle.num_threads()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": el * 1e3 / a.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (Q8_0 activations x Q8_0 weights)",
        "data": "synthetic: seeded random-init Q8_0 Qwen3-0.6B weights, synthetic f16 KV cache",
        "config": {"workload": f"steady-state decode at {ctx}-token context, Qwen3-0.6B 28 layers, "
                               f"2-sequence sample per step on the host cores", "ctx": ctx, "rows": rows},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{a.steps} steps x {rows} sequences; CPU restatement of the reference "
                                   f"(ggml unavailable: third_party/ggml is not vendored)"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "attention":
        run_attention(args)
    elif args.workload == "gemm":
        run_gemm(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "serve":
        run_serve(args)
    elif args.workload == "pipeline":
        run_pipeline(args)
    elif args.workload == "append":
        run_append(args)
    else:
        run_ours(args)
