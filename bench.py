"""Decode benchmark: aggregate tok/s for tenants sharing Llama-2-7B Q4_K_M weights.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Llama-2-7B shape (32 layers, hidden 4096,
32 MHA heads x 128, FFN 11008, vocab 32000), random-init N(0, 0.02) weights
quantised to Q4_K (attn_v and output Q6_K) on the device, 8 tenants per GPU
with fp16 paged KV, prompts U[128, 512] tokens (seed 4), greedy decode. One
step = one decode token for every tenant on the GPU (one rb_forward call).
Under torchrun each rank drives one GPU with its own 8 tenants (weak scaling,
no collective on the decode path; the barrier and the max-over-ranks time
reduction are plumbing).

`value` = tokens / device time of the K decode-step graphs (inputs resident);
`e2e` = the same K steps timed on the device stream from the H2D copy of each
step's token ids through the D2H copy of its greedy ids, via the C ABI with
host buffers. The weights (3.9 GB) dwarf the 126 MB L2, so no flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000,
           max_seq=1024, rms_eps=1e-5, layer_eps=1e-5, rope_theta=10000.0)
TENANTS_PER_GPU = 8       # configs[3] on one GPU
TOTAL_TENANTS_MULTI = 64  # configs[3] at 2/4/8 GPUs: 32/16/8 per GPU
METRIC = "aggregate decode tok/s, 8 tenants Llama-7B Q4_K; paged-KV attn HBM GB/s vs peak"
Q4K_BPW, Q6K_BPW = 144 / 256, 210 / 256
# dram__bytes_read.sum + dram__bytes_write.sum of one gate|up GEMV launch (22016 x 4096
# Q4_K, M = 8), from `ncu --set full` of `bench.py --case gemv`: 50.87 + 0.07 MB.
GEMV_NCU_TRAFFIC = 50941440
# the same for one config-2 attention launch (`bench.py --case attn`): 282.53 + 4.43 MB
ATTN_NCU_TRAFFIC = 286963456


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def weight_bytes(cfg):
    H, Q, KV, F, V, L = (cfg["hidden"], cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"],
                         cfg["ffn"], cfg["vocab"], cfg["n_layers"])
    layer = (Q * H + KV * H + Q * H + 3 * F * H) * Q4K_BPW + KV * H * Q6K_BPW
    return L * layer + V * H * Q6K_BPW


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        time.sleep(0.5)  # let the sampler start before the timed region
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.p:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                out, _ = self.p.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def build_model(rb, torch, ctx, dev, n_tenants, host_copy=None, base=None):
    """Random-init Q4_K_M weights generated and quantised on the device. If
    host_copy is a dict, the GGUF bytes of every tensor are also copied into it
    (for the CPU baseline on identical weights)."""
    base = base or CFG
    cfg = dict(base, kv_dtype=rb.F16, max_tenants=n_tenants, kv_pages=n_tenants * (base["max_seq"] // 16))
    m = rb.Model(ctx, cfg)
    g = torch.Generator(device=dev)
    H, Q, KV, F, V = base["hidden"], base["n_heads"] * base["head_dim"], base["n_kv_heads"] * base["head_dim"], \
        base["ffn"], base["vocab"]
    seed = [3]

    def qt(dt, rows, cols):
        g.manual_seed(seed[0])
        seed[0] += 1
        x = torch.randn(rows, cols, generator=g, device=dev, dtype=torch.float32).mul_(0.02)
        be, bb = rb.BLOCK_ELEMS[dt], rb.BLOCK_BYTES[dt]
        out = torch.empty(rows * cols // be * bb, dtype=torch.uint8, device=dev)
        ctx.quantize(dt, x.view(-1), out)
        return out

    def put(which, layer, dt, t):
        m.set_weight(which, layer, dt, t)
        if host_copy is not None:
            host_copy[(which, layer)] = (dt, t.cpu().numpy())

    ones = torch.ones(H, dtype=torch.float32, device=dev)
    put(rb.W_TOKEN_EMBD, -1, rb.Q4_K, qt(rb.Q4_K, V, H))
    put(rb.W_OUTPUT_NORM, -1, rb.F32, ones)
    put(rb.W_OUTPUT, -1, rb.Q6_K, qt(rb.Q6_K, V, H))
    shapes = [(rb.W_Q, Q, H, rb.Q4_K), (rb.W_K, KV, H, rb.Q4_K), (rb.W_V, KV, H, rb.Q6_K), (rb.W_O, H, Q, rb.Q4_K),
              (rb.W_GATE, F, H, rb.Q4_K), (rb.W_UP, F, H, rb.Q4_K), (rb.W_DOWN, H, F, rb.Q4_K)]
    for l in range(base["n_layers"]):
        put(rb.W_ATTN_NORM, l, rb.F32, ones)
        put(rb.W_FFN_NORM, l, rb.F32, ones)
        for which, r, c, dt in shapes:
            put(which, l, dt, qt(dt, r, c))
    m.finalize()
    torch.cuda.synchronize(dev)
    return m


def gemv_roofline(rb, torch, ctx, dev, hbm_peak, peak_kind):
    """Dominant kernel: the Q4_K gate|up GEMV (22016 x 4096, M = 8 tenants).
    Device time per launch from CUDA events around a CUDA graph of 48
    back-to-back launches on the context stream, rotating 4 weight copies
    (200 MB > L2, so every launch streams its weights from HBM)."""
    n, k, m = 2 * CFG["ffn"], CFG["hidden"], TENANTS_PER_GPU
    g = torch.Generator(device=dev)
    ws = []
    for i in range(4):
        g.manual_seed(100 + i)
        x = torch.randn(n, k, generator=g, device=dev).mul_(0.02)
        blk = torch.empty(n * k // 256 * 144, dtype=torch.uint8, device=dev)
        ctx.quantize(rb.Q4_K, x.view(-1), blk)
        ws.append(rb.Weight(ctx, rb.Q4_K, n, k, blk))
        del x
    avg_us = ctx.gemv_timing(ws, m, iters=48, reps=3)
    alg_bytes = n * k * Q4K_BPW + m * k * 4 + m * n * 4
    achieved = alg_bytes / (avg_us * 1e-6) / 1e9
    for w in ws:
        w.free()
    # dram__bytes_read.sum + write.sum of one launch of this kernel and shape
    traffic = GEMV_NCU_TRAFFIC
    return {"kernel": "gemv_kernel<Q4_K, NT=1> (gate|up 22016x4096, M=8)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "algorithmic_bytes": int(alg_bytes),
            "avg_launch_us": round(avg_us, 2)}


def attention_roofline(rb, torch, ctx, dev, hbm_peak, peak_kind):
    """Config 2: 16 tenants, 32 q / 8 kv heads, hd 128, fp16 K/V ~ N(0,1) (seed 2),
    contexts U[512, 8192], 16-token pages from a permuted pool; one new token per
    tenant appended then attended. Timed: the attention kernel (events)."""
    rng = np.random.default_rng(2)
    n_t, hq, hkv, hd = 16, 32, 8, 128
    ctxs = rng.integers(512, 8193, n_t)
    pool = ctx.kv_pool(1, hkv, hd, rb.F16, n_pages=int(sum((c + 17) // 16 for c in ctxs)) + 16,
                       max_tenants=n_t, max_seq=8208)
    pool.shuffle(2)
    for t in range(n_t):
        pool.create(t)
        L = int(ctxs[t])
        kk = torch.randn(L, hkv * hd, device=dev)
        vv = torch.randn(L, hkv * hd, device=dev)
        pool.append(t, 0, kk, vv)
    q = torch.randn(n_t, hq * hd, device=dev)
    kn = torch.randn(n_t, hkv * hd, device=dev)
    vn = torch.randn(n_t, hkv * hd, device=dev)
    out = torch.empty(n_t, hq * hd, device=dev)
    tenants = list(range(n_t))
    pos = [int(c) for c in ctxs]
    pool.attention_forward(0, tenants, q, hq, 1 / np.sqrt(hd), positions=pos, k_new=kn, v_new=vn, out=out)
    torch.cuda.synchronize(dev)
    ms = []
    for _ in range(20):
        pool.attention_forward(0, tenants, q, hq, 1 / np.sqrt(hd), positions=[p for p in pos], out=out)
        ms.append(ctx.last_forward_ms())
    avg = float(np.mean(ms[3:]))
    kv_bytes = sum((p + 1) * hkv * hd * 2 * 2 for p in pos)
    pages = sum(p // 16 + 1 for p in pos)
    alg = kv_bytes + pages * 4 + 2 * n_t * hq * hd * 4
    achieved = alg / (avg * 1e-3) / 1e9
    return {"kernel": "attn_kernel<HD=128, NREP=4, fp16> (config 2)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "traffic": ATTN_NCU_TRAFFIC, "algorithmic_bytes": int(alg),
            "avg_launch_us": round(avg * 1e3, 2)}


def decode_step_line(step_bytes, step_ms, prof_ms, hbm_peak, nt):
    """Per-GPU decode-step roofline, plus the GEMV chains' figure inside the
    step: their share of a kernel-by-kernel run of one step (no overlap),
    applied to the graph-replayed step time, against the weight bytes they
    stream."""
    tot = sum(prof_ms.values())
    share = prof_ms["gemv"] / tot if tot > 0 else None
    wb = weight_bytes(CFG)
    line = {"tenants_per_gpu": nt, "bytes_per_step": int(step_bytes),
            "achieved_GBps": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
            "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / hbm_peak, 4),
            "kernel_ms_serialised": {k: round(v, 4) for k, v in prof_ms.items()}}
    if share:
        chain_ms = step_ms * share
        line["chain"] = {"share": round(share, 4), "ms_in_step": round(chain_ms, 4), "weight_bytes": int(wb),
                         "GBps": round(wb / (chain_ms * 1e-3) / 1e9, 1),
                         "frac": round(wb / (chain_ms * 1e-3) / 1e9 / hbm_peak, 4)}
    return line


SWEEP_SHAPES = [(4096, 4096, "q4k"), (11008, 4096, "q4k"), (4096, 11008, "q4k"), (32000, 4096, "q6k")]
SWEEP_M = (1, 8, 16, 64)


def gemv_sweep(rb, torch, ctx, dev, hbm_peak, peak_kind):
    """the fused dequant GEMV/GEMM at Llama-7B shapes, weights
    N(0, 0.02) quantised on the device (seed 3 per shape), M = 1, 8, 16, 64.
    Device time per launch from a CUDA graph of 48 launches rotating weight
    copies that together exceed the 126 MB L2 (each launch streams from HBM)."""
    out = []
    g = torch.Generator(device=dev)
    for n, k, fmt in SWEEP_SHAPES:
        dt = rb.Q4_K if fmt == "q4k" else rb.Q6_K
        bpw = Q4K_BPW if fmt == "q4k" else Q6K_BPW
        wbytes = n * k * bpw
        copies = max(2, int(np.ceil(300e6 / wbytes)))
        g.manual_seed(3)
        x = torch.randn(n, k, generator=g, device=dev).mul_(0.02)
        blk = torch.empty(int(wbytes), dtype=torch.uint8, device=dev)
        ctx.quantize(dt, x.view(-1), blk)
        del x
        ws = [rb.Weight(ctx, dt, n, k, blk) for _ in range(copies)]
        for m in SWEEP_M:
            us = ctx.gemv_timing(ws, m, iters=48, reps=3)
            alg = wbytes + 4 * m * k + 4 * m * n
            gbps = alg / (us * 1e-6) / 1e9
            out.append({"n": n, "k": k, "fmt": fmt, "m": m, "us": round(us, 2), "GBps": round(gbps, 1),
                        "frac": round(gbps / hbm_peak, 4), "path": "tcgen05" if (fmt == "q4k" and ctx.uses_tcgen05(m)) else "mma.sync"})
        for w in ws:
            w.free()
        del blk
    return {"workload": "configs[2]: N x K weights N(0,0.02) seed 3, fp32 activations, M rows", "peak": hbm_peak,
            "peak_kind": peak_kind, "points": out}


def cpu_sweep(threads, budget_s=1.0):
    """configs[2] on the host cores, timed on a row sample of each weight (the
    cost per output row is constant, so time x N / rows sampled is the full
    call). B1: the reference's fused kernel restated (fused.rs:229-374 /
    1128-1259) on one thread; B2: the same on every thread; B3: dequantise then
    an fp32 GEMM (CandleCpuBackend semantics, candle_cpu_backend.rs:92-114) on
    every thread."""
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    pts = []
    for n, k, fmt in SWEEP_SHAPES:
        dt = O.Q4K if fmt == "q4k" else O.Q6K
        rows = 256
        blocks = O.quantize(dt, rng.normal(0, 0.02, size=(rows, k)).astype(np.float32))
        wbytes = n * k * O.BLOCK_BYTES[dt] / 256
        for m in SWEEP_M:
            x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
            rec = {"n": n, "k": k, "fmt": fmt, "m": m, "rows_sampled": rows}
            for name, fn in (("B1", lambda: O.fused_matmul(dt, blocks, x, m, rows, k, threads=1)),
                             ("B2", lambda: O.fused_matmul(dt, blocks, x, m, rows, k, threads=threads)),
                             ("B3", lambda: O.dequant_matmul(dt, blocks, x, m, rows, k, threads=threads))):
                fn()
                t0, reps = time.perf_counter(), 0
                while True:
                    fn()
                    reps += 1
                    if time.perf_counter() - t0 > budget_s / 8 or reps >= 50:
                        break
                per_call = (time.perf_counter() - t0) / reps * (n / rows)
                rec[name] = {"us": round(per_call * 1e6, 1), "GBps": round(wbytes / per_call / 1e9, 3)}
            pts.append(rec)
    return {"threads": threads, "points": pts}


def cpu_attention_config2(threads):
    """configs[1] on the host: the oracle's attention (compute_attention restated,
    attention.rs:310-380, over a contiguous fp16-rounded cache) for the 16 tenants
    of the bench's microbench (contexts U[512, 8192] from seed 2, 32 q / 8 kv heads,
    hd 128), one query each. Single-threaded restatement: `cores` 1."""
    from oracle import oracle as O
    rng = np.random.default_rng(2)
    n_t, hq, hkv, hd = 16, 32, 8, 128
    ctxs = rng.integers(512, 8193, n_t)
    t_total, kv_bytes = 0.0, 0
    for t in range(n_t):
        L = int(ctxs[t]) + 1
        k = rng.normal(size=L * hkv * hd).astype(np.float16).astype(np.float32)
        v = rng.normal(size=L * hkv * hd).astype(np.float16).astype(np.float32)
        q = rng.normal(size=hq * hd).astype(np.float32)
        t0 = time.perf_counter()
        O.attention(q, k, v, 1, L, L - 1, hq, hkv, hd)
        t_total += time.perf_counter() - t0
        kv_bytes += L * hkv * hd * 2 * 2
    return {"us": round(t_total * 1e6, 1), "GBps_fp16_equiv": round(kv_bytes / t_total / 1e9, 3), "cores": 1,
            "kind": "port", "sample": "the 16 tenants of configs[1], one query each (fp32 math over fp16-rounded K/V)"}


def cpu_tinyllama_config1(threads, n_gen=8):
    """configs[0] on the host: TinyLlama-1.1B shape, Q4_K_M random-init weights
    (seed 0), 40-token prompt (seed 1), greedy decode through the oracle's
    Model::generate (model.rs:749-847); timed over n_gen decode tokens."""
    from oracle import oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import synth
    cfg = dict(synth.TINYLLAMA)
    W = synth.make_weights(cfg, seed=0)
    om = O.Model(dict(cfg, kv_fp16=0), W, threads=threads)
    prompt = np.random.default_rng(1).integers(0, cfg["vocab"], 40).astype(np.uint32)
    t0 = time.perf_counter()
    for cs in range(0, 40, 8):
        lg = om.forward(prompt[cs:cs + 8], cs)
    t1 = time.perf_counter()
    tok = O.argmax(lg)
    for g in range(n_gen):
        lg = om.forward([tok], 40 + g)
        tok = O.argmax(lg)
    t2 = time.perf_counter()
    return {"prefill_tok_per_s": round(40 / (t1 - t0), 2), "decode_tok_per_s": round(n_gen / (t2 - t1), 2),
            "cores": threads, "kind": "port", "sample": f"40-token prefill in 8-token chunks, {n_gen} greedy decode tokens"}


def cpu_baseline(weights, threads, max_s=20.0):
    """The oracle (C++ restatement of the reference CPU path, all host threads)
    on a bounded sample: single-token decode forwards of one tenant at context
    length 448 (the workload's mean), timed until ~max_s seconds."""
    from oracle import oracle as O
    cfg = dict(CFG, kv_fp16=1)
    om = O.Model(cfg, weights, threads=threads)
    om.kv_fill(448, seed=0)
    t0 = time.perf_counter()
    n = 0
    while True:
        om.forward([1], 448 + n)
        n += 1
        if time.perf_counter() - t0 > max_s or n >= 8:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} single-token decode forwards of one tenant at ctx 448 (Llama-2-7B Q4_K_M, "
                      f"oracle dequant+fp32 GEMV path, {threads} threads); tenants are served one token at a time"}


def run_ours(args):
    import torch
    import realm_b200 as rb
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    hbm_peak, peak_kind = peaks()
    ctx = rb.Context(local)
    ledger = None
    if dist:
        from realm_b200.sharding import StepLedger
        ledger = StepLedger.from_default_group("bench")
    # 8 tenants on one GPU; 64 tenants sharded over 2/4/8 GPUs by
    # LPT on prompt length (equal counts, so every rank runs the same row count)
    rng = np.random.default_rng(4)
    n_total = TENANTS_PER_GPU if world == 1 else TOTAL_TENANTS_MULTI
    all_lens = rng.integers(128, 513, n_total)
    all_ids = [rng.integers(0, CFG["vocab"], int(n)).astype(np.uint32) for n in all_lens]
    if world == 1:
        mine = list(range(n_total))
    else:
        from realm_b200.sharding import lpt_shard
        mine = lpt_shard([int(x) for x in all_lens], world, equal_counts=True)[rank]
    nt = len(mine)
    lens = all_lens[mine]
    host_w = {} if (world == 1 and not args.no_cpu) else None
    m = build_model(rb, torch, ctx, dev, nt, host_w)
    last = []
    for t, g in enumerate(mine):
        m.tenant_create(t)
        ids = all_ids[g]
        for cs in range(0, len(ids), 64):
            chunk = ids[cs:cs + 64]
            _, am = m.forward_rows([t] * len(chunk), chunk, want_logits=False)
        last.append(int(am[-1]))
    tenants = np.arange(nt, dtype=np.uint32)
    tok = np.array(last, np.uint32)
    for _ in range(args.warmup):
        _, tok = m.forward_rows(tenants, tok, want_logits=False)
    if ledger:  # every rank is alive and warmed up before anyone times
        ledger.done(1)
        ledger.wait_peers(1, timeout_s=600)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    dev_ms = 0.0
    launches = 0
    with Clocks(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            _, tok = m.forward_rows(tenants, tok, want_logits=False)
            dev_ms += ctx.last_forward_ms()
            launches += ctx.last_forward_launches()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    e2e_ms = ev0.elapsed_time(ev1)
    # one more step run kernel by kernel: the shares of the step's device time
    prof_ms, _ = m.forward_profile(tenants, tok)
    if ledger:
        ledger.done(2)
        ledger.wait_peers(2, timeout_s=600)
    if dist:
        t = torch.tensor([dev_ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, e2e_ms = float(t[0]), float(t[1])
        dist.barrier()
    tokens = nt * world * args.steps  # equal tenant counts per rank
    value = tokens / (dev_ms * 1e-3)
    e2e = tokens / (e2e_ms * 1e-3)
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    roof = gemv_roofline(rb, torch, ctx, dev, hbm_peak, peak_kind)
    attn = attention_roofline(rb, torch, ctx, dev, hbm_peak, peak_kind)
    sweep = gemv_sweep(rb, torch, ctx, dev, hbm_peak, peak_kind) if world == 1 else None
    # decode-step roofline: weights once + KV of every tenant per step
    mean_ctx = float(np.mean(lens)) + args.warmup + args.steps / 2
    step_bytes = weight_bytes(CFG) + nt * mean_ctx * CFG["n_layers"] * 2 * CFG["n_kv_heads"] * CFG["head_dim"] * 2
    step_ms = dev_ms / args.steps
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        # 64 tenants in total at every N >= 2 (total work fixed)
        "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None, "dtype": "f32 (Q4_K/Q6_K weights exact in fp16 tensor-core operands, fp16 hi/lo "
                                      "activations, fp32 accumulate)",
        "data": "synthetic: random-init N(0,0.02) weights quantised on device, prompts U[128,512] seed 4",
        "config": {"workload": ("Llama-2-7B Q4_K_M decode (configs[3]), 8 tenants on 1 GPU" if world == 1 else
                                f"Llama-2-7B Q4_K_M decode (configs[3]), 64 tenants sharded over {world} GPUs "
                                f"(LPT by prompt length), weights replicated") + ", fp16 paged KV",
                   "tenants": nt * world, "tenants_per_gpu": nt,
                   "prompt_lens": [int(x) for x in lens] if world == 1 else None,
                   "parallelism": f"tenant-sharded x{world}",
                   "l2": "weights 3.9 GB per step > 126 MB L2 (no flush needed)"},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * (2 + 3 * 64),
                "d2h_bytes_per_step": 8 * nt},
        "gpu_launches": launches,
        "roofline": roof,
        "attention": attn,
        "gemv_sweep": sweep,
        "decode_step": decode_step_line(step_bytes, step_ms, prof_ms, hbm_peak, nt),
        "clocks": clk.summary(),
    }
    if host_w is not None:
        try:
            line["cpu_baseline"] = cpu_baseline(host_w, os.cpu_count() or 1)
        except Exception as e:  # a baseline failure must not hide the GPU number
            line["cpu_baseline"] = {"error": str(e)[:200]}
        for key, fn in (("cpu_sweep", cpu_sweep), ("cpu_config2_attention", cpu_attention_config2),
                        ("cpu_config1_tinyllama", cpu_tinyllama_config1)):
            try:
                line[key] = fn(os.cpu_count() or 1)
            except Exception as e:
                line[key] = {"error": str(e)[:200]}
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def run_reference(args):
    """The reference arm: the oracle (C++ restatement of the reference's CPU
    path; the Rust reference cannot be built here) on all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(3)
    H, Q, KV, F, V = CFG["hidden"], CFG["n_heads"] * CFG["head_dim"], CFG["n_kv_heads"] * CFG["head_dim"], \
        CFG["ffn"], CFG["vocab"]

    def qt(dt, rows, cols):
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        x *= 0.02
        return dt, O.quantize(dt, x)

    W = {(O.W_TOKEN_EMBD, -1): qt(O.Q4K, V, H), (O.W_OUTPUT_NORM, -1): (O.F32, np.ones(H, np.float32)),
         (O.W_OUTPUT, -1): qt(O.Q6K, V, H)}
    for l in range(CFG["n_layers"]):
        W[(O.W_ATTN_NORM, l)] = (O.F32, np.ones(H, np.float32))
        W[(O.W_FFN_NORM, l)] = (O.F32, np.ones(H, np.float32))
        for which, r, c, dt in [(O.W_Q, Q, H, O.Q4K), (O.W_K, KV, H, O.Q4K), (O.W_V, KV, H, O.Q6K),
                                (O.W_O, H, Q, O.Q4K), (O.W_GATE, F, H, O.Q4K), (O.W_UP, F, H, O.Q4K),
                                (O.W_DOWN, H, F, O.Q4K)]:
            W[(which, l)] = qt(dt, r, c)
    om = O.Model(dict(CFG, kv_fp16=1), W, threads=threads)
    om.kv_fill(448, seed=0)
    pos = 448
    for _ in range(min(args.warmup, 3)):
        om.forward([1], pos)
        pos += 1
    k = max(1, min(args.steps, 4))
    t0 = time.perf_counter()
    for _ in range(k):
        om.forward([1], pos)
        pos += 1
    dt = time.perf_counter() - t0
    v = k / dt
    sample = (f"{k} single-token decode forwards of one tenant at ctx ~448 (oracle restatement of the reference CPU "
              f"path: dequant + fp32 GEMV, {threads} threads); the reference serves tenants one token at a time, so "
              f"aggregate tok/s over tenants equals this rate")
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s",
                      "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": k, "warmup": min(args.warmup, 3),
                      "ms_per_step": round(dt / k * 1e3, 2), "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic (numpy N(0,0.02), seed 3)",
                      "config": {"workload": "Llama-2-7B Q4_K_M decode (configs[3]), one tenant-token per sample"},
                      "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                      "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                                       "sample": sample}}), flush=True)


def run_case(args):
    """Small workloads for ncu captures (no timing, no JSON line).
    attn: 6 calls of the config-2 paged attention (16 tenants, GQA 4, hd 128,
    contexts U[512, 8192], 0.3 GB of fp16 K/V).
    gemv: 8 launches of the Q4_K gate|up GEMV (22016 x 4096, M = 8) over 8
    weight copies (400 MB, > L2). decode: the bench model, 8 tenants with
    caches of U[128, 512] random entries, then 3 decode steps of 66 launches each.
    serve: continuous batching through the scheduler (run_serve); prints a JSON line."""
    import torch
    import realm_b200 as rb
    dev = torch.device("cuda", 0)
    ctx = rb.Context(0)
    if args.case == "attn":
        # config 2 (as attention_roofline): 6 calls of the paged attention kernel
        rng = np.random.default_rng(2)
        n_t, hq, hkv, hd = 16, 32, 8, 128
        ctxs = rng.integers(512, 8193, n_t)
        pool = ctx.kv_pool(1, hkv, hd, rb.F16, n_pages=int(sum((c + 17) // 16 for c in ctxs)) + 16,
                           max_tenants=n_t, max_seq=8208)
        pool.shuffle(2)
        for t in range(n_t):
            pool.create(t)
            pool.append(t, 0, torch.randn(int(ctxs[t]), hkv * hd, device=dev),
                        torch.randn(int(ctxs[t]), hkv * hd, device=dev))
        q = torch.randn(n_t, hq * hd, device=dev)
        out = torch.empty(n_t, hq * hd, device=dev)
        for _ in range(6):
            pool.attention_forward(0, list(range(n_t)), q, hq, 1 / np.sqrt(hd),
                                   positions=[int(c) - 1 for c in ctxs], out=out)
        torch.cuda.synchronize(dev)
        print("attn case done", flush=True)
        return
    if args.case == "chunk":
        run_chunk_attn(rb, torch, dev)
        return
    if args.case == "gemv":
        n, k, m = 2 * CFG["ffn"], CFG["hidden"], TENANTS_PER_GPU
        ws = []
        for i in range(8):
            x = torch.randn(n, k, device=dev).mul_(0.02)
            blk = torch.empty(n * k // 256 * 144, dtype=torch.uint8, device=dev)
            ctx.quantize(rb.Q4_K, x.view(-1), blk)
            ws.append(rb.Weight(ctx, rb.Q4_K, n, k, blk))
            del x
        xs = torch.randn(m, k, device=dev)
        y = torch.empty(m, n, device=dev)
        for w in ws:
            w.matmul(xs, m, out=y)
        torch.cuda.synchronize(dev)
        print("gemv case done", flush=True)
        return
    if args.case == "serve":
        run_serve(rb, torch, ctx, dev)
        return
    if args.case == "serve_sampled":
        run_serve(rb, torch, ctx, dev, sampling=rb.SamplingParams(0.8, 0.9, 40, 1.1))
        return
    if args.case == "load":
        run_load(rb, torch, ctx, dev)
        return
    if args.case == "sample":
        run_sample(rb, torch, ctx, dev)
        return
    if args.case == "llama70b":
        run_llama70b(rb, torch, ctx, dev, args)
        return
    if args.case == "qgemm":
        # the tcgen05 dequant-GEMM (opt-in path): 8 launches of a 4096 x 4096 Q4_K
        # weight over 8 copies (75 MB > L2), 64 rows
        ctx.close()
        os.environ["RB_QGEMM"] = "1"
        qctx = rb.Context(0)
        n, k, m = 4096, 4096, 64
        ws = []
        for i in range(8):
            x = torch.randn(n, k, device=dev).mul_(0.02)
            blk = torch.empty(n * k // 256 * 144, dtype=torch.uint8, device=dev)
            qctx.quantize(rb.Q4_K, x.view(-1), blk)
            ws.append(rb.Weight(qctx, rb.Q4_K, n, k, blk))
        xs = torch.randn(m, k, device=dev)
        y = torch.empty(m, n, device=dev)
        for w in ws:
            w.matmul(xs, m, out=y)
        torch.cuda.synchronize(dev)
        print("qgemm case done", flush=True)
        return
    base = dict(CFG, n_layers=args.layers) if args.layers else CFG
    m = build_model(rb, torch, ctx, dev, TENANTS_PER_GPU, base=base)
    rng = np.random.default_rng(4)
    lens = rng.integers(128, 513, TENANTS_PER_GPU)
    kvw = CFG["n_kv_heads"] * CFG["head_dim"]
    for t in range(TENANTS_PER_GPU):  # caches filled directly (K/V ~ N(0,1)) instead of a prefill
        m.tenant_create(t)
        for l in range(base["n_layers"]):
            m.kv.append(t, l, torch.randn(int(lens[t]), kvw, device=dev), torch.randn(int(lens[t]), kvw, device=dev))
    tenants = np.arange(TENANTS_PER_GPU, dtype=np.uint32)
    tok = tenants.copy()
    for s in range(3):
        _, tok = m.forward_rows(tenants, tok, want_logits=False)
        print("decode step", s, ctx.last_forward_launches(), "launches", flush=True)


def run_chunk_attn(rb, torch, dev, ctx_len=4032, rows=64, reps=7):
    """Prompt-chunk attention: one tenant whose fp16 cache holds ctx_len
    N(0,1) entries, a rows-long chunk at the next positions (GQA 8, hd 128, the
    configs[4] heads), through rb_attention_forward on device buffers. Median
    device us of the prompt-chunk kernel (grouped rows) against one decode pair
    per row (RB_ATTN_GROUP=0), and the K/V bytes each requests (the per-row
    pairs of one tenant mostly hit L2). Prints one JSON line."""
    out = {}
    for n_heads, n_kv in ((64, 8),):
        hd = 128
        res = {}
        for grouped in (1, 0):
            os.environ["RB_ATTN_GROUP"] = str(grouped)
            ctx = rb.Context(0)
            del os.environ["RB_ATTN_GROUP"]
            n_pages = (ctx_len + rows) // 16 + 2
            pool = ctx.kv_pool(1, n_kv, hd, rb.F16, n_pages=n_pages, max_tenants=1, max_seq=ctx_len + rows)
            pool.shuffle(3)
            pool.create(0)
            g = torch.Generator(device=dev)
            g.manual_seed(7)
            pool.append(0, 0, torch.randn(ctx_len + rows, n_kv * hd, generator=g, device=dev),
                        torch.randn(ctx_len + rows, n_kv * hd, generator=g, device=dev))
            q = torch.randn(rows, n_heads * hd, generator=g, device=dev)
            o = torch.empty(rows, n_heads * hd, device=dev)
            pos = list(range(ctx_len, ctx_len + rows))
            ms = []
            for _ in range(reps):
                pool.attention_forward(0, [0] * rows, q, n_heads, 1 / np.sqrt(hd), positions=pos, out=o)
                ms.append(ctx.last_forward_ms())
            res["chunk_kernel" if grouped else "per_row_pairs"] = round(float(np.median(ms[2:])) * 1e3, 1)
            ctx.close()
        pages = (ctx_len + rows) // 16
        out[f"gqa{n_heads // n_kv}"] = {
            "us": res, "kv_MB_per_kv_head_tile": round(pages * 16 * hd * 2 * 2 / 1e6, 2),
            "kv_MB_read": {"chunk_kernel": round(n_kv * (rows * n_heads // n_kv // 64) * pages * 8192 / 1e6, 1),
                           "per_row_pairs": round(n_kv * rows * pages * 8192 / 1e6, 1)}}
    print(json.dumps({"case": "chunk_attention", "ctx": ctx_len, "rows": rows, "hd": 128, "results": out}),
          flush=True)


CFG70B = dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=32000,
              max_seq=4096, rms_eps=1e-5, layer_eps=1e-5, rope_theta=10000.0)


def run_llama70b(rb, torch, ctx, dev, args):
    """Llama-2-70B shape (80 layers, hidden 8192, 64 q / 8 kv heads
    of 128, FFN 28672, vocab 32000), random-init N(0, 0.02) weights quantised
    to Q4_K_M on the device (about 40 GB), 16 tenants with fp16 paged KV.
    Decode: every tenant's cache holds 3840 random entries (the prompt's K/V
    stand-in), then 16-row decode steps are timed (CUDA events over the graph
    replays). Prefill: one tenant's 3840-token prompt in 64-row steps, timed.
    Prints one JSON line."""
    hbm_peak, peak_kind = peaks()
    nt, prompt = 16, 3840
    m = build_model(rb, torch, ctx, dev, nt, base=CFG70B)
    kvw = CFG70B["n_kv_heads"] * CFG70B["head_dim"]
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    for t in range(nt):
        m.tenant_create(t)
        for l in range(CFG70B["n_layers"]):
            m.kv.append(t, l, torch.randn(prompt, kvw, generator=g, device=dev),
                        torch.randn(prompt, kvw, generator=g, device=dev))
    tenants = np.arange(nt, dtype=np.uint32)
    tok = np.random.default_rng(5).integers(0, CFG70B["vocab"], nt).astype(np.uint32)
    for _ in range(3):
        _, tok = m.forward_rows(tenants, tok, want_logits=False)
    steps = max(4, min(args.steps, 32))
    dev_ms = 0.0
    with Clocks(0) as clk:
        for _ in range(steps):
            _, tok = m.forward_rows(tenants, tok, want_logits=False)
            dev_ms += ctx.last_forward_ms()
    step_ms = dev_ms / steps
    prof_ms, _ = m.forward_profile(tenants, tok)
    ctx_mean = prompt + 3 + steps / 2
    wb = weight_bytes(CFG70B)
    kvb = nt * ctx_mean * CFG70B["n_layers"] * 2 * kvw * 2
    # prefill: one more tenant-sized prompt through 64-row steps (the cache of
    # tenant 0 is reset and refilled by the prompt itself)
    m.tenant_reset(0)
    ids = np.random.default_rng(55).integers(0, CFG70B["vocab"], prompt).astype(np.uint32)
    torch.cuda.synchronize(dev)
    pre_ms = 0.0
    for cs in range(0, prompt, 64):
        m.forward_rows([0] * 64, ids[cs:cs + 64], want_logits=False)
        pre_ms += ctx.last_forward_ms()
    # one more 64-row chunk (positions 3840..3903) run kernel by kernel: where a deep chunk's time goes
    pre_prof, _ = m.forward_profile([0] * 64, np.random.default_rng(56).integers(0, CFG70B["vocab"], 64).astype(np.uint32))
    line = {"metric": "configs[4] Llama-2-70B Q4_K_M decode tok/s (16 tenants, ctx 3840+)", "unit": "tok/s",
            "value": round(nt / (step_ms * 1e-3), 1), "ms_per_step": round(step_ms, 3), "steps": steps,
            "decode_step": {"bytes_per_step": int(wb + kvb), "weight_bytes": int(wb), "kv_bytes": int(kvb),
                            "achieved_GBps": round((wb + kvb) / (step_ms * 1e-3) / 1e9, 1),
                            "frac": round((wb + kvb) / (step_ms * 1e-3) / 1e9 / hbm_peak, 4),
                            "peak": hbm_peak, "peak_kind": peak_kind,
                            "kernel_ms_serialised": {k: round(v, 3) for k, v in prof_ms.items()}},
            "prefill": {"tokens": prompt, "rows_per_step": 64, "ms": round(pre_ms, 1),
                        "tok_per_s": round(prompt / (pre_ms * 1e-3), 1),
                        "path": "tcgen05" if ctx.uses_tcgen05(64) else "mma.sync",
                        "chunk_ms_serialised": {k: round(v, 3) for k, v in pre_prof.items()}},
            "config": {"workload": "Llama-2-70B shape, random-init Q4_K_M (attn_v, output Q6_K), 16 tenants, "
                                   "fp16 paged KV, caches of 3840 N(0,1) entries; prefill of a 3840-token prompt",
                       "weights_GB": round(wb / 1e9, 2)},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def run_serve(rb, torch, ctx, dev, n_req=96, max_batch=32, max_tokens=128, sampling=None):
    """Continuous batching through rb_scheduler on the bench model: n_req
    requests (prompts U[128, 512] from seed 5) all queued at t = 0, at most
    max_batch live, max_tokens each. Every step is one rb_forward over the live
    requests' decode rows plus prompt chunks that fill the 64-row budget.
    Prints one JSON line: generated tok/s by the wall clock around the whole
    run (host scheduling, copies and prefill included) and by summed device time."""
    import time
    m = build_model(rb, torch, ctx, dev, max_batch)
    rng = np.random.default_rng(5)
    lens = rng.integers(128, 513, n_req)
    # warm-up: capture the decode-step graph of every row count 1..64 once
    m.tenant_create(0)
    used = 0
    for r in range(1, 65):
        if used + r > CFG["max_seq"]:
            m.tenant_reset(0)
            used = 0
        m.forward_rows([0] * r, rng.integers(0, CFG["vocab"], r).astype(np.uint32), want_logits=False)
        used += r
    m.tenant_reset(0)
    s = rb.Scheduler(m, max_batch_size=max_batch)
    st0 = s.stats()
    for i in range(n_req):
        s.submit(i, rng.integers(0, CFG["vocab"], int(lens[i])).tolist(), max_tokens, sampling=sampling, seed=i)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    with Clocks(0) as clk:
        out = s.run()
    wall = time.perf_counter() - t0
    st = s.stats()
    steps = st["steps"] - st0["steps"]
    gen = st["tokens_generated"] - st0["tokens_generated"]
    dev_ms = st["device_ms"] - st0["device_ms"]
    assert gen == n_req * max_tokens and all(len(v) == max_tokens for v in out.values())
    line = {
        "metric": "serve_generated_tok_per_s" + ("_sampled" if sampling else ""), "value": round(gen / wall, 1),
        "unit": "tok/s",
        "sampling": None if sampling is None else vars(sampling),
        "device_tok_per_s": round(gen / (dev_ms * 1e-3), 1),
        "prompt_tok_per_s": round(int(lens.sum()) / wall, 1),
        "steps": steps, "rows_per_step": round((st["rows"] - st0["rows"]) / steps, 2),
        "prefill_rows": st["prefill_rows"] - st0["prefill_rows"], "decode_rows": st["decode_rows"] - st0["decode_rows"],
        "wall_s": round(wall, 3), "device_s": round(dev_ms * 1e-3, 3),
        "config": {"workload": f"Llama-2-7B Q4_K_M, {n_req} requests, prompts U[128,512], {max_tokens} tokens each, "
                               f"<= {max_batch} live, fp16 paged KV", "data": "synthetic, random-init weights"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    s.close()


def run_load(rb, torch, ctx, dev):
    """GGUF load of the bench model: the weights are generated on the device,
    written once as a llama-architecture GGUF file, then opened (parse + mmap)
    and loaded with rb_model_load_gguf (upload + re-tiling) while timed. The file
    is in the page cache after the write, so this is the host-to-device path,
    not the disk. Prints one JSON line."""
    import sys
    import tempfile
    import time
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests"))
    import gguf_writer as GW
    host = {}
    m = build_model(rb, torch, ctx, dev, 8, host_copy=host)
    m.close()
    cfg = dict(CFG)
    blob = GW.model_gguf(cfg, host)
    del host
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "llama7b_q4km.gguf")
        with open(path, "wb") as f:
            f.write(blob)
        nbytes = len(blob)
        del blob
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            g = rb.GGUFFile(path)
            t1 = time.perf_counter()
            mg = g.load_model(ctx, max_tenants=8)
            torch.cuda.synchronize(dev)
            t2 = time.perf_counter()
            times.append((t1 - t0, t2 - t1))
            mg.close()
            g.close()
    parse_s, load_s = min(times, key=lambda x: x[0] + x[1])
    print(json.dumps({"metric": "gguf_load_GBps", "value": round(nbytes / (parse_s + load_s) / 1e9, 2),
                      "unit": "GB/s", "file_bytes": nbytes, "parse_s": round(parse_s, 4), "load_s": round(load_s, 3),
                      "runs": [[round(a, 4), round(b, 3)] for a, b in times],
                      "config": {"workload": "Llama-2-7B Q4_K_M GGUF (synthetic weights) from the page cache"}}),
          flush=True)


def run_sample(rb, torch, ctx, dev, n_rows=64, vocab=32000):
    """Fused sampling on the device: 64 logits rows of the Llama vocabulary,
    top-k 40 + top-p 0.9 + temperature 0.8 + repetition penalty 1.1 over 64
    previous tokens per row, timed with CUDA events over 50 launches on the
    context stream (device pointers). Prints one JSON line."""
    import ctypes as C
    from realm_b200 import sampling as S
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    lg = torch.randn(n_rows, vocab, generator=g, device=dev).mul_(3.0)
    params = S._params_array([rb.SamplingParams(0.8, 0.9, 40, 1.1)] * n_rows)
    dparams = torch.frombuffer(bytearray(bytes(params)), dtype=torch.uint8).to(dev)
    prev = torch.randint(0, vocab, (n_rows * 64,), generator=g, device=dev, dtype=torch.int32)
    off = torch.arange(0, n_rows * 64 + 1, 64, device=dev, dtype=torch.int32)
    uni = torch.rand(n_rows, generator=g, device=dev)
    out = torch.empty(n_rows, device=dev, dtype=torch.int32)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)

    def call():
        r = rb.lib().rb_sample_logits(ctx.handle, lg.data_ptr(), vocab, n_rows, vocab, dparams.data_ptr(),
                                      prev.data_ptr(), off.data_ptr(), uni.data_ptr(), out.data_ptr(), rb.PTR_DEVICE)
        assert r == n_rows, rb.last_error()
    for _ in range(5):
        call()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    for _ in range(50):
        call()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    us = ev0.elapsed_time(ev1) * 1e3 / 50
    print(json.dumps({"metric": "sample_us_per_call", "value": round(us, 2), "unit": "us", "rows": n_rows,
                      "vocab": vocab, "strategy": "T 0.8, top-k 40, top-p 0.9, penalty 1.1 over 64 tokens",
                      "note": "each call includes its host synchronisation and the 256-byte token copy back"}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--layers", type=int, default=0,
                    help="decode case only: build the 7B model with this many layers (small ncu captures)")
    ap.add_argument("--case", choices=["gemv", "decode", "attn", "chunk", "serve", "serve_sampled", "load", "sample", "qgemm",
                             "llama70b"],
                    help="profiling case for ncu: run a small workload of one kernel family and exit")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
