"""Benchmark of the B200 INT8 KV-cache decode path.

Default workload: one full decode step over the model's
8 full-attention layers for 128 sequences at 32768 cached tokens each
(16 Q / 4 KV heads, head_dim 128).  Per layer a step appends one token per
sequence (quantize-on-append) and then runs split-K decode attention.  The
128 sequences are sharded by sequence across ranks with no collective.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3|1|2|4]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference     # the reference's CPU code on the host

Config 4 (one 1,048,576-token sequence split along context) runs a partial
(m, l, O) per rank; at N > 1 the ranks exchange and merge the partials in one
kernel over NVLink peer memory (``--cp-nccl``: an NCCL all-gather plus the
log-sum-exp combine kernel instead).  Config 5 is the chunked prefill,
``--kv-fp32`` the fp32-cache decode.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "echo-core_b200"))

import ranks  # noqa: E402
import workloads as W  # noqa: E402

METRIC = "INT8-KV decode attention HBM GB/s (% of peak) and decode tok/s at 32k ctx"
D = 128
HKV = 4
H = 16
BYTES_PER_TOKEN = W.kv_bytes_per_token(HKV, D)  # 1056: K+V codes + K/V scales, per layer


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic():
    """dram bytes per decode launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------ CPU legs
class CpuDecode:
    """Single-sequence decode steps at `ctx` on the host (setup once, time steps).

    use_ref: the reference's own InferenceEngine::attention (oracle/_ref), one
    engine per thread, each holding one copy of the cache, run through the
    reference's weight-absent branch so that the Q/K/V/O matvecs around the
    loop are not timed (src/inference.cpp:313-319,410-411); else the C
    restatement (oracle/liboracle.so) on one thread."""

    def __init__(self, ctx, threads, use_ref):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        self.O, self.ctx, self.threads, self.use_ref = O, ctx, threads, use_ref
        rng = np.random.default_rng(2)
        self.kq, self.ks = O.quantize_kv(W.kv_rows(rng, ctx, HKV, D), HKV, D)
        self.vq, self.vs = O.quantize_kv(W.kv_rows(rng, ctx, HKV, D), HKV, D)
        self.q = W.queries(rng, 1, H, D)[0]
        self.engines = []
        if use_ref:
            for _ in range(threads):
                e = O.RefAttention(H, HKV, D, ctx + 1, projections=False)
                e.load(self.kq, self.vq, self.ks, self.vs, ctx)
                self.engines.append(e)

    def run(self, n_units):
        """Seconds for n_units decode steps."""
        O = self.O
        if not self.use_ref:
            t0 = time.perf_counter()
            for _ in range(n_units):
                O.decode_attention(self.kq, self.vq, self.ks, self.vs, self.ctx, self.q, H, HKV,
                                   D, W.softmax_scale(D))
            return time.perf_counter() - t0
        from concurrent.futures import ThreadPoolExecutor
        T = self.threads

        def work(i):
            e = self.engines[i]
            out = np.zeros(H * D, np.float32)
            for _ in range(n_units // T + (1 if i < n_units % T else 0)):
                e.step(self.q, out)

        t0 = time.perf_counter()
        with ThreadPoolExecutor(T) as ex:
            list(ex.map(work, range(T)))
        return time.perf_counter() - t0

    def close(self):
        for e in self.engines:
            e.close()


def cpu_baseline_line(ctx=32768, units=None):
    units = units or int(os.environ.get("EC_CPU_UNITS", "96"))
    cd = CpuDecode(ctx, 1, use_ref=False)
    dt = cd.run(units)
    gbs = units * ctx * BYTES_PER_TOKEN / dt / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{units} single-sequence decode steps (one layer) at ctx {ctx}, "
                      f"16 Q / 4 KV heads, d 128; {dt:.1f} s on 1 host core"}


def run_reference_arm(args, rank):
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    threads = max(1, min(threads, int(os.environ.get("EC_REF_THREADS", "64"))))
    ctx = 32768
    use_ref = O.ref_available()
    kind = "reference" if use_ref else "port"
    if not use_ref:
        threads = 1
    per_step_units = int(os.environ.get("EC_REF_UNITS", str(threads)))
    cd = CpuDecode(ctx, threads, use_ref)
    for _ in range(args.warmup):
        cd.run(threads)
    times = [cd.run(per_step_units) for _ in range(args.steps)]
    cd.close()
    dt = sum(times)
    gbs = args.steps * per_step_units * ctx * BYTES_PER_TOKEN / dt / 1e9
    ms = dt / args.steps * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "cfg3_decode_8layers_128x32k", "sample_units_per_step": per_step_units,
                   "ctx": ctx, "q_heads": H, "kv_heads": HKV, "head_dim": D},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{per_step_units} (sequence, layer) decode steps of config 3 "
                                   f"per step on {threads} host threads, "
                                   + ("the reference's InferenceEngine::attention (oracle/_ref), "
                                      "projections excluded: its weight-absent branch skips the "
                                      "Q/K/V/O matvecs; the attention loop and the append are timed"
                                      if use_ref else "C restatement (oracle)")},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def fill_layer(torch, eckv, bc, lens, gen, chunk_tokens=1 << 20):
    """Fills a BatchCache's slabs with quantized N(0,1)+outlier K/V (setup)."""
    stream = torch.cuda.current_stream()
    for s, L in enumerate(lens):
        off = int(bc.offsets_host[s])
        done = 0
        while done < L:
            n = min(chunk_tokens, L - done)
            for dst_codes, dst_scales in ((bc.keys, bc.key_scales), (bc.values, bc.val_scales)):
                x = torch.randn((n, HKV, D), generator=gen, device="cuda", dtype=torch.float32)
                x[:, :, list(W.OUTLIER_CHANNELS)] *= W.OUTLIER_FACTOR
                slot = off + done
                codes = dst_codes[slot:slot + n]
                scales = dst_scales[slot * HKV:(slot + n) * HKV]
                eckv.quantize_per_token_symmetric(x, codes, scales, n * HKV, D, stream)
            done += n
    bc.length.copy_(torch.tensor(lens, dtype=torch.int32, device="cuda"))


def run_gpu_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import eckv
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfgn = args.config
    cfg = W.config(cfgn)
    if args.seqs:
        cfg.ctx = (cfg.ctx * ((args.seqs + len(cfg.ctx) - 1) // len(cfg.ctx)))[:args.seqs]
        cfg.num_seqs = args.seqs
        cfg.name += f"_seqs{args.seqs}"
    if args.layers:
        cfg.num_layers = args.layers
        cfg.name += f"_layers{args.layers}"
    if args.ctx:
        cfg.ctx = [args.ctx] * len(cfg.ctx)
        cfg.name += f"_ctx{args.ctx}"
    if args.kv_fp32:
        return run_f32_arm(args, rank, world, local_rank, cfg)
    if cfgn == 4:
        return run_cp_arm(args, rank, world, local_rank)
    if cfgn == 5:
        return run_prefill_arm(args, rank, world, local_rank)
    # ---- shard sequences
    nseq_total = cfg.num_seqs
    # contiguous blocks balanced by cached tokens (equal blocks for equal lengths)
    lo, hi = ranks.shard_weighted(cfg.ctx[:nseq_total], rank, world)
    lens0 = cfg.ctx[lo:hi]
    nseq = hi - lo
    layers = cfg.num_layers
    new_tok = 1
    # capacities, grid bound and split-K token hint (shared with the parity
    # test at this size, so that both run the same plan)
    caps, max_len, hint = W.decode_bench_batch(lens0, args.warmup, args.steps, new_tok)
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed * 1000 + rank)
    caches = []
    for _ in range(layers):
        bc = eckv.BatchCache(caps, num_kv_heads=HKV, device=dev, max_seq_len=max_len)
        fill_layer(torch, eckv, bc, lens0, gen)
        caches.append(bc)
    q = torch.randn((layers, nseq, H, D), generator=gen, device=dev)
    kn = torch.randn((layers, nseq, HKV * D), generator=gen, device=dev)
    vn = torch.randn((layers, nseq, HKV * D), generator=gen, device=dev)
    out = torch.empty((layers, nseq, H, D), device=dev)
    for bc in caches:
        # host estimate of the cached tokens at the timed decodes: sizes the
        # split-K plan for ragged batches (config 2)
        bc.tokens_hint = hint
        bc.workspace(H)
    torch.cuda.synchronize()
    scale = W.softmax_scale(D)
    stream = torch.cuda.current_stream()
    d0 = caches[0].desc()
    plan_chunks = eckv.lib().ec_decode_workspace_size_batch(ctypes.byref(d0), H)
    # append (its length bump folded in for one new token), decode, split-K merge
    launches_per_layer = (1 if new_tok == 1 else 2) + 1 + (1 if plan_chunks > 0 else 0)

    def step(ev=None, st=None):
        st = st or stream
        for l, bc in enumerate(caches):
            bc.append(kn[l], vn[l], 1, st)
            if ev is not None:
                ev[l][0].record(st)
            bc.decode(q[l], out[l], H, scale, st)
            if ev is not None:
                ev[l][1].record(st)

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    sync_all()
    for bc in caches:
        assert bc.device_error() == 0
    # bytes of the timed steps: per layer, every cached token after the append
    lens_t = np.asarray(lens0, dtype=np.int64)
    bytes_steps = 0
    for k in range(args.steps):
        cur = lens_t + (args.warmup + k + 1) * new_tok
        bytes_steps += layers * int(cur.sum()) * BYTES_PER_TOKEN
    qo_bytes = 2 * nseq * H * D * 4
    dec_events = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(layers)]
                  for _ in range(args.steps)]
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    sync_all()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    graph = None
    if args.graph:
        # the step's launches captured once and replayed: the timed region then
        # holds no host launch gaps (the kernels read the device length table,
        # so every replay appends and attends at the next position).  The
        # per-launch decode timing comes from an eager pass of the same steps.
        for k in range(args.steps):
            step(dec_events[k])
        torch.cuda.synchronize()
        for bc in caches:
            bc.length.sub_(args.steps * new_tok)
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step(st=side)              # uncaptured run on the capture stream
        torch.cuda.synchronize()
        for bc in caches:
            bc.length.sub_(new_tok)
        with torch.cuda.graph(graph, stream=side):
            step(st=torch.cuda.current_stream())
        torch.cuda.synchronize()
        sync_all()
        t_start.record(stream)
        for k in range(args.steps):
            graph.replay()
        t_end.record(stream)
    else:
        t_start.record(stream)
        for k in range(args.steps):
            step(dec_events[k])
        t_end.record(stream)
    torch.cuda.synchronize()
    ms = t_start.elapsed_time(t_end)
    clk = clocks.stop() if clocks else None
    dec_ms = [dec_events[k][l][0].elapsed_time(dec_events[k][l][1])
              for k in range(args.steps) for l in range(layers)]
    for bc in caches:
        assert bc.device_error() == 0
    # max over ranks
    t = torch.tensor([ms, float(bytes_steps), float(np.mean(dec_ms))], dtype=torch.float64, device=dev)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax[:1], op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum[1:2], op=dist.ReduceOp.SUM)
        ms_max, total_bytes = float(tmax[0]), float(tsum[1])
    else:
        ms_max, total_bytes = ms, float(bytes_steps)

    # ---- e2e: same step through the C ABI from pinned host buffers
    e2e = None
    if not args.no_e2e:
        q_h = torch.empty((layers, nseq, H, D), pin_memory=True)
        kn_h = torch.empty((layers, nseq, HKV * D), pin_memory=True)
        vn_h = torch.empty((layers, nseq, HKV * D), pin_memory=True)
        out_h = torch.empty((layers, nseq, H, D), pin_memory=True)
        q_h.copy_(q.cpu()); kn_h.copy_(kn.cpu()); vn_h.copy_(vn.cpu())
        # roll lengths back so the e2e run sees the same contexts
        for bc in caches:
            bc.length.sub_(args.steps * new_tok)
        sync_all()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        # Copies overlap the kernels on two copy streams: layer l's inputs go
        # up while earlier layers attend, and its output comes down while
        # later layers attend.  Events order each buffer's reuse.
        up, down = torch.cuda.Stream(), torch.cuda.Stream()
        consumed = [None] * layers    # decode of layer l done with q/kn/vn[l]
        read = [None] * layers        # out[l] copied down
        e0.record(stream)
        up.wait_event(e0)
        for k in range(args.steps):
            for l, bc in enumerate(caches):
                if consumed[l] is not None:
                    up.wait_event(consumed[l])
                with torch.cuda.stream(up):
                    q[l].copy_(q_h[l], non_blocking=True)
                    kn[l].copy_(kn_h[l], non_blocking=True)
                    vn[l].copy_(vn_h[l], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(up)
                stream.wait_event(ready)
                if read[l] is not None:
                    stream.wait_event(read[l])
                bc.append(kn[l], vn[l], 1, stream)
                bc.decode(q[l], out[l], H, scale, stream)
                done = torch.cuda.Event()
                done.record(stream)
                consumed[l] = done
                down.wait_event(done)
                with torch.cuda.stream(down):
                    out_h[l].copy_(out[l], non_blocking=True)
                read[l] = torch.cuda.Event()
                read[l].record(down)
        for l in range(layers):
            stream.wait_event(read[l])
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        te = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        h2d = (q_h.numel() + kn_h.numel() + vn_h.numel()) * 4
        d2h = out_h.numel() * 4
        if world > 1:
            hb = torch.tensor([float(h2d), float(d2h)], dtype=torch.float64, device=dev)
            dist.all_reduce(hb, op=dist.ReduceOp.SUM)
            h2d, d2h = int(hb[0]), int(hb[1])
        e2e = {"value": round(total_bytes / (float(te[0]) * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(float(te[0]) / args.steps, 4),
               "tok_s": round(nseq_total * args.steps / (float(te[0]) * 1e-3), 1),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    if rank != 0:
        return
    peak, peak_kind = peaks()
    gbs = total_bytes / (ms_max * 1e-3) / 1e9
    # roofline of the dominant kernel (decode, incl. its combine) on this rank
    dec_avg_ms = float(np.mean(dec_ms))
    lens_mid = lens_t + (args.warmup + 1) * new_tok
    alg_bytes = int(lens_mid.sum()) * BYTES_PER_TOKEN + qo_bytes
    achieved = alg_bytes / (dec_avg_ms * 1e-3) / 1e9
    tr = committed_traffic()
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: N(0,1) K/V with 4 outlier channels x8 per KV head, N(0,1) Q; "
                "quantized on device",
        "config": {"workload": cfg.name, "layers": layers, "seqs": nseq_total, "ctx": lens0[0],
                   "q_heads": H, "kv_heads": HKV, "head_dim": D,
                   "parallelism": f"sequence-shard x{world} (no collective)",
                   "launch": "CUDA graph replay" if args.graph else "eager",
                   "l2": "inputs larger than L2 (KV working set per step >> 126 MB)"},
        "tok_s": round(nseq_total * args.steps / (ms_max * 1e-3), 1),
        "pct_of_hbm_peak": round(100 * gbs / (peak * world), 1),
        # (the library's plan: stream-K for 32 to 1024 sequences a rank, else the chunked grid)
        "roofline": {"bound": "hbm",
                     "kernel": ("decode_sk_kernel" if 32 <= nseq <= 1024
                                else "decode_kernel") + "+combine_kernel",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "alg_bytes_per_launch": alg_bytes,
                     # measured DRAM bytes per cached token (ncu) x this launch's tokens
                     "traffic": (int(int(lens_mid.sum()) * tr["bytes_per_token_measured"])
                                 if tr and "bytes_per_token_measured" in tr else None)},
        "gpu_launches": launches_per_layer * layers * args.steps,
        "clocks": clk,
    }
    if e2e:
        line["e2e"] = e2e
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_line()
    print(json.dumps(line), flush=True)


def run_f32_arm(args, rank, world, local_rank, cfg):
    """Decode over the fp32 cache mode (use_kv_quantization = false): one
    sequence of 65,536 tokens (or --ctx) per rank through the cache object,
    16 Q / 4 KV heads; bytes = the K and V rows, 4096 per token (268 MB per
    rank, above L2)."""
    import torch
    import torch.distributed as dist
    import eckv
    dev = torch.device("cuda", local_rank)
    L = args.ctx or 65536
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed * 1000 + rank)
    c = eckv.KVCache(num_heads=H, num_kv_heads=HKV, head_dim=D, num_layers=1, max_seq_len=L,
                     use_kv_quantization=False)
    row = HKV * D
    # the cache's own append (a plain fp32 copy per token, src/kv_cache.cpp:106-110)
    kbuf = torch.randn((L, row), generator=gen, device=dev)
    vbuf = torch.randn((L, row), generator=gen, device=dev)
    for t in range(L):
        c.append(0, kbuf[t], vbuf[t])
    del kbuf, vbuf
    q = torch.randn((H, D), generator=gen, device=dev)
    out = torch.empty((H, D), device=dev)
    scale = W.softmax_scale(D)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        c.attention(0, q, out, scale, stream)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    graph = None
    if args.graph:
        # the attention call's launches (decode + merge) captured once and
        # replayed, as a serving loop would: no host launch gaps in the timing
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.graph(graph, stream=side):
            c.attention(0, q, out, scale, torch.cuda.current_stream())
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    else:
        e0.record(stream)
        for _ in range(args.steps):
            c.attention(0, q, out, scale, stream)
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del graph
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        peak, kind = peaks()
        nbytes = L * row * 4 * 2 * world
        gbs = nbytes * args.steps / (float(t[0]) * 1e-3) / 1e9
        print(json.dumps({
            "metric": "decode attention over the fp32 KV cache (use_kv_quantization=false) GB/s",
            "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(float(t[0]) / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic N(0,1) K/V/Q",
            "config": {"workload": f"fp32_cache_decode_ctx{L}", "ctx": L, "q_heads": H,
                       "kv_heads": HKV, "head_dim": D,
                       "launch": "CUDA graph replay" if args.graph else "eager"},
            "pct_of_hbm_peak": round(100 * gbs / (peak * world), 1), "peak_kind": kind}), flush=True)
    c.close()


def run_prefill_arm(args, rank, world, local_rank):
    """Config 5: 32 sequences each append a 4096-token chunk (quantize-on-append)
    onto an 8192-token int8 cache, then causal GQA attention of the chunk's
    bf16-cast queries over the cache on tcgen05.  Sequences are sharded across
    ranks with no collective.  Every step restores the 8192-token lengths first,
    so each step is the same workload."""
    import torch
    import torch.distributed as dist
    import eckv
    dev = torch.device("cuda", local_rank)
    cfg = W.config(5)
    nseq_total = args.seqs or cfg.num_seqs
    lo, hi = ranks.shard(nseq_total, rank, world)
    nseq = hi - lo
    past, n_new = cfg.ctx[0], cfg.new_tokens
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed * 1000 + rank)
    bc = eckv.BatchCache([past + n_new] * nseq, num_kv_heads=HKV, device=dev)
    fill_layer(torch, eckv, bc, [past] * nseq, gen)
    base_len = bc.length.clone()
    kn = torch.randn((nseq, n_new, HKV * D), generator=gen, device=dev)
    vn = torch.randn((nseq, n_new, HKV * D), generator=gen, device=dev)
    kn[:, :, :].view(nseq, n_new, HKV, D)[:, :, :, list(W.OUTLIER_CHANNELS)] *= W.OUTLIER_FACTOR
    vn[:, :, :].view(nseq, n_new, HKV, D)[:, :, :, list(W.OUTLIER_CHANNELS)] *= W.OUTLIER_FACTOR
    q = torch.randn((nseq, n_new, H, D), generator=gen, device=dev)
    out = torch.empty((nseq, n_new, H, D), device=dev)
    scale = W.softmax_scale(D)
    stream = torch.cuda.current_stream()
    ev = []

    def step(record=False):
        bc.length.copy_(base_len)
        if record:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record(stream)
        bc.append(kn, vn, n_new, stream)
        if record:
            e[1].record(stream)
        bc.prefill(q, out, n_new, H, scale, stream)
        if record:
            e[2].record(stream)
            ev.append(e)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    assert bc.device_error() == 0
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step(record=True)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    clk = clocks.stop() if clocks else None
    pre_ms = float(np.mean([e[1].elapsed_time(e[2]) for e in ev]))
    app_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    pairs = n_new * past + n_new * (n_new + 1) // 2
    flops_rank = 4.0 * D * pairs * H * nseq
    t = torch.tensor([ms, flops_rank], dtype=torch.float64, device=dev)
    if world > 1:
        tm = t.clone()
        dist.all_reduce(tm[:1], op=dist.ReduceOp.MAX)
        ts = t.clone()
        dist.all_reduce(ts[1:], op=dist.ReduceOp.SUM)
        ms_max, flops = float(tm[0]), float(ts[1])
    else:
        ms_max, flops = ms, flops_rank
    if rank != 0:
        return
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = float(pk.get("bf16_tflops_sustained", 1400.0))
    achieved = flops_rank / (pre_ms * 1e-3) / 1e12
    append_bytes = nseq * n_new * (2 * HKV * D * 4 + BYTES_PER_TOKEN)
    print(json.dumps({
        "metric": "chunked-prefill attention TFLOP/s over the int8 KV cache (config 5)",
        "value": round(flops * args.steps / (ms_max * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 (bf16-cast Q, exact int8 K/V codes), f16 hi/lo P, fp32 accumulate",
        "data": "synthetic", "config": {"workload": cfg.name, "seqs": nseq_total, "past": past,
                                          "new_tokens": n_new, "q_heads": H, "kv_heads": HKV,
                                          "head_dim": D, "flops_per_step": flops},
        "roofline": {"bound": "tensor", "kernel": "prefill_kernel", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_kind": "measured sustained" if pk else "fallback",
                     "note": "algorithmic FLOPs (QK^T and PV, causal); PV runs as two f16 MMAs (p' hi/lo)"},
        "append": {"kernel": "append_kernel+bump_lengths_kernel", "ms": round(app_ms, 4),
                   "gbs": round(append_bytes / (app_ms * 1e-3) / 1e9, 1),
                   "frac": round(append_bytes / (app_ms * 1e-3) / 1e9 / peaks()[0], 4),
                   "bytes": append_bytes, "bound": "hbm",
                   "note": "fp32 K/V rows read + int8 codes and scales written, per rank"},
        "gpu_launches": 3 * args.steps, "clocks": clk}), flush=True)


def run_cp_arm(args, rank, world, local_rank):
    """Config 4: 1,048,576-token sequence split contiguously across ranks;
    per-rank partial state, NCCL all-gather, log-sum-exp combine."""
    import torch
    import torch.distributed as dist
    import eckv
    dev = torch.device("cuda", local_rank)
    cfg = W.config(4)
    total = cfg.ctx[0]
    lo, hi = ranks.shard(total, rank, world)
    n = hi - lo
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed * 1000 + rank)
    bc = eckv.BatchCache([n], num_kv_heads=HKV, device=dev)
    fill_layer(torch, eckv, bc, [n], gen)
    q = torch.randn((1, H, D), generator=gen, device=dev)
    qg = q.clone()
    if world > 1:
        dist.broadcast(qg, 0)
    po_local = torch.empty((1, H, D), device=dev)
    pml_local = torch.empty((1, H, 2), device=dev)
    out = torch.empty((1, H, D), device=dev)
    scale = W.softmax_scale(D)
    stream = torch.cuda.current_stream()

    # N > 1: the decode kernel, then one kernel that merges this rank's split-K
    # chunks, exchanges the state over peer memory and merges the ranks (two
    # launches a step); --cp-unfused keeps the chunk merge as its own launch
    # before the exchange; --cp-nccl exchanges with an NCCL all-gather.
    # N = 1: the plain decode (decode + chunk merge).
    peer = world > 1 and not args.cp_nccl
    fused = peer and not args.cp_unfused
    # graph replay at one GPU; with ranks the step stays eager (measured at 2
    # GPUs: fused step 0.1061-0.1066 ms eager against 0.1099-0.1101 ms
    # replayed with device epochs; unfused 0.1157 against 0.1191 ms)
    use_graph = args.graph and world == 1
    cx = ranks.CPExchange(1, H) if peer else None
    # this library's kernels a step: decode (+ its split-K merge when the plan
    # splits), or decode + exchange (fused), or decode (+ merge) + exchange /
    # + ec_lse_combine (the NCCL all-gather between is NCCL's)
    split = 1 if bc.workspace(H)[1] > 0 else 0
    own_launches = 1 + split if world == 1 else 2 if fused else 2 + split

    def step():
        if world == 1:
            bc.decode(qg, out, H, scale, stream)
            return
        if fused:
            cx.decode_exchange(bc, qg, out, H, scale, stream)
            return
        bc.decode_partial(qg, po_local, pml_local, H, scale, stream)
        if peer:
            cx.combine(po_local, pml_local, out, stream)     # exchange + merge, one kernel
            return
        po, pml = ranks.gather_partials(po_local, pml_local)
        eckv.lse_combine(po, pml, world, 1, H, D, out, stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    graph = None
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        outer = stream
        with torch.cuda.graph(graph, stream=side):
            stream = torch.cuda.current_stream()
            step()
        stream = outer
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del graph
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        peak, kind = peaks()
        gbs = total * BYTES_PER_TOKEN * args.steps / (float(t[0]) * 1e-3) / 1e9
        print(json.dumps({
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(float(t[0]) / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": cfg.name, "ctx": total, "parallelism": f"context-split x{world}",
                       "exchange": ("chunk merge + peer stores + rank merge in one kernel "
                                    "(ec_cp_decode_exchange)" if fused else
                                    "peer stores + merge in one kernel (ec_cp_exchange_combine)"
                                    if peer else "NCCL all-gather + ec_lse_combine"
                                    if world > 1 else "none"),
                       "launch": "CUDA graph replay" if use_graph else "eager"},
            "gpu_launches": own_launches * args.steps,
            "pct_of_hbm_peak": round(100 * gbs / (peak * world), 1)}), flush=True)
    if cx is not None:
        cx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seqs", type=int, default=None,
                    help="override the sequence count (small profiling cases)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count")
    ap.add_argument("--ctx", type=int, default=None, help="override every sequence's context")
    ap.add_argument("--eager", action="store_true",
                    help="decode configs: launch every kernel from the host each step instead of "
                         "replaying the step as a captured CUDA graph")
    ap.add_argument("--cp-nccl", action="store_true",
                    help="config 4: exchange partials with an NCCL all-gather instead of peer stores")
    ap.add_argument("--cp-unfused", action="store_true",
                    help="config 4: merge each rank's split-K chunks in their own launch before "
                         "the peer exchange")
    ap.add_argument("--kv-fp32", action="store_true",
                    help="decode over the fp32 cache mode (one sequence per rank)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.graph = not args.eager
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank)
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_gpu_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
