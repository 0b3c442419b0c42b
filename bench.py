"""bench.py -- Qwen3.5-0.8B-shape Q4_K_M bs1 greedy decode at ctx 4k on B200.

Workload: a random-init Qwen3.5-0.8B-shaped hybrid
decoder in the Q4_K_M mix (hidden 1024, 24 layers = [GDN x3, ATT] x6, FFN 3584,
vocab 248320 tied Q6_K head), written as a synthetic GGUF; the KV cache and
R/S state are prefilled from 4096 seeded random tokens (untimed); each timed
step decodes one token (one CUDA-graph replay of the whole forward + LM-head
argmax).  Weights (513 MB) exceed L2 (126 MB), so no flush is needed.

  value  tokens/s over all GPUs (independent replicas, weak scaling), device-timed
  e2e    the same metric through the public C ABI with host buffers: per step
         kib_qwen35_forward() copies the token and position host->device and
         reads the argmax back (the reference's per-token loop)
  roofline  the dominant kernel, decode_persistent_kernel (one launch per
         token, with the embedding row gather before it): algorithmic bytes
         per token / device time per token, against the measured HBM copy peak
  matvec_config1  BASELINE config 1 on its own: the Q4_K 3584x1024 GEMV kernel
         over a rotating pool of weight copies > 4x L2
  cpu_baseline  the CPU oracle's decode step on the host cores (bounded sample)

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kib|reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "kraken-infer_b200"), os.path.join(ROOT, "tests")]

METRIC = "Qwen3.5-0.8B-shape Q4_K_M bs1 decode tok/s @ctx4k"
UNIT = "tok/s"
CONTEXT = 4096
WORKLOAD = "qwen35-0.8b-shape-q4_k_m-bs1-greedy-decode-ctx4096"
# HBM bytes per decoded token at ctx 4096 (algorithmic): weights 513.3 MB
# (24 layers 304.7 + Q6_K LM head 208.6), GDN S r+w 37.7, conv R r+w 2.7,
# KV read 50.3 (6 layers x 4096 x 2 heads x 256 x 2 B x K,V).
TOKEN_BYTES = 604.0e6
# DRAM bytes per token of decode_persistent_kernel from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of a 4-layer model: 70.51 MB
# read + 0.46 MB written against 72.44 MB algorithmic, scaled to the full model
# by algorithmic bytes, traffic/algorithmic = 0.980.
PK_TRAFFIC = 591.7e6  # 0.980 x 604 MB


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu):
        self.gpu = gpu
        self.samples = []
        self.stop = threading.Event()

    def _run(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        while not self.stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self.stop.wait(0.2)

    def __enter__(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 2 + i and s[2 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def dist_setup(n):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo")
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allmax(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


MODEL_OVERRIDES = {}


def model_path(rank, world):
    d = os.environ.get("KIB_BENCH_DIR", os.path.join(tempfile.gettempdir(), "kib_bench"))
    os.makedirs(d, exist_ok=True)
    tag = "".join(f"_{k}{v}" for k, v in sorted(MODEL_OVERRIDES.items()))
    return os.path.join(d, f"qwen35_0p8b_shape_q4_k_m_seed1234{tag}.gguf")


def ensure_model(path, rank, world):
    import kib
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".tmp"
        kib.write_synthetic_qwen35(tmp, threads=min(os.cpu_count() or 8, 64), seed=1234, **MODEL_OVERRIDES)
        os.replace(tmp, path)
    barrier(world)


def matvec_roofline(ctx, hbm_peak, reps=5, profile=False, qtype=None, rows=3584, cols=1024):
    """Config 1 (Q4_K 3584x1024, x ~ N(0,1)) over a rotating pool of distinct
    weight copies > 4x L2, launched back to back from one CUDA graph; CUDA
    events on the stream the kernels run on."""
    import numpy as np
    import torch
    import kib
    qtype = kib.Q4_K if qtype is None else qtype
    w = kib.quantize(qtype, (np.random.default_rng(1).standard_normal(rows * cols) * 0.02).astype(np.float32))
    wbytes = w.size
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    copies = int(max(8, (4 * l2) // wbytes + 1))
    pool = torch.from_numpy(np.tile(w, copies)).cuda()
    x = torch.randn(cols, device="cuda")
    y = torch.zeros(copies, rows, device="cuda")
    stream = torch.cuda.ExternalStream(ctx.lib.kib_stream(ctx.h))
    base = pool.data_ptr()

    def launch_all():
        for i in range(copies):
            ctx.matvec_kquant(qtype, base + i * wbytes, rows, cols, x, y[i])

    ctx.begin_graph()
    launch_all()  # warm-up, eager
    ctx.commit_graph()
    if profile:  # ncu --profile-from-start off: three launches
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        ctx.begin_graph()
        for i in range(3):
            ctx.matvec_kquant(qtype, base + i * wbytes, rows, cols, x, y[i])
        ctx.commit_graph()
        torch.cuda.profiler.stop()
    g = torch.cuda.CUDAGraph()
    ctx.begin_graph()
    with torch.cuda.graph(g, stream=stream):
        launch_all()
    ctx.commit_graph()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * copies)
    alg = wbytes + cols * 4 + rows * 4  # 2,082,816 B per call
    achieved = alg / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "traffic": None,
            "kernel": f"kquant_gemv2_kernel<{qtype},1> ({rows}x{cols} matvec)",
            "bytes_per_launch": alg, "us_per_launch": round(ms * 1e3, 3), "launches": reps * copies,
            "pool_copies": copies}


MTP_CONTEXT = 2048
# HBM bytes of one (k+1)-token verify forward at ctx 2048 (algorithmic, nearly
# independent of k): weights 513.3 MB + GDN S/R read+write 40.4 MB + K/V read
# once for all k+1 queries 25.2 MB.
VERIFY_BYTES = 578.8e6


def mtp_verify_bench(ctx, hbm_peak, reps=20):
    """the config-1 model plus one NextN layer, prompt of
    2048 seeded tokens.  For draft budgets k = 1..4: the latency of one verify
    forward over k+1 tokens through kib_qwen35_forward (argmax per row on the
    device, no state advance; device time by CUDA events on the engine's
    stream and the call's wall time), and tokens per verify step of greedy MTP
    generation with the budget fixed at k."""
    import numpy as np
    import torch
    import kib
    d = os.environ.get("KIB_BENCH_DIR", os.path.join(tempfile.gettempdir(), "kib_bench"))
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "qwen35_0p8b_shape_q4_k_m_nextn1_seed1234.gguf")
    if not os.path.exists(path):
        tmp = path + ".tmp"
        kib.write_synthetic_qwen35(tmp, threads=min(os.cpu_count() or 8, 64), seed=1234, nextn_layers=1)
        os.replace(tmp, path)
    m = kib.Qwen35(ctx, path, context_tokens=MTP_CONTEXT + 256, decode_tokens=64, prefill_chunk=1024, enable_mtp=True)
    rng = np.random.default_rng(2048)
    prompt = rng.integers(0, m.plan.vocab_size, MTP_CONTEXT).astype(np.int32)
    m.prefill(prompt, 1024)
    stream = torch.cuda.ExternalStream(ctx.lib.kib_stream(ctx.h))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    res = {}
    for k in (1, 2, 3, 4):
        toks = rng.integers(0, m.plan.vocab_size, k + 1).astype(np.int32)
        for _ in range(3):
            m.forward(toks, advance=False)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0.record(stream)
        for _ in range(reps):
            m.forward(toks, advance=False)
        e1.record(stream)
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - t0) * 1e3 / reps
        dev_ms = e0.elapsed_time(e1) / reps
        res[f"k{k}"] = {"verify_tokens": k + 1, "verify_ms_device": round(dev_ms, 4),
                        "verify_ms_call": round(wall_ms, 4),
                        "verify_hbm_gbs": round(VERIFY_BYTES / (dev_ms * 1e-3) / 1e9, 1)}
    for k in (1, 2, 3, 4):
        m.reset()
        out, r = m.generate(prompt, 48, enable_mtp=True, mtp_draft_tokens=k, mtp_adaptive=False, ignore_eos=True)
        steps = max(int(r.mtp.verify_steps), 1)
        res[f"k{k}"].update({"generated": int(r.generated_tokens), "verify_steps": int(r.mtp.verify_steps),
                             "drafted": int(r.mtp.drafted_tokens), "accepted": int(r.mtp.accepted_tokens),
                             "tokens_per_step": round(int(r.generated_tokens) / steps, 3),
                             "decode_ms": round(float(r.decode_ms), 2)})
    m.close()
    return {"workload": "BASELINE config 3: MTP verify at ctx 2048, fixed draft budget k (random-init weights: "
                        "drafts rarely match, so tokens/step sits near 1)",
            "bytes_per_verify": VERIFY_BYTES, "peak": hbm_peak, "by_k": res}



PREFILL_TOKENS = 8192
# FLOPs of the 8192-token prefill (algorithmic): linear projections 8.15 TFLOP,
# causal attention 1.65 TFLOP, delta-rule GDN 0.23 TFLOP.
PREFILL_FLOP = 10.03e12


def prefill_bench(ctx, path):
    """an 8192-token prompt of seeded uniform token ids
    through kib_qwen35_prefill in 1024-token chunks (device time by CUDA events
    on the engine's stream), against the measured dense bf16 tensor peak."""
    import numpy as np
    import torch
    import kib
    m = kib.Qwen35(ctx, path, context_tokens=PREFILL_TOKENS + 16, decode_tokens=8, prefill_chunk=1024, enable_mtp=False)
    prompt = np.random.default_rng(8192).integers(0, m.plan.vocab_size, PREFILL_TOKENS).astype(np.int32)
    stream = torch.cuda.ExternalStream(ctx.lib.kib_stream(ctx.h))
    m.prefill(prompt[:1024], 1024)  # warm-up: graphs and kernels
    m.reset()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()  # ncu --profile-from-start off captures the timed prefill only
    e0.record(stream)
    nxt = m.prefill(prompt, 1024)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1)
    m.close()
    tflops = PREFILL_FLOP / (ms * 1e-3) / 1e12
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, kind = (float(json.load(open(pk))["bf16_tflops_sustained"]), "measured sustained bf16") if os.path.exists(pk) \
        else (1400.0, "fallback")
    return {"workload": "BASELINE config 4: 8192-token prefill in 1024-token chunks (tcgen05 GEMMs with TMEM "
                        "accumulators on resident f16 weights, split-key mma.sync flash attention, chunked delta rule on split-TF32 mma.sync)", "tokens": PREFILL_TOKENS, "ms": round(ms, 2),
            "tok_per_s": round(PREFILL_TOKENS / (ms * 1e-3), 1), "bound": "tensor", "achieved": round(tflops, 2),
            "peak": peak, "unit": "TFLOP/s", "frac": round(tflops / peak, 4), "peak_kind": kind,
            "flop": PREFILL_FLOP, "next_token": int(nxt)}



BATCH_SLOTS = 32
BATCH_CONTEXT = 2048
BATCH_STEPS = 128


def batched_bench(ctx, path, hbm_peak, steps=BATCH_STEPS):
    """BASELINE config 5 on one GPU: 32 independent sequences, each with a
    seeded random 2048-token context, then `steps` greedy decode steps for all
    of them (device time by CUDA events on the engine's stream).  Algorithmic
    HBM bytes per step: the f16 projection weights read by the slot GEMMs, the
    Q6_K head, and per slot its KV rows, conv state and delta-rule state."""
    import numpy as np
    import torch
    import kib
    m = kib.Qwen35(ctx, path, context_tokens=BATCH_CONTEXT + 16, decode_tokens=8, prefill_chunk=1024,
                   enable_mtp=False)
    b = kib.Qwen35Batch(m, BATCH_SLOTS, context_tokens=BATCH_CONTEXT + steps + 16, max_steps=steps + 8)
    rng = np.random.default_rng(5)
    first = np.array([b.prefill(s, rng.integers(0, m.plan.vocab_size, BATCH_CONTEXT).astype(np.int32))
                      for s in range(BATCH_SLOTS)], np.int32)
    warm = b.decode(first, 4)  # captures the step graph
    stream = torch.cuda.ExternalStream(ctx.lib.kib_stream(ctx.h))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()  # ncu --profile-from-start off captures the timed steps only
    e0.record(stream)
    out = b.decode(warm[-1], steps)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1)
    p = m.plan
    ctx_mid = BATCH_CONTEXT + 4 + steps / 2
    w16 = 2.0 * (p.linear_attention_layers * (1024 * (6144 + 2048 + 32) + 2048 * 1024) +
                 p.full_attention_layers * (1024 * (4096 + 512 + 512) + 2048 * 1024) +
                 p.main_layers * 3 * 1024 * 3584)
    head = p.vocab_size * 4 * 210
    per_slot = (p.full_attention_layers * ctx_mid * 2 * 512 * 2 +            # K and V rows read
                p.linear_attention_layers * (16 * 128 * 128 * 4 * 2 + 6144 * 3 * 4 * 2))  # S and R read + written
    step_bytes = w16 + head + BATCH_SLOTS * per_slot
    step_ms = ms / steps
    gbs = step_bytes / (step_ms * 1e-3) / 1e9
    b.close()
    m.close()
    return {"workload": "BASELINE config 5: 32 sequences x 2048-token seeded contexts, greedy steps for all "
                        "(one GEMM over the slots per projection: the M > 8 numerics bucket)",
            "slots": BATCH_SLOTS, "steps": steps, "ms_per_step": round(step_ms, 4),
            "tok_per_s": round(BATCH_SLOTS * steps / (ms * 1e-3), 1), "bytes_per_step": round(step_bytes),
            "bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(gbs / hbm_peak, 4), "tokens_head": [int(x) for x in out[0][:8]]}


def cpu_decode_sample(path, threads, budget_s=20.0, max_tokens=6):
    """The oracle's bs1 decode step at position 4096 on the host cores (state
    content does not change the work)."""
    import numpy as np
    import oracle_lib
    o = oracle_lib.Oracle(threads=threads)
    om = oracle_lib.OracleModel(o, path, CONTEXT + max_tokens + 16)
    tok = 1
    t0 = time.perf_counter()
    n = 0
    while n < max_tokens:
        _, _, lg = om.forward([tok], CONTEXT + n)
        tok = int(np.argmax(lg[0]))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    om.close()
    return n / dt, n, dt


def run_reference(args, rank, world):
    if rank != 0:
        return
    path = model_path(rank, world)
    ensure_model(path, 0, 1)
    threads = os.cpu_count() or 1
    for _ in range(max(args.warmup, 0) and 1):
        cpu_decode_sample(path, threads, budget_s=5.0, max_tokens=1)
    vals = []
    toks = 0
    secs = 0.0
    for _ in range(args.steps):
        v, n, dt = cpu_decode_sample(path, threads, budget_s=10.0, max_tokens=2)
        vals.append(v)
        toks += n
        secs += dt
    value = toks / secs
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * secs / max(toks, 1), 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "context": CONTEXT, "quant_mix": "Q4_K + Q6_K ffn_down/head",
                       "l2": "weights 513 MB > L2", "reduced_model_for_profiling": bool(MODEL_OVERRIDES),
                       "parallelism": f"rank 0 of {world} (CPU arm)"},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{toks} decode steps at position {CONTEXT} (oracle/kib_oracle.cpp, "
                                       f"{threads} threads)"},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="kib", choices=["kib", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--no-mtp", action="store_true", help="skip the config-3 MTP verify measurement")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill measurement")
    ap.add_argument("--no-batch", action="store_true", help="skip the config-5 batched decode measurement")
    ap.add_argument("--workload", default="decode", choices=["decode", "matvec", "prefill", "batch", "verify"],
                    help="matvec: BASELINE config 1 only (Q4_K 3584x1024 GEMV roofline); verify: one MTP verify "
                         "forward of --verify-tokens tokens at ctx 2048 inside cudaProfilerStart/Stop (profiling)")
    ap.add_argument("--verify-tokens", type=int, default=2)
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: fewer layers than the BASELINE model (the JSON line says so)")
    ap.add_argument("--vocab", type=int, default=None, help="profiling only: smaller vocabulary")
    ap.add_argument("--mv-type", type=int, default=12, help="matvec workload: GGML type (12/13/14)")
    ap.add_argument("--mv-rows", type=int, default=3584)
    ap.add_argument("--mv-cols", type=int, default=1024)
    args = ap.parse_args()
    rank, world, local = dist_setup(args.gpus)
    if args.layers:
        MODEL_OVERRIDES["layers"] = args.layers
    if args.vocab:
        MODEL_OVERRIDES["vocab"] = args.vocab
    if args.workload == "matvec":
        import torch
        import kib
        torch.cuda.set_device(local)
        ctx = kib.Context(local)
        hbm, kind = peaks()
        r = matvec_roofline(ctx, hbm, profile=True, qtype=args.mv_type, rows=args.mv_rows, cols=args.mv_cols)
        r["peak_kind"] = kind
        print(json.dumps({"metric": f"K-quant type {args.mv_type} {args.mv_rows}x{args.mv_cols} matvec GB/s", "value": r["achieved"], "unit": "GB/s",
                          "roofline": r}), flush=True)
        ctx.close()
        return
    if args.workload == "prefill":
        import torch
        import kib
        torch.cuda.set_device(local)
        path = model_path(rank, world)
        ensure_model(path, rank, world)
        ctx = kib.Context(local)
        r = prefill_bench(ctx, path)
        print(json.dumps({"metric": "Qwen3.5-0.8B-shape 8192-token chunked prefill tok/s", "value": r["tok_per_s"],
                          "unit": "tok/s", "prefill_config4": r}), flush=True)
        ctx.close()
        return
    if args.workload == "verify":
        import numpy as np
        import torch
        import kib
        torch.cuda.set_device(local)
        ctx = kib.Context(local)
        d = os.environ.get("KIB_BENCH_DIR", os.path.join(tempfile.gettempdir(), "kib_bench"))
        os.makedirs(d, exist_ok=True)
        path = os.path.join(d, "qwen35_0p8b_shape_q4_k_m_nextn1_seed1234.gguf")
        if not os.path.exists(path):
            kib.write_synthetic_qwen35(path + ".tmp", threads=min(os.cpu_count() or 8, 64), seed=1234, nextn_layers=1)
            os.replace(path + ".tmp", path)
        m = kib.Qwen35(ctx, path, context_tokens=MTP_CONTEXT + 256, decode_tokens=64, prefill_chunk=1024,
                       enable_mtp=True)
        rng = np.random.default_rng(2048)
        m.prefill(rng.integers(0, m.plan.vocab_size, MTP_CONTEXT).astype(np.int32), 1024)
        toks = rng.integers(0, m.plan.vocab_size, args.verify_tokens).astype(np.int32)
        for _ in range(3):
            m.forward(toks, advance=False)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        m.forward(toks, advance=False)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"workload": "verify", "tokens": args.verify_tokens}), flush=True)
        m.close()
        ctx.close()
        return
    if args.workload == "batch":
        import torch
        import kib
        torch.cuda.set_device(local)
        path = model_path(rank, world)
        ensure_model(path, rank, world)
        ctx = kib.Context(local)
        hbm, _ = peaks()
        r = batched_bench(ctx, path, hbm)
        print(json.dumps({"metric": "Qwen3.5-0.8B-shape 32-sequence batched decode tok/s", "value": r["tok_per_s"],
                          "unit": "tok/s", "batched_config5": r}), flush=True)
        ctx.close()
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    import numpy as np
    import torch
    import kib
    torch.cuda.set_device(local)
    path = model_path(rank, world)
    ensure_model(path, rank, world)
    ctx = kib.Context(local)
    total = CONTEXT + args.warmup + args.steps + args.e2e_steps + 8
    m = kib.Qwen35(ctx, path, context_tokens=total, decode_tokens=8, prefill_chunk=1024, enable_mtp=False)
    prompt = np.random.default_rng(4096 + rank).integers(0, m.plan.vocab_size, CONTEXT).astype(np.int32)
    first = m.prefill(prompt, 1024)
    # warm-up (captures the decode graph)
    toks = m.decode_greedy(first, args.warmup)
    stream = torch.cuda.ExternalStream(ctx.lib.kib_stream(ctx.h))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pos0 = m.position
    lib = ctx.lib
    # timed region: K graph replays, token and position resident on the device
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        h = m.h
        # same call kib_qwen35_decode_greedy makes, with events around it on the engine's stream
        out = np.zeros(args.steps, np.int32)
        torch.cuda.profiler.start()  # ncu --profile-from-start off captures the timed region only
        e0.record(stream)
        rc = lib.kib_qwen35_decode_greedy(h, int(toks[-1]), args.steps, out.ctypes.data)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    assert rc == 0
    barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = allmax(ms, world)
    value = world * args.steps / (ms_max / 1e3)
    # e2e through the public C ABI with host buffers, per-token sync
    tok = int(out[-1])
    e2e_tokens = np.zeros(1, np.int32)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        am, _, _ = m.forward([tok], advance=True)
        tok = int(am[0])
    t1 = time.perf_counter()
    e2e_s = allmax(t1 - t0, world)
    e2e = world * args.e2e_steps / e2e_s
    hbm_peak, peak_kind = peaks()
    line = None
    if rank == 0:
        mv = matvec_roofline(ctx, hbm_peak)
        mv["peak_kind"] = f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"
        step_achieved = TOKEN_BYTES / (ms / args.steps * 1e-3) / 1e9
        persistent = os.environ.get("KIB_PERSISTENT", "1") != "0"
        roof = {"bound": "hbm", "achieved": round(step_achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(step_achieved / hbm_peak, 4), "traffic": PK_TRAFFIC,
                "kernel": "decode_persistent_kernel" if persistent else "per-kernel decode graph",
                "bytes_per_launch": TOKEN_BYTES, "us_per_launch": round(ms / args.steps * 1e3, 2),
                "peak_kind": mv["peak_kind"]}
        mtp = None
        if not args.no_mtp and world == 1:
            mtp = mtp_verify_bench(ctx, hbm_peak)
        pre = None
        if not args.no_prefill and world == 1:
            pre = prefill_bench(ctx, path)
        bat = None
        if not args.no_batch and world == 1:
            bat = batched_bench(ctx, path, hbm_peak)
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            threads = os.cpu_count() or 1
            v, n, dt = cpu_decode_sample(path, threads, budget_s=12.0, max_tokens=256)
            cpu = {"value": round(v, 4), "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"{n} oracle decode steps at position {CONTEXT} in {dt:.1f} s "
                             f"(oracle/kib_oracle.cpp, {threads} threads)"}
        # persistent path: embedding gather + the persistent kernel; otherwise
        # the per-kernel graph (embedding, 5 per layer... plus the head)
        launches_per_step = 2 if persistent else 2 + 5 * int(m.plan.main_layers)
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32 (K-quant weights, F16 KV)",
                "data": "synthetic (random-init weights, seeded random token ids)",
                "config": {"workload": WORKLOAD, "context": CONTEXT, "position_start": pos0,
                           "quant_mix": "Q4_K projections, Q6_K ffn_down + tied head",
                           "layers": int(m.plan.main_layers), "vocab": int(m.plan.vocab_size),
                           "reduced_model_for_profiling": bool(MODEL_OVERRIDES),
                           "parallelism": f"replicas x{world}", "l2": "inputs larger than L2 (weights 513 MB)"},
                "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 20, "d2h_bytes_per_step": 8,
                        "api": "kib_qwen35_forward (one graph launch per token: position, step counter and token H2D in one 20-byte copy, argmax and error flag D2H, per-token sync)"},
                "roofline": roof,
                "matvec_config1": mv,
                "mtp_verify_config3": mtp,
                "prefill_config4": pre,
                "batched_config5": bat,
                "cpu_baseline": cpu, "gpu_launches": launches_per_step * args.steps,
                "clocks": clk.summary(),
                "tokens_head": [int(x) for x in out[:8]]}
    m.close()
    ctx.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier(world)


if __name__ == "__main__":
    main()
