"""Benchmark: decode tokens/s of katgpt-rs's per-token forward on B200.

Workloads (`--workload`):
  c5 (default, the metric's configuration): n_layer 32, n_embd 4096, 32 heads
      of 128, mlp 16384, vocab 32000, bf16 weights ~N(0, 0.02), 4-bit
      TurboQuant KV (forward_quantized). 256 sequences in total: a 4096-token
      prefill from uniform random ids (untimed setup), then teacher-forced
      decode steps over positions 4096..4223 (the cache's 128 decode slots;
      a run longer than that wraps back to 4096). One step = one token for
      every sequence. `--gpus N` splits the FIXED 256 sequences, 256/N per
      rank (strong scaling), weights replicated; an NCCL all-gather of each
      step's logits is the only collective.
  c3: n_layer 12, n_embd 768, 12 heads, mlp 3072, vocab 32000, block 2048,
      4-bit TurboQuant KV; 64 sequences per GPU, 1024-token prefill (weak
      scaling).
  c4: n_layer 24, n_embd 2048, mlp 8192, standard bf16 KV, TwELL with ~90%-zero
      hidden activations; 512 sequences per GPU, 512-token prefill (weak).
  c1: Config::micro with AttentionMode::Standard (forward_base, f32): 4,096
      sequences x [BOS + 15 tokens] per GPU, teacher-forced (weak).
  c2: Config::micro with AttentionMode::SpKvQuant and the 3-bit codec;
      65,536 sequences x 16 positions per GPU (weak).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c5|c3|c4|c2|c1]

Prints one JSON line on rank 0.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "katgpt-rs_b200"))

METRIC = "decode tokens/s (box)"
UNIT = "tokens/s"
SEED = 42

# Decode workloads. `seqs` is per GPU for weak scaling and the whole job for
# strong scaling; positions [prefill, block_size) are the decode slots.
WORKLOADS = {
    "c5": dict(cfg=dict(vocab_size=32000, block_size=4096 + 128, n_embd=4096, n_head=32, head_dim=128,
                        n_kv_head=32, mlp_hidden=16384, n_layer=32, key_bits=4, val_bits=4),
               kv="tq", seqs=256, prefill=4096, scaling="strong", keep=0.0,
               text="c5: n_layer 32, n_embd 4096, 32 heads of 128, mlp 16384, vocab 32000, bf16 weights N(0,0.02), "
                    "4-bit TurboQuant KV (forward_quantized); 256 sequences in total split across the GPUs, "
                    "4096-token prefill then teacher-forced decode at positions 4096-4223"),
    "c3": dict(cfg=dict(vocab_size=32000, block_size=2048, n_embd=768, n_head=12, head_dim=64, n_kv_head=12,
                        mlp_hidden=3072, n_layer=12, key_bits=4, val_bits=4),
               kv="tq", seqs=64, prefill=1024, scaling="weak", keep=0.0,
               text="c3: n_layer 12, n_embd 768, 12 heads, mlp 3072, vocab 32000, block 2048, bf16 weights "
                    "N(0,0.02), 4-bit TurboQuant KV (forward_quantized); 64 sequences per GPU, 1024-token prefill "
                    "then teacher-forced decode"),
    # c4: vocab and decode steps are not given by the workload: 32000 and up to 64 (block 512 + 64)
    "c4": dict(cfg=dict(vocab_size=32000, block_size=576, n_embd=2048, n_head=16, head_dim=128, n_kv_head=16,
                        mlp_hidden=8192, n_layer=24),
               kv="std", seqs=512, prefill=512, scaling="weak", keep=0.1,
               text="c4: n_layer 24, n_embd 2048, 16 heads, mlp 8192, vocab 32000 (assumed), bf16 weights "
                    "N(0,0.02), standard attention with a bf16 KV cache, TwELL with ~90%-zero hidden activations "
                    "(benchmark hook: per-token Bernoulli keep 0.1, |N(0,1)| survivors (post-ReLU)); 512 sequences "
                    "per GPU, 512-token prefill then teacher-forced decode"),
}
C2_SEQS, C2_T = 65536, 16
C1_SEQS = 4096
# the micro-model workloads (Config::micro, BOS + 15 teacher-forced tokens):
# sequences per GPU, attention mode, the reference forward they time
MICRO = {
    "c1": dict(seqs=C1_SEQS, kv="f32", fwd="forward_base",
               text="c1: Config::micro + AttentionMode::Standard (forward_base, f32), 4096 sequences x 16 positions "
                    "per GPU"),
    "c2": dict(seqs=C2_SEQS, kv="spkv", fwd="forward_sp_kv_quant",
               text="c2: Config::micro + SpKvQuant + TurboQuant 3-bit, 65536 sequences x 16 positions per GPU"),
}
E2E_STEPS = 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c5", choices=["c5", "c3", "c4", "c2", "c1"])
    ap.add_argument("--seqs", type=int, default=0,
                    help="sequences per GPU (0 = the workload's; smaller for profiler captures)")
    ap.add_argument("--layers", type=int, default=0,
                    help="n_layer override for profiler captures of one kernel (0 = the workload's)")
    return ap.parse_args()


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms (one
    long-running nvidia-smi process), started before the warm-up steps and
    stopped after the timed steps."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.rows = [[x.strip() for x in ln.split(",")] for ln in out.splitlines() if ln.strip()]

    def summary(self):
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in self.rows if len(r) > 2 and num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if len(r) > 2 and num(r[2]) is not None]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU legs: the oracle (C++ restatement of the reference's x86 AVX2 path)

def profiled_traffic(name):
    """DRAM bytes per launch recorded by the ncu capture summarised in profiles/."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as fh:
            for line in fh:
                if line.startswith("traffic_bytes_per_layer:") or line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except OSError:
        pass
    return None


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    return oracle


class CpuDecode:
    """The reference's per-token decode on host cores at the GPU's context
    length (oracle.time_decode): one sequence per thread, each decoding the
    next position over a cache whose earlier positions hold synthetic codes.
    The timing weights are one random f32 layer shared by every layer (each
    layer's matrices still stream from DRAM, so the work per token is the
    same; all 32 distinct C5 layers would need 27 GB of host memory)."""

    def __init__(self, workload):
        self.oracle = _oracle()
        spec = WORKLOADS[workload]
        c = spec["cfg"]
        o = self.oracle
        self.cfg = o.config(vocab_size=c["vocab_size"], block_size=c["block_size"], n_embd=c["n_embd"],
                            n_head=c["n_head"], head_dim=c["head_dim"], n_kv_head=c["n_kv_head"],
                            mlp_hidden=c["mlp_hidden"], n_layer=c["n_layer"])
        c1 = o.config(vocab_size=c["vocab_size"], block_size=c["block_size"], n_embd=c["n_embd"],
                      n_head=c["n_head"], head_dim=c["head_dim"], n_kv_head=c["n_kv_head"],
                      mlp_hidden=c["mlp_hidden"], n_layer=1)
        n = o.lib().or_weights_count(ctypes.byref(c1))
        self.w1 = np.random.default_rng(SEED).standard_normal(n, dtype=np.float32) * np.float32(0.02)
        self.mode = o.MODE_QUANT if spec["kv"] == "tq" else o.MODE_BASE
        self.prefill = spec["prefill"]
        self.threads = os.cpu_count() or 1
        self.fwd = "forward_quantized" if self.mode == o.MODE_QUANT else "forward_base"

    def step(self, ctx, n_pos=1):
        """tokens/s of n_pos positions per thread starting at context ctx."""
        return self.oracle.time_decode(self.cfg, self.w1, ctx, n_pos, mode=self.mode, threads=self.threads)

    def sample(self, budget_s=15.0):
        n_pos, t0 = 1, time.perf_counter()
        while True:
            v = self.step(self.prefill, n_pos)
            el = self.threads * n_pos / v
            if time.perf_counter() - t0 + 2 * el > budget_s or n_pos >= 64:
                break
            n_pos *= 2
        return v, (f"{self.threads} sequences (one per thread) x {n_pos} decode positions from position "
                   f"{self.prefill} ({self.fwd}, {el:.1f} s of decode; one f32 layer shared by all layers)")


def cpu_sample_micro(workload, budget_s=10.0, threads=None):
    """tokens/s of the oracle's micro-model forward on the host cores."""
    oracle = _oracle()
    threads = threads or os.cpu_count() or 1
    cfg = oracle.config()
    w = oracle.weights(cfg, SEED)
    spec = MICRO[workload]
    mode = oracle.MODE_SPKV if spec["kv"] == "spkv" else oracle.MODE_BASE
    toks = c2_tokens(0, spec["seqs"])
    n, done, t0 = 1024, 0, time.perf_counter()
    while True:
        oracle.run_batch(cfg, mode, w, toks[:n], threads=threads, keep_logits=False)
        done += n * C2_T
        el = time.perf_counter() - t0
        if el > budget_s:
            break
        n = min(spec["seqs"], n * 2)
    return done / el, threads, f"{done // C2_T} sequences x {C2_T} positions ({spec['fwd']}, {el:.1f} s)"


def per_rank_seqs(workload, world, seqs_arg):
    """(sequences on this rank, sequences in the whole job)."""
    if workload in MICRO:
        return MICRO[workload]["seqs"], MICRO[workload]["seqs"] * world
    spec = WORKLOADS[workload]
    if seqs_arg:
        return seqs_arg, seqs_arg * world
    if spec["scaling"] == "strong":
        if spec["seqs"] % world:
            raise SystemExit(f"{workload}: {spec['seqs']} sequences do not split across {world} GPUs")
        return spec["seqs"] // world, spec["seqs"]
    return spec["seqs"], spec["seqs"] * world


def workload_config(workload, world, seqs_arg=0, layers=0):
    """The `config` of a bench line (identical in both arms)."""
    l2 = "inputs larger than L2 (KV cache and weights); L2 also flushed between steps (256 MiB write)"
    if workload in MICRO:
        return {"workload": MICRO[workload]["text"], "global_batch": world * MICRO[workload]["seqs"],
                "seq_len": C2_T, "parallelism": f"dp{world} (sequence shards)", "l2": l2}
    spec = WORKLOADS[workload]
    n, tot = per_rank_seqs(workload, world, seqs_arg)
    text = spec["text"] + (f" [n_layer {layers}]" if layers else "")
    return {"workload": text, "global_batch": tot, "seq_len": spec["prefill"],
            "parallelism": f"dp{world} (sequence shards, {n} per GPU)", "l2": l2}


def run_reference(args):
    """The reference arm: the oracle on all host cores, rank 0 only. One step =
    one decode position for one sequence per host thread, at the GPU arm's
    context (position prefill + step, wrapping within the decode slots)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    config = workload_config(args.workload, args.gpus, args.seqs)
    if args.workload in MICRO:
        vals = []
        for _ in range(args.warmup + args.steps):
            v, cores, sample = cpu_sample_micro(args.workload, budget_s=3.0)
            vals.append(v)
        v = float(np.median(vals[args.warmup:]))
        ms = 1000.0 * MICRO[args.workload]["seqs"] * C2_T / v
    else:
        cpu = CpuDecode(args.workload)
        spec = WORKLOADS[args.workload]
        dec = spec["cfg"]["block_size"] - spec["prefill"]
        secs = []
        for s in range(args.warmup + args.steps):
            v = cpu.step(spec["prefill"] + s % dec)
            if s >= args.warmup:
                secs.append(cpu.threads / v)
        cores = cpu.threads
        v = cpu.threads * len(secs) / float(np.sum(secs))
        ms = 1000.0 * float(np.mean(secs))
        sample = (f"each step: {cores} sequences (one per thread) x 1 decode position at context "
                  f"{spec['prefill']}+step ({cpu.fwd}; one f32 layer shared by all layers)")
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": WORKLOADS[args.workload]["scaling"] if args.workload not in MICRO else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference", "config": config,
            "note": "reference = its x86 AVX2 CPU path restated in C++ (the Rust reference cannot be built here), "
                    "timed on the host cores",
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                             "cpu_model": cpu_model()},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------

def c2_tokens(rank, n_seq):
    rng = np.random.default_rng(1000 + rank)
    t = rng.integers(1, 27, size=(n_seq, C2_T)).astype(np.int32)
    t[:, 0] = 26  # BOS
    return t


def timed_steps(torch, stream, steps, step_fn, flush):
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s in range(steps):
        flush.fill_(s & 0xFF)
        ev[s][0].record(stream)
        step_fn(s)
        ev[s][1].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def bench_decode(args, torch, dist, kgcuda, world, rank, local):
    """Prefill every sequence of this rank, then time teacher-forced decode
    steps (one token per sequence per step) on the device."""
    spec = WORKLOADS[args.workload]
    C = dict(spec["cfg"])
    if args.layers:
        C["n_layer"] = args.layers
    n, n_tot = per_rank_seqs(args.workload, world, args.seqs)
    PRE = spec["prefill"]
    DEC = C["block_size"] - PRE                  # decode slots; longer runs wrap
    dev = torch.device("cuda", local)
    kv_mode = kgcuda.KG_KV_TQ if spec["kv"] == "tq" else kgcuda.KG_KV_F32
    cfg = kgcuda.micro_config(kv_mode=kv_mode, weight_dtype=kgcuda.KG_W_BF16, max_seqs=n, **C)
    be = kgcuda.CudaBackend(cfg, device=local)
    be.random_weights(seed=SEED, std=0.02)
    if spec["keep"] > 0:
        be.set_mlp_hook(spec["keep"], SEED + rank)
    V, d, m, L = C["vocab_size"], C["n_embd"], C["mlp_hidden"], C["n_layer"]
    kvd = C["n_kv_head"] * C["head_dim"]
    n_prof = min(args.steps, 8)
    rng = np.random.default_rng(1000 + rank)
    toks = rng.integers(0, V, size=(n, C["block_size"])).astype(np.int32)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = ctypes.c_void_p(stream.cuda_stream)
    d_ids = torch.arange(n, dtype=torch.int32, device=dev)
    d_pre = torch.from_numpy(np.ascontiguousarray(toks[:, :PRE])).to(dev)
    d_dec = torch.from_numpy(np.ascontiguousarray(toks[:, PRE:].T)).to(dev)       # [slot][seq]
    d_pos = (torch.arange(DEC, dtype=torch.int32, device=dev)[:, None] + PRE).expand(-1, n).contiguous()
    d_log = torch.empty((n, V), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    slot = lambda s: s % DEC  # noqa: E731

    # prefill (untimed setup of the decode benchmark; its device time is reported)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    be.profile_read()
    be.profile(True)
    e0.record(stream)
    be.forward_batch_dev(n, PRE, P(d_ids), P(d_pre), None, None, None, sp)
    e1.record(stream)
    torch.cuda.synchronize()
    be.profile(False)
    pf_ms, _ = be.profile_read()
    prefill_ms = e0.elapsed_time(e1)
    # prefill weight GEMMs (QKV, Wo, W1, W2): algorithmic FLOPs = 2 x params x
    # tokens; the device issues twice that (activations as bf16 hi + lo)
    qd = C["n_head"] * C["head_dim"]
    layer_w = qd * d + 2 * kvd * d + d * qd + 2 * d * m
    pf_flops = 2.0 * n * PRE * L * layer_w
    pf_gemm_tf = pf_flops / (float(pf_ms[2]) * 1e-3) / 1e12 if pf_ms[2] > 0 else None

    # N > 1: each rank decodes its own sequences; the library's NCCL
    # all-gather (kg_decode_gather_dev, on the decode stream right after the
    # step) collects every rank's logits (the only collective on the path)
    d_all = torch.empty((world, n, V), dtype=torch.float32, device=dev)
    if world > 1:
        obj = [kgcuda.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        be.comm_init(obj[0], world, rank)

    def step(s):
        k = slot(s)
        be.decode_gather_dev(n, P(d_ids), P(d_dec[k]), P(d_pos[k]), P(d_all), None, sp)

    # warm-up: the first step of a batch shape runs eagerly, the second
    # captures the decode step as a CUDA graph, later steps replay it
    with ClockSampler(local) as clk:
        for s in range(args.warmup):
            step(s)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push(f"{args.workload}_decode")  # lets a profiler select the timed steps
        step_ms = timed_steps(torch, stream, args.steps, lambda s: step(args.warmup + s), flush)
        torch.cuda.nvtx.range_pop()
    graph_kernels = be.graph_kernels()
    if world > 1:
        dist.barrier()
    # phase breakdown: more steps, eagerly, with CUDA events around each phase
    # (attention, encode, GEMMs) on the launching stream
    p0 = args.warmup + args.steps
    be.profile_read()          # clear
    be.profile(True)
    timed_steps(torch, stream, n_prof, lambda s: step(p0 + s), flush)
    be.profile(False)
    ph_ms, _ = be.profile_read()
    ph_ms = [float(x) / n_prof for x in ph_ms]
    t = torch.tensor([float(np.sum(step_ms))], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    value = n_tot / (ms_per_step / 1000.0)

    # end to end through the public host API (kg_forward_batch) with pinned
    # host buffers: token/position/id upload and the logits read-back inside
    # every step; two untimed calls first (the first runs eagerly, the second
    # captures the decode graph)
    e0s = p0 + n_prof
    h_tok = torch.from_numpy(np.ascontiguousarray(toks[:, PRE:].T)).pin_memory()
    h_ids = torch.arange(n, dtype=torch.int32).pin_memory()
    h_pos = (torch.arange(DEC, dtype=torch.int32)[:, None] + PRE).expand(-1, n).contiguous().pin_memory()
    h_log = torch.empty((n, V), dtype=torch.float32).pin_memory()
    lib = kgcuda.lib()

    def e2e_step(s):
        k = slot(s)
        rc = lib.kg_forward_batch(be._h, n, P(h_ids), P(h_tok[k]), P(h_pos[k]), 1, P(h_log), None)
        if rc:
            raise RuntimeError(lib.kg_last_error(be._h))

    e2e_step(e0s)
    e2e_step(e0s + 1)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for s in range(E2E_STEPS):
        e2e_step(e0s + 2 + s)
    te = torch.tensor([time.perf_counter() - t0], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = n_tot * E2E_STEPS / float(te.item())

    positions = [PRE + slot(p0 + s) for s in range(n_prof)]
    kv_bytes_per_pos = (2 * (kvd // 2) + 8) if spec["kv"] == "tq" else 2 * kvd * 2
    attn_bytes = sum(n * L * (p + 1) * kv_bytes_per_pos for p in positions) / n_prof  # per step
    attn_gbs = attn_bytes / (ph_ms[0] / 1000.0) / 1e9 if ph_ms[0] > 0 else None
    gemm_bytes = (L * layer_w + V * d) * 2  # per step: streamed weights (wte/wpe gathered, not streamed)
    gemm_gbs = gemm_bytes / (ph_ms[2] / 1000.0) / 1e9 if ph_ms[2] > 0 else None
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    tpeak = peaks.get("bf16_tflops", 1590.0)
    prof_name = f"decode_attention_{args.workload}.txt"
    traffic = profiled_traffic(prof_name)
    attn_kernel = ("decode KV attention over 4-bit codes (scores + softmax + values, rotated domain)"
                   if spec["kv"] == "tq" else "decode KV attention (standard, bf16 K/V rows, GQA)")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": spec["scaling"],
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args.workload, world, args.seqs, args.layers),
        "collective": (f"NCCL all-gather of each rank's logits ({n} x {V} f32) per step inside the library "
                       f"(kg_decode_gather_dev)" if world > 1 else None),
        "gpu_launches": int(graph_kernels * args.steps),
        "decode_step": "one CUDA graph per step" if graph_kernels else "eager",
        "kernels_per_step": int(graph_kernels),
        "roofline": {"bound": "hbm", "kernel": attn_kernel,
                     "achieved": attn_gbs, "peak": peak, "unit": "GB/s",
                     "frac": (attn_gbs / peak) if attn_gbs else None, "traffic": traffic,
                     "traffic_unit": "DRAM read+write bytes per layer (ncu, the attention launches of one layer, "
                                     "scaled to this rank's sequences)",
                     "algorithmic_bytes_per_layer": attn_bytes / L,
                     "algorithmic_bytes_per_step": attn_bytes,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        "phases_ms_per_step": {"kv_attention": ph_ms[0], "kv_encode": ph_ms[1], "weight_gemms": ph_ms[2],
                               "note": f"{n_prof} eager steps after the timed ones, CUDA events per phase"},
        "weight_gemm_gbs": gemm_gbs,
        "prefill": {"tokens": n * PRE, "ms": prefill_ms, "tokens_per_s": n * PRE / (prefill_ms / 1000.0),
                    "weight_gemm_ms": float(pf_ms[2]),
                    "weight_gemm_tensor": {"achieved": pf_gemm_tf, "unit": "TFLOP/s", "peak": tpeak,
                                           "frac": (pf_gemm_tf / tpeak) if pf_gemm_tf else None,
                                           "flops": "algorithmic, 2 x weight params x tokens (QKV, Wo, W1, W2)",
                                           "issued_tensor_flops": "2x algorithmic: activations enter as bf16 hi + lo "
                                                                  "against bf16 weights",
                                           "kernel": "tcgen05 GEMM (QKV, Wo, W1, W2)"}},
        "e2e": {"value": e2e_val, "unit": UNIT, "steps": E2E_STEPS, "h2d_bytes_per_step": int(n * 4 * 3),
                "d2h_bytes_per_step": int(n * V * 4 + 4)},
        "clocks": clk.summary(),
    }
    if spec["keep"] > 0:
        line["mlp_hook"] = {"keep": spec["keep"], "note": "hidden activations after W1 replaced by Bernoulli(keep) "
                                                          "|N(0,1)| values (post-ReLU activations are non-negative; the "
                                                          "sparsity a trained TwELL model shows)"}
    if world > 1:
        be.comm_destroy()
    be.close()
    return line


def bench_micro(args, torch, dist, kgcuda, world, rank, local):
    """c1 / c2: teacher-forced forward of the micro model, one position per call
    for every sequence (the exact-order kernel)."""
    dev = torch.device("cuda", local)
    spec = MICRO[args.workload]
    n_seq = spec["seqs"]
    kv_mode = kgcuda.KG_KV_SPKV_TQ if spec["kv"] == "spkv" else kgcuda.KG_KV_F32
    cfg = kgcuda.micro_config(kv_mode=kv_mode, max_seqs=n_seq)
    be = kgcuda.CudaBackend(cfg, device=local)
    be.compile(kgcuda.reference_weights(cfg, SEED))
    toks = c2_tokens(rank, n_seq)
    d_tok = torch.from_numpy(np.ascontiguousarray(toks.T)).to(dev)        # [T][n_seq]
    d_ids = torch.arange(n_seq, dtype=torch.int32, device=dev)
    d_pos = torch.arange(C2_T, dtype=torch.int32, device=dev)[:, None].expand(C2_T, n_seq).contiguous()
    d_log = torch.empty((C2_T, n_seq, 27), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step(_s):
        for t in range(C2_T):
            be.forward_batch_dev(n_seq, 1, P(d_ids), P(d_tok[t]), P(d_pos[t]), P(d_log[t]), None, sp)

    with ClockSampler(local) as clk:
        for s in range(max(3, args.warmup)):
            step(s)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        step_ms = timed_steps(torch, stream, args.steps, step, flush)
    tm = torch.tensor([float(np.sum(step_ms))], device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms_per_step = float(tm.item()) / args.steps
    value = world * n_seq * C2_T / (ms_per_step / 1000.0)
    lo_dec = d_log[:, :64].permute(1, 0, 2).cpu().numpy()
    h_tok = torch.from_numpy(np.ascontiguousarray(toks.T)).pin_memory()
    h_ids = torch.arange(n_seq, dtype=torch.int32).pin_memory()
    h_pos = torch.arange(C2_T, dtype=torch.int32)[:, None].expand(C2_T, n_seq).contiguous().pin_memory()
    h_log = torch.empty((C2_T, n_seq, 27), dtype=torch.float32).pin_memory()
    lib = kgcuda.lib()

    def e2e_step():
        for t in range(C2_T):
            rc = lib.kg_forward_batch(be._h, n_seq, P(h_ids), P(h_tok[t]), P(h_pos[t]), 1, P(h_log[t]), None)
            if rc:
                raise RuntimeError(lib.kg_last_error(be._h))

    e2e_step()
    e2e_step()
    e_steps = 10
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e_steps):
        e2e_step()
    te = torch.tensor([time.perf_counter() - t0], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = world * n_seq * C2_T * e_steps / float(te.item())
    self_diff = float(np.abs(h_log[:, :64].permute(1, 0, 2).numpy() - lo_dec).max())
    # per position read / written: token, the cached K/V rows (c2: 3-bit codes of
    # K and V + two norms; c1: f32 K and V rows), the new row, (c2) its
    # utility, the logits
    row_b = 2 * 12 + 2 * 4 if spec["kv"] == "spkv" else 2 * 16 * 4
    util_b = 4 if spec["kv"] == "spkv" else 0
    bytes_per_step = n_seq * sum(4 + t * row_b + row_b + util_b + 27 * 4 for t in range(C2_T))
    achieved = bytes_per_step / (ms_per_step / 1000.0) / 1e9
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.workload, world),
        "gpu_launches": C2_T * args.steps,
        "roofline": {"bound": "hbm", "kernel": "micro_forward", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None,
                     "note": "exact-order f32 kernel: issue-bound, not HBM-bound",
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        "e2e": {"value": e2e_val, "unit": UNIT, "steps": e_steps, "h2d_bytes_per_step": int(3 * C2_T * n_seq * 4),
                "d2h_bytes_per_step": int(h_log.numel() * 4)},
        "self_check_max_abs_diff": self_diff,
        "clocks": clk.summary(),
    }
    be.close()
    return line


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist
    import kgcuda

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    fn = bench_micro if args.workload in MICRO else bench_decode
    line = fn(args, torch, dist, kgcuda, world, rank, local)
    if rank == 0 and world == 1:
        try:
            if args.workload in MICRO:
                v, cores, sample = cpu_sample_micro(args.workload)
            else:
                cpu = CpuDecode(args.workload)
                v, sample = cpu.sample()
                cores = cpu.threads
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                                    "cpu_model": cpu_model()}
        except Exception as ex:  # the baseline must not break the bench line
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": 0, "kind": "port", "sample": f"failed: {ex}"}
    if rank == 0:
        print(json.dumps(line, default=float), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
