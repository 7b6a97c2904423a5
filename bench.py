#!/usr/bin/env python
"""Phi-3-mini INT8 EAGLE-style speculative decoding on B200 (bs1, greedy
chain, k = 4 drafted tokens per step).

Workload (one "step" of this benchmark): decode 128 new tokens with the
speculative engine from a prefilled 128-token seeded prompt. Base model
Phi-3-mini-shaped (32 layers, d 3072, 32 heads x 96, SwiGLU 8192, vocab
32064) plus a 4-layer draft sharing the embedding and LM head; weights are
seeded N(0, 0.02) -> Q4_0 -> INT8 [-8, 7] with fp16 block scales, random
init (no checkpoints are available offline). Every step streams ~6.4 GB of
weights per speculative step, far more than the 126 MB L2, so no L2 flush is
needed between timed iterations.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    python bench.py --workload sampled-batch [--seqs 64 --prompt-len 1024 --new-tokens 512 --k 6]
    torchrun --nproc-per-node N bench.py --gpus N --workload tp-medium [--prompt-len 512] [--batch 4] [--tree 8]
    python bench.py --workload medusa [--prompt-len 512 --new-tokens 256]
    python bench.py --workload step-breakdown [--steps 3 --warmup 1]

One process per GPU (torchrun for N > 1); this path does not shard (batch 1),
so N GPUs run N independent replicas and `value` sums their tokens/s.
--impl reference times the CPU implementation of the same path (the oracle's
restatement built on the reference's primitives -- the reference ships no
speculative decoder) on the host cores, rank 0 only.

--workload sampled-batch is the batched stochastic configuration: independent
sequences (temperature 0.8, top-p 0.95, k = 6, Philox seed 1234 keyed by
sequence id) split across the ranks with no exchange, each rank decoding its
share as one in-GPU batch (the verify pass runs sequences x (k + 1) rows
through the tcgen05 GEMM); `value` = all ranks' tokens / the slowest rank's
device time for its share, prefills included (strong scaling: the sequence
count is fixed); `spec.decode_only_tok_s` leaves the prefills out. Not the
default line.

--workload tp-medium is the tensor-parallel configuration: a Phi-3-medium-
shaped base (40 layers, d 5120, 40 query / 10 KV heads x 128, SwiGLU 17920,
vocab 32064) with a 2-layer draft of the same dims, greedy chain k = 4, bs1,
sharded over the ranks (NCCL all-reduce after o and down); `value` = tokens/s
of all sequences (strong scaling), device-timed, max over ranks. `--batch B`
decodes B sequences as one in-GPU batch; `--tree W` verifies a static draft
tree of 1 + k W nodes per step (with `--batch`, one tree per sequence, all
in one pass; prefills outside the timing).

--workload medusa is the Medusa configuration: the Phi-3-mini base with 4
residual Medusa heads (3072 x 3072 INT8 each, shared LM head), per-head
top-k 10/5/3/2, a 64-node candidate tree verified in one tree-masked pass
(65 rows through the tcgen05 GEMM), greedy path acceptance and KV compaction;
`value` = new tokens / device time of the decode (prefill included), bs1.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "fast-llm-inference_b200"))

import numpy as np  # noqa: E402

METRIC = "Phi-3-mini spec-decode accepted tok/s @bs1"
DIMS = dict(vocab=32064, d=3072, ffn=8192, layers=32, heads=32, kv_heads=32, head_dim=96, theta=10000.0, eps=1e-5)
DRAFT_LAYERS = 4
SEED = 1
PROMPT_SEED = 2024


def engine_cfg(max_seq_len):
    return dict(vocab_size=DIMS["vocab"], hidden_size=DIMS["d"], intermediate_size=DIMS["ffn"],
                num_layers=DIMS["layers"], num_heads=DIMS["heads"], num_kv_heads=DIMS["kv_heads"],
                head_dim=DIMS["head_dim"], draft_layers=DRAFT_LAYERS, medusa_heads=0, max_seq_len=max_seq_len,
                rope_theta=DIMS["theta"], norm_eps=DIMS["eps"])


def step_bytes(k, ctx, wbytes=1.0):
    """Algorithmic HBM bytes of one speculative step: k draft passes (4
    layers + LM head) and one verify pass (32 layers + LM head) of weights
    (wbytes per weight: 1 INT8, 0.5 packed 4-bit) with fp16 block scales,
    plus the fp16 KV read by attention."""
    d, F, V = DIMS["d"], DIMS["ffn"], DIMS["vocab"]
    layer = (3 * d * d + d * d + 2 * F * d + d * F) * (wbytes + 1 / 16)
    lm = V * d * (wbytes + 1 / 16)
    kv_pos = 2 * d * 2  # K and V, fp16, one layer
    draft = k * (DRAFT_LAYERS * layer + lm + DRAFT_LAYERS * kv_pos * ctx)
    verify = DIMS["layers"] * layer + lm + DIMS["layers"] * kv_pos * ctx
    return draft + verify


def medusa_step_bytes(rows, heads, ctx):
    """Algorithmic HBM bytes of one Medusa tree step: the heads (one INT8
    d x d linear each, their LM head pass over `heads` rows), one verify pass
    over the tree's rows (32 layers, each weight read once; LM head in
    ceil(rows / 8) eight-row passes) and the fp16 KV read by attention."""
    d, F, V = DIMS["d"], DIMS["ffn"], DIMS["vocab"]
    layer = (3 * d * d + d * d + 2 * F * d + d * F) * (1 + 1 / 16)
    lm = V * d * (1 + 1 / 16)
    kv = DIMS["layers"] * 2 * d * 2 * ctx
    return heads * d * d * (1 + 1 / 16) + lm + DIMS["layers"] * layer + -(-rows // 8) * lm + kv


def profiled_traffic(summary, m):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch of a kernel at
    M = m, from the ncu summary committed under profiles/ (its line
    `traffic_bytes_per_launch M=<m>: <bytes>`); None when absent."""
    import re
    try:
        with open(os.path.join(ROOT, "profiles", summary)) as f:
            for line in f:
                r = re.match(r"\s*traffic_bytes_per_launch M=(\d+): (\d+)", line)
                if r and int(r.group(1)) == m:
                    return int(r.group(2))
    except OSError:
        pass
    return None


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def tensor_id(stack, layer, proj):
    """FL_TENSOR_ID of include/fl_cuda.h."""
    return (stack << 24) | (layer << 8) | proj


def workload_config(a, world):
    """The `config` of both arms' lines (same workload, same keys)."""
    return {"workload": f"phi3-mini int8 (32L d3072 ffn8192 vocab32064) + {DRAFT_LAYERS}-layer draft, "
                        f"greedy chain k={a.k}, bs1, prompt {a.prompt_len}, {a.new_tokens} new tokens per step",
            "parallelism": "replicas only" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (6.4 GB of weights per speculative step)"}


def oracle_weights(orc):
    """Every tensor of the model from the oracle's restatement of the seeded
    generator: the bits fl_engine_synthesize puts on the device, with no
    product library loaded."""
    d, F = DIMS["d"], DIMS["ffn"]
    qd = kd = DIMS["heads"] * DIMS["head_dim"]
    shapes = [(qd, d), (kd, d), (kd, d), (d, qd), (F, d), (F, d), (d, F)]
    w = {}
    for s_, nl in ((0, DIMS["layers"]), (1, DRAFT_LAYERS)):
        for l in range(nl):
            for p, (r, c) in enumerate(shapes):
                w[(s_, l, p)] = orc.synth_q4_0_i8(SEED, tensor_id(s_, l, p), r, c)
    w[(3, 0, 1)] = orc.synth_q4_0_i8(SEED, tensor_id(3, 0, 1), DIMS["vocab"], d)
    embed = orc.synth_q4_0_f32(SEED, tensor_id(3, 0, 0), DIMS["vocab"], d)
    return w, embed


def kernel_comparison(orc, ref, reps=10):
    """The gate/up projection at the verify width (16384 x 3072, 5 rows):
    the oracle's packed block matmul (the arm's kernel) against the
    reference's compiled matmul_dequantized on the per-row form of the same
    INT8 values, median ms over `reps` calls each. Shows that the arm's
    kernel runs at the reference kernel's speed."""
    import ctypes as C
    rng = np.random.default_rng(7)
    M, N, K = 5, 16384, 3072
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float32)
    wq, dq = orc.synth_q4_0_i8(SEED, tensor_id(0, 0, 4), N, K)
    wp, sp = np.empty_like(wq), np.empty(dq.shape, np.float32)
    P = lambda x: x.ctypes.data_as(C.c_void_p)
    orc.so.orc_pack_rows8(P(wq), P(dq), N, K, P(wp), P(sp))
    out = np.empty((M, N), np.float32)

    def med(f):
        f()
        ts = []
        for _ in range(reps):
            t = time.perf_counter()
            f()
            ts.append(time.perf_counter() - t)
        return float(statistics.median(ts)) * 1e3

    res = {"shape": f"{M}x{K} @ {N}x{K}",
           "port_ms": med(lambda: orc.so.orc_matmul_packed(P(A), P(wp), P(sp), P(out), M, N, K))}
    if ref is not None:
        rs = np.ascontiguousarray(dq[:, 0].view(np.float16).astype(np.float32) * 16.0)
        res["reference_matmul_dequantized_ms"] = med(
            lambda: ref.so.ref_matmul_dequantized(P(A), P(wq), P(rs), P(out), M, N, K))
    return res


def cpu_reference_decode(a, n_tokens, warmup, steps):
    """The reference's CPU path on the host cores, restated by the oracle:
    the speculative decode loop (draft chain, one verify pass of k + 1 rows,
    greedy acceptance) over the layer math of inference.c and the INT8
    matmul of dequantized_tensor.c (u8 activations, maddubs dots) in its
    per-32-block-scale form, which is what the workload's weights need. The
    reference's compiled matmul_dequantized has a per-row scale only; on
    these weights it computes a different model, one whose stream accepts
    every draft, so it would be timed on other work per token. The oracle's
    kernel runs on weights repacked for 8-lane integer dots and matches the
    reference kernel's speed (kernel_comparison, in the same run). Same
    weights (the oracle's restatement of the seeded generator: no product
    library is loaded), prompt and draft length as the GPU arm, all host
    threads, and the same tokens. Returns the median decode-loop rate over
    `steps` decodes of n_tokens (each after its own prefill, excluded)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    import bind
    t0 = time.time()
    orc = bind.Oracle()
    try:
        ref = bind.Ref()
    except RuntimeError:
        ref = None
    w, embed = oracle_weights(orc)
    om = bind.OracleModel(orc, DIMS, embed, w, draft_layers=DRAFT_LAYERS, packed=True)
    del w
    prompt = np.random.default_rng(PROMPT_SEED).integers(0, DIMS["vocab"], a.prompt_len).astype(np.int32)
    setup_s = time.time() - t0
    kernels = kernel_comparison(orc, ref)
    for _ in range(warmup):  # warms caches and threads: short decodes
        om.spec(prompt, 8, a.k)
    vals, hist = [], []
    for _ in range(steps):
        toks, acc, margins = om.spec(prompt, n_tokens, a.k)
        dec = orc.so.orc_last_decode_seconds()
        vals.append(((n_tokens - 1) / dec, dec))
        hist.append(acc)
    acc_cat = np.concatenate(hist)
    return {"value": float(statistics.median(x[0] for x in vals)),
            "ms": float(statistics.median(x[1] for x in vals)) * 1000.0,
            "kind": "port", "cores": threads, "setup_s": setup_s,
            "matmul": "oracle block matmul on 8-row packed weights (reference's u8 x s8 maddubs rule, "
                      "per-32-block scales)",
            "kernel_comparison": kernels, "tokens": toks, "margins": margins,
            "accepted_hist": np.bincount(acc_cat, minlength=a.k + 1).tolist()}


def stream_check(cpu_toks, margins, gpu_toks):
    """Greedy streams of the CPU arm and the GPU decode from the same prompt:
    the identical prefix and, where they part, the CPU's relative top-2
    margin there (a near-tie below 1e-2 is the allowed divergence)."""
    n = min(len(cpu_toks), len(gpu_toks))
    same = int(np.argmin(np.asarray(cpu_toks[:n]) == np.asarray(gpu_toks[:n]))) \
        if not np.array_equal(cpu_toks[:n], gpu_toks[:n]) else n
    out = {"tokens": n, "identical_prefix": same}
    if same < n:
        out["margin_at_divergence"] = float(margins[same])
    return out


def run_reference(a, rank, world):
    if rank != 0:
        return 0
    r = cpu_reference_decode(a, a.new_tokens, a.warmup, a.steps)
    line = {
        "metric": METRIC, "value": r["value"], "unit": "tok/s", "impl": "reference", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": r["ms"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8xs8->s32, f32",
        "data": "synthetic (seeded N(0,0.02) -> Q4_0 -> INT8 weights, uniform prompt ids)",
        "config": workload_config(a, world),
        "cpu_baseline": {"value": r["value"], "unit": "tok/s", "cores": r["cores"], "kind": r["kind"],
                         "sample": f"each step: one {a.new_tokens}-token speculative decode after the "
                                   f"{a.prompt_len}-token prefill (prefill excluded from the rate; warm-up steps "
                                   f"decode 8 tokens)",
                         "matmul": r["matmul"], "kernel_comparison": r["kernel_comparison"],
                         "accepted_hist": r["accepted_hist"]},
        "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": r["setup_s"],
    }
    print(json.dumps(line), flush=True)
    return 0


MICRO_SHAPES = {"gateup": (16384, 3072), "qkv": (9216, 3072), "o": (3072, 3072), "down": (3072, 8192),
                "lm": (32064, 3072)}


def run_microbench(a):
    """One GEMV shape of the model in isolation (for ncu captures and kernel
    timing): NT device copies of the weights (> 300 MB together, so launches
    stream from HBM), M activation rows, fl_cuda_matmul_i8 launches back to
    back on the library stream, timed with CUDA events."""
    import ctypes as C
    import torch
    import flb200
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(0), "init")
    N, K = MICRO_SHAPES[a.microbench]
    w, d = lib.synth_q4_0_i8(SEED, 7000 + N + K, N, K)
    nt = max(4, int(np.ceil(300e6 / (N * K * 17 / 16))))
    ts = []
    for _ in range(nt):
        t = flb200.block_tensor(w, d)
        lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
        ts.append(t)
    x = torch.randn(a.m, K, device="cuda")
    out = torch.empty(a.m, N, device="cuda")
    s = lib.fl_cuda_stream()
    stream = torch.cuda.ExternalStream(s)

    def sweep():
        for t in ts:
            lib.check(lib.fl_cuda_matmul_i8(x.data_ptr(), C.byref(t), out.data_ptr(), a.m, N, K, s), "matmul")

    sweep()
    lib.check(lib.fl_cuda_sync(), "sync")
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.iters):
        sweep()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (a.iters * nt)
    byts = N * K * 17 / 16 + a.m * K * 4 + a.m * N * 4
    print(json.dumps({"microbench": a.microbench, "N": N, "K": K, "M": a.m, "launches": a.iters * nt,
                      "us_per_launch": us, "GBps": byts / us / 1e3, "TOPS": 2.0 * a.m * N * K / us / 1e6}),
          flush=True)
    return 0


MEDIUM = dict(vocab_size=32064, hidden_size=5120, intermediate_size=17920, num_layers=40, num_heads=40,
              num_kv_heads=10, head_dim=128, draft_layers=2, medusa_heads=0, rope_theta=10000.0, norm_eps=1e-5)


def run_tp_medium(a):
    """Phi-3-medium-shaped spec decode, tensor-parallel over the ranks."""
    import datetime
    import torch
    import flb200
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(local), "init")
    cfg = dict(MEDIUM, max_seq_len=((a.prompt_len + a.new_tokens + a.k + 2 + 63) // 64) * 64)
    tp = None
    if world > 1:
        box = [flb200.tp_unique_id(lib) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = (rank, world, box[0])
    t0 = time.time()
    eng = flb200.Engine(lib, cfg, local, tp=tp)
    eng.synthesize(SEED)
    B = max(1, a.batch)
    rng = np.random.default_rng(PROMPT_SEED)
    prompts = rng.integers(0, MEDIUM["vocab_size"], (B, a.prompt_len)).astype(np.int32)
    tree_us = []
    if a.tree > 0 and B > 1:
        # a draft tree of 1 + k * width nodes for each of B sequences, all
        # verified in one pass (prefills inside each call, outside its timing)
        eng.batch_reserve(B, a.prompt_len + a.new_tokens + 1 + a.k * a.tree + a.k + 3)
        def decode():
            toks, steps, _ = eng.batch_tree_generate(prompts, a.new_tokens, a.k, a.tree)
            tree_us.append(eng.last_timing()[2])
            return toks, np.zeros(int(steps.max()), np.int32)
    elif a.tree > 0:
        # static draft tree of 1 + k * width nodes (prefill inside each call,
        # outside its device timing)
        def decode():
            toks, acc = eng.spec_tree_generate(prompts[0], a.new_tokens, a.k, a.tree)
            tree_us.append(eng.last_timing()[2])
            return toks, acc
    elif B == 1:
        eng.spec_prefill(prompts[0], a.k)
        decode = lambda: eng.spec_decode(a.new_tokens)
    else:
        # B independent sequences as one in-GPU batch on every rank
        eng.batch_reserve(B, a.prompt_len + a.new_tokens + a.k + 3)
        eng.batch_prefill(prompts, a.k)
        def decode():
            toks, steps, _ = eng.batch_decode(a.new_tokens)
            return toks, np.zeros(int(steps.max()), np.int32)
    setup_s = time.time() - t0
    for _ in range(a.warmup):
        decode()
    stream = torch.cuda.ExternalStream(eng.stream(), device=local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    steps_total, launches = 0, 0
    for _ in range(a.steps):
        toks, acc = decode()
        steps_total += len(acc)
        launches += eng.last_launches()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if a.tree > 0:
        ms = sum(tree_us[-a.steps:]) / 1e3  # the decode loops alone (prefills excluded)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if rank == 0:
        line = {
            "metric": f"Phi-3-medium spec-decode tok/s @bs{B}, tensor parallel",
            "value": B * a.steps * a.new_tokens / (ms / 1e3),
            "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8xs8->s32, f32",
            "data": "synthetic (seeded N(0,0.02) -> Q4_0 -> INT8 weights, uniform prompt ids)",
            "config": {"workload": f"phi3-medium int8 (40L d5120 40/10 heads x128 ffn17920 vocab32064) + 2-layer draft, "
                                   + (f"greedy draft tree k={a.k} x width {a.tree} ({1 + a.k * a.tree} nodes)"
                                      if a.tree > 0 else f"greedy chain k={a.k}")
                                   + f", batch {B}, prompt {a.prompt_len}, "
                                   f"{a.new_tokens} new tokens per sequence per step",
                       "parallelism": f"tensor parallel x{world} (NCCL all-reduce after o and down)"},
            "spec": {"spec_steps_per_decode": steps_total / a.steps, "step_us": ms * 1e3 / max(1, steps_total)},
            "gpu_launches": int(launches), "clocks": clk, "setup_s": setup_s,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_step_breakdown(a):
    """Where the config-0 speculative step goes, from whole-step device times
    of engines that differ only in layer counts and k (every launch of each
    step runs; nothing is skipped): the Phi-3-mini widths with (base, draft,
    k) = (32, 4, 4), (16, 4, 4), (32, 2, 4), (32, 4, 2), 128-token prompt,
    128 new tokens, zero acceptance on random weights. A verify layer is the
    difference of the first two over 16 layers; a draft layer's cost per step
    (its catch-up pass and k - 1 chain passes) the difference of the first
    and third over 2; the rest (LM heads, picks, control kernels) what
    remains of the full step. One JSON line."""
    import torch
    import flb200
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(0), "init")
    prompt = np.random.default_rng(PROMPT_SEED).integers(0, DIMS["vocab"], 128).astype(np.int32)
    cases = [(32, 4, 4), (16, 4, 4), (32, 2, 4), (32, 4, 2)]
    us = {}
    for L, D, k in cases:
        cfg = engine_cfg(512)
        cfg["num_layers"], cfg["draft_layers"] = L, D
        eng = flb200.Engine(lib, cfg, 0)
        eng.synthesize(SEED)
        stream = torch.cuda.ExternalStream(eng.stream())
        times = []
        for r in range(max(a.warmup, 1) + a.steps):
            eng.spec_prefill(prompt, k)
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            toks, acc = eng.spec_decode(128)
            e1.record(stream)
            torch.cuda.synchronize()
            if r >= max(a.warmup, 1):
                times.append(e0.elapsed_time(e1) * 1e3 / len(acc))
        us[(L, D, k)] = statistics.median(times)
        eng.close()
    full = us[(32, 4, 4)]
    verify_layer = (full - us[(16, 4, 4)]) / 16
    draft_layer = (full - us[(32, 2, 4)]) / 2
    line = {"workload": "step-breakdown: phi3-mini widths, 128-token prompt, 128 new tokens, zero acceptance",
            "step_us": {f"L{L}_D{D}_k{k}": v for (L, D, k), v in us.items()},
            "verify_layer_us": verify_layer, "verify_layers_us": 32 * verify_layer,
            "draft_layer_per_step_us": draft_layer, "draft_layer_pass_us": draft_layer / 4,
            "draft_us": 4 * draft_layer, "rest_us": full - 32 * verify_layer - 4 * draft_layer,
            "k4_minus_k2_us": full - us[(32, 4, 2)]}
    print(json.dumps(line), flush=True)
    return 0


def run_profile_step(a):
    """A small case of the config-0 decode for ncu captures: the full widths
    (d 3072, 32 heads of 96, ffn 8192, vocab 32064) with 4 base and 2 draft
    layers, a 64-token prompt and 12 new tokens (the same kernels, tiles and
    launch shapes as the full model, about 1 GB on the device), then one
    pass of each decode attention over the 4 layers at a 192-position
    context. --step-kernel selects the one-kernel step."""
    if a.step_kernel:
        os.environ["FL_STEP_KERNEL"] = "1"
    import flb200
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(0), "init")
    cfg = engine_cfg(256)
    cfg["num_layers"], cfg["draft_layers"] = 4, 2
    eng = flb200.Engine(lib, cfg, 0)
    eng.synthesize(SEED)
    prompt = np.random.default_rng(PROMPT_SEED).integers(0, DIMS["vocab"], 64).astype(np.int32)
    eng.spec_prefill(prompt, a.k)
    toks, acc = eng.spec_decode(12)
    att = eng.bench_attention(0, a.k + 1, 192, reps=1)
    att1 = eng.bench_attention(1, 1, 192, reps=1)
    print(json.dumps({"profile_case": "phi3-mini widths, 4 + 2 layers", "step_kernel": bool(eng.step_kernel()),
                      "spec_steps": len(acc), "attention_us": [att, att1]}), flush=True)
    eng.close()
    return 0


def run_medusa(a):
    """Medusa heads on the Phi-3-mini base, bs1, one timed generate per step."""
    import torch
    import flb200
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(0), "init")
    topk, nodes = [10, 5, 3, 2], 64
    cfg = dict(engine_cfg(((a.prompt_len + a.new_tokens + nodes + 2 + 63) // 64) * 64), draft_layers=0, medusa_heads=4)
    eng = flb200.Engine(lib, cfg, 0)
    eng.synthesize(SEED)
    prompt = np.random.default_rng(PROMPT_SEED).integers(0, DIMS["vocab"], a.prompt_len).astype(np.int32)
    for _ in range(a.warmup):
        eng.medusa_generate(prompt, 16, topk, nodes)
    stream = torch.cuda.ExternalStream(eng.stream())
    torch.cuda.synchronize()
    clocks = Clocks(0)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    accs, dec_us = [], []
    for _ in range(a.steps):
        toks, acc = eng.medusa_generate(prompt, a.new_tokens, topk, nodes)
        accs.append(acc)
        dec_us.append(eng.last_timing()[2])  # the tree-step loop alone (after the prefill)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    acc_cat = np.concatenate(accs)
    step_us = sum(dec_us) / max(1, len(acc_cat))
    tree_bytes = medusa_step_bytes(nodes, 4, a.prompt_len + a.new_tokens // 2)  # the root is one of the nodes
    tree_gbs = tree_bytes / (step_us * 1e-6) / 1e9
    peak, peak_kind = measured_peaks()
    line = {
        "metric": "Phi-3-mini Medusa decode tok/s @bs1", "value": a.steps * a.new_tokens / (ms / 1e3), "unit": "tok/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8xs8->s32, f32",
        "data": "synthetic (seeded N(0,0.02) -> Q4_0 -> INT8 weights, uniform prompt ids)",
        "config": {"workload": f"phi3-mini int8 + 4 Medusa heads, top-k {topk}, {nodes}-node tree, bs1, "
                               f"prompt {a.prompt_len}, {a.new_tokens} new tokens per step (prefill included)"},
        "medusa": {"tree_steps_per_generate": len(acc_cat) / a.steps, "mean_accepted": float(acc_cat.mean()),
                   "step_us": step_us, "decode_tok_s": (a.new_tokens - 1) * len(dec_us) / (sum(dec_us) * 1e-6)},
        "roofline": {"bound": "hbm", "achieved": tree_gbs, "peak": peak, "unit": "GB/s", "frac": tree_gbs / peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": f"whole tree step ({nodes} verify rows: tcgen05 GEMM, LM head in 8-row GEMVs)",
                     "bytes_per_step": tree_bytes},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    eng.close()
    return 0


SHARD_T, SHARD_TOP_P, SHARD_SEED = 0.8, 0.95, 1234


def sharded_decode(a, dist, rank, nranks, local):
    """Config 3's sequences decoded by ranks 0 .. nranks - 1 (each its share
    as one in-GPU batch, no collective on the data path); ranks at or past
    nranks only take part in the barriers. Returns (slowest rank's seconds
    with prefills, slowest decode seconds, speculative steps, stream
    checksum over all sequences, launches of this rank)."""
    import torch
    import flb200
    import shard
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(local), "init")
    max_seq = ((a.prompt_len + a.new_tokens + a.k + 2 + 63) // 64) * 64
    ids = shard.shard_of(a.seqs, rank, nranks) if rank < nranks else []
    eng = None
    if ids:
        eng = flb200.Engine(lib, engine_cfg(max_seq), local)
        eng.synthesize(SEED)
        eng.set_sampling(SHARD_T, SHARD_TOP_P, SHARD_SEED)
        # KV regions reserved once, outside the timed region; warm-up on as
        # many other sequences (same batch size: the same kernels and tiles)
        eng.batch_reserve(len(ids), a.prompt_len + a.new_tokens + a.k + 3)
        wid = list(range(a.seqs + rank * len(ids), a.seqs + (rank + 1) * len(ids)))
        warm = shard.prompts_for(wid, 64, DIMS["vocab"], PROMPT_SEED)
        for _ in range(max(a.warmup, 3)):
            eng.spec_generate_batch(warm, 16, a.k, seq_ids=wid)

    def barrier():
        if dist:
            dist.barrier()

    barrier()
    torch.cuda.synchronize()
    secs = dec = 0.0
    nsteps, launches, toks, got_ids = 0, 0, np.zeros((0, a.new_tokens), np.int32), []
    if ids:
        got_ids, toks, steps, secs = shard.run_shard(eng, ids, a.prompt_len, a.new_tokens, a.k, DIMS["vocab"],
                                                     PROMPT_SEED)
        dec = eng.last_timing()[1] * 1e-6  # decode loops alone
        launches = eng.last_launches()
        nsteps = int(steps.sum())
    torch.cuda.synchronize()
    barrier()
    if dist:
        t = torch.tensor([secs, dec], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs, dec = float(t[0].item()), float(t[1].item())
        full = shard.gather_tokens(dist, list(got_ids), toks, a.seqs)
        t = torch.tensor([nsteps], device="cuda", dtype=torch.float64)
        dist.all_reduce(t)
        nsteps = int(t.item())
    else:
        full = toks
    if eng:
        eng.close()
    # gather_tokens gives the full set on rank 0 only
    return secs, dec, nsteps, int(np.asarray(full, np.int64).sum()) if full is not None else 0, launches


def run_sampled_batch(a):
    """Independent sampled sequences sharded across ranks (see the module
    docstring); one timed pass over each rank's share."""
    import datetime
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    clocks = Clocks(local)
    clocks.start()
    secs, dec, nsteps, checksum, launches = sharded_decode(a, dist, rank, world, local)
    clk = clocks.stop()
    tokens = a.seqs * a.new_tokens
    if rank == 0:
        line = {
            "metric": "sampled spec-decode tok/s, batch of independent sequences", "value": tokens / secs,
            "unit": "tok/s", "n_gpus": world, "steps": 1, "warmup": max(a.warmup, 3),
            "ms_per_step": secs * 1000.0, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u8xs8->s32, f32",
            "data": "synthetic (seeded N(0,0.02) -> Q4_0 -> INT8 weights, uniform prompt ids per sequence)",
            "config": {"workload": f"phi3-mini int8 + {DRAFT_LAYERS}-layer draft, rejection sampling T={SHARD_T} "
                                   f"top-p={SHARD_TOP_P} k={a.k}, Philox seed {SHARD_SEED} keyed by sequence id, "
                                   f"{a.seqs} sequences x ({a.prompt_len} prompt + {a.new_tokens} new), "
                                   f"split over {world} rank(s), prefill included",
                       "parallelism": f"sequence sharding over {world} GPU(s), no collective",
                       "step": "each rank's share as one in-GPU batch (prefills + batched decode)"},
            "spec": {"speculative_steps": nsteps, "tokens_per_step": tokens / max(1, nsteps),
                     "decode_only_tok_s": tokens / dec if dec > 0 else None,
                     "batch_per_gpu": (a.seqs + world - 1) // world, "decode_s": dec, "prefill_s": secs - dec,
                     "stream_checksum": checksum},
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# Strong-scaling ceiling of config 3 from HBM bytes alone: every rank still
# streams the replicated weights once per pass (about 7.47 GB), only the KV
# reads shrink with the share (64 / g x 0.566 GB).
SHARD_CEILING = {1: 1.0, 2: 1.71, 4: 2.64, 8: 3.64}


def split_host_threads(impl):
    """OpenMP threads of this process, set before the libraries (and their
    OpenMP runtimes) load. The ranks of one node share the host cores for
    the weight generator; the reference arm runs on rank 0 alone and takes
    them all. torchrun exports OMP_NUM_THREADS=1 to every rank when the
    variable is unset, so 1 counts as unset under it."""
    world = int(os.environ.get("LOCAL_WORLD_SIZE", os.environ.get("WORLD_SIZE", "1")))
    cur = os.environ.get("OMP_NUM_THREADS")
    if cur is not None and not (world > 1 and cur == "1"):
        return
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores if impl == "reference" else max(1, cores // world))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--cpu-tokens", type=int, default=16, help="tokens of the bounded CPU decode sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--microbench", choices=sorted(MICRO_SHAPES), help="time one GEMV shape in isolation")
    ap.add_argument("--w4", action="store_true",
                    help="decode passes stream packed 4-bit weights (fl_engine_set_weight_bits 4)")
    ap.add_argument("--step-kernel", action="store_true",
                    help="one persistent tcgen05 kernel per speculative step (128-byte panels)")
    ap.add_argument("--m", type=int, default=5, help="activation rows for --microbench")
    ap.add_argument("--iters", type=int, default=10, help="sweeps for --microbench")
    ap.add_argument("--workload", default="spec-bs1",
                    choices=["spec-bs1", "sampled-batch", "tp-medium", "medusa", "profile-step", "step-breakdown"])
    ap.add_argument("--seqs", type=int, default=64, help="sequences of --workload sampled-batch")
    ap.add_argument("--batch", type=int, default=1, help="sequences decoded together by --workload tp-medium")
    ap.add_argument("--tree", type=int, default=0, help="draft-tree width for --workload tp-medium (0: chain)")
    a = ap.parse_args()
    split_host_threads(a.impl)
    if a.microbench:
        return run_microbench(a)
    if a.workload == "sampled-batch":
        return run_sampled_batch(a)
    if a.workload == "tp-medium":
        return run_tp_medium(a)
    if a.workload == "medusa":
        return run_medusa(a)
    if a.workload == "profile-step":
        return run_profile_step(a)
    if a.workload == "step-breakdown":
        return run_step_breakdown(a)
    a.warmup = max(a.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if a.impl == "reference":
        return run_reference(a, rank, world)
    if a.step_kernel:
        os.environ["FL_STEP_KERNEL"] = "1"

    import torch
    import flb200
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    lib = flb200.Lib()
    lib.check(lib.fl_cuda_init(local), "init")
    t_setup = time.time()
    max_seq = 512
    eng = flb200.Engine(lib, engine_cfg(max_seq), local)
    eng.synthesize(SEED)  # the seeded generator on the device: the tensors the CPU arm generates
    if a.w4:
        eng.set_weight_bits(4)
    wbytes = 0.5 if a.w4 else 1.0
    prompt = np.random.default_rng(PROMPT_SEED).integers(0, DIMS["vocab"], a.prompt_len).astype(np.int32)
    eng.spec_prefill(prompt, a.k)
    setup_s = time.time() - t_setup

    stream = torch.cuda.ExternalStream(eng.stream(), device=local)
    for _ in range(a.warmup):
        toks, acc = eng.spec_decode(a.new_tokens)

    def barrier():
        if dist:
            dist.barrier()

    clocks = Clocks(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launches = 0
    steps_total = 0
    acc_all = []
    for _ in range(a.steps):
        toks, acc = eng.spec_decode(a.new_tokens)
        launches += eng.last_launches()
        steps_total += len(acc)
        acc_all.append(acc)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / a.steps
    value = world * a.steps * a.new_tokens / (ms / 1000.0)
    acc_cat = np.concatenate(acc_all)
    spec_steps = steps_total / a.steps
    step_us = ms_per_step * 1000.0 / spec_steps
    ctx_mid = a.prompt_len + a.new_tokens // 2
    peak, peak_kind = measured_peaks()
    step_gbs = step_bytes(a.k, ctx_mid, wbytes) / (step_us * 1e-6) / 1e9

    # Dominant kernel: the verify pass's gate/up GEMV (M = k + 1), timed live
    # as captured back-to-back launches over all 32 layers (1.6 GB > L2).
    us_gu, by_gu = eng.bench_linear(0, 2, a.k + 1, reps=5)
    us_dn, by_dn = eng.bench_linear(0, 3, a.k + 1, reps=5)
    us_qkv, by_qkv = eng.bench_linear(0, 0, a.k + 1, reps=5)
    us_o, by_o = eng.bench_linear(0, 1, a.k + 1, reps=5)
    us_d1, by_d1 = eng.bench_linear(1, 2, 1, reps=20)
    us_att = eng.bench_attention(0, a.k + 1, ctx_mid, reps=20)
    us_att1 = eng.bench_attention(1, 1, ctx_mid, reps=20)
    kern_gbs = by_gu / (us_gu * 1e-6) / 1e9

    # End to end through the reference-facing API: speculative_generate() with
    # host buffers (prompt ids as floats in, tokens out), prefill included.
    import ctypes as C
    dm = lib.draft_model_create(DRAFT_LAYERS, DIMS["d"], DIMS["ffn"], DIMS["vocab"])
    lib.check(0 if lib.draft_model_load(dm, f"synthetic:{SEED}".encode()) == 0 else -1, "draft_model_load")
    cfg = flb200.SpecConfig(a.k, 0.0, a.k)
    ph = prompt.astype(np.float32)
    out = np.empty(a.new_tokens, np.int32)
    tf = C.cast(lib.so.fl_cuda_target_forward, C.c_void_p)
    n = lib.speculative_generate(dm, eng.h, tf, flb200.ptr(ph), len(prompt), flb200.ptr(out), a.new_tokens,
                                 C.byref(cfg))
    lib.check(0 if n == a.new_tokens else -1, "speculative_generate")
    e2e_times = []
    for _ in range(max(3, a.steps // 2)):
        t0 = time.perf_counter()
        n = lib.speculative_generate(dm, eng.h, tf, flb200.ptr(ph), len(prompt), flb200.ptr(out), a.new_tokens,
                                     C.byref(cfg))
        e2e_times.append(time.perf_counter() - t0)
    e2e_ok = n == a.new_tokens and np.array_equal(out, toks)
    e2e_val = world * a.new_tokens / statistics.median(e2e_times)
    if dist:
        t = torch.tensor([statistics.median(e2e_times)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_val = world * a.new_tokens / float(t.item())
    lib.draft_model_free(dm)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        r = cpu_reference_decode(a, a.cpu_tokens, 0, 1)
        cpu = {"value": r["value"], "unit": "tok/s", "cores": r["cores"], "kind": r["kind"],
               "sample": f"one {a.cpu_tokens}-token speculative decode after the same {a.prompt_len}-token prefill "
                         f"(prefill excluded)", "matmul": r["matmul"],
               "stream_check": stream_check(r["tokens"], r["margins"], toks)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8xs8->s32, f32",
            "data": "synthetic (seeded N(0,0.02) -> Q4_0 -> INT8 weights, uniform prompt ids)",
            "config": dict(workload_config(a, world),
                           weights="packed 4-bit in the decode passes" if a.w4 else "INT8"),
            "step_path": "one persistent cooperative kernel per step" if eng.step_kernel()
            else "multi-kernel CUDA graph per step",
            "spec": {"spec_steps_per_decode": spec_steps, "mean_accepted": float(acc_cat.mean()),
                     "accepted_hist": np.bincount(acc_cat, minlength=a.k + 1).tolist(),
                     "step_us": step_us, "step_bytes": step_bytes(a.k, ctx_mid, wbytes), "step_gbs": step_gbs,
                     "step_frac_of_hbm": step_gbs / peak},
            # the 32 layers' four verify GEMVs, each timed in a chain of its own
            # launches (inside the step they cost more: --workload step-breakdown)
            "verify_gemvs_us_isolated": 32 * (us_gu + us_dn + us_qkv + us_o),
            "roofline": {"bound": "hbm", "achieved": kern_gbs, "peak": peak, "unit": "GB/s",
                         "frac": kern_gbs / peak,
                         "traffic": None if eng.step_kernel() or a.w4 else profiled_traffic(
                             "gemv_tma_gateup_16384x3072.md", a.k + 1),
                         "peak_kind": peak_kind,
                         "kernel": "gemv_tma_kernel (verify gate/up, 16384x3072, M=%d)" % (a.k + 1),
                         "per_launch_us": us_gu, "bytes_per_launch": by_gu,
                         "others": {"qkv_M5": [us_qkv, by_qkv / (us_qkv * 1e-6) / 1e9],
                                    "o_M5": [us_o, by_o / (us_o * 1e-6) / 1e9],
                                    "down_M5": [us_dn, by_dn / (us_dn * 1e-6) / 1e9],
                                    "draft_gateup_M1": [us_d1, by_d1 / (us_d1 * 1e-6) / 1e9],
                                    "attention_M%d_us" % (a.k + 1): us_att, "draft_attention_M1_us": us_att1}},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": int(ph.nbytes),
                    "d2h_bytes_per_step": int(out.nbytes), "api": "speculative_generate (prefill included)",
                    "tokens_match": bool(e2e_ok)},
            "gpu_launches": int(launches),
            "clocks": clk,
            "setup_s": setup_s,
        }
    eng.close()
    if dist:
        # The batch-1 path above does not shard (replicas only). Config 3 does:
        # its 64 sampled sequences decoded by rank 0 alone, then split over all
        # ranks with no collective on the data path (strong scaling, same run).
        c3 = argparse.Namespace(seqs=64, prompt_len=1024, new_tokens=512, k=6, warmup=1)
        one = sharded_decode(c3, dist, rank, 1, local)
        many = sharded_decode(c3, dist, rank, world, local)
        if rank == 0:
            tok = c3.seqs * c3.new_tokens
            line["sharded"] = {
                "workload": "config 3: 64 independent sampled sequences (T 0.8, top-p 0.95, k 6, Philox seed 1234 "
                            "by sequence id) x (1024 prompt + 512 new), prefills included",
                "scaling": "strong", "tok_s_1gpu": tok / one[0], f"tok_s_{world}gpu": tok / many[0],
                "speedup": one[0] / many[0], "hbm_ceiling_speedup": SHARD_CEILING.get(world),
                "decode_only_speedup": one[1] / many[1] if many[1] > 0 else None,
                "streams_identical": one[3] == many[3]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
