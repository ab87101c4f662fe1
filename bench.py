#!/usr/bin/env python
"""Benchmark of the attention hot path (BASELINE metric: decode/verify attention HBM GB/s, prefill TFLOP/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nvattn|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N ...

Headline workload: BASELINE config 2 (Qwen3-8B paged decode: 32 q / 8 kv heads, head_dim 128, block 256,
context U[512, 4096]).  A step is one Attention.forward of the decode branch over the batch: the KV scatter of
the new tokens plus paged decode attention.  Multi-GPU follows nano-vllm's tensor-parallel head split: rank r
owns kv heads [r*8/N, (r+1)*8/N) and their q heads, for a global batch of 64*N sequences (weak scaling: every
rank reads the same ~640 MB of KV per step as one GPU does at N=1).  No collective runs inside attention; the
only NCCL calls are the barrier and the max-over-ranks of the timings.

value      algorithmic bytes (KV read once per kv head + q + o + the scatter's read and write) of all ranks,
           divided by the slowest rank's device time (CUDA events), inputs resident in HBM, L2 flushed between
           timed steps outside the events (a 256 MiB write, then a 256 MiB read that writes the dirty lines back).
e2e        the same bytes through the public nvattn.attention.Attention.forward with the step's inputs copied
           host->device from pinned memory and the output copied back inside the timed region.
roofline   the decode launch (one kernel: split-KV pieces merged in the same launch) timed alone with CUDA events vs
           measured HBM peak.
The reference arm (--impl reference) times the reference semantics (the FP32 torch oracle) on host cores.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "nano-vllm-spec-decode_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

GiB = 1 << 30


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return dict(hbm=float(d["hbm_gbs"]), bf16=float(d["bf16_tflops"]),
                    bf16_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


def traffic_summary():
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.gpu_index = gpu_index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
                self.lines = [l for l in out.splitlines() if l.strip()]
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------------------------------------- work
def decode_shard(world, rank, seed=0, B_per_gpu=64, k=0):
    """This rank's KV-head shard of the (weak-scaled) decode / verify batch."""
    from nvattn.workloads import paged_decode_batch
    B = B_per_gpu * world
    g = torch.Generator().manual_seed(seed)
    if k == 0:
        lens = torch.randint(512, 4097, (B,), generator=g).tolist()
    else:
        lens = torch.randint(256, 2049, (B,), generator=g).tolist()
    H, KVH = 32 // world, 8 // world
    b = paged_decode_batch(lens, k + 1, H, KVH, 128, 2048 * world, 0.5, seed + 1 + rank, device="cuda",
                           device_fill=True)
    return b, lens, H, KVH


def decode_strong_shard(world, rank, seed=0):
    """This rank's KV-head shard of BASELINE config 2 itself (64 sequences at every N): strong scaling over the
    tensor-parallel head split, 32/N q heads and 8/N kv heads per rank."""
    from nvattn.workloads import paged_decode_batch
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(512, 4097, (64,), generator=g).tolist()
    H, KVH = 32 // world, 8 // world
    b = paged_decode_batch(lens, 1, H, KVH, 128, 2048, 0.5, seed + 1 + rank, device="cuda", device_fill=True)
    return b, lens, H, KVH


def decode_kernel_name(n, H, KVH):
    """The paged_decode_kernel<NP, Spec> instantiation a decode / verify call (fixed-length batch) runs, as profilers
    name it: the packed rows q_per_seq x group of one kv head, padded to 16, 32 or 48 (decode_rows_padded in
    csrc/paged_decode.cu); Spec = 1, the speculative-weights variant, at 48 rows."""
    rows = n * (H // KVH)
    np_ = next(x for x in (16, 32, 48) if rows <= x)
    return f"paged_decode_kernel<{np_}, {1 if np_ == 48 else 0}>"


def attn_bytes(lens, n, H, KVH):
    from nvattn.workloads import bytes_decode
    return bytes_decode(lens, n, H, KVH)


def scatter_bytes(T, KVH):
    return 2.0 * T * KVH * 128 * 2 * 2     # k and v rows, read + write


def capture(fn):
    """CUDA graph of fn (warmed up on a side stream first), the way nano-vllm replays its decode steps."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


class L2Flush:
    """Flushes the 126 MB L2 between timed steps, outside the events: a 256 MiB write, then a read of another
    256 MiB buffer, which evicts the written (dirty) lines and writes them back before the step starts, so the timed
    step neither finds its inputs in L2 nor pays for someone else's write-backs."""

    def __init__(self):
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.r = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")

    def __call__(self):
        self.w.zero_()
        torch.count_nonzero(self.r)


def time_steps(fn, steps, warmup, flush):
    """Per-step device time (ms) with CUDA events on the current stream; L2 flushed (`flush()`) before each step
    outside the events.  Returns the list of step times."""
    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def run_nvattn(args, world, rank, local):
    from nvattn import ops
    from nvattn.attention import Attention
    from nvattn.context import set_context, reset_context
    pk = peaks()
    b, lens, H, KVH = decode_shard(world, rank, args.seed)
    B = b.num_seqs
    q4 = b.q.view(B, 1, H, 128)
    out = torch.empty_like(q4)
    flush = L2Flush()
    a_bytes = attn_bytes(lens, 1, H, KVH)
    s_bytes = scatter_bytes(B, KVH)

    def step():
        ops.store_kvcache(b.k_new, b.v_new, b.k_cache, b.v_cache, b.slot_mapping)
        ops.flash_attn_with_kvcache(q4, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                    block_table=b.block_tables, softmax_scale=b.scale, out=out)

    def attn_only():
        ops.flash_attn_with_kvcache(q4, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                    block_table=b.block_tables, softmax_scale=b.scale, out=out)

    g_step = capture(step)
    g_attn = capture(attn_only)

    # ---- headline: device-resident inputs, one graph replay (scatter + attention) per step
    barrier(world)
    with ClockSampler(local) as clk:
        barrier(world)
        times = time_steps(g_step.replay, args.steps, args.warmup, flush)
        barrier(world)
    total_ms = max_over_ranks(sum(times), world)
    ms_step = total_ms / args.steps
    value = world * (a_bytes + s_bytes) / (ms_step * 1e-3) / 1e9

    # ---- roofline: the decode launch alone
    k_times = time_steps(g_attn.replay, args.steps, args.warmup, flush)
    k_ms = max_over_ranks(statistics.mean(k_times), world)
    achieved = a_bytes / (k_ms * 1e-3) / 1e9
    tr = traffic_summary().get("paged_decode_config2")
    traffic = None
    if tr:
        # per-launch DRAM bytes of the captured case, scaled by the KV bytes this launch reads
        traffic = tr["dram_bytes"] * (a_bytes / tr["algorithmic_bytes"])

    # ---- e2e through the public Attention.forward with host buffers
    attn = Attention(H, 128, b.scale, KVH)
    attn.k_cache, attn.v_cache = b.k_cache, b.v_cache
    host = {n: t.cpu().pin_memory() for n, t in dict(q=b.q, k=b.k_new, v=b.v_new, slots=b.slot_mapping,
                                                      ctx=b.context_lens, bt=b.block_tables).items()}
    dev = {n: torch.empty_like(t, device="cuda") for n, t in host.items()}
    out_host = torch.empty(B, H, 128, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()

    # Attention.forward captured once over static device buffers (ModelRunner.capture_cudagraph); each step copies
    # the step's inputs in from pinned host memory, replays, and copies the output back (ModelRunner.run_model).
    for n in host:
        dev[n].copy_(host[n])
    set_context(False, slot_mapping=dev["slots"], context_lens=dev["ctx"], block_tables=dev["bt"])
    o_static = {}

    def fwd():
        o_static["o"] = attn(dev["q"], dev["k"], dev["v"])
    g_fwd = capture(fwd)
    reset_context()

    def e2e_step():
        for n in host:
            dev[n].copy_(host[n], non_blocking=True)
        g_fwd.replay()
        out_host.copy_(o_static["o"], non_blocking=True)

    barrier(world)
    e_times = time_steps(e2e_step, args.steps, args.warmup, flush)
    e_ms = max_over_ranks(sum(e_times), world) / args.steps
    e2e_value = world * (a_bytes + s_bytes) / (e_ms * 1e-3) / 1e9

    # ---- secondary rows: verify (config 3) and greedy accept at this N
    secondary = {}
    for k in (1, 2, 4, 8):
        # one batch of contexts for every k (B = 32, contexts U[256, 2048]), so the k rows differ
        # only in their query tokens
        vb, vl, _, _ = decode_shard(world, rank, args.seed + 10, B_per_gpu=32, k=k)
        vq = vb.q.view(vb.num_seqs, k + 1, H, 128)
        vout = torch.empty_like(vq)

        def vstep():
            ops.flash_attn_with_kvcache(vq, vb.k_cache, vb.v_cache, cache_seqlens=vb.context_lens,
                                        block_table=vb.block_tables, softmax_scale=vb.scale, out=vout)
        vt = time_steps(capture(vstep).replay, max(10, args.steps // 2), args.warmup, flush)
        v_ms = max_over_ranks(statistics.mean(vt), world)
        vbytes = attn_bytes(vl, k + 1, H, KVH)
        from nvattn.workloads import flops_decode
        secondary[f"verify_k{k}"] = {"GBps": round(world * vbytes / (v_ms * 1e-3) / 1e9, 1),
                                     "frac_hbm": round(vbytes / (v_ms * 1e-3) / 1e9 / pk["hbm"], 3),
                                     "us": round(v_ms * 1e3, 2),
                                     "TFLOPs": round(world * flops_decode(vl, k + 1, H) / (v_ms * 1e-3) / 1e12, 1)}
        del vb, vq, vout
    if world > 1:
        secondary["strong_tp"] = strong_row(world, rank, args, flush, pk)
    else:
        secondary.update(aux_rows(args, flush, pk))
    secondary.update(varlen_rows(world, rank, args, flush, pk))
    secondary["flash_attn_2_8_3_same_workloads"] = fa2_rows(world, rank, args, flush, b, q4, lens, H, KVH)
    from nvattn.workloads import accept_config
    t_ids, d_ids, nd = (x.cuda() for x in accept_config(8, S=32, seed=args.seed))
    acc_out = {}

    def accept():
        acc_out["r"] = ops.greedy_accept(t_ids, d_ids, nd)
    at = time_steps(capture(accept).replay, 50, 5, flush)
    secondary["greedy_accept_k8_S32_us"] = round(statistics.median(at) * 1e3, 2)

    line = {
        "metric": "decode attention HBM GB/s (BASELINE config 2: Qwen3-8B paged decode)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded; BASELINE config 2 shapes)",
        "config": {"workload": "paged decode step = KV scatter + GQA paged attention, BASELINE config 2",
                   "timing": "CUDA-graph replay per step, CUDA events, max over ranks",
                   "global_batch": B, "per_rank_q_heads": H, "per_rank_kv_heads": KVH, "head_dim": 128,
                   "block_size": 256, "context": "U[512, 4096]", "parallelism": f"kv-head shards x{world}",
                   "l2": "flushed between timed steps outside the events: 256 MiB write, then a 256 MiB read that "
                         "writes the dirty lines back"},
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e_ms, 5),
                "api": "nvattn.attention.Attention.forward (CUDA-graph replay, inputs H2D from pinned memory, output D2H)"},
        "roofline": {"kernel": decode_kernel_name(1, H, KVH), "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": pk["hbm"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm"], 4), "peak_source": pk["source"],
                     "traffic": None if traffic is None else round(traffic),
                     "algorithmic_bytes": round(a_bytes), "us": round(k_ms * 1e3, 2)},
        "gpu_launches": 2 * args.steps,   # per timed headline step: store_kvcache_kernel + paged_decode_kernel
        "secondary": secondary,
    }
    if world == 1 and rank == 0 and not args.no_e2e_model:
        del b, q4, out, flush
        torch.cuda.empty_cache()
        secondary["e2e_config5"] = e2e_model_rows(args)
    clocks = clk.summary()
    line["clocks"] = clocks
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.seed, budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)


def strong_row(world, rank, args, flush, pk):
    """Strong scaling: BASELINE config 2's fixed batch of 64 sequences split over the N ranks by kv heads (at N = 8
    one kv head, ~80 MB of KV per rank and step).  us = the slowest rank's decode launch; frac_per_rank = one rank's
    algorithmic bytes / that time / measured HBM peak; GBps = all ranks' bytes / that time."""
    from nvattn import ops
    b, lens, H, KVH = decode_strong_shard(world, rank, args.seed)
    q = b.q.view(b.num_seqs, 1, H, 128)
    out = torch.empty_like(q)

    def call():
        ops.flash_attn_with_kvcache(q, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                    block_table=b.block_tables, softmax_scale=b.scale, out=out)
    t = time_steps(capture(call).replay, max(10, args.steps // 2), args.warmup, flush)
    ms = max_over_ranks(statistics.mean(t), world)
    by = attn_bytes(lens, 1, H, KVH)
    return {"global_batch": 64, "per_rank_q_heads": H, "per_rank_kv_heads": KVH, "us": round(ms * 1e3, 2),
            "MB_per_rank": round(by / 1e6, 1), "GBps": round(world * by / (ms * 1e-3) / 1e9, 1),
            "frac_per_rank": round(by / (ms * 1e-3) / 1e9 / pk["hbm"], 3),
            "hbm_floor_us": round(by / (pk["hbm"] * 1e9) * 1e6, 2)}


def e2e_model_rows(args):
    """BASELINE config 5 end to end (nvattn/e2e.py): random-init Qwen3-8B under the reference's own engine, greedy
    n-gram speculative decoding with dynamic k over a fixed injected step-cost table, 64 requests of 1024 prompt
    tokens, 256 new tokens each; the reference arm (its flash-attn 2.8.3 + Triton scatter) and this package's full
    drop-in (attention, fused q/k-norm + rotary + scatter prologue, sharded greedy verify), each in its own process,
    one after the other.  Output tokens / generate() wall time, after the reference bench's warm-up and one more on
    requests of the measured shape (other ids), so that first calls at the measured batch sizes (torch.compile work)
    stay outside the timed call in both arms.  With random weights the model does not repeat its
    own text, so n-gram guesses rarely fire; the second pair of rows lets the model guess for itself (every decode
    step a k = 4 verify step, ~93% of guesses accepted)."""
    import tempfile
    rows = {}
    with tempfile.TemporaryDirectory() as tmp:
        costs = os.path.join(tmp, "costs.json")
        model = os.path.join(tmp, "qwen3_8b_random")
        env = dict(os.environ, PYTHONPATH=os.path.join(REPO, "nano-vllm-spec-decode_b200"))
        for variant, extra in (("spec_ngram_dynk_graph", ["--step-costs", costs, "--synthetic-step-costs"]),
                               ("spec_draft_graph", ["--max-num-seqs", "64"])):
            for arm in ("reference", "nvattn+all"):
                out = os.path.join(tmp, f"{variant}_{arm}.json")
                cmd = [sys.executable, "-m", "nvattn.e2e", "--arm", arm, "--variant", variant, "--model-dir", model,
                       "--out", out, "--shape-warmup"] + extra
                try:
                    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
                except subprocess.TimeoutExpired:
                    rows[f"{variant}/{arm}"] = {"unavailable": "timed out after 600 s"}
                    continue
                if r.returncode != 0:
                    rows[f"{variant}/{arm}"] = {"unavailable": (r.stderr.strip().splitlines() or ["failed"])[-1][:200]}
                    continue
                with open(out) as f:
                    d = json.load(f)
                spec = d.get("spec") or {}
                rows[f"{variant}/{arm}"] = {
                    "output_tok_per_s": round(d["output_tok_per_s"], 1), "generate_s": round(d["generate_s"], 3),
                    "output_tokens": d["output_tokens"], "k_steps": spec.get("k_steps"),
                    "accepted": spec.get("num_accepted"), "drafts": spec.get("num_drafts"),
                    "device_error": d.get("device_error")}
            ref, own = rows.get(f"{variant}/reference", {}), rows.get(f"{variant}/nvattn+all", {})
            if "output_tok_per_s" in ref and "output_tok_per_s" in own:
                rows[f"{variant}/speedup"] = round(own["output_tok_per_s"] / ref["output_tok_per_s"], 3)
    rows["workload"] = "64 requests x 1024-token seeded prompts (128-token span repeated 4x), 256 new tokens, T=0"
    return rows


def prefill_flops(q_lens, k_lens, H, D=128):
    """Causal prefill FLOPs: 4*H*D per visible (query, key) pair; query i of a run of q sees k - q + i + 1 keys."""
    pairs = sum(q * (k - q) + q * (q + 1) // 2 for q, k in zip(q_lens, k_lens))
    return 4.0 * H * D * pairs


def varlen_rows(world, rank, args, flush, pk):
    """BASELINE config 4 rows at this rank's head shard: the prefill chunks alone (paged prefix, tensor-core bound),
    a 2048-token prefill without prefix (contiguous K/V), sixteen 1024-token prompts (config 5's prompt shape), and
    the whole mixed step (decode rows HBM-bound)."""
    from nvattn import ops
    from nvattn.workloads import mixed_config, varlen_batch
    H, KVH = 32 // world, 8 // world
    rows = {}

    def timed(b, paged):
        k, v, bt = (b.k_cache, b.v_cache, b.block_tables) if paged else (b.k_new, b.v_new, None)
        out = torch.empty_like(b.q)

        def call():
            ops.flash_attn_varlen_func(b.q, k, v, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=b.cu_seqlens_q,
                                       max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=b.cu_seqlens_k,
                                       softmax_scale=b.scale, causal=True, block_table=bt, out=out)
        t = time_steps(capture(call).replay, max(10, args.steps // 2), args.warmup, flush)
        return max_over_ranks(statistics.mean(t), world)

    chunks, prefixes = [512, 640, 640], [0, 256, 1024]
    kl = [c + p for c, p in zip(chunks, prefixes)]
    b = varlen_batch(chunks, kl, H, KVH, 128, 64, 0.5, args.seed + 40, device="cuda")
    ms = timed(b, True)
    fl = prefill_flops(chunks, kl, H)
    rows["prefill_config4_chunks"] = {"us": round(ms * 1e3, 2), "TFLOPs": round(world * fl / (ms * 1e-3) / 1e12, 1),
                                      "frac_bf16": round(fl / (ms * 1e-3) / 1e12 / pk["bf16"], 3),
                                      "GFLOP_per_rank": round(fl / 1e9, 2)}
    del b
    lens = [512] * 4
    b = varlen_batch(lens, lens, H, KVH, 128, 64, 0.5, args.seed + 41, device="cuda", paged=False)
    ms = timed(b, False)
    fl = prefill_flops(lens, lens, H)
    rows["prefill_4x512_contiguous"] = {"us": round(ms * 1e3, 2), "TFLOPs": round(world * fl / (ms * 1e-3) / 1e12, 1),
                                        "frac_bf16": round(fl / (ms * 1e-3) / 1e12 / pk["bf16"], 3)}
    del b
    # the prompt shape of BASELINE config 5 (1024-token prompts), 16 of them in one prefill step
    lens = [1024] * 16
    b = varlen_batch(lens, lens, H, KVH, 128, 64, 0.5, args.seed + 42, device="cuda", paged=False)
    ms = timed(b, False)
    fl = prefill_flops(lens, lens, H)
    rows["prefill_16x1024_contiguous"] = {"us": round(ms * 1e3, 2),
                                          "TFLOPs": round(world * fl / (ms * 1e-3) / 1e12, 1),
                                          "frac_bf16": round(fl / (ms * 1e-3) / 1e12 / pk["bf16"], 3)}
    del b
    b = mixed_config(seed=args.seed, device="cuda", num_heads=H, num_kv_heads=KVH)
    ms = timed(b, True)
    nd = b.meta["num_decode"]
    dec_bytes = attn_bytes(b.meta["k_lens"][:nd], 1, H, KVH)
    fl = prefill_flops(b.meta["q_lens"][nd:], b.meta["k_lens"][nd:], H)
    bound_us = max(fl / (pk["bf16"] * 1e12), dec_bytes / (pk["hbm"] * 1e9)) * 1e6
    rows["mixed_config4"] = {"us": round(ms * 1e3, 2), "roofline_us": round(bound_us, 2),
                             "frac_of_roofline": round(bound_us / (ms * 1e3), 3),
                             "decode_part_MB": round(dec_bytes / 1e6, 1), "prefill_part_GFLOP": round(fl / 1e9, 2)}
    del b
    return rows


def fa2_rows(world, rank, args, flush, b, q4, lens, H, KVH):
    """The reference's own GPU attention (flash-attn 2.8.3, the calls of attention.py:67-77) on the same workloads,
    same graph-replay timing: context for the numbers above, not part of this arm's measurement."""
    try:
        from flash_attn import flash_attn_varlen_func, flash_attn_with_kvcache
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    rows = {}
    out = {}

    def dec():
        out["o"] = flash_attn_with_kvcache(q4, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                           block_table=b.block_tables, softmax_scale=b.scale, causal=True)
    t = time_steps(capture(dec).replay, max(10, args.steps // 2), args.warmup, flush)
    ms = max_over_ranks(statistics.mean(t), world)
    by = attn_bytes(lens, 1, H, KVH)
    rows["decode_config2"] = {"us": round(ms * 1e3, 2), "GBps": round(world * by / (ms * 1e-3) / 1e9, 1)}
    from nvattn.workloads import varlen_batch
    chunks, prefixes = [512, 640, 640], [0, 256, 1024]
    kl = [c + p for c, p in zip(chunks, prefixes)]
    vb = varlen_batch(chunks, kl, H, KVH, 128, 64, 0.5, args.seed + 40, device="cuda")

    def pre():
        out["p"] = flash_attn_varlen_func(vb.q, vb.k_cache, vb.v_cache, max_seqlen_q=vb.max_seqlen_q,
                                          cu_seqlens_q=vb.cu_seqlens_q, max_seqlen_k=vb.max_seqlen_k,
                                          cu_seqlens_k=vb.cu_seqlens_k, softmax_scale=vb.scale, causal=True,
                                          block_table=vb.block_tables)
    t = time_steps(capture(pre).replay, max(10, args.steps // 2), args.warmup, flush)
    ms = max_over_ranks(statistics.mean(t), world)
    fl = prefill_flops(chunks, kl, H)
    rows["prefill_config4_chunks"] = {"us": round(ms * 1e3, 2), "TFLOPs": round(world * fl / (ms * 1e-3) / 1e12, 1)}
    return rows


def cpu_sample(seed, nseq, total=64):
    """The first nseq sequences of the config-2 batch of `total` sequences (the GPU arm's lengths at N = total / 64),
    generated on the CPU."""
    from nvattn.workloads import paged_decode_batch
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(512, 4097, (total,), generator=g).tolist()[:nseq]
    nblk = sum((L + 255) // 256 for L in lens)
    b = paged_decode_batch(lens, 1, 32, 8, 128, nblk, 0.5, seed + 1, device="cpu")
    return b, lens


def time_oracle(b, lens, reps):
    import oracle
    q = b.q.view(len(lens), 1, 32, 128)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.paged_attention_ref(q, b.k_cache, b.v_cache, b.context_lens, b.block_tables, b.scale)
        best = min(best, time.perf_counter() - t0)
    return best


def cpu_baseline(seed, budget_s=10.0):
    """The FP32 torch restatement of the reference semantics (oracle.paged_attention_ref) on host cores, on a
    bounded sample of the config-2 batch; same metric (algorithmic bytes / s)."""
    b, lens = cpu_sample(seed, 1)
    t1 = time_oracle(b, lens, 1)
    nseq = max(1, min(64, int(budget_s / 3 / max(t1, 1e-3))))
    b, lens = cpu_sample(seed, nseq)
    best = time_oracle(b, lens, 3)
    by = attn_bytes(lens, 1, 32, 8)
    return {"value": round(by / best / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"first {nseq} of the 64 config-2 sequences ({sum(lens)} tokens), best of 3, FP32 torch oracle",
            "host_cpu_count": os.cpu_count()}


def run_reference(args, world, rank):
    """Reference arm: the reference semantics on the host cores (FP32 torch oracle) with every host thread, on this
    arm's whole config-2 job: all 64 x N sequences and all 32 q / 8 kv heads per step (the GPU arm splits the heads
    over its N ranks).  Rank 0 alone runs it."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    nseq = 64 * world
    b, lens = cpu_sample(args.seed, nseq, total=nseq)
    by = attn_bytes(lens, 1, 32, 8)
    import oracle
    q = b.q.view(len(lens), 1, 32, 128)
    warmup = 1 if world > 1 else max(1, min(args.warmup, 3))
    for _ in range(warmup):
        oracle.paged_attention_ref(q, b.k_cache, b.v_cache, b.context_lens, b.block_tables, b.scale)
    steps = max(1, min(args.steps, 20 if world == 1 else 10))
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.paged_attention_ref(q, b.k_cache, b.v_cache, b.context_lens, b.block_tables, b.scale)
    dt = (time.perf_counter() - t0) / steps
    value = by / dt / 1e9
    sample = f"the whole job: all {nseq} config-2 sequences ({sum(lens)} tokens), all heads, per step; {steps} steps"
    line = {"impl": "reference", "metric": "decode attention HBM GB/s (BASELINE config 2: Qwen3-8B paged decode)",
            "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded; BASELINE config 2 shapes)",
            "config": {"workload": "paged decode attention, BASELINE config 2", "global_batch": nseq,
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def aux_kernel_call(case, seed):
    """The two kernels around attention, on workloads larger than L2 (HBM-bound, one pass each):
      argmax    nva_shard_argmax + nva_shard_accept on the largest k = 4 verify step of config 3's shape: 510 rows
                (102 sequences x 5) of 151936 bf16 logits (155 MB), whole vocabulary on one GPU;
      prologue  nva_qk_norm_rope_store on an 8192-token prefill chunk of Qwen3-8B (qkv 8192 x 6144 bf16 in; q, the
                cache rows of k and v out).
    Returns (call, algorithmic bytes per call)."""
    from nvattn import ops
    g = torch.Generator(device="cuda").manual_seed(seed)
    if case == "argmax":
        S, k, V = 102, 4, 151936
        logits = (torch.randn(S * (k + 1), V, generator=g, device="cuda") * 1.3).to(torch.bfloat16)
        drafts = torch.randint(0, V, (S, k), generator=g, device="cuda")
        nd = torch.full((S,), k, dtype=torch.int64, device="cuda")

        def call():
            keys = ops.shard_argmax(logits, 0)
            ops.shard_accept(keys.view(1, S, k + 1), drafts, nd)
        return call, logits.numel() * 2 + S * (k + 1) * 8 * 2
    T, H, KVH, D = 8192, 32, 8, 128
    qkv = (torch.randn(T, (H + 2 * KVH) * D, generator=g, device="cuda")).to(torch.bfloat16)
    pos = torch.arange(T, device="cuda", dtype=torch.int64)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32, device="cuda") / D))
    angles = torch.arange(T, dtype=torch.float32, device="cuda")[:, None] * inv_freq[None, :]
    table = torch.cat((angles.cos(), angles.sin()), dim=-1).contiguous()    # RotaryEmbedding's cos / sin rows
    w = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(T // 256, 256, KVH, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.randperm(T, generator=g, device="cuda").to(torch.int32)

    def call():
        ops.qk_norm_rope_store(qkv, pos, table, w, w, 1e-6, H, KVH, kc, vc, slots)
    # read qkv (+ positions, slots), write q and the k / v cache rows; the cos / sin rows read once per token
    return call, qkv.numel() * 2 + T * H * D * 2 + 2 * T * KVH * D * 2 + T * (8 + 4 + D * 4)


def aux_rows(args, flush, pk):
    """Secondary rows of the kernels around attention (aux_kernel_call): device time of one call, algorithmic
    GB/s, fraction of the measured HBM peak."""
    rows = {}
    for case, name in (("argmax", "shard_argmax_accept_510x151936"), ("prologue", "qk_prologue_8192_tokens")):
        call, by = aux_kernel_call(case, args.seed)
        t = time_steps(capture(call).replay, max(10, args.steps // 2), args.warmup, flush)
        ms = statistics.mean(t)
        rows[name] = {"us": round(ms * 1e3, 2), "GBps": round(by / (ms * 1e-3) / 1e9, 1),
                      "frac_hbm": round(by / (ms * 1e-3) / 1e9 / pk["hbm"], 3), "MB": round(by / 1e6, 1)}
        del call
    return rows


def profile_case(args):
    """One workload launched `--steps` times (after `--warmup` launches) and nothing else: the command the ncu
    summaries under profiles/ capture.  Prints the mean device time per launch (CUDA events, no L2 flush)."""
    from nvattn import ops
    from nvattn.workloads import mixed_config, varlen_batch
    case = args.profile_case
    if case in ("argmax", "prologue"):
        call = aux_kernel_call(case, args.seed)[0]
    elif case in ("decode", "verify4", "verify8"):
        k = 0 if case == "decode" else int(case[len("verify"):])
        b, _, H, KVH = decode_shard(1, 0, args.seed if k == 0 else args.seed + 10, B_per_gpu=64 if k == 0 else 32,
                                    k=k)
        q = b.q.view(b.num_seqs, k + 1, H, 128)
        out = torch.empty_like(q)

        def call():
            ops.flash_attn_with_kvcache(q, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                        block_table=b.block_tables, softmax_scale=b.scale, out=out)
    else:
        if case == "prefill4":
            chunks, prefixes = [512, 640, 640], [0, 256, 1024]
            b = varlen_batch(chunks, [c + p for c, p in zip(chunks, prefixes)], 32, 8, 128, 64, 0.5, args.seed + 40,
                             device="cuda")
        elif case == "prefill16k":
            lens = [1024] * 16
            b = varlen_batch(lens, lens, 32, 8, 128, 64, 0.5, args.seed + 42, device="cuda", paged=False)
        else:
            b = mixed_config(seed=args.seed, device="cuda")
        out = torch.empty_like(b.q)
        paged = b.meta.get("paged", True)
        kk, vv, bt = (b.k_cache, b.v_cache, b.block_tables) if paged else (b.k_new, b.v_new, None)

        def call():
            ops.flash_attn_varlen_func(b.q, kk, vv, max_seqlen_q=b.max_seqlen_q,
                                       cu_seqlens_q=b.cu_seqlens_q, max_seqlen_k=b.max_seqlen_k,
                                       cu_seqlens_k=b.cu_seqlens_k, softmax_scale=b.scale, causal=True,
                                       block_table=bt, out=out)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "launches": args.steps,
                      "us_per_launch": round(e0.elapsed_time(e1) * 1e3 / args.steps, 2)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["nvattn", "reference"], default="nvattn")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e-model", action="store_true", help="skip the config-5 end-to-end rows (N = 1 only)")
    ap.add_argument("--profile-case", choices=["decode", "verify4", "verify8", "prefill4", "prefill16k", "mixed4",
                                               "argmax", "prologue"],
                    help="run one workload --steps times on one GPU (for ncu captures) and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile_case:
        profile_case(args)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    assert world == args.gpus or "WORLD_SIZE" not in os.environ, "--gpus must match the launcher's world size"
    assert 8 % world == 0, "kv heads (8) must split evenly across ranks"
    try:
        run_nvattn(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
