"""Benchmark: batch-1 Qwen3-0.6B bf16 greedy decode on B200 (the benchmark metric: decode tok/s at batch 1 and the HBM roofline fraction).

Workload (configs[0], the configuration the reference's headline tok/s is quoted on,
metal_infrence_engine/README.md:15-24): the Qwen3-0.6B geometry with seeded random-init bf16
weights, a 130-id seeded prompt fed token by token, then 128 greedy decode steps at positions
130..257, batch 1, f32 KV cache. One bench STEP = one 128-token greedy decode from the prefilled
cache (one launch of the persistent decode kernel). `--config long` selects configs[1] instead
(2048-id prompt, 512 decode steps at positions 2048..2559).

Printed JSON (one line, rank 0):
  value        decode tok/s over all ranks: 128 x steps x N / (max over ranks of the device time of
               the timed steps), tokens and logits resident in HBM (qw_decode_device)
  e2e          the same metric through the public host API qw_decode (host first token in, every
               token streamed back to the host callback), timed with CUDA events on the model's
               stream around each call
  roofline     the decode kernel against the measured HBM copy bandwidth (MEASURED_PEAKS.json):
               achieved = the reference's bytes-per-token rule (tests/mbu.rs:19-37: all weights
               but the embedding table + one embedding row + f32 K/V of positions 0..pos) summed
               over the 128 positions of a launch / average launch time (CUDA events)
  cpu_baseline the CPU oracle (C++ restatement of cpu_inference.rs, all host threads) on a bounded
               sample of the same decode positions
Multi-GPU (torchrun): every rank holds a weight replica and decodes its own independent sequences
(replicas.shard: one per rank for configs[0]/[1], prompt seed 1 + rank; `--config box` shards
configs[4]'s 64 sequences); no collective touches the decode path (weak scaling), and `value` is
all ranks' tokens over the slowest rank's device time.
`--impl reference` times the reference's CPU engine (its C++ restatement; the Rust original cannot
be built here) on the same config, rank 0 only, the way the reference's own bench times it
(metal_infrence_engine/src/bin/bench.rs:166-191: untimed warm-up, a prefill of the prompt, then each
decode token timed as the gap since the previous one).
`--config gemv` is configs[2], the isolated GEMV microbenchmark; `--profile-case decode|prefill|batch`
runs a small fixed workload for ncu captures and prints no bench line.
Cross-rank bookkeeping (the barrier around the timed region and the gather of the ranks' times)
goes through a gloo process group on CPU tensors: nothing on the GPUs is collective.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "mac-gpu-compiler_b200"))

import randmodel  # noqa: E402
import replicas  # noqa: E402

CONFIGS = {
    "ai130": dict(prompt=130, decode=128, label="configs[0]: 130-id prompt token-by-token, then 128 greedy decode steps (pos 130..257)"),
    "long": dict(prompt=2048, decode=512, label="configs[1]: 2048-id prompt token-by-token, then 512 greedy decode steps (pos 2048..2559)"),
    "prefill": dict(prompt=512, decode=64,
                    label="configs[3]: 512-id prompt in one batched prefill pass (tcgen05 GEMMs), then 64 greedy decode steps"),
    "box": dict(prompt=130, decode=128, sequences=64,
                label="configs[4]: 64 independent sequences (130-id prompt + 128 greedy steps each) sharded over the GPUs"),
    "lookup": dict(prompt=130, decode=128, ngram=3, draft=15,
                   label="configs[0] workload with prompt-lookup speculation (qw_decode_lookup, n-gram <= 3, "
                         "draft <= 15): 130-id prompt, then 128 greedy tokens"),
    "box8": dict(prompt=130, decode=128, sequences=64, batch=8,
                 label="configs[4], batch-8 variant: 64 independent sequences (130-id prompt + 128 greedy steps each) "
                       "sharded over the GPUs, decoded 8 at a time per GPU (qw_decode_batch)"),
    "gemv": dict(label="configs[2]: isolated bf16 GEMV y = W x (W ~ N(0, 0.02) bf16, x ~ N(0, 1) f32) at the q 2048x1024, "
                       "k+v 1024x1024, o 1024x2048, gate+up 6144x1024, down 1024x3072 and lm_head 151936x1024 shapes"),
}
GEMV_SHAPES = {"q": (2048, 1024), "kv": (1024, 1024), "o": (1024, 2048), "gate_up": (6144, 1024),
               "down": (1024, 3072), "lm_head": (151936, 1024)}
L2_BYTES = 126 << 20
HBM_SPEC_GBS = 8000.0   # B200 HBM3e, NVIDIA's DGX figure (the HGX figure is 7.7 TB/s)
DECODE_METRIC = "Qwen3-0.6B bf16 decode tok/s @bs1 & % of HBM roofline; box tok/s at 1-8 GPUs"
PREFILL_METRIC = "Qwen3-0.6B bf16 batched prefill tok/s (512-token prompt, per-position logits)"
GEMV_METRIC = "bf16 GEMV GB/s at the decode step's shapes (configs[2]), algorithmic bytes R*C*2 + C*4 + R*4"


def workload_config(name: str, world: int, rows: int = 0) -> dict:
    """The `config` object of a bench line. Both arms (ours and --impl reference) print exactly this
    dict for the same --config and world size: it names the workload, not the engine."""
    c = CONFIGS[name]
    label = c["label"]
    if name == "gemv":
        return {"workload": label, "shapes": {k: list(v) for k, v in GEMV_SHAPES.items()},
                "l2": "every launch reads weight copies larger than 2x the 126 MB L2"}
    d = {"workload": label, "model": "Qwen3-0.6B geometry, random-init bf16 (seed 0)"}
    if name in ("box", "box8"):
        B = rows or c.get("batch", 1)
        if name == "box8" and B != c["batch"]:
            d["workload"] = label.replace("8 at a time", f"{B} at a time")
        d.update(global_batch=c["sequences"], seq_len=c["prompt"] + c["decode"],
                 parallelism=f"replicas x{world}: the {c['sequences']} sequences sharded over the GPUs, no collective")
        if name == "box8":
            d["per_gpu_batch"] = B
    else:
        d.update(global_batch=world, seq_len=c["prompt"] + c["decode"],
                 parallelism=f"replicas x{world}: one independent sequence per GPU, no collective")
    d["l2"] = "inputs larger than L2: 1.19 GB of weights streamed per weight pass"
    return d


# reference's published decode tok/s for this metric and config: Metal engine, f32 KV cache, Apple M1
# (metal_infrence_engine/README.md:22)
PUBLISHED_TPS = 46.37
# DRAM traffic of the decode kernel relative to its algorithmic bytes, from one ncu capture of
# `bench.py --profile-case decode`'s decode launch: a 4-token launch at positions 8..11 read
# 4,777,358,000 B and wrote 4,609,280 B against 4,778,041,344 algorithmic bytes. The bench launch
# (128 tokens, ~158 GB) is too large to capture, and its traffic grows with the same weight + K/V
# bytes per token, so roofline.traffic is that ratio times the launch's algorithmic bytes.
NCU_TRAFFIC_RATIO = (4_777_358_000 + 4_609_280) / 4_778_041_344


def kv_bytes_at(cfg, pos: int) -> int:
    """tests/mbu.rs:32-37 — f32 K and V for every cached position (0..=pos) in every layer."""
    return 2 * cfg.num_hidden_layers * (pos + 1) * cfg.num_key_value_heads * cfg.head_dim * 4


def load_tensor_peak() -> tuple[float, str]:
    """Sustained dense bf16 TFLOP/s (a prefill is a multi-millisecond chain of GEMMs)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), "measured sustained"
        except (ValueError, KeyError):
            pass
    return 1400.0, "fallback sustained"


def prefill_flops(cfg, n: int, start: int = 0) -> float:
    """Algorithmic FLOPs of one prefill pass over n tokens: 2 per weight per token for every
    projection and the lm_head, plus q.k and p.v over each token's causal window (the split-bf16
    operands double the tensor-core work; that is not counted)."""
    H, I, L, V = cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers, cfg.vocab_size
    QD = cfg.num_attention_heads * cfg.head_dim
    KVD = cfg.num_key_value_heads * cfg.head_dim
    per_tok = 2 * L * ((QD + 2 * KVD) * H + H * QD + 2 * I * H + H * I) + 2 * V * H
    attn = sum(4 * QD * (start + t + 1) for t in range(n)) * L
    return float(per_tok * n + attn)


def run_prefill(args, world: int, rank: int, local: int, pg) -> None:
    """one batched prefill of a 512-id prompt per step (device-resident ids and logits,
    CUDA events on the model stream), then 64 greedy decode steps from the prefilled cache."""
    import numpy as np
    import torch
    import cuda_inference as ci
    c = CONFIGS["prefill"]
    n, n_dec = c["prompt"], c["decode"]
    path = randmodel.make_model("qwen3-0.6b", 0)
    model = ci.CudaModel.load_model(path, device=local)
    cfg = model.config
    cache = ci.CudaKVCache(model, n + n_dec + 1)
    ids = randmodel.prompt_ids(n, cfg.vocab_size, seed=replicas.prompt_seed(rank))
    d_ids = torch.tensor(ids, dtype=torch.int32, device=f"cuda:{local}")
    d_logits = torch.empty(n, cfg.vocab_size, dtype=torch.float32, device=f"cuda:{local}")
    stream = torch.cuda.ExternalStream(model.stream)

    def step():
        model.prefill_device(cache, d_ids.data_ptr(), n, 0, d_logits.data_ptr(), stream=model.stream)

    for _ in range(args.warmup):
        step()
    model.sync()
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    model.sync()
    elapsed = t0.elapsed_time(t1) / 1e3
    step_s = statistics.mean(a.elapsed_time(b) for a, b in evs) / 1e3
    timings = replicas.reduce_timings(replicas.RankTiming(n * args.steps, elapsed),
                                      group=pg.group.WORLD if pg is not None else None)
    box = replicas.aggregate(timings)
    # then 64 greedy decode steps from the prefilled cache (the rest of configs[3])
    first = int(torch.argmax(d_logits[-1]).item())
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    toks = model.decode(first, n, n_dec, cache)
    b.record(stream)
    torch.cuda.synchronize()
    dec_s = a.elapsed_time(b) / 1e3
    # e2e through the host API: ids from page-locked host memory in, all logits (n x vocab f32)
    # back out into a page-locked host buffer the caller keeps (one DMA); beside it, a new pageable
    # array per call (the library's pinned stages and host copy threads)
    h_ids = torch.tensor(ids, dtype=torch.int32).pin_memory().numpy().view(np.uint32)
    h_out = torch.empty((n, cfg.vocab_size), dtype=torch.float32).pin_memory().numpy()

    def host_calls(out_fn, reps=4):
        times = []
        for i in range(reps):
            ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ea.record(stream)
            model.prefill(h_ids, 0, cache, out=out_fn())
            eb.record(stream)
            torch.cuda.synchronize()
            if i:
                times.append(ea.elapsed_time(eb) / 1e3)
        return replicas.aggregate(replicas.reduce_timings(replicas.RankTiming(n * len(times), sum(times)),
                                                          group=pg.group.WORLD if pg is not None else None))
    e2e_box = host_calls(lambda: h_out)
    e2e_new = host_calls(lambda: np.empty((n, cfg.vocab_size), np.float32))
    if rank == 0:
        flops = prefill_flops(cfg, n)
        peak, kind = load_tensor_peak()
        achieved = flops / step_s / 1e12
        print(json.dumps({
            "metric": PREFILL_METRIC,
            "value": box["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": box["seconds"] / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "accumulate": "f32 (split-bf16 activations)", "data": "synthetic",
            "config": workload_config("prefill", world),
            "step": f"one {n}-token prefill pass incl. the lm_head over all positions",
            "e2e": {"value": e2e_box["tok_per_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * n * cfg.vocab_size,
                    "api": "qw_prefill (ids from page-locked host memory, logits into a page-locked host buffer)",
                    "new_pageable_array_tok_per_s": e2e_new["tok_per_s"]},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": f"{kind} (bf16_tflops_sustained, cuBLAS)", "traffic": None,
                         "algorithmic_flops_per_step": flops, "kernel": "prefill pass (qw::tc::gemm_bf16x2_kernel + elementwise)"},
            "decode_after_prefill": {"steps": n_dec, "tok_per_s": n_dec / dec_s, "first_tokens": toks[:8]},
            "gpu_launches": args.steps * (1 + 9 * cfg.num_hidden_layers + 2),
            "clocks": clocks.summary(),
        }), flush=True)
    model.close()


def run_batch(args, world: int, rank: int, local: int, pg) -> None:
    """configs[4]'s batch-8 variant: this rank's share of the 64 sequences, in groups of 8 that
    decode together (one captured graph step per token of all 8 rows). A bench step is one
    128-token greedy decode of every group. The weights are read once per step of a group."""
    import numpy as np
    import torch
    import cuda_inference as ci
    c = CONFIGS["box8"]
    n_prompt, n_dec, B = c["prompt"], c["decode"], args.rows or c["batch"]
    path = randmodel.make_model("qwen3-0.6b", 0)
    model = ci.CudaModel.load_model(path, device=local)
    cfg = model.config
    seqs = list(replicas.shard(c["sequences"], world, rank))
    groups = [seqs[i:i + B] for i in range(0, len(seqs), B)]
    caches, firsts = {}, {}
    for sq in seqs:                                    # untimed: batched prefill of all but the last id
        cache = ci.CudaKVCache(model, n_prompt + n_dec + 1)
        ids = randmodel.prompt_ids(n_prompt, cfg.vocab_size, seed=replicas.prompt_seed(sq))
        model.prefill(ids[:-1], 0, cache, logits=False)
        firsts[sq] = int(np.argmax(model.forward(ids[-1], n_prompt - 1, cache)))
        caches[sq] = cache
    dev = f"cuda:{local}"
    d_first = [torch.tensor([firsts[s] for s in g], dtype=torch.int32, device=dev) for g in groups]
    d_out = [torch.zeros(n_dec * len(g), dtype=torch.int32, device=dev) for g in groups]
    stream = torch.cuda.ExternalStream(model.stream)
    torch.cuda.synchronize()

    def step():
        for g, f, o in zip(groups, d_first, d_out):
            model.decode_batch_device(f.data_ptr(), [n_prompt] * len(g), n_dec, [caches[s] for s in g], o.data_ptr(),
                                      stream=model.stream)

    for _ in range(args.warmup):
        step()
    model.sync()
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    model.sync()
    elapsed = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    if pg is not None:
        pg.barrier()
    group_arg = pg.group.WORLD if pg is not None else None
    box = replicas.aggregate(replicas.reduce_timings(replicas.RankTiming(n_dec * args.steps * len(seqs), elapsed),
                                                     group=group_arg))
    dev_tokens = [o.view(n_dec, -1).t().cpu().numpy() for o in d_out]

    # e2e: the host API (qw_decode_batch: host first tokens and positions in, [B][steps] tokens out)
    rounds = max(2, min(args.steps, 3))
    e2e_sec = 0.0
    for i in range(rounds + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for k, g in enumerate(groups):
            got = model.decode_batch([firsts[s] for s in g], [n_prompt] * len(g), n_dec, [caches[s] for s in g])
            assert (got == dev_tokens[k].astype(np.uint32)).all(), "host-API batch decode disagrees with the device one"
        b.record(stream)
        torch.cuda.synchronize()
        if i > 0:
            e2e_sec += a.elapsed_time(b) / 1e3
    e2e_box = replicas.aggregate(replicas.reduce_timings(replicas.RankTiming(n_dec * rounds * len(seqs), e2e_sec),
                                                         group=group_arg))
    if rank == 0:
        W = model.weight_bytes_per_token()
        # algorithmic bytes of one graph step of a group: the weights once, plus every row's K/V history
        step_bytes = [W + sum(kv_bytes_at(cfg, pos) for _ in g) for g in groups[:1] for pos in range(n_prompt, n_prompt + n_dec)]
        bytes_group = sum(step_bytes)
        group_s = elapsed / args.steps / max(1, len(groups))
        achieved = bytes_group / group_s / 1e9
        peak, peak_kind = load_peaks()
        per_step_kernels = 10 * cfg.num_hidden_layers + 4
        line = {
            "metric": DECODE_METRIC,
            "value": box["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": box["seconds"] / args.steps * 1e3,
            "ms_per_batch_token_step": group_s / n_dec * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "accumulate": "f32 (split-bf16 activations)", "data": "synthetic",
            "config": workload_config("box8", world, B),
            "step": f"one {n_dec}-token greedy decode of every group of {B} ({n_dec} graph replays per group; "
                    f"{len(seqs)} sequences on rank 0)",
            "e2e": {"value": e2e_box["tok_per_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * len(seqs) + 8 * len(seqs),
                    "d2h_bytes_per_step": 4 * n_dec * len(seqs), "api": "qw_decode_batch (host tokens in and out)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} (hbm_gbs, copy)", "traffic": None,
                         "algorithmic_bytes_per_group_decode": bytes_group,
                         "kernel": "batch step graph (skinny tcgen05 GEMMs, row attention, elementwise)"},
            "gpu_launches": args.steps * len(groups) * n_dec * per_step_kernels,
            "clocks": clocks.summary(),
            "first_tokens": [int(x) for x in dev_tokens[0][0][:8]] if groups else [],
        }
        print(json.dumps(line), flush=True)
    model.close()


def run_lookup(args, world: int, rank: int, local: int, pg) -> None:
    """configs[0]'s decode through prompt-lookup speculation: a step is one qw_decode_lookup call
    (128 greedy tokens from position 130, drafts looked up in the prompt and the output), timed
    with CUDA events on the model stream. The call is host-driven (each pass's accepted tokens come
    back to the host), so `value` and `e2e` are the same call: host first token in, tokens out."""
    import numpy as np
    import torch
    import cuda_inference as ci
    c = CONFIGS["lookup"]
    n_prompt, n_dec = c["prompt"], c["decode"]
    path = randmodel.make_model("qwen3-0.6b", 0)
    model = ci.CudaModel.load_model(path, device=local)
    cfg = model.config
    ids = randmodel.prompt_ids(n_prompt, cfg.vocab_size, seed=replicas.prompt_seed(rank))
    cache = ci.CudaKVCache(model, n_prompt + n_dec + 1)
    model.prefill(ids[:-1], 0, cache, logits=False)
    first = int(np.argmax(model.forward(ids[-1], n_prompt - 1, cache)))
    plain = model.decode(first, n_prompt, n_dec, cache)
    stream = torch.cuda.ExternalStream(model.stream)

    def step():
        return model.decode_lookup(ids, first, n_prompt, n_dec, cache, max_ngram=c["ngram"], draft_max=c["draft"])

    for _ in range(args.warmup):
        toks, st = step()
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            evs[i][0].record(stream)
            toks, st = step()
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    elapsed = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    box = replicas.aggregate(replicas.reduce_timings(replicas.RankTiming(n_dec * args.steps, elapsed),
                                                     group=pg.group.WORLD if pg is not None else None))
    same = next((i for i in range(n_dec) if toks[i] != plain[i]), n_dec)
    if rank == 0:
        line = {
            "metric": DECODE_METRIC,
            "value": box["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": box["seconds"] / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": box["tok_per_s"] / PUBLISHED_TPS, "dtype": "bf16", "accumulate": "f32", "data": "synthetic",
            "config": workload_config("lookup", world),
            "step": f"one qw_decode_lookup call producing {n_dec} greedy tokens",
            "e2e": {"value": box["tok_per_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * (n_prompt + 1),
                    "d2h_bytes_per_step": 4 * n_dec, "api": "qw_decode_lookup (host-driven passes)"},
            "speculation": {"passes": st["passes"], "drafted": st["drafted"], "accepted": st["accepted"],
                            "tokens_per_pass": n_dec / st["passes"],
                            "equal_to_plain_decode_for_first": same},
            "clocks": clocks.summary(),
            "first_tokens": toks[:8],
        }
        print(json.dumps(line), flush=True)
    model.close()


def read_probe_gbs(local: int, gib: int = 4, reps: int = 5) -> float:
    """Best read-only streaming rate of this GPU (qw_read_probe: the CUDA twin of the reference's
    tests/read_bandwidth.rs:16-54) over a buffer far larger than L2; a second roofline denominator
    next to the measured copy bandwidth."""
    import torch
    import cuda_inference as ci
    n = (gib << 30) // 4
    src = torch.ones(n, dtype=torch.float32, device=f"cuda:{local}")
    parts = torch.empty(4096, dtype=torch.float32, device=f"cuda:{local}")
    ci.read_probe(local, src.data_ptr(), n, parts.data_ptr(), parts.numel())
    best = float("inf")
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ci.read_probe(local, src.data_ptr(), n, parts.data_ptr(), parts.numel())
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / 1e3)
    del src
    return n * 4 / best / 1e9


def run_gemv(args, world: int, rank: int, local: int, pg) -> None:
    """the isolated GEMV at the decode step's shapes. Per shape, enough stacked copies of
    W that their bytes exceed 2x L2 are multiplied by one x in ONE qw_gemv_bf16_seq launch (every
    CTA streams its rows of copy after copy, as the decode kernel streams layer after layer), timed
    with CUDA events over `steps` launches; single qw_gemv_bf16 launches over the rotated copies are
    timed too (launch-bound for the layer shapes). value = all shapes' algorithmic bytes over their
    streaming time."""
    import torch
    import cuda_inference as ci
    dev = f"cuda:{local}"
    stream = torch.cuda.current_stream().cuda_stream
    shapes, tot_b, tot_s, e2e_s = {}, 0, 0.0, 0.0
    h2d = d2h = 0
    with ClockSampler(local) as clocks:
        for name, (R, C) in GEMV_SHAPES.items():
            g = torch.Generator(device=dev).manual_seed(R + C)
            count = max(2, -(-2 * L2_BYTES // (R * C * 2)))
            w = (torch.randn(count, R, C, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            x = torch.randn(C, device=dev, generator=g)
            y = torch.empty(count, R, device=dev)
            for _ in range(args.warmup):
                ci.gemv_bf16_seq(local, w.data_ptr(), x.data_ptr(), y.data_ptr(), R, C, count, stream)
            torch.cuda.synchronize()
            err = float((y[count - 1].double() - w[count - 1].double() @ x.double()).abs().max())
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                ci.gemv_bf16_seq(local, w.data_ptr(), x.data_ptr(), y.data_ptr(), R, C, count, stream)
            b.record()
            torch.cuda.synchronize()
            seq_s = a.elapsed_time(b) / 1e3 / args.steps
            a.record()
            for i in range(args.steps * 4):
                m = i % count
                ci.gemv_bf16(local, w[m].data_ptr(), x.data_ptr(), y[m].data_ptr(), R, C, stream)
            b.record()
            torch.cuda.synchronize()
            one_s = a.elapsed_time(b) / 1e3 / (args.steps * 4)
            # e2e: x from pinned host memory in, all count outputs back to pinned host memory
            hx = x.cpu().pin_memory()
            hy = torch.empty(count, R, pin_memory=True)
            a.record()
            for _ in range(args.steps):
                x.copy_(hx, non_blocking=True)
                ci.gemv_bf16_seq(local, w.data_ptr(), x.data_ptr(), y.data_ptr(), R, C, count, stream)
                hy.copy_(y, non_blocking=True)
            b.record()
            torch.cuda.synchronize()
            e2e_one = a.elapsed_time(b) / 1e3 / args.steps
            algo = R * C * 2 + C * 4 + R * 4
            shapes[name] = {"rows": R, "cols": C, "copies": count, "stream_GB_s": count * algo / seq_s / 1e9,
                            "stream_us_per_matrix": seq_s / count * 1e6, "single_launch_us": one_s * 1e6,
                            "single_launch_GB_s": algo / one_s / 1e9, "max_abs_err_vs_f64": err}
            tot_b += count * algo
            tot_s += seq_s
            e2e_s += e2e_one
            h2d += C * 4
            d2h += count * R * 4
            del w, y
    peak, peak_kind = load_peaks()
    value = tot_b / tot_s / 1e9
    if rank == 0:
        for v in shapes.values():
            v["frac_of_measured_copy"] = v["stream_GB_s"] / peak
        print(json.dumps({
            "metric": GEMV_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tot_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "accumulate": "f32", "data": "synthetic",
            "config": workload_config("gemv", world),
            "step": "one qw_gemv_bf16_seq launch per shape over its stacked copies",
            "e2e": {"value": tot_b / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "qw_gemv_bf16_seq with x copied in from pinned host memory and y copied back"},
            "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                         "peak_kind": f"{peak_kind} (hbm_gbs, copy)", "traffic": None,
                         "peak_spec": HBM_SPEC_GBS, "frac_of_spec": value / HBM_SPEC_GBS,
                         "kernel": "gemv_kernel (the decode kernel's ring producer and GEMV consumer)"},
            "shapes": shapes, "gpu_launches": len(GEMV_SHAPES) * (args.warmup + 2 * args.steps + 4 * args.steps),
            "clocks": clocks.summary(),
        }), flush=True)


def run_profile_case(args) -> None:
    """Small fixed workloads for ncu captures (no bench line). decode: --case-prompt single-token
    forward() launches, then one --case-steps-step decode() launch (every launch is
    qw::decode_kernel). prefill: --case-steps passes of qw_prefill_device over a --case-prompt-id
    prompt. batch: --case-batch caches prefilled with --case-prompt ids, then --case-steps greedy
    batch steps (one graph replay each)."""
    import numpy as np
    import torch
    import cuda_inference as ci
    geom = args.case_geometry
    m = ci.CudaModel.load_model(randmodel.make_model(geom, 0))
    V = m.config.vocab_size
    if args.profile_case == "decode":
        cache = ci.CudaKVCache(m, args.case_prompt + args.case_steps + 1)
        ids = randmodel.prompt_ids(args.case_prompt, V, seed=1)
        logits = None
        for pos, tok in enumerate(ids):
            logits = m.forward(tok, pos, cache)
        toks = m.decode(int(np.argmax(logits)), args.case_prompt, args.case_steps, cache)
        print(f"{geom}: {args.case_prompt} forward launches + 1 decode launch of {args.case_steps} steps -> {toks}")
    elif args.profile_case == "prefill":
        cache = ci.CudaKVCache(m, args.case_prompt + 1)
        ids = torch.tensor(randmodel.prompt_ids(args.case_prompt, V, seed=1), dtype=torch.int32, device="cuda")
        logits = torch.empty(args.case_prompt, V, device="cuda")
        for _ in range(args.case_steps):
            m.prefill_device(cache, ids.data_ptr(), args.case_prompt, 0, logits.data_ptr())
        m.sync()
        print(f"{geom}: {args.case_steps} prefill passes of {args.case_prompt} tokens; last argmax {int(logits[-1].argmax())}")
    else:
        caches, firsts = [], []
        for b in range(args.case_batch):
            c = ci.CudaKVCache(m, args.case_prompt + args.case_steps + 1)
            ids = randmodel.prompt_ids(args.case_prompt, V, seed=1 + b)
            m.prefill(ids[:-1], 0, c, logits=False)
            firsts.append(int(np.argmax(m.forward(ids[-1], args.case_prompt - 1, c))))
            caches.append(c)
        out = m.decode_batch(firsts, [args.case_prompt] * args.case_batch, args.case_steps, caches)
        print(f"{geom}: batch {args.case_batch}, {args.case_steps} steps from position {args.case_prompt}; "
              f"first row {out[0].tolist()}")
    m.close()


def load_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        # a reader thread collects samples; entering waits (up to 3 s) for the first one, so a short
        # timed region still falls inside the sampling window
        self.lines = []
        self._thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        first = threading.Event()

        def read():
            for l in self.proc.stdout:
                if l.strip():
                    self.lines.append(l.strip())
                    first.set()
            first.set()

        self._thread = threading.Thread(target=read, daemon=True)
        self._thread.start()
        first.wait(timeout=3.0)
        self._start = len(self.lines)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            n = len(self.lines)
            deadline = time.time() + 0.5
            while len(self.lines) <= n and time.time() < deadline:  # one sample at the end of the region
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            if self._thread is not None:
                self._thread.join(timeout=5)
        return False

    def summary(self) -> dict:
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
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_oracle as co
    return co


def model_file(geometry: str = "qwen3-0.6b") -> Path:
    """The seeded random-init model file. A child process writes it if it is missing, so the CPU-engine
    timings map only the oracle's library, never one of this repository's product libraries."""
    subprocess.run([sys.executable, str(ROOT / "mac-gpu-compiler_b200" / "randmodel.py"), "--geometry", geometry,
                    "--seed", "0"], check=True, stdout=subprocess.DEVNULL)
    return randmodel.make_model(geometry, 0)   # present now: returns the path without writing


def cpu_decode_timing(co, m, cfg_name: str, warmup: int, n_tokens: int, chunks: int = 1,
                      budget_s: float | None = None) -> dict:
    """The reference bench's decode timing on the CPU engine (metal_infrence_engine/src/bin/bench.rs:
    166-191): untimed warm-up, a prefill of the workload's prompt, then greedy decode from the
    prompt's argmax with each token timed as the gap since the previous one (forward + argmax).
    The prefill runs layer by layer over the prompt (forward_seq), which leaves the same cache, bit
    for bit, as the reference's token-by-token loop; it is not timed there either. At most
    n_tokens tokens are timed (fewer once budget_s is spent), split into `chunks` bench steps."""
    c = CONFIGS[cfg_name]
    V = m.config.vocab_size
    scratch = co.KVCache(m)
    for i in range(warmup):                      # pages in the mmap'd weights, warms the threads
        m.forward(1 + i, i, scratch)
    del scratch
    ids = randmodel.prompt_ids(c["prompt"], V, seed=replicas.prompt_seed(0))
    cache = co.KVCache(m)
    last = m.forward_seq(ids, 0, cache, out_positions=[len(ids) - 1])[0]
    tok, pos = co.argmax(last), len(ids)
    gaps, chunk_s = [], []
    per = max(1, -(-n_tokens // max(1, chunks)))
    t_last = time.perf_counter()
    for k in range(max(1, chunks)):
        t_chunk = time.perf_counter()
        for _ in range(per):
            if len(gaps) >= n_tokens or (budget_s is not None and sum(gaps) > budget_s):
                break
            tok = co.argmax(m.forward(tok, pos, cache))
            pos += 1
            now = time.perf_counter()
            gaps.append(now - t_last)
            t_last = now
        chunk_s.append(time.perf_counter() - t_chunk)
        t_last = time.perf_counter()
    n = len(gaps)
    return {"tokens": n, "seconds": sum(gaps), "tok_per_s": n / sum(gaps), "first_pos": len(ids),
            "last_pos": len(ids) + n - 1, "chunk_s": chunk_s, "threads": co.threads()}


def cpu_prefill_timing(co, m, warmup: int, n_tokens: int) -> dict:
    """The reference's prefill of the 512-id prompt: token-by-token forward from an empty cache at
    positions 0..n-1 (cpu_inference.rs:100-179), each token timed; at most n_tokens are timed."""
    c = CONFIGS["prefill"]
    ids = randmodel.prompt_ids(c["prompt"], m.config.vocab_size, seed=replicas.prompt_seed(0))
    scratch = co.KVCache(m)
    for i in range(warmup):
        m.forward(ids[i % len(ids)], i, scratch)
    del scratch
    cache = co.KVCache(m)
    t0 = time.perf_counter()
    n = min(n_tokens, len(ids))
    for pos in range(n):
        m.forward(ids[pos], pos, cache)
    dt = time.perf_counter() - t0
    return {"tokens": n, "seconds": dt, "tok_per_s": n / dt, "first_pos": 0, "last_pos": n - 1, "threads": co.threads()}


def cpu_gemv_timing(co, reps: int = 3) -> dict:
    """The reference's matvec (cpu_inference.rs:225-257, host threads over rows) at configs[2]'s
    shapes: GB/s of the algorithmic bytes R*C*2 + C*4 + R*4, best of `reps` calls per shape."""
    import numpy as np
    rng = np.random.Generator(np.random.PCG64(7))
    per, tot_b, tot_s = {}, 0, 0.0
    for name, (R, C) in GEMV_SHAPES.items():
        w = (rng.standard_normal((R, C), dtype=np.float32) * 0.02).view(np.uint32) >> 16
        w = w.astype(np.uint16)
        x = rng.standard_normal(C, dtype=np.float32)
        best = float("inf")
        for _ in range(reps):
            t0 = time.perf_counter()
            co.matvec(w, x)
            best = min(best, time.perf_counter() - t0)
        b = R * C * 2 + C * 4 + R * 4
        per[name] = {"us_per_call": best * 1e6, "GB_s": b / best / 1e9}
        tot_b += b
        tot_s += best
    return {"GB_s": tot_b / tot_s / 1e9, "shapes": per, "threads": co.threads()}


def cpu_sample(path, cfg_name: str, budget_s: float = 15.0) -> dict:
    """cpu_baseline of our arm: the CPU oracle on the host cores, on a bounded sample of the same
    workload, timed like the reference bench (see cpu_decode_timing)."""
    co = _oracle()
    m = co.Model.load_model(path)
    if cfg_name == "prefill":
        r = cpu_prefill_timing(co, m, warmup=2, n_tokens=96)
        return {"value": r["tok_per_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                "sample": f"token-by-token prefill of positions 0..{r['last_pos']} of the 512-id prompt from an "
                          f"empty cache, {r['threads']} host threads"}
    n = CONFIGS[cfg_name].get("decode", 128)
    r = cpu_decode_timing(co, m, "ai130" if cfg_name in ("box", "box8", "lookup") else cfg_name, warmup=2,
                          n_tokens=min(n, 128), budget_s=budget_s)
    return {"value": r["tok_per_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
            "sample": f"{r['tokens']} greedy decode tokens at positions {r['first_pos']}..{r['last_pos']} after the "
                      f"workload's real {r['first_pos']}-id prompt prefill, each timed as the gap between tokens "
                      f"(bench.rs:166-191), {r['threads']} host threads"}


def run_reference(args, cfg_name: str) -> None:
    """The reference's CPU engine (the oracle: C++ restatement of cpu_inference.rs, all host threads)
    on our arm's metric, unit and config. Rank 0 runs it; other ranks exit without work."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    co = _oracle()
    c = CONFIGS[cfg_name]
    path = model_file("qwen3-0.6b")
    m = co.Model.load_model(path)
    line = {"impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong" if cfg_name in ("box", "box8") else "weak",
            "dtype": "bf16", "accumulate": "f32", "data": "synthetic", "config": workload_config(cfg_name, world),
            "engine": "CPU oracle: C++ restatement of metal_infrence_engine/src/cpu_inference.rs (the Rust "
                      "original needs cargo, absent on these machines)"}
    if cfg_name == "gemv":
        r = cpu_gemv_timing(co)
        v, unit = r["GB_s"], "GB/s"
        line.update(metric=GEMV_METRIC, value=v, unit=unit, ms_per_step=None, shapes=r["shapes"])
        sample = f"one matvec per shape (best of 3), {r['threads']} host threads"
    elif cfg_name == "prefill":
        n = max(args.steps, min(c["prompt"], 4 * args.steps))
        r = cpu_prefill_timing(co, m, warmup=args.warmup, n_tokens=n)
        v, unit = r["tok_per_s"], "tok/s"
        line.update(metric=PREFILL_METRIC, value=v, unit=unit, ms_per_step=r["seconds"] / args.steps * 1e3)
        sample = (f"token-by-token prefill (how the reference prefills) of positions 0..{r['last_pos']} of the "
                  f"{c['prompt']}-id prompt from an empty cache, {r['threads']} host threads")
    else:
        base = "ai130" if cfg_name in ("box", "box8", "lookup") else cfg_name
        n_dec = CONFIGS[base]["decode"]
        n = max(args.steps, min(n_dec, 128))
        r = cpu_decode_timing(co, m, base, warmup=args.warmup, n_tokens=n, chunks=args.steps)
        v, unit = r["tok_per_s"], "tok/s"
        line.update(metric=DECODE_METRIC, value=v, unit=unit, ms_per_step=r["seconds"] / args.steps * 1e3)
        sample = (f"{r['tokens']} greedy decode tokens at positions {r['first_pos']}..{r['last_pos']} after a prefill "
                  f"of the workload's {r['first_pos']}-id prompt, each timed as the gap since the previous token "
                  f"(bench.rs:166-191), {args.warmup} untimed warm-up forwards, {r['threads']} host threads")
    line["cpu_baseline"] = {"value": v, "unit": unit, "cores": co.threads(), "kind": "port", "sample": sample}
    line["e2e"] = {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="ai130", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=0, help="box8: sequences decoded together per GPU (default 8, at most 16)")
    ap.add_argument("--profile-case", choices=["decode", "prefill", "batch"], default=None,
                    help="run a small fixed workload for an ncu capture instead of the bench")
    ap.add_argument("--case-geometry", default="qwen3-0.6b", choices=sorted(randmodel.GEOMETRIES))
    ap.add_argument("--case-prompt", type=int, default=None, help="profile case prompt ids (decode 8, prefill 512, batch 130)")
    ap.add_argument("--case-steps", type=int, default=None, help="profile case steps / passes (decode 4, prefill 2, batch 4)")
    ap.add_argument("--case-batch", type=int, default=8)
    args = ap.parse_args()
    if args.profile_case:
        dflt = {"decode": (8, 4), "prefill": (512, 2), "batch": (130, 4)}[args.profile_case]
        args.case_prompt = args.case_prompt or dflt[0]
        args.case_steps = args.case_steps or dflt[1]
        run_profile_case(args)
        return
    if args.impl == "reference":
        run_reference(args, args.config)
        return

    import numpy as np
    import torch
    import cuda_inference as ci

    world, rank, local = dist_setup()
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # gloo on CPU tensors: only the barrier and the gather of the ranks' times cross ranks
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        pg = dist
    if args.config in ("prefill", "box8", "lookup", "gemv"):
        {"prefill": run_prefill, "box8": run_batch, "lookup": run_lookup, "gemv": run_gemv}[args.config](
            args, world, rank, local, pg)
        if pg is not None:
            pg.barrier()
            pg.destroy_process_group()
        return

    c = CONFIGS[args.config]
    n_prompt, n_dec = c["prompt"], c["decode"]
    path = randmodel.make_model("qwen3-0.6b", 0)
    model = ci.CudaModel.load_model(path, device=local)
    cfg = model.config
    # this rank's independent sequences: one per rank (its own prompt seed), or a share of configs[4]'s 64
    seqs = replicas.shard(c.get("sequences", world), world, rank)
    caches, toks_dev, firsts = [], [], []
    for sq in seqs:
        cache = ci.CudaKVCache(model, n_prompt + n_dec + 1)
        ids = randmodel.prompt_ids(n_prompt, cfg.vocab_size, seed=replicas.prompt_seed(sq))
        logits = None
        for pos, tok in enumerate(ids):              # token-by-token prefill (untimed)
            logits = model.forward(tok, pos, cache)
        first = int(np.argmax(logits))
        t = torch.zeros(n_dec + 1, dtype=torch.int32, device=f"cuda:{local}")
        t[0] = first
        caches.append(cache)
        toks_dev.append(t)
        firsts.append(first)
    stream = torch.cuda.ExternalStream(model.stream)
    torch.cuda.synchronize()

    def barrier():
        if pg is not None:
            pg.barrier()

    def step():  # one greedy decode of n_dec tokens per sequence of this rank, one launch each
        for cache, t in zip(caches, toks_dev):
            model.decode_device(cache, t.data_ptr(), n_prompt, n_dec, stream=model.stream)

    for _ in range(args.warmup):
        step()
    model.sync()
    barrier()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t_start.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    model.sync()
    elapsed = t_start.elapsed_time(t_end) / 1e3
    launch_ms = [a.elapsed_time(b) / max(1, len(seqs)) for a, b in evs]
    barrier()
    # every rank's (tokens, device seconds): whole-box tok/s = all tokens / the slowest rank's time
    timings = replicas.reduce_timings(replicas.RankTiming(n_dec * args.steps * len(seqs), elapsed),
                                      group=pg.group.WORLD if pg is not None else None)
    box = replicas.aggregate(timings)
    elapsed_max = box["seconds"]

    out_tokens = toks_dev[0].cpu().tolist() if seqs else []

    # e2e through the public host API (qw_decode: host first token in, every token streamed to the
    # host callback), each sequence of this rank once per round, timed with events on the model stream
    rounds = max(2, min(args.steps, 5))
    e2e_sec = 0.0
    for i in range(rounds + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for k, cache in enumerate(caches):
            got = model.decode(firsts[k], n_prompt, n_dec, cache)
            if k == 0:
                assert got == out_tokens[1:], "host-API decode disagrees with the device-resident decode"
        b.record(stream)
        torch.cuda.synchronize()
        if i > 0:
            e2e_sec += a.elapsed_time(b) / 1e3
    e2e_box = replicas.aggregate(replicas.reduce_timings(replicas.RankTiming(n_dec * rounds * len(seqs), e2e_sec),
                                                         group=pg.group.WORLD if pg is not None else None))

    if rank == 0:
        probe = read_probe_gbs(local)
        W = model.weight_bytes_per_token()
        bytes_launch = sum(W + kv_bytes_at(cfg, pos) for pos in range(n_prompt, n_prompt + n_dec))
        avg_launch = statistics.mean(launch_ms) / 1e3
        achieved = bytes_launch / avg_launch / 1e9
        peak, peak_kind = load_peaks()
        value = box["tok_per_s"]
        traffic = NCU_TRAFFIC_RATIO * bytes_launch
        line = {
            "metric": DECODE_METRIC,
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_max / args.steps * 1e3,
            "ms_per_token": elapsed_max / args.steps / n_dec / max(1, len(seqs)) * 1e3,
            "higher_is_better": True, "scaling": "strong" if args.config == "box" else "weak",
            "vs_baseline": value / PUBLISHED_TPS if args.config == "ai130" else None,
            "vs_baseline_ref": "reference Metal engine, f32 KV, Apple M1: 46.37 tok/s (README.md:22)",
            "dtype": "bf16", "accumulate": "f32", "data": "synthetic",
            "config": workload_config(args.config, world),
            "step": f"one {n_dec}-token greedy decode per sequence = one decode-kernel launch each "
                    f"({len(seqs)} sequences on rank 0)",
            "e2e": {"value": e2e_box["tok_per_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * len(seqs),
                    "d2h_bytes_per_step": 4 * n_dec * len(seqs), "api": "qw_decode (host callback per token)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} (hbm_gbs, copy)", "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-token launch, scaled by algorithmic bytes",
                         "algorithmic_bytes_per_launch": bytes_launch,
                         "kernel": "qw::decode_kernel", "avg_launch_ms": avg_launch * 1e3,
                         "peak_spec": HBM_SPEC_GBS, "frac_of_spec": achieved / HBM_SPEC_GBS,
                         "peak_read_probe": probe, "frac_of_read_probe": achieved / probe,
                         "read_probe": "qw_read_probe over 4 GiB (read-only stream, best of 5), this GPU, this run"},
            "gpu_launches": args.steps * len(seqs),
            "clocks": clocks.summary(),
            "first_tokens": out_tokens[1:9],
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_sample(path, args.config)
        print(json.dumps(line), flush=True)
    model.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
