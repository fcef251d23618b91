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
be built here) on the same config, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
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
}
# reference's published decode tok/s for this metric and config: Metal engine, f32 KV cache, Apple M1
# (metal_infrence_engine/README.md:22)
PUBLISHED_TPS = 46.37
# DRAM traffic of the decode kernel relative to its algorithmic bytes, from one ncu capture of
# mac-gpu-compiler_b200/profile_case.py's decode launch: a 4-token launch at positions 8..11 read
# 4,777,855,000 B and wrote 5,338,112 B against 4,778,041,344 algorithmic bytes. The bench launch
# (128 tokens, ~158 GB) is too large to capture, and its traffic grows with the same weight + K/V
# bytes per token, so roofline.traffic is that ratio times the launch's algorithmic bytes.
NCU_TRAFFIC_RATIO = (4_777_855_000 + 5_338_112) / 4_778_041_344


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
    # e2e through the host API: ids from host memory in, all logits (n x vocab f32) back out
    e2e = []
    for i in range(3):
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record(stream)
        model.prefill(ids, 0, cache)
        eb.record(stream)
        torch.cuda.synchronize()
        if i:
            e2e.append(ea.elapsed_time(eb) / 1e3)
    e2e_box = replicas.aggregate(replicas.reduce_timings(replicas.RankTiming(n * len(e2e), sum(e2e)),
                                                         group=pg.group.WORLD if pg is not None else None))
    if rank == 0:
        flops = prefill_flops(cfg, n)
        peak, kind = load_tensor_peak()
        achieved = flops / step_s / 1e12
        print(json.dumps({
            "metric": "Qwen3-0.6B bf16 batched prefill tok/s (512-token prompt, per-position logits)",
            "value": box["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": box["seconds"] / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "accumulate": "f32 (split-bf16 activations)", "data": "synthetic",
            "config": {"workload": c["label"], "model": "Qwen3-0.6B geometry, random-init bf16 (seed 0)",
                       "global_batch": world, "seq_len": n + n_dec,
                       "parallelism": f"replicas x{world}, one independent prompt per GPU, no collective",
                       "step": f"one {n}-token prefill pass incl. the lm_head over all positions"},
            "e2e": {"value": e2e_box["tok_per_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * n * cfg.vocab_size, "api": "qw_prefill (host ids in, host logits out)"},
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
            "metric": "Qwen3-0.6B bf16 decode tok/s @bs1 & % of HBM roofline; box tok/s at 1-8 GPUs",
            "value": box["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": box["seconds"] / args.steps * 1e3,
            "ms_per_batch_token_step": group_s / n_dec * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "accumulate": "f32 (split-bf16 activations)", "data": "synthetic",
            "config": {"workload": c["label"] if B == c["batch"] else c["label"].replace("8 at a time", f"{B} at a time"),
                       "model": "Qwen3-0.6B geometry, random-init bf16 (seed 0)",
                       "global_batch": c["sequences"], "per_gpu_batch": B, "seq_len": n_prompt + n_dec,
                       "parallelism": f"replicas x{world}, {len(seqs)} sequences on rank 0 in groups of {B}, no collective",
                       "l2": "inputs larger than L2: 1.19 GB of weights streamed per batch step",
                       "step": f"one {n_dec}-token greedy decode of every group ({n_dec} graph replays per group)"},
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
            "metric": "Qwen3-0.6B bf16 decode tok/s @bs1 & % of HBM roofline; box tok/s at 1-8 GPUs",
            "value": box["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": box["seconds"] / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": box["tok_per_s"] / PUBLISHED_TPS, "dtype": "bf16", "accumulate": "f32", "data": "synthetic",
            "config": {"workload": c["label"], "model": "Qwen3-0.6B geometry, random-init bf16 (seed 0)",
                       "global_batch": world, "seq_len": n_prompt + n_dec,
                       "parallelism": f"replicas x{world}, one sequence per rank, no collective",
                       "step": f"one qw_decode_lookup call producing {n_dec} greedy tokens"},
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
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
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


def cpu_sample(path, cfg_name: str, budget_s: float = 12.0) -> dict:
    """Times the CPU oracle on decode positions of the workload: the cache is pre-filled with
    synthetic K/V for the prompt positions (untimed), then decode tokens are timed."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_oracle as co
    c = CONFIGS[cfg_name]
    m = co.Model.load_model(path)
    cache = co.KVCache(m)
    cache.fill_synthetic(c["prompt"], seed=0)
    tok, pos = 1, c["prompt"]
    t0 = time.perf_counter()
    m.forward(tok, pos, cache)   # warm-up token (pages in the mmap)
    first = time.perf_counter() - t0
    n = max(2, min(c["decode"], int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for i in range(n):
        lg = m.forward(tok, pos + 1 + i, cache)
        tok = co.argmax(lg)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": co.threads(), "kind": "port",
            "sample": f"{n} greedy decode tokens at positions {pos + 1}..{pos + n} after a synthetic "
                      f"{c['prompt'] + 1}-position K/V cache, {co.threads()} host threads"}


def run_reference(args, cfg_name: str) -> None:
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_oracle as co
    c = CONFIGS[cfg_name]
    path = randmodel.make_model("qwen3-0.6b", 0)
    m = co.Model.load_model(path)
    cache = co.KVCache(m)
    cache.fill_synthetic(c["prompt"], seed=0)
    per_step = 2   # decode tokens per bench step: keeps the whole run within a few minutes
    pos, tok = c["prompt"], 1
    for _ in range(args.warmup):
        for _ in range(per_step):
            tok = co.argmax(m.forward(tok, pos, cache))
            pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(per_step):
            tok = co.argmax(m.forward(tok, pos, cache))
            pos += 1
    dt = time.perf_counter() - t0
    v = per_step * args.steps / dt
    sample = (f"{per_step} greedy decode tokens per step at positions {c['prompt']}..{pos - 1} after a "
              f"synthetic {c['prompt']}-position K/V cache, {co.threads()} host threads")
    print(json.dumps({
        "impl": "reference",
        "metric": ("Qwen3-0.6B bf16 batched prefill tok/s (512-token prompt, per-position logits)" if cfg_name == "prefill"
                   else "Qwen3-0.6B bf16 decode tok/s @bs1 & % of HBM roofline; box tok/s at 1-8 GPUs"),
        "value": v, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
        "config": {"workload": c["label"], "model": "Qwen3-0.6B geometry, random-init bf16 (seed 0)",
                   "global_batch": c.get("sequences", 1), "seq_len": c["prompt"] + c["decode"],
                   "engine": "CPU oracle: C++ restatement of metal_infrence_engine/src/cpu_inference.rs "
                             "(the Rust original needs cargo, absent on these machines)"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": co.threads(), "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="ai130", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=0, help="box8: sequences decoded together per GPU (default 8, at most 16)")
    args = ap.parse_args()
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    if args.config in ("prefill", "box8", "lookup"):
        {"prefill": run_prefill, "box8": run_batch, "lookup": run_lookup}[args.config](args, world, rank, local, pg)
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
        W = model.weight_bytes_per_token()
        bytes_launch = sum(W + kv_bytes_at(cfg, pos) for pos in range(n_prompt, n_prompt + n_dec))
        avg_launch = statistics.mean(launch_ms) / 1e3
        achieved = bytes_launch / avg_launch / 1e9
        peak, peak_kind = load_peaks()
        value = box["tok_per_s"]
        traffic = NCU_TRAFFIC_RATIO * bytes_launch
        line = {
            "metric": "Qwen3-0.6B bf16 decode tok/s @bs1 & % of HBM roofline; box tok/s at 1-8 GPUs",
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_max / args.steps * 1e3,
            "ms_per_token": elapsed_max / args.steps / n_dec / max(1, len(seqs)) * 1e3,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / PUBLISHED_TPS if args.config == "ai130" else None,
            "vs_baseline_ref": "reference Metal engine, f32 KV, Apple M1: 46.37 tok/s (README.md:22)",
            "dtype": "bf16", "accumulate": "f32", "data": "synthetic",
            "config": {"workload": c["label"], "model": "Qwen3-0.6B geometry, random-init bf16 (seed 0)",
                       "global_batch": box["tokens"] // (n_dec * args.steps), "seq_len": n_prompt + n_dec,
                       "parallelism": f"replicas x{world}, independent sequences sharded over the GPUs "
                                      f"({len(seqs)} on rank 0), no collective",
                       "l2": "inputs larger than L2: 1.19 GB of weights streamed per token",
                       "step": f"one {n_dec}-token greedy decode per sequence = one decode-kernel launch each"},
            "e2e": {"value": e2e_box["tok_per_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * len(seqs),
                    "d2h_bytes_per_step": 4 * n_dec * len(seqs), "api": "qw_decode (host callback per token)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} (hbm_gbs, copy)", "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-token launch, scaled by algorithmic bytes",
                         "algorithmic_bytes_per_launch": bytes_launch,
                         "kernel": "qw::decode_kernel", "avg_launch_ms": avg_launch * 1e3},
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
