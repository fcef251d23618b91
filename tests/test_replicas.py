"""Multi-process host logic of the multi-GPU runner, on CPU with the gloo backend (world size 2).

Each rank owns a disjoint, contiguous share of the independent sequences, decodes them with no
collective on the data path (here with the CPU oracle, standing in for the per-GPU engine), and the
ranks only exchange their token counts and times afterwards; the whole-box throughput is all tokens
over the slowest rank's time. The tokens each rank produces must equal a single-process run of the
same sequences: sharding changes who decodes a sequence, never what it decodes.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import replicas


def test_shard_covers_every_item_once():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            got = [i for r in range(world) for i in replicas.shard(n, world, r)]
            assert got == list(range(n))
            sizes = [len(replicas.shard(n, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= (1 if n % world else 0)
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)


def test_aggregate_uses_the_slowest_rank():
    agg = replicas.aggregate([replicas.RankTiming(100, 2.0), replicas.RankTiming(100, 4.0)])
    assert agg["tokens"] == 200 and agg["seconds"] == 4.0 and agg["tok_per_s"] == 50.0


def _decode_sequences(model_path: str, seqs, prompt_len: int, steps: int) -> dict:
    import cpu_oracle as co
    import randmodel
    m = co.Model.load_model(model_path)
    out = {}
    for s in seqs:
        cache = co.KVCache(m)
        ids = randmodel.prompt_ids(prompt_len, m.config.vocab_size, seed=replicas.prompt_seed(s))
        logits = None
        for pos, tok in enumerate(ids):
            logits = m.forward(tok, pos, cache)
        tok, toks = co.argmax(logits), []
        for i in range(steps):
            toks.append(tok)
            tok = co.argmax(m.forward(tok, prompt_len + i, cache))
        out[s] = toks
    return out


def _rank_main(rank: int, world: int, port: int, model_path: str, result_path: str) -> None:
    import json
    import time
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = replicas.shard(5, world, rank)
        dist.barrier()
        t0 = time.perf_counter()
        toks = _decode_sequences(model_path, mine, prompt_len=6, steps=4)
        dt = time.perf_counter() - t0
        timings = replicas.reduce_timings(replicas.RankTiming(sum(len(v) for v in toks.values()), dt), group=dist.group.WORLD)
        gathered = [None] * world
        dist.all_gather_object(gathered, toks)
        if rank == 0:
            merged = {int(k): v for d in gathered for k, v in d.items()}
            with open(result_path, "w") as f:
                json.dump({"tokens": merged, "agg": replicas.aggregate(timings),
                           "times": [t.seconds for t in timings]}, f)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_decode_their_shards_like_one_process(tiny_model_path, tmp_path):
    import json
    import torch.multiprocessing as mp
    result = tmp_path / "result.json"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tiny_model_path), str(result)), nprocs=2,
                       join=True, start_method="spawn")
    got = json.loads(result.read_text())
    want = _decode_sequences(str(tiny_model_path), range(5), prompt_len=6, steps=4)
    assert {int(k): v for k, v in got["tokens"].items()} == want
    assert got["agg"]["tokens"] == 5 * 4 and got["agg"]["ranks"] == 2
    assert got["agg"]["seconds"] == pytest.approx(max(got["times"]))
