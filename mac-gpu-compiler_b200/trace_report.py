"""Phase-timeline report of one decode token (the engine's tracing facility).

Prefills `--pos` tokens with forward(), enables tracing, runs one more forward() (one launch =
one token) and prints, per phase hand-off, the median and max over CTAs of each interval
(averaged over layers), plus the whole token's span. Stamps are %globaltimer (ns) taken by each
CTA's thread 0 at the points listed in decode_kernel.cuh (TRACE_PER_LAYER).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import numpy as np  # noqa: E402

import cuda_inference as ci  # noqa: E402
import randmodel  # noqa: E402

TPL = 14
# the cluster kernel's stamps per layer (cluster_decode.cuh): 0 layer start, 1 x*ln1 in hand, 2 q|k|v
# of the head group in hand, 3 q/k norm + RoPE done, 4 this CTA's attention partial ready,
# 5 all 16 partials in hand, 6 attention merged, 7 o_proj rows published, 8 x*ln2 in hand,
# 9 the cluster's h in hand, 10 down rows published, 11 residual updated and the next x pushed
CLUSTER_INTERVALS = [
    ("E1 wait (x*ln1 from the residual exchange)", 0, 1), ("A q|k|v GEMV + push + E2 wait", 1, 2),
    ("B q/k norm + RoPE (+ K/V append)", 2, 3), ("B attention over own positions", 3, 4),
    ("B partials push + E3 wait", 4, 5), ("B merge the cluster's partials", 5, 6), ("C o_proj rows + publish", 6, 7),
    ("G1 residual poll + E4 push + wait", 7, 8), ("D gate|up + SiLU + E5 push + wait", 8, 9),
    ("E down rows + publish", 9, 10), ("G2 residual poll + E1 push", 10, 11),
]
INTERVALS = [  # (name, from stamp, to stamp) of the grid kernel (decode_kernel.cuh)
    ("A input (gather x + rmsnorm)", 0, 1), ("A q|k|v GEMV + store", 1, 2),
    ("B wait q/k/v + norm/RoPE", 2, 3), ("B attention chunk", 3, 4), ("B merge / publish", 4, 5),
    ("C input (gather att)", 5, 6), ("C o GEMV + residual", 6, 7),
    ("D input (gather x + rmsnorm)", 7, 8), ("D gate|up GEMV + SiLU", 8, 9),
    ("E input (gather h)", 9, 10), ("E down GEMV + residual", 10, 11),
    ("B merge: poll partials (merging CTAs)", 4, 12), ("B merge: combine + publish", 12, 13),
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--geometry", default="qwen3-0.6b", choices=sorted(randmodel.GEOMETRIES))
    ap.add_argument("--pos", type=int, default=130)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    model = ci.CudaModel.load_model(randmodel.make_model(a.geometry, 0))
    L = model.config.num_hidden_layers
    cache = ci.CudaKVCache(model, a.pos + 2)
    ids = randmodel.prompt_ids(a.pos + 1, model.config.vocab_size, seed=1)
    for pos in range(a.pos):
        model.forward(ids[pos], pos, cache)
    model.set_trace(True)
    model.forward(ids[a.pos], a.pos, cache)
    tr = model.read_trace().astype(np.int64)
    model.set_trace(False)
    t0 = tr[:, 0].min()
    rel = tr - t0
    rows = []
    kind = model.decoder_kind
    for name, i, j in (CLUSTER_INTERVALS if kind == "cluster" else INTERVALS):
        vals = []
        for l in range(L):
            d = rel[:, l * TPL + j] - rel[:, l * TPL + i]
            ok = (tr[:, l * TPL + i] > 0) & (tr[:, l * TPL + j] > 0)
            if ok.any():
                vals.append(d[ok])
        v = np.concatenate(vals) if vals else np.zeros(1)
        rows.append({"interval": name, "median_us": float(np.median(v)) / 1e3, "max_us": float(v.max()) / 1e3})
    layer_span = [(rel[:, l * TPL + 11].max() - (rel[:, l * TPL + 0].min())) / 1e3 for l in range(L)]
    tail = L * TPL
    out = {
        "geometry": a.geometry, "pos": a.pos, "ctas": int(tr.shape[0]), "decoder": kind,
        "token_span_us": float(rel[:, tail + 3].max()) / 1e3,
        "layers_span_us": float(rel[:, (L - 1) * TPL + 11].max()) / 1e3,
        "layer_span_us_median": float(np.median(layer_span)),
        "lm_head_us": float(np.median(rel[:, tail + 1] - rel[:, tail + 0])) / 1e3,
        "lm_input_wait_us": float(np.median(rel[:, tail + 0] - rel[:, (L - 1) * TPL + 11])) / 1e3,
        "barrier_us": float(np.median(rel[:, tail + 2] - rel[:, tail + 1])) / 1e3,
        "intervals": rows,
    }
    if a.json:
        print(json.dumps(out))
        return
    print(f"{a.geometry} pos {a.pos} ({kind} decoder): token span {out['token_span_us']:.1f} us over {out['ctas']} CTAs; "
          f"layers {out['layers_span_us']:.1f} us (median layer {out['layer_span_us_median']:.2f} us); "
          f"lm_head {out['lm_head_us']:.1f} us; end barrier {out['barrier_us']:.2f} us")
    for r in rows:
        print(f"  {r['interval']:32s} median {r['median_us']:7.2f} us   max {r['max_us']:7.2f} us")


if __name__ == "__main__":
    main()
