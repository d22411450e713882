"""Time each decode operation of the config-2 model in isolation on B200.

    python -m gfxinfer_b200.bench_ops [--layers 64] [--position 256] [--launches 96] [--ops gdn_step,attention]

One engine with config-2 widths (hidden 5120, MLP 17408 W3, GDN/attention W4, A4) and a session filled to
`position` by chunked prefill; every operation is launched `launches` times (gfxb_session_time_operation),
cycling over the layers that carry it so each launch reads its weights or states from HBM, replayed from a
CUDA graph and timed with CUDA events on the session stream. Prints one JSON line per operation: mean
launch time, algorithmic bytes per launch, GB/s and the fraction of the measured HBM copy bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from . import session as gs

OPS = {"mlp_gate_up": 0, "mlp_down": 1, "gdn_in": 2, "gdn_out": 3, "attn_qkv": 4, "attn_o": 5, "lm_head": 6,
       "gdn_step": 7, "attention": 8, "norm_pack": 9, "silu_pack": 10}


def measured_peak() -> tuple[float, str]:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def run(layers: int, position: int, launches: int, names: list[str], graph: bool = True, **overrides) -> list[dict]:
    cfg = dict(gs.CONFIG2, layers=layers, **overrides)
    cfg["max_context"] = max(cfg["max_context"], -(-(position + 1) // 128) * 128)
    engine = gs.Engine.create(gs.model_config(**cfg), include_mtp=False)
    session = gs.QwenDecodeSession.create(engine, use_graphs=False)
    rng = np.random.default_rng(cfg["seed"])
    if position > 0:
        session.prefill([int(t) for t in rng.integers(0, cfg["vocab"], size=position)])
    peak, source = measured_peak()
    out = []
    for name in names:
        us, per_launch = session.time_operation(OPS[name], launches, graph)
        gbps = per_launch / (us * 1e-6) / 1e9
        out.append({"op": name, "us": round(us, 3), "bytes": per_launch, "GBps": round(gbps, 1),
                    "frac": round(gbps / peak, 4), "peak": peak, "peak_source": source, "position": position,
                    "layers": layers, "graph": graph})
    session.close()
    engine.close()
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--layers", type=int, default=64)
    parser.add_argument("--position", type=int, default=256)
    parser.add_argument("--launches", type=int, default=96)
    parser.add_argument("--ops", default=",".join(OPS))
    parser.add_argument("--no-graph", action="store_true")
    args = parser.parse_args()
    for line in run(args.layers, args.position, args.launches, args.ops.split(","), graph=not args.no_graph):
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
