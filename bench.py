"""Benchmark: batch-1 W3A4 decode tokens/s of the 64-layer config-2 model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one greedy decode token (64 layers + LM head + argmax) of the
BASELINE config-2 model (hidden 5120, MLP 17408 W3, GDN/attention W4, W4 LM
head over vocab 151936, A4 activations, context 512) with seeded random-init
weights and a 64-token uniform-random prompt. N > 1 runs tensor parallelism
over N GPUs (one process per GPU under torchrun, NCCL all-reduce), so the
total work per token is fixed: "scaling": "strong".

value: K greedy steps replayed back to back from device memory (each step's
argmax feeds the next), CUDA events on the session stream, max over ranks.
e2e:   K steps through the public greedy_step call: pinned host token in,
       host token out, synchronised every step.
The weights (11.2 GB) exceed L2 (126 MB), so no flush is needed.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 W3A4 decode tokens/s"
UNIT = "tokens/s"


def _config_dict():
    from gfxinfer_b200.session import CONFIG2

    return dict(CONFIG2)


def _kernels_per_step(cfg: dict, tp: int) -> int:
    layers = cfg["layers"]
    attention = layers // cfg["attention_interval"]
    gdn = layers - attention
    # see gfxinfer_b200/csrc/host/runtime.cu enqueue_forward: a GDN layer is in-projection GEMV, recurrent step
    # (causal conv inside), out-projection, norm, gate/up, SiLU pack, down, norm; an attention layer has q/k/v,
    # the single-token attention (Q/K norm + RoPE, KV append, chunks and merge in one launch), o_proj, then
    # the same five
    per_gdn, per_attention = 8, 8
    head = 1 + 2 + (2 if tp > 1 else 0)  # LM-head GEMV, argmax (2), TP exchange/select
    return 1 + gdn * per_gdn + attention * per_attention + head + 1  # embed+norm ... advance


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


class _PeerWatchdog:
    """Aborts the engine's NCCL communicator when another rank reports a failure through the
    torch.distributed store, so this rank's pending collectives end with an error instead of
    waiting for a peer that is gone."""

    def __init__(self, engine) -> None:
        import torch.distributed as dist

        self.engine = engine
        self.store = dist.distributed_c10d._get_default_store()
        self.done = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self) -> None:
        while not self.done.wait(1.0):
            try:
                if self.store.add("gfxb_failures", 0) > 0:
                    self.engine.abort()
                    return
            except Exception:
                return

    def stop(self) -> None:
        self.done.set()

    @staticmethod
    def report_failure() -> None:
        try:
            import torch.distributed as dist

            dist.distributed_c10d._get_default_store().add("gfxb_failures", 1)
        except Exception:
            pass


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class CpuSample:
    """The reference path's CPU implementation on this host: the oracle's C forward (OpenMP over all host
    cores, AVX2 integer group dots), the reference having no CPU forward of its own. Every token runs all 64
    config-2 layers (48 GDN + 16 attention, each with its own recurrent state and KV cache) and the full LM
    head; the weights of 4 layers (the repeating 3 GDN + 1 attention unit) are reused 16 times so that the
    model fits host memory. Each step is one whole greedy token, timed by the host clock."""

    def __init__(self) -> None:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from oracle_lib import Oracle, OracleModel, model_config

        self.oracle = Oracle()
        self.cores = int(self.oracle.lib.or_set_threads(os.cpu_count() or 1))
        cfg = model_config(max_context=512)
        start = time.perf_counter()
        self.model = OracleModel(self.oracle, cfg, include_mtp=False, resident_layers=4)
        self.build_seconds = time.perf_counter() - start
        self.token = 1

    def step(self) -> float:
        """One full greedy token (64 layers + LM head + argmax); returns its seconds."""
        start = time.perf_counter()
        self.token = self.model.greedy_step(self.token)
        return time.perf_counter() - start

    def describe(self, tokens: int) -> str:
        return (f"{tokens} greedy tokens, each through all 64 config-2 layers (weights of 4 layers reused 16x) "
                f"and the full LM head (vocab 151936), C forward with AVX2 integer dots on {self.cores} threads, "
                f"host clock per token")


def cpu_baseline(tokens: int = 5) -> dict:
    sample = CpuSample()
    sample.step()  # first-touch warm-up
    seconds = [sample.step() for _ in range(tokens)]
    value = 1.0 / statistics.mean(seconds)
    return {"value": round(value, 4), "unit": UNIT, "cores": sample.cores, "kind": "port",
            "sample": sample.describe(tokens)}


def run_reference(args) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    sample = CpuSample()
    seconds = []
    for i in range(args.warmup + args.steps):
        t = sample.step()
        if i >= args.warmup:
            seconds.append(t)
    per_token = statistics.mean(seconds)
    tokens_per_s = 1.0 / per_token
    line = {"impl": "reference", "metric": METRIC, "value": round(tokens_per_s, 4), "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 * per_token, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "config-2 decode: 64-layer hybrid (48 GDN + 16 gated GQA), hidden 5120, "
                                   "MLP 17408 W3, GDN/attention W4, W4 LM head vocab 151936, A4, batch 1, ctx 512",
                       "global_batch": 1, "seq_len": 512, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(tokens_per_s, 4), "unit": UNIT, "cores": sample.cores, "kind": "port",
                             "sample": sample.describe(args.steps)},
            "e2e": {"value": round(tokens_per_s, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "timed_seconds": round(sum(seconds), 3), "model_build_seconds": round(sample.build_seconds, 3)}
    print(json.dumps(line), flush=True)


def measure_verifier(gs, np, torch, local: int, widths=(5, 32), blocks: int = 6) -> dict:
    """The causal verifier alone (the reference's block-bench: `QwenDecodeSession::block_step`, evaluated tokens
    per second) on the config-2 model: after a 64-token prefill, `blocks` timed blocks of each width (one warm-up
    block first), device-timed with CUDA events on the session stream."""
    cfg = dict(gs.CONFIG2, max_context=512)
    engine = gs.Engine.create(gs.model_config(**cfg), device=local, include_mtp=False)
    rng = np.random.default_rng(cfg["seed"] + 5)
    out = {"workload": "config-2 causal verifier blocks after a 64-token prompt, evaluated tokens/s", "widths": {}}
    for width in widths:
        session = gs.QwenDecodeSession.create(engine, maximum_context_tokens=512)
        stream = torch.cuda.ExternalStream(session.stream(), device=torch.device("cuda", local))
        session.prefill([int(t) for t in rng.integers(0, cfg["vocab"], size=64)])
        tokens = [[int(t) for t in rng.integers(0, cfg["vocab"], size=width)] for _ in range(blocks + 1)]
        session.block_step(tokens[0])
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for block in tokens[1:]:
            session.block_step(block)
        stop.record(stream)
        stop.synchronize()
        ms = start.elapsed_time(stop)
        out["widths"][str(width)] = {"evaluated_tokens_per_s": round(width * blocks / (ms / 1000.0), 3),
                                     "ms_per_block": round(ms / blocks, 3)}
        session.close()
    engine.close()
    return out


def measure_mtp(gs, np, torch, local: int, depths=(4, 8), emitted_target: int = 256) -> dict:
    """the config-2 model plus one MTP layer, context 2048; speculative rounds
    (MTP draft chain + causal verifier, one captured CUDA graph per depth) until 256 tokens are
    emitted after a 64-token prompt. Emitted tokens/s over the device-timed loop (the host accept
    step included) and the draft acceptance rate. Random-init weights: acceptance is low."""
    cfg = dict(gs.CONFIG2, max_context=2048)
    engine = gs.Engine.create(gs.model_config(**cfg), device=local, include_mtp=True)
    rng = np.random.default_rng(cfg["seed"] + 3)
    prompt = [int(t) for t in rng.integers(0, cfg["vocab"], size=64)]
    out = {"workload": "config-3: config-2 model + 1 MTP layer (draft head = first 98304 LM-head rows), "
                       "ctx 2048, 64-token prompt, 256 emitted tokens per depth", "depths": {}}
    for depth in depths:
        session = gs.QwenDecodeSession.create(engine, maximum_context_tokens=2048, graph_verifier_batch=depth + 1)
        stream = torch.cuda.ExternalStream(session.stream(), device=torch.device("cuda", local))
        token = None
        for t in prompt:
            token = session.greedy_step(t)
            session.mtp_draft(token)  # keep the MTP cache aligned with the target (spec-bench warm-up)
        seed = session.greedy_step(token)
        for _ in range(2):  # warm-up rounds
            seed = session.speculative_step(seed, depth).tokens[-1]
        emitted = proposed = accepted = rounds = 0
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        while emitted < emitted_target:
            result = session.speculative_step(seed, depth)
            emitted += len(result.tokens)
            proposed += result.proposed_drafts
            accepted += result.accepted_drafts
            rounds += 1
            seed = result.tokens[-1]
        stop.record(stream)
        stop.synchronize()
        ms = start.elapsed_time(stop)
        out["depths"][str(depth)] = {"emitted_tokens_per_s": round(emitted / (ms / 1000.0), 3),
                                     "emitted_tokens": emitted, "rounds": rounds,
                                     "acceptance": round(accepted / max(proposed, 1), 4),
                                     "ms_per_round": round(ms / rounds, 3)}
        session.close()
    engine.close()
    return out


def measure_config4(gs, np, torch, world: int, rank: int, local: int, nccl_id, steps: int, barrier) -> dict:
    """the config-2 model with W2 MLP, W4 attention/GDN/head, A8 activations and
    a 4096-token context, tensor-parallel over the job's GPUs. The session is filled to position
    3968 with 32-token verifier blocks, then `steps` greedy steps run device-resident; plus the
    per-GPU W2 MLP gate+up GEMV bandwidth."""
    cfg = dict(gs.CONFIG2, mlp_bits=2, activation_bits=8, max_context=4096)
    engine = gs.Engine.create(gs.model_config(**cfg), device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id,
                              include_mtp=False)
    session = gs.QwenDecodeSession.create(engine, maximum_context_tokens=4096)
    stream = torch.cuda.ExternalStream(session.stream(), device=torch.device("cuda", local))
    rng = np.random.default_rng(cfg["seed"] + 4)
    fill = 4096 - 128
    tokens = [int(t) for t in rng.integers(0, cfg["vocab"], size=fill)]
    token = None
    for i in range(0, fill, 32):
        token = session.block_step(tokens[i:i + 32])[-1]
    for _ in range(3):
        token = session.greedy_step(token)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record(stream)
    session.enqueue_greedy(token, steps)
    stop.record(stream)
    stop.synchronize()
    barrier()
    decode_ms = start.elapsed_time(stop)
    launches = 48
    session.enqueue_gemv(0, 8)
    torch.cuda.synchronize()
    start.record(stream)
    gemv_bytes = session.enqueue_gemv(0, launches)
    stop.record(stream)
    stop.synchronize()
    gemv_us = start.elapsed_time(stop) * 1000.0 / launches
    times = torch.tensor([decode_ms, gemv_us], dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    decode_ms, gemv_us = times.tolist()
    weight_bytes = engine.weight_bytes()
    session.close()
    engine.close()
    return {"workload": "config-4: config-2 model, W2 MLP / W4 attention+GDN+head, A8, ctx 4096 "
                        f"(decode at positions {fill + 3}..{fill + 3 + steps}), tp{world}",
            "tokens_per_s": round(steps / (decode_ms / 1000.0), 3), "ms_per_token": round(decode_ms / steps, 4),
            "weight_bytes_per_gpu": weight_bytes,
            "per_gpu_GBps": round(weight_bytes / (decode_ms / steps / 1000.0) / 1e9, 1),
            "mlp_gate_up_gemv_GBps_per_gpu": round(gemv_bytes / (gemv_us * 1e-6) / 1e9, 1),
            "mlp_gate_up_gemv_us": round(gemv_us, 3)}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one W3A4 MLP gate+up launch, from the ncu
# capture summarised in profiles/gemv_pipe_w3_gate_up_config2_ncu.md.
GATE_UP_DRAM_BYTES = 69711872


def measure_config0(peak: float) -> dict:
    """BASELINE config 0 on the device: the W3A4 [17408 x 5120] GEMV at batch 1 and 5 (bench-gemv's
    workload: six weight copies rotated so every launch reads HBM, launches replayed from a CUDA
    graph, CUDA events), against the north star's >= 60 % of HBM roofline."""
    from gfxinfer_b200 import bench_gemv

    out = {"workload": "config-0 W3A4 GEMV [17408x5120], fp16 group scales, A4 activations, fp32 out",
           "peak_GBps": peak}
    for batch in (1, 5):
        r = bench_gemv.run("w3", 17408, 5120, batch, "a4", 60, 6, True)
        out[f"b{batch}"] = {"us": r["mean_launch_us"], "GBps": r["algorithmic_GBps"],
                            "packed_code_GBps": r["packed_GBps"], "algorithmic_bytes": r["algorithmic_bytes"],
                            "frac": round(r["algorithmic_GBps"] / peak, 4)}
    return out


def run_b200(args) -> None:
    import numpy as np
    import torch

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        # gloo carries only host-side plumbing (NCCL id, barriers, timing max); the data path is the
        # engine's own NCCL communicator.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    from gfxinfer_b200 import build

    if rank == 0 and not os.path.exists(os.path.join(ROOT, "gfxinfer_b200", "libgfxb200.so")):
        build.build()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    from gfxinfer_b200 import session as gs

    cfg = _config_dict()
    nccl_id = None
    if world > 1:
        import torch.distributed as dist

        holder = [gs.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(holder, src=0)
        nccl_id = holder[0]
    engine = gs.Engine.create(gs.model_config(**cfg), device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id,
                              include_mtp=False)
    watchdog = _PeerWatchdog(engine) if world > 1 else None
    session = gs.QwenDecodeSession.create(engine, maximum_context_tokens=cfg["max_context"])
    stream = torch.cuda.ExternalStream(session.stream(), device=torch.device("cuda", local))
    rng = np.random.default_rng(cfg["seed"])
    prompt = [int(t) for t in rng.integers(0, cfg["vocab"], size=64)]

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    token = None
    for t in prompt:  # serial prefill through the public step, as the reference does
        token = session.greedy_step(t)
    for _ in range(args.warmup):
        token = session.greedy_step(token)

    # --- value: device-resident greedy loop -----------------------------------
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        session.enqueue_greedy(token, args.steps)
        stop.record(stream)
        stop.synchronize()
    barrier()
    device_ms = start.elapsed_time(stop)
    token = session.last_token()

    # --- e2e: public greedy_step with host buffers ------------------------------
    for _ in range(args.warmup):
        token = session.greedy_step(token)
    barrier()
    start.record(stream)
    for _ in range(args.steps):
        token = session.greedy_step(token)
    stop.record(stream)
    stop.synchronize()
    barrier()
    e2e_ms = start.elapsed_time(stop)

    # --- dominant kernel: W3 MLP gate+up GEMV in isolation -------------------------
    launches = 96
    gemv_start, gemv_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    session.enqueue_gemv(0, 8)
    torch.cuda.synchronize()
    gemv_start.record(stream)
    gemv_bytes = session.enqueue_gemv(0, launches)
    gemv_stop.record(stream)
    gemv_stop.synchronize()
    gemv_us = gemv_start.elapsed_time(gemv_stop) * 1000.0 / launches

    times = torch.tensor([device_ms, e2e_ms, gemv_us], dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    device_ms, e2e_ms, gemv_us = times.tolist()
    if rank == 0:
        peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        peak, peak_note = 6650.0, "fallback"
        if os.path.exists(peaks_path):
            with open(peaks_path) as f:
                peak = float(json.load(f)["hbm_gbs"])
            peak_note = "measured"
        achieved = gemv_bytes / (gemv_us * 1e-6) / 1e9
        per_step_bytes = engine.weight_bytes()
        line = {
            "metric": METRIC, "value": round(args.steps / (device_ms / 1000.0), 3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(device_ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded random-init weights, random prompt)",
            "config": {"workload": "config-2 decode: 64-layer hybrid (48 GDN + 16 gated GQA), hidden 5120, "
                                   "MLP 17408 W3, GDN/attention W4, W4 LM head vocab 151936, A4, batch 1, ctx 512",
                       "global_batch": 1, "seq_len": cfg["max_context"], "parallelism": f"tp{world}",
                       "prompt_tokens": 64, "l2": "weights 11.2 GB per token >> 126 MB L2; no flush needed"},
            "e2e": {"value": round(args.steps / (e2e_ms / 1000.0), 3), "unit": UNIT,
                    "h2d_bytes_per_step": 4 + 8, "d2h_bytes_per_step": 4},
            "gpu_launches": _kernels_per_step(cfg, world) * args.steps,
            "roofline": {"bound": "hbm", "kernel": "W3A4 MLP gate+up GEMV [2x17408x5120] (one launch)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_note,
                         "traffic": GATE_UP_DRAM_BYTES,
                         "algorithmic_bytes_per_launch": gemv_bytes, "launch_us": round(gemv_us, 3)},
            "decode_roofline": {"weight_bytes_per_token_per_gpu": per_step_bytes,
                                "achieved_GBps_per_gpu": round(per_step_bytes / (device_ms / args.steps / 1000.0) / 1e9, 1),
                                "frac": round(per_step_bytes / (device_ms / args.steps / 1000.0) / 1e9 / peak, 4)},
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(5)
    if watchdog is not None:
        watchdog.stop()
    session.close()
    engine.close()
    extras = {}
    if not args.no_extra:
        config4_id = None
        if world > 1:
            import torch.distributed as dist

            holder = [gs.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(holder, src=0)
            config4_id = holder[0]
        extras["config4"] = measure_config4(gs, np, torch, world, rank, local, config4_id, min(args.steps, 96), barrier)
        if world == 1:
            extras["mtp"] = measure_mtp(gs, np, torch, local)
            extras["verifier"] = measure_verifier(gs, np, torch, local)
            extras["config0"] = measure_config0(line["roofline"]["peak"])
    if rank == 0:
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=128)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-extra", action="store_true", help="skip the config-3 (MTP) and config-4 (TP W2/A8) lines")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    if 64 + 2 * (args.warmup + args.steps) > 512:
        parser.error("prompt + warm-up + timed steps exceed the 512-token context")
    if args.impl == "reference":
        run_reference(args)
        return
    try:
        run_b200(args)
    except BaseException:
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            _PeerWatchdog.report_failure()
        raise


if __name__ == "__main__":
    main()
