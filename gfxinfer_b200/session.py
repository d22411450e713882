"""Engine and decode-session handles over the C ABI.

Mirrors the reference's public runtime API (include/gfxinfer/engine.h:77-97,
include/gfxinfer/qwen_runtime.h:47-77): Engine.create, QwenDecodeSession.create,
greedy_step, block_step, mtp_draft, speculative_step, position. Failures raise
GfxbError carrying the reference's ErrorCode value.
"""
from __future__ import annotations

import atexit
import ctypes
import weakref
from dataclasses import dataclass, field

from . import abi, check, lib

CONFIG2 = dict(hidden=5120, intermediate=17408, layers=64, attention_interval=4, gdn_key_heads=16,
               gdn_value_heads=48, q_heads=24, kv_heads=4, vocab=151936, draft_vocab=98304, mlp_bits=3,
               proj_bits=4, head_bits=4, emb_bits=4, activation_bits=4, max_context=512, seed=0x5EED)
"""BASELINE config 2: 64-layer hybrid decoder, W3 MLP, W4 projections/head, A4, context 512."""


def model_config(**overrides) -> abi.ModelConfig:
    values = dict(CONFIG2)
    values.update(overrides)
    return abi.ModelConfig(**values)


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib().gfxb_nccl_unique_id(buf))
    return buf.raw


def tp_shard(config: abi.ModelConfig, tp_rank: int, tp_size: int) -> abi.TpShardInfo:
    """This rank's slice of every tensor-parallel dimension (host-side; no GPU needed)."""
    out = abi.TpShardInfo()
    check(lib().gfxb_tp_shard(ctypes.byref(config), tp_rank, tp_size, ctypes.byref(out)))
    return out


class Engine:
    """Resident weights of one model (or one tensor-parallel shard) on one GPU."""

    def __init__(self, handle: int, config: abi.ModelConfig) -> None:
        self._handle = ctypes.c_void_p(handle)
        self.config = config
        # raw handles of the sessions still open on this engine: close() destroys them before the engine
        # even when their Python objects are unreachable (cyclic garbage finalises in any order)
        self._session_handles: set[int] = set()
        _LIVE.add(self)

    @classmethod
    def create(cls, config: abi.ModelConfig | None = None, device: int = 0, tp_rank: int = 0, tp_size: int = 1,
               nccl_id: bytes | None = None, include_mtp: bool = True) -> "Engine":
        config = config or model_config()
        handle = ctypes.c_void_p()
        check(lib().gfxb_engine_create_synthetic(ctypes.byref(config), device, tp_rank, tp_size, nccl_id,
                                                 int(include_mtp), ctypes.byref(handle)))
        return cls(handle.value, config)

    @classmethod
    def from_artifact(cls, path: str, device: int = 0, activation_bits: int = 4, max_context: int = 512,
                      draft_vocab: int = 0, include_mtp: bool = True, verify_checksums: bool = True,
                      tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None) -> "Engine":
        """Engine::create from a `.gfxi` artifact (engine.cpp:62-216); the shape comes from the tensors."""
        options = abi.ArtifactLoadOptions(activation_bits, max_context, draft_vocab, int(include_mtp),
                                          int(verify_checksums))
        handle = ctypes.c_void_p()
        check(lib().gfxb_engine_create_from_artifact(str(path).encode(), ctypes.byref(options), device, tp_rank,
                                                     tp_size, nccl_id, ctypes.byref(handle)))
        engine = cls(handle.value, abi.ModelConfig())
        check(lib().gfxb_engine_config(engine.handle, ctypes.byref(engine.config)))
        return engine

    def export_artifact(self, path: str, weights_id: str = "synthetic") -> None:
        """Write this (single-GPU) engine's weights as a "b200-v1" artifact."""
        check(lib().gfxb_engine_export_artifact(self._handle, str(path).encode(), weights_id.encode()))

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def abort(self) -> None:
        """Abort the NCCL communicator so a step blocked on a failed peer returns an error."""
        if self._handle:
            check(lib().gfxb_engine_abort(self._handle))

    def weight_bytes(self) -> int:
        out = ctypes.c_uint64()
        check(lib().gfxb_engine_weight_bytes(self._handle, ctypes.byref(out)))
        return out.value

    def _release_session(self, handle: int) -> bool:
        """True when the session handle is still open and the caller must destroy it."""
        if handle in self._session_handles:
            self._session_handles.discard(handle)
            return True
        return False

    def close(self) -> None:
        """Destroys the engine; sessions created from it are destroyed first."""
        for handle in list(self._session_handles):
            lib().gfxb_session_destroy(ctypes.c_void_p(handle))
        self._session_handles.clear()
        if self._handle:
            lib().gfxb_engine_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


@dataclass
class SpeculativeStepResult:
    tokens: list[int] = field(default_factory=list)
    proposed_drafts: int = 0
    accepted_drafts: int = 0


class QwenDecodeSession:
    """Batch-1 decode session (qwen_runtime.h:47-77)."""

    def __init__(self, handle: int, engine: Engine) -> None:
        self._handle = ctypes.c_void_p(handle)
        self.engine = engine
        engine._session_handles.add(handle)

    @classmethod
    def create(cls, engine: Engine, maximum_context_tokens: int | None = None, graph_verifier_batch: int = 0,
               use_graphs: bool = True, step_kernel: int = abi.STEP_AUTO) -> "QwenDecodeSession":
        """step_kernel: abi.STEP_AUTO (the faster path on B200: per-operation kernels today),
        abi.STEP_LAUNCHES (per-operation kernels) or abi.STEP_PERSISTENT (token kernel or
        GFXB_UNSUPPORTED)."""
        ctx = maximum_context_tokens or engine.config.max_context
        config = abi.SessionConfig(ctx, graph_verifier_batch, int(use_graphs), step_kernel)
        handle = ctypes.c_void_p()
        check(lib().gfxb_session_create(engine.handle, ctypes.byref(config), ctypes.byref(handle)))
        return cls(handle.value, engine)

    def greedy_step(self, token: int) -> int:
        out = ctypes.c_uint32()
        check(lib().gfxb_session_greedy_step(self._handle, token, ctypes.byref(out)))
        return out.value

    def block_step(self, tokens: list[int]) -> list[int]:
        n = len(tokens)
        arr = (ctypes.c_uint32 * max(n, 1))(*tokens)
        out = (ctypes.c_uint32 * max(n, 1))()
        check(lib().gfxb_session_block_step(self._handle, arr, n, out))
        return list(out)[:n]

    def mtp_draft(self, next_token: int) -> int:
        out = ctypes.c_uint32()
        check(lib().gfxb_session_mtp_draft(self._handle, next_token, ctypes.byref(out)))
        return out.value

    def speculative_step(self, seed_token: int, draft_count: int,
                         drafts: list[int] | None = None) -> SpeculativeStepResult:
        """One MTP speculative round; with `drafts`, the round verifies those tokens instead of the
        MTP proposals (gfxb_session_speculative_step_with_drafts)."""
        out = (ctypes.c_uint32 * 32)()
        count = ctypes.c_uint()
        accepted = ctypes.c_uint()
        if drafts is None:
            check(lib().gfxb_session_speculative_step(self._handle, seed_token, draft_count, out, ctypes.byref(count),
                                                      ctypes.byref(accepted)))
        else:
            draft_count = len(drafts)
            arr = (ctypes.c_uint32 * max(draft_count, 1))(*drafts)
            check(lib().gfxb_session_speculative_step_with_drafts(self._handle, seed_token, arr, draft_count, out,
                                                                  ctypes.byref(count), ctypes.byref(accepted)))
        return SpeculativeStepResult(list(out)[:count.value], draft_count, accepted.value)

    def prefill(self, tokens: list[int]) -> int:
        """Chunked prefill of a prompt (32-token causal blocks, LM head on the last token only);
        returns the argmax after the prompt's last token."""
        n = len(tokens)
        arr = (ctypes.c_uint32 * max(n, 1))(*tokens)
        out = ctypes.c_uint32()
        check(lib().gfxb_session_prefill(self._handle, arr, n, ctypes.byref(out)))
        return out.value

    def position(self) -> int:
        out = ctypes.c_uint64()
        check(lib().gfxb_session_position(self._handle, ctypes.byref(out)))
        return out.value

    def enqueue_greedy(self, first_token: int, steps: int) -> None:
        check(lib().gfxb_session_enqueue_greedy(self._handle, first_token, steps))

    def sync(self) -> None:
        check(lib().gfxb_session_sync(self._handle))

    def last_token(self) -> int:
        out = ctypes.c_uint32()
        check(lib().gfxb_session_last_token(self._handle, ctypes.byref(out)))
        return out.value

    def stream(self) -> int:
        return lib().gfxb_session_stream(self._handle) or 0

    def enqueue_gemv(self, kind: int, launches: int) -> int:
        """Enqueue standalone GEMV launches (0 MLP gate+up, 1 MLP down, 2 GDN in); returns bytes per launch."""
        out = ctypes.c_uint64()
        check(lib().gfxb_session_enqueue_gemv(self._handle, kind, launches, ctypes.byref(out)))
        return out.value

    def enqueue_operation(self, kind: int, launches: int) -> int:
        """Enqueue standalone launches of one decode operation (gfxb.h GFXB_OP_*); returns bytes per launch."""
        out = ctypes.c_uint64()
        check(lib().gfxb_session_enqueue_operation(self._handle, kind, launches, ctypes.byref(out)))
        return out.value

    def time_operation(self, kind: int, launches: int, graph: bool = True) -> tuple[float, int]:
        """(microseconds per launch, bytes per launch) of one decode operation timed in isolation."""
        us, out = ctypes.c_float(), ctypes.c_uint64()
        check(lib().gfxb_session_time_operation(self._handle, kind, launches, int(graph), ctypes.byref(us),
                                                ctypes.byref(out)))
        return us.value, out.value

    def read_state(self, logits_count: int = 0):
        import numpy as np

        hidden = np.zeros(self.engine.config.hidden, np.uint16)
        logits = np.zeros(max(logits_count, 1), np.float32)
        check(lib().gfxb_session_read_state(self._handle, hidden.ctypes.data,
                                            logits.ctypes.data if logits_count else None, logits_count))
        return hidden, logits[:logits_count]

    def trace_step(self, token: int):
        """One greedy step on the persistent token kernel with its timeline recorded.

        Returns (next_token, timeline, op_kinds): timeline is int64 nanoseconds
        [op_count + 1][2][ctas] (barrier arrival, barrier release per operation
        and CTA; see gfxb_session_trace_step), op_kinds the operation codes."""
        import numpy as np

        ops, ctas = ctypes.c_uint(), ctypes.c_uint()
        out = ctypes.c_uint32()
        probe = lib().gfxb_session_trace_step(self._handle, token, ctypes.byref(out), None, 0, ctypes.byref(ops),
                                              ctypes.byref(ctas), None)
        if probe not in (0, 1):  # 1: the probe's missing buffer; anything else is a real failure
            check(probe)
        timeline = np.zeros((ops.value + 1, 2, ctas.value), np.uint64)
        kinds = np.zeros(ops.value, np.uint32)
        check(lib().gfxb_session_trace_step(self._handle, token, ctypes.byref(out), timeline.ctypes.data,
                                            timeline.size, ctypes.byref(ops), ctypes.byref(ctas),
                                            kinds.ctypes.data))
        return out.value, timeline.astype(np.int64), kinds

    def close(self) -> None:
        if self._handle:
            if self.engine._release_session(self._handle.value):
                lib().gfxb_session_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


_LIVE: weakref.WeakSet = weakref.WeakSet()


@atexit.register
def _close_all() -> None:
    # Release device objects before the CUDA runtime is torn down at exit.
    for engine in list(_LIVE):
        engine.close()


def read_device_errors() -> int:
    flags = ctypes.c_uint32()
    check(lib().gfxb_read_device_errors(ctypes.byref(flags)))
    return flags.value
