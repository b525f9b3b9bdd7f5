"""Greedy top-1 generation: the host-side state machine that drives decode steps.

Restates the reference's deterministic generation contract
(crates/pvlc-cpu-ref/src/lib.rs:2046-2420):

* ``TopKEntry`` ordering (``compare_top_k_entries`` :2051-2056): larger value
  first under IEEE total order (so -0.0 sorts after +0.0), ties broken by the
  smaller vocabulary index;
* ``GreedyGenerationState`` (:2201-2279): the prefill's top-1 is the first
  generated token; generation stops on the EOS token (which is kept) or when
  ``max_new_tokens`` tokens exist; each decode step must return well-formed
  candidates and caches one token longer than before;
* ``greedy_generate`` (:2282-2305) and ``greedy_generate_chunked``
  (:2309-2366): the callback and chunked drivers, with every malformed input
  rejected before the next callback.

Caches are opaque to the state machine: any object with ``tokens``,
``key_value_heads`` and ``head_dim`` attributes.  When it also carries
``keys`` / ``values`` sequences their lengths are checked as the reference's
``validate_kv_geometry`` does (:756-780).  The GPU engine passes light
descriptors of its device-resident caches.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

# CpuRefErrorCode (crates/pvlc-cpu-ref/src/lib.rs:16-30), numbered from 1 as the
# CPU oracle and the C ABI number them (0 = ok).
DIMENSION_MISMATCH = 1
INVALID_K = 6
NON_FINITE_INPUT = 7
INVALID_TILE_SIZE = 12

_CODE_NAMES = {DIMENSION_MISMATCH: "DimensionMismatch", INVALID_K: "InvalidK",
               NON_FINITE_INPUT: "NonFiniteInput", INVALID_TILE_SIZE: "InvalidTileSize"}

PINNED_DECODER_LAYERS = 18
PINNED_DECODER_VOCAB_SIZE = 103_424
PINNED_DECODER_KEY_VALUE_HEADS = 2
PINNED_DECODER_HEAD_DIM = 128
PINNED_DECODER_EOS_TOKEN_ID = 2


class GreedyError(ValueError):
    """A rejected generation input; ``code`` is the reference's CpuRefErrorCode number."""

    def __init__(self, code: int, message: str = ""):
        super().__init__(f"{_CODE_NAMES.get(code, code)}: {message}" if message else
                         _CODE_NAMES.get(code, str(code)))
        self.code = code


class CallbackError(RuntimeError):
    """Raised by a decode callback to stop generation; propagated unchanged."""


def _f32(value: float) -> float:
    return struct.unpack("<f", struct.pack("<f", value))[0]


def _total_order_key(value: float) -> int:
    """Rust ``f32::total_cmp`` as an integer key: flip the magnitude bits of negatives."""
    bits = struct.unpack("<i", struct.pack("<f", value))[0]
    return bits ^ ((bits >> 31) & 0x7FFFFFFF)


@dataclass(frozen=True)
class TopKEntry:
    index: int
    value: float

    def sort_key(self):
        # compare_top_k_entries: right.value.total_cmp(left.value), then index ascending
        return (-_total_order_key(self.value), self.index)


def compare_top_k_entries(left: TopKEntry, right: TopKEntry) -> int:
    a, b = left.sort_key(), right.sort_key()
    return (a > b) - (a < b)


def top_k(values: Sequence[float], k: int) -> List[TopKEntry]:
    """crates/pvlc-cpu-ref/src/lib.rs:2065-2080."""
    if k > len(values):
        raise GreedyError(INVALID_K, "top-k exceeds the number of logits")
    if not all(math.isfinite(v) for v in values):
        raise GreedyError(NON_FINITE_INPUT)
    entries = sorted((TopKEntry(i, _f32(float(v))) for i, v in enumerate(values)),
                     key=TopKEntry.sort_key)
    return entries[:k]


@dataclass(frozen=True)
class GreedyGenerationConfig:
    layers: int
    vocab_size: int
    key_value_heads: int
    head_dim: int
    max_new_tokens: int
    eos_token_id: int


def pinned_greedy_generation_config(max_new_tokens: int) -> GreedyGenerationConfig:
    """crates/pvlc-cpu-ref/src/lib.rs:2369-2378: PaddleOCR-VL-1.6 decoder topology."""
    return GreedyGenerationConfig(PINNED_DECODER_LAYERS, PINNED_DECODER_VOCAB_SIZE,
                                  PINNED_DECODER_KEY_VALUE_HEADS, PINNED_DECODER_HEAD_DIM,
                                  max_new_tokens, PINNED_DECODER_EOS_TOKEN_ID)


@dataclass
class GreedyDecodeStep:
    top_k: List[TopKEntry]
    kv_caches: list


@dataclass
class GreedyGenerationTrace:
    generated_tokens: List[int]
    kv_caches: list
    decode_steps: int
    stop_reason: str            # "max_new_tokens" | "eos_token"


@dataclass
class GreedyChunkedGenerationTrace:
    generation: GreedyGenerationTrace
    decode_chunks: int


MAX_NEW_TOKENS = "max_new_tokens"
EOS_TOKEN = "eos_token"


def _validate_config(config: GreedyGenerationConfig) -> None:
    # crates/pvlc-cpu-ref/src/lib.rs:2128-2139
    if (config.layers == 0 or config.vocab_size == 0 or config.key_value_heads == 0
            or config.head_dim == 0 or config.max_new_tokens == 0
            or config.eos_token_id >= config.vocab_size):
        raise GreedyError(DIMENSION_MISMATCH, "generation config")


def _validate_candidates(candidates: Sequence[TopKEntry], vocab_size: int) -> None:
    # crates/pvlc-cpu-ref/src/lib.rs:2141-2168
    if not candidates or len(candidates) > vocab_size:
        raise GreedyError(DIMENSION_MISMATCH, "candidate count")
    for c in candidates:
        if not math.isfinite(c.value):
            raise GreedyError(NON_FINITE_INPUT, "candidate value")
    seen = set()
    for c in candidates:
        if c.index < 0 or c.index >= vocab_size or c.index in seen:
            raise GreedyError(DIMENSION_MISMATCH, "candidate index")
        seen.add(c.index)
    for a, b in zip(candidates, candidates[1:]):
        if compare_top_k_entries(a, b) >= 0:
            raise GreedyError(DIMENSION_MISMATCH, "candidates out of order")


def _validate_caches(caches, config: GreedyGenerationConfig,
                     expected_tokens: Optional[int]) -> int:
    # crates/pvlc-cpu-ref/src/lib.rs:2170-2198 with validate_kv_geometry :756-780
    if len(caches) != config.layers:
        raise GreedyError(DIMENSION_MISMATCH, "layer count")
    tokens = caches[0].tokens
    if tokens == 0 or (expected_tokens is not None and tokens != expected_tokens):
        raise GreedyError(DIMENSION_MISMATCH, "cache tokens")
    for c in caches:
        if (c.tokens != tokens or c.key_value_heads != config.key_value_heads
                or c.head_dim != config.head_dim):
            raise GreedyError(DIMENSION_MISMATCH, "cache geometry")
        keys = getattr(c, "keys", None)
        values = getattr(c, "values", None)
        if keys is not None or values is not None:
            n = tokens * config.key_value_heads * config.head_dim
            if keys is None or values is None or len(keys) != n or len(values) != n:
                raise GreedyError(DIMENSION_MISMATCH, "cache length")
            if not (all(math.isfinite(v) for v in keys) and all(math.isfinite(v) for v in values)):
                raise GreedyError(NON_FINITE_INPUT, "cache values")
    return tokens


@dataclass
class GreedyGenerationState:
    """One request's generation state (crates/pvlc-cpu-ref/src/lib.rs:2201-2279)."""

    config: GreedyGenerationConfig
    generated_tokens: List[int] = field(default_factory=list)
    current_token: int = 0
    current_caches: list = field(default_factory=list)
    cache_tokens: int = 0
    decode_steps: int = 0

    @classmethod
    def initialize(cls, prefill_top_k, initial_kv_caches, config):
        _validate_config(config)
        _validate_candidates(prefill_top_k, config.vocab_size)
        cache_tokens = _validate_caches(initial_kv_caches, config, None)
        token = prefill_top_k[0].index
        return cls(config, [token], token, initial_kv_caches, cache_tokens, 0)

    def terminal_reason(self) -> Optional[str]:
        if self.current_token == self.config.eos_token_id:
            return EOS_TOKEN
        if len(self.generated_tokens) == self.config.max_new_tokens:
            return MAX_NEW_TOKENS
        return None

    def remaining_decode_steps(self) -> int:
        remaining = self.config.max_new_tokens - len(self.generated_tokens)
        if remaining < 0:
            raise GreedyError(DIMENSION_MISMATCH, "generation overran its budget")
        return remaining

    def apply_decode_step(self, decoded: GreedyDecodeStep) -> Optional[str]:
        _validate_candidates(decoded.top_k, self.config.vocab_size)
        _validate_caches(decoded.kv_caches, self.config, self.cache_tokens + 1)
        self.current_token = decoded.top_k[0].index
        self.current_caches = decoded.kv_caches
        self.cache_tokens += 1
        self.generated_tokens.append(self.current_token)
        self.decode_steps += 1
        return self.terminal_reason()

    def into_trace(self, stop_reason: str) -> GreedyGenerationTrace:
        return GreedyGenerationTrace(self.generated_tokens, self.current_caches,
                                     self.decode_steps, stop_reason)


DecodeStepFn = Callable[[int, int, list], GreedyDecodeStep]


def greedy_generate(prefill_top_k, initial_kv_caches, config: GreedyGenerationConfig,
                    decode_step: DecodeStepFn) -> GreedyGenerationTrace:
    """crates/pvlc-cpu-ref/src/lib.rs:2282-2305: decode_step(step_index, input_token, caches)."""
    state = GreedyGenerationState.initialize(prefill_top_k, initial_kv_caches, config)
    reason = state.terminal_reason()
    if reason is not None:
        return state.into_trace(reason)
    while True:
        decoded = decode_step(state.decode_steps, state.current_token, state.current_caches)
        reason = state.apply_decode_step(decoded)
        if reason is not None:
            return state.into_trace(reason)


def greedy_generate_chunked(prefill_top_k, initial_kv_caches, config: GreedyGenerationConfig,
                            decode_chunk_size: int, decode_chunk) -> GreedyChunkedGenerationTrace:
    """crates/pvlc-cpu-ref/src/lib.rs:2309-2366.

    decode_chunk(chunk_index, input_token, caches, requested_steps) returns a
    list of GreedyDecodeStep with 1..requested_steps entries; a terminal step
    (EOS or the token budget) must be the chunk's last.
    """
    if decode_chunk_size == 0:
        raise GreedyError(DIMENSION_MISMATCH, "decode chunk size")
    state = GreedyGenerationState.initialize(prefill_top_k, initial_kv_caches, config)
    reason = state.terminal_reason()
    if reason is not None:
        return GreedyChunkedGenerationTrace(state.into_trace(reason), 0)
    chunks = 0
    while True:
        requested = min(decode_chunk_size, state.remaining_decode_steps())
        steps = decode_chunk(chunks, state.current_token, state.current_caches, requested)
        if len(steps) == 0 or len(steps) > requested:
            raise GreedyError(DIMENSION_MISMATCH, "decode chunk length")
        terminal = None
        for i, decoded in enumerate(steps):
            terminal = state.apply_decode_step(decoded)
            if terminal is not None and i + 1 != len(steps):
                raise GreedyError(DIMENSION_MISMATCH, "steps after a terminal token")
        chunks += 1
        if terminal is not None:
            return GreedyChunkedGenerationTrace(state.into_trace(terminal), chunks)


class BatchedGreedyState:
    """The rules of GreedyGenerationState applied to B requests at once.

    The batched engine decodes every request of a batch in lockstep and
    reads back [steps, B] top-1 tokens per chunk; per request this applies
    exactly GreedyGenerationState's rules (first token from the prefill, EOS
    kept and terminal, stop at max_new_tokens, steps after a stop ignored)
    without a Python object per request, layer and step.  Top-1 ties are
    resolved on the device by argmax's first (smallest) index, the same rule
    as compare_top_k_entries for finite logits.
    """

    def __init__(self, first_tokens, max_new_tokens: int, eos_token_id: int):
        import numpy as np
        first = np.asarray(first_tokens, dtype=np.int64).reshape(-1)
        if max_new_tokens <= 0 or first.size == 0:
            raise GreedyError(DIMENSION_MISMATCH, "generation config")
        self.max_new_tokens = int(max_new_tokens)
        self.eos = int(eos_token_id)
        self.tokens = np.zeros((first.size, self.max_new_tokens), np.int64)
        self.tokens[:, 0] = first
        self.count = np.ones(first.size, np.int64)
        self.eos_stop = first == self.eos
        self.done = self.eos_stop | (self.count == self.max_new_tokens)
        self.decode_steps = np.zeros(first.size, np.int64)

    def remaining_decode_steps(self) -> int:
        import numpy as np
        active = ~self.done
        return int((self.max_new_tokens - self.count[active]).max()) if active.any() else 0

    def apply_steps(self, steps) -> None:
        """steps: [S, B] top-1 tokens of S consecutive decode steps."""
        import numpy as np
        steps = np.asarray(steps, dtype=np.int64)
        for row in steps:
            active = ~self.done
            if not active.any():
                break
            idx = np.nonzero(active)[0]
            self.tokens[idx, self.count[idx]] = row[idx]
            self.count[idx] += 1
            self.decode_steps[idx] += 1
            eos = row[idx] == self.eos
            self.eos_stop[idx] |= eos
            self.done[idx] = eos | (self.count[idx] == self.max_new_tokens)

    def all_done(self) -> bool:
        return bool(self.done.all())

    def generated(self, b: int) -> List[int]:
        return self.tokens[b, : self.count[b]].tolist()

    def stop_reason(self, b: int) -> str:
        return EOS_TOKEN if self.eos_stop[b] else MAX_NEW_TOKENS


def pinned_greedy_generate(prefill_top_k, initial_kv_caches, max_new_tokens: int,
                           decode_step: DecodeStepFn) -> GreedyGenerationTrace:
    """crates/pvlc-cpu-ref/src/lib.rs:2381-2397."""
    return greedy_generate(prefill_top_k, initial_kv_caches,
                           pinned_greedy_generation_config(max_new_tokens), decode_step)
