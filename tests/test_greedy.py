"""Greedy generation state machine (pvlc_b200.greedy) against the reference's contract.

Fixtures and literal digests follow
crates/pvlc-cpu-ref/tests/greedy_generation_contract.rs and
crates/pvlc-cpu-ref/tests/greedy_decode_chunk_contract.rs (digest schemas at
:125-160 and :170-200 respectively).
"""
import struct
from dataclasses import dataclass

import blake3
import numpy as np
import pytest

from pvlc_b200 import greedy as G


@dataclass
class Cache:
    tokens: int
    key_value_heads: int
    head_dim: int
    keys: list
    values: list


def f32(v):
    return struct.unpack("<f", struct.pack("<f", v))[0]


def cache(tokens, keys, values):
    return Cache(tokens, 1, 2, [f32(v) for v in keys], [f32(v) for v in values])


def shaped_cache(tokens, kvh, hd, layer, generation):
    n = tokens * kvh * hd
    base = float(generation * 100 + layer * 20)
    keys = (np.float32(base) + np.arange(n, dtype=np.float32) / np.float32(16.0)).tolist()
    values = (-np.float32(base) - np.arange(n, dtype=np.float32) / np.float32(32.0)).tolist()
    return Cache(tokens, kvh, hd, keys, values)


def synthetic_caches(tokens, layers, generation):
    return [shaped_cache(tokens, 1, 2, layer, generation) for layer in range(layers)]


def config(layers, max_new, eos, vocab=8):
    return G.GreedyGenerationConfig(layers, vocab, 1, 2, max_new, eos)


def E(i, v):
    return G.TopKEntry(i, f32(v))


def _u(h, v):
    h.update(struct.pack("<Q", v))


def _f(h, values):
    _u(h, len(values))
    for v in values:
        h.update(struct.pack("<f", v))


def _trace_body(h, trace):
    _u(h, len(trace.generated_tokens))
    for t in trace.generated_tokens:
        _u(h, t)
    _u(h, len(trace.kv_caches))
    for c in trace.kv_caches:
        _u(h, c.tokens)
        _u(h, c.key_value_heads)
        _u(h, c.head_dim)
        _f(h, c.keys)
        _f(h, c.values)
    h.update(bytes([0 if trace.stop_reason == G.MAX_NEW_TOKENS else 1]))
    _u(h, trace.decode_steps)


def trace_digest(trace):
    # greedy_generation_contract.rs:136-160
    h = blake3.blake3()
    h.update(b"pvlc-greedy-generation-v1\0")
    _trace_body(h, trace)
    return h.hexdigest()


def chunk_trace_digest(trace):
    # greedy_decode_chunk_contract.rs:176-200
    h = blake3.blake3()
    h.update(b"pvlc-greedy-decode-chunk-v1\0")
    _trace_body(h, trace.generation)
    _u(h, trace.decode_chunks)
    return h.hexdigest()


def test_literal_four_token_trace_matches_fixed_digest():
    # greedy_generation_contract.rs:162-240
    initial = [cache(2, [0.10, 0.11, 0.12, 0.13], [1.10, 1.11, 1.12, 1.13]),
               cache(2, [2.10, 2.11, 2.12, 2.13], [3.10, 3.11, 3.12, 3.13])]
    after_five = [cache(3, [0.20, 0.21, 0.22, 0.23, 0.24, 0.25], [1.20, 1.21, 1.22, 1.23, 1.24, 1.25]),
                  cache(3, [2.20, 2.21, 2.22, 2.23, 2.24, 2.25], [3.20, 3.21, 3.22, 3.23, 3.24, 3.25])]
    after_one = [cache(4, [0.30, 0.31, 0.32, 0.33, 0.34, 0.35, 0.36, 0.37],
                       [1.30, 1.31, 1.32, 1.33, 1.34, 1.35, 1.36, 1.37]),
                 cache(4, [2.30, 2.31, 2.32, 2.33, 2.34, 2.35, 2.36, 2.37],
                       [3.30, 3.31, 3.32, 3.33, 3.34, 3.35, 3.36, 3.37])]
    after_six = [cache(5, [0.40, 0.41, 0.42, 0.43, 0.44, 0.45, 0.46, 0.47, 0.48, 0.49],
                       [1.40, 1.41, 1.42, 1.43, 1.44, 1.45, 1.46, 1.47, 1.48, 1.49]),
                 cache(5, [2.40, 2.41, 2.42, 2.43, 2.44, 2.45, 2.46, 2.47, 2.48, 2.49],
                       [3.40, 3.41, 3.42, 3.43, 3.44, 3.45, 3.46, 3.47, 3.48, 3.49])]
    expected_inputs = [initial, after_five, after_one]
    outputs = [after_five, after_one, after_six]
    tokens_in = [3, 5, 1]
    tops = [[E(5, 9.5), E(4, 8.0)], [E(1, 7.25), E(0, 6.0)], [E(6, 5.5), E(2, 4.0)]]
    calls = []

    def step(i, tok, caches):
        assert i == len(calls)
        assert tok == tokens_in[i]
        assert caches is expected_inputs[i]
        calls.append(i)
        return G.GreedyDecodeStep(tops[i], outputs[i])

    trace = G.greedy_generate([E(3, 10.0), E(1, 9.0)], initial, config(2, 4, 7), step)
    assert len(calls) == 3
    assert trace.generated_tokens == [3, 5, 1, 6]
    assert trace.kv_caches is after_six
    assert trace.decode_steps == 3
    assert trace.stop_reason == G.MAX_NEW_TOKENS
    assert trace_digest(trace) == "f830d7fe54c0fb87f45e6a0ae1ba8f2fd9d0ffdfbcfe9bc786f194dd6baf80ba"


def test_max_one_returns_prefill_top_one_without_callback():
    initial = synthetic_caches(3, 2, 0)

    def never(*a):
        raise AssertionError("max_new_tokens=1 must not decode")

    trace = G.greedy_generate([E(4, 3.0), E(2, 1.0)], initial, config(2, 1, 7), never)
    assert trace.generated_tokens == [4]
    assert trace.decode_steps == 0
    assert trace.stop_reason == G.MAX_NEW_TOKENS
    assert trace.kv_caches is initial


def test_prefill_eos_stops_before_decode():
    initial = synthetic_caches(1, 2, 0)
    trace = G.greedy_generate([E(2, 5.0), E(1, 4.0)], initial, config(2, 8, 2),
                              lambda *a: pytest.fail("prefill EOS must stop"))
    assert trace.generated_tokens == [2]
    assert trace.stop_reason == G.EOS_TOKEN
    assert trace.decode_steps == 0


def test_decode_eos_is_appended_and_stops():
    initial = synthetic_caches(2, 1, 0)
    final = synthetic_caches(3, 1, 1)
    calls = []

    def step(i, tok, caches):
        calls.append((i, tok, caches[0].tokens))
        return G.GreedyDecodeStep([E(2, 7.0), E(1, 6.0)], final)

    trace = G.greedy_generate([E(4, 5.0)], initial, config(1, 6, 2), step)
    assert calls == [(0, 4, 2)]
    assert trace.generated_tokens == [4, 2]
    assert trace.kv_caches is final
    assert trace.stop_reason == G.EOS_TOKEN


def test_callback_error_propagates_and_prevents_later_calls():
    calls = []

    def step(i, tok, caches):
        calls.append(i)
        raise G.CallbackError("boom")

    with pytest.raises(G.CallbackError):
        G.greedy_generate([E(4, 5.0)], synthetic_caches(2, 2, 0), config(2, 4, 7), step)
    assert calls == [0]


@pytest.mark.parametrize("cfg", [
    G.GreedyGenerationConfig(0, 8, 1, 2, 2, 7), G.GreedyGenerationConfig(2, 0, 1, 2, 2, 0),
    G.GreedyGenerationConfig(2, 8, 0, 2, 2, 7), G.GreedyGenerationConfig(2, 8, 1, 0, 2, 7),
    G.GreedyGenerationConfig(2, 8, 1, 2, 0, 7), G.GreedyGenerationConfig(2, 8, 1, 2, 2, 8),
    G.GreedyGenerationConfig(2, 8, 1, 2, 2, 9)])
def test_malformed_config_rejected_before_callback(cfg):
    with pytest.raises(G.GreedyError) as e:
        G.greedy_generate([E(4, 5.0), E(1, 3.0)], synthetic_caches(2, 2, 0), cfg,
                          lambda *a: pytest.fail("reached callback"))
    assert e.value.code == G.DIMENSION_MISMATCH


@pytest.mark.parametrize("candidates,code", [
    ([], G.DIMENSION_MISMATCH),
    ([E(t, 20.0 - t) for t in range(9)], G.DIMENSION_MISMATCH),
    ([E(1, 4.0), E(1, 3.0)], G.DIMENSION_MISMATCH),
    ([E(8, 4.0)], G.DIMENSION_MISMATCH),
    ([E(1, 3.0), E(2, 4.0)], G.DIMENSION_MISMATCH),
    ([E(2, 4.0), E(1, 4.0)], G.DIMENSION_MISMATCH),
    ([G.TopKEntry(1, float("nan"))], G.NON_FINITE_INPUT),
    ([G.TopKEntry(1, float("inf"))], G.NON_FINITE_INPUT),
    ([G.TopKEntry(1, float("-inf"))], G.NON_FINITE_INPUT)])
def test_malformed_prefill_candidates_rejected_before_callback(candidates, code):
    # greedy_generation_contract.rs:401-458
    with pytest.raises(G.GreedyError) as e:
        G.greedy_generate(candidates, synthetic_caches(2, 2, 0), config(2, 2, 7),
                          lambda *a: pytest.fail("reached callback"))
    assert e.value.code == code


def test_malformed_step_caches_fail_before_later_callback():
    calls = []

    def step(i, tok, caches):
        calls.append(i)
        # wrong length: cache not one token longer
        return G.GreedyDecodeStep([E(5, 1.0)], synthetic_caches(2, 2, 1))

    with pytest.raises(G.GreedyError) as e:
        G.greedy_generate([E(4, 5.0)], synthetic_caches(2, 2, 0), config(2, 4, 7), step)
    assert e.value.code == G.DIMENSION_MISMATCH
    assert calls == [0]


def test_top_k_orders_by_value_then_smaller_index_under_total_order():
    vals = [1.0, 3.0, 3.0, -0.0, 0.0, 2.5]
    got = [(e.index, e.value) for e in G.top_k(vals, 6)]
    assert got == [(1, 3.0), (2, 3.0), (5, 2.5), (0, 1.0), (4, 0.0), (3, -0.0)]
    with pytest.raises(G.GreedyError) as e:
        G.top_k(vals, 7)
    assert e.value.code == G.INVALID_K


# ---------------------------------------------------------------- chunked
PREFILL_TOKEN, EOS, NEXT = 4, 63, [5, 6, 7, 8, 9, 10, 11, 12]


def chunk_caches(tokens, generation):
    return [shaped_cache(tokens, 1, 2, layer, generation) for layer in range(2)]


def chunk_step(tok, i):
    return G.GreedyDecodeStep([E(tok, 100.0 - i)], chunk_caches(2 + i + 1, i + 1))


def run_exact_chunks(size):
    decoded = [0]
    chunks = [0]

    def chunk(ci, tok, current, requested):
        assert ci == chunks[0]
        assert tok == (PREFILL_TOKEN if decoded[0] == 0 else NEXT[decoded[0] - 1])
        assert requested == min(size, len(NEXT) - decoded[0])
        steps = [chunk_step(NEXT[decoded[0] + o], decoded[0] + o) for o in range(requested)]
        decoded[0] += requested
        chunks[0] += 1
        return steps

    cfg = G.GreedyGenerationConfig(2, 64, 1, 2, 9, EOS)
    return G.greedy_generate_chunked([E(PREFILL_TOKEN, 101.0)], chunk_caches(2, 0), cfg, size,
                                     chunk)


def test_literal_nine_token_three_chunk_trace_matches_fixed_digest():
    # greedy_decode_chunk_contract.rs:242-251
    trace = run_exact_chunks(3)
    assert trace.generation.generated_tokens == [PREFILL_TOKEN] + NEXT
    assert trace.decode_chunks == 3
    assert chunk_trace_digest(trace) == \
        "2bd4512d55393ab9f9115b0827edf7821a54d6ea6be963d0be5caabe88e60259"


@pytest.mark.parametrize("size,chunks", [(1, 8), (2, 4), (4, 2), (8, 1)])
def test_chunk_sizes_equal_single_step_generation(size, chunks):
    trace = run_exact_chunks(size)
    assert trace.generation.generated_tokens == [PREFILL_TOKEN] + NEXT
    assert trace.decode_chunks == chunks
    assert trace.generation.stop_reason == G.MAX_NEW_TOKENS


def test_chunk_with_steps_after_eos_is_rejected():
    def chunk(ci, tok, current, requested):
        return [G.GreedyDecodeStep([E(EOS, 1.0)], chunk_caches(3, 1)),
                G.GreedyDecodeStep([E(7, 1.0)], chunk_caches(4, 2))]

    cfg = G.GreedyGenerationConfig(2, 64, 1, 2, 9, EOS)
    with pytest.raises(G.GreedyError):
        G.greedy_generate_chunked([E(PREFILL_TOKEN, 101.0)], chunk_caches(2, 0), cfg, 4, chunk)


def test_pinned_config_freezes_topology():
    cfg = G.pinned_greedy_generation_config(512)
    assert (cfg.layers, cfg.vocab_size, cfg.key_value_heads, cfg.head_dim, cfg.eos_token_id) == \
        (18, 103424, 2, 128, 2)


def test_batched_state_applies_the_single_request_rules():
    """BatchedGreedyState == GreedyGenerationState per request on random step streams."""
    rng = np.random.default_rng(3)
    eos, max_new, B, S = 2, 9, 6, 12
    first = rng.integers(0, 6, B)
    first[0] = eos                       # prefill EOS
    steps = rng.integers(0, 6, (S, B))
    batched = G.BatchedGreedyState(first, max_new, eos)
    batched.apply_steps(steps[:5])
    batched.apply_steps(steps[5:])
    for b in range(B):
        cfg = G.GreedyGenerationConfig(1, 8, 1, 2, max_new, eos)
        it = iter(range(S))

        def step(i, tok, caches, b=b):
            s = next(it)
            return G.GreedyDecodeStep([G.TopKEntry(int(steps[s, b]), 1.0)],
                                      [Cache(caches[0].tokens + 1, 1, 2, None, None)])

        ref = G.greedy_generate([G.TopKEntry(int(first[b]), 1.0)],
                                [Cache(3, 1, 2, None, None)], cfg, step)
        assert batched.generated(b) == ref.generated_tokens
        assert batched.stop_reason(b) == ref.stop_reason
        assert int(batched.decode_steps[b]) == ref.decode_steps
    assert batched.all_done()
