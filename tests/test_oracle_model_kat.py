"""Known-answer pins of the oracle's model-level composition (oracle/pvlc_model_oracle.cpp).

* decoder layer prefill: the literal COMBINED_BLAKE3 of
  crates/pvlc-cpu-ref/tests/decoder_layer_contract.rs:18 over the fixture of
  :144-181 (digest schema :413-450);
* prefill LM head: the literal logits bits and blake3 of
  crates/pvlc-cpu-ref/tests/prefill_lm_head_contract.rs:11-39;
* RMSNorm / LayerNorm / linear: order-of-operation checks against plain loops.
"""
import struct

import blake3
import numpy as np

import pvlc_oracle as O

F = np.float32


def dense(n, mul, add, mod, div):
    # decoder_layer_contract.rs:144-148
    i = np.arange(n, dtype=np.int64)
    return (((i * mul + add) % mod).astype(F) - F(mod // 2)) / F(div)


def test_decoder_layer_prefill_matches_reference_combined_digest():
    T, H, I, QH, KVH, HD = 3, 5, 7, 4, 2, 6
    k = np.arange(H)
    w = [F(0.7) + ((k * 3 + 1) % 7).astype(F) / F(20.0),
         dense(QH * HD * H, 7, 3, 29, 19.0), dense(KVH * HD * H, 11, 5, 31, 23.0),
         dense(KVH * HD * H, 13, 7, 37, 29.0), dense(H * QH * HD, 17, 2, 41, 31.0),
         F(0.65) + ((k * 5 + 2) % 9).astype(F) / F(24.0),
         dense(I * H, 19, 1, 43, 37.0), dense(I * H, 23, 4, 47, 41.0),
         dense(H * I, 29, 6, 53, 43.0)]
    x = dense(T * H, 17, 3, 29, 11.0)
    a, t, d = np.meshgrid(np.arange(3), np.arange(T), np.arange(HD), indexing="ij")
    cos = F(0.55) + a.astype(F) * F(0.13) + t.astype(F) * F(0.02) + d.astype(F) * F(0.007)
    sin = F(-0.3) - a.astype(F) * F(0.11) + t.astype(F) * F(0.015) - d.astype(F) * F(0.005)
    tr = O.decoder_layer_prefill(x, T, H, I, QH, KVH, HD, 1e-5, (1, 1, 1), cos, sin, w)
    h = blake3.blake3()
    for name in ("norm1", "query", "key", "value", "mrope_query", "mrope_key", "mrope_key",
                 "value"):                      # cache keys / values are copies
        h.update(tr[name].astype("<f4").tobytes())
    for meta in (T, KVH, HD):
        h.update(struct.pack("<Q", meta))
    for name in ("attention_context", "attention_output", "attention_residual", "norm2",
                 "mlp_gate", "mlp_up", "mlp_activation", "mlp_down", "output"):
        h.update(tr[name].astype("<f4").tobytes())
    assert h.hexdigest() == "61ab6647b035c78971b02d51c4600f5e78d92686deda863809ea0e7f9c35740e"


def test_prefill_lm_head_matches_reference_literal_bits_and_digest():
    final_norm = np.array([0.125, -1.75, 2.5, 0.33333334, 9.25, -0.5, 1.125, -3.75, 0.2, -1.3,
                           2.7, 0.0625], F)
    lm = np.array([0.7, -1.1, 0.3, 2.0, -0.4, 0.9, -1.7, 0.125, 1.2, 0.25, -0.75, 0.6, -2.0, 1.5,
                   0.5, -0.2, 0.05, -0.08, 0.13, -0.21], F).reshape(5, 4)
    logits = O.prefill_last_logits(final_norm.reshape(3, 4), lm)
    assert [int(b) for b in logits.view(np.uint32)] == \
        [0x402051ec, 0xc0baa148, 0xc004a3d8, 0xbf819999, 0x3ee75c28]
    assert blake3.blake3(logits.astype("<f4").tobytes()).hexdigest() == \
        "330604b81e09bab80b697069dbae035d946b5b29c05afebf011a73052afdd6c7"


def _loop_norms(x, w, b, eps, kind):
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        s = x[r]
        if kind == "rms":
            acc = F(0)
            for v in s:
                acc = F(acc + v * v)
            acc = F(acc / F(len(s)))
            inv = F(F(1) / F(np.sqrt(F(acc + F(eps)))))
            out[r] = s * inv * w
        else:
            mean = F(0)
            for v in s:
                mean = F(mean + v)
            mean = F(mean / F(len(s)))
            var = F(0)
            for v in s:
                c = F(v - mean)
                var = F(var + c * c)
            var = F(var / F(len(s)))
            inv = F(F(1) / F(np.sqrt(F(var + F(eps)))))
            out[r] = (s - mean) * inv * w + b
    return out


def test_norms_and_linear_follow_reference_operation_order():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, 37)).astype(F)
    w = rng.standard_normal(37).astype(F)
    b = rng.standard_normal(37).astype(F)
    assert np.array_equal(O.rms_norm(x, w, 1e-5), _loop_norms(x, w, b, 1e-5, "rms"))
    assert np.array_equal(O.layer_norm(x, w, b, 1e-6), _loop_norms(x, w, b, 1e-6, "ln"))
    W = rng.standard_normal((5, 37)).astype(F)
    bias = rng.standard_normal(5).astype(F)
    ref = np.empty((4, 5), F)
    for r in range(4):
        for o in range(5):
            acc = bias[o]
            for d in range(37):
                acc = F(acc + F(x[r, d] * W[o, d]))
            ref[r, o] = acc
    assert np.array_equal(O.linear(x, W, bias), ref)
