"""B200 (sm_100a) attention backend for the PaddleOCR-VL engine.

Three attention paths behind the reference's operator contract, exported as a
C ABI (include/pvlc_cuda_attn.h, libpvlc_cuda_attn.so):
  * vision varlen bidirectional attention with fused 2-D RoPE  (ops.vision_varlen_attention)
  * decoder causal GQA prefill with fused M-RoPE + KV write     (ops.decoder_prefill)
  * batched split-KV GQA decode with fused M-RoPE + KV append   (ops.decode, session.DecoderKvSession)
"""
from . import abi, positions  # noqa: F401

__all__ = ["abi", "positions"]
