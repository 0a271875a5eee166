"""B200-native fused single-query decode attention (fp16 / int8-KV / int4-KV / GQA / split-K).

Drop-in for the operator surface of emirabayer/Fused-Quantized-KV-Decode-
Attention: the same five attention operators and the two per-token KV
quantizers, computed by hand-written sm_100a CUDA kernels in
``libfqkv_b200.so`` (C ABI: ``include/fqkv_b200.h``).

The directory name is not a Python identifier, so import it with
``importlib.import_module("fused-quantized-kv-decode-attention_b200")``.
"""
from __future__ import annotations

from . import _native, hf_integration, ops, sharding, tp_exchange
from .ops import (
    decode_attn_fp16_mw,
    decode_attn_gqa,
    decode_attn_gqa_int8,
    decode_attn_gqa_int8_kvcache,
    decode_attn_gqa_kvcache,
    decode_attn_int4,
    decode_attn_int8_mw,
    decode_attn_kvcache_tp,
    gqa_sk_fast,
    qpt,
    quant_int4_per_token,
    add_rmsnorm,
    gemv,
    gemv_rope_append,
    gemv_swiglu,
    quantize_into_cache,
    rope_qkv_append,
    silu_mul,
    tp_wait,
    workspace_bytes,
)

__all__ = [
    "decode_attn_fp16_mw",
    "decode_attn_int8_mw",
    "decode_attn_int4",
    "decode_attn_gqa",
    "decode_attn_gqa_kvcache",
    "decode_attn_gqa_int8",
    "decode_attn_gqa_int8_kvcache",
    "quantize_into_cache",
    "rope_qkv_append",
    "add_rmsnorm",
    "gemv",
    "gemv_rope_append",
    "gemv_swiglu",
    "silu_mul",
    "decode_attn_kvcache_tp",
    "tp_wait",
    "gqa_sk_fast",
    "qpt",
    "quant_int4_per_token",
    "workspace_bytes",
    "build",
    "library_path",
    "native",
    "sharding",
    "hf_integration",
    "tp_exchange",
    "ops",
]

native = _native


def library_path() -> str:
    return str(_native.LIB_PATH)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libfqkv_b200.so`` in-tree (nvcc, sm_100a) if it is out of date."""
    import importlib.util
    import pathlib

    spec = importlib.util.spec_from_file_location(
        "_fqkv_build", pathlib.Path(__file__).resolve().with_name("build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return str(mod.build(force=force, verbose=verbose))
