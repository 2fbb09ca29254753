"""k8v4_xpu_b200: a B200-native (sm_100a) quantized-KV LLM serving framework.

Int8-K / int4-V paged KV cache (``int8_k_int4_v``), GPTQ INT4 weights with an
INT8 embedding side file, MLP-only W4A8 prefill, tensor and context
parallelism over NVLink, MTP speculative decoding, CUDA-graph decode, chunked
prefill and prefix caching, served through an OpenAI-compatible endpoint.
"""
from .kv.layout import CACHE_DTYPE, PageLayout  # noqa: F401

__version__ = "0.1.0"
