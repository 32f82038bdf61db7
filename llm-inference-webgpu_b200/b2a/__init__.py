"""b2a: the Qwen2.5 grouped-query attention hot path of abho7/llm-inference-webgpu,
rebuilt as CUDA kernels for B200 (sm_100a) behind a C ABI (include/b2a.h).

This package is the host-side mirror of the reference's attention / KV-cache
operator API (src/core/attention.js, src/core/ops.js, src/cpu/cache.js,
src/gpu/model.js) over libb2a.so. There is no CPU fallback: without the built
library, or without a CUDA device, calls raise.
"""
from ._lib import B2AError, BusyError, RangeError, load, lib_path  # noqa: F401
from .attention import (appendRope, attentionDecode, attentionDecodeAsync, attentionPrefill, attentionPrefillBatch, decodePartial, decodeSplit, decodeSplitNccl,  # noqa: F401
                        default_context, groupedAttention, kvHeadFor, linearInt8, lseCombine, qkvInt8,
                        quantizeInt8PerChannel, ropeFrequencies, ropeTables)
from .model import Model, ModelConfig  # noqa: F401
from .weights import Safetensors, TensorInfo, write_safetensors  # noqa: F401
from .runtime import CacheConfig, Context, Exchange, GpuKVCache, PagePool, RopeTable  # noqa: F401
