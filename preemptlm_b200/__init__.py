"""B200-native SlottedGLU MoE hot path (preemptLM's slotted MoE block).

Python host code over libsg_b200.so (hand-written sm_100a kernels behind the
C-ABI in include/sg_abi.h).  There is no CPU fallback: the ops raise if the
shared library is missing.
"""

from .arena import GLU_PROJECTION_NAMES, SlottedGLU
from .bank import (ExpertBankManifest, ExpertBankWriter, ModelMoESpec, PreadExpertBank, ReadPriority,
                   SerializedExpert, TensorSpec, decode_serialized_expert, parse_encoding_tag)
from .cache_manager import CacheEvictionPolicy, ExpertCacheManager
from .layer import BaseMoEWrapper, Qwen3_xMoEWrapper, SlottedMoE, SparseMoeBlock
from .loader import DiskBackedExpertLoader, GenerationMetrics, HostExpertCache
from .quant import MlxQuantMode, QuantSettings, dequantize_affine, quantize_affine
from .trace import (ExpertTraceRecorder, ListTraceSink, ParquetTraceSink, TraceRunContext, TraceStepContext,
                    arrow_schema)

__all__ = [
    "GLU_PROJECTION_NAMES", "SlottedGLU", "ExpertBankManifest", "ExpertBankWriter", "ModelMoESpec",
    "PreadExpertBank", "ReadPriority", "SerializedExpert", "TensorSpec", "decode_serialized_expert",
    "parse_encoding_tag", "CacheEvictionPolicy", "ExpertCacheManager", "BaseMoEWrapper", "Qwen3_xMoEWrapper",
    "SlottedMoE", "SparseMoeBlock", "DiskBackedExpertLoader", "GenerationMetrics", "HostExpertCache",
    "MlxQuantMode", "QuantSettings", "dequantize_affine", "quantize_affine", "ExpertTraceRecorder",
    "ListTraceSink", "ParquetTraceSink", "TraceRunContext", "TraceStepContext", "arrow_schema",
]
