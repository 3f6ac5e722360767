"""cdclq - B200-native (sm_100a) CDCL-GPTQ per-layer quantization path.

Python mirror of the reference crate's library surface (tailot/CDCL-GPTQ: engine, quant, linalg, pipeline),
backed by the CUDA library libcdclq_cuda.so through its C ABI (include/cdclq.h).
"""
from ._lib import CdclqError, LIB_PATH, lib
from .abi import Config, LayerStats, effective_group, num_groups
from .engine import PrepCache, proxy_loss, quantize_layer, row_chunk, rtn_layer, validate
from .quant import F16_MIN_NORMAL, QLayer, find_params, row_bytes

__all__ = [
    "CdclqError", "LIB_PATH", "lib", "Config", "LayerStats", "effective_group", "num_groups", "PrepCache",
    "proxy_loss", "quantize_layer", "row_chunk", "rtn_layer", "validate", "F16_MIN_NORMAL", "QLayer",
    "find_params", "row_bytes",
]
