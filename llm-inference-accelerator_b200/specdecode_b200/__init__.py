"""specdecode_b200 — the paged INT8 KV-cache hot path of a speculative decoder
on B200 (sm_100a).

Python host code over one C-ABI CUDA library (libspecdecode_cuda.so, built
in-tree by ``llm-inference-accelerator_b200/csrc/build.py``) that holds the
quantize-and-append, rollback, paged verify-attention and gather/dequantize
kernels.  There is no CPU implementation of any of these: without the
library or a CUDA device the cache raises instead of computing.
"""

from ._lib import NativeBackendError, NativeLibraryNotFound, load_library
from .kv_cache import (
    CudaUnavailableError,
    DequantizedKVToken,
    KVCacheCapacityError,
    KVCacheCheckpoint,
    KVCacheConfig,
    KVCacheError,
    KVCacheStats,
    KVQuantizer,
    PagedKVCache,
    QuantizedKVToken,
    QuantizedVector,
)
from .page_table import PageTable

__all__ = [
    "CudaUnavailableError",
    "DequantizedKVToken",
    "KVCacheCapacityError",
    "KVCacheCheckpoint",
    "KVCacheConfig",
    "KVCacheError",
    "KVCacheStats",
    "KVQuantizer",
    "NativeBackendError",
    "NativeLibraryNotFound",
    "PageTable",
    "PagedKVCache",
    "QuantizedKVToken",
    "QuantizedVector",
    "load_library",
]
