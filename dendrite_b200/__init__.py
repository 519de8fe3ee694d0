"""dendrite_b200 — B200-native (sm_100a) paged cascade decode attention over
copy-on-write block tables, with the FP8 E4M3 / MXFP8 KV-page codec.

The compute path is ``libdendrite_b200.so`` (C ABI: include/dendrite_b200.h);
this package is its host-side binding and the mirror of Dendrite's
AttentionBackend interface. Importing it loads the native library and raises
if it is missing: there is no CPU fallback.
"""
from ._lib import (AllocationFailed, CudaError, FfiError, InvalidArgument, NotAvailable,  # noqa: F401
                   WorkspaceTooSmall, version)
from .backend import (PAGE_SIZE, SUPPORTED_HEAD_DIMS, AttentionConfig, B200Backend,  # noqa: F401
                      BlockTable, CascadePlan, append_kv_batch, cascade_decode, copy_pages,
                      decode_paged, dequantize_kv_pages,
                      make_config, merge_states, quantize_kv_pages, scatter_head_shards,
                      selftest_wait, workspace_status)

from .paged_cache import PagedKVCache  # noqa: F401

__version__ = "0.1.0"
