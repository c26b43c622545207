"""B200-native (sm_100a) PrismKV decode-time sparse retrieval.

The reference's operator API (src/prismkv/__init__.py: FeatureIndex,
SharedSAE, build_index, select_buckets, attend, append_index, plus
bucket_scores and summarize from core.py) over hand-written CUDA kernels, and
the batched device operator ``SparseDecode`` (the role of the reference's
Native8B / DecodeOps).  The CUDA library is loaded on first use; without it
every operation raises -- there is no CPU path.
"""
from .core import (FeatureIndex, SharedSAE, append_index, attend, bucket_scores, build_index, select_buckets,
                   summarize)
from .decode import SparseDecode, kv_append
from .index import DeviceIndex, SAEParams

__all__ = ["FeatureIndex", "SharedSAE", "build_index", "select_buckets", "attend", "append_index",
           "bucket_scores", "summarize", "SparseDecode", "kv_append", "DeviceIndex", "SAEParams"]
