"""Import-path alias of sparse/module/spatial_sparse_attention.py."""
from lsrm_sparse.module import (  # noqa: F401
    SpatialSparseAttentionIn,
    SpatialSparseAttentionMid,
    SpatialSparseAttentionOut,
)
