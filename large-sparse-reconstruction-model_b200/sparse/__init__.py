"""Drop-in package with the reference's import paths (``sparse``,
``sparse.ops``, ``sparse.module``), backed by lsrm_sparse."""

from .module.spatial_sparse_attention import (
    SpatialSparseAttentionIn,
    SpatialSparseAttentionMid,
    SpatialSparseAttentionOut,
)
