"""B200 (sm_100a) variable-block native sparse attention for LSRM.

``lsrm_sparse.api`` and ``lsrm_sparse.module`` mirror the reference's
``sparse.ops`` and ``sparse.module``; the sibling ``sparse`` package re-exports
them under the reference's import paths.  All compute runs in
``liblsrm_sparse.so`` (built by ``build.py``)."""

from .api import (compressed_attention, get_block_score, native_sparse_attend, set_variant,
                  sliding_window_attention, sparse_window_attention, spatial_selection_attention)
from .module import (SparseResBlock, SpatialSparseAttentionIn, SpatialSparseAttentionMid,
                     SpatialSparseAttentionOut)
