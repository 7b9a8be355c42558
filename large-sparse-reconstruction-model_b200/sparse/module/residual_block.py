"""Import-path alias of sparse/module/residual_block.py."""
from lsrm_sparse.module import LayerNorm32, SparseResBlock  # noqa: F401
