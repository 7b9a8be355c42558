"""Import-path alias of sparse/ops/block_window_attention.py; implemented in CUDA."""
from lsrm_sparse.api import sparse_window_attention  # noqa: F401
