"""Import-path alias of sparse/ops/block_score.py; implemented in CUDA."""
from lsrm_sparse.api import get_block_score  # noqa: F401
