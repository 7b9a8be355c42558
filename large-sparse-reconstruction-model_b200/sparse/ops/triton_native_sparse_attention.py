"""Import-path alias of the reference module of this name so callers need no
edit; the implementation is the sm_100a CUDA library (no Triton)."""
from lsrm_sparse.api import spatial_selection_attention  # noqa: F401
