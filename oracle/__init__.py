"""CPU oracle for LSRM's variable-block native sparse attention.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or as the timed CPU restatement of the reference.

Parity status: pinned.  ``tests/golden/make_golden.py`` runs the reference's
own code (``sparse.ops.get_block_score``, ``SparseResBlock``,
``torch.segment_reduce``, ``SpatialSparseAttentionOut`` and the Triton
``native_sparse_attend`` under ``TRITON_INTERPRET=1`` in fp16) and stores its
outputs as fixtures; ``tests/test_oracle_golden.py`` checks this oracle
against them.
"""

from .nsa_oracle import *  # noqa: F401,F403
from .attn_maps import (camera_terms, fma32, image_sort_keys, image_token_points,  # noqa: F401
                        image_volume_block_topk,
                        project_to_blocks, view_block_geometry, view_block_topk, view_rows_equivalent,
                        voxel_points)
