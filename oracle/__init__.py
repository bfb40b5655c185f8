"""CPU oracle for Palu compressed-KV decode attention.

TEST INFRASTRUCTURE ONLY. This package restates, in plain fp32 PyTorch on the CPU, the reference's
own CPU model of the hot path (``palu_tt/fused.py:82-107`` ``reference_decode`` and
``palu_tt/reference.py:14-55`` ``PaluRefAttention``) plus the host table builders it depends on.
It is the checker the CUDA path is compared against. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) may import it; the product
package never does, and the product fails loudly instead of falling back to it.

Pinning: the restatement is checked against golden vectors produced by the reference's own Python
code (``tests/golden/make_golden.py``, run where the reference tree is mounted) and, where the
reference tree is present, against the reference functions directly.
"""
from oracle.palu_ref import (  # noqa: F401
    MAX_CHUNK,
    chunk_size,
    cos_sin_tables,
    cs_table,
    expand_groups,
    llama3_scale_freqs,
    phase2_tables,
    reference_decode,
    reference_decode_streamed,
    rope_freqs,
    rope_transformation_matrix,
    rot_step_table,
    trans_mat_tile,
    w_rot_from_u_k,
    PaluRefAttention,
    reverse_permute,
    seeded_decode_inputs,
    input_checksums,
)
from oracle.metrics import rel_errors, rowwise_rel_errors  # noqa: F401
from oracle import f4, f8  # noqa: F401
from oracle.paged import paged_append, paged_gather, paged_scatter, shuffled_page_table  # noqa: F401
