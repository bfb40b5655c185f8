"""Stand-ins for the three tt-metal helpers the reference imports but does not vendor, so that the
reference's own CPU code (``palu_tt/fused.py``, ``palu_tt/convert.py``, ``palu_tt/reference.py``) can be
imported where the reference tree is mounted. Used only by ``make_golden.py`` (fixture generation) and
as a pytest plugin (``-p _ref_stubs``) to run the reference's own CPU tests against these stand-ins.

The stand-ins are this repository's oracle restatements (``oracle/palu_ref.py``): the reference's tests
tests/test_fused.py:8-73 and tests/test_convert.py pin them. ``ttnn`` is an empty module (only
``tests/conftest.py`` and ``palu_tt/device.py`` import it in the CPU files).
"""
import sys
import types


def _rope_scaling_dict(rs):
    if rs is None or isinstance(rs, dict):
        return rs
    keys = ("rope_type", "factor", "low_freq_factor", "high_freq_factor", "original_max_position_embeddings")
    return {k: getattr(rs, k) for k in keys if hasattr(rs, k)}


def install():
    from oracle import palu_ref as P

    def get_rot_transformation_mat(dhead):
        return P.rope_transformation_matrix(dhead)[None, None]

    def compute_gather_cos_sin(dhead, end, theta, rope_scaling):
        f = P.rope_freqs(dhead, theta, _rope_scaling_dict(rope_scaling))
        import torch
        ang = torch.outer(torch.arange(end).float(), f).float()
        cos = torch.cos(ang).repeat_interleave(2, dim=-1)[None, None]
        sin = torch.sin(ang).repeat_interleave(2, dim=-1)[None, None]
        return cos, sin

    def reverse_permute(tensor, n_heads, dim1, dim2):
        return P.reverse_permute(tensor, n_heads, dim1, dim2)

    mods = {}
    for name in ("ttnn", "models", "models.common", "models.common.tensor_utils", "models.tt_transformers",
                 "models.tt_transformers.tt", "models.tt_transformers.tt.rope",
                 "models.tt_transformers.tt.load_checkpoints"):
        mods[name] = sys.modules.get(name) or types.ModuleType(name)
    mods["models.common.tensor_utils"].get_rot_transformation_mat = get_rot_transformation_mat
    mods["models.tt_transformers.tt.rope"].compute_gather_cos_sin = compute_gather_cos_sin
    mods["models.tt_transformers.tt.load_checkpoints"].reverse_permute = reverse_permute
    sys.modules.update(mods)


if __name__ == "_ref_stubs":  # loaded as a pytest plugin (``-p _ref_stubs``): install before any conftest
    install()
