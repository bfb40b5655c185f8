"""The C ABI library without a GPU: it loads, exports every symbol include/palu_b200.h declares, and its
host-side planning and validation answer without touching a device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from palu_b200 import _lib, build, fused

HEADER = Path(__file__).resolve().parents[1] / "include" / "palu_b200.h"


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(palu_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_library_is_built_and_loads():
    build.build()
    lib = _lib.load()
    assert b"sm_100a" in lib.palu_version()


def test_every_declared_symbol_is_exported():
    syms = declared_symbols()
    assert set(syms) == set(_lib.EXPORTED), syms
    lib = ctypes.CDLL(str(build.build()))
    for s in syms:
        assert hasattr(lib, s), s


def _call_invalid(dims, **kw):
    lib = _lib.load()
    z = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    args = dict(q=z, k=z, v=z, u_k=z, ld=128, u_v=None, cs=z, pos=z, out=z, odt=0, ws=z, wsb=1 << 30)
    args.update(kw)
    st = lib.palu_decode_attn(args["q"], args["k"], args["v"], args["u_k"], args["ld"], args["u_v"], args["cs"],
                              args["pos"], args["out"], args["odt"], args["ws"], args["wsb"], ctypes.byref(dims),
                              1.0, None)
    return st, lib.palu_last_error().decode()


@pytest.mark.parametrize("change,needle", [
    (dict(head_dim=64), "head_dim"),
    (dict(r_k=40), "r_k"),
    (dict(r_v=24), "r_v"),
    (dict(r_k=144), "r_k"),   # above 128 widths step by 32
    (dict(r_v=288), "r_v"),   # widest supported latent is 256
    (dict(n_groups=3), "heads_per_group"),
    (dict(n_q_heads=30), "KV head count"),
    (dict(n_groups=2), "u_v"),
])
def test_envelope_errors_from_the_abi(change, needle):
    base = dict(batch=2, n_q_heads=32, n_kv_heads=8, n_groups=8, head_dim=128, r_k=64, r_v=64, max_seq=256, splits=0)
    base.update(change)
    st, msg = _call_invalid(_lib.DecodeDims(**base))
    assert st == _lib.PALU_ERR_INVALID and needle in msg, msg


def test_workspace_too_small_is_reported():
    d = _lib.dims(2, 32, 8, 8, 64, 64, 256)
    st, msg = _call_invalid(d, wsb=16)
    assert st == _lib.PALU_ERR_WORKSPACE and "workspace" in msg


def test_split_planning_is_deterministic_and_bounded():
    d = _lib.dims(32, 32, 8, 8, 64, 64, 8192)
    s = _lib.choose_splits(d)
    assert 1 <= s <= 256 and s == _lib.choose_splits(d)
    # s = CTAs per KV head for the tcgen05 kernel: partial records, one pair per (batch row, KV head) and two
    # edge pairs per CTA, each 4 heads x (64 latent floats + m + 4 quarter sums of l)
    assert _lib.workspace_bytes(d) >= (32 * 8 * 2 + 8 * s * 4) * 4 * (64 + 5) * 4
    assert _lib.choose_splits(_lib.dims(1, 32, 8, 8, 64, 64, 128)) == 1     # tiny cache: one split
    assert _lib.choose_splits(_lib.dims(2, 32, 8, 8, 64, 64, 4096, splits=9)) == 9


# The reference op's envelope messages (tests/test_palu_sdpa_device.py:115-138, 301-316, 391-399, 466-503),
# raised by the wrapper before any device work.
def _args(B=1, S=256, r_k=64, r_v=64, n_groups=4, n_kv=4, nh=16):
    q = torch.zeros(1, B, nh, 128)
    k = torch.zeros(B, n_groups, S, r_k, dtype=torch.bfloat16)
    v = torch.zeros(B, n_groups, S, r_v, dtype=torch.bfloat16)
    w = torch.zeros(1, n_kv, r_k, 256)
    cs = torch.zeros(1, 1, S, 256)
    pos = torch.zeros(B, dtype=torch.int32)
    return q, k, w, cs, v, pos


class _PC:
    def __init__(self, chunk, grid=(8, 8)):
        self.k_chunk_size = chunk
        self.compute_with_storage_grid_size = grid


def test_reference_envelope_messages():
    q, k, w, cs, v, pos = _args()
    with pytest.raises(RuntimeError, match="r_k"):
        fused.palu_sdpa_decode(q, torch.zeros(1, 4, 256, 48, dtype=torch.bfloat16), w, cs, v, 64, pos)
    with pytest.raises(RuntimeError, match="cs_tab"):
        fused.palu_sdpa_decode(q, k, w, cs[:, :, :128], v, 64, pos)
    with pytest.raises(RuntimeError, match="w_rot"):
        fused.palu_sdpa_decode(q, k, w[..., :128], cs, v, 64, pos)
    with pytest.raises(RuntimeError, match="optional together"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 64, pos, trans_mat=fused.trans_mat_tile())
    with pytest.raises(RuntimeError, match="Phase 1"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 64, pos, program_config=_PC(256))
    with pytest.raises(RuntimeError, match="rot_mode must be"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 64, pos, rot_mode="bogus")
    with pytest.raises(RuntimeError, match="head_dim_v"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 128, pos)


def test_reference_group_envelope_messages():
    q, k, w, cs, v, pos = _args(r_k=128, r_v=128, n_groups=1)
    uv = torch.zeros(1, 4, 128, 128)
    with pytest.raises(RuntimeError, match="heads_per_group"):
        fused.palu_sdpa_decode(q, torch.zeros(1, 3, 256, 128, dtype=torch.bfloat16), w, cs,
                               torch.zeros(1, 3, 256, 128, dtype=torch.bfloat16), 128, pos, u_v=uv)
    with pytest.raises(RuntimeError, match="u_v"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 128, pos)
    with pytest.raises(RuntimeError, match="head_dim_v"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 256, pos, u_v=uv)
    with pytest.raises(RuntimeError, match="heads_per_core"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 128, pos, u_v=uv, heads_per_core=3)
    with pytest.raises(RuntimeError, match="KV head count"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 128, pos, u_v=uv, heads_per_core=8)
    k2 = torch.zeros(1, 2, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="heads_per_group"):
        fused.palu_sdpa_decode(q, k2, w, cs, k2, 128, pos, u_v=uv, heads_per_core=4)
    k1 = torch.zeros(1, 4, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="grouped latents"):
        fused.palu_sdpa_decode(q, k1, w, cs, k1, 128, pos, u_v=uv, heads_per_core=2)
    q4, k4, w4, cs4, v4, pos4 = _args(B=4, r_k=128, r_v=128, n_groups=1)
    with pytest.raises(RuntimeError, match="only 4 available"):
        fused.palu_sdpa_decode(q4, k4, w4, cs4, v4, 128, pos4, u_v=uv, heads_per_core=2, program_config=_PC(128, (2, 2)))


def test_cpu_tensors_are_refused_loudly():
    q, k, w, cs, v, pos = _args()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 64, pos)


def test_decoder_step_entry_points_validate_before_any_cuda_call():
    """palu_rope_q_append, palu_add_rms_norm and palu_swiglu reject bad shapes with PALU_ERR_INVALID and a
    message naming the problem (the pointers are dummies: validation fails first)."""
    lib = _lib.load()
    z = ctypes.c_void_p(16)
    d = _lib.dims(4, 32, 8, 8, 64, 64, 256)
    width = 32 * 128 + 8 * (64 + 64)
    st = lib.palu_rope_q_append(z, width - 1, _lib.PALU_BF16, z, z, z, z, z, z, None, ctypes.byref(d), None)
    assert st == _lib.PALU_ERR_INVALID and "cannot hold" in lib.palu_last_error().decode()
    st = lib.palu_rope_q_append(z, width, 7, z, z, z, z, z, z, None, ctypes.byref(d), None)
    assert st == _lib.PALU_ERR_INVALID and "dtype" in lib.palu_last_error().decode()
    st = lib.palu_add_rms_norm(z, None, _lib.PALU_F32, z, z, 4, 4098, 1e-5, None)
    assert st == _lib.PALU_ERR_INVALID and "multiple of 4" in lib.palu_last_error().decode()
    st = lib.palu_add_rms_norm(z, z, 9, z, z, 4, 4096, 1e-5, None)
    assert st == _lib.PALU_ERR_INVALID and "dtype" in lib.palu_last_error().decode()
    st = lib.palu_swiglu(z, 100, 64, z, 4, None)
    assert st == _lib.PALU_ERR_INVALID and "2 f" in lib.palu_last_error().decode()


def test_rope_mode_setter_validates_without_a_gpu():
    """palu_set_rope_mode (the op's Phase 1 / Phase 2 switch) takes the two modes and refuses others."""
    lib = _lib.load()
    assert lib.palu_set_rope_mode(_lib.PALU_ROPE_CHUNK_RELATIVE) == _lib.PALU_OK
    assert lib.palu_set_rope_mode(_lib.PALU_ROPE_ABSOLUTE) == _lib.PALU_OK
    assert lib.palu_set_rope_mode(7) == _lib.PALU_ERR_INVALID
    assert b"RoPE mode" in lib.palu_last_error()
