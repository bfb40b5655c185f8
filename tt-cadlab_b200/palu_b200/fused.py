"""Host side of the fused decode op: the RoPE table builders and the ``palu_sdpa_decode`` wrapper.

Mirrors the reference's ``palu_tt/fused.py`` surface (table builders fused.py:36-79) and the
``ttnn.transformer.palu_sdpa_decode`` keyword surface (called at palu_tt/attention.py:633-639 and
tests/test_palu_sdpa_device.py:84-88, 255-258). The op itself runs in libpalu_b200 (CUDA, sm_100a):

* K is rebuilt on the tensor cores from the latent (``w_rot``'s first 128 columns are ``u_k``; the
  ``u_k T`` half is not read because the pair swap is free in registers), rotated in registers from the
  packed [cos | sin] table, and scored against the rotated query;
* V is either the latent itself (absorbed into ``wo``, M-LRD) or rebuilt per head through ``u_v``
  (G-LRD), and the split-K partials are merged by a second kernel.

``rot_step``/``trans_mat`` keep the reference's meaning as the Phase 2 switch (fused.py:1-14): passed
together, the keys are rotated by chunk-relative angles (table rows 0..127, read once per CTA) and the
query by each 128-position chunk's base row, R_p = R_{128 t} R_j; their contents are not read (the B200
kernel takes the base rotation from the table row itself, so no fp32 recurrence accumulates). Without
them (Phase 1) every key is rotated by its own table row. The other Tensix-only knobs (``rot_mode``,
``table_mcast``, ``heads_per_core``, ``program_config``, ``compute_kernel_config``, ``memory_config``)
are accepted and validated the way the reference validates them and do not change the B200
computation: the B200 kernels always share a group latent across the group.
"""
from __future__ import annotations

import ctypes
import math
import os
import weakref
from typing import Optional

import torch

from palu_b200 import _lib

MAX_CHUNK = 512
HEAD_DIM = 128
ROT_MODES = ("legacy", "pack", "dst")


# ----------------------------------------------------------------------------------------------
# Table builders (host, once per model) -- fused.py:36-79
# ----------------------------------------------------------------------------------------------

def rope_transformation_matrix(head_dim: int) -> torch.Tensor:
    """[hd, hd] T such that x @ T maps each adjacent pair (x0, x1) to (-x1, x0) (fused.py:36-41)."""
    idx = torch.arange(0, head_dim, 2)
    T = torch.zeros(head_dim, head_dim)
    T[idx, idx + 1] = 1.0
    T[idx + 1, idx] = -1.0
    return T


def trans_mat_tile() -> torch.Tensor:
    """The [1, 1, 32, 32] pair-rotation tile (fused.py:44-46)."""
    return rope_transformation_matrix(32).reshape(1, 1, 32, 32)


def w_rot_from_u_k(u_k: torch.Tensor) -> torch.Tensor:
    """u_k [n_kv, r_k, hd] -> w_rot [n_kv, r_k, 2 hd] = [u_k | u_k @ T] (fused.py:49-51)."""
    return torch.cat([u_k, u_k @ rope_transformation_matrix(u_k.shape[-1]).to(u_k.device, u_k.dtype)], dim=-1)


def chunk_size(seq_len: int) -> int:
    """Largest power of two dividing seq_len, at most 512 (fused.py:54-59)."""
    assert seq_len > 0, f"chunk_size requires seq_len > 0, got {seq_len}"
    return min(MAX_CHUNK, seq_len & -seq_len)


def _llama3_freqs(f: torch.Tensor, rs: dict) -> torch.Tensor:
    factor, lo, hi = float(rs["factor"]), float(rs["low_freq_factor"]), float(rs["high_freq_factor"])
    orig = float(rs["original_max_position_embeddings"])
    wl = 2.0 * math.pi / f
    t = (orig / wl - lo) / (hi - lo)
    mid = (1.0 - t) * (f / factor) + t * f
    return torch.where(wl < orig / hi, f, torch.where(wl > orig / lo, f / factor, mid)).float()


def _scaling_dict(rope_scaling):
    if rope_scaling is None or isinstance(rope_scaling, dict):
        return rope_scaling
    keys = ("rope_type", "factor", "low_freq_factor", "high_freq_factor", "original_max_position_embeddings")
    return {k: getattr(rope_scaling, k) for k in keys if hasattr(rope_scaling, k)}


def rope_frequencies(head_dim: int, theta: float, rope_scaling=None) -> torch.Tensor:
    """fp32 inverse frequencies theta ** (-2i/d), with Llama-3.1 scaling when rope_scaling asks for it."""
    f = 1.0 / (theta ** (torch.arange(0, head_dim, 2)[: head_dim // 2].float() / head_dim))
    rs = _scaling_dict(rope_scaling)
    if rs:
        kind = rs.get("rope_type", rs.get("type", "llama3"))
        if kind != "llama3":
            raise ValueError(f"rope_scaling type {kind!r} is not supported (llama3 only)")
        f = _llama3_freqs(f, rs)
    return f


def cos_sin_tables(head_dim: int, seq_len: int, theta: float, rope_scaling=None):
    """Meta-interleaved cos / sin, fp32, each [seq_len + 513, head_dim] (fused.py:62-68)."""
    n = seq_len + MAX_CHUNK + 1
    ang = torch.outer(torch.arange(n).float(), rope_frequencies(head_dim, theta, rope_scaling)).float()
    return torch.cos(ang).repeat_interleave(2, -1).contiguous(), torch.sin(ang).repeat_interleave(2, -1).contiguous()


def cs_table(cos: torch.Tensor, sin: torch.Tensor, seq_len: int) -> torch.Tensor:
    """[seq_len, 2 hd] = [cos | sin] for positions 0..seq_len-1 (fused.py:71-73)."""
    return torch.cat([cos[:seq_len], sin[:seq_len]], dim=-1)


def rot_step_table(cos: torch.Tensor, sin: torch.Tensor, chunk: int) -> torch.Tensor:
    """[32, 2 hd] fp32 [cos(c f) | sin(c f)] rows (fused.py:76-79). Passing it (with ``trans_mat``) to
    ``palu_sdpa_decode`` selects Phase 2; the B200 kernel reads each chunk's base rotation from the table
    row itself, so the contents are not used."""
    return torch.cat([cos[chunk], sin[chunk]]).expand(32, -1).contiguous().float()


# ----------------------------------------------------------------------------------------------
# Device-side table packing (cached per cs_tab tensor)
# ----------------------------------------------------------------------------------------------

# id(cs_tab) -> (weak reference to cs_tab, its version counter, packed table). Keyed by the table tensor
# object, not its address: a freed table's memory can be reused by a new table of the same shape, and an
# address-keyed entry would then hand back the old table's values.
_PACK_CACHE: dict = {}


def pack_cs_table(cs_tab: torch.Tensor) -> torch.Tensor:
    """[.., S, 256] [cos | sin] (bf16 or fp32, CUDA) -> [S, 64] int32 rows of packed fp16 (per row 4 blocks
    of 16 frequencies: 16 cosines, then the same frequencies' sines), computed by the library's pack kernel
    and cached while the same table tensor is alive and unchanged (in-place writes bump its version)."""
    _lib.require_cuda(cs_tab)
    hit = _PACK_CACHE.get(id(cs_tab))
    if hit is not None and hit[0]() is cs_tab and hit[1] == cs_tab._version:
        return hit[2]
    t = cs_tab.reshape(-1, cs_tab.shape[-1])
    if t.stride(-1) != 1:
        t = t.contiguous()
    if t.dtype not in (torch.bfloat16, torch.float32):
        t = t.float()
    out = torch.empty(t.shape[0], 64, dtype=torch.int32, device=t.device)
    dt = _lib.PALU_F32 if t.dtype == torch.float32 else _lib.PALU_BF16
    _lib.check(_lib.load().palu_pack_cs_table(t.data_ptr(), t.stride(0), dt, out.data_ptr(), t.shape[0],
                                              _lib.stream_handle(t.device)))
    if len(_PACK_CACHE) > 256:  # one entry per live table (a model holds one per layer): drop the dead ones
        for k in [k for k, v in _PACK_CACHE.items() if v[0]() is None]:
            del _PACK_CACHE[k]
    _PACK_CACHE[id(cs_tab)] = (weakref.ref(cs_tab), cs_tab._version, out)
    return out


# ----------------------------------------------------------------------------------------------
# The op
# ----------------------------------------------------------------------------------------------

def _bf16(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is None:
        return None
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t.contiguous()


def _grid_cores(program_config) -> Optional[int]:
    grid = getattr(program_config, "compute_with_storage_grid_size", None)
    if grid is None:
        return None
    try:
        gx, gy = (grid.x, grid.y) if hasattr(grid, "x") else tuple(grid)
    except TypeError:
        return None
    return int(gx) * int(gy)


_WS_CACHE: dict = {}


def _workspace_for(d, device, need=None) -> torch.Tensor:
    """A zeroed workspace, cached per (device, size) so that repeated calls reuse it; calls that overlap on
    different streams must pass their own ``workspace``."""
    if need is None:
        need = _lib.workspace_bytes(d)
    key = (device.index if device.index is not None else torch.cuda.current_device(), need)
    ws = _WS_CACHE.get(key)
    if ws is None:
        if len(_WS_CACHE) > 8:
            _WS_CACHE.clear()
        ws = _WS_CACHE[key] = _lib.new_workspace(d, device)
    return ws


def workspace_status() -> int:
    """Read and clear the status words of the cached workspaces: 0 when no bounded device wait expired
    in any call since the last read (a nonzero value marks that call's output as invalid)."""
    st = 0
    for ws in list(_WS_CACHE.values()):
        st = max(st, _lib.read_status(ws))
    return st


def _check_status(workspace, what: str) -> None:
    """Wait for the call and raise if one of its bounded device waits expired (its output is then NaN)."""
    st = _lib.read_status(workspace)
    if st != 0:
        raise RuntimeError(f"{what}: a bounded device wait expired (status {st}); the output is invalid")


def _check_by_default() -> bool:
    return os.environ.get("PALU_CHECK_STATUS", "") not in ("", "0")


# ----------------------------------------------------------------------------------------------
# fp8 latent caches: the B200 form of the reference's block-float latent caches (bfp8_b by default,
# palu_tt/attention.py:159-169)
# ----------------------------------------------------------------------------------------------

class F8Latents:
    """A latent cache held as e4m3 codes plus one power-of-two exponent per row: ``codes`` uint8
    [..., r], ``exp`` int8 [...] (the codes' leading dims); the cached value is code * 2^exp. The
    decode op takes a pair of these where it takes bf16 caches (``palu_sdpa_decode``, ``decode``)."""

    __slots__ = ("codes", "exp")
    fmt = "f8"

    def __init__(self, codes: torch.Tensor, exp: torch.Tensor):
        if codes.dtype != torch.uint8 or exp.dtype != torch.int8:
            raise RuntimeError(f"fp8 latents need uint8 codes and int8 exponents, got {codes.dtype} / {exp.dtype}")
        if tuple(exp.shape) != tuple(codes.shape[:-1]):
            raise RuntimeError(f"fp8 latents: exponents {tuple(exp.shape)} must be the codes' leading dims "
                               f"{tuple(codes.shape[:-1])}")
        self.codes, self.exp = codes, exp

    @classmethod
    def empty(cls, *shape, device=None) -> "F8Latents":
        return cls(torch.zeros(*shape, dtype=torch.uint8, device=device),
                   torch.zeros(*shape[:-1], dtype=torch.int8, device=device))

    @property
    def shape(self):
        return self.codes.shape

    @property
    def device(self):
        return self.codes.device

    @property
    def is_cuda(self) -> bool:
        return self.codes.is_cuda

    def dim(self) -> int:
        return self.codes.dim()

    def contiguous(self) -> "F8Latents":
        return F8Latents(self.codes.contiguous(), self.exp.contiguous())

    def __getitem__(self, rows):
        """Leading-dimension selection (cache rows): a view of the same format."""
        if not isinstance(rows, slice):
            raise TypeError("low-bit latent caches index their leading (batch row) dimension by a slice")
        return type(self)(self.codes[rows], self.exp[rows])

    def dequantize(self) -> torch.Tensor:
        """float32 values code * 2^exp (host-side inspection; the decode op reads the codes directly)."""
        return self.codes.view(torch.float8_e4m3fn).float() * torch.exp2(self.exp.float()).unsqueeze(-1)


class F4Latents(F8Latents):
    """A latent cache held as e2m1 codes, two per byte (the first value in the low nibble), plus one
    power-of-two exponent per block of 16 values: ``codes`` uint8 [..., r / 2], ``exp`` int8 [..., r / 16];
    the cached value is code * 2^exp. ``shape`` reports the logical [..., r]."""

    __slots__ = ()
    fmt = "f4"

    def __init__(self, codes: torch.Tensor, exp: torch.Tensor):
        if codes.dtype != torch.uint8 or exp.dtype != torch.int8:
            raise RuntimeError(f"fp4 latents need uint8 codes and int8 exponents, got {codes.dtype} / {exp.dtype}")
        if codes.shape[-1] % 8 or tuple(exp.shape) != (*codes.shape[:-1], codes.shape[-1] // 8):
            raise RuntimeError(f"fp4 latents: exponents {tuple(exp.shape)} must be [..., r / 16] for codes "
                               f"{tuple(codes.shape)}")
        self.codes, self.exp = codes, exp

    @classmethod
    def empty(cls, *shape, device=None) -> "F4Latents":
        *lead, r = shape
        return cls(torch.zeros(*lead, r // 2, dtype=torch.uint8, device=device),
                   torch.zeros(*lead, r // 16, dtype=torch.int8, device=device))

    @property
    def shape(self):
        return torch.Size((*self.codes.shape[:-1], 2 * self.codes.shape[-1]))

    def contiguous(self) -> "F4Latents":
        return F4Latents(self.codes.contiguous(), self.exp.contiguous())

    def dequantize(self) -> torch.Tensor:
        """float32 values code * 2^exp (host-side inspection)."""
        lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], device=self.codes.device)
        c = self.codes.long()
        nib = torch.stack([c & 15, c >> 4], dim=-1).flatten(-2)
        val = lut[nib & 7] * torch.where(nib >= 8, -1.0, 1.0)
        sc = torch.exp2(self.exp.float()).repeat_interleave(16, dim=-1)
        return val * sc


def quantize_latents_f8(x: torch.Tensor) -> F8Latents:
    """bf16 latents [..., r] (CUDA) -> F8Latents (palu_quantize_latents_f8): per row, the smallest exponent
    k with max|row| <= 448 * 2^k (kept in [-120, 7]), codes = row * 2^-k rounded to nearest even e4m3."""
    _lib.require_cuda(x)
    xb = _bf16(x).contiguous()
    r = xb.shape[-1]
    out = F8Latents.empty(*xb.shape, device=xb.device)
    _lib.check(_lib.load().palu_quantize_latents_f8(xb.data_ptr(), xb.numel() // r, r, out.codes.data_ptr(),
                                                    out.exp.data_ptr(), _lib.stream_handle(xb.device)))
    return out


def quantize_latents_f4(x: torch.Tensor) -> F4Latents:
    """bf16 latents [..., r] (CUDA, r a multiple of 16) -> F4Latents (palu_quantize_latents_f4): per block of 16
    values the smallest exponent k with max|block| <= 6 * 2^k (kept in [-120, 7]), codes = block * 2^-k
    rounded to nearest even e2m1."""
    _lib.require_cuda(x)
    xb = _bf16(x).contiguous()
    r = xb.shape[-1]
    out = F4Latents.empty(*xb.shape, device=xb.device)
    _lib.check(_lib.load().palu_quantize_latents_f4(xb.data_ptr(), xb.numel() // r, r, out.codes.data_ptr(),
                                                    out.exp.data_ptr(), _lib.stream_handle(xb.device)))
    return out


def append_latents_f8(new_k, new_v, cur_pos, k_cache: F8Latents, v_cache: F8Latents) -> None:
    """Quantize one step's latents [B, n_groups, r] (bf16) into fp8 (or fp4, with F4Latents) caches at
    cur_pos[b] (palu_append_latents_f8 / _f4); rows with cur_pos outside [0, S) are skipped."""
    if k_cache.fmt != v_cache.fmt:
        raise RuntimeError("k and v caches must hold the same low-bit format")
    _lib.require_cuda(new_k, new_v, cur_pos, k_cache.codes, v_cache.codes)
    B, G, S, r_k = k_cache.shape
    r_v = v_cache.shape[3]
    d = _lib.dims(B, G, G, G, r_k, r_v, S)
    nk, nv = _bf16(new_k).contiguous(), _bf16(new_v).contiguous()
    fn = _lib.load().palu_append_latents_f4 if k_cache.fmt == "f4" else _lib.load().palu_append_latents_f8
    _lib.check(fn(
        nk.data_ptr(), nv.data_ptr(), cur_pos.to(torch.int32).contiguous().data_ptr(), k_cache.codes.data_ptr(),
        v_cache.codes.data_ptr(), k_cache.exp.data_ptr(), v_cache.exp.data_ptr(), ctypes.byref(d),
        _lib.stream_handle(nk.device)))


def decode(q, k_latent, v_latent, u_k, cs_pairs, cur_pos, *, u_k_ld=HEAD_DIM, u_v=None, scale=None,
           out=None, out_dtype=torch.bfloat16, splits=0, workspace=None, page_table=None,
           check_status=None, chunk_relative=False, _checked=False) -> torch.Tensor:
    """Low-level entry (no reference-surface validation): the arrays are already in the library's layout.

    q [B, nh, 128] bf16; k_latent [B, n_groups, S, r_k]; v_latent [B, n_groups, S, r_v]; u_k rows of
    ``u_k_ld`` elements ([n_kv, r_k, u_k_ld]); cs_pairs [>= S, 64] int32 from ``pack_cs_table``;
    cur_pos [B] int32; u_v [n_kv, r_v, 128] or None. Returns [B, nh, r_v or 128].
    Paged caches: ``page_table`` [B, blocks per row] int32 and k_latent [n_blocks, n_groups, block_size,
    r_k], v_latent [n_blocks, n_groups, block_size, r_v]; a row then holds blocks per row x block_size
    positions (palu_decode_attn_paged).
    fp8 caches: k_latent and v_latent as ``F8Latents`` (palu_decode_attn_f8; contiguous caches).
    ``check_status`` (default: the PALU_CHECK_STATUS environment variable) waits for the call and raises
    RuntimeError if a bounded device wait expired, as the reference op raises on a failed run.
    ``chunk_relative`` selects the reference op's Phase 2 RoPE (palu_set_rope_mode): key position
    p = 128 t + j rotated by table row j and the query of chunk t rotated back by row 128 t."""
    f8 = isinstance(k_latent, F8Latents)
    if f8 != isinstance(v_latent, F8Latents) or (f8 and k_latent.fmt != v_latent.fmt):
        raise RuntimeError("k_latent and v_latent must both be bf16 or both fp8 (F8Latents) or both fp4 (F4Latents)")
    if f8 and page_table is not None:
        raise RuntimeError("fp8 latent caches are contiguous (no page table)")
    if not _checked:
        _lib.require_cuda(q, u_k, cs_pairs, cur_pos, u_v, page_table,
                          *((k_latent.codes, k_latent.exp, v_latent.codes, v_latent.exp) if f8 else (k_latent, v_latent)))
    B, nh = q.shape[0], q.shape[1]
    n_groups, S, r_k = k_latent.shape[1], k_latent.shape[2], k_latent.shape[3]
    r_v = v_latent.shape[3]
    if page_table is not None:
        S = page_table.shape[1] * k_latent.shape[2]
    n_kv = u_k.shape[0]
    d = _lib.dims(B, nh, n_kv, n_groups, r_k, r_v, S, splits or _lib.env_splits())
    width = HEAD_DIM if u_v is not None else r_v
    if out is None:
        out = torch.empty(B, nh, width, dtype=out_dtype, device=q.device)
    need = _lib.workspace_bytes(d)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace_for(d, q.device, need)
    odt = _lib.PALU_F32 if out.dtype == torch.float32 else _lib.PALU_BF16
    sc = HEAD_DIM ** -0.5 if scale is None else float(scale)
    _lib.set_rope_mode(_lib.PALU_ROPE_CHUNK_RELATIVE if chunk_relative else _lib.PALU_ROPE_ABSOLUTE)
    if f8:
        fn = _lib.load().palu_decode_attn_f4 if k_latent.fmt == "f4" else _lib.load().palu_decode_attn_f8
        _lib.check(fn(
            q.data_ptr(), k_latent.codes.data_ptr(), v_latent.codes.data_ptr(), k_latent.exp.data_ptr(),
            v_latent.exp.data_ptr(), u_k.data_ptr(), int(u_k_ld), _lib.ptr(u_v), cs_pairs.data_ptr(),
            cur_pos.data_ptr(), out.data_ptr(), odt, workspace.data_ptr(), workspace.numel(), ctypes.byref(d), sc,
            _lib.stream_handle(q.device)))
    elif page_table is None:
        _lib.check(_lib.load().palu_decode_attn(
            q.data_ptr(), k_latent.data_ptr(), v_latent.data_ptr(), u_k.data_ptr(), int(u_k_ld), _lib.ptr(u_v),
            cs_pairs.data_ptr(), cur_pos.data_ptr(), out.data_ptr(), odt, workspace.data_ptr(), workspace.numel(),
            ctypes.byref(d), sc, _lib.stream_handle(q.device)))
    else:
        pg = _lib.pages(page_table, k_latent.shape[2], k_latent.shape[0])
        _lib.check(_lib.load().palu_decode_attn_paged(
            q.data_ptr(), k_latent.data_ptr(), v_latent.data_ptr(), u_k.data_ptr(), int(u_k_ld), _lib.ptr(u_v),
            cs_pairs.data_ptr(), cur_pos.data_ptr(), ctypes.byref(pg), out.data_ptr(), odt, workspace.data_ptr(),
            workspace.numel(), ctypes.byref(d), sc, _lib.stream_handle(q.device)))
    if check_status if check_status is not None else _check_by_default():
        _check_status(workspace, "palu_sdpa_decode")
    return out


def palu_sdpa_decode(q, k_latent, w_rot, cs_tab, v_latent, head_dim_v, cur_pos_tensor, *, rot_step=None,
                     trans_mat=None, u_v=None, scale=None, heads_per_core=None, rot_mode="dst", table_mcast=True,
                     program_config=None, compute_kernel_config=None, memory_config=None,
                     out_dtype=torch.bfloat16, splits=0, page_table_tensor=None, check_status=None) -> torch.Tensor:
    """B200 implementation of ``ttnn.transformer.palu_sdpa_decode`` (same positional / keyword surface).

    q [1, B, nh, 128] (rotated), k_latent [B, n_groups, S, r_k], w_rot [1, n_kv, r_k, 256],
    cs_tab [1, 1, >= S, 256], v_latent [B, n_groups, S, r_v], cur_pos_tensor [B] ints,
    u_v [1, n_kv, r_v, 128] (in-kernel V). Returns [1, B, nh, head_dim_v]. Raises RuntimeError with
    the reference's message substrings on envelope violations.

    ``page_table_tensor`` [B, blocks per row] int32 (the stock paged decode op's keyword; the paged
    variant the reference plans, HANDOFF.md:126-127): the caches are then paged, k_latent
    [n_blocks, n_groups, block_size, r_k] and v_latent [n_blocks, n_groups, block_size, r_v], and
    S = blocks per row x block_size. ``check_status`` True (or PALU_CHECK_STATUS=1 in the environment)
    waits for the call and raises RuntimeError when a bounded device wait expired."""
    if rot_mode not in ROT_MODES:
        raise RuntimeError(f"rot_mode must be one of {ROT_MODES}, got {rot_mode!r}")
    if (rot_step is None) != (trans_mat is None):
        raise RuntimeError("rot_step and trans_mat are optional together: pass both (Phase 2) or neither (Phase 1)")
    chunk = getattr(program_config, "k_chunk_size", 0) or 0
    if rot_step is None and chunk > 128:
        raise RuntimeError(f"Phase 1 (no rot_step) needs k_chunk_size <= 128, got {chunk}")
    if q.dim() != 4 or q.shape[0] != 1 or q.shape[-1] != HEAD_DIM:
        raise RuntimeError(f"q must be [1, B, nh, 128], got {tuple(q.shape)}")
    B, nh = q.shape[1], q.shape[2]
    if k_latent.dim() != 4 or v_latent.dim() != 4:
        raise RuntimeError("k_latent and v_latent must be [B, n_groups, S, r]")
    n_groups, S, r_k = k_latent.shape[1], k_latent.shape[2], k_latent.shape[3]
    r_v = v_latent.shape[3]
    if page_table_tensor is None:
        if k_latent.shape[0] != B or v_latent.shape[:3] != k_latent.shape[:3]:
            raise RuntimeError("k_latent / v_latent batch, group or sequence dims do not match q")
    else:
        pt = page_table_tensor
        if pt.dim() != 2 or pt.shape[0] != B:
            raise RuntimeError(f"page_table_tensor must be [B={B}, blocks per row], got {tuple(pt.shape)}")
        if v_latent.shape[:3] != k_latent.shape[:3]:
            raise RuntimeError("paged k_latent / v_latent block, group or block_size dims do not match")
        S = pt.shape[1] * k_latent.shape[2]
    w = w_rot.reshape(-1, *w_rot.shape[-2:]) if w_rot.dim() >= 3 else w_rot
    if w.dim() != 3 or w.shape[-1] != 2 * HEAD_DIM:
        raise RuntimeError(f"w_rot must be [1, n_kv, r_k, 256] = [u_k | u_k T], got {tuple(w_rot.shape)}")
    n_kv = w.shape[0]
    if r_k % 16 or not 16 <= r_k <= 512 or w.shape[1] != r_k:
        raise RuntimeError(f"r_k: latent width {r_k} must be a multiple of 16 in [16, 512] and match w_rot's "
                           f"{w.shape[1]} rows")
    if cs_tab.shape[-1] != 2 * HEAD_DIM or cs_tab.shape[-2] < S:
        raise RuntimeError(f"cs_tab must be [1, 1, >= {S}, 256] ([cos | sin] per position), got {tuple(cs_tab.shape)}")
    if n_kv % n_groups:
        raise RuntimeError(f"heads_per_group: {n_groups} latent heads do not divide {n_kv} KV heads (w_rot)")
    if nh % n_kv:
        raise RuntimeError(f"KV head count {n_kv} must divide the {nh} query heads")
    hpg = n_kv // n_groups
    if hpg > 1 and u_v is None:
        raise RuntimeError(f"grouped latents ({hpg} KV heads per latent) need u_v (in-kernel V)")
    if u_v is not None:
        if head_dim_v != HEAD_DIM:
            raise RuntimeError(f"head_dim_v must be {HEAD_DIM} when u_v is given, got {head_dim_v}")
        uv = u_v.reshape(-1, *u_v.shape[-2:])
        if tuple(uv.shape) != (n_kv, r_v, HEAD_DIM):
            raise RuntimeError(f"u_v must be [1, {n_kv}, {r_v}, 128], got {tuple(u_v.shape)}")
    elif head_dim_v != r_v:
        raise RuntimeError(f"head_dim_v {head_dim_v} must equal the V latent width {r_v} (absorbed V)")
    if heads_per_core is not None:
        h = int(heads_per_core)
        if h > n_kv:
            raise RuntimeError(f"heads_per_core {h} exceeds the KV head count {n_kv}")
        if h > 1 and hpg == 1:
            raise RuntimeError("heads_per_core > 1 shares a latent read and needs grouped latents")
        if h < 1 or hpg % h:
            raise RuntimeError(f"heads_per_core {h} must divide heads_per_group {hpg}")
        cores = _grid_cores(program_config)
        if h > 1 and cores is not None and B * (n_kv // h) > cores:
            raise RuntimeError(f"heads_per_core {h} needs {B * (n_kv // h)} cores, only {cores} available")
    f8 = isinstance(k_latent, F8Latents)
    if f8 != isinstance(v_latent, F8Latents) or (f8 and k_latent.fmt != v_latent.fmt):
        raise RuntimeError("k_latent and v_latent must both be bf16 or both fp8 (F8Latents) or both fp4 (F4Latents)")
    if f8:
        if page_table_tensor is not None:
            raise RuntimeError("fp8 latent caches are contiguous (no page_table_tensor)")
        if r_k > 128 or r_v > 128:
            raise RuntimeError(f"fp8 latent caches: r_k and r_v must be at most 128, got {r_k} / {r_v}")
    elif k_latent.dtype != torch.bfloat16 or v_latent.dtype != torch.bfloat16:
        raise RuntimeError("latent caches must be bf16 tensors or fp8 F8Latents")
    _lib.require_cuda(q, w_rot, cs_tab, cur_pos_tensor, u_v,
                      *((k_latent.codes, v_latent.codes) if f8 else (k_latent, v_latent)))
    pos = cur_pos_tensor.reshape(-1)
    if pos.numel() != B:
        raise RuntimeError(f"cur_pos_tensor must hold {B} positions, got {pos.numel()}")
    pos = pos.to(torch.int32).contiguous()
    wb = _bf16(w)
    pt = None if page_table_tensor is None else page_table_tensor.to(torch.int32).contiguous()
    out = decode(_bf16(q[0]), k_latent.contiguous(), v_latent.contiguous(), wb, pack_cs_table(cs_tab), pos,
                 u_k_ld=wb.shape[-1], u_v=_bf16(u_v.reshape(n_kv, r_v, HEAD_DIM)) if u_v is not None else None,
                 scale=scale, out_dtype=out_dtype, splits=splits, page_table=pt, check_status=check_status,
                 chunk_relative=rot_step is not None, _checked=True)
    return out.unsqueeze(0)


def plain_gqa_decode(q, k, v, cur_pos, *, scale=None, out_dtype=torch.bfloat16, splits=0) -> torch.Tensor:
    """Plain GQA flash-decode over already-rotated full K (the stock decode op the identity
    factorisation must match, tests/test_palu_sdpa_device.py:58-65). q [1, B, nh, 128],
    k [B, n_kv, S, 128], v [B, n_kv, S, d_v] -> [1, B, nh, d_v]."""
    _lib.require_cuda(q, k, v, cur_pos)
    B, nh = q.shape[1], q.shape[2]
    n_kv, S, d_v = k.shape[1], k.shape[2], v.shape[3]
    d = _lib.dims(B, nh, n_kv, n_kv, HEAD_DIM, d_v, S, splits or _lib.env_splits())
    out = torch.empty(B, nh, d_v, dtype=out_dtype, device=q.device)
    ws = _workspace_for(d, q.device)
    odt = _lib.PALU_F32 if out_dtype == torch.float32 else _lib.PALU_BF16
    sc = HEAD_DIM ** -0.5 if scale is None else float(scale)
    qb, kb, vb = _bf16(q[0]), _bf16(k), _bf16(v)
    _lib.check(_lib.load().palu_plain_gqa_decode(
        qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), cur_pos.to(torch.int32).contiguous().data_ptr(),
        out.data_ptr(), odt, ws.data_ptr(), ws.numel(), ctypes.byref(d), sc, _lib.stream_handle(q.device)))
    return out.unsqueeze(0)


def append_latents(new_k, new_v, cur_pos, k_cache, v_cache, page_table=None) -> None:
    """Write one step's latents [B, n_groups, r] into the caches [B, n_groups, S, r] at cur_pos[b]
    (the reference's paged_update_cache pair, attention.py:622-623). With ``page_table`` [B, blocks per
    row] int32 (paged_update_cache's keyword) the caches are paged, [n_blocks, n_groups, block_size, r]."""
    _lib.require_cuda(new_k, new_v, cur_pos, k_cache, v_cache, page_table)
    if page_table is not None:
        return _append_paged(new_k, new_v, cur_pos, k_cache, v_cache, page_table)
    B, G, S, r_k = k_cache.shape
    r_v = v_cache.shape[-1]
    if tuple(new_k.shape[-3:]) != (B, G, r_k) or tuple(new_v.shape[-3:]) != (B, G, r_v):
        raise RuntimeError(f"new latents must be [B, n_groups, r]: got {tuple(new_k.shape)}, {tuple(new_v.shape)}")
    d = _lib.dims(B, G, G, G, r_k, r_v, S)
    nk, nv = _bf16(new_k), _bf16(new_v)
    _lib.check(_lib.load().palu_append_latents(nk.data_ptr(), nv.data_ptr(),
                                               cur_pos.to(torch.int32).contiguous().data_ptr(),
                                               k_cache.data_ptr(), v_cache.data_ptr(), ctypes.byref(d),
                                               _lib.stream_handle(k_cache.device)))


def _append_paged(new_k, new_v, cur_pos, k_cache, v_cache, page_table) -> None:
    n_blocks, G, bs, r_k = k_cache.shape
    r_v = v_cache.shape[-1]
    B = page_table.shape[0]
    if tuple(new_k.shape[-3:]) != (B, G, r_k) or tuple(new_v.shape[-3:]) != (B, G, r_v):
        raise RuntimeError(f"new latents must be [B, n_groups, r]: got {tuple(new_k.shape)}, {tuple(new_v.shape)}")
    if tuple(v_cache.shape[:3]) != (n_blocks, G, bs):
        raise RuntimeError("paged k / v caches must share n_blocks, n_groups and block_size")
    pt = page_table.to(torch.int32).contiguous()
    d = _lib.dims(B, G, G, G, r_k, r_v, pt.shape[1] * bs)
    pg = _lib.pages(pt, bs, n_blocks)
    nk, nv = _bf16(new_k), _bf16(new_v)
    _lib.check(_lib.load().palu_append_latents_paged(nk.data_ptr(), nv.data_ptr(),
                                                     cur_pos.to(torch.int32).contiguous().data_ptr(), ctypes.byref(pg),
                                                     k_cache.data_ptr(), v_cache.data_ptr(), ctypes.byref(d),
                                                     _lib.stream_handle(k_cache.device)))


def rope_q_append(qkv, cos, sin, cur_pos, k_cache, v_cache, n_q, page_table=None) -> torch.Tensor:
    """One decode step's q rotation and latent append in one kernel (palu_rope_q_append; the reference's
    nlp_create_qkv_heads_decode split, rotary_embedding_llama on q and paged_update_cache x2,
    attention.py:601-625). qkv [B, n_q * 128 + n_groups * (r_k + r_v)] bf16 or fp32 (the fused
    projection, rows contiguous); cos / sin [>= S, 128] fp32; cur_pos [B] int32; caches contiguous
    [B, n_groups, S, r] or, with ``page_table``, paged [n_blocks, n_groups, block_size, r]. Returns the
    rotated q [B, n_q, 128] bf16, bit-identical to rotating in fp32 torch ops and rounding to bf16."""
    _lib.require_cuda(qkv, cos, sin, cur_pos, k_cache, v_cache, page_table)
    if qkv.dtype not in (torch.bfloat16, torch.float32) or qkv.dim() != 2 or qkv.stride(1) != 1:
        raise RuntimeError(f"qkv must be a row-major bf16 or fp32 [B, width] tensor, got {qkv.dtype} {tuple(qkv.shape)}")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or not cos.is_contiguous() or not sin.is_contiguous():
        raise RuntimeError("cos / sin must be contiguous fp32 [S, 128] tables")
    B = qkv.shape[0]
    G, r_k, r_v = k_cache.shape[1], k_cache.shape[3], v_cache.shape[3]
    if page_table is None:
        S = k_cache.shape[2]
        pg = None
    else:
        page_table = page_table.to(torch.int32).contiguous()
        S = page_table.shape[1] * k_cache.shape[2]
        pg = ctypes.byref(_lib.pages(page_table, k_cache.shape[2], k_cache.shape[0]))
    if cos.shape[0] < S or sin.shape[0] < S:
        raise RuntimeError(f"cos / sin tables of {cos.shape[0]} rows are shorter than the {S} cache positions")
    q = torch.empty(B, n_q, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device)
    d = _lib.dims(B, n_q, G, G, r_k, r_v, S)
    _lib.check(_lib.load().palu_rope_q_append(
        qkv.data_ptr(), qkv.stride(0), _lib.PALU_F32 if qkv.dtype == torch.float32 else _lib.PALU_BF16,
        cos.data_ptr(), sin.data_ptr(), cur_pos.to(torch.int32).contiguous().data_ptr(), q.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), pg, ctypes.byref(d), _lib.stream_handle(qkv.device)))
    return q


def add_rms_norm(h, delta, w, eps) -> torch.Tensor:
    """Residual add + RMSNorm of the decoder (palu_add_rms_norm): h [N, D] fp32 (contiguous) += delta
    (fp32 or bf16 [N, D], or None) in place, then returns bf16(h * rsqrt(mean(h^2) + eps) * w), w [D] fp32."""
    _lib.require_cuda(h, delta, w)
    if h.dtype != torch.float32 or not h.is_contiguous() or h.dim() != 2:
        raise RuntimeError("h must be a contiguous fp32 [N, D] tensor")
    if delta is not None and (delta.dtype not in (torch.float32, torch.bfloat16) or not delta.is_contiguous()
                              or delta.shape != h.shape):
        raise RuntimeError("delta must be a contiguous fp32 or bf16 tensor shaped like h")
    ddt = _lib.PALU_BF16 if delta is not None and delta.dtype == torch.bfloat16 else _lib.PALU_F32
    w = w.float().contiguous()
    out = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device)
    _lib.check(_lib.load().palu_add_rms_norm(h.data_ptr(), _lib.ptr(delta), ddt, w.data_ptr(), out.data_ptr(),
                                             h.shape[0], h.shape[1], float(eps), _lib.stream_handle(h.device)))
    return out


def swiglu(gu, f) -> torch.Tensor:
    """SwiGLU on the fused gate/up GEMM output (palu_swiglu): gu [N, >= 2f] bf16, gate in columns 0..f-1 and
    up in f..2f-1 -> bf16(bf16(silu(gate)) * up) [N, f]."""
    _lib.require_cuda(gu)
    if gu.dtype != torch.bfloat16 or gu.dim() != 2 or gu.stride(1) != 1:
        raise RuntimeError("gu must be a row-major bf16 [N, 2f] tensor")
    out = torch.empty(gu.shape[0], f, dtype=torch.bfloat16, device=gu.device)
    _lib.check(_lib.load().palu_swiglu(gu.data_ptr(), gu.stride(0), int(f), out.data_ptr(), gu.shape[0],
                                       _lib.stream_handle(gu.device)))
    return out
