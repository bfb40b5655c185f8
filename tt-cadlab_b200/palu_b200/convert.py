"""Palu low-rank factors -> the tensors ``PaluAttention`` loads (mirrors palu_tt/convert.py).

On-disk format (Palu's dump, read by ``load_palu_dir``; convert.py:148-199 in the reference):

* ``config.json["head_wise_ranks"]["model.layers.{i}.self_attn.{k,v}_proj"]``: one rank per *group*
  (group size 1 = M-LRD, one group per KV head; group size > 1 = G-LRD);
* ``{key}.VT.weight`` [sum of group ranks, dim]: the groups' VT blocks stacked;
* ``{key}.U.{g}.weight`` [group_size * head_dim, r_g]: group g's up-projection.

Per-layer device layout (``palu_layer_tensors``; convert.py:227-288): the latent projections sit in the
K/V slots of a fused QKV weight (``wk_lat_pad`` / ``wv_lat_pad``), ``u_k`` is in Meta (interleaved pair)
order so K comes out in the order the RoPE tables use, ``wo_fused`` absorbs U_v into the output
projection (M-LRD), and ``w_rot = [u_k | u_k T]``. Ranks are zero-padded to the layer maximum rounded up
to ``rank_multiple``, which changes nothing numerically.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional

import torch

from palu_b200.fused import w_rot_from_u_k

# Version of the tensor layout produced by palu_layer_tensors (convert.py:23 in the reference: v4 =
# group-aware layout). Part of every cache tag so a layout change never reuses stale tensors.
CONVERT_VERSION = 4


@dataclass
class PaluRuntime:
    """Runtime switches (convert.py:26-58). On B200 the fused op is the only decode path worth running,
    so ``use_fused_k`` selects it; the Tensix rebuild modes are accepted and recorded."""
    recon_len: Optional[int] = None
    check: bool = False
    use_fused_k: bool = False
    cs_recurrence: bool = False
    fused_k_chunk: Optional[int] = None
    group_heads_per_core: Optional[int] = None
    rot_mode: str = "dst"
    table_mcast: bool = True
    latent_quant_in_prefill: bool = True


@dataclass
class PaluConfig:
    """Per-model Palu description (convert.py:61-90)."""
    rank_k: List[int]
    rank_v: List[int]
    cache_id: str
    runtime: PaluRuntime = field(default_factory=PaluRuntime)
    latent_dtype: Optional[object] = None
    k_latent_dtype: Optional[object] = None
    v_latent_dtype: Optional[object] = None
    group_size: int = 1
    latent_scale: str = "balanced"
    device_tables: dict = field(default_factory=dict, repr=False, compare=False)


@dataclass
class LowRank:
    """Per-head factors W_h ~= U_h @ VT_h: k_VT [n_kv, r, dim], k_U [n_kv, hd, r] (same for v). For a group
    size > 1 every head of a group carries the group's VT and its own hd-row slice of the group's U."""
    k_VT: torch.Tensor
    k_U: torch.Tensor
    v_VT: torch.Tensor
    v_U: torch.Tensor
    group_size: int = 1

    @property
    def r_k(self) -> int:
        return self.k_VT.shape[1]

    @property
    def r_v(self) -> int:
        return self.v_VT.shape[1]


def reverse_permute(t: torch.Tensor, n_heads: int, dim1: int, dim2: int) -> torch.Tensor:
    """HF head order (first half / second half of each head) -> Meta order (adjacent pairs)."""
    return t.reshape(n_heads, 2, dim1 // n_heads // 2, dim2).transpose(1, 2).reshape(dim1, dim2)


def _unit_scale_pair(VT: torch.Tensor, U: torch.Tensor, gs: int):
    VT2, U2 = VT.clone(), U.clone()
    for g0 in range(0, U.shape[0], gs):
        heads = slice(g0, g0 + gs)
        norm = U[heads].pow(2).sum(dim=(0, 1)).sqrt()              # [r], over the group's gs*hd rows
        norm = torch.where(norm > 0, norm, torch.ones_like(norm))  # rank padding stays untouched
        U2[heads] = U[heads] * norm
        VT2[heads] = VT[heads] / norm[:, None]
    return VT2, U2


def unit_scale_lowrank(lr: LowRank) -> LowRank:
    """Rescale so every latent component has unit norm in U (convert.py:115-136): column j of U is
    multiplied and row j of VT divided by ||U[:, j]|| over the group; U @ VT is unchanged."""
    k_VT, k_U = _unit_scale_pair(lr.k_VT, lr.k_U, lr.group_size)
    v_VT, v_U = _unit_scale_pair(lr.v_VT, lr.v_U, lr.group_size)
    return LowRank(k_VT=k_VT, k_U=k_U, v_VT=v_VT, v_U=v_U, group_size=lr.group_size)


def identity_lowrank(hf_attn: Dict[str, torch.Tensor], n_kv_heads: int, head_dim: int) -> LowRank:
    """VT = the head's rows of the projection, U = I (rank = head_dim): the stock model through the
    Palu path (convert.py:139-145)."""
    eye = torch.eye(head_dim).expand(n_kv_heads, head_dim, head_dim).contiguous()
    k = hf_attn["k"].float().reshape(n_kv_heads, head_dim, -1).contiguous()
    v = hf_attn["v"].float().reshape(n_kv_heads, head_dim, -1).contiguous()
    return LowRank(k_VT=k, k_U=eye.clone(), v_VT=v, v_U=eye.clone())


def _read_palu_layer(tensors, ranks, layer, proj, n_kv_heads, head_dim, rank_multiple):
    """One projection of one layer -> per-head (VT, U, group size) (convert.py:148-172)."""
    key = f"model.layers.{layer}.self_attn.{proj}"
    group_ranks = [int(r) for r in ranks[key]]
    n_groups = len(group_ranks)
    if n_kv_heads % n_groups:
        raise ValueError(f"{key}: {n_groups} groups do not divide {n_kv_heads} KV heads")
    gs = n_kv_heads // n_groups
    r_pad = int(math.ceil(max(group_ranks) / rank_multiple) * rank_multiple)
    stacked = tensors[f"{key}.VT.weight"]
    dim = stacked.shape[1]
    VT = torch.zeros(n_kv_heads, r_pad, dim)
    U = torch.zeros(n_kv_heads, head_dim, r_pad)
    row = 0
    for g, r in enumerate(group_ranks):
        Ug = tensors[f"{key}.U.{g}.weight"]
        if tuple(Ug.shape) != (gs * head_dim, r):
            raise ValueError(f"{key}.U.{g}: shape {tuple(Ug.shape)}, expected {(gs * head_dim, r)}")
        for hh in range(gs):
            VT[g * gs + hh, :r] = stacked[row:row + r]
            U[g * gs + hh, :, :r] = Ug[hh * head_dim:(hh + 1) * head_dim]
        row += r
    return VT, U, gs


def load_palu_dir(palu_dir, n_layers: int, n_kv_heads: int, head_dim: int, rank_multiple: int = 32,
                  latent_scale: str = "balanced") -> Dict[int, LowRank]:
    """Read a Palu dump (factors-only or full HF dump with the same key names) into per-layer LowRank
    factors, ranks zero-padded per layer (convert.py:175-199)."""
    from safetensors import safe_open
    if latent_scale not in ("balanced", "unit"):
        raise ValueError(f"latent_scale must be 'balanced' or 'unit', got {latent_scale!r}")
    palu_dir = Path(palu_dir)
    ranks = json.loads((palu_dir / "config.json").read_text())["head_wise_ranks"]
    tensors = {}
    for f in sorted(palu_dir.glob("*.safetensors")):
        with safe_open(str(f), framework="pt") as sf:
            for k in sf.keys():
                if ".k_proj." in k or ".v_proj." in k:
                    tensors[k] = sf.get_tensor(k).float()
    out = {}
    for i in range(n_layers):
        k_VT, k_U, gk = _read_palu_layer(tensors, ranks, i, "k_proj", n_kv_heads, head_dim, rank_multiple)
        v_VT, v_U, gv = _read_palu_layer(tensors, ranks, i, "v_proj", n_kv_heads, head_dim, rank_multiple)
        if gk != gv:
            raise ValueError(f"layer {i}: K group size {gk} != V group size {gv}")
        lr = LowRank(k_VT, k_U, v_VT, v_U, group_size=gk)
        out[i] = unit_scale_lowrank(lr) if latent_scale == "unit" else lr
    return out


def palu_layer_tensors(hf_attn: Dict[str, torch.Tensor], lr: LowRank, n_heads: int, n_kv_heads: int,
                       head_dim: int) -> Dict[str, torch.Tensor]:
    """Per-layer tensors (convert.py:227-288):

    * ``wk_lat_pad`` / ``wv_lat_pad`` [n_kv*hd, dim]: a group's VT in the first r rows of the group's
      gs*hd slot, zeros elsewhere. Per-head full rank collapses: r_k == hd puts the factorised K weight
      (Meta order) in the slot (the stock K path), r_v == hd puts U_v @ VT_v in the slot with U_v := I.
    * ``u_k`` [n_kv, r_k, hd] = U_kᵀ in Meta order; ``u_v`` [n_kv, r_v, hd] = U_vᵀ (I on the full-rank V
      path); ``w_rot`` = [u_k | u_k T].
    * ``wo_fused`` [dim, nh*hd]: per head, the first r_v columns are wo_h @ U_v[kv] (M-LRD absorbed V);
      for grouped factors V is rebuilt per head, so wo_fused == wo.
    """
    dim = hf_attn["q"].shape[1]
    gs, r_k, r_v = lr.group_size, lr.r_k, lr.r_v
    fast_v = gs == 1 and r_v == head_dim
    u_v_eff = torch.eye(head_dim).expand(n_kv_heads, head_dim, head_dim) if fast_v else lr.v_U
    wk = torch.zeros(n_kv_heads * head_dim, dim)
    wv = torch.zeros(n_kv_heads * head_dim, dim)
    u_k = torch.zeros(n_kv_heads, r_k, head_dim)
    u_v = torch.zeros(n_kv_heads, r_v, head_dim)
    for h in range(n_kv_heads):
        slot = slice(h * head_dim, (h + 1) * head_dim)
        g, first = h // gs, h % gs == 0
        gbase = g * gs * head_dim
        if gs == 1 and r_k == head_dim:
            wk[slot] = reverse_permute(lr.k_U[h] @ lr.k_VT[h], 1, head_dim, dim)
        elif first:
            wk[gbase:gbase + r_k] = lr.k_VT[h]
        if fast_v:
            wv[slot] = lr.v_U[h] @ lr.v_VT[h]
        elif first:
            wv[gbase:gbase + r_v] = lr.v_VT[h]
        u_k[h] = reverse_permute(lr.k_U[h], 1, head_dim, r_k).T
        u_v[h] = u_v_eff[h].T
    wo = hf_attn["o"].float()
    if gs > 1:
        wo_fused = wo.clone()
    else:
        wo_fused = torch.zeros_like(wo)
        rep = n_heads // n_kv_heads
        for qh in range(n_heads):
            cols = slice(qh * head_dim, (qh + 1) * head_dim)
            wo_fused[:, qh * head_dim:qh * head_dim + r_v] = wo[:, cols] @ u_v_eff[qh // rep]
    return {"wk_lat_pad": wk, "wv_lat_pad": wv, "u_k": u_k, "u_v": u_v, "wo_fused": wo_fused,
            "w_rot": w_rot_from_u_k(u_k)}
