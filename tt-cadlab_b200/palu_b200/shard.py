"""KV-head sharding of one Palu attention layer over the GPUs of one node.

Each rank owns a contiguous block of KV heads (M-LRD) or of latent groups (G-LRD), the query heads that
attend them, their latent caches and up-projections, and the matching input-column block of
``wo_fused``. The decode op then needs no communication; the layer output is the sum over ranks of each
rank's ``o_local @ wo_block^T``, i.e. one all-reduce of ``[B, dim]`` after ``wo`` — the reference's tail
(palu_tt/attention.py:718-733: concat heads, ``wo_fused`` linear, ``tt_all_reduce``).

The helpers are pure tensor slicing plus one ``torch.distributed.all_reduce`` (NCCL on GPUs, gloo on
CPU in the tests); nothing here launches a kernel of this library.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HEAD_DIM = 128


@dataclass(frozen=True)
class KVShard:
    """The heads rank ``rank`` of ``world`` owns: ``n_kv / world`` consecutive KV heads, their query heads
    and the latent groups those heads read.

    Latent groups shard whole when ``n_groups % world == 0``. With more ranks than groups (a G-LRD layer of
    2 groups on 4 or 8 GPUs), a group's KV heads are split over ``world / n_groups`` ranks and each of them
    holds the whole group latent: its latent projection and cache are replicated, so the latent bytes each
    GPU reads stop shrinking past ``world == n_groups`` (the cap of head sharding for grouped latents; a
    sequence split with an exchange of partial softmax states would lift it)."""
    rank: int
    world: int
    n_kv: int
    n_q: int
    n_groups: int

    def __post_init__(self):
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world {self.world}")
        if self.n_q % self.n_kv or self.n_kv % self.n_groups:
            raise ValueError(f"heads do not nest: n_q {self.n_q}, n_kv {self.n_kv}, n_groups {self.n_groups}")
        if self.n_kv % self.world:
            raise ValueError(f"{self.n_kv} KV heads do not shard over {self.world} ranks")
        if self.n_groups % self.world and self.world % self.n_groups:
            raise ValueError(f"{self.n_groups} latent groups do not shard over {self.world} ranks (neither "
                             "divides the other)")

    @property
    def kv(self) -> range:
        per = self.n_kv // self.world
        return range(self.rank * per, (self.rank + 1) * per)

    @property
    def q(self) -> range:
        rep = self.n_q // self.n_kv
        return range(self.kv.start * rep, self.kv.stop * rep)

    @property
    def groups(self) -> range:
        """The latent groups this rank's KV heads read (whole groups, or the one group its heads belong to
        when a group is split over ranks)."""
        gs = self.n_kv // self.n_groups
        return range(self.kv.start // gs, (self.kv.stop - 1) // gs + 1)

    @property
    def latent_replicas(self) -> int:
        """How many ranks hold a copy of each latent group: 1 when groups shard whole."""
        return max(1, self.world // self.n_groups)


def shard_layer_inputs(shard: KVShard, q, k_lat, v_lat, u_k, wo_fused, u_v=None) -> dict:
    """Slice one layer's decode inputs to ``shard``.

    q [B, n_q, hd]; k_lat / v_lat [B, n_groups, S, r]; u_k [n_kv, r_k, ld]; u_v [n_kv, r_v, hd] or None;
    wo_fused [dim, n_q * hd] (input columns grouped by query head). Returns views (no copies)."""
    qs, ks, gs = shard.q, shard.kv, shard.groups
    return {
        "q": q[:, qs.start:qs.stop],
        "k_lat": k_lat[:, gs.start:gs.stop],
        "v_lat": v_lat[:, gs.start:gs.stop],
        "u_k": u_k[ks.start:ks.stop],
        "u_v": None if u_v is None else u_v[ks.start:ks.stop],
        "wo": wo_fused[:, qs.start * HEAD_DIM:qs.stop * HEAD_DIM],
    }


def layer_output_partial(o_local: torch.Tensor, wo_local: torch.Tensor) -> torch.Tensor:
    """This rank's share of the layer output: attention output [B, n_q_local, w] (w = r_v for absorbed V,
    128 with V rebuilt) laid into head_dim slots (``wo_fused`` keeps the first r_v columns of each head
    slot, attention.py:718-727) and multiplied by the rank's ``wo`` column block -> [B, dim] fp32. The
    product runs in ``wo_local``'s dtype (fp32 weights: fp32 throughout; bf16 weights: a bf16 GEMM)."""
    B, nq, w = o_local.shape
    if w > HEAD_DIM:
        raise ValueError(f"attention output width {w} > head_dim {HEAD_DIM}")
    slots = o_local.new_zeros(B, nq, HEAD_DIM, dtype=wo_local.dtype)
    slots[..., :w] = o_local.to(wo_local.dtype)
    return (slots.reshape(B, nq * HEAD_DIM) @ wo_local.t()).float()


def all_reduce_layer_output(partial: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the ranks' partials in place (the one collective of the sharded layer)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
