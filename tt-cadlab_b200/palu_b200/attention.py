"""Palu attention layer on B200: the decode path of palu_tt/attention.py's ``PaluAttention``.

Per decode step (attention.py:585-733):

1. q = x @ wq (Meta head order), rotated at each row's position (``rotary_embedding_llama``);
2. the step's latents h_k = x @ VT_k, h_v = x @ VT_v, one per latent group, appended to the caches at
   cur_pos (two ``paged_update_cache`` calls, attention.py:612-625 -> ``fused.append_latents``);
3. the fused op (``ttnn.transformer.palu_sdpa_decode``, attention.py:633-639 -> ``fused.palu_sdpa_decode``):
   K rebuilt from the latent cache, RoPE, online softmax; V absorbed into ``wo_fused`` (M-LRD) or
   rebuilt per head from the group latent (G-LRD);
4. heads concatenated into their head_dim slots, ``@ wo_fused^T``, and with KV heads sharded over ranks,
   one all-reduce of [B, dim] (attention.py:718-733).

``forward_prefill`` fills the caches for a prompt and returns the prompt's attention output with torch
SDPA on the rebuilt K / V (the reference runs its prefill on full K / V too, attention.py:382-516).

Paged caches: with ``paged_attention_config`` (tt_transformers' argument, which the reference accepts and
asserts is None, attention.py:83-86) the caches are [max_num_blocks, n_groups, block_size, r] and the
forward methods take the ``page_table`` [B, blocks per row] int32 (attention.py:585-586); the decode
step then runs palu_decode_attn_paged / palu_append_latents_paged.

Weights follow the reference's layout (palu_tt/convert.py): q / K in Meta (interleaved-pair) head order
so they meet the interleaved RoPE tables, ``u_k`` = U_kᵀ in Meta order, ``wo_fused`` absorbing U_v.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Optional

import torch

from palu_b200 import fused
from palu_b200.convert import LowRank, reverse_permute
from palu_b200.shard import KVShard, all_reduce_layer_output, layer_output_partial

LLAMA3_SCALING = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                  "original_max_position_embeddings": 8192}


class Mode(str, Enum):
    """Forward mode (tt_transformers' ``Mode``, which the reference's ``forward`` dispatches on,
    attention.py:735-740). Plain strings "decode" / "prefill" are accepted too."""
    DECODE = "decode"
    PREFILL = "prefill"


@dataclass
class PagedAttentionConfig:
    """Paged cache geometry (the fields of tt_transformers' PagedAttentionConfig)."""
    block_size: int = 64
    max_num_blocks: int = 2048


class PaluAttention:
    """One attention layer with per-head (M-LRD) or per-group (G-LRD) latent K/V caches.

    wq, wo: [dim, n_heads * head_dim] in HF order (as in the checkpoint); ``lowrank``: the layer's
    factors (``convert.LowRank``: k_VT [n_kv, r_k, dim], k_U [n_kv, head_dim, r_k], v_VT, v_U, with
    G-LRD groups repeated per head as ``load_palu_dir`` returns them). ``shard`` selects this rank's
    KV heads (``shard.KVShard``); the layer output is then all-reduced over the default process group.
    ``proj_dtype`` is the dtype of the q / latent / output projections: fp32 (default) keeps the checkpoint
    values exact, bf16 halves their weight traffic (the reference's device weights are bf16).
    """

    def __init__(self, wq: torch.Tensor, wo: torch.Tensor, lowrank: LowRank, n_heads: int, n_kv_heads: int, *,
                 max_batch: int, max_seq: int, head_dim: int = 128, rope_theta: float = 500000.0,
                 rope_scaling: Optional[dict] = LLAMA3_SCALING, shard: Optional[KVShard] = None,
                 device: str = "cuda", cache_dtype: torch.dtype = torch.bfloat16,
                 proj_dtype: torch.dtype = torch.float32,
                 paged_attention_config: Optional[PagedAttentionConfig] = None, latent_dtype: str = "bf16",
                 cs_recurrence: bool = False):
        if head_dim != fused.HEAD_DIM:
            raise RuntimeError(f"head_dim must be {fused.HEAD_DIM}, got {head_dim}")
        gs = lowrank.group_size
        n_groups = n_kv_heads // gs
        self.shard = shard or KVShard(0, 1, n_kv_heads, n_heads, n_groups)
        sh = self.shard
        self.n_heads, self.n_kv_heads, self.head_dim, self.group_size = n_heads, n_kv_heads, head_dim, gs
        self.nh, self.nkv, self.ng = len(sh.q), len(sh.kv), len(sh.groups)  # local counts
        self.max_batch, self.max_seq, self.device = max_batch, max_seq, torch.device(device)
        self.r_k, self.r_v = lowrank.r_k, lowrank.r_v
        self.grouped = gs > 1
        dim = wq.shape[1]
        self.dim = dim
        dev, bf = self.device, torch.bfloat16

        qs, ks = sh.q, sh.kv
        wq_meta = reverse_permute(wq.float(), n_heads, n_heads * head_dim, dim)
        # Projections in proj_dtype (fp32 by default: the checkpoint values are exact in it, and the only
        # rounding left on the path is the bf16 of q and of the cached latents, as on the device).
        f32 = proj_dtype
        self.proj_dtype = proj_dtype
        self.wq = wq_meta[qs.start * head_dim:qs.stop * head_dim].to(dev, f32)           # [nh*hd, dim]
        # one latent projection per local group: the group's first head carries its VT (convert.py:266-276)
        first = [g * gs for g in sh.groups]
        self.wk_lat = torch.cat([lowrank.k_VT[h].float() for h in first]).to(dev, f32)  # [ng*r_k, dim]
        self.wv_lat = torch.cat([lowrank.v_VT[h].float() for h in first]).to(dev, f32)  # [ng*r_v, dim]
        # one GEMM per decode step for q and both latents: wq, wk_lat, wv_lat become views of w_qkv
        self.w_qkv = torch.cat([self.wq, self.wk_lat, self.wv_lat])
        nq_rows, nk_rows = self.wq.shape[0], self.wk_lat.shape[0]
        self.wq, self.wk_lat, self.wv_lat = (self.w_qkv[:nq_rows], self.w_qkv[nq_rows:nq_rows + nk_rows],
                                             self.w_qkv[nq_rows + nk_rows:])
        u_k = torch.stack([reverse_permute(lowrank.k_U[h].float(), 1, head_dim, self.r_k).T for h in ks])
        self.u_k = u_k.to(dev, bf)                                                        # [nkv, r_k, hd]
        self.w_rot = fused.w_rot_from_u_k(u_k)[None].to(dev, bf)                          # [1, nkv, r_k, 2hd]
        # fp32 copies of U for the prefill path (K / V rebuilt over the prompt)
        self._u_k32 = u_k.to(dev)
        self._u_v32 = torch.stack([lowrank.v_U[h].float().T for h in ks]).to(dev)          # [nkv, r_v, hd]
        wo = wo.float()
        cols = slice(qs.start * head_dim, qs.stop * head_dim)
        if self.grouped:
            self.u_v = self._u_v32[None].to(bf)                                            # [1, nkv, r_v, hd]
            self.wo = wo[:, cols].to(dev, f32)
            self.head_dim_v = head_dim
        else:
            # M-LRD: the attention output stays in latent space; U_v folds into wo (convert.py:278-286)
            rep = n_heads // n_kv_heads
            wf = torch.zeros(dim, self.nh * head_dim)
            for i, qh in enumerate(qs):
                blk = wo[:, qh * head_dim:(qh + 1) * head_dim] @ lowrank.v_U[qh // rep].float()
                wf[:, i * head_dim:i * head_dim + self.r_v] = blk
            self.u_v = None
            self.wo = wf.to(dev, f32)
            self.head_dim_v = self.r_v
        # M-LRD: only the first r_v columns of each head slot of wo_fused are nonzero; the decode step
        # multiplies the [B, nh * r_v] attention output by those columns alone
        self.wo_compact = (None if self.grouped else
                           self.wo.view(dim, self.nh, head_dim)[:, :, :self.r_v].reshape(dim, self.nh * self.r_v)
                           .contiguous())

        self.paged = paged_attention_config
        # Latent-cache format (the reference's latent_dtype: bfp8 by default, bfp4 per side, attention.py:
        # 159-169): "bf16", or the B200 block-scaled forms "f8" (e4m3) and "f4" (e2m1), contiguous caches.
        if latent_dtype not in ("bf16", "f8", "f4"):
            raise RuntimeError(f"latent_dtype must be bf16, f8 or f4, got {latent_dtype!r}")
        if latent_dtype != "bf16" and paged_attention_config is not None:
            raise RuntimeError("low-bit latent caches are contiguous (no paged_attention_config)")
        self.latent_dtype = latent_dtype
        # a paged row holds whole blocks: the tables cover max_seq rounded up to a block
        tab_len = max_seq if self.paged is None else -(-max_seq // self.paged.block_size) * self.paged.block_size
        cos, sin = fused.cos_sin_tables(head_dim, tab_len, rope_theta, rope_scaling)
        self.cos, self.sin = cos.to(dev), sin.to(dev)                                      # fp32 [>= S, hd]
        self.cs_tab = fused.cs_table(cos, sin, tab_len)[None, None].to(dev, bf)           # [1, 1, S, 2hd]
        # The reference's PaluRuntime.cs_recurrence (convert.py:36; attention.py:74-75, 152): the op's Phase 2,
        # chunk-relative key angles with the query rotated per chunk, switched on by rot_step / trans_mat.
        self.phase2 = {}
        if cs_recurrence:
            self.phase2 = {"rot_step": fused.rot_step_table(cos, sin, min(128, tab_len - 1)).to(dev),
                           "trans_mat": fused.trans_mat_tile()}
        if latent_dtype != "bf16":
            cls = fused.F4Latents if latent_dtype == "f4" else fused.F8Latents
            self.k_cache = cls.empty(max_batch, self.ng, max_seq, self.r_k, device=dev)
            self.v_cache = cls.empty(max_batch, self.ng, max_seq, self.r_v, device=dev)
        elif self.paged is None:
            self.k_cache = torch.zeros(max_batch, self.ng, max_seq, self.r_k, dtype=cache_dtype, device=dev)
            self.v_cache = torch.zeros(max_batch, self.ng, max_seq, self.r_v, dtype=cache_dtype, device=dev)
        else:
            nb, bs = self.paged.max_num_blocks, self.paged.block_size
            self.k_cache = torch.zeros(nb, self.ng, bs, self.r_k, dtype=cache_dtype, device=dev)
            self.v_cache = torch.zeros(nb, self.ng, bs, self.r_v, dtype=cache_dtype, device=dev)
        self.scale = head_dim ** -0.5
        # The two device ops of a decode step (the CUDA library; the tests substitute CPU models here to
        # check the layer algebra on a machine without a GPU).
        self.append_op = fused.append_latents if latent_dtype == "bf16" else fused.append_latents_f8
        self.attend_op = fused.palu_sdpa_decode

    # ---- RoPE on q (Meta-interleaved pairs, rotary_embedding_llama) ----------------------------------
    def _rotate(self, t: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """t [..., n, hd] fp32 at positions pos (broadcast over the head axis): pairs (2j, 2j+1) rotate by
        pos * f_j."""
        c = self.cos[pos].unsqueeze(-2)
        s = self.sin[pos].unsqueeze(-2)
        tr = torch.stack([-t[..., 1::2], t[..., 0::2]], dim=-1).flatten(-2)  # (-x1, x0) per pair
        return t * c + tr * s

    def _out(self, attn: torch.Tensor, fp32: bool = True) -> torch.Tensor:
        """[B, nh_local, w] attention output -> [B, dim] layer output (summed over ranks), fp32, or in the
        projection dtype when ``fp32`` is False on one rank."""
        if self.wo_compact is not None and attn.shape[-1] == self.r_v:
            y = attn.reshape(attn.shape[0], -1).to(self.wo_compact.dtype) @ self.wo_compact.t()
            if fp32 or self.shard.world > 1:
                y = y.float()
        else:
            y = layer_output_partial(attn, self.wo)
        return all_reduce_layer_output(y) if self.shard.world > 1 else y

    def _fused_prep(self, qkv: torch.Tensor) -> bool:
        """Whether the step's q rotation and latent append run as the library's one fused kernel: on CUDA,
        with bf16 caches and the library's append (tests that substitute CPU models of the device ops take
        the tensor-op path, which computes the same values)."""
        return (qkv.is_cuda and self.append_op is fused.append_latents and self.latent_dtype == "bf16"
                and self.k_cache.dtype == torch.bfloat16
                and qkv.dtype in (torch.bfloat16, torch.float32))

    def _check_pages(self, page_table: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        if (page_table is None) != (self.paged is None):
            raise RuntimeError("page_table is required with paged caches and refused without them")
        if page_table is None:
            return None
        if page_table.shape[-1] * self.paged.block_size < self.max_seq:
            raise RuntimeError(f"page_table rows of {page_table.shape[-1]} blocks of {self.paged.block_size} "
                               f"cannot hold max_seq {self.max_seq}")
        return page_table.to(self.device, torch.int32).contiguous()

    @torch.no_grad()
    def forward(self, x: torch.Tensor, current_pos: Optional[torch.Tensor] = None, rot_mats=None, user_id: int = 0,
                mode=Mode.DECODE, page_table: Optional[torch.Tensor] = None, chunk_page_table=None,
                chunk_start_idx=None, kv_cache=None) -> torch.Tensor:
        """The reference layer's entry point (attention.py:735-740): ``mode`` PREFILL runs
        ``forward_prefill``, DECODE ``forward_decode``, with the same arguments."""
        m = Mode(mode.value if isinstance(mode, Enum) else str(mode).lower())
        if m is Mode.PREFILL:
            return self.forward_prefill(x, rot_mats, user_id, page_table=page_table, chunk_page_table=chunk_page_table,
                                        chunk_start_idx=chunk_start_idx, kv_cache=kv_cache)
        return self.forward_decode(x, current_pos, rot_mats, page_table=page_table, kv_cache=kv_cache)

    @torch.no_grad()
    def forward_decode(self, x: torch.Tensor, current_pos: torch.Tensor, rot_mats=None,
                       page_table: Optional[torch.Tensor] = None, kv_cache=None, *,
                       out_fp32: bool = True) -> torch.Tensor:
        """The reference's ``forward_decode(x, current_pos, rot_mats=None, page_table=None, kv_cache=None)``
        (attention.py:585). x [B, dim] or [1, 1, B, dim]; current_pos [B] ints (each row's position; < 0
        skips the row); ``rot_mats`` is accepted and not used: q is rotated at ``current_pos`` from the
        layer's own tables inside the fused q-rotation kernel. page_table [B, blocks per row] with paged
        caches; ``kv_cache`` must be None (the layer owns its latent caches, as the reference asserts).
        Returns the layer output in x's layout, fp32 (or, with ``out_fp32`` False on one rank, the output
        GEMM's dtype, for a consumer that widens it itself)."""
        if kv_cache is not None:
            raise RuntimeError("kv_cache must be None: the layer owns its latent caches (attention.py:586)")
        shape4 = x.dim() == 4
        xb = (x.reshape(-1, x.shape[-1]) if shape4 else x).to(self.device)
        B = xb.shape[0]
        if B > self.max_batch:
            raise RuntimeError(f"batch {B} exceeds the cache's {self.max_batch} rows")
        pos = current_pos.to(self.device, torch.int32).reshape(B)
        # x arrives in fp32, or already in the projection dtype (the decoder's fused norm writes bf16)
        xp = xb if xb.dtype == self.proj_dtype else xb.float().to(self.proj_dtype)
        qkv = xp @ self.w_qkv.T
        pt = self._check_pages(page_table)
        if pt is None:
            kc, vc, paged = self.k_cache[:B], self.v_cache[:B], {}
        else:
            pt = pt[:B, :(self.max_seq + self.paged.block_size - 1) // self.paged.block_size]
            kc, vc, paged = self.k_cache, self.v_cache, {"page_table": pt}
        if self._fused_prep(qkv):
            # q rotation + latent append in one kernel (attention.py:601-625), bit-identical to the path below
            q = fused.rope_q_append(qkv, self.cos, self.sin, pos, kc, vc, self.nh, **paged)
        else:
            nq, nk = self.nh * self.head_dim, self.ng * self.r_k
            q = qkv[:, :nq].float().view(B, self.nh, self.head_dim)
            q = self._rotate(q, pos.clamp(min=0).long()).to(torch.bfloat16)
            cdt = self.k_cache.dtype if self.latent_dtype == "bf16" else torch.bfloat16
            k_new = qkv[:, nq:nq + nk].reshape(B, self.ng, self.r_k).to(cdt)
            v_new = qkv[:, nq + nk:].reshape(B, self.ng, self.r_v).to(cdt)
            self.append_op(k_new, v_new, pos, kc, vc, **paged)
        # bf16 projections take the op's output in bf16: the rounding _out's input cast would apply anyway
        odt = torch.bfloat16 if self.proj_dtype == torch.bfloat16 else torch.float32
        attn = self.attend_op(q[None], kc, self.w_rot, self.cs_tab, vc, self.head_dim_v, pos, u_v=self.u_v,
                              scale=self.scale, out_dtype=odt, **self.phase2,
                              **({"page_table_tensor": pt} if pt is not None else {}))[0]
        y = self._out(attn, out_fp32)
        return y.view(1, 1, B, self.dim) if shape4 else y

    @torch.no_grad()
    def forward_prefill(self, x: torch.Tensor, rot_mats=None, user_id: int = 0,
                        page_table: Optional[torch.Tensor] = None, chunk_page_table=None, chunk_start_idx=None,
                        kv_cache=None) -> torch.Tensor:
        """The reference's ``forward_prefill(x_11SH, rot_mats, user_id=0, page_table=None, ...)``
        (attention.py:382). Prompt of P tokens at positions 0..P-1: x [B, P, dim] (cache rows user_id ..
        user_id + B - 1, so a long batch can be prefilled a few rows at a time), or [1, 1, P, dim] for cache
        row ``user_id`` (the reference's per-user prefill). ``rot_mats`` is accepted
        and not used (the layer rotates from its own tables); chunked prefill (``chunk_page_table``,
        ``chunk_start_idx``) and an external ``kv_cache`` are not supported. Writes the prompt's latents into
        the caches and returns its causal attention output (fp32, x's layout) computed with torch SDPA on K
        and V rebuilt from the cached (bf16) latents. With paged caches, ``page_table`` is the whole batch's
        table [max_batch or B, blocks per row] and the rows' latents go through it (paged_fill_cache)."""
        if chunk_page_table is not None or chunk_start_idx is not None or kv_cache is not None:
            raise RuntimeError("chunked prefill and an external kv_cache are not supported")
        shape4 = x.dim() == 4
        xb = (x.reshape(1, x.shape[-2], x.shape[-1]) if shape4 else x).to(self.device, torch.float32)
        B, P, _ = xb.shape
        rows = slice(user_id, user_id + B)
        if P > self.max_seq or rows.stop > self.max_batch:
            raise RuntimeError(f"prompt of {P} tokens / cache rows {rows} exceed the cache")
        xp = xb.to(self.proj_dtype)
        lat_k = (xp @ self.wk_lat.T).float().view(B, P, self.ng, self.r_k).transpose(1, 2)
        lat_v = (xp @ self.wv_lat.T).float().view(B, P, self.ng, self.r_v).transpose(1, 2)
        pt = self._check_pages(page_table)
        if self.latent_dtype != "bf16":
            # quantize the prompt's rows into the low-bit caches; attention runs on the values they hold
            quant = fused.quantize_latents_f4 if self.latent_dtype == "f4" else fused.quantize_latents_f8
            ck_q, cv_q = quant(lat_k.to(torch.bfloat16)), quant(lat_v.to(torch.bfloat16))
            for cache, qd in ((self.k_cache, ck_q), (self.v_cache, cv_q)):
                cache.codes[rows, :, :P] = qd.codes
                cache.exp[rows, :, :P] = qd.exp
            ck, cv = ck_q.dequantize(), cv_q.dequantize()
        elif pt is None:
            self.k_cache[rows, :, :P] = lat_k.to(self.k_cache.dtype)
            self.v_cache[rows, :, :P] = lat_v.to(self.v_cache.dtype)
            ck, cv = self.k_cache[rows, :, :P], self.v_cache[rows, :, :P]
        else:
            # position t of a row: row t % bs of block table[row, t // bs]; [B, P] indices
            bs = self.paged.block_size
            t = torch.arange(P, device=self.device)
            blk = pt[rows][:, t // bs].long()
            off = (t % bs)[None].expand(B, P)
            self.k_cache[blk, :, off] = lat_k.transpose(1, 2).to(self.k_cache.dtype)
            self.v_cache[blk, :, off] = lat_v.transpose(1, 2).to(self.v_cache.dtype)
            ck, cv = self.k_cache[blk, :, off].transpose(1, 2), self.v_cache[blk, :, off].transpose(1, 2)
        gs_local = self.nkv // self.ng
        rep = self.nh // self.nkv
        lk = ck.float().repeat_interleave(gs_local, dim=1)                               # [B, nkv, P, r_k]
        lv = cv.float().repeat_interleave(gs_local, dim=1)
        K = torch.einsum("bhpr,hrd->bhpd", lk, self._u_k32)
        V = torch.einsum("bhpr,hrd->bhpd", lv, self._u_v32) if self.grouped else lv
        p_idx = torch.arange(P, device=self.device)
        K = self._rotate(K.transpose(1, 2), p_idx[None]).transpose(1, 2)                # [B, nkv, P, hd]
        q = (xp @ self.wq.T).float().view(B, P, self.nh, self.head_dim)
        q = self._rotate(q, p_idx[None]).transpose(1, 2)                               # [B, nh, P, hd]
        attn = torch.nn.functional.scaled_dot_product_attention(
            q, K.repeat_interleave(rep, dim=1), V.repeat_interleave(rep, dim=1), is_causal=True, scale=self.scale)
        attn = attn.transpose(1, 2).reshape(B * P, self.nh, -1)
        y = self._out(attn).view(B, P, self.dim)
        return y.view(1, 1, P, self.dim) if shape4 else y
