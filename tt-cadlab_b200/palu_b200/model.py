"""Palu decoder on B200: a Llama-3.1-8B-shaped decoder whose attention layers are ``PaluAttention``.

The reference assembles its model from tt_transformers (palu_tt/model.py:52-95, ``build_model``) and
decodes greedily (palu_tt/generate.py:40-62: ``decode_step`` runs one token for every batch row at a
position, ``greedy`` takes the argmax). This module is the B200 counterpart of that loop around the hot
path: per layer RMSNorm -> Palu attention (latent caches + the fused decode op) -> residual -> RMSNorm ->
SwiGLU MLP -> residual; then the final RMSNorm, the LM head and the argmax.

Parallelism across ranks (one process per GPU, ``torch.distributed`` over NCCL): attention shards KV heads
(``shard.KVShard``), the MLP shards its hidden dimension (w1 / w3 rows, w2 columns); each layer
all-reduces its attention output and its MLP output, [B, dim] each. Embedding and LM head are replicated.

Weights are random (seeded), in the checkpoint layouts ``PaluAttention`` takes (HF head order for wq / wo,
``convert.LowRank`` factors); no checkpoint is read. GEMMs outside the fused op run in bf16 through torch
(cuBLAS): library GEMMs, not this package's kernels.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import torch

from palu_b200 import fused
from palu_b200.attention import LLAMA3_SCALING, PagedAttentionConfig, PaluAttention
from palu_b200.convert import LowRank
from palu_b200.shard import KVShard


@dataclass
class DecoderConfig:
    """Model shape (Llama-3.1-8B by default)."""
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 8
    ffn_dim: int = 14336
    vocab: int = 128256
    norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: Optional[dict] = field(default_factory=lambda: dict(LLAMA3_SCALING))
    head_dim: int = 128


RANK_CHOICES = (32, 48, 64, 96, 128)


def mixed_ranks(n_layers: int, seed: int, choices: Sequence[int] = RANK_CHOICES) -> List[Tuple[int, int]]:
    """Per-layer (r_k, r_v), drawn from ``choices`` with ``seed``: every KV head of a layer gets the same
    ranks (a lighter variant of the mixed-rank config, for tests)."""
    g = torch.Generator().manual_seed(seed)
    pick = lambda: int(choices[int(torch.randint(len(choices), (1,), generator=g))])
    return [(pick(), pick()) for _ in range(n_layers)]


def mixed_head_ranks(n_layers: int, n_kv_heads: int, seed: int,
                     choices: Sequence[int] = RANK_CHOICES) -> List[Tuple[List[int], List[int]]]:
    """The mixed-rank decoder config as BASELINE states it: ranks drawn from ``choices`` per layer AND per
    KV head, K and V separately -> per layer (K ranks per head, V ranks per head)."""
    g = torch.Generator().manual_seed(seed)
    pick = lambda: [int(choices[int(i)]) for i in torch.randint(len(choices), (n_kv_heads,), generator=g)]
    return [(pick(), pick()) for _ in range(n_layers)]


def padded_rank(head_ranks: Sequence[int], multiple: int = 32) -> int:
    """A layer's cache width: the largest per-head rank rounded up to ``multiple`` (load_palu_dir's padding,
    convert.py:148-199; the padded rows and columns of the factors are zero)."""
    r = max(head_ranks)
    return -(-r // multiple) * multiple


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x [..., dim] fp32 -> x / rms(x) * w, fp32 (torch's fused rms_norm: one kernel instead of four)."""
    return torch.nn.functional.rms_norm(x, (x.shape[-1],), w.float(), eps)


class PaluDecoder:
    """Decoder of ``cfg.n_layers`` layers with Palu attention, random weights from ``seed``.

    ``ranks``: per layer either (r_k, r_v) for every KV head (``mixed_ranks``) or per-head rank lists
    (K ranks, V ranks) (``mixed_head_ranks``), zero-padded per layer to ``padded_rank`` as the reference's
    loader pads them; ``world`` / ``rank``: tensor-parallel ranks (the
    default process group, when world > 1). Caches hold ``max_batch`` rows of ``max_seq`` positions.
    ``proj_dtype``: dtype of every weight matrix (bf16 for the full model; fp32 for exact comparisons).
    ``keep_source`` keeps each layer's checkpoint-layout weights (wq, wo, LowRank, full w1 / w3 / w2) in
    ``layers[i]["src"]``, for comparisons against a reference model built from the same weights.
    ``paged_attention_config``: paged latent caches in every layer (``PagedAttentionConfig``); the prefill
    and decode calls then take the batch's ``page_table`` [B, blocks per row] (tt_transformers' argument).
    """

    def __init__(self, cfg: DecoderConfig, ranks: Sequence[Tuple[int, int]], *, max_batch: int, max_seq: int,
                 seed: int = 0, device: str = "cuda", rank: int = 0, world: int = 1,
                 proj_dtype: torch.dtype = torch.bfloat16, keep_source: bool = False,
                 paged_attention_config: Optional[PagedAttentionConfig] = None, latent_dtype: str = "bf16",
                 cs_recurrence: bool = False):
        if len(ranks) != cfg.n_layers:
            raise ValueError(f"{len(ranks)} rank pairs for {cfg.n_layers} layers")
        if cfg.ffn_dim % world or cfg.n_kv_heads % world:
            raise ValueError(f"ffn_dim {cfg.ffn_dim} and n_kv_heads {cfg.n_kv_heads} must divide by world {world}")
        self.cfg, self.rank, self.world = cfg, rank, world
        self.device, self.dtype = torch.device(device), proj_dtype
        dev, dt = self.device, proj_dtype
        g = torch.Generator(device=dev).manual_seed(seed)
        D, hd = cfg.dim, cfg.head_dim

        def randn(*shape, scale):
            # drawn on the model's device from one seed: every rank of a run draws the same weights
            return (torch.randn(*shape, generator=g, device=dev) * scale).to(dt)

        self.embed = randn(cfg.vocab, D, scale=1.0)
        self.layers = []
        f_lo, f_hi = rank * cfg.ffn_dim // world, (rank + 1) * cfg.ffn_dim // world
        for (rk_spec, rv_spec) in ranks:
            wq = randn(cfg.n_heads * hd, D, scale=D ** -0.5)          # q_proj weight [n_heads * hd, dim]
            wo = randn(D, cfg.n_heads * hd, scale=(cfg.n_heads * hd) ** -0.5)  # o_proj weight [dim, n_heads * hd]
            heads_k = [int(rk_spec)] * cfg.n_kv_heads if isinstance(rk_spec, int) else [int(r) for r in rk_spec]
            heads_v = [int(rv_spec)] * cfg.n_kv_heads if isinstance(rv_spec, int) else [int(r) for r in rv_spec]
            r_k = rk_spec if isinstance(rk_spec, int) else padded_rank(heads_k)
            r_v = rv_spec if isinstance(rv_spec, int) else padded_rank(heads_v)

            def factors(head_ranks, r_pad):
                # per head: VT rows and U columns beyond the head's rank are zero (the loader's padding)
                VT = randn(cfg.n_kv_heads, r_pad, D, scale=D ** -0.5).float()
                U = randn(cfg.n_kv_heads, hd, r_pad, scale=1.0).float()
                for h, r in enumerate(head_ranks):
                    VT[h, r:] = 0
                    U[h, :, r:] = 0
                    U[h, :, :r] *= r ** -0.5
                return VT, U

            k_VT, k_U = factors(heads_k, r_k)
            v_VT, v_U = factors(heads_v, r_v)
            lr = LowRank(k_VT=k_VT, k_U=k_U, v_VT=v_VT, v_U=v_U)
            shard = KVShard(rank, world, cfg.n_kv_heads, cfg.n_heads, cfg.n_kv_heads) if world > 1 else None
            attn = PaluAttention(wq, wo, lr, cfg.n_heads, cfg.n_kv_heads, max_batch=max_batch,
                                 max_seq=max_seq, head_dim=hd, rope_theta=cfg.rope_theta,
                                 rope_scaling=cfg.rope_scaling, shard=shard, device=device, proj_dtype=dt,
                                 paged_attention_config=paged_attention_config, latent_dtype=latent_dtype,
                                 cs_recurrence=cs_recurrence)
            w1f = randn(cfg.ffn_dim, D, scale=D ** -0.5)
            w3f = randn(cfg.ffn_dim, D, scale=D ** -0.5)
            w2f = randn(D, cfg.ffn_dim, scale=cfg.ffn_dim ** -0.5)
            # w1 and w3 rows of this rank as one matrix: the gate and up projections are one GEMM
            w13 = torch.cat([w1f[f_lo:f_hi], w3f[f_lo:f_hi]])
            layer = dict(attn=attn, attn_norm=torch.ones(D, device=dev), ffn_norm=torch.ones(D, device=dev),
                         w13=w13, w1=w13[:f_hi - f_lo], w3=w13[f_hi - f_lo:], w2=w2f[:, f_lo:f_hi].contiguous())
            if keep_source:
                layer["src"] = dict(wq=wq, wo=wo, lowrank=lr, w1=w1f, w3=w3f, w2=w2f)
            self.layers.append(layer)
        self.norm = torch.ones(D, device=dev)
        self.lm_head = randn(cfg.vocab, D, scale=D ** -0.5)

    # ---- pieces -------------------------------------------------------------------------------------
    def _fused_elementwise(self) -> bool:
        """Decode steps on CUDA with bf16 weights run the residual adds, RMSNorms and SwiGLU as the library's
        fused kernels (the tensor-op path below computes the same steps, for CPU runs and fp32 weights)."""
        return self.device.type == "cuda" and self.dtype == torch.bfloat16

    def _mlp(self, L: dict, x: torch.Tensor, fp32: bool = True) -> torch.Tensor:
        """SwiGLU on this rank's hidden slice, summed over ranks: x [N, dim] -> [N, dim] fp32 (in the weights'
        dtype when ``fp32`` is False on one rank)."""
        h = x.to(self.dtype)
        gu = h @ L["w13"].t()
        f = L["w1"].shape[0]
        if self._fused_elementwise():
            a = fused.swiglu(gu, f)
        else:
            a = torch.nn.functional.silu(gu[:, :f]) * gu[:, f:]
        y = a @ L["w2"].t()
        if fp32 or self.world > 1:
            y = y.float()
        if self.world > 1:
            torch.distributed.all_reduce(y)
        return y

    def _logits(self, h: torch.Tensor) -> torch.Tensor:
        """Final norm and LM head: h [N, dim] fp32 -> logits [N, vocab] fp32."""
        return (rms_norm(h, self.norm, self.cfg.norm_eps).to(self.dtype) @ self.lm_head.t()).float()

    # ---- decode ---------------------------------------------------------------------------------------
    @torch.no_grad()
    def decode_logits(self, tokens: torch.Tensor, pos: torch.Tensor,
                      page_table: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step for every batch row (generate.py:40-50): tokens [B] at positions pos [B] ->
        logits [B, vocab] fp32. Appends the step's latents to every layer's caches."""
        h = self.embed[tokens.to(self.device)].float()
        if self._fused_elementwise():
            # residual adds, RMSNorms and the bf16 casts as one library kernel each time (fp32 residual h)
            eps = self.cfg.norm_eps
            x = fused.add_rms_norm(h, None, self.layers[0]["attn_norm"], eps)
            for i, L in enumerate(self.layers):
                # on one rank the GEMM outputs stay bf16: the norm kernel widens them while adding
                x = fused.add_rms_norm(h, L["attn"].forward_decode(x, pos, page_table=page_table, out_fp32=False),
                                       L["ffn_norm"], eps)
                nxt = self.layers[i + 1]["attn_norm"] if i + 1 < len(self.layers) else self.norm
                x = fused.add_rms_norm(h, self._mlp(L, x, fp32=False), nxt, eps)
            return (x @ self.lm_head.t()).float()
        for L in self.layers:
            h = h + L["attn"].forward_decode(rms_norm(h, L["attn_norm"], self.cfg.norm_eps), pos,
                                                  page_table=page_table)
            h = h + self._mlp(L, rms_norm(h, L["ffn_norm"], self.cfg.norm_eps))
        return self._logits(h)

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor,
                    page_table: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Greedy next tokens [B] (generate.py:53-62)."""
        return self.decode_logits(tokens, pos, page_table).argmax(-1)

    # ---- prefill --------------------------------------------------------------------------------------
    @torch.no_grad()
    def prefill_logits(self, tokens: torch.Tensor, page_table: Optional[torch.Tensor] = None,
                       row0: int = 0) -> torch.Tensor:
        """Prompt tokens [B, P] at positions 0..P-1 (cache rows row0 .. row0 + B - 1): fills every layer's
        caches and returns the logits of the last prompt position [B, vocab] fp32 (generate.py:28-37)."""
        tokens = tokens.to(self.device)
        B, P = tokens.shape
        h = self.embed[tokens].float()                                   # [B, P, dim]
        for L in self.layers:
            h = h + L["attn"].forward_prefill(rms_norm(h, L["attn_norm"], self.cfg.norm_eps), None, row0,
                                              page_table=page_table)
            h = h + self._mlp(L, rms_norm(h, L["ffn_norm"], self.cfg.norm_eps).reshape(B * P, -1)).view(B, P, -1)
        return self._logits(h[:, -1])

    # ---- CUDA graph of one decode step ------------------------------------------------------------------
    def capture_decode(self, batch: int, page_table: Optional[torch.Tensor] = None) -> "DecodeGraph":
        """A CUDA graph of ``decode_step`` for ``batch`` rows: set ``graph.tokens`` / ``graph.pos`` (and, with
        paged caches, ``graph.page_table``, captured from ``page_table``) and call ``graph.replay()``; the
        next tokens land in ``graph.next``. The warm-up call (which builds the library's packed tables and
        workspaces outside the capture) runs every row at position -1, which the append and the decode op
        skip, so it leaves the caches as they were."""
        return DecodeGraph(self, batch, page_table)


class DecodeGraph:
    """One captured decode step (see ``PaluDecoder.capture_decode``)."""

    def __init__(self, model: PaluDecoder, batch: int, page_table: Optional[torch.Tensor] = None):
        dev = model.device
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.pos = torch.full((batch,), -1, dtype=torch.int32, device=dev)
        # the table the graph reads (rewrite it in place between replays as blocks are allocated)
        self.page_table = None if page_table is None else page_table.to(dev, torch.int32).contiguous().clone()
        self.next = model.decode_step(self.tokens, self.pos, self.page_table)  # warm-up: position -1 writes nothing
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.next = model.decode_step(self.tokens, self.pos, self.page_table)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.next
