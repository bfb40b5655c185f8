"""fp32 CPU restatement of the reference's decode-attention model (TEST INFRASTRUCTURE ONLY).

Every function cites the reference line it restates (paths inside the ryankert01/tt-cadlab tree).
Three helpers come from tt-metal, which the reference imports but does not vendor
(``third_party/tt-metal`` at the ``palu-sdpa`` branch off v0.78.0; absent from the mounted tree):

* ``get_rot_transformation_mat`` (fused.py:30, 36-46): restated as ``rope_transformation_matrix``;
  pinned exactly by the reference's tests/test_fused.py:8-17.
* ``compute_gather_cos_sin`` (fused.py:31, 62-68): restated as ``cos_sin_tables`` from the published
  RoPE definition (inverse frequencies ``theta ** (-2i/d)``, fp32 angles ``t * f``) with the published
  Llama-3.1 frequency scaling; pinned structurally by tests/test_fused.py:33-73 and numerically
  against HF ``LlamaRotaryEmbedding`` (the frequencies the layer oracle reference.py:22,41-46 uses).
* ``reverse_permute`` (convert.py:13): restated; pinned by tests/test_convert.py:18-28,144-160,388-412.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

MAX_CHUNK = 512  # fused.py:33


# ----------------------------------------------------------------------------------------------
# RoPE helpers (fused.py:36-79)
# ----------------------------------------------------------------------------------------------

def rope_transformation_matrix(head_dim: int) -> torch.Tensor:
    """[hd, hd] pair rotation T with (x @ T) mapping each adjacent pair (x0, x1) to (-x1, x0).

    Restates fused.py:36-41 (tt-metal ``get_rot_transformation_mat``)."""
    assert head_dim % 2 == 0
    T = torch.zeros(head_dim, head_dim)
    even = torch.arange(0, head_dim, 2)
    T[even, even + 1] = 1.0       # (xT)[2j+1] = x[2j]
    T[even + 1, even] = -1.0      # (xT)[2j]   = -x[2j+1]
    return T


def trans_mat_tile() -> torch.Tensor:
    """[1, 1, 32, 32] tile of T (fused.py:44-46)."""
    return rope_transformation_matrix(32)[None, None]


def w_rot_from_u_k(u_k: torch.Tensor) -> torch.Tensor:
    """[n_kv, r_k, hd] -> [n_kv, r_k, 2 hd] = [u_k | u_k @ T] (fused.py:49-51)."""
    return torch.cat([u_k, u_k @ rope_transformation_matrix(u_k.shape[-1])], dim=-1)


def chunk_size(seq_len: int) -> int:
    """Largest power of two dividing seq_len, capped at 512 (fused.py:54-59)."""
    assert seq_len > 0
    return min(MAX_CHUNK, seq_len & -seq_len)


def llama3_scale_freqs(freqs: torch.Tensor, factor: float, low_freq_factor: float,
                       high_freq_factor: float, original_max_position_embeddings: int) -> torch.Tensor:
    """The published Llama-3.1 RoPE frequency scaling, elementwise in fp32.

    Wavelengths shorter than ``orig / high`` keep their frequency, wavelengths longer than
    ``orig / low`` are divided by ``factor``, and the band between is a linear blend in
    ``orig / wavelength``."""
    f = freqs.float()
    wavelen = (2.0 * math.pi) / f
    lo_wl = original_max_position_embeddings / low_freq_factor
    hi_wl = original_max_position_embeddings / high_freq_factor
    smooth = (original_max_position_embeddings / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
    blended = (1.0 - smooth) * (f / factor) + smooth * f
    out = torch.where(wavelen < hi_wl, f, torch.where(wavelen > lo_wl, f / factor, blended))
    return out.float()


def rope_freqs(head_dim: int, theta: float, rope_scaling: Optional[dict]) -> torch.Tensor:
    """Inverse frequencies ``1 / theta ** (2i / d)`` (fp32), llama3-scaled when ``rope_scaling`` says so."""
    f = 1.0 / (theta ** (torch.arange(0, head_dim, 2)[: head_dim // 2].float() / head_dim))
    if rope_scaling:
        kind = rope_scaling.get("rope_type", rope_scaling.get("type", "llama3"))
        assert kind == "llama3", f"only llama3 rope scaling is restated, got {kind!r}"
        f = llama3_scale_freqs(f, float(rope_scaling["factor"]), float(rope_scaling["low_freq_factor"]),
                               float(rope_scaling["high_freq_factor"]),
                               int(rope_scaling["original_max_position_embeddings"]))
    return f


def cos_sin_tables(head_dim: int, seq_len: int, theta: float, rope_scaling: Optional[dict]):
    """Meta-interleaved cos/sin, fp32, each [seq_len + 513, head_dim] (fused.py:62-68).

    Angles are the fp32 products ``t * f``; each frequency fills two adjacent columns."""
    n = seq_len + MAX_CHUNK + 1
    f = rope_freqs(head_dim, theta, rope_scaling)
    ang = torch.outer(torch.arange(n).float(), f).float()
    cos = torch.cos(ang).repeat_interleave(2, dim=-1)
    sin = torch.sin(ang).repeat_interleave(2, dim=-1)
    return cos.contiguous(), sin.contiguous()


def cs_table(cos: torch.Tensor, sin: torch.Tensor, seq_len: int) -> torch.Tensor:
    """[seq_len, 2 hd] = [cos | sin] (fused.py:71-73)."""
    return torch.cat([cos[:seq_len], sin[:seq_len]], dim=-1)


def rot_step_table(cos: torch.Tensor, sin: torch.Tensor, chunk: int) -> torch.Tensor:
    """[32, 2 hd] fp32 rows [cos(c f) | sin(c f)] (fused.py:76-79)."""
    return torch.cat([cos[chunk], sin[chunk]]).expand(32, -1).contiguous().float()


def phase2_tables(cos: torch.Tensor, sin: torch.Tensor, chunk: int = 128):
    """Effective per-position [cos | sin] of chunk-relative RoPE (the reference's Phase 2, fused.py:1-14):
    key position p = chunk * t + j is rotated by the table's chunk-relative row j and the query by row
    chunk * t the other way, which equals rotating the key by the composition R_{chunk t} R_j
    (2-D rotations commute, fused.py:9-11):
    cos'(p) = cos(p0) cos(j) - sin(p0) sin(j), sin'(p) = sin(p0) cos(j) + cos(p0) sin(j), p0 = chunk * t,
    in fp32 from the given table values. For an exact table this is the table itself; a rounded table
    (bf16, fp16) gives a rotation that differs from row p by the rounding of rows p0 and j. The B200 form
    uses chunk 128 and reads the base rotation from row p0 directly (the reference steps it with the fp32
    rot_step recurrence, fused.py:76-79)."""
    S = cos.shape[0]
    p = torch.arange(S)
    p0, j = (p // chunk) * chunk, p % chunk
    c, s = cos.float(), sin.float()
    return c[p0] * c[j] - s[p0] * s[j], s[p0] * c[j] + c[p0] * s[j]


# ----------------------------------------------------------------------------------------------
# The op model (fused.py:82-107)
# ----------------------------------------------------------------------------------------------

def reference_decode(q, k_lat, u_k, v_lat, cur_pos, cos, sin, scale: float, u_v=None) -> torch.Tensor:
    """fp32 model of ``palu_sdpa_decode`` (restates fused.py:82-107).

    q [1, B, nh, hd] (already rotated), k_lat [B, nkv, S, r_k], u_k [nkv, r_k, hd],
    v_lat [B, nkv, S, r_v], cur_pos [B] (inclusive last valid position), cos/sin [>= S, hd].
    Query head h attends KV head h // (nh // nkv). With ``u_v`` [nkv, r_v, hd] V is rebuilt per head
    (in-kernel V mode); without it the latent is attended over directly (absorbed V).
    Returns [1, B, nh, r_v] (or [1, B, nh, hd] with u_v)."""
    B, nkv, S, _ = k_lat.shape
    nh = q.shape[2]
    T = rope_transformation_matrix(u_k.shape[-1])
    K = torch.einsum("bhsr,hrd->bhsd", k_lat.float(), u_k.float())
    K = K * cos[None, None, :S] + (K @ T) * sin[None, None, :S]
    rep = nh // nkv
    K = K.repeat_interleave(rep, dim=1)
    V = v_lat.float()
    if u_v is not None:
        V = torch.einsum("bhsr,hrd->bhsd", V, u_v.float())
    V = V.repeat_interleave(rep, dim=1)
    Q = q.float().permute(1, 2, 0, 3)
    mask = torch.zeros(B, 1, 1, S)
    for b in range(B):
        mask[b, :, :, int(cur_pos[b]) + 1:] = float("-inf")
    out = torch.nn.functional.scaled_dot_product_attention(Q, K, V, attn_mask=mask, scale=scale)
    return out.permute(2, 0, 1, 3)


def reference_decode_streamed(q, k_lat, u_k, v_lat, cur_pos, cos, sin, scale: float, u_v=None,
                              group_size: int = 1) -> torch.Tensor:
    """Same math as ``reference_decode``, one (batch row, KV head) at a time, so that large shapes fit
    host memory (the full-config cells of the sweep); latents may be grouped (``group_size`` KV heads
    share latent ``h // group_size``, test_palu_sdpa_device.py:234-235).

    Only the positions 0..cur_pos[b] are touched; the masked tail contributes exactly zero to the
    reference's softmax, so the result equals ``reference_decode`` up to fp32 summation order."""
    B, n_lat, S, _ = k_lat.shape
    nkv = u_k.shape[0]
    nh = q.shape[2]
    rep = nh // nkv
    hd = u_k.shape[-1]
    r_v_out = hd if u_v is not None else v_lat.shape[-1]
    out = torch.zeros(1, B, nh, r_v_out)
    T = rope_transformation_matrix(hd)
    for b in range(B):
        n = int(cur_pos[b]) + 1
        if n <= 0:
            out[0, b] = float("nan")
            continue
        c, s = cos[:n].float(), sin[:n].float()
        for h in range(nkv):
            g = h // group_size
            K = k_lat[b, g, :n].float() @ u_k[h].float()
            K = K * c + (K @ T) * s
            V = v_lat[b, g, :n].float()
            if u_v is not None:
                V = V @ u_v[h].float()
            Qh = q[0, b, h * rep:(h + 1) * rep].float()
            att = torch.softmax((Qh @ K.T) * scale, dim=-1)
            out[0, b, h * rep:(h + 1) * rep] = att @ V
    return out


def seeded_decode_inputs(seed: int, B: int, n_kv: int, n_q: int, S: int, r_k: int, r_v: int, group_size: int = 1):
    """Seeded CPU inputs in the reference device tests' recipe (test_palu_sdpa_device.py:45-55, 218-231):
    bf16-rounded q ~ N(0,1) [1, B, n_q, 128], latents ~ N(0,1) [B, n_kv // group_size, S, r], U_k ~ N(0, 1/r_k)
    [n_kv, r_k, 128] and, for grouped latents, U_v ~ N(0, 1/r_v) [n_kv, r_v, 128]; drawn in this order from one
    generator, so that a long-context fixture can store its seed instead of hundreds of MB of latents.
    Returns (q, k_lat, v_lat, u_k, u_v or None), fp32 holding bf16 values."""
    g = torch.Generator().manual_seed(seed)
    bf = lambda t: t.to(torch.bfloat16).float()
    n_lat = n_kv // group_size
    q = bf(torch.randn(1, B, n_q, 128, generator=g))
    k_lat = bf(torch.randn(B, n_lat, S, r_k, generator=g))
    v_lat = bf(torch.randn(B, n_lat, S, r_v, generator=g))
    u_k = bf(torch.randn(n_kv, r_k, 128, generator=g) / r_k ** 0.5)
    u_v = bf(torch.randn(n_kv, r_v, 128, generator=g) / r_v ** 0.5) if group_size > 1 else None
    return q, k_lat, v_lat, u_k, u_v


def input_checksums(*tensors) -> torch.Tensor:
    """float64 sums of each tensor and of its squares (None -> 0, 0): a fingerprint that a regenerated
    input set must reproduce before its stored output is trusted."""
    out = []
    for t in tensors:
        out += [0.0, 0.0] if t is None else [t.double().sum().item(), t.double().square().sum().item()]
    return torch.tensor(out, dtype=torch.float64)


def expand_groups(lat: torch.Tensor, group_size: int) -> torch.Tensor:
    """[B, n_groups, S, r] -> [B, n_groups * gs, S, r] (test_palu_sdpa_device.py:234-235)."""
    return lat.repeat_interleave(group_size, dim=1)


# ----------------------------------------------------------------------------------------------
# Weight-order helper (tt-metal reverse_permute, used at convert.py:266,276)
# ----------------------------------------------------------------------------------------------

def reverse_permute(t: torch.Tensor, n_heads: int, dim1: int, dim2: int) -> torch.Tensor:
    """HF half-split head order -> Meta interleaved order, per head (restated tt-metal helper)."""
    return t.reshape(n_heads, 2, dim1 // n_heads // 2, dim2).transpose(1, 2).reshape(dim1, dim2)


# ----------------------------------------------------------------------------------------------
# Layer oracle (reference.py:14-55): HF conventions, fp32
# ----------------------------------------------------------------------------------------------

class PaluRefAttention:
    """Restates reference.py:14-55: q from wq, per-head latents from VT, caches of latents,
    K = lat_k @ U_kᵀ and V = lat_v @ U_vᵀ rebuilt over the whole cache, HF rotate-half RoPE,
    GQA, causal mask ``tril(start_pos)``, softmax, ``@ woᵀ``.

    ``lowrank`` is any object with ``k_VT [nkv, r_k, dim]``, ``k_U [nkv, hd, r_k]``, ``v_VT``, ``v_U``.

    ``device_rounding`` (off by default, which is the reference as written) applies the roundings of the
    values the device path stores, so that a comparison measures the kernels rather than those roundings:
    the latent caches in bf16 (the caches are bf16, attention.py:159-169) and, for a one-token decode step,
    q rounded to bf16 after RoPE (the op's q input) and K rotated with the bf16 [cos | sin] table the op
    reads (attention.py:52-78)."""

    def __init__(self, hf_cfg: dict, w: dict, lowrank, device_rounding: bool = False):
        from transformers import LlamaConfig
        from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
        self.cfg = LlamaConfig(**{k: v for k, v in hf_cfg.items() if k != "architectures"})
        self.nh = self.cfg.num_attention_heads
        self.nkv = self.cfg.num_key_value_heads
        self.hd = self.cfg.hidden_size // self.nh
        self.wq, self.wo = w["q"].float(), w["o"].float()
        self.lr = lowrank
        self.rotary = LlamaRotaryEmbedding(config=self.cfg)
        self.cache_k_lat = None
        self.cache_v_lat = None
        self.device_rounding = device_rounding

    @torch.no_grad()
    def forward(self, x: torch.Tensor, start_pos: int) -> torch.Tensor:
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        B, S, _ = x.shape
        q = (x @ self.wq.T).view(B, S, self.nh, self.hd).transpose(1, 2)
        k_lat = torch.einsum("bsd,hrd->bhsr", x, self.lr.k_VT.float())
        v_lat = torch.einsum("bsd,hrd->bhsr", x, self.lr.v_VT.float())
        rnd = lambda t: t.to(torch.bfloat16).float() if self.device_rounding else t
        k_lat, v_lat = rnd(k_lat), rnd(v_lat)
        decode = self.device_rounding and S == 1
        if self.cache_k_lat is None or start_pos == 0:
            self.cache_k_lat, self.cache_v_lat = k_lat, v_lat
        else:
            assert self.cache_k_lat.shape[2] == start_pos
            self.cache_k_lat = torch.cat([self.cache_k_lat, k_lat], dim=2)
            self.cache_v_lat = torch.cat([self.cache_v_lat, v_lat], dim=2)
        T = self.cache_k_lat.shape[2]
        K = torch.einsum("bhtr,hdr->bhtd", self.cache_k_lat, self.lr.k_U.float())
        V = torch.einsum("bhtr,hdr->bhtd", self.cache_v_lat, self.lr.v_U.float())
        pos_q = torch.arange(start_pos, start_pos + S)[None].expand(B, -1)
        pos_k = torch.arange(0, T)[None].expand(B, -1)
        cos_q, sin_q = self.rotary(x, pos_q)
        cos_k, sin_k = self.rotary(x, pos_k)
        if decode:
            cos_k, sin_k = rnd(cos_k), rnd(sin_k)
        q, _ = apply_rotary_pos_emb(q, q, cos_q, sin_q)
        if decode:
            q = rnd(q)
        _, K = apply_rotary_pos_emb(K, K, cos_k, sin_k)
        rep = self.nh // self.nkv
        K = K.repeat_interleave(rep, dim=1)
        V = V.repeat_interleave(rep, dim=1)
        scores = q @ K.transpose(-1, -2) / math.sqrt(self.hd)
        mask = torch.ones(S, T, dtype=torch.bool).tril(diagonal=start_pos)
        scores = scores.masked_fill(~mask, float("-inf"))
        attn = torch.softmax(scores, dim=-1)
        out = (attn @ V).transpose(1, 2).reshape(B, S, self.nh * self.hd)
        return out @ self.wo.T
