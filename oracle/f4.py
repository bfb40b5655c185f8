"""fp4 latent rows: the CPU statement of the library's e2m1 latent-cache format.

TEST INFRASTRUCTURE ONLY (see the package docstring). The reference keeps latent caches in block-float
bfp4_b on request (per side, palu_tt/attention.py:159-169; its device test holds the op to PCC >= 0.95 on
bfp4 latents, tests/test_palu_sdpa_device.py:558-575). The B200 library's form is e2m1 codes (values 0, 0.5,
1, 1.5, 2, 3, 4, 6 and their negatives) with one power-of-two scale per block of 16 values of a row:

* k = the smallest integer with max|block| <= 6 * 2^k, kept in [-120, 7]; an all-zero block has k = 0;
* codes = e2m1(block * 2^-k), round to nearest with ties to the even code, saturating at +-6; the sign
  bit (bit 3) follows the sign of the scaled value, zeros included;
* two codes per byte, the first value in the low nibble; value = code * 2^k.

``quantize_rows`` restates that rule; ``dequantize_rows`` gives the float32 values the decode op must
attend over. The GPU tests check the library's quantizer against this bit for bit.
"""
from __future__ import annotations

import torch

E2M1_MAX = 6.0
K_MIN, K_MAX = -120, 7
GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def block_exponents(amax: torch.Tensor) -> torch.Tensor:
    """int32 k per block: amax = m * 2^e, m in [0.5, 1) (frexp); 6 * 2^k = 0.75 * 2^(k + 3), so k = e - 3 when
    m <= 0.75, else e - 2; clamped to [K_MIN, K_MAX]; 0 where amax == 0."""
    m, e = torch.frexp(amax.float())
    k = torch.where(m <= 0.75, e - 3, e - 2)
    k = torch.where(amax > 0, k, torch.zeros_like(k))
    return k.clamp(K_MIN, K_MAX).to(torch.int32)


def _e2m1_codes(y: torch.Tensor) -> torch.Tensor:
    """Nearest e2m1 code of each value (ties to the even code), with the sign in bit 3."""
    a = y.abs().clamp(max=E2M1_MAX)
    lo = (torch.searchsorted(GRID, a.contiguous(), right=True) - 1).clamp(0, 6)  # GRID[lo] <= a
    hi = lo + 1
    dl, dh = a - GRID[lo], GRID[hi] - a
    pick_hi = (dh < dl) | ((dh == dl) & (lo % 2 == 1))
    code = torch.where(pick_hi, hi, lo)
    code = torch.where(a >= E2M1_MAX, torch.full_like(code, 7), code)
    return (code | (torch.signbit(y).long() << 3)).to(torch.uint8)


def quantize_rows(x: torch.Tensor):
    """x [..., r] (r a multiple of 16) -> (codes uint8 [..., r / 2], exp int8 [..., r / 16])."""
    x32 = x.float()
    *lead, r = x32.shape
    blocks = x32.reshape(*lead, r // 16, 16)
    k = block_exponents(blocks.abs().amax(dim=-1))
    y = torch.ldexp(blocks, (-k).unsqueeze(-1).to(x32.dtype)).reshape(*lead, r)
    c = _e2m1_codes(y).reshape(*lead, r // 2, 2)
    return (c[..., 0] | (c[..., 1] << 4)).to(torch.uint8), k.to(torch.int8)


def dequantize_rows(codes: torch.Tensor, exp: torch.Tensor) -> torch.Tensor:
    """float32 code * 2^exp, [..., r]."""
    c = codes.long()
    nib = torch.stack([c & 15, c >> 4], dim=-1).flatten(-2)
    val = GRID[nib & 7] * torch.where(nib >= 8, -1.0, 1.0)
    return val * torch.exp2(exp.float()).repeat_interleave(16, dim=-1)
