"""fp8 latent rows: the CPU statement of the library's e4m3 latent-cache format.

TEST INFRASTRUCTURE ONLY (see the package docstring). The reference keeps its latent caches in
block-float formats (bfp8_b by default, bfp4_b per side; palu_tt/attention.py:159-169; the bfp4 device
test, tests/test_palu_sdpa_device.py:558-575, holds the op to PCC >= 0.95 against the fp32
``reference_decode`` on the unquantized latents). Those are Tensix formats; the B200 library's form is
e4m3 codes with one power-of-two scale per row (one position of one latent head):

* k = the smallest integer with max|row| <= 448 * 2^k (448 = the largest e4m3 value), kept in
  [-120, 7]; an all-zero row has k = 0;
* codes = e4m3(row * 2^-k), round to nearest even, saturating at +-448;
* codes whose exponent field is 0 (e4m3 subnormals) are stored as a signed zero;
* value = code * 2^k.

``quantize_rows`` restates that rule with torch's float8_e4m3fn conversion; ``dequantize_rows`` gives the
float32 values the decode op must attend over. The GPU tests check the library's quantizer against this
bit for bit, and the fp8 decode op against ``reference_decode`` on ``dequantize_rows`` of the same caches.
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0
K_MIN, K_MAX = -120, 7


def row_exponents(amax: torch.Tensor) -> torch.Tensor:
    """int32 k per row: amax = m * 2^e with m in [0.5, 1) (frexp), and 448 * 2^k = 0.875 * 2^(k + 9), so
    k = e - 9 when m <= 0.875, else e - 8; clamped to [K_MIN, K_MAX]; 0 where amax == 0."""
    m, e = torch.frexp(amax.float())
    k = torch.where(m <= 0.875, e - 9, e - 8)
    k = torch.where(amax > 0, k, torch.zeros_like(k))
    return k.clamp(K_MIN, K_MAX).to(torch.int32)


def quantize_rows(x: torch.Tensor):
    """x [..., r] (any float dtype; the library quantizes bf16) -> (codes uint8 [..., r], exp int8 [...])."""
    x32 = x.float()
    k = row_exponents(x32.abs().amax(dim=-1))
    y = torch.ldexp(x32, (-k).unsqueeze(-1).to(x32.dtype)).clamp(-E4M3_MAX, E4M3_MAX)
    codes = y.to(torch.float8_e4m3fn).view(torch.uint8)
    codes = torch.where((codes & 0x78) == 0, codes & 0x80, codes)
    return codes, k.to(torch.int8)


def dequantize_rows(codes: torch.Tensor, exp: torch.Tensor) -> torch.Tensor:
    """float32 code * 2^exp."""
    return codes.view(torch.float8_e4m3fn).float() * torch.exp2(exp.float()).unsqueeze(-1)
