"""fp8 latent caches without a GPU: the oracle's format rule (oracle/f8.py) and the fp8 entry points'
validation through the C ABI (dummy pointers: validation fails before any CUDA call).

The format is the B200 form of the reference's block-float latent caches (bfp8_b by default,
palu_tt/attention.py:159-169): e4m3 codes and one power-of-two exponent per row."""
import ctypes

import pytest
import torch

import oracle
from oracle import f8


def test_row_exponent_is_the_smallest_that_fits():
    g = torch.Generator().manual_seed(3)
    amax = torch.exp(torch.randn(20000, generator=g) * 8)  # magnitudes over ~2^-30 .. 2^30
    amax = torch.cat([amax, torch.tensor([448.0, 449.0, 0.875 * 512, 0.876 * 512, 1.0, 2.0 ** -130])])
    k = f8.row_exponents(amax).double()
    inside = (k > f8.K_MIN) & (k < f8.K_MAX)
    a = amax.double()
    assert torch.all(a[inside] <= 448 * torch.exp2(k[inside]))
    assert torch.all(a[inside] > 448 * torch.exp2(k[inside] - 1))
    assert f8.row_exponents(torch.tensor([0.0])).item() == 0
    assert f8.row_exponents(torch.tensor([1e30])).item() == f8.K_MAX
    assert f8.row_exponents(torch.tensor([1e-40])).item() == f8.K_MIN


def test_quantized_rows_round_trip_within_e4m3_precision():
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(4096, 64, generator=g) * torch.exp(torch.randn(4096, 1, generator=g) * 3)).bfloat16()
    codes, exp = f8.quantize_rows(x)
    assert codes.dtype == torch.uint8 and exp.dtype == torch.int8 and codes.shape == x.shape
    d = f8.dequantize_rows(codes, exp)
    xf = x.float()
    step = torch.exp2(exp.float()).unsqueeze(-1)
    # normal codes: half an ulp of 3 mantissa bits; flushed codes: below the smallest normal (2^-6 * 2^k)
    err = (d - xf).abs()
    fits = (xf.abs().amax(-1) <= 448 * 2.0 ** f8.K_MAX).unsqueeze(-1)  # rows past that saturate
    assert fits.float().mean() > 0.9
    ok = err <= torch.maximum(xf.abs() * 2.0 ** -4, step * 2.0 ** -6) * (1 + 1e-6)
    assert torch.all(ok | ~fits)
    sat = ~fits & (xf.abs() > 448 * 2.0 ** f8.K_MAX)
    assert torch.all(d[sat].abs() == 448 * 2.0 ** f8.K_MAX)
    # the row maximum is never clipped and every code is normal or zero
    assert torch.all(d.abs().amax(-1) <= 448 * step.squeeze(-1))
    sub = (codes & 0x78) == 0
    assert torch.all((codes[sub] & 0x7F) == 0)


def test_exact_values_survive_and_zero_rows_stay_zero():
    x = torch.tensor([[1.0, -3.0, 0.5, 448.0 / 64], [0.0, 0.0, 0.0, 0.0]]).repeat(1, 4).bfloat16()
    codes, exp = f8.quantize_rows(x)
    assert torch.equal(f8.dequantize_rows(codes, exp), x.float())
    assert exp[1].item() == 0 and torch.all(codes[1] == 0)


def test_f8_entry_points_validate_before_any_cuda_call():
    from palu_b200 import _lib
    lib = _lib.load()
    z = ctypes.c_void_p(16)
    st = lib.palu_quantize_latents_f8(z, 10, 40, z, z, None)
    assert st == _lib.PALU_ERR_INVALID and "multiple of 16" in lib.palu_last_error().decode()
    d = _lib.dims(2, 32, 8, 8, 64, 64, 256)
    st = lib.palu_append_latents_f8(z, z, z, z, z, None, z, ctypes.byref(d), None)
    assert st == _lib.PALU_ERR_INVALID and "every pointer" in lib.palu_last_error().decode()
    wide = _lib.dims(2, 32, 8, 2, 256, 256, 256)
    ws = ctypes.c_void_p(256)
    st = lib.palu_decode_attn_f8(z, z, z, z, z, z, 128, z, z, z, z, 0, ws, 1 << 30, ctypes.byref(wide), 0.1, None)
    assert st == _lib.PALU_ERR_INVALID and "at most 128" in lib.palu_last_error().decode()
    st = lib.palu_decode_attn_f8(z, z, z, None, z, z, 128, None, z, z, z, 0, ws, 1 << 30, ctypes.byref(d), 0.1, None)
    assert st == _lib.PALU_ERR_INVALID and "exponent" in lib.palu_last_error().decode()


def test_fp8_caches_through_the_reference_surface_are_checked():
    from palu_b200 import fused
    k = fused.F8Latents.empty(2, 8, 256, 64)
    v = torch.zeros(2, 8, 256, 64, dtype=torch.bfloat16)
    q = torch.zeros(1, 2, 32, 128, dtype=torch.bfloat16)
    w = torch.zeros(1, 8, 64, 256, dtype=torch.bfloat16)
    cs = torch.zeros(1, 1, 256, 256, dtype=torch.bfloat16)
    pos = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="both be bf16 or both fp8"):
        fused.palu_sdpa_decode(q, k, w, cs, v, 64, pos)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused.palu_sdpa_decode(q, k, w, cs, fused.F8Latents.empty(2, 8, 256, 64), 64, pos)
    with pytest.raises(RuntimeError, match="leading dims"):
        fused.F8Latents(torch.zeros(2, 4, dtype=torch.uint8), torch.zeros(3, dtype=torch.int8))


def test_fp4_block_exponents_and_rounding():
    """The e2m1 rule (oracle/f4.py): the smallest exponent that fits 6 * 2^k, nearest code with ties to
    the even code, saturation at 6."""
    from oracle import f4
    g = torch.Generator().manual_seed(6)
    amax = torch.exp(torch.randn(20000, generator=g) * 6)
    k = f4.block_exponents(amax).double()
    inside = (k > f4.K_MIN) & (k < f4.K_MAX)
    a = amax.double()
    assert torch.all(a[inside] <= 6 * torch.exp2(k[inside]))
    assert torch.all(a[inside] > 6 * torch.exp2(k[inside] - 1))
    # one block scaled by 2^1 (max 7): ties go to the even code
    x = torch.tensor([[0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.25, -0.75, 0, 0, 0, 0, 0, 6.0]])
    codes, exp = f4.quantize_rows(x)
    assert exp.item() == 1
    want = torch.tensor([[0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 8.0, -0.0, -1.0, 0, 0, 0, 0, 0, 6.0]])
    assert torch.equal(f4.dequantize_rows(codes, exp), want)
    assert codes.shape == (1, 8) and (codes[0, 0] & 15).item() == 0 and (codes[0, 0] >> 4).item() == 1


def test_fp4_round_trip_within_e2m1_precision():
    from oracle import f4
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(2048, 128, generator=g) * torch.exp(torch.randn(2048, 1, generator=g))).bfloat16()
    codes, exp = f4.quantize_rows(x)
    assert codes.shape == (2048, 64) and exp.shape == (2048, 8)
    d, xf = f4.dequantize_rows(codes, exp), x.float()
    step = torch.exp2(exp.float()).repeat_interleave(16, dim=-1)
    # e2m1 spacing is at most 2 (between 4 and 6) in units of 2^k: half a step is at most 1
    assert torch.all((d - xf).abs() <= step * (1 + 1e-6))
    assert torch.all(d.abs() <= 6 * step)
