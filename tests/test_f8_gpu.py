"""fp8 latent caches on the GPU: the quantizer and the append against the oracle's format rule bit for bit,
and the fp8 decode op (palu_decode_attn_f8) against the oracle on the dequantized caches.

The fp8 op converts each staged tile to f16 exactly (every e4m3 code is an f16 value; V rows are scaled by
their 2^k, K row scales are applied to the scores), reconstructs K against U rounded to f16 and feeds P to
the PV product as f16 hi + lo. On the dequantized caches it is held to the bf16 path's oracle bar (max-abs
relative error <= 2e-2, mean-abs relative error <= 1e-3, fp32 output per row) and to within
F8_VS_BF16 of the bf16 op on the same values. Against the unquantized latents the bar is a PCC, like the
reference's block-float test (tests/test_palu_sdpa_device.py:558-575: bfp4 latents, PCC >= 0.95); e4m3
rows are held to 0.99.
"""
import pytest
import torch

import oracle
from oracle import f8
from oracle.metrics import MAX_REL, MEAN_REL, rel_errors, rowwise_rel_errors

pytestmark = pytest.mark.gpu

THETA = 500000.0
LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
SCALE = 128 ** -0.5
F8_VS_BF16 = (5e-3, 2e-4)  # max-abs / mean-abs relative difference of the fp8 and bf16 ops on the same values


def _close(out, ref, what):
    mx, mn = rel_errors(out, ref)
    assert mx <= MAX_REL and mn <= MEAN_REL, f"{what}: global max {mx:.3e} mean {mn:.3e}"
    rmx, rmn = rowwise_rel_errors(out, ref)
    assert rmx <= MAX_REL and rmn <= MEAN_REL, f"{what}: worst row max {rmx:.3e} mean {rmn:.3e}"


def _pcc(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    a, b = a - a.mean(), b - b.mean()
    return float((a @ b) / (a.norm() * b.norm()))


def _case(seed, B, n_kv, n_groups, S, r_k, r_v, grouped=False, spread=0.0):
    """BASELINE's distributions (latents and q ~ N(0,1), U ~ N(0, 1/rank)); ``spread`` > 0 scales each
    cached row by e^(N(0, spread^2)), so that the rows' exponents cover a wide range."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, B, 4 * n_kv, 128, generator=g).bfloat16()
    k = (torch.randn(B, n_groups, S, r_k, generator=g) *
         torch.exp(spread * torch.randn(B, n_groups, S, 1, generator=g))).bfloat16()
    v = (torch.randn(B, n_groups, S, r_v, generator=g) *
         torch.exp(spread * torch.randn(B, n_groups, S, 1, generator=g))).bfloat16()
    u_k = (torch.randn(n_kv, r_k, 128, generator=g) / r_k ** 0.5).bfloat16()
    u_v = (torch.randn(n_kv, r_v, 128, generator=g) / r_v ** 0.5).bfloat16() if grouped else None
    pos = torch.randint(S // 2, S, (B,), generator=g, dtype=torch.int32)
    pos[0] = S - 1
    special = [0, 127, 128, 200]
    for i in range(1, min(B, 1 + len(special))):
        pos[i] = min(special[i - 1], S - 1)
    cos, sin = oracle.cos_sin_tables(128, S, THETA, LLAMA3)
    return q, k, v, u_k, u_v, pos, cos[:S].bfloat16().float(), sin[:S].bfloat16().float()


def _run(dev, q, kc, vc, u_k, u_v, pos, cos, sin, out_dtype=torch.float32, splits=0):
    from palu_b200 import fused
    S = kc.shape[2]
    w_rot = fused.w_rot_from_u_k(u_k.float())[None].to(dev, torch.bfloat16)
    cs = fused.cs_table(cos, sin, S)[None, None].to(dev, torch.bfloat16)
    hd_v = 128 if u_v is not None else vc.shape[-1]
    out = fused.palu_sdpa_decode(q.to(dev), kc, w_rot, cs, vc, hd_v, pos.to(dev), scale=SCALE,
                                 u_v=None if u_v is None else u_v[None].to(dev), out_dtype=out_dtype, splits=splits,
                                 check_status=True)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("r", [16, 64, 96, 128, 256])
def test_quantizer_matches_the_format_rule_bit_for_bit(cuda, r):
    from palu_b200 import fused
    g = torch.Generator().manual_seed(r)
    x = torch.randn(3000, r, generator=g) * torch.exp(torch.randn(3000, 1, generator=g) * 4)
    x[5] = 0
    x[6, :] = 1e-39  # below bf16's normal range
    x[7, 0] = 3e5  # saturates at 448 * 2^7
    x = x.bfloat16()
    got = fused.quantize_latents_f8(x.to(cuda))
    codes, exp = f8.quantize_rows(x)
    assert torch.equal(got.exp.cpu(), exp)
    assert torch.equal(got.codes.cpu(), codes)


def test_append_writes_quantized_rows_at_cur_pos_only(cuda):
    from palu_b200 import fused
    B, G, S, r_k, r_v = 5, 4, 300, 64, 96
    g = torch.Generator().manual_seed(9)
    kc = fused.F8Latents.empty(B, G, S, r_k, device=cuda)
    vc = fused.F8Latents.empty(B, G, S, r_v, device=cuda)
    nk = torch.randn(B, G, r_k, generator=g).bfloat16()
    nv = (torch.randn(B, G, r_v, generator=g) * 50).bfloat16()
    pos = torch.tensor([0, 299, 17, -1, 300], dtype=torch.int32)
    fused.append_latents_f8(nk.to(cuda), nv.to(cuda), pos.to(cuda), kc, vc)
    torch.cuda.synchronize()
    for cache, new in ((kc, nk), (vc, nv)):
        codes, exp = f8.quantize_rows(new)
        want_c = torch.zeros_like(cache.codes.cpu())
        want_e = torch.zeros_like(cache.exp.cpu())
        for b in range(B):
            if 0 <= int(pos[b]) < S:
                want_c[b, :, int(pos[b])] = codes[b]
                want_e[b, :, int(pos[b])] = exp[b]
        assert torch.equal(cache.codes.cpu(), want_c)
        assert torch.equal(cache.exp.cpu(), want_e)


CASES = [  # (B, n_kv, n_groups, S, r_k, r_v, grouped)
    (4, 8, 8, 2000, 64, 64, False),
    (3, 8, 8, 1500, 32, 128, False),
    (2, 8, 8, 3000, 128, 128, False),
    (3, 8, 8, 700, 48, 96, False),
    (2, 8, 2, 1200, 128, 128, True),
]


@pytest.mark.parametrize("case", CASES, ids=[f"rk{c[4]}_rv{c[5]}_g{c[2]}" for c in CASES])
def test_fp8_decode_matches_the_oracle_on_the_dequantized_caches(cuda, case):
    from palu_b200 import fused
    B, n_kv, G, S, r_k, r_v, grouped = case
    q, k, v, u_k, u_v, pos, cos, sin = _case(sum(case[:6]), B, n_kv, G, S, r_k, r_v, grouped)
    kc, vc = fused.quantize_latents_f8(k.to(cuda)), fused.quantize_latents_f8(v.to(cuda))
    kd, vd = f8.dequantize_rows(kc.codes.cpu(), kc.exp.cpu()), f8.dequantize_rows(vc.codes.cpu(), vc.exp.cpu())
    out = _run(cuda, q, kc, vc, u_k, u_v, pos, cos, sin).cpu()
    # the same values as bf16 caches through the bf16 op
    bf = _run(cuda, q, kd.bfloat16().to(cuda), vd.bfloat16().to(cuda), u_k, u_v, pos, cos, sin).cpu()
    mx, mn = rel_errors(out, bf)
    assert mx <= F8_VS_BF16[0] and mn <= F8_VS_BF16[1], f"fp8 vs bf16 op: max {mx:.3e} mean {mn:.3e}"
    gs = n_kv // G
    ref = oracle.reference_decode(q.float(), oracle.expand_groups(kd, gs), u_k.float(), oracle.expand_groups(vd, gs),
                                  pos, cos, sin, SCALE, u_v=None if u_v is None else u_v.float())
    _close(out, ref, f"fp8 {case}")


def test_fp8_matches_bf16_on_rows_of_every_magnitude(cuda):
    """Rows scaled by e^(N(0, 2^2)) (exponents from about -20 to 7, V rows below 2^-14 carried as f16
    subnormals): the fp8 op against the bf16 op on the dequantized caches."""
    from palu_b200 import fused
    q, k, v, u_k, _, pos, cos, sin = _case(44, 3, 8, 8, 1000, 64, 128, spread=2.0)
    kc, vc = fused.quantize_latents_f8(k.to(cuda)), fused.quantize_latents_f8(v.to(cuda))
    assert int(kc.exp.min()) < -14 and int(kc.exp.max()) > 0
    kd, vd = f8.dequantize_rows(kc.codes.cpu(), kc.exp.cpu()), f8.dequantize_rows(vc.codes.cpu(), vc.exp.cpu())
    out = _run(cuda, q, kc, vc, u_k, None, pos, cos, sin).cpu()
    bf = _run(cuda, q, kd.bfloat16().to(cuda), vd.bfloat16().to(cuda), u_k, None, pos, cos, sin).cpu()
    mx, mn = rel_errors(out, bf)
    assert mx <= 2e-2 and mn <= 1e-3, f"fp8 vs bf16 op: max {mx:.3e} mean {mn:.3e}"


def test_fp8_latents_track_the_unquantized_reference(cuda):
    """The reference's block-float test shape (B 32, S 1024, r_k 64, r_v 128; bfp4 -> PCC >= 0.95):
    e4m3 rows against the fp32 reference on the unquantized latents, PCC >= 0.99, bf16 output."""
    from palu_b200 import fused
    q, k, v, u_k, _, pos, cos, sin = _case(21, 32, 8, 8, 1024, 64, 128)
    kc, vc = fused.quantize_latents_f8(k.to(cuda)), fused.quantize_latents_f8(v.to(cuda))
    out = _run(cuda, q, kc, vc, u_k, None, pos, cos, sin, out_dtype=torch.bfloat16).cpu().float()
    ref = oracle.reference_decode(q.float(), k.float(), u_k.float(), v.float(), pos, cos, sin, SCALE)
    assert _pcc(out, ref) >= 0.99


@pytest.mark.parametrize("splits", [1, 3, 64])
def test_fp8_split_counts_and_garbage_past_cur_pos(cuda, splits):
    """Codes past cur_pos hold e4m3 NaN and their exponents junk: masked positions contribute nothing."""
    from palu_b200 import fused
    q, k, v, u_k, _, pos, cos, sin = _case(33, 4, 8, 8, 900, 64, 64)
    kc, vc = fused.quantize_latents_f8(k.to(cuda)), fused.quantize_latents_f8(v.to(cuda))
    kd, vd = f8.dequantize_rows(kc.codes.cpu(), kc.exp.cpu()), f8.dequantize_rows(vc.codes.cpu(), vc.exp.cpu())
    for b in range(4):
        p = int(pos[b]) + 1
        for c in (kc, vc):
            c.codes[b, :, p:] = 0x7F
            c.exp[b, :, p:] = 100
    out = _run(cuda, q, kc, vc, u_k, None, pos, cos, sin, splits=splits).cpu()
    assert torch.isfinite(out).all()
    ref = oracle.reference_decode(q.float(), kd, u_k.float(), vd, pos, cos, sin, SCALE)
    _close(out, ref, f"fp8 splits={splits}")
