"""fp4 latent caches on the GPU: the quantizer and the append against the oracle's e2m1 rule (oracle/f4.py)
bit for bit, and palu_decode_attn_f4 against the oracle on the dequantized caches.

The fp4 op converts each staged tile to f16 exactly (every e2m1 value times its block's 2^k is an f16 value
for k >= -23) through the same producers as the fp8 op, so it is held to the same bars: the bf16 path's oracle
bar on the dequantized caches (max-abs relative error <= 2e-2, mean-abs <= 1e-3, fp32 output per row), within
F8_VS_BF16 of the bf16 op on the same values, and — against the unquantized latents — the reference's own
bar for bfp4 latents, PCC >= 0.95 at its test shape (tests/test_palu_sdpa_device.py:558-575: B 32,
S 1024, r_k 64, r_v 128).
"""
import pytest
import torch

import oracle
from oracle import f4
from oracle.metrics import rel_errors
from tests.test_f8_gpu import F8_VS_BF16, SCALE, _case, _close, _pcc, _run

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("r", [16, 64, 128, 256])
def test_fp4_quantizer_matches_the_format_rule_bit_for_bit(cuda, r):
    from palu_b200 import fused
    g = torch.Generator().manual_seed(100 + r)
    x = torch.randn(2000, r, generator=g) * torch.exp(torch.randn(2000, r // 16, generator=g).repeat_interleave(16, -1) * 3)
    x[5] = 0
    x[7, 0] = 1e4  # saturates at 6 * 2^7
    x = x.bfloat16()
    got = fused.quantize_latents_f4(x.to(cuda))
    codes, exp = f4.quantize_rows(x)
    assert torch.equal(got.exp.cpu(), exp)
    # codes bit for bit, except the sign of a zero code (both decode to 0)
    gc, wc = got.codes.cpu(), codes
    zero_lo, zero_hi = (wc & 7) == 0, ((wc >> 4) & 7) == 0
    mask = torch.where(zero_lo, 0xF0, 0xFF) & torch.where(zero_hi, 0x0F, 0xFF)
    assert torch.equal(gc & mask.to(torch.uint8), wc & mask.to(torch.uint8))
    assert torch.equal(f4.dequantize_rows(gc, got.exp.cpu()), f4.dequantize_rows(wc, exp))


def test_fp4_append_writes_quantized_rows_at_cur_pos_only(cuda):
    from palu_b200 import fused
    B, G, S, r_k, r_v = 4, 2, 200, 64, 128
    g = torch.Generator().manual_seed(8)
    kc = fused.F4Latents.empty(B, G, S, r_k, device=cuda)
    vc = fused.F4Latents.empty(B, G, S, r_v, device=cuda)
    nk = torch.randn(B, G, r_k, generator=g).bfloat16()
    nv = (torch.randn(B, G, r_v, generator=g) * 30).bfloat16()
    pos = torch.tensor([0, 199, -1, 57], dtype=torch.int32)
    fused.append_latents_f8(nk.to(cuda), nv.to(cuda), pos.to(cuda), kc, vc)
    torch.cuda.synchronize()
    for cache, new in ((kc, nk), (vc, nv)):
        want = torch.zeros(B, G, S, new.shape[-1])
        for b in range(B):
            if 0 <= int(pos[b]) < S:
                c, e = f4.quantize_rows(new[b])
                want[b, :, int(pos[b])] = f4.dequantize_rows(c, e)
        assert torch.equal(f4.dequantize_rows(cache.codes.cpu(), cache.exp.cpu()), want)


CASES = [  # (B, n_kv, n_groups, S, r_k, r_v, grouped)
    (4, 8, 8, 2000, 64, 64, False),
    (3, 8, 8, 1500, 64, 128, False),
    (2, 8, 8, 3000, 128, 128, False),
    (2, 8, 2, 1200, 128, 128, True),
]


@pytest.mark.parametrize("case", CASES, ids=[f"rk{c[4]}_rv{c[5]}_g{c[2]}" for c in CASES])
def test_fp4_decode_matches_the_oracle_on_the_dequantized_caches(cuda, case):
    from palu_b200 import fused
    B, n_kv, G, S, r_k, r_v, grouped = case
    q, k, v, u_k, u_v, pos, cos, sin = _case(sum(case[:6]) + 1, B, n_kv, G, S, r_k, r_v, grouped)
    kc, vc = fused.quantize_latents_f4(k.to(cuda)), fused.quantize_latents_f4(v.to(cuda))
    kd, vd = f4.dequantize_rows(kc.codes.cpu(), kc.exp.cpu()), f4.dequantize_rows(vc.codes.cpu(), vc.exp.cpu())
    out = _run(cuda, q, kc, vc, u_k, u_v, pos, cos, sin).cpu()
    bf = _run(cuda, q, kd.bfloat16().to(cuda), vd.bfloat16().to(cuda), u_k, u_v, pos, cos, sin).cpu()
    mx, mn = rel_errors(out, bf)
    assert mx <= F8_VS_BF16[0] and mn <= F8_VS_BF16[1], f"fp4 vs bf16 op: max {mx:.3e} mean {mn:.3e}"
    gs = n_kv // G
    ref = oracle.reference_decode(q.float(), oracle.expand_groups(kd, gs), u_k.float(), oracle.expand_groups(vd, gs),
                                  pos, cos, sin, SCALE, u_v=None if u_v is None else u_v.float())
    _close(out, ref, f"fp4 {case}")


def test_fp4_latents_track_the_unquantized_reference(cuda):
    """The reference's bfp4 test shape and bar: PCC >= 0.95 against the fp32 reference on the unquantized
    latents (bf16 output)."""
    from palu_b200 import fused
    q, k, v, u_k, _, pos, cos, sin = _case(23, 32, 8, 8, 1024, 64, 128)
    kc, vc = fused.quantize_latents_f4(k.to(cuda)), fused.quantize_latents_f4(v.to(cuda))
    out = _run(cuda, q, kc, vc, u_k, None, pos, cos, sin, out_dtype=torch.bfloat16).cpu().float()
    ref = oracle.reference_decode(q.float(), k.float(), u_k.float(), v.float(), pos, cos, sin, SCALE)
    assert _pcc(out, ref) >= 0.95


@pytest.mark.parametrize("splits", [1, 64])
def test_fp4_split_counts_and_garbage_past_cur_pos(cuda, splits):
    from palu_b200 import fused
    q, k, v, u_k, _, pos, cos, sin = _case(35, 4, 8, 8, 900, 64, 64)
    kc, vc = fused.quantize_latents_f4(k.to(cuda)), fused.quantize_latents_f4(v.to(cuda))
    kd, vd = f4.dequantize_rows(kc.codes.cpu(), kc.exp.cpu()), f4.dequantize_rows(vc.codes.cpu(), vc.exp.cpu())
    for b in range(4):
        p = int(pos[b]) + 1
        for c in (kc, vc):
            c.codes[b, :, p:] = 0x77
            c.exp[b, :, p:] = 100
    out = _run(cuda, q, kc, vc, u_k, None, pos, cos, sin, splits=splits).cpu()
    assert torch.isfinite(out).all()
    ref = oracle.reference_decode(q.float(), kd, u_k.float(), vd, pos, cos, sin, SCALE)
    _close(out, ref, f"fp4 splits={splits}")
