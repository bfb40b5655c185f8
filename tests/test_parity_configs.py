"""Parity of the CUDA decode op with the oracle at the BASELINE configs' full sizes.

Each case launches the op on the config's whole shape (inputs generated on the GPU from a seed, with the
configs' distributions: latents and q ~ N(0,1), U ~ N(0, 1/rank), llama3 RoPE) and compares a seeded
subset of batch rows, all heads, with ``oracle.reference_decode_streamed`` (the reference's fp32
``reference_decode``, palu_tt/fused.py:82-107, one (row, KV head) at a time so the large shapes fit host
memory). Checked rows include a full-context row (cur_pos = S - 1) and ragged ones.

Bar (the north star's, written here): max-abs relative error <= 2e-2 and mean-abs relative error <= 1e-3,
on the fp32 output per (batch row, query head) row and globally, and on the bf16 output globally against
the oracle rounded to bf16.

* ``mlrd_r64_b32_s8192``: the bench workload (BASELINE's target row), every row checked;
* ``identity_r128_b32_s8192``: BASELINE config 2, U = I at rank 128, also against plain GQA flash-decode
  over the rotated full K (``palu_plain_gqa_decode``), which it must match within the same bar;
* ``glrd_gs4_r256_b16_s16384``: BASELINE config 3, 2 groups of 4 KV heads sharing rank-256 latents, V
  rebuilt per head through u_v;
* ``sweep_*``: BASELINE config 5's mixed-path layer (r_k 32, r_v 128) at 32k and 128k cached positions,
  batch 1 and 8.
The reference's own reference_decode at 32768 positions is pinned separately by the golden fixture
``decode_long_rk32_rv128_s32768`` (inputs regenerated from its seed, checksums verified).
"""
import pytest
import torch

import oracle
from oracle.metrics import MAX_REL, MEAN_REL, rel_errors, rowwise_rel_errors
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

THETA = 500000.0
LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
SCALE = 128 ** -0.5


def _close(out, ref, what, per_row=True):
    mx, mn = rel_errors(out, ref)
    assert mx <= MAX_REL and mn <= MEAN_REL, f"{what}: global max {mx:.3e} mean {mn:.3e}"
    if per_row:
        rmx, rmn = rowwise_rel_errors(out, ref)
        assert rmx <= MAX_REL and rmn <= MEAN_REL, f"{what}: worst row max {rmx:.3e} mean {rmn:.3e}"


def _tables(S, dev):
    from palu_b200 import fused
    cos, sin = oracle.cos_sin_tables(128, S, THETA, LLAMA3)
    cos, sin = cos[:S].bfloat16().float(), sin[:S].bfloat16().float()
    cs = fused.cs_table(cos, sin, S)[None, None].to(dev, torch.bfloat16)
    return cos, sin, cs


def _gpu_case(dev, seed, B, n_kv, n_lat, S, r_k, r_v, *, grouped=False, identity=False, full_rows=False):
    g = torch.Generator(device=dev).manual_seed(seed)
    bf = torch.bfloat16
    q = torch.randn(1, B, 4 * n_kv, 128, generator=g, device=dev, dtype=bf)
    k = torch.randn(B, n_lat, S, r_k, generator=g, device=dev, dtype=bf)
    v = torch.randn(B, n_lat, S, r_v, generator=g, device=dev, dtype=bf)
    if identity:
        u_k = torch.eye(128, device=dev, dtype=bf).expand(n_kv, 128, 128).contiguous()
    else:
        u_k = (torch.randn(n_kv, r_k, 128, generator=g, device=dev) / r_k ** 0.5).to(bf)
    u_v = (torch.randn(n_kv, r_v, 128, generator=g, device=dev) / r_v ** 0.5).to(bf) if grouped else None
    if full_rows:
        pos = torch.full((B,), S - 1, dtype=torch.int32)
    else:
        gp = torch.Generator().manual_seed(seed)
        pos = torch.randint(S // 2, S, (B,), generator=gp, dtype=torch.int32)
        pos[0] = S - 1
    return q, k, v, u_k, u_v, pos


def _run(q, k, v, u_k, u_v, pos, cs, out_dtype):
    from palu_b200 import fused
    w_rot = fused.w_rot_from_u_k(u_k.float()).to(torch.bfloat16)[None]
    head_dim_v = 128 if u_v is not None else v.shape[-1]
    out = fused.palu_sdpa_decode(q, k, w_rot, cs, v, head_dim_v, pos.to(q.device), scale=SCALE,
                                 u_v=None if u_v is None else u_v[None], out_dtype=out_dtype, check_status=True)
    return out


def _oracle_rows(q, k, v, u_k, u_v, pos, cos, sin, rows, group_size):
    r = torch.tensor(rows)
    return oracle.reference_decode_streamed(
        q[:, r].float().cpu(), k[r].float().cpu(), u_k.float().cpu(), v[r].float().cpu(), pos[r], cos, sin, SCALE,
        u_v=None if u_v is None else u_v.float().cpu(), group_size=group_size)


def _check_config(dev, seed, B, n_kv, n_lat, S, r_k, r_v, rows, *, grouped=False, identity=False, full_rows=False,
                  name=""):
    q, k, v, u_k, u_v, pos = _gpu_case(dev, seed, B, n_kv, n_lat, S, r_k, r_v, grouped=grouped, identity=identity,
                                       full_rows=full_rows)
    cos, sin, cs = _tables(S, dev)
    out32 = _run(q, k, v, u_k, u_v, pos, cs, torch.float32)
    out16 = _run(q, k, v, u_k, u_v, pos, cs, torch.bfloat16)
    torch.cuda.synchronize()
    ref = _oracle_rows(q, k, v, u_k, u_v, pos, cos, sin, rows, n_kv // n_lat)
    r = torch.tensor(rows)
    _close(out32[:, r].cpu(), ref, f"{name} fp32 output")
    _close(out16[:, r].float().cpu(), ref.to(torch.bfloat16).float(), f"{name} bf16 output", per_row=False)
    return q, k, v, u_k, u_v, pos, cos, sin, out32


def test_bench_workload_mlrd_r64_b32_s8192(cuda):
    """BASELINE's target row at full size (the shape the bench times): every batch row checked."""
    _check_config(cuda, 101, 32, 8, 8, 8192, 64, 64, list(range(32)), full_rows=True, name="mlrd_r64_b32_s8192")


def test_identity_r128_b32_s8192_matches_oracle_and_plain_gqa(cuda):
    """U = I at rank 128 equals plain GQA flash-decode over the rotated full K.

    A stock cache holds the rotated K in bf16, so the plain path attends over K_rot rounded to bf16 while
    the identity path rotates the exact latent. Each path is first held to the bar against the oracle on
    its own inputs (plain: the oracle with K_rot as the latent, U = I and no rotation). The two kernels
    must then agree with each other to within what that input rounding alone moves the result (the two
    oracles' difference) plus the bar."""
    from palu_b200 import fused
    rows = [0, 5, 13, 31]
    q, k, v, u_k, u_v, pos, cos, sin, out32 = _check_config(
        cuda, 102, 32, 8, 8, 8192, 128, 128, rows, identity=True, full_rows=True, name="identity_r128_b32_s8192")
    # plain GQA on K rotated with the same bf16 tables (K = latent when U = I), rounded to bf16
    S = k.shape[2]
    kf = k.float()
    kr = torch.stack([-kf[..., 1::2], kf[..., 0::2]], dim=-1).flatten(-2)
    k_rot = (kf * cos.to(cuda) + kr * sin.to(cuda)).to(torch.bfloat16)
    del kf, kr
    plain = fused.plain_gqa_decode(q, k_rot, v, pos.to(cuda), scale=SCALE, out_dtype=torch.float32)
    torch.cuda.synchronize()
    r = torch.tensor(rows)
    ref_plain = _oracle_rows(q, k_rot, v, u_k, None, pos, torch.ones(S, 128), torch.zeros(S, 128), rows, 1)
    _close(plain[:, r].cpu(), ref_plain, "plain GQA vs oracle on the bf16 K cache")
    ref_latent = _oracle_rows(q, k, v, u_k, None, pos, cos, sin, rows, 1)
    imx, imn = rel_errors(ref_plain, ref_latent)  # the stock cache's bf16 K rounding alone
    mx, mn = rel_errors(plain[:, r].cpu(), out32[:, r].cpu())
    assert mx <= imx + MAX_REL and mn <= imn + MEAN_REL, \
        f"plain GQA vs identity palu: max {mx:.3e} mean {mn:.3e} (input rounding alone: {imx:.3e} / {imn:.3e})"


def test_glrd_gs4_r256_b16_s16384(cuda):
    """grouped rank-256 latents (2 groups x 4 KV heads), V rebuilt per head."""
    _check_config(cuda, 103, 16, 8, 2, 16384, 256, 256, [0, 7, 15], grouped=True, name="glrd_gs4_r256_b16_s16384")


@pytest.mark.parametrize("B,S", [(1, 32768), (8, 32768), (1, 131072), (8, 131072)],
                         ids=["b1_s32k", "b8_s32k", "b1_s128k", "b8_s128k"])
def test_sweep_cells_rk32_rv128(cuda, B, S):
    """BASELINE config 5's mixed-path layer (r_k 32, r_v 128) at long context."""
    rows = [0] if B == 1 else [0, B - 1]
    _check_config(cuda, 104 + B + S // 1024, B, 8, 8, S, 32, 128, rows, name=f"sweep_b{B}_s{S}")
    torch.cuda.empty_cache()


def test_long_context_golden_fixture(cuda):
    """The reference's own reference_decode at 32768 positions (tests/golden/make_golden.py): the inputs
    are regenerated from the fixture's seed and must reproduce its checksums first."""
    from palu_b200 import fused
    d = load_golden("decode_long_rk32_rv128_s32768")
    B, nkv, nh, S, r_k, r_v = (int(x) for x in d["dims"])
    q, k, v, u_k, _ = oracle.seeded_decode_inputs(int(d["seed"]), B, nkv, nh, S, r_k, r_v)
    assert torch.allclose(oracle.input_checksums(q, k, v, u_k), d["checksums"], rtol=1e-12, atol=0), \
        "regenerated inputs differ from the fixture's"
    cos, sin, cs = _tables(S, cuda)
    out = _run(q.to(cuda, torch.bfloat16), k.to(cuda, torch.bfloat16), v.to(cuda, torch.bfloat16),
               u_k.to(cuda), None, d["cur_pos"], cs, torch.float32)
    torch.cuda.synchronize()
    _close(out.cpu(), d["out"], "long-context golden")
