"""Chunk-relative RoPE (the reference op's Phase 2, palu_tt/fused.py:1-14) on the GPU.

Passing ``rot_step`` and ``trans_mat`` to ``palu_sdpa_decode`` selects Phase 2: key position p = 128 t + j
is rotated by the table's row j and the query of chunk t back by row 128 t, so the key sees the rotation
R_{128 t} R_j. Its oracle is the reference's fp32 model (``reference_decode``, fused.py:82-107) run on the
effective table of that rule (``oracle.phase2_tables``: the composition in fp32 of the same table values).

Bar: the north star's, max-abs relative <= 2e-2 and mean-abs relative <= 1e-3, on the fp32 output per
(batch row, query head) row and globally, and on the bf16 output globally against the oracle rounded to bf16.

Cases: the bench workload at full size (every row), BASELINE config 3 (rank-256 G-LRD on the one-pipeline
kernel), a config-5 cell at 128k positions, ragged rows and a cache shorter than one chunk, paged caches
(bit-identical to the contiguous op), fp8 and fp4 caches (on their dequantized values). With an fp32 table
the chunk-relative op also meets the bar against the plain (Phase 1) oracle on that table, and the mma.sync
kernel, which has no chunk-relative form, refuses the call.
"""
import pytest
import torch

import oracle
from oracle import f4 as of4
from oracle import f8 as of8
from tests.test_parity_configs import LLAMA3, SCALE, THETA, _close, _gpu_case, _tables

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _absolute_afterwards():
    """The RoPE form is per host thread: later tests that call the C ABI directly expect the default."""
    yield
    from palu_b200 import _lib
    _lib.set_rope_mode(_lib.PALU_ROPE_ABSOLUTE)


def _phase2_kw(cos, sin, dev):
    from palu_b200 import fused
    # the reference builds rot_step for its chunk; only its presence selects Phase 2 here
    return {"rot_step": fused.rot_step_table(cos, sin, min(128, cos.shape[0] - 1)).to(dev),
            "trans_mat": fused.trans_mat_tile()}


def _run(q, k, v, u_k, u_v, pos, cs, cos, sin, out_dtype, page_table=None):
    from palu_b200 import fused
    w_rot = fused.w_rot_from_u_k(u_k.float()).to(torch.bfloat16)[None]
    width = 128 if u_v is not None else v.shape[-1]
    kw = {} if page_table is None else {"page_table_tensor": page_table}
    return fused.palu_sdpa_decode(q, k, w_rot, cs, v, width, pos.to(q.device), scale=SCALE,
                                  u_v=None if u_v is None else u_v[None], out_dtype=out_dtype, check_status=True,
                                  **_phase2_kw(cos, sin, q.device), **kw)


def _oracle(q, k, v, u_k, u_v, pos, cos, sin, rows, group_size):
    r = torch.tensor(rows)
    c2, s2 = oracle.phase2_tables(cos, sin)
    return oracle.reference_decode_streamed(
        q[:, r].float().cpu(), k[r].float().cpu(), u_k.float().cpu(), v[r].float().cpu(), pos[r], c2, s2, SCALE,
        u_v=None if u_v is None else u_v.float().cpu(), group_size=group_size)


def _check(dev, seed, B, n_kv, n_lat, S, r_k, r_v, rows, *, grouped=False, full_rows=False, name=""):
    q, k, v, u_k, u_v, pos = _gpu_case(dev, seed, B, n_kv, n_lat, S, r_k, r_v, grouped=grouped, full_rows=full_rows)
    cos, sin, cs = _tables(S, dev)
    out32 = _run(q, k, v, u_k, u_v, pos, cs, cos, sin, torch.float32)
    out16 = _run(q, k, v, u_k, u_v, pos, cs, cos, sin, torch.bfloat16)
    torch.cuda.synchronize()
    ref = _oracle(q, k, v, u_k, u_v, pos, cos, sin, rows, n_kv // n_lat)
    r = torch.tensor(rows)
    _close(out32[:, r].cpu(), ref, f"{name} fp32 output")
    _close(out16[:, r].float().cpu(), ref.to(torch.bfloat16).float(), f"{name} bf16 output", per_row=False)


def test_bench_workload_mlrd_r64_b32_s8192(cuda):
    """BASELINE's target row at full size, every batch row."""
    _check(cuda, 201, 32, 8, 8, 8192, 64, 64, list(range(32)), full_rows=True, name="phase2 mlrd_r64_b32_s8192")


def test_glrd_gs4_r256_b16_s16384(cuda):
    """BASELINE config 3 on the one-pipeline kernel (both RoPE halves side by side on 8 warps)."""
    _check(cuda, 202, 16, 8, 2, 16384, 256, 256, [0, 7, 15], grouped=True, name="phase2 glrd_gs4_r256")


def test_sweep_cell_b1_s128k(cuda):
    """BASELINE config 5's r_k 32 / r_v 128 layer at 131072 positions (1024 chunks of query rotation)."""
    _check(cuda, 203, 1, 8, 8, 131072, 32, 128, [0], name="phase2 sweep_b1_s128k")
    torch.cuda.empty_cache()


@pytest.mark.parametrize("S,pos", [(100, [0, 50, 99, 7, 63]), (1500, [1499, 0, 127, 128, 1000])],
                         ids=["short_cache", "ragged"])
def test_ragged_rows_and_short_cache(cuda, S, pos):
    """Rows ending inside, at and just past a chunk boundary; a cache shorter than one chunk (rows past the
    table are the TMA's zero fill, all of them masked)."""
    B = len(pos)
    q, k, v, u_k, u_v, _ = _gpu_case(cuda, 204 + S, B, 8, 8, S, 64, 64)
    p = torch.tensor(pos, dtype=torch.int32)
    cos, sin, cs = _tables(S, cuda)
    out = _run(q, k, v, u_k, u_v, p, cs, cos, sin, torch.float32)
    torch.cuda.synchronize()
    _close(out.cpu(), _oracle(q, k, v, u_k, u_v, p, cos, sin, list(range(B)), 1), f"phase2 S={S}")


def test_paged_equals_contiguous(cuda):
    """Paged caches (blocks of 32, a shuffled page table): bit-identical to the contiguous Phase 2 op."""
    B, S, bs = 4, 2048, 32
    q, k, v, u_k, u_v, pos = _gpu_case(cuda, 205, B, 8, 8, S, 64, 64)
    cos, sin, cs = _tables(S, cuda)
    ref = _run(q, k, v, u_k, u_v, pos, cs, cos, sin, torch.float32)
    per_row = S // bs
    g = torch.Generator(device=cuda).manual_seed(7)
    pt = torch.randperm(B * per_row, generator=g, device=cuda).view(B, per_row).to(torch.int32)

    def paged(c):
        out = torch.empty(B * per_row, c.shape[1], bs, c.shape[-1], dtype=c.dtype, device=cuda)
        out[pt.long().view(-1)] = c.view(B, c.shape[1], per_row, bs, c.shape[-1]).transpose(1, 2).reshape(
            -1, c.shape[1], bs, c.shape[-1])
        return out

    got = _run(q, paged(k), paged(v), u_k, u_v, pos, cs, cos, sin, torch.float32, page_table=pt)
    torch.cuda.synchronize()
    assert torch.equal(got, ref), "paged Phase 2 output differs from the contiguous op"


@pytest.mark.parametrize("fmt", ["f8", "f4"])
def test_low_bit_caches_on_dequantized_values(cuda, fmt):
    """fp8 / fp4 caches: the Phase 2 op against the Phase 2 oracle on the dequantized caches."""
    from palu_b200 import fused
    B, S = 4, 3000
    q, k, v, u_k, u_v, pos = _gpu_case(cuda, 206, B, 8, 8, S, 64, 64)
    quant = fused.quantize_latents_f4 if fmt == "f4" else fused.quantize_latents_f8
    deq = of4.dequantize_rows if fmt == "f4" else of8.dequantize_rows
    kc, vc = quant(k), quant(v)
    kd, vd = deq(kc.codes.cpu(), kc.exp.cpu()), deq(vc.codes.cpu(), vc.exp.cpu())
    cos, sin, cs = _tables(S, cuda)
    w_rot = fused.w_rot_from_u_k(u_k.float()).to(torch.bfloat16)[None]
    out = fused.palu_sdpa_decode(q, kc, w_rot, cs, vc, 64, pos.to(cuda), scale=SCALE, out_dtype=torch.float32,
                                 check_status=True, **_phase2_kw(cos, sin, cuda))
    torch.cuda.synchronize()
    ref = _oracle(q, kd, vd, u_k, None, pos, cos, sin, list(range(B)), 1)
    _close(out.cpu(), ref, f"phase2 {fmt} caches")


def test_fp32_table_meets_the_bar_against_the_plain_oracle(cuda):
    """With an fp32 table (packed to fp16 by the library) the chunk-relative rotation is the exact RoPE
    within the table's rounding: the Phase 2 op meets the bar against the Phase 1 oracle on that table."""
    from palu_b200 import fused
    B, S = 8, 8192
    q, k, v, u_k, u_v, pos = _gpu_case(cuda, 207, B, 8, 8, S, 64, 64, full_rows=True)
    cos, sin = oracle.cos_sin_tables(128, S, THETA, LLAMA3)
    cos, sin = cos[:S].float(), sin[:S].float()
    cs = fused.cs_table(cos, sin, S)[None, None].to(cuda)
    out = _run(q, k, v, u_k, u_v, pos, cs, cos, sin, torch.float32)
    torch.cuda.synchronize()
    r = torch.arange(B)
    ref = oracle.reference_decode_streamed(q.float().cpu(), k.float().cpu(), u_k.float().cpu(), v.float().cpu(),
                                           pos, cos, sin, SCALE)
    _close(out[:, r].cpu(), ref, "phase2 on an fp32 table vs the Phase 1 oracle")


def test_mma_kernel_refuses_the_chunk_relative_form(cuda):
    from palu_b200 import _lib
    q, k, v, u_k, u_v, pos = _gpu_case(cuda, 208, 2, 8, 8, 512, 64, 64)
    cos, sin, cs = _tables(512, cuda)
    _lib.set_kernel(_lib.PALU_KERNEL_MMA)
    try:
        with pytest.raises(RuntimeError, match="chunk-relative"):
            _run(q, k, v, u_k, u_v, pos, cs, cos, sin, torch.float32)
    finally:
        _lib.set_kernel(_lib.PALU_KERNEL_AUTO)
