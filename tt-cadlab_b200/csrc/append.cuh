// Small bandwidth kernels around the decode op:
//  * palu_append_kernel: write one decode step's latents into the caches at cur_pos[b], contiguous or
//    through a page table (the reference's paged_update_cache calls, attention.py:612-625);
//  * palu_pack_cs_kernel: turn the reference's [S, 256] [cos | sin] table (pair-duplicated,
//    Meta-interleaved, fused.py:62-73) into the packed 256-byte rows the decode kernels read (half the
//    bytes): per row, 4 blocks of 16 frequencies, each block 16 fp16 cosines then their 16 sines. One
//    block is one 64-byte TMA row segment, and consecutive frequencies sit side by side so that the
//    rotation runs on two frequencies per packed half2 instruction. fp16 holds every bf16 table value
//    exactly (|cos|, |sin| <= 1; below 6e-5 fp16 is subnormal, an absolute error under 3e-8).
#pragma once
#include <cuda_fp16.h>

#include "palu_common.cuh"

namespace palu {

struct AppendParams {
  const __nv_bfloat16* new_k;  // [B][n_groups][r_k]
  const __nv_bfloat16* new_v;  // [B][n_groups][r_v]
  const int32_t* cur_pos;      // [B]
  __nv_bfloat16* k_cache;      // [B][n_groups][max_seq][r_k]
  __nv_bfloat16* v_cache;      // [B][n_groups][max_seq][r_v]
  int batch, n_groups, r_k, r_v, max_seq;
  // Paged caches (null page_table: the layouts above): position pos of row b goes to row pos % bs of
  // block page_table[b * table_ld + pos / bs] of [n_blocks][n_groups][bs][r] (bs = 1 << blk_shift).
  const int32_t* page_table;
  int table_ld, blk_shift, n_blocks;
};

// One thread per 16-byte chunk of the step's K and V latents.
__global__ void palu_append_kernel(const AppendParams p) {
  const int kc = p.r_k / 8, vc = p.r_v / 8, per = kc + vc;
  const long total = (long)p.batch * p.n_groups * per;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % per);
    const long bg = i / per;
    const int b = (int)(bg / p.n_groups);
    const int pos = p.cur_pos[b];
    if (pos < 0 || pos >= p.max_seq) continue;
    long row = bg * p.max_seq + pos;  // cache row, in rows of r elements
    if (p.page_table) {
      const int e = p.page_table[(long)b * p.table_ld + (pos >> p.blk_shift)];
      if ((unsigned)e >= (unsigned)p.n_blocks) continue;  // an entry outside the caches drops the write
      row = (((long)e * p.n_groups + (bg - (long)b * p.n_groups)) << p.blk_shift) + (pos & ((1 << p.blk_shift) - 1));
    }
    if (c < kc) {
      const uint4 v = reinterpret_cast<const uint4*>(p.new_k + bg * p.r_k)[c];
      reinterpret_cast<uint4*>(p.k_cache + row * p.r_k)[c] = v;
    } else {
      const uint4 v = reinterpret_cast<const uint4*>(p.new_v + bg * p.r_v)[c - kc];
      reinterpret_cast<uint4*>(p.v_cache + row * p.r_v)[c - kc] = v;
    }
  }
}

// cs_tab row s: cos at columns 2j (== 2j+1), sin at 128 + 2j. in_f32 selects an fp32 table
// (rounded to bf16 here) instead of bf16. Output word w of row s (w = 16 blk + x):
// x < 8: (cos f0, cos f0+1), x >= 8: (sin f1, sin f1+1), f0 = 16 blk + 2x, f1 = f0 - 16 (low half first).
__global__ void palu_pack_cs_kernel(const void* cs_tab, long ld, int in_f32, uint32_t* out, int rows) {
  const long total = (long)rows * 64;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long s = i >> 6;
    const int w = (int)(i & 63), x = w & 15;
    const int f = (w & ~15) + 2 * (x & 7);       // first of the word's two frequencies
    const int col = (x < 8 ? 0 : kHeadDim) + 2 * f;  // cos_f at 2f, sin_f at 128 + 2f
    float a, bv;
    if (in_f32) {
      const float* r = reinterpret_cast<const float*>(cs_tab) + s * ld;
      a = r[col];
      bv = r[col + 2];
    } else {
      const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(cs_tab) + s * ld;
      a = __bfloat162float(r[col]);
      bv = __bfloat162float(r[col + 2]);
    }
    const __half2 h = __floats2half2_rn(a, bv);
    out[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
}

}  // namespace palu
