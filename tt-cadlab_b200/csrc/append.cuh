// Small bandwidth kernels around the decode op:
//  * palu_append_kernel: write one decode step's latents into the caches at cur_pos[b], contiguous or
//    through a page table (the reference's paged_update_cache calls, attention.py:612-625);
//  * palu_pack_cs_kernel: turn the reference's [S, 256] [cos | sin] table (pair-duplicated,
//    Meta-interleaved, fused.py:62-73) into the packed 256-byte rows the decode kernels read (half the
//    bytes): per row, 4 blocks of 16 frequencies, each block 16 fp16 cosines then their 16 sines. One
//    block is one 64-byte TMA row segment, and consecutive frequencies sit side by side so that the
//    rotation runs on two frequencies per packed half2 instruction. fp16 holds every bf16 table value
//    exactly (|cos|, |sin| <= 1; below 6e-5 fp16 is subnormal, an absolute error under 3e-8).
//  * palu_quantize_f8_kernel: fp8 latent caches (the B200 form of the reference's block-float bfp8 latent
//    caches, attention.py:159-169): each row of r latent values (one position of one latent head) becomes
//    r e4m3 codes and one power-of-two exponent k, value = code * 2^k. k is the smallest integer with
//    amax <= 448 * 2^k (448 = the largest e4m3 value), kept in [-120, 7]; scaling by 2^-k is exact, the codes
//    round to nearest even with saturation, and codes below the smallest normal e4m3 value (exponent
//    field 0) are flushed to a signed zero, so every stored code converts to bf16 by moving bit fields.
//  * palu_quantize_f4_kernel: fp4 latent caches (the B200 form of the reference's bfp4 latent caches): e2m1
//    codes, two per byte (the first value in the low nibble), with one power-of-two exponent per block of 16
//    values: k is the smallest integer with max|block| <= 6 * 2^k (6 = the largest e2m1 value), kept in
//    [-120, 7]; the codes are the block times 2^-k rounded to nearest even with saturation.
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

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

// ---- fp8 latent rows ---------------------------------------------------------------------------------
struct QuantF8Params {
  const __nv_bfloat16* src;  // rows of r bf16 values
  long rows;                 // rows to quantize
  int r;                     // values per row (<= 256)
  uint8_t* codes;            // destination rows of r e4m3 codes
  int8_t* exps;              // destination exponents, one per row
  // Append mode (cur_pos set): source row i = (b, latent head) = (i / n_groups, i % n_groups) goes to
  // destination row i * max_seq + cur_pos[b]; rows with cur_pos outside [0, max_seq) are skipped.
  const int32_t* cur_pos;
  int n_groups, max_seq;
};

// The row exponent: the smallest k with amax <= 448 * 2^k, kept in [-120, 7] (0 for an all-zero row). With
// amax = m * 2^e, m in [0.5, 1): 448 * 2^k = 0.875 * 2^(k + 9), so k = e - 9 when m <= 0.875, else e - 8.
PALU_DEVINL int f8_row_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  int e;
  const float m = frexpf(amax, &e);
  const int k = m <= 0.875f ? e - 9 : e - 8;
  return k > 7 ? 7 : (k < -120 ? -120 : k);
}
PALU_DEVINL uint8_t f8_code(float y) {
  uint8_t c = (uint8_t)__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
  return (c & 0x78) ? c : (uint8_t)(c & 0x80);  // exponent field 0: flush to a signed zero
}

// One warp per row: lane l holds values l, l + 32, ... (up to 8).
__global__ void palu_quantize_f8_kernel(const QuantF8Params p) {
  const int lane = threadIdx.x & 31;
  const long warps = (long)gridDim.x * (blockDim.x >> 5);
  for (long i = blockIdx.x * (long)(blockDim.x >> 5) + (threadIdx.x >> 5); i < p.rows; i += warps) {
    long dst = i;
    if (p.cur_pos) {
      const int pos = p.cur_pos[i / p.n_groups];
      if (pos < 0 || pos >= p.max_seq) continue;
      dst = i * p.max_seq + pos;
    }
    float x[8];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int d = lane + 32 * c;
      x[c] = d < p.r ? __bfloat162float(p.src[i * p.r + d]) : 0.f;
      amax = fmaxf(amax, fabsf(x[c]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const int k = f8_row_exponent(amax);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int d = lane + 32 * c;
      if (d < p.r) p.codes[dst * p.r + d] = f8_code(ldexpf(x[c], -k));
    }
    if (lane == 0) p.exps[dst] = (int8_t)k;
  }
}

// ---- fp4 latent rows -----------------------------------------------------------------------------------
struct QuantF4Params {
  const __nv_bfloat16* src;  // rows of r bf16 values
  long rows;
  int r;                     // values per row: a multiple of 16, <= 256
  uint8_t* codes;            // destination rows of r / 2 bytes
  int8_t* exps;              // destination rows of r / 16 block exponents
  const int32_t* cur_pos;    // append mode, as QuantF8Params
  int n_groups, max_seq;
};

// amax = m * 2^e, m in [0.5, 1): 6 * 2^k = 0.75 * 2^(k + 3), so k = e - 3 when m <= 0.75, else e - 2.
PALU_DEVINL int f4_block_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  int e;
  const float m = frexpf(amax, &e);
  const int k = m <= 0.75f ? e - 3 : e - 2;
  return k > 7 ? 7 : (k < -120 ? -120 : k);
}

// One warp per row: lane l holds the value pairs 2 (l + 32 c), 2 (l + 32 c) + 1; a block of 16 values is 8 lanes.
__global__ void palu_quantize_f4_kernel(const QuantF4Params p) {
  const int lane = threadIdx.x & 31;
  const long warps = (long)gridDim.x * (blockDim.x >> 5);
  for (long i = blockIdx.x * (long)(blockDim.x >> 5) + (threadIdx.x >> 5); i < p.rows; i += warps) {
    long dst = i;
    if (p.cur_pos) {
      const int pos = p.cur_pos[i / p.n_groups];
      if (pos < 0 || pos >= p.max_seq) continue;
      dst = i * p.max_seq + pos;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int pr = lane + 32 * c, d0 = 2 * pr;  // value pair index, first value
      const bool in = d0 < p.r;
      const float x0 = in ? __bfloat162float(p.src[i * p.r + d0]) : 0.f;
      const float x1 = in ? __bfloat162float(p.src[i * p.r + d0 + 1]) : 0.f;
      float amax = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
      for (int o = 4; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const int k = f4_block_exponent(amax);
      if (in) {
        p.codes[dst * (p.r / 2) + pr] = (uint8_t)__nv_cvt_float2_to_fp4x2(make_float2(ldexpf(x0, -k), ldexpf(x1, -k)),
                                                                          __NV_E2M1, cudaRoundNearest);
        if ((lane & 7) == 0) p.exps[dst * (p.r / 16) + (pr >> 3)] = (int8_t)k;
      }
    }
  }
}

}  // namespace palu

namespace palu {

// One decode step's q rotation and latent append in one pass over the step's fused projection output
// (the reference's nlp_create_qkv_heads_decode split, rotary_embedding_llama on q and the two
// paged_update_cache calls, attention.py:601-625).
struct RopeAppendParams {
  const void* qkv;        // [B][ld] bf16 or f32: n_q * 128 q values (Meta pair order), then n_groups * r_k
                          // K latents, then n_groups * r_v V latents
  long ld;
  const float* cos;       // [>= max_seq][128] fp32: cos of frequency j at columns 2j and 2j + 1
  const float* sin;       // the same layout
  const int32_t* cur_pos; // [B]
  __nv_bfloat16* q_out;   // [B][n_q][128]
  __nv_bfloat16* k_cache; // as AppendParams (contiguous or paged)
  __nv_bfloat16* v_cache;
  int batch, n_q, n_groups, r_k, r_v, max_seq;
  const int32_t* page_table;
  int table_ld, blk_shift, n_blocks;
};

template <typename T>
PALU_DEVINL float load_f32(const T* p, long i);
template <>
PALU_DEVINL float load_f32<float>(const float* p, long i) { return p[i]; }
template <>
PALU_DEVINL float load_f32<__nv_bfloat16>(const __nv_bfloat16* p, long i) { return __bfloat162float(p[i]); }

// Items per batch row: n_q * 64 q pairs, then n_groups * (r_k + r_v) latent elements. The q rotation is
// out(2j) = x(2j) cos(2j) + (-x(2j+1)) sin(2j), out(2j+1) = x(2j+1) cos(2j+1) + x(2j) sin(2j+1) with each
// product and the sum rounded separately (no fused multiply-add), at cur_pos clamped to [0, max_seq), the
// decode op's clamp. Latents are appended at cur_pos; rows outside [0, max_seq) append nothing.
template <typename T>
__global__ void palu_rope_q_append_kernel(const RopeAppendParams p) {
  const T* qkv = static_cast<const T*>(p.qkv);
  const int qp = p.n_q * 64, nk = p.n_groups * p.r_k, per = qp + nk + p.n_groups * p.r_v;
  const long total = (long)p.batch * per;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int b = (int)(i / per), e = (int)(i - (long)b * per);
    const long row = (long)b * p.ld;
    const int pos = p.cur_pos[b];
    if (e < qp) {
      const int h = e >> 6, j = e & 63, d = h * 128 + 2 * j;
      const int pr = pos < 0 ? 0 : (pos >= p.max_seq ? p.max_seq - 1 : pos);
      const float x0 = load_f32(qkv, row + d), x1 = load_f32(qkv, row + d + 1);
      const float* c = p.cos + (long)pr * 128 + 2 * j;
      const float* s = p.sin + (long)pr * 128 + 2 * j;
      const float o0 = __fadd_rn(__fmul_rn(x0, c[0]), __fmul_rn(-x1, s[0]));
      const float o1 = __fadd_rn(__fmul_rn(x1, c[1]), __fmul_rn(x0, s[1]));
      __nv_bfloat162 o;
      o.x = __float2bfloat16_rn(o0);
      o.y = __float2bfloat16_rn(o1);
      *reinterpret_cast<__nv_bfloat162*>(p.q_out + ((long)b * p.n_q + h) * 128 + 2 * j) = o;
      continue;
    }
    if (pos < 0 || pos >= p.max_seq) continue;
    const int el = e - qp;
    const bool is_k = el < nk;
    const int r = is_k ? p.r_k : p.r_v, x = is_k ? el : el - nk, g = x / r, c = x - g * r;
    long crow = ((long)b * p.n_groups + g) * p.max_seq + pos;
    if (p.page_table) {
      const int blk = p.page_table[(long)b * p.table_ld + (pos >> p.blk_shift)];
      if ((unsigned)blk >= (unsigned)p.n_blocks) continue;  // an entry outside the caches drops the write
      crow = (((long)blk * p.n_groups + g) << p.blk_shift) + (pos & ((1 << p.blk_shift) - 1));
    }
    const __nv_bfloat16 v = __float2bfloat16_rn(load_f32(qkv, row + p.n_q * 128 + el));
    (is_k ? p.k_cache : p.v_cache)[crow * r + c] = v;
  }
}

}  // namespace palu

namespace palu {

// Decoder elementwise steps around the attention layer (the stock RMSNorm and SwiGLU MLP that the
// reference's model assembles, palu_tt/model.py:52-95), fused so that one decode step launches fewer kernels.

// Residual add + RMSNorm, one CTA per row: h += delta (fp32 or bf16, in place; delta may be null), then
// out = bf16(h * rsqrt(mean(h^2) + eps) * w). dim is a multiple of 4.
constexpr int kNormThreads = 512;
PALU_DEVINL float4 load4(const float* p, int i) { return reinterpret_cast<const float4*>(p)[i]; }
PALU_DEVINL float4 load4(const __nv_bfloat16* p, int i) {
  const uint2 u = reinterpret_cast<const uint2*>(p)[i];
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <typename TD>
__global__ void __launch_bounds__(kNormThreads) palu_add_rms_norm_kernel(float* h, const TD* delta, const float* w,
                                                                          __nv_bfloat16* out, int dim, float eps) {
  __shared__ float s_part[kNormThreads / 32];
  const long row = blockIdx.x;
  float4* hr = reinterpret_cast<float4*>(h + row * dim);
  const TD* dr = delta ? delta + row * dim : nullptr;
  const int n4 = dim / 4;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n4; i += kNormThreads) {
    float4 x = hr[i];
    if (dr) {
      const float4 d = load4(dr, i);
      x.x += d.x;
      x.y += d.y;
      x.z += d.z;
      x.w += d.w;
      hr[i] = x;
    }
    ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kNormThreads / 32 ? s_part[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) s_part[0] = rsqrtf(v / dim + eps);
  }
  __syncthreads();
  const float inv = s_part[0];
  const float4* wr = reinterpret_cast<const float4*>(w);
  __nv_bfloat162* orow = reinterpret_cast<__nv_bfloat162*>(out + row * dim);
  for (int i = threadIdx.x; i < n4; i += kNormThreads) {
    const float4 x = hr[i], g = wr[i];
    orow[2 * i] = __floats2bfloat162_rn(x.x * inv * g.x, x.y * inv * g.y);
    orow[2 * i + 1] = __floats2bfloat162_rn(x.z * inv * g.z, x.w * inv * g.w);
  }
}

// SwiGLU on the gate/up GEMM output: gu [rows][ld] bf16 holds gate (columns 0..f-1) then up (f..2f-1);
// out[r][i] = bf16(bf16(silu(gate)) * up), the rounding of a silu kernel followed by a multiply kernel.
PALU_DEVINL __nv_bfloat16 swiglu1(__nv_bfloat16 gate, __nv_bfloat16 up) {
  const float g = __bfloat162float(gate);
  const float a = __bfloat162float(__float2bfloat16_rn(g / (1.0f + expf(-g))));
  return __float2bfloat16_rn(a * __bfloat162float(up));
}
__global__ void palu_swiglu_kernel(const __nv_bfloat16* gu, long ld, int f, __nv_bfloat16* out, int rows) {
  const long total = (long)rows * f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / f;
    const int c = (int)(i - r * f);
    out[i] = swiglu1(gu[r * ld + c], gu[r * ld + f + c]);
  }
}
// The same with 8 columns per thread (16-byte loads and stores): row blockIdx.y, f and ld multiples of 8,
// gu and out 16-byte aligned.
__global__ void palu_swiglu8_kernel(const __nv_bfloat16* gu, long ld, int f, __nv_bfloat16* out) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 * 8 >= f) return;
  const long r = blockIdx.y;
  const uint4 gv = reinterpret_cast<const uint4*>(gu + r * ld)[c8];
  const uint4 uv = reinterpret_cast<const uint4*>(gu + r * ld + f)[c8];
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&gv);
  const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uv);
  uint4 ov;
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = swiglu1(g[k], u[k]);
  reinterpret_cast<uint4*>(out + r * f)[c8] = ov;
}

}  // namespace palu
