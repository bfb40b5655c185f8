// Shared device helpers for the Palu decode kernels (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define PALU_DEVINL __device__ __forceinline__

namespace palu {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kHeadDim = 128;

PALU_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global->shared copy; bytes beyond src_bytes (0 or 16) are zero-filled.
PALU_DEVINL void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
PALU_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
PALU_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

PALU_DEVINL void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
PALU_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
PALU_DEVINL void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// D += A * B, m16n8k16, bf16 inputs, fp32 accumulate.
PALU_DEVINL void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Packed RoPE table rows (palu_pack_cs_kernel): 128 fp16 per position, 4 blocks of 16 frequencies,
// each block 16 cosines then the same 16 frequencies' sines. Element index of cos / sin of frequency f:
PALU_DEVINL int packed_cos_index(int f) { return 32 * (f >> 4) + (f & 15); }
PALU_DEVINL int packed_sin_index(int f) { return 32 * (f >> 4) + 16 + (f & 15); }

// Two fp32 -> packed bf16x2 (round to nearest even); x0 in the low half.
PALU_DEVINL uint32_t pack_bf16(float x0, float x1) {
  __nv_bfloat162 v = __floats2bfloat162_rn(x0, x1);
  return *reinterpret_cast<uint32_t*>(&v);
}
// hi = bf16(x), lo = bf16(x - hi): hi + lo carries ~16 significant bits of x.
PALU_DEVINL void split_bf16(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  float2 hf = __bfloat1622float2(h);
  __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
  hi = *reinterpret_cast<uint32_t*>(&h);
  lo = *reinterpret_cast<uint32_t*>(&l);
}
PALU_DEVINL float2 unpack_bf16(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// Partial records of the tcgen05 decode (decode_tc.cuh: one CTA per (tile range, KV head), two groups
// per CTA, or one for latents wider than 128, whose second record of each pair stays unused): a batch row
// wholly inside one CTA has a direct pair (one record per group); a CTA's first
// segment, when its row began in an earlier CTA (side 0), and its last segment, when its row continues in
// a later one (side 1), have the CTA's edge pairs. Each record: O [rep][r_v] and (m, l x 4) [rep][5].
__host__ __device__ inline size_t tc_rec_direct(int b, int kvh, int n_kv, int g) {
  return ((size_t)b * n_kv + kvh) * 2 + g;
}
__host__ __device__ inline size_t tc_rec_edge(int batch, int n_kv, int ctas, int kvh, int c, int side, int g) {
  return (size_t)batch * n_kv * 2 + (((size_t)kvh * ctas + c) * 2 + side) * 2 + g;
}
__host__ __device__ inline size_t tc_n_records(int batch, int n_kv, int ctas) {
  return (size_t)batch * n_kv * 2 + (size_t)n_kv * ctas * 4;
}
// 128-token tiles of a row that attends positions 0..cur_pos (clamped to [0, max_seq)).
PALU_DEVINL int tc_row_tiles(const int32_t* cur_pos, int b, int max_seq) {
  int L = cur_pos[b] + 1;
  L = L < 0 ? 0 : (L > max_seq ? max_seq : L);
  return (L + 127) / 128;
}

PALU_DEVINL float fast_exp2(float x) {  // ex2.approx: exp2(-inf) = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace palu
