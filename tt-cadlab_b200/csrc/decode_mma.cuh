// Split-K flash-decode over Palu latent caches, warp-level tensor-core path (mma.sync m16n8k16).
//
// One CTA owns (batch row b, KV head h, split s): a contiguous range of 64-token tiles of the
// positions 0..cur_pos[b]. Per tile, each of the 4 warps takes 16 tokens and
//   1. rebuilds K = lat_k @ U_k (16 x 128, fp32 accumulators) on the tensor cores,
//   2. applies RoPE in registers from the packed (cos, sin) table: each accumulator fragment keeps a
//      frequency pair (columns 2j, 2j+1) inside one thread,
//   3. scores the group's query heads against K_rot on the tensor cores, with K_rot split into two
//      bf16 terms (hi + lo) so the product keeps ~16 significant bits,
//   4. runs an online softmax per warp (exp2 domain),
//   5. accumulates O^T += lat_v^T @ P on the tensor cores, P again split hi + lo.
// The warps merge their (O, m, l) in shared memory and the CTA writes one partial; the combine
// kernel (combine.cuh) merges the splits. K and V are never written to global memory.
//
// RECON = false is plain GQA flash-decode over an already-rotated full K cache (the identity
// comparison path): the K tile feeds step 3 directly.
//
// The semantics follow the reference's fp32 model of palu_sdpa_decode (palu_tt/fused.py:82-107):
// query head qh attends KV head qh / rep; position p is visible iff p <= cur_pos[b].
#pragma once
#include <cuda_fp16.h>

#include "palu_common.cuh"

namespace palu {

struct DecodeParams {
  const __nv_bfloat16* q;   // [B][n_q][128], already rotated
  const __nv_bfloat16* k;   // RECON: [B][n_groups][max_seq][rk]; plain: [B][n_kv][max_seq][128] (rotated)
  const __nv_bfloat16* v;   // [B][n_groups][max_seq][rv]
  const __nv_bfloat16* u_k; // [n_kv][rk] rows of ld_u elements (first 128 used); RECON only
  const uint32_t* cs;       // [max_seq][64] words: packed table rows (append.cuh); RECON only
  const int32_t* cur_pos;   // [B]
  float* ws_o;              // [B][n_kv][splits][rep][rv]
  float* ws_ml;             // [B][n_kv][splits][rep][2]  (m in log2 units, l)
  int batch, n_q, n_kv, n_groups, rk, rv, max_seq, splits, ld_u, rep;
  float scale_log2;         // softmax scale * log2(e)
  // Paged caches (null page_table: the contiguous layouts above): row b's position t sits at row t % bs of
  // physical block page_table[b * table_ld + t / bs] (bs = 1 << blk_shift) of [n_blocks][n_lat][bs][r].
  const int32_t* page_table;
  int table_ld, blk_shift, n_blocks;
};

constexpr int kMmaThreads = 128;
constexpr int kMmaTile = 64;     // tokens per pipeline stage (16 per warp)
constexpr int kCsLd = 68;        // packed-table smem row stride (words): 64 pairs + 4 pad, conflict-free
constexpr int kULd = 136;        // U_k smem row stride (bf16): 128 + 8 pad

template <int RV16, bool RECON>
struct MmaSmem {
  int rk;
  __host__ __device__ explicit MmaSmem(int rk_) : rk(RECON ? rk_ : 128) {}
  __host__ __device__ int ldk() const { return rk + 8; }
  static constexpr int ldv = RV16 * 16 + 8;
  __host__ __device__ int u_bytes() const { return RECON ? rk * kULd * 2 : 0; }
  __host__ __device__ int k_bytes() const { return kMmaTile * ldk() * 2; }
  static constexpr int v_bytes = kMmaTile * ldv * 2;
  static constexpr int t_bytes = RECON ? kMmaTile * kCsLd * 4 : 0;
  __host__ __device__ int stage_bytes() const { return k_bytes() + v_bytes + t_bytes; }
  static constexpr int p_bytes = 4 * 8 * 24 * 2;
  __host__ __device__ int total(int ns) const { return u_bytes() + ns * stage_bytes() + p_bytes; }
};

template <int RV16, bool RECON, int NS>
__global__ void __launch_bounds__(kMmaThreads, 2) palu_decode_mma_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const MmaSmem<RV16, RECON> lay(p.rk);
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int rk = lay.rk;
  constexpr int rv = RV16 * 16;
  const int ldk = lay.ldk();
  constexpr int ldv = MmaSmem<RV16, RECON>::ldv;
  const int group = RECON ? kvh / (p.n_kv / p.n_groups) : kvh;
  const int n_lat = RECON ? p.n_groups : p.n_kv;

  int L = p.cur_pos[b] + 1;
  L = L < 0 ? 0 : (L > p.max_seq ? p.max_seq : L);
  const int n_tiles = (L + kMmaTile - 1) / kMmaTile;
  const int per = (n_tiles + p.splits - 1) / p.splits;
  const int tile0 = split * per;
  const int tile1 = min(n_tiles, tile0 + per);
  const int my_tiles = max(0, tile1 - tile0);

  const __nv_bfloat16* k_base = p.k + (size_t)(b * n_lat + group) * p.max_seq * rk;
  const __nv_bfloat16* v_base = p.v + (size_t)(b * n_lat + group) * p.max_seq * rv;

  unsigned char* sU = smem;
  unsigned char* sStages = smem + lay.u_bytes();
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(sStages + NS * lay.stage_bytes()) + warp * 8 * 24;

  // Cache row of position tok (tok < L), as an offset in rows of r elements; -1 for a page-table entry
  // outside [0, n_blocks), whose rows are read as zeros.
  const int32_t* page_row = p.page_table ? p.page_table + (size_t)b * p.table_ld : nullptr;
  auto cache_row = [&](int tok) -> long {
    if (!page_row) return tok;
    const int e = __ldg(page_row + (tok >> p.blk_shift));
    if ((unsigned)e >= (unsigned)p.n_blocks) return -1;
    return (((long)e * n_lat + group) << p.blk_shift) + (tok & ((1 << p.blk_shift) - 1));
  };
  const __nv_bfloat16* k_rows = page_row ? p.k : k_base;
  const __nv_bfloat16* v_rows = page_row ? p.v : v_base;

  auto load_tile = [&](int tile, int stage) {
    unsigned char* st = sStages + stage * lay.stage_bytes();
    const uint32_t sK = smem_u32(st), sV = smem_u32(st + lay.k_bytes());
    const int row0 = tile * kMmaTile;
    const int kc = rk / 8;
    for (int c = tid; c < kMmaTile * kc; c += kMmaThreads) {
      const int r = c / kc, col = c - r * kc, tok = row0 + r;
      const long cr = tok < L ? cache_row(tok) : -1;
      const bool ok = cr >= 0;
      cp_async16(sK + (r * ldk + col * 8) * 2, k_rows + (size_t)(ok ? cr : 0) * rk + col * 8, ok ? 16 : 0);
    }
    constexpr int vc = rv / 8;
    for (int c = tid; c < kMmaTile * vc; c += kMmaThreads) {
      const int r = c / vc, col = c - r * vc, tok = row0 + r;
      const long cr = tok < L ? cache_row(tok) : -1;
      const bool ok = cr >= 0;
      cp_async16(sV + (r * ldv + col * 8) * 2, v_rows + (size_t)(ok ? cr : 0) * rv + col * 8, ok ? 16 : 0);
    }
    if constexpr (RECON) {
      const uint32_t sT = smem_u32(st + lay.k_bytes() + MmaSmem<RV16, RECON>::v_bytes);
      for (int c = tid; c < kMmaTile * 16; c += kMmaThreads) {
        const int r = c >> 4, col = c & 15, tok = row0 + r;
        const bool ok = tok < L;
        cp_async16(sT + (r * kCsLd + col * 4) * 4, p.cs + (size_t)(ok ? tok : 0) * 64 + col * 4, ok ? 16 : 0);
      }
    }
  };

  // Resident operands: U_k (RECON) through shared memory, the query B-fragments in registers.
  if constexpr (RECON) {
    const uint32_t su = smem_u32(sU);
    for (int c = tid; c < rk * 16; c += kMmaThreads) {
      const int r = c >> 4, col = c & 15;
      cp_async16(su + (r * kULd + col * 8) * 2, p.u_k + ((size_t)kvh * rk + r) * p.ld_u + col * 8, 16);
    }
  }
  uint32_t bq[8][2];
  {
    const bool ok = g < p.rep;
    const __nv_bfloat16* qrow = p.q + ((size_t)b * p.n_q + kvh * p.rep + (ok ? g : 0)) * kHeadDim;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      bq[kk][0] = ok ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t) : 0u;
      bq[kk][1] = ok ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t + 8) : 0u;
    }
  }

#pragma unroll
  for (int s = 0; s < NS - 1; ++s) {
    if (s < my_tiles) load_tile(tile0 + s, s);
    cp_async_commit();
  }

  // Softmax state for the two heads this thread's output columns belong to: head 2*(t&1)+e.
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[RV16][4];
#pragma unroll
  for (int i = 0; i < RV16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  const int lrow = (lane & 7) + ((lane >> 3) & 1) * 8;  // ldmatrix row within a 16-row block
  const int lcol = (lane >> 4) * 8;                     // ldmatrix column offset (A / trans-B order)

  for (int it = 0; it < my_tiles; ++it) {
    if constexpr (NS == 1) {
      // One stage (wide latents): every warp is done with the previous tile before it is overwritten.
      __syncthreads();
      load_tile(tile0 + it, 0);
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
    } else {
      cp_async_wait<NS - 2>();
      __syncthreads();
      if (it + NS - 1 < my_tiles) load_tile(tile0 + it + NS - 1, (it + NS - 1) % NS);
      cp_async_commit();
    }

    unsigned char* st = sStages + (it % NS) * lay.stage_bytes();
    const uint32_t sK = smem_u32(st), sV = smem_u32(st + lay.k_bytes());
    float s[4] = {0.f, 0.f, 0.f, 0.f};

    if constexpr (RECON) {
      float acc[16][4];
#pragma unroll
      for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
      const uint32_t su = smem_u32(sU);
      for (int kk = 0; kk < rk / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(sK + ((warp * 16 + lrow) * ldk + kk * 16 + lcol) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(su + ((kk * 16 + lrow) * kULd + np * 16 + lcol) * 2, b0, b1, b2, b3);
          mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
          mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // RoPE: K_rot[2j] = K[2j] cos - K[2j+1] sin ; K_rot[2j+1] = K[2j+1] cos + K[2j] sin.
      const uint32_t* sT = reinterpret_cast<const uint32_t*>(st + lay.k_bytes() + MmaSmem<RV16, RECON>::v_bytes);
      const __half* t0 = reinterpret_cast<const __half*>(sT + (warp * 16 + g) * kCsLd);
      const __half* t1 = t0 + 16 * kCsLd;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int f = 4 * n + t;  // frequency pair of this thread's two accumulator columns
        const float2 c0 = make_float2(__half2float(t0[packed_cos_index(f)]), __half2float(t0[packed_sin_index(f)]));
        const float2 c1 = make_float2(__half2float(t1[packed_cos_index(f)]), __half2float(t1[packed_sin_index(f)]));
        const float k0 = acc[n][0], k1 = acc[n][1], k2 = acc[n][2], k3 = acc[n][3];
        acc[n][0] = k0 * c0.x - k1 * c0.y;
        acc[n][1] = k1 * c0.x + k0 * c0.y;
        acc[n][2] = k2 * c1.x - k3 * c1.y;
        acc[n][3] = k3 * c1.x + k2 * c1.y;
      }
      // Scores: accumulator fragments of two adjacent n-tiles form one A fragment (k = 16 dims).
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
        split_bf16(acc[2 * kk][0], acc[2 * kk][1], h0, l0);
        split_bf16(acc[2 * kk][2], acc[2 * kk][3], h1, l1);
        split_bf16(acc[2 * kk + 1][0], acc[2 * kk + 1][1], h2, l2);
        split_bf16(acc[2 * kk + 1][2], acc[2 * kk + 1][3], h3, l3);
        mma_bf16(s, h0, h1, h2, h3, bq[kk][0], bq[kk][1]);
        mma_bf16(s, l0, l1, l2, l3, bq[kk][0], bq[kk][1]);
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(sK + ((warp * 16 + lrow) * ldk + kk * 16 + lcol) * 2, a0, a1, a2, a3);
        mma_bf16(s, a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
      }
    }

    // Online softmax. s[i]: token g (i<2) or g+8 (i>=2), head 2t + (i&1).
    const int tok0 = (tile0 + it) * kMmaTile + warp * 16 + g;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = tok0 + (i >> 1) * 8;
      const int head = 2 * t + (i & 1);
      x[i] = (tok < L && head < p.rep) ? s[i] * p.scale_log2 : -INFINITY;
    }
    float mx[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
      const float other = __shfl_xor_sync(0xffffffffu, mx[e], 2);
      if (t >= 2) mx[e] = other;
    }
    float alpha[2], pm[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float m_new = fmaxf(m_run[e], mx[e]);
      alpha[e] = (m_new == -INFINITY) ? 1.f : fast_exp2(m_run[e] - m_new);
      pm[e] = m_new;
      m_run[e] = m_new;
    }
    float pv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float m_e = pm[i & 1];
      pv[i] = (t < 2 && m_e != -INFINITY) ? fast_exp2(x[i] - m_e) : 0.f;
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float rs = pv[e] + pv[2 + e];
      rs += __shfl_xor_sync(0xffffffffu, rs, 4);
      rs += __shfl_xor_sync(0xffffffffu, rs, 8);
      rs += __shfl_xor_sync(0xffffffffu, rs, 16);
      const float other = __shfl_xor_sync(0xffffffffu, rs, 2);
      if (t >= 2) rs = other;
      l_run[e] = l_run[e] * alpha[e] + rs;
    }
    // P^T (rows: heads hi 0..3 then lo 0..3; columns: the warp's 16 tokens) -> B fragment.
    if (t < 2) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int h = 2 * t + (i & 1), col = g + (i >> 1) * 8;
        const __nv_bfloat16 hi = __float2bfloat16_rn(pv[i]);
        sP[h * 24 + col] = hi;
        sP[(4 + h) * 24 + col] = __float2bfloat16_rn(pv[i] - __bfloat162float(hi));
      }
    }
    __syncwarp();
    uint32_t bp0, bp1;
    ldsm_x2(smem_u32(sP + (lane & 7) * 24 + ((lane >> 3) & 1) * 8), bp0, bp1);
#pragma unroll
    for (int mt = 0; mt < RV16; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
      uint32_t a0, a1, a2, a3;
      const int vrow = warp * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
      const int vcol = mt * 16 + ((lane >> 3) & 1) * 8;
      ldsm_x4_t(sV + (vrow * ldv + vcol) * 2, a0, a1, a2, a3);
      mma_bf16(o[mt], a0, a1, a2, a3, bp0, bp1);
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  __syncthreads();

  // hi + lo columns: lane ^ 2 holds the other term of the same (head, column).
#pragma unroll
  for (int mt = 0; mt < RV16; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[mt][i] += __shfl_xor_sync(0xffffffffu, o[mt][i], 2);

  // Merge the 4 warps through shared memory (the stage buffers are free now).
  float* sm = reinterpret_cast<float*>(sStages);          // [4 warps][4 heads][2]
  float* so = sm + 32;                                     // [4 warps][4 heads][rv]
  if (t < 2) {
    if (g == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sm[(warp * 4 + 2 * t + e) * 2 + 0] = m_run[e];
        sm[(warp * 4 + 2 * t + e) * 2 + 1] = l_run[e];
      }
    }
#pragma unroll
    for (int mt = 0; mt < RV16; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int h = 2 * t + (i & 1), c = mt * 16 + g + (i >> 1) * 8;
        so[(warp * 4 + h) * rv + c] = o[mt][i];
      }
  }
  __syncthreads();
  const size_t item = ((size_t)(b * p.n_kv + kvh) * p.splits + split) * p.rep;
  for (int idx = tid; idx < p.rep * rv; idx += kMmaThreads) {
    const int h = idx / rv, c = idx - h * rv;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[(w * 4 + h) * 2]);
    float acc = 0.f, lsum = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = fast_exp2(sm[(w * 4 + h) * 2] - M);
        acc += so[(w * 4 + h) * rv + c] * f;
        lsum += sm[(w * 4 + h) * 2 + 1] * f;
      }
    }
    p.ws_o[(item + h) * rv + c] = acc;
    if (c == 0) {
      p.ws_ml[(item + h) * 2 + 0] = M;
      p.ws_ml[(item + h) * 2 + 1] = lsum;
    }
  }
}

}  // namespace palu
