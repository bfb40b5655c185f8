// Second pass of the split-K decode: merge the per-split (O, m, l) partials of one (batch row,
// query head) with the log-sum-exp rule, normalise, and store bf16 or fp32. For the in-kernel-V
// mode (G-LRD) the merged latent-space output is multiplied by the head's U_v here, which is exact
// linear algebra: softmax(s) @ (lat_v @ U_v) == (softmax(s) @ lat_v) @ U_v.
// A nonzero status word (a bounded wait of the decode kernel expired, so some partials were never
// written and others may be stale) makes the merge write NaN instead: a failed call never returns
// numbers that look valid. The word stays set until palu_read_status clears it.
#pragma once
#include "palu_common.cuh"

namespace palu {

struct CombineParams {
  const int* status;         // the workspace's status word
  const float* ws_o;         // [B][n_kv][splits][rep][r_lat]
  const float* ws_ml;        // [B][n_kv][splits][rep][2]
  const __nv_bfloat16* u_v;  // optional [n_kv][r_lat][128]
  void* out;                 // [B][n_q][r_out]
  int out_f32;
  int batch, n_q, n_kv, rep, splits, r_lat, r_out;
};

constexpr int kCombineThreads = 128;
constexpr int kMaxSplits = 256;

// Output row of a call whose decode kernel gave up on a wait: NaN everywhere.
PALU_DEVINL void write_nan_row(void* out, int out_f32, size_t orow, int width) {
  for (int c = threadIdx.x; c < width; c += kCombineThreads) {
    if (out_f32)
      reinterpret_cast<float*>(out)[orow + c] = __int_as_float(0x7fc00000);
    else
      reinterpret_cast<__nv_bfloat16*>(out)[orow + c] = __ushort_as_bfloat16((unsigned short)0x7fc0);
  }
}

__global__ void __launch_bounds__(kCombineThreads) palu_combine_kernel(const CombineParams p) {
  __shared__ float s_w[kMaxSplits];
  __shared__ float s_inv_l;
  extern __shared__ float s_lat[];  // r_lat floats (u_v mode only)
  const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int kvh = qh / p.rep, hl = qh - kvh * p.rep;
  if (*reinterpret_cast<const volatile int*>(p.status) != 0) {
    write_nan_row(p.out, p.out_f32, ((size_t)b * p.n_q + qh) * p.r_out, p.r_out);
    return;
  }
  const size_t base = (size_t)(b * p.n_kv + kvh) * p.splits;
  auto idx = [&](int s) { return (base + s) * p.rep + hl; };

  if (tid < 32) {
    float M = -INFINITY;
    for (int s = tid; s < p.splits; s += 32) M = fmaxf(M, p.ws_ml[idx(s) * 2]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int s = tid; s < p.splits; s += 32) {
      const float m = p.ws_ml[idx(s) * 2];
      const float w = (M == -INFINITY || m == -INFINITY) ? 0.f : fast_exp2(m - M);
      s_w[s] = w;
      L += w * p.ws_ml[idx(s) * 2 + 1];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (tid == 0) s_inv_l = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const float inv_l = s_inv_l;
  const size_t orow = ((size_t)b * p.n_q + qh) * p.r_out;
  for (int c = tid; c < p.r_lat; c += kCombineThreads) {
    float acc = 0.f;
    for (int s = 0; s < p.splits; ++s) acc += p.ws_o[idx(s) * p.r_lat + c] * s_w[s];
    acc *= inv_l;
    if (p.u_v) {
      s_lat[c] = acc;
    } else if (p.out_f32) {
      reinterpret_cast<float*>(p.out)[orow + c] = acc;
    } else {
      reinterpret_cast<__nv_bfloat16*>(p.out)[orow + c] = __float2bfloat16_rn(acc);
    }
  }
  if (p.u_v) {
    __syncthreads();
    const __nv_bfloat16* u = p.u_v + (size_t)kvh * p.r_lat * kHeadDim;
    for (int d = tid; d < kHeadDim; d += kCombineThreads) {
      float acc = 0.f;
      for (int c = 0; c < p.r_lat; ++c) acc += s_lat[c] * __bfloat162float(u[(size_t)c * kHeadDim + d]);
      if (p.out_f32)
        reinterpret_cast<float*>(p.out)[orow + d] = acc;
      else
        reinterpret_cast<__nv_bfloat16*>(p.out)[orow + d] = __float2bfloat16_rn(acc);
    }
  }
}

// Merge for the tcgen05 decode's balanced split (decode_tc.cuh): the records of (batch row b, query head)
// are found from the same cut of the KV head's row-ordered tile list into `ctas` ranges: T tiles in all,
// row b's tiles are s_b .. s_b + n_b - 1, and tile x lies in range ((x + 1) * ctas - 1) / T. Rows with no
// tile (cur_pos < 0) come out zero. Launched as a programmatic dependent of the decode kernel: the record
// lists come from cur_pos alone, so they are built before griddepcontrol.wait, which then waits for the
// decode grid's completion and memory before any record is read.
struct CombineTcParams {
  const int* status;         // the workspace's status word
  const float* ws_o;         // records [rec][rep][r_lat]
  const float* ws_ml;        // records [rec][rep][5]: m, l of the 4 row quarters
  const int32_t* cur_pos;    // [B]
  const __nv_bfloat16* u_v;  // optional [n_kv][r_lat][128]
  void* out;                 // [B][n_q][r_out]
  int out_f32;
  int batch, n_q, n_kv, rep, ctas, r_lat, r_out, max_seq;
  int npipe;                 // pipelines per decode CTA (1 or 2): records g < npipe of each pair are written
};
constexpr int kMaxTcRecords = 2 * kMaxSplits;

__global__ void __launch_bounds__(kCombineThreads) palu_combine_tc_kernel(const CombineTcParams p) {
  __shared__ int s_rec[kMaxTcRecords];
  __shared__ int s_nrec;
  extern __shared__ float s_lat[];  // r_lat floats (u_v mode only)
  const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int kvh = qh / p.rep, hl = qh - kvh * p.rep;
  if (tid < 32) {
    long long T = 0, sb = 0;
    for (int bb = tid; bb < p.batch; bb += 32) {
      const int nb = tc_row_tiles(p.cur_pos, bb, p.max_seq);
      T += nb;
      if (bb < b) sb += nb;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      T += __shfl_xor_sync(0xffffffffu, T, o);
      sb += __shfl_xor_sync(0xffffffffu, sb, o);
    }
    if (tid == 0) {
      const int nb = tc_row_tiles(p.cur_pos, b, p.max_seq);
      int cnt = 0;
      if (nb > 0 && T > 0) {
        const int cf = (int)(((sb + 1) * p.ctas - 1) / T), cl = (int)(((sb + nb) * p.ctas - 1) / T);
        if (cf == cl) {
          for (int g = 0; g < p.npipe; ++g) s_rec[cnt++] = (int)tc_rec_direct(b, kvh, p.n_kv, g);
        } else {
          for (int g = 0; g < p.npipe; ++g) s_rec[cnt++] = (int)tc_rec_edge(p.batch, p.n_kv, p.ctas, kvh, cf, 1, g);
          for (int c = cf + 1; c <= cl && cnt + 2 <= kMaxTcRecords; ++c) {
            if ((long long)c * T / p.ctas == (long long)(c + 1) * T / p.ctas) continue;  // empty range: no records
            for (int g = 0; g < p.npipe; ++g) s_rec[cnt++] = (int)tc_rec_edge(p.batch, p.n_kv, p.ctas, kvh, c, 0, g);
          }
        }
      }
      s_nrec = cnt;
    }
  }
  __syncthreads();
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const size_t orow = ((size_t)b * p.n_q + qh) * p.r_out;
  if (*reinterpret_cast<const volatile int*>(p.status) != 0) {
    write_nan_row(p.out, p.out_f32, orow, p.r_out);
    return;
  }
  // Every thread merges its own latent dims (c = tid, tid + 128) over all records. Records are taken 8 at a
  // time and every load of a batch (m, the 4 quarter sums l, O) is issued before any is used, so the merge
  // costs about one round trip to L2 per 8 records; the running (M, L, acc) are rescaled between batches.
  const int nrec = s_nrec;
  constexpr int kBatch = 8;
  float M = -INFINITY, Lsum = 0.f, acc0 = 0.f, acc1 = 0.f;
  const int c0 = tid, c1 = tid + kCombineThreads;
  for (int i0 = 0; i0 < nrec; i0 += kBatch) {
    float m[kBatch], l[kBatch], o0[kBatch], o1[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      m[k] = -INFINITY;
      l[k] = o0[k] = o1[k] = 0.f;
      if (i0 + k < nrec) {
        const size_t rh = (size_t)s_rec[i0 + k] * p.rep + hl;
        const float* ml = p.ws_ml + rh * 5;
        m[k] = ml[0];
        l[k] = (ml[1] + ml[2]) + (ml[3] + ml[4]);
        const float* o = p.ws_o + rh * p.r_lat;
        if (c0 < p.r_lat) o0[k] = o[c0];
        if (c1 < p.r_lat) o1[k] = o[c1];
      }
    }
    float mb = M;
#pragma unroll
    for (int k = 0; k < kBatch; ++k) mb = fmaxf(mb, m[k]);
    if (mb != -INFINITY) {
      const float sc = M == -INFINITY ? 0.f : fast_exp2(M - mb);
      Lsum *= sc;
      acc0 *= sc;
      acc1 *= sc;
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const float w = m[k] == -INFINITY ? 0.f : fast_exp2(m[k] - mb);
        Lsum += w * l[k];
        acc0 += w * o0[k];
        acc1 += w * o1[k];
      }
      M = mb;
    }
  }
  const float inv_l = Lsum > 0.f ? 1.f / Lsum : 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = h ? c1 : c0;
    if (c >= p.r_lat) continue;
    const float v = (h ? acc1 : acc0) * inv_l;
    if (p.u_v) {
      s_lat[c] = v;
    } else if (p.out_f32) {
      reinterpret_cast<float*>(p.out)[orow + c] = v;
    } else {
      reinterpret_cast<__nv_bfloat16*>(p.out)[orow + c] = __float2bfloat16_rn(v);
    }
  }
  if (p.u_v) {
    __syncthreads();
    const __nv_bfloat16* u = p.u_v + (size_t)kvh * p.r_lat * kHeadDim;
    for (int d = tid; d < kHeadDim; d += kCombineThreads) {
      float acc = 0.f;
#pragma unroll 8
      for (int c = 0; c < p.r_lat; ++c) acc += s_lat[c] * __bfloat162float(u[(size_t)c * kHeadDim + d]);
      if (p.out_f32)
        reinterpret_cast<float*>(p.out)[orow + d] = acc;
      else
        reinterpret_cast<__nv_bfloat16*>(p.out)[orow + d] = __float2bfloat16_rn(acc);
    }
  }
}

}  // namespace palu
