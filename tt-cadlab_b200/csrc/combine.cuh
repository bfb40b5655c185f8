// Second pass of the split-K decode: merge the per-split (O, m, l) partials of one (batch row,
// query head) with the log-sum-exp rule, normalise, and store bf16 or fp32. For the in-kernel-V
// mode (G-LRD) the merged latent-space output is multiplied by the head's U_v here, which is exact
// linear algebra: softmax(s) @ (lat_v @ U_v) == (softmax(s) @ lat_v) @ U_v.
#pragma once
#include "palu_common.cuh"

namespace palu {

struct CombineParams {
  const float* ws_o;         // [B][n_kv][splits][rep][r_lat]
  const float* ws_ml;        // [B][n_kv][splits][rep][2]
  const __nv_bfloat16* u_v;  // optional [n_kv][r_lat][128]
  void* out;                 // [B][n_q][r_out]
  int out_f32;
  int batch, n_q, n_kv, rep, splits, r_lat, r_out;
};

constexpr int kCombineThreads = 128;
constexpr int kMaxSplits = 256;

__global__ void __launch_bounds__(kCombineThreads) palu_combine_kernel(const CombineParams p) {
  __shared__ float s_w[kMaxSplits];
  __shared__ float s_inv_l;
  extern __shared__ float s_lat[];  // r_lat floats (u_v mode only)
  const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int kvh = qh / p.rep, hl = qh - kvh * p.rep;
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

}  // namespace palu
