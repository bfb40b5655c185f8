// C ABI of libpalu_b200 (declared in include/palu_b200.h): envelope validation, split planning,
// workspace layout and kernel dispatch. Everything here runs on the host; the kernels live in the
// .cuh files next to it.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/palu_b200.h"
#include "append.cuh"
#include "combine.cuh"
#include "decode_mma.cuh"
#include "decode_tc.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_check(const char* where) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(PALU_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
  return PALU_OK;
}

// SM count of the current device, cached per device. Several host threads may race on the first lookup;
// each stores the same value, and the atomics make those stores and the loads well defined.
int device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int rep_of(const palu_decode_dims* d) { return d->n_q_heads / d->n_kv_heads; }

// Shape envelope shared by every decode entry point. `latent` = latent caches (palu_decode_attn).
int validate(const palu_decode_dims* d, bool latent, bool has_uv) {
  if (!d) return fail(PALU_ERR_INVALID, "dims is NULL");
  if (d->batch <= 0 || d->n_q_heads <= 0 || d->n_kv_heads <= 0 || d->n_groups <= 0 || d->max_seq <= 0)
    return fail(PALU_ERR_INVALID, "batch, head counts and max_seq must be positive (got B=%d n_q=%d n_kv=%d "
                "n_groups=%d max_seq=%d)", d->batch, d->n_q_heads, d->n_kv_heads, d->n_groups, d->max_seq);
  if (d->head_dim != 128) return fail(PALU_ERR_INVALID, "head_dim must be 128, got %d", d->head_dim);
  if (d->n_q_heads % d->n_kv_heads != 0)
    return fail(PALU_ERR_INVALID, "KV head count %d must divide the %d query heads", d->n_kv_heads, d->n_q_heads);
  if (rep_of(d) > 4)
    return fail(PALU_ERR_INVALID, "at most 4 query heads per KV head are supported, got %d", rep_of(d));
  if (d->n_kv_heads % d->n_groups != 0)
    return fail(PALU_ERR_INVALID, "heads_per_group: %d latent heads do not divide %d KV heads", d->n_groups,
                d->n_kv_heads);
  // Latent widths: multiples of 16 up to 128, multiples of 32 up to 256 (wider ones run on the mma.sync
  // kernel with a single pipeline stage).
  auto rank_ok = [](int r) { return r >= 16 && ((r <= 128 && r % 16 == 0) || (r <= 256 && r % 32 == 0)); };
  if (!rank_ok(d->r_v))
    return fail(PALU_ERR_INVALID, "r_v must be a multiple of 16 in [16, 128] or of 32 in (128, 256], got %d",
                d->r_v);
  if (latent) {
    if (!rank_ok(d->r_k))
      return fail(PALU_ERR_INVALID, "r_k must be a multiple of 16 in [16, 128] or of 32 in (128, 256], got %d",
                  d->r_k);
    if (d->n_groups != d->n_kv_heads && !has_uv)
      return fail(PALU_ERR_INVALID, "grouped latents (%d groups for %d KV heads) need u_v", d->n_groups,
                  d->n_kv_heads);
  } else {
    if (d->n_groups != d->n_kv_heads) return fail(PALU_ERR_INVALID, "plain decode needs n_groups == n_kv_heads");
    if (d->r_k != 128) return fail(PALU_ERR_INVALID, "plain decode needs r_k == head_dim == 128");
  }
  if (d->splits < 0) return fail(PALU_ERR_INVALID, "splits must be >= 0");
  return PALU_OK;
}

int choose_splits(const palu_decode_dims* d) {
  if (d->splits > 0) return d->splits < palu::kMaxSplits ? d->splits : palu::kMaxSplits;
  const long items = (long)d->batch * d->n_kv_heads;
  const int tiles = (d->max_seq + palu::kMmaTile - 1) / palu::kMmaTile;
  const long target = 16L * device_sms();  // ~8 waves at 2 CTAs per SM
  long s = (target + items - 1) / items;
  const long cap = tiles / 4 > 1 ? tiles / 4 : 1;  // keep >= 4 tiles per split
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  if (s > palu::kMaxSplits) s = palu::kMaxSplits;
  return (int)s;
}

// Workspace layout: [256 B status header: int32 status word][O partials][(m, l) partials].
constexpr size_t kWsHeader = 256;

size_t ws_floats_o(const palu_decode_dims* d, int splits) {
  return (size_t)d->batch * d->n_kv_heads * splits * rep_of(d) * d->r_v;
}
size_t ws_floats_ml(const palu_decode_dims* d, int splits) {
  return (size_t)d->batch * d->n_kv_heads * splits * rep_of(d) * 2;
}
size_t ws_bytes(const palu_decode_dims* d, int splits) {
  const size_t o = (ws_floats_o(d, splits) * 4 + 255) / 256 * 256;
  return kWsHeader + o + ws_floats_ml(d, splits) * 4 + 256;
}

// ---- tcgen05 path: availability, split planning, tensor maps ---------------------------------------

int g_kernel_choice = PALU_KERNEL_AUTO;
// RoPE form of this host thread's decode calls (palu_set_rope_mode).
thread_local int g_rope_mode = PALU_ROPE_ABSOLUTE;
// Timeout-path test hook (palu_set_wait_limit): the bound on every device wait, and the V-starve switch.
std::atomic<unsigned long long> g_wait_ns{palu::tc::kWaitNs};
std::atomic<int> g_starve_v{0};

// Latents up to 128 wide run two pipelines per CTA; up to 256 wide, one (tc_pipes).
bool tc_supported(const palu_decode_dims* d, bool recon) {
  return recon && d->r_k <= 256 && d->r_v <= 256 && rep_of(d) <= 4;
}
int tc_pipes(const palu_decode_dims* d) { return d->r_k > 128 || d->r_v > 128 ? 1 : 2; }

bool use_tc(const palu_decode_dims* d, bool recon) {
  if (g_kernel_choice == PALU_KERNEL_MMA) return false;
  return tc_supported(d, recon);
}

// CTAs per KV head for the tcgen05 kernel, whose CTAs split each KV head's row-ordered tiles into equal
// ranges: one CTA per SM in a single wave (SMs / n_kv per KV head), but at least 4 tiles per CTA when every
// row attends the whole cache.
int choose_splits_tc(const palu_decode_dims* d) {
  if (d->splits > 0) return d->splits < palu::kMaxSplits ? d->splits : palu::kMaxSplits;
  const long tiles = (long)d->batch * ((d->max_seq + palu::tc::kTile - 1) / palu::tc::kTile);
  long c = device_sms() / d->n_kv_heads;
  if (c > tiles / 4) c = tiles / 4;
  if (c < 1) c = 1;
  if (c > palu::kMaxSplits) c = palu::kMaxSplits;
  return (int)c;
}

// Workspace of the tcgen05 path: [256 B status header][O records][(m, l x 4) records].
size_t ws_tc_o_bytes(const palu_decode_dims* d, int ctas) {
  return (palu::tc_n_records(d->batch, d->n_kv_heads, ctas) * rep_of(d) * d->r_v * 4 + 255) / 256 * 256;
}
size_t ws_tc_bytes(const palu_decode_dims* d, int ctas) {
  return kWsHeader + ws_tc_o_bytes(d, ctas) + palu::tc_n_records(d->batch, d->n_kv_heads, ctas) * rep_of(d) * 5 * 4 +
         256;
}

int splits_for(const palu_decode_dims* d, bool recon) {
  return use_tc(d, recon) ? choose_splits_tc(d) : choose_splits(d);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's cuTensorMapEncodeTiled, looked up once. A function-local static is initialised exactly once
// even when several host threads make their first call at the same time.
EncodeTiledFn encode_fn() {
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(ptr);
    return nullptr;
  }();
  return fn;
}

int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box, const char* what,
           CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PALU_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PALU_ERR_INVALID, "tensor map for %s rejected (CUresult %d)", what, (int)r);
  return PALU_OK;
}

// Page-table fields of the kernel parameters (all zero for contiguous caches).
template <class Params>
void set_pages(Params& p, const palu_page_table* pg) {
  p.page_table = pg ? pg->table : nullptr;
  p.table_ld = pg ? pg->table_ld : 0;
  p.n_blocks = pg ? pg->n_blocks : 0;
  p.blk_shift = 0;
  while (pg && (1 << p.blk_shift) < pg->block_size) ++p.blk_shift;
}

template <int KBK, int KBV, bool PAGED, int NP, bool F8, bool F4, bool REL>
int launch_tc_form(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mt, const palu::tc::TcParams& p,
                   cudaStream_t stream) {
  using Lay = palu::tc::Layout<KBK, KBV, NP, F8>;
  auto kern = palu::tc::palu_decode_tc_kernel<KBK, KBV, PAGED, NP, F8, F4, REL>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::TOTAL) != cudaSuccess)
    return cuda_check("cudaFuncSetAttribute(decode tc)");
  kern<<<dim3(p.ctas, p.n_kv, 1), palu::tc::kThreads, Lay::TOTAL, stream>>>(mk, mv, mt, p);
  return cuda_check("decode tc kernel launch");
}

// The RoPE form is a template parameter of the kernel (one body per form); p.rel picks the instantiation.
template <int KBK, int KBV, bool PAGED, int NP = 2, bool F8 = false, bool F4 = false>
int launch_tc(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mt, const palu::tc::TcParams& p,
              cudaStream_t stream) {
  using Lay = palu::tc::Layout<KBK, KBV, NP, F8>;
  if (!p.rel) return launch_tc_form<KBK, KBV, PAGED, NP, F8, F4, false>(mk, mv, mt, p, stream);
  if (!palu::tc::rel_fits<Lay, NP>())
    return fail(PALU_ERR_INVALID, "chunk-relative RoPE: this kernel layout has no room for the fixed table rows");
  return launch_tc_form<KBK, KBV, PAGED, NP, F8, F4, true>(mk, mv, mt, p, stream);
}

int run_tc(const void* q, const void* k, const void* v, const void* u_k, int64_t u_k_ld, const void* cs_pairs,
           const int32_t* cur_pos, void* workspace, float* ws_o, float* ws_ml, const palu_decode_dims* d, int splits,
           float scale, const palu_page_table* pg, cudaStream_t stream, const int8_t* k_exp = nullptr,
           const int8_t* v_exp = nullptr, bool f4 = false) {
  const bool f8 = k_exp != nullptr;
  CUtensorMap mk, mv, mt;
  // Contiguous caches: one item per (batch row, latent head) of max_seq rows, 128-row boxes. Paged caches:
  // one item per (physical block, latent head) of block_size rows, one block per box.
  const cuuint64_t items = pg ? (cuuint64_t)pg->n_blocks * d->n_groups : (cuuint64_t)d->batch * d->n_groups;
  const cuuint64_t rows = pg ? (cuuint64_t)pg->block_size : (cuuint64_t)d->max_seq;
  const cuuint32_t box_rows = pg ? (cuuint32_t)pg->block_size : 128;
  if (f8) {
    // e4m3 codes: one box per tile of 64 or 128 codes per row (the kernel's staged rows), no swizzle; e2m1
    // codes: rows of r / 2 bytes, one box of 32 or 64 bytes per row
    const cuuint64_t wk = f4 ? d->r_k / 2 : d->r_k, wv = f4 ? d->r_v / 2 : d->r_v;
    const cuuint64_t dk[3] = {wk, rows, items}, dv[3] = {wv, rows, items};
    const cuuint64_t sk[2] = {wk, rows * wk}, sv[2] = {wv, rows * wv};
    const cuuint32_t unit = f4 ? 32u : 64u;
    const cuuint32_t bk[3] = {d->r_k > 64 ? 2 * unit : unit, box_rows, 1}, bv[3] = {d->r_v > 64 ? 2 * unit : unit, box_rows, 1};
    if (int st = encode(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, k, dk, sk, bk, "k_lat (fp8)", CU_TENSOR_MAP_SWIZZLE_NONE))
      return st;
    if (int st = encode(&mv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, v, dv, sv, bv, "v_lat (fp8)", CU_TENSOR_MAP_SWIZZLE_NONE))
      return st;
  } else {
    {
      const cuuint64_t dims[3] = {(cuuint64_t)d->r_k, rows, items};
      const cuuint64_t str[2] = {(cuuint64_t)d->r_k * 2, rows * d->r_k * 2};
      const cuuint32_t box[3] = {64, box_rows, 1};
      if (int st = encode(&mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims, str, box, "k_lat")) return st;
    }
    {
      const cuuint64_t dims[3] = {(cuuint64_t)d->r_v, rows, items};
      const cuuint64_t str[2] = {(cuuint64_t)d->r_v * 2, rows * d->r_v * 2};
      const cuuint32_t box[3] = {64, box_rows, 1};
      if (int st = encode(&mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v, dims, str, box, "v_lat")) return st;
    }
  }
  {
    const cuuint64_t dims[2] = {64, (cuuint64_t)d->max_seq};
    const cuuint64_t str[1] = {256};
    const cuuint32_t box[2] = {16, 128};  // one 16-frequency block (16 cos + 16 sin, 64 B) x 128 positions
    if (int st = encode(&mt, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, cs_pairs, dims, str, box, "cs_tab",
                        CU_TENSOR_MAP_SWIZZLE_64B))
      return st;
  }
  palu::tc::TcParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.u_k = static_cast<const __nv_bfloat16*>(u_k);
  p.ld_u = (int)u_k_ld;
  p.cur_pos = cur_pos;
  p.ws_o = ws_o;
  p.ws_ml = ws_ml;
  p.status = static_cast<int*>(workspace);
  p.batch = d->batch;
  p.n_q = d->n_q_heads;
  p.n_kv = d->n_kv_heads;
  p.n_groups = d->n_groups;
  p.rk = d->r_k;
  p.rv = d->r_v;
  p.max_seq = d->max_seq;
  p.ctas = splits;
  p.rep = rep_of(d);
  p.scale_log2 = scale * palu::kLog2e;
  set_pages(p, pg);
  p.wait_ns = g_wait_ns.load(std::memory_order_relaxed);
  p.starve_v = g_starve_v.load(std::memory_order_relaxed);
  p.pdl_early = (long)splits * d->n_kv_heads <= device_sms();
  p.k_exp = k_exp;
  p.v_exp = v_exp;
  p.rel = g_rope_mode == PALU_ROPE_CHUNK_RELATIVE;
  p.cs = static_cast<const uint32_t*>(cs_pairs);
  if (f8) {  // fp8 caches: contiguous, latents at most 128 wide (checked by the caller)
    const int kbk8 = d->r_k > 64 ? 2 : 1, kbv8 = d->r_v > 64 ? 2 : 1;
    if (f4) {
      if (kbk8 == 1 && kbv8 == 1) return launch_tc<1, 1, false, 2, true, true>(mk, mv, mt, p, stream);
      if (kbk8 == 1 && kbv8 == 2) return launch_tc<1, 2, false, 2, true, true>(mk, mv, mt, p, stream);
      if (kbk8 == 2 && kbv8 == 1) return launch_tc<2, 1, false, 2, true, true>(mk, mv, mt, p, stream);
      return launch_tc<2, 2, false, 2, true, true>(mk, mv, mt, p, stream);
    }
    if (kbk8 == 1 && kbv8 == 1) return launch_tc<1, 1, false, 2, true>(mk, mv, mt, p, stream);
    if (kbk8 == 1 && kbv8 == 2) return launch_tc<1, 2, false, 2, true>(mk, mv, mt, p, stream);
    if (kbk8 == 2 && kbv8 == 1) return launch_tc<2, 1, false, 2, true>(mk, mv, mt, p, stream);
    return launch_tc<2, 2, false, 2, true>(mk, mv, mt, p, stream);
  }
  if (tc_pipes(d) == 1)  // latents wider than 128: one pipeline, four 64-wide boxes per K and V tile
    return pg ? launch_tc<4, 4, true, 1>(mk, mv, mt, p, stream) : launch_tc<4, 4, false, 1>(mk, mv, mt, p, stream);
  const int kbk = d->r_k > 64 ? 2 : 1, kbv = d->r_v > 64 ? 2 : 1;
  if (pg) {
    if (kbk == 1 && kbv == 1) return launch_tc<1, 1, true>(mk, mv, mt, p, stream);
    if (kbk == 1 && kbv == 2) return launch_tc<1, 2, true>(mk, mv, mt, p, stream);
    if (kbk == 2 && kbv == 1) return launch_tc<2, 1, true>(mk, mv, mt, p, stream);
    return launch_tc<2, 2, true>(mk, mv, mt, p, stream);
  }
  if (kbk == 1 && kbv == 1) return launch_tc<1, 1, false>(mk, mv, mt, p, stream);
  if (kbk == 1 && kbv == 2) return launch_tc<1, 2, false>(mk, mv, mt, p, stream);
  if (kbk == 2 && kbv == 1) return launch_tc<2, 1, false>(mk, mv, mt, p, stream);
  return launch_tc<2, 2, false>(mk, mv, mt, p, stream);
}

template <int RV16, bool RECON, int NS>
int launch_mma_ns(const palu::DecodeParams& p, int bytes, cudaStream_t stream) {
  auto kern = palu::palu_decode_mma_kernel<RV16, RECON, NS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return cuda_check("cudaFuncSetAttribute(decode)");
  kern<<<dim3(p.splits, p.n_kv, p.batch), palu::kMmaThreads, bytes, stream>>>(p);
  return cuda_check("decode kernel launch");
}

// Two pipeline stages where they fit in shared memory, else one (latents wider than 128).
template <int RV16, bool RECON>
int launch_mma(const palu::DecodeParams& p, cudaStream_t stream) {
  constexpr int kSmemMax = 227 * 1024;
  const palu::MmaSmem<RV16, RECON> lay(p.rk);
  if (lay.total(2) <= kSmemMax) return launch_mma_ns<RV16, RECON, 2>(p, lay.total(2), stream);
  if (lay.total(1) <= kSmemMax) return launch_mma_ns<RV16, RECON, 1>(p, lay.total(1), stream);
  return fail(PALU_ERR_INVALID, "r_k %d / r_v %d need %d bytes of shared memory", p.rk, p.rv, lay.total(1));
}

template <bool RECON>
int dispatch_rv(const palu::DecodeParams& p, cudaStream_t s) {
  switch (p.rv / 16) {
    case 1: return launch_mma<1, RECON>(p, s);
    case 2: return launch_mma<2, RECON>(p, s);
    case 3: return launch_mma<3, RECON>(p, s);
    case 4: return launch_mma<4, RECON>(p, s);
    case 5: return launch_mma<5, RECON>(p, s);
    case 6: return launch_mma<6, RECON>(p, s);
    case 7: return launch_mma<7, RECON>(p, s);
    case 8: return launch_mma<8, RECON>(p, s);
    case 10: return launch_mma<10, RECON>(p, s);
    case 12: return launch_mma<12, RECON>(p, s);
    case 14: return launch_mma<14, RECON>(p, s);
    case 16: return launch_mma<16, RECON>(p, s);
  }
  return fail(PALU_ERR_INVALID, "r_v %d unsupported", p.rv);
}

int run_decode(bool recon, const void* q, const void* k, const void* v, const void* u_k, int64_t u_k_ld,
               const void* u_v, const void* cs_pairs, const int32_t* cur_pos, void* out, int32_t out_dtype,
               void* workspace, size_t workspace_bytes, const palu_decode_dims* d, float scale,
               cudaStream_t stream, const palu_page_table* pg = nullptr, const int8_t* k_exp = nullptr,
               const int8_t* v_exp = nullptr, bool f4 = false) {
  int st = validate(d, recon, u_v != nullptr);
  if (st) return st;
  const bool f8 = k_exp != nullptr || v_exp != nullptr;
  if (f8) {
    if (!k_exp || !v_exp) return fail(PALU_ERR_INVALID, "fp8 latents need both exponent arrays");
    if (d->r_k > 128 || d->r_v > 128)
      return fail(PALU_ERR_INVALID, "fp8 latents: r_k and r_v must be at most 128 (got %d, %d)", d->r_k, d->r_v);
    if (f4 && ((d->r_k != 64 && d->r_k != 128) || (d->r_v != 64 && d->r_v != 128)))
      return fail(PALU_ERR_INVALID, "fp4 latents: r_k and r_v must be 64 or 128 (got %d, %d)", d->r_k, d->r_v);
    if (!use_tc(d, recon))
      return fail(PALU_ERR_INVALID, "fp8 latents run on the tcgen05 kernel only (palu_set_kernel selects mma.sync)");
  }
  if (!q || !k || !v || !cur_pos || !out) return fail(PALU_ERR_INVALID, "q, caches, cur_pos and out must be set");
  if (recon && (!u_k || !cs_pairs)) return fail(PALU_ERR_INVALID, "u_k (w_rot) and cs_tab must be set");
  if (recon && (u_k_ld < 128 || u_k_ld % 8 != 0))
    return fail(PALU_ERR_INVALID, "w_rot/u_k row length %lld must be >= 128 and a multiple of 8", (long long)u_k_ld);
  if (out_dtype != PALU_BF16 && out_dtype != PALU_F32) return fail(PALU_ERR_INVALID, "out_dtype must be bf16 or f32");
  const bool tc = use_tc(d, recon);
  if (recon && !tc && g_rope_mode == PALU_ROPE_CHUNK_RELATIVE)
    return fail(PALU_ERR_INVALID, "chunk-relative RoPE runs on the tcgen05 kernel only (palu_set_kernel selects mma.sync)");
  const int splits = tc ? choose_splits_tc(d) : choose_splits(d);
  const size_t need = tc ? ws_tc_bytes(d, splits) : ws_bytes(d, splits);
  if (!workspace || workspace_bytes < need)
    return fail(PALU_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes needed", workspace_bytes,
                need);
  if (tc && reinterpret_cast<uintptr_t>(cs_pairs) % 16 != 0)
    return fail(PALU_ERR_INVALID, "cs_tab (packed) must be 16-byte aligned");
  if (tc && reinterpret_cast<uintptr_t>(u_k) % 16 != 0)
    return fail(PALU_ERR_INVALID, "w_rot/u_k must be 16-byte aligned");
  float* ws_o = reinterpret_cast<float*>(static_cast<char*>(workspace) + kWsHeader);
  float* ws_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + kWsHeader +
                                          (tc ? ws_tc_o_bytes(d, splits) : (ws_floats_o(d, splits) * 4 + 255) / 256 * 256));

  palu::DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.u_k = static_cast<const __nv_bfloat16*>(u_k);
  p.cs = static_cast<const uint32_t*>(cs_pairs);
  p.cur_pos = cur_pos;
  p.ws_o = ws_o;
  p.ws_ml = ws_ml;
  p.batch = d->batch;
  p.n_q = d->n_q_heads;
  p.n_kv = d->n_kv_heads;
  p.n_groups = d->n_groups;
  p.rk = d->r_k;
  p.rv = d->r_v;
  p.max_seq = d->max_seq;
  p.splits = splits;
  p.ld_u = (int)u_k_ld;
  p.rep = rep_of(d);
  p.scale_log2 = scale * palu::kLog2e;
  set_pages(p, pg);
  if (tc) {
    st = run_tc(q, k, v, u_k, u_k_ld, cs_pairs, cur_pos, workspace, ws_o, ws_ml, d, splits, scale, pg, stream, k_exp,
                v_exp, f4);
    if (st) return st;
    palu::CombineTcParams c;
    c.status = static_cast<const int*>(workspace);
    c.ws_o = ws_o;
    c.ws_ml = ws_ml;
    c.cur_pos = cur_pos;
    c.u_v = static_cast<const __nv_bfloat16*>(u_v);
    c.out = out;
    c.out_f32 = out_dtype == PALU_F32;
    c.batch = d->batch;
    c.n_q = d->n_q_heads;
    c.n_kv = d->n_kv_heads;
    c.rep = p.rep;
    c.ctas = splits;
    c.r_lat = d->r_v;
    c.r_out = u_v ? 128 : d->r_v;
    c.max_seq = d->max_seq;
    c.npipe = tc_pipes(d);
    // Programmatic dependent launch: the merge's prologue overlaps the decode kernel's tail.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d->n_q_heads, d->batch);
    cfg.blockDim = dim3(palu::kCombineThreads);
    cfg.dynamicSmemBytes = u_v ? d->r_v * 4 : 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, palu::palu_combine_tc_kernel, c) != cudaSuccess) return cuda_check("combine kernel launch");
    return cuda_check("combine kernel launch");
  }
  st = recon ? dispatch_rv<true>(p, stream) : dispatch_rv<false>(p, stream);
  if (st) return st;

  palu::CombineParams c;
  c.status = static_cast<const int*>(workspace);
  c.ws_o = ws_o;
  c.ws_ml = ws_ml;
  c.u_v = static_cast<const __nv_bfloat16*>(u_v);
  c.out = out;
  c.out_f32 = out_dtype == PALU_F32;
  c.batch = d->batch;
  c.n_q = d->n_q_heads;
  c.n_kv = d->n_kv_heads;
  c.rep = p.rep;
  c.splits = splits;
  c.r_lat = d->r_v;
  c.r_out = u_v ? 128 : d->r_v;
  palu::palu_combine_kernel<<<dim3(d->n_q_heads, d->batch), palu::kCombineThreads, u_v ? d->r_v * 4 : 0, stream>>>(c);
  return cuda_check("combine kernel launch");
}

// ---- static-scratch variant (palu_decode_attn_static) ----------------------------------------------

// The partial results and status word of palu_decode_attn_static live in this module-global array, one
// copy per device, so that entry point allocates nothing. 8 MiB holds every call whose
// palu_workspace_bytes() fits it, e.g. B = 32, 8 KV heads, 4 query heads each, r_v = 64 (1.2 MB of
// partial records for the tcgen05 kernel). All calls on one device share it: calls that overlap in time
// (other streams, other host threads) race on it.
constexpr size_t kStaticScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {nullptr};

// Per-device setup, once: resolve the array's address on the current device and zero its status word.
// Runs synchronous CUDA calls, so the first call on a device must come before any stream capture.
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(PALU_ERR_CUDA, "palu_decode_attn_static: no current device");
  if (dev < 0 || dev >= kMaxDevices) return fail(PALU_ERR_CUDA, "palu_decode_attn_static: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(PALU_ERR_CUDA, "palu_decode_attn_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    e = cudaMemset(p, 0, sizeof(int32_t));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess)
      return fail(PALU_ERR_CUDA, "palu_decode_attn_static: clearing the status word: %s", cudaGetErrorString(e));
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return PALU_OK;
}

// Page-table checks shared by the paged decode and append entry points.
int validate_pages(const palu_page_table* pg, const palu_decode_dims* d) {
  if (!pg) return fail(PALU_ERR_INVALID, "pages is NULL");
  if (!pg->table) return fail(PALU_ERR_INVALID, "page table pointer is NULL");
  if (reinterpret_cast<uintptr_t>(pg->table) % 4 != 0) return fail(PALU_ERR_INVALID, "page table must be 4-byte aligned");
  const int bs = pg->block_size;
  if (bs != 16 && bs != 32 && bs != 64 && bs != 128)
    return fail(PALU_ERR_INVALID, "block_size must be 16, 32, 64 or 128, got %d", bs);
  if (pg->n_blocks <= 0) return fail(PALU_ERR_INVALID, "n_blocks must be positive, got %d", pg->n_blocks);
  if ((long long)pg->n_blocks * d->n_groups * bs > 0x7fffffffLL)
    return fail(PALU_ERR_INVALID, "n_blocks %d x n_groups %d x block_size %d cache rows exceed 2^31", pg->n_blocks,
                d->n_groups, bs);
  const long long need = ((long long)d->max_seq + bs - 1) / bs;
  if (pg->table_ld < need)
    return fail(PALU_ERR_INVALID, "table_ld %d is below the %lld blocks max_seq %d needs", pg->table_ld, need,
                d->max_seq);
  return PALU_OK;
}

int append(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_cache, void* v_cache,
           const palu_decode_dims* d, const palu_page_table* pg, palu_stream_t stream) {
  if (!new_k || !new_v || !cur_pos || !k_cache || !v_cache)
    return fail(PALU_ERR_INVALID, "append: every pointer must be set");
  if (d->batch <= 0 || d->n_groups <= 0 || d->max_seq <= 0)
    return fail(PALU_ERR_INVALID, "append: batch, n_groups and max_seq must be positive");
  if (d->r_k % 8 != 0 || d->r_v % 8 != 0 || d->r_k <= 0 || d->r_v <= 0)
    return fail(PALU_ERR_INVALID, "append: r_k and r_v must be positive multiples of 8 (got %d, %d)", d->r_k, d->r_v);
  palu::AppendParams p;
  p.new_k = static_cast<const __nv_bfloat16*>(new_k);
  p.new_v = static_cast<const __nv_bfloat16*>(new_v);
  p.cur_pos = cur_pos;
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.batch = d->batch;
  p.n_groups = d->n_groups;
  p.r_k = d->r_k;
  p.r_v = d->r_v;
  p.max_seq = d->max_seq;
  set_pages(p, pg);
  const long total = (long)d->batch * d->n_groups * (d->r_k / 8 + d->r_v / 8);
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  palu::palu_append_kernel<<<blocks, 256, 0, stream>>>(p);
  return cuda_check("append kernel launch");
}

// fp8 rows: `rows` source rows of r bf16 values -> codes + exponents (append mode when cur_pos is set).
int quantize_f8(const void* src, long rows, int r, void* codes, void* exps, const int32_t* cur_pos, int n_groups,
                int max_seq, cudaStream_t stream) {
  if (rows <= 0) return PALU_OK;
  palu::QuantF8Params p;
  p.src = static_cast<const __nv_bfloat16*>(src);
  p.rows = rows;
  p.r = r;
  p.codes = static_cast<uint8_t*>(codes);
  p.exps = static_cast<int8_t*>(exps);
  p.cur_pos = cur_pos;
  p.n_groups = n_groups;
  p.max_seq = max_seq;
  const long blocks = (rows + 7) / 8;  // 8 warps per block
  palu::palu_quantize_f8_kernel<<<(int)(blocks < 8192 ? blocks : 8192), 256, 0, stream>>>(p);
  return cuda_check("fp8 quantize kernel launch");
}

// fp4 rows: as quantize_f8, into r / 2 code bytes and r / 16 block exponents per row.
int quantize_f4(const void* src, long rows, int r, void* codes, void* exps, const int32_t* cur_pos, int n_groups,
                int max_seq, cudaStream_t stream) {
  if (rows <= 0) return PALU_OK;
  palu::QuantF4Params p;
  p.src = static_cast<const __nv_bfloat16*>(src);
  p.rows = rows;
  p.r = r;
  p.codes = static_cast<uint8_t*>(codes);
  p.exps = static_cast<int8_t*>(exps);
  p.cur_pos = cur_pos;
  p.n_groups = n_groups;
  p.max_seq = max_seq;
  const long blocks = (rows + 7) / 8;
  palu::palu_quantize_f4_kernel<<<(int)(blocks < 8192 ? blocks : 8192), 256, 0, stream>>>(p);
  return cuda_check("fp4 quantize kernel launch");
}

}  // namespace

extern "C" {

const char* palu_last_error(void) { return g_err.c_str(); }

const char* palu_version(void) { return "palu_b200 0.1.0 (sm_100a)"; }

int32_t palu_choose_splits(const palu_decode_dims* dims) {
  if (!dims || dims->n_kv_heads <= 0 || dims->n_q_heads <= 0) return 0;
  return splits_for(dims, true);
}

size_t palu_workspace_bytes(const palu_decode_dims* dims) {
  if (!dims || dims->n_kv_heads <= 0 || dims->n_q_heads <= 0) return 0;
  // enough for either kernel family, so palu_set_kernel may switch between calls
  const size_t a = ws_bytes(dims, choose_splits(dims)), b = ws_tc_bytes(dims, choose_splits_tc(dims));
  return a > b ? a : b;
}

int palu_set_kernel(int32_t which) {
  g_err.clear();
  if (which != PALU_KERNEL_AUTO && which != PALU_KERNEL_MMA && which != PALU_KERNEL_TC)
    return fail(PALU_ERR_INVALID, "kernel choice must be PALU_KERNEL_AUTO, _MMA or _TC");
  g_kernel_choice = which;
  return PALU_OK;
}

int palu_set_rope_mode(int32_t mode) {
  g_err.clear();
  if (mode != PALU_ROPE_ABSOLUTE && mode != PALU_ROPE_CHUNK_RELATIVE)
    return fail(PALU_ERR_INVALID, "RoPE mode must be PALU_ROPE_ABSOLUTE or PALU_ROPE_CHUNK_RELATIVE");
  g_rope_mode = mode;
  return PALU_OK;
}

int palu_set_wait_limit(int64_t wait_ns, int32_t starve_v) {
  g_err.clear();
  if (wait_ns < 0) return fail(PALU_ERR_INVALID, "wait_ns must be >= 0");
  g_wait_ns.store(wait_ns == 0 ? palu::tc::kWaitNs : (unsigned long long)wait_ns, std::memory_order_relaxed);
  g_starve_v.store(starve_v != 0, std::memory_order_relaxed);
  return PALU_OK;
}

int32_t palu_kernel_for(const palu_decode_dims* dims) {
  if (!dims) return -1;
  return use_tc(dims, true) ? PALU_KERNEL_TC : PALU_KERNEL_MMA;
}

int palu_read_status(void* workspace, int32_t* status, palu_stream_t stream) {
  g_err.clear();
  if (!status) return fail(PALU_ERR_INVALID, "status must be set");
  if (!workspace) {  // the static scratch of palu_decode_attn_static on the current device
    if (int st = static_scratch(&workspace)) return st;
  }
  if (cudaMemcpyAsync(status, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return cuda_check("reading the status word");
  if (*status != 0 && cudaMemsetAsync(workspace, 0, sizeof(int32_t), stream) != cudaSuccess)
    return cuda_check("clearing the status word");
  return PALU_OK;
}

int palu_decode_attn(const void* q, const void* k_lat, const void* v_lat, const void* u_k, int64_t u_k_ld,
                     const void* u_v, const void* cs_pairs, const int32_t* cur_pos, void* out, int32_t out_dtype,
                     void* workspace, size_t workspace_bytes, const palu_decode_dims* dims, float scale,
                     palu_stream_t stream) {
  g_err.clear();
  return run_decode(true, q, k_lat, v_lat, u_k, u_k_ld, u_v, cs_pairs, cur_pos, out, out_dtype, workspace,
                    workspace_bytes, dims, scale, stream);
}

int palu_decode_attn_static(const void* q, const void* k_lat, const void* v_lat, const void* u_k, int64_t u_k_ld,
                            const void* u_v, const void* cs_pairs, const int32_t* cur_pos, void* out,
                            int32_t out_dtype, const palu_decode_dims* dims, float scale, palu_stream_t stream) {
  g_err.clear();
  int st = validate(dims, true, u_v != nullptr);
  if (st) return st;
  // The same bound for every kernel family, so whether a shape is accepted does not depend on
  // palu_set_kernel: what palu_workspace_bytes() reports must fit.
  const size_t need = palu_workspace_bytes(dims);
  if (need > kStaticScratchBytes)
    return fail(PALU_ERR_WORKSPACE, "palu_decode_attn_static: these shapes need %zu bytes of scratch, more than the "
                "%zu-byte static scratch; use palu_decode_attn with a caller workspace", need, kStaticScratchBytes);
  void* scratch = nullptr;
  st = static_scratch(&scratch);
  if (st) return st;
  return run_decode(true, q, k_lat, v_lat, u_k, u_k_ld, u_v, cs_pairs, cur_pos, out, out_dtype, scratch,
                    kStaticScratchBytes, dims, scale, stream);
}

int palu_decode_attn_f8(const void* q, const void* k_codes, const void* v_codes, const int8_t* k_exp,
                        const int8_t* v_exp, const void* u_k, int64_t u_k_ld, const void* u_v, const void* cs_pairs,
                        const int32_t* cur_pos, void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                        const palu_decode_dims* dims, float scale, palu_stream_t stream) {
  g_err.clear();
  if (!k_exp || !v_exp) return fail(PALU_ERR_INVALID, "fp8 latents need both exponent arrays");
  return run_decode(true, q, k_codes, v_codes, u_k, u_k_ld, u_v, cs_pairs, cur_pos, out, out_dtype, workspace,
                    workspace_bytes, dims, scale, stream, nullptr, k_exp, v_exp);
}

int palu_quantize_latents_f8(const void* latents, int64_t rows, int32_t r, void* codes, int8_t* exps,
                             palu_stream_t stream) {
  g_err.clear();
  if (rows < 0 || r < 16 || r > 256 || r % 16 != 0)
    return fail(PALU_ERR_INVALID, "quantize_latents_f8: rows >= 0 and r a multiple of 16 in [16, 256] (got %lld, %d)",
                (long long)rows, r);
  if (rows > 0 && (!latents || !codes || !exps)) return fail(PALU_ERR_INVALID, "quantize_latents_f8: every pointer must be set");
  return quantize_f8(latents, (long)rows, r, codes, exps, nullptr, 1, 1, stream);
}

int palu_append_latents_f8(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_codes, void* v_codes,
                           int8_t* k_exp, int8_t* v_exp, const palu_decode_dims* d, palu_stream_t stream) {
  g_err.clear();
  if (!d) return fail(PALU_ERR_INVALID, "dims is NULL");
  if (!new_k || !new_v || !cur_pos || !k_codes || !v_codes || !k_exp || !v_exp)
    return fail(PALU_ERR_INVALID, "append_latents_f8: every pointer must be set");
  if (d->batch <= 0 || d->n_groups <= 0 || d->max_seq <= 0)
    return fail(PALU_ERR_INVALID, "append: batch, n_groups and max_seq must be positive");
  auto r_ok = [](int r) { return r >= 16 && r <= 256 && r % 16 == 0; };
  if (!r_ok(d->r_k) || !r_ok(d->r_v))
    return fail(PALU_ERR_INVALID, "append_latents_f8: r_k and r_v must be multiples of 16 in [16, 256] (got %d, %d)",
                d->r_k, d->r_v);
  const long rows = (long)d->batch * d->n_groups;
  if (int st = quantize_f8(new_k, rows, d->r_k, k_codes, k_exp, cur_pos, d->n_groups, d->max_seq, stream)) return st;
  return quantize_f8(new_v, rows, d->r_v, v_codes, v_exp, cur_pos, d->n_groups, d->max_seq, stream);
}

int palu_decode_attn_f4(const void* q, const void* k_codes, const void* v_codes, const int8_t* k_exp,
                        const int8_t* v_exp, const void* u_k, int64_t u_k_ld, const void* u_v, const void* cs_pairs,
                        const int32_t* cur_pos, void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                        const palu_decode_dims* dims, float scale, palu_stream_t stream) {
  g_err.clear();
  if (!k_exp || !v_exp) return fail(PALU_ERR_INVALID, "fp4 latents need both exponent arrays");
  return run_decode(true, q, k_codes, v_codes, u_k, u_k_ld, u_v, cs_pairs, cur_pos, out, out_dtype, workspace,
                    workspace_bytes, dims, scale, stream, nullptr, k_exp, v_exp, true);
}

int palu_quantize_latents_f4(const void* latents, int64_t rows, int32_t r, void* codes, int8_t* exps,
                             palu_stream_t stream) {
  g_err.clear();
  if (rows < 0 || r < 16 || r > 256 || r % 16 != 0)
    return fail(PALU_ERR_INVALID, "quantize_latents_f4: rows >= 0 and r a multiple of 16 in [16, 256] (got %lld, %d)",
                (long long)rows, r);
  if (rows > 0 && (!latents || !codes || !exps)) return fail(PALU_ERR_INVALID, "quantize_latents_f4: every pointer must be set");
  return quantize_f4(latents, (long)rows, r, codes, exps, nullptr, 1, 1, stream);
}

int palu_append_latents_f4(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_codes, void* v_codes,
                           int8_t* k_exp, int8_t* v_exp, const palu_decode_dims* d, palu_stream_t stream) {
  g_err.clear();
  if (!d) return fail(PALU_ERR_INVALID, "dims is NULL");
  if (!new_k || !new_v || !cur_pos || !k_codes || !v_codes || !k_exp || !v_exp)
    return fail(PALU_ERR_INVALID, "append_latents_f4: every pointer must be set");
  if (d->batch <= 0 || d->n_groups <= 0 || d->max_seq <= 0)
    return fail(PALU_ERR_INVALID, "append: batch, n_groups and max_seq must be positive");
  auto r_ok = [](int r) { return r >= 16 && r <= 256 && r % 16 == 0; };
  if (!r_ok(d->r_k) || !r_ok(d->r_v))
    return fail(PALU_ERR_INVALID, "append_latents_f4: r_k and r_v must be multiples of 16 in [16, 256] (got %d, %d)",
                d->r_k, d->r_v);
  const long rows = (long)d->batch * d->n_groups;
  if (int st = quantize_f4(new_k, rows, d->r_k, k_codes, k_exp, cur_pos, d->n_groups, d->max_seq, stream)) return st;
  return quantize_f4(new_v, rows, d->r_v, v_codes, v_exp, cur_pos, d->n_groups, d->max_seq, stream);
}

int palu_decode_attn_paged(const void* q, const void* k_cache, const void* v_cache, const void* u_k, int64_t u_k_ld,
                           const void* u_v, const void* cs_pairs, const int32_t* cur_pos, const palu_page_table* pages,
                           void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                           const palu_decode_dims* dims, float scale, palu_stream_t stream) {
  g_err.clear();
  if (!dims) return fail(PALU_ERR_INVALID, "dims is NULL");
  if (int st = validate_pages(pages, dims)) return st;
  return run_decode(true, q, k_cache, v_cache, u_k, u_k_ld, u_v, cs_pairs, cur_pos, out, out_dtype, workspace,
                    workspace_bytes, dims, scale, stream, pages);
}

int palu_plain_gqa_decode(const void* q, const void* k, const void* v, const int32_t* cur_pos, void* out,
                          int32_t out_dtype, void* workspace, size_t workspace_bytes, const palu_decode_dims* dims,
                          float scale, palu_stream_t stream) {
  g_err.clear();
  return run_decode(false, q, k, v, nullptr, 128, nullptr, nullptr, cur_pos, out, out_dtype, workspace,
                    workspace_bytes, dims, scale, stream);
}


int palu_append_latents(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_cache, void* v_cache,
                        const palu_decode_dims* d, palu_stream_t stream) {
  g_err.clear();
  if (!d) return fail(PALU_ERR_INVALID, "dims is NULL");
  return append(new_k, new_v, cur_pos, k_cache, v_cache, d, nullptr, stream);
}

int palu_append_latents_paged(const void* new_k, const void* new_v, const int32_t* cur_pos,
                              const palu_page_table* pages, void* k_cache, void* v_cache, const palu_decode_dims* d,
                              palu_stream_t stream) {
  g_err.clear();
  if (!d) return fail(PALU_ERR_INVALID, "dims is NULL");
  if (d->n_groups <= 0 || d->max_seq <= 0) return fail(PALU_ERR_INVALID, "append: n_groups and max_seq must be positive");
  if (int st = validate_pages(pages, d)) return st;
  return append(new_k, new_v, cur_pos, k_cache, v_cache, d, pages, stream);
}

int palu_rope_q_append(const void* qkv, int64_t ld, int32_t qkv_dtype, const float* cos, const float* sin,
                       const int32_t* cur_pos, void* q_out, void* k_cache, void* v_cache, const palu_page_table* pages,
                       const palu_decode_dims* d, palu_stream_t stream) {
  g_err.clear();
  if (!d) return fail(PALU_ERR_INVALID, "dims is NULL");
  if (!qkv || !cos || !sin || !cur_pos || !q_out || !k_cache || !v_cache)
    return fail(PALU_ERR_INVALID, "rope_q_append: every pointer must be set");
  if (d->batch <= 0 || d->n_q_heads <= 0 || d->n_groups <= 0 || d->max_seq <= 0 || d->r_k <= 0 || d->r_v <= 0)
    return fail(PALU_ERR_INVALID, "rope_q_append: batch, n_q_heads, n_groups, r_k, r_v and max_seq must be positive");
  if (d->head_dim != 128) return fail(PALU_ERR_INVALID, "head_dim must be 128, got %d", d->head_dim);
  if (qkv_dtype != PALU_BF16 && qkv_dtype != PALU_F32) return fail(PALU_ERR_INVALID, "qkv dtype must be bf16 or f32");
  const long long width = (long long)d->n_q_heads * 128 + (long long)d->n_groups * (d->r_k + d->r_v);
  if (ld < width)
    return fail(PALU_ERR_INVALID, "qkv rows of %lld elements cannot hold the %lld q and latent values", (long long)ld,
                width);
  if (reinterpret_cast<uintptr_t>(q_out) % 4 != 0) return fail(PALU_ERR_INVALID, "q_out must be 4-byte aligned");
  if (pages)
    if (int st = validate_pages(pages, d)) return st;
  palu::RopeAppendParams p;
  p.qkv = qkv;
  p.ld = (long)ld;
  p.cos = cos;
  p.sin = sin;
  p.cur_pos = cur_pos;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.batch = d->batch;
  p.n_q = d->n_q_heads;
  p.n_groups = d->n_groups;
  p.r_k = d->r_k;
  p.r_v = d->r_v;
  p.max_seq = d->max_seq;
  set_pages(p, pages);
  const long total = (long)d->batch * (d->n_q_heads * 64 + d->n_groups * (d->r_k + d->r_v));
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  if (qkv_dtype == PALU_F32)
    palu::palu_rope_q_append_kernel<float><<<blocks, 256, 0, stream>>>(p);
  else
    palu::palu_rope_q_append_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(p);
  return cuda_check("rope_q_append kernel launch");
}

int palu_add_rms_norm(float* h, const void* delta, int32_t delta_dtype, const float* w, void* out, int32_t rows,
                      int32_t dim, float eps, palu_stream_t stream) {
  g_err.clear();
  if (!h || !w || !out) return fail(PALU_ERR_INVALID, "add_rms_norm: h, w and out must be set");
  if (delta_dtype != PALU_BF16 && delta_dtype != PALU_F32)
    return fail(PALU_ERR_INVALID, "add_rms_norm: delta dtype must be bf16 or f32");
  if (rows <= 0 || dim <= 0 || dim % 4 != 0)
    return fail(PALU_ERR_INVALID, "add_rms_norm: rows must be positive and dim a positive multiple of 4 (got %d, %d)",
                rows, dim);
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(out)) % 16 != 0)
    return fail(PALU_ERR_INVALID, "add_rms_norm: h, delta, w and out must be 16-byte aligned");
  if (delta_dtype == PALU_BF16)
    palu::palu_add_rms_norm_kernel<__nv_bfloat16><<<rows, palu::kNormThreads, 0, stream>>>(
        h, static_cast<const __nv_bfloat16*>(delta), w, static_cast<__nv_bfloat16*>(out), dim, eps);
  else
    palu::palu_add_rms_norm_kernel<float><<<rows, palu::kNormThreads, 0, stream>>>(
        h, static_cast<const float*>(delta), w, static_cast<__nv_bfloat16*>(out), dim, eps);
  return cuda_check("add_rms_norm kernel launch");
}

int palu_swiglu(const void* gu, int64_t ld, int32_t f, void* out, int32_t rows, palu_stream_t stream) {
  g_err.clear();
  if (!gu || !out) return fail(PALU_ERR_INVALID, "swiglu: gu and out must be set");
  if (rows <= 0 || f <= 0 || ld < 2LL * f)
    return fail(PALU_ERR_INVALID, "swiglu: rows and f must be positive and rows of gu hold 2 f values (got %d, %d, %lld)",
                rows, f, (long long)ld);
  if (f % 8 == 0 && ld % 8 == 0 && rows <= 65535 &&
      (reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(out)) % 16 == 0) {
    const dim3 grid((f / 8 + 127) / 128, rows);
    palu::palu_swiglu8_kernel<<<grid, 128, 0, stream>>>(static_cast<const __nv_bfloat16*>(gu), (long)ld, f,
                                                        static_cast<__nv_bfloat16*>(out));
    return cuda_check("swiglu kernel launch");
  }
  const long total = (long)rows * f;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  palu::palu_swiglu_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(gu), (long)ld, f,
                                                       static_cast<__nv_bfloat16*>(out), rows);
  return cuda_check("swiglu kernel launch");
}

int palu_pack_cs_table(const void* cs_tab, int64_t ld, int32_t in_dtype, void* cs_pairs, int32_t rows,
                       palu_stream_t stream) {
  g_err.clear();
  if (!cs_tab || !cs_pairs || rows <= 0) return fail(PALU_ERR_INVALID, "cs_tab: table, output and rows must be set");
  if (ld < 256) return fail(PALU_ERR_INVALID, "cs_tab rows must hold [cos | sin] (>= 256 columns), got %lld",
                            (long long)ld);
  if (in_dtype != PALU_BF16 && in_dtype != PALU_F32) return fail(PALU_ERR_INVALID, "cs_tab dtype must be bf16 or f32");
  const long total = (long)rows * 64;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  palu::palu_pack_cs_kernel<<<blocks, 256, 0, stream>>>(cs_tab, ld, in_dtype == PALU_F32,
                                                         static_cast<uint32_t*>(cs_pairs), rows);
  return cuda_check("cs_tab pack kernel launch");
}

}  // extern "C"
