// Flash-decode over Palu latent caches on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA per (range, KV head): the KV head's 128-token tiles over all batch rows (positions 0..cur_pos[b]
// of each row, rows in order) are cut into `ctas` equal contiguous ranges (see TcParams), so every CTA
// streams the same number of tiles in a single wave whatever the batch and the rows' lengths; the pipeline
// runs on across row boundaries, where each group writes a partial (O, m, l) for the row it leaves
// (combine.cuh merges a row's partials). Two groups work on alternate tiles of the range (group g on
// CTA-local tiles t with t % 2 == g), so two tiles are in flight per CTA. Each group has its own warps,
// rings, barriers and TMEM columns (24 warps in all, see role_of): a K+table TMA producer, a V producer, a
// QK+PV issuer, a reconstruct issuer (a single thread issues at most one tcgen05.mma per ~64 cycles
// whatever its shape, measured on B200, so the MMAs are split over two threads; QK(j) and PV(j - 1) stay on
// one thread, in that order: with PV on a third thread its MMAs interleave with QK's in the tensor pipe and
// the op measured 20 % slower on B200), 4 RoPE warps and 4 softmax warps (a warp of either kind owns the 32
// TMEM lanes of its SMSP quarter: 32 token rows of the tile, or 32 latent dims of the PV output).
// At start the RoPE warps stage U_k (bf16) in shared memory with its head dims reordered as
// [even dims | odd dims] per half of the frequencies, so that D_k holds each rotation pair (2f, 2f+1) 32
// columns apart and the rotation of two adjacent frequencies is one packed half2 operation. The softmax
// warps stage Q^T (fp16, the same reordering) per batch row, double-buffered per group.
// Per group-local tile j (CTA-local tile t = g + 2 j):
//   MMA      D_k[128 tok x 128 dim] (f32) = lat_k (smem, K-major) x U_k (smem, MN-major), as two N = 64 halves
//            (frequencies 0..31 and 32..63, each half its even dims then its odd dims)
//   RoPE     K row -> fp16, rotated in half2 arithmetic with the fp16 table -> K_rot into its own TMEM
//            columns: the A operand of QK (fp16 keeps 11 significant bits; q is bf16, exact in fp16)
//   MMA      D_s[128 tok x 16] (f32) = K_rot (TMEM) x Q^T (smem, fp16)
//   softmax  online softmax over the query heads (exp2 domain); P^T as bf16 hi + lo -> smem
//   MMA      D_o[128 lat x 16] (f32) = V^T (smem, MN-major: the V tile exactly as TMA wrote it) x P^T
//   softmax  thread c (latent dim c) accumulates O[h][c] = O * alpha + hi + lo in registers
// RoPE works by halves of D_k: as soon as RoPE(j) has finished half h, the reconstruction of half h of
// tile j + 1 and the QK MMAs of half h of tile j are issued, so the reconstruct latency overlaps the
// rotation of the other half; RoPE(j + 1) overlaps softmax(j) and PV(j - 1). D_s, D_o and P are
// double-buffered by j % 2, and every consumer releases what it read with its own barrier, so no barrier
// runs two phases ahead of a waiter. Every wait is bounded (1 s of globaltimer by default): on expiry the CTA records a
// status code, all roles stop (the multi-lane warps agree on it, so none is left divergent), copies and
// MMAs in flight are drained, and TMEM is freed.
// Latents wider than 128 (up to 256: the grouped G-LRD caches) run the same roles with ONE pipeline per CTA
// (NP = 1; group 1's warps only help stage U_k): U_k alone is then 64 KB and a K or V tile 64 KB, so K streams
// through a ring of 64-wide boxes into a double-buffered D_k, a single V stage fits, and V^T is two M = 128
// blocks (latent dims 0..127 and 128..255) whose PV results sit in TMEM columns 256..319, the columns group 1
// would have used.
// Low-bit latent caches (F8: e4m3 codes with a scale per row; F4: e2m1 codes with a scale per 16 values) keep
// the two pipelines; their K and V producer warps work as whole warps, converting each tile landed by TMA in
// place into the f16 tile the MMAs read, and the reconstruction and PV run on f16 operands.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "palu_common.cuh"

namespace palu {
namespace tc {

// Warps: 8 role warps (see role_of; single-lane, except the low-bit producers), then 8 RoPE warps and 8
// softmax warps (4 per group). A RoPE or softmax warp w owns TMEM lanes 32 (w % 4) .. + 31.
constexpr int kRoleWarps = 8;
constexpr int kRopeWarp0 = kRoleWarps;
constexpr int kSoftWarp0 = kRoleWarps + 8;
constexpr int kThreads = (kRoleWarps + 16) * 32;
constexpr int kTile = 128;
constexpr int kBox = 16384;             // one TMA box: 128 rows x 128 B
constexpr int kTmemCols = 512;
constexpr int kGrpCols = 256;           // TMEM columns reserved per softmax group
constexpr int kColDk = 0;               // 128 columns: f32 K tile, two halves of [even | odd] dims (reconstruct output)
constexpr int kColA = 128;              // 64 columns: fp16 K_rot, the A operand of QK (packed 2 per column)
constexpr int kColDs = 192;             // 2 x 16 columns: scores, double-buffered
constexpr int kColDo = 224;             // 2 x 16 columns: PV result, double-buffered (two pipelines)
constexpr int kColDoWide = 256;         // one pipeline: 2 buffers x 2 M-blocks x 16 columns at 256..319
constexpr int kColDk2 = 320;            // one pipeline: the second D_k buffer (128 columns)
constexpr unsigned long long kWaitNs = 1000000000ull;  // bound on any single wait

enum : int { kStatusOk = 0, kStatusTimeout = 1 };

struct TcParams {
  const __nv_bfloat16* q;   // [B][n_q][128]
  const __nv_bfloat16* u_k; // [n_kv][r_k] rows of ld_u elements (U_k in the first 128)
  const int32_t* cur_pos;   // [B]
  float* ws_o;              // partial records (tc_rec_direct / tc_rec_edge), each [rep][rv]
  float* ws_ml;             // the same records' [rep][5]: m, then the 4 row quarters' l
  int* status;              // device status word, 0 = ok
  int batch, n_q, n_kv, n_groups, rk, rv, max_seq, ctas, rep, ld_u;
  float scale_log2;
  // Paged caches (null page_table: contiguous [B][n_groups][max_seq][r] caches). Row b's positions
  // j*bs .. j*bs+bs-1 (bs = 1 << blk_shift) sit in physical block page_table[b * table_ld + j] of the
  // [n_blocks][n_groups][bs][r] caches; the tensor maps then have boxes of bs rows.
  const int32_t* page_table;
  int table_ld, blk_shift, n_blocks;
  // Bound on any single wait (ns), and a test switch: nonzero makes group 0's V producer issue no loads, so
  // that a wait runs out on purpose (the test of the timeout path; never set in normal use).
  unsigned long long wait_ns;
  int starve_v;
  // Nonzero when every CTA of the grid is resident at once (one wave): the merge, a programmatic dependent,
  // may then be launched as soon as the CTAs start, so its CTAs take SMs as decode CTAs finish and wait there
  // (griddepcontrol.wait) instead of being launched after the last one. With more CTAs than one wave the
  // trigger stays implicit at exit, so no merge CTA can hold an SM a decode CTA is still waiting for.
  int pdl_early;
  // fp8 latent caches (the F8 kernels): e4m3 codes in the caches above, and per (batch row, latent head,
  // position) the power-of-two exponent k of the row's scale, [B][n_groups][max_seq] int8 each; a cached
  // value is code * 2^k. fp4 caches (F8 and F4): e2m1 codes, two per byte (the first in the low nibble),
  // and one exponent per 16 values of a row, [B][n_groups][max_seq][r / 16].
  const int8_t* k_exp;
  const int8_t* v_exp;
  // Chunk-relative RoPE (the reference's Phase 2, fused.py:1-14): nonzero rotates key position
  // p = 128 t + j by the table rows j (0..127, loaded once per CTA) and rotates the query of tile t by
  // row 128 t the other way, R_p = R_{128 t} R_j, instead of reading row p for every key. The host launches
  // the kernel's REL instantiation for it. `cs` is the packed table (palu_pack_cs_table rows) the query
  // rotation reads.
  int rel;
  const uint32_t* cs;
};
// Whether a layout holds the four table chunk slots that chunk-relative RoPE keeps for rows 0..127.
template <class Lay, int NP>
__host__ __device__ constexpr bool rel_fits() { return NP * Lay::T_SLOTS >= 4; }

// Work split: the tiles of one KV head over all batch rows, in row order (row b has ceil(L_b / 128)
// tiles, L_b = cur_pos[b] + 1 clamped to [0, max_seq]), are cut into `ctas` equal contiguous ranges, one
// per CTA, so every CTA streams the same number of tiles whatever the rows' lengths. A row's tiles inside
// one CTA form a segment; each group of the CTA writes one partial record (O, m, l) per segment
// (tc_rec_direct / tc_rec_edge). The merge (combine.cuh) finds a row's records from the same split.
PALU_DEVINL int row_len(const TcParams& p, int b) {
  const int L = p.cur_pos[b] + 1;
  return L < 0 ? 0 : (L > p.max_seq ? p.max_seq : L);
}
PALU_DEVINL int row_tiles(const TcParams& p, int b) { return tc_row_tiles(p.cur_pos, b, p.max_seq); }

// A batch row's tiles inside this CTA's range: tiles ta .. ta + cnt - 1 of row b, which are the CTA's
// tiles kb .. kb + cnt - 1 (CTA-local order). cnt == 0 marks the end of the range.
struct RowSeg {
  int b, ta, cnt, kb;
};
PALU_DEVINL RowSeg seg_next(const TcParams& p, int n, const RowSeg& s) {
  RowSeg r{s.b, 0, 0, s.kb + s.cnt};
  if (r.kb >= n) return r;
  int nb = 0;
  do {
    if (++r.b >= p.batch) return RowSeg{r.b, 0, 0, n};  // unreachable while cur_pos is unchanged
    nb = row_tiles(p, r.b);
  } while (nb == 0);
  r.cnt = min(nb, n - r.kb);
  return r;
}
// With np pipelines (groups) per CTA (1 or 2), group g takes the CTA-local tiles k with k % np == g: its first
// tile in segment s and their count.
template <int NP>
PALU_DEVINL int seg_group_first(const RowSeg& s, int g) { return s.kb + ((g - s.kb) & (NP - 1)); }
template <int NP>
PALU_DEVINL int seg_group_count(const RowSeg& s, int g) {
  const int kf = seg_group_first<NP>(s, g);
  return kf < s.kb + s.cnt ? (s.kb + s.cnt - kf + NP - 1) / NP : 0;
}
// Group g's tiles in order, with their row, tile within the row and group-segment index (segments in which
// the group has tiles, counted from 0).
template <int NP>
struct GroupTiles {
  RowSeg s;
  int g, n, x, cnt, kf, sigma, len;  // len: positions the current row attends
  PALU_DEVINL void init(const TcParams& p, const RowSeg& s0, int g_, int n_) {
    s = s0;
    g = g_;
    n = n_;
    sigma = -1;
    settle(p);
  }
  PALU_DEVINL void settle(const TcParams& p) {
    while (s.cnt > 0 && (cnt = seg_group_count<NP>(s, g)) == 0) s = seg_next(p, n, s);
    if (s.cnt > 0) {
      kf = seg_group_first<NP>(s, g);
      x = 0;
      ++sigma;
      len = row_len(p, s.b);
    }
  }
  PALU_DEVINL bool valid() const { return s.cnt > 0; }
  PALU_DEVINL int tile() const { return s.ta + (kf - s.kb) + NP * x; }
  PALU_DEVINL bool first() const { return x == 0; }
  PALU_DEVINL void next(const TcParams& p) {
    if (++x >= cnt) {
      s = seg_next(p, n, s);
      settle(p);
    }
  }
  PALU_DEVINL void next_segment(const TcParams& p) {
    s = seg_next(p, n, s);
    settle(p);
  }
};

// Shared memory per CTA: the fixed buffers plus three rings, K (NS_K stages), V (NS_V stages) and the RoPE
// table (T_SLOTS chunk slots per group). With two pipelines, stage i of the K and V rings holds tiles of
// group i % 2 only. The first (NS_K, NS_V, T_SLOTS) choice that fits is used: with two pipelines, two K
// stages per group, one V stage per group and a whole tile of table chunks when the latents are at most 64
// wide. With one pipeline (latents up to 256 wide) a K stage is one 64-wide box (the reconstruction streams
// a tile box by box), and the choice is three K boxes, one V tile and a whole tile of table chunks.
constexpr int kTabChunkBytes = 8192;  // table chunk: 128 rows x 16 pairs x 4 B (SWIZZLE_64B)
constexpr int kSmemBudget = 227 * 1024;
constexpr int layout_need(int fixed, int kb, int vb, int nk, int nv, int t, int np) {
  return fixed + nk * kb + nv * vb + np * t * kTabChunkBytes;
}
constexpr int layout_pick(int fixed, int kb, int vb, int np, bool lowbit = false) {
  // low-bit caches: a second V stage per group first (the V conversion sits between a slot's release and
  // the next PV; measured 3 % faster at r 64), at the cost of one table chunk slot per group
  if (np == 2 && lowbit && layout_need(fixed, kb, vb, 4, 4, 3, 2) <= kSmemBudget) return 443;
  constexpr int c2[4][3] = {{4, 2, 4}, {2, 2, 4}, {4, 2, 2}, {2, 2, 2}};
  constexpr int c1[5][3] = {{4, 1, 4}, {3, 1, 4}, {2, 1, 4}, {2, 1, 2}, {1, 1, 2}};
  if (np == 2) {
    for (int i = 0; i < 4; ++i)
      if (layout_need(fixed, kb, vb, c2[i][0], c2[i][1], c2[i][2], 2) <= kSmemBudget)
        return c2[i][0] * 100 + c2[i][1] * 10 + c2[i][2];
    return 222;
  }
  for (int i = 0; i < 5; ++i)
    if (layout_need(fixed, kb, vb, c1[i][0], c1[i][1], c1[i][2], 1) <= kSmemBudget)
      return c1[i][0] * 100 + c1[i][1] * 10 + c1[i][2];
  return 112;
}

// NP pipelines per CTA: 2 (latents at most 128 wide), or 1 (up to 256 wide: U_k alone is then 64 KB and a
// K or V tile 64 KB, so one pipeline, a ring of K boxes and a single V stage is what fits).
template <int KBK, int KBV, int NP, bool LOWBIT = false>
struct Layout {
  static constexpr int K_BYTES = NP == 1 ? kBox : KBK * kBox;  // one pipeline: a K ring stage is one box
  static constexpr int V_BYTES = KBV * kBox;
  static constexpr int TCH_BYTES = kTabChunkBytes;
  static constexpr int U_BYTES = KBK * 2 * 64 * 128;  // 2 N-blocks x (<= 64 KBK rows) x 128 B
  static constexpr int Q_BYTES = 2 * 2048;            // one buffer: 2 K-blocks x 16 rows x 128 B (fp16)
  static constexpr int P_BYTES = 2 * 2048;            // one buffer: 2 K-blocks x 16 rows x 128 B (bf16)
  static constexpr int MISC_BYTES = 2048;
  static constexpr int FIXED = U_BYTES + 2 * NP * Q_BYTES + 2 * NP * P_BYTES + MISC_BYTES + 1024;
  static constexpr int PICK = layout_pick(FIXED, K_BYTES, V_BYTES, NP, LOWBIT);
  static constexpr int NS_K = PICK / 100, NS_V = PICK / 10 % 10, T_SLOTS = PICK % 10;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + NS_K * K_BYTES;
  static constexpr int OFF_TAB = OFF_V + NS_V * V_BYTES;
  static constexpr int OFF_U = OFF_TAB + NP * T_SLOTS * TCH_BYTES;
  static constexpr int OFF_Q = OFF_U + U_BYTES;
  static constexpr int OFF_P = OFF_Q + 2 * NP * Q_BYTES;  // Q: [group][segment parity], P: [group][tile parity]
  static constexpr int OFF_MISC = OFF_P + 2 * NP * P_BYTES;
  static constexpr int TOTAL = OFF_MISC + MISC_BYTES + 1024;  // + slack to align the base to 1024
  static_assert(TOTAL <= kSmemBudget, "shared memory budget");
  static_assert(NS_K % NP == 0 && NS_V % NP == 0, "every group owns the same number of K and V stages");
};

// ---- PTX wrappers -----------------------------------------------------------------------------------

PALU_DEVINL void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
PALU_DEVINL void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
PALU_DEVINL void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
PALU_DEVINL bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
PALU_DEVINL bool mbar_test(uint32_t bar, uint32_t parity) {  // non-blocking
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
PALU_DEVINL unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}

// Bounded wait for `parity` on `bar` (at most `limit_ns`). Returns false on timeout or when another role
// already gave up. The polling loop is one out-of-line function: inlined at each of the ~20 wait sites it
// grew the kernel body past what the instruction cache serves well (no_instruction stalls), and the op
// measured 2-4 % faster on B200 with one shared copy.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                            unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return mbar_try(bar, parity);
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      atomicExch(status, kStatusTimeout);
      return false;
    }
  }
}
PALU_DEVINL bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                           unsigned long long limit_ns) {
  if (mbar_try(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, abort_flag, status, limit_ns);
}

// Bounded wait used on the abort path, to let copies already in flight land before the CTA exits.
PALU_DEVINL void mbar_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

PALU_DEVINL void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
PALU_DEVINL void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
PALU_DEVINL void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor, SWIZZLE_128B, version 1 (sm_100). Offsets in bytes.
PALU_DEVINL uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16 with f32 accumulate, M = 128. fmt: 0 = f16, 1 = bf16 (A and B alike).
// M = 128 or 64 (an M = 64 accumulator holds its rows in lanes 0..15 of each 32-lane quarter).
__host__ __device__ constexpr uint32_t idesc_f16(int n, uint32_t fmt, bool a_mn_major, bool b_mn_major, int m = 128) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

PALU_DEVINL void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
PALU_DEVINL void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
PALU_DEVINL void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
PALU_DEVINL void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
PALU_DEVINL void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// Four e4m3 codes (one 32-bit word, lowest byte first) -> two f16 pairs, exactly (every e4m3 value is an f16
// value).
PALU_DEVINL void e4m3x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 a, b;\n mov.b32 {a, b}, %2;\n cvt.rn.f16x2.e4m3x2 %0, a;\n cvt.rn.f16x2.e4m3x2 %1, b;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}
PALU_DEVINL uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  const __half2 m = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&m);
}
// 16 staged e4m3 codes of one cached row (v) -> codes 16 c .. 16 c + 15 of row r of f16 K-major SWIZZLE_128B
// box `box` of the tile (its 16-byte chunks 2 c and 2 c + 1), converted exactly and, when SCALED,
// multiplied by the f16 pair s2 = (2^k, 2^k).
template <bool SCALED>
PALU_DEVINL void f8_store_chunk(unsigned char* tile, int r, uint4 v, uint32_t s2, int box, int c) {
  uint32_t o[8];
  e4m3x4_to_f16x4(v.x, o[0], o[1]);
  e4m3x4_to_f16x4(v.y, o[2], o[3]);
  e4m3x4_to_f16x4(v.z, o[4], o[5]);
  e4m3x4_to_f16x4(v.w, o[6], o[7]);
  if constexpr (SCALED) {
#pragma unroll
    for (int x = 0; x < 8; ++x) o[x] = hmul2_u32(o[x], s2);
  }
  unsigned char* brow = tile + box * kBox + r * 128;
  *reinterpret_cast<uint4*>(brow + (((2 * c) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(brow + (((2 * c + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
}
// The f16 pair (2^k, 2^k): normal for k >= -14, subnormal down to 2^-24, 0 below (rows that small hold
// values under 448 * 2^-25, which the f16 tile cannot carry).
PALU_DEVINL uint32_t f8_scale_pair(int k) {
  const uint32_t h = k >= -14 ? (uint32_t)(k + 15) << 10 : (k >= -24 ? 1u << (k + 24) : 0u);
  return h | (h << 16);
}
// One cached row r of an NBOX-box tile converted in place, the codes staged at `stage` (NBOX x 64 per row).
// One box: f16 row r overlaps staged rows 2 r - 128 and 2 r - 127 (other threads'), so `all_read` must
// return only once every thread that owns those rows has read them (false: that wait gave up). Two boxes:
// box 0 lies below the staging half, converted 16 codes at a time; box 1's row r is the staged row r
// itself, so its 64 codes are read before any is written. Each thread starts at a chunk rotated by its row
// so that the 8 threads of a shared-memory phase read distinct banks.
template <int NBOX, bool SCALED, class AllRead>
PALU_DEVINL bool f8_convert_row(unsigned char* tile, const unsigned char* stage, int r, int k, AllRead all_read) {
  const uint32_t s2 = SCALED ? f8_scale_pair(k) : 0u;
  const uint4* src = reinterpret_cast<const uint4*>(stage + r * (NBOX * 64));
  const int rot = NBOX == 1 ? (r >> 1) : r;
  if constexpr (NBOX == 1) {
    uint4 in[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) in[i] = src[(i + rot) & 3];
    if (!all_read()) return false;
#pragma unroll
    for (int i = 0; i < 4; ++i) f8_store_chunk<SCALED>(tile, r, in[i], s2, 0, (i + rot) & 3);
  } else {
#pragma unroll 1
    for (int i = 0; i < 4; ++i) f8_store_chunk<SCALED>(tile, r, src[(i + rot) & 3], s2, 0, (i + rot) & 3);
    uint4 in[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) in[i] = src[4 + ((i + rot) & 3)];
#pragma unroll
    for (int i = 0; i < 4; ++i) f8_store_chunk<SCALED>(tile, r, in[i], s2, 1, (i + rot) & 3);
  }
  return true;
}
// fp4: 16 staged e2m1 codes of one row (v: 8 bytes, the first code of each byte in its low nibble) ->
// codes 16 c .. 16 c + 15 of row r of f16 box `box` (chunks 2 c, 2 c + 1), converted exactly and multiplied by
// the block's f16 pair s2 = (2^k, 2^k).
PALU_DEVINL void e2m1x8_to_f16x8(uint32_t w, uint32_t& o0, uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  asm("{\n .reg .b8 a, b, c, d;\n mov.b32 {a, b, c, d}, %4;\n cvt.rn.f16x2.e2m1x2 %0, a;\n"
      " cvt.rn.f16x2.e2m1x2 %1, b;\n cvt.rn.f16x2.e2m1x2 %2, c;\n cvt.rn.f16x2.e2m1x2 %3, d;\n}\n"
      : "=r"(o0), "=r"(o1), "=r"(o2), "=r"(o3)
      : "r"(w));
}
PALU_DEVINL void f4_store_chunk(unsigned char* tile, int r, uint2 v, uint32_t s2, int box, int c) {
  uint32_t o[8];
  e2m1x8_to_f16x8(v.x, o[0], o[1], o[2], o[3]);
  e2m1x8_to_f16x8(v.y, o[4], o[5], o[6], o[7]);
#pragma unroll
  for (int x = 0; x < 8; ++x) o[x] = hmul2_u32(o[x], s2);
  unsigned char* brow = tile + box * kBox + r * 128;
  *reinterpret_cast<uint4*>(brow + (((2 * c) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(brow + (((2 * c + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
}
// One fp4 row r of an NBOX-box tile converted in place: staged at `stage`, NBOX x 32 bytes per row, with the
// staged tile at the end of the slot. f16 rows of 32-row batches 0..2 lie below the staging area; batch 3's
// overlap staged rows of every batch, this one's included, so `all_read` returns once every thread of the warp
// has read its staged row. e8: the row's NBOX x 4 block exponents, one byte each.
template <int NBOX, class AllRead>
PALU_DEVINL bool f4_convert_row(unsigned char* tile, const unsigned char* stage, int r, const uint32_t (&e8)[2],
                                AllRead all_read) {
  const uint2* src = reinterpret_cast<const uint2*>(stage + r * (NBOX * 32));
  uint2 in[NBOX * 4];
#pragma unroll
  for (int i = 0; i < NBOX * 4; ++i) in[i] = src[i];
  if (!all_read()) return false;
#pragma unroll
  for (int i = 0; i < NBOX * 4; ++i)
    f4_store_chunk(tile, r, in[i], f8_scale_pair((int)(int8_t)(e8[i >> 2] >> (8 * (i & 3)))), i >> 2, i & 3);
  return true;
}
PALU_DEVINL void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
PALU_DEVINL void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
PALU_DEVINL void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// tcgen05.ld returns before its registers are written, and the compiler treats an inline-asm load's
// outputs as ready at once: a register-only use could be scheduled above a plain wait::ld. These waits
// take the loaded registers as read-write operands, so every use depends on the wait.
PALU_DEVINL void tmem_wait_ld_regs(uint32_t (&r)[4]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3])::"memory");
}
PALU_DEVINL void tmem_wait_ld_regs(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])::"memory");
}
PALU_DEVINL void tmem_wait_ld_regs(uint32_t (&a)[8], uint32_t (&b)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])::"memory");
}
// tcgen05.st may read its source registers after it issues: keep them unmodified until the wait, which
// takes them as read-write operands so the compiler cannot reuse them earlier.
PALU_DEVINL void tmem_wait_st_regs(uint32_t (&a)[4], uint32_t (&b)[4], uint32_t (&c)[4], uint32_t (&d)[4]) {
  asm volatile("tcgen05.wait::st.sync.aligned;\n"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]),
                 "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]), "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])::"memory");
}
PALU_DEVINL void tmem_wait_ld_regs(uint32_t (&a)[16], uint32_t (&b)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]),
                 "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                 "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15])::"memory");
}
PALU_DEVINL void tmem_wait_st_regs(uint32_t (&a)[8], uint32_t (&b)[8]) {
  asm volatile("tcgen05.wait::st.sync.aligned;\n"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])::"memory");
}
PALU_DEVINL __half2 u32_as_half2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
PALU_DEVINL uint32_t half2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

PALU_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
PALU_DEVINL void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
PALU_DEVINL void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
PALU_DEVINL float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;\n" : "=f"(r) : "f"(v));
  return r;
}
PALU_DEVINL void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
PALU_DEVINL void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
PALU_DEVINL void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

PALU_DEVINL uint32_t pack_half2(float x0, float x1) {
  __half2 h = __floats2half2_rn(x0, x1);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-bit element (row, k) of a K-major SWIZZLE_128B operand stored as 64-element
// K-blocks of `rows` rows each.
PALU_DEVINL uint32_t sw128_offset(int row, int k, int rows) {
  const int blk = k >> 6, kk = k & 63;
  return (uint32_t)(blk * rows * 128 + row * 128 + ((((kk >> 3) ^ (row & 7))) << 4) + (kk & 7) * 2);
}

// ---- the kernel --------------------------------------------------------------------------------------

PALU_DEVINL void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// Roles of the single-lane warps, two of each per group; warp w runs on SMSP w % 4:
//   group 0: 0 = K+table producer, 1 = QK+PV issuer, 2 = reconstruct issuer, 3 = V producer
//   group 1: 4 = QK+PV issuer, 5 = K+table producer, 6 = V producer, 7 = reconstruct issuer
enum : int { kRoleKT = 0, kRoleQK = 1, kRoleRC = 2, kRoleV = 3 };
PALU_DEVINL int role_of(int warp) {
  switch (warp) {
    case 0:
    case 5: return kRoleKT;
    case 1:
    case 4: return kRoleQK;
    case 2:
    case 7: return kRoleRC;
    default: return kRoleV;
  }
}

// PAGED: the caches are paged (TcParams.page_table set). A template parameter rather than a runtime branch,
// so that the contiguous-cache kernel carries none of the paged producers' code: with it the body fit the
// instruction cache worse, and dropping it measured 2-4 % faster on B200.
// REL: chunk-relative RoPE (TcParams.rel), likewise a template parameter: with both RoPE forms behind a runtime
// flag the chunk-relative kernel measured 151.9 us at the bench workload against 141.5 us for the specialised
// body (no_instruction stalls 1.47 per issued instruction against 0.83 before the flag).
template <int KBK, int KBV, bool PAGED, int NP, bool F8 = false, bool F4 = false, bool REL = false>
__global__ void __launch_bounds__(kThreads, 1)
    palu_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_tab, const TcParams p) {
  static_assert(!F8 || (NP == 2 && !PAGED), "fp8 latent caches: contiguous caches, latents at most 128 wide");
  static_assert(!F4 || F8, "fp4 caches run the low-bit producers of the F8 kernels");
  using Lay = Layout<KBK, KBV, NP, F8>;
  constexpr int NS_K = Lay::NS_K, NS_V = Lay::NS_V, T_SLOTS = Lay::T_SLOTS;
  constexpr int NS_T = NP * T_SLOTS;  // table chunk slots, [group][slot]
  // Chunk-relative RoPE: slots 0..3 hold table rows 0..127 (chunk c in slot c) for the whole kernel, loaded
  // once by group 0's K producer; nothing releases or refills them.
  constexpr bool rel = REL && rel_fits<Lay, NP>();
  // V^T as PV's A operand: one M = 64 block (V at most 64 wide), one M = 128 block (at most 128), or two M = 128
  // blocks (at most 256; a block's rows past the latent width are the TMA's zero fill).
  constexpr int NMB = KBV <= 2 ? 1 : 2;
  const int nmb = NMB == 1 || p.rv <= 128 ? 1 : 2;  // M-blocks that hold latent dims
  // PV result columns of buffer b, M-block mb (relative to the group's TMEM base)
  auto do_col = [](int b, int mb) -> uint32_t { return NP == 1 ? kColDoWide + mb * 32 + b * 16 : kColDo + b * 16; };
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);

  const int cta = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lat_head = kvh / (p.n_kv / p.n_groups);  // latent head of this KV head (its group)

  // ---- barriers and scalars (misc area) ----
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::OFF_MISC);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  // [g][x] pairs are double-buffered by the group-local tile index parity x.
  // V-full barriers are per (slot, use parity), so a parity wait is never more than one phase behind.
  // Drain barriers: [g][QK+PV issuer, reconstruct issuer]. One pipeline: REC[x] marks D_k[x] reconstructed
  // (tiles j with j % 2 == x) and DKF[x] marks it read by RoPE. fp8 caches: ST[slot] marks a slot's e4m3
  // tile landed in its staging half (K slots, then V slots); KF / VF then mark it converted to f16.
  constexpr int B_KF = 0, B_KE = B_KF + NS_K, B_VF = B_KE + NS_K, B_VE = B_VF + 2 * NS_V, B_TF = B_VE + NS_V,
                B_TE = B_TF + NS_T, B_UF = B_TE + NS_T, B_REC = B_UF + 1, B_AF = B_REC + 4, B_AE = B_AF + 4,
                B_SF = B_AE + 2, B_SR = B_SF + 4, B_PF = B_SR + 4, B_OF = B_PF + 4, B_OR = B_OF + 4,
                B_MX = B_OR + 4, B_QF = B_MX + 4, B_DRAIN = B_QF + 4, B_DKF = B_DRAIN + 4, B_STK = B_DKF + 2, B_STV = B_STK + NS_K,
                B_COUNT = B_STV + NS_V;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  int* s_range = reinterpret_cast<int*>(s_tmem + 4);      // n, b0, t0, cnt0 of this CTA's range
  float* s_max = reinterpret_cast<float*>(s_tmem + 8);    // [2 groups][2 bufs][4 warps][4 heads]
  static_assert((B_COUNT + 8) * 8 + 64 * 4 <= Lay::MISC_BYTES, "misc area");

  // Bounded waits. The RoPE and softmax warps use wait_all: every lane of the warp gets the same answer, so
  // that when the CTA gives up no warp is left divergent before its next .sync.aligned instruction. A phase
  // that has already completed is seen by the whole converged warp in one try_wait, so the vote is taken on
  // the spinning path only.
  auto wait = [&](uint32_t b, uint32_t ph) -> bool { return mbar_wait(b, ph, s_abort, p.status, p.wait_ns); };
  auto wait_all = [&](uint32_t b, uint32_t ph) -> bool {
    if (__all_sync(0xffffffffu, mbar_try(b, ph))) return true;
    return __all_sync(0xffffffffu, mbar_wait_slow(b, ph, s_abort, p.status, p.wait_ns)) != 0;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS_K; ++s) {
      mbar_init(bar(B_KF + s), 1);
      mbar_init(bar(B_KE + s), 1);
    }
    for (int s = 0; s < NS_V; ++s) {
      mbar_init(bar(B_VF + 2 * s), 1);
      mbar_init(bar(B_VF + 2 * s + 1), 1);
      mbar_init(bar(B_VE + s), 1);
    }
    for (int s = 0; s < NS_T; ++s) {
      mbar_init(bar(B_TF + s), 1);
      mbar_init(bar(B_TE + s), 4);  // the group's 4 RoPE warps
    }
    mbar_init(bar(B_UF), 8);  // the 8 RoPE warps stage U_k
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(B_AE + g), 1);
      for (int h = 0; h < 2; ++h) {
        mbar_init(bar(B_REC + 2 * g + h), 1);
        mbar_init(bar(B_AF + 2 * g + h), 4);
      }
      for (int x = 0; x < 2; ++x) {
        mbar_init(bar(B_SF + 2 * g + x), 1);
        mbar_init(bar(B_SR + 2 * g + x), 4);
        mbar_init(bar(B_PF + 2 * g + x), 4);
        mbar_init(bar(B_OF + 2 * g + x), 1);
        mbar_init(bar(B_OR + 2 * g + x), 4);
        mbar_init(bar(B_MX + 2 * g + x), 4);
        mbar_init(bar(B_QF + 2 * g + x), 4);  // the group's 4 softmax warps stage Q
      }
    }
    for (int x = 0; x < 4; ++x) mbar_init(bar(B_DRAIN + x), 1);
    for (int x = 0; x < 2; ++x) mbar_init(bar(B_DKF + x), 8);  // one pipeline: the 8 RoPE warps read D_k[x]
    for (int s = 0; s < NS_K + NS_V; ++s) mbar_init(bar(B_STK + s), 1);  // fp8: a staged tile has landed
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {  // TMEM: 512 columns; the base address lands in shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (warp == 2) {
    // This CTA's range of the KV head's tiles, and where it starts (row b0, tile t0 of that row).
    long long T = 0;
    for (int bb = lane; bb < p.batch; bb += 32) T += row_tiles(p, bb);
#pragma unroll
    for (int o = 16; o; o >>= 1) T += __shfl_xor_sync(0xffffffffu, T, o);
    if (lane == 0) {
      const long long k0 = (long long)cta * T / p.ctas, k1 = (long long)(cta + 1) * T / p.ctas;
      const int n = (int)(k1 - k0);
      int b0 = 0, t0 = 0, cnt0 = 0;
      if (n > 0) {
        long long acc = 0;
        for (b0 = 0; b0 < p.batch; ++b0) {
          const int nb = row_tiles(p, b0);
          if (acc + nb > k0) break;
          acc += nb;
        }
        if (b0 < p.batch) {
          t0 = (int)(k0 - acc);
          cnt0 = min(row_tiles(p, b0) - t0, n);
        }
      }
      s_range[0] = cnt0 > 0 ? n : 0;
      s_range[1] = b0;
      s_range[2] = t0;
      s_range[3] = cnt0;
    }
  }
  if (warp >= kSoftWarp0) {
    // Q buffers (4 x 4 KB) and P buffers (4 x 4 KB): rows past the query heads stay zero throughout.
    for (int e = (warp - kSoftWarp0) * 32 + lane; e < (2 * NP * Lay::Q_BYTES + 2 * NP * Lay::P_BYTES) / 16; e += 256)
      reinterpret_cast<uint4*>(smem + Lay::OFF_Q)[e] = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (p.pdl_early) asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const uint32_t tmem = *s_tmem;
  const int n = s_range[0];                                  // tiles of this CTA
  const RowSeg seg0{s_range[1], s_range[2], s_range[3], 0};  // its first segment

  if (warp < kRoleWarps) {
    // ============================== role warps ==============================
    const int g = warp < 4 ? 0 : 1, role = role_of(warp);
    const int n_g = g < NP ? (n - g + NP - 1) / NP : 0;  // this group's tiles: CTA-local t = g + NP j, j < n_g
    if (F8 && (role == kRoleKT || role == kRoleV)) {
      if (n_g > 0) {
        // ---- fp8 producers (whole warp). Lane 0 issues the TMA of a tile's e4m3 codes into the upper half of
        // its ring slot, up to the ring's depth ahead; the warp converts each landed tile in place into the
        // f16 tile the MMAs read (SWIZZLE_128B K-major boxes of 64 dims): K codes as they are (their row
        // scales are applied to the scores), V codes times their row's 2^k. The K warp then issues the
        // tile's 4 table chunks (after the conversion: RoPE of the previous tile, which frees their slots,
        // waits for it).
        const bool kt = role == kRoleKT;
        const int NS = kt ? NS_K : NS_V, ring = NS / NP;
        const uint32_t slot_bytes = kt ? Lay::K_BYTES : Lay::V_BYTES, off0 = kt ? Lay::OFF_K : Lay::OFF_V;
        const int row8 = (kt ? KBK : KBV) * (F4 ? 32 : 64);        // staged bytes per row
        const uint32_t stage_off = slot_bytes - (uint32_t)row8 * kTile;  // the staged tile ends the slot
        const CUtensorMap* tm = kt ? &tm_k : &tm_v;
        const int b_st = kt ? B_STK : B_STV;
        if (lane == 0) {
          tma_prefetch_map(tm);
          if (kt) tma_prefetch_map(&tm_tab);
          if (kt && rel && g == 0) {  // chunk-relative RoPE: table rows 0..127 into slots 0..3, once
            for (int c = 0; c < 4; ++c) {
              mbar_expect_tx(bar(B_TF + c), Lay::TCH_BYTES);
              tma_load_2d(sbase + Lay::OFF_TAB + c * Lay::TCH_BYTES, &tm_tab, bar(B_TF + c), c * 16, 0);
            }
          }
        }
        GroupTiles<NP> iss, cv;
        iss.init(p, seg0, g, n);
        cv.init(p, seg0, g, n);
        int ji = 0, jc = 0, issued_t = 0;
        // The TMA of tile ji into its slot, once the slot's previous tile is consumed. A tile is issued `ring`
        // tiles ahead, after the conversion of the tile before it, so a conversion starts as soon as its
        // slot's previous tile is consumed, with its codes already landed.
        auto issue_next = [&]() -> bool {
          const int t = g + NP * ji, sb = t % NS, use = t / NS;
          if (use >= 1 && !wait_all(bar((kt ? B_KE : B_VE) + sb), (use - 1) & 1)) return false;
          if (lane == 0) {
            mbar_expect_tx(bar(b_st + sb), row8 * kTile);
            tma_load_3d(sbase + off0 + sb * slot_bytes + stage_off, tm, bar(b_st + sb), 0, iss.tile() * kTile,
                        iss.s.b * p.n_groups + lat_head);
          }
          ++ji;
          iss.next(p);
          return true;
        };
        bool ok = true;
        while (ok && ji < n_g && ji < ring && iss.valid()) ok = issue_next();
        for (int j = 0; ok && j < n_g && cv.valid(); ++j, cv.next(p)) {
          const int t = g + NP * j, sb = t % NS, use = t / NS, row0 = cv.tile() * kTile;
          uint32_t ex4 = 0;  // V: the exponents of rows lane, 32 + lane, 64 + lane, 96 + lane, one byte each
          if (!kt && !F4) {
            const int8_t* erow = p.v_exp + ((size_t)cv.s.b * p.n_groups + lat_head) * p.max_seq;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int pos = row0 + 32 * q + lane;
              ex4 |= (uint32_t)(uint8_t)(pos < p.max_seq ? __ldg(erow + pos) : 0) << (8 * q);
            }
          }
          if (!wait_all(bar(b_st + sb), use & 1)) {
            ok = false;
            break;
          }
          unsigned char* slot = smem + off0 + sb * slot_bytes;
          const unsigned char* stage = slot + stage_off;
          // rows 32 q .. 32 q + 31, one per lane, batch by batch: with 64-code rows the f16 rows of a batch
          // overlap staged rows of this batch and earlier ones only
          auto warp_read = [] {
            __syncwarp();
            return true;
          };
#pragma unroll 1
          for (int q = 0; q < 4; ++q) {
            const int r = 32 * q + lane;
            if constexpr (F4) {
              // fp4: the row's block exponents (r / 16 of them), then the row
              const int nb = kt ? KBK : KBV, pos = row0 + r;
              const int8_t* ep = (kt ? p.k_exp : p.v_exp) +
                                 (((size_t)cv.s.b * p.n_groups + lat_head) * p.max_seq + pos) * (nb * 4);
              uint32_t e8[2] = {0u, 0u};
              if (pos < p.max_seq) {
                e8[0] = __ldg(reinterpret_cast<const uint32_t*>(ep));
                if (nb == 2) e8[1] = __ldg(reinterpret_cast<const uint32_t*>(ep) + 1);
              }
              if (kt) f4_convert_row<KBK>(slot, stage, r, e8, warp_read);
              else f4_convert_row<KBV>(slot, stage, r, e8, warp_read);
            } else if (kt) {
              f8_convert_row<KBK, false>(slot, stage, r, 0, warp_read);
            } else {
              f8_convert_row<KBV, true>(slot, stage, r, (int)(int8_t)(ex4 >> (8 * q)), warp_read);
            }
          }
          fence_proxy_async();  // generic writes -> visible to the tensor core's reads
          __syncwarp();
          if (lane == 0) mbar_arrive(kt ? bar(B_KF + sb) : bar(B_VF + 2 * sb + (use & 1)));
          jc = j + 1;
          if (kt && !rel) {
            for (int c = 0; c < 4; ++c) {
              const int nc = 4 * j + c, ts = g * T_SLOTS + nc % T_SLOTS, tuse = nc / T_SLOTS;
              if (tuse >= 1 && !wait_all(bar(B_TE + ts), (tuse - 1) & 1)) {
                ok = false;
                break;
              }
              if (lane == 0) {
                mbar_expect_tx(bar(B_TF + ts), Lay::TCH_BYTES);
                tma_load_2d(sbase + Lay::OFF_TAB + ts * Lay::TCH_BYTES, &tm_tab, bar(B_TF + ts), c * 16, row0);
              }
              issued_t = nc + 1;
            }
          }
          if (ok && ji < n_g && iss.valid()) ok = issue_next();
        }
        if (*s_abort && lane == 0) {  // let every copy already issued land before the CTA can exit
          for (int jj = jc; jj < ji; ++jj) {
            const int t = g + NP * jj;
            mbar_drain(bar(b_st + t % NS), (t / NS) & 1);
          }
          for (int nc = max(0, issued_t - T_SLOTS); nc < issued_t; ++nc)
            mbar_drain(bar(B_TF + g * T_SLOTS + nc % T_SLOTS), (nc / T_SLOTS) & 1);
          if (kt && rel && g == 0)
            for (int c = 0; c < 4; ++c) mbar_drain(bar(B_TF + c), 0);
        }
      }
    } else if (lane == 0 && n_g > 0) {
      if (role == kRoleKT || role == kRoleV) {
        // ---- TMA producers: K tile then its 4 table chunks (KT), or the V tile (V), per group tile.
        const bool kt = role == kRoleKT;
        const bool starve = !kt && g == 0 && p.starve_v;  // test of the timeout path only
        tma_prefetch_map(kt ? &tm_k : &tm_v);
        if (kt) tma_prefetch_map(&tm_tab);
        int issued_kv = 0, issued_t = 0;
        // One pipeline: K streams through a ring of single boxes (kbn: boxes issued so far).
        const bool box_ring = NP == 1 && kt;
        const int nbk = (p.rk + 63) >> 6;
        int kbn = 0;
        GroupTiles<NP> it;
        it.init(p, seg0, g, n);
        if (kt && rel && g == 0) {  // chunk-relative RoPE: table rows 0..127 into slots 0..3, once
          for (int c = 0; c < 4; ++c) {
            mbar_expect_tx(bar(B_TF + c), Lay::TCH_BYTES);
            tma_load_2d(sbase + Lay::OFF_TAB + c * Lay::TCH_BYTES, &tm_tab, bar(B_TF + c), c * 16, 0);
          }
        }
        for (int j = 0; j < n_g && it.valid(); ++j, it.next(p)) {
          const int t = g + NP * j, row = it.tile() * kTile, item_lat = it.s.b * p.n_groups + lat_head;
          const int sb = kt ? t % NS_K : t % NS_V, use = kt ? t / NS_K : t / NS_V;
          const uint32_t full = kt ? bar(B_KF + sb) : bar(B_VF + 2 * sb + (use & 1));
          const uint32_t empty = bar((kt ? B_KE : B_VE) + sb);
          // Paged caches: the tile's blocks, looked up before the wait so the loads overlap it. Blocks
          // past the row's last position repeat its last block (those rows are masked), so no table
          // entry beyond the row's length is read; an entry outside [0, n_blocks) becomes a coordinate
          // past the tensor map, which the copy fills with zeros.
          int blk[kTile / 16];
          if constexpr (PAGED) {
            const int32_t* pt = p.page_table + (size_t)it.s.b * p.table_ld;
            const int last = (it.len - 1) >> p.blk_shift, lb0 = row >> p.blk_shift;
#pragma unroll
            for (int i = 0; i < kTile / 16; ++i)
              if (i < (kTile >> p.blk_shift)) {
                const int e = __ldg(pt + min(lb0 + i, last));
                blk[i] = (unsigned)e < (unsigned)p.n_blocks ? e * p.n_groups + lat_head : p.n_blocks * p.n_groups;
              }
          }
          if (box_ring) {
            bool ok = true;
            for (int c = 0; c < nbk; ++c, ++kbn) {
              const int s = kbn % NS_K, u = kbn / NS_K;
              if (u >= 1 && !wait(bar(B_KE + s), (u - 1) & 1)) {
                ok = false;
                break;
              }
              const uint32_t kf = bar(B_KF + s), dst = sbase + Lay::OFF_K + s * Lay::K_BYTES;
              mbar_expect_tx(kf, kBox);
              if constexpr (!PAGED) {
                tma_load_3d(dst, &tm_k, kf, c * 64, row, item_lat);
              } else {
                const int nsub = kTile >> p.blk_shift, sub_bytes = 128 << p.blk_shift;
#pragma unroll
                for (int i = 0; i < kTile / 16; ++i)
                  if (i < nsub) tma_load_3d(dst + i * sub_bytes, &tm_k, kf, c * 64, 0, blk[i]);
              }
              issued_kv = kbn + 1;
            }
            if (!ok) break;
          } else if (use >= 1 && !wait(empty, (use - 1) & 1)) {
            break;
          } else if (!starve) {
            const CUtensorMap* tm = kt ? &tm_k : &tm_v;
            const uint32_t dst = sbase + (kt ? Lay::OFF_K + sb * Lay::K_BYTES : Lay::OFF_V + sb * Lay::V_BYTES);
            // boxes that hold latent dims (the wide layout reserves four; a tile of a narrower latent skips
            // the boxes wholly past it, which its MMAs never read)
            const int nbox = kt ? min(KBK, (p.rk + 63) >> 6) : min(KBV, (p.rv + 63) >> 6);
            mbar_expect_tx(full, nbox * kBox);
            if constexpr (!PAGED) {
              for (int c = 0; c < nbox; ++c) tma_load_3d(dst + c * kBox, tm, full, c * 64, row, item_lat);
            } else {
              // one box of bs rows per block; bs * 128 B is a whole number of 1 KB swizzle atoms, so the
              // rows land exactly where one 128-row box would put them
              const int nsub = kTile >> p.blk_shift, sub_bytes = 128 << p.blk_shift;
#pragma unroll
              for (int i = 0; i < kTile / 16; ++i)
                if (i < nsub)
                  for (int c = 0; c < nbox; ++c)
                    tma_load_3d(dst + c * kBox + i * sub_bytes, tm, full, c * 64, 0, blk[i]);
            }
            issued_kv = j + 1;
          }
          if (kt && !rel) {
            bool ok = true;
            for (int c = 0; c < 4; ++c) {
              const int nc = 4 * j + c, ts = g * T_SLOTS + nc % T_SLOTS, tuse = nc / T_SLOTS;
              if (tuse >= 1 && !wait(bar(B_TE + ts), (tuse - 1) & 1)) {
                ok = false;
                break;
              }
              mbar_expect_tx(bar(B_TF + ts), Lay::TCH_BYTES);
              tma_load_2d(sbase + Lay::OFF_TAB + ts * Lay::TCH_BYTES, &tm_tab, bar(B_TF + ts), c * 16, row);
              issued_t = nc + 1;
            }
            if (!ok) break;
          }
        }
        if (*s_abort) {  // let every copy already issued land before the CTA can exit
          const int ring = kt ? NS_K / NP : NS_V / NP;
          if (box_ring) {
            for (int u = max(0, issued_kv - NS_K); u < issued_kv; ++u)
              mbar_drain(bar(B_KF + u % NS_K), (u / NS_K) & 1);
          } else {
            for (int j = max(0, issued_kv - ring); j < issued_kv; ++j) {
              const int t = g + NP * j;
              if (kt) mbar_drain(bar(B_KF + t % NS_K), (t / NS_K) & 1);
              else mbar_drain(bar(B_VF + 2 * (t % NS_V) + ((t / NS_V) & 1)), (t / NS_V >> 1) & 1);
            }
          }
          for (int nc = max(0, issued_t - T_SLOTS); nc < issued_t; ++nc)
            mbar_drain(bar(B_TF + g * T_SLOTS + nc % T_SLOTS), (nc / T_SLOTS) & 1);
          if (kt && rel && g == 0)
            for (int c = 0; c < 4; ++c) mbar_drain(bar(B_TF + c), 0);
        }
      } else {
        const uint32_t tg = tmem + g * kGrpCols;
        const int drain = B_DRAIN + 2 * g + (role == kRoleQK ? 0 : 1);
        if (role == kRoleQK) {
          // ---- QK(j): D_s[j & 1] = K_rot (TMEM, fp16) x Q^T in two halves, half h once RoPE(j) wrote A half h
          // (and, first, once softmax(j - 2) read D_s[j & 1]); then PV(j - 1) once softmax(j - 1) wrote P.
          // (PV first measured slower on B200: waiting for P(j - 1) then delays QK(j) and the RoPE chain.)
          // The commit after QK(j) also covers PV(j - 2), issued before it by this thread: once softmax(j) sees
          // D_s[j & 1], P[j & 1] is free to rewrite.
          // Q: the group's buffer of the tile's row, staged by the softmax warps per group segment.
          constexpr uint32_t ID_QK = idesc_f16(16, 0, false, false);
          // bf16 V^T (MN-major) x bf16 P. A V latent at most 64 wide is one M = 64 block: with M = 128 the
          // MMA read every V row twice (measured 1.6 % faster at the bench workload with M = 64).
          constexpr uint32_t ID_PV = idesc_f16(16, F8 ? 0 : 1, true, false, KBV == 1 ? 64 : 128);  // f16 | bf16
          static_assert(KBV != 1 || NMB == 1, "an M = 64 PV block holds the whole V latent");
          const uint32_t v_lbo = p.rv > 64 ? kBox : 0;  // V: stride between the 64-dim halves of an M = 128 block
          GroupTiles<NP> it, pit;  // QK(j) and PV(j - 1) tiles
          it.init(p, seg0, g, n);
          pit.init(p, seg0, g, n);
          for (int j = 0; j <= n_g; ++j) {
            if (j < n_g) {
              // Q buffer: per group segment (the row's q), or per tile with chunk-relative RoPE (the q of the
              // tile's row rotated by the tile's base position)
              const int qb = rel ? (j & 1) : (it.sigma & 1);
              if ((rel || it.first()) && !wait(bar(B_QF + 2 * g + qb), ((rel ? j : it.sigma) >> 1) & 1)) break;
              if (j >= 2 && !wait(bar(B_SR + 2 * g + (j & 1)), ((j >> 1) - 1) & 1)) break;
              const uint32_t sQ = sbase + Lay::OFF_Q + (2 * g + qb) * Lay::Q_BYTES;
              it.next(p);
              bool ok = true;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (!wait(bar(B_AF + 2 * g + h), j & 1)) {
                  ok = false;
                  break;
                }
                fence_after();
                // A half h: the 16-element K steps kk = 2h, 2h + 1 (even dims) and 4 + 2h, 5 + 2h (odd dims).
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                  const int kk = (x >> 1) * 4 + 2 * h + (x & 1);
                  mma_ts(tg + kColDs + (j & 1) * 16, tg + kColA + kk * 8,
                         sdesc(sQ + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), ID_QK, (h | x) != 0);
                }
                mma_commit(bar(h == 0 ? B_AE + g : B_SF + 2 * g + (j & 1)));
              }
              if (!ok) break;
            }
            if (j >= 1) {  // PV(j - 1)
              const int jp = j - 1, tp = g + NP * jp, sv = tp % NS_V;
              if (!wait(bar(B_PF + 2 * g + (jp & 1)), (jp >> 1) & 1)) break;
              if (jp >= 2 && !wait(bar(B_OR + 2 * g + (jp & 1)), ((jp >> 1) - 1) & 1)) break;
              if (!wait(bar(B_VF + 2 * sv + ((tp / NS_V) & 1)), (tp / NS_V >> 1) & 1)) break;
              // A row's last tile may be partial. V rows past cur_pos may hold anything (NaN included) and
              // 0 * NaN is not 0, so for such a tile the MMA takes only the 16-token K-steps that hold valid
              // rows, and the invalid rows inside the last of them are zeroed here first: by this thread, whose
              // proxy fence orders its own writes before its MMAs. (Zeroing them from the softmax warps, with a
              // proxy fence and an mbarrier hand-off, let the zeros land in the slot's next tile on B200.)
              const int nv = pit.len - pit.tile() * kTile;  // valid rows (> 0)
              pit.next(p);
              const uint32_t sV = sbase + Lay::OFF_V + sv * Lay::V_BYTES;
              const uint32_t sP = sbase + Lay::OFF_P + (2 * g + (jp & 1)) * Lay::P_BYTES;
              if (nv >= kTile) {
                fence_after();
#pragma unroll
                for (int mb = 0; mb < NMB; ++mb)
                  if (mb < nmb)
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                      mma_ss(tg + do_col(jp & 1, mb), sdesc(sV + mb * 2 * kBox + kk * 2048, v_lbo, 1024),
                           sdesc(sP + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), ID_PV, kk > 0);
              } else {
                const int ksteps = (nv + 15) >> 4;
                for (int rr = nv; rr < ksteps * 16; ++rr)
                  for (int vb = 0; vb < KBV; ++vb)
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                      reinterpret_cast<uint4*>(smem + Lay::OFF_V + sv * Lay::V_BYTES + vb * kBox + rr * 128)[c] =
                          make_uint4(0, 0, 0, 0);
                fence_proxy_async();
                fence_after();
                for (int mb = 0; mb < nmb; ++mb)
                  for (int kk = 0; kk < ksteps; ++kk)
                    mma_ss(tg + do_col(jp & 1, mb), sdesc(sV + mb * 2 * kBox + kk * 2048, v_lbo, 1024),
                           sdesc(sP + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), ID_PV, kk > 0);
              }
              mma_commit(bar(B_OF + 2 * g + (jp & 1)));
              mma_commit(bar(B_VE + sv));
            }
          }
        } else {
          // ---- reconstruct(j + 1) in two halves: D_k columns 64 h .. 64 h + 63 (frequencies 32 h .. + 31) once
          // RoPE(j) has read them, so the reconstruction of one half overlaps the rotation of the other.
          // bf16 lat x bf16 U (MN-major), N = 64; f16 x f16 for fp8 caches
          constexpr uint32_t ID_REC = idesc_f16(64, F8 ? 0 : 1, false, true);
          const uint32_t sU = sbase + Lay::OFF_U;
          const uint32_t u_lbo = p.rk * 128;  // U: stride between the two 64-column N-blocks
          auto recon = [&](int j, int h) -> bool {
            const int t = g + NP * j, s = t % NS_K;
            if (h == 0 && !wait(bar(B_KF + s), (t / NS_K) & 1)) return false;
            fence_after();
            const uint32_t sK = sbase + Lay::OFF_K + s * Lay::K_BYTES;
            for (int kk = 0; kk < p.rk / 16; ++kk)
              mma_ss(tg + kColDk + 64 * h, sdesc(sK + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024),
                     sdesc(sU + h * u_lbo + kk * 2048, u_lbo, 1024), ID_REC, kk > 0);
            if (h == 1) mma_commit(bar(B_KE + s));
            mma_commit(bar(B_REC + 2 * g + h));
            return true;
          };
          if constexpr (NP == 2) {
            bool ok = wait(bar(B_UF), 0) && recon(0, 0) && recon(0, 1);
            for (int j = 0; ok && j + 1 < n_g; ++j)
              for (int h = 0; ok && h < 2; ++h) ok = wait(bar(B_AF + 2 * g + h), j & 1) && recon(j + 1, h);
          } else {
            // One pipeline: D_k is double-buffered by tile parity (columns kColDk / kColDk2), so reconstruct(j)
            // runs a whole tile ahead of RoPE(j - 1): it waits only for RoPE(j - 2) to have read its buffer.
            // It is one N = 128 pass streamed box by box through the K ring (4 K-steps per 64-wide box), each
            // box released as soon as its MMAs complete.
            constexpr uint32_t ID_REC2 = idesc_f16(128, 1, false, true);  // N = 128: both frequency halves
            const int nbk = (p.rk + 63) >> 6, nks = p.rk >> 4;
            int kbn = 0;
            bool ok = wait(bar(B_UF), 0);
            for (int j = 0; ok && j < n_g; ++j) {
              if (j >= 2 && !(ok = wait(bar(B_DKF + (j & 1)), ((j >> 1) - 1) & 1))) break;
              fence_after();
              const uint32_t dk = tg + ((j & 1) ? kColDk2 : kColDk);
              for (int c = 0; c < nbk; ++c, ++kbn) {
                const int s = kbn % NS_K;
                if (!(ok = wait(bar(B_KF + s), (kbn / NS_K) & 1))) break;
                fence_after();
                const uint32_t sK = sbase + Lay::OFF_K + s * Lay::K_BYTES;
                for (int kk = 4 * c; kk < min(4 * c + 4, nks); ++kk)
                  mma_ss(dk, sdesc(sK + (kk & 3) * 32, 16, 1024), sdesc(sU + kk * 2048, u_lbo, 1024), ID_REC2,
                         kk > 0);
                mma_commit(bar(B_KE + s));
              }
              if (ok) mma_commit(bar(B_REC + (j & 1)));
            }
          }
        }
        // Drain: every MMA this thread issued has completed once this barrier flips.
        mma_commit(bar(drain));
        mbar_drain(bar(drain), 0);
      }
    }
    __syncwarp();
  } else if (warp < kSoftWarp0) {
    // ============================== RoPE warps ==============================
    // Two pipelines: warps 4 g .. 4 g + 3 rotate pipeline g's tiles, all four chunks each. One pipeline: all
    // 8 warps rotate every tile, warps 4 hh .. 4 hh + 3 its frequency half hh (chunks 2 hh, 2 hh + 1), so
    // the two halves of a tile run side by side.
    const int g = NP == 2 ? (warp - kRopeWarp0) >> 2 : 0, quarter = warp & 3, row = quarter * 32 + lane;
    const int ch0 = NP == 2 ? 0 : ((warp - kRopeWarp0) >> 2) * 2, nch = NP == 2 ? 4 : 2;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + g * kGrpCols;
    {
      // U_k -> shared memory as the MN-major SWIZZLE_128B B operand of the reconstruction, one 64-column
      // N-block per half of the frequencies: N-block h holds the even dims of frequencies 32 h .. 32 h + 31
      // (columns 0..31), then their odd dims (columns 32..63).
      // Item: (latent row r, source dims 16 a .. 16 a + 15 = frequencies 8 a .. 8 a + 7) -> 16-byte chunks
      // a % 4 (even dims) and 4 + a % 4 (odd dims) of row r of N-block a / 4.
      for (int e = (warp - kRopeWarp0) * 32 + lane; e < p.rk * 8; e += 256) {
        const int r = e >> 3, a = e & 7;
        const uint4* src = reinterpret_cast<const uint4*>(p.u_k + ((size_t)kvh * p.rk + r) * p.ld_u + 16 * a);
        const uint4 x0 = src[0], x1 = src[1];
        uint4 ev = make_uint4(__byte_perm(x0.x, x0.y, 0x5410), __byte_perm(x0.z, x0.w, 0x5410),
                              __byte_perm(x1.x, x1.y, 0x5410), __byte_perm(x1.z, x1.w, 0x5410));
        uint4 od = make_uint4(__byte_perm(x0.x, x0.y, 0x7632), __byte_perm(x0.z, x0.w, 0x7632),
                              __byte_perm(x1.x, x1.y, 0x7632), __byte_perm(x1.z, x1.w, 0x7632));
        if constexpr (F8) {  // fp8 caches: the reconstruction runs on f16 operands (U rounded to f16)
          auto h2 = [](uint32_t w) {
            const float2 f = unpack_bf16(w);
            return pack_half2(f.x, f.y);
          };
          ev = make_uint4(h2(ev.x), h2(ev.y), h2(ev.z), h2(ev.w));
          od = make_uint4(h2(od.x), h2(od.y), h2(od.z), h2(od.w));
        }
        unsigned char* urow = smem + Lay::OFF_U + (a >> 2) * p.rk * 128 + r * 128;
        *reinterpret_cast<uint4*>(urow + (((a & 3) ^ (r & 7)) << 4)) = ev;
        *reinterpret_cast<uint4*>(urow + (((4 + (a & 3)) ^ (r & 7)) << 4)) = od;
      }
      fence_proxy_async();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_UF));
    }
    const int n_g = NP == 2 ? (n - g + 1) / 2 : n;
    // chunk-relative RoPE: the fixed table rows 0..127 (slots 0..3), waited for once
    bool tab_ok = true;
    if (rel && n_g > 0)
      for (int c = 0; c < 4 && tab_ok; ++c) tab_ok = wait_all(bar(B_TF + c), 0);
    for (int i = 0; tab_ok && i < n_g; ++i) {
      // ---- RoPE(i), by halves: D_k columns 64 h .. 64 h + 31 hold the even dims of frequencies 32 h + c,
      // columns 64 h + 32 + c their odd dims; chunk ch = 2 h + sub rotates frequencies 16 ch .. 16 ch + 15.
      // K_rot -> fp16 A columns. Finishing half h releases D_k half h (reconstruction of tile i + 1) and
      // hands A half h to QK(i).
      // One pipeline: D_k[i % 2] holds the whole tile once REC[i % 2] flips; reading it is signalled on DKF.
      bool ok = true;
      const uint32_t dk = trow + (NP == 1 && (i & 1) ? kColDk2 : kColDk);
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int ch = ch0 + c, h = ch >> 1, sub = ch & 1;
        if (sub == 0) {
          if (!(NP == 2 ? wait_all(bar(B_REC + 2 * g + h), i & 1) : wait_all(bar(B_REC + (i & 1)), (i >> 1) & 1))) {
            ok = false;
            break;
          }
          fence_after();
        }
        const int n = i * 4 + ch, sb = rel ? ch : g * T_SLOTS + n % T_SLOTS;
        // The chunk's D_k columns load while this warp waits for and reads its table chunk.
        uint32_t ke[16], ko[16];
        tmem_ld16(dk + 64 * h + 16 * sub, ke);
        tmem_ld16(dk + 64 * h + 32 + 16 * sub, ko);
        if (!rel && !wait_all(bar(B_TF + sb), (n / T_SLOTS) & 1)) {
          tmem_wait_ld_regs(ke, ko);
          ok = false;
          break;
        }
        // SWIZZLE_64B rows of 64 B: 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3). Words 0..7:
        // cos of frequency pairs (f, f+1), words 8..15: their sines (fp16, low half first).
        const unsigned char* tb = smem + Lay::OFF_TAB + sb * Lay::TCH_BYTES + row * 64;
        uint32_t cs[16];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const uint4 w = *reinterpret_cast<const uint4*>(tb + ((c4 ^ ((row >> 1) & 3)) << 4));
          cs[4 * c4 + 0] = w.x;
          cs[4 * c4 + 1] = w.y;
          cs[4 * c4 + 2] = w.z;
          cs[4 * c4 + 3] = w.w;
        }
        tmem_wait_ld_regs(ke, ko);
        if (NP == 1 && sub == 1) {  // this warp's last read of D_k[i % 2]
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_DKF + (i & 1)));
        }
        uint32_t ae[8], ao[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          // half2 math on two adjacent frequencies: K to fp16 first (the A operand is fp16 anyway), then
          // rot(2f) = k(2f) cos - k(2f+1) sin ; rot(2f+1) = k(2f+1) cos + k(2f) sin
          const __half2 c = u32_as_half2(cs[x]), sn = u32_as_half2(cs[8 + x]);
          const __half2 e = __floats2half2_rn(__uint_as_float(ke[2 * x]), __uint_as_float(ke[2 * x + 1]));
          const __half2 o = __floats2half2_rn(__uint_as_float(ko[2 * x]), __uint_as_float(ko[2 * x + 1]));
          ae[x] = half2_as_u32(__hfma2(__hneg2(o), sn, __hmul2(e, c)));
          ao[x] = half2_as_u32(__hfma2(e, sn, __hmul2(o, c)));
        }
        // Every lane has used its table values: the slot may refill. (An arrive issued while this warp's
        // tcgen05.ld is in flight waits for that load, measured at ~260 cycles on B200, hence after the math.)
        // The chunk was read through the generic proxy and the refill writes it through the async proxy
        // (TMA), so the reads are ordered before the release by fence.proxy.async. Without the fence the
        // refill overwrote rows whose reads were still in flight (the first rows of the chunk, which the TMA
        // writes first): on B200 a few percent of calls then differed in the last bits of one batch row.
        if (!rel) {
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_TE + sb));
        }
        if (sub == 0 && i >= 1) {
          // A half h still feeds half h of QK(i - 1) until those MMAs complete: their commit is AE (h = 0)
          // or the scores barrier (h = 1).
          const int jq = i - 1;
          const bool freed = h == 0 ? wait_all(bar(B_AE + g), jq & 1)
                                    : wait_all(bar(B_SF + 2 * g + (jq & 1)), (jq >> 1) & 1);
          if (!freed) {
            ok = false;
            break;
          }
          fence_after();
        }
        // A column 8 ch + x: K_rot dims (2f, 2f + 2) of f = 16 ch + 2x (reordered elements f, f + 1);
        // column 32 + the same: the odd dims of those frequencies.
        tmem_st8(trow + kColA + 8 * ch, ae);
        tmem_st8(trow + kColA + 32 + 8 * ch, ao);
        tmem_wait_st_regs(ae, ao);
        if (sub == 1) {
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_AF + 2 * g + h));
        }
      }
      if (!ok) break;
    }
  } else {
    // ============================== softmax warps ==============================
    const int g = (warp - kSoftWarp0) >> 2, quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + g * kGrpCols;
    // Q^T of a batch row into the group's Q buffer `buf`: fp16, K-major SWIZZLE_128B, 16 rows (this KV
    // head's query heads; the rest stay zero) x 128 dims in [even | odd] order: K-block 0 = even dims,
    // K-block 1 = odd dims (64 fp16 per 128-B row). Item (row, 16-byte chunk of 8 reordered dims); bf16
    // q is exact in fp16. The QK issuer waits for the buffer's barrier.
    // Chunk-relative RoPE (`rel`; `tile` is then the tile's index in its row, else -1): the q of the tile's
    // row rotated by the tile's base position
    // p0 = 128 tile the other way, q' = R_{p0}^T q (q'(2f) = q(2f) cos + q(2f+1) sin, q'(2f+1) = q(2f+1) cos -
    // q(2f) sin, with the packed table's row p0), in fp32 and rounded once to fp16, so that
    // q' . R_j k = q . R_{p0 + j} k.
    auto stage_q = [&](int b_row, int tile, int buf) {
      const int tq = quarter * 32 + lane;
      if (tq < p.rep * 16) {
        const int r = tq >> 4, chunk = tq & 15, c8 = chunk & 7;
        const uint4* qr = reinterpret_cast<const uint4*>(p.q + ((size_t)b_row * p.n_q + kvh * p.rep + r) * kHeadDim +
                                                         16 * c8);
        const uint4 x0 = qr[0], x1 = qr[1];  // source dims 16 c8 .. + 15: (even, odd) of frequencies 8 c8 .. + 7
        uint32_t w[4];
        if (rel) {  // a constant of the instantiation: each body keeps one of the two paths
          // cosines of frequencies 8 c8 .. + 7 at p0: packed words 16 (c8 >> 1) + 4 (c8 & 1) .. + 3; sines 8 words on
          const uint4* tr = reinterpret_cast<const uint4*>(p.cs + (size_t)tile * kTile * 64 + 16 * (c8 >> 1) + 4 * (c8 & 1));
          const uint4 cw = __ldg(tr), sw = __ldg(tr + 2);
          const uint32_t qw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          const uint32_t cv[4] = {cw.x, cw.y, cw.z, cw.w}, sv[4] = {sw.x, sw.y, sw.z, sw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // frequencies 8 c8 + 2 i (a) and 8 c8 + 2 i + 1 (b)
            const float2 c = __half22float2(u32_as_half2(cv[i])), sn = __half22float2(u32_as_half2(sv[i]));
            const float2 a = unpack_bf16(qw[2 * i]), b = unpack_bf16(qw[2 * i + 1]);
            w[i] = chunk < 8 ? pack_half2(a.x * c.x + a.y * sn.x, b.x * c.y + b.y * sn.y)
                             : pack_half2(a.y * c.x - a.x * sn.x, b.y * c.y - b.x * sn.y);
          }
        } else {
          const uint32_t sel = chunk < 8 ? 0x5410u : 0x7632u;  // even (low) or odd (high) halves
          const uint32_t bw[4] = {__byte_perm(x0.x, x0.y, sel), __byte_perm(x0.z, x0.w, sel),
                                  __byte_perm(x1.x, x1.y, sel), __byte_perm(x1.z, x1.w, sel)};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack_bf16(bw[i]);
            w[i] = pack_half2(f.x, f.y);
          }
        }
        const uint32_t off = (chunk >> 3) * 2048 + r * 128 + ((c8 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(smem + Lay::OFF_Q + (2 * g + buf) * Lay::Q_BYTES + off) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_QF + 2 * g + buf));
    };
    // Q for the group's first two segments now; at the start of segment sigma >= 1, the one after it
    // (buffer (sigma + 1) & 1 last fed QK of segment sigma - 1, all of whose scores are read by then).
    // Chunk-relative RoPE: Q per tile instead, tiles 0 and 1 now and tile j + 2 once softmax(j) has seen the
    // scores of QK(j), the last reader of buffer j & 1.
    GroupTiles<NP> qa;
    qa.init(p, seg0, g, n);
    if (g < NP && qa.valid()) {
      if (rel) {
        stage_q(qa.s.b, qa.tile(), 0);
        qa.next(p);
        if (qa.valid()) {
          stage_q(qa.s.b, qa.tile(), 1);
          qa.next(p);
        }
      } else {
        stage_q(qa.s.b, -1, 0);
        qa.next_segment(p);
        if (qa.valid()) stage_q(qa.s.b, -1, 1);
      }
    }
    // alphaN: softmax scale of tiles j with j%2 == N; o_acc[mb][h]: latent dim 128 mb + row of head h
    float m_run[4], l_run[4], o_acc[NMB][4], alpha0[4], alpha1[4];
    int j0 = 0, sigma = 0;
    bool ok = true;
    for (RowSeg sg = seg0; g < NP && sg.cnt > 0; sg = seg_next(p, n, sg)) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.f;
#pragma unroll
        for (int mb = 0; mb < NMB; ++mb) o_acc[mb][h] = 0.f;
        alpha0[h] = alpha1[h] = 1.f;
      }
      const int cnt = seg_group_count<NP>(sg, g), kf = seg_group_first<NP>(sg, g);
      if (cnt > 0) {
        if (sigma >= 1 && !rel) {
          qa.next_segment(p);
          if (qa.valid()) stage_q(qa.s.b, -1, (sigma + 1) & 1);
        }
        const int L = row_len(p, sg.b);
        // softmax(j) then accumulate(j - 1) per step; the segment's last tile is accumulated before its
        // record is written (the QK+PV issuer issues each PV as soon as its P is written, so this waits
        // for one PV only).
        for (int x = 0; x <= cnt; ++x) {
          // ---- softmax(j) -------------------------------------------------------------------------------
          if (x < cnt) {
            const int j = j0 + x;
            // fp8 caches: K rows were rebuilt from their codes, so the score of row t carries its row scale
            // 2^k (RoPE and the dot product are linear in the row), applied here with the softmax scale
            float sl2 = p.scale_log2;
            if constexpr (F8 && !F4) {
              const int kpos = (sg.ta + (kf - sg.kb) + NP * x) * kTile + row;
              if (kpos < p.max_seq)
                sl2 = ldexpf(sl2, __ldg(p.k_exp + ((size_t)sg.b * p.n_groups + lat_head) * p.max_seq + kpos));
            }
            if (!wait_all(bar(B_SF + 2 * g + (j & 1)), (j >> 1) & 1)) {
              ok = false;
              break;
            }
            fence_after();
            uint32_t sc[4];
            tmem_ld4(trow + kColDs + (j & 1) * 16, sc);
            tmem_wait_ld_regs(sc);
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_SR + 2 * g + (j & 1)));  // D_s[j & 1] may be overwritten
            const int tile_start = (sg.ta + (kf - sg.kb) + NP * x) * kTile;
            const bool valid = tile_start + row < L;
            float xs[4], mx[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              xs[h] = (valid && h < p.rep) ? __uint_as_float(sc[h]) * sl2 : -INFINITY;
              mx[h] = warp_max(xs[h]);
            }
            // The 4 warps' maxima meet through a double-buffered mbarrier (bounded wait, unlike bar.sync).
            float* smx = s_max + ((g * 2 + (j & 1)) * 4) * 4;
            if (lane == 0) {
#pragma unroll
              for (int h = 0; h < 4; ++h) smx[quarter * 4 + h] = mx[h];
              mbar_arrive(bar(B_MX + 2 * g + (j & 1)));
            }
            if (!wait_all(bar(B_MX + 2 * g + (j & 1)), (j >> 1) & 1)) {
              ok = false;
              break;
            }
            unsigned char* sP = smem + Lay::OFF_P + (2 * g + (j & 1)) * Lay::P_BYTES;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float tmax = fmaxf(fmaxf(smx[h], smx[4 + h]), fmaxf(smx[8 + h], smx[12 + h]));
              const float m_new = fmaxf(m_run[h], tmax);
              const float alpha = (m_new == -INFINITY) ? 1.f : fast_exp2(m_run[h] - m_new);
              const float pv = (m_new == -INFINITY) ? 0.f : fast_exp2(xs[h] - m_new);
              if (j & 1)
                alpha1[h] = alpha;
              else
                alpha0[h] = alpha;
              l_run[h] = l_run[h] * alpha + pv;
              m_run[h] = m_new;
              if constexpr (F8) {  // P as f16 hi + lo (the V tile is f16)
                const __half hi = __float2half_rn(pv);
                const __half lo = __float2half_rn(pv - __half2float(hi));
                *reinterpret_cast<__half*>(sP + sw128_offset(h, row, 16)) = hi;
                *reinterpret_cast<__half*>(sP + sw128_offset(4 + h, row, 16)) = lo;
                continue;
              }
              const __nv_bfloat16 hi = __float2bfloat16_rn(pv);
              const __nv_bfloat16 lo = __float2bfloat16_rn(pv - __bfloat162float(hi));
              *reinterpret_cast<__nv_bfloat16*>(sP + sw128_offset(h, row, 16)) = hi;
              *reinterpret_cast<__nv_bfloat16*>(sP + sw128_offset(4 + h, row, 16)) = lo;
            }
            fence_proxy_async();
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_PF + 2 * g + (j & 1)));
            if (rel && qa.valid()) {  // Q of tile j + 2 into buffer j & 1
              stage_q(qa.s.b, qa.tile(), j & 1);
              qa.next(p);
            }
          }
          // ---- accumulate(j - 1) --------------------------------------------------------------------------
          if (x >= 1) {
            const int ja = j0 + x - 1;
            if (!wait_all(bar(B_OF + 2 * g + (ja & 1)), (ja >> 1) & 1)) {
              ok = false;
              break;
            }
            fence_after();
#pragma unroll
            for (int mb = 0; mb < NMB; ++mb) {
              if (mb >= nmb) break;
              uint32_t ov[8];
              tmem_ld8(trow + do_col(ja & 1, mb), ov);
              tmem_wait_ld_regs(ov);
#pragma unroll
              for (int h = 0; h < 4; ++h)
                o_acc[mb][h] = o_acc[mb][h] * ((ja & 1) ? alpha1[h] : alpha0[h]) + __uint_as_float(ov[h]) +
                               __uint_as_float(ov[4 + h]);
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_OR + 2 * g + (ja & 1)));
          }
        }
        if (!ok) break;
        j0 += cnt;
        ++sigma;
      }
      // ---- this group's partial of the segment (empty when the group had no tile in it) ----------------
      const bool starts_before = sg.kb == 0 && sg.ta > 0;
      const bool ends_after = sg.kb + sg.cnt == n && sg.ta + sg.cnt < row_tiles(p, sg.b);
      const size_t rec = (!starts_before && !ends_after)
                             ? tc_rec_direct(sg.b, kvh, p.n_kv, g)
                             : tc_rec_edge(p.batch, p.n_kv, p.ctas, kvh, cta, starts_before ? 0 : 1, g);
      float* wo = p.ws_o + rec * p.rep * p.rv;
      float* wml = p.ws_ml + rec * p.rep * 5;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float v = l_run[h];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (h < p.rep) {
          if (lane == 0) wml[h * 5 + 1 + quarter] = v;
          if (quarter == 0 && lane == 0) wml[h * 5] = m_run[h];
          // D_o rows (latent dims): lane 32 q + l holds row 32 q + l (M = 128), or row 16 q + l for l < 16 (M = 64);
          // M-block mb holds latent dims 128 mb + row.
#pragma unroll
          for (int mb = 0; mb < NMB; ++mb) {
            const int orow = KBV == 1 ? 16 * quarter + lane : 128 * mb + row;
            if ((KBV != 1 || lane < 16) && orow < p.rv) wo[h * p.rv + orow] = o_acc[mb][h];
          }
        }
      }
    }
  }
  // every role reaches this point warp-converged
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace tc
}  // namespace palu
