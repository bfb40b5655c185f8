/*
 * palu_b200.h -- C ABI of the B200 (sm_100a) Palu compressed-KV decode-attention library.
 *
 * Conventions for every entry point:
 *   - all tensor pointers are device pointers, owned by the caller, row-major and contiguous in the
 *     layouts stated below; bf16 means IEEE bfloat16 (cuda_bf16.h __nv_bfloat16);
 *   - work is enqueued on `stream` (NULL = the legacy default stream) and the call returns without
 *     synchronising; errors found before launch return a nonzero status and launch nothing;
 *   - the return value is PALU_OK (0) or a PALU_ERR_* code; palu_last_error() then describes the
 *     failure in the calling thread (thread-local). The messages reuse the substrings of the
 *     reference op's validation errors ("r_k", "cs_tab", "heads_per_group", "u_v", "head_dim_v", ...).
 *   - head_dim is 128 throughout (the reference envelope).
 *
 * Reference interfaces replaced (paths inside the ryankert01/tt-cadlab tree):
 *   palu_decode_attn       <- ttnn.transformer.palu_sdpa_decode, called at palu_tt/attention.py:633-639,
 *                             CPU model palu_tt/fused.py:82-107
 *   palu_workspace_bytes   <- (no reference counterpart: the Tensix op sizes its own circular buffers,
 *                             palu_tt/fused.py:145-201); the split-K partials live in caller memory here
 *   palu_append_latents    <- ttnn.experimental.paged_update_cache x2, palu_tt/attention.py:612-625
 *   palu_plain_gqa_decode  <- ttnn.transformer.flash_multi_latent_attention_decode / stock
 *                             scaled_dot_product_attention_decode on full K, palu_tt/attention.py:703-706,
 *                             tests/test_palu_sdpa_device.py:58-65, 238-241
 *   palu_pack_cs_table     <- the cs_tab upload of palu_tt/attention.py:70-72 (fused.py:62-73 layout)
 *   palu_rope_q_append     <- nlp_create_qkv_heads_decode's split + rotary_embedding_llama on q + the two
 *                             paged_update_cache calls, palu_tt/attention.py:601-625, in one kernel
 *   palu_add_rms_norm, palu_swiglu
 *                          <- the decoder's stock RMSNorm and SwiGLU (palu_tt/model.py:52-95, tt_transformers)
 *   palu_decode_attn_paged / palu_append_latents_paged
 *                          <- the paged variant of palu_sdpa_decode and paged_update_cache with a page
 *                             table, which the reference plans but has not built (HANDOFF.md:54-55,
 *                             126-127; palu_tt/attention.py:86 and :586 assert a non-paged cache). The
 *                             page-table convention is the stock paged flash-decode op's the plan names
 *                             as its template: caches [n_blocks][heads][block_size][width], a table
 *                             [B][blocks per row] of physical block indices.
 *   palu_decode_attn_f8 / palu_append_latents_f8 / palu_quantize_latents_f8
 *                          <- palu_sdpa_decode and paged_update_cache over block-float latent caches
 *                             (bfp8_b by default, bfp4_b per side: palu_tt/attention.py:159-169;
 *                             tests/test_palu_sdpa_device.py:558-575), in the B200 form: e4m3 codes with
 *                             one power-of-two scale per (position, latent head).
 *   palu_decode_attn_f4 / palu_append_latents_f4 / palu_quantize_latents_f4
 *                          <- the same over bfp4_b latent caches, in the B200 form: e2m1 codes with one
 *                             power-of-two scale per block of 16 values.
 */
#ifndef PALU_B200_H
#define PALU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* palu_stream_t; /* the same handle type as cudaStream_t */

enum palu_status {
  PALU_OK = 0,
  PALU_ERR_INVALID = 1,   /* shapes / envelope / null pointers */
  PALU_ERR_WORKSPACE = 2, /* workspace missing or smaller than palu_workspace_bytes() */
  PALU_ERR_CUDA = 3       /* a CUDA runtime error (launch failure, no device, ...) */
};

enum palu_dtype { PALU_BF16 = 0, PALU_F32 = 1 };

/* Decode kernel families: the tcgen05/TMEM/TMA kernel (the product path, used wherever its envelope
 * covers the shapes) and the warp-level mma.sync kernel (the legacy tensor-core baseline). */
enum palu_kernel { PALU_KERNEL_AUTO = 0, PALU_KERNEL_MMA = 1, PALU_KERNEL_TC = 2 };

/* Shapes of one decode-attention call (the local shard on this GPU). */
typedef struct palu_decode_dims {
  int32_t batch;      /* B */
  int32_t n_q_heads;  /* query heads; n_q_heads / n_kv_heads query heads share a KV head */
  int32_t n_kv_heads; /* KV heads */
  int32_t n_groups;   /* latent heads in the caches: n_kv_heads (M-LRD) or n_kv_heads / group size (G-LRD) */
  int32_t head_dim;   /* must be 128 */
  int32_t r_k;        /* K latent width: a multiple of 16 up to 128, or of 32 up to 256 */
  int32_t r_v;        /* V latent width: a multiple of 16 up to 128, or of 32 up to 256 */
  int32_t max_seq;    /* cache rows per (batch row, latent head) */
  int32_t splits;     /* work partitions; 0 = choose for this GPU. tcgen05 kernel: CTAs per KV head, each
                         taking an equal share of the KV head's 128-token tiles over all batch rows;
                         mma.sync kernel: split-K partitions per (batch row, KV head) */
} palu_decode_dims;

/*
 * Fused decode attention over latent caches (replaces palu_sdpa_decode).
 *
 *   q        [B][n_q_heads][128] bf16, already rotated (RoPE at the query position)
 *   k_lat    [B][n_groups][max_seq][r_k] bf16 latent K cache
 *   v_lat    [B][n_groups][max_seq][r_v] bf16 latent V cache
 *   u_k      [n_kv_heads][r_k] rows of u_k_ld bf16 elements; the first 128 of a row are U_k in Meta
 *            (interleaved-pair) order. u_k_ld = 128 for u_k itself, 256 for w_rot = [u_k | u_k T].
 *   u_v      NULL: absorbed V (M-LRD) -- the output is the attention-weighted V latent, r_v wide;
 *            else [n_kv_heads][r_v][128] bf16 -- V rebuilt per head (G-LRD), the output is 128 wide.
 *   cs_pairs [>= max_seq][64] 32-bit words: packed rows from palu_pack_cs_table (16-byte aligned)
 *   cur_pos  [B] int32: last visible position of each row (inclusive); < 0 skips the row (zeros out)
 *   out      [B][n_q_heads][r_v or 128], out_dtype PALU_BF16 or PALU_F32
 *   workspace / workspace_bytes: >= palu_workspace_bytes(dims) bytes of device memory; its first 4
 *            bytes are a status word that must be zero when the workspace is first used (zero the
 *            buffer once after allocating it); see palu_read_status. While that word is nonzero (a
 *            bounded device wait expired in an earlier call and nobody has cleared it), every call that
 *            uses the workspace writes NaN to `out`
 *   scale    softmax scale (the reference passes head_dim ** -0.5)
 * Query head h attends KV head h / (n_q_heads / n_kv_heads), which reads latent head
 * kv / (n_kv_heads / n_groups). Positions above cur_pos[b] are masked; cur_pos[b] >= max_seq is
 * clamped to max_seq - 1.
 */
int palu_decode_attn(const void* q, const void* k_lat, const void* v_lat, const void* u_k, int64_t u_k_ld,
                     const void* u_v, const void* cs_pairs, const int32_t* cur_pos, void* out, int32_t out_dtype,
                     void* workspace, size_t workspace_bytes, const palu_decode_dims* dims, float scale,
                     palu_stream_t stream);

/*
 * palu_decode_attn without a caller workspace: allocates nothing. No counterpart in the reference (the
 * Tensix op sizes its own circular buffers). It is for callers that hold only the tensors a framework
 * hands them and have no device allocator of their own, e.g. a plugin bound over a plain C FFI inside a
 * framework whose caching allocator owns most of device memory (a raw cudaMalloc there can fail, and
 * would bypass the framework's accounting), or a decode loop that must not call cudaMalloc/cudaFree per
 * step because those calls can synchronize the device.
 * Arguments and results as palu_decode_attn. The partial results and status word live in a static
 * 8 MiB device array, one per device, held until the process exits: shapes whose palu_workspace_bytes()
 * exceeds 8 MiB are rejected with PALU_ERR_WORKSPACE. Every call rewrites each partial result that its
 * merge reads, so stale contents from the previous call are never used. Calls that overlap in time on
 * one device (other streams, other host threads) race on that array; calls in one stream are ordered
 * and safe. The first call on each device sets the array up (its address, and a zeroed status word) with
 * synchronous CUDA calls, so make it before any stream capture.
 * A bounded device wait that expires is recorded in the array's status word, and the merge then writes
 * NaN in place of the call's output; palu_read_status(NULL, &status, stream) reads (and clears) that
 * word for the current device.
 */
int palu_decode_attn_static(const void* q, const void* k_lat, const void* v_lat, const void* u_k, int64_t u_k_ld,
                            const void* u_v, const void* cs_pairs, const int32_t* cur_pos, void* out,
                            int32_t out_dtype, const palu_decode_dims* dims, float scale, palu_stream_t stream);

/*
 * Paged latent caches: fixed-size blocks of positions shared by all rows through a page table.
 *   table       [batch][table_ld] int32: entry j of row b is the physical block that holds the row's
 *               positions j*block_size .. (j+1)*block_size - 1
 *   table_ld    entries per table row, >= ceil(dims->max_seq / block_size)
 *   block_size  positions per block: 16, 32, 64 or 128
 *   n_blocks    physical blocks in each cache
 * The caches are then k_cache [n_blocks][n_groups][block_size][r_k] and v_cache
 * [n_blocks][n_groups][block_size][r_v] bf16; dims->max_seq is the positions a row may hold. A decode
 * call reads only the entries that cover positions 0..cur_pos[b]; an entry outside [0, n_blocks) reads
 * as zero latents (decode) or drops the write (append) rather than touching memory outside the caches.
 */
typedef struct palu_page_table {
  const int32_t* table;
  int32_t table_ld;
  int32_t block_size;
  int32_t n_blocks;
} palu_page_table;

/*
 * fp8 latent caches. k_codes [B][n_groups][max_seq][r_k] and v_codes [B][n_groups][max_seq][r_v] hold
 * e4m3 codes (one byte each), k_exp and v_exp [B][n_groups][max_seq] int8 the exponent k of each row's
 * scale: the cached value is code * 2^k. palu_quantize_latents_f8 and palu_append_latents_f8 write them:
 * k is the smallest integer with max|row| <= 448 * 2^k, kept in [-120, 7] (0 for an all-zero row); the
 * codes are the row times 2^-k rounded to nearest even with saturation, codes below the smallest normal
 * e4m3 value stored as a signed zero.
 *
 * palu_decode_attn_f8: palu_decode_attn over such caches (every other argument, the workspace and the
 * output as palu_decode_attn; same palu_workspace_bytes(dims)). The result equals palu_decode_attn's on
 * the dequantized caches (the kernel rebuilds each row's bf16 values exactly). Envelope: r_k, r_v <= 128,
 * contiguous caches, the tcgen05 kernel (PALU_ERR_INVALID under palu_set_kernel(PALU_KERNEL_MMA)).
 */
int palu_decode_attn_f8(const void* q, const void* k_codes, const void* v_codes, const int8_t* k_exp,
                        const int8_t* v_exp, const void* u_k, int64_t u_k_ld, const void* u_v, const void* cs_pairs,
                        const int32_t* cur_pos, void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                        const palu_decode_dims* dims, float scale, palu_stream_t stream);

/* rows x r bf16 values (r a multiple of 16 in [16, 256]) -> rows x r e4m3 codes and rows exponents. */
int palu_quantize_latents_f8(const void* latents, int64_t rows, int32_t r, void* codes, int8_t* exps,
                             palu_stream_t stream);

/* palu_append_latents into fp8 caches: new_k [B][n_groups][r_k], new_v [B][n_groups][r_v] bf16 quantized
 * row by row into position cur_pos[b]; rows with cur_pos outside [0, max_seq) are skipped. */
int palu_append_latents_f8(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_codes, void* v_codes,
                           int8_t* k_exp, int8_t* v_exp, const palu_decode_dims* dims, palu_stream_t stream);

/*
 * fp4 latent caches. k_codes [B][n_groups][max_seq][r_k / 2] and v_codes [...][r_v / 2] hold two e2m1 codes per
 * byte (the first value in the low nibble), k_exp [B][n_groups][max_seq][r_k / 16] and v_exp [...][r_v / 16]
 * int8 the exponent k of each block of 16 values: the cached value is code * 2^k. k is the smallest integer
 * with max|block| <= 6 * 2^k, kept in [-120, 7] (0 for an all-zero block); the codes round to nearest even
 * with saturation. palu_decode_attn_f4 is palu_decode_attn over such caches, envelope r_k, r_v in {64, 128},
 * contiguous caches, the tcgen05 kernel; the others as their fp8 counterparts (r a multiple of 16).
 */
int palu_decode_attn_f4(const void* q, const void* k_codes, const void* v_codes, const int8_t* k_exp,
                        const int8_t* v_exp, const void* u_k, int64_t u_k_ld, const void* u_v, const void* cs_pairs,
                        const int32_t* cur_pos, void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                        const palu_decode_dims* dims, float scale, palu_stream_t stream);
int palu_quantize_latents_f4(const void* latents, int64_t rows, int32_t r, void* codes, int8_t* exps,
                             palu_stream_t stream);
int palu_append_latents_f4(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_codes, void* v_codes,
                           int8_t* k_exp, int8_t* v_exp, const palu_decode_dims* dims, palu_stream_t stream);

/*
 * palu_decode_attn over paged caches: every other argument, the workspace and the output as
 * palu_decode_attn (same palu_workspace_bytes(dims)). With the same latents at the same logical
 * positions the result is bit-identical to palu_decode_attn on contiguous caches.
 */
int palu_decode_attn_paged(const void* q, const void* k_cache, const void* v_cache, const void* u_k, int64_t u_k_ld,
                           const void* u_v, const void* cs_pairs, const int32_t* cur_pos,
                           const palu_page_table* pages, void* out, int32_t out_dtype, void* workspace,
                           size_t workspace_bytes, const palu_decode_dims* dims, float scale, palu_stream_t stream);

/*
 * palu_append_latents into paged caches: row b's latents go to row cur_pos[b] % block_size of block
 * table[b][cur_pos[b] / block_size]. Rows with cur_pos outside [0, max_seq) are skipped.
 */
int palu_append_latents_paged(const void* new_k, const void* new_v, const int32_t* cur_pos,
                              const palu_page_table* pages, void* k_cache, void* v_cache,
                              const palu_decode_dims* dims, palu_stream_t stream);

/*
 * One decode step's q rotation and latent append in one kernel (replaces the split of
 * nlp_create_qkv_heads_decode, rotary_embedding_llama on q and the two paged_update_cache calls,
 * palu_tt/attention.py:601-625).
 *   qkv      [B][ld] (qkv_dtype PALU_BF16 or PALU_F32): per row the n_q_heads * 128 query values (Meta pair
 *            order), then n_groups * r_k K latents, then n_groups * r_v V latents (the fused projection)
 *   cos, sin [>= max_seq][128] f32: cos / sin of frequency j at columns 2j and 2j + 1
 *   cur_pos  [B]: q is rotated at cur_pos clamped to [0, max_seq); the latents are appended at cur_pos
 *            (rows outside [0, max_seq) append nothing)
 *   q_out    [B][n_q_heads][128] bf16 (4-byte aligned), the decode op's q
 *   k_cache, v_cache, pages: as palu_append_latents (pages NULL) or palu_append_latents_paged
 * dims: batch, n_q_heads, n_groups, head_dim (128), r_k, r_v, max_seq. Each product of the rotation and
 * their sum are rounded separately, so q is bit-identical to rotating in fp32 tensor ops and rounding to bf16.
 */
int palu_rope_q_append(const void* qkv, int64_t ld, int32_t qkv_dtype, const float* cos, const float* sin,
                       const int32_t* cur_pos, void* q_out, void* k_cache, void* v_cache, const palu_page_table* pages,
                       const palu_decode_dims* dims, palu_stream_t stream);

/*
 * Decoder steps around the attention layer (the stock RMSNorm and SwiGLU MLP of the decoder the reference
 * assembles, palu_tt/model.py:52-95), fused to cut a decode step's kernel count.
 * palu_add_rms_norm: h [rows][dim] f32 in place += delta ([rows][dim] of delta_dtype PALU_F32 or PALU_BF16,
 *   or NULL), then out [rows][dim] bf16 = h * rsqrt(mean(h^2) + eps) * w (w [dim] f32). dim a multiple of 4;
 *   pointers 16-byte aligned.
 * palu_swiglu: gu [rows][ld] bf16 = gate (columns 0..f-1) then up (f..2f-1); out [rows][f] bf16 =
 *   bf16(bf16(silu(gate)) * up).
 */
int palu_add_rms_norm(float* h, const void* delta, int32_t delta_dtype, const float* w, void* out, int32_t rows,
                      int32_t dim, float eps, palu_stream_t stream);
int palu_swiglu(const void* gu, int64_t ld, int32_t f, void* out, int32_t rows, palu_stream_t stream);

/* Device bytes palu_decode_attn / palu_plain_gqa_decode need for their partial results (enough for either
 * kernel family, so palu_set_kernel may change between calls). */
size_t palu_workspace_bytes(const palu_decode_dims* dims);

/* The partition count (see palu_decode_dims.splits) a call with dims->splits == 0 uses on the current device. */
int32_t palu_choose_splits(const palu_decode_dims* dims);

/*
 * Append one decode step's latents at cur_pos[b] (replaces the two paged_update_cache calls).
 *   new_k [B][n_groups][r_k] bf16, new_v [B][n_groups][r_v] bf16; rows with cur_pos outside
 *   [0, max_seq) are skipped. Caches as in palu_decode_attn.
 */
int palu_append_latents(const void* new_k, const void* new_v, const int32_t* cur_pos, void* k_cache, void* v_cache,
                        const palu_decode_dims* dims, palu_stream_t stream);

/*
 * Plain GQA flash-decode over full, already-rotated K (the identity comparison path).
 *   k [B][n_kv_heads][max_seq][128] bf16, v [B][n_kv_heads][max_seq][dims->r_v] bf16,
 *   out [B][n_q_heads][r_v]. dims->n_groups must equal n_kv_heads and dims->r_k must be 128.
 */
int palu_plain_gqa_decode(const void* q, const void* k, const void* v, const int32_t* cur_pos, void* out,
                          int32_t out_dtype, void* workspace, size_t workspace_bytes, const palu_decode_dims* dims,
                          float scale, palu_stream_t stream);

/*
 * Pack the reference's [rows][ld] [cos | sin] table (bf16 or fp32, pair-duplicated frequency
 * columns: cos_j at column 2j, sin_j at 128 + 2j) into rows of 128 fp16 (= 64 32-bit words): 4 blocks
 * of 16 frequencies, each block the 16 cosines (frequency order) followed by the same 16 sines.
 */
int palu_pack_cs_table(const void* cs_tab, int64_t ld, int32_t in_dtype, void* cs_pairs, int32_t rows,
                       palu_stream_t stream);

/*
 * Select the decode kernel family for subsequent calls in this process (PALU_KERNEL_AUTO by default:
 * the tcgen05 kernel where its envelope covers the shapes, else the mma.sync kernel). No reference
 * counterpart (the Tensix op has one program); used to benchmark the legacy path against the product.
 */
int palu_set_kernel(int32_t which);

/*
 * Test hook for the timeout path of the tcgen05 decode kernel (no reference counterpart; not needed in
 * normal use). For subsequent decode calls in this process: wait_ns > 0 bounds every device-side wait at
 * wait_ns nanoseconds instead of the default 1 s (0 restores the default); starve_v nonzero makes one V
 * producer per CTA issue no loads, so that a wait runs out on purpose. Such a call records status 1 in its
 * workspace (palu_read_status), its merge writes NaN, and the device stays usable for the next call.
 */
int palu_set_wait_limit(int64_t wait_ns, int32_t starve_v);

/*
 * RoPE form of the decode calls this host thread makes after it (thread-local; PALU_ROPE_ABSOLUTE by
 * default). Replaces the reference op's Phase 1 / Phase 2 switch: palu_sdpa_decode rotates each key with
 * the table row of its position unless rot_step and trans_mat are passed (Phase 2: chunk-relative
 * angles, the query rotated per chunk; palu_tt/fused.py:1-14, attention.py:74-75 and 633-639, switched
 * by PaluRuntime.cs_recurrence, convert.py:36).
 *   PALU_ROPE_ABSOLUTE         key position p rotated by table row p (Phase 1).
 *   PALU_ROPE_CHUNK_RELATIVE   Phase 2 with 128-position chunks: key position p = 128 t + j rotated by
 *                              table row j, the query of chunk t rotated back by row 128 t (fp32, rounded
 *                              once to fp16), so R_p is taken as R_{128 t} R_j. Equal to the absolute form
 *                              for an exact rotation table, within the table's rounding otherwise (a bf16
 *                              table moves the output by ~2e-3 mean relative; an fp32 table, packed to fp16,
 *                              by ~2e-4). The tcgen05 kernel reads rows 0..127 once per CTA instead of every
 *                              key's row. The mma.sync kernel has no chunk-relative form: its calls fail.
 */
enum palu_rope_mode { PALU_ROPE_ABSOLUTE = 0, PALU_ROPE_CHUNK_RELATIVE = 1 };
int palu_set_rope_mode(int32_t mode);

/* The kernel family a palu_decode_attn call with these dims would run (PALU_KERNEL_MMA or _TC). */
int32_t palu_kernel_for(const palu_decode_dims* dims);

/*
 * Read (and clear) the status word a decode call left in `workspace`: 0 = ok, 1 = a bounded device
 * wait expired (the call's output is then NaN). workspace NULL reads the static scratch of
 * palu_decode_attn_static on the current device. Synchronises `stream`. No reference counterpart:
 * the Tensix op has no bounded waits (its known hangs were capped by the host, README.md:301-329).
 */
int palu_read_status(void* workspace, int32_t* status, palu_stream_t stream);

/* Description of the last failure in this thread ("" if none). */
const char* palu_last_error(void);

/* Library version string. */
const char* palu_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PALU_B200_H */
