/*
 * sparse_attn_b200.h - C ABI of the B200 (sm_100a) dynamic block-sparse prefill path.
 *
 * Drop-in native layer under the Python package `sm120_attn` (same module and function names as
 * accion-intelligence/Qwen38-sparse-attn).  Every entry point takes raw device pointers, element
 * strides and sizes, runs asynchronously on the given CUDA stream (a `cudaStream_t` passed as
 * `void*`; NULL = legacy default stream), allocates nothing, and returns SA_OK or a negative
 * SA_ERR_* code; `sa_last_error()` gives a message for the calling thread's last failure.
 * Tensors are row-major with explicit element strides; bf16 data is passed as 16-bit words and
 * e4m3 (float8_e4m3fn) data as bytes.
 *
 * Kernels that wait on barriers bound every wait (about 2 s of wall time).  When a wait expires
 * the kernel writes SA_DEV_* bits into the caller's `status` word (device int32, may be NULL),
 * stops, frees its tensor memory and returns; `sa_read_status` fetches and clears the word.
 */
#ifndef SPARSE_ATTN_B200_H
#define SPARSE_ATTN_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SA_API __attribute__((visibility("default")))
#else
#define SA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define SA_OK 0
#define SA_ERR_ARG (-1)          /* bad shape, size or argument combination              */
#define SA_ERR_ALIGN (-2)        /* pointer or stride not aligned as the kernel requires  */
#define SA_ERR_UNSUPPORTED (-3)  /* head_dim, block size or mode not implemented          */
#define SA_ERR_CUDA (-4)         /* CUDA runtime error (launch, attribute, symbol)        */
#define SA_ERR_TMA (-5)          /* TMA tensor-map encoding failed                        */
#define SA_ERR_DEVICE (-6)       /* a kernel reported a device-side failure (status word) */

/* bits a kernel may set in the device status word */
#define SA_DEV_WAIT_Q 0x1        /* a wait for the query tile expired                     */
#define SA_DEV_WAIT_KV 0x2       /* a wait for a key/value stage expired                  */
#define SA_DEV_WAIT_S 0x4        /* a wait for the score (S) tile expired                 */
#define SA_DEV_WAIT_P 0x8        /* a wait for the probability (P) tile expired           */
#define SA_DEV_WAIT_O 0x10       /* a wait for the output accumulator expired             */
#define SA_DEV_BAD_LIST 0x20     /* a block index in a list was out of range              */
#define SA_DEV_BAD_PAGE 0x40     /* a page id in a page table was out of range (read as 0) */
#define SA_DEV_WAIT_KM 0x80      /* a wait for key means staged by the one-pass selection expired */
#define SA_DEV_WAIT_TEST 0x100   /* the wait of sa_wait_selftest expired (as it always does)  */

/* selection modes for sa_select */
#define SA_SELECT_PER_HEAD 0     /* one row per (query head, q block): union=False         */
#define SA_SELECT_KV_UNION 1     /* one row per (kv head, q block): union over the group   */
#define SA_SELECT_PAIR_UNION 2   /* one row per (query head, pair of q blocks)             */

SA_API int sa_version(void);
SA_API const char* sa_last_error(void);

/* Copy the device status word to the host (synchronises `stream`) and reset it to 0.
 * Returns SA_OK and stores the word in *value. */
SA_API int sa_read_status(int32_t* status, int32_t* value, void* stream);

/* Diagnostic of the failure path every waiting kernel shares: one CTA waits, with the library's
 * bounded mbarrier wait, for a barrier phase that nothing completes.  The wait gives up after
 * limit_ns (1000 .. about 2e9) of wall time, the kernel sets SA_DEV_WAIT_TEST in *status and
 * returns; the context stays usable.  No reference counterpart (the reference's kernels do not
 * bound their waits).  Asynchronous on `stream`; read the word with sa_read_status. */
SA_API int sa_wait_selftest(int32_t* status, int64_t limit_ns, void* stream);

/*
 * (a) Block summary.  Replaces the ATen pooling of
 *   sm120_attn/sparse_prefill.py:437-446 (`_cached_block_means`: append the chunk's K block means
 *   to the cache, partial boundary blocks averaged over the rows this chunk holds) and
 *   sm120_attn/sparse_prefill.py:58-63 (`block_masks`: mean of the valid rows of each q block).
 * x: bf16 [n, heads, head_dim] with rows at absolute positions pos0 .. pos0+n-1.  For every block
 * b in [pos0/block, ceil((pos0+n)/block)) and head h writes the fp32 mean of its rows to
 *   out[h*out_head_stride + (b - out_block0)*out_block_stride + d].
 * The mean divides by the number of rows the block holds in x, or by `fixed_divisor` when it is
 * > 0 (the reference's `km is None` path averages zero-padded blocks over BLOCK rows,
 * sparse_prefill.py:166-168, :216-218).
 * Optionally (q8 != NULL) also writes the e4m3 quantisation of every row read,
 *   q8[r*q8_row_stride + h*q8_head_stride + d] = e4m3(bf16(x * inv_scale[h*inv_scale_stride]))
 * (the glue's bf16-arithmetic quantisation, sparse_prefill.py:230), so one HBM pass serves both.
 * head_dim % 8 == 0; x 16-byte aligned with strides multiples of 8 elements.
 */
SA_API int sa_block_means_bf16(const void* x, int64_t x_row_stride, int64_t x_head_stride, int n, int heads,
                        int head_dim, int pos0, int block, float* out, int64_t out_head_stride,
                        int64_t out_block_stride, int out_block0, uint8_t* q8, int64_t q8_row_stride,
                        int64_t q8_head_stride, const float* inv_scale, int inv_scale_stride, int fixed_divisor,
                        void* stream);

/*
 * Paged KV caches.  The reference gathers a request's whole key/value history out of vLLM's paged
 * cache on every chunk (sm120_attn/sparse_prefill.py:521-522, `key_cache[pages].reshape(...)`);
 * these entries read the pages in place instead.  cache: bf16 [num_pages, page_size, heads,
 * head_dim] viewed through element strides page_stride / row_stride / head_stride (vLLM's
 * key_cache or value_cache, page_stride % 8 == 0); the row at logical position l of the request is
 * slot l % page_size of page page_table[l / page_size] (the request's row of vLLM's block table,
 * int32).  page_table must hold an entry for every page the call reads.
 */
/* sa_block_means_bf16 (no fixed divisor, no q8) over the keys at positions pos0 .. pos0+n-1 of a
 * paged cache; the same launch shape and summation order as sa_block_means_bf16 over the gathered
 * rows, so the two give the same bits. */
SA_API int sa_block_means_paged_bf16(const void* cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                     const int32_t* page_table, int page_size, int n, int heads, int head_dim,
                                     int pos0, int block, float* out, int64_t out_head_stride,
                                     int64_t out_block_stride, int out_block0, void* stream);
/* sa_absmax_bf16 over the rows at positions row0 .. row0+rows-1 of a paged cache. */
SA_API int sa_absmax_paged_bf16(const void* cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                const int32_t* page_table, int page_size, int row0, int rows, int heads, int head_dim,
                                int per_head, float* out, void* stream);
/* sa_quantize_e4m3 (row-major output) of the rows at positions row0 .. row0+rows-1 of a paged cache:
 * out row r holds position row0 + r. */
SA_API int sa_quantize_paged_e4m3(const void* cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                  const int32_t* page_table, int page_size, int row0, int rows, int heads,
                                  int head_dim, const float* scale, int scale_stride, int mode, uint8_t* out,
                                  int64_t out_row_stride, int64_t out_head_stride, void* stream);

/*
 * (b) Block selection.  Replaces `SparsePrefill.block_masks` (sm120_attn/sparse_prefill.py:41-85)
 * and the list build of sm120_attn/sparse_prefill.py:172-174 / :223-225.
 * qm: fp32 [MB, num_heads, head_dim] pooled query blocks (block strides given), q block m sits at
 * absolute block index qblk0 + m.  km: fp32 [num_kv_heads, nb_km, head_dim] cached key-block means;
 * blocks nb_km .. nb_total-1 are scored as zero vectors (the driver's zero padding,
 * sparse_prefill.py:219-221).  Per (head, q block): logits = qm.km * scale with future blocks
 * (j > qblk0+m) at -inf, softmax, keep the smallest top set (ties: lower block id first) whose
 * float64-accumulated mass rounded to fp32 reaches fp32(tau), force the diagonal and the sink
 * block, clear the future.  Rows per `mode` (SA_SELECT_*): PER_HEAD row = h*MB + m; KV_UNION
 * row = hk*MB + m; PAIR_UNION row = h*(MB/2) + t (MB even).
 * Outputs (any may be NULL): counts[row]; lists[row*list_stride + i] = selected block ids in
 * ascending order for i < counts[row] (entries past counts[row] are not written);
 * masks[row*nb_total + j] = 0/1.
 * workspace: device scratch of at least sa_select_workspace_bytes(num_heads, MB, nb_total) bytes,
 * 16-byte aligned (the fp32 logits of every row); its contents on entry do not matter.  head_dim
 * must be a multiple of 32; qm and km 16-byte aligned with strides that are multiples of 4.
 */
SA_API int sa_select(const float* qm, int64_t qm_block_stride, int64_t qm_head_stride, const float* km,
              int64_t km_head_stride, int64_t km_block_stride, int nb_km, int num_heads, int num_kv_heads,
              int head_dim, int MB, int nb_total, int qblk0, float scale, float tau, int mode, int32_t* counts,
              int32_t* lists, int64_t list_stride, uint8_t* masks, void* workspace, size_t workspace_bytes,
              void* stream);

/* Bytes of workspace sa_select needs for these sizes (0 for invalid sizes). */
SA_API size_t sa_select_workspace_bytes(int num_heads, int MB, int nb_total);

/*
 * (a)+(b) in one pass: block selection straight from the query rows.  Replaces the query pooling
 * and scoring of sm120_attn/sparse_prefill.py:58-84 (`block_masks`) like sa_block_means_bf16 +
 * sa_select, without the pooled-query tensor or the logits workspace: one CTA per (query block, or
 * pair of query blocks for SA_SELECT_PAIR_UNION; KV head) pools its rows, scores them against km
 * in shared memory and selects.
 * q: bf16 [n, num_heads, head_dim] at absolute positions q_start .. q_start+n-1, which must lie in
 * the query blocks qblk0 .. qblk0+MB-1 of `block` rows; each block's mean is taken over the rows
 * of q it holds (0 for a block without rows).  km, nb_km, nb_total, scale, tau, mode, counts,
 * lists, list_stride, masks: as sa_select (query block m is block qblk0 + m).  q8 (optional):
 * e4m3 copy of every query row as in sa_block_means_bf16 (inv_scale per head or scalar).
 * status (device int32, may be NULL): SA_DEV_WAIT_KM is set there if a wait for key means staged in
 * shared memory expires (the unit's rows are then not written).
 * Returns SA_ERR_UNSUPPORTED, launching nothing, for shapes outside the kernel's limits (head_dim
 * 128; at most 16 query heads per KV head; rows of at most 1024 key blocks; query blocks per unit
 * x query heads per KV head x nb_total rounded up to 32 at most 16384); use sa_block_means_bf16 +
 * sa_select there.
 */
SA_API int sa_select_q(const void* q, int64_t q_row_stride, int64_t q_head_stride, int n, int q_start, int block,
              int qblk0, int MB, const float* km, int64_t km_head_stride, int64_t km_block_stride, int nb_km,
              int num_heads, int num_kv_heads, int head_dim, int nb_total, float scale, float tau, int mode,
              int32_t* counts, int32_t* lists, int64_t list_stride, uint8_t* masks, uint8_t* q8,
              int64_t q8_row_stride, int64_t q8_head_stride, const float* inv_scale, int inv_scale_stride,
              int32_t* status, void* stream);

/*
 * sa_select without a workspace argument: the same selection, with its scratch taken from a
 * 40 MiB (41943040-byte) buffer that is compiled into the library, one per device.  It has no
 * counterpart in the reference, whose selection allocates through PyTorch.  It is meant for
 * callers that cannot allocate device memory at the point where they select blocks - a C or C++
 * host runtime driving this library through plain pointers with no device allocator of its own,
 * or a serving loop that must not allocate (and possibly synchronise the device) per request.
 *   - Sizes whose sa_select_workspace_bytes() exceeds 41943040 are refused with
 *     SA_ERR_UNSUPPORTED and a message naming the sizes; use sa_select then.  (64 heads x 64
 *     q blocks fit up to 2560 key blocks.)
 *   - The first call made with a given device current looks up the buffer's address on that
 *     device; later calls on that device only reuse it.  Make that first call before capturing
 *     any stream.  The address is tied to the device's CUDA context: after cudaDeviceReset (a
 *     new primary context loads the library's module again) the next call looks it up anew.
 *   - Nothing in the buffer needs to start at zero: each call writes every entry it reads.
 *   - All calls on one device share the buffer: calls whose work overlaps on the GPU (different
 *     streams, or host threads without ordering) race.  Order them on one stream.
 *   - No device memory is allocated or freed by this call.
 */
SA_API int sa_select_static(const float* qm, int64_t qm_block_stride, int64_t qm_head_stride, const float* km,
              int64_t km_head_stride, int64_t km_block_stride, int nb_km, int num_heads, int num_kv_heads,
              int head_dim, int MB, int nb_total, int qblk0, float scale, float tau, int mode, int32_t* counts,
              int32_t* lists, int64_t list_stride, uint8_t* masks, void* stream);

/* scale modes of sa_quantize_e4m3 */
#define SA_QUANT_MUL 0           /* e4m3(x * s)            fp32 multiply by s = 1/scale        */
#define SA_QUANT_MUL_BF16 1      /* e4m3(bf16(x * s))      the glue, sparse_prefill.py:230-233 */
#define SA_QUANT_DIV 2           /* e4m3(x / s)            fp32 division, kai_fa_fp8.py:327    */

/*
 * e4m3 quantisation of a bf16 [rows, heads, head_dim] tensor.  Replaces
 * sm120_attn/sparse_prefill.py:230-233 (mode SA_QUANT_MUL_BF16 with s = 1/scale) and
 * sm120_attn/kernels/kai_fa_fp8.py:325-328 (`quantize_e4m3`: mode SA_QUANT_DIV with s = scale).
 * s (`scale`) is per head (stride 1) or one scalar (stride 0).  Conversion rounds to nearest even and
 * saturates at +-448 (torch's cast gives NaN above 464; in-range values match bit for bit).
 * transpose = 0: out[r*out_row_stride + h*out_head_stride + d];
 * transpose = 1: out[h*out_head_stride + d*out_row_stride + r] (V^T, keys contiguous), rows
 *                rows..rows_pad-1 written as zeros.  This is the reference's pre-quantised vT8
 *                layout before its key permutation; the attention entry points take V untransposed.
 */
SA_API int sa_quantize_e4m3(const void* x, int64_t x_row_stride, int64_t x_head_stride, int rows, int heads,
                     int head_dim, const float* scale, int scale_stride, int mode, uint8_t* out,
                     int64_t out_row_stride, int64_t out_head_stride, int transpose, int rows_pad, void* stream);

/* amax over a bf16 [rows, heads, head_dim] tensor: out[h] (per_head = 1) or out[0] (per tensor).
 * Replaces the `.abs().amax()` reductions of sm120_attn/sparse_prefill.py:227 / :465 and
 * kai_fa_fp8.py:326. */
SA_API int sa_absmax_bf16(const void* x, int64_t x_row_stride, int64_t x_head_stride, int rows, int heads, int head_dim,
                   int per_head, float* out, void* stream);

/*
 * (c) Block-sparse causal attention forward on tcgen05 tensor cores.  Replaces
 * `attention_sm120_fp8_tma` / `attention_sm120_fp8` (sm120_attn/kernels/kai_fa_fp8_tma.py:447-490,
 * kai_fa_fp8.py:331-375) for sa_attn_fwd_fp8 and `attention_sm120` (kai_fa_bf16.py:1206-1243) for
 * sa_attn_fwd_bf16.
 * q: [n_q, num_heads, head_dim]; k, v: [kv_len, num_kv_heads, head_dim] (the natural NHD layout:
 * no transposed or key-permuted V is needed); out: bf16 [n_q, num_heads, head_dim].  Element strides.  Query tile m (128 rows) covers
 * q rows m*128 - q_front .. +127 (rows outside [0, n_q) read as zero, not written) at absolute
 * positions q_offset + m*128 + r; a key at position j is visible when j <= position and
 * j < kv_len.  Block lists (counts != NULL): tile m of head h walks
 * lists[row*list_stride + i], i < counts[row], row = h*ceil((q_front+n_q)/128) + m, each entry a
 * kv_block-key block (kv_block 64 or 128; q_block must be 128); counts == NULL walks every causal
 * block.  FP8 scales: softmax uses softmax_scale*q_scale[h]*k_scale[hk] and the output is
 * multiplied by v_scale[hk] (scale strides 0 = one scalar, 1 = per head); P is rounded to e4m3
 * after scaling by 448 (kai_fa_fp8.py:248-253).  head_dim must be 128.
 */
SA_API int sa_attn_fwd_fp8(const uint8_t* q, int64_t q_row_stride, int64_t q_head_stride, const uint8_t* k,
                    int64_t k_row_stride, int64_t k_head_stride, const uint8_t* v, int64_t v_row_stride,
                    int64_t v_head_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                    int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                    const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block, int kv_block,
                    const float* q_scale, int q_scale_stride, const float* k_scale, int k_scale_stride,
                    const float* v_scale, int v_scale_stride, float softmax_scale, int32_t* status, void* stream);

/*
 * sa_attn_fwd_fp8 with the partial last wave split.  The (query tile, head) units that fill whole
 * waves of the GPU's resident CTAs (2 per SM) run as in sa_attn_fwd_fp8; each unit of the partial
 * last wave (tail_units < 0; else the last tail_units units of the launch order: tiles from the last
 * to the first, heads in order) has its walk cut into `splits` contiguous ranges of its 64-key
 * steps, run as separate CTAs; the last of them to finish combines the ranges (the rescaled sums of
 * their unnormalised outputs), counting arrivals in the workspace (zeroed by a memset on the stream).
 * With few units of nearly equal cost (a tensor-parallel rank holding one or two KV heads) that last
 * wave is otherwise mostly idle; the reference's grid has no such split (kai_fa_fp8_tma.py:447-490
 * launches one CTA per tile and head).  Tail units whose walk has fewer than 32 * splits steps run
 * whole.  workspace: device memory of sa_attn_split_workspace_bytes(n_q, q_front, num_heads, splits,
 * tail_units) bytes (0 when nothing splits), 16-byte aligned; splits 1..16 (1: as sa_attn_fwd_fp8).
 * P is rounded to e4m3 against each range's own running max, so split rows differ from the unsplit
 * kernel's within the FP8 tolerance.  sa_attn_split_count suggests a split count for this GPU (1 when
 * the units fill less than one wave, or no split shortens the launch by 5% or more).
 */
SA_API int sa_attn_split_count(int n_q, int q_front, int num_heads);
SA_API int64_t sa_attn_split_workspace_bytes(int n_q, int q_front, int num_heads, int splits, int tail_units);
SA_API int sa_attn_fwd_fp8_split(const uint8_t* q, int64_t q_row_stride, int64_t q_head_stride, const uint8_t* k,
                                 int64_t k_row_stride, int64_t k_head_stride, const uint8_t* v, int64_t v_row_stride,
                                 int64_t v_head_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                                 int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                                 const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                                 int kv_block, const float* q_scale, int q_scale_stride, const float* k_scale,
                                 int k_scale_stride, const float* v_scale, int v_scale_stride, float softmax_scale,
                                 int32_t* status, int splits, int tail_units, void* workspace, int64_t workspace_bytes,
                                 void* stream);

SA_API int sa_attn_fwd_bf16(const void* q, int64_t q_row_stride, int64_t q_head_stride, const void* k,
                     int64_t k_row_stride, int64_t k_head_stride, const void* v, int64_t v_row_stride,
                     int64_t v_head_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                     int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                     const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block, int kv_block,
                     float softmax_scale, int32_t* status, void* stream);

/*
 * sa_attn_fwd_bf16 reading K and V from paged caches in place (the reference gathers the request's
 * history into contiguous tensors first, sm120_attn/sparse_prefill.py:521-522).  k_cache, v_cache:
 * bf16 [num_pages, page_size, num_kv_heads, head_dim] with the same element strides page_stride /
 * row_stride / head_stride (multiples of 8); the key at position j is slot j % page_size of page
 * page_table[j / page_size], for j < kv_len (page_table holds ceil(kv_len / page_size) ids in
 * [0, num_pages)).  page_size 8, 16, 32 or a multiple of 64.  Keys past kv_len read as zero, as in
 * sa_attn_fwd_bf16; a page id out of range sets SA_DEV_BAD_PAGE in status and reads as zeros.
 * Every other argument as sa_attn_fwd_bf16.
 */
SA_API int sa_attn_fwd_bf16_paged(const void* q, int64_t q_row_stride, int64_t q_head_stride, const void* k_cache,
                                  const void* v_cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                  const int32_t* page_table, int page_size, int num_pages, void* out,
                                  int64_t o_row_stride, int64_t o_head_stride, int n_q, int num_heads, int num_kv_heads,
                                  int head_dim, int kv_len, int q_front, int q_offset, const int32_t* counts,
                                  const int32_t* lists, int64_t list_stride, int q_block, int kv_block,
                                  float softmax_scale, int32_t* status, void* stream);

/*
 * Elementwise kernels of the end-to-end prefill harness (benchmark configuration 5: a random-init dense
 * GQA decoder whose TTFT the reference measures through vLLM, scripts/bench_ttft.py:1-12).  The
 * reference has no entry points of its own here: these compute what vLLM 0.22's model layers do
 * (model_executor/layers/layernorm.py fused-add RMSNorm, rotary_embedding/base.py neox rotary
 * embedding, activation.py SiluAndMul).  bf16 tensors, element strides, fp32 arithmetic.
 */

/* h <- bf16(h + delta) (delta may be NULL: no add), x <- bf16(s * rsqrt(mean(s^2) + eps) * weight)
 * with s the fp32 sum; rows x hidden, hidden % 8 == 0 and <= 8192. */
SA_API int sa_add_rmsnorm_bf16(const void* delta, int64_t delta_row_stride, void* h, int64_t h_row_stride,
                               const void* weight, void* x, int64_t x_row_stride, int rows, int hidden, float eps,
                               void* stream);

/* qkv rows [q heads | k heads | v heads] x head_dim at positions pos0 + row: neox rotary embedding
 * (element i < head_dim/2 pairs with i + head_dim/2) of the q and k heads with the fp32 table
 * cos_sin [max_pos, head_dim] (cos of the head_dim/2 angles, then their sin); q goes to
 * q_out [rows, num_heads, head_dim], k and v to k_out / v_out rows (heads contiguous). */
SA_API int sa_rope_qkv_bf16(const void* qkv, int64_t qkv_row_stride, int rows, int num_heads, int num_kv_heads,
                            int head_dim, const float* cos_sin, int pos0, int max_pos, void* q_out, void* k_out,
                            int64_t k_row_stride, void* v_out, int64_t v_row_stride, void* stream);

/* sa_rope_qkv_bf16 that also writes the fp32 block means of the rotated k rows it stores (the key
 * block summary of sm120_attn/sparse_prefill.py:437-446 taken at KV-write time, with no second pass
 * over the keys): for every block b in [pos0/block, ceil((pos0+rows)/block)) and KV head h,
 *   km[h*km_head_stride + (b - km_block0)*km_block_stride + d] = mean of k_out rows of block b
 * (the rows this call writes).  Bit for bit what sa_block_means_bf16(k_out, ..., pos0, block, km,
 * ..., km_block0) computes afterwards. */
SA_API int sa_rope_qkv_means_bf16(const void* qkv, int64_t qkv_row_stride, int rows, int num_heads, int num_kv_heads,
                                  int head_dim, const float* cos_sin, int pos0, int max_pos, void* q_out, void* k_out,
                                  int64_t k_row_stride, void* v_out, int64_t v_row_stride, int block, float* km,
                                  int64_t km_head_stride, int64_t km_block_stride, int km_block0, void* stream);

/* out[r, j] = silu(gate_up[r, j]) * gate_up[r, inter + j], j < inter (inter % 8 == 0). */
SA_API int sa_silu_mul_bf16(const void* gate_up, int64_t gate_up_row_stride, int rows, int inter, void* out,
                            int64_t out_row_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_ATTN_B200_H */
