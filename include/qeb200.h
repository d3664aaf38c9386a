/*
 * qeb200.h — C ABI of libqeb200.so, the B200 (sm_100a) implementation of QwenEdit's
 * paged prefix K/V cache and fused NVFP4 activation quantisers.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes (no torch types), and returns an
 * int status (QE_OK == 0). On failure a human-readable message is available from qe_last_error()
 * (thread-local). Device entry points take an explicit cudaStream_t (passed as void*) and are
 * asynchronous with respect to the host; they never synchronise the stream.
 *
 * Reference interfaces replaced (paths inside the QwenEdit project, shauray8/QwenEdit):
 *   multi_turn/cache/paged.py:40-131   PagedKVPool (match / alloc / insert / gather / write / usage / clear)
 *   multi_turn/pipeline/hooks.py:126-139  _store_computed (2*L per-layer index_copy_)
 *   multi_turn/cache/encoder.py:114,131-138  extra index_select / index_copy_
 *   multi_turn/fibo/fp4.py:37-116       _e2m1 / _quantize_store / _norm_scale_fp4_kernel / _silu_mul_fp4_kernel
 *   SGLang RadixCache + TokenToKVPoolAllocator as driven by paged.py:52-55,75,79,93,95,99,102
 */
#ifndef QEB200_H
#define QEB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------- */
enum {
  QE_OK = 0,
  QE_ERR_INVALID = 1,   /* bad argument: null pointer, negative size, misalignment, stale handle */
  QE_ERR_CUDA = 2,      /* a CUDA runtime call or kernel launch failed */
  QE_ERR_NOMEM = 3,     /* host allocation failed */
  QE_ERR_TIMEOUT = 4,   /* a bounded device-side wait gave up (kernel returned early) */
  QE_ERR_STATE = 5      /* misuse of an object (e.g. unlocking a node that holds no lock) */
};

/* Message for the last failing call on this thread ("" when none). */
const char *qe_last_error(void);
/* Library version string. */
const char *qe_version(void);

/* ---- paged K/V data movement (device) --------------------------------------------------------
 *
 * A "plane" is one [rows, row_bytes] slab of a pool: for the DiT pool kv[L, 2, cap+1, H, D] there
 * are 2*L planes (layer l, K/V c) of row_bytes = H*D*elem. Plane p starts at
 *     base + (p / planes_inner) * outer_stride + (p % planes_inner) * inner_stride      (bytes)
 * so both the contiguous pool and strided caller views (e.g. kv[:, :, m:] of a larger tensor)
 * are expressed without copies. Rows inside a plane are row_bytes apart (row-contiguous).
 *
 * Token-slot form: `slots` is a device int64 array, one pool row per token (page_size 1,
 * the reference's token-granular RadixCache indices, paged.py:80).
 * Block-table form: `block_table` is a device int32 array of page ids; token t lives in pool row
 * block_table[t / page_size] * page_size + t % page_size.
 *
 * Requirements: row_bytes, strides and base pointers multiples of 16 bytes; slots / pages in range
 * (checked on the device: an out-of-range slot is skipped and reported through *err_flag when
 * err_flag is non-null; pass the pool's row count in pool_rows).
 * *err_flag bits (OR-ed by the device, never cleared by it): 1 = a slot or page out of range (row skipped),
 * 2 = a bounded wait of the bulk-copy kernel gave up, 4 = a per-plane source pointer (pointer forms) null or
 * misaligned (plane skipped).
 */
typedef struct qe_planes {
  void *base;            /* device pointer of plane 0 */
  int64_t outer_stride;  /* bytes between planes p and p + planes_inner */
  int64_t inner_stride;  /* bytes between planes p and p + 1 inside one outer group */
  int32_t planes_inner;  /* planes per outer group (2 for K/V, 1 for a plain stack) */
  int32_t _pad;
} qe_planes;

/* gather: out plane p row t = pool plane p row slots[t]  (paged.py:106-113, index_select dim 2;
 * encoder.py:114 extra.index_select). n_planes planes, n_tokens rows each. */
int qe_gather_slots(qe_planes pool, int64_t pool_rows, qe_planes out, int32_t n_planes, int64_t row_bytes,
                    const int64_t *slots, int64_t n_tokens, int32_t *err_flag, void *stream);

/* gather through a page table (page_size tokens per page; the paged mode the 1K / 2K edit benchmark uses). */
int qe_gather_pages(qe_planes pool, int64_t pool_rows, qe_planes out, int32_t n_planes, int64_t row_bytes,
                    const int32_t *block_table, int32_t page_size, int64_t n_tokens, int32_t *err_flag,
                    void *stream);

/* append (scatter): pool plane p row slots[t] = src plane p row t  (paged.py:115-116 index_copy_ dim 2;
 * encoder.py:135 extra.index_copy_). */
int qe_append_slots(qe_planes pool, int64_t pool_rows, qe_planes src, int32_t n_planes, int64_t row_bytes,
                    const int64_t *slots, int64_t n_tokens, int32_t *err_flag, void *stream);

/* append through a page table. */
int qe_append_pages(qe_planes pool, int64_t pool_rows, qe_planes src, int32_t n_planes, int64_t row_bytes,
                    const int32_t *block_table, int32_t page_size, int64_t n_tokens, int32_t *err_flag,
                    void *stream);

/* append from one source pointer per plane (hooks.py:136-138: 2*L separate index_copy_ calls from
 * the per-layer caches layer["key"][0] / layer["value"][0]) in ONE launch. src_ptrs is a DEVICE
 * array of n_planes device pointers; each source plane is row-contiguous ([n_tokens, row_bytes]).
 * Every source pointer must be 16-byte aligned (the host cannot see them; the kernel checks each one against
 * the vector width it was launched with and skips a null or misaligned plane, setting bit 4 of *err_flag). */
int qe_append_slots_ptrs(qe_planes pool, int64_t pool_rows, const void *const *src_ptrs, int32_t n_planes,
                         int64_t row_bytes, const int64_t *slots, int64_t n_tokens, int32_t *err_flag,
                         void *stream);

/* qe_append_slots_ptrs for callers that cannot allocate device memory: the per-plane source pointers are
 * passed as a HOST array and copied into a table inside this library's own device memory, so the caller
 * allocates nothing (qe_append_slots_ptrs needs a caller-allocated device array of pointers). Meant for hosts
 * whose device memory is all owned by another allocator (e.g. a serving process that reserved the GPU's memory
 * up front), or code paths that must not allocate. No counterpart in the reference.
 * Limits: n_planes <= 1024 (an 8 KiB table per GPU that loads the library, held until exit); larger calls fail
 * with QE_ERR_INVALID before any work. The first call on each device looks the table up with
 * cudaGetSymbolAddress (a set-up step, done once per device with that device current), so make that first call
 * before any stream capture. Every call rewrites the table's
 * first n_planes entries on `stream` and the kernel reads them from there: calls whose work can overlap on the
 * GPU (different streams) race on the shared table; issue them on one stream. Host threads calling on one stream
 * are serialised by a per-device lock held from the table write through the launch, so their table writes and
 * kernels cannot interleave. Allocates nothing: no cudaMalloc, cudaFree or allocating library call. The host
 * array is copied with cudaMemcpyAsync: pageable memory may be reused once the call returns, pinned memory once
 * `stream` has passed the call. Null source pointers are rejected; the vector width follows the least-aligned
 * source pointer. */
int qe_append_slots_ptrs_noalloc(qe_planes pool, int64_t pool_rows, const void *const *src_ptrs_host,
                                 int32_t n_planes, int64_t row_bytes, const int64_t *slots, int64_t n_tokens,
                                 int32_t *err_flag, void *stream);

/* Gather into a head-major layout with room for a tail (the text encoder's partial hit, cache/encoder.py:173-182,
 * which gathers [L, 2, m, H, D] and then builds [1, H, m + n, D] per layer by transpose + cat): for every plane
 * p, token t < n_tokens and head h, the head_bytes of head h of pool row slots[t] go to
 *   out.plane(p) + h * out_head_stride + t * out_token_stride.
 * row_bytes = heads * head_bytes; everything 16-byte aligned. When everything is also 32-byte aligned (and the
 * copy mode is not 4) the copy moves 256-bit vectors, else 16-byte ones; the result is the same. Slots outside
 * [0, pool_rows) are skipped and set *err_flag. No counterpart as such in the reference (it is index_select +
 * transpose + cat). */
int qe_gather_slots_heads(qe_planes pool, int64_t pool_rows, qe_planes out, int32_t n_planes, int64_t row_bytes,
                          int64_t head_bytes, int64_t out_head_stride, int64_t out_token_stride, const int64_t *slots,
                          int64_t n_tokens, int32_t *err_flag, void *stream);

/* Kernel used by the copies above (process-wide): 0 = default, 1 = warp-vectorised LDG/STG kernel (rows of at
 * most 1 KiB are moved several per warp pass; on 32-byte aligned planes in 256-bit vectors, else 16-byte
 * ones), 2 = TMA bulk-copy pipeline (cp.async.bulk through shared memory; 16-byte aligned
 * rows of <= 32 KiB, else the warp kernel), 3 = the warp kernel with one row per warp pass whatever the row
 * size, 4 = the warp kernel with 16-byte vectors only (also for qe_gather_slots_heads). No counterpart in the
 * reference; for measurement and tuning. */
int qe_set_paged_copy_mode(int32_t mode);

/* ---- fused NVFP4 activation quantisers (device) ---------------------------------------------
 *
 * Output contract (fibo/fp4.py:29-34, :46-61, :94-98): q [M, K/2] uint8, e2m1 pairs, low nibble =
 * even column; sf [pad128(M), K/16] uint8 e4m3 block scales in the 128x4-swizzled layout
 *   offset(m, g) = (m/128)*(K/64*512) + (g/4)*512 + (m%32)*16 + (m%128/32)*4 + g%4
 * Rows M..pad128(M)-1 receive zero scales. K must be a multiple of 64. gs is a device fp32 scalar
 * (the layer's global activation scale, pipeline/fp4.py:33-35).
 */

/* RMSNorm + adaLN scale (+ optional shift) -> NVFP4   (fibo/fp4.py:64-80, wrapper :101-109).
 *   x [M, K] bf16 row-major (M = B*S), w [K] bf16,
 *   noisy / clean: bf16 rows of length >= K, row b at noisy + b*mod_stride (elements; 0 = one row
 *   shared by every batch);
 *   mask: uint8 [S] or null (null: every token uses `noisy`); clean may be null when mask is null;
 *   shift / shift_clean: optional bf16 adaLN shift rows with the same layout and mask select
 *   (the adaLN form x*(1+scale)+shift of the benchmark; the reference has no shift). */
int qe_norm_scale_fp4(const void *x, const void *w, const void *noisy, const void *clean, const uint8_t *mask,
                      const void *shift, const void *shift_clean, const float *gs, int64_t M, int64_t S,
                      int64_t K, int64_t mod_stride, float eps, uint8_t *q, uint8_t *sf, void *stream);

/* Where qe_norm_scale_fp4 / qe_norm_scale_amax keep the per-column constants (process-wide): 0 = default
 * (tensor memory when K is the specialised width 3072, M >= 12288 rows and they fit 256 TMEM columns, else
 * shared memory or global memory), 1 = never tensor memory, 2 = always global memory (read through L1). Results
 * are identical in every mode. No counterpart in the reference; for measurement and tests. */
int qe_set_norm_table_mode(int32_t mode);

/* Where qe_silu_mul_fp4 / qe_silu_mul_amax read the SiLU table from (process-wide): 0 = by size (default),
 * 1 = staged in shared memory by every CTA, 2 = global memory through the L1 cache (by size: below 1,024
 * rows). Results are identical.
 * No counterpart in the reference; for measurement and tests. */
int qe_set_silu_table_mode(int32_t mode);

/* How the fp32 divisions and the reciprocal square root that the reference leaves to its compiler are evaluated
 * by qe_norm_scale_fp4 / qe_silu_mul_fp4 (process-wide): `1.0 / gs` and `1.0 / (sff * (1.0 / gs))` of the
 * quantiser (fibo/fp4.py:53-55), `sum / K` and `tl.rsqrt` of the norm (fibo/fp4.py:70). Bits 0-1: the
 * quantiser's reciprocals, bits 2-3: the norm's mean division (0 = IEEE round-to-nearest, 1 = PTX div.full.f32,
 * 2 = div.approx.f32, 3 = rcp.approx.f32 then a multiply); bit 4: rsqrt (0 = correctly rounded 1 / sqrt,
 * 1 = rsqrt.approx.f32). 0 = IEEE everywhere, the rounding of a CPU restatement. The default, 21 = 1 | 1 << 2 |
 * 1 << 4, reproduces the reference's Triton kernels as Triton compiles them for sm_100 (codes and scales measured
 * bit-identical on a B200 except for rare row-sum ordering differences of the norm, 2 codes in 100.7 M at
 * T = 32768). No counterpart in the reference. */
int qe_set_nvfp4_numerics(int32_t numerics);

/* Launch of qe_norm_scale_fp4 / qe_silu_mul_fp4 and their amax modes (process-wide): 1 (default) = with
 * programmatic stream serialization, so that the next kernel on the stream may place its CTAs on SMs this launch has
 * left while its last CTAs run (each quantiser waits for the grids it depends on before its first global read);
 * 0 = plain stream order. Results are identical. No counterpart in the reference; for measurement. */
int qe_set_nvfp4_pdl(int32_t on);

/* SiLU kernel load schedule (process-wide): 0 = load then compute (1024 threads per CTA); 1 = the next item's
 * loads issued before the current one is computed (1024 threads; default); 2 = the same with two items per
 * iteration (512 threads). Results are identical. No counterpart in the reference. */
int qe_set_silu_pipeline(int32_t on);

/* Fill `table` (65,536 uint16, 16-byte aligned device memory) with bf16(silu(g)) for every bf16 bit pattern g:
 * bf16(g / (1 + exp(-g))) exactly as the fused kernel's arithmetic rounds it (fibo/fp4.py:90). Build it once
 * per device; it is the workspace of qe_silu_mul_fp4. */
int qe_silu_table_init(uint16_t *table, void *stream);

/* SiLU(gate) * value -> NVFP4   (fibo/fp4.py:83-91, wrapper :112-116). gate, value [M, K] bf16; silu_table
 * from qe_silu_table_init on the same device. q must be 8-byte aligned. */
int qe_silu_mul_fp4(const void *gate, const void *value, const float *gs, int64_t M, int64_t K, uint8_t *q,
                    uint8_t *sf, const uint16_t *silu_table, void *stream);

/* Calibration pre-passes: *amax = max |y| over all M*K values of the y the matching quantiser would encode
 * (the bf16 result of the norm/adaLN or SiLU*mul arithmetic, as fp32). Replaces the bf16 pass the reference
 * runs on a layer's first call to set its activation scale, `x2.float().abs().amax()` in
 * pipeline/fp4.py:33-35 (fused caller: fibo/fp4.py:128-134); gs = 448*6 / (max(amax, 1e-8) * headroom).
 * amax is one device fp32, cleared on `stream` by the call; M = 0 leaves it 0. No codes or scales are
 * written. Arguments otherwise as the quantisers above. */
int qe_norm_scale_amax(const void *x, const void *w, const void *noisy, const void *clean, const uint8_t *mask,
                       const void *shift, const void *shift_clean, int64_t M, int64_t S, int64_t K,
                       int64_t mod_stride, float eps, float *amax, void *stream);
int qe_silu_mul_amax(const void *gate, const void *value, int64_t M, int64_t K, const uint16_t *silu_table,
                     float *amax, void *stream);

/* ---- paged joint attention (device) ----------------------------------------------------------
 *
 * out = softmax(scale * q K^T) V, K / V = [the first n_prefix tokens of a prefix held in pool pages; n_local own
 * tokens], in one launch that reads the prefix K/V tiles from the pool through the block table (TMA tile loads)
 * and runs both products on the tensor cores (tcgen05, fp32 accumulation). Replaces the per-step gather of the
 * matched prefix (multi_turn/pipeline/hooks.py:101-105 -> cache/paged.py:106-113) that feeds the DiT's joint
 * attention through the per-layer caches (hooks.py:81-83), and the text encoder's partial-hit attention over
 * [gathered prefix; tail] (cache/encoder.py:173-190: grouped-query heads, causal tail).
 *   q        bf16 [n_q][heads_q][128]: element (i, h, d) at q + i * q_token_stride + h * q_head_stride (bytes)
 *   k_pool / v_pool  the layer's K and V planes of the pool: rows of heads_kv x 128 bf16, row r at
 *            plane + r * heads_kv * 256; pool_rows = rows of a plane (a multiple of page_size)
 *   block_table  device int32 page ids, ceil(n_prefix / page_size) of them; prefix token t is pool row
 *            block_table[t / page_size] * page_size + t % page_size. page_size: 8, 16, 32, 64 or 128, or a
 *            multiple of 128. Pages outside the pool read as zeros and set bit 1 of *err_flag.
 *   k_local / v_local  bf16 [n_local][heads_kv][128] with the given strides (may be null when n_local == 0)
 *   causal   query i sees every prefix token and own tokens j <= i + n_local - n_q (bottom-right alignment)
 *   heads_q  a multiple of heads_kv (query head h reads K/V head h / (heads_q / heads_kv))
 *   out      bf16 [n_q][heads_q][128] (strides in bytes); lse (optional) fp32 [heads_q][n_q]: the natural log of
 *            the softmax denominator of the scaled scores.
 * Everything 16-byte aligned with 16-byte multiple strides. Every internal wait is bounded; a wait that gives up
 * sets bit 2 of *err_flag. No counterpart as one operation in the reference (gather + the model's attention). */
int qe_paged_attention(const void *q, int64_t q_token_stride, int64_t q_head_stride, int32_t n_q, int32_t heads_q,
                       const void *k_pool, const void *v_pool, int64_t pool_rows, int32_t heads_kv,
                       const int32_t *block_table, int32_t page_size, int32_t n_prefix, const void *k_local,
                       const void *v_local, int64_t local_token_stride, int64_t local_head_stride, int32_t n_local,
                       int32_t causal, float scale, void *out, int64_t out_token_stride, int64_t out_head_stride,
                       float *lse, int32_t *err_flag, void *stream);

/* qe_paged_attention with the own tokens appended to the pool in the same launch: the arguments of
 * qe_paged_attention plus append_table, device int32 page ids, ceil(n_local / page_size) of them; own token t
 * (row t of k_local / v_local) is written to pool row append_table[t / page_size] * page_size + t % page_size of
 * k_pool and v_pool (page_size and the pool planes as above; block_table may be null when n_prefix == 0).
 * Rows of the last page past own token n_local - 1 are not written. Each own K/V tile is stored by exactly one
 * of the CTAs that load it for the attention (spread over the query-tile CTAs and the query heads of its group),
 * from the same shared-memory stage, so the own K/V are read from HBM once for both. Pages outside the pool are
 * skipped and set bit 1 of *err_flag (err_flag must not be null). Needs n_q >= 1 and n_local >= 1. Replaces the
 * separate store of freshly computed prefix K/V after the forward (multi_turn/cache/prefill.py:69-72, the
 * encoder's _store, multi_turn/cache/encoder.py:131-138); no counterpart as one operation in the reference. */
int qe_paged_attention_append(const void *q, int64_t q_token_stride, int64_t q_head_stride, int32_t n_q,
                              int32_t heads_q, const void *k_pool, const void *v_pool, int64_t pool_rows,
                              int32_t heads_kv, const int32_t *block_table, int32_t page_size, int32_t n_prefix,
                              const void *k_local, const void *v_local, int64_t local_token_stride,
                              int64_t local_head_stride, int32_t n_local, int32_t causal, float scale, void *out,
                              int64_t out_token_stride, int64_t out_head_stride, float *lse,
                              const int32_t *append_table, int32_t *err_flag, void *stream);

/* Query tiles (of 128 queries) per CTA of qe_paged_attention / qe_paged_attention_append (process-wide): 0 = by
 * grid size (default: one tile per CTA when ceil(n_q / 128) x heads_q CTAs fit on the GPU's SMs at once, which
 * doubles the CTAs of small launches such as the encoder tail's; else two, whose softmax phases hide each
 * other's), 1 or 2 forced. Results are the same within the kernel's rounding. No counterpart in the reference;
 * for measurement and tests. */
int qe_set_attention_q_tiles(int32_t q_tiles);

/* ---- head-sharded pools across the GPUs of one node ------------------------------------------
 *
 * No counterpart in the reference, which keeps a prefix on one GPU and disables the pool under tensor or
 * sequence parallelism (multi_turn/pipeline/encoding.py:214-220). Rank r of an n-GPU group owns heads
 * [r H/n, (r+1) H/n) of every pooled token; every rank runs the same index decisions, so slots agree.
 */

/* CUDA IPC plumbing: qe_ipc_alloc makes a `bytes` device allocation on the current device and writes its
 * 64-byte cudaIpcMemHandle to `handle`; qe_ipc_open maps a handle made by another process into this one (peer
 * access enabled on first use); qe_ipc_close / qe_ipc_free undo them. */
int qe_ipc_alloc(int64_t bytes, void **ptr, uint8_t *handle);
int qe_ipc_free(void *ptr);
int qe_ipc_open(const uint8_t *handle, void **ptr);
int qe_ipc_close(void *ptr);

/* Append with the head scatter fused in: `src` holds n_tokens rows of all heads (n_peers * slice_bytes bytes
 * per plane row, planes as for the copies above); slice r of the row of token t is written to row slots[t] of
 * plane p of rank r's pool, whose base is peer_pools[r] (a host array of n_peers device pointers, this rank's
 * own pool at its rank; mapped peer pools from qe_ipc_open). `pool` gives the plane strides shared by every
 * rank's pool (its base is ignored); its rows are slice_bytes long. Slots outside [0, pool_rows) are skipped
 * and set *err_flag. The peer writes are visible to the other ranks after a stream-ordered barrier that follows
 * this launch on `stream` (for example an NCCL all-reduce). n_peers <= 8. */
int qe_append_scatter(const void *const *peer_pools, int32_t n_peers, qe_planes pool, int64_t pool_rows,
                      qe_planes src, int32_t n_planes, int64_t slice_bytes, const int64_t *slots, int64_t n_tokens,
                      int32_t *err_flag, void *stream);

/* ---- per-step latent ops (device) -----------------------------------------------------------
 *
 * dtype codes: 0 = fp32, 1 = bf16, 2 = fp16.
 */

/* MaskState.blend (multi_turn/pipeline/masking.py:82-89) in one launch:
 *   s = sigma.to(dtype); keep = (1 - s) x0 + s eps; out = m lat + (1 - m) keep,   m = mask.to(dtype)
 * with torch's eager rounding: each op in fp32, rounded to `dtype`. latents / out [B, N, C] contiguous in
 * `dtype`; x0 / eps [*, N, C] in `dtype` with x0_bstride / eps_bstride elements between batch entries (0 =
 * broadcast); mask [*, N, mask_channels] (1 or C) in mask_dtype with mask_bstride; sigma one value of
 * sigma_dtype on the device, or sigma_dtype 3: two fp32 values {s, 1 - s} kept unrounded (a Python-float sigma). */
int qe_mask_blend(const void *latents, const void *x0, const void *eps, const void *mask, const void *sigma,
                  void *out, int64_t B, int64_t N, int64_t C, int64_t x0_bstride, int64_t eps_bstride,
                  int64_t mask_bstride, int32_t mask_channels, int32_t dtype, int32_t mask_dtype, int32_t sigma_dtype,
                  void *stream);

/* _compose (multi_turn/pipeline/hooks.py:234-247) in one launch: out [h, w] cells = base, except the box
 * [y0, y1) x [x0, x1) taken from crop [(y1 - y0), (x1 - x0)] cells; a cell is row_bytes bytes (C latent values). */
int qe_latent_compose(const void *base, const void *crop, void *out, int64_t h, int64_t w, int64_t row_bytes,
                      int64_t x0, int64_t y0, int64_t x1, int64_t y1, void *stream);

/* stored_latents with a crop box (multi_turn/state.py:52-62): out = src cells of the box, row-major. */
int qe_latent_crop(const void *src, void *out, int64_t h, int64_t w, int64_t row_bytes, int64_t x0, int64_t y0,
                   int64_t x1, int64_t y1, void *stream);

/* ---- prefix index: radix tree + slot allocator + LRU eviction (host) -------------------------
 *
 * Restates the behaviour of SGLang's RadixCache (page_size 1 and paged) and TokenToKVPoolAllocator
 * (need_sort=True) as PagedKVPool drives them (paged.py:52-55, :72-103, :118-131). Keys are int64
 * virtual ids. Slots are pool rows 1..capacity (page mode: pages 1..capacity/page_size; page 0 is
 * padding). Node handles are opaque 64-bit values; 0 means "no node". A handle stays valid while the
 * node holds a lock (match + qe_index_lock). Not internally synchronised: callers serialise (the
 * Python pool holds an RLock, paged.py:57).
 */
typedef struct qe_index qe_index;

int qe_index_create(int64_t capacity_tokens, int32_t page_size, qe_index **out);
int qe_index_destroy(qe_index *ix);
/* RadixCache.reset + allocator.clear (paged.py:128-131). */
int qe_index_clear(qe_index *ix);
/* match_prefix (paged.py:75-80): longest cached prefix of key[0..n). Writes *out_len, the slots along
 * the path into out_slots[0..*out_len) (capacity n), and the last node (0 when *out_len == 0).
 * Touches the LRU clock of every node on the path and may split a node, as the reference does. */
int qe_index_match(qe_index *ix, const int64_t *key, int64_t n, int64_t *out_len, int64_t *out_slots,
                   uint64_t *out_node);
/* inc_lock_ref / dec_lock_ref (paged.py:79, :36). */
int qe_index_lock(qe_index *ix, uint64_t node);
int qe_index_unlock(qe_index *ix, uint64_t node);
/* insert (paged.py:99): returns the already-present prefix length in *out_present. */
int qe_index_insert(qe_index *ix, const int64_t *key, const int64_t *slots, int64_t n, int64_t *out_present);
/* evict up to num_tokens from unlocked leaves in LRU order (paged.py:93). Evicted slots return to
 * the allocator. *out_evicted = tokens evicted. */
int qe_index_evict(qe_index *ix, int64_t num_tokens, int64_t *out_evicted);
/* allocator.alloc(n) (paged.py:95): *out_ok = 1 and n slots in out_slots, or *out_ok = 0 (no change). */
int qe_index_alloc(qe_index *ix, int64_t n, int64_t *out_slots, int32_t *out_ok);
/* allocator.free(slots) (paged.py:102). */
int qe_index_free(qe_index *ix, const int64_t *slots, int64_t n);
/* Permute the free list (seeded) so later allocations come from scattered pages. No counterpart in the
 * reference, whose allocator starts sorted: it builds a fragmented pool for tests and benchmarks. */
int qe_index_shuffle_free(qe_index *ix, uint64_t seed);
/* usage (paged.py:118-126): out[0] = available slots, out[1] = evictable tokens, out[2] = protected
 * tokens, out[3] = live tree nodes (excluding the root). */
int qe_index_usage(qe_index *ix, int64_t out[4]);

/* ---- prefix keys (host) -------------------------------------------------------------------------
 * Chained 63-bit ids of multi_turn/cache/keys.py, computed natively (the reference loops over text tokens in
 * Python, keys.py:81-84, :94-96, :100-102). BLAKE2b-128 of length-prefixed parts, RFC 7693. */

/* BLAKE2b with a 16-byte digest of msg[0..len) (hashlib.blake2b(digest_size=16)). */
int qe_blake2b16(const uint8_t *msg, int64_t len, uint8_t *out16);
/* out[i] = id of text token i chained from `prev` (keys.py:57-58 applied along tokens[0..n)). */
int qe_keys_text_chain(int64_t prev, const int64_t *tokens, int64_t n, int64_t *out);
/* out[i] = id of token i of an n-token image block after `prev` with content key content[0..len)
 * (keys.py:42-54). */
int qe_keys_block_ids(int64_t prev, const uint8_t *content, int64_t len, int64_t n, int64_t *out);

#ifdef __cplusplus
}
#endif

#endif /* QEB200_H */
