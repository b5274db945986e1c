/*
 * helix_kv.h - C ABI of the B200 (sm_100a) long-context KV hot path.
 *
 * Plain C: pointers, sizes and status codes only. Every entry point is
 * asynchronous on the CUDA stream it is given (a cudaStream_t passed as
 * void*), allocates nothing, and returns HX_OK (0) when the launch was
 * accepted or a nonzero HX_ERR_* for invalid arguments. Faults found on the
 * device (a full outlier arena, an out-of-range index, a wait that ran out)
 * are OR-ed into the caller's device word `dev_err` as HX_DEV_ERR_* bits;
 * read it after synchronising.
 *
 * Pointers marked "device" are device memory. fp16 data is passed as
 * uint16_t bit patterns.
 *
 * Reference interfaces replaced (paths inside xFuzzitx/helix-lite):
 *   src/kvquant/compact_pool.py   CompactKVPool.write_kv / unpack_to_staging
 *   src/kvquant/triton_batched.py pack_/unpack_{keys_per_channel,values_per_token}_batched
 *   src/kvquant/nuq.py            quantize_nuq / dequantize_nuq (torch spec)
 *   src/quest/reference.py        compute_page_stats / page_upper_bound /
 *                                 topk_pages_with_sinks / selected_attention
 *   src/quest/triton_kernels.py   page_upper_bound_triton
 *   src/kvquant/quest_selector.py select_top_blocks_for_layer
 *   src/kvquant/compact_backend.py KVQuantCompactImpl.forward (staging + FA)
 */
#ifndef HELIX_KV_H
#define HELIX_KV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define HX_API __attribute__((visibility("default")))
#else
#define HX_API
#endif

/* host status codes */
#define HX_OK              0
#define HX_ERR_ARG         1   /* shape, pointer or size rejected */
#define HX_ERR_UNSUPPORTED 2   /* valid request this build has no kernel for */
#define HX_ERR_LAUNCH      3   /* the CUDA launch itself failed */
#define HX_ERR_SCRATCH_LIMIT 4 /* request exceeds a fixed scratch array's size */

/* device error bits, OR-ed into *dev_err */
#define HX_DEV_ERR_ARENA_FULL 0x1u  /* outlier arena exhausted: entries dropped */
#define HX_DEV_ERR_BOUNDS     0x2u  /* an index (page, slot, level) out of range */
#define HX_DEV_ERR_TIMEOUT    0x4u  /* a bounded wait on a bulk copy ran out */
#define HX_DEV_ERR_SELECT     0x8u  /* selection could not isolate a threshold */

/* Calibrated nuq scales of one layer (src/kvquant/scales.py:14-70). */
typedef struct hx_layer_scales {
  const uint16_t* k_poles;   /* device fp16 (H, D, levels_k): per channel   */
  const uint16_t* k_upper;   /* device fp16 (H, D)                          */
  const uint16_t* k_lower;   /* device fp16 (H, D)                          */
  const uint16_t* v_poles;   /* device fp16 (H, t_cal, levels_v): per token */
  const uint16_t* v_upper;   /* device fp16 (H, t_cal)                      */
  const uint16_t* v_lower;   /* device fp16 (H, t_cal)                      */
  int32_t levels_k;          /* 2..16 */
  int32_t levels_v;          /* 2..16 */
  int32_t t_cal;             /* V positions >= t_cal use row t_cal - 1     */
  int32_t reserved;
  /* Code thresholds written by hx_scales_prepare (device, 16-byte aligned),
   * or NULL: hx_pack_append then takes its level-scan kernel.            */
  const uint32_t* k_thresh;  /* (H, D/2, 16) fp16 pairs                   */
  const uint32_t* v_thresh;  /* (H, t_cal, 16) fp16 duplicated in both halves */
} hx_layer_scales;

/*
 * One layer of the compact paged pool. Codes of a (head, page) live in one
 * contiguous segment: K rows (S x D*bits_k/8 bytes) then V rows
 * (S x D*bits_v/8). A row packs channel codes little-end first: nuq4 byte i
 * = c[2i] | c[2i+1] << 4, nuq2 byte i = c[4i] | c[4i+1] << 2 | c[4i+2] << 4
 * | c[4i+3] << 6. Outliers are sparse: every (head, page, K|V) has a
 * directory record {offset, capacity, count, rows} into the layer's arena
 * of 32-bit entries (bits 0-15 fp16 value, 16-23 channel, 24-28 slot).
 */
typedef struct hx_pool_layer {
  uint8_t*  codes;         /* device (H, NB, seg_bytes)                     */
  uint16_t* stats;         /* device fp16 (H, NB, 2, D): K min, K max       */
  uint32_t* dir;           /* device (H, NB, 2, 4)                          */
  uint32_t* arena;         /* device (arena_capacity,) outlier entries      */
  uint32_t* arena_top;     /* device, one counter: entries handed out       */
  int64_t   arena_capacity;
  int32_t   num_blocks;    /* NB */
  int32_t   block_size;    /* S, tokens per page, 1..32 */
  int32_t   num_kv_heads;  /* H */
  int32_t   head_size;     /* D, multiple of 8, <= 256 */
  int32_t   bits_k;        /* 2 or 4 */
  int32_t   bits_v;        /* 2 or 4 */
} hx_pool_layer;

/* ---- pool maintenance ------------------------------------------------- */

/* Set every page of the layer to empty: stats to +inf / -inf, directory
 * records to zero, arena counter to zero. Replaces the allocation-time
 * initialisation of CompactKVPool.__post_init__ (compact_pool.py:418-444). */
HX_API int hx_pool_init(void* stream, const hx_pool_layer* pool);

/* Empty the listed pages (stats and outlier lists) so they can be reused. */
HX_API int hx_pool_reset_pages(void* stream, const hx_pool_layer* pool,
                               const int32_t* pages, int32_t n, uint32_t* dev_err);

/* ---- pack on write (Kernel A) ----------------------------------------- */

/* Quantise, bit-pack and append T tokens of one layer: K per channel, V per
 * token at position min(abs_positions[t], t_cal - 1); outliers (outside the
 * band) appended to the page lists; K page stats updated with the running
 * min / max of the reconstructed K. slot_mapping[t] < 0 skips the token.
 * Tokens may come in any slot order: a page whose slots arrive as several
 * runs in one call (a run = input tokens filling consecutive slots) is
 * updated one run at a time under a per-page lock, so no outlier entry or
 * stat is lost. A slot written twice in one call keeps one of its tokens,
 * unspecified which (the reference's parallel kernels race the same way).
 * The order of entries inside a page's outlier list is unspecified.
 * With 16-token pages, head_size 128 and the scales' thresholds
 * (hx_scales_prepare) a bandwidth kernel runs; otherwise a level-scan kernel.
 * Both give the same bytes. Replaces CompactKVPool.write_kv
 * (compact_pool.py:447-489). */
HX_API int hx_pack_append(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                          const uint16_t* key, const uint16_t* value,      /* (T, H, D) fp16 */
                          const int64_t* slot_mapping, const int64_t* abs_positions,
                          int32_t T, uint32_t* dev_err);

/* Code thresholds of a layer's codebooks for the bandwidth path of
 * hx_pack_append (16-token pages, head_size 128). For a codebook row with
 * poles p_0 < ... < p_{L-1} (finite), entry l < L-1 is the largest fp16 x for
 * which the reference's scan does not prefer level l+1 over level l
 * (|x - p_{l+1}| < |x - p_l| in fp32, compact_pool.py:258-268), entries up to
 * 14 are +inf, and entry 15 is a bound X below which the count of thresholds
 * under x is the scan's code (X = p_0 + 2^22 * smallest gap, rounded down).
 * Rows whose poles are not finite and strictly increasing get X = -inf; the
 * pack kernel runs the scan itself for every element with !(x < X). Layout:
 * k_thresh (H, D/2, 16) u32, half e of entry l of pair P from channel 2P+e;
 * v_thresh (H, t_cal, 16) u32, each entry's fp16 in both halves. Computed once
 * per scales (no reference counterpart: the reference scans every level). */
HX_API int hx_scales_prepare(void* stream, const hx_layer_scales* sc, int32_t H, int32_t D,
                             uint32_t* k_thresh, uint32_t* v_thresh);

/* Dequantise whole pages to fp16 staging (NK, S, H, D) for K and V.
 * Replaces CompactKVPool.unpack_to_staging (compact_pool.py:492-537). */
HX_API int hx_unpack_pages(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                           const int64_t* block_ids, const int64_t* first_pos, int32_t nk,
                           uint16_t* staging_k, uint16_t* staging_v, uint32_t* dev_err);

/* ---- calibration statistics ------------------------------------------ */

/* One group of samples per row: sorted (rows, n) float32, each row ascending.
 * lower / upper (rows) receive numpy.quantile(row, q_low) / (row, q_high)
 * (method "linear", numpy's own float32 value for float32 samples), centers
 * (rows, k) the sorted centres of a 1-D k-means of the samples with lower <=
 * x <= upper: the exact optimum (dynamic programming) over the samples, or
 * over 4096 of them stratified by rank, equal values merged, then at most
 * max_iter Lloyd steps over every band sample (a sample on a midpoint joins
 * the lower centre); fewer samples than k: the samples and zeros, sorted.
 * iters_done (rows, optional): the Lloyd steps run. scratch:
 * hx_calib_scratch_bytes(rows, n) bytes. k <= 16. Replaces the statistics
 * loop of src/kvquant/calibration.py:127-188 (there: np.quantile and
 * sklearn's KMeans on a random subsample of 5,000). */
HX_API int64_t hx_calib_scratch_bytes(int32_t rows, int64_t n);
HX_API int hx_calib_rows(void* stream, const float* sorted, int32_t rows, int64_t n, double q_low,
                         double q_high, int32_t k, int32_t max_iter, float* lower, float* upper,
                         float* centers, double* scratch, int32_t* iters_done);

/* ---- dense quantisation (the batched Triton API) ---------------------- */

/* mode 0: K, poles (H, D, L), thresholds (H, D); mode 1: V, poles (H, T, L),
 * thresholds (H, T). values (T, H, D) fp16 -> codes u8, outlier values fp16
 * (0 elsewhere), outlier mask u8. Replaces pack_keys_per_channel_batched /
 * pack_values_per_token_batched (triton_batched.py:125-148, :275-303). */
HX_API int hx_nuq_pack_dense(void* stream, int32_t mode, const uint16_t* values,
                             const uint16_t* poles, const uint16_t* upper, const uint16_t* lower,
                             int32_t T, int32_t H, int32_t D, int32_t L,
                             uint8_t* codes, uint16_t* outv, uint8_t* outm);

/* Inverse of hx_nuq_pack_dense (triton_batched.py:151-171, :306-326). */
HX_API int hx_nuq_unpack_dense(void* stream, int32_t mode, const uint8_t* codes,
                               const uint16_t* outv, const uint8_t* outm, const uint16_t* poles,
                               int32_t T, int32_t H, int32_t D, int32_t L, uint16_t* out);

/* Flat quantise_nuq: n elements, poles (n, L) row-major, values and
 * thresholds of one dtype (0 = fp32, 1 = fp16). Writes the reconstruction
 * (same dtype) and the outlier mask (u8). Differences are taken in the
 * input dtype as the torch spec does (nuq.py:22-38). Mask: the band test
 * (nuq.py:72); with cap > 0 only the cap largest |normalised deviation|
 * entries of each row of `row` elements stay (nuq.py:74-87, ties to the
 * lower index); elements with (i / seq_stride) % seq_size < first_few are
 * forced outliers (nuq.py:89-92). scratch_mask: n bytes, needed when cap > 0. */
HX_API int hx_nuq_quantize_flat(void* stream, int32_t dtype, const void* values, const void* poles,
                                const void* upper, const void* lower, int64_t n, int32_t L,
                                int32_t cap, int64_t row, int64_t seq_stride, int64_t seq_size,
                                int32_t first_few, void* recon, uint8_t* mask, uint8_t* scratch_mask);

/* dequantize_nuq: out[i] = mask[i] ? outliers[i] : poles[i*L + codes[i]] in
 * the dtype of outliers (nuq.py:135-156). codes are int64. */
HX_API int hx_nuq_dequantize_flat(void* stream, int32_t dtype, const int64_t* codes,
                                  const void* outliers, const uint8_t* mask, const void* poles,
                                  int64_t n, int32_t L, void* out, uint32_t* dev_err);

/* ---- Quest (Kernel B) -------------------------------------------------- */

/* compute_page_stats: (P, S, H, D) -> min, max (P, H, D), dtype 0 fp32 / 1 fp16
 * (quest/reference.py:38-56). */
HX_API int hx_page_stats(void* stream, int32_t dtype, const void* k_pages,
                         int32_t P, int32_t S, int32_t H, int32_t D, void* kmin, void* kmax);

/*
 * Page scores: for batch b, KV head h and logical page j < ceil(seq_lens[b]/S)
 *   score = sum_d Qp[d] * kmax[d] + Qn[d] * kmin[d]
 * with Qp / Qn the group terms of the `group` query heads of h (gqa_mode 0:
 * sum of per-head clamps, 1: clamp of the fp16-rounded mean). Arithmetic
 * order is pinned (32 lanes x ceil(D/32) channels, butterfly); products and
 * sums are rounded to fp32 separately. Stats rows are addressed as
 *   kmin + phys*page_stride + h*head_stride (same for kmax), phys =
 *   block_table ? block_table[b*bt_stride + j] : j,
 * with dtype 0 fp32 / 1 fp16. q is (B, H*group, D) fp16. Scores (B, H,
 * max_pages) fp32. If hist != NULL, each non-sink page is counted into
 * hist (B*H, 2, 4096) [level 1; level 2 is used by hx_quest_threshold] at bin
 * clamp((key - anchor) / 2^16 + 2048, 0, 4095), key = the order key of its
 * score and anchor = that of page sinks (the first non-sink page). hist must
 * be zero on entry (hx_quest_threshold leaves it zero again).
 * Replaces page_upper_bound / page_upper_bound_triton (reference.py:59-93,
 * triton_kernels.py:26-91) and the GQA contraction (compact_backend.py:231).
 */
HX_API int hx_quest_scores(void* stream, const uint16_t* q, int32_t B, int32_t H, int32_t group,
                           int32_t D, int32_t gqa_mode, int32_t stats_dtype,
                           const void* kmin, const void* kmax, int64_t page_stride, int64_t head_stride,
                           const int32_t* block_table, int32_t bt_stride,
                           const int32_t* seq_lens, int32_t page_size, int32_t max_pages,
                           int32_t sink_pages, float* scores, uint32_t* hist);

/*
 * Exact top-K threshold per (b, h): k_b = frac_den > 0 ? n_b*frac_num/frac_den
 * : k_fixed pages, k_eff = min(k_b, n_b - sinks), sinks = min(sink_pages, n_b).
 * Page j >= sinks is selected iff key64(j) >= thresh[b*H+h], key64 =
 * order_key(score) << 32 | ~j; thresh = ~0 when k_eff == 0.
 * Scratch: hist as above (filled by hx_quest_scores when hist_ready != 0,
 * else counted here from `scores`); cand (B*H*max_pages) u64; counters
 * (B*H*2) u32; all zero on entry and left zero. Rows of up to 2048 pages
 * (max_pages) are resolved by one CTA each; longer ones by one CTA per 1024
 * pages, the last of them finishing the row. Replaces the torch.topk of
 * topk_pages_with_sinks (reference.py:96-133) with a deterministic order.
 */
HX_API int hx_quest_threshold(void* stream, const float* scores, int32_t B, int32_t H,
                              const int32_t* seq_lens, int32_t page_size, int32_t max_pages,
                              int32_t sink_pages, int32_t k_fixed, int32_t frac_num, int32_t frac_den,
                              int32_t hist_ready, uint32_t* hist, uint64_t* cand, uint32_t* counters,
                              uint64_t* thresh, uint32_t* dev_err);

/* hx_quest_threshold plus the per-slice counts the decode balances its splits
 * over (HX_SEL_SLICES): the non-sink pages [sinks, n_b) of each (b, h) are
 * cut into C = hx_quest_slices(max_pages) slices of ceil((n_b - sinks) / C)
 * pages, and slice_off (B*H, C + 1) int32 receives the exclusive prefix of
 * the slices' selected counts (slice_off[C] = selected non-sink pages). No
 * reference counterpart (the reference hands FlashAttention a page list). */
HX_API int32_t hx_quest_slices(int32_t max_pages);
HX_API int hx_quest_threshold_slices(void* stream, const float* scores, int32_t B, int32_t H,
                                     const int32_t* seq_lens, int32_t page_size, int32_t max_pages,
                                     int32_t sink_pages, int32_t k_fixed, int32_t frac_num, int32_t frac_den,
                                     int32_t hist_ready, uint32_t* hist, uint64_t* cand, uint32_t* counters,
                                     uint64_t* thresh, int32_t* slice_off, uint32_t* dev_err);

/* Selected logical pages, ascending, per (b, h): out (B, H, max_out) int32
 * and counts (B, H). union_heads != 0 writes the union over heads instead:
 * out (B, max_out), counts (B). */
HX_API int hx_quest_compact(void* stream, const float* scores, const uint64_t* thresh,
                            int32_t B, int32_t H, const int32_t* seq_lens, int32_t page_size,
                            int32_t max_pages, int32_t sink_pages, int32_t union_heads,
                            int32_t max_out, int32_t* out, int32_t* counts);

/* The same per-(b, h) ascending lists as hx_quest_compact without the union,
 * written by ceil(max_pages / HX_LIST_CHUNK) CTAs per (b, h) in two passes so
 * that long sequences are compacted at full bandwidth; this is the list the
 * decode balances its splits over (HX_SEL_LIST). chunk_counts: scratch of
 * B*H*ceil(max_pages / HX_LIST_CHUNK) int32 (no initial value; may be NULL
 * when max_pages <= HX_LIST_CHUNK). No reference counterpart: the reference
 * selects with torch.topk and hands FlashAttention a page list
 * (src/kvquant/quest_selector.py:38-97). */
#define HX_LIST_CHUNK 2048
HX_API int hx_quest_lists(void* stream, const float* scores, const uint64_t* thresh,
                          int32_t B, int32_t H, const int32_t* seq_lens, int32_t page_size,
                          int32_t max_pages, int32_t sink_pages, int32_t max_out,
                          int32_t* out, int32_t* counts, int32_t* chunk_counts);

/* Global top-K over split-KV shards. thresh_global (B*H) holds thresholds
 * that hx_quest_threshold computed over the whole sequence's scores (every
 * shard's pages, in global page order); this shard's pages are global pages
 * page_begin .. page_begin + max_pages - 1 and its scores (B, H, max_pages)
 * are indexed locally. Writes the shard's own thresholds (thresh, B*H), which
 * select with local indices exactly the global selection's pages in this
 * shard (score ties broken by the global index), and the decode's slice
 * counts (slice_off (B*H, hx_quest_slices(max_pages) + 1), as
 * hx_quest_threshold_slices writes them). sink_pages: the global sinks that
 * fall on this shard, max(0, min(sinks - page_begin, max_pages)). One kernel. The
 * reference selects on one GPU only (src/kvquant/quest_selector.py:70-83);
 * this keeps that selection bit for bit when the pages are split. */
HX_API int hx_quest_localize(void* stream, const uint64_t* thresh_global, const float* scores,
                             int32_t B, int32_t H, const int32_t* seq_lens, int32_t page_size,
                             int32_t max_pages, int32_t sink_pages, int32_t page_begin,
                             uint64_t* thresh, int32_t* slice_off);

/* ---- fused-dequant decode attention (Kernel C) ------------------------ */

#define HX_SEL_DENSE     0   /* every page of the sequence                  */
#define HX_SEL_THRESHOLD 1   /* sinks + pages with key64 >= thresh          */
#define HX_SEL_LIST      2   /* explicit per-(b, h) logical page lists      */
#define HX_SEL_SLICES    3   /* sinks + key64 >= thresh, ranks located by slice_off */
#define HX_SEL_MODE_MASK 0xFF
/* OR-ed into sel_mode: the V scale row of page j's slot t is
 * min((page_begin + block_table[j]) * 16 + t, t_cal - 1), i.e. the token's
 * physical slot, the rule of the reference pool, which packs V with
 * abs_positions = slot_mapping and unpacks block b from position b * 16
 * (compact_backend.py:157-167, compact_pool.py:370-372, quest_selector.py:89).
 * Without it the row is that of the logical position (page_begin + j) * 16 + t. */
#define HX_VPOS_PHYSICAL 0x100
/* OR-ed into sel_mode: QK and PV in fp32 FFMA on the CUDA cores instead of
 * the tensor cores (mma.sync), with the same pipeline, dequant and softmax.
 * Slower; kept as the comparison the design choice rests on. */
#define HX_DECODE_CUDA_CORES 0x200

/* Scratch bytes hx_decode_attn needs for B sequences, H heads, n_splits. */
HX_API int64_t hx_decode_scratch_bytes(int32_t B, int32_t H, int32_t n_splits);

/*
 * One decode token per sequence over the compact pool. q (B, H*group, D) fp16
 * (group <= 8, D = 128, page_size = 16). Logical page j of sequence b is pool
 * page block_table[b*bt_stride + j] and starts at absolute position
 * (page_begin + j) * 16 (V tail clamp; (page_begin + block_table[...]) * 16
 * with HX_VPOS_PHYSICAL in sel_mode); tokens >= seq_lens[b] are masked.
 * Selection: HX_SEL_DENSE; HX_SEL_THRESHOLD with scores / thresh from
 * hx_quest_scores / hx_quest_threshold; HX_SEL_LIST with lists (B, H,
 * list_stride) and list_counts (B, H); HX_SEL_SLICES with scores / thresh
 * and slice_off from hx_quest_threshold_slices passed as lists, list_stride
 * = C + 1 (list_counts unused): the splits balance over the selected pages
 * as with lists, and each CTA finds its pages by scanning its slices. The sequence is split n_splits ways
 * per (b, h); the last CTA of each (b, h) merges the splits. Writes o (B,
 * H*group, D) fp32 normalised, lse (B, H*group) natural log (-inf for an
 * empty selection), and out16 (same shape, fp16) when non-NULL. scratch:
 * hx_decode_scratch_bytes bytes: a 64 KB region of split counters (B*H <=
 * 16384) that must be zero the first time and is left zero, then the split
 * partials.
 * Replaces unpack_to_staging + flash_attn_varlen_func in
 * KVQuantCompactImpl.forward (compact_backend.py:233-299).
 */
HX_API int hx_decode_attn(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                          const uint16_t* q, int32_t B, int32_t group, float softmax_scale,
                          const int32_t* block_table, int32_t bt_stride, const int32_t* seq_lens,
                          int32_t page_begin, int32_t max_pages, int32_t sel_mode,
                          const float* scores, const uint64_t* thresh, int32_t sink_pages,
                          const int32_t* lists, int32_t list_stride, const int32_t* list_counts,
                          int32_t n_splits, void* scratch, float* o, float* lse, uint16_t* out16,
                          uint32_t* dev_err);

/*
 * Quest selection and decode in one kernel, for rows of at most 16384 pages
 * (split-KV shards, batched sequences): hx_decode_attn in HX_SEL_SLICES mode
 * whose CTAs each compute their row's exact threshold and slice counts from
 * `scores` and the level-1 histogram `hist` that hx_quest_scores wrote (the
 * work of hx_quest_threshold_slices, same selection: k_b = frac_den > 0 ?
 * n_b*frac_num/frac_den : k_fixed, sinks forced, ties to the lower page), so
 * the threshold kernel and its chain of global round trips go away. The
 * row's last CTA leaves its histogram zero for the next scoring. flags:
 * HX_VPOS_PHYSICAL (HX_DECODE_CUDA_CORES: HX_ERR_UNSUPPORTED, the CUDA-core
 * comparison runs with the threshold kernel). thresh_out (B*H) and slice_out
 * (B*H, hx_quest_slices(max_pages) + 1), when non-NULL, receive the row's
 * threshold and slice offsets. max_pages > 16384: HX_ERR_UNSUPPORTED.
 * Replaces select_top_blocks_for_layer + unpack_to_staging + FlashAttention
 * in KVQuantCompactImpl.forward (compact_backend.py:225-299).
 */
HX_API int hx_decode_attn_select(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                                 const uint16_t* q, int32_t B, int32_t group, float softmax_scale,
                                 const int32_t* block_table, int32_t bt_stride, const int32_t* seq_lens,
                                 int32_t page_begin, int32_t max_pages, int32_t flags,
                                 const float* scores, uint32_t* hist, int32_t sink_pages,
                                 int32_t k_fixed, int32_t frac_num, int32_t frac_den, int32_t n_splits,
                                 void* scratch, float* o, float* lse, uint16_t* out16,
                                 uint64_t* thresh_out, int32_t* slice_out, uint32_t* dev_err);

/*
 * Chunked-prefill attention over the compact pool. q (Tq, H*group, D) fp16
 * holds B sequences' query tokens back to back: sequence b's are rows
 * q_start[b] .. q_start[b+1] - 1 (q_start (B+1) int32, device), the last
 * q_len_b tokens of its seq_lens[b] tokens, already packed into the pool
 * (hx_pack_append). Query token i of sequence b (position seq_lens[b] -
 * q_len_b + i) attends causally to positions 0 .. its own, read and
 * dequantised from the pages block_table[b*bt_stride + j]; V rows by the
 * logical position, or the physical one with HX_VPOS_PHYSICAL in flags.
 * max_q_len bounds q_len_b (grid size). Writes out16 (Tq, H*group, D) fp16
 * and, when non-NULL, out32 (the same in fp32) and lse (Tq, H*group) fp32
 * natural log. D = 128, page
 * size 16. No reference counterpart: the reference's prefill reads vLLM's
 * fp16 cache, which it keeps beside the compact pool for that reason
 * (src/kvquant/compact_backend.py:12-15).
 */
HX_API int hx_prefill_attn(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                           const uint16_t* q, const int32_t* q_start, int32_t B, int32_t group,
                           float softmax_scale, const int32_t* block_table, int32_t bt_stride,
                           const int32_t* seq_lens, int32_t max_q_len, int32_t flags,
                           uint16_t* out16, float* out32, float* lse, uint32_t* dev_err);

/*
 * hx_decode_attn without a caller scratch buffer: no counterpart in the
 * reference. Its scratch is a fixed array inside this library (64 KB of split
 * counters + 1024 split partials, about 4.3 MB per GPU that loads the
 * library, held until exit), so the call allocates nothing and needs nothing
 * allocated for it. Meant for callers that cannot call cudaMalloc: a serving
 * engine that has reserved nearly all HBM for its own KV pool and forbids
 * allocation during decode, or a foreign-language binding that holds raw
 * device pointers but no allocator. B * H * n_splits must be <= 1024, else
 * HX_ERR_SCRATCH_LIMIT and nothing runs. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture. Each call clears the
 * counters it needs (a memset on `stream`) because the array keeps the last
 * call's contents. All calls share the one array: calls that overlap on the
 * GPU (other streams, other threads) race and must be serialised by the caller.
 */
HX_API int hx_decode_attn_noalloc(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                                  const uint16_t* q, int32_t B, int32_t group, float softmax_scale,
                                  const int32_t* block_table, int32_t bt_stride, const int32_t* seq_lens,
                                  int32_t page_begin, int32_t max_pages, int32_t sel_mode,
                                  const float* scores, const uint64_t* thresh, int32_t sink_pages,
                                  const int32_t* lists, int32_t list_stride, const int32_t* list_counts,
                                  int32_t n_splits, float* o, float* lse, uint16_t* out16,
                                  uint32_t* dev_err);

/* Merge R shards' (o, lse): o_parts (R, N, D) fp32, lse_parts (R, N) ->
 * o (N, D) fp32, lse (N), out16 (N, D) fp16 if non-NULL. Used after the
 * all-gather of split-KV partials across GPUs. */
HX_API int hx_merge_partials(void* stream, const float* o_parts, const float* lse_parts,
                             int32_t R, int32_t N, int32_t D, float* o, float* lse, uint16_t* out16);

/* The same merge over the buffer an all-gather of per-rank rows
 * [o (N x D) | lse (N)] fills: gathered (R, N * (D + 1)) fp32, read in place
 * (the exchange of the split-KV step sends one such row per rank). */
HX_API int hx_merge_gathered(void* stream, const float* gathered, int32_t R, int32_t N, int32_t D, float* o,
                             float* lse, uint16_t* out16);

/*
 * The split-KV exchange and merge of one layer over peer memory (no NCCL):
 * peer_rows / peer_flags are device arrays of R device pointers (this
 * process's view of every rank's symmetric buffers, e.g. from CUDA IPC):
 * rank r's rows (slots, N * (D + 1)) fp32, row `slot` = [o (N x D) | lse (N)]
 * written by its decode, and its flags (slots, R) uint32, zero at start.
 * The kernel sets flag (slot, rank) on every rank, waits until all R flags
 * (slot, *) of its own array are set (at most max_polls polls, then
 * HX_DEV_ERR_TIMEOUT and nothing merged), merges the R rows read from the
 * peers into o (N, D), lse (N) (and out16 if non-NULL), then clears its own
 * (slot, *) flags. Each rank calls it once per slot per step, slots in the
 * same order on every rank. R <= 32, N <= 64. No reference counterpart (the
 * reference decodes on one GPU; this replaces an all-gather plus
 * hx_merge_partials).
 */
HX_API int hx_exchange_merge(void* stream, const uint64_t* peer_rows, const uint64_t* peer_flags, int32_t R,
                             int32_t rank, int32_t slot, int32_t N, int32_t D, float* o, float* lse,
                             uint16_t* out16, uint32_t max_polls, uint32_t* dev_err);

/*
 * selected_attention on dense pages (quest/reference.py:136-168), fp32
 * arithmetic, grouped-query: q (Hq, D), K / V pages (P, S, H, D) (dtype 0
 * fp32 / 1 fp16), page_idx (k, H) int64 (column h: pages of KV head h).
 * Query head i reads KV head i / (Hq / H). out (Hq, D) in the dtype of q.
 */
HX_API int hx_selected_attention(void* stream, int32_t dtype, const void* q, const void* k_pages,
                                 const void* v_pages, const int64_t* page_idx, int32_t k,
                                 int32_t P, int32_t S, int32_t H, int32_t Hq, int32_t D,
                                 float softmax_scale, void* out);

/* Library version and build arch string ("sm_100a"). */
HX_API const char* hx_version(void);

#ifdef __cplusplus
}
#endif
#endif /* HELIX_KV_H */
