/*
 * musc_b200.h -- C ABI of the B200 (sm_100a) MuSc scoring library.
 *
 * The library replaces the reference's scoring hot path: LNAMD neighbourhood
 * aggregation, MSM mutual scoring with the interval average, the score
 * reduction, and the ViT block softmax attention.  Each entry point names the
 * reference interface it replaces (paths relative to the MuSc checkout).
 *
 * Conventions (all entry points):
 *   - Return an int status: MUSC_B200_OK (0) or one of the error codes below.
 *     musc_b200_last_error() returns a thread-local message for the last
 *     failure on the calling thread.  No exception crosses the ABI.
 *   - Every tensor argument is caller-owned device memory of the current
 *     device; the library never allocates or frees it.  Scratch memory comes
 *     from a caller-provided workspace sized by the matching *_bytes query.
 *   - Work is enqueued on `stream` (a cudaStream_t; 0 = legacy default
 *     stream) and is asynchronous to the host, like the reference's launches
 *     on torch's current stream (models/modules/_cuda_runtime.py:95-100).
 *   - Entry points are stateless and reentrant per stream.
 *   - The device must be sm_100 (B200); anything else returns
 *     MUSC_B200_ERR_DEVICE.  There is no CPU fallback.
 */
#ifndef MUSC_B200_H
#define MUSC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* musc_b200_stream; /* same type as cudaStream_t */

enum musc_b200_status {
  MUSC_B200_OK = 0,
  MUSC_B200_ERR_INVALID = 1,   /* shape / dtype / rank contract: the reference raises ValueError
                                  (models/modules/_MSM_gpu.py:702-711, _backend.py:6-7) */
  MUSC_B200_ERR_CUDA = 2,      /* CUDA runtime or driver failure: the reference raises RuntimeError
                                  (models/modules/_cuda_runtime.py:47-55) */
  MUSC_B200_ERR_DEVICE = 3,    /* current device is not sm_100 */
  MUSC_B200_ERR_WORKSPACE = 4, /* workspace smaller than the *_bytes query */
  MUSC_B200_ERR_TIMEOUT = 5    /* a device-side bounded wait expired (reported by
                                  musc_b200_take_device_error) */
};

enum musc_b200_dtype { MUSC_B200_F32 = 0, MUSC_B200_F16 = 1, MUSC_B200_BF16 = 2 };

/* ABI version of this header (bumped on any signature change): 3. */
int musc_b200_abi_version(void);

/* Thread-local message of the last failing call on this thread ("" if none). */
const char* musc_b200_last_error(void);

/* Reads and clears the device-side error word of the current device
 * (MUSC_B200_OK or MUSC_B200_ERR_TIMEOUT).  Synchronises the device.
 *
 * The pipelined kernels (nearest GEMM, attention, staged LNAMD stencil) never
 * hang: a bounded wait that expires sets this word and the kernel returns
 * early, leaving its output incomplete.  While the word is set, the interval
 * average (musc_b200_trimmed_mean, musc_b200_msm, musc_b200_score_pool), the
 * score maps and RsCIN write NaN instead of scores, so an incomplete result is
 * never a plausible number.  Callers of musc_b200_score_pool, musc_b200_msm,
 * musc_b200_nearest_pool, musc_b200_nearest and musc_b200_attention_fwd call
 * this once, where they synchronise anyway, before trusting the outputs. */
int musc_b200_take_device_error(int* code);

/* Self-test of the device-side bounded wait that every pipelined kernel here
 * uses (no counterpart in the reference, whose kernels have no waits): a
 * single thread waits on an mbarrier for at most limit_ns nanoseconds.  With
 * arrive == 0 nothing arrives, the wait expires and the device error word
 * becomes MUSC_B200_ERR_TIMEOUT (read it with musc_b200_take_device_error);
 * with arrive != 0 it completes at once.  The context stays usable either way. */
int musc_b200_selftest_wait(long long limit_ns, int arrive, musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * LNAMD (models/modules/_LNAMD.py)
 * Replaces LNAMD._embed (models/modules/_LNAMD.py:72-129), its direct-pool
 * form aggregate_features (models/modules/_encoder_gpu.py:14-42) with the
 * radius cache (models/modules/_aggregation_cache.py:15-58), and the
 * L2 normalisation of models/musc.py:238.
 *
 * tokens: [n_images][tokens_per_image][channels] of `dtype`; token 0 is the
 *         CLS token and is skipped; tokens_per_image - 1 = side*side.
 * For each requested radius r in {1, 3, 5}: LayerNorm over the whole
 * (channels, side, side) image (weight 1, bias 0, eps 1e-5, biased variance),
 * then the zero-padded r x r mean with divisor r^2, then (l2_normalize != 0)
 * division by the per-patch L2 norm over channels.
 * out[i] receives radius radii[i] at
 *     out[i][image * out_image_stride + patch * out_patch_stride + channel]
 * (float32), so the reference's (B, P, layers, C) stack and a contiguous
 * (N, P, C) scoring bank are both expressible.  channels % 4 == 0,
 * channels <= 2048, strides % 4 == 0.
 * ---------------------------------------------------------------------- */
size_t musc_b200_lnamd_workspace_bytes(int n_images);

int musc_b200_lnamd(const void* tokens, int dtype, int n_images, int tokens_per_image,
                    int channels, int n_radii, const int* radii, float* const* out,
                    long long out_image_stride, long long out_patch_stride, int l2_normalize,
                    void* workspace, size_t workspace_bytes, musc_b200_stream stream);

/* musc_b200_lnamd without a workspace argument, for callers that cannot
 * allocate device memory: hosts that hand the library only the tensors they
 * already own -- a plug-in inside another runtime's memory arena, a service
 * that forbids device allocation after start-up, or a foreign-language caller
 * with no CUDA allocator of its own.  This entry point has no counterpart in
 * the reference.  Its scratch (the per-image LayerNorm sums) is a 256 KB
 * array in the library's static device memory, so:
 *   - at most 2048 images per call; larger n_images returns
 *     MUSC_B200_ERR_INVALID before any work is enqueued;
 *   - every call looks the array's address up for the current device
 *     (cudaGetSymbolAddress, a host-side query that allocates nothing; the
 *     first one on a device may load the library's module there) -- make the
 *     first call on a device before any stream capture on it;
 *   - every call shares the one array: nothing in it needs to start at zero
 *     (each call overwrites the slots it reads before reading them), but calls
 *     that overlap on the GPU -- concurrent streams, or other host threads --
 *     race on it; serialise them.
 * Inputs, outputs and results are exactly those of musc_b200_lnamd.  No
 * cudaMalloc, cudaFree or allocating library routine is called. */
int musc_b200_lnamd_noalloc(const void* tokens, int dtype, int n_images, int tokens_per_image,
                            int channels, int n_radii, const int* radii, float* const* out,
                            long long out_image_stride, long long out_patch_stride, int l2_normalize,
                            musc_b200_stream stream);

/* Super-fast profile: r = 3 LNAMD on the side x side grid, then
 * adaptive_avg_pool2d to out_side x out_side (fp32), then optional L2
 * normalisation.  Replaces SuperFastAggregation.__call__
 * (models/modules/_super_fast.py:17-27) followed by models/musc.py:238. */
int musc_b200_lnamd_super_fast(const void* tokens, int dtype, int n_images,
                               int tokens_per_image, int channels, int out_side, float* out,
                               long long out_image_stride, long long out_patch_stride,
                               int l2_normalize, void* workspace, size_t workspace_bytes,
                               musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * MSM mutual scoring (models/modules/_MSM.py, models/modules/_MSM_gpu.py)
 * Replaces models/modules/_MSM.py:10-59 (original) and
 * models/modules/_MSM_gpu.py:701-830 (the reference GPU driver).
 *
 * A "bank" is the tensor-core operand form of a block of feature rows
 * z[rows][channels] (fp32): each row scaled by a power of two and split into
 * fp16 hi + lo halves, plus fp32 squared norms and the inverse scales.
 * ---------------------------------------------------------------------- */
size_t musc_b200_bank_bytes(long long rows, int channels);

/* Byte offsets of the bank's five planes (hi, lo, |z|^2, 2^-k, residual norm
 * |lo| 2^-k) for `rows` rows: plane_offsets[0..4].  The hi/lo planes hold
 * rows * channels fp16 each and the vectors rows fp32, row-contiguous, so the
 * banks of consecutive row blocks (one per rank) are gathered plane by plane
 * into the bank of the concatenated rows. */
int musc_b200_bank_layout(long long rows, int channels, size_t* plane_offsets);

/* z: [rows][channels] fp32, channels % 8 == 0.  bank: >= bank_bytes.  The bank
 * holds z itself (no centring). */
int musc_b200_prep_bank(const float* z, long long rows, int channels, void* bank,
                        size_t bank_bytes, musc_b200_stream stream);

/* Centring statistics of z [rows][channels] fp32 (rows >= 0) into
 * stats[channels + 1] fp64: the column sums, then the smallest squared row norm
 * (+inf for no rows), in a fixed order (the same rows give the same statistics
 * bit for bit).  workspace: musc_b200_center_stats_bytes(channels) bytes,
 * 16-byte aligned.  channels <= 6400. */
size_t musc_b200_center_stats_bytes(int channels);
int musc_b200_center_stats(const float* z, long long rows, int channels, double* stats, void* workspace,
                           size_t workspace_bytes, musc_b200_stream stream);

/* prep_bank of the centred rows z - mu, from the statistics of one or more row
 * blocks (e.g. one per rank) stats[n_parts][channels + 1] and the number of rows
 * they cover: mu[c] = (sum over the parts of the column sums) / count, applied
 * only if |mu|^2 <= 4 x the smallest squared row norm of all parts (then
 * |z - mu| <= 3 |z| for every row; otherwise the bank holds z, as
 * musc_b200_prep_bank).  Squared distances do not change under a common shift,
 * and the split's error scales with the row norms, so for clustered rows
 * (L2-normalised ViT features) centring tightens every bound the screened pass
 * relies on.  Every bank scored against another (musc_b200_nearest's query and
 * reference banks, the ranks' blocks of a gathered pool bank) must be prepared
 * from the same statistics. */
int musc_b200_prep_bank_centered(const float* z, long long rows, int channels, const double* stats,
                                 int n_parts, long long count, void* bank, size_t bank_bytes,
                                 musc_b200_stream stream);

/* Nearest-patch minima, squared: for every query row q (global row
 * query_first_row + q, image (query_first_row + q) / patches_per_image) and
 * every reference image j != that image,
 *   nearest_sq[j * query_rows + q] = min over the patches p of image j of
 *                                    |z_q - z_p|^2   (clamped at 0),
 * and FLT_MAX in the query's own image slot (_MSM_gpu.py:202).  This is
 * _MSM.py:16-17 before the square root.  The reference bank holds rows
 * [0, ref_rows) = images [0, ref_rows / patches_per_image).
 * n_images = ref_rows / patches_per_image.  tcgen05 split-fp16 GEMM with the
 * min fused into the epilogue; the distance matrix never reaches memory. */
int musc_b200_nearest(const void* query_bank, long long query_rows, long long query_first_row,
                      const void* ref_bank, long long ref_rows, int channels,
                      int patches_per_image, float* nearest_sq, musc_b200_stream stream);

/* Pool form of the above, for a bank scored against itself: every unordered
 * pair of patches from different images is evaluated once (symmetric tiles:
 * row minima give one direction, column minima the other; the reference GPU
 * driver pairs forward/reverse the same way, _MSM_gpu.py:749-767), halving
 * the tensor-core work.  The tile list is split into n_parts balanced parts
 * and this call evaluates part `part` (multi-GPU: one part per rank, then an
 * element-wise MIN reduction of the tables).
 * The bank is laid out for bank_rows >= rows rows (a padded, gathered bank);
 * only its first `rows` rows are scored.
 * Layout: nearest_sq[block][image][r], block = row / rows_per_block,
 * r = row % rows_per_block, n_images = rows / patches_per_image; the call
 * first fills the whole table with FLT_MAX.  The buffer must hold
 * musc_b200_nearest_pool_bytes: the table plus a 256-byte word after it (at
 * the table size rounded up to 256 bytes) that the kernel's dynamic tile
 * scheduler uses; CTAs claim tiles from it, so ones that start late take
 * fewer.  max_ctas (0 = one per SM) caps the persistent grid: a multi-GPU
 * caller leaves a few SMs free so the collectives of the neighbouring banks
 * (which cannot share an SM with this kernel's ~200 KB of shared memory) run
 * concurrently instead of after it.  The kernel runs as CTA pairs on two SMs
 * (cta_group::2, 256 x 256 tiles; MUSC_B200_NEAREST_PAIR=0 in the
 * environment selects single-CTA 128 x 256 tiles, same table bit for bit), so
 * the cap is rounded down to an even number of CTAs.
 * rows_per_block = rows gives the plain [image][row] table;
 * rows_per_block = one rank's rows makes each rank's rows contiguous for a
 * reduce-scatter. */
size_t musc_b200_nearest_pool_bytes(long long rows, int patches_per_image, long long rows_per_block);

int musc_b200_nearest_pool(const void* bank, long long bank_rows, long long rows, int channels,
                           int patches_per_image, int part, int n_parts, long long rows_per_block,
                           int max_ctas, float* nearest_sq, musc_b200_stream stream);

/* Screened pool pass: the rank-deferred form of musc_b200_nearest_pool, the
 * default path of musc_b200_msm and musc_b200_score_pool.  Replaces the
 * reference GPU driver's fp16 screening (models/modules/_MSM_gpu.py:739-767,
 * deferred_half_min :307-419): the same symmetric tile list evaluated with
 * one fp16 hi*hi MMA pass (a third of the exact path's tensor-core work).  For
 * every (row, reference image) it stores, in the layout of
 * musc_b200_nearest_pool ([block][image][r], blocks = ceil(rows /
 * rows_per_block)):
 *   k1: uint64 key (bits of the smallest screened squared distance, low 8
 *       mantissa bits cleared) << 32 | the patch of the image attaining it;
 *   m2: uint32 bits of the second-smallest screened squared distance over
 *       the image's other patches (low 8 bits cleared),
 * both 0xFF.. where unset (the call fills both first).  sched_word: 8 bytes
 * the kernel's tile scheduler counts in.  Parts of a multi-GPU split combine
 * through musc_b200_refine, not by a plain minimum. */
int musc_b200_screen_pool(const void* bank, long long bank_rows, long long rows, int channels,
                          int patches_per_image, int part, int n_parts, long long rows_per_block,
                          int max_ctas, void* k1, void* m2, void* sched_word, musc_b200_stream stream);

/* Exact minima from screened tables (the reference's rank-deferred exact
 * evaluation, models/modules/_MSM_gpu.py:770-786: kthvalue threshold,
 * rank_anchor_rows, rank_candidates, rank_finish).  For the query rows
 * [first_row, first_row + query_rows) of the pool bank (all `rows` rows
 * gathered, laid out for bank_rows), with n_partials screen tables (partial g
 * at k1 + g * partial_stride entries, likewise m2, each [n_images][table_rows],
 * local row index = row - first_row), writes exact_sq[n_images][query_rows]:
 *   - FLT_MAX for the query's own image and for images whose certified lower
 *     bound lies above the rank_hi-th smallest certified upper bound (they
 *     cannot reach the trimmed ranks [.., rank_hi));
 *   - the exact squared minimum (fp32-class, as musc_b200_nearest_pool) for
 *     every other image: the exact distance to the screened argmin when the
 *     second-smallest screened value rules out every other patch, else the
 *     exact 3-pass minimum over the image's patches.
 * So musc_b200_trimmed_mean over exact_sq gives the reference's scores for any
 * rank_lo < rank_hi.  Scratch in `workspace` (1024-byte aligned): its fixed
 * part (the queue of uncertified pairs, n_images * query_rows ints) plus a
 * staging bank for the exact fallback, which runs in rounds of as many rows as
 * the staging bank holds.  musc_b200_refine_bytes is the default size (up to 2 M
 * staged rows); any size >= musc_b200_refine_min_bytes (128 staged rows) gives
 * the same results in more rounds. */
size_t musc_b200_refine_bytes(int n_images, long long query_rows, int channels);

size_t musc_b200_refine_min_bytes(int n_images, long long query_rows, int channels);

/* Kernels one musc_b200_refine call with this workspace size enqueues (2 plus 3 per
 * fallback round; rounds past the end of the queue return at once). */
int musc_b200_refine_launches(int n_images, long long query_rows, int channels, size_t workspace_bytes);

int musc_b200_refine(const void* bank, long long bank_rows, long long rows, int channels,
                     int patches_per_image, long long first_row, long long query_rows, int rank_hi,
                     const void* k1, const void* m2, int n_partials, long long partial_stride,
                     long long table_rows, float* exact_sq, void* workspace, size_t workspace_bytes,
                     musc_b200_stream stream);

/* Interval average: scores[q] = mean of ranks [rank_lo, rank_hi) of
 * sqrt(nearest_sq[:, q]) over the n_images - 1 other images, in float32,
 * stored as float64 (_MSM.py:19-30).  0 <= rank_lo < rank_hi <= n_images-1.
 * Pool size limit: a CTA stages 32 rows x n_images keys in shared memory, so
 * n_images <= 1790 on a B200 (227 KB per CTA); larger pools return
 * MUSC_B200_ERR_INVALID (the reference's MSM has no such limit). */
int musc_b200_trimmed_mean(const float* nearest_sq, long long query_rows, int n_images,
                           int rank_lo, int rank_hi, double* scores, musc_b200_stream stream);

/* Whole MSM for one bank: z [n][p][c] fp32 -> scores [n][p] float64: column
 * centring statistics and the centred bank prep, screened pool pass, refinement to exact
 * minima, interval average
 * (MUSC_B200_MSM_EXACT=1 in the environment: the 3-pass musc_b200_nearest_pool
 * instead of screen + refinement).  The workspace holds the bank, the tables and the statistics.  n <= 1790 (the
 * interval average's shared-memory limit, see musc_b200_trimmed_mean). */
size_t musc_b200_msm_workspace_bytes(int n, int p, int c);

int musc_b200_msm(const float* z, int n, int p, int c, int rank_lo, int rank_hi,
                  double* scores, void* workspace, size_t workspace_bytes,
                  musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * Score reduction: models/musc.py:259-288.
 * scores: [n_radii][n_layers][n][side*side] float64.  maps[n][side*side] =
 * mean over layers, then over radii; image_max[n] = max of the bilinear
 * (align_corners=True) up-sampling of each map to image_size^2; upsampled
 * (nullable) receives that [n][image_size][image_size] map.
 * ---------------------------------------------------------------------- */
int musc_b200_score_maps(const double* scores, int n_radii, int n_layers, int n, int side,
                         int image_size, double* maps, double* image_max, double* upsampled,
                         musc_b200_stream stream);

/* RsCIN image-score refinement (models/modules/_RsCIN.py:5-31, applied by
 * models/musc.py:287-296).  cls_tokens [n_images][dim] float32 (the
 * L2-normalised pooled class features), image_scores [n_images] float64 ->
 * scores_out [n_images] float64 (must not alias image_scores).  For each k of
 * k_list (at most 8 values, each <= min(n_images, 64)), every image averages
 * the min-max normalised scores of the k images most similar to it (itself
 * included) weighted by the similarity; the result is the mean over the
 * list.  As in the reference, cls_tokens == NULL, n_k == 0 or a 0 in k_list
 * returns the scores unchanged (a device copy). */
int musc_b200_rscin(const float* cls_tokens, int n_images, int dim, const double* image_scores, int n_k,
                    const int* k_list, double* scores_out, musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * Whole-pool scoring on one GPU (LNAMD, MSM and reduction in one call): the scoring
 * half of MuSc.make_category_data (models/musc.py:224-288) for non-Python
 * hosts.  tokens[l] points at layer l's [n_images][tokens_per_image][channels]
 * tokens (`dtype`).  For every layer: LNAMD of the given radii (one pass,
 * L2-normalised banks); for every (radius, layer) bank: split-fp16 prep,
 * symmetric nearest GEMM, interval average over ranks
 * [int((N-1)*topmin_min), int((N-1)*topmin_max)) (values >= 1 are ranks, as
 * in models/modules/_MSM_gpu.py:706-709).  Outputs: scores
 * [n_radii][n_layers][n_images][P] float64, maps [n_images][P] float64 (layer
 * mean then radius mean) and image_max [n_images] float64 (maximum of the
 * bilinear align_corners=True up-sampling to image_size^2).
 * ---------------------------------------------------------------------- */
size_t musc_b200_score_pool_bytes(int n_images, int tokens_per_image, int channels, int n_radii);

int musc_b200_score_pool(const void* const* tokens, int dtype, int n_images, int tokens_per_image,
                         int channels, int n_layers, int n_radii, const int* radii, double topmin_min,
                         double topmin_max, int image_size, double* scores, double* maps,
                         double* image_max, void* workspace, size_t workspace_bytes,
                         musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * Block attention of the ViT-L/14 encoder: out = softmax(q k^T * scale) v per
 * (batch item, head), the core of nn.MultiheadAttention as the reference's ViT
 * blocks call it (models/backbone/open_clip/transformer.py:221-234), with the
 * reference's row-softmax kernel (models/modules/_attention_gpu.py:41-81)
 * fused in: the tokens x tokens logits never reach memory.
 * q, k, v: fp16 or bf16 (dtype MUSC_B200_F16 / MUSC_B200_BF16), element
 * (b, t, h, d) at base[(b * tokens + t) * qkv_row_stride
 * + h * head_dim + d] (so the three slices of one packed QKV projection are
 * addressed by base, base + heads*head_dim, base + 2*heads*head_dim);
 * out: same type, same addressing with out_row_stride.  Softmax and
 * accumulation in fp32; P is rounded to the input type for the second MMA.  head_dim == 64; strides
 * multiples of 8 elements; pointers 16-byte aligned.
 * ---------------------------------------------------------------------- */
int musc_b200_attention_fwd(const void* q, const void* k, const void* v, void* out, int dtype,
                            int batch, int tokens, int heads, int head_dim, long long qkv_row_stride,
                            long long out_row_stride, float scale, musc_b200_stream stream);

/* Residual add + LayerNorm of a ViT block (models/backbone/open_clip/transformer.py:236-249,
 * the ln_1 / ln_2 normalisations with the preceding branch's residual add fused in):
 * per row of x [rows][channels] fp32 (updated in place), x += delta (delta: the branch's
 * [rows][channels] output in delta_dtype, f16 or bf16, widened exactly; NULL = no add),
 * then out = (x - mean) / sqrt(var + eps) * gamma + beta in out_dtype (f16 or bf16), with
 * the mean and biased variance in fp32 (two-pass).  channels a multiple of 128, at most
 * 2048; all pointers 16-byte aligned. */
int musc_b200_add_layernorm(float* x, const void* delta, int delta_dtype, const float* gamma,
                            const float* beta, float eps, void* out, int out_dtype, long long rows,
                            int channels, musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * Pool-image preprocessing: the evaluation transform the reference applies to
 * each image before the encoder -- Resize((out_h, out_w), BICUBIC), CenterCrop
 * of the same size (the identity), ToTensor, Normalize(mean, std)
 * (models/backbone/open_clip/transform.py:124-133, applied per item in
 * datasets/mvtec.py:98-99, batched by models/modules/_loader.py:8-43 and
 * moved to the device at models/musc.py:197) -- on the device, bit for bit.
 * The resize is Pillow's antialiased separable resample (fixed-point weights
 * with 22 fractional bits, 8-bit horizontal pass, then vertical pass);
 * MUSC_B200_BILINEAR gives Pillow's bilinear, the reference's non-CLIP path
 * (datasets/mvtec.py:53-60).
 * images: n_images 8-bit RGB images, H x W x 3 row-major (decoded on the host,
 * e.g. PIL convert("RGB")), image i at images + i * image_stride_bytes.
 * mean, std: 3 host floats each (copied at the call).  out: n_images x 3 x
 * out_h x out_w in out_dtype (F32 = the reference's tensor bit for bit; F16 /
 * BF16 = that tensor rounded to nearest).  An input side may be at most 15.75x
 * (bicubic) / 31.5x (bilinear) its output side.  workspace: the two axes'
 * weight tables, musc_b200_preprocess_workspace_bytes (0 = invalid sizes).
 * ---------------------------------------------------------------------- */
enum musc_b200_filter { MUSC_B200_BICUBIC = 0, MUSC_B200_BILINEAR = 1 };

size_t musc_b200_preprocess_workspace_bytes(int in_h, int in_w, int out_h, int out_w, int filter);

int musc_b200_preprocess_images(const uint8_t* images, int n_images, int in_h, int in_w,
                                long long image_stride_bytes, int out_h, int out_w, int filter,
                                const float* mean, const float* std, int out_dtype, void* out,
                                void* workspace, size_t workspace_bytes, musc_b200_stream stream);

/* ------------------------------------------------------------------------
 * Copy-engine exchange between the GPUs of one node (multi-GPU pool scoring;
 * no counterpart in the reference, which is single-device).
 *
 * musc_b200_ipc_get: the 64-byte CUDA IPC handle of the allocation holding
 *     device pointer `ptr` and the offset of `ptr` inside it.
 * musc_b200_ipc_open: maps a peer's handle into this process (peer access
 *     enabled lazily); *base is what musc_b200_ipc_close takes, *ptr = *base +
 *     offset.  A mapped pointer is only ever a cudaMemcpyAsync source or a
 *     flag address here -- never a kernel or library operand.
 * musc_b200_stream_signal: stream-ordered write of `value` to a 32-bit flag
 *     (this device's or a peer's mapped memory); the stream's prior work is
 *     made visible first.
 * musc_b200_stream_wait: the stream waits until the flag (this device's
 *     memory) is >= value (cyclic 32-bit comparison).  Counters only grow.
 * musc_b200_copy_async: cudaMemcpyAsync of `bytes` between two device
 *     pointers of the unified address space (peer copies run on copy engines).
 * ---------------------------------------------------------------------- */
int musc_b200_ipc_get(const void* ptr, void* handle, size_t* offset);

int musc_b200_ipc_open(const void* handle, size_t offset, void** base, void** ptr);

int musc_b200_ipc_close(void* base);

int musc_b200_stream_signal(unsigned int* flag, unsigned int value, musc_b200_stream stream);

int musc_b200_stream_wait(const unsigned int* flag, unsigned int value, musc_b200_stream stream);

int musc_b200_copy_async(void* dst, const void* src, size_t bytes, musc_b200_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* MUSC_B200_H */
