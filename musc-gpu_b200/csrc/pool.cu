// Whole-pool scoring on one GPU through the C ABI: the scoring half of
// MuSc.make_category_data (models/musc.py:224-288) for callers that are not
// Python -- LNAMD of every hooked layer (all radii in one pass), then per
// (radius, layer) bank the centring statistics and the centred split-fp16 prep, the
// screened symmetric pass and its refinement to exact minima (or the 3-pass exact
// pass, MUSC_B200_MSM_EXACT=1) and the interval average, then the layer/radius
// means, up-sampling and image maxima.
// Every launch goes to the caller's stream; scratch lives in one caller
// workspace sized by musc_b200_score_pool_bytes.
#include "common.cuh"

#include <algorithm>

// Implemented in msm.cu: one prepared bank -> scores, and its scratch size.
int msm_bank(const void* bank, int n, int p, int c, int rank_lo, int rank_hi, double* scores, void* scratch,
             cudaStream_t s);
size_t msm_bank_scratch_bytes(int n, int p, int c);

namespace musc {
namespace {

size_t align_1k(size_t v) { return (v + 1023) / 1024 * 1024; }

struct PoolWorkspace {
  size_t stats, z, bank, table, center, partial, total;
};

PoolWorkspace pool_layout(int n, int p, int c, int n_radii) {
  PoolWorkspace w;
  const long long rows = (long long)n * p;
  w.stats = 0;
  w.z = align_1k(musc_b200_lnamd_workspace_bytes(n));
  w.bank = w.z + align_1k((size_t)n_radii * rows * c * sizeof(float));
  w.table = w.bank + align_1k(musc_b200_bank_bytes(rows, c));
  w.center = w.table + align_1k(msm_bank_scratch_bytes(n, p, c));
  w.partial = w.center + align_1k((size_t)(c + 1) * sizeof(double));
  w.total = w.partial + align_1k(musc_b200_center_stats_bytes(c));
  return w;
}

int side_of(int tokens_per_image) {
  int s = 0;
  while ((s + 1) * (s + 1) <= tokens_per_image - 1) ++s;
  return s * s == tokens_per_image - 1 ? s : 0;
}

}  // namespace
}  // namespace musc

using namespace musc;

extern "C" size_t musc_b200_score_pool_bytes(int n_images, int tokens_per_image, int channels, int n_radii) {
  if (n_images <= 0 || tokens_per_image < 2 || channels <= 0 || n_radii <= 0) return 0;
  return pool_layout(n_images, tokens_per_image - 1, channels, n_radii).total;
}

extern "C" int musc_b200_score_pool(const void* const* tokens, int dtype, int n_images, int tokens_per_image,
                                    int channels, int n_layers, int n_radii, const int* radii,
                                    double topmin_min, double topmin_max, int image_size, double* scores,
                                    double* maps, double* image_max, void* workspace, size_t workspace_bytes,
                                    musc_b200_stream stream) {
  if (!tokens || !radii || !maps || !image_max || !workspace)
    return fail(MUSC_B200_ERR_INVALID, "score_pool: null pointer");
  if (n_layers <= 0 || n_radii <= 0 || n_radii > 3)
    return fail(MUSC_B200_ERR_INVALID, "score_pool: 1 or more layers and 1 to 3 radii are required");
  const int side = side_of(tokens_per_image);
  if (side == 0) return fail(MUSC_B200_ERR_INVALID, "score_pool: tokens_per_image - 1 must be a square");
  const int p = side * side;
  // Rank interval exactly as models/modules/_MSM_gpu.py:706-709 derives it.
  int a = topmin_min < 1 ? (int)((n_images - 1) * topmin_min) : (int)topmin_min;
  int b = topmin_max < 1 ? (int)((n_images - 1) * topmin_max) : (int)topmin_max;
  if (a > b) std::swap(a, b);
  if (!(n_images >= 2 && 0 <= a && a < b && b <= n_images - 1))
    return fail(MUSC_B200_ERR_INVALID, "Require valid nonempty trimmed ranks 0<=a<b<=N-1.");
  const PoolWorkspace w = pool_layout(n_images, p, channels, n_radii);
  if (workspace_bytes < w.total)
    return fail(MUSC_B200_ERR_WORKSPACE, "score_pool: workspace smaller than musc_b200_score_pool_bytes");
  if (reinterpret_cast<uintptr_t>(workspace) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "score_pool: workspace must be 1024-byte aligned");
  if (!scores) return fail(MUSC_B200_ERR_INVALID, "score_pool: scores [R][L][N][P] float64 is required");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const long long rows = (long long)n_images * p;
  float* z = reinterpret_cast<float*>(ws + w.z);
  for (int li = 0; li < n_layers; ++li) {
    float* outs[3];
    for (int ri = 0; ri < n_radii; ++ri) outs[ri] = z + (size_t)ri * rows * channels;
    MUSC_TRY(musc_b200_lnamd(tokens[li], dtype, n_images, tokens_per_image, channels, n_radii, radii, outs,
                             (long long)p * channels, channels, 1, ws + w.stats, w.z - w.stats, stream));
    for (int ri = 0; ri < n_radii; ++ri) {
      double* center = reinterpret_cast<double*>(ws + w.center);
      MUSC_TRY(musc_b200_center_stats(outs[ri], rows, channels, center, ws + w.partial, w.total - w.partial, stream));
      MUSC_TRY(musc_b200_prep_bank_centered(outs[ri], rows, channels, center, 1, rows, ws + w.bank,
                                            w.table - w.bank, stream));
      MUSC_TRY(msm_bank(ws + w.bank, n_images, p, channels, a, b, scores + ((size_t)ri * n_layers + li) * rows,
                        ws + w.table, reinterpret_cast<cudaStream_t>(stream)));
    }
  }
  return musc_b200_score_maps(scores, n_radii, n_layers, n_images, side, image_size, maps, image_max, nullptr,
                              stream);
}
