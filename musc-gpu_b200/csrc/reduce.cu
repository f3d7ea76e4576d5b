// Score reduction: models/musc.py:259-288.
//
// One CTA per image: the (side*side) map is the mean over layers of each
// radius's MSM scores, then the mean over radii (float64, models/musc.py:259,
// 263); the per-image score is the maximum of the bilinear, align_corners=True
// up-sampling of the map to image_size^2 (models/musc.py:269-273, 288), with
// the interpolation evaluated in the same order as torch's
// upsample_bilinear2d: h0w * (w0w * a + w1w * b) + h1w * (w0w * c + w1w * d).
//
// RsCIN (models/modules/_RsCIN.py:5-31), the image-score refinement applied
// after it (models/musc.py:287-296): one CTA per image i forms row i of the
// class-token similarity W = T T^T (fp32 dot products, one warp per column),
// takes its kmax largest entries by kmax rounds of a block arg-max, and for
// each k of the list averages the min-max normalised scores (rounded to fp32,
// as the reference's .float() does) with weights W[i, j] / sum over the kept
// j, in float64; the output is the mean over the k list.
#include "common.cuh"

#include <cfloat>
#include <climits>

namespace musc {

constexpr int kReduceThreads = 256;

__global__ void __launch_bounds__(kReduceThreads)
score_maps_kernel(const double* __restrict__ scores, int n_radii, int n_layers, int n, int side,
                  int image_size, double* __restrict__ maps, double* __restrict__ image_max,
                  double* __restrict__ upsampled, const int* err) {
  extern __shared__ double map[];
  const int img = blockIdx.x;
  const int P = side * side;
  // Device error word set (an expired bounded wait upstream): NaN maps and maxima.
  const double nan = __longlong_as_double(0x7FF8000000000000LL);
  const bool poisoned = *reinterpret_cast<const volatile int*>(err) != 0;
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    double acc_r = 0.0;
    for (int r = 0; r < n_radii; ++r) {
      double acc_l = 0.0;
      for (int l = 0; l < n_layers; ++l)
        acc_l += scores[(((long long)r * n_layers + l) * n + img) * P + p];
      acc_r += acc_l / (double)n_layers;
    }
    const double v = poisoned ? nan : acc_r / (double)n_radii;
    map[p] = v;
    maps[(long long)img * P + p] = v;
  }
  __syncthreads();
  const double scale = image_size > 1 ? (double)(side - 1) / (double)(image_size - 1) : 0.0;
  double best = -DBL_MAX;
  const long long total = (long long)image_size * image_size;
  for (long long idx = threadIdx.x; idx < total; idx += blockDim.x) {
    const int oy = (int)(idx / image_size), ox = (int)(idx - (long long)oy * image_size);
    const double sy = scale * oy, sx = scale * ox;
    const int y0 = (int)sy, x0 = (int)sx;
    const int yp = y0 < side - 1 ? 1 : 0, xp = x0 < side - 1 ? 1 : 0;
    const double h1 = sy - y0, h0 = 1.0 - h1;
    const double w1 = sx - x0, w0 = 1.0 - w1;
    const double* r0 = map + y0 * side + x0;
    const double* r1 = r0 + yp * side;
    const double v = h0 * (w0 * r0[0] + w1 * r0[xp]) + h1 * (w0 * r1[0] + w1 * r1[xp]);
    if (upsampled) upsampled[(long long)img * total + idx] = v;
    best = v > best ? v : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ double red[kReduceThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = red[0];
    for (int w = 1; w < kReduceThreads / 32; ++w) b = red[w] > b ? red[w] : b;
    image_max[img] = poisoned ? nan : b;
  }
}

constexpr int kRscinThreads = 256;
constexpr int kRscinMaxK = 64;
constexpr int kRscinMaxList = 8;

struct KList {
  int count;
  int k[kRscinMaxList];
};

__global__ void __launch_bounds__(kRscinThreads)
rscin_kernel(const float* __restrict__ cls, int n, int dim, const double* __restrict__ scores, KList klist,
             int kmax, double* __restrict__ out, const int* err) {
  extern __shared__ float w[];  // row i of W
  __shared__ double red_lo[kRscinThreads / 32], red_hi[kRscinThreads / 32];
  __shared__ float red_v[kRscinThreads / 32];
  __shared__ int red_j[kRscinThreads / 32];
  __shared__ float sel_w[kRscinMaxK];
  __shared__ int sel_j[kRscinMaxK];
  const int i = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;

  // min and max of the image scores (_RsCIN.py:26)
  double lo = DBL_MAX, hi = -DBL_MAX;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const double v = scores[j];
    lo = v < lo ? v : lo;
    hi = v > hi ? v : hi;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double a = __shfl_xor_sync(0xffffffffu, lo, o), b = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = a < lo ? a : lo;
    hi = b > hi ? b : hi;
  }
  if (lane == 0) red_lo[warp] = lo, red_hi[warp] = hi;

  // row i of the similarity matrix (_RsCIN.py:27)
  const float* ci = cls + (long long)i * dim;
  for (int j = warp; j < n; j += nwarps) {
    const float* cj = cls + (long long)j * dim;
    float acc = 0.f;
    for (int d = lane; d < dim; d += 32) acc = fmaf(__ldg(ci + d), __ldg(cj + d), acc);
    acc = warp_sum(acc);
    if (lane == 0) w[j] = acc;
  }
  __syncthreads();
  lo = red_lo[0];
  hi = red_hi[0];
  for (int k = 1; k < nwarps; ++k) {
    lo = red_lo[k] < lo ? red_lo[k] : lo;
    hi = red_hi[k] > hi ? red_hi[k] : hi;
  }

  // the kmax largest entries, largest first (ties: lower index first)
  for (int t = 0; t < kmax; ++t) {
    float best = -FLT_MAX;
    int bj = INT_MAX;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const float v = w[j];
      if (v > best || (v == best && j < bj)) best = v, bj = j;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ov > best || (ov == best && oj < bj)) best = ov, bj = oj;
    }
    if (lane == 0) red_v[warp] = best, red_j[warp] = bj;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int k = 1; k < nwarps; ++k)
        if (red_v[k] > best || (red_v[k] == best && red_j[k] < bj)) best = red_v[k], bj = red_j[k];
      sel_w[t] = best;
      sel_j[t] = bj;
      w[bj] = -FLT_MAX;
    }
    __syncthreads();
  }

  // MMO (_RsCIN.py:5-20): per k, the W-weighted mean of the normalised scores of the k kept
  // columns; then the mean over the k list
  if (threadIdx.x == 0) {
    const double range = hi - lo;
    double acc = 0.0;
    for (int q = 0; q < klist.count; ++q) {
      double num = 0.0, den = 0.0;
      for (int t = 0; t < klist.k[q]; ++t) {
        const double s = (double)(float)((scores[sel_j[t]] - lo) / range);
        num += (double)sel_w[t] * s;
        den += (double)sel_w[t];
      }
      acc += num / den;
    }
    // Device error word set (an expired bounded wait upstream): NaN instead of a score.
    out[i] = *reinterpret_cast<const volatile int*>(err) != 0 ? __longlong_as_double(0x7FF8000000000000LL)
                                                              : acc / (double)klist.count;
  }
}

}  // namespace musc

using namespace musc;

extern "C" int musc_b200_rscin(const float* cls_tokens, int n_images, int dim, const double* image_scores, int n_k,
                               const int* k_list, double* scores_out, musc_b200_stream stream) {
  if (!image_scores || !scores_out || (n_k > 0 && !k_list))
    return fail(MUSC_B200_ERR_INVALID, "rscin: null pointer");
  if (n_images <= 0 || n_k < 0 || n_k > kRscinMaxList)
    return fail(MUSC_B200_ERR_INVALID, "rscin: requires n_images > 0 and at most 8 k values");
  MUSC_TRY(require_sm100());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  bool passthrough = cls_tokens == nullptr || n_k == 0;
  for (int q = 0; q < n_k; ++q) passthrough = passthrough || k_list[q] == 0;
  if (passthrough) {  // _RsCIN.py:23-24: the scores come back unchanged
    if (scores_out != image_scores)
      MUSC_CUDA(cudaMemcpyAsync(scores_out, image_scores, (size_t)n_images * sizeof(double),
                                cudaMemcpyDeviceToDevice, s));
    return MUSC_B200_OK;
  }
  if (dim <= 0) return fail(MUSC_B200_ERR_INVALID, "rscin: dim must be positive");
  if (scores_out == image_scores)
    return fail(MUSC_B200_ERR_INVALID, "rscin: scores_out must not alias image_scores (every image reads all scores)");
  KList kl{};
  kl.count = n_k;
  int kmax = 0;
  for (int q = 0; q < n_k; ++q) {
    if (k_list[q] < 0 || k_list[q] > n_images || k_list[q] > kRscinMaxK)
      return fail(MUSC_B200_ERR_INVALID, "rscin: every k must lie in [0, min(n_images, 64)]");
    kl.k[q] = k_list[q];
    kmax = k_list[q] > kmax ? k_list[q] : kmax;
  }
  const size_t smem = (size_t)n_images * sizeof(float);
  if ((long long)smem > smem_optin() - 2048)
    return fail(MUSC_B200_ERR_INVALID, "rscin: too many images for one similarity row in shared memory");
  if (smem > 48 * 1024)
    MUSC_CUDA(cudaFuncSetAttribute(rscin_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int* err = device_error_ptr();
  if (!err) return fail(MUSC_B200_ERR_CUDA, "rscin: device error word unavailable");
  rscin_kernel<<<n_images, kRscinThreads, smem, s>>>(cls_tokens, n_images, dim, image_scores, kl, kmax, scores_out,
                                                     err);
  return check_launch("rscin_kernel");
}

extern "C" int musc_b200_score_maps(const double* scores, int n_radii, int n_layers, int n, int side,
                                    int image_size, double* maps, double* image_max, double* upsampled,
                                    musc_b200_stream stream) {
  if (!scores || !maps || !image_max) return fail(MUSC_B200_ERR_INVALID, "score_maps: null pointer");
  if (n_radii <= 0 || n_layers <= 0 || n <= 0 || side <= 0 || image_size <= 0)
    return fail(MUSC_B200_ERR_INVALID, "score_maps: sizes must be positive");
  const size_t smem = (size_t)side * side * sizeof(double);
  if (smem > 48 * 1024) return fail(MUSC_B200_ERR_INVALID, "score_maps: side too large (side*side <= 6144)");
  MUSC_TRY(require_sm100());
  int* err = device_error_ptr();
  if (!err) return fail(MUSC_B200_ERR_CUDA, "score_maps: device error word unavailable");
  score_maps_kernel<<<n, kReduceThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      scores, n_radii, n_layers, n, side, image_size, maps, image_max, upsampled, err);
  return check_launch("score_maps_kernel");
}
