// Score reduction: models/musc.py:259-288.
//
// One CTA per image: the (side*side) map is the mean over layers of each
// radius's MSM scores, then the mean over radii (float64, models/musc.py:259,
// 263); the per-image score is the maximum of the bilinear, align_corners=True
// up-sampling of the map to image_size^2 (models/musc.py:269-273, 288), with
// the interpolation evaluated in the same order as torch's
// upsample_bilinear2d: h0w * (w0w * a + w1w * b) + h1w * (w0w * c + w1w * d).
#include "common.cuh"

#include <cfloat>

namespace musc {

constexpr int kReduceThreads = 256;

__global__ void __launch_bounds__(kReduceThreads)
score_maps_kernel(const double* __restrict__ scores, int n_radii, int n_layers, int n, int side,
                  int image_size, double* __restrict__ maps, double* __restrict__ image_max,
                  double* __restrict__ upsampled) {
  extern __shared__ double map[];
  const int img = blockIdx.x;
  const int P = side * side;
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    double acc_r = 0.0;
    for (int r = 0; r < n_radii; ++r) {
      double acc_l = 0.0;
      for (int l = 0; l < n_layers; ++l)
        acc_l += scores[(((long long)r * n_layers + l) * n + img) * P + p];
      acc_r += acc_l / (double)n_layers;
    }
    const double v = acc_r / (double)n_radii;
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
    image_max[img] = b;
  }
}

}  // namespace musc

using namespace musc;

extern "C" int musc_b200_score_maps(const double* scores, int n_radii, int n_layers, int n, int side,
                                    int image_size, double* maps, double* image_max, double* upsampled,
                                    musc_b200_stream stream) {
  if (!scores || !maps || !image_max) return fail(MUSC_B200_ERR_INVALID, "score_maps: null pointer");
  if (n_radii <= 0 || n_layers <= 0 || n <= 0 || side <= 0 || image_size <= 0)
    return fail(MUSC_B200_ERR_INVALID, "score_maps: sizes must be positive");
  const size_t smem = (size_t)side * side * sizeof(double);
  if (smem > 48 * 1024) return fail(MUSC_B200_ERR_INVALID, "score_maps: side too large (side*side <= 6144)");
  MUSC_TRY(require_sm100());
  score_maps_kernel<<<n, kReduceThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      scores, n_radii, n_layers, n, side, image_size, maps, image_max, upsampled);
  return check_launch("score_maps_kernel");
}
