// LNAMD neighbourhood aggregation: models/modules/_LNAMD.py and its call in models/musc.py.
//
// Reference: LNAMD._embed (models/modules/_LNAMD.py:72-129), its direct-pool
// form aggregate_features (models/modules/_encoder_gpu.py:14-42), the radius
// cache (models/modules/_aggregation_cache.py:15-58), the super-fast pooling
// (models/modules/_super_fast.py:17-27) and the L2 normalisation of
// models/musc.py:238.
//
// Two passes over the tokens of one layer:
//   1. lnamd_stats: per image sum and sum of squares of the (side*side, C)
//      body in float64 (the LayerNorm statistics over the whole image),
//      split over kStatSplit CTAs per image.
//   2. lnamd_stencil: one CTA per (output row y, image); thread t owns
//      channels [4t, 4t+4).  Walking x along the row it keeps vertical
//      window sums of the centred values for r = 1, 3, 5 in a register ring,
//      forms the r x r box sums (zero padding, divisor r^2), scales by the
//      LayerNorm rstd and -- when asked -- divides by the per-patch L2 norm
//      over channels (one block reduction per patch).  All radii come from one
//      read of the tokens; the five input rows a CTA reads are re-read by the
//      neighbouring rows' CTAs, which run next to it, mostly from L2.  The
//      default (staged) form streams each column's input tokens into a
//      shared-memory ring with bulk copies; the register-pipelined form
//      serves rows whose byte length is not a multiple of 16.
// Algorithmic bytes per layer: n * (1 + P) * C * sizeof(T) read for the
// statistics, the same again for the stencil, and n_radii * n * P * C * 4
// written.
#include "common.cuh"
#include "tc.cuh"

#include <cstdlib>
#include <mutex>
#include <vector>

namespace musc {

constexpr int kStatSplit = 8;
constexpr int kStatThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kStatThreads)
lnamd_stats_kernel(const T* __restrict__ tokens, long long image_elems, int channels,
                   long long body_vec4, double* __restrict__ partial) {
  const int img = blockIdx.y;
  const T* body = tokens + (long long)img * image_elems + channels;  // skip CLS
  const long long per = (body_vec4 + gridDim.x - 1) / gridDim.x;
  const long long begin = (long long)blockIdx.x * per;
  const long long end = begin + per < body_vec4 ? begin + per : body_vec4;
  double s = 0.0, ss = 0.0;
  for (long long i = begin + threadIdx.x; i < end; i += blockDim.x) {
    float4 v = load4<T>(body + 4 * i);
    s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
    ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  s = warp_sum(s);
  ss = warp_sum(ss);
  __shared__ double red[2][kStatThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][warp] = s;
    red[1][warp] = ss;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < kStatThreads / 32; ++w) {
      a += red[0][w];
      b += red[1][w];
    }
    partial[((long long)img * gridDim.x + blockIdx.x) * 2 + 0] = a;
    partial[((long long)img * gridDim.x + blockIdx.x) * 2 + 1] = b;
  }
}

// LayerNorm mean and rstd of one image from the split partial sums.
__device__ __forceinline__ void image_moments(const double* partial, int img, double count,
                                              float* mu, float* rstd) {
  double s = 0.0, ss = 0.0;
#pragma unroll
  for (int k = 0; k < kStatSplit; ++k) {
    s += partial[((long long)img * kStatSplit + k) * 2 + 0];
    ss += partial[((long long)img * kStatSplit + k) * 2 + 1];
  }
  double mean = s / count;
  double var = ss / count - mean * mean;
  if (var < 0.0) var = 0.0;
  *mu = (float)mean;
  *rstd = (float)(1.0 / sqrt(var + 1e-5));
}

__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4scale(float4 a, float s) {
  return make_float4(a.x * s, a.y * s, a.z * s, a.w * s);
}
// Explicit FMA chain: nothing left for the compiler to contract, so every
// kernel that uses it rounds identically.
__device__ __forceinline__ float f4dot(float4 a) {
  return __fmaf_rn(a.w, a.w, __fmaf_rn(a.z, a.z, __fmaf_rn(a.y, a.y, __fmul_rn(a.x, a.x))));
}

// Block-wide sum of up to three values; `buf` alternates between calls so a
// single __syncthreads per call suffices.  Every thread gets the totals.
template <int K>
__device__ __forceinline__ void block_sum(float (&v)[K], float* red, int buf) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int k = 0; k < K; ++k) v[k] = warp_sum(v[k]);
  float* slot = red + buf * 32 * K;
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < K; ++k) slot[warp * K + k] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < K; ++k) v[k] = 0.f;
  for (int w = 0; w < nwarps; ++w) {
#pragma unroll
    for (int k = 0; k < K; ++k) v[k] += slot[w * K + k];
  }
}

constexpr int kMaxStencilThreads = 512;  // channels <= 2048

template <typename T>
__global__ void __launch_bounds__(kMaxStencilThreads)
lnamd_stencil_kernel(const T* __restrict__ tokens, int tokens_per_image, int channels, int side,
                     const double* __restrict__ partial, float* out1, float* out3, float* out5,
                     long long out_image_stride, long long out_patch_stride, int normalize) {
  __shared__ float red[2 * 32 * 3];
  const int y = blockIdx.x;
  const int img = blockIdx.y;
  const int cg = threadIdx.x;  // channel group of 4
  const bool active = cg * 4 < channels;
  float mu, rstd;
  image_moments(partial, img, (double)side * side * channels, &mu, &rstd);
  const T* body = tokens + (long long)img * tokens_per_image * channels + channels + cg * 4;

  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 a1[3] = {zero, zero, zero};        // V1 at x'-2 .. x'
  float4 a3[4] = {zero, zero, zero, zero};  // V3 at x'-3 .. x'
  float4 a5[5] = {zero, zero, zero, zero, zero};
  const bool want1 = out1 != nullptr, want3 = out3 != nullptr, want5 = out5 != nullptr;
  const float s1 = rstd, s3 = rstd / 9.f, s5 = rstd / 25.f;
  float* o1p = want1 ? out1 + (long long)img * out_image_stride + cg * 4 : nullptr;
  float* o3p = want3 ? out3 + (long long)img * out_image_stride + cg * 4 : nullptr;
  float* o5p = want5 ? out5 + (long long)img * out_image_stride + cg * 4 : nullptr;

  // Software pipeline: the five rows of column x'+1 are loaded while column x' is
  // reduced, so the loads overlap the per-patch block reduction.
  float4 cur[5], nxt[5];
  auto load_col = [&](int xc, float4 (&r)[5]) {
#pragma unroll
    for (int d = 0; d < 5; ++d) {
      const int yy = y + d - 2;
      if (xc < side && active && yy >= 0 && yy < side) {
        float4 t = load4<T>(body + ((long long)yy * side + xc) * channels);
        r[d] = make_float4(t.x - mu, t.y - mu, t.z - mu, t.w - mu);
      } else {
        r[d] = zero;
      }
    }
  };
  load_col(0, cur);
  for (int xp = 0; xp < side + 2; ++xp) {
    load_col(xp + 1, nxt);
    const float4 v1 = cur[2];
    const float4 v3 = f4add(f4add(cur[1], cur[2]), cur[3]);
    const float4 v5 = f4add(f4add(v3, cur[0]), cur[4]);
#pragma unroll
    for (int d = 0; d < 5; ++d) cur[d] = nxt[d];
    a1[0] = a1[1]; a1[1] = a1[2]; a1[2] = v1;
    a3[0] = a3[1]; a3[1] = a3[2]; a3[2] = a3[3]; a3[3] = v3;
    a5[0] = a5[1]; a5[1] = a5[2]; a5[2] = a5[3]; a5[3] = a5[4]; a5[4] = v5;
    const int x = xp - 2;
    if (x < 0) continue;
    float4 o1 = f4scale(a1[0], s1);
    float4 o3 = f4scale(f4add(f4add(a3[0], a3[1]), a3[2]), s3);
    float4 o5 = f4scale(f4add(f4add(f4add(a5[0], a5[1]), f4add(a5[2], a5[3])), a5[4]), s5);
    if (normalize) {
      float sq[3] = {want1 ? f4dot(o1) : 0.f, want3 ? f4dot(o3) : 0.f, want5 ? f4dot(o5) : 0.f};
      if (!active) sq[0] = sq[1] = sq[2] = 0.f;
      block_sum<3>(sq, red, x & 1);
      o1 = f4scale(o1, 1.f / sqrtf(sq[0]));
      o3 = f4scale(o3, 1.f / sqrtf(sq[1]));
      o5 = f4scale(o5, 1.f / sqrtf(sq[2]));
    }
    if (active) {
      const long long off = (long long)(y * side + x) * out_patch_stride;
      if (want1) *reinterpret_cast<float4*>(o1p + off) = o1;
      if (want3) *reinterpret_cast<float4*>(o3p + off) = o3;
      if (want5) *reinterpret_cast<float4*>(o5p + off) = o5;
    }
  }
}

// Staged form of lnamd_stencil_kernel with the same arithmetic in the same
// order (bit-identical outputs).  Thread 0 streams the (up to five) input
// tokens of each column into a kBulkDepth-deep shared-memory ring with untiled
// bulk copies, kBulkDepth columns ahead, so every CTA keeps its next columns'
// reads in flight without holding them in registers (which lets three
// 256-thread CTAs share an SM); the other threads read their four channels
// from shared memory.  One __syncthreads per column (the L2-norm reduction's)
// frees the column's slot for the next copy.  Requires channels * sizeof(T)
// % 16 == 0 (bulk-copy granularity).
constexpr uint64_t kBulkWaitNs = 2000000000ull;  // 2 s per column

template <typename T, int kBulkDepth, int kThreads, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
lnamd_stencil_bulk_kernel(const T* __restrict__ tokens, int tokens_per_image, int channels, int side,
                          const double* __restrict__ partial, float* out1, float* out3, float* out5,
                          long long out_image_stride, long long out_patch_stride, int normalize, int* err) {
  extern __shared__ __align__(128) uint8_t ring_raw[];  // [kBulkDepth][5][channels] of T
  __shared__ float red[2 * 32 * 3];
  __shared__ __align__(8) uint64_t full[kBulkDepth];
  __shared__ int aborted;
  const T* ring = reinterpret_cast<const T*>(ring_raw);
  const int y = blockIdx.x;
  const int img = blockIdx.y;
  const int cg = threadIdx.x;  // channel group of 4
  const bool active = cg * 4 < channels;
  const uint32_t row_bytes = (uint32_t)channels * (uint32_t)sizeof(T);
  const T* body = tokens + (long long)img * tokens_per_image * channels + channels;
  const int y_lo = y - 2 < 0 ? 0 : y - 2;
  const int y_hi = y + 2 > side - 1 ? side - 1 : y + 2;
  const uint32_t col_bytes = (uint32_t)(y_hi - y_lo + 1) * row_bytes;

  __shared__ int last_issued;  // thread 0: the last column whose copies were issued
  auto issue = [&](int xc) {  // thread 0: column xc into slot xc % kBulkDepth
    last_issued = xc;
    const int slot = xc % kBulkDepth;
    const uint32_t bar = tc::smem_u32(&full[slot]);
    tc::mbar_arrive_expect_tx(bar, col_bytes);
    for (int yy = y_lo; yy <= y_hi; ++yy) {
      const uint32_t dst = tc::smem_u32(ring_raw + ((size_t)slot * 5 + (yy - y + 2)) * row_bytes);
      tc::bulk_load(dst, body + ((long long)yy * side + xc) * channels, row_bytes, bar);
    }
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkDepth; ++s) tc::mbar_init(tc::smem_u32(&full[s]), 1);
    aborted = 0;
    last_issued = -1;
    tc::fence_barrier_init();
    for (int xc = 0; xc < kBulkDepth && xc < side; ++xc) issue(xc);
  }
  float mu, rstd;
  image_moments(partial, img, (double)side * side * channels, &mu, &rstd);
  __syncthreads();

  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 a1[3] = {zero, zero, zero};        // V1 at x'-2 .. x'
  float4 a3[4] = {zero, zero, zero, zero};  // V3 at x'-3 .. x'
  float4 a5[5] = {zero, zero, zero, zero, zero};
  const bool want1 = out1 != nullptr, want3 = out3 != nullptr, want5 = out5 != nullptr;
  const float s1 = rstd, s3 = rstd / 9.f, s5 = rstd / 25.f;
  float* o1p = want1 ? out1 + (long long)img * out_image_stride + cg * 4 : nullptr;
  float* o3p = want3 ? out3 + (long long)img * out_image_stride + cg * 4 : nullptr;
  float* o5p = want5 ? out5 + (long long)img * out_image_stride + cg * 4 : nullptr;

  for (int xp = 0; xp < side + 2; ++xp) {
    float4 cur[5];
    if (xp < side) {
      const int slot = xp % kBulkDepth;
      const uint32_t bar = tc::smem_u32(&full[slot]);
      const uint32_t parity = (uint32_t)(xp / kBulkDepth) & 1u;
      if (!tc::mbar_try_wait(bar, parity)) {
        const uint64_t start = global_ns();
        while (!tc::mbar_try_wait(bar, parity)) {
          if (*reinterpret_cast<volatile int*>(&aborted)) break;
          if (global_ns() - start > kBulkWaitNs) {
            aborted = 1;
            atomicExch(err, MUSC_B200_ERR_TIMEOUT);
            break;
          }
        }
      }
#pragma unroll
      for (int d = 0; d < 5; ++d) {
        const int yy = y + d - 2;
        if (active && yy >= 0 && yy < side) {
          const float4 t = load4_shared(ring + ((size_t)slot * 5 + d) * channels + cg * 4);
          cur[d] = make_float4(t.x - mu, t.y - mu, t.z - mu, t.w - mu);
        } else {
          cur[d] = zero;
        }
      }
    } else {
#pragma unroll
      for (int d = 0; d < 5; ++d) cur[d] = zero;
    }
    const float4 v1 = cur[2];
    const float4 v3 = f4add(f4add(cur[1], cur[2]), cur[3]);
    const float4 v5 = f4add(f4add(v3, cur[0]), cur[4]);
    a1[0] = a1[1]; a1[1] = a1[2]; a1[2] = v1;
    a3[0] = a3[1]; a3[1] = a3[2]; a3[2] = a3[3]; a3[3] = v3;
    a5[0] = a5[1]; a5[1] = a5[2]; a5[2] = a5[3]; a5[3] = a5[4]; a5[4] = v5;
    const int x = xp - 2;
    float4 o1 = zero, o3 = zero, o5 = zero;
    if (x >= 0) {
      o1 = f4scale(a1[0], s1);
      o3 = f4scale(f4add(f4add(a3[0], a3[1]), a3[2]), s3);
      o5 = f4scale(f4add(f4add(f4add(a5[0], a5[1]), f4add(a5[2], a5[3])), a5[4]), s5);
    }
    if (x >= 0 && normalize) {
      float sq[3] = {want1 ? f4dot(o1) : 0.f, want3 ? f4dot(o3) : 0.f, want5 ? f4dot(o5) : 0.f};
      if (!active) sq[0] = sq[1] = sq[2] = 0.f;
      block_sum<3>(sq, red, x & 1);  // its __syncthreads also frees this column's slot
      o1 = f4scale(o1, 1.f / sqrtf(sq[0]));
      o3 = f4scale(o3, 1.f / sqrtf(sq[1]));
      o5 = f4scale(o5, 1.f / sqrtf(sq[2]));
    } else {
      __syncthreads();
    }
    if (threadIdx.x == 0 && xp + kBulkDepth < side && !aborted) {
      tc::fence_proxy_async_smem();
      issue(xp + kBulkDepth);
    }
    if (x >= 0 && active) {
      const long long off = (long long)(y * side + x) * out_patch_stride;
      if (want1) *reinterpret_cast<float4*>(o1p + off) = o1;
      if (want3) *reinterpret_cast<float4*>(o3p + off) = o3;
      if (want5) *reinterpret_cast<float4*>(o5p + off) = o5;
    }
  }
  if (threadIdx.x == 0 && aborted) {
    // Let copies still in flight land before the CTA's shared memory goes away.  Only
    // the last kBulkDepth issued columns can be in flight: each occupies its own slot,
    // armed for that column's phase and never re-armed, so waiting on that phase's
    // parity waits for exactly those copies (earlier columns of the same slots were
    // consumed before the slot was reused; columns never issued are not waited on).
    const uint64_t start = global_ns();
    const int first = last_issued - kBulkDepth + 1 < 0 ? 0 : last_issued - kBulkDepth + 1;
    for (int xc = first; xc <= last_issued; ++xc) {
      const uint32_t bar = tc::smem_u32(&full[xc % kBulkDepth]);
      while (!tc::mbar_try_wait(bar, (uint32_t)(xc / kBulkDepth) & 1u) && global_ns() - start < kBulkWaitNs) {
      }
    }
  }
}

// Super-fast: r = 3 box mean on the side x side grid, adaptive average
// pooling to out_side x out_side, optional L2 normalisation.  One CTA per
// (output row i, image).  With T[x] = sum_y m_y (x(y, x) - mu), where m_y
// counts the 3-row windows of the pooled grid rows [h0, h1) that cover input
// row y, the pooled value of output (i, j) is
//   rstd / (9 (h1-h0)(w1-w0)) * sum_{w in [w0, w1)} (T[w-1] + T[w] + T[w+1]).
constexpr int kMaxSfRows = 8;
constexpr int kMaxSfWindow = 4;

template <typename T>
__global__ void __launch_bounds__(kMaxStencilThreads)
lnamd_super_fast_kernel(const T* __restrict__ tokens, int tokens_per_image, int channels, int side,
                        int out_side, const double* __restrict__ partial, float* out,
                        long long out_image_stride, long long out_patch_stride, int normalize) {
  __shared__ float red[2 * 32];
  const int i = blockIdx.x;
  const int img = blockIdx.y;
  const int cg = threadIdx.x;
  const bool active = cg * 4 < channels;
  float mu, rstd;
  image_moments(partial, img, (double)side * side * channels, &mu, &rstd);
  const T* body = tokens + (long long)img * tokens_per_image * channels + channels + cg * 4;

  const int h0 = (i * side) / out_side;
  const int h1 = ((i + 1) * side + out_side - 1) / out_side;
  const int y_lo = h0 - 1 < 0 ? 0 : h0 - 1;
  const int y_hi = h1 < side - 1 ? h1 : side - 1;  // inclusive
  float mult[kMaxSfRows];
#pragma unroll
  for (int k = 0; k < kMaxSfRows; ++k) {
    const int yy = y_lo + k;
    int m = 0;
    for (int h = h0; h < h1; ++h) m += (yy >= h - 1 && yy <= h + 1) ? 1 : 0;
    mult[k] = (yy <= y_hi) ? (float)m : 0.f;
  }
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 t[3] = {zero, zero, zero};                 // T at x'-2 .. x'
  float4 cs[kMaxSfWindow] = {zero, zero, zero, zero};  // CS at w-3 .. w
  int j = 0;
  float* op = out + (long long)img * out_image_stride + cg * 4;
  const float base_scale = rstd / (9.f * (float)(h1 - h0));

  for (int xp = 0; xp <= side; ++xp) {
    float4 tv = zero;
    if (xp < side && active) {
      for (int k = 0; k < kMaxSfRows; ++k) {
        const int yy = y_lo + k;
        if (yy > y_hi) break;
        float4 v = load4<T>(body + ((long long)yy * side + xp) * channels);
        const float m = mult[k];
        tv.x += m * (v.x - mu);
        tv.y += m * (v.y - mu);
        tv.z += m * (v.z - mu);
        tv.w += m * (v.w - mu);
      }
    }
    t[0] = t[1]; t[1] = t[2]; t[2] = tv;
    const int w = xp - 1;
    if (w < 0) continue;
#pragma unroll
    for (int k = 0; k < kMaxSfWindow - 1; ++k) cs[k] = cs[k + 1];
    cs[kMaxSfWindow - 1] = f4add(f4add(t[0], t[1]), t[2]);
    while (j < out_side) {
      const int w0 = (j * side) / out_side;
      const int w1 = ((j + 1) * side + out_side - 1) / out_side;
      if (w1 - 1 != w) break;
      float4 acc = zero;
      for (int k = 0; k < w1 - w0; ++k) acc = f4add(acc, cs[kMaxSfWindow - 1 - k]);
      float4 o = f4scale(acc, base_scale / (float)(w1 - w0));
      if (normalize) {
        float sq[1] = {active ? f4dot(o) : 0.f};
        block_sum<1>(sq, red, j & 1);
        o = f4scale(o, 1.f / sqrtf(sq[0]));
      }
      if (active) *reinterpret_cast<float4*>(op + (long long)(i * out_side + j) * out_patch_stride) = o;
      ++j;
    }
  }
}

namespace {

int check_tokens(const void* tokens, int dtype, int n_images, int tokens_per_image, int channels,
                 int* side) {
  if (!tokens) return fail(MUSC_B200_ERR_INVALID, "lnamd: null tokens");
  if (dtype < MUSC_B200_F32 || dtype > MUSC_B200_BF16)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: dtype must be f32, f16 or bf16");
  if (n_images <= 0 || channels <= 0 || tokens_per_image < 2)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: requires n_images > 0, channels > 0, tokens > 1");
  if (channels % 4 != 0 || channels > 4 * kMaxStencilThreads)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: channels must be a multiple of 4 and <= 2048");
  int s = 0;
  while ((s + 1) * (s + 1) <= tokens_per_image - 1) ++s;
  if (s * s != tokens_per_image - 1)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: tokens_per_image - 1 must be a square (CLS + side*side)");
  if (reinterpret_cast<uintptr_t>(tokens) % 16 != 0)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: tokens must be 16-byte aligned");
  *side = s;
  return MUSC_B200_OK;
}

template <typename T>
int launch_stats(const void* tokens, int n_images, int tokens_per_image, int channels, int side,
                 double* partial, cudaStream_t stream) {
  dim3 grid(kStatSplit, n_images);
  lnamd_stats_kernel<T><<<grid, kStatThreads, 0, stream>>>(
      static_cast<const T*>(tokens), (long long)tokens_per_image * channels, channels,
      (long long)side * side * channels / 4, partial);
  return check_launch("lnamd_stats_kernel");
}

int stats_dispatch(const void* tokens, int dtype, int n_images, int tokens_per_image, int channels,
                   int side, double* partial, cudaStream_t stream) {
  switch (dtype) {
    case MUSC_B200_F32:
      return launch_stats<float>(tokens, n_images, tokens_per_image, channels, side, partial, stream);
    case MUSC_B200_F16:
      return launch_stats<__half>(tokens, n_images, tokens_per_image, channels, side, partial, stream);
    default:
      return launch_stats<__nv_bfloat16>(tokens, n_images, tokens_per_image, channels, side, partial,
                                         stream);
  }
}

int block_threads(int channels) { return ((channels / 4 + 31) / 32) * 32; }

// The staged stencil is the default; MUSC_B200_LNAMD_BULK=0 selects the
// register-pipelined kernel (same outputs, bit for bit).
int bulk_stencil_mode() {
  const char* e = std::getenv("MUSC_B200_LNAMD_BULK");
  return (e && e[0] == '0') ? 0 : 1;
}

template <typename T, int D, int NT, int MB>
int launch_bulk(const void* tokens, int tokens_per_image, int channels, int side, const double* partial,
                float* const* o, long long out_image_stride, long long out_patch_stride, int l2_normalize, int* err,
                dim3 grid, int threads, cudaStream_t s) {
  static std::mutex m;
  static size_t done[64] = {0};
  const size_t ring = (size_t)D * 5 * channels * sizeof(T);
  int dev = 0;
  MUSC_CUDA(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lock(m);
    if (dev >= 64 || done[dev] < ring) {
      MUSC_CUDA(cudaFuncSetAttribute(lnamd_stencil_bulk_kernel<T, D, NT, MB>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ring));
      if (dev < 64) done[dev] = ring;
    }
  }
  lnamd_stencil_bulk_kernel<T, D, NT, MB><<<grid, threads, ring, s>>>(
      static_cast<const T*>(tokens), tokens_per_image, channels, side, partial, o[0], o[1], o[2], out_image_stride,
      out_patch_stride, l2_normalize, err);
  return check_launch("lnamd_stencil_bulk_kernel");
}

}  // namespace
}  // namespace musc

using namespace musc;

extern "C" size_t musc_b200_lnamd_workspace_bytes(int n_images) {
  return n_images > 0 ? (size_t)n_images * kStatSplit * 2 * sizeof(double) : 0;
}

extern "C" int musc_b200_lnamd(const void* tokens, int dtype, int n_images, int tokens_per_image,
                               int channels, int n_radii, const int* radii, float* const* out,
                               long long out_image_stride, long long out_patch_stride,
                               int l2_normalize, void* workspace, size_t workspace_bytes,
                               musc_b200_stream stream) {
  int side = 0;
  MUSC_TRY(check_tokens(tokens, dtype, n_images, tokens_per_image, channels, &side));
  if (n_radii <= 0 || n_radii > 3 || !radii || !out)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: 1 to 3 radii with output pointers are required");
  float* o[3] = {nullptr, nullptr, nullptr};  // r = 1, 3, 5
  for (int i = 0; i < n_radii; ++i) {
    const int r = radii[i];
    if (r != 1 && r != 3 && r != 5)
      return fail(MUSC_B200_ERR_INVALID, "lnamd: radius must be 1, 3 or 5 (the reference's direct-pool set)");
    if (!out[i] || reinterpret_cast<uintptr_t>(out[i]) % 16 != 0)
      return fail(MUSC_B200_ERR_INVALID, "lnamd: output pointers must be non-null and 16-byte aligned");
    if (o[r / 2]) return fail(MUSC_B200_ERR_INVALID, "lnamd: duplicate radius");
    o[r / 2] = out[i];
  }
  if (out_patch_stride < channels || out_patch_stride % 4 != 0 || out_image_stride % 4 != 0 ||
      out_image_stride < channels)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: strides must be multiples of 4 and hold a patch");
  if (!workspace || workspace_bytes < musc_b200_lnamd_workspace_bytes(n_images))
    return fail(MUSC_B200_ERR_WORKSPACE, "lnamd: workspace smaller than musc_b200_lnamd_workspace_bytes");
  if (reinterpret_cast<uintptr_t>(workspace) % 8 != 0)
    return fail(MUSC_B200_ERR_INVALID, "lnamd: workspace must be 8-byte aligned");
  MUSC_TRY(require_sm100());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  MUSC_TRY(stats_dispatch(tokens, dtype, n_images, tokens_per_image, channels, side, partial, s));
  dim3 grid(side, n_images);
  const int threads = block_threads(channels);
  const int elem = dtype == MUSC_B200_F32 ? 4 : 2;
  const int bulk = bulk_stencil_mode();
  if ((channels * elem) % 16 == 0 && bulk != 0) {
    int* err = device_error_ptr();
    if (!err) return fail(MUSC_B200_ERR_CUDA, "lnamd: device error word unavailable");
    // Up to 1024 channels: 256 threads, 2-deep ring, 3 CTAs per SM; wider rows: 512 threads, 3-deep.
    if (threads <= 256) {
      switch (dtype) {
        case MUSC_B200_F32:
          return launch_bulk<float, 2, 256, 3>(tokens, tokens_per_image, channels, side, partial, o, out_image_stride,
                                               out_patch_stride, l2_normalize, err, grid, threads, s);
        case MUSC_B200_F16:
          return launch_bulk<__half, 2, 256, 3>(tokens, tokens_per_image, channels, side, partial, o, out_image_stride,
                                                out_patch_stride, l2_normalize, err, grid, threads, s);
        default:
          return launch_bulk<__nv_bfloat16, 2, 256, 3>(tokens, tokens_per_image, channels, side, partial, o,
                                                       out_image_stride, out_patch_stride, l2_normalize, err, grid,
                                                       threads, s);
      }
    }
    switch (dtype) {
      case MUSC_B200_F32:
        return launch_bulk<float, 3, kMaxStencilThreads, 1>(tokens, tokens_per_image, channels, side, partial, o,
                                                            out_image_stride, out_patch_stride, l2_normalize, err,
                                                            grid, threads, s);
      case MUSC_B200_F16:
        return launch_bulk<__half, 3, kMaxStencilThreads, 1>(tokens, tokens_per_image, channels, side, partial, o,
                                                             out_image_stride, out_patch_stride, l2_normalize, err,
                                                             grid, threads, s);
      default:
        return launch_bulk<__nv_bfloat16, 3, kMaxStencilThreads, 1>(tokens, tokens_per_image, channels, side, partial,
                                                                    o, out_image_stride, out_patch_stride,
                                                                    l2_normalize, err, grid, threads, s);
    }
  }
  switch (dtype) {
    case MUSC_B200_F32:
      lnamd_stencil_kernel<float><<<grid, threads, 0, s>>>(
          static_cast<const float*>(tokens), tokens_per_image, channels, side, partial, o[0], o[1],
          o[2], out_image_stride, out_patch_stride, l2_normalize);
      break;
    case MUSC_B200_F16:
      lnamd_stencil_kernel<__half><<<grid, threads, 0, s>>>(
          static_cast<const __half*>(tokens), tokens_per_image, channels, side, partial, o[0], o[1],
          o[2], out_image_stride, out_patch_stride, l2_normalize);
      break;
    default:
      lnamd_stencil_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(tokens), tokens_per_image, channels, side, partial, o[0],
          o[1], o[2], out_image_stride, out_patch_stride, l2_normalize);
      break;
  }
  return check_launch("lnamd_stencil_kernel");
}

extern "C" int musc_b200_lnamd_super_fast(const void* tokens, int dtype, int n_images,
                                          int tokens_per_image, int channels, int out_side,
                                          float* out, long long out_image_stride,
                                          long long out_patch_stride, int l2_normalize,
                                          void* workspace, size_t workspace_bytes,
                                          musc_b200_stream stream) {
  int side = 0;
  MUSC_TRY(check_tokens(tokens, dtype, n_images, tokens_per_image, channels, &side));
  if (out_side <= 0 || out_side > side)
    return fail(MUSC_B200_ERR_INVALID, "lnamd_super_fast: out_side must be in [1, side]");
  // Pooled windows span at most ceil(side/out_side)+1 grid rows; with the
  // 3-row box this must fit kMaxSfRows input rows and kMaxSfWindow columns.
  const int win = (side + out_side - 1) / out_side + 1;
  if (win > kMaxSfWindow || win + 2 > kMaxSfRows)
    return fail(MUSC_B200_ERR_INVALID, "lnamd_super_fast: side / out_side must be <= 3");
  if (!out || reinterpret_cast<uintptr_t>(out) % 16 != 0 || out_patch_stride % 4 != 0 ||
      out_image_stride % 4 != 0 || out_patch_stride < channels)
    return fail(MUSC_B200_ERR_INVALID, "lnamd_super_fast: output must be 16-byte aligned, strides % 4 == 0");
  if (!workspace || workspace_bytes < musc_b200_lnamd_workspace_bytes(n_images))
    return fail(MUSC_B200_ERR_WORKSPACE, "lnamd_super_fast: workspace too small");
  MUSC_TRY(require_sm100());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  MUSC_TRY(stats_dispatch(tokens, dtype, n_images, tokens_per_image, channels, side, partial, s));
  dim3 grid(out_side, n_images);
  const int threads = block_threads(channels);
  switch (dtype) {
    case MUSC_B200_F32:
      lnamd_super_fast_kernel<float><<<grid, threads, 0, s>>>(
          static_cast<const float*>(tokens), tokens_per_image, channels, side, out_side, partial, out,
          out_image_stride, out_patch_stride, l2_normalize);
      break;
    case MUSC_B200_F16:
      lnamd_super_fast_kernel<__half><<<grid, threads, 0, s>>>(
          static_cast<const __half*>(tokens), tokens_per_image, channels, side, out_side, partial, out,
          out_image_stride, out_patch_stride, l2_normalize);
      break;
    default:
      lnamd_super_fast_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(tokens), tokens_per_image, channels, side, out_side,
          partial, out, out_image_stride, out_patch_stride, l2_normalize);
      break;
  }
  return check_launch("lnamd_super_fast_kernel");
}

// ---------------------------------------------------------------------------
// musc_b200_lnamd_noalloc: the same LNAMD call for callers that cannot
// allocate device memory.  Its only scratch -- the per-image LayerNorm
// partial sums, 16 doubles per image -- lives in this file-scope device array,
// so the call allocates nothing.  Every GPU that loads the library holds the
// array (256 KB) until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxImages = 2048;
__device__ __align__(256) double g_lnamd_noalloc_scratch[kNoAllocMaxImages * kStatSplit * 2];

// Device address of the scratch array on the current device.  Host code may
// not pass the array's name to a kernel (on the host it is only a stand-in
// symbol), so the address is looked up with the device current.  It is looked
// up on every call (a host-side query that allocates nothing) rather than
// cached, so a context torn down and recreated (cudaDeviceReset) never leaves
// a stale address behind.
int noalloc_scratch(double** out) {
  void* p = nullptr;
  cudaError_t err = cudaGetSymbolAddress(&p, g_lnamd_noalloc_scratch);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(g_lnamd_noalloc_scratch)");
  *out = static_cast<double*>(p);
  return MUSC_B200_OK;
}

}  // namespace

extern "C" int musc_b200_lnamd_noalloc(const void* tokens, int dtype, int n_images, int tokens_per_image,
                                       int channels, int n_radii, const int* radii, float* const* out,
                                       long long out_image_stride, long long out_patch_stride,
                                       int l2_normalize, musc_b200_stream stream) {
  if (n_images > kNoAllocMaxImages)
    return fail(MUSC_B200_ERR_INVALID,
                "lnamd_noalloc: n_images exceeds the static scratch limit of 2048 images per call "
                "(split the batch, or use musc_b200_lnamd with a workspace)");
  double* scratch = nullptr;
  MUSC_TRY(noalloc_scratch(&scratch));
  return musc_b200_lnamd(tokens, dtype, n_images, tokens_per_image, channels, n_radii, radii, out,
                         out_image_stride, out_patch_stride, l2_normalize, scratch,
                         sizeof(g_lnamd_noalloc_scratch), stream);
}
