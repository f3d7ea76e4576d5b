// MSM mutual scoring: models/modules/_MSM.py and models/modules/_MSM_gpu.py.
//
// Reference: compute_scores_fast / MSM (models/modules/_MSM.py:10-59) and the
// reference GPU driver models/modules/_MSM_gpu.py:701-830.
//
// Pipeline for one (layer, radius) bank z[N*P][C] fp32:
//   0. center_partial_kernel / center_finish_kernel: the pool's column sums and
//      smallest row norm (fixed order), from which mu = the column mean and the
//      gate |mu| <= 2 min |z|; the bank then holds the centred rows z - mu (same
//      distances, smaller split-fp16 error).
//   1. prep_bank_kernel: per row, a power-of-two scale 2^k putting max|z - mu|
//      in [2^14, 2^15), the split (z - mu)*2^k = hi + lo with hi = fp16(.) and
//      lo = fp16(. - hi) (together ~22 significant bits, fp32-class accuracy),
//      the fp32 squared norm (float64 accumulation), 2^-k and the residual norm.
//   2. nearest_kernel: persistent, warp-specialised tcgen05 GEMM.  Each tile
//      is 128 query rows x 256 reference rows; per 32-wide K slice TMA brings
//      A_hi, A_lo, B_hi, B_lo (48 KB) into a 4-deep shared-memory ring, and one
//      thread issues hi*hi + hi*lo + lo*hi (6 MMAs of 128x256x16) into a
//      fp32 TMEM accumulator (2 x 256 columns, double-buffered).  The pool
//      form runs as CTA pairs by default: 256 x 256 tiles, cta_group::2 MMAs of
//      256x256x16, each CTA loading half of A and half of B.  Four
//      epilogue warps read the accumulator (tcgen05.ld), form
//      d^2 = |q|^2 + |r|^2 - 2 q.r, keep a running minimum per reference
//      image segment and atomically lower nearest_sq[image][row].  The
//      N*P x N*P distance matrix never reaches memory.
//   3. trimmed_mean_kernel: per query row (four threads), the sum of the
//      smallest m distances by a binary search on the order-preserving bit
//      pattern of the squared minima (exact threshold, ties handled by count),
//      for m = rank_hi and rank_lo; score = mean of ranks [rank_lo, rank_hi)
//      rounded to fp32 like the reference's fp32 mean, stored as float64.
#include "common.cuh"
#include "nearest.cuh"
#include "tc.cuh"

#include <algorithm>
#include <cfloat>
#include <cstdlib>
#include <mutex>
#include <vector>

namespace musc {

// Implemented in refine.cu.
size_t refine_workspace_bytes(int n_images, long long q_rows, int channels);
size_t refine_min_workspace_bytes(int n_images, long long q_rows, int channels);
long long refine_rounds(int n_images, long long q_rows, int channels, size_t bytes);
int refine_launch(const void* bank, long long bank_rows, long long rows, int channels, int patches,
                  long long first_row, long long q_rows, int rank_hi, const unsigned long long* k1,
                  const unsigned int* m2, int n_parts, long long part_stride, long long table_rows,
                  float* exact, void* workspace, size_t workspace_bytes, cudaStream_t s);

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct BankLayout {
  size_t hi, lo, norm, inv, lnorm, total;
};

// Planes: hi, lo (fp16 [rows][C]), |z|^2, 2^-k and the residual norm |lo| 2^-k (fp32 [rows]),
// each 1024-byte aligned.
static BankLayout bank_layout(long long rows, int channels) {
  const size_t plane = align_up((size_t)rows * channels * 2, 1024);
  const size_t vec = align_up((size_t)rows * 4, 1024);
  return {0, plane, 2 * plane, 2 * plane + vec, 2 * plane + 2 * vec, 2 * plane + 3 * vec};
}

// ------------------------------------------------------------------ centring statistics
// Centring.  Squared distances are invariant under a common shift of every row, and
// the error of a split-fp16 dot product scales with |a| |b|, so the bank may hold
// z - mu with mu the pool's column mean: for features clustered around a common
// direction (L2-normalised ViT tokens lie in a narrow cone, |z - mu| ~ 0.05-0.4)
// the screen's error bound shrinks by |a - mu| |b - mu| / (|a| |b|).  The shift is
// applied only when |mu| <= 2 x the smallest row norm, which keeps |z - mu| <= 3 |z| for
// every row (a pool mixing rows of very different norms would otherwise lose the
// small rows' digits to the rounding of z - mu); L2-normalised rows always pass, and so
// do clusters far from the origin.
// mu and the gate must be the same for every row of a pool, so they are formed from
// statistics [C column sums, smallest squared row norm] that the ranks of a multi-GPU
// pool exchange (each over its own rows).  Everything is evaluated in a fixed order:
// the same rows give the same statistics, mu and gate bit for bit.
constexpr int kStatBlocks = 296;  // 2 per SM
constexpr int kStatWarps = 8;

// Warp w of block b takes rows (b * 8 + w) + k * 8G; lane l owns columns 4l + 128j.  Each
// warp accumulates its column sums (fp32) in its own shared-memory row and the smallest
// squared row norm in a register; the block then adds its 8 warp rows in order.
__global__ void __launch_bounds__(kStatWarps * 32)
center_partial_kernel(const float* __restrict__ z, long long rows, int channels, float* __restrict__ partial,
                      float* __restrict__ partial_min) {
  extern __shared__ float acc[];  // [kStatWarps][channels]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* mine = acc + (size_t)warp * channels;
  for (int c = lane * 4; c < channels; c += 128) *reinterpret_cast<float4*>(mine + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  float mn = __int_as_float(0x7f800000);
  for (long long row = (long long)blockIdx.x * kStatWarps + warp; row < rows;
       row += (long long)gridDim.x * kStatWarps) {
    const float* zr = z + row * channels;
    float ss = 0.f;
    for (int c = lane * 4; c < channels; c += 128) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(zr + c));
      float4 a = *reinterpret_cast<float4*>(mine + c);
      a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      *reinterpret_cast<float4*>(mine + c) = a;
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
    mn = fminf(mn, warp_sum(ss));
  }
  __shared__ float wmin[kStatWarps];
  if (lane == 0) wmin[warp] = mn;
  __syncthreads();
  for (int c = threadIdx.x; c < channels; c += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < kStatWarps; ++w) t += acc[(size_t)w * channels + c];
    partial[(size_t)blockIdx.x * channels + c] = t;
  }
  if (threadIdx.x == 0) {
    float m = wmin[0];
    for (int w = 1; w < kStatWarps; ++w) m = fminf(m, wmin[w]);
    partial_min[blockIdx.x] = m;
  }
}

// stats[c] = the block partials of column c added in block order (fp64); stats[C] = the
// smallest squared row norm (+inf for no rows), widened by 2^-20 against the fp32
// accumulation of the norms.
__global__ void center_finish_kernel(const float* __restrict__ partial, const float* __restrict__ partial_min,
                                     int blocks, int channels, double* __restrict__ stats) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < channels) {
    double s = 0.0;
    for (int b = 0; b < blocks; ++b) s += partial[(size_t)b * channels + c];
    stats[c] = s;
  }
  if (c == 0) {
    float m = partial_min[0];
    for (int b = 1; b < blocks; ++b) m = fminf(m, partial_min[b]);
    stats[channels] = (double)m * (1.0 - 0x1p-20);
  }
}

// ------------------------------------------------------------------ prep
constexpr int kPrepWarps = 8;
constexpr int kPrepBlocksPerSm = 8;

// Grid-stride over rows, one warp per row.  With `stats` ([n_parts][C + 1] fp64, or null
// for no centring) each block first forms mu[c] = (sum over the parts of the column sums)
// / count and the gate |mu|^2 <= 4 x the smallest squared row norm of all parts, both in a
// fixed order (every block of every rank reaches the same mu and decision); if the gate
// holds every row is split as (z - mu) 2^k, otherwise as z 2^k.
__global__ void __launch_bounds__(kPrepWarps * 32)
prep_bank_kernel(const float* __restrict__ z, long long rows, int channels, const double* __restrict__ stats,
                 int n_parts, double inv_count, __half* __restrict__ hi, __half* __restrict__ lo,
                 float* __restrict__ norm2, float* __restrict__ inv_scale, float* __restrict__ lo_norm) {
  extern __shared__ float mu[];
  __shared__ double red[kPrepWarps];
  double mu2 = 0.0;
  for (int c = threadIdx.x; c < channels; c += blockDim.x) {
    double s = 0.0;
    if (stats)
      for (int p = 0; p < n_parts; ++p) s += stats[(size_t)p * (channels + 1) + c];
    const float m = (float)(s * inv_count);
    mu[c] = m;
    mu2 += (double)m * m;
  }
  mu2 = warp_sum(mu2);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mu2;
  __syncthreads();
  if (stats) {
    double t = 0.0, mn = stats[channels];
    for (int w = 0; w < kPrepWarps; ++w) t += red[w];
    for (int p = 1; p < n_parts; ++p) mn = fmin(mn, stats[(size_t)p * (channels + 1) + channels]);
    if (!(t <= 4.0 * mn))  // gate closed: no shift (every thread reaches the same decision)
      for (int c = threadIdx.x; c < channels; c += blockDim.x) mu[c] = 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (long long row = (long long)blockIdx.x * kPrepWarps + (threadIdx.x >> 5); row < rows;
       row += (long long)gridDim.x * kPrepWarps) {
    const float* zr = z + row * channels;
    float m = 0.f;
    double ss = 0.0;
    for (int c = lane * 4; c < channels; c += 128) {
      float4 v = __ldg(reinterpret_cast<const float4*>(zr + c));
      const float4 u = *reinterpret_cast<const float4*>(mu + c);
      v.x -= u.x; v.y -= u.y; v.z -= u.z; v.w -= u.w;
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
    m = warp_max(m);
    ss = warp_sum(ss);
    int k = 0;
    if (m > 0.f) {
      k = 14 - ilogbf(m);
      k = k > 126 ? 126 : (k < -126 ? -126 : k);
    }
    const float s = ldexpf(1.f, k);
    __half* hr = hi + row * channels;
    __half* lr = lo + row * channels;
    double ll = 0.0;
    for (int c = lane * 4; c < channels; c += 128) {
      float4 v = __ldg(reinterpret_cast<const float4*>(zr + c));
      const float4 u = *reinterpret_cast<const float4*>(mu + c);
      v.x -= u.x; v.y -= u.y; v.z -= u.z; v.w -= u.w;
      const float x[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
      __half h[4], l[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        h[e] = __float2half_rn(x[e]);
        l[e] = __float2half_rn(x[e] - __half2float(h[e]));
        const double le = (double)__half2float(l[e]);
        ll += le * le;
      }
      uint2 ph, pl;
      __half2 t;
      t = __halves2half2(h[0], h[1]); ph.x = *reinterpret_cast<uint32_t*>(&t);
      t = __halves2half2(h[2], h[3]); ph.y = *reinterpret_cast<uint32_t*>(&t);
      t = __halves2half2(l[0], l[1]); pl.x = *reinterpret_cast<uint32_t*>(&t);
      t = __halves2half2(l[2], l[3]); pl.y = *reinterpret_cast<uint32_t*>(&t);
      *reinterpret_cast<uint2*>(hr + c) = ph;
      *reinterpret_cast<uint2*>(lr + c) = pl;
    }
    ll = warp_sum(ll);
    if (lane == 0) {
      norm2[row] = (float)ss;
      inv_scale[row] = ldexpf(1.f, -k);
      // Residual norm |z 2^k - hi| in original units, rounded up, for the screen's error
      // bound: lo carries z 2^k - hi to fp16 rounding (relative 2^-11, absolute 2^-25 for
      // subnormal lo), so |z 2^k - hi| <= |lo| (1 + 2^-10) + sqrt(C) 2^-24.
      lo_norm[row] = (float)((sqrt(ll) * (1.0 + 0x1p-10) + sqrt((double)channels) * 0x1p-24) * (1.0 + 1.0e-6)) *
                     ldexpf(1.f, -k);
    }
  }
}


// ------------------------------------------------------------------ fill
__global__ void fill_u32_kernel(unsigned int* p, long long n, unsigned int v) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    p[i] = v;
}

// ------------------------------------------------------------------ trimmed mean
// Four threads (a quad) per query row: each pass of the threshold search counts a
// quarter of the row's keys per thread and combines the counts with two shuffles,
// so the sequential search passes are four times shorter.  The CTA stages a
// [32 rows][pitch] transposed tile of the image-major table in shared memory
// (pitch = 4 mod 32 words, so a warp's 8 rows x 4 quad lanes hit 32 banks).
constexpr int kSelRows = 32;
constexpr int kSelThreads = 4 * kSelRows;

__device__ __forceinline__ int quad_sum(int v, unsigned mask) {
  v += __shfl_xor_sync(mask, v, 1);
  v += __shfl_xor_sync(mask, v, 2);
  return v;
}

__device__ __forceinline__ double quad_sum(double v, unsigned mask) {
  v += __shfl_xor_sync(mask, v, 1);
  v += __shfl_xor_sync(mask, v, 2);
  return v;
}

struct SelRow {
  const unsigned int* keys;  // this row's keys in shared memory
  int n, sub;
  unsigned mask;

  __device__ __forceinline__ int count_below(unsigned int t) const {
    int c = 0;
    for (int j = sub; j < n; j += 4) c += keys[j] < t ? 1 : 0;
    return quad_sum(c, mask);
  }
  __device__ __forceinline__ double sum_below(unsigned int t) const {
    double acc = 0.0;
    for (int j = sub; j < n; j += 4) {
      const unsigned int k = keys[j];
      if (k < t) acc += (double)sqrtf(__uint_as_float(k));
    }
    return quad_sum(acc, mask);
  }
  // Sum of the m smallest sqrt(values) (keys are non-negative float bit patterns,
  // so integer order is value order); a binary search for the m-th key, stopping
  // as soon as exactly m keys lie below the bracket's upper end.
  __device__ double sum_smallest(int m, unsigned int kmin, unsigned int kmax) const {
    if (m <= 0) return 0.0;
    const int k = m - 1;
    unsigned int lo = kmin;        // count(< lo) == 0 <= k
    unsigned int hi = kmax + 1u;   // count(< hi) == n > k
    while (hi - lo > 1u) {
      const unsigned int mid = lo + (hi - lo) / 2u;
      const int c = count_below(mid);
      if (c <= k) {
        lo = mid;
      } else {
        hi = mid;
        if (c == m) return sum_below(hi);
      }
    }
    // lo is the k-th smallest key: count(< lo) <= k < count(<= lo).
    const int c_lo = count_below(lo);
    return sum_below(lo) + (double)(m - c_lo) * (double)sqrtf(__uint_as_float(lo));
  }
};

__global__ void __launch_bounds__(kSelThreads)
trimmed_mean_kernel(const unsigned int* __restrict__ nearest, long long q_rows, int n, int pitch,
                    int rank_lo, int rank_hi, double* __restrict__ scores, const int* err) {
  extern __shared__ unsigned int tile[];  // [kSelRows][pitch]
  // A bounded wait that expired earlier on this device (device error word set and not yet
  // taken) means some table may be incomplete: every score becomes NaN instead.
  const bool poisoned = *reinterpret_cast<const volatile int*>(err) != 0;
  const long long row0 = (long long)blockIdx.x * kSelRows;
  for (int idx = threadIdx.x; idx < n * kSelRows; idx += kSelThreads) {
    const int j = idx / kSelRows, r = idx - j * kSelRows;
    const long long row = row0 + r;
    tile[r * pitch + j] = row < q_rows ? __ldg(nearest + (long long)j * q_rows + row) : 0u;
  }
  __syncthreads();
  const int r = threadIdx.x >> 2, sub = threadIdx.x & 3;
  const long long row = row0 + r;
  if (row >= q_rows) return;  // quad-uniform
  const unsigned lane = threadIdx.x & 31;
  SelRow sel{tile + r * pitch, n, sub, 0xFu << (lane & ~3u)};
  unsigned int kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int j = sub; j < n; j += 4) {
    const unsigned int k = sel.keys[j];
    kmin = k < kmin ? k : kmin;
    kmax = k > kmax ? k : kmax;
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    const unsigned int a = __shfl_xor_sync(sel.mask, kmin, o), b = __shfl_xor_sync(sel.mask, kmax, o);
    kmin = a < kmin ? a : kmin;
    kmax = b > kmax ? b : kmax;
  }
  const double hi = sel.sum_smallest(rank_hi, kmin, kmax);
  const double lo = sel.sum_smallest(rank_lo, kmin, kmax);
  if (sub == 0) scores[row] = poisoned ? __longlong_as_double(0x7FF8000000000000LL)
                                      : (double)(float)((hi - lo) / (double)(rank_hi - rank_lo));
}

// ------------------------------------------------------------------ host helpers
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* fn) {
  static std::mutex m;
  static EncodeTiledFn cached = nullptr;
  std::lock_guard<std::mutex> lock(m);
  if (!cached) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
      return fail(MUSC_B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    cached = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  *fn = cached;
  return MUSC_B200_OK;
}

int check_bank_args(long long rows, int channels) {
  if (rows <= 0 || channels <= 0) return fail(MUSC_B200_ERR_INVALID, "bank: requires rows > 0, channels > 0");
  if (channels % 8 != 0) return fail(MUSC_B200_ERR_INVALID, "bank: channels must be a multiple of 8");
  if (rows > 0x7FFFFFFFLL) return fail(MUSC_B200_ERR_INVALID, "bank: rows must fit in int32");
  return MUSC_B200_OK;
}

int trimmed_pitch(int n) { return n + (((4 - n) % 32) + 32) % 32; }  // >= n, == 4 (mod 32)

}  // namespace

// 2-D fp16 plane [rows][channels], box = k_box channels x box_rows; k_box 32 (64-byte rows,
// 64-byte swizzle) or 64 (128-byte rows, 128-byte swizzle).
int make_plane_map(CUtensorMap* map, const void* base, long long rows, int channels, int box_rows, int k_box) {
  EncodeTiledFn encode;
  MUSC_TRY(get_encode_fn(&encode));
  if (k_box != 32 && k_box != 64) return fail(MUSC_B200_ERR_INVALID, "make_plane_map: k_box must be 32 or 64");
  cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)channels * 2};
  cuuint32_t box[2] = {(cuuint32_t)k_box, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      k_box == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MUSC_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return MUSC_B200_OK;
}

// Balanced split of the symmetric tile list.  Tiles are visited in the
// kernel's linear order (groups of GROUP_M m-tiles, n outer, m inner); the
// needed tiles of one (group, n) column are counted in closed form from
// n_start(m), the first n-tile holding a column of a later image than the
// m-tile's first row.  Part k starts at the first column whose preceding
// count reaches total * k / parts.
static void sym_part_range(long long rows, int patches, int n_images, int num_m, int num_n, int tile_m,
                           int group_m, int part, int parts, long long* tile_begin, long long* tile_end) {
  using nearest::BN;
  const int GROUP_M = group_m;
  std::vector<int> n_start(num_m);
  for (int m = 0; m < num_m; ++m) {
    const long long img = (long long)m * tile_m / patches;
    if (img >= n_images - 1) {
      n_start[m] = num_n;
    } else {
      const long long need = (img + 1) * patches - BN + 1;  // n*BN + BN - 1 >= (img+1)*P
      n_start[m] = need <= 0 ? 0 : (int)((need + BN - 1) / BN);
    }
  }
  const int groups = (num_m + GROUP_M - 1) / GROUP_M;
  long long total = 0;
  for (int m = 0; m < num_m; ++m) total += num_n - n_start[m];
  const long long lin_total = (long long)num_m * num_n;
  auto start_of = [&](int k) -> long long {
    if (k <= 0) return 0;
    if (k >= parts) return lin_total;
    const long long target = total * k / parts;
    long long acc = 0;
    for (int g = 0; g < groups; ++g) {
      const int first_m = g * GROUP_M;
      const int gm = std::min(GROUP_M, num_m - first_m);
      int ptr = first_m;  // m in [first_m, ptr) have n_start <= n
      for (int n = 0; n < num_n; ++n) {
        while (ptr < first_m + gm && n_start[ptr] <= n) ++ptr;
        if (acc >= target) return (long long)g * GROUP_M * num_n + (long long)n * gm;
        acc += ptr - first_m;
      }
    }
    return lin_total;
  };
  *tile_begin = start_of(part);
  *tile_end = start_of(part + 1);
}

template <int MODE, bool PAIR>
static int set_attr_one() {
  return cudaFuncSetAttribute(nearest::nearest_kernel<MODE, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)nearest::smem_bytes<MODE, PAIR>()) == cudaSuccess
             ? MUSC_B200_OK
             : fail(MUSC_B200_ERR_CUDA, "cudaFuncSetAttribute(nearest_kernel) failed");
}

// Opt every instantiation of the nearest kernel in to its shared memory (once per device).
int set_nearest_smem_attrs() {
  static std::mutex m;
  static bool done[64] = {false};
  int dev = 0;
  MUSC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(m);
  if (dev >= 64 || !done[dev]) {
    using namespace nearest;
    MUSC_TRY((set_attr_one<DIRECTED, false>()));
    MUSC_TRY((set_attr_one<SYM, false>()));
    MUSC_TRY((set_attr_one<SYM, true>()));
    MUSC_TRY((set_attr_one<SCREEN, false>()));
    MUSC_TRY((set_attr_one<SCREEN, true>()));
    MUSC_TRY((set_attr_one<GATHER, false>()));
    if (dev < 64) done[dev] = true;
  }
  return MUSC_B200_OK;
}

// The symmetric pool kernels run as CTA pairs (cta_group::2) unless
// MUSC_B200_NEAREST_PAIR=0 selects the single-CTA kernels; both compute the
// same tables bit for bit.
static bool use_cta_pairs() {
  const char* e = std::getenv("MUSC_B200_NEAREST_PAIR");
  return !(e && e[0] == '0');
}

static int fill_table(float* table, long long count, cudaStream_t s) {
  fill_u32_kernel<<<1184, 256, 0, s>>>(reinterpret_cast<unsigned int*>(table), count, 0x7F7FFFFFu);
  return check_launch("fill_u32_kernel");
}

int nearest_launch(const void* query_bank, long long query_rows, long long query_first_row,
                   const void* ref_bank, long long ref_rows, int channels, int patches,
                   float* nearest_sq, cudaStream_t s) {
  using namespace nearest;
  const BankLayout ql = bank_layout(query_rows, channels);
  const BankLayout rl = bank_layout(ref_rows, channels);
  const uint8_t* qb = static_cast<const uint8_t*>(query_bank);
  const uint8_t* rb = static_cast<const uint8_t*>(ref_bank);
  CUtensorMap mqh, mql, mrh, mrl;
  MUSC_TRY(make_plane_map(&mqh, qb + ql.hi, query_rows, channels, CTA_M, BK));
  MUSC_TRY(make_plane_map(&mql, qb + ql.lo, query_rows, channels, CTA_M, BK));
  MUSC_TRY(make_plane_map(&mrh, rb + rl.hi, ref_rows, channels, BN, BK));
  MUSC_TRY(make_plane_map(&mrl, rb + rl.lo, ref_rows, channels, BN, BK));
  const int n_images = (int)(ref_rows / patches);
  MUSC_TRY(fill_table(nearest_sq, (long long)n_images * query_rows, s));
  Params p{};
  p.q_norm = reinterpret_cast<const float*>(qb + ql.norm);
  p.q_inv = reinterpret_cast<const float*>(qb + ql.inv);
  p.r_norm = reinterpret_cast<const float*>(rb + rl.norm);
  p.r_inv = reinterpret_cast<const float*>(rb + rl.inv);
  p.nearest = reinterpret_cast<unsigned int*>(nearest_sq);
  p.err = device_error_ptr();
  if (!p.err) return fail(MUSC_B200_ERR_CUDA, "nearest: device error word unavailable");
  p.q_rows = query_rows;
  p.r_rows = ref_rows;
  p.q_first_row = query_first_row;
  p.rows_per_block = query_rows;
  p.blocked = 0;
  p.patches = patches;
  p.n_images = n_images;
  p.num_kb = (channels + BK - 1) / BK;
  p.num_m = (int)((query_rows + CTA_M - 1) / CTA_M);
  p.num_n = (int)((ref_rows + BN - 1) / BN);
  p.tile_begin = 0;
  p.tile_end = (long long)p.num_m * p.num_n;
  p.sched = nullptr;  // static schedule
  MUSC_TRY(set_nearest_smem_attrs());
  const int grid = (int)std::min<long long>(p.tile_end, sm_count());
  nearest_kernel<DIRECTED, false><<<grid, Cfg<DIRECTED, false>::THREADS, smem_bytes<DIRECTED, false>(), s>>>(
      mqh, mql, mrh, mrl, p);
  return check_launch("nearest_kernel<directed>");
}

// Launch a symmetric pool kernel (SYM or SCREEN) over part `part` of `parts` of the
// tile list; p holds the outputs, the caller has filled them.
template <int MODE>
static int pool_kernel_launch(const void* bank, long long bank_rows, long long rows, int channels, int patches,
                              int part, int parts, int max_ctas, nearest::Params& p, cudaStream_t s) {
  using namespace nearest;
  const BankLayout l = bank_layout(bank_rows, channels);
  const uint8_t* b = static_cast<const uint8_t*>(bank);
  const bool pair = use_cta_pairs();
  const int b_box = pair ? Cfg<MODE, true>::CTA_N : Cfg<MODE, false>::CTA_N;
  CUtensorMap mah, mal, mbh, mbl;
  const int kb = Cfg<MODE, false>::KB;
  MUSC_TRY(make_plane_map(&mah, b + l.hi, rows, channels, CTA_M, kb));
  MUSC_TRY(make_plane_map(&mal, b + l.lo, rows, channels, CTA_M, kb));
  MUSC_TRY(make_plane_map(&mbh, b + l.hi, rows, channels, b_box, kb));
  MUSC_TRY(make_plane_map(&mbl, b + l.lo, rows, channels, b_box, kb));
  p.q_norm = p.r_norm = reinterpret_cast<const float*>(b + l.norm);
  p.q_inv = p.r_inv = reinterpret_cast<const float*>(b + l.inv);
  p.err = device_error_ptr();
  if (!p.err) return fail(MUSC_B200_ERR_CUDA, "nearest_pool: device error word unavailable");
  p.q_rows = p.r_rows = rows;
  p.q_first_row = 0;
  p.patches = patches;
  p.n_images = (int)(rows / patches);
  p.num_kb = (channels + kb - 1) / kb;
  const int tile_m = pair ? Cfg<MODE, true>::TILE_M : Cfg<MODE, false>::TILE_M;
  const int group_m = pair ? Cfg<MODE, true>::GROUP_M : Cfg<MODE, false>::GROUP_M;
  p.num_m = (int)((rows + tile_m - 1) / tile_m);
  p.num_n = (int)((rows + BN - 1) / BN);
  sym_part_range(rows, patches, p.n_images, p.num_m, p.num_n, tile_m, group_m, part, parts, &p.tile_begin,
                 &p.tile_end);
  if (p.tile_end <= p.tile_begin) return MUSC_B200_OK;  // nothing to do for this part
  MUSC_TRY(set_nearest_smem_attrs());
  const int sms = sm_count();
  const int ctas = max_ctas > 0 && max_ctas < sms ? max_ctas : sms;
  if (!pair) {
    nearest_kernel<MODE, false><<<ctas, Cfg<MODE, false>::THREADS, smem_bytes<MODE, false>(), s>>>(mah, mal, mbh,
                                                                                                   mbl, p);
    return check_launch(MODE == SCREEN ? "nearest_kernel<screen>" : "nearest_kernel<symmetric>");
  }
  // One cluster of two CTAs per SM pair, as many as can be resident at once.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(Cfg<MODE, true>::THREADS);
  cfg.dynamicSmemBytes = smem_bytes<MODE, true>();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  MUSC_CUDA(cudaOccupancyMaxActiveClusters(&clusters, nearest_kernel<MODE, true>, &cfg));
  if (clusters <= 0) return fail(MUSC_B200_ERR_CUDA, "nearest_pool: no CTA pair fits on this device");
  clusters = std::min(clusters, std::max(1, ctas / 2));
  cfg.gridDim = dim3(2 * clusters);
  MUSC_CUDA(cudaLaunchKernelEx(&cfg, nearest_kernel<MODE, true>, mah, mal, mbh, mbl, p));
  return check_launch(MODE == SCREEN ? "nearest_kernel<screen, pair>" : "nearest_kernel<symmetric, pair>");
}

static size_t table_entries(long long rows, int patches, long long rows_per_block) {
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  return (size_t)blocks * (size_t)(rows / patches) * (size_t)rows_per_block;
}

int nearest_pool_launch(const void* bank, long long bank_rows, long long rows, int channels, int patches,
                        int part, int parts, long long rows_per_block, int max_ctas, float* nearest_sq,
                        cudaStream_t s) {
  const size_t table = table_entries(rows, patches, rows_per_block);
  MUSC_TRY(fill_table(nearest_sq, (long long)table, s));
  // The scheduler counter lives in the 256 bytes after the table (musc_b200_nearest_pool_bytes).
  unsigned long long* sched = reinterpret_cast<unsigned long long*>(
      reinterpret_cast<uint8_t*>(nearest_sq) + (table * sizeof(float) + 255) / 256 * 256);
  MUSC_CUDA(cudaMemsetAsync(sched, 0, sizeof(unsigned long long), s));
  nearest::Params p{};
  p.nearest = reinterpret_cast<unsigned int*>(nearest_sq);
  p.sched = sched;
  p.rows_per_block = rows_per_block;
  p.blocked = rows_per_block < rows ? 1 : 0;
  return pool_kernel_launch<nearest::SYM>(bank, bank_rows, rows, channels, patches, part, parts, max_ctas, p, s);
}

// Screen tables: k1 [blocks][N][rpb] uint64 and m2 (same shape, uint32), filled with
// 0xFF bytes first ("unset", above every value); the scheduler word is zeroed.
int screen_pool_launch(const void* bank, long long bank_rows, long long rows, int channels, int patches,
                       int part, int parts, long long rows_per_block, int max_ctas, unsigned long long* k1,
                       unsigned int* m2, unsigned long long* sched, cudaStream_t s) {
  const size_t n = table_entries(rows, patches, rows_per_block);
  MUSC_CUDA(cudaMemsetAsync(k1, 0xFF, n * sizeof(unsigned long long), s));
  MUSC_CUDA(cudaMemsetAsync(m2, 0xFF, n * sizeof(unsigned int), s));
  MUSC_CUDA(cudaMemsetAsync(sched, 0, sizeof(unsigned long long), s));
  nearest::Params p{};
  p.k1 = k1;
  p.m2 = m2;
  p.sched = sched;
  p.rows_per_block = rows_per_block;
  p.blocked = rows_per_block < rows ? 1 : 0;
  return pool_kernel_launch<nearest::SCREEN>(bank, bank_rows, rows, channels, patches, part, parts, max_ctas, p,
                                             s);
}

int trimmed_launch(const float* nearest_sq, long long query_rows, int n_images, int rank_lo, int rank_hi,
                   double* scores, cudaStream_t s) {
  const int pitch = trimmed_pitch(n_images);
  const size_t smem = (size_t)kSelRows * pitch * 4;
  if ((long long)smem > smem_optin() - 1024)
    return fail(MUSC_B200_ERR_INVALID, "trimmed_mean: too many images for shared memory (N <= ~1700)");
  MUSC_CUDA(cudaFuncSetAttribute(trimmed_mean_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int* err = device_error_ptr();
  if (!err) return fail(MUSC_B200_ERR_CUDA, "trimmed_mean: device error word unavailable");
  const long long blocks = (query_rows + kSelRows - 1) / kSelRows;
  trimmed_mean_kernel<<<(unsigned)blocks, kSelThreads, smem, s>>>(
      reinterpret_cast<const unsigned int*>(nearest_sq), query_rows, n_images, pitch, rank_lo, rank_hi, scores,
      err);
  return check_launch("trimmed_mean_kernel");
}

}  // namespace musc

using namespace musc;

extern "C" size_t musc_b200_bank_bytes(long long rows, int channels) {
  if (rows <= 0 || channels <= 0) return 0;
  return bank_layout(rows, channels).total;
}

// Workspace of musc_b200_center_stats: fp32 block partials [G][C] and block minima [G].
extern "C" size_t musc_b200_center_stats_bytes(int channels) {
  if (channels <= 0) return 0;
  return align_up((size_t)kStatBlocks * channels * sizeof(float), 256) + kStatBlocks * sizeof(float);
}

extern "C" int musc_b200_center_stats(const float* z, long long rows, int channels, double* stats, void* workspace,
                                      size_t workspace_bytes, musc_b200_stream stream) {
  if (rows < 0 || channels <= 0 || channels % 8 != 0)
    return fail(MUSC_B200_ERR_INVALID, "center_stats: requires rows >= 0 and channels a positive multiple of 8");
  if (!stats || !workspace || (rows > 0 && !z)) return fail(MUSC_B200_ERR_INVALID, "center_stats: null pointer");
  if ((rows > 0 && reinterpret_cast<uintptr_t>(z) % 16 != 0) || reinterpret_cast<uintptr_t>(stats) % 8 != 0 ||
      reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
    return fail(MUSC_B200_ERR_INVALID, "center_stats: z and workspace must be 16-byte and stats 8-byte aligned");
  const size_t smem = (size_t)kStatWarps * channels * sizeof(float);
  if (smem > 200 * 1024) return fail(MUSC_B200_ERR_INVALID, "center_stats: channels above 6400");
  if (workspace_bytes < musc_b200_center_stats_bytes(channels))
    return fail(MUSC_B200_ERR_WORKSPACE, "center_stats: workspace smaller than musc_b200_center_stats_bytes");
  MUSC_TRY(require_sm100());
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(center_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  MUSC_CUDA(attr);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(workspace);
  float* pmin = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         align_up((size_t)kStatBlocks * channels * sizeof(float), 256));
  center_partial_kernel<<<kStatBlocks, kStatWarps * 32, smem, s>>>(z, rows, channels, partial, pmin);
  MUSC_TRY(check_launch("center_partial_kernel"));
  center_finish_kernel<<<(channels + 255) / 256, 256, 0, s>>>(partial, pmin, kStatBlocks, channels, stats);
  return check_launch("center_finish_kernel");
}

static int prep_bank_launch(const float* z, long long rows, int channels, const double* stats, int n_parts,
                            long long count, void* bank, size_t bank_bytes, cudaStream_t s) {
  MUSC_TRY(check_bank_args(rows, channels));
  if (!z || !bank) return fail(MUSC_B200_ERR_INVALID, "prep_bank: null pointer");
  if (reinterpret_cast<uintptr_t>(z) % 16 != 0 || reinterpret_cast<uintptr_t>(bank) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "prep_bank: z must be 16-byte and bank 1024-byte aligned");
  if (stats && (n_parts <= 0 || count <= 0 || reinterpret_cast<uintptr_t>(stats) % 8 != 0))
    return fail(MUSC_B200_ERR_INVALID, "prep_bank: centring needs n_parts > 0, count > 0 and 8-byte aligned stats");
  const BankLayout l = bank_layout(rows, channels);
  if (bank_bytes < l.total) return fail(MUSC_B200_ERR_WORKSPACE, "prep_bank: bank smaller than musc_b200_bank_bytes");
  const size_t smem = (size_t)channels * sizeof(float);
  if (smem > 200 * 1024) return fail(MUSC_B200_ERR_INVALID, "prep_bank: channels above 51200");
  MUSC_TRY(require_sm100());
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(prep_bank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  MUSC_CUDA(attr);
  const int sms = std::max(1, sm_count());
  uint8_t* b = static_cast<uint8_t*>(bank);
  const long long need = (rows + kPrepWarps - 1) / kPrepWarps;
  const long long blocks = std::min<long long>(need, (long long)sms * kPrepBlocksPerSm);
  prep_bank_kernel<<<(unsigned)blocks, kPrepWarps * 32, smem, s>>>(
      z, rows, channels, stats, stats ? n_parts : 0, stats ? 1.0 / (double)count : 0.0,
      reinterpret_cast<__half*>(b + l.hi), reinterpret_cast<__half*>(b + l.lo),
      reinterpret_cast<float*>(b + l.norm), reinterpret_cast<float*>(b + l.inv), reinterpret_cast<float*>(b + l.lnorm));
  return check_launch("prep_bank_kernel");
}

extern "C" int musc_b200_prep_bank(const float* z, long long rows, int channels, void* bank,
                                   size_t bank_bytes, musc_b200_stream stream) {
  return prep_bank_launch(z, rows, channels, nullptr, 0, 0, bank, bank_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int musc_b200_prep_bank_centered(const float* z, long long rows, int channels, const double* stats,
                                            int n_parts, long long count, void* bank, size_t bank_bytes,
                                            musc_b200_stream stream) {
  if (!stats) return fail(MUSC_B200_ERR_INVALID, "prep_bank_centered: null stats");
  return prep_bank_launch(z, rows, channels, stats, n_parts, count, bank, bank_bytes,
                          reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int musc_b200_nearest(const void* query_bank, long long query_rows, long long query_first_row,
                                 const void* ref_bank, long long ref_rows, int channels,
                                 int patches_per_image, float* nearest_sq, musc_b200_stream stream) {
  MUSC_TRY(check_bank_args(query_rows, channels));
  MUSC_TRY(check_bank_args(ref_rows, channels));
  if (!query_bank || !ref_bank || !nearest_sq) return fail(MUSC_B200_ERR_INVALID, "nearest: null pointer");
  if (reinterpret_cast<uintptr_t>(query_bank) % 1024 != 0 || reinterpret_cast<uintptr_t>(ref_bank) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "nearest: banks must be 1024-byte aligned");
  if (patches_per_image <= 0 || ref_rows % patches_per_image != 0)
    return fail(MUSC_B200_ERR_INVALID, "nearest: ref_rows must be a multiple of patches_per_image");
  if (query_first_row < 0 || query_first_row + query_rows > ref_rows)
    return fail(MUSC_B200_ERR_INVALID, "nearest: query rows must lie inside the reference pool");
  if (reinterpret_cast<uintptr_t>(nearest_sq) % 4 != 0)
    return fail(MUSC_B200_ERR_INVALID, "nearest: output must be 4-byte aligned");
  MUSC_TRY(require_sm100());
  return nearest_launch(query_bank, query_rows, query_first_row, ref_bank, ref_rows, channels,
                        patches_per_image, nearest_sq, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t musc_b200_nearest_pool_bytes(long long rows, int patches_per_image,
                                               long long rows_per_block) {
  if (rows <= 0 || patches_per_image <= 0 || rows_per_block <= 0) return 0;
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  const size_t table = (size_t)blocks * (size_t)(rows / patches_per_image) * (size_t)rows_per_block * sizeof(float);
  return (table + 255) / 256 * 256 + 256;  // + the dynamic scheduler's counter
}

extern "C" int musc_b200_bank_layout(long long rows, int channels, size_t* plane_offsets) {
  MUSC_TRY(check_bank_args(rows, channels));
  if (!plane_offsets) return fail(MUSC_B200_ERR_INVALID, "bank_layout: null output");
  const BankLayout l = bank_layout(rows, channels);
  plane_offsets[0] = l.hi;
  plane_offsets[1] = l.lo;
  plane_offsets[2] = l.norm;
  plane_offsets[3] = l.inv;
  plane_offsets[4] = l.lnorm;
  return MUSC_B200_OK;
}

extern "C" int musc_b200_nearest_pool(const void* bank, long long bank_rows, long long rows, int channels,
                                      int patches_per_image, int part, int n_parts, long long rows_per_block,
                                      int max_ctas, float* nearest_sq, musc_b200_stream stream) {
  MUSC_TRY(check_bank_args(rows, channels));
  if (bank_rows < rows) return fail(MUSC_B200_ERR_INVALID, "nearest_pool: bank_rows must be >= rows");
  if (!bank || !nearest_sq) return fail(MUSC_B200_ERR_INVALID, "nearest_pool: null pointer");
  if (reinterpret_cast<uintptr_t>(bank) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "nearest_pool: bank must be 1024-byte aligned");
  if (patches_per_image <= 0 || rows % patches_per_image != 0 || rows / patches_per_image < 2)
    return fail(MUSC_B200_ERR_INVALID, "nearest_pool: rows must hold N >= 2 whole images");
  if (n_parts <= 0 || part < 0 || part >= n_parts)
    return fail(MUSC_B200_ERR_INVALID, "nearest_pool: requires 0 <= part < n_parts");
  if (rows_per_block <= 0 || rows_per_block % patches_per_image != 0)
    return fail(MUSC_B200_ERR_INVALID, "nearest_pool: rows_per_block must be a positive multiple of P");
  if (reinterpret_cast<uintptr_t>(nearest_sq) % 4 != 0)
    return fail(MUSC_B200_ERR_INVALID, "nearest_pool: output must be 4-byte aligned");
  MUSC_TRY(require_sm100());
  return nearest_pool_launch(bank, bank_rows, rows, channels, patches_per_image, part, n_parts, rows_per_block,
                             max_ctas, nearest_sq, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int musc_b200_trimmed_mean(const float* nearest_sq, long long query_rows, int n_images,
                                      int rank_lo, int rank_hi, double* scores, musc_b200_stream stream) {
  if (!nearest_sq || !scores) return fail(MUSC_B200_ERR_INVALID, "trimmed_mean: null pointer");
  if (query_rows <= 0 || n_images < 2)
    return fail(MUSC_B200_ERR_INVALID, "trimmed_mean: requires rows > 0 and N >= 2");
  if (!(0 <= rank_lo && rank_lo < rank_hi && rank_hi <= n_images - 1))
    return fail(MUSC_B200_ERR_INVALID, "Require valid nonempty trimmed ranks 0<=a<b<=N-1.");
  if (query_rows > 0x7FFFFFFFLL * 32) return fail(MUSC_B200_ERR_INVALID, "trimmed_mean: too many rows");
  MUSC_TRY(require_sm100());
  return trimmed_launch(nearest_sq, query_rows, n_images, rank_lo, rank_hi, scores,
                        reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int musc_b200_screen_pool(const void* bank, long long bank_rows, long long rows, int channels,
                                     int patches_per_image, int part, int n_parts, long long rows_per_block,
                                     int max_ctas, void* k1, void* m2, void* sched_word, musc_b200_stream stream) {
  MUSC_TRY(check_bank_args(rows, channels));
  if (bank_rows < rows) return fail(MUSC_B200_ERR_INVALID, "screen_pool: bank_rows must be >= rows");
  if (!bank || !k1 || !m2 || !sched_word) return fail(MUSC_B200_ERR_INVALID, "screen_pool: null pointer");
  if (reinterpret_cast<uintptr_t>(bank) % 1024 != 0 || reinterpret_cast<uintptr_t>(k1) % 8 != 0 ||
      reinterpret_cast<uintptr_t>(m2) % 4 != 0 || reinterpret_cast<uintptr_t>(sched_word) % 8 != 0)
    return fail(MUSC_B200_ERR_INVALID, "screen_pool: bank must be 1024-byte aligned, k1 and the word 8-byte, m2 4-byte");
  if (patches_per_image <= 0 || rows % patches_per_image != 0 || rows / patches_per_image < 2)
    return fail(MUSC_B200_ERR_INVALID, "screen_pool: rows must hold N >= 2 whole images");
  if (patches_per_image > (1 << 24))
    return fail(MUSC_B200_ERR_INVALID, "screen_pool: patches_per_image must be below 2^24");
  if (n_parts <= 0 || part < 0 || part >= n_parts)
    return fail(MUSC_B200_ERR_INVALID, "screen_pool: requires 0 <= part < n_parts");
  if (rows_per_block <= 0 || rows_per_block % patches_per_image != 0)
    return fail(MUSC_B200_ERR_INVALID, "screen_pool: rows_per_block must be a positive multiple of P");
  MUSC_TRY(require_sm100());
  return screen_pool_launch(bank, bank_rows, rows, channels, patches_per_image, part, n_parts, rows_per_block,
                            max_ctas, static_cast<unsigned long long*>(k1), static_cast<unsigned int*>(m2),
                            static_cast<unsigned long long*>(sched_word), reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t musc_b200_refine_bytes(int n_images, long long query_rows, int channels) {
  if (n_images <= 0 || query_rows <= 0 || channels <= 0) return 0;
  return refine_workspace_bytes(n_images, query_rows, channels);
}

extern "C" int musc_b200_refine_launches(int n_images, long long query_rows, int channels,
                                         size_t workspace_bytes) {
  if (n_images <= 0 || query_rows <= 0 || channels <= 0) return 0;
  return (int)(2 + 3 * refine_rounds(n_images, query_rows, channels, workspace_bytes));
}

extern "C" size_t musc_b200_refine_min_bytes(int n_images, long long query_rows, int channels) {
  if (n_images <= 0 || query_rows <= 0 || channels <= 0) return 0;
  return refine_min_workspace_bytes(n_images, query_rows, channels);
}

extern "C" int musc_b200_refine(const void* bank, long long bank_rows, long long rows, int channels,
                                int patches_per_image, long long first_row, long long query_rows, int rank_hi,
                                const void* k1, const void* m2, int n_partials, long long partial_stride,
                                long long table_rows, float* exact_sq, void* workspace, size_t workspace_bytes,
                                musc_b200_stream stream) {
  MUSC_TRY(check_bank_args(rows, channels));
  if (!bank || !k1 || !m2 || !exact_sq || !workspace) return fail(MUSC_B200_ERR_INVALID, "refine: null pointer");
  if (bank_rows < rows) return fail(MUSC_B200_ERR_INVALID, "refine: bank_rows must be >= rows");
  if (reinterpret_cast<uintptr_t>(bank) % 1024 != 0 || reinterpret_cast<uintptr_t>(workspace) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "refine: bank and workspace must be 1024-byte aligned");
  if (reinterpret_cast<uintptr_t>(k1) % 8 != 0 || reinterpret_cast<uintptr_t>(m2) % 4 != 0 ||
      reinterpret_cast<uintptr_t>(exact_sq) % 4 != 0)
    return fail(MUSC_B200_ERR_INVALID, "refine: misaligned table");
  if (patches_per_image <= 0 || rows % patches_per_image != 0 || rows / patches_per_image < 2)
    return fail(MUSC_B200_ERR_INVALID, "refine: rows must hold N >= 2 whole images");
  const int n_images = (int)(rows / patches_per_image);
  if (!(rank_hi >= 1 && rank_hi <= n_images - 1))
    return fail(MUSC_B200_ERR_INVALID, "refine: requires 1 <= rank_hi <= N-1");
  if (query_rows <= 0 || first_row < 0 || first_row + query_rows > rows || table_rows < query_rows)
    return fail(MUSC_B200_ERR_INVALID, "refine: query rows must lie in the pool and in the tables");
  if (n_partials <= 0 || (n_partials > 1 && partial_stride < (long long)n_images * table_rows))
    return fail(MUSC_B200_ERR_INVALID, "refine: partial tables overlap");
  if (workspace_bytes < refine_min_workspace_bytes(n_images, query_rows, channels))
    return fail(MUSC_B200_ERR_WORKSPACE, "refine: workspace smaller than musc_b200_refine_min_bytes");
  MUSC_TRY(require_sm100());
  return refine_launch(bank, bank_rows, rows, channels, patches_per_image, first_row, query_rows, rank_hi,
                       static_cast<const unsigned long long*>(k1), static_cast<const unsigned int*>(m2), n_partials,
                       partial_stride, table_rows, exact_sq, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream));
}

// MUSC_B200_MSM_EXACT=1 in the environment selects the 3-pass symmetric kernel for every
// bank instead of the screen + refinement (same results within fp32 rounding).
static bool use_exact_pool() {
  const char* e = std::getenv("MUSC_B200_MSM_EXACT");
  return e && e[0] == '1';
}

// Scratch of one bank's MSM after the bank itself: the exact path's table, or the screen
// tables, the exact table and the refinement's workspace.
static size_t msm_scratch_bytes(int n, int p, int c) {
  const long long rows = (long long)n * p;
  const size_t exact_path = align_up(musc_b200_nearest_pool_bytes(rows, p, rows), 1024);
  const size_t entries = (size_t)n * rows;
  const size_t deferred = align_up(entries * 8, 1024) + align_up(entries * 4, 1024) + 1024 +
                          align_up(entries * sizeof(float), 1024) + align_up(refine_workspace_bytes(n, rows, c), 1024);
  return std::max(exact_path, deferred);
}

// One prepared bank -> scores (the whole pool is one part).
int msm_bank(const void* bank, int n, int p, int c, int rank_lo, int rank_hi, double* scores, void* scratch,
             cudaStream_t s) {
  const long long rows = (long long)n * p;
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  musc_b200_stream st = reinterpret_cast<musc_b200_stream>(s);
  if (use_exact_pool()) {
    float* table = reinterpret_cast<float*>(ws);
    MUSC_TRY(musc_b200_nearest_pool(bank, rows, rows, c, p, 0, 1, rows, 0, table, st));
    return musc_b200_trimmed_mean(table, rows, n, rank_lo, rank_hi, scores, st);
  }
  const size_t entries = (size_t)n * rows;
  uint8_t* k1 = ws;
  uint8_t* m2 = k1 + align_up(entries * 8, 1024);
  uint8_t* word = m2 + align_up(entries * 4, 1024);
  float* exact = reinterpret_cast<float*>(word + 1024);
  uint8_t* rws = word + 1024 + align_up(entries * sizeof(float), 1024);
  MUSC_TRY(musc_b200_screen_pool(bank, rows, rows, c, p, 0, 1, rows, 0, k1, m2, word, st));
  MUSC_TRY(musc_b200_refine(bank, rows, rows, c, p, 0, rows, rank_hi, k1, m2, 1, 0, rows, exact, rws,
                            refine_workspace_bytes(n, rows, c), st));
  return musc_b200_trimmed_mean(exact, rows, n, rank_lo, rank_hi, scores, st);
}

size_t msm_bank_scratch_bytes(int n, int p, int c) { return msm_scratch_bytes(n, p, c); }

// The centring statistics and their workspace, after the bank and the MSM scratch.
static size_t msm_center_bytes(int c) {
  return align_up((size_t)(c + 1) * sizeof(double), 1024) + align_up(musc_b200_center_stats_bytes(c), 1024);
}

extern "C" size_t musc_b200_msm_workspace_bytes(int n, int p, int c) {
  if (n <= 0 || p <= 0 || c <= 0) return 0;
  const long long rows = (long long)n * p;
  return bank_layout(rows, c).total + align_up(msm_scratch_bytes(n, p, c), 1024) + msm_center_bytes(c);
}

extern "C" int musc_b200_msm(const float* z, int n, int p, int c, int rank_lo, int rank_hi, double* scores,
                             void* workspace, size_t workspace_bytes, musc_b200_stream stream) {
  if (!z || !scores || !workspace) return fail(MUSC_B200_ERR_INVALID, "msm: null pointer");
  if (!(n >= 2 && p > 0 && c > 0)) return fail(MUSC_B200_ERR_INVALID, "Requires N>=2, P>0, C>0.");
  if (!(0 <= rank_lo && rank_lo < rank_hi && rank_hi <= n - 1))
    return fail(MUSC_B200_ERR_INVALID, "Require valid nonempty trimmed ranks 0<=a<b<=N-1.");
  const long long rows = (long long)n * p;
  MUSC_TRY(check_bank_args(rows, c));
  if (workspace_bytes < musc_b200_msm_workspace_bytes(n, p, c))
    return fail(MUSC_B200_ERR_WORKSPACE, "msm: workspace smaller than musc_b200_msm_workspace_bytes");
  if (reinterpret_cast<uintptr_t>(workspace) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "msm: workspace must be 1024-byte aligned");
  const size_t bank_size = bank_layout(rows, c).total;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* center = ws + bank_size + align_up(msm_scratch_bytes(n, p, c), 1024);
  double* stats = reinterpret_cast<double*>(center);
  uint8_t* partial = center + align_up((size_t)(c + 1) * sizeof(double), 1024);
  MUSC_TRY(musc_b200_center_stats(z, rows, c, stats, partial, musc_b200_center_stats_bytes(c), stream));
  MUSC_TRY(musc_b200_prep_bank_centered(z, rows, c, stats, 1, rows, ws, bank_size, stream));
  return msm_bank(ws, n, p, c, rank_lo, rank_hi, scores, ws + bank_size, reinterpret_cast<cudaStream_t>(stream));
}
