// Exact minima from the screened pool pass: the rank-deferred half of MSM.
//
// The reference's GPU driver (models/modules/_MSM_gpu.py:701-830) screens every
// (query patch, reference image) pair with fp16 dot products and certified error
// bounds, takes the rank threshold of the upper bounds (kthvalue, :770), evaluates
// exactly only the pairs that can reach the trimmed ranks (rank_anchor_rows,
// :585-629) and their recorded candidates (rank_candidates, :471-487).  This file
// does the same job on the screen tables of nearest_kernel<SCREEN>:
//
//   1. image_bounds_kernel: per reference image the largest |z|^2 and residual
//      norm (the inputs of the error bound).
//   2. refine_kernel: per query row, the screened minimum of every image (its
//      value, the patch attaining it, and the second-smallest value over the
//      image's other patches, combined over the partial tables of a multi-GPU
//      split) gives certified bounds [L_j, U_j] on the exact minimum.  The
//      threshold T = the rank_hi-th smallest U_j; images with L_j > T lie beyond
//      the trimmed ranks and get FLT_MAX (the interval average never reaches
//      them).  For every other image the exact distance D to the screened argmin
//      is evaluated in fp32 from the bank's hi + lo planes; when the second
//      smallest screened value, lowered by its error bound, is still >= D, no
//      other patch can be closer and D is the exact minimum.  Otherwise D is
//      stored as an upper bound and the row is queued for image j.
//   3. fallback_plan_kernel / fallback_gather_kernel: the queued rows are
//      copied, image by image, into a staging bank (128-row tiles), and
//      nearest_kernel<GATHER> evaluates each tile exactly (3-pass split fp16)
//      against its image, lowering the table entries with atomic minima -- in
//      rounds of at most the staging bank's capacity, until the queue is drained.
// The interval average then runs on the exact table as before.
//
// Error bound of a screened distance (original units, a = query, b = reference,
// H = |hi| 2^-k, L = |lo| 2^-k (1 + 2^-11) the residual norm, K the padded
// channel count, gamma = K u / (1 - K u) with u = 2^-23):
//   |d2~ - d2| <= 2 (H_a L_b + L_a H_b + L_a L_b + gamma H_a H_b)
//                 + 2^-21 (|a|^2 + |b|^2),
// the split residual terms, the fp32 accumulation of the fp16 products and
// the fp32 evaluation of |a|^2 + |b|^2 - 2 a.b.  The keys store the value
// with its low 8 mantissa bits replaced, a relative change below 2^-15; the
// bounds allow 2^-14.
#include "common.cuh"
#include "nearest.cuh"

#include <algorithm>
#include <cfloat>
#include <cstdlib>
#include <vector>

namespace musc {

// Implemented in msm.cu.
int make_plane_map(CUtensorMap* map, const void* base, long long rows, int channels, int box_rows, int k_box);
int set_nearest_smem_attrs();

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr int kRefineThreads = 256;     // 8 warps, one per row
constexpr int kRefineMaxThreads = 768;  // large pools: 24 warps sharing fewer rows

struct BankPlanes {
  const __half* hi;
  const __half* lo;
  const float* norm;
  const float* inv;
  const float* lnorm;
};

// Same layout as the bank of msm.cu (planes hi, lo, |z|^2, 2^-k, residual norm).
BankPlanes bank_planes(const void* bank, long long bank_rows, int channels) {
  const size_t plane = align_up((size_t)bank_rows * channels * 2, 1024);
  const size_t vec = align_up((size_t)bank_rows * 4, 1024);
  const uint8_t* b = static_cast<const uint8_t*>(bank);
  return {reinterpret_cast<const __half*>(b), reinterpret_cast<const __half*>(b + plane),
          reinterpret_cast<const float*>(b + 2 * plane), reinterpret_cast<const float*>(b + 2 * plane + vec),
          reinterpret_cast<const float*>(b + 2 * plane + 2 * vec)};
}

// Workspace of one refinement (rank-local rows): the queue, the staging bank and the
// small planning arrays.  Offsets in bytes, each 1024-aligned.  The staging bank holds
// `cap` rows; the fallback stages the queue in rounds of at most `cap` rows, so any
// capacity >= 128 rows works (a smaller workspace means more rounds).
struct RefineLayout {
  size_t bounds, counts, lists, words, tile_img, tile_off, row_map, s_norm, s_inv, s_hi, s_lo, total;
  long long cap;  // staging rows (multiple of 128)
};

constexpr long long kMaxStagingRows = 1LL << 21;  // 2 M rows: 8 GB of hi + lo at C = 1024

// Default staging capacity: 4 queued images per row on average (far above the typical
// certified fraction), at most every pair plus padding, at most kMaxStagingRows.
long long default_staging_rows(int n_images, long long q_rows) {
  const long long full = (long long)n_images * q_rows + 128LL * n_images;
  long long cap = std::min(4 * q_rows + 128LL * n_images, full);
  cap = std::min(cap, kMaxStagingRows);
  return std::max(128LL, (cap + 127) / 128 * 128);
}

RefineLayout refine_layout(int n_images, long long q_rows, int channels, long long cap) {
  RefineLayout l;
  l.cap = cap;
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = align_up(o + bytes, 1024); return at; };
  l.bounds = take((size_t)n_images * 4 * sizeof(float));
  l.counts = take((size_t)n_images * sizeof(int));
  l.lists = take((size_t)n_images * q_rows * sizeof(int));
  l.words = take(8 * sizeof(long long));  // tiles, staged rows, scheduler, cursor image, cursor offset
  l.tile_img = take((size_t)(cap / nearest::CTA_M) * sizeof(int));
  l.tile_off = take((size_t)(cap / nearest::CTA_M) * sizeof(int));
  l.row_map = take((size_t)cap * sizeof(int));
  l.s_norm = take((size_t)cap * sizeof(float));
  l.s_inv = take((size_t)cap * sizeof(float));
  l.s_hi = take((size_t)cap * channels * 2);
  l.s_lo = take((size_t)cap * channels * 2);
  l.total = o;
  return l;
}

// The largest staging capacity (multiple of 128, at most the default) whose layout fits
// `bytes`; 0 when even 128 rows do not fit.
long long staging_rows_for(int n_images, long long q_rows, int channels, size_t bytes) {
  long long hi = default_staging_rows(n_images, q_rows) / 128, lo = 0;
  if (refine_layout(n_images, q_rows, channels, hi * 128).total <= bytes) return hi * 128;
  while (hi - lo > 1) {
    const long long mid = (lo + hi) / 2;
    if (refine_layout(n_images, q_rows, channels, mid * 128).total <= bytes) lo = mid;
    else hi = mid;
  }
  return lo * 128;
}

// ------------------------------------------------------------------ image bounds
// bounds[j] = {max |z|^2, max residual norm} over image j's rows.
__global__ void __launch_bounds__(256)
image_bounds_kernel(const float* __restrict__ norm, const float* __restrict__ lnorm, int patches,
                    float* __restrict__ bounds) {
  const int j = blockIdx.x;
  float mn = 0.f, ml = 0.f;
  for (int r = threadIdx.x; r < patches; r += blockDim.x) {
    const long long row = (long long)j * patches + r;
    mn = fmaxf(mn, __ldg(norm + row));
    ml = fmaxf(ml, __ldg(lnorm + row));
  }
  mn = warp_max(mn);
  ml = warp_max(ml);
  __shared__ float red[2][8];
  if ((threadIdx.x & 31) == 0) red[0][threadIdx.x >> 5] = mn, red[1][threadIdx.x >> 5] = ml;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mn = fmaxf(mn, red[0][w]), ml = fmaxf(ml, red[1][w]);
    mn = fmaxf(mn, red[0][0]);
    ml = fmaxf(ml, red[1][0]);
    bounds[4 * j + 0] = mn;                                           // max |z|^2
    bounds[4 * j + 1] = ml;                                           // max L
    bounds[4 * j + 2] = sqrtf(mn) * (1.f + 1.0e-6f) + ml;             // max H (|hi| <= |z| + |lo|)
    bounds[4 * j + 3] = 0.f;
  }
}

// ------------------------------------------------------------------ refine
struct RefineParams {
  BankPlanes bank;
  const unsigned long long* k1;  // partial g at k1 + g * part_stride, [n_images][table_rows]
  const unsigned int* m2;
  long long part_stride;
  int n_parts;
  long long table_rows;          // rows per image in the partial tables
  long long first_row;           // global row of local row 0
  long long q_rows;
  int n_images, patches, channels;
  int rank_hi;
  float gamma;
  const float* bounds;
  float* exact;                  // [n_images][q_rows] (float bits, exact or FLT_MAX or an upper bound)
  int* counts;                   // [n_images] queued rows per image
  int* lists;                    // [n_images][q_rows] queued local rows
  int rows_per_cta;
  int pitch;                     // smem row pitch (>= n_images)
  int warps_per_row;             // warps sharing a row's bounds and exact evaluations
};

__device__ __forceinline__ float key_value(unsigned long long k) {
  return __uint_as_float((uint32_t)(k >> 32));
}

// Exact squared distance of two bank rows, one warp: sum over channels of the squared
// difference of the fp32 reconstructions (hi + lo) 2^-k.
__device__ float exact_d2(const BankPlanes& b, long long qa, long long pb, int channels, int lane) {
  const float ia = __ldg(b.inv + qa), ib = __ldg(b.inv + pb);
  const __half* ha = b.hi + qa * channels;
  const __half* la = b.lo + qa * channels;
  const __half* hb = b.hi + pb * channels;
  const __half* lb = b.lo + pb * channels;
  float acc = 0.f;
#pragma unroll 4
  for (int c = lane * 8; c < channels; c += 256) {
    const uint4 vha = __ldg(reinterpret_cast<const uint4*>(ha + c));
    const uint4 vla = __ldg(reinterpret_cast<const uint4*>(la + c));
    const uint4 vhb = __ldg(reinterpret_cast<const uint4*>(hb + c));
    const uint4 vlb = __ldg(reinterpret_cast<const uint4*>(lb + c));
    const __half* pha = reinterpret_cast<const __half*>(&vha);
    const __half* pla = reinterpret_cast<const __half*>(&vla);
    const __half* phb = reinterpret_cast<const __half*>(&vhb);
    const __half* plb = reinterpret_cast<const __half*>(&vlb);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xa = (__half2float(pha[e]) + __half2float(pla[e])) * ia;
      const float xb = (__half2float(phb[e]) + __half2float(plb[e])) * ib;
      const float d = xa - xb;
      acc = fmaf(d, d, acc);
    }
  }
  return warp_sum(acc);
}

// The same for two reference rows at once (the query row's loads shared): twice the
// loads in flight per warp, for the latency-bound gathers of the refinement.
__device__ void exact_d2_pair(const BankPlanes& b, long long qa, long long p0, long long p1, int channels, int lane,
                              float* d0, float* d1) {
  const float ia = __ldg(b.inv + qa), i0 = __ldg(b.inv + p0), i1 = __ldg(b.inv + p1);
  const __half* ha = b.hi + qa * channels;
  const __half* la = b.lo + qa * channels;
  const __half* h0 = b.hi + p0 * channels;
  const __half* l0 = b.lo + p0 * channels;
  const __half* h1 = b.hi + p1 * channels;
  const __half* l1 = b.lo + p1 * channels;
  float a0 = 0.f, a1 = 0.f;
#pragma unroll 2
  for (int c = lane * 8; c < channels; c += 256) {
    const uint4 vha = __ldg(reinterpret_cast<const uint4*>(ha + c));
    const uint4 vla = __ldg(reinterpret_cast<const uint4*>(la + c));
    const uint4 vh0 = __ldg(reinterpret_cast<const uint4*>(h0 + c));
    const uint4 vl0 = __ldg(reinterpret_cast<const uint4*>(l0 + c));
    const uint4 vh1 = __ldg(reinterpret_cast<const uint4*>(h1 + c));
    const uint4 vl1 = __ldg(reinterpret_cast<const uint4*>(l1 + c));
    const __half* pha = reinterpret_cast<const __half*>(&vha);
    const __half* pla = reinterpret_cast<const __half*>(&vla);
    const __half* ph0 = reinterpret_cast<const __half*>(&vh0);
    const __half* pl0 = reinterpret_cast<const __half*>(&vl0);
    const __half* ph1 = reinterpret_cast<const __half*>(&vh1);
    const __half* pl1 = reinterpret_cast<const __half*>(&vl1);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xa = (__half2float(pha[e]) + __half2float(pla[e])) * ia;
      const float x0 = (__half2float(ph0[e]) + __half2float(pl0[e])) * i0;
      const float x1 = (__half2float(ph1[e]) + __half2float(pl1[e])) * i1;
      const float e0 = xa - x0, e1 = xa - x1;
      a0 = fmaf(e0, e0, a0);
      a1 = fmaf(e1, e1, a1);
    }
  }
  *d0 = warp_sum(a0);
  *d1 = warp_sum(a1);
}

__global__ void __launch_bounds__(kRefineMaxThreads)
refine_kernel(const RefineParams rp) {
  extern __shared__ uint8_t smem_raw[];
  // [rows_per_cta][pitch] combined keys, second minima and the output row.
  unsigned long long* sk = reinterpret_cast<unsigned long long*>(smem_raw);
  uint32_t* sm2 = reinterpret_cast<uint32_t*>(sk + (size_t)rp.rows_per_cta * rp.pitch);
  float* sx = reinterpret_cast<float*>(sm2 + (size_t)rp.rows_per_cta * rp.pitch);
  float* su = sx + (size_t)rp.rows_per_cta * rp.pitch;  // per-group scratch [groups][pitch]: upper bounds
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r0 = (long long)blockIdx.x * rp.rows_per_cta;
  const int R = rp.rows_per_cta, N = rp.n_images;

  // 1. Stage the combined screen results of this CTA's rows, coalesced along rows.
  for (int idx = threadIdx.x; idx < N * R; idx += blockDim.x) {
    const int j = idx / R, r = idx - j * R;
    const long long q = r0 + r;
    unsigned long long best = ~0ull;
    uint32_t second = nearest::UMAX;
    if (q < rp.q_rows) {
      for (int g = 0; g < rp.n_parts; ++g) {
        const long long at = g * rp.part_stride + (long long)j * rp.table_rows + q;
        const unsigned long long k = __ldg(rp.k1 + at);
        second = min(second, __ldg(rp.m2 + at));
        if (k < best) {
          second = min(second, (uint32_t)(best >> 32));
          best = k;
        } else {
          second = min(second, (uint32_t)(k >> 32));
        }
      }
    }
    sk[(size_t)r * rp.pitch + j] = best;
    sm2[(size_t)r * rp.pitch + j] = second & ~0xFFu;
  }
  __syncthreads();

  // 2. One warp per row, or (large pools, few rows per CTA) a group of `warps_per_row`
  // warps per row: the group fills the row's upper bounds together (every wpr-th block of
  // 32 images per warp, one shared array, a named barrier per group), each warp finds the
  // threshold, and each evaluates its own blocks -- more row gathers in flight per SM.
  const int wpr = rp.warps_per_row, sub = warp % wpr, group = warp / wpr;
  float* u = su + (size_t)group * rp.pitch;
  const float lo_scale = 1.f - 6.2e-5f, hi_scale = 1.f + 6.2e-5f;  // 2^-14 on either side
  auto group_sync = [&]() {
    if (wpr == 1) __syncwarp();
    else asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(32 * wpr) : "memory");
  };
  for (int r = group; r < R; r += (int)(blockDim.x >> 5) / wpr) {
    const long long q = r0 + r;
    if (q >= rp.q_rows) break;  // warp-uniform
    const long long grow = rp.first_row + q;
    const int img = (int)(grow / rp.patches);
    const float nq = __ldg(rp.bank.norm + grow);
    const float lq = __ldg(rp.bank.lnorm + grow);
    const float hq = sqrtf(nq) * (1.f + 1.0e-6f) + lq;
    unsigned long long* kr = sk + (size_t)r * rp.pitch;
    uint32_t* mr = sm2 + (size_t)r * rp.pitch;
    float* xr = sx + (size_t)r * rp.pitch;
    auto bound = [&](int j) {
      const float nmax = __ldg(rp.bounds + 4 * j + 0), lmax = __ldg(rp.bounds + 4 * j + 1);
      const float hmax = __ldg(rp.bounds + 4 * j + 2);
      const float e = 2.f * (hq * lmax + lq * hmax + lq * lmax + rp.gamma * hq * hmax) + 4.8e-7f * (nq + nmax);
      return e * (1.f + 1.0e-5f);
    };
    // upper bounds U_j (FLT_MAX-like for the self image and unset pairs)
    group_sync();  // the group has finished reading the previous row's bounds
    for (int j = sub * 32 + lane; j < N; j += 32 * wpr) {
      const unsigned long long k = kr[j];
      float uj = __int_as_float(0x7f800000);  // +inf: never among the smallest
      if (j != img && k != ~0ull) uj = key_value(k) * hi_scale + bound(j);
      u[j] = uj;
    }
    group_sync();
    // T = the rank_hi-th smallest U_j: the largest bit pattern t with #{U < t} < rank_hi.
    uint32_t lo = 0u, hi = 0x7f800001u;
    while (hi - lo > 1u) {
      const uint32_t mid = lo + (hi - lo) / 2u;
      int c = 0;
      for (int j = lane; j < N; j += 32) c += __float_as_uint(u[j]) < mid ? 1 : 0;
      c = __reduce_add_sync(0xffffffffu, c);
      if (c < rp.rank_hi) lo = mid;
      else hi = mid;
    }
    const float T = __uint_as_float(lo);
    // Per image: excluded (FLT_MAX), certified exact, or an upper bound queued for the
    // exact fallback.
    for (int jb = sub * 32; jb < N; jb += 32 * wpr) {
      const int j = jb + lane;
      bool need = false;
      float lower = 0.f, e = 0.f;
      if (j < N) {
        const unsigned long long k = kr[j];
        if (j == img) {
          xr[j] = FLT_MAX;
        } else if (k == ~0ull) {
          // Never screened (cannot happen for a complete set of partial tables): queue
          // it with no bound; the fallback evaluates it exactly.
          xr[j] = FLT_MAX;
          const int slot = atomicAdd(rp.counts + j, 1);
          rp.lists[(long long)j * rp.q_rows + slot] = (int)q;
        } else {
          e = bound(j);
          lower = key_value(k) * lo_scale - e;
          need = lower <= T;
          if (!need) xr[j] = FLT_MAX;
        }
      }
      uint32_t mask = __ballot_sync(0xffffffffu, need);
      // The exact distance to each needed image's screened argmin, two images at a time;
      // the lane that owns the image stores it and decides its certification.
      auto settle = [&](int src, float d) {
        if (lane == src) {
          const int jj = jb + src;
          xr[jj] = d;
          const float m2v = __uint_as_float(mr[jj]);
          const bool certified = mr[jj] == (nearest::UMAX & ~0xFFu) || m2v * lo_scale - e >= d;
          if (!certified) {
            const int slot = atomicAdd(rp.counts + jj, 1);
            rp.lists[(long long)jj * rp.q_rows + slot] = (int)q;
          }
        }
      };
      while (mask) {
        const int s0 = __ffs(mask) - 1;
        mask &= mask - 1;
        const long long p0 = (long long)(jb + s0) * rp.patches + (long long)(uint32_t)kr[jb + s0];
        if (mask) {
          const int s1 = __ffs(mask) - 1;
          mask &= mask - 1;
          const long long p1 = (long long)(jb + s1) * rp.patches + (long long)(uint32_t)kr[jb + s1];
          float d0, d1;
          exact_d2_pair(rp.bank, grow, p0, p1, rp.channels, lane, &d0, &d1);
          settle(s0, fmaxf(d0, 0.f));
          settle(s1, fmaxf(d1, 0.f));
        } else {
          settle(s0, fmaxf(exact_d2(rp.bank, grow, p0, rp.channels, lane), 0.f));
        }
      }
    }
    __syncwarp();
  }
  __syncthreads();
  // 3. Write the exact table rows, coalesced along rows.
  for (int idx = threadIdx.x; idx < N * R; idx += blockDim.x) {
    const int j = idx / R, r = idx - j * R;
    const long long q = r0 + r;
    if (q < rp.q_rows) rp.exact[(long long)j * rp.q_rows + q] = sx[(size_t)r * rp.pitch + j];
  }
}

// ------------------------------------------------------------------ fallback rounds
// One thread: the next round's 128-row tiles, image after image from the cursor
// (words[3] = image, words[4] = offset in its queue) until the staging bank is full.
// tile_img / tile_off: each tile's image and the queue offset of its first row;
// words[0] = tiles x nsub for the GATHER kernel, words[1] = staged rows, words[2] = the
// GATHER kernel's scheduler (zeroed).  A round after the last does nothing.
__global__ void fallback_plan_kernel(const int* __restrict__ counts, int n_images, long long cap_tiles, int nsub,
                                     int* __restrict__ tile_img, int* __restrict__ tile_off,
                                     long long* __restrict__ words) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  long long j = words[3], off = words[4], tiles = 0;
  while (j < n_images && tiles < cap_tiles) {
    if (off >= counts[j]) {
      ++j;
      off = 0;
      continue;
    }
    tile_img[tiles] = (int)j;
    tile_off[tiles] = (int)off;
    ++tiles;
    off += nearest::CTA_M;
  }
  words[0] = tiles * nsub;
  words[1] = tiles * nearest::CTA_M;
  words[2] = 0;
  words[3] = j;
  words[4] = off;
}

// One warp per staged row of the round: copy the queued row's hi and lo planes, |z|^2
// and 2^-k from the pool bank into the staging bank; padding rows get row_map = -1.
__global__ void __launch_bounds__(256)
fallback_gather_kernel(BankPlanes bank, long long first_row, int channels, const int* __restrict__ counts,
                       const int* __restrict__ tile_img, const int* __restrict__ tile_off,
                       const int* __restrict__ lists, long long q_rows, const long long* __restrict__ words,
                       __half* __restrict__ s_hi, __half* __restrict__ s_lo, float* __restrict__ s_norm,
                       float* __restrict__ s_inv, int* __restrict__ row_map) {
  const long long staged = words[1];
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long s = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); s < staged; s += warps) {
    const long long mt = s / nearest::CTA_M;
    const int j = tile_img[mt];
    const long long k = tile_off[mt] + (s - mt * nearest::CTA_M);
    if (k >= counts[j]) {
      if (lane == 0) row_map[s] = -1;
      continue;
    }
    const int q = lists[(long long)j * q_rows + k];
    const long long g = first_row + q;
    for (int c = lane * 8; c < channels; c += 256) {
      *reinterpret_cast<uint4*>(s_hi + s * channels + c) = __ldg(reinterpret_cast<const uint4*>(bank.hi + g * channels + c));
      *reinterpret_cast<uint4*>(s_lo + s * channels + c) = __ldg(reinterpret_cast<const uint4*>(bank.lo + g * channels + c));
    }
    if (lane == 0) {
      s_norm[s] = __ldg(bank.norm + g);
      s_inv[s] = __ldg(bank.inv + g);
      row_map[s] = q;
    }
  }
}

// Rows per CTA, threads and warps per row.  Eight one-row warps per CTA over the most rows
// (32, 16 or 8) that still let three CTAs share an SM, the most its registers allow; where
// none does (large pools), one group of warps per row (24 warps per CTA) sharing the row's
// upper bounds.
int refine_rows_per_cta(int n_images, int* pitch, size_t* smem, int* threads, int* wpr) {
  const int pt = n_images + ((2 - n_images % 2) % 2);  // even, so the 8-byte keys stay aligned
  const long long per_sm = smem_optin(), budget = per_sm - 4096;
  auto bytes_for = [&](int r, int groups) {
    return (long long)r * pt * (8 + 4 + 4) + (long long)groups * pt * 4;
  };
  *pitch = pt;
  for (int rows = 32; rows >= 8; rows >>= 1) {
    if (per_sm / (bytes_for(rows, 8) + 1024) >= 3) {
      *threads = kRefineThreads;
      *wpr = 1;
      *smem = (size_t)bytes_for(rows, 8);
      return rows;
    }
  }
  int rows = 16;
  while (rows > 1 && bytes_for(rows, rows) > budget) rows >>= 1;
  *wpr = std::max(1, (kRefineMaxThreads / 32) / rows);
  *threads = 32 * rows * *wpr;
  *smem = (size_t)bytes_for(rows, rows);
  return rows;
}

}  // namespace

size_t refine_workspace_bytes(int n_images, long long q_rows, int channels) {
  return refine_layout(n_images, q_rows, channels, default_staging_rows(n_images, q_rows)).total;
}

size_t refine_min_workspace_bytes(int n_images, long long q_rows, int channels) {
  return refine_layout(n_images, q_rows, channels, 128).total;
}

// Fallback rounds enqueued for a workspace of `bytes`: enough for every (row, image) pair.
long long refine_rounds(int n_images, long long q_rows, int channels, size_t bytes) {
  const long long cap = staging_rows_for(n_images, q_rows, channels, bytes);
  if (cap < 128) return 0;
  const long long worst_tiles = ((long long)n_images * q_rows) / nearest::CTA_M + n_images;
  const long long cap_tiles = cap / nearest::CTA_M;
  return (worst_tiles + cap_tiles - 1) / cap_tiles;
}

// The whole refinement of one bank for rows [first_row, first_row + q_rows) of the pool.
int refine_launch(const void* bank, long long bank_rows, long long rows, int channels, int patches,
                  long long first_row, long long q_rows, int rank_hi, const unsigned long long* k1,
                  const unsigned int* m2, int n_parts, long long part_stride, long long table_rows,
                  float* exact, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  const int n_images = (int)(rows / patches);
  const long long cap = staging_rows_for(n_images, q_rows, channels, workspace_bytes);
  if (cap < 128) return fail(MUSC_B200_ERR_WORKSPACE, "refine: workspace below musc_b200_refine_min_bytes");
  const RefineLayout l = refine_layout(n_images, q_rows, channels, cap);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const BankPlanes bp = bank_planes(bank, bank_rows, channels);
  float* bounds = reinterpret_cast<float*>(ws + l.bounds);
  int* counts = reinterpret_cast<int*>(ws + l.counts);
  int* lists = reinterpret_cast<int*>(ws + l.lists);
  int* tile_img = reinterpret_cast<int*>(ws + l.tile_img);
  int* tile_off = reinterpret_cast<int*>(ws + l.tile_off);
  int* row_map = reinterpret_cast<int*>(ws + l.row_map);
  float* s_norm = reinterpret_cast<float*>(ws + l.s_norm);
  float* s_inv = reinterpret_cast<float*>(ws + l.s_inv);
  __half* s_hi = reinterpret_cast<__half*>(ws + l.s_hi);
  __half* s_lo = reinterpret_cast<__half*>(ws + l.s_lo);
  long long* words = reinterpret_cast<long long*>(ws + l.words);

  MUSC_CUDA(cudaMemsetAsync(counts, 0, (size_t)n_images * sizeof(int), s));
  MUSC_CUDA(cudaMemsetAsync(words, 0, 8 * sizeof(long long), s));
  image_bounds_kernel<<<n_images, 256, 0, s>>>(bp.norm, bp.lnorm, patches, bounds);
  MUSC_TRY(check_launch("image_bounds_kernel"));

  RefineParams rp;
  rp.bank = bp;
  rp.k1 = k1;
  rp.m2 = m2;
  rp.part_stride = part_stride;
  rp.n_parts = n_parts;
  rp.table_rows = table_rows;
  rp.first_row = first_row;
  rp.q_rows = q_rows;
  rp.n_images = n_images;
  rp.patches = patches;
  rp.channels = channels;
  rp.rank_hi = rank_hi;
  const double kpad = (double)((channels + nearest::BK - 1) / nearest::BK * nearest::BK);
  const double ku = kpad * 1.1920928955078125e-7;  // K * 2^-23
  rp.gamma = (float)(ku / (1.0 - ku));
  rp.bounds = bounds;
  rp.exact = exact;
  rp.counts = counts;
  rp.lists = lists;
  size_t smem = 0;
  int threads = kRefineThreads;
  rp.rows_per_cta = refine_rows_per_cta(n_images, &rp.pitch, &smem, &threads, &rp.warps_per_row);
  if (rp.rows_per_cta < 1 || (long long)smem > smem_optin())
    return fail(MUSC_B200_ERR_INVALID, "refine: too many images for the refinement's shared memory");
  MUSC_CUDA(cudaFuncSetAttribute(refine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const long long blocks = (q_rows + rp.rows_per_cta - 1) / rp.rows_per_cta;
  refine_kernel<<<(unsigned)blocks, (unsigned)threads, smem, s>>>(rp);
  MUSC_TRY(check_launch("refine_kernel"));

  // Exact 3-pass evaluation of the queued rows against their images, in rounds of at
  // most `cap` staged rows.  The host cannot see the queue's length without a
  // synchronisation, so it enqueues the worst-case number of rounds; rounds after the
  // queue is drained find nothing to plan and their kernels return at once.
  const int nsub = (patches + nearest::BN - 1) / nearest::BN;
  const int sms = sm_count();
  CUtensorMap mqh, mql, mrh, mrl;
  MUSC_TRY(make_plane_map(&mqh, s_hi, l.cap, channels, nearest::CTA_M, nearest::BK));
  MUSC_TRY(make_plane_map(&mql, s_lo, l.cap, channels, nearest::CTA_M, nearest::BK));
  MUSC_TRY(make_plane_map(&mrh, bp.hi, rows, channels, nearest::BN, nearest::BK));
  MUSC_TRY(make_plane_map(&mrl, bp.lo, rows, channels, nearest::BN, nearest::BK));
  nearest::Params p{};
  p.q_norm = s_norm;
  p.q_inv = s_inv;
  p.r_norm = bp.norm;
  p.r_inv = bp.inv;
  p.nearest = reinterpret_cast<unsigned int*>(exact);
  p.sched = reinterpret_cast<unsigned long long*>(words + 2);
  p.tile_img = tile_img;
  p.row_map = row_map;
  p.tile_total = words;
  p.err = device_error_ptr();
  if (!p.err) return fail(MUSC_B200_ERR_CUDA, "refine: device error word unavailable");
  p.q_rows = l.cap;
  p.r_rows = rows;
  p.q_first_row = 0;
  p.tile_begin = 0;
  p.tile_end = 0x7FFFFFFFFFFFFFFFLL;
  p.rows_per_block = q_rows;
  p.blocked = 0;
  p.patches = patches;
  p.n_images = n_images;
  p.num_kb = (channels + nearest::BK - 1) / nearest::BK;
  p.nsub = nsub;
  MUSC_TRY(set_nearest_smem_attrs());
  // worst case: every (row, image) pair queued, each image's queue padded to whole tiles
  const long long cap_tiles = l.cap / nearest::CTA_M;
  const long long rounds = refine_rounds(n_images, q_rows, channels, workspace_bytes);
  for (long long r = 0; r < rounds; ++r) {
    fallback_plan_kernel<<<1, 32, 0, s>>>(counts, n_images, cap_tiles, nsub, tile_img, tile_off, words);
    MUSC_TRY(check_launch("fallback_plan_kernel"));
    fallback_gather_kernel<<<sms * 4, 256, 0, s>>>(bp, first_row, channels, counts, tile_img, tile_off, lists,
                                                    q_rows, words, s_hi, s_lo, s_norm, s_inv, row_map);
    MUSC_TRY(check_launch("fallback_gather_kernel"));
    nearest::nearest_kernel<nearest::GATHER, false>
        <<<sms, nearest::Cfg<nearest::GATHER, false>::THREADS, nearest::smem_bytes<nearest::GATHER, false>(), s>>>(
            mqh, mql, mrh, mrl, p);
    MUSC_TRY(check_launch("nearest_kernel<gather>"));
  }
  return MUSC_B200_OK;
}

}  // namespace musc
