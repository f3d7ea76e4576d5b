// Pool-image preprocessing on the device: the reference's evaluation transform
// (models/backbone/open_clip/transform.py:124-133 -- Resize((S, S), BICUBIC),
// CenterCrop((S, S)), ToTensor, Normalize) applied to a batch of 8-bit RGB
// images that were decoded on the host and copied in as bytes, so the host
// neither resizes nor converts to float and the copy moves 3 bytes per input
// pixel instead of 12 per output pixel.
//
// The resize is Pillow's separable antialiased resample, bit for bit: per axis
// a table of fixed-point weights (22 fractional bits) computed in IEEE double
// exactly as Pillow computes it, a horizontal pass over the input rows the
// vertical pass needs (8-bit, clipped), then the vertical pass.  One CTA owns a
// band of TY output rows of one image: it resamples the band's input rows
// horizontally into shared memory (channel-planar bytes), then each thread
// produces output pixels of one channel from the staged rows, normalises them
// through a 256-entry table per channel ((u8 / 255 - mean) / std in fp32, the
// torchvision operations) and stores the planar (3, S, S) result coalesced.
// HBM traffic: the input bytes once (plus the band halo, from L2) and the
// output once.
#include "common.cuh"

#include <math.h>

namespace musc {
namespace image {

constexpr int kPrecisionBits = 22;
constexpr int kMaxTaps = 65;        // 2 * ceil(support) + 1 for a 15.75x bicubic reduction
constexpr int kThreads = 256;
constexpr int kMaxSmem = 200 * 1024;

struct Axis {
  int in_size, out_size, ksize;
  double scale, support, inv_filterscale;
};

// Filter support and table width of one axis, as Pillow derives them.
inline Axis make_axis(int in_size, int out_size, int filter) {
  Axis a;
  a.in_size = in_size;
  a.out_size = out_size;
  a.scale = static_cast<double>(static_cast<float>(in_size)) / out_size;
  double filterscale = a.scale < 1.0 ? 1.0 : a.scale;
  a.support = (filter == MUSC_B200_BILINEAR ? 1.0 : 2.0) * filterscale;
  a.ksize = static_cast<int>(ceil(a.support)) * 2 + 1;
  a.inv_filterscale = 1.0 / filterscale;
  return a;
}

// Upper bound of the input rows a band of `ty` output rows reads: the first
// tap of the band's first row is >= centre - support - 0.5 and the end of its
// last row <= centre + support + 0.5, (ty - 1) * scale apart.
inline int band_rows(const Axis& v, int ty, bool need_vertical) {
  if (!need_vertical) return ty;
  return static_cast<int>(ceil((ty - 1) * v.scale + 2.0 * v.support)) + 2;
}

// Pillow's filters, evaluated with explicitly rounded double operations so the
// compiler cannot contract them into fused multiply-adds (Pillow's x86 build
// rounds every product and sum).
__device__ __forceinline__ double filter_weight(int filter, double x) {
  x = fabs(x);
  if (filter == MUSC_B200_BILINEAR) return x < 1.0 ? __dsub_rn(1.0, x) : 0.0;
  if (x < 1.0) return __dadd_rn(__dmul_rn(__dmul_rn(__dsub_rn(__dmul_rn(1.5, x), 2.5), x), x), 1.0);
  if (x < 2.0)
    return __dmul_rn(__dsub_rn(__dmul_rn(__dadd_rn(__dmul_rn(__dsub_rn(x, 5.0), x), 8.0), x), 4.0), -0.5);
  return 0.0;
}

// One thread per output index of one axis: tap range and fixed-point weights
// (Resample.c's precompute_coeffs + normalize_coeffs_8bpc, restated).
__device__ void axis_table(const Axis& a, int filter, int o, int2* bounds, int* weights) {
  double centre = __dmul_rn(__dadd_rn(static_cast<double>(o), 0.5), a.scale);
  int xmin = __double2int_rz(__dadd_rn(__dsub_rn(centre, a.support), 0.5));
  if (xmin < 0) xmin = 0;
  int xmax = __double2int_rz(__dadd_rn(__dadd_rn(centre, a.support), 0.5));
  if (xmax > a.in_size) xmax = a.in_size;
  xmax -= xmin;
  if (xmax > a.ksize) xmax = a.ksize;   // never binds: the taps span at most 2 * ceil(support) + 1
  double w[kMaxTaps];
  double ww = 0.0;
  for (int x = 0; x < xmax; ++x) {
    double arg = __dmul_rn(__dadd_rn(__dsub_rn(static_cast<double>(x + xmin), centre), 0.5), a.inv_filterscale);
    w[x] = filter_weight(filter, arg);
    ww = __dadd_rn(ww, w[x]);
  }
  int* k = weights + static_cast<long long>(o) * a.ksize;
  for (int x = 0; x < a.ksize; ++x) {
    int fixed = 0;
    if (x < xmax) {
      double v = ww != 0.0 ? __ddiv_rn(w[x], ww) : w[x];
      double scaled = __dmul_rn(v, static_cast<double>(1 << kPrecisionBits));
      fixed = __double2int_rz(v < 0 ? __dadd_rn(-0.5, scaled) : __dadd_rn(0.5, scaled));
    }
    k[x] = fixed;
  }
  bounds[o] = make_int2(xmin, xmax);
}

__global__ void __launch_bounds__(128) tables_kernel(Axis h, Axis v, int filter, int2* hb, int* hw, int2* vb,
                                                     int* vw) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < h.out_size) axis_table(h, filter, i, hb, hw);
  else if (i < h.out_size + v.out_size) axis_table(v, filter, i - h.out_size, vb, vw);
}

__device__ __forceinline__ int clip8(int acc) {
  int v = acc >> kPrecisionBits;
  return v < 0 ? 0 : (v > 255 ? 255 : v);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

struct Params {
  const uint8_t* images;
  long long image_stride;   // bytes between images
  int in_h, in_w, out_h, out_w;
  int kh, kv, ty, max_rows;
  int need_h, need_v;
  float mean[3], stdev[3];
  const int2* hb;
  const int* hw;
  const int2* vb;
  const int* vw;
  void* out;
};

template <typename OutT>
__global__ void __launch_bounds__(kThreads) resample_kernel(Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* lut = reinterpret_cast<float*>(smem);                 // [3][256]
  uint8_t* band = smem + 3 * 256 * sizeof(float);             // [3][max_rows][out_w]
  const int img = blockIdx.y;
  const int y0 = blockIdx.x * p.ty;
  const int y1 = min(y0 + p.ty, p.out_h);
  const uint8_t* src = p.images + static_cast<long long>(img) * p.image_stride;
  const long long row_bytes = 3LL * p.in_w;

  for (int i = threadIdx.x; i < 3 * 256; i += kThreads) {
    int c = i >> 8;
    float x = __fdiv_rn(static_cast<float>(i & 255), 255.0f);
    float m = c == 0 ? p.mean[0] : (c == 1 ? p.mean[1] : p.mean[2]);
    float sd = c == 0 ? p.stdev[0] : (c == 1 ? p.stdev[1] : p.stdev[2]);
    lut[i] = __fdiv_rn(__fsub_rn(x, m), sd);
  }

  // Input rows of the band: [r0, r0 + rows).
  int r0, rows;
  if (p.need_v) {
    int2 first = p.vb[y0], last = p.vb[y1 - 1];
    r0 = first.x;
    rows = last.x + last.y - first.x;
  } else {
    r0 = y0;
    rows = y1 - y0;
  }
  rows = min(rows, p.max_rows);   // never binds: max_rows is an upper bound (band_rows)
  const int plane = p.max_rows * p.out_w;

  // Horizontal pass into the band (or a plain copy when the width is kept).
  const int band_items = rows * p.out_w;
  for (int i = threadIdx.x; i < band_items; i += kThreads) {
    int r = i / p.out_w, x = i - r * p.out_w;
    const uint8_t* row = src + (r0 + r) * row_bytes;
    int a0, a1, a2;
    if (p.need_h) {
      int2 b = __ldg(p.hb + x);
      const int* k = p.hw + static_cast<long long>(x) * p.kh;
      const uint8_t* px = row + 3 * b.x;
      a0 = a1 = a2 = 1 << (kPrecisionBits - 1);
      for (int t = 0; t < b.y; ++t) {
        int w = __ldg(k + t);
        a0 += static_cast<int>(__ldg(px + 3 * t + 0)) * w;
        a1 += static_cast<int>(__ldg(px + 3 * t + 1)) * w;
        a2 += static_cast<int>(__ldg(px + 3 * t + 2)) * w;
      }
      a0 = clip8(a0);
      a1 = clip8(a1);
      a2 = clip8(a2);
    } else {
      a0 = __ldg(row + 3 * x + 0);
      a1 = __ldg(row + 3 * x + 1);
      a2 = __ldg(row + 3 * x + 2);
    }
    band[i] = static_cast<uint8_t>(a0);
    band[plane + i] = static_cast<uint8_t>(a1);
    band[2 * plane + i] = static_cast<uint8_t>(a2);
  }
  __syncthreads();

  // Vertical pass, normalisation, planar store.
  OutT* out = reinterpret_cast<OutT*>(p.out) + static_cast<long long>(img) * 3 * p.out_h * p.out_w;
  const int band_out = (y1 - y0) * p.out_w;
  for (int i = threadIdx.x; i < 3 * band_out; i += kThreads) {
    int c = i / band_out;
    int rem = i - c * band_out;
    int dy = rem / p.out_w, x = rem - dy * p.out_w;
    int y = y0 + dy;
    const uint8_t* col = band + c * plane + x;
    int u;
    if (p.need_v) {
      int2 b = __ldg(p.vb + y);
      const int* k = p.vw + static_cast<long long>(y) * p.kv;
      int first = b.x - r0;
      int taps = min(b.y, rows - first);   // never binds (see max_rows)
      int acc = 1 << (kPrecisionBits - 1);
      for (int t = 0; t < taps; ++t) acc += static_cast<int>(col[(first + t) * p.out_w]) * __ldg(k + t);
      u = clip8(acc);
    } else {
      u = col[dy * p.out_w];
    }
    out[(static_cast<long long>(c) * p.out_h + y) * p.out_w + x] = from_f32<OutT>(lut[c * 256 + u]);
  }
}

// Staged form for the common case (both axes resized, at most 17 horizontal
// taps: an input at most 4x its output).  The band's input rows are copied
// into shared memory with 16-byte loads; the horizontal pass gives each thread
// one output column with its weights in registers and a run of rows; the
// vertical pass gives each thread four adjacent columns of one channel (one
// 32-bit shared load per tap) with the row's weights broadcast from shared
// memory.  Shared memory: LUT | band rows' vertical bounds + weights | 8-bit
// horizontal result [3][max_rows][pitch] | input rows (+ slack for the taps
// past a row's end, whose weights are zero).
constexpr int kRowsPerItem = 2;

// Threads of the staged kernel: 512 for up to 9 taps (64 registers, two CTAs per SM),
// 256 for the wider tap buckets.
__host__ __device__ constexpr int staged_threads(int kh) { return kh <= 9 ? 512 : 256; }

__host__ __device__ inline int band_pitch(int out_w) { return (out_w + 3) & ~3; }

__host__ __device__ inline size_t staged_smem(int ty, int kv, int max_rows, int out_w, long long row_bytes,
                                              int kh_max) {
  size_t off = 3 * 256 * sizeof(float) + 16 * sizeof(int2);
  off += (static_cast<size_t>(ty) * kv * sizeof(int) + 15) & ~static_cast<size_t>(15);
  off += 3ULL * max_rows * band_pitch(out_w);
  off = (off + 15) & ~static_cast<size_t>(15);
  return off + static_cast<size_t>(max_rows) * row_bytes + 16 + 3 * kh_max + 16;
}

template <typename OutT, int KH>
__global__ void __launch_bounds__(staged_threads(KH), 2) resample_staged_kernel(Params p) {
  constexpr int kT = staged_threads(KH);
  extern __shared__ __align__(16) uint8_t smem[];
  float* lut = reinterpret_cast<float*>(smem);
  int2* vb_s = reinterpret_cast<int2*>(smem + 3 * 256 * sizeof(float));
  int* vw_s = reinterpret_cast<int*>(vb_s + 16);
  uint8_t* band = reinterpret_cast<uint8_t*>(vw_s) + ((p.ty * p.kv * sizeof(int) + 15) & ~static_cast<size_t>(15));
  const int pitch = band_pitch(p.out_w);
  const int plane = p.max_rows * pitch;
  uint8_t* in_s = band + ((3 * plane + 15) & ~15);
  const int img = blockIdx.y;
  const int y0 = blockIdx.x * p.ty;
  const int y1 = min(y0 + p.ty, p.out_h);
  const int tid = threadIdx.x;
  const long long row_bytes = 3LL * p.in_w;

  for (int i = tid; i < 3 * 256; i += kT) {
    int c = i >> 8;
    float x = __fdiv_rn(static_cast<float>(i & 255), 255.0f);
    float m = c == 0 ? p.mean[0] : (c == 1 ? p.mean[1] : p.mean[2]);
    float sd = c == 0 ? p.stdev[0] : (c == 1 ? p.stdev[1] : p.stdev[2]);
    lut[i] = __fdiv_rn(__fsub_rn(x, m), sd);
  }
  for (int i = tid; i < (y1 - y0) * p.kv; i += kT) {
    int dy = i / p.kv;
    vw_s[i] = __ldg(p.vw + static_cast<long long>(y0) * p.kv + i);
    if (i - dy * p.kv == 0) vb_s[dy] = p.vb[y0 + dy];
  }
  int2 first = p.vb[y0], last = p.vb[y1 - 1];
  const int r0 = first.x;
  const int rows = min(last.x + last.y - first.x, p.max_rows);   // the min never binds (band_rows)

  // Input rows [r0, r0 + rows) -> in_s[off0 ...]: whole 16-byte chunks by vector loads,
  // the partial chunks at both ends byte by byte (every access inside the image).
  {
    const uint8_t* start = p.images + static_cast<long long>(img) * p.image_stride + r0 * row_bytes;
    const long long n = rows * row_bytes;
    const int off0 = static_cast<int>(reinterpret_cast<uintptr_t>(start) & 15);
    const uint8_t* a0 = start - off0;
    const long long chunks = (off0 + n + 15) >> 4;
    for (long long k = tid; k < chunks; k += kT) {
      long long lo = k << 4, hi = lo + 16;
      if (lo >= off0 && hi <= off0 + n) {
        *reinterpret_cast<uint4*>(in_s + lo) = __ldg(reinterpret_cast<const uint4*>(a0 + lo));
      } else {
        for (long long b = max(lo, static_cast<long long>(off0)); b < min(hi, off0 + n); ++b) in_s[b] = __ldg(a0 + b);
      }
    }
    in_s += off0;
  }
  __syncthreads();

  // Horizontal pass: item = (column, run of kRowsPerItem rows).
  const int runs = (rows + kRowsPerItem - 1) / kRowsPerItem;
  for (int i = tid; i < runs * p.out_w; i += kT) {
    int run = i / p.out_w;
    int x = i - run * p.out_w;
    int2 b = __ldg(p.hb + x);
    const int* k = p.hw + static_cast<long long>(x) * p.kh;
    int w[KH];
#pragma unroll
    for (int t = 0; t < KH; ++t) w[t] = t < p.kh ? __ldg(k + t) : 0;   // zero past the taps
    const uint8_t* base = in_s + 3 * b.x;
    int rend = min(run * kRowsPerItem + kRowsPerItem, rows);
    for (int r = run * kRowsPerItem; r < rend; ++r) {
      // The 3 * KH tap bytes as 32-bit shared loads: NW aligned words from the window's
      // aligned-down start, re-aligned to the window by funnel shifts (the last bytes may
      // lie past the row: their weights are zero, and the slack after the staged rows
      // covers them).
      constexpr int NV = (3 * KH + 3) / 4, NW = NV + 1;
      const uint8_t* px = base + r * row_bytes;
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(px) & ~uintptr_t(3));
      const int sh = static_cast<int>(reinterpret_cast<uintptr_t>(px) & 3) * 8;
      uint32_t wv[NW];
#pragma unroll
      for (int k = 0; k < NW; ++k) wv[k] = wp[k];
      uint32_t v[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) v[k] = __funnelshift_r(wv[k], wv[k + 1], sh);
      int a0 = 1 << (kPrecisionBits - 1), a1 = a0, a2 = a0;
#pragma unroll
      for (int t = 0; t < KH; ++t) {
        // byte j of the window: one byte permute (selector j & 3 for the low byte, 4 = zero)
        a0 += static_cast<int>(__byte_perm(v[(3 * t + 0) >> 2], 0u, 0x4440u | ((3 * t + 0) & 3))) * w[t];
        a1 += static_cast<int>(__byte_perm(v[(3 * t + 1) >> 2], 0u, 0x4440u | ((3 * t + 1) & 3))) * w[t];
        a2 += static_cast<int>(__byte_perm(v[(3 * t + 2) >> 2], 0u, 0x4440u | ((3 * t + 2) & 3))) * w[t];
      }
      uint8_t* dst = band + r * pitch + x;
      dst[0] = static_cast<uint8_t>(clip8(a0));
      dst[plane] = static_cast<uint8_t>(clip8(a1));
      dst[2 * plane] = static_cast<uint8_t>(clip8(a2));
    }
  }
  __syncthreads();

  // Vertical pass: item = (output row, channel, four columns).
  OutT* out = reinterpret_cast<OutT*>(p.out) + static_cast<long long>(img) * 3 * p.out_h * p.out_w;
  const int nq = pitch >> 2;
  for (int i = tid; i < (y1 - y0) * 3 * nq; i += kT) {
    const int dy = i / (3 * nq);
    const int y = y0 + dy;
    const int2 b = vb_s[dy];
    const int f = b.x - r0;
    const int taps = min(b.y, rows - f);   // never binds (see max_rows)
    const int* wy = vw_s + dy * p.kv;
    int rem = i - dy * 3 * nq;
    int c = rem >= 2 * nq ? 2 : (rem >= nq ? 1 : 0);
    int xq = rem - c * nq;
    const uint32_t* col = reinterpret_cast<const uint32_t*>(band + c * plane) + xq;
    int acc0 = 1 << (kPrecisionBits - 1), acc1 = acc0, acc2 = acc0, acc3 = acc0;
    for (int t = 0; t < taps; ++t) {
      uint32_t v = col[(f + t) * nq];
      int w = wy[t];
      acc0 += static_cast<int>(v & 255u) * w;
      acc1 += static_cast<int>((v >> 8) & 255u) * w;
      acc2 += static_cast<int>((v >> 16) & 255u) * w;
      acc3 += static_cast<int>(v >> 24) * w;
    }
    const float* l = lut + c * 256;
    OutT* o = out + (static_cast<long long>(c) * p.out_h + y) * p.out_w + 4 * xq;
    int x = 4 * xq;
    if (x + 0 < p.out_w) o[0] = from_f32<OutT>(l[clip8(acc0)]);
    if (x + 1 < p.out_w) o[1] = from_f32<OutT>(l[clip8(acc1)]);
    if (x + 2 < p.out_w) o[2] = from_f32<OutT>(l[clip8(acc2)]);
    if (x + 3 < p.out_w) o[3] = from_f32<OutT>(l[clip8(acc3)]);
  }
}

struct Plan {
  Axis h, v;
  int need_h, need_v, ty, max_rows;
  size_t smem;
  size_t offsets[5];   // hb, hw, vb, vw, end
  int staged_kh;       // 0 = the general kernel, else the staged kernel's tap bucket
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int make_plan(int in_h, int in_w, int out_h, int out_w, int filter, int n_images, Plan* plan) {
  if (in_h < 1 || in_w < 1 || out_h < 1 || out_w < 1)
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: image sizes must be positive");
  if (filter != MUSC_B200_BICUBIC && filter != MUSC_B200_BILINEAR)
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: filter must be MUSC_B200_BICUBIC or MUSC_B200_BILINEAR");
  if (in_h >= (1 << 24) || in_w >= (1 << 24) || 3LL * in_w * in_h > (1LL << 40))
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: input image too large");
  plan->h = make_axis(in_w, out_w, filter);
  plan->v = make_axis(in_h, out_h, filter);
  if (plan->h.ksize > kMaxTaps || plan->v.ksize > kMaxTaps)
    return fail(MUSC_B200_ERR_INVALID,
                "preprocess_images: an input side is more than 15.75x (bicubic) / 31.5x (bilinear) its output side");
  plan->need_h = in_w != out_w;
  plan->need_v = in_h != out_h;
  int sms = n_images > 0 ? sm_count() : 148;
  // Staged kernel: both axes resized and at most 17 horizontal taps.  Tallest band of
  // 16, 8 or 4 rows whose shared memory lets two CTAs share an SM (and that gives two
  // CTAs per SM over the grid, where the batch allows).
  plan->staged_kh = 0;
  if (plan->need_h && plan->need_v && plan->h.ksize <= 17) {
    int kh = plan->h.ksize <= 9 ? 9 : (plan->h.ksize <= 13 ? 13 : 17);
    for (int ty = 16; ty >= 4; ty >>= 1) {
      int rows = band_rows(plan->v, ty, true);
      size_t smem = staged_smem(ty, plan->v.ksize, rows, out_w, 3LL * in_w, kh);
      if (smem > 113 * 1024) continue;
      long long ctas = static_cast<long long>((out_h + ty - 1) / ty) * (n_images > 0 ? n_images : 1);
      plan->staged_kh = kh;
      plan->ty = ty;
      plan->max_rows = rows;
      plan->smem = smem;
      if (ctas >= 2LL * sms) break;
    }
  }
  // General kernel: tallest band that fits the shared memory and still gives two CTAs per SM.
  if (!plan->staged_kh) plan->ty = 0;
  for (int ty = 16; !plan->staged_kh && ty >= 1; ty >>= 1) {
    int rows = band_rows(plan->v, ty, plan->need_v);
    size_t smem = 3 * 256 * sizeof(float) + 3ULL * rows * out_w;
    if (smem > kMaxSmem) continue;
    long long ctas = static_cast<long long>((out_h + ty - 1) / ty) * (n_images > 0 ? n_images : 1);
    plan->ty = ty;
    plan->max_rows = rows;
    plan->smem = smem;
    if (ctas >= 2LL * sms) break;
  }
  if (plan->ty == 0)
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: output row too wide for one band in shared memory");
  size_t off = 0;
  plan->offsets[0] = off; off = align256(off + sizeof(int2) * out_w);
  plan->offsets[1] = off; off = align256(off + sizeof(int) * static_cast<size_t>(out_w) * plan->h.ksize);
  plan->offsets[2] = off; off = align256(off + sizeof(int2) * out_h);
  plan->offsets[3] = off; off = align256(off + sizeof(int) * static_cast<size_t>(out_h) * plan->v.ksize);
  plan->offsets[4] = off;
  return MUSC_B200_OK;
}

template <typename OutT>
int launch(const Params& p, const Plan& plan, int n_images, cudaStream_t stream) {
  auto kern = plan.staged_kh == 9    ? resample_staged_kernel<OutT, 9>
              : plan.staged_kh == 13 ? resample_staged_kernel<OutT, 13>
              : plan.staged_kh == 17 ? resample_staged_kernel<OutT, 17>
                                     : resample_kernel<OutT>;
  int threads = plan.staged_kh ? staged_threads(plan.staged_kh) : kThreads;
  MUSC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem)));
  // gridDim.y is at most 65535: larger batches go in slices of that many images
  constexpr int kMaxGridY = 65535;
  for (int first = 0; first < n_images; first += kMaxGridY) {
    Params q = p;
    q.images = p.images + static_cast<long long>(first) * p.image_stride;
    q.out = static_cast<OutT*>(p.out) + static_cast<long long>(first) * 3 * p.out_h * p.out_w;
    dim3 grid((p.out_h + p.ty - 1) / p.ty, min(kMaxGridY, n_images - first));
    kern<<<grid, threads, plan.smem, stream>>>(q);
    MUSC_TRY(check_launch("resample_kernel"));
  }
  return MUSC_B200_OK;
}

}  // namespace image
}  // namespace musc

using namespace musc;

extern "C" size_t musc_b200_preprocess_workspace_bytes(int in_h, int in_w, int out_h, int out_w, int filter) {
  image::Plan plan;
  if (image::make_plan(in_h, in_w, out_h, out_w, filter, 0, &plan) != MUSC_B200_OK) return 0;
  return plan.offsets[4];
}

extern "C" int musc_b200_preprocess_images(const uint8_t* images, int n_images, int in_h, int in_w,
                                           long long image_stride_bytes, int out_h, int out_w, int filter,
                                           const float* mean, const float* stdev, int out_dtype, void* out,
                                           void* workspace, size_t workspace_bytes, musc_b200_stream stream) {
  if (n_images < 0) return fail(MUSC_B200_ERR_INVALID, "preprocess_images: n_images must be >= 0");
  if (!mean || !stdev) return fail(MUSC_B200_ERR_INVALID, "preprocess_images: mean and std must be given");
  if (out_dtype != MUSC_B200_F32 && out_dtype != MUSC_B200_F16 && out_dtype != MUSC_B200_BF16)
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: unknown output dtype");
  if (image_stride_bytes < 3LL * in_h * in_w)
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: image stride smaller than one H x W x 3 image");
  for (int c = 0; c < 3; ++c)
    if (!(stdev[c] != 0.0f)) return fail(MUSC_B200_ERR_INVALID, "preprocess_images: std must be non-zero");
  image::Plan plan;
  MUSC_TRY(image::make_plan(in_h, in_w, out_h, out_w, filter, n_images, &plan));
  if (n_images == 0) return MUSC_B200_OK;
  if (!images || !out || !workspace)
    return fail(MUSC_B200_ERR_INVALID, "preprocess_images: null images, output or workspace");
  if (workspace_bytes < plan.offsets[4])
    return fail(MUSC_B200_ERR_WORKSPACE, "preprocess_images: workspace smaller than musc_b200_preprocess_workspace_bytes");
  MUSC_TRY(require_sm100());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int2* hb = reinterpret_cast<int2*>(ws + plan.offsets[0]);
  int* hw = reinterpret_cast<int*>(ws + plan.offsets[1]);
  int2* vb = reinterpret_cast<int2*>(ws + plan.offsets[2]);
  int* vw = reinterpret_cast<int*>(ws + plan.offsets[3]);
  int table_items = out_w + out_h;
  image::tables_kernel<<<(table_items + 127) / 128, 128, 0, s>>>(plan.h, plan.v, filter, hb, hw, vb, vw);
  MUSC_TRY(check_launch("tables_kernel"));

  image::Params p;
  p.images = images;
  p.image_stride = image_stride_bytes;
  p.in_h = in_h;
  p.in_w = in_w;
  p.out_h = out_h;
  p.out_w = out_w;
  p.kh = plan.h.ksize;
  p.kv = plan.v.ksize;
  p.ty = plan.ty;
  p.max_rows = plan.max_rows;
  p.need_h = plan.need_h;
  p.need_v = plan.need_v;
  for (int c = 0; c < 3; ++c) {
    p.mean[c] = mean[c];
    p.stdev[c] = stdev[c];
  }
  p.hb = hb;
  p.hw = hw;
  p.vb = vb;
  p.vw = vw;
  p.out = out;
  switch (out_dtype) {
    case MUSC_B200_F32: return image::launch<float>(p, plan, n_images, s);
    case MUSC_B200_F16: return image::launch<__half>(p, plan, n_images, s);
    default: return image::launch<__nv_bfloat16>(p, plan, n_images, s);
  }
}
