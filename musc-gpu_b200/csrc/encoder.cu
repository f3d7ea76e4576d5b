// Residual add + LayerNorm of the ViT-L/14 blocks: the two normalisation points of
// each residual block of the reference's CLIP vision tower
// (models/backbone/open_clip/transformer.py:236-249: x = x + attn(ln_1(x));
// x = x + mlp(ln_2(x))), with the residual add of the preceding branch fused in:
//
//   x[row] += delta[row]            (fp32 residual stream; delta is the branch's 16-bit
//                                    GEMM output, widened exactly, or absent)
//   out[row] = 16-bit( (x - mean) / sqrt(var + eps) * gamma + beta )
//
// one read of x and delta and one write of x and out per row, where the unfused form
// makes separate passes for the add, the fp32 LayerNorm and the cast.  One warp per row;
// mean and the biased variance in fp32 with the two-pass (centred) form, as torch's
// layer_norm, so results agree with it to fp32 rounding.
#include "common.cuh"

#include <cuda_bf16.h>

namespace musc {
namespace {

constexpr int kLnWarps = 8;
constexpr int kLnMaxVec = 16;  // float4s per lane: channels <= 2048

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __half2 a = *reinterpret_cast<const __half2*>(&u.x), b = *reinterpret_cast<const __half2*>(&u.y);
  const float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float4 v);
template <>
__device__ __forceinline__ void store4<__half>(__half* p, float4 v) {
  __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// DT: the type of delta (ignored when has_delta is false); OT: the output type.
template <typename DT, typename OT>
__global__ void __launch_bounds__(kLnWarps * 32)
add_layernorm_kernel(float* __restrict__ x, const DT* __restrict__ delta, bool has_delta,
                     const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                     OT* __restrict__ out, long long rows, int channels) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;  // warp-uniform
  float* xr = x + row * channels;
  const int nvec = channels / 128;  // float4s per lane
  float4 v[kLnMaxVec];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    if (i < nvec) {
      const int c = i * 128 + lane * 4;
      float4 a = *reinterpret_cast<const float4*>(xr + c);
      if (has_delta) {
        const float4 d = load4<DT>(delta + row * channels + c);
        a.x += d.x; a.y += d.y; a.z += d.z; a.w += d.w;
        *reinterpret_cast<float4*>(xr + c) = a;
      }
      v[i] = a;
      s += (a.x + a.y) + (a.z + a.w);
    }
  }
  const float mean = warp_sum(s) / (float)channels;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    if (i < nvec) {
      const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
      q = fmaf(dx, dx, fmaf(dy, dy, fmaf(dz, dz, fmaf(dw, dw, q))));
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / (float)channels + eps);
  OT* orow = out + row * channels;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    if (i < nvec) {
      const int c = i * 128 + lane * 4;
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma + c));
      const float4 b = __ldg(reinterpret_cast<const float4*>(beta + c));
      store4<OT>(orow + c, make_float4((v[i].x - mean) * rstd * g.x + b.x, (v[i].y - mean) * rstd * g.y + b.y,
                                       (v[i].z - mean) * rstd * g.z + b.z, (v[i].w - mean) * rstd * g.w + b.w));
    }
  }
}

template <typename DT, typename OT>
int launch(float* x, const void* delta, const float* gamma, const float* beta, float eps, void* out,
           long long rows, int channels, cudaStream_t s) {
  const long long blocks = (rows + kLnWarps - 1) / kLnWarps;
  add_layernorm_kernel<DT, OT><<<(unsigned)blocks, kLnWarps * 32, 0, s>>>(
      x, static_cast<const DT*>(delta), delta != nullptr, gamma, beta, eps, static_cast<OT*>(out), rows, channels);
  return check_launch("add_layernorm_kernel");
}

}  // namespace
}  // namespace musc

using namespace musc;

extern "C" int musc_b200_add_layernorm(float* x, const void* delta, int delta_dtype, const float* gamma,
                                       const float* beta, float eps, void* out, int out_dtype, long long rows,
                                       int channels, musc_b200_stream stream) {
  if (!x || !gamma || !beta || !out) return fail(MUSC_B200_ERR_INVALID, "add_layernorm: null pointer");
  if (rows <= 0 || channels <= 0 || channels % 128 != 0 || channels > 128 * kLnMaxVec)
    return fail(MUSC_B200_ERR_INVALID, "add_layernorm: rows > 0 and channels a multiple of 128 up to 2048");
  if (rows > 0x7FFFFFFFLL * kLnWarps) return fail(MUSC_B200_ERR_INVALID, "add_layernorm: too many rows");
  if (out_dtype != MUSC_B200_F16 && out_dtype != MUSC_B200_BF16)
    return fail(MUSC_B200_ERR_INVALID, "add_layernorm: out dtype must be f16 or bf16");
  if (delta && delta_dtype != MUSC_B200_F16 && delta_dtype != MUSC_B200_BF16)
    return fail(MUSC_B200_ERR_INVALID, "add_layernorm: delta dtype must be f16 or bf16");
  for (const void* p : {(const void*)x, delta, (const void*)gamma, (const void*)beta, (const void*)out})
    if (p && reinterpret_cast<uintptr_t>(p) % 16 != 0)
      return fail(MUSC_B200_ERR_INVALID, "add_layernorm: pointers must be 16-byte aligned");
  MUSC_TRY(require_sm100());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool dh = delta_dtype != MUSC_B200_BF16, oh = out_dtype == MUSC_B200_F16;
  if (dh && oh) return launch<__half, __half>(x, delta, gamma, beta, eps, out, rows, channels, s);
  if (dh && !oh) return launch<__half, __nv_bfloat16>(x, delta, gamma, beta, eps, out, rows, channels, s);
  if (!dh && oh) return launch<__nv_bfloat16, __half>(x, delta, gamma, beta, eps, out, rows, channels, s);
  return launch<__nv_bfloat16, __nv_bfloat16>(x, delta, gamma, beta, eps, out, rows, channels, s);
}
