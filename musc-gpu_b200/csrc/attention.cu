// Fused block attention of the ViT-L/14 encoder: out = softmax(q k^T * scale) v per
// (batch, head), the core of nn.MultiheadAttention as the reference's ViT
// blocks call it (models/backbone/open_clip/transformer.py:221-234), with the
// row softmax the reference moves into its aligned_dual kernel
// (models/modules/_attention_gpu.py:41-81) fused in, so the (L x L) logits and
// probabilities never reach memory.
//
// One CTA per (batch, head, 128-query tile); head_dim 64, fp16 or bf16 in/out
// (both operands of every MMA share the type), fp32 softmax and accumulation.  Warp roles:
//   warp 0     TMA: Q once, then K_j / V_j tiles of 128 keys into 2-deep rings;
//   warp 1     one thread issues tcgen05.mma: S_j = Q K_j^T (128x128x64) into a
//              double-buffered TMEM S, and PV_j = P_j V_j (128x64x128) into a
//              double-buffered TMEM PV (V is the MN-major B operand);
//   warps 2-9  softmax, two warps per query row (one per 64-key half of the
//              tile, exchanging partial row maxima through shared memory):
//              tcgen05.ld of S_j, online max / exp2 / row sum in fp32, P_j
//              written to shared memory in the input type, K-major 128-byte
//              swizzle layout the MMA reads; one tile later the same threads
//              read their 32 output dims of PV_j and accumulate
//              O = O * alpha_j + PV_j in registers (so the tensor core never
//              waits for a rescale); finally O / l goes out in the input type.
// QK_{j+1} overlaps softmax_j; PV_j overlaps softmax_{j+1}.
// Algorithmic work: 4 * L^2 * d flop per (batch, head); L^2 exponentials.
#include "common.cuh"
#include "tc.cuh"

#include <cfloat>
#include <mutex>
#include <vector>

namespace musc {
namespace attn {

constexpr int BQ = 128;       // query rows per CTA (TMEM lanes)
constexpr int BKV = 128;      // keys per tile
constexpr int D = 64;         // head dim: one 128-byte swizzle row of bf16
constexpr int KV_STAGES = 2;
constexpr int TILE_BYTES = BKV * D * 2;  // 16 KB (Q, K_j, V_j tiles)
constexpr int P_BYTES = BQ * BKV * 2;    // 32 KB (two 64-key swizzle column blocks)
constexpr int SOFTMAX_WARPS = 8;  // two per TMEM lane quarter
constexpr int THREADS = 32 * (2 + SOFTMAX_WARPS);
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0;      // S buffers at columns 0 and 128
constexpr int PV_COL = 256;   // PV buffers at columns 256 and 320
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;
// kind::f16 operand format: 0 = fp16, 1 = bf16 (A and B always share it).
template <bool FP16> constexpr uint32_t idesc_qk() { return tc::idesc_f16(BQ, BKV, FP16 ? 0 : 1); }
template <bool FP16> constexpr uint32_t idesc_pv() {
  return tc::idesc_f16(BQ, D, FP16 ? 0 : 1) | (1u << 16);  // B (V) MN-major
}

struct Smem {
  uint8_t q[TILE_BYTES];
  uint8_t k[KV_STAGES][TILE_BYTES];
  uint8_t v[KV_STAGES][TILE_BYTES];
  uint8_t p[2][P_BYTES];
  uint64_t q_full;
  uint64_t k_full[KV_STAGES], k_empty[KV_STAGES];
  uint64_t v_full[KV_STAGES], v_empty[KV_STAGES];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2];
  uint64_t o_full[2], o_empty[2];
  uint64_t drain;
  float red[2][2][BQ];  // [tile parity][column half][row]: partial row maxima / final sums
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;

struct Params {
  void* out;
  long long out_row_stride;  // elements between consecutive tokens of out
  int* err;
  int tokens, heads, n_q_tiles, n_kv;
  float scale_log2;          // scale * log2(e)
};

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (tc::mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  uint32_t iter = 0;
  while (true) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if ((++iter & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - start > WAIT_LIMIT_NS) {
        *abort_flag = 1;
        atomicExch(err, MUSC_B200_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// MN-major operand in the 128-byte swizzle (B = V tile: 64 head dims contiguous per key,
// 8-key groups 1024 bytes apart): leading byte offset = distance between 64-element MN
// blocks (unused with one block), stride byte offset 1024, layout type 2.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)(TILE_BYTES >> 4) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Barrier of the two softmax warps that share a TMEM lane quarter (named barrier
// 2 + quarter, 64 threads) that also ORs `flag` across them.
__device__ __forceinline__ bool pair_sync_any(int quarter, bool flag) {
  uint32_t res;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(res)
      : "r"((uint32_t)flag), "r"(2 + quarter)
      : "memory");
  return res != 0;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool FP16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (FP16) {
    __half2 t = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&t);
  } else {
    __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&t);
  }
}

template <bool FP16>
__global__ void __launch_bounds__(THREADS, 1)
attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                 const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;
  const int q_tile = blockIdx.x % p.n_q_tiles;
  const int bh = blockIdx.x / p.n_q_tiles;
  const int b = bh / p.heads, h = bh % p.heads;
  const int row0 = b * p.tokens;  // first token row of this batch item in the 2-D maps

  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_u32(&sm.q_full), 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      tc::mbar_init(tc::smem_u32(&sm.k_full[s]), 1);
      tc::mbar_init(tc::smem_u32(&sm.k_empty[s]), 1);
      tc::mbar_init(tc::smem_u32(&sm.v_full[s]), 1);
      tc::mbar_init(tc::smem_u32(&sm.v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(tc::smem_u32(&sm.s_full[s]), 1);
      tc::mbar_init(tc::smem_u32(&sm.s_empty[s]), SOFTMAX_WARPS);
      tc::mbar_init(tc::smem_u32(&sm.p_full[s]), SOFTMAX_WARPS);
      tc::mbar_init(tc::smem_u32(&sm.o_full[s]), 1);
      tc::mbar_init(tc::smem_u32(&sm.o_empty[s]), SOFTMAX_WARPS);
    }
    tc::mbar_init(tc::smem_u32(&sm.drain), 1);
    sm.abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tensormap(&map_q);
    tc::prefetch_tensormap(&map_k);
    tc::prefetch_tensormap(&map_v);
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_u32(&sm.tmem_base), TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = sm.tmem_base;
  const int n_kv = p.n_kv;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      const uint32_t qf = tc::smem_u32(&sm.q_full);
      tc::mbar_arrive_expect_tx(qf, TILE_BYTES);
      tc::tma_load_2d(tc::smem_u32(sm.q), &map_q, h * D, row0 + q_tile * BQ, qf);
      uint32_t issued_phase_k[KV_STAGES] = {0, 0}, issued_phase_v[KV_STAGES] = {0, 0};
      bool issued_k[KV_STAGES] = {false, false}, issued_v[KV_STAGES] = {false, false};
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (uint32_t)(j / KV_STAGES) & 1u;
        if (!wait_bounded(tc::smem_u32(&sm.k_empty[s]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        const uint32_t kf = tc::smem_u32(&sm.k_full[s]);
        tc::mbar_arrive_expect_tx(kf, TILE_BYTES);
        tc::tma_load_2d(tc::smem_u32(sm.k[s]), &map_k, h * D, row0 + j * BKV, kf);
        issued_k[s] = true, issued_phase_k[s] = ph;
        if (!wait_bounded(tc::smem_u32(&sm.v_empty[s]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        const uint32_t vf = tc::smem_u32(&sm.v_full[s]);
        tc::mbar_arrive_expect_tx(vf, TILE_BYTES);
        tc::tma_load_2d(tc::smem_u32(sm.v[s]), &map_v, h * D, row0 + j * BKV, vf);
        issued_v[s] = true, issued_phase_v[s] = ph;
      }
      // Let every copy this thread issued land before the CTA can exit.
      const uint64_t start = global_ns();
      while (!tc::mbar_try_wait(qf, 0) && global_ns() - start < WAIT_LIMIT_NS) {
      }
      for (int s = 0; s < KV_STAGES && !ok; ++s) {
        const uint64_t t0 = global_ns();
        if (issued_k[s])
          while (!tc::mbar_try_wait(tc::smem_u32(&sm.k_full[s]), issued_phase_k[s]) &&
                 global_ns() - t0 < WAIT_LIMIT_NS) {
          }
        if (issued_v[s])
          while (!tc::mbar_try_wait(tc::smem_u32(&sm.v_full[s]), issued_phase_v[s]) &&
                 global_ns() - t0 < WAIT_LIMIT_NS) {
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = wait_bounded(tc::smem_u32(&sm.q_full), 0, abort_flag, p.err);
      tc::fence_after_sync();
      const uint32_t q_addr = tc::smem_u32(sm.q);
      for (int j = 0; j <= n_kv && ok; ++j) {
        if (j < n_kv) {
          // S_j = Q K_j^T
          const int s = j % KV_STAGES, sb = j & 1;
          const uint32_t ph = (uint32_t)(j / KV_STAGES) & 1u, sph = (uint32_t)(j >> 1) & 1u;
          if (!wait_bounded(tc::smem_u32(&sm.k_full[s]), ph, abort_flag, p.err) ||
              !wait_bounded(tc::smem_u32(&sm.s_empty[sb]), sph ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t k_addr = tc::smem_u32(sm.k[s]);
          const uint32_t d_tmem = tmem_base + (uint32_t)(S_COL + sb * BKV);
#pragma unroll
          for (int k16 = 0; k16 < D / 16; ++k16)
            tc::mma_f16_ss(d_tmem, tc::desc_k_sw128(q_addr + k16 * 32), tc::desc_k_sw128(k_addr + k16 * 32),
                           idesc_qk<FP16>(), k16 ? 1u : 0u);
          tc::mma_commit(tc::smem_u32(&sm.k_empty[s]));
          tc::mma_commit(tc::smem_u32(&sm.s_full[sb]));
        }
        if (j >= 1) {
          // PV_{j-1} = P_{j-1} V_{j-1}
          const int i = j - 1;
          const int s = i % KV_STAGES, pb = i & 1;
          const uint32_t ph = (uint32_t)(i / KV_STAGES) & 1u, pph = (uint32_t)(i >> 1) & 1u;
          if (!wait_bounded(tc::smem_u32(&sm.v_full[s]), ph, abort_flag, p.err) ||
              !wait_bounded(tc::smem_u32(&sm.p_full[pb]), pph, abort_flag, p.err) ||
              !wait_bounded(tc::smem_u32(&sm.o_empty[pb]), pph ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t p_addr = tc::smem_u32(sm.p[pb]);
          const uint32_t v_addr = tc::smem_u32(sm.v[s]);
          const uint32_t d_tmem = tmem_base + (uint32_t)(PV_COL + pb * D);
#pragma unroll
          for (int k16 = 0; k16 < BKV / 16; ++k16) {
            const uint32_t pa = p_addr + (uint32_t)((k16 >> 2) * (BQ * 128) + (k16 & 3) * 32);
            const uint32_t va = v_addr + (uint32_t)(k16 * 2048);  // 16 keys = two 8-key groups
            tc::mma_f16_ss(d_tmem, tc::desc_k_sw128(pa), desc_mn_sw128(va), idesc_pv<FP16>(), k16 ? 1u : 0u);
          }
          tc::mma_commit(tc::smem_u32(&sm.v_empty[s]));
          tc::mma_commit(tc::smem_u32(&sm.o_full[pb]));
        }
      }
      if (!ok) {
        tc::mma_commit(tc::smem_u32(&sm.drain));
        const uint64_t start = global_ns();
        while (!tc::mbar_try_wait(tc::smem_u32(&sm.drain), 0) && global_ns() - start < WAIT_LIMIT_NS) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + output
    // Two warps per TMEM lane quarter: warp half h owns key columns [64h, 64h + 64) of S
    // and output dims [32h, 32h + 32); the pair exchanges its partial row maxima once per
    // tile through shared memory (named barrier 2 + quarter, 64 threads).  Every stop
    // decision is taken at a pair barrier, so the two warps always leave together.
    const int quarter = warp & 3;
    const int half = (warp - 2) / 4;
    const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    float o[D / 2];
#pragma unroll
    for (int d = 0; d < D / 2; ++d) o[d] = 0.f;
    float m_run = -FLT_MAX, l_half = 0.f, alpha_prev = 1.f;
    bool ok = true;
    int j = 0;
    for (; j < n_kv; ++j) {
      const int sb = j & 1;
      ok = ok && wait_bounded(tc::smem_u32(&sm.s_full[sb]), (uint32_t)(j >> 1) & 1u, abort_flag, p.err);
      float sv[BKV / 2];
      float mt = -FLT_MAX;
      const int valid = p.tokens - j * BKV - half * (BKV / 2);  // keys past the sequence end are masked
      if (__all_sync(0xffffffffu, ok)) {
        tc::fence_after_sync();
        {
          // both 32-column loads in flight before one wait
          uint32_t raw0[32], raw1[32];
          static_assert(BKV / 2 == 64, "two 32-column TMEM loads per half tile");
          tc::tmem_ld_32x32b_x32(lane_base + (uint32_t)(S_COL + sb * BKV + half * (BKV / 2)), raw0);
          tc::tmem_ld_32x32b_x32(lane_base + (uint32_t)(S_COL + sb * BKV + half * (BKV / 2) + 32), raw1);
          tc::tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) sv[t] = __uint_as_float(raw0[t]), sv[32 + t] = __uint_as_float(raw1[t]);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(tc::smem_u32(&sm.s_empty[sb]));
        // row maximum over four independent partial maxima (exact: max is order-free)
        float mq[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
#pragma unroll
        for (int c = 0; c < BKV / 2; ++c) {
          sv[c] = c < valid ? sv[c] * p.scale_log2 : -FLT_MAX;
          mq[c & 3] = fmaxf(mq[c & 3], sv[c]);
        }
        mt = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        sm.red[j & 1][half][r] = mt;
      } else {
        ok = false;
      }
      if (pair_sync_any(quarter, !ok)) break;
      mt = fmaxf(mt, sm.red[j & 1][half ^ 1][r]);
      const float m_new = fmaxf(m_run, mt);
      const float alpha = ex2(m_run - m_new);
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // four independent partial row sums
      uint8_t* prow = sm.p[sb] + half * (BQ * 128) + r * 128;  // this half's 64-key column block
#pragma unroll
      for (int ch = 0; ch < BKV / 16; ++ch) {  // 16-byte chunks of 8 keys
        float e[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int c = ch * 8 + t;
          e[t] = c < valid ? ex2(sv[c] - m_new) : 0.f;
          ls[t & 3] += e[t];
        }
        uint4 pk = make_uint4(pack2<FP16>(e[0], e[1]), pack2<FP16>(e[2], e[3]), pack2<FP16>(e[4], e[5]),
                              pack2<FP16>(e[6], e[7]));
        *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = pk;
      }
      const float lsum = (ls[0] + ls[1]) + (ls[2] + ls[3]);
      l_half = l_half * alpha + lsum;
      m_run = m_new;
      tc::fence_proxy_async_smem();  // P stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(tc::smem_u32(&sm.p_full[sb]));
      if (j >= 1) {
        // accumulate this half's dims of PV_{j-1}
        const int pb = (j - 1) & 1;
        ok = wait_bounded(tc::smem_u32(&sm.o_full[pb]), (uint32_t)((j - 1) >> 1) & 1u, abort_flag, p.err);
        if (__all_sync(0xffffffffu, ok)) {
          tc::fence_after_sync();
          uint32_t raw[32];
          tc::tmem_ld_32x32b_x32(lane_base + (uint32_t)(PV_COL + pb * D + half * 32), raw);
          tc::tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) o[t] = fmaf(o[t], alpha_prev, __uint_as_float(raw[t]));
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(tc::smem_u32(&sm.o_empty[pb]));
        } else {
          ok = false;
        }
      }
      alpha_prev = alpha;
    }
    if (j == n_kv) {
      // last PV
      const int pb = (n_kv - 1) & 1;
      ok = ok && wait_bounded(tc::smem_u32(&sm.o_full[pb]), (uint32_t)((n_kv - 1) >> 1) & 1u, abort_flag, p.err);
      if (__all_sync(0xffffffffu, ok)) {
        tc::fence_after_sync();
        uint32_t raw[32];
        tc::tmem_ld_32x32b_x32(lane_base + (uint32_t)(PV_COL + pb * D + half * 32), raw);
        tc::tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) o[t] = fmaf(o[t], alpha_prev, __uint_as_float(raw[t]));
      } else {
        ok = false;
      }
      // row sum = both halves' partial sums, exchanged in the parity buffer the last
      // tile did not use (the partner may still be reading the last tile's maxima)
      const int pf = n_kv & 1;
      sm.red[pf][half][r] = l_half;
      const bool stop = pair_sync_any(quarter, !ok);
      const float l_run = l_half + sm.red[pf][half ^ 1][r];
      const int token = q_tile * BQ + r;
      if (!stop && token < p.tokens) {
        const float inv = 1.f / l_run;
        uint16_t* dst = static_cast<uint16_t*>(p.out) + ((long long)b * p.tokens + token) * p.out_row_stride +
                        h * D + half * 32;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint4 pk = make_uint4(pack2<FP16>(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv),
                                pack2<FP16>(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv),
                                pack2<FP16>(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv),
                                pack2<FP16>(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv));
          *reinterpret_cast<uint4*>(dst + c8 * 8) = pk;
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace attn

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* fn) {
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

// bf16 [rows][row_stride] with the head slices as the inner dimension; box = one head
// (64 elements = 128 bytes) x 128 token rows, 128-byte swizzle.
int make_token_map(CUtensorMap* map, const void* base, long long rows, int inner, long long row_stride,
                   bool fp16) {
  EncodeTiledFn encode;
  MUSC_TRY(encode_fn(&encode));
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)attn::D, (cuuint32_t)attn::BKV};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                      const_cast<void*>(base), dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MUSC_B200_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed: " + std::to_string((int)r));
  return MUSC_B200_OK;
}

}  // namespace
}  // namespace musc

using namespace musc;

extern "C" int musc_b200_attention_fwd(const void* q, const void* k, const void* v, void* out, int dtype,
                                       int batch, int tokens, int heads, int head_dim,
                                       long long qkv_row_stride, long long out_row_stride, float scale,
                                       musc_b200_stream stream) {
  if (!q || !k || !v || !out) return fail(MUSC_B200_ERR_INVALID, "attention: null pointer");
  if (dtype != MUSC_B200_F16 && dtype != MUSC_B200_BF16)
    return fail(MUSC_B200_ERR_INVALID, "attention: dtype must be f16 or bf16");
  const bool fp16 = dtype == MUSC_B200_F16;
  if (batch <= 0 || tokens <= 0 || heads <= 0)
    return fail(MUSC_B200_ERR_INVALID, "attention: batch, tokens and heads must be positive");
  if (head_dim != attn::D) return fail(MUSC_B200_ERR_INVALID, "attention: head_dim must be 64");
  if (qkv_row_stride < (long long)heads * head_dim || out_row_stride < (long long)heads * head_dim ||
      qkv_row_stride % 8 != 0 || out_row_stride % 8 != 0)
    return fail(MUSC_B200_ERR_INVALID, "attention: row strides must hold heads*head_dim and be multiples of 8");
  for (const void* ptr : {q, k, v, (const void*)out})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return fail(MUSC_B200_ERR_INVALID, "attention: q, k, v and out must be 16-byte aligned");
  const long long rows = (long long)batch * tokens;
  if (rows > 0x7FFFFFFFLL) return fail(MUSC_B200_ERR_INVALID, "attention: batch*tokens must fit in int32");
  MUSC_TRY(require_sm100());
  const int inner = heads * head_dim;
  CUtensorMap mq, mk, mv;
  MUSC_TRY(make_token_map(&mq, q, rows, inner, qkv_row_stride, fp16));
  MUSC_TRY(make_token_map(&mk, k, rows, inner, qkv_row_stride, fp16));
  MUSC_TRY(make_token_map(&mv, v, rows, inner, qkv_row_stride, fp16));
  attn::Params p;
  p.out = out;
  p.out_row_stride = out_row_stride;
  p.err = device_error_ptr();
  if (!p.err) return fail(MUSC_B200_ERR_CUDA, "attention: device error word unavailable");
  p.tokens = tokens;
  p.heads = heads;
  p.n_q_tiles = (tokens + attn::BQ - 1) / attn::BQ;
  p.n_kv = (tokens + attn::BKV - 1) / attn::BKV;
  p.scale_log2 = scale * 1.4426950408889634f;
  static std::mutex m;
  static bool attr_done[64] = {false};
  int dev = 0;
  MUSC_CUDA(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lock(m);
    if (dev >= 64 || !attr_done[dev]) {
      MUSC_CUDA(cudaFuncSetAttribute(attn::attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)attn::SMEM_BYTES));
      MUSC_CUDA(cudaFuncSetAttribute(attn::attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)attn::SMEM_BYTES));
      if (dev < 64) attr_done[dev] = true;
    }
  }
  const long long grid = (long long)batch * heads * p.n_q_tiles;
  if (grid > 0x7FFFFFFFLL) return fail(MUSC_B200_ERR_INVALID, "attention: grid too large");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (fp16)
    attn::attention_kernel<true><<<(unsigned)grid, attn::THREADS, attn::SMEM_BYTES, s>>>(mq, mk, mv, p);
  else
    attn::attention_kernel<false><<<(unsigned)grid, attn::THREADS, attn::SMEM_BYTES, s>>>(mq, mk, mv, p);
  return check_launch("attention_kernel");
}
