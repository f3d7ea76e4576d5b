// MSM mutual scoring: models/modules/_MSM.py and models/modules/_MSM_gpu.py.
//
// Reference: compute_scores_fast / MSM (models/modules/_MSM.py:10-59) and the
// reference GPU driver models/modules/_MSM_gpu.py:701-830.
//
// Pipeline for one (layer, radius) bank z[N*P][C] fp32:
//   1. prep_bank_kernel: per row, a power-of-two scale 2^k putting max|z|
//      in [2^14, 2^15), the split z*2^k = hi + lo with hi = fp16(z*2^k) and
//      lo = fp16(z*2^k - hi) (together ~22 significant bits, fp32-class
//      accuracy), the fp32 squared norm (float64 accumulation) and 2^-k.
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
#include "tc.cuh"

#include <algorithm>
#include <cfloat>
#include <cstdlib>
#include <mutex>
#include <vector>

namespace musc {

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct BankLayout {
  size_t hi, lo, norm, inv, total;
};

static BankLayout bank_layout(long long rows, int channels) {
  const size_t plane = align_up((size_t)rows * channels * 2, 1024);
  const size_t vec = align_up((size_t)rows * 4, 1024);
  return {0, plane, 2 * plane, 2 * plane + vec, 2 * plane + 2 * vec};
}

// ------------------------------------------------------------------ prep
constexpr int kPrepWarps = 8;

__global__ void __launch_bounds__(kPrepWarps * 32)
prep_bank_kernel(const float* __restrict__ z, long long rows, int channels, __half* __restrict__ hi,
                 __half* __restrict__ lo, float* __restrict__ norm2, float* __restrict__ inv_scale) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
  if (row >= rows) return;  // warp-uniform
  const float* zr = z + row * channels;
  float m = 0.f;
  double ss = 0.0;
  for (int c = lane * 4; c < channels; c += 128) {
    float4 v = __ldg(reinterpret_cast<const float4*>(zr + c));
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
  for (int c = lane * 4; c < channels; c += 128) {
    float4 v = __ldg(reinterpret_cast<const float4*>(zr + c));
    const float x[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
    __half h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = __float2half_rn(x[e]);
      l[e] = __float2half_rn(x[e] - __half2float(h[e]));
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
  if (lane == 0) {
    norm2[row] = (float)ss;
    inv_scale[row] = ldexpf(1.f, -k);
  }
}

// ------------------------------------------------------------------ nearest
namespace nearest {
constexpr int CTA_M = 128;        // query rows per CTA (TMEM lanes)
constexpr int BN = 256;           // reference rows per tile (TMEM columns per accumulator)
constexpr int BK = 32;            // fp16 elements per K slice = one 64-byte swizzle row
constexpr int A_BYTES = CTA_M * BK * 2;  // 8 KB per plane
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;  // 4 s per wait
constexpr float INF = FLT_MAX;
constexpr int RING = 8;      // tile indices handed from the producer to the MMA and epilogue warps
constexpr int CHUNK = 8;     // tiles claimed per atomic by the dynamic scheduler

// Tile shapes.  Single CTA: 128 x 256 tiles, the CTA holds all 256 B rows of
// a K slice.  CTA pair (cta_group::2): 256 x 256 tiles over two SMs; each CTA
// loads 128 A rows and 128 B rows, so per MMA an SM reads 8 KB of operands
// from shared memory instead of 12 KB and fetches a third fewer bytes from
// L2, and the smaller stages allow a 6-deep ring in the same shared memory.
template <bool PAIR>
struct Cfg {
  static constexpr int TILE_M = PAIR ? 256 : 128;
  static constexpr int CTA_N = PAIR ? 128 : 256;
  static constexpr int B_BYTES = CTA_N * BK * 2;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;  // 48 KB / 32 KB
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int GROUP_M = PAIR ? 32 : 64;  // m-tiles swept together (8192 query rows)
  static constexpr uint32_t IDESC = tc::idesc_f16(TILE_M, BN, /*fp16*/ 0);
  static constexpr int EPI_ARRIVALS = (PAIR ? 2 : 1) * EPI_WARPS;  // epilogue warps releasing a tile
};

template <int STAGES, int STAGE_BYTES>
struct Smem {
  uint8_t tiles[STAGES][STAGE_BYTES];  // 1024-aligned base
  float col_norm[BN];
  float col_w[BN];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[NUM_ACC];
  uint64_t acc_empty[NUM_ACC];
  uint64_t drain;
  uint64_t ring_full[RING];
  uint64_t ring_empty[RING];
  long long tile_ring[RING];
  uint32_t tmem_base;
  int abort_flag;
};
template <bool PAIR>
using SmemT = Smem<Cfg<PAIR>::STAGES, Cfg<PAIR>::STAGE_BYTES>;
template <bool PAIR>
constexpr size_t smem_bytes() {
  return sizeof(SmemT<PAIR>) + 1024;
}

struct Params {
  const float* q_norm;
  const float* q_inv;
  const float* r_norm;
  const float* r_inv;
  unsigned int* nearest;  // float bits, layout [row / rpb][image][row % rpb]
  unsigned long long* sched;  // dynamic-scheduler counter (zeroed before the launch), or nullptr
  int* err;
  long long q_rows, r_rows, q_first_row;
  long long tile_begin, tile_end;  // linear tile range processed by this launch
  long long rows_per_block;        // rpb of the nearest layout
  int blocked;                     // 0: rows_per_block covers every row addressed
  int patches;                     // P
  int n_images;
  int num_kb;
  int num_m, num_n;
};

__host__ __device__ inline void tile_coords(long long tile, int num_m, int num_n, int group_m, int* m_blk,
                                            int* n_blk) {
  const long long group = tile / ((long long)group_m * num_n);
  const int first_m = (int)(group * group_m);
  const int gm = num_m - first_m < group_m ? num_m - first_m : group_m;
  const long long local = tile - group * group_m * (long long)num_n;
  *m_blk = first_m + (int)(local % gm);
  *n_blk = (int)(local / gm);
}

// Symmetric mode: tile (m, n) holds an element (r, c) with img(r) < img(c).
__host__ __device__ inline bool sym_needed(int m, int n, long long rows, int patches, int n_images, int tile_m) {
  const long long r0 = (long long)m * tile_m;
  const long long img_r = r0 / patches;
  if (img_r >= n_images - 1) return false;
  long long c_last = (long long)n * BN + BN - 1;
  if (c_last > rows - 1) c_last = rows - 1;
  return c_last / patches > img_r;
}

// Bounded wait: true when the phase completed; false after the time limit
// (which raises this CTA's abort flag, the peer CTA's when `peer_abort` is a
// cluster address, and the device error word) or when an abort was already
// raised.  CLUSTER selects acquire at cluster scope, for phases completed by
// the other CTA of a pair.
template <bool CLUSTER>
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                                             uint32_t peer_abort) {
  auto ready = [&]() { return CLUSTER ? tc::mbar_try_wait_cluster(bar, parity) : tc::mbar_try_wait(bar, parity); };
  if (ready()) return true;
  const uint64_t start = global_ns();
  uint32_t iter = 0;
  while (true) {
    if (ready()) return true;
    if ((++iter & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - start > WAIT_LIMIT_NS) {
        *abort_flag = 1;
        if (peer_abort) tc::st_cluster_u32(peer_abort, 1u);
        atomicExch(err, MUSC_B200_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void named_sync_epi() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}

// Barrier over the epilogue warps that also ORs `flag` across them, so every
// epilogue thread takes the same branch afterwards.
__device__ __forceinline__ bool named_sync_epi_any(int flag) {
  uint32_t res;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(res)
      : "r"(flag), "n"(EPI_WARPS * 32)
      : "memory");
  return res != 0;
}

__device__ __forceinline__ long long table_index(const Params& p, int img, long long row) {
  if (!p.blocked) return (long long)img * p.rows_per_block + row;
  const long long blk = row / p.rows_per_block;
  return (blk * p.n_images + img) * p.rows_per_block + (row - blk * p.rows_per_block);
}

__device__ __forceinline__ void flush_min(const Params& p, long long row, int img, float m) {
  if (m < INF) {
    const float v = m > 0.f ? m : 0.f;
    atomicMin(p.nearest + table_index(p, img, row), __float_as_uint(v));
  }
}

// After the call lane l holds min over the warp's 32 lanes of v[l] (a
// transposing butterfly: 31 shuffles for 32 columns).
__device__ __forceinline__ float warp_column_min(float (&v)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = upper ? v[i] : v[i + s];
      const float keep = upper ? v[i + s] : v[i];
      const float recv = __shfl_xor_sync(0xffffffffu, send, s);
      v[i] = fminf(keep, recv);
    }
  }
  return v[0];
}

// Roles (one CTA, or each CTA of a pair): warp 0 lane 0 loads (TMA), warp 1
// lane 0 issues the MMAs (the even CTA only, for a pair), warps 2-5 are the
// epilogue.  In a pair the even CTA (rank 0) owns the schedule: its producer
// claims each tile, writes the index into both CTAs' rings and both CTAs'
// loads complete on its `full` barriers; its MMA thread signals both CTAs'
// `empty` and `acc_full` barriers; both epilogues release the accumulator and
// the ring slot on its barriers.
template <bool SYM, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
nearest_kernel(const __grid_constant__ CUtensorMap map_q_hi, const __grid_constant__ CUtensorMap map_q_lo,
               const __grid_constant__ CUtensorMap map_r_hi, const __grid_constant__ CUtensorMap map_r_lo,
               const Params p) {
  using C = Cfg<PAIR>;
  extern __shared__ uint8_t smem_raw[];
  SmemT<PAIR>& sm =
      *reinterpret_cast<SmemT<PAIR>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;
  const uint32_t rank = PAIR ? tc::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const uint32_t peer_abort = PAIR ? tc::mapa(tc::smem_u32(&sm.abort_flag), rank ^ 1u) : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      tc::mbar_init(tc::smem_u32(&sm.full[s]), 1);
      tc::mbar_init(tc::smem_u32(&sm.empty[s]), 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      tc::mbar_init(tc::smem_u32(&sm.acc_full[a]), 1);
      tc::mbar_init(tc::smem_u32(&sm.acc_empty[a]), C::EPI_ARRIVALS);
    }
    tc::mbar_init(tc::smem_u32(&sm.drain), 1);
    for (int i = 0; i < RING; ++i) {
      tc::mbar_init(tc::smem_u32(&sm.ring_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&sm.ring_empty[i]), C::EPI_ARRIVALS);
    }
    sm.abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tensormap(&map_q_hi);
    tc::prefetch_tensormap(&map_q_lo);
    tc::prefetch_tensormap(&map_r_hi);
    tc::prefetch_tensormap(&map_r_lo);
  }
  if (warp == 1) {
    if (PAIR) {
      tc::tmem_alloc_pair(tc::smem_u32(&sm.tmem_base), TMEM_COLS);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(tc::smem_u32(&sm.tmem_base), TMEM_COLS);
      tc::tmem_relinquish();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (PAIR) tc::cluster_sync();  // the peer's barriers exist before anything arrives on them
  tc::fence_after_sync();
  const uint32_t tmem_base = sm.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[C::STAGES];
      bool issued[C::STAGES];
      for (int s = 0; s < C::STAGES; ++s) issued[s] = false, issued_phase[s] = 0;
      bool ok = true;
      const long long group_id = PAIR ? (long long)tc::cluster_id_x() : (long long)blockIdx.x;
      const long long n_groups = PAIR ? (long long)tc::cluster_count_x() : (long long)gridDim.x;
      long long next_static = p.tile_begin + group_id, chunk_cur = 0, chunk_end = 0;
      // Next tile (linear index), or -1.  Static: stride = number of CTAs (pairs).
      // Dynamic: claim CHUNK consecutive indices per atomic, so CTAs that start late
      // (their SM busy with another kernel, e.g. a collective) simply take fewer.
      auto next_tile = [&]() -> long long {
        while (true) {
          long long t;
          if (p.sched) {
            if (chunk_cur >= chunk_end) {
              const long long c = (long long)atomicAdd(p.sched, 1ull);
              chunk_cur = p.tile_begin + c * CHUNK;
              chunk_end = chunk_cur + CHUNK < p.tile_end ? chunk_cur + CHUNK : p.tile_end;
              if (chunk_cur >= p.tile_end) return -1;
            }
            t = chunk_cur++;
          } else {
            t = next_static;
            if (t >= p.tile_end) return -1;
            next_static += n_groups;
          }
          if (!SYM) return t;
          int mb, nb;
          tile_coords(t, p.num_m, p.num_n, C::GROUP_M, &mb, &nb);
          if (sym_needed(mb, nb, p.r_rows, p.patches, p.n_images, C::TILE_M)) return t;
        }
      };
      for (int local = 0; ok; ++local) {
        const int slot = local % RING;
        const uint32_t ring_parity = (uint32_t)(local / RING) & 1u;
        long long tile;
        if (leader) {
          if (!wait_bounded<PAIR>(tc::smem_u32(&sm.ring_empty[slot]), ring_parity ^ 1u, abort_flag, p.err,
                                  peer_abort)) {
            ok = false;
            break;
          }
          tile = next_tile();
          sm.tile_ring[slot] = tile;
          if (PAIR) {
            tc::st_cluster_s64(tc::mapa(tc::smem_u32(&sm.tile_ring[slot]), 1u), tile);
            tc::mbar_arrive_cluster(tc::mapa(tc::smem_u32(&sm.ring_full[slot]), 1u));
          }
          tc::mbar_arrive(tc::smem_u32(&sm.ring_full[slot]));
        } else {
          if (!wait_bounded<true>(tc::smem_u32(&sm.ring_full[slot]), ring_parity, abort_flag, p.err, peer_abort)) {
            ok = false;
            break;
          }
          tile = sm.tile_ring[slot];
        }
        if (tile < 0) break;
        int m_blk, n_blk;
        tile_coords(tile, p.num_m, p.num_n, C::GROUP_M, &m_blk, &n_blk);
        const int a_row = m_blk * C::TILE_M + (int)rank * CTA_M;
        const int b_row = n_blk * BN + (int)rank * C::CTA_N;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!wait_bounded<false>(tc::smem_u32(&sm.empty[stage]), phase ^ 1, abort_flag, p.err, peer_abort)) {
            ok = false;
            break;
          }
          const uint32_t full_local = tc::smem_u32(&sm.full[stage]);
          // The leader's barrier counts both CTAs' bytes of this stage.
          if (leader) tc::mbar_arrive_expect_tx(full_local, (PAIR ? 2 : 1) * C::STAGE_BYTES);
          const uint32_t base = tc::smem_u32(sm.tiles[stage]);
          const int kc = kb * BK;
          if (PAIR) {
            const uint32_t full = tc::mapa(full_local, 0u);
            tc::tma_load_2d_pair(base, &map_q_hi, kc, a_row, full);
            tc::tma_load_2d_pair(base + A_BYTES, &map_q_lo, kc, a_row, full);
            tc::tma_load_2d_pair(base + 2 * A_BYTES, &map_r_hi, kc, b_row, full);
            tc::tma_load_2d_pair(base + 2 * A_BYTES + C::B_BYTES, &map_r_lo, kc, b_row, full);
          } else {
            tc::tma_load_2d(base, &map_q_hi, kc, a_row, full_local);
            tc::tma_load_2d(base + A_BYTES, &map_q_lo, kc, a_row, full_local);
            tc::tma_load_2d(base + 2 * A_BYTES, &map_r_hi, kc, b_row, full_local);
            tc::tma_load_2d(base + 2 * A_BYTES + C::B_BYTES, &map_r_lo, kc, b_row, full_local);
          }
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == C::STAGES) stage = 0, phase ^= 1;
        }
      }
      if (!ok) {
        // Let the copies already in flight land before the CTA exits.  The
        // leader watches its `full` barriers (one deadline for all stages); the
        // peer's copies complete on the leader's barriers, so it gives them a
        // fixed 2 ms, far above the latency of one copy.
        const uint64_t start = global_ns();
        if (leader) {
          for (int s = 0; s < C::STAGES; ++s) {
            if (!issued[s]) continue;
            while (!tc::mbar_try_wait(tc::smem_u32(&sm.full[s]), issued_phase[s]) &&
                   global_ns() - start < WAIT_LIMIT_NS) {
            }
          }
        } else {
          while (global_ns() - start < 2000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int local = 0; ok; ++local) {
        const int slot = local % RING;
        if (!wait_bounded<false>(tc::smem_u32(&sm.ring_full[slot]), (uint32_t)(local / RING) & 1u, abort_flag,
                                 p.err, peer_abort)) {
          ok = false;
          break;
        }
        if (sm.tile_ring[slot] < 0) break;
        if (!wait_bounded<PAIR>(tc::smem_u32(&sm.acc_empty[acc]), acc_phase ^ 1, abort_flag, p.err, peer_abort)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!wait_bounded<false>(tc::smem_u32(&sm.full[stage]), phase, abort_flag, p.err, peer_abort)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t base = tc::smem_u32(sm.tiles[stage]);
#pragma unroll
          for (int k16 = 0; k16 < BK / 16; ++k16) {
            const uint32_t koff = (uint32_t)(k16 * 32);  // 16 fp16 = 32 bytes along the swizzled row
            const uint64_t a_hi = tc::desc_k_sw64(base + koff);
            const uint64_t a_lo = tc::desc_k_sw64(base + A_BYTES + koff);
            const uint64_t b_hi = tc::desc_k_sw64(base + 2 * A_BYTES + koff);
            const uint64_t b_lo = tc::desc_k_sw64(base + 2 * A_BYTES + C::B_BYTES + koff);
            const uint32_t first = (kb | k16) != 0 ? 1u : 0u;
            if (PAIR) {
              tc::mma_f16_ss_pair(d_tmem, a_hi, b_hi, C::IDESC, first);
              tc::mma_f16_ss_pair(d_tmem, a_hi, b_lo, C::IDESC, 1u);
              tc::mma_f16_ss_pair(d_tmem, a_lo, b_hi, C::IDESC, 1u);
            } else {
              tc::mma_f16_ss(d_tmem, a_hi, b_hi, C::IDESC, first);
              tc::mma_f16_ss(d_tmem, a_hi, b_lo, C::IDESC, 1u);
              tc::mma_f16_ss(d_tmem, a_lo, b_hi, C::IDESC, 1u);
            }
          }
          const uint32_t empty = tc::smem_u32(&sm.empty[stage]);
          if (PAIR) {
            tc::mma_commit_pair(empty);
            tc::mma_commit_pair(tc::mapa(empty, 1u));
          } else {
            tc::mma_commit(empty);
          }
          if (++stage == C::STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        const uint32_t accf = tc::smem_u32(&sm.acc_full[acc]);
        if (PAIR) {
          tc::mma_commit_pair(accf);
          tc::mma_commit_pair(tc::mapa(accf, 1u));
        } else {
          tc::mma_commit(accf);
        }
        if (++acc == NUM_ACC) acc = 0, acc_phase ^= 1;
      }
      if (!ok) {
        // Wait for this thread's MMAs in flight before TMEM is released.
        if (PAIR) tc::mma_commit_pair(tc::smem_u32(&sm.drain));
        else tc::mma_commit(tc::smem_u32(&sm.drain));
        const uint64_t start = global_ns();
        while (!tc::mbar_try_wait(tc::smem_u32(&sm.drain), 0) && global_ns() - start < WAIT_LIMIT_NS) {
        }
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int et = threadIdx.x - 64;         // 0..127
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int P = p.patches;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int local = 0;; ++local) {
      const int slot = local % RING;
      const bool got = wait_bounded<PAIR>(tc::smem_u32(&sm.ring_full[slot]), (uint32_t)(local / RING) & 1u,
                                          abort_flag, p.err, peer_abort);
      const long long tile = got ? sm.tile_ring[slot] : -1;
      if (named_sync_epi_any(tile < 0)) break;  // uniform: every epilogue thread read the same slot
      int m_blk, n_blk;
      tile_coords(tile, p.num_m, p.num_n, C::GROUP_M, &m_blk, &n_blk);
      const long long n0 = (long long)n_blk * BN;
      named_sync_epi();  // previous tile's readers are done with col_norm / col_w
      for (int j = et; j < BN; j += EPI_WARPS * 32) {
        const long long col = n0 + j;
        const bool ok = col < p.r_rows;
        sm.col_norm[j] = ok ? __ldg(p.r_norm + col) : 0.f;
        sm.col_w[j] = ok ? 2.f * __ldg(p.r_inv + col) : 0.f;
      }
      wait_bounded<false>(tc::smem_u32(&sm.acc_full[acc]), acc_phase, abort_flag, p.err, peer_abort);
      if (named_sync_epi_any(*abort_flag)) break;  // uniform decision across the epilogue warps
      tc::fence_after_sync();

      const long long cta_row0 = (long long)m_blk * C::TILE_M + (long long)rank * CTA_M;
      const long long warp_row0 = cta_row0 + quarter * 32;
      const long long row = warp_row0 + lane;
      const bool row_ok = row < p.q_rows;
      const float qn = row_ok ? __ldg(p.q_norm + row) : 0.f;
      const float qi = row_ok ? __ldg(p.q_inv + row) : 0.f;
      const int q_img = (int)((p.q_first_row + row) / P);
      // Symmetric mode keeps only columns of a later image than the row's.
      const long long col_from = SYM ? (long long)(q_img + 1) * P : 0;
      long long cta_last_row = cta_row0 + CTA_M - 1;
      if (cta_last_row > p.q_rows - 1) cta_last_row = p.q_rows - 1;
      const bool rows_full = cta_row0 + CTA_M <= p.q_rows;
      const bool clean = !SYM || (rows_full && (cta_last_row / P) < (n0 / P));
      // row images covered by this warp (symmetric column minima)
      const bool warp_any = warp_row0 < p.q_rows;
      long long warp_last = warp_row0 + 31;
      if (warp_last > p.q_rows - 1) warp_last = p.q_rows - 1;
      const int w_img0 = (int)(warp_row0 / P), w_img1 = warp_any ? (int)(warp_last / P) : w_img0 - 1;

      int seg_img = (int)(n0 / P);
      long long seg_end = (long long)(seg_img + 1) * P;
      float m = INF;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        const long long c0 = n0 + chunk * 32;
        if (c0 >= p.r_rows) break;
        uint32_t raw[32];
        tc::tmem_ld_32x32b_x32(tbase + (uint32_t)(chunk * 32), raw);
        tc::tmem_wait_ld();
        float v[32];
        const bool full_chunk = c0 + 32 <= p.r_rows;
        if (clean && full_chunk) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int jj = chunk * 32 + j;
            v[j] = fmaf(-__uint_as_float(raw[j]), qi * sm.col_w[jj], qn + sm.col_norm[jj]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int jj = chunk * 32 + j;
            const long long col = c0 + j;
            const bool ok = row_ok && col < p.r_rows && col >= col_from;
            v[j] = ok ? fmaf(-__uint_as_float(raw[j]), qi * sm.col_w[jj], qn + sm.col_norm[jj]) : INF;
          }
        }
        // Row minima per reference-image segment.
        if (c0 + 32 <= seg_end) {
#pragma unroll
          for (int j = 0; j < 32; ++j) m = fminf(m, v[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j >= seg_end) {
              if (row_ok && seg_img != q_img) flush_min(p, row, seg_img, m);
              ++seg_img;
              seg_end += P;
              m = INF;
            }
            m = fminf(m, v[j]);
          }
        }
        if (SYM) {
          // Column minima over this warp's rows, one per row image.
          const long long col = c0 + lane;
          if (w_img0 == w_img1) {
            const float cm = warp_column_min(v, lane);
            if (col < p.r_rows) flush_min(p, col, w_img0, cm);
          } else {
            for (int ri = w_img0; ri <= w_img1; ++ri) {
              float u[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) u[j] = (q_img == ri) ? v[j] : INF;
              const float cm = warp_column_min(u, lane);
              if (col < p.r_rows) flush_min(p, col, ri, cm);
            }
          }
        }
      }
      if (row_ok && seg_img != q_img) flush_min(p, row, seg_img, m);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        const uint32_t acc_e = tc::smem_u32(&sm.acc_empty[acc]);
        const uint32_t ring_e = tc::smem_u32(&sm.ring_empty[slot]);
        if (leader) {
          tc::mbar_arrive(acc_e);
          tc::mbar_arrive(ring_e);
        } else {
          tc::mbar_arrive_cluster(tc::mapa(acc_e, 0u));
          tc::mbar_arrive_cluster(tc::mapa(ring_e, 0u));
        }
      }
      if (++acc == NUM_ACC) acc = 0, acc_phase ^= 1;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (PAIR) tc::cluster_sync();  // no access to the other CTA's shared memory or TMEM is still pending
  if (warp == 1) {
    tc::fence_after_sync();
    if (PAIR) tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (PAIR) tc::cluster_sync();
}

}  // namespace nearest

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

// 2-D fp16 plane [rows][channels], box = 32 channels x box_rows, 64-byte swizzle.
int make_plane_map(CUtensorMap* map, const void* base, long long rows, int channels, int box_rows) {
  EncodeTiledFn encode;
  MUSC_TRY(get_encode_fn(&encode));
  cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)channels * 2};
  cuuint32_t box[2] = {(cuuint32_t)nearest::BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MUSC_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
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

static int set_smem_attr() {
  static std::mutex m;
  static bool done[64] = {false};
  int dev = 0;
  MUSC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(m);
  if (dev >= 64 || !done[dev]) {
    MUSC_CUDA(cudaFuncSetAttribute(nearest::nearest_kernel<false, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)nearest::smem_bytes<false>()));
    MUSC_CUDA(cudaFuncSetAttribute(nearest::nearest_kernel<true, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)nearest::smem_bytes<false>()));
    MUSC_CUDA(cudaFuncSetAttribute(nearest::nearest_kernel<true, true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)nearest::smem_bytes<true>()));
    if (dev < 64) done[dev] = true;
  }
  return MUSC_B200_OK;
}

// The symmetric pool kernel runs as CTA pairs (cta_group::2) unless
// MUSC_B200_NEAREST_PAIR=0 selects the single-CTA kernel; both compute the
// same table bit for bit.
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
  const BankLayout ql = bank_layout(query_rows, channels);
  const BankLayout rl = bank_layout(ref_rows, channels);
  const uint8_t* qb = static_cast<const uint8_t*>(query_bank);
  const uint8_t* rb = static_cast<const uint8_t*>(ref_bank);
  CUtensorMap mqh, mql, mrh, mrl;
  MUSC_TRY(make_plane_map(&mqh, qb + ql.hi, query_rows, channels, nearest::CTA_M));
  MUSC_TRY(make_plane_map(&mql, qb + ql.lo, query_rows, channels, nearest::CTA_M));
  MUSC_TRY(make_plane_map(&mrh, rb + rl.hi, ref_rows, channels, nearest::BN));
  MUSC_TRY(make_plane_map(&mrl, rb + rl.lo, ref_rows, channels, nearest::BN));
  const int n_images = (int)(ref_rows / patches);
  MUSC_TRY(fill_table(nearest_sq, (long long)n_images * query_rows, s));
  nearest::Params p;
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
  p.num_kb = (channels + nearest::BK - 1) / nearest::BK;
  p.num_m = (int)((query_rows + nearest::CTA_M - 1) / nearest::CTA_M);
  p.num_n = (int)((ref_rows + nearest::BN - 1) / nearest::BN);
  p.tile_begin = 0;
  p.tile_end = (long long)p.num_m * p.num_n;
  p.sched = nullptr;  // static schedule
  MUSC_TRY(set_smem_attr());
  const int grid = (int)std::min<long long>(p.tile_end, sm_count());
  nearest::nearest_kernel<false, false><<<grid, nearest::THREADS, nearest::smem_bytes<false>(), s>>>(
      mqh, mql, mrh, mrl, p);
  return check_launch("nearest_kernel<directed>");
}

int nearest_pool_launch(const void* bank, long long bank_rows, long long rows, int channels, int patches,
                        int part, int parts, long long rows_per_block, int max_ctas, float* nearest_sq,
                        cudaStream_t s) {
  const BankLayout l = bank_layout(bank_rows, channels);
  const uint8_t* b = static_cast<const uint8_t*>(bank);
  const bool pair = use_cta_pairs();
  const int b_box = pair ? nearest::Cfg<true>::CTA_N : nearest::Cfg<false>::CTA_N;
  CUtensorMap mah, mal, mbh, mbl;
  MUSC_TRY(make_plane_map(&mah, b + l.hi, rows, channels, nearest::CTA_M));
  MUSC_TRY(make_plane_map(&mal, b + l.lo, rows, channels, nearest::CTA_M));
  MUSC_TRY(make_plane_map(&mbh, b + l.hi, rows, channels, b_box));
  MUSC_TRY(make_plane_map(&mbl, b + l.lo, rows, channels, b_box));
  const int n_images = (int)(rows / patches);
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  const long long table = blocks * n_images * rows_per_block;
  MUSC_TRY(fill_table(nearest_sq, table, s));
  // The scheduler counter lives in the 256 bytes after the table (musc_b200_nearest_pool_bytes).
  unsigned long long* sched = reinterpret_cast<unsigned long long*>(
      reinterpret_cast<uint8_t*>(nearest_sq) + ((size_t)table * sizeof(float) + 255) / 256 * 256);
  MUSC_CUDA(cudaMemsetAsync(sched, 0, sizeof(unsigned long long), s));
  nearest::Params p;
  p.q_norm = p.r_norm = reinterpret_cast<const float*>(b + l.norm);
  p.q_inv = p.r_inv = reinterpret_cast<const float*>(b + l.inv);
  p.nearest = reinterpret_cast<unsigned int*>(nearest_sq);
  p.sched = sched;
  p.err = device_error_ptr();
  if (!p.err) return fail(MUSC_B200_ERR_CUDA, "nearest_pool: device error word unavailable");
  p.q_rows = p.r_rows = rows;
  p.q_first_row = 0;
  p.rows_per_block = rows_per_block;
  p.blocked = blocks > 1 ? 1 : 0;
  p.patches = patches;
  p.n_images = n_images;
  p.num_kb = (channels + nearest::BK - 1) / nearest::BK;
  const int tile_m = pair ? nearest::Cfg<true>::TILE_M : nearest::Cfg<false>::TILE_M;
  const int group_m = pair ? nearest::Cfg<true>::GROUP_M : nearest::Cfg<false>::GROUP_M;
  p.num_m = (int)((rows + tile_m - 1) / tile_m);
  p.num_n = (int)((rows + nearest::BN - 1) / nearest::BN);
  sym_part_range(rows, patches, n_images, p.num_m, p.num_n, tile_m, group_m, part, parts, &p.tile_begin,
                 &p.tile_end);
  if (p.tile_end <= p.tile_begin) return MUSC_B200_OK;  // nothing to do for this part
  MUSC_TRY(set_smem_attr());
  const int sms = sm_count();
  const int ctas = max_ctas > 0 && max_ctas < sms ? max_ctas : sms;
  if (!pair) {
    nearest::nearest_kernel<true, false><<<ctas, nearest::THREADS, nearest::smem_bytes<false>(), s>>>(
        mah, mal, mbh, mbl, p);
    return check_launch("nearest_kernel<symmetric>");
  }
  // One cluster of two CTAs per SM pair, as many as can be resident at once.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(nearest::THREADS);
  cfg.dynamicSmemBytes = nearest::smem_bytes<true>();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  MUSC_CUDA(cudaOccupancyMaxActiveClusters(&clusters, nearest::nearest_kernel<true, true>, &cfg));
  if (clusters <= 0) return fail(MUSC_B200_ERR_CUDA, "nearest_pool: no CTA pair fits on this device");
  clusters = std::min(clusters, std::max(1, ctas / 2));
  cfg.gridDim = dim3(2 * clusters);
  MUSC_CUDA(cudaLaunchKernelEx(&cfg, nearest::nearest_kernel<true, true>, mah, mal, mbh, mbl, p));
  return check_launch("nearest_kernel<symmetric, pair>");
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

extern "C" int musc_b200_prep_bank(const float* z, long long rows, int channels, void* bank,
                                   size_t bank_bytes, musc_b200_stream stream) {
  MUSC_TRY(check_bank_args(rows, channels));
  if (!z || !bank) return fail(MUSC_B200_ERR_INVALID, "prep_bank: null pointer");
  if (reinterpret_cast<uintptr_t>(z) % 16 != 0 || reinterpret_cast<uintptr_t>(bank) % 1024 != 0)
    return fail(MUSC_B200_ERR_INVALID, "prep_bank: z must be 16-byte and bank 1024-byte aligned");
  const BankLayout l = bank_layout(rows, channels);
  if (bank_bytes < l.total) return fail(MUSC_B200_ERR_WORKSPACE, "prep_bank: bank smaller than musc_b200_bank_bytes");
  MUSC_TRY(require_sm100());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* b = static_cast<uint8_t*>(bank);
  const long long blocks = (rows + kPrepWarps - 1) / kPrepWarps;
  prep_bank_kernel<<<(unsigned)blocks, kPrepWarps * 32, 0, s>>>(
      z, rows, channels, reinterpret_cast<__half*>(b + l.hi), reinterpret_cast<__half*>(b + l.lo),
      reinterpret_cast<float*>(b + l.norm), reinterpret_cast<float*>(b + l.inv));
  return check_launch("prep_bank_kernel");
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

extern "C" size_t musc_b200_msm_workspace_bytes(int n, int p, int c) {
  if (n <= 0 || p <= 0 || c <= 0) return 0;
  const long long rows = (long long)n * p;
  return bank_layout(rows, c).total + align_up(musc_b200_nearest_pool_bytes(rows, p, rows), 1024);
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
  float* table = reinterpret_cast<float*>(ws + bank_size);
  MUSC_TRY(musc_b200_prep_bank(z, rows, c, ws, bank_size, stream));
  MUSC_TRY(musc_b200_nearest_pool(ws, rows, rows, c, p, 0, 1, rows, 0, table, stream));
  return musc_b200_trimmed_mean(table, rows, n, rank_lo, rank_hi, scores, stream);
}
