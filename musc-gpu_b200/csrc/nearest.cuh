// The persistent tcgen05 distance GEMM with fused per-image minima (MSM's
// dense contraction, models/modules/_MSM.py:16-17), in four modes:
//
//   DIRECTED  query bank x reference bank, split-fp16 3-pass (hi*hi + hi*lo +
//             lo*hi), exact fp32-class minima per (query row, reference image)
//             into a float table (musc_b200_nearest).
//   SYM       the pool against itself over the symmetric tile list (each
//             unordered pair of patches from different images once): row minima
//             give one direction, a transposing warp butterfly the other; 3-pass,
//             exact (musc_b200_nearest_pool, the exact pool path).
//   SCREEN    SYM with the hi*hi pass only: a third of the tensor-core work.  Per
//             (row, image) it keeps the smallest screened distance with the patch
//             that attains it (a 64-bit key: value bits << 32 | patch) and the
//             second-smallest screened distance over the image's other patches.
//             Both are combined across tiles with atomic minima; the second
//             minimum uses the value each key-minimum displaces, so the result is
//             the true second smallest whatever the order of the updates.  The
//             refinement kernel (refine.cu) turns these into exact minima.
//   GATHER    exact 3-pass rows of a staged query bank, each 128-row tile against
//             one reference image only (the pairs the refinement could not
//             certify).
//
// Warp roles: warp 0 lane 0 loads (TMA), warp 1 lane 0 issues the MMAs (the even
// CTA of a pair), the remaining warps are the epilogue.  In a CTA pair (cta_group::2,
// 256 x 256 tiles over two SMs) the even CTA owns the schedule: its producer claims
// each tile, writes the index into both CTAs' rings, and both CTAs' loads complete on
// its `full` barriers; its MMA thread signals both CTAs' `empty` and `acc_full`
// barriers; both epilogues release the accumulator and the ring slot on its barriers.
// Every wait is bounded (4 s): on expiry the kernel raises the device error word,
// drains its copies and MMAs, frees TMEM and returns.
#pragma once

#include "common.cuh"
#include "tc.cuh"

#include <cfloat>

namespace musc {
namespace nearest {

enum Mode { DIRECTED = 0, SYM = 1, SCREEN = 2, GATHER = 3 };

constexpr int CTA_M = 128;        // query rows per CTA (TMEM lanes)
constexpr int BN = 256;           // reference rows per tile (TMEM columns per accumulator)
constexpr int BK = 32;            // fp16 elements per K slice of the 3-pass modes (64-byte swizzle rows)
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;  // 4 s per wait
constexpr float INF = FLT_MAX;
constexpr uint32_t UMAX = 0xFFFFFFFFu;
constexpr int RING = 8;      // tile indices handed from the producer to the MMA and epilogue warps
constexpr int CHUNK = 8;     // tiles claimed per atomic by the dynamic scheduler

// Tile shapes.  Single CTA: 128 x 256 tiles, the CTA holds all 256 B rows of a K slice.
// CTA pair (cta_group::2): 256 x 256 tiles over two SMs; each CTA loads 128 A rows and
// 128 B rows, so per MMA an SM reads 8 KB of operands from shared memory instead of
// 12 KB and fetches a third fewer bytes from L2.  SCREEN loads only the hi planes, so
// its stages are half as large and twice as many; it runs eight epilogue warps (two
// per TMEM lane quarter, one per 128-column half) because a tile's MMA work is a third
// of the other modes'.
template <int MODE, bool PAIR>
struct Cfg {
  static constexpr bool SYMM = MODE == SYM || MODE == SCREEN;
  static constexpr int PASSES = MODE == SCREEN ? 1 : 3;
  static constexpr int PLANES = MODE == SCREEN ? 1 : 2;
  // K slice: 32 fp16 (64-byte rows, 64-byte swizzle) for the 3-pass modes, whose stages
  // carry four planes; 64 fp16 (128-byte rows, 128-byte swizzle) for the screen, whose
  // one-pass MMAs consume operands three times faster -- whole 128-byte lines halve the
  // copy engine's row requests per byte.
  static constexpr int KB = MODE == SCREEN ? 64 : BK;
  static constexpr int TILE_M = PAIR ? 256 : 128;
  static constexpr int CTA_N = PAIR ? 128 : 256;
  static constexpr int A_PLANE = CTA_M * KB * 2;
  static constexpr int B_PLANE = CTA_N * KB * 2;
  static constexpr int STAGE_BYTES = PLANES * (A_PLANE + B_PLANE);  // 48/32 KB, screen 48/32 KB
  static constexpr int STAGES = MODE == SCREEN ? (PAIR ? 5 : 3) : (PAIR ? 6 : 4);
  static constexpr int GROUP_M = PAIR ? 32 : 64;  // m-tiles swept together (8192 query rows)
  static constexpr uint32_t IDESC = tc::idesc_f16(TILE_M, BN, /*fp16*/ 0);
  static constexpr int EPI_WARPS = MODE == SCREEN ? 8 : 4;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int EPI_ARRIVALS = (PAIR ? 2 : 1) * EPI_WARPS;  // epilogue warps releasing a tile
  // SCREEN: per epilogue warp a 32 x 33-word transpose buffer (conflict-free both ways)
  static constexpr int XPOSE_WORDS = MODE == SCREEN ? EPI_WARPS * 32 * 33 : 1;
  // SCREEN: per-tile merge buffers -- column partials [4 row quarters][256 columns] x (min,
  // second) and row partials [2 column halves][128 rows] x (min, second, image).
  static constexpr int MERGE_WORDS = MODE == SCREEN ? 4 * 256 * 2 + 2 * 128 * 3 + 4 : 1;
};

template <int STAGES, int STAGE_BYTES, int XPOSE_WORDS, int MERGE_WORDS>
struct Smem {
  uint8_t tiles[STAGES][STAGE_BYTES];  // 1024-aligned base
  uint32_t xpose[XPOSE_WORDS];
  uint32_t merge[MERGE_WORDS];
  float col_norm[BN];
  float col_w[BN];
  float2 col_stat[2][BN];  // SCREEN: (|r|^2, 2 * 2^-k_r) per column, double-buffered by tile
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
template <int MODE, bool PAIR>
using SmemT = Smem<Cfg<MODE, PAIR>::STAGES, Cfg<MODE, PAIR>::STAGE_BYTES, Cfg<MODE, PAIR>::XPOSE_WORDS,
                   Cfg<MODE, PAIR>::MERGE_WORDS>;
template <int MODE, bool PAIR>
constexpr size_t smem_bytes() {
  return sizeof(SmemT<MODE, PAIR>) + 1024;
}

struct Params {
  const float* q_norm;
  const float* q_inv;
  const float* r_norm;
  const float* r_inv;
  unsigned int* nearest;        // float bits, layout [row / rpb][image][row % rpb] (DIRECTED/SYM/GATHER)
  unsigned long long* k1;       // SCREEN: min key (value bits << 32 | patch), same layout
  unsigned int* m2;             // SCREEN: second-smallest value bits, same layout
  unsigned long long* sched;    // dynamic-scheduler counter (zeroed before the launch), or nullptr
  const int* tile_img;          // GATHER: reference image of each staged 128-row m-tile
  const int* row_map;           // GATHER: table row of each staged row (-1 = padding)
  const long long* tile_total;  // GATHER: number of tiles (written by the planning kernel)
  int* err;
  long long q_rows, r_rows, q_first_row;
  long long tile_begin, tile_end;  // linear tile range processed by this launch
  long long rows_per_block;        // rpb of the table layout
  int blocked;                     // 0: rows_per_block covers every row addressed
  int patches;                     // P
  int n_images;
  int num_kb;
  int num_m, num_n;
  int nsub;                        // GATHER: n-tiles per reference image
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

// Symmetric modes: tile (m, n) holds an element (r, c) with img(r) < img(c).
__host__ __device__ inline bool sym_needed(int m, int n, long long rows, int patches, int n_images, int tile_m) {
  const long long r0 = (long long)m * tile_m;
  const long long img_r = r0 / patches;
  if (img_r >= n_images - 1) return false;
  long long c_last = (long long)n * BN + BN - 1;
  if (c_last > rows - 1) c_last = rows - 1;
  return c_last / patches > img_r;
}

// Bounded wait: true when the phase completed; false after the time limit (which
// raises this CTA's abort flag, the peer CTA's when `peer_abort` is a cluster address,
// and the device error word) or when an abort was already raised.  CLUSTER selects
// acquire at cluster scope, for phases completed by the other CTA of a pair.
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

template <int EPI_WARPS>
__device__ __forceinline__ void named_sync_epi() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}

// Barrier over the epilogue warps that also ORs `flag` across them, so every epilogue
// thread takes the same branch afterwards.
template <int EPI_WARPS>
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

// After the call lane l holds min over the warp's 32 lanes of v[l] (a transposing
// butterfly: 31 shuffles for 32 columns).
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

// Same butterfly over (smallest key, second-smallest key) pairs: after the call lane l
// holds the smallest and second-smallest of column l's 32 keys.
__device__ __forceinline__ void warp_column_min2(uint32_t (&k)[32], uint32_t (&m)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const uint32_t send_k = upper ? k[i] : k[i + s];
      const uint32_t send_m = upper ? m[i] : m[i + s];
      const uint32_t keep_k = upper ? k[i + s] : k[i];
      const uint32_t keep_m = upper ? m[i + s] : m[i];
      const uint32_t rk = __shfl_xor_sync(0xffffffffu, send_k, s);
      const uint32_t rm = __shfl_xor_sync(0xffffffffu, send_m, s);
      k[i] = min(keep_k, rk);
      m[i] = min(max(keep_k, rk), min(keep_m, rm));
    }
  }
}

// Screened distance -> sortable key: non-negative float bits with the low `bits`
// bits replaced by a local index (the value keeps 15+ significant bits).
__device__ __forceinline__ uint32_t pack_key(float v, uint32_t low_mask, uint32_t idx) {
  return (__float_as_uint(v) & ~low_mask) | idx;
}

// Smallest and second-smallest of 32 keys by a pairwise tree (depth 5 instead of a
// 32-long dependency chain); `v` is clobbered.
__device__ __forceinline__ void min2_tree(uint32_t (&v)[32], uint32_t& m1, uint32_t& m2) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    w[i] = max(v[2 * i], v[2 * i + 1]);
    v[i] = min(v[2 * i], v[2 * i + 1]);
  }
#pragma unroll
  for (int n = 8; n >= 1; n >>= 1) {
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const uint32_t a1 = v[2 * i], b1 = v[2 * i + 1];
      w[i] = min(max(a1, b1), min(w[2 * i], w[2 * i + 1]));
      v[i] = min(a1, b1);
    }
  }
  m1 = v[0];
  m2 = w[0];
}

// One screened partial result awaiting its second-minimum update.  push() issues the
// key minimum (returning the old key) and completes the previous partial: its
// second-minimum candidate is the larger of its key and the key it met, so the table's
// second minimum ends as the second smallest value over all partials, in any order.
struct ScreenFlush {
  long long idx = -1;
  unsigned long long key = 0, old = 0;
  uint32_t m = UMAX;

  __device__ __forceinline__ void finish(const Params& p) {
    if (idx < 0) return;
    const unsigned long long larger = old > key ? old : key;
    const uint32_t shadow = (uint32_t)(larger >> 32) & ~0xFFu;
    const uint32_t v = min(m & ~0xFFu, shadow);
    if (v != (UMAX & ~0xFFu)) atomicMin(p.m2 + idx, v);
    idx = -1;
  }
  __device__ __forceinline__ void push(const Params& p, long long table_idx, uint32_t value_bits, uint32_t patch,
                                       uint32_t second) {
    const unsigned long long k = ((unsigned long long)(value_bits & ~0xFFu) << 32) | patch;
    const unsigned long long o = atomicMin(p.k1 + table_idx, k);
    finish(p);
    idx = table_idx;
    key = k;
    old = o;
    m = second;
  }
};

template <int MODE, bool PAIR>
__global__ void __launch_bounds__(Cfg<MODE, PAIR>::THREADS, 1)
nearest_kernel(const __grid_constant__ CUtensorMap map_q_hi, const __grid_constant__ CUtensorMap map_q_lo,
               const __grid_constant__ CUtensorMap map_r_hi, const __grid_constant__ CUtensorMap map_r_lo,
               const Params p) {
  using C = Cfg<MODE, PAIR>;
  constexpr int EPI = C::EPI_WARPS;
  extern __shared__ uint8_t smem_raw[];
  SmemT<MODE, PAIR>& sm =
      *reinterpret_cast<SmemT<MODE, PAIR>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;
  const uint32_t rank = PAIR ? tc::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const uint32_t peer_abort = PAIR ? tc::mapa(tc::smem_u32(&sm.abort_flag), rank ^ 1u) : 0u;
  // A fallback round that planned nothing: leave before any setup (every thread reads
  // the same word, so the whole grid returns).
  if (MODE == GATHER && *reinterpret_cast<const volatile long long*>(p.tile_total) == 0) return;

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
    tc::prefetch_tensormap(&map_r_hi);
    if (C::PLANES > 1) {
      tc::prefetch_tensormap(&map_q_lo);
      tc::prefetch_tensormap(&map_r_lo);
    }
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
      long long tile_end = p.tile_end;
      if (MODE == GATHER) {
        const long long t = *reinterpret_cast<const volatile long long*>(p.tile_total);
        tile_end = t < tile_end ? t : tile_end;
      }
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
              chunk_end = chunk_cur + CHUNK < tile_end ? chunk_cur + CHUNK : tile_end;
              if (chunk_cur >= tile_end) return -1;
            }
            t = chunk_cur++;
          } else {
            t = next_static;
            if (t >= tile_end) return -1;
            next_static += n_groups;
          }
          if (!C::SYMM) return t;
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
        int a_row, b_row;
        if (MODE == GATHER) {
          const int mt = (int)(tile / p.nsub), ns = (int)(tile - (long long)mt * p.nsub);
          a_row = mt * CTA_M;
          b_row = p.tile_img[mt] * p.patches + ns * BN;
        } else {
          int m_blk, n_blk;
          tile_coords(tile, p.num_m, p.num_n, C::GROUP_M, &m_blk, &n_blk);
          a_row = m_blk * C::TILE_M + (int)rank * CTA_M;
          b_row = n_blk * BN + (int)rank * C::CTA_N;
        }
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!wait_bounded<false>(tc::smem_u32(&sm.empty[stage]), phase ^ 1, abort_flag, p.err, peer_abort)) {
            ok = false;
            break;
          }
          const uint32_t full_local = tc::smem_u32(&sm.full[stage]);
          // The leader's barrier counts both CTAs' bytes of this stage.
          if (leader) tc::mbar_arrive_expect_tx(full_local, (PAIR ? 2 : 1) * C::STAGE_BYTES);
          const uint32_t base = tc::smem_u32(sm.tiles[stage]);
          const uint32_t b_base = base + C::PLANES * C::A_PLANE;
          const int kc = kb * C::KB;
          if (PAIR) {
            const uint32_t full = tc::mapa(full_local, 0u);
            tc::tma_load_2d_pair(base, &map_q_hi, kc, a_row, full);
            tc::tma_load_2d_pair(b_base, &map_r_hi, kc, b_row, full);
            if (C::PLANES > 1) {
              tc::tma_load_2d_pair(base + C::A_PLANE, &map_q_lo, kc, a_row, full);
              tc::tma_load_2d_pair(b_base + C::B_PLANE, &map_r_lo, kc, b_row, full);
            }
          } else {
            tc::tma_load_2d(base, &map_q_hi, kc, a_row, full_local);
            tc::tma_load_2d(b_base, &map_r_hi, kc, b_row, full_local);
            if (C::PLANES > 1) {
              tc::tma_load_2d(base + C::A_PLANE, &map_q_lo, kc, a_row, full_local);
              tc::tma_load_2d(b_base + C::B_PLANE, &map_r_lo, kc, b_row, full_local);
            }
          }
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == C::STAGES) stage = 0, phase ^= 1;
        }
      }
      if (!ok) {
        // Let the copies already in flight land before the CTA exits.  The leader
        // watches its `full` barriers (one deadline for all stages); the peer's copies
        // complete on the leader's barriers, so it gives them a fixed 2 ms, far above
        // the latency of one copy.
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
          const uint32_t b_base = base + C::PLANES * C::A_PLANE;
          auto desc = [](uint32_t a) { return C::KB == 64 ? tc::desc_k_sw128(a) : tc::desc_k_sw64(a); };
#pragma unroll
          for (int k16 = 0; k16 < C::KB / 16; ++k16) {
            const uint32_t koff = (uint32_t)(k16 * 32);  // 16 fp16 = 32 bytes along the swizzled row
            const uint64_t a_hi = desc(base + koff);
            const uint64_t b_hi = desc(b_base + koff);
            const uint32_t first = (kb | k16) != 0 ? 1u : 0u;
            if (PAIR) tc::mma_f16_ss_pair(d_tmem, a_hi, b_hi, C::IDESC, first);
            else tc::mma_f16_ss(d_tmem, a_hi, b_hi, C::IDESC, first);
            if (C::PASSES > 1) {
              const uint64_t a_lo = desc(base + C::A_PLANE + koff);
              const uint64_t b_lo = desc(b_base + C::B_PLANE + koff);
              if (PAIR) {
                tc::mma_f16_ss_pair(d_tmem, a_hi, b_lo, C::IDESC, 1u);
                tc::mma_f16_ss_pair(d_tmem, a_lo, b_hi, C::IDESC, 1u);
              } else {
                tc::mma_f16_ss(d_tmem, a_hi, b_lo, C::IDESC, 1u);
                tc::mma_f16_ss(d_tmem, a_lo, b_hi, C::IDESC, 1u);
              }
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
  } else if constexpr (MODE == SCREEN) {
    // ---------------------------------------------------------- screen epilogue
    // Eight warps: warp w reads TMEM lane quarter w % 4 and one 128-column half of the
    // tile.  One named barrier per tile: the column statistics are double-buffered (a warp
    // that writes tile t's buffer has passed tile t-1's barrier, so every warp is done
    // with tile t-2's), and the same barrier makes the end / abort decision uniform.
    const int et = threadIdx.x - 64;
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int c_begin = half * (BN / 2);
    const int P = p.patches;
    int acc = 0;
    uint32_t acc_phase = 0;
    // Pending second-minimum updates: `pend` for partials pushed from the chunk loop,
    // `pend_col` / `pend_row` for the one column and one row partial each thread pushes
    // per tile after the merge -- each is completed a whole tile later, when its key
    // atomic has long returned.
    ScreenFlush pend, pend_col, pend_row;
    for (int local = 0;; ++local) {
      const int slot = local % RING;
      const int buf = local & 1;
      const bool got = wait_bounded<PAIR>(tc::smem_u32(&sm.ring_full[slot]), (uint32_t)(local / RING) & 1u,
                                          abort_flag, p.err, peer_abort);
      const long long tile = got ? sm.tile_ring[slot] : -1;
      long long n0 = 0, cta_row0 = 0;
      if (tile >= 0) {
        int m_blk, n_blk;
        tile_coords(tile, p.num_m, p.num_n, C::GROUP_M, &m_blk, &n_blk);
        n0 = (long long)n_blk * BN;
        cta_row0 = (long long)m_blk * C::TILE_M + (long long)rank * CTA_M;
        for (int j = et; j < BN; j += EPI * 32) {
          const long long col = n0 + j;
          const bool ok = col < p.r_rows;
          sm.col_stat[buf][j] = make_float2(ok ? __ldg(p.r_norm + col) : 0.f, ok ? 2.f * __ldg(p.r_inv + col) : 0.f);
        }
        wait_bounded<false>(tc::smem_u32(&sm.acc_full[acc]), acc_phase, abort_flag, p.err, peer_abort);
      }
      if (named_sync_epi_any<EPI>(tile < 0 || *abort_flag)) break;
      tc::fence_after_sync();

      const long long warp_row0 = cta_row0 + quarter * 32;
      const long long row = warp_row0 + lane;
      const bool row_ok = row < p.q_rows;
      const float qn = row_ok ? __ldg(p.q_norm + row) : 0.f;
      const float qi = row_ok ? __ldg(p.q_inv + row) : 0.f;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      const int q_img = (int)((p.q_first_row + row) / P);
      const long long col_from = (long long)(q_img + 1) * P;  // columns of a later image than the row's
      // Clean tile: all 128 rows valid and of images before the first column's image, and
      // every column inside the pool -- no per-element masks (the common case).
      long long cta_last = cta_row0 + CTA_M - 1;
      const bool clean = cta_last < p.q_rows && cta_last / P < n0 / P && n0 + BN <= p.r_rows;
      if (cta_last > p.q_rows - 1) cta_last = p.q_rows - 1;
      const bool warp_any = warp_row0 < p.q_rows;
      long long warp_last = warp_row0 + 31;
      if (warp_last > p.q_rows - 1) warp_last = p.q_rows - 1;
      const int w_img0 = (int)(warp_row0 / P), w_img1 = warp_any ? (int)(warp_last / P) : w_img0 - 1;
      int seg_img = (int)((n0 + c_begin) / P);
      long long seg_end = (long long)(seg_img + 1) * P;
      uint32_t k1 = UMAX, m2 = UMAX;  // row direction: packed keys (value | column in the tile)
      // Merge buffers: column partials per row quarter, row partials per column half.
      uint32_t* colbuf = sm.merge;                  // [4][256][2]
      uint32_t* rowbuf = sm.merge + 4 * 256 * 2;    // [2][128][3]
      int* qimg = reinterpret_cast<int*>(sm.merge + 4 * 256 * 2 + 2 * 128 * 3);  // [4] image of each quarter
      const int rin = quarter * 32 + lane;          // this thread's row within the CTA's 128
      // The segment touching the middle of the tile (half 0's last, half 1's first) goes to
      // the row merge buffer (merged with the other half's there); others are pushed.  A
      // segment with no valid column keeps a key of all ones above the low byte.
      bool to_buffer = half == 1;
      auto row_flush = [&]() {
        const bool valid = row_ok && (k1 | 0xFFu) != UMAX && seg_img != q_img;
        if (to_buffer) {
          uint32_t* e = rowbuf + (half * 128 + rin) * 3;
          e[0] = valid ? k1 : UMAX;
          e[1] = m2;
          e[2] = (uint32_t)seg_img;
          to_buffer = false;
        } else if (valid) {
          const uint32_t patch = (uint32_t)(n0 + (k1 & 0xFFu) - (long long)seg_img * P);
          pend.push(p, table_index(p, seg_img, row), k1, patch, m2);
        }
      };
      const float2* cs = sm.col_stat[buf];
      // Column direction through this warp's transpose buffer: lane r writes row r's 32
      // keys (packed with r) at word r*33 + j, lane c reads column c's 32 keys at
      // r*33 + c; both conflict-free.  Where the warp's rows span several row images,
      // each image's rows give their own result.
      uint32_t* xp = sm.xpose + (warp - 2) * (32 * 33);
      int nchunks = 0;
      while (nchunks < BN / 64 && n0 + c_begin + nchunks * 32 < p.r_rows) ++nchunks;
      uint32_t raw[32];
      if (nchunks > 0) tc::tmem_ld_32x32b_x32(tbase + (uint32_t)c_begin, raw);
#pragma unroll 1
      for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int cl = c_begin + chunk * 32;
        const long long c0 = n0 + cl;
        tc::tmem_wait_ld();
        uint32_t kk[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) kk[j] = raw[j];
        if (chunk + 1 < nchunks) tc::tmem_ld_32x32b_x32(tbase + (uint32_t)(cl + 32), raw);  // next chunk in flight
        if (clean) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float2 st = cs[cl + j];
            const float v = fmaxf(fmaf(-__uint_as_float(kk[j]), qi * st.y, qn + st.x), 0.f);
            kk[j] = __float_as_uint(v);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float2 st = cs[cl + j];
            const long long col = c0 + j;
            const bool ok = row_ok && col < p.r_rows && col >= col_from;
            const float v = fmaxf(fmaf(-__uint_as_float(kk[j]), qi * st.y, qn + st.x), 0.f);
            kk[j] = ok ? __float_as_uint(v) : UMAX;
          }
        }
        // Row direction: smallest and second-smallest per reference-image segment (keys
        // carry the column in the tile; an invalid element stays all ones above the low byte).
        if (c0 + 32 <= seg_end) {
          uint32_t t[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = (kk[j] & ~0xFFu) | (uint32_t)(cl + j);
          uint32_t t1, t2;
          min2_tree(t, t1, t2);
          m2 = min(max(k1, t1), min(m2, t2));
          k1 = min(k1, t1);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j >= seg_end) {
              row_flush();
              ++seg_img;
              seg_end += P;
              k1 = m2 = UMAX;
            }
            const uint32_t key = (kk[j] & ~0xFFu) | (uint32_t)(cl + j);
            m2 = min(m2, max(k1, key));
            k1 = min(k1, key);
          }
        }
        // Column direction.
#pragma unroll
        for (int j = 0; j < 32; ++j) xp[lane * 33 + j] = (kk[j] & ~0x1Fu) | (uint32_t)lane;
        __syncwarp();
        const long long col = c0 + lane;
        uint32_t c1 = UMAX, c2 = UMAX;
        if (w_img0 == w_img1) {
          uint32_t t[32];
#pragma unroll
          for (int r = 0; r < 32; ++r) t[r] = xp[r * 33 + lane];
          min2_tree(t, c1, c2);
          // to the merge buffer, the winning row re-packed as its index in the CTA's 128 rows
          uint32_t* e = colbuf + (quarter * 256 + cl + lane) * 2;
          e[0] = (col < p.r_rows && (c1 | 0x1Fu) != UMAX) ? ((c1 & ~0x7Fu) | (uint32_t)(quarter * 32) | (c1 & 0x1Fu))
                                                          : UMAX;
          e[1] = c2;
        } else {
          // the warp's rows span several row images: one result per image
          int ri = w_img0;
          long long next = (long long)(ri + 1) * P - warp_row0;  // first row of the next image
          for (int r = 0; r < 32; ++r) {
            if (r == next) {
              if (col < p.r_rows && (c1 | 0x1Fu) != UMAX)
                pend.push(p, table_index(p, ri, col), c1 & ~0x1Fu,
                          (uint32_t)(warp_row0 + (c1 & 0x1Fu) - (long long)ri * P), c2);
              c1 = c2 = UMAX;
              ++ri;
              next += P;
            }
            const uint32_t x = xp[r * 33 + lane];
            c2 = min(c2, max(c1, x));
            c1 = min(c1, x);
          }
          if (col < p.r_rows && (c1 | 0x1Fu) != UMAX && ri <= w_img1)
            pend.push(p, table_index(p, ri, col), c1 & ~0x1Fu,
                      (uint32_t)(warp_row0 + (c1 & 0x1Fu) - (long long)ri * P), c2);
          uint32_t* e = colbuf + (quarter * 256 + cl + lane) * 2;  // nothing left to merge
          e[0] = UMAX;
          e[1] = UMAX;
        }
        __syncwarp();  // every lane has read the buffer before the next chunk overwrites it
      }
      if (half == 0) to_buffer = true;  // half 0's last segment touches the middle
      row_flush();
      if (nchunks < BN / 64) {           // chunks of this half past the pool's last column
        for (int c = nchunks; c < BN / 64; ++c) {
          uint32_t* e = colbuf + (quarter * 256 + c_begin + c * 32 + lane) * 2;
          e[0] = UMAX;
          e[1] = UMAX;
        }
      }
      if (lane == 0 && half == 0) qimg[quarter] = (w_img0 == w_img1) ? w_img0 : -1;
      // TMEM is read: release the accumulator before merging.
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        const uint32_t acc_e = tc::smem_u32(&sm.acc_empty[acc]);
        if (leader) tc::mbar_arrive(acc_e);
        else tc::mbar_arrive_cluster(tc::mapa(acc_e, 0u));
      }
      named_sync_epi<EPI>();
      // Column merge: thread t owns column t of the tile; quarters holding the same row
      // image (consecutive) combine into one partial.
      {
        const int t = et;
        const long long col = n0 + t;
        uint32_t a1 = UMAX, a2 = UMAX;
        int cur = -1;
        for (int q = 0; q < 4; ++q) {
          const int im = qimg[q];
          const uint32_t b1 = colbuf[(q * 256 + t) * 2], b2 = colbuf[(q * 256 + t) * 2 + 1];
          if (im < 0 || b1 == UMAX) continue;
          if (im != cur) {
            if (cur >= 0 && a1 != UMAX)
              pend.push(p, table_index(p, cur, col), a1 & ~0x7Fu,
                        (uint32_t)(cta_row0 + (a1 & 0x7Fu) - (long long)cur * P), a2);
            cur = im;
            a1 = b1;
            a2 = b2;
          } else {
            a2 = min(max(a1, b1), min(a2, b2));
            a1 = min(a1, b1);
          }
        }
        if (cur >= 0 && a1 != UMAX)
          pend_col.push(p, table_index(p, cur, col), a1 & ~0x7Fu,
                        (uint32_t)(cta_row0 + (a1 & 0x7Fu) - (long long)cur * P), a2);
      }
      // Row merge: thread t < 128 owns row t of the CTA; the two halves' middle segments
      // combine when they are the same reference image.
      if (et < 128) {
        const uint32_t* e0 = rowbuf + et * 3;
        const uint32_t* e1 = rowbuf + (128 + et) * 3;
        const long long grow = cta_row0 + et;
        uint32_t a1 = e0[0], a2 = e0[1], b1 = e1[0], b2 = e1[1];
        const int ia = (int)e0[2], ib = (int)e1[2];
        if (a1 != UMAX && b1 != UMAX && ia == ib) {
          a2 = min(max(a1, b1), min(a2, b2));
          a1 = min(a1, b1);
          b1 = UMAX;
        }
        if (a1 != UMAX)
          pend_row.push(p, table_index(p, ia, grow), a1, (uint32_t)(n0 + (a1 & 0xFFu) - (long long)ia * P), a2);
        if (b1 != UMAX)
          pend.push(p, table_index(p, ib, grow), b1, (uint32_t)(n0 + (b1 & 0xFFu) - (long long)ib * P), b2);
      }
      __syncwarp();
      if (lane == 0) {
        const uint32_t ring_e = tc::smem_u32(&sm.ring_empty[slot]);
        if (leader) tc::mbar_arrive(ring_e);
        else tc::mbar_arrive_cluster(tc::mapa(ring_e, 0u));
      }
      if (++acc == NUM_ACC) acc = 0, acc_phase ^= 1;
    }
    pend.finish(p);
    pend_col.finish(p);
    pend_row.finish(p);
  } else {
    // ---------------------------------------------------------- epilogue
    const int et = threadIdx.x - 64;     // 0 .. 32*EPI-1
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int P = p.patches;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int local = 0;; ++local) {
      const int slot = local % RING;
      const bool got = wait_bounded<PAIR>(tc::smem_u32(&sm.ring_full[slot]), (uint32_t)(local / RING) & 1u,
                                          abort_flag, p.err, peer_abort);
      const long long tile = got ? sm.tile_ring[slot] : -1;
      if (named_sync_epi_any<EPI>(tile < 0)) break;  // uniform: every epilogue thread read the same slot
      long long n0, cta_row0;
      int g_img = 0;  // GATHER: the tile's reference image
      if (MODE == GATHER) {
        const int mt = (int)(tile / p.nsub), ns = (int)(tile - (long long)mt * p.nsub);
        g_img = p.tile_img[mt];
        n0 = (long long)g_img * P + (long long)ns * BN;
        cta_row0 = (long long)mt * CTA_M;
      } else {
        int m_blk, n_blk;
        tile_coords(tile, p.num_m, p.num_n, C::GROUP_M, &m_blk, &n_blk);
        n0 = (long long)n_blk * BN;
        cta_row0 = (long long)m_blk * C::TILE_M + (long long)rank * CTA_M;
      }
      named_sync_epi<EPI>();  // previous tile's readers are done with col_norm / col_w
      for (int j = et; j < BN; j += EPI * 32) {
        const long long col = n0 + j;
        const bool ok = col < p.r_rows;
        sm.col_norm[j] = ok ? __ldg(p.r_norm + col) : 0.f;
        sm.col_w[j] = ok ? 2.f * __ldg(p.r_inv + col) : 0.f;
      }
      wait_bounded<false>(tc::smem_u32(&sm.acc_full[acc]), acc_phase, abort_flag, p.err, peer_abort);
      if (named_sync_epi_any<EPI>(*abort_flag)) break;  // uniform decision across the epilogue warps
      tc::fence_after_sync();

      const long long warp_row0 = cta_row0 + quarter * 32;
      const long long row = warp_row0 + lane;
      const bool row_ok = row < p.q_rows;
      const float qn = row_ok ? __ldg(p.q_norm + row) : 0.f;
      const float qi = row_ok ? __ldg(p.q_inv + row) : 0.f;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);

      if constexpr (MODE == GATHER) {
        // Rows of a staged tile, columns of one reference image: the minimum over the
        // image's columns in this tile, folded into the exact table.
        const int trow = row_ok ? __ldg(p.row_map + row) : -1;
        const long long c_end = (long long)(g_img + 1) * P;
        float m = INF;
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          const long long c0 = n0 + chunk * 32;
          if (c0 >= c_end) break;
          uint32_t raw[32];
          tc::tmem_ld_32x32b_x32(tbase + (uint32_t)(chunk * 32), raw);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int jj = chunk * 32 + j;
            const float v = fmaf(-__uint_as_float(raw[j]), qi * sm.col_w[jj], qn + sm.col_norm[jj]);
            m = (c0 + j < c_end) ? fminf(m, v) : m;
          }
        }
        if (trow >= 0) flush_min(p, trow, g_img, m);
      } else {
        const int q_img = (int)((p.q_first_row + row) / P);
        // Symmetric mode keeps only columns of a later image than the row's.
        const long long col_from = C::SYMM ? (long long)(q_img + 1) * P : 0;
        long long cta_last_row = cta_row0 + CTA_M - 1;
        if (cta_last_row > p.q_rows - 1) cta_last_row = p.q_rows - 1;
        const bool rows_full = cta_row0 + CTA_M <= p.q_rows;
        const bool clean = !C::SYMM || (rows_full && (cta_last_row / P) < (n0 / P));
        // row images covered by this warp (symmetric column minima)
        const bool warp_any = warp_row0 < p.q_rows;
        long long warp_last = warp_row0 + 31;
        if (warp_last > p.q_rows - 1) warp_last = p.q_rows - 1;
        const int w_img0 = (int)(warp_row0 / P), w_img1 = warp_any ? (int)(warp_last / P) : w_img0 - 1;

        int seg_img = (int)(n0 / P);
        long long seg_end = (long long)(seg_img + 1) * P;
        float m = INF;
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
          if (C::SYMM) {
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
      }
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
}  // namespace musc
