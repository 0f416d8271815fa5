// Persistent, warp-specialised tcgen05 GEMM core shared by every contraction of the engine:
//
//   D[m, n] = sum_k A[m, k] * B[n, k]     (bf16 operands, fp32 accumulation in TMEM)
//
// with a pluggable epilogue that consumes each finished 128 x 256 fp32 accumulator tile
// straight from tensor memory (the forward CE/entropy reduction, a bf16/fp32 store, ...).
//
// CTA layout (192 threads, one CTA per SM):
//   warp 0      TMA producer: streams 128x64 A and 256x64 B bf16 tiles into a 4-deep
//               shared-memory ring (128-byte swizzle), completion counted on mbarriers.
//   warp 1      MMA issuer: owns the 512-column TMEM allocation; one thread issues
//               tcgen05.mma (M=128, N=256, K=16) into one of two 256-column accumulators,
//               so the epilogue of tile i overlaps the mainloop of tile i+1.
//   warps 2..5  epilogue: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32), i.e. one thread
//               per output row, and runs Epi::run on the tile.
//
// Operands may be K-major (row-major [rows, K], one 64-element box per tile row) or
// MN-major (row-major [K, rows], 64x64 boxes side by side), selected per operand at compile
// time; this is how the backward GEMMs read dlogits / weight / hidden in place without any
// transpose copies.
#pragma once

#include "frx_ptx.cuh"

namespace frx {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kGemmThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kABytes = kBM * kBK * 2;  // 16 KiB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KiB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kMNBoxBytes = 64 * kBK * 2;  // one 64 (MN) x 64 (K) bf16 box, 8 KiB
constexpr int kGemmSmemBytes = kStages * kStageBytes + 1024 /*barriers*/ + 1024 /*alignment slack*/;

// Dynamic shared memory of a GEMM kernel whose epilogue needs `epi_bytes` of staging space.
constexpr int gemm_smem_bytes(int ring_bytes, int epi_bytes) { return ring_bytes + epi_bytes + 2048; }

// Grouped rasterisation over (m-block, n-block) tiles: tiles are taken in bands of `group`
// m-blocks; inside a band the m-block index runs fastest. Concurrently resident CTAs then
// share both the band's A rows and a narrow slice of B in L2.
struct TileSched {
  int num_m;
  int num_n;
  int group;
  int num_tiles;
  int n256;  // number of 256-column blocks of the output (epilogue bound for wide tiles)
  int f16;   // operands are fp16 (else bf16)
  // Failure-detection testing only: when >= 0, the producer of the (leading) CTA leaves k-block
  // stall_kb of its first tile unfilled (no expect-tx, no copies), so the MMA warp's bounded wait
  // on that stage runs out. wait_limit_ns bounds every pipeline wait of the launch.
  int stall_kb;
  unsigned long long wait_limit_ns;
  __device__ __forceinline__ void get(int t, int& m_blk, int& n_blk) const {
    const int per_band = group * num_n;
    const int band = t / per_band;
    const int r = t - band * per_band;
    const int first_m = band * group;
    const int gm = min(group, num_m - first_m);
    n_blk = r / gm;
    m_blk = first_m + (r - n_blk * gm);
  }
};

template <bool kAMN, bool kBMN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        TileSched sched, int num_k_blocks, const __grid_constant__ typename Epi::Params ep,
                        int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + kStages * kABytes;
  uint8_t* s_epi = s_b + kStages * kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_epi + Epi::kSmemBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // uniform over the grid, so an early return skips every barrier together
  if (!device_check(reinterpret_cast<const uint8_t*>(tmem_slot + 2) - smem_raw <=
                        static_cast<ptrdiff_t>(dynamic_smem_bytes()),
                    threadIdx.x == 0 ? status : nullptr))
    return;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < sched.num_tiles && ok; t += gridDim.x) {
        int m_blk, n_blk;
        sched.get(t, m_blk, n_blk);
        const int m0 = m_blk * kBM;
        const int n0 = n_blk * kBN;
        for (int kb = 0; kb < num_k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, status, kStatusTimeoutProducer,
                                 sched.wait_limit_ns)) {
            ok = false;
            break;
          }
          if (kb == sched.stall_kb && t == static_cast<int>(blockIdx.x)) {
            ++issued;  // left unfilled on purpose (failure-detection testing); nothing is in flight
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          const int k0 = kb * kBK;
          uint8_t* da = s_a + stage * kABytes;
          uint8_t* db = s_b + stage * kBBytes;
          if (kAMN) {
#pragma unroll
            for (int g = 0; g < kBM / 64; ++g) tma_load_2d(da + g * kMNBoxBytes, &tm_a, &full[stage], m0 + 64 * g, k0);
          } else {
            tma_load_2d(da, &tm_a, &full[stage], k0, m0);
          }
          if (kBMN) {
#pragma unroll
            for (int g = 0; g < kBN / 64; ++g) tma_load_2d(db + g * kMNBoxBytes, &tm_b, &full[stage], n0 + 64 * g, k0);
          } else {
            tma_load_2d(db, &tm_b, &full[stage], k0, n0);
          }
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every copy still in flight land before the CTA's shared memory goes away.
        const long long first = issued > kStages ? issued - kStages : 0;
        for (long long j = first; j < issued; ++j)
          mbar_wait_drain(&full[j % kStages], static_cast<uint32_t>((j / kStages) & 1), status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f32acc(kBM, kBN, kAMN, kBMN, sched.f16 != 0);
      constexpr uint32_t a_lbo = kAMN ? kMNBoxBytes : 16;
      constexpr uint32_t b_lbo = kBMN ? kMNBoxBytes : 16;
      constexpr uint32_t a_kstep = kAMN ? 16 * 128 : 32;  // bytes per UMMA_K (=16) step
      constexpr uint32_t b_kstep = kBMN ? 16 * 128 : 32;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < sched.num_tiles && ok; t += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1u, abort_flag, status, kStatusTimeoutMma,
                               sched.wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBN);
        for (int kb = 0; kb < num_k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, status, kStatusTimeoutMma,
                                 sched.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(s_a + stage * kABytes);
          const uint32_t b_addr = smem_u32(s_b + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = make_smem_desc_sw128(a_addr + k * a_kstep, a_lbo, 1024);
            const uint64_t bdesc = make_smem_desc_sw128(b_addr + k * b_kstep, b_lbo, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // frees this smem slot once the MMAs have read it
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      // All MMAs issued by this thread must finish before TMEM is released.
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int t = blockIdx.x; t < sched.num_tiles; t += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_bounded(&acc_full[buf], acc_phase, abort_flag, status, kStatusTimeoutEpilogue,
                                   sched.wait_limit_ns) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int m_blk, n_blk;
      sched.get(t, m_blk, n_blk);
      const uint32_t tacc = tmem_base + static_cast<uint32_t>(buf * kBN) + (static_cast<uint32_t>(q * 32) << 16);
      Epi::run(ep, s_epi + q * Epi::kSmemPerWarp, tacc, m_blk, n_blk, q, lane, [&]() {
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
      });
    }
    Epi::finish(ep, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace frx

namespace frx {

// ---------------------------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2): a cluster of two CTAs on neighbouring SMs computes a
// 256 x (256 * kNH) output tile with M = 256 MMAs issued by the even CTA. Each CTA stages only its
// own 128 rows of A and its own 128-row halves of B, so per-SM shared-memory and L2 traffic per
// FLOP drop by a third against the single-CTA kernel. Each CTA's TMEM holds the fp32 accumulator
// of its 128 rows, and each CTA runs the epilogue on its own rows. No TMA multicast is used: every
// CTA loads its own operands; only MMA-completion commits are multicast to both CTAs.
//
// Two shapes share the code:
//   kNH = 1: 256 x 256 tiles, stage K = 128 (two 64-deep sub-tiles per operand), 3 stages, two
//            256-column TMEM accumulators (tile i's epilogue overlaps tile i+1's mainloop);
//            used by the forward, whose K (= hidden size) is short.
//   kNH = 2: 256 x 512 tiles, stage K = 64 with two 256-wide N halves sharing the A sub-tile,
//            4 stages, one 512-column accumulator; A is re-read half as often, which matters for
//            the backward GEMMs whose K (= vocabulary or batch) is long enough to hide the
//            epilogue.
// Either way a stage is 8 MMAs per tcgen05.commit: every commit costs the tensor pipe a drain
// bubble of roughly one MMA, which at 4 MMAs per commit held the pipe to ~79% busy and at 8 lets
// it run at ~99%.
//
// Barriers: the even CTA's full[s] counts the bytes of both CTAs' loads (the odd CTA's TMA
// completes on it through its shared::cluster address); the MMA commit frees empty[s] in both
// CTAs; acc_full[b] is signalled in both CTAs; the even CTA's acc_empty[b] collects one arrival
// per epilogue warp of both CTAs.
// ---------------------------------------------------------------------------------------------
constexpr int kPairSubBytes = 128 * 64 * 2;  // 128 rows x 64 K of bf16 (one SW128 sub-tile), 16 KiB

template <int kNH>
struct PairCfg {
  static constexpr int kKS = 2 / kNH;                    // 64-deep K sub-tiles per stage
  static constexpr int kStageK = 64 * kKS;                // K per stage
  static constexpr int kStages = kNH == 1 ? 3 : 4;
  static constexpr int kABytes = kKS * kPairSubBytes;     // this CTA's 128 rows of A
  static constexpr int kBBytes = kKS * kNH * kPairSubBytes;  // this CTA's 128-row slice of each N half
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kNumAcc = 2 / kNH;                 // TMEM accumulator buffers
  static constexpr int kTileN = 256 * kNH;
};

template <bool kAMN, bool kBMN, int kNH, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                             TileSched sched, int num_k_blocks, const __grid_constant__ typename Epi::Params ep,
                             int* status) {
  using Cfg = PairCfg<kNH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + Cfg::kStages * Cfg::kABytes;
  uint8_t* s_epi = s_b + Cfg::kStages * Cfg::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_epi + Epi::kSmemBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* acc_full = empty + Cfg::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // uniform over the grid (both CTAs of every pair), so an early return skips every barrier together
  if (!device_check(reinterpret_cast<const uint8_t*>(tmem_slot + 2) - smem_raw <=
                        static_cast<ptrdiff_t>(dynamic_smem_bytes()),
                    threadIdx.x == 0 ? status : nullptr))
    return;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();
  const bool leader = rank == 0;
  const int pair_id = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = pair_id; t < sched.num_tiles && ok; t += num_pairs) {
        int pm, pn;
        sched.get(t, pm, pn);
        const int m0 = pm * 2 * kBM + static_cast<int>(rank) * kBM;
        const int n0 = pn * Cfg::kTileN + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < num_k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, status, kStatusTimeoutProducer,
                                 sched.wait_limit_ns)) {
            ok = false;
            break;
          }
          if (leader && kb == sched.stall_kb && t == pair_id) {
            ++issued;  // left unfilled on purpose (failure-detection testing); nothing is in flight
            if (++stage == Cfg::kStages) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          const uint32_t bar = map_to_cta(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          uint8_t* da = s_a + stage * Cfg::kABytes;
          uint8_t* db = s_b + stage * Cfg::kBBytes;
#pragma unroll
          for (int ks = 0; ks < Cfg::kKS; ++ks) {
            const int kk = kb * Cfg::kStageK + 64 * ks;
            uint8_t* da_s = da + ks * kPairSubBytes;
            if (kAMN) {
#pragma unroll
              for (int g = 0; g < kBM / 64; ++g) tma_load_2d_pair(da_s + g * kMNBoxBytes, &tm_a, bar, m0 + 64 * g, kk);
            } else {
              tma_load_2d_pair(da_s, &tm_a, bar, kk, m0);
            }
#pragma unroll
            for (int h = 0; h < kNH; ++h) {
              uint8_t* db_s = db + (ks * kNH + h) * kPairSubBytes;
              const int nh = n0 + 256 * h;
              if (kBMN) {
#pragma unroll
                for (int g = 0; g < 2; ++g) tma_load_2d_pair(db_s + g * kMNBoxBytes, &tm_b, bar, nh + 64 * g, kk);
              } else {
                tma_load_2d_pair(db_s, &tm_b, bar, kk, nh);
              }
            }
          }
          ++issued;
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        if (leader) {
          const long long first = issued > Cfg::kStages ? issued - Cfg::kStages : 0;
          for (long long j = first; j < issued; ++j)
            mbar_wait_drain(&full[j % Cfg::kStages], static_cast<uint32_t>((j / Cfg::kStages) & 1), status);
        } else {
          // The odd CTA's copies complete on the even CTA's barriers; give them time to land.
          const uint64_t t0 = global_timer_ns();
          while (global_timer_ns() - t0 < kDrainLimitNs / 10) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && leader) {
      const uint32_t idesc = make_idesc_f32acc(2 * kBM, 256, kAMN, kBMN, sched.f16 != 0);
      constexpr uint32_t a_lbo = kAMN ? kMNBoxBytes : 16;
      constexpr uint32_t b_lbo = kBMN ? kMNBoxBytes : 16;
      constexpr uint32_t a_kstep = kAMN ? 16 * 128 : 32;  // bytes per UMMA_K (= 16) step
      constexpr uint32_t b_kstep = kBMN ? 16 * 128 : 32;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair_id; t < sched.num_tiles && ok; t += num_pairs, ++local) {
        const int buf = local % Cfg::kNumAcc;
        const uint32_t acc_phase = static_cast<uint32_t>((local / Cfg::kNumAcc) & 1);
        if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1u, abort_flag, status, kStatusTimeoutMma,
                               sched.wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * 256);
        for (int kb = 0; kb < num_k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, status, kStatusTimeoutMma,
                                 sched.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(s_a + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(s_b + stage * Cfg::kBBytes);
#pragma unroll
          for (int ks = 0; ks < Cfg::kKS; ++ks) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t adesc =
                  make_smem_desc_sw128(a_addr + ks * kPairSubBytes + k * a_kstep, a_lbo, 1024);
              const uint32_t acc = (kb | ks | k) != 0 ? 1u : 0u;
#pragma unroll
              for (int h = 0; h < kNH; ++h) {
                const uint64_t bdesc =
                    make_smem_desc_sw128(b_addr + (ks * kNH + h) * kPairSubBytes + k * b_kstep, b_lbo, 1024);
                umma_f16_pair(d_tmem + static_cast<uint32_t>(h * 256), adesc, bdesc, idesc, acc);
              }
            }
          }
          umma_commit_pair_mc(&empty[stage], 0x3);  // frees this slot in both CTAs
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair_mc(&acc_full[buf], 0x3);
      }
      umma_commit_pair(mma_done);
      mbar_wait_drain(mma_done, 0, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue warps (both CTAs)
    const int q = warp & 3;
    int local = 0;
    for (int t = pair_id; t < sched.num_tiles; t += num_pairs, ++local) {
      const int buf = local % Cfg::kNumAcc;
      const uint32_t acc_phase = static_cast<uint32_t>((local / Cfg::kNumAcc) & 1);
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_bounded(&acc_full[buf], acc_phase, abort_flag, status, kStatusTimeoutEpilogue,
                                   sched.wait_limit_ns) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int pm, pn;
      sched.get(t, pm, pn);
      const uint32_t tacc = tmem_base + static_cast<uint32_t>(buf * 256) + (static_cast<uint32_t>(q * 32) << 16);
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&acc_empty[buf]), 0));
      };
#pragma unroll 1
      for (int h = 0; h < kNH; ++h) {
        const int n_blk = pn * kNH + h;  // 256-column block index
        const bool last = h == kNH - 1;
        if (n_blk < sched.n256) {
          if (last) {
            Epi::run(ep, s_epi + q * Epi::kSmemPerWarp, tacc + static_cast<uint32_t>(h * 256),
                     pm * 2 + static_cast<int>(rank), n_blk, q, lane, release);
          } else {
            Epi::run(ep, s_epi + q * Epi::kSmemPerWarp, tacc + static_cast<uint32_t>(h * 256),
                     pm * 2 + static_cast<int>(rank), n_blk, q, lane, [] {});
          }
        } else if (last) {
          release();
        }
      }
    }
    Epi::finish(ep, lane);
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its barriers or smem
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace frx
