// Host-side helpers shared by the C-ABI entry points: the thread-local error string,
// argument checks, per-device attribute cache, TMA descriptor encoding and the launcher
// for the tcgen05 GEMM core.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "frx.h"
#include "frx_gemm.cuh"

namespace frx {

void set_error(const char* fmt, ...);

#define FRX_REQUIRE(cond, code, ...)   \
  do {                                 \
    if (!(cond)) {                     \
      ::frx::set_error(__VA_ARGS__);   \
      return (code);                   \
    }                                  \
  } while (0)

#define FRX_CUDA_CHECK(expr)                                                                    \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess) {                                                                    \
      ::frx::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
      return FRX_ERR_CUDA;                                                                      \
    }                                                                                           \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device ordinal).
int sm_count(int* out);

// Encodes a 2-D bf16 TMA descriptor over a row-major matrix [rows, cols] with row stride
// `ld` elements, box [box_rows, box_cols] (box_cols * 2 bytes == 128 for the swizzle),
// 128-byte swizzle, zero fill outside the matrix.
int encode_bf16_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                   int box_cols);

// Opts the kernel into the large dynamic shared memory carve-out (once per device).
template <class Kernel>
int ensure_smem_attr(Kernel kernel, std::atomic<uint64_t>& done_mask, int bytes) {
  int dev = 0;
  FRX_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return FRX_OK;
  FRX_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return FRX_OK;
}

// Operand descriptor for the GEMM core: a row-major bf16 matrix plus how the GEMM reads it.
// K-major: the matrix is [mn_extent, k_extent]; MN-major: the matrix is [k_extent, mn_extent].
struct Operand {
  const void* ptr;
  int64_t ld;
  int64_t mn_extent;
  int64_t k_extent;
  bool mn_major;
};

inline int encode_operand(CUtensorMap* map, const Operand& op, int tile_mn) {
  if (op.mn_major) return encode_bf16_2d(map, op.ptr, op.k_extent, op.mn_extent, op.ld, kBK, 64);
  return encode_bf16_2d(map, op.ptr, op.mn_extent, op.k_extent, op.ld, tile_mn, kBK);
}

template <bool kAMN, bool kBMN, class Epi>
int launch_gemm(const Operand& a, const Operand& b, int64_t M, int64_t N, int64_t K, int group_m,
                const typename Epi::Params& ep, int* status, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_done{0};
  CUtensorMap tm_a, tm_b;
  int rc = encode_operand(&tm_a, a, kBM);
  if (rc) return rc;
  rc = encode_operand(&tm_b, b, kBN);
  if (rc) return rc;
  auto kernel = gemm_tcgen05_kernel<kAMN, kBMN, Epi>;
  rc = ensure_smem_attr(kernel, attr_done, kGemmSmemBytes);
  if (rc) return rc;
  int sms = 0;
  rc = sm_count(&sms);
  if (rc) return rc;
  TileSched sched;
  sched.num_m = static_cast<int>((M + kBM - 1) / kBM);
  sched.num_n = static_cast<int>((N + kBN - 1) / kBN);
  sched.group = group_m < 1 ? 1 : (group_m > sched.num_m ? sched.num_m : group_m);
  const long long tiles = static_cast<long long>(sched.num_m) * sched.num_n;
  FRX_REQUIRE(tiles < (1ll << 31), FRX_ERR_INVALID_ARG, "problem too large: %lld output tiles", tiles);
  sched.num_tiles = static_cast<int>(tiles);
  const int num_k_blocks = static_cast<int>((K + kBK - 1) / kBK);
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  kernel<<<grid, kGemmThreads, kGemmSmemBytes, stream>>>(tm_a, tm_b, sched, num_k_blocks, ep, status);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}

}  // namespace frx
