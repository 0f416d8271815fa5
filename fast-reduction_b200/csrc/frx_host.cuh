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

// FRX_OK when [p, p + bytes) lies inside one device allocation (cuMemGetAddressRange), else
// FRX_ERR_INVALID_ARG with a message naming `what`. NULL / empty ranges pass.
int check_range(const void* p, int64_t bytes, const char* what);

// Declares a device range that is a valid buffer without being a driver allocation (a module
// __device__ array) to check_range.
void register_static_range(const void* base, size_t size);

// Bytes spanned by a row-major matrix of `rows` rows of `cols` elements with row stride `ld`.
inline int64_t matrix_bytes(int64_t rows, int64_t cols, int64_t ld, int64_t elem) {
  return rows <= 0 || cols <= 0 ? 0 : ((rows - 1) * ld + cols) * elem;
}

// Checked builds (FRX_CHECKED=1) verify before every launch that each buffer an entry point will
// touch lies inside a device allocation; release builds skip the (driver) query.
#if FRX_CHECKED
#define FRX_CHECK_RANGE(p, bytes, what)                    \
  do {                                                     \
    const int _rc = ::frx::check_range((p), (bytes), (what)); \
    if (_rc) return _rc;                                   \
  } while (0)
#else
#define FRX_CHECK_RANGE(p, bytes, what) \
  do {                                  \
  } while (0)
#endif

// Encodes a 2-D TMA descriptor over a row-major bf16 (or fp16, `f16`) matrix [rows, cols] with row
// stride `ld` elements, box [box_rows, box_cols] (box_cols * 2 bytes == 128 for the swizzle),
// 128-byte swizzle, zero fill outside the matrix.
int encode_16bit_2d(CUtensorMap* map, bool f16, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows, int box_cols);

// Same for an fp32 matrix (box_cols * 4 bytes == 128), used for TMA stores of logits tiles.
int encode_f32_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
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

// Operand descriptor for the GEMM core: a row-major bf16 / fp16 matrix plus how the GEMM reads it.
// K-major: the matrix is [mn_extent, k_extent]; MN-major: the matrix is [k_extent, mn_extent].
struct Operand {
  const void* ptr;
  int64_t ld;
  int64_t mn_extent;
  int64_t k_extent;
  bool mn_major;
  int dtype = FRX_DTYPE_BF16;  // FRX_DTYPE_BF16 or FRX_DTYPE_F16
};

// The 16-bit operand formats of the GEMM core.
inline bool is_gemm_dtype(int dtype) { return dtype == FRX_DTYPE_BF16 || dtype == FRX_DTYPE_F16; }

inline int encode_operand(CUtensorMap* map, const Operand& op, int tile_mn) {
  const bool f16 = op.dtype == FRX_DTYPE_F16;
  if (op.mn_major) return encode_16bit_2d(map, f16, op.ptr, op.k_extent, op.mn_extent, op.ld, kBK, 64);
  return encode_16bit_2d(map, f16, op.ptr, op.mn_extent, op.k_extent, op.ld, tile_mn, kBK);
}

// Which GEMM core runs: the CTA-pair kernel (default) or the single-CTA kernel. The
// FRX_GEMM_VARIANT environment variable ("pair" / "single") overrides it, for tuning only.
bool use_pair_kernel();

// Positive integer from the environment variable `name`, else `fallback` (tuning knobs only).
int env_int(const char* name, int fallback);

// Co-resident 2-CTA clusters of `kernel` on the current device (cached per device).
template <class Kernel>
int max_pair_clusters(Kernel kernel, std::atomic<int>* cache, int smem_bytes, int* out) {
  int dev = 0;
  FRX_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) {
      *out = c;
      return FRX_OK;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  FRX_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
  FRX_REQUIRE(n >= 1, FRX_ERR_CUDA, "no 2-CTA cluster of the GEMM kernel fits on this device");
  if (dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  *out = n;
  return FRX_OK;
}

// Launches the GEMM core. kWide selects 256 x 512 pair tiles (backward GEMMs, long K) instead of
// 256 x 256 double-buffered tiles (forward); it only applies to the pair kernel.
// max_sms > 0 caps the persistent grid at that many SMs (the others stay free for concurrent work,
// e.g. a collective on another stream); 0 uses every SM.
template <bool kAMN, bool kBMN, bool kWide, class Epi>
int launch_gemm(const Operand& a, const Operand& b, int64_t M, int64_t N, int64_t K, int group_m,
                const typename Epi::Params& ep, int* status, cudaStream_t stream, int stall_kb = -1,
                uint64_t wait_limit_ns = kWaitLimitNs, int max_sms = 0) {
  FRX_REQUIRE(is_gemm_dtype(a.dtype) && a.dtype == b.dtype, FRX_ERR_INVALID_ARG,
              "GEMM operands must both be bf16 or both fp16 (dtype codes %d, %d)", a.dtype, b.dtype);
  const bool pair = use_pair_kernel();
  const int b_rows = pair ? 128 : kBN;
  CUtensorMap tm_a, tm_b;
  int rc = encode_operand(&tm_a, a, kBM);
  if (rc) return rc;
  rc = encode_operand(&tm_b, b, b_rows);
  if (rc) return rc;
  constexpr int kNH = kWide ? 2 : 1;
  const int tile_m = pair ? 2 * kBM : kBM;
  const int tile_n = pair ? 256 * kNH : kBN;
  TileSched sched;
  sched.num_m = static_cast<int>((M + tile_m - 1) / tile_m);
  sched.num_n = static_cast<int>((N + tile_n - 1) / tile_n);
  sched.n256 = static_cast<int>((N + 255) / 256);
  sched.f16 = a.dtype == FRX_DTYPE_F16 ? 1 : 0;
  sched.stall_kb = stall_kb;
  sched.wait_limit_ns = wait_limit_ns;
  const int group = pair ? (group_m + 1) / 2 : group_m;
  sched.group = group < 1 ? 1 : (group > sched.num_m ? sched.num_m : group);
  const long long tiles = static_cast<long long>(sched.num_m) * sched.num_n;
  FRX_REQUIRE(tiles < (1ll << 31), FRX_ERR_INVALID_ARG, "problem too large: %lld output tiles", tiles);
  sched.num_tiles = static_cast<int>(tiles);
  if (pair) {
    using Cfg = PairCfg<kNH>;
    const int num_k_blocks = static_cast<int>((K + Cfg::kStageK - 1) / Cfg::kStageK);
    static std::atomic<uint64_t> attr_done{0};
    static std::atomic<int> clusters_cache[64];
    auto kernel = gemm_tcgen05_pair_kernel<kAMN, kBMN, kNH, Epi>;
    constexpr int smem = gemm_smem_bytes(Cfg::kStages * Cfg::kStageBytes, Epi::kSmemBytes);
    static_assert(smem <= 232448, "shared memory budget exceeded");
    rc = ensure_smem_attr(kernel, attr_done, smem);
    if (rc) return rc;
    int clusters = 0;
    rc = max_pair_clusters(kernel, clusters_cache, smem, &clusters);
    if (rc) return rc;
    if (max_sms > 0 && max_sms / 2 < clusters) clusters = max_sms / 2 < 1 ? 1 : max_sms / 2;
    const long long pairs = tiles < clusters ? tiles : clusters;
    kernel<<<static_cast<unsigned>(2 * pairs), kGemmThreads, smem, stream>>>(tm_a, tm_b, sched, num_k_blocks, ep,
                                                                             status);
  } else {
    const int num_k_blocks = static_cast<int>((K + kBK - 1) / kBK);
    static std::atomic<uint64_t> attr_done{0};
    auto kernel = gemm_tcgen05_kernel<kAMN, kBMN, Epi>;
    constexpr int smem = gemm_smem_bytes(kStages * kStageBytes, Epi::kSmemBytes);
    static_assert(smem <= 232448, "shared memory budget exceeded");
    rc = ensure_smem_attr(kernel, attr_done, smem);
    if (rc) return rc;
    int sms = 0;
    rc = sm_count(&sms);
    if (rc) return rc;
    if (max_sms > 0 && max_sms < sms) sms = max_sms;
    const int grid = static_cast<int>(tiles < sms ? tiles : sms);
    kernel<<<grid, kGemmThreads, smem, stream>>>(tm_a, tm_b, sched, num_k_blocks, ep, status);
  }
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}

}  // namespace frx
