// Forward CE / entropy entry point that allocates no device memory at all.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocator) on their call path --
// e.g. a plugin running inside a host framework that owns every byte of device memory and
// forbids foreign allocations, a latency-critical serving loop that must not pay cudaMalloc's
// implicit device synchronisation, or an embedded deployment whose memory budget is fixed at
// load time. frx_fwd_partials + frx_finalize need a caller-provided partials buffer between
// the two kernels; this entry point instead keeps that scratch in a fixed-size array that is
// part of the library image itself.
//
// Limits and sharing rules:
//   * hidden and weight must be bf16: the call passes FRX_DTYPE_BF16 to the GEMM and takes no
//     dtype argument.
//   * The scratch array is kFwdScratchBytes (32 MiB) per GPU; a call needs
//     ceil(vocab_size / 256) * rows * 16 bytes of it, so at most
//     floor(2097152 / ceil(vocab_size / 256)) rows per call (4185 at V = 128256). Larger calls
//     are rejected with FRX_ERR_INVALID_ARG before any GPU work.
//   * Every GPU that has the library's module loaded holds the 32 MiB until the process exits.
//     With CUDA's lazy module loading (the default) the driver loads the module, and reserves
//     the array, on the first call on that device (its cudaGetSymbolAddress); a caller that
//     hands all remaining device memory to its own allocator should make one small warm-up
//     call before doing so.
//   * All calls on a device share the one array. Calls whose kernels overlap on the GPU (for
//     example on two streams without ordering between them) race on it; serialise them.
//   * The array keeps the previous call's contents. Nothing needs to start at zero: the GEMM
//     writes every (tile, row) slot the finalize reads within the same call.
//   * The first call on each device looks up the array's device address (cudaGetSymbolAddress,
//     with that device current) and caches it; make that first call before any stream capture.
#include <mutex>

#include "frx_host.cuh"

namespace frx {

constexpr size_t kFwdScratchBytes = size_t(32) << 20;

// Host code must not use this name as a device pointer (in host code it denotes a host-side
// shadow); the device address comes from fwd_scratch_device_ptr().
static __device__ __align__(256) float4 g_fwd_scratch[kFwdScratchBytes / sizeof(float4)];

namespace {
std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};
}  // namespace

// Device address of g_fwd_scratch on the current device (looked up once per device).
static int fwd_scratch_device_ptr(void** out) {
  int dev = 0;
  FRX_CUDA_CHECK(cudaGetDevice(&dev));
  FRX_REQUIRE(dev >= 0 && dev < 64, FRX_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    FRX_CUDA_CHECK(cudaGetSymbolAddress(&p, g_fwd_scratch));
    register_static_range(p, kFwdScratchBytes);
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FRX_OK;
}

}  // namespace frx

extern "C" int frx_fwd_ce_entropy_noalloc(const void* hidden, int64_t ld_hidden, const void* weight,
                                          int64_t ld_weight, const int64_t* target, int64_t rows,
                                          int64_t vocab_size, int64_t hidden_dim, int64_t ignore_index, float* ce,
                                          float* entropy, float* lse, float* log_probs, int* status, void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && vocab_size >= 1 && hidden_dim >= 1, FRX_ERR_INVALID_ARG,
              "frx_fwd_ce_entropy_noalloc: bad sizes rows=%lld vocab_size=%lld hidden_dim=%lld", (long long)rows,
              (long long)vocab_size, (long long)hidden_dim);
  if (rows == 0) return FRX_OK;
  const int64_t n_tiles = (vocab_size + FRX_VOCAB_TILE - 1) / FRX_VOCAB_TILE;
  const int64_t max_rows = static_cast<int64_t>(kFwdScratchBytes / sizeof(float4)) / n_tiles;
  FRX_REQUIRE(rows <= max_rows, FRX_ERR_INVALID_ARG,
              "frx_fwd_ce_entropy_noalloc: %lld rows x %lld vocabulary tiles need %lld bytes of scratch, but the "
              "static scratch holds %zu bytes; call with at most %lld rows at this vocabulary size",
              (long long)rows, (long long)n_tiles, (long long)(rows * n_tiles * 16), kFwdScratchBytes,
              (long long)max_rows);
  void* scratch = nullptr;
  int rc = fwd_scratch_device_ptr(&scratch);
  if (rc) return rc;
  float* partials = static_cast<float*>(scratch);
  rc = frx_fwd_partials(hidden, ld_hidden, weight, ld_weight, FRX_DTYPE_BF16, nullptr, target, rows, vocab_size,
                        hidden_dim, 0, partials, rows, nullptr, 0, status, stream);
  if (rc) return rc;
  return frx_finalize(partials, n_tiles, rows, rows, 0, target, vocab_size, ignore_index, ce, entropy, lse, log_probs,
                      nullptr, status, stream);
}
