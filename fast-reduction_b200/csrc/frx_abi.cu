// Library-wide host plumbing: error string, version, device attribute cache and TMA
// descriptor encoding (cuTensorMapEncodeTiled is fetched through the runtime's driver
// entry-point query, so the library does not link libcuda directly).
#include <cstring>

#include "frx_host.cuh"

namespace frx {

namespace {
thread_local char g_last_error[512] = {0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

std::atomic<int> g_sm_count[64];

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn get_address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}
}  // namespace

namespace {
// Device ranges that are not driver allocations (module __device__ arrays) but are valid buffers.
std::mutex g_static_mu;
struct StaticRange {
  uintptr_t base;
  size_t size;
};
StaticRange g_static_ranges[64];
int g_num_static = 0;
}  // namespace

void register_static_range(const void* base, size_t size) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  for (int i = 0; i < g_num_static; ++i)
    if (g_static_ranges[i].base == reinterpret_cast<uintptr_t>(base)) return;
  if (g_num_static < 64) g_static_ranges[g_num_static++] = {reinterpret_cast<uintptr_t>(base), size};
}

int check_range(const void* p, int64_t bytes, const char* what) {
  if (p == nullptr || bytes <= 0) return FRX_OK;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    for (int i = 0; i < g_num_static; ++i) {
      const StaticRange& r = g_static_ranges[i];
      if (a >= r.base && a < r.base + r.size)
        return a + static_cast<uint64_t>(bytes) <= r.base + r.size
                   ? FRX_OK
                   : (set_error("%s: %lld bytes from %p run past a %zu-byte static device array", what,
                                (long long)bytes, p, r.size),
                      FRX_ERR_INVALID_ARG);
    }
  }
  AddressRangeFn fn = get_address_range_fn();
  FRX_REQUIRE(fn != nullptr, FRX_ERR_CUDA, "cuMemGetAddressRange is unavailable from the CUDA driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(p));
  FRX_REQUIRE(r == CUDA_SUCCESS, FRX_ERR_INVALID_ARG, "%s: %p is not in a device allocation (CUresult %d)", what, p,
              static_cast<int>(r));
  const uint64_t end = static_cast<uint64_t>(base) + size;
  const uint64_t need = reinterpret_cast<uint64_t>(p) + static_cast<uint64_t>(bytes);
  FRX_REQUIRE(need <= end, FRX_ERR_INVALID_ARG,
              "%s: %lld bytes from %p run %llu bytes past the end of its device allocation", what,
              (long long)bytes, p, (unsigned long long)(need - end));
  return FRX_OK;
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

bool use_pair_kernel() {
  static const bool pair = [] {
    const char* v = getenv("FRX_GEMM_VARIANT");
    return !(v != nullptr && strcmp(v, "single") == 0);
  }();
  return pair;
}

int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  if (v == nullptr || *v == '\0') return fallback;
  char* end = nullptr;
  const long x = strtol(v, &end, 10);
  return (end != v && x > 0 && x < (1 << 20)) ? static_cast<int>(x) : fallback;
}

int sm_count(int* out) {
  int dev = 0;
  FRX_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64) {
    int cached = g_sm_count[dev].load(std::memory_order_relaxed);
    if (cached > 0) {
      *out = cached;
      return FRX_OK;
    }
  }
  int n = 0;
  FRX_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev < 64) g_sm_count[dev].store(n, std::memory_order_relaxed);
  *out = n;
  return FRX_OK;
}

static int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, int64_t rows,
                     int64_t cols, int64_t ld, int box_rows, int box_cols) {
  EncodeTiledFn fn = get_encode_fn();
  FRX_REQUIRE(fn != nullptr, FRX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  FRX_REQUIRE(aligned16(base), FRX_ERR_INVALID_ARG, "matrix base %p is not 16-byte aligned", base);
  FRX_REQUIRE((ld * elem_bytes) % 16 == 0, FRX_ERR_INVALID_ARG,
              "matrix leading dimension %lld x %d bytes is not a multiple of 16", (long long)ld, elem_bytes);
  FRX_REQUIRE(rows >= 1 && cols >= 1 && ld >= cols, FRX_ERR_INVALID_ARG,
              "bad matrix extents rows=%lld cols=%lld ld=%lld", (long long)rows, (long long)cols, (long long)ld);
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld) * static_cast<cuuint64_t>(elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FRX_REQUIRE(r == CUDA_SUCCESS, FRX_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return FRX_OK;
}

int encode_16bit_2d(CUtensorMap* map, bool f16, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows, int box_cols) {
  return encode_2d(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols,
                   ld, box_rows, box_cols);
}

int encode_f32_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                  int box_cols) {
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, rows, cols, ld, box_rows, box_cols);
}

}  // namespace frx

extern "C" int frx_abi_version(void) { return FRX_ABI_VERSION; }

extern "C" const char* frx_last_error(void) { return frx::g_last_error; }

extern "C" int frx_check_range(const void* ptr, int64_t bytes) {
  return frx::check_range(ptr, bytes, "frx_check_range");
}

namespace frx {

// One thread per block stamps its SM's cycle counter and the global nanosecond timer into the SM's
// slot. Cycle counters are per SM, so a clock is only read from two stamps of the same SM.
__global__ void clock_probe_kernel(unsigned long long* out, int max_sms) {
  if (threadIdx.x != 0) return;
  unsigned int smid;
  unsigned long long c, t;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (smid < static_cast<unsigned int>(max_sms)) {
    out[2 * smid] = c;
    out[2 * smid + 1] = t;
  }
}

}  // namespace frx

extern "C" int frx_clock_probe(uint64_t* out, int max_sms, void* stream) {
  FRX_REQUIRE(out != nullptr && max_sms >= 1 && max_sms <= 4096, FRX_ERR_INVALID_ARG,
              "frx_clock_probe: need an output of 2 * max_sms stamps, 1 <= max_sms <= 4096");
  frx::clock_probe_kernel<<<static_cast<unsigned>(4 * max_sms), 32, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<unsigned long long*>(out), max_sms);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}
