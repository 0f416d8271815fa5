// fp32 -> bf16 hi / mid / lo parts for the bf16x6 emulation of fp32 matrix products on the bf16
// tensor cores (Henry, Tang, Heinecke, ARITH 2019): hi = bf16(x), mid = bf16(x - hi),
// lo = bf16(x - hi - mid). Each subtraction is exact in fp32 (the operands agree in their leading
// bits), so hi + mid + lo reproduces x to about 24 significant bits. Pure streaming kernel:
// 4 B read, 2 B written per requested part.
#include <algorithm>

#include "frx_host.cuh"

namespace frx {

constexpr int kSplitThreads = 256;

__device__ __forceinline__ void split3(float x, uint16_t (&part)[3]) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(hi);
  const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(mid);
  const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
  part[0] = __bfloat16_as_ushort(hi);
  part[1] = __bfloat16_as_ushort(mid);
  part[2] = __bfloat16_as_ushort(lo);
}

__device__ __forceinline__ void split_store(const float (&v)[4], uint32_t parts, int n_parts, uint16_t* out,
                                            int64_t part_stride, bool full, int64_t c0, int64_t cols) {
  uint16_t pr[4][3];
#pragma unroll
  for (int i = 0; i < 4; ++i) split3(v[i], pr[i]);
  for (int p = 0; p < n_parts; ++p) {
    const int sel = static_cast<int>((parts >> (2 * p)) & 3u);
    uint16_t* o = out + p * part_stride;
    uint16_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = sel == 0 ? pr[i][0] : (sel == 1 ? pr[i][1] : pr[i][2]);
    if (full) {
      const uint2 pk = make_uint2(static_cast<uint32_t>(w[0]) | (static_cast<uint32_t>(w[1]) << 16),
                                  static_cast<uint32_t>(w[2]) | (static_cast<uint32_t>(w[3]) << 16));
      __stcs(reinterpret_cast<uint2*>(o), pk);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (c0 + i < cols) o[i] = w[i];
    }
  }
}

__device__ __forceinline__ void load4(const float* xr, bool full, int64_t c0, int64_t cols, float (&v)[4]) {
  if (full) {
    const float4 q = __ldcs(reinterpret_cast<const float4*>(xr));
    v[0] = q.x;
    v[1] = q.y;
    v[2] = q.z;
    v[3] = q.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = c0 + i < cols ? xr[i] : 0.0f;
  }
}

// One thread per 4 consecutive columns of a row; grid.y (a few CTAs per SM) walks the rows two at a
// time, both rows' loads issued before either is split.
__global__ void __launch_bounds__(kSplitThreads)
    split_f32_kernel(const float* __restrict__ x, int64_t ld_x, int64_t rows, int64_t cols, uint32_t parts,
                     int n_parts, uint16_t* __restrict__ out, int64_t ld_out, int64_t part_stride, int vec_ok) {
  const int64_t c0 = (static_cast<int64_t>(blockIdx.x) * kSplitThreads + threadIdx.x) * 4;
  if (c0 >= cols) return;
  const bool full = vec_ok && c0 + 4 <= cols;
  const int64_t step = gridDim.y;
  int64_t r = blockIdx.y;
  for (; r + step < rows; r += 2 * step) {
    float a[4], b[4];
    load4(x + r * ld_x + c0, full, c0, cols, a);
    load4(x + (r + step) * ld_x + c0, full, c0, cols, b);
    split_store(a, parts, n_parts, out + r * ld_out + c0, part_stride, full, c0, cols);
    split_store(b, parts, n_parts, out + (r + step) * ld_out + c0, part_stride, full, c0, cols);
  }
  if (r < rows) {
    float a[4];
    load4(x + r * ld_x + c0, full, c0, cols, a);
    split_store(a, parts, n_parts, out + r * ld_out + c0, part_stride, full, c0, cols);
  }
}

}  // namespace frx

extern "C" int frx_split_f32(const float* x, int64_t ld_x, int64_t rows, int64_t cols, uint32_t parts, int n_parts,
                             void* out, int64_t ld_out, int64_t part_stride, void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && cols >= 0 && ld_x >= cols && ld_out >= cols && n_parts >= 1 && n_parts <= 16,
              FRX_ERR_INVALID_ARG, "frx_split_f32: bad sizes rows=%lld cols=%lld ld_x=%lld ld_out=%lld n_parts=%d",
              (long long)rows, (long long)cols, (long long)ld_x, (long long)ld_out, n_parts);
  if (rows == 0 || cols == 0) return FRX_OK;
  FRX_REQUIRE(x != nullptr && out != nullptr, FRX_ERR_INVALID_ARG, "frx_split_f32: null pointer");
  for (int p = 0; p < n_parts; ++p)
    FRX_REQUIRE(((parts >> (2 * p)) & 3u) <= FRX_PART_LO, FRX_ERR_INVALID_ARG,
                "frx_split_f32: part %d selector must be FRX_PART_HI, _MID or _LO", p);
  const int vec_ok = aligned16(x) && ld_x % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 7u) == 0 &&
                     ld_out % 4 == 0 && part_stride % 4 == 0;
  FRX_CHECK_RANGE(x, matrix_bytes(rows, cols, ld_x, 4), "frx_split_f32: x");
  FRX_CHECK_RANGE(out, ((n_parts - 1) * part_stride + matrix_bytes(rows, cols, ld_out, 1)) * 2, "frx_split_f32: out");
  const int64_t gx = (cols + 4 * kSplitThreads - 1) / (4 * kSplitThreads);
  FRX_REQUIRE(gx < (1ll << 31), FRX_ERR_INVALID_ARG, "frx_split_f32: too many columns");
  int sms = 0;
  const int rc = sm_count(&sms);
  if (rc) return rc;
  const int64_t max_gy = std::max<int64_t>(1, 8LL * sms / gx);  // a few resident CTAs per SM in all
  const unsigned gy = static_cast<unsigned>(std::min<int64_t>(rows, std::min<int64_t>(max_gy, 65535)));
  split_f32_kernel<<<dim3(static_cast<unsigned>(gx), gy), kSplitThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, ld_x, rows, cols, parts, n_parts, static_cast<uint16_t*>(out), ld_out, part_stride, vec_ok);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}
