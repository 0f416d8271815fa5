// Softmax partials of given logits (no GEMM): the standalone cross-entropy / entropy /
// logsumexp reductions over a materialised [rows, cols] logits matrix.
//
// One warp reduces one (row, column tile) to the same (m, s, u, zt) partial the fused GEMM
// epilogue writes, so frx_finalize produces ce / entropy / lse from it, and a long row is
// spread over several warps when there are few rows. Each lane streams 16-byte vectors and
// keeps an online (max, sum exp, sum (x - max) exp) over them; shuffles merge the lanes.
// HBM-bound: cols * sizeof(T) bytes read per row.
// Reference: fast_reduction/cute_cross_entropy.py:171-578 (CrossEntropyOnly, EntropyOnly,
// CrossEntropyEntropy), wrappers :583-735.
#include <cuda_fp16.h>

#include "frx_host.cuh"

namespace frx {

constexpr int kRowThreads = 256;

struct OnlineStat {
  float m, s, u;
};

__device__ __forceinline__ void online_merge(OnlineStat& a, const OnlineStat& b) {
  if (b.m == -INFINITY) return;
  if (a.m == -INFINITY) {
    a = b;
    return;
  }
  const float M = fmaxf(a.m, b.m);
  const float da = a.m - M, db = b.m - M;
  const float ea = ex2_approx(da * kLog2e), eb = ex2_approx(db * kLog2e);
  a.u = fmaf(da, a.s, a.u) * ea + fmaf(db, b.s, b.u) * eb;
  a.s = a.s * ea + b.s * eb;
  a.m = M;
}

// Adds n_valid values to the running stats. The reference point m only moves up when a vector
// holds a larger value (rare after the first few vectors of a row), so the steady state costs one
// ex2 per element; a raise rescales s and u to the new m first:
//   s' = s e^(m - M),  u' = (u + (m - M) s) e^(m - M).
template <int N>
__device__ __forceinline__ void online_add(OnlineStat& st, const float (&v)[N], int n_valid) {
  float vm = -INFINITY;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n_valid) vm = fmaxf(vm, v[i]);
  if (vm > st.m) {
    if (st.m != -INFINITY) {
      const float d = st.m - vm;
      const float e = ex2_approx(d * kLog2e);
      st.u = fmaf(d, st.s, st.u) * e;
      st.s *= e;
    }
    st.m = vm;
  }
  if (vm == -INFINITY) return;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    if (i < n_valid) {
      const float d = v[i] - st.m;  // formed first: exact 1 at the max, error independent of |m|
      const float e = ex2_approx(d * kLog2e);
      st.s += e;
      st.u = fmaf(d, e, st.u);
    }
  }
}

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 q = __ldcs(reinterpret_cast<const float4*>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  }
  __device__ static float scalar(const float* p) { return *p; }
};
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __device__ static float scalar(const __nv_bfloat16* p) { return __bfloat162float(*p); }
};
template <>
struct Vec16<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float (&v)[8]) {
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ static float scalar(const __half* p) { return __half2float(*p); }
};

// One warp reduces one (row, column tile): each lane streams 16-byte vectors (two loads in flight)
// into its own online stats, then five shuffle merges combine the lanes. No shared memory and no
// block barrier, so short tiles (a few thousand columns) cost no more per byte than long ones.
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
    logits_partials_kernel(const T* __restrict__ x, int64_t ld, int64_t rows, int64_t cols,
                           const int64_t* __restrict__ target, int64_t tile_cols, float4* __restrict__ partials,
                           int64_t tile_stride, int vec_ok) {
  using V = Vec16<T>;
  constexpr int N = V::N;
  constexpr int kWarps = kRowThreads / 32;
  const int lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  const int64_t c_begin = tile * tile_cols;
  const int64_t c_end = min(cols, c_begin + tile_cols);
  for (int64_t row = static_cast<int64_t>(blockIdx.y) * kWarps + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.y) * kWarps) {
    const T* xr = x + row * ld;
    OnlineStat st{-INFINITY, 0.f, 0.f};
    if (vec_ok) {
      constexpr int64_t kStride = 32 * N;
      int64_t c = c_begin + static_cast<int64_t>(lane) * N;
      // two full vectors per step, both loads issued before the math (same element order as below)
      for (; c + kStride + N <= c_end; c += 2 * kStride) {
        float a[N], b[N];
        V::load(xr + c, a);
        V::load(xr + c + kStride, b);
        online_add<N>(st, a, N);
        online_add<N>(st, b, N);
      }
      for (; c < c_end; c += kStride) {
        float v[N];
        if (c + N <= c_end) {
          V::load(xr + c, v);
          online_add<N>(st, v, N);
        } else {
#pragma unroll
          for (int i = 0; i < N; ++i) v[i] = (c + i < c_end) ? V::scalar(xr + c + i) : 0.f;
          online_add<N>(st, v, static_cast<int>(c_end - c));
        }
      }
    } else {
      for (int64_t c = c_begin + lane; c < c_end; c += 32) {
        float v[1] = {V::scalar(xr + c)};
        online_add<1>(st, v, 1);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      OnlineStat o{__shfl_xor_sync(0xffffffffu, st.m, off), __shfl_xor_sync(0xffffffffu, st.s, off),
                   __shfl_xor_sync(0xffffffffu, st.u, off)};
      online_merge(st, o);
    }
    if (lane == 0) {
      float zt = 0.f;
      if (target != nullptr) {
        const int64_t t = target[row];
        if (t >= c_begin && t < c_end) zt = V::scalar(xr + t);
      }
      partials[tile * tile_stride + row] = make_float4(st.m, st.s, st.u, zt);
    }
  }
}

}  // namespace frx

extern "C" int frx_logits_partials(const void* logits, int dtype, int64_t ld, int64_t rows, int64_t cols,
                                   const int64_t* target, int64_t tile_cols, float* partials, int64_t tile_stride,
                                   void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && cols >= 1 && tile_cols >= 1 && ld >= cols && tile_stride >= rows, FRX_ERR_INVALID_ARG,
              "frx_logits_partials: bad sizes rows=%lld cols=%lld ld=%lld tile_cols=%lld tile_stride=%lld",
              (long long)rows, (long long)cols, (long long)ld, (long long)tile_cols, (long long)tile_stride);
  if (rows == 0) return FRX_OK;
  FRX_REQUIRE(logits != nullptr && partials != nullptr && aligned16(partials), FRX_ERR_INVALID_ARG,
              "frx_logits_partials: null logits/partials or unaligned partials");
  const int64_t n_tiles = (cols + tile_cols - 1) / tile_cols;
  FRX_REQUIRE(n_tiles < (1ll << 31), FRX_ERR_INVALID_ARG, "frx_logits_partials: too many tiles");
  [[maybe_unused]] const int64_t esz = dtype == FRX_DTYPE_F32 ? 4 : 2;
  FRX_CHECK_RANGE(logits, matrix_bytes(rows, cols, ld, esz), "frx_logits_partials: logits");
  FRX_CHECK_RANGE(target, rows * 8, "frx_logits_partials: target");
  FRX_CHECK_RANGE(partials, matrix_bytes(n_tiles, rows, tile_stride, 16), "frx_logits_partials: partials");
  const int64_t row_blocks = (rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
  const dim3 grid(static_cast<unsigned>(n_tiles), static_cast<unsigned>(row_blocks < 65535 ? row_blocks : 65535));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FRX_DTYPE_F32) {
    const int vec_ok = aligned16(logits) && ld % 4 == 0 && tile_cols % 4 == 0;
    logits_partials_kernel<float><<<grid, kRowThreads, 0, st>>>(static_cast<const float*>(logits), ld, rows, cols,
                                                                 target, tile_cols,
                                                                 reinterpret_cast<float4*>(partials), tile_stride,
                                                                 vec_ok);
  } else if (dtype == FRX_DTYPE_BF16) {
    const int vec_ok = aligned16(logits) && ld % 8 == 0 && tile_cols % 8 == 0;
    logits_partials_kernel<__nv_bfloat16><<<grid, kRowThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), ld, rows, cols, target, tile_cols,
        reinterpret_cast<float4*>(partials), tile_stride, vec_ok);
  } else if (dtype == FRX_DTYPE_F16) {
    const int vec_ok = aligned16(logits) && ld % 8 == 0 && tile_cols % 8 == 0;
    logits_partials_kernel<__half><<<grid, kRowThreads, 0, st>>>(static_cast<const __half*>(logits), ld, rows, cols,
                                                                  target, tile_cols,
                                                                  reinterpret_cast<float4*>(partials), tile_stride,
                                                                  vec_ok);
  } else {
    FRX_REQUIRE(false, FRX_ERR_INVALID_ARG, "frx_logits_partials: unknown dtype %d", dtype);
  }
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}

namespace frx {

// acc[i] += the 8 16-bit values of q (bf16, or fp16 when kF16).
template <bool kF16>
__device__ __forceinline__ void add8(float (&acc)[8], const uint4& q) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (kF16) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    } else {
      acc[2 * i] += __uint_as_float(w[i] << 16);
      acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
}

// out[c] = sum over rows of x[r, c] (x bf16, or fp16 when kF16): a CTA owns 256 columns (8 per
// lane, 16-byte loads); its 8 warps take every 8th row, four rows in flight each, and the per-warp
// sums are added in a fixed order through shared memory.
template <bool kF16>
__global__ void __launch_bounds__(256)
    column_sums_kernel(const uint16_t* __restrict__ x, int64_t ld, int64_t rows, int64_t cols,
                       float* __restrict__ out, int vec_ok) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 256 + lane * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
    const bool full = vec_ok && c0 + 8 <= cols;
    int64_t r = warp;
    if (full) {
      // four rows per step with all four loads issued first; rows are added in increasing order,
      // exactly as the one-row loop below would add them
      for (; r + 24 < rows; r += 32) {
        uint4 q[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = __ldcs(reinterpret_cast<const uint4*>(x + (r + 8 * k) * ld + c0));
#pragma unroll
        for (int k = 0; k < 4; ++k) add8<kF16>(acc, q[k]);
      }
    }
    for (; r < rows; r += 8) {
      const uint16_t* xr = x + r * ld + c0;
      if (full) {
        add8<kF16>(acc, __ldcs(reinterpret_cast<const uint4*>(xr)));
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (c0 + i < cols) {
            const uint16_t b = xr[i];
            acc[i] += kF16 ? __half2float(__ushort_as_half(b)) : __uint_as_float(static_cast<uint32_t>(b) << 16);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[warp][lane * 8 + i] = acc[i];
  __syncthreads();
  const int64_t c = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (c < cols) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][threadIdx.x];
    out[c] = s;
  }
}

}  // namespace frx

extern "C" int frx_column_sums(const void* x, int dtype, int64_t ld, int64_t rows, int64_t cols, float* out,
                               void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && cols >= 0 && ld >= cols, FRX_ERR_INVALID_ARG, "frx_column_sums: bad sizes");
  FRX_REQUIRE(dtype == FRX_DTYPE_BF16 || dtype == FRX_DTYPE_F16, FRX_ERR_INVALID_ARG,
              "frx_column_sums: dtype must be FRX_DTYPE_BF16 or FRX_DTYPE_F16");
  if (cols == 0) return FRX_OK;
  FRX_REQUIRE(out != nullptr && (x != nullptr || rows == 0), FRX_ERR_INVALID_ARG, "frx_column_sums: null pointer");
  const int vec_ok = aligned16(x) && ld % 8 == 0;
  FRX_CHECK_RANGE(x, matrix_bytes(rows, cols, ld, 2), "frx_column_sums: x");
  FRX_CHECK_RANGE(out, cols * 4, "frx_column_sums: out");
  const int64_t blocks = (cols + 255) / 256;
  FRX_REQUIRE(blocks < (1ll << 31), FRX_ERR_INVALID_ARG, "frx_column_sums: too many columns");
  auto kernel = dtype == FRX_DTYPE_F16 ? column_sums_kernel<true> : column_sums_kernel<false>;
  kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), ld, rows, cols, out, vec_ok);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}
