// The two small pieces of the training op around the GEMMs:
//
//   frx_loss_sum      loss = ce_weight * sum_r ce[r] + ent_weight * sum_r entropy[r]
//                     (the reference's `ce_weight * ce.sum() + ent_weight * ent.sum()`,
//                     fast_reduction/gemm_kernel.py:897), one CTA, fp64 accumulation in a fixed
//                     order, so the result does not depend on the launch or the GPU.
//   frx_scale_inplace x *= *scale for the precomputed gradients when autograd hands them over
//                     (the reference's `d_hidden * dloss`, gemm_kernel.py:905-913). The scale is
//                     read on the device, so the host never waits for it; when it is exactly 1
//                     (loss.backward() without an explicit gradient) every thread returns after
//                     one load.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstring>

#include "frx_host.cuh"

namespace frx {

constexpr int kLossThreads = 512;

__global__ void __launch_bounds__(kLossThreads)
    loss_sum_kernel(const float* __restrict__ ce, const float* __restrict__ ent, int64_t rows, float ce_weight,
                    float ent_weight, float* __restrict__ loss) {
  double sc = 0.0, se = 0.0;
  for (int64_t r = threadIdx.x; r < rows; r += kLossThreads) {
    if (ce != nullptr) sc += static_cast<double>(ce[r]);
    if (ent != nullptr) se += static_cast<double>(ent[r]);
  }
  double v = static_cast<double>(ce_weight) * sc + static_cast<double>(ent_weight) * se;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  __shared__ double part[kLossThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kLossThreads / 32; ++w) t += part[w];
    *loss = static_cast<float>(t);
  }
}

constexpr int kScaleThreads = 256;

// 16-bit values: bf16 (f16 = false) or fp16. Each element is multiplied by the fp32 scale in fp32
// and rounded to nearest once (torch's `g * dloss` would round dloss to the 16-bit type first).
__device__ __forceinline__ uint16_t scale16(uint16_t x, float s, bool f16) {
  if (f16) {
    __half h;
    memcpy(&h, &x, 2);
    const __half r = __float2half_rn(__half2float(h) * s);
    uint16_t o;
    memcpy(&o, &r, 2);
    return o;
  }
  __nv_bfloat16 b;
  memcpy(&b, &x, 2);
  const __nv_bfloat16 r = __float2bfloat16_rn(__bfloat162float(b) * s);
  uint16_t o;
  memcpy(&o, &r, 2);
  return o;
}

__global__ void __launch_bounds__(kScaleThreads)
    scale_inplace_kernel(void* __restrict__ x, int dtype, int64_t n, const float* __restrict__ scale, int vec_ok) {
  const float s = __ldg(scale);
  if (s == 1.0f) return;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kScaleThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kScaleThreads;
  if (dtype == FRX_DTYPE_F32) {
    float* p = static_cast<float*>(x);
    const int64_t nv = vec_ok ? n / 4 : 0;
    for (int64_t i = tid; i < nv; i += stride) {
      float4 v = reinterpret_cast<float4*>(p)[i];
      v.x *= s;
      v.y *= s;
      v.z *= s;
      v.w *= s;
      reinterpret_cast<float4*>(p)[i] = v;
    }
    for (int64_t i = nv * 4 + tid; i < n; i += stride) p[i] *= s;
    return;
  }
  const bool f16 = dtype == FRX_DTYPE_F16;
  uint16_t* p = static_cast<uint16_t*>(x);
  const int64_t nv = vec_ok ? n / 8 : 0;
  for (int64_t i = tid; i < nv; i += stride) {
    uint4 v = reinterpret_cast<uint4*>(p)[i];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = scale16(static_cast<uint16_t>(w[j] & 0xFFFFu), s, f16);
      const uint32_t hi = scale16(static_cast<uint16_t>(w[j] >> 16), s, f16);
      w[j] = lo | (hi << 16);
    }
    reinterpret_cast<uint4*>(p)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int64_t i = nv * 8 + tid; i < n; i += stride) p[i] = scale16(p[i], s, f16);
}

}  // namespace frx

extern "C" int frx_loss_sum(const float* ce, const float* entropy, int64_t rows, float ce_weight, float ent_weight,
                            float* loss, void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0, FRX_ERR_INVALID_ARG, "frx_loss_sum: rows %lld < 0", (long long)rows);
  FRX_REQUIRE(loss != nullptr, FRX_ERR_INVALID_ARG, "frx_loss_sum: null loss pointer");
  FRX_REQUIRE(rows == 0 || ce != nullptr || entropy != nullptr, FRX_ERR_INVALID_ARG,
              "frx_loss_sum: ce and entropy are both NULL");
  FRX_CHECK_RANGE(ce, rows * 4, "frx_loss_sum: ce");
  FRX_CHECK_RANGE(entropy, rows * 4, "frx_loss_sum: entropy");
  FRX_CHECK_RANGE(loss, 4, "frx_loss_sum: loss");
  loss_sum_kernel<<<1, kLossThreads, 0, static_cast<cudaStream_t>(stream)>>>(ce, entropy, rows, ce_weight, ent_weight,
                                                                             loss);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}

extern "C" int frx_scale_inplace(void* x, int dtype, int64_t n, const float* scale, void* stream) {
  using namespace frx;
  FRX_REQUIRE(n >= 0, FRX_ERR_INVALID_ARG, "frx_scale_inplace: n %lld < 0", (long long)n);
  if (n == 0) return FRX_OK;
  FRX_REQUIRE(x != nullptr && scale != nullptr, FRX_ERR_INVALID_ARG, "frx_scale_inplace: null pointer");
  FRX_REQUIRE(dtype == FRX_DTYPE_BF16 || dtype == FRX_DTYPE_F16 || dtype == FRX_DTYPE_F32, FRX_ERR_INVALID_ARG,
              "frx_scale_inplace: dtype must be FRX_DTYPE_BF16, FRX_DTYPE_F16 or FRX_DTYPE_F32");
  const int64_t esz = dtype == FRX_DTYPE_F32 ? 4 : 2;
  FRX_CHECK_RANGE(x, n * esz, "frx_scale_inplace: x");
  FRX_CHECK_RANGE(scale, 4, "frx_scale_inplace: scale");
  int sms = 0;
  const int rc = sm_count(&sms);
  if (rc) return rc;
  const int64_t per_block = static_cast<int64_t>(kScaleThreads) * (16 / esz);
  int64_t blocks = (n + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  if (blocks > cap) blocks = cap;
  scale_inplace_kernel<<<static_cast<unsigned>(blocks), kScaleThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, dtype, n, scale, aligned16(x) ? 1 : 0);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}
