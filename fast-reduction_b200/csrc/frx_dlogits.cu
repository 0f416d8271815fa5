// dlogits for loss = sum_r g_ce[r] ce[r] + g_ent[r] H[r] over one vocabulary shard:
//
//   p_j  = exp(z_j - lse)
//   dz_j = p_j * (g_ce - g_ent * (log p_j + H)) - g_ce * [j == target]
//
// (reference: fast_reduction/cute_dlogits.py:87-100). Pure streaming kernel, HBM-bound:
// reads fp32 logits once, writes bf16 (or fp32) dlogits once. Each thread handles 8
// consecutive columns (two 16-byte loads, one 16-byte bf16 store); the per-row constants
// A = g_ce - g_ent * H and B = -g_ent are formed once per thread.
#include "frx_host.cuh"

namespace frx {

constexpr int kDlThreads = 256;
constexpr int kDlVec = 8;
constexpr int kDlColsPerBlock = kDlThreads * kDlVec;

__device__ __forceinline__ float dz_value(float z, float row_lse, float a, float b) {
  const float lp = z - row_lse;
  const float p = ex2_approx(lp * kLog2e);
  return p * fmaf(b, lp, a);
}

__global__ void __launch_bounds__(kDlThreads)
    dlogits_kernel(const float* __restrict__ logits, int64_t ld_logits, const int64_t* __restrict__ target,
                   const float* __restrict__ lse, const float* __restrict__ ent, const float* __restrict__ g_ce,
                   const float* __restrict__ g_ent, float ce_weight, float ent_weight, void* __restrict__ out,
                   int64_t ld_out, int out_f32, int64_t rows, int64_t cols, int64_t vocab_offset,
                   int64_t ignore_index, int vec_ok) {
  const int64_t c0 = (static_cast<int64_t>(blockIdx.x) * kDlThreads + threadIdx.x) * kDlVec;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const float gc = g_ce != nullptr ? g_ce[row] : ce_weight;
    const float ge = g_ent != nullptr ? g_ent[row] : ent_weight;
    const float row_lse = lse[row];
    const float h = ent[row];
    int64_t tcol = -1;
    float gc_t = gc;
    if (target != nullptr) {
      const int64_t t = target[row];
      if (t == ignore_index) gc_t = 0.0f;
      tcol = t - vocab_offset;
    }
    // CE term dropped for ignored rows; entropy term kept.
    const float a = gc_t - ge * h;
    const float b = -ge;
    if (c0 >= cols) continue;
    const float* zrow = logits + row * ld_logits;
    float z[kDlVec];
    const bool full = c0 + kDlVec <= cols;
    if (full && vec_ok) {
      const float4 z0 = __ldcs(reinterpret_cast<const float4*>(zrow + c0));
      const float4 z1 = __ldcs(reinterpret_cast<const float4*>(zrow + c0 + 4));
      z[0] = z0.x; z[1] = z0.y; z[2] = z0.z; z[3] = z0.w;
      z[4] = z1.x; z[5] = z1.y; z[6] = z1.z; z[7] = z1.w;
    } else {
#pragma unroll
      for (int i = 0; i < kDlVec; ++i) z[i] = (c0 + i < cols) ? zrow[c0 + i] : 0.0f;
    }
    float d[kDlVec];
#pragma unroll
    for (int i = 0; i < kDlVec; ++i) {
      d[i] = dz_value(z[i], row_lse, a, b);
      if (c0 + i == tcol) d[i] -= gc_t;
    }
    if (out_f32) {
      float* orow = static_cast<float*>(out) + row * ld_out;
      if (full && vec_ok) {
        __stcs(reinterpret_cast<float4*>(orow + c0), make_float4(d[0], d[1], d[2], d[3]));
        __stcs(reinterpret_cast<float4*>(orow + c0 + 4), make_float4(d[4], d[5], d[6], d[7]));
      } else {
#pragma unroll
        for (int i = 0; i < kDlVec; ++i)
          if (c0 + i < cols) orow[c0 + i] = d[i];
      }
    } else {
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(out) + row * ld_out;
      if (full && vec_ok) {
        uint4 pk;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(d[0], d[1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(d[2], d[3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(d[4], d[5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(d[6], d[7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(orow + c0) = pk;
      } else {
#pragma unroll
        for (int i = 0; i < kDlVec; ++i)
          if (c0 + i < cols) orow[c0 + i] = __float2bfloat16_rn(d[i]);
      }
    }
  }
}

}  // namespace frx

extern "C" int frx_dlogits(const float* logits, int64_t ld_logits, const int64_t* target, const float* lse,
                           const float* entropy, const float* g_ce, const float* g_ent, float ce_weight,
                           float ent_weight, void* dlogits, int64_t ld_dlogits, int out_dtype, int64_t rows,
                           int64_t vocab_shard, int64_t vocab_offset, int64_t ignore_index, void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && vocab_shard >= 0, FRX_ERR_INVALID_ARG, "frx_dlogits: bad sizes");
  if (rows == 0 || vocab_shard == 0) return FRX_OK;
  FRX_REQUIRE(logits != nullptr && lse != nullptr && entropy != nullptr && dlogits != nullptr, FRX_ERR_INVALID_ARG,
              "frx_dlogits: null logits/lse/entropy/dlogits pointer");
  FRX_REQUIRE(out_dtype == FRX_DTYPE_BF16 || out_dtype == FRX_DTYPE_F32, FRX_ERR_INVALID_ARG,
              "frx_dlogits: out_dtype must be FRX_DTYPE_BF16 or FRX_DTYPE_F32");
  FRX_REQUIRE(ld_logits >= vocab_shard && ld_dlogits >= vocab_shard, FRX_ERR_INVALID_ARG,
              "frx_dlogits: leading dimensions must be >= vocab_shard");
  const int out_f32 = out_dtype == FRX_DTYPE_F32 ? 1 : 0;
  const int64_t out_elem = out_f32 ? 4 : 2;
  const int vec_ok = aligned16(logits) && aligned16(dlogits) && (ld_logits % 4 == 0) &&
                     ((ld_dlogits * out_elem) % 16 == 0);
  const int64_t gx = (vocab_shard + kDlColsPerBlock - 1) / kDlColsPerBlock;
  FRX_REQUIRE(gx < (1ll << 31), FRX_ERR_INVALID_ARG, "frx_dlogits: vocab_shard too large");
  const unsigned gy = static_cast<unsigned>(rows < 65535 ? rows : 65535);
  dim3 grid(static_cast<unsigned>(gx), gy);
  dlogits_kernel<<<grid, kDlThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, ld_logits, target, lse, entropy, g_ce, g_ent, ce_weight, ent_weight, dlogits, ld_dlogits, out_f32,
      rows, vocab_shard, vocab_offset, ignore_index, vec_ok);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}
