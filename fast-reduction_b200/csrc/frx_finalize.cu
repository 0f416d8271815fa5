// Finalize: merge the per-(vocabulary tile, row) softmax partials into per-row
// cross-entropy, entropy, logsumexp and log-probability.
//
// Layout: partials[t * tile_stride + r] (float4) for t < n_tiles, r < rows. A CTA owns 32
// consecutive rows and splits the tile axis over 8 warps (warp w merges tiles w, w+8, ...),
// so every warp-wide load is one contiguous 512-byte segment and 256 threads keep many
// loads in flight; the 8 per-warp results are merged through shared memory.
//
// Merge rule (associative; identical to the reference's online-softmax merge in
// fast_reduction/gemm_ce_entropy_finalize.py:78-92, restated for the centred third slot):
//   M = max(m_a, m_b), a = exp(m_a - M), b = exp(m_b - M)   (one of the two is exactly 1)
//   S = s_a a + s_b b,  U = (u_a + (m_a - M) s_a) a + (u_b + (m_b - M) s_b) b,  ZT = zt_a + zt_b
// Final: lse = M + log S, H = log S - U / S, ce = lse - ZT (reference: :94-97).
#include <cmath>

#include "frx_host.cuh"

namespace frx {

struct RowStat {
  float m, s, u, zt;
};

__device__ __forceinline__ RowStat merge_stats(RowStat a, const RowStat& b) {
  if (b.m == -INFINITY) {
    a.zt += b.zt;
    return a;
  }
  if (a.m == -INFINITY) {
    RowStat r = b;
    r.zt += a.zt;
    return r;
  }
  // Only the smaller of the two maxima needs rescaling: one exp per merge, no branch.
  const bool a_hi = a.m >= b.m;
  const float m_hi = a_hi ? a.m : b.m, m_lo = a_hi ? b.m : a.m;
  const float s_hi = a_hi ? a.s : b.s, s_lo = a_hi ? b.s : a.s;
  const float u_hi = a_hi ? a.u : b.u, u_lo = a_hi ? b.u : a.u;
  const float d = m_lo - m_hi;  // <= 0
  const float e = ex2_approx(d * kLog2e);
  RowStat r;
  r.m = m_hi;
  r.s = fmaf(s_lo, e, s_hi);
  r.u = fmaf(fmaf(d, s_lo, u_lo), e, u_hi);
  r.zt = a.zt + b.zt;
  return r;
}

constexpr int kFinRows = 32;
constexpr int kFinSplits = 8;

__global__ void __launch_bounds__(kFinRows * kFinSplits)
    finalize_kernel(const float4* __restrict__ partials, int64_t n_tiles, int64_t rows, int64_t tile_stride,
                    int ref_layout, int ignore_negative, const int64_t* __restrict__ target, int64_t vocab_size,
                    int64_t ignore_index,
                    float* __restrict__ ce, float* __restrict__ ent, float* __restrict__ lse,
                    float* __restrict__ logp, float4* __restrict__ merged, int* status) {
  __shared__ RowStat red[kFinSplits][kFinRows];
  const int lane = threadIdx.x & 31;
  const int split = threadIdx.x >> 5;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kFinRows + lane;
  RowStat acc{-INFINITY, 0.f, 0.f, 0.f};
  if (row < rows) {
    int64_t t = split;
    // Four independent loads in flight per thread.
    for (; t + 3 * kFinSplits < n_tiles; t += 4 * kFinSplits) {
      float4 p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = __ldg(&partials[(t + i * kFinSplits) * tile_stride + row]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        RowStat b{p[i].x, p[i].y, ref_layout ? fmaf(-p[i].x, p[i].y, p[i].z) : p[i].z, p[i].w};
        acc = merge_stats(acc, b);
      }
    }
    for (; t < n_tiles; t += kFinSplits) {
      const float4 p = __ldg(&partials[t * tile_stride + row]);
      RowStat b{p.x, p.y, ref_layout ? fmaf(-p.x, p.y, p.z) : p.z, p.w};
      acc = merge_stats(acc, b);
    }
  }
  red[split][lane] = acc;
  __syncthreads();
  if (split != 0 || row >= rows) return;
#pragma unroll
  for (int i = 1; i < kFinSplits; ++i) acc = merge_stats(acc, red[i][lane]);

  if (merged != nullptr) merged[row] = make_float4(acc.m, acc.s, acc.u, acc.zt);
  const float log_s = logf(acc.s);
  const float row_lse = acc.m + log_s;
  const float row_ent = log_s - acc.u / acc.s;
  float row_ce = row_lse - acc.zt;
  if (target != nullptr) {
    const int64_t t = target[row];
    if (t == ignore_index || (ignore_negative && t < 0)) {
      row_ce = 0.0f;
    } else if (t < 0 || t >= vocab_size) {
      row_ce = __int_as_float(0x7fc00000);
      if (status) atomicOr(status, kStatusBadTarget);
    }
  }
  if (ce != nullptr) ce[row] = row_ce;
  if (ent != nullptr) ent[row] = row_ent;
  if (lse != nullptr) lse[row] = row_lse;
  if (logp != nullptr) logp[row] = -row_ce;
}

}  // namespace frx

extern "C" int frx_finalize(const float* partials, int64_t n_tiles, int64_t rows, int64_t tile_stride, int flags,
                            const int64_t* target, int64_t vocab_size, int64_t ignore_index, float* ce,
                            float* entropy, float* lse, float* log_probs, float* merged, int* status,
                            void* stream) {
  using namespace frx;
  FRX_REQUIRE(n_tiles >= 0 && rows >= 0 && tile_stride >= rows, FRX_ERR_INVALID_ARG,
              "frx_finalize: bad sizes n_tiles=%lld rows=%lld tile_stride=%lld", (long long)n_tiles,
              (long long)rows, (long long)tile_stride);
  FRX_REQUIRE((flags & ~(FRX_PARTIALS_REF_LAYOUT | FRX_IGNORE_NEGATIVE_TARGETS)) == 0, FRX_ERR_INVALID_ARG,
              "frx_finalize: unknown flags 0x%x", flags);
  if (rows == 0) return FRX_OK;
  FRX_REQUIRE(partials != nullptr || n_tiles == 0, FRX_ERR_INVALID_ARG, "frx_finalize: null partials");
  FRX_REQUIRE(partials == nullptr || aligned16(partials), FRX_ERR_INVALID_ARG,
              "frx_finalize: partials must be 16-byte aligned");
  FRX_REQUIRE(merged == nullptr || aligned16(merged), FRX_ERR_INVALID_ARG,
              "frx_finalize: merged must be 16-byte aligned");
  FRX_CHECK_RANGE(partials, matrix_bytes(n_tiles, rows, tile_stride, 16), "frx_finalize: partials");
  FRX_CHECK_RANGE(target, rows * 8, "frx_finalize: target");
  FRX_CHECK_RANGE(ce, rows * 4, "frx_finalize: ce");
  FRX_CHECK_RANGE(entropy, rows * 4, "frx_finalize: entropy");
  FRX_CHECK_RANGE(lse, rows * 4, "frx_finalize: lse");
  FRX_CHECK_RANGE(log_probs, rows * 4, "frx_finalize: log_probs");
  FRX_CHECK_RANGE(merged, rows * 16, "frx_finalize: merged");
  const int64_t blocks = (rows + kFinRows - 1) / kFinRows;
  FRX_REQUIRE(blocks < (1ll << 31), FRX_ERR_INVALID_ARG, "frx_finalize: too many rows");
  finalize_kernel<<<static_cast<unsigned>(blocks), kFinRows * kFinSplits, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(partials), n_tiles, rows, tile_stride, (flags & FRX_PARTIALS_REF_LAYOUT) ? 1 : 0,
      (flags & FRX_IGNORE_NEGATIVE_TARGETS) ? 1 : 0, target, vocab_size, ignore_index, ce, entropy, lse, log_probs,
      reinterpret_cast<float4*>(merged), status);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}
