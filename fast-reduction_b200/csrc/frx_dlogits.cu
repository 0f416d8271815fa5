// dlogits for loss = sum_r g_ce[r] ce[r] + g_ent[r] H[r] over one vocabulary shard:
//
//   p_j  = exp(z_j - lse)
//   dz_j = p_j * (g_ce - g_ent * (log p_j + H)) - g_ce * [j == target]
//
// (reference: fast_reduction/cute_dlogits.py:87-100). Pure streaming kernel, HBM-bound:
// reads fp32 logits once, writes bf16 (or fp16 / fp32) dlogits once. Each thread handles 16
// consecutive columns of a row (four 16-byte streaming loads issued back to back, two 16-byte
// 16-bit stores); the per-row constants A = g_ce - g_ent * H and B = -g_ent are formed once per
// thread, after the loads are in flight.
//
// Two inputs: fp32 logits z (frx_dlogits), or fp16 tile-relative logits d = z - m_t with the tile
// maximum m_t taken from the forward partials (frx_dlogits_tilerel, 2 bytes per logit read instead
// of 4). Then log p = d - (lse - m_t), and the rest is the same.
#include <cstring>

#include "frx_host.cuh"

namespace frx {

constexpr int kDlThreads = 256;
constexpr int kDlVec = 16;  // columns per thread: four 16-byte loads in flight
constexpr int kDlColsPerBlock = kDlThreads * kDlVec;

// dz for one logit given lp = z - shift (shift = lse for fp32 logits, lse - m_t for tile-relative ones).
__device__ __forceinline__ float dz_value(float z, float shift, float a, float b) {
  const float lp = z - shift;
  const float p = ex2_approx(lp * kLog2e);
  return p * fmaf(b, lp, a);
}

__device__ __forceinline__ uint32_t pack_16x2(float lo, float hi, bool f16) {
  if (f16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The fp16 value in the low (hi = false) or high half of `w` as a float, with integer and FMA-pipe
// instructions only: the magnitude bits moved into an fp32 exponent / mantissa and scaled by 2^112
// (exact for every finite fp16, subnormals included), then the sign. A conversion instruction per
// element would run on the same low-throughput unit as the exponential and made this HBM-bound
// kernel compute-bound (3.2 TB/s at the headline shape). fp16 infinities come out as +-65536.
__device__ __forceinline__ float half_of(uint32_t w, bool hi) {
  const uint32_t h = hi ? (w >> 16) : w;
  const float mag = __uint_as_float((h & 0x7FFFu) << 13) * 0x1p112f;
  return __uint_as_float(__float_as_uint(mag) | ((h & 0x8000u) << 16));
}

// Tile-relative logits are stored saturated at the fp16 range: -inf (a logit more than 65504 below
// its tile maximum, read as -65536) is floored to -65504, whose probability is 0, so
// p * (a + b log p) stays 0 and never becomes 0 * inf.
constexpr float kRelFloor = -65504.0f;

// kRel = false: `in` is fp32 logits z [rows, ld_in]. kRel = true: `in` is fp16 tile-relative
// logits d = z - m_t [rows, ld_in], and m_t is slot 0 of partials[t * tile_stride + row] for the
// 256-column tile t of the column.
template <bool kRel>
__global__ void __launch_bounds__(kDlThreads)
    dlogits_kernel(const void* __restrict__ in, int64_t ld_in, const float4* __restrict__ partials,
                   int64_t tile_stride, const int64_t* __restrict__ target, const float* __restrict__ lse,
                   const float* __restrict__ ent, const float* __restrict__ g_ce, const float* __restrict__ g_ent,
                   float ce_weight, float ent_weight, void* __restrict__ out, int64_t ld_out, int out_f32,
                   int out_f16, int64_t rows, int64_t cols, int64_t vocab_offset, int64_t ignore_index, int vec_ok) {
  const int64_t c0 = (static_cast<int64_t>(blockIdx.x) * kDlThreads + threadIdx.x) * kDlVec;
  if (c0 >= cols) return;
  const bool full = vec_ok && c0 + kDlVec <= cols;
  const int64_t tile = c0 / FRX_VOCAB_TILE;  // kDlVec divides the tile width: one tile per thread
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    float z[kDlVec];
    if (kRel) {
      const uint16_t* zrow = static_cast<const uint16_t*>(in) + row * ld_in;
      if (full) {
#pragma unroll
        for (int i = 0; i < kDlVec; i += 8) {
          const uint4 q = __ldcs(reinterpret_cast<const uint4*>(zrow + c0 + i));
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            z[i + 2 * j] = half_of(w[j], false);
            z[i + 2 * j + 1] = half_of(w[j], true);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kDlVec; ++i) z[i] = (c0 + i < cols) ? half_of(zrow[c0 + i], false) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < kDlVec; ++i) z[i] = fmaxf(z[i], kRelFloor);
    } else {
      const float* zrow = static_cast<const float*>(in) + row * ld_in;
      if (full) {
#pragma unroll
        for (int i = 0; i < kDlVec; i += 4) {
          const float4 q = __ldcs(reinterpret_cast<const float4*>(zrow + c0 + i));
          z[i] = q.x;
          z[i + 1] = q.y;
          z[i + 2] = q.z;
          z[i + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < kDlVec; ++i) z[i] = (c0 + i < cols) ? zrow[c0 + i] : 0.0f;
      }
    }
    const float gc = g_ce != nullptr ? g_ce[row] : ce_weight;
    const float ge = g_ent != nullptr ? g_ent[row] : ent_weight;
    const float row_lse = kRel ? lse[row] - __ldg(&partials[tile * tile_stride + row].x) : lse[row];
    const float h = ent[row];
    int64_t tcol = -1;
    float gc_t = gc;
    if (target != nullptr) {
      const int64_t t = target[row];
      if (t == ignore_index) gc_t = 0.0f;  // CE term dropped for ignored rows; entropy term kept
      tcol = t - vocab_offset;
    }
    const float a = gc_t - ge * h;
    const float b = -ge;
    float d[kDlVec];
#pragma unroll
    for (int i = 0; i < kDlVec; ++i) d[i] = dz_value(z[i], row_lse, a, b);
    if (tcol >= c0 && tcol < c0 + kDlVec) {
#pragma unroll
      for (int i = 0; i < kDlVec; ++i)
        if (c0 + i == tcol) d[i] -= gc_t;
    }
    if (out_f32) {
      float* orow = static_cast<float*>(out) + row * ld_out;
      if (full) {
#pragma unroll
        for (int i = 0; i < kDlVec; i += 4)
          __stcs(reinterpret_cast<float4*>(orow + c0 + i), make_float4(d[i], d[i + 1], d[i + 2], d[i + 3]));
      } else {
#pragma unroll
        for (int i = 0; i < kDlVec; ++i)
          if (c0 + i < cols) orow[c0 + i] = d[i];
      }
    } else {
      const bool f16 = out_f16 != 0;
      uint16_t* orow = static_cast<uint16_t*>(out) + row * ld_out;
      if (full) {
#pragma unroll
        for (int i = 0; i < kDlVec; i += 8) {
          uint4 pk;
          pk.x = pack_16x2(d[i], d[i + 1], f16);
          pk.y = pack_16x2(d[i + 2], d[i + 3], f16);
          pk.z = pack_16x2(d[i + 4], d[i + 5], f16);
          pk.w = pack_16x2(d[i + 6], d[i + 7], f16);
          __stcs(reinterpret_cast<uint4*>(orow + c0 + i), pk);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kDlVec; ++i)
          if (c0 + i < cols) orow[c0 + i] = static_cast<uint16_t>(pack_16x2(d[i], 0.0f, f16) & 0xFFFFu);
      }
    }
  }
}

}  // namespace frx

namespace frx {

// Shared host side of frx_dlogits (rel = false: fp32 logits) and frx_dlogits_tilerel (rel = true:
// fp16 tile-relative logits plus the partials that hold each tile's maximum).
static int dlogits_impl(bool rel, const char* name, const void* in, int64_t ld_in, const float* partials,
                        int64_t tile_stride, const int64_t* target, const float* lse, const float* entropy,
                        const float* g_ce, const float* g_ent, float ce_weight, float ent_weight, void* dlogits,
                        int64_t ld_dlogits, int out_dtype, int64_t rows, int64_t vocab_shard, int64_t vocab_offset,
                        int64_t ignore_index, void* stream) {
  FRX_REQUIRE(rows >= 0 && vocab_shard >= 0, FRX_ERR_INVALID_ARG, "%s: bad sizes", name);
  if (rows == 0 || vocab_shard == 0) return FRX_OK;
  FRX_REQUIRE(in != nullptr && lse != nullptr && entropy != nullptr && dlogits != nullptr, FRX_ERR_INVALID_ARG,
              "%s: null logits/lse/entropy/dlogits pointer", name);
  FRX_REQUIRE(!rel || (partials != nullptr && tile_stride >= rows), FRX_ERR_INVALID_ARG,
              "%s: tile-relative logits need the partials (tile_stride %lld >= rows %lld)", name,
              (long long)tile_stride, (long long)rows);
  FRX_REQUIRE(out_dtype == FRX_DTYPE_BF16 || out_dtype == FRX_DTYPE_F16 || out_dtype == FRX_DTYPE_F32,
              FRX_ERR_INVALID_ARG, "%s: out_dtype must be FRX_DTYPE_BF16, FRX_DTYPE_F16 or FRX_DTYPE_F32", name);
  FRX_REQUIRE(ld_in >= vocab_shard && ld_dlogits >= vocab_shard, FRX_ERR_INVALID_ARG,
              "%s: leading dimensions must be >= vocab_shard", name);
  const int out_f32 = out_dtype == FRX_DTYPE_F32 ? 1 : 0;
  const int out_f16 = out_dtype == FRX_DTYPE_F16 ? 1 : 0;
  const int64_t out_elem = out_f32 ? 4 : 2;
  const int64_t in_elem = rel ? 2 : 4;
  const int vec_ok = aligned16(in) && aligned16(dlogits) && ((ld_in * in_elem) % 16 == 0) &&
                     ((ld_dlogits * out_elem) % 16 == 0);
  [[maybe_unused]] const int64_t n_tiles = (vocab_shard + FRX_VOCAB_TILE - 1) / FRX_VOCAB_TILE;
  FRX_CHECK_RANGE(in, matrix_bytes(rows, vocab_shard, ld_in, in_elem), "dlogits: logits");
  FRX_CHECK_RANGE(partials, rel ? matrix_bytes(n_tiles, rows, tile_stride, 16) : 0, "dlogits: partials");
  FRX_CHECK_RANGE(dlogits, matrix_bytes(rows, vocab_shard, ld_dlogits, out_elem), "dlogits: dlogits");
  FRX_CHECK_RANGE(target, rows * 8, "dlogits: target");
  FRX_CHECK_RANGE(lse, rows * 4, "dlogits: lse");
  FRX_CHECK_RANGE(entropy, rows * 4, "dlogits: entropy");
  FRX_CHECK_RANGE(g_ce, rows * 4, "dlogits: g_ce");
  FRX_CHECK_RANGE(g_ent, rows * 4, "dlogits: g_ent");
  const int64_t gx = (vocab_shard + kDlColsPerBlock - 1) / kDlColsPerBlock;
  FRX_REQUIRE(gx < (1ll << 31), FRX_ERR_INVALID_ARG, "%s: vocab_shard too large", name);
  const unsigned gy = static_cast<unsigned>(rows < 65535 ? rows : 65535);
  dim3 grid(static_cast<unsigned>(gx), gy);
  auto kernel = rel ? dlogits_kernel<true> : dlogits_kernel<false>;
  kernel<<<grid, kDlThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      in, ld_in, reinterpret_cast<const float4*>(partials), tile_stride, target, lse, entropy, g_ce, g_ent, ce_weight,
      ent_weight, dlogits, ld_dlogits, out_f32, out_f16, rows, vocab_shard, vocab_offset, ignore_index, vec_ok);
  FRX_CUDA_CHECK(cudaGetLastError());
  return FRX_OK;
}

}  // namespace frx

extern "C" int frx_dlogits(const float* logits, int64_t ld_logits, const int64_t* target, const float* lse,
                           const float* entropy, const float* g_ce, const float* g_ent, float ce_weight,
                           float ent_weight, void* dlogits, int64_t ld_dlogits, int out_dtype, int64_t rows,
                           int64_t vocab_shard, int64_t vocab_offset, int64_t ignore_index, void* stream) {
  return frx::dlogits_impl(false, "frx_dlogits", logits, ld_logits, nullptr, 0, target, lse, entropy, g_ce, g_ent,
                           ce_weight, ent_weight, dlogits, ld_dlogits, out_dtype, rows, vocab_shard, vocab_offset,
                           ignore_index, stream);
}

extern "C" int frx_dlogits_tilerel(const void* logits_rel, int64_t ld_logits_rel, const float* partials,
                                   int64_t tile_stride, const int64_t* target, const float* lse, const float* entropy,
                                   const float* g_ce, const float* g_ent, float ce_weight, float ent_weight,
                                   void* dlogits, int64_t ld_dlogits, int out_dtype, int64_t rows, int64_t vocab_shard,
                                   int64_t vocab_offset, int64_t ignore_index, void* stream) {
  return frx::dlogits_impl(true, "frx_dlogits_tilerel", logits_rel, ld_logits_rel, partials, tile_stride, target, lse,
                           entropy, g_ce, g_ent, ce_weight, ent_weight, dlogits, ld_dlogits, out_dtype, rows,
                           vocab_shard, vocab_offset, ignore_index, stream);
}
