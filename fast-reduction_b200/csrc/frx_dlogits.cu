// dlogits for loss = sum_r g_ce[r] ce[r] + g_ent[r] H[r] over one vocabulary shard:
//
//   p_j  = exp(z_j - lse)
//   dz_j = p_j * (g_ce - g_ent * (log p_j + H)) - g_ce * [j == target]
//
// (reference: fast_reduction/cute_dlogits.py:87-100). Pure streaming kernels, HBM-bound: they read
// the logits once and write bf16 (or fp16 / fp32) dlogits once. Two inputs: fp32 logits z
// (frx_dlogits), or fp16 tile-relative logits d = z - m_t with the tile maximum m_t taken from the
// forward partials (frx_dlogits_tilerel, 2 bytes per logit read instead of 4); then
// log p = d - (lse - m_t).
//
// Layout: a warp owns whole rows of a column span; each lane covers 32 fp32 or 64 fp16 columns of
// the row in 16-byte vectors placed so that consecutive lanes read consecutive 16 bytes (every load
// is fully coalesced), all eight loads of the row are issued before any arithmetic (128 bytes in
// flight per thread, 1024 threads per SM), and the per-row work (six constant loads, the target and
// ignore test, the row pointer) is spread over those columns. Measured at the headline chunk
// (4096 x 128256): one row and 16 columns per thread left the fp16 variant latency-bound at
// 4.1 TB/s (32 bytes of loads in flight per thread); 8 columns per lane per row made both variants
// issue-bound (25-30 instructions per logit, three of the four schedulers of every SM busy);
// 32 fp16 columns per lane (64 bytes in flight) gave 4.6-5.0 TB/s. Neither staging the fp16 loads in
// shared memory with LDGSTS two rows ahead (3.9 TB/s) nor a one-wave grid with L2 bulk prefetches
// two rows ahead (3.5 TB/s fp16, 4.8 TB/s fp32) helped.
#include <cstring>

#include "frx_host.cuh"

namespace frx {

constexpr int kDlThreads = 256;
constexpr int kDlWarps = kDlThreads / 32;
// Four CTAs (1024 threads) per SM: the register cap (64) under which the loads in flight fit.
constexpr int kDlMinBlocks = 4;

// Per-lane shape: kVec elements per 16-byte load, kSlots loads per row at stride 32 * kVec columns
// (the warp's loads of one slot are contiguous), one row per iteration. Either input keeps eight
// 16-byte loads (128 bytes) in flight per thread: 32 fp32 or 64 fp16 columns per lane, a warp span of
// 1024 or 2048 columns (four or eight vocabulary tiles).
template <bool kRel>
struct DlShape {
  static constexpr int kVec = kRel ? 8 : 4;
  static constexpr int kSlots = 8;
  static constexpr int kSpan = 32 * kVec * kSlots;
};

// dz for one logit from q = log2 p = log p * log2(e): p * (a + b log p) = 2^q * (a + (b ln 2) q), with
// b2 = b ln 2 formed once per row. Working in base 2 saves the multiply by log2(e) per logit: q comes
// straight out of the FMA that forms log p.
__device__ __forceinline__ float dz_of(float q, float a, float b2) { return ex2_approx(q) * fmaf(b2, q, a); }
constexpr float kLn2 = 0.6931471805599453f;

// Output element types of the kernels (template argument): bf16, fp16 or fp32.
constexpr int kOutBf16 = 0, kOutF16 = 1, kOutF32 = 2;

template <int kOut>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kOut == kOutF16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Tile-relative logits d = z - m_t are never positive (m_t is the maximum of the tile's z), so an
// fp16 d is decoded from its magnitude bits alone: moved into an fp32 exponent / mantissa they read
// as |d| * 2^-112 (exact for every finite fp16, subnormals included), and the factor -2^112 is folded
// into the FMA that forms log p = d - (lse - m_t). Two integer instructions per logit: an fp16
// conversion instruction runs on the same low-throughput unit as the exponential and made this
// kernel compute-bound (3.2 TB/s at the headline chunk), and a general decode with the sign took six.
// fp16 -inf (a logit more than 65504 below its tile maximum) decodes to -65536, a finite value whose
// probability is 0, so p * (a + b log p) stays 0 and never becomes 0 * inf.
__device__ __forceinline__ float rel_mag(uint32_t w, bool hi) {
  return __uint_as_float(hi ? ((w >> 3) & 0x0FFFE000u) : ((w << 13) & 0x0FFFE000u));
}
constexpr float kRelScale = -0x1p112f;
constexpr float kRelScale2 = kRelScale * kLog2e;  // the decode's scale times log2(e), for q = log2 p

// The per-row constants of the dz formula and the row's target column relative to the span
// [cw, cw + span) (-1 when outside it).
struct DlRow {
  float a, b, gc_t, lse;
  int tl;
};

__device__ __forceinline__ DlRow dl_row(int64_t row, int cw, int span, const int64_t* target, const float* lse,
                                        const float* ent, const float* g_ce, const float* g_ent, float ce_weight,
                                        float ent_weight, int64_t vocab_offset, int64_t ignore_index) {
  const float gc = g_ce != nullptr ? g_ce[row] : ce_weight;
  const float ge = g_ent != nullptr ? g_ent[row] : ent_weight;
  DlRow r;
  r.lse = lse[row];
  r.tl = -1;
  r.gc_t = gc;
  if (target != nullptr) {
    const int64_t t = target[row];
    if (t == ignore_index) r.gc_t = 0.0f;  // CE term dropped for ignored rows; entropy term kept
    const int64_t rel = t - vocab_offset - cw;
    if (rel >= 0 && rel < span) r.tl = static_cast<int>(rel);
  }
  r.a = r.gc_t - ge * ent[row];
  r.b = -ge;
  return r;
}

// Writes the kVec dlogits d of one slot to o: one vector store when all are valid and the output
// rows are 16-byte aligned, else element by element (n_valid of them).
template <int kOut, int kVec>
__device__ __forceinline__ void dl_store(void* o, const float (&d)[kVec], int n_valid, bool vec) {
  if constexpr (kOut == kOutF32) {
    float* of = static_cast<float*>(o);
    if (vec && n_valid == kVec) {
#pragma unroll
      for (int i = 0; i < kVec; i += 4)
        __stcs(reinterpret_cast<float4*>(of + i), make_float4(d[i], d[i + 1], d[i + 2], d[i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < kVec; ++i)
        if (i < n_valid) of[i] = d[i];
    }
  } else {
    uint16_t* oh = static_cast<uint16_t*>(o);
    if (vec && n_valid == kVec) {
      uint32_t w[kVec / 2];
#pragma unroll
      for (int i = 0; i < kVec / 2; ++i) w[i] = pack2<kOut>(d[2 * i], d[2 * i + 1]);
      if constexpr (kVec == 8)
        __stcs(reinterpret_cast<uint4*>(oh), make_uint4(w[0], w[1], w[2], w[3]));
      else
        __stcs(reinterpret_cast<uint2*>(oh), make_uint2(w[0], w[1]));
    } else {
#pragma unroll
      for (int i = 0; i < kVec; ++i)
        if (i < n_valid) oh[i] = static_cast<uint16_t>(pack2<kOut>(d[i], 0.0f) & 0xFFFFu);
    }
  }
}

// One warp's rows of the kernel below. kFull: every slot of the span is in bounds and both the input
// and output rows are 16-byte aligned, so no slot needs a bounds check (every span but a shard's
// last one, on the training pass's buffers).
template <bool kRel, int kOut, bool kFull>
__device__ __forceinline__ void dlogits_rows(const void* __restrict__ in, int64_t ld_in,
                                             const float4* __restrict__ partials, int64_t tile_stride,
                                             const int64_t* __restrict__ target, const float* __restrict__ lse,
                                             const float* __restrict__ ent, const float* __restrict__ g_ce,
                                             const float* __restrict__ g_ent, float ce_weight, float ent_weight,
                                             void* __restrict__ out, int64_t ld_out, int64_t rows, int cols,
                                             int64_t vocab_offset, int64_t ignore_index, bool in_vec, bool out_vec,
                                             int cw, int c0, int64_t row0, int64_t row_step) {
  using S = DlShape<kRel>;
  constexpr int kVec = S::kVec, kSlots = S::kSlots;
  constexpr int kInBytes = kRel ? 2 : 4;
  constexpr int kOutBytes = kOut == kOutF32 ? 4 : 2;
  for (int64_t row = row0; row < rows; row += row_step) {
    const char* rp = static_cast<const char*>(in) + row * ld_in * kInBytes;
    // All loads of the row first.
    uint4 raw[kSlots];
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      const int c = c0 + s * 32 * kVec;
      raw[s] = make_uint4(0u, 0u, 0u, 0u);
      if (kFull || (in_vec && c + kVec <= cols)) raw[s] = __ldcs(reinterpret_cast<const uint4*>(rp + c * kInBytes));
    }
    const DlRow r = dl_row(row, cw, S::kSpan, target, lse, ent, g_ce, g_ent, ce_weight, ent_weight, vocab_offset,
                           ignore_index);
    const float b2 = r.b * kLn2;
    const float lse2 = r.lse * kLog2e;
    // tile maximum of this lane's first slot (kRel: one 256-column tile per slot)
    const float4* pm = partials + static_cast<int64_t>(c0 / FRX_VOCAB_TILE) * tile_stride + row;
    char* op = static_cast<char*>(out) + row * ld_out * kOutBytes;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      const int c = c0 + s * 32 * kVec;
      const int nv = kFull ? kVec : min(cols - c, kVec);  // valid columns of this slot
      if (!kFull && nv <= 0) continue;
      const bool vec_in = kFull || (in_vec && nv == kVec);
      float q[kVec];  // log2 p
      if constexpr (kRel) {
        const float nshift2 = fmaf(__ldg(&pm[s * tile_stride].x), kLog2e, -lse2);  // (m_t - lse) log2(e)
        if (vec_in) {
          const uint32_t w[4] = {raw[s].x, raw[s].y, raw[s].z, raw[s].w};
#pragma unroll
          for (int i = 0; i < kVec; ++i) q[i] = fmaf(rel_mag(w[i >> 1], (i & 1) != 0), kRelScale2, nshift2);
        } else {
#pragma unroll
          for (int i = 0; i < kVec; ++i)
            q[i] = i < nv ? fmaf(rel_mag(reinterpret_cast<const uint16_t*>(rp)[c + i], false), kRelScale2, nshift2)
                          : 0.0f;
        }
      } else {
        if (vec_in) {
          const uint32_t w[4] = {raw[s].x, raw[s].y, raw[s].z, raw[s].w};
#pragma unroll
          for (int i = 0; i < kVec; ++i) q[i] = fmaf(__uint_as_float(w[i]), kLog2e, -lse2);
        } else {
#pragma unroll
          for (int i = 0; i < kVec; ++i)
            q[i] = i < nv ? fmaf(reinterpret_cast<const float*>(rp)[c + i], kLog2e, -lse2) : 0.0f;
        }
      }
      float d[kVec];
#pragma unroll
      for (int i = 0; i < kVec; ++i) d[i] = dz_of(q[i], r.a, b2);
      const int hit = r.tl - (c - cw);
      if (hit >= 0 && hit < kVec) {
#pragma unroll
        for (int i = 0; i < kVec; ++i)
          if (i == hit) d[i] -= r.gc_t;
      }
      dl_store<kOut, kVec>(op + static_cast<int64_t>(c) * kOutBytes, d, nv, kFull || out_vec);
    }
  }
}

// kRel = false: `in` is fp32 logits z [rows, ld_in]. kRel = true: `in` is fp16 tile-relative logits
// d = z - m_t <= 0 [rows, ld_in], and m_t is slot 0 of partials[t * tile_stride + row] for the
// 256-column tile t of the column. kOut: the dlogits type. Column indices are 32-bit
// (vocab_shard < 2^31 - span). in_vec / out_vec: rows 16-byte aligned (vector loads / stores).
template <bool kRel, int kOut>
__global__ void __launch_bounds__(kDlThreads, kDlMinBlocks)
    dlogits_kernel(const void* __restrict__ in, int64_t ld_in, const float4* __restrict__ partials,
                   int64_t tile_stride, const int64_t* __restrict__ target, const float* __restrict__ lse,
                   const float* __restrict__ ent, const float* __restrict__ g_ce, const float* __restrict__ g_ent,
                   float ce_weight, float ent_weight, void* __restrict__ out, int64_t ld_out, int64_t rows, int cols,
                   int64_t vocab_offset, int64_t ignore_index, int in_vec, int out_vec) {
  using S = DlShape<kRel>;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int cw = blockIdx.x * S::kSpan;
  const int c0 = cw + lane * S::kVec;  // this lane's first column; slot s starts 32 * kVec * s further
  const int64_t row_step = static_cast<int64_t>(gridDim.y) * kDlWarps;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kDlWarps + warp;
  if (in_vec && out_vec && cw + S::kSpan <= cols)  // uniform over the CTA
    dlogits_rows<kRel, kOut, true>(in, ld_in, partials, tile_stride, target, lse, ent, g_ce, g_ent, ce_weight,
                                   ent_weight, out, ld_out, rows, cols, vocab_offset, ignore_index, true, true, cw,
                                   c0, row0, row_step);
  else
    dlogits_rows<kRel, kOut, false>(in, ld_in, partials, tile_stride, target, lse, ent, g_ce, g_ent, ce_weight,
                                    ent_weight, out, ld_out, rows, cols, vocab_offset, ignore_index, in_vec != 0,
                                    out_vec != 0, cw, c0, row0, row_step);
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
  const int in_vec = aligned16(in) && ((ld_in * in_elem) % 16 == 0) ? 1 : 0;
  const int out_vec = aligned16(dlogits) && ((ld_dlogits * out_elem) % 16 == 0) ? 1 : 0;
  [[maybe_unused]] const int64_t n_tiles = (vocab_shard + FRX_VOCAB_TILE - 1) / FRX_VOCAB_TILE;
  FRX_CHECK_RANGE(in, matrix_bytes(rows, vocab_shard, ld_in, in_elem), "dlogits: logits");
  FRX_CHECK_RANGE(partials, rel ? matrix_bytes(n_tiles, rows, tile_stride, 16) : 0, "dlogits: partials");
  FRX_CHECK_RANGE(dlogits, matrix_bytes(rows, vocab_shard, ld_dlogits, out_elem), "dlogits: dlogits");
  FRX_CHECK_RANGE(target, rows * 8, "dlogits: target");
  FRX_CHECK_RANGE(lse, rows * 4, "dlogits: lse");
  FRX_CHECK_RANGE(entropy, rows * 4, "dlogits: entropy");
  FRX_CHECK_RANGE(g_ce, rows * 4, "dlogits: g_ce");
  FRX_CHECK_RANGE(g_ent, rows * 4, "dlogits: g_ent");
  const int span = rel ? DlShape<true>::kSpan : DlShape<false>::kSpan;
  FRX_REQUIRE(vocab_shard < (1ll << 31) - span, FRX_ERR_INVALID_ARG, "%s: vocab_shard too large", name);
  const int cols = static_cast<int>(vocab_shard);
  const int64_t gx = (vocab_shard + span - 1) / span;
  const int64_t row_blocks = (rows + kDlWarps - 1) / kDlWarps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned gy = static_cast<unsigned>(row_blocks < 65535 ? row_blocks : 65535);
  const int okind = out_f32 ? kOutF32 : (out_f16 ? kOutF16 : kOutBf16);
  auto kernel = rel ? (okind == kOutF32 ? dlogits_kernel<true, kOutF32>
                       : okind == kOutF16 ? dlogits_kernel<true, kOutF16> : dlogits_kernel<true, kOutBf16>)
                    : (okind == kOutF32 ? dlogits_kernel<false, kOutF32>
                       : okind == kOutF16 ? dlogits_kernel<false, kOutF16> : dlogits_kernel<false, kOutBf16>);
  kernel<<<dim3(static_cast<unsigned>(gx), gy), kDlThreads, 0, st>>>(
      in, ld_in, reinterpret_cast<const float4*>(partials), tile_stride, target, lse, entropy, g_ce, g_ent, ce_weight,
      ent_weight, dlogits, ld_dlogits, rows, cols, vocab_offset, ignore_index, in_vec, out_vec);
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
