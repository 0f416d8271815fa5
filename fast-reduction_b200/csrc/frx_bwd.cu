// Backward contractions of the training path, both on the tcgen05 GEMM core:
//
//   d_hidden[B, H] = dlogits[B, V] @ weight[V, H]      A = dlogits (K-major), B = weight (MN-major)
//   d_weight[V, H] = dlogits[B, V]^T @ hidden[B, H]    A = dlogits (MN-major), B = hidden (MN-major)
//
// Both read their operands in place (no transposed copies): the MN-major operands are
// fetched as 64 x 64 TMA boxes and described to tcgen05.mma with the MN-major bit. d_weight
// is accumulated over the whole batch in fp32 tensor memory and written once.
#include <cstring>

#include "frx_host.cuh"

namespace frx {

// Packs two floats into a bf16x2 or fp16x2 word (round to nearest even), low half first.
__device__ __forceinline__ uint32_t pack2(float a, float b, bool f16) {
  uint32_t w;
  if (f16) {
    const __half2 h = __floats2half2_rn(a, b);
    memcpy(&w, &h, sizeof(w));
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    memcpy(&w, &h, sizeof(w));
  }
  return w;
}

// Writes the fp32 accumulator tile as bf16, fp16 or fp32 rows: each thread owns one output row and
// stores 32 consecutive columns per TMEM load.
struct StoreEpilogue {
  static constexpr int kSmemPerWarp = 0;
  static constexpr int kSmemBytes = 0;

  struct Params {
    void* out;
    int64_t ld_out;
    int rows;
    int cols;
    int out_f32;
    int out_f16;  // 16-bit output is fp16 (else bf16)
    int accumulate;  // fp32 output: add the product to what the output holds
    int vec_ok;   // base and ld allow 16-byte vector stores
  };

  template <class Release>
  __device__ __forceinline__ static void run(const Params& p, uint8_t* /*stage*/, uint32_t tacc, int m_blk, int n_blk,
                                             int q, int lane, Release release) {
    const int row = m_blk * kBM + q * 32 + lane;
    const int n0 = n_blk * kBN;
    const int ncols = min(kBN, p.cols - n0);
    const bool row_ok = row < p.rows;
    float v[32];
#pragma unroll 1
    for (int c = 0; c < kBN / 32; ++c) {
      const int lim = ncols - c * 32;
      if (lim <= 0) break;
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after per-row branches
      tmem_load_32cols(tacc + static_cast<uint32_t>(c * 32), v);
      if (!row_ok) continue;  // uniform reconvergence is restored by the __syncwarp above
      const int64_t off = static_cast<int64_t>(row) * p.ld_out + n0 + c * 32;
      if (p.out_f32) {
        float* dst = static_cast<float*>(p.out) + off;
        if (lim >= 32 && p.vec_ok) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            if (p.accumulate) {
              const float4 prev = *reinterpret_cast<const float4*>(dst + j);
              o.x += prev.x;
              o.y += prev.y;
              o.z += prev.z;
              o.w += prev.w;
            }
            *reinterpret_cast<float4*>(dst + j) = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < lim) dst[j] = p.accumulate ? dst[j] + v[j] : v[j];
        }
      } else {
        const bool f16 = p.out_f16 != 0;
        uint16_t* dst = static_cast<uint16_t*>(p.out) + off;
        if (lim >= 32 && p.vec_ok) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            pk.x = pack2(v[j], v[j + 1], f16);
            pk.y = pack2(v[j + 2], v[j + 3], f16);
            pk.z = pack2(v[j + 4], v[j + 5], f16);
            pk.w = pack2(v[j + 6], v[j + 7], f16);
            *reinterpret_cast<uint4*>(dst + j) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < lim) dst[j] = static_cast<uint16_t>(pack2(v[j], 0.0f, f16) & 0xFFFFu);
        }
      }
    }
    release();
  }

  __device__ __forceinline__ static void finish(const Params&, int) {}
};

// Adds the fp32 accumulator tile into a multicast (NVLS) view of an fp32 matrix that every rank
// of the vocabulary-parallel group holds: the NVSwitch sums all ranks' contributions into every
// copy, so the d_hidden all-reduce happens inside this GEMM, tile by tile, while it computes.
struct MultimemAddEpilogue {
  // Two 32 x 32 fp32 staging blocks per epilogue warp: rows are re-read row-contiguously so each
  // warp-wide reduction covers four full 128-byte row segments instead of 32 scattered 16-byte ones.
  static constexpr int kSmemPerWarp = 2 * 32 * 32 * 4;
  static constexpr int kSmemBytes = 4 * kSmemPerWarp;

  struct Params {
    float* mc_out;  // multicast address of the fp32 [rows, cols] accumulation buffer
    int64_t ld_out;
    int rows;
    int cols;
  };

  template <class Release>
  __device__ __forceinline__ static void run(const Params& p, uint8_t* stage, uint32_t tacc, int m_blk, int n_blk,
                                             int q, int lane, Release release) {
    const int row0 = m_blk * kBM + q * 32;
    const int n0 = n_blk * kBN;
    const int ncols = min(kBN, p.cols - n0);
    const uint32_t stage_base = smem_u32(stage);
    float v[32];
#pragma unroll 1
    for (int c = 0; c < kBN / 32; ++c) {
      const int lim = ncols - c * 32;
      if (lim <= 0) break;
      __syncwarp();
      tmem_load_32cols(tacc + static_cast<uint32_t>(c * 32), v);
      // lane = row: write the row's 8 16-byte chunks XOR-swizzled by row % 8 (bank-conflict free)
      const uint32_t buf = stage_base + static_cast<uint32_t>((c & 1) * 4096);
      const uint32_t rowb = buf + static_cast<uint32_t>(lane * 128);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        st_shared_v4(rowb + static_cast<uint32_t>((j ^ (lane & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                     v[4 * j + 3]);
      __syncwarp();
      // read back: lane = (row-in-group, chunk); 8 lanes cover one row's 128 bytes
      const int j = lane & 7;
      const int col = c * 32 + 4 * j;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 4 * i + (lane >> 3);
        const int row = row0 + r;
        float4 x;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                     : "r"(buf + static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4))));
        if (row < p.rows) {
          float* dst = p.mc_out + static_cast<int64_t>(row) * p.ld_out + n0 + col;
          if (col + 4 <= ncols) {
            multimem_red_add_v4(dst, x.x, x.y, x.z, x.w);
          } else {
            if (col + 0 < ncols) multimem_red_add(dst + 0, x.x);
            if (col + 1 < ncols) multimem_red_add(dst + 1, x.y);
            if (col + 2 < ncols) multimem_red_add(dst + 2, x.z);
          }
        }
      }
    }
    release();
  }

  // Order this thread's reductions before anything that follows the kernel at system scope.
  __device__ __forceinline__ static void finish(const Params&, int) { __threadfence_system(); }
};

static int check_out(void* out, int64_t ld, int64_t cols, int out_dtype, const char* who) {
  FRX_REQUIRE(out != nullptr, FRX_ERR_INVALID_ARG, "%s: null output pointer", who);
  FRX_REQUIRE((out_dtype & FRX_OUT_ACCUMULATE) == 0 || (out_dtype & ~FRX_OUT_ACCUMULATE) == FRX_DTYPE_F32,
              FRX_ERR_INVALID_ARG, "%s: FRX_OUT_ACCUMULATE needs an fp32 output", who);
  out_dtype &= ~FRX_OUT_ACCUMULATE;
  FRX_REQUIRE(out_dtype == FRX_DTYPE_BF16 || out_dtype == FRX_DTYPE_F16 || out_dtype == FRX_DTYPE_F32,
              FRX_ERR_INVALID_ARG, "%s: out_dtype must be FRX_DTYPE_BF16, FRX_DTYPE_F16 or FRX_DTYPE_F32", who);
  FRX_REQUIRE(ld >= cols, FRX_ERR_INVALID_ARG, "%s: output leading dimension %lld < %lld columns", who,
              (long long)ld, (long long)cols);
  return FRX_OK;
}

[[maybe_unused]] static int64_t out_elem_bytes(int out_dtype) {
  return (out_dtype & ~FRX_OUT_ACCUMULATE) == FRX_DTYPE_F32 ? 4 : 2;
}

static StoreEpilogue::Params store_params(void* out, int64_t ld, int64_t rows, int64_t cols, int out_dtype) {
  StoreEpilogue::Params ep;
  ep.out = out;
  ep.ld_out = ld;
  ep.rows = static_cast<int>(rows);
  ep.cols = static_cast<int>(cols);
  ep.accumulate = (out_dtype & FRX_OUT_ACCUMULATE) ? 1 : 0;
  out_dtype &= ~FRX_OUT_ACCUMULATE;
  ep.out_f32 = out_dtype == FRX_DTYPE_F32 ? 1 : 0;
  ep.out_f16 = out_dtype == FRX_DTYPE_F16 ? 1 : 0;
  const int64_t elem = ep.out_f32 ? 4 : 2;
  ep.vec_ok = aligned16(out) && ((ld * elem) % 16 == 0) ? 1 : 0;
  return ep;
}

}  // namespace frx

extern "C" int frx_gemm_dhidden(const void* dlogits, int64_t ld_dlogits, const void* weight, int64_t ld_weight,
                                int in_dtype, void* d_hidden, int64_t ld_d_hidden, int out_dtype, int64_t rows,
                                int64_t hidden_dim, int64_t vocab_shard, int* status, void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && hidden_dim >= 1 && vocab_shard >= 1 && rows < (1ll << 31) && hidden_dim < (1ll << 31) &&
                  vocab_shard < (1ll << 31),
              FRX_ERR_INVALID_ARG, "frx_gemm_dhidden: bad sizes rows=%lld hidden_dim=%lld vocab_shard=%lld",
              (long long)rows, (long long)hidden_dim, (long long)vocab_shard);
  if (rows == 0) return FRX_OK;
  FRX_REQUIRE(dlogits != nullptr && weight != nullptr, FRX_ERR_INVALID_ARG, "frx_gemm_dhidden: null input pointer");
  int rc = check_out(d_hidden, ld_d_hidden, hidden_dim, out_dtype, "frx_gemm_dhidden");
  if (rc) return rc;
  FRX_CHECK_RANGE(dlogits, matrix_bytes(rows, vocab_shard, ld_dlogits, 2), "frx_gemm_dhidden: dlogits");
  FRX_CHECK_RANGE(weight, matrix_bytes(vocab_shard, hidden_dim, ld_weight, 2), "frx_gemm_dhidden: weight");
  FRX_CHECK_RANGE(d_hidden, matrix_bytes(rows, hidden_dim, ld_d_hidden, out_elem_bytes(out_dtype)),
                  "frx_gemm_dhidden: d_hidden");
  Operand a{dlogits, ld_dlogits, rows, vocab_shard, false, in_dtype};  // [rows, V] row-major, K = V contiguous
  Operand b{weight, ld_weight, hidden_dim, vocab_shard, true, in_dtype};  // [V, H] row-major, N = H contiguous
  return launch_gemm<false, true, true, StoreEpilogue>(a, b, rows, hidden_dim, vocab_shard, 8,
                                                 store_params(d_hidden, ld_d_hidden, rows, hidden_dim, out_dtype),
                                                 status, static_cast<cudaStream_t>(stream));
}

namespace frx {

static int gemm_dweight_impl(const void* dlogits, int64_t ld_dlogits, const void* hidden, int64_t ld_hidden,
                             int in_dtype, void* d_weight, int64_t ld_d_weight, int out_dtype, int64_t vocab_shard,
                             int64_t hidden_dim, int64_t rows, int max_sms, int* status, void* stream) {
  FRX_REQUIRE(rows >= 1 && hidden_dim >= 1 && vocab_shard >= 0 && rows < (1ll << 31) && hidden_dim < (1ll << 31) &&
                  vocab_shard < (1ll << 31),
              FRX_ERR_INVALID_ARG, "frx_gemm_dweight: bad sizes rows=%lld hidden_dim=%lld vocab_shard=%lld",
              (long long)rows, (long long)hidden_dim, (long long)vocab_shard);
  if (vocab_shard == 0) return FRX_OK;
  FRX_REQUIRE(dlogits != nullptr && hidden != nullptr, FRX_ERR_INVALID_ARG, "frx_gemm_dweight: null input pointer");
  int rc = check_out(d_weight, ld_d_weight, hidden_dim, out_dtype, "frx_gemm_dweight");
  if (rc) return rc;
  FRX_CHECK_RANGE(dlogits, matrix_bytes(rows, vocab_shard, ld_dlogits, 2), "frx_gemm_dweight: dlogits");
  FRX_CHECK_RANGE(hidden, matrix_bytes(rows, hidden_dim, ld_hidden, 2), "frx_gemm_dweight: hidden");
  FRX_CHECK_RANGE(d_weight, matrix_bytes(vocab_shard, hidden_dim, ld_d_weight, out_elem_bytes(out_dtype)),
                  "frx_gemm_dweight: d_weight");
  Operand a{dlogits, ld_dlogits, vocab_shard, rows, true, in_dtype};  // [rows, V] row-major, M = V contiguous
  Operand b{hidden, ld_hidden, hidden_dim, rows, true, in_dtype};     // [rows, H] row-major, N = H contiguous
  return launch_gemm<true, true, true, StoreEpilogue>(a, b, vocab_shard, hidden_dim, rows, 8,
                                                store_params(d_weight, ld_d_weight, vocab_shard, hidden_dim, out_dtype),
                                                status, static_cast<cudaStream_t>(stream), -1, kWaitLimitNs, max_sms);
}

}  // namespace frx

extern "C" int frx_gemm_dweight(const void* dlogits, int64_t ld_dlogits, const void* hidden, int64_t ld_hidden,
                                int in_dtype, void* d_weight, int64_t ld_d_weight, int out_dtype, int64_t vocab_shard,
                                int64_t hidden_dim, int64_t rows, int* status, void* stream) {
  return frx::gemm_dweight_impl(dlogits, ld_dlogits, hidden, ld_hidden, in_dtype, d_weight, ld_d_weight, out_dtype,
                                vocab_shard, hidden_dim, rows, 0, status, stream);
}

extern "C" int frx_gemm_dweight_sms(const void* dlogits, int64_t ld_dlogits, const void* hidden, int64_t ld_hidden,
                                    int in_dtype, void* d_weight, int64_t ld_d_weight, int out_dtype,
                                    int64_t vocab_shard, int64_t hidden_dim, int64_t rows, int max_sms, int* status,
                                    void* stream) {
  FRX_REQUIRE(max_sms >= 0, FRX_ERR_INVALID_ARG, "frx_gemm_dweight_sms: max_sms %d < 0", max_sms);
  return frx::gemm_dweight_impl(dlogits, ld_dlogits, hidden, ld_hidden, in_dtype, d_weight, ld_d_weight, out_dtype,
                                vocab_shard, hidden_dim, rows, max_sms, status, stream);
}

extern "C" int frx_gemm_dhidden_multicast(const void* dlogits, int64_t ld_dlogits, const void* weight,
                                          int64_t ld_weight, int in_dtype, void* d_hidden_mc, int64_t ld_d_hidden,
                                          int64_t rows, int64_t hidden_dim, int64_t vocab_shard, int* status,
                                          void* stream) {
  using namespace frx;
  FRX_REQUIRE(rows >= 0 && hidden_dim >= 1 && vocab_shard >= 1 && rows < (1ll << 31) && hidden_dim < (1ll << 31) &&
                  vocab_shard < (1ll << 31),
              FRX_ERR_INVALID_ARG, "frx_gemm_dhidden_multicast: bad sizes");
  if (rows == 0) return FRX_OK;
  FRX_REQUIRE(dlogits != nullptr && weight != nullptr && d_hidden_mc != nullptr, FRX_ERR_INVALID_ARG,
              "frx_gemm_dhidden_multicast: null pointer");
  FRX_REQUIRE(ld_d_hidden >= hidden_dim, FRX_ERR_INVALID_ARG, "frx_gemm_dhidden_multicast: ld_d_hidden < hidden_dim");
  MultimemAddEpilogue::Params ep;
  ep.mc_out = static_cast<float*>(d_hidden_mc);
  ep.ld_out = ld_d_hidden;
  ep.rows = static_cast<int>(rows);
  ep.cols = static_cast<int>(hidden_dim);
  FRX_REQUIRE(aligned16(d_hidden_mc) && ld_d_hidden % 4 == 0, FRX_ERR_INVALID_ARG,
              "frx_gemm_dhidden_multicast: the multicast buffer must be 16-byte aligned with ld a multiple of 4");
  FRX_CHECK_RANGE(dlogits, matrix_bytes(rows, vocab_shard, ld_dlogits, 2), "frx_gemm_dhidden_multicast: dlogits");
  FRX_CHECK_RANGE(weight, matrix_bytes(vocab_shard, hidden_dim, ld_weight, 2), "frx_gemm_dhidden_multicast: weight");
  Operand a{dlogits, ld_dlogits, rows, vocab_shard, false, in_dtype};
  Operand b{weight, ld_weight, hidden_dim, vocab_shard, true, in_dtype};
  // 256 x 256 tiles with the double-buffered TMEM accumulator: each tile's NVLink reductions run
  // while the next tile's MMAs do, instead of stalling a single-buffered 256 x 512 tile.
  return launch_gemm<false, true, false, MultimemAddEpilogue>(a, b, rows, hidden_dim, vocab_shard, 8, ep, status,
                                                              static_cast<cudaStream_t>(stream));
}
