// Forward GEMM with the cross-entropy / entropy row reduction fused into its epilogue.
//
// Each finished 128 x 256 fp32 accumulator tile is read from tensor memory by the four
// epilogue warps, one thread per row (TMEM lane == row), so the row statistics need no
// shared memory and no shuffles. Two passes over the tile's TMEM columns:
//   pass 1: tile max m (and the target logit when the row's target lies in the tile;
//           optionally the fp32 logits are streamed out to HBM here),
//   pass 2: s = sum exp(z - m) and u = sum (z - m) exp(z - m) against that exact tile max.
// The reference computes the same four numbers per (row, 256-column tile) in
// fast_reduction/gemm_ce_entropy_epilogue.py:184-271 (its third slot is sum z exp(z - m)).
// Columns at or beyond the shard's vocabulary size are skipped, not sentinel-filled. An optional
// bias (bf16 or fp16, the operands' type) is added to each column before the reductions (and
// before the logits store).
//
// Two optional logits outputs feed the training pass's dlogits kernel:
//   fp32 logits z (pass 1, 4 bytes per logit; the reference's layout), or
//   fp16 tile-relative logits z - m (pass 2, 2 bytes per logit), where m is the tile maximum the
//   same launch writes into the partials; the reader adds m back (frx_dlogits_tilerel).
#include <cstring>

#include "frx_host.cuh"

namespace frx {

// v[idx] for a runtime idx in [0, 32) as a 5-level select tree, so the array stays in
// registers (an indexed read would demote it to local memory).
__device__ __forceinline__ float select32(const float (&v)[32], int idx) {
  float w16[16], w8[8], w4[4], w2[2];
#pragma unroll
  for (int j = 0; j < 16; ++j) w16[j] = (idx & 16) ? v[j + 16] : v[j];
#pragma unroll
  for (int j = 0; j < 8; ++j) w8[j] = (idx & 8) ? w16[j + 8] : w16[j];
#pragma unroll
  for (int j = 0; j < 4; ++j) w4[j] = (idx & 4) ? w8[j + 4] : w8[j];
#pragma unroll
  for (int j = 0; j < 2; ++j) w2[j] = (idx & 2) ? w4[j + 2] : w4[j];
  return (idx & 1) ? w2[1] : w2[0];
}

// The two 16-bit values packed in `w` (low half first) as floats: bf16 or fp16.
__device__ __forceinline__ float2 unpack2(uint32_t w, bool f16) {
  if (f16) {
    __half2 h;
    memcpy(&h, &w, sizeof(h));
    return __half22float2(h);
  }
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// Two floats as one fp16x2 word (round to nearest; low half = first value, the lower column).
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  uint32_t w;
  memcpy(&w, &h, sizeof(w));
  return w;
}

// v[j] += bias[j] for the valid columns of a 32-column chunk (16-bit bias, fp32 add).
__device__ __forceinline__ void add_bias32(float (&v)[32], const uint16_t* b, int lim, bool vec, bool f16) {
  if (lim >= 32 && vec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(b) + q);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack2(u[i], f16);
        v[8 * q + 2 * i] += f.x;
        v[8 * q + 2 * i + 1] += f.y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < lim) v[j] += unpack2(b[j], f16).x;
  }
}

struct CEPartialsEpilogue {
  // Two 32 x 32 fp32 staging blocks per epilogue warp for the optional logits store.
  static constexpr int kSmemPerWarp = 2 * 32 * 32 * 4;
  static constexpr int kSmemBytes = 4 * kSmemPerWarp;

  struct Params {
    CUtensorMap tm_logits;  // fp32 [rows, vocab_shard] logits, 32 x 32 boxes, 128B swizzle
    CUtensorMap tm_rel;     // fp16 [rows, vocab_shard] tile-relative logits, 32 x 64 boxes, 128B swizzle
    const int64_t* target;
    const uint16_t* bias;  // optional [vocab_shard] bias of this shard (bf16 or fp16 bits)
    int64_t vocab_offset;
    int rows;
    int vocab_shard;
    float4* partials;
    int64_t tile_stride;
    int has_logits;
    int has_rel;
    int bias_vec;  // bias base 16-byte aligned
    int f16;       // bias is fp16 (else bf16)
    int n_tiles;   // vocabulary tiles the partials buffer holds (checked builds verify the index)
    int* status;
  };

  template <class Release>
  __device__ __forceinline__ static void run(const Params& p, uint8_t* stage, uint32_t tacc, int m_blk, int n_blk,
                                             int q, int lane, Release release) {
    // Row handled by this thread: TMEM lane (q * 32 + lane) of the tile.
    const int row0 = m_blk * kBM + q * 32;
    const int row = row0 + lane;
    const int n0 = n_blk * kBN;
    const int ncols = min(kBN, p.vocab_shard - n0);
    const bool row_ok = row < p.rows;
    int tcol = -1;
    if (row_ok && p.target != nullptr) {
      const long long lt = static_cast<long long>(p.target[row]) - p.vocab_offset - n0;
      if (lt >= 0 && lt < ncols) tcol = static_cast<int>(lt);
    }
    const uint32_t stage_base = smem_u32(stage);

    float v[32];
    float mx0 = -INFINITY, mx1 = -INFINITY, zt = 0.0f;
#pragma unroll 1
    for (int c = 0; c < kBN / 32; ++c) {
      const int lim = ncols - c * 32;  // warp-uniform
      if (lim <= 0) break;
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after per-row branches
      tmem_load_32cols(tacc + static_cast<uint32_t>(c * 32), v);
      if (p.bias != nullptr) add_bias32(v, p.bias + n0 + c * 32, lim, p.bias_vec != 0, p.f16 != 0);
      if (lim >= 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          mx0 = fmaxf(mx0, v[j]);
          mx1 = fmaxf(mx1, v[j + 1]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < lim) mx0 = fmaxf(mx0, v[j]);
      }
      if ((tcol >> 5) == c) zt = select32(v, tcol & 31);
      if (p.has_logits) {
        // Stage this warp's 32 x 32 block in shared memory (row = lane, 16-byte chunks XOR-swizzled
        // by row % 8, which is both bank-conflict free and the TMA 128B-swizzle layout) and write it
        // with one TMA store; rows / columns outside the matrix are clipped by the TMA unit.
        const int buf = c & 1;
        // The store that last used this buffer has read it. At a tile's first chunk wait for all of
        // them: the previous tile may have ended on either buffer (a ragged last vocabulary tile).
        if (lane == 0) {
          if (c == 0)
            bulk_wait_group_read<0>();
          else
            bulk_wait_group_read<1>();
        }
        __syncwarp();
        const uint32_t rowb = stage_base + static_cast<uint32_t>(buf * 4096 + lane * 128);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(rowb + static_cast<uint32_t>((j ^ (lane & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                       v[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // Evict-first: the 4 bytes per logit (2.1 GB per 4096-row chunk at V = 128256) are read
          // back only by the dlogits pass, from DRAM. At normal priority they displaced this GEMM's
          // operand tiles from L2 (ncu, rows 4096, V 128256: L2 hit rate 93% without logits, 78%
          // with them, 0.85 GB of extra operand reads per launch); evict-first gives 81% and
          // 0.62 GB. The tensor pipe stays ~90% active either way (97.5% without logits).
          tma_store_2d_hint(&p.tm_logits, stage + buf * 4096, n0 + c * 32, row0, l2_policy_evict_first());
          bulk_commit_group();
        }
      }
    }
    const float mx = fmaxf(mx0, mx1);
    // exp(z - m) as 2^((z - m) log2 e) with z - m formed first: the largest logit gets exactly 1 and
    // the error does not grow with |m| (folding m into one FMA, z log2e - m log2e, would carry the
    // rounding of m log2e, about |m| 2^-24).
    float s0 = 0.f, s1 = 0.f, u0 = 0.f, u1 = 0.f;
#pragma unroll 1
    for (int c = 0; c < kBN / 32; ++c) {
      const int lim = ncols - c * 32;
      if (lim <= 0) break;
      __syncwarp();
      tmem_load_32cols(tacc + static_cast<uint32_t>(c * 32), v);
      if (p.bias != nullptr) add_bias32(v, p.bias + n0 + c * 32, lim, p.bias_vec != 0, p.f16 != 0);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] -= mx;  // d = z - m
      if (p.has_rel) store_rel(p, stage, stage_base, v, c, lim, lane, row0, n0);
      if (lim >= 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float e0 = ex2_approx(v[j] * kLog2e);
          const float e1 = ex2_approx(v[j + 1] * kLog2e);
          s0 += e0;
          s1 += e1;
          u0 = fmaf(v[j], e0, u0);
          u1 = fmaf(v[j + 1], e1, u1);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j < lim) {
            const float e = ex2_approx(v[j] * kLog2e);
            s0 += e;
            u0 = fmaf(v[j], e, u0);
          }
        }
      }
    }
    release();  // accumulator buffer may now be overwritten by the next tile's MMAs
    if (row_ok && device_check(n_blk < p.n_tiles, p.status))
      p.partials[static_cast<int64_t>(n_blk) * p.tile_stride + row] = make_float4(mx, s0 + s1, u0 + u1, zt);
  }

  // Called once per epilogue warp after its last tile: outstanding logits stores must finish
  // before the CTA (and its staging shared memory) goes away.
  __device__ __forceinline__ static void finish(const Params& p, int lane) {
    if ((p.has_logits || p.has_rel) && lane == 0) bulk_wait_all();
  }

  // Pass-2 store of the tile-relative logits d = z - m of 32-column chunk c (this thread's row =
  // lane): packed to fp16 into one half of a 32 x 64 staging block (row = lane, 128 bytes per row,
  // 16-byte chunks XOR-swizzled by row % 8: bank-conflict free and the TMA 128B-swizzle layout);
  // each completed 64-column block (or the tile's last, partial one) leaves with one TMA store.
  // Columns past the shard's vocabulary are clipped by the TMA unit.
  __device__ __forceinline__ static void store_rel(const Params& p, uint8_t* stage, uint32_t stage_base,
                                                   const float (&v)[32], int c, int lim, int lane, int row0, int n0) {
    const int blk = c >> 1;
    const int buf = blk & 1;
    if ((c & 1) == 0) {
      // The store that last used this buffer has read it (at a tile's first block: every store,
      // since the previous tile may have ended on either buffer).
      if (lane == 0) {
        if (blk == 0)
          bulk_wait_group_read<0>();
        else
          bulk_wait_group_read<1>();
      }
      __syncwarp();
    }
    const uint32_t rowb = stage_base + static_cast<uint32_t>(buf * 4096 + lane * 128);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t w0 = pack_half2(v[8 * k], v[8 * k + 1]);
      const uint32_t w1 = pack_half2(v[8 * k + 2], v[8 * k + 3]);
      const uint32_t w2 = pack_half2(v[8 * k + 4], v[8 * k + 5]);
      const uint32_t w3 = pack_half2(v[8 * k + 6], v[8 * k + 7]);
      st_shared_v4_u32(rowb + static_cast<uint32_t>((((c & 1) * 4 + k) ^ (lane & 7)) << 4), w0, w1, w2, w3);
    }
    if ((c & 1) == 1 || lim <= 32) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        // Evict-first, as for the fp32 logits: the dlogits pass reads them back from DRAM.
        tma_store_2d_hint(&p.tm_rel, stage + buf * 4096, n0 + 64 * blk, row0, l2_policy_evict_first());
        bulk_commit_group();
      }
    }
  }
};

}  // namespace frx

namespace frx {

static int fwd_partials_impl(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight, int dtype,
                             const void* bias, const int64_t* target, int64_t rows, int64_t vocab_shard,
                             int64_t hidden_dim, int64_t vocab_offset, float* partials, int64_t tile_stride,
                             float* logits, int64_t ld_logits, void* zrel, int64_t ld_zrel, int* status, void* stream,
                             int stall_kb, uint64_t wait_limit_ns) {
  FRX_REQUIRE(rows >= 0 && vocab_shard >= 1 && hidden_dim >= 1, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: bad sizes rows=%lld vocab_shard=%lld hidden_dim=%lld", (long long)rows,
              (long long)vocab_shard, (long long)hidden_dim);
  FRX_REQUIRE(rows < (1ll << 31) && vocab_shard < (1ll << 31) && hidden_dim < (1ll << 31), FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: sizes must be below 2^31");
  if (rows == 0) return FRX_OK;
  FRX_REQUIRE(hidden != nullptr && weight != nullptr && partials != nullptr, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: null hidden/weight/partials pointer");
  FRX_REQUIRE(hidden_dim % 8 == 0, FRX_ERR_UNSUPPORTED, "frx_fwd_partials: hidden_dim %lld must be a multiple of 8",
              (long long)hidden_dim);
  FRX_REQUIRE(is_gemm_dtype(dtype), FRX_ERR_UNSUPPORTED,
              "frx_fwd_partials: dtype %d must be FRX_DTYPE_BF16 or FRX_DTYPE_F16", dtype);
  FRX_REQUIRE(tile_stride >= rows, FRX_ERR_INVALID_ARG, "frx_fwd_partials: tile_stride %lld < rows %lld",
              (long long)tile_stride, (long long)rows);
  FRX_REQUIRE((reinterpret_cast<uintptr_t>(partials) & 15u) == 0, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: partials must be 16-byte aligned");
  FRX_REQUIRE(logits == nullptr || ld_logits >= vocab_shard, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: ld_logits %lld < vocab_shard %lld", (long long)ld_logits, (long long)vocab_shard);
  FRX_REQUIRE(logits == nullptr || (ld_logits % 4 == 0 && aligned16(logits)), FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: logits must be 16-byte aligned with ld_logits a multiple of 4 (got %lld)",
              (long long)ld_logits);
  FRX_REQUIRE(logits == nullptr || zrel == nullptr, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials: at most one of fp32 logits and tile-relative logits per launch");
  FRX_REQUIRE(zrel == nullptr || ld_zrel >= vocab_shard, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials_tilerel: ld_logits_rel %lld < vocab_shard %lld", (long long)ld_zrel,
              (long long)vocab_shard);
  FRX_REQUIRE(zrel == nullptr || (ld_zrel % 8 == 0 && aligned16(zrel)), FRX_ERR_INVALID_ARG,
              "frx_fwd_partials_tilerel: logits_rel must be 16-byte aligned with ld_logits_rel a multiple of 8 "
              "(got %lld)", (long long)ld_zrel);
  const int64_t n_tiles = (vocab_shard + kBN - 1) / kBN;
  [[maybe_unused]] const int64_t esz = 2;
  FRX_CHECK_RANGE(hidden, matrix_bytes(rows, hidden_dim, ld_hidden, esz), "frx_fwd_partials: hidden");
  FRX_CHECK_RANGE(weight, matrix_bytes(vocab_shard, hidden_dim, ld_weight, esz), "frx_fwd_partials: weight");
  FRX_CHECK_RANGE(bias, vocab_shard * esz, "frx_fwd_partials: bias");
  FRX_CHECK_RANGE(target, rows * 8, "frx_fwd_partials: target");
  FRX_CHECK_RANGE(partials, matrix_bytes(n_tiles, rows, tile_stride, 16), "frx_fwd_partials: partials");
  // The TMA stores write whole 16-byte chunks: each row's pad columns up to the next 16-byte boundary.
  FRX_CHECK_RANGE(logits, matrix_bytes(rows, (vocab_shard + 3) / 4 * 4, ld_logits, 4), "frx_fwd_partials: logits");
  FRX_CHECK_RANGE(zrel, matrix_bytes(rows, (vocab_shard + 7) / 8 * 8, ld_zrel, 2),
                  "frx_fwd_partials_tilerel: logits_rel");
  CEPartialsEpilogue::Params ep;
  memset(&ep, 0, sizeof(ep));
  ep.n_tiles = static_cast<int>(n_tiles);
  ep.status = status;
  if (logits != nullptr) {
    const int rc = encode_f32_2d(&ep.tm_logits, logits, rows, vocab_shard, ld_logits, 32, 32);
    if (rc) return rc;
    ep.has_logits = 1;
  }
  if (zrel != nullptr) {
    const int rc = encode_16bit_2d(&ep.tm_rel, true, zrel, rows, vocab_shard, ld_zrel, 32, 64);
    if (rc) return rc;
    ep.has_rel = 1;
  }
  ep.target = target;
  ep.bias = static_cast<const uint16_t*>(bias);
  ep.bias_vec = aligned16(bias) ? 1 : 0;
  ep.f16 = dtype == FRX_DTYPE_F16 ? 1 : 0;
  ep.vocab_offset = vocab_offset;
  ep.rows = static_cast<int>(rows);
  ep.vocab_shard = static_cast<int>(vocab_shard);
  ep.partials = reinterpret_cast<float4*>(partials);
  ep.tile_stride = tile_stride;
  Operand a{hidden, ld_hidden, rows, hidden_dim, false, dtype};
  Operand b{weight, ld_weight, vocab_shard, hidden_dim, false, dtype};
  // A band of up to 32 row blocks (4096 rows, 32 MiB of bf16 hidden at H=4096) stays in L2
  // while the CTAs sweep the vocabulary. Measured on one B200 at vocabulary shards of 16032 to
  // 128256 rows: 4096-row bands beat 8192- and 16384-row bands everywhere (e.g. 2.64 / 2.93 /
  // 3.25 ms over 32768 rows at 16032), and 2048-row bands lose at 128256.
  // FRX_FWD_GROUP_M (tuning only) overrides the band height in 128-row blocks.
  static const int group_m = env_int("FRX_FWD_GROUP_M", 32);
  return launch_gemm<false, false, false, CEPartialsEpilogue>(a, b, rows, vocab_shard, hidden_dim, group_m, ep, status,
                                                              static_cast<cudaStream_t>(stream), stall_kb,
                                                              wait_limit_ns);
}

}  // namespace frx

extern "C" int frx_fwd_partials(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight,
                                int dtype, const void* bias, const int64_t* target, int64_t rows, int64_t vocab_shard,
                                int64_t hidden_dim, int64_t vocab_offset, float* partials, int64_t tile_stride,
                                float* logits, int64_t ld_logits, int* status, void* stream) {
  return frx::fwd_partials_impl(hidden, ld_hidden, weight, ld_weight, dtype, bias, target, rows, vocab_shard,
                                hidden_dim, vocab_offset, partials, tile_stride, logits, ld_logits, nullptr, 0, status,
                                stream, -1, frx::kWaitLimitNs);
}

extern "C" int frx_fwd_partials_tilerel(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight,
                                        int dtype, const void* bias, const int64_t* target, int64_t rows,
                                        int64_t vocab_shard, int64_t hidden_dim, int64_t vocab_offset, float* partials,
                                        int64_t tile_stride, void* logits_rel, int64_t ld_logits_rel, int* status,
                                        void* stream) {
  FRX_REQUIRE(rows == 0 || logits_rel != nullptr, FRX_ERR_INVALID_ARG,
              "frx_fwd_partials_tilerel: null logits_rel pointer");
  return frx::fwd_partials_impl(hidden, ld_hidden, weight, ld_weight, dtype, bias, target, rows, vocab_shard,
                                hidden_dim, vocab_offset, partials, tile_stride, nullptr, 0, logits_rel, ld_logits_rel,
                                status, stream, -1, frx::kWaitLimitNs);
}

extern "C" int frx_test_stalled_fwd(const void* hidden, int64_t ld_hidden, const void* weight, int64_t ld_weight,
                                    const int64_t* target, int64_t rows, int64_t vocab_shard, int64_t hidden_dim,
                                    float* partials, int64_t tile_stride, int stall_kb, int64_t wait_limit_us,
                                    int* status, void* stream) {
  using namespace frx;
  FRX_REQUIRE(stall_kb >= 0 && wait_limit_us >= 1 && wait_limit_us <= 1000000, FRX_ERR_INVALID_ARG,
              "frx_test_stalled_fwd: need stall_kb >= 0 and 1 <= wait_limit_us <= 1e6");
  FRX_REQUIRE(stall_kb * 128 < hidden_dim, FRX_ERR_INVALID_ARG,
              "frx_test_stalled_fwd: stall_kb %d is past the last k-block of hidden_dim %lld", stall_kb,
              (long long)hidden_dim);
  return fwd_partials_impl(hidden, ld_hidden, weight, ld_weight, FRX_DTYPE_BF16, nullptr, target, rows, vocab_shard,
                           hidden_dim, 0, partials, tile_stride, nullptr, 0, nullptr, 0, status, stream, stall_kb,
                           static_cast<uint64_t>(wait_limit_us) * 1000ull);
}
