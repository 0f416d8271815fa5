/*
 * A plain C caller of libfrx.so (no Python, no torch in the process): the training pass of the
 * fused linear + cross-entropy + entropy head through the C ABI of include/frx.h, checked against a
 * double-precision computation on the host.
 *
 * It runs the same sequence the reference's megakernel runs per chunk
 * (fast_reduction/gemm_kernel.py:823-871): the forward GEMM-epilogue with fp32 logits out
 * (frx_fwd_partials), the merge into ce / entropy / lse (frx_finalize), dlogits in bf16
 * (frx_dlogits), then d_hidden = dlogits @ W and d_weight = dlogits^T @ X (frx_gemm_dhidden,
 * frx_gemm_dweight), with ce_weight 1 and ent_weight -1, a ragged last vocabulary tile and some
 * rows ignored (target -100). Exit status 0 and a final "ok" line mean every check passed.
 *
 * Build: gcc -std=c11 -O2 -I include -I $CUDA/include frx_c_caller.c -L <dir of libfrx.so> -lfrx
 *        -L $CUDA/lib64 -lcudart -lm
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "frx.h"

#define CUDA_OK(x)                                                                              \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) {                                                                    \
      fprintf(stderr, "%s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e_));               \
      return 2;                                                                                 \
    }                                                                                           \
  } while (0)

#define FRX_CALL(x)                                                                             \
  do {                                                                                          \
    int rc_ = (x);                                                                              \
    if (rc_ != FRX_OK) {                                                                        \
      fprintf(stderr, "%s:%d: libfrx error %d: %s\n", __FILE__, __LINE__, rc_, frx_last_error()); \
      return 3;                                                                                 \
    }                                                                                           \
  } while (0)

enum { B = 300, H = 256, V = 1000, IGNORE = -100 };

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;

static double uniform01(void) { /* xorshift64 */
  rng_state ^= rng_state << 13;
  rng_state ^= rng_state >> 7;
  rng_state ^= rng_state << 17;
  return (double)(rng_state >> 11) * (1.0 / 9007199254740992.0);
}

static double normal01(void) { /* Box-Muller */
  double u1 = uniform01(), u2 = uniform01();
  if (u1 < 1e-300) u1 = 1e-300;
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static uint16_t to_bf16(float f) { /* round to nearest even (finite inputs) */
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static double from_bf16(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static int n_bad = 0;

static void check(const char* what, int64_t i, double got, double want, double tol) {
  if (!(fabs(got - want) <= tol)) {
    if (n_bad < 10) fprintf(stderr, "%s[%lld]: got %.9g want %.9g (tol %.3g)\n", what, (long long)i, got, want, tol);
    ++n_bad;
  }
}

int main(void) {
  if (frx_abi_version() != FRX_ABI_VERSION) {
    fprintf(stderr, "ABI version %d, header %d\n", frx_abi_version(), FRX_ABI_VERSION);
    return 4;
  }
  const int64_t T = (V + FRX_VOCAB_TILE - 1) / FRX_VOCAB_TILE;
  uint16_t* h_x = malloc(sizeof(uint16_t) * B * H);
  uint16_t* h_w = malloc(sizeof(uint16_t) * V * H);
  int64_t* h_t = malloc(sizeof(int64_t) * B);
  for (int64_t i = 0; i < (int64_t)B * H; ++i) h_x[i] = to_bf16((float)normal01());
  for (int64_t i = 0; i < (int64_t)V * H; ++i) h_w[i] = to_bf16((float)(0.15 * normal01()));
  for (int64_t r = 0; r < B; ++r) {
    if (r % 17 == 5) h_t[r] = IGNORE;
    else if (r % 11 == 3) h_t[r] = V - 1 - (r % 232); /* inside the ragged last tile (232 columns) */
    else h_t[r] = (int64_t)(uniform01() * V) % V;
  }

  void *d_x, *d_w, *d_dz;
  int64_t* d_t;
  float *d_part, *d_logits, *d_ce, *d_ent, *d_lse, *d_dh, *d_dw;
  int* d_status;
  cudaStream_t stream;
  CUDA_OK(cudaStreamCreate(&stream));
  CUDA_OK(cudaMalloc(&d_x, sizeof(uint16_t) * B * H));
  CUDA_OK(cudaMalloc(&d_w, sizeof(uint16_t) * V * H));
  CUDA_OK(cudaMalloc((void**)&d_t, sizeof(int64_t) * B));
  CUDA_OK(cudaMalloc((void**)&d_part, sizeof(float) * 4 * T * B));
  CUDA_OK(cudaMalloc((void**)&d_logits, sizeof(float) * B * V));
  CUDA_OK(cudaMalloc((void**)&d_ce, sizeof(float) * B));
  CUDA_OK(cudaMalloc((void**)&d_ent, sizeof(float) * B));
  CUDA_OK(cudaMalloc((void**)&d_lse, sizeof(float) * B));
  CUDA_OK(cudaMalloc(&d_dz, sizeof(uint16_t) * B * V));
  CUDA_OK(cudaMalloc((void**)&d_dh, sizeof(float) * B * H));
  CUDA_OK(cudaMalloc((void**)&d_dw, sizeof(float) * V * H));
  CUDA_OK(cudaMalloc((void**)&d_status, sizeof(int)));
  CUDA_OK(cudaMemcpyAsync(d_x, h_x, sizeof(uint16_t) * B * H, cudaMemcpyHostToDevice, stream));
  CUDA_OK(cudaMemcpyAsync(d_w, h_w, sizeof(uint16_t) * V * H, cudaMemcpyHostToDevice, stream));
  CUDA_OK(cudaMemcpyAsync(d_t, h_t, sizeof(int64_t) * B, cudaMemcpyHostToDevice, stream));
  CUDA_OK(cudaMemsetAsync(d_status, 0, sizeof(int), stream));

  /* V = 1000 is a multiple of 8, so every row stride below is the matrix width */
  FRX_CALL(frx_fwd_partials(d_x, H, d_w, H, FRX_DTYPE_BF16, NULL, d_t, B, V, H, 0, d_part, B, d_logits, V,
                            d_status, stream));
  FRX_CALL(frx_finalize(d_part, T, B, B, 0, d_t, V, IGNORE, d_ce, d_ent, d_lse, NULL, NULL, d_status, stream));
  FRX_CALL(frx_dlogits(d_logits, V, d_t, d_lse, d_ent, NULL, NULL, 1.0f, -1.0f, d_dz, V, FRX_DTYPE_BF16, B, V, 0,
                       IGNORE, stream));
  FRX_CALL(frx_gemm_dhidden(d_dz, V, d_w, H, FRX_DTYPE_BF16, d_dh, H, FRX_DTYPE_F32, B, H, V, d_status, stream));
  FRX_CALL(frx_gemm_dweight(d_dz, V, d_x, H, FRX_DTYPE_BF16, d_dw, H, FRX_DTYPE_F32, V, H, B, d_status, stream));

  float* g_logits = malloc(sizeof(float) * B * V);
  float *g_ce = malloc(sizeof(float) * B), *g_ent = malloc(sizeof(float) * B), *g_lse = malloc(sizeof(float) * B);
  uint16_t* g_dz = malloc(sizeof(uint16_t) * B * V);
  float* g_dh = malloc(sizeof(float) * B * H);
  float* g_dw = malloc(sizeof(float) * V * H);
  int g_status = -1;
  CUDA_OK(cudaMemcpyAsync(g_logits, d_logits, sizeof(float) * B * V, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(g_ce, d_ce, sizeof(float) * B, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(g_ent, d_ent, sizeof(float) * B, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(g_lse, d_lse, sizeof(float) * B, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(g_dz, d_dz, sizeof(uint16_t) * B * V, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(g_dh, d_dh, sizeof(float) * B * H, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(g_dw, d_dw, sizeof(float) * V * H, cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaMemcpyAsync(&g_status, d_status, sizeof(int), cudaMemcpyDeviceToHost, stream));
  CUDA_OK(cudaStreamSynchronize(stream));
  if (g_status != 0) {
    fprintf(stderr, "device status bits 0x%x\n", g_status);
    return 5;
  }

  /* host reference in double over the same bf16 inputs */
  double* z = malloc(sizeof(double) * V);
  double* dz = malloc(sizeof(double) * V);
  double max_dz_rel = 0.0;
  for (int64_t r = 0; r < B; ++r) {
    double m = -INFINITY;
    for (int64_t j = 0; j < V; ++j) {
      double acc = 0.0;
      for (int64_t k = 0; k < H; ++k) acc += from_bf16(h_x[r * H + k]) * from_bf16(h_w[j * H + k]);
      z[j] = acc;
      if (acc > m) m = acc;
      check("logits", r * V + j, g_logits[r * V + j], acc, 1e-4 + 1e-5 * fabs(acc));
    }
    double s = 0.0, u = 0.0;
    for (int64_t j = 0; j < V; ++j) {
      double e = exp(z[j] - m);
      s += e;
      u += (z[j] - m) * e;
    }
    double lse = m + log(s), ent = log(s) - u / s;
    double ce = h_t[r] == IGNORE ? 0.0 : lse - z[h_t[r]];
    check("lse", r, g_lse[r], lse, 1e-4 + 1e-5 * fabs(lse));
    check("entropy", r, g_ent[r], ent, 1e-4 + 1e-5 * fabs(ent));
    check("ce", r, g_ce[r], ce, 1e-4 + 1e-5 * fabs(ce));
    /* dz = p (g_ce + (log p + H)) - g_ce [j == t] with ent_weight -1; g_ce = 1, or 0 on an ignored
       row, which (nll_loss semantics) drops the whole CE term and keeps the entropy term */
    const double g_ce = h_t[r] == IGNORE ? 0.0 : 1.0;
    for (int64_t j = 0; j < V; ++j) {
      double lp = z[j] - lse, p = exp(lp);
      dz[j] = p * (g_ce + (lp + ent)) - (j == h_t[r] ? g_ce : 0.0);
      double got = from_bf16(g_dz[r * V + j]);
      /* bf16 keeps 8 significant bits (half an ulp is 2^-9 relative); the fp32 logits and lse add
         ~1e-6 absolute to log p, i.e. ~1e-6 p to dz, which dominates where 1 + log p + H cancels */
      check("dlogits", r * V + j, got, dz[j], 4.0e-3 * fabs(dz[j]) + 1e-5 * p + 1e-7);
      if (fabs(dz[j]) > 1e-3) {
        double rel = fabs(got - dz[j]) / fabs(dz[j]);
        if (rel > max_dz_rel) max_dz_rel = rel;
      }
    }
  }
  /* the backward GEMMs against the device's own bf16 dlogits: only the fp32 accumulation differs
     (bounded by a multiple of the sum of |terms|; a wrong tile or stride errs by O(sum |terms|)) */
  for (int64_t r = 0; r < B; ++r)
    for (int64_t k = 0; k < H; ++k) {
      double acc = 0.0, mag = 0.0;
      for (int64_t j = 0; j < V; ++j) {
        double t = from_bf16(g_dz[r * V + j]) * from_bf16(h_w[j * H + k]);
        acc += t;
        mag += fabs(t);
      }
      check("d_hidden", r * H + k, g_dh[r * H + k], acc, 1e-4 * mag + 1e-7);
    }
  for (int64_t j = 0; j < V; ++j)
    for (int64_t k = 0; k < H; ++k) {
      double acc = 0.0, mag = 0.0;
      for (int64_t r = 0; r < B; ++r) {
        double t = from_bf16(g_dz[r * V + j]) * from_bf16(h_x[r * H + k]);
        acc += t;
        mag += fabs(t);
      }
      check("d_weight", j * H + k, g_dw[j * H + k], acc, 1e-4 * mag + 1e-7);
    }

  cudaFree(d_x); cudaFree(d_w); cudaFree(d_t); cudaFree(d_part); cudaFree(d_logits); cudaFree(d_ce);
  cudaFree(d_ent); cudaFree(d_lse); cudaFree(d_dz); cudaFree(d_dh); cudaFree(d_dw); cudaFree(d_status);
  cudaStreamDestroy(stream);
  if (n_bad) {
    fprintf(stderr, "%d mismatches\n", n_bad);
    return 1;
  }
  printf("frx C caller ok: B=%d H=%d V=%d, %lld vocabulary tiles, max dlogits rel err %.2e\n", B, H, V,
         (long long)T, max_dz_rel);
  return 0;
}
