/* CPU restatement of the CB3 expert layer in C with OpenMP: TEST INFRASTRUCTURE and the timed CPU baseline.
 *
 * Never linked into the product: only tests/ (checked against the NumPy oracle) and bench.py's CPU-baseline legs
 * load it. It computes what the NumPy oracle computes (oracle/moe.py), in fp32 instead of fp64:
 *   cb3 matvec        moe_matvec_ref, pallas_moe.py:310-323: W[r, j] = cb[r, q(r, j)] (exact bf16), f32 sums
 *   layer             ResidentFetch._apply_kernel, resident.py:110-120: per (token, slot) gate/up matvec,
 *                     swiglu_clamped (model.py:119-122), down matvec, routing-weighted sum over the k slots;
 *                     every slot recomputes its expert, as the reference's per-slot kernel does
 *   shared expert     mlp_partial (model.py:125-127) with W = bf16(f32(q) * s) (quant8.py:91-99)
 * Paths are relative to launcher/glm53-flash/engine/glm53/ in the reference repository.
 * Build: make -C oracle  (-> oracle/libcbmoe_cpu.so).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* float -> bf16 bits, round to nearest even (finite inputs) */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline uint32_t cb3_index(const uint32_t* row, int j) {
  const int bit = 3 * j, w = bit >> 5, off = bit & 31;
  uint32_t v = row[w] >> off;
  if (off > 29) v |= row[w + 1] << (32 - off);
  return v & 7u;
}

/* y[r] = sum_j cb[r, q(r, j)] * x[j] for rows [r0, r1) of one CB3 matrix [rows, K]. */
static void cb3_rows(const uint32_t* idx, const uint16_t* cb, int K, const float* x, float* y, int r0, int r1) {
  const int wpr = K * 3 / 32;
  for (int r = r0; r < r1; ++r) {
    const uint32_t* row = idx + (size_t)r * wpr;
    float lut[8];
    for (int v = 0; v < 8; ++v) lut[v] = bf16_to_f32(cb[(size_t)r * 8 + v]);
    float acc = 0.f;
    /* 32 indices = 3 words */
    for (int m = 0; m < wpr; m += 3) {
      const uint64_t lo = (uint64_t)row[m] | ((uint64_t)row[m + 1] << 32);
      const uint32_t hi = row[m + 2];
      const float* xs = x + (size_t)(m / 3) * 32;
      for (int i = 0; i < 21; ++i) acc += lut[(lo >> (3 * i)) & 7u] * xs[i];
      const uint32_t mid = (uint32_t)(lo >> 63) | (hi << 1);       /* index 21: bits 63, 64, 65 */
      acc += lut[mid & 7u] * xs[21];
      for (int i = 22; i < 32; ++i) acc += lut[(hi >> (3 * i - 64)) & 7u] * xs[i];
    }
    y[r] = acc;
  }
}

void cbmoe_cpu_cb3_matvec(const uint32_t* idx, const uint16_t* cb, int rows, int K, const float* x, int N,
                          float* y, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
  for (int n = 0; n < N; ++n) {
#pragma omp parallel for schedule(static)
    for (int r0 = 0; r0 < rows; r0 += 16) {
      const int r1 = r0 + 16 < rows ? r0 + 16 : rows;
      cb3_rows(idx, cb, K, x + (size_t)n * K, y + (size_t)n * rows, r0, r1);
    }
  }
}

static inline float swiglu(float g, float u, float limit) {
  g = g < limit ? g : limit;
  u = u < -limit ? -limit : (u > limit ? limit : u);
  return g / (1.f + expf(-g)) * u;
}

/* y[o] = sum_i x[i] * bf16(q[i, o] * s) for a [in, out] int8 leaf; scale_axis 1: s[o], 0: s[i]. */
static void q8_cols(const int8_t* q, const float* s, int scale_axis, int n_in, int n_out, const float* x, float* y,
                    int o0, int o1) {
  for (int o = o0; o < o1; ++o) y[o] = 0.f;
  for (int i = 0; i < n_in; ++i) {
    const float xi = x[i];
    const int8_t* qr = q + (size_t)i * n_out;
    for (int o = o0; o < o1; ++o) {
      const float sc = scale_axis == 1 ? s[o] : s[i];
      y[o] += xi * bf16_to_f32(f32_to_bf16((float)qr[o] * sc));
    }
  }
}

static void q8_matvec(const int8_t* q, const float* s, int scale_axis, int n_in, int n_out, const float* x,
                      float* y) {
#pragma omp parallel for schedule(static)
  for (int o0 = 0; o0 < n_out; o0 += 64) {
    const int o1 = o0 + 64 < n_out ? o0 + 64 : n_out;
    q8_cols(q, s, scale_axis, n_in, n_out, x, y, o0, o1);
  }
}

static void cb3_matvec_par(const uint32_t* idx, const uint16_t* cb, int rows, int K, const float* x, float* y) {
#pragma omp parallel for schedule(static)
  for (int r0 = 0; r0 < rows; r0 += 16) {
    const int r1 = r0 + 16 < rows ? r0 + 16 : rows;
    cb3_rows(idx, cb, K, x, y, r0, r1);
  }
}

/* The layer for N tokens: routed experts (per slot) + optional int8 shared expert -> out f32 [N, H].
 * Expert tables in the CB3 format: gate/up idx [E, I, H*3/32], cb [E, I, 8]; down idx [E, H, I*3/32], cb [E, H, 8].
 * Shared leaves (may be NULL): gate/up q [H, I] int8, down q [I, H] int8. */
int cbmoe_cpu_moe_layer(int E, int H, int I, const uint32_t* gi, const uint16_t* gc, const uint32_t* ui,
                        const uint16_t* uc, const uint32_t* di, const uint16_t* dc, const int8_t* sgq,
                        const float* sgs, const int8_t* suq, const float* sus, const int8_t* sdq, const float* sds,
                        int scale_axis, const float* x, int N, const int32_t* idx, const float* w, int k,
                        float limit, float* out, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
  float* g = (float*)malloc(sizeof(float) * I);
  float* u = (float*)malloc(sizeof(float) * I);
  float* y = (float*)malloc(sizeof(float) * H);
  if (!g || !u || !y) return -1;
  const size_t gu_w = (size_t)I * (H * 3 / 32), dn_w = (size_t)H * (I * 3 / 32);
  for (int n = 0; n < N; ++n) {
    const float* xn = x + (size_t)n * H;
    float* on = out + (size_t)n * H;
    for (int r = 0; r < H; ++r) on[r] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int e = idx[n * k + j];
      if (e < 0 || e >= E) continue;
      cb3_matvec_par(gi + e * gu_w, gc + (size_t)e * I * 8, I, H, xn, g);
      cb3_matvec_par(ui + e * gu_w, uc + (size_t)e * I * 8, I, H, xn, u);
      for (int i = 0; i < I; ++i) g[i] = swiglu(g[i], u[i], limit);
      cb3_matvec_par(di + e * dn_w, dc + (size_t)e * H * 8, H, I, g, y);
      const float wt = w[n * k + j];
      for (int r = 0; r < H; ++r) on[r] += wt * y[r];
    }
    if (sgq) {
      q8_matvec(sgq, sgs, scale_axis, H, I, xn, g);
      q8_matvec(suq, sus, scale_axis, H, I, xn, u);
      for (int i = 0; i < I; ++i) g[i] = swiglu(g[i], u[i], limit);
      q8_matvec(sdq, sds, scale_axis, I, H, g, y);
      for (int r = 0; r < H; ++r) on[r] += y[r];
    }
  }
  free(g);
  free(u);
  free(y);
  return 0;
}

int cbmoe_cpu_max_threads(void) { return omp_get_max_threads(); }
