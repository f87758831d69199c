// The reference's IQ2_S and IQ3_S expert tables on the int8 tensor cores: the load-time transcode into the IQ8
// layout (iq8lane.cuh), the activations split into X8 digits in the order the kernels' B fragments want, and the
// expert matvec over a routing plan's passes.
//
// Counterpart of the reference's moe_matvec on its GGUF planes (pallas_moe.py:238-307 with the dequant of
// iqquant.py:108-134): the same weights, exactly (d * k * v), multiplied against the activations' X8 digits with
// exact int32 sums per group, the group factor k applied to each group's int32 partial and d once per 256-weight
// block. One warp per (pass, 16 weight rows), four per CTA (a 64-row block), a persistent grid over the items; each
// stage's codes, group factors and block scales are loaded one stage ahead (coalesced 16-byte loads, lane-major
// units), the B fragments from the pass's X8 rows (L1/L2: every warp of the pass reads them).
#include "iq8lane.cuh"
#include "layer.cuh"
#include "layout.cuh"
#include "profile.cuh"

namespace cbmoe {

namespace {

// ------------------------------------------------------------------------------------------------- transcode
template <int T>
__global__ void iq8_units_kernel(const uint8_t* __restrict__ raw, const float* __restrict__ table, int E, int rows,
                                 int KS, uint32_t* __restrict__ units, int* __restrict__ bad) {
  constexpr int BB = IqFmt<T>::kBytes, LW = Iq8Fmt<T>::kLaneWords;
  const int RB = rows / kRowsPerBlock;
  const long long n_warps = (long long)E * RB * KS * 4;
  const int lane = threadIdx.x & 31;
  const long long stride = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long wi = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < n_warps; wi += stride) {
    long long r = wi;
    const int w = (int)(r % 4);
    r /= 4;
    const int ks = (int)(r % KS);
    r /= KS;
    const int rb = (int)(r % RB);
    const int e = (int)(r / RB);
    const int row_g = rb * kRowsPerBlock + w * kRowsPerWarp + (lane >> 2);
    const uint8_t* bg = raw + (((size_t)e * rows + row_g) * KS + ks) * BB;
    const uint8_t* bh = bg + (size_t)8 * KS * BB;
    uint32_t words[LW];
    const bool ok = iq8_lane_words<T>(bg, bh, table, lane, words);
    uint4* dst = reinterpret_cast<uint4*>(units + ((size_t)wi * 32 + lane) * LW);
#pragma unroll
    for (int i = 0; i < LW / 4; ++i)
      dst[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
    if (!ok) atomicOr(bad, 1);
  }
}

template <int T>
__global__ void iq8_scales_kernel(const uint8_t* __restrict__ raw, long long n_blocks, uint8_t* __restrict__ groups,
                                  float* __restrict__ scales) {
  constexpr int BB = IqFmt<T>::kBytes, NG = Iq8Fmt<T>::kGroups;
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks;
       b += (long long)gridDim.x * blockDim.x) {
    const uint8_t* blk = raw + (size_t)b * BB;
#pragma unroll
    for (int m = 0; m < NG; ++m) groups[(size_t)b * NG + m] = (uint8_t)iq8_group_factor<T>(blk, m);
    scales[b] = iq8_block_scale<T>(blk);
  }
}

// ------------------------------------------------------------------------------------------- X8 activations
// One CTA per row: X = rint(v 2^t) with the row's largest |X| in [2^13, 2^14), digits d1 = (X + 128) >> 8 and
// d0 = X - 256 d1, factor 2^-t; stored per stage as [chunk 4][digit 2][64], storage byte s of a chunk's plane
// holding input iq8_perm<T>(s). Rows without a finite maximum (padding rows of the routing plan) get factor 1 and
// clamped digits; no pass reads them.
// IN: 0 = bf16 rows x, 1 = f32 rows x, 2 = swiglu_clamped(x, u, limit) of f32 rows x (gate) and u (up).
template <int T, int IN>
__global__ void __launch_bounds__(256) iq8_split_kernel(const void* __restrict__ x, const float* __restrict__ u,
                                                        float limit, int R, int K, uint8_t* __restrict__ x8,
                                                        float* __restrict__ scale) {
  __shared__ float red[8];
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    auto val = [&](int i) -> float {
      if constexpr (IN == 1) return static_cast<const float*>(x)[(size_t)r * K + i];
      else if constexpr (IN == 2)
        return swiglu_clamped(static_cast<const float*>(x)[(size_t)r * K + i], u[(size_t)r * K + i], limit);
      else return __uint_as_float((uint32_t)static_cast<const uint16_t*>(x)[(size_t)r * K + i] << 16);
    };
    float mx = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(val(i)));
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();   // red is reused by the next row
    const int sh = shift_for(mx, 14);
    uint8_t* out = x8 + (size_t)r * K * 2;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
      const int stage = i >> 8, c = (i >> 6) & 3, s = i & 63;
      const float v = val(stage * 256 + c * 64 + iq8_perm<T>(s));
      int X = __float2int_rn(ldexpf(v, sh));
      X = X > 32639 ? 32639 : (X < -32768 ? -32768 : X);
      const int d1 = (X + 128) >> 8, d0 = X - 256 * d1;
      uint8_t* o = out + stage * kX8StageBytes + c * 128 + s;
      o[0] = (uint8_t)d0;
      o[64] = (uint8_t)d1;
    }
    if (threadIdx.x == 0) scale[r] = ldexpf(1.f, -sh);
  }
}

// ------------------------------------------------------------------------------------------------- matvec
struct Iq8Params {
  const uint32_t* units;
  const uint8_t* groups;
  const float* scales;
  int rows, K, E;
  const int* pass_expert;
  const int* pass_row0;
  const int* pass_cnt;
  const int* n_pass;
  const int* tok_row;        // sorted row -> X8 row (nullptr: the sorted row itself)
  const uint8_t* x8;         // X8 rows in this format's storage order
  const float* x8_scale;     // per X8 row
  float* out;                // f32 [sorted row][rows]
};

constexpr int kIq8Tiles = 2;   // token tiles of 4: passes of up to 8 tokens

__device__ __forceinline__ void mma_i8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ uint32_t word_of(const uint4& q, int i) {
  return i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
}

template <int T>
struct Iq8Stage {
  uint32_t w[Iq8Fmt<T>::kLaneWords];
  uint32_t fg[Iq8Fmt<T>::kGroups / 4], fh[Iq8Fmt<T>::kGroups / 4];   // group factors of rows g, g + 8
  float dg, dh;
};

template <int T>
__device__ __forceinline__ void iq8_load(Iq8Stage<T>& s, const uint32_t* u, const uint8_t* gg, const uint8_t* gh,
                                         const float* sg, const float* sh, int ks) {
  constexpr int LW = Iq8Fmt<T>::kLaneWords, NG = Iq8Fmt<T>::kGroups;
#pragma unroll
  for (int i = 0; i < LW / 4; ++i) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(u) + i);
    s.w[4 * i] = q.x;
    s.w[4 * i + 1] = q.y;
    s.w[4 * i + 2] = q.z;
    s.w[4 * i + 3] = q.w;
  }
  if constexpr (NG == 16) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(gg + (size_t)ks * NG));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(gh + (size_t)ks * NG));
    s.fg[0] = a.x; s.fg[1] = a.y; s.fg[2] = a.z; s.fg[3] = a.w;
    s.fh[0] = b.x; s.fh[1] = b.y; s.fh[2] = b.z; s.fh[3] = b.w;
  } else {
    const uint2 a = __ldg(reinterpret_cast<const uint2*>(gg + (size_t)ks * NG));
    const uint2 b = __ldg(reinterpret_cast<const uint2*>(gh + (size_t)ks * NG));
    s.fg[0] = a.x; s.fg[1] = a.y;
    s.fh[0] = b.x; s.fh[1] = b.y;
  }
  s.dg = __ldg(sg + ks);
  s.dh = __ldg(sh + ks);
}

template <int T>
__global__ void __launch_bounds__(128, 4) iq8_matvec_kernel(const Iq8Params p) {
  constexpr int LW = Iq8Fmt<T>::kLaneWords, NG = Iq8Fmt<T>::kGroups, NT = kIq8Tiles;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int KS = p.K >> 8, RB = p.rows / kRowsPerBlock;
  const int n_items = *p.n_pass * RB;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int pass = item / RB, rb = item - pass * RB;
    const int e = p.pass_expert[pass], row0 = p.pass_row0[pass];
    const int cnt = min(p.pass_cnt[pass], 4 * NT);
    if (e < 0 || e >= p.E || cnt <= 0) continue;
    const int rbase = rb * kRowsPerBlock + warp * kRowsPerWarp;
    // B column g of tile n: token n*4 + g/2 of the pass, digit g%2
    const uint8_t* bsrc[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int j = n * 4 + (g >> 1), jj = j < cnt ? j : 0;
      const int xr = p.tok_row ? p.tok_row[row0 + jj] : row0 + jj;
      bsrc[n] = p.x8 + (size_t)xr * KS * kX8StageBytes + (g & 1) * 64 + 16 * t;
    }
    const uint32_t* u = p.units + ((((size_t)e * RB + rb) * KS * 4 + warp) * 32 + lane) * LW;
    const size_t ustride = (size_t)4 * 32 * LW;
    const size_t rg = (size_t)e * p.rows + rbase + g, rh = rg + 8;
    const uint8_t* gg = p.groups + rg * KS * NG;
    const uint8_t* gh = p.groups + rh * KS * NG;
    const float* sg = p.scales + rg * KS;
    const float* sh = p.scales + rh * KS;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
    Iq8Stage<T> cur, nxt;
    iq8_load<T>(cur, u, gg, gh, sg, sh, 0);
    for (int ks = 0; ks < KS; ++ks) {
      if (ks + 1 < KS) iq8_load<T>(nxt, u + (ks + 1) * ustride, gg, gh, sg, sh, ks + 1);
      int ai[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) ai[n][i] = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 bx[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n)
          if (n == 0 || n * 4 < cnt)
            bx[n] = __ldg(reinterpret_cast<const uint4*>(bsrc[n] + ks * kX8StageBytes + c * 128));
        if constexpr (T == CBMOE_GGML_IQ2_S) {
          uint32_t ag[4], ah[4];
          iq8_frag_iq2(cur.w[3 * c], cur.w[3 * c + 1], cur.w[3 * c + 2], ag, ah);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int kg = (int)((cur.fg[c] >> (8 * j)) & 255u), kh = (int)((cur.fh[c] >> (8 * j)) & 255u);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              if (!(n == 0 || n * 4 < cnt)) continue;
              int D[4] = {0, 0, 0, 0};
              mma_i8_k16(D, ag[j], ah[j], word_of(bx[n], j));
              ai[n][0] += kg * D[0];
              ai[n][1] += kg * D[1];
              ai[n][2] += kh * D[2];
              ai[n][3] += kh * D[3];
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t a[4];
            iq8_frag_iq3(cur.w[4 * c + 2 * h], cur.w[4 * c + 2 * h + 1], a);
            const uint32_t ones[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
            const int m = 2 * c + h;
            const int kg = (int)((cur.fg[m >> 2] >> (8 * (m & 3))) & 255u);
            const int kh = (int)((cur.fh[m >> 2] >> (8 * (m & 3))) & 255u);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              if (!(n == 0 || n * 4 < cnt)) continue;
              int D[4] = {0, 0, 0, 0}, S[4] = {0, 0, 0, 0};
              mma_i8<true>(D, a, word_of(bx[n], 2 * h), word_of(bx[n], 2 * h + 1));
              mma_i8<true>(S, ones, word_of(bx[n], 2 * h), word_of(bx[n], 2 * h + 1));
#pragma unroll
              for (int i = 0; i < 4; ++i) ai[n][i] += ((i & 2) ? kh : kg) * (2 * D[i] - 15 * S[i]);
            }
          }
        }
      }
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[n][i] += (float)ai[n][i] * ((i & 2) ? cur.dh : cur.dg);
      if (ks + 1 < KS) cur = nxt;
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int j = n * 4 + t;
      if (j >= cnt) continue;
      const float fx = p.x8_scale[p.tok_row ? p.tok_row[row0 + j] : row0 + j];
      float* o = p.out + (size_t)(row0 + j) * p.rows + rbase + g;
      o[0] = (acc[n][0] + acc[n][1] * 256.f) * fx;
      o[8] = (acc[n][2] + acc[n][3] * 256.f) * fx;
    }
  }
}

template <int T>
int launch_iq8_matvec(const Iq8Params& p, int kind, cudaStream_t s) {
  static PerDevice s_grid;
  long long grid = 0;
  int rc = per_device(s_grid, [&](long long& v) -> int {
    int per_sm = 0;
    CBMOE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, iq8_matvec_kernel<T>, 128, 0));
    v = (long long)num_sms() * (per_sm > 0 ? per_sm : 1);
    return CBMOE_OK;
  }, &grid);
  if (rc) return rc;
  prof_begin(kind, s);
  iq8_matvec_kernel<T><<<(int)grid, 128, 0, s>>>(p);
  prof_end(kind, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

template <int T>
int launch_iq8_split(const void* x, const float* u, float limit, int in, int R, int K, uint8_t* x8, float* scale,
                     cudaStream_t s) {
  if (R <= 0) return CBMOE_OK;
  const int blocks = R < num_sms() * 4 ? R : num_sms() * 4;
  prof_begin(kProfOther, s);
  if (in == 1) iq8_split_kernel<T, 1><<<blocks, 256, 0, s>>>(x, u, limit, R, K, x8, scale);
  else if (in == 2) iq8_split_kernel<T, 2><<<blocks, 256, 0, s>>>(x, u, limit, R, K, x8, scale);
  else iq8_split_kernel<T, 0><<<blocks, 256, 0, s>>>(x, u, limit, R, K, x8, scale);
  prof_end(kProfOther, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

template <int T>
int iq8_build_t(const void* raw, const float* table, int E, int rows, int K, void* out, cudaStream_t stream) {
  const Iq8Sizes sz = iq8_sizes<T>(E, rows, K);
  uint8_t* base = static_cast<uint8_t*>(out);
  const int KS = K / 256;
  int* bad = nullptr;
  CBMOE_CUDA_TRY(cudaMalloc(&bad, sizeof(int)));
  int rc = CBMOE_OK;
  if (cudaMemsetAsync(bad, 0, sizeof(int), stream) != cudaSuccess) rc = CBMOE_ERR_CUDA;
  if (!rc) {
    const long long n_warps = (long long)E * (rows / kRowsPerBlock) * KS * 4;
    long long blocks = (n_warps + 7) / 8;
    if (blocks > (long long)num_sms() * 16) blocks = (long long)num_sms() * 16;
    iq8_units_kernel<T><<<(int)blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(raw), table, E, rows, KS,
                                                         reinterpret_cast<uint32_t*>(base), bad);
    const long long n_blocks = (long long)E * rows * KS;
    long long b2 = (n_blocks + 255) / 256;
    if (b2 > (long long)num_sms() * 16) b2 = (long long)num_sms() * 16;
    iq8_scales_kernel<T><<<(int)b2, 256, 0, stream>>>(static_cast<const uint8_t*>(raw), n_blocks, base + sz.units,
                                                       reinterpret_cast<float*>(base + sz.units + sz.groups));
    if (cudaGetLastError() != cudaSuccess) rc = CBMOE_ERR_CUDA;
  }
  int hbad = 0;
  if (!rc && (cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
              cudaStreamSynchronize(stream) != cudaSuccess))
    rc = CBMOE_ERR_CUDA;
  cudaFree(bad);
  if (!rc && hbad) rc = CBMOE_ERR_UNSUPPORTED;
  return rc;
}

}  // namespace

// ------------------------------------------------------------------------------------- library-internal API
bool iq8_type(int t) { return t == CBMOE_GGML_IQ2_S || t == CBMOE_GGML_IQ3_S; }

size_t iq8_table_bytes(int t, int E, int rows, int K) {
  if (t == CBMOE_GGML_IQ2_S) return iq8_sizes<CBMOE_GGML_IQ2_S>(E, rows, K).total;
  if (t == CBMOE_GGML_IQ3_S) return iq8_sizes<CBMOE_GGML_IQ3_S>(E, rows, K).total;
  return 0;
}

int iq8_split(int t, const void* x, bool f32, int R, int K, uint8_t* x8, float* scale, cudaStream_t s) {
  return t == CBMOE_GGML_IQ2_S ? launch_iq8_split<CBMOE_GGML_IQ2_S>(x, nullptr, 0.f, f32 ? 1 : 0, R, K, x8, scale, s)
                               : launch_iq8_split<CBMOE_GGML_IQ3_S>(x, nullptr, 0.f, f32 ? 1 : 0, R, K, x8, scale, s);
}

int iq8_swiglu_split(int t, const float* g, const float* u, float limit, int R, int K, uint8_t* x8, float* scale,
                     cudaStream_t s) {
  return t == CBMOE_GGML_IQ2_S ? launch_iq8_split<CBMOE_GGML_IQ2_S>(g, u, limit, 2, R, K, x8, scale, s)
                               : launch_iq8_split<CBMOE_GGML_IQ3_S>(g, u, limit, 2, R, K, x8, scale, s);
}

int iq8_matvec(int t, const void* table8, int E, int rows, int K, const int32_t* plan_pass_expert,
               const int32_t* plan_pass_row0, const int32_t* plan_pass_cnt, const int32_t* n_pass,
               const int32_t* tok_row, const uint8_t* x8, const float* x8_scale, float* out, int kind,
               cudaStream_t s) {
  Iq8Params p{};
  const uint8_t* base = static_cast<const uint8_t*>(table8);
  p.rows = rows;
  p.K = K;
  p.E = E;
  p.pass_expert = plan_pass_expert;
  p.pass_row0 = plan_pass_row0;
  p.pass_cnt = plan_pass_cnt;
  p.n_pass = n_pass;
  p.tok_row = tok_row;
  p.x8 = x8;
  p.x8_scale = x8_scale;
  p.out = out;
  if (t == CBMOE_GGML_IQ2_S) {
    const Iq8Sizes sz = iq8_sizes<CBMOE_GGML_IQ2_S>(E, rows, K);
    p.units = reinterpret_cast<const uint32_t*>(base);
    p.groups = base + sz.units;
    p.scales = reinterpret_cast<const float*>(base + sz.units + sz.groups);
    return launch_iq8_matvec<CBMOE_GGML_IQ2_S>(p, kind, s);
  }
  const Iq8Sizes sz = iq8_sizes<CBMOE_GGML_IQ3_S>(E, rows, K);
  p.units = reinterpret_cast<const uint32_t*>(base);
  p.groups = base + sz.units;
  p.scales = reinterpret_cast<const float*>(base + sz.units + sz.groups);
  return launch_iq8_matvec<CBMOE_GGML_IQ3_S>(p, kind, s);
}

}  // namespace cbmoe

using namespace cbmoe;

extern "C" size_t cbmoe_iq8_bytes(int ggml_type, int E, int rows, int K) {
  if (!iq8_type(ggml_type) || E <= 0 || rows <= 0 || K <= 0 || rows % kRowsPerBlock || K % 256) return 0;
  return iq8_table_bytes(ggml_type, E, rows, K);
}

extern "C" int cbmoe_iq8_build(int ggml_type, const void* raw, const float* table, int E, int rows, int K, void* out,
                               cudaStream_t stream) {
  if (!iq8_type(ggml_type)) return CBMOE_ERR_UNSUPPORTED;
  if (!raw || !table || !out || E <= 0 || rows <= 0 || K <= 0 || rows % kRowsPerBlock || K % 256 ||
      (reinterpret_cast<uintptr_t>(out) & 255) || (reinterpret_cast<uintptr_t>(table) & 3))
    return CBMOE_ERR_INVALID;
  return ggml_type == CBMOE_GGML_IQ2_S ? iq8_build_t<CBMOE_GGML_IQ2_S>(raw, table, E, rows, K, out, stream)
                                       : iq8_build_t<CBMOE_GGML_IQ3_S>(raw, table, E, rows, K, out, stream);
}
