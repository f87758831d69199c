// Kernel layouts of the expert tables and the register-level dequant that reads them.
//
// Both layouts are organized around the bf16 m16n8k16 tensor-core fragment of one decode warp:
//   a warp owns 16 weight rows; lane (g = lane/4, t = lane%4) owns rows g and g+8;
//   a 64-input "chunk" gives lane t the 16 consecutive inputs [16t, 16t+16) of both rows; within the chunk, MMA
//   step s (0..3) covers inputs 16t+4s .. 16t+4s+3: fragment a0/a2 = row g, inputs {+0,+1}/{+2,+3}; a1/a3 = row g+8.
//   The activation fragment of the same step is x[16t+4s .. +3] of token g, so a lane's activations for a chunk
//   are 16 consecutive bf16 (two 16-byte loads).
// A "unit" is one warp's 16 rows x 256 inputs (4 chunks) of one matrix; a "stage" is the 4 warps' units of a
// 64-row block (times nmat matrices), which is contiguous in memory and streamed with one bulk copy.
//   offset(e, rb, ks, w, m) = ((((e*RB + rb)*KS + ks)*4 + w)*nmat + m) * UNIT_BYTES,  RB = rows/64, KS = K/256
//
// CB3K unit (1536 B): lane-major, 48 B per lane = 4 chunks x 3 words (w0, w1, w2). For chunk c:
//   w0 nibble n = 4s+i (s = 0,1): index of row g, input 16t+4s+i (bits 0-2)
//   w1 nibble n = 4(s-2)+i (s = 2,3): row g
//   w2 nibble n = 4s+i (s = 0,1): row g+8
//   row g+8, s = 2,3, nibble n = 4(s-2)+i: bit 0 in bit 3 of w0's nibble n, bit 1 in bit 3 of w1's, bit 2 of w2's.
// So every 4-index selector is 4 nibbles whose low 3 bits are the indices: one `prmt` over the codebook's 8 low
// bytes and one over its 8 high bytes look up 4 weights; two more interleave them into bf16 pairs.
// CB3K codebooks: 16 B per row, byte-planar: word0 = low bytes of entries 0-3, word1 = low bytes of 4-7,
// word2 = high bytes of 0-3, word3 = high bytes of 4-7; ordered [e][rb][w][m][row 0..15].
//
// W8K unit (4096 B): int8, ordered [chunk c][row half h][lane][16 B]: lane (g, t)'s 16 inputs [16t, 16t+16) of
// row g (h = 0) or g+8 (h = 1); lanes contiguous so a warp's 16-byte shared loads are conflict-free.
//
// CB8 (the decode kernels' codebooks, built at load time from the CB3K ones): every row's 8 bf16 entries as 16-bit
// fixed point, T = rint(v 2^s) with the row's largest magnitude times 2^s in [2^14, 2^15), stored as two byte
// tables: hi = T >> 8 (int8) and lo = T & 255 (uint8), so T = 256 hi + lo, plus the row factor 2^-s. T equals
// v 2^s exactly for every entry within 2^7 of the row's largest (bf16 has 8 significant bits); smaller entries are
// rounded to within 2^-15 of the largest. The same CB3K index bits select the bytes: one `prmt` looks up 4
// weights' hi bytes, one their lo bytes, and each feeds an int8 m16n8k32 MMA (exact int32 sums).
// Per (expert, 64-row block): tables [w][m][row 0..15] x 16 B (hi bytes of entries 0-3 | 4-7, lo bytes of 0-3 |
// 4-7), then row factors 2^-s [w][m][row 0..15] x f32.
// The m16n8k32 fragment: a lane's A register 0 / 2 hold row g's physical inputs 16t+8h+{0..3} / {4..7} of MMA step
// h (0, 1) of a chunk, registers 1 / 3 row g+8's; B register 0 / 1 hold the same inputs of one column: the CB3K
// selector groups s = 2h, 2h+1 unchanged, and a column's 8 inputs of step h are 8 consecutive bytes.
// Activations reach these kernels split into signed digits the same way: "X8" rows (split_x_row) hold, per
// 256-input stage, [chunk 4][digit 2][64] int8 with one factor f per row: x = f (256 d1 + d0), the row's largest
// |x| / f in [2^13, 2^14) (exact for bf16 within 2^6 of the row's largest, else to within 2^-14 of it); "H8" rows
// (the SwiGLU epilogue of the CB8 gate/up kernel) hold [chunk 4][digit 4][64] int8 then 4 f32 factors (one per
// 64-input chunk): h = f_c sum_p 256^p d_p, the chunk's largest |h| / f_c in [2^28, 2^29) (the fp32 value itself
// for every element within 2^5 of the chunk's largest).
#pragma once
#include <cstdint>
#include "common.cuh"

namespace cbmoe {

constexpr int kRowsPerWarp = 16;
constexpr int kWarpsPerBlock = 4;
constexpr int kRowsPerBlock = kRowsPerWarp * kWarpsPerBlock;  // 64
constexpr int kStageK = 256;
constexpr int kChunkK = 64;
constexpr int kCb3kUnitBytes = 32 * 48;                       // 1536
constexpr int kW8kUnitBytes = 4 * 2 * 32 * 16;                // 4096
constexpr int kFmtCB3 = 0;
constexpr int kFmtW8 = 1;
constexpr int kFmtCB8 = 2;
constexpr int kFmtW8I = 4;   // int8 leaves (W8K) multiplied as stored against X8 digits: the int8 lm_head
constexpr int kCb8RowBytes = 16 + 4;                           // tables + row factor
constexpr int kCb8BlockBytes = kRowsPerBlock * kCb8RowBytes;   // per matrix and 64-row block: 1280
constexpr int kX8StageBytes = 4 * 2 * 64;                      // 512
constexpr int kH8StageBytes = 4 * 4 * 64 + 16;                 // 1040: parts + 4 chunk factors

template <int FMT>
struct Fmt;
template <>
struct Fmt<kFmtCB3> {
  static constexpr int kUnitBytes = kCb3kUnitBytes;
};
template <>
struct Fmt<kFmtW8> {
  static constexpr int kUnitBytes = kW8kUnitBytes;
};
template <>
struct Fmt<kFmtCB8> {
  static constexpr int kUnitBytes = kCb3kUnitBytes;   // the CB3K index bits
};
template <>
struct Fmt<kFmtW8I> {
  static constexpr int kUnitBytes = kW8kUnitBytes;
};

struct Codebook {
  uint32_t la, lb, ha, hb;
};

// CB8 tables of one row: hi bytes (int8) of entries 0-3 | 4-7, lo bytes (uint8) of 0-3 | 4-7.
struct Cb8 {
  uint32_t ha, hb, la, lb;
};

// One chunk of one CB8 matrix: the 3 CB3K index words of this lane -> int8 A fragments of the hi and lo bytes for
// the chunk's two k32 MMA steps: ah[h] / al[h] = {row g group 2h, row g+8 group 2h, row g group 2h+1, row g+8
// group 2h+1}. Selectors as cb3k_dequant_chunk (shifts and masks; moving the spare-bit word and the upper halves to
// multiply-adds on the FMA pipe measured slower).
__device__ __forceinline__ void cb8_dequant_chunk(uint32_t w0, uint32_t w1, uint32_t w2, const Cb8& cg,
                                                  const Cb8& ch, uint32_t (&ah)[2][4], uint32_t (&al)[2][4]) {
  const uint32_t g01 = w0 & 0x77777777u;
  const uint32_t g23 = w1 & 0x77777777u;
  const uint32_t h01 = w2 & 0x77777777u;
  const uint32_t h23 = ((w0 >> 3) & 0x11111111u) | ((w1 >> 2) & 0x22222222u) | ((w2 >> 1) & 0x44444444u);
  const uint32_t g01u = g01 >> 16, g23u = g23 >> 16, h01u = h01 >> 16, h23u = h23 >> 16;
  ah[0][0] = prmt(cg.ha, cg.hb, g01);
  ah[0][1] = prmt(ch.ha, ch.hb, h01);
  ah[0][2] = prmt(cg.ha, cg.hb, g01u);
  ah[0][3] = prmt(ch.ha, ch.hb, h01u);
  ah[1][0] = prmt(cg.ha, cg.hb, g23);
  ah[1][1] = prmt(ch.ha, ch.hb, h23);
  ah[1][2] = prmt(cg.ha, cg.hb, g23u);
  ah[1][3] = prmt(ch.ha, ch.hb, h23u);
  al[0][0] = prmt(cg.la, cg.lb, g01);
  al[0][1] = prmt(ch.la, ch.lb, h01);
  al[0][2] = prmt(cg.la, cg.lb, g01u);
  al[0][3] = prmt(ch.la, ch.lb, h01u);
  al[1][0] = prmt(cg.la, cg.lb, g23);
  al[1][1] = prmt(ch.la, ch.lb, h23);
  al[1][2] = prmt(cg.la, cg.lb, g23u);
  al[1][3] = prmt(ch.la, ch.lb, h23u);
}

// The shift that brings the largest magnitude m into [2^(top-1), 2^top): top - e, where m = f 2^e, f in [0.5, 1)
// (frexp's exponent); 0 when m is zero or not finite (nothing to scale).
__device__ __forceinline__ int shift_for(float m, int top) {
  if (!(m > 0.f && m < 3e38f)) return 0;
  int ex = 0;
  frexpf(m, &ex);
  return top - ex;
}

// 2^k as a float (k in [-126, 127]).
__device__ __forceinline__ float pow2f(int k) { return __int_as_float((127 + k) << 23); }

// One chunk of one matrix: 3 index words of this lane -> fragments a[s][0..3] for the 4 MMA steps.
//   selectors of row g:   w0 & 0x7.. (s = 0 low half, s = 1 high half), w1 & 0x7.. (s = 2, 3)
//   selectors of row g+8: w2 & 0x7.. (s = 0, 1); s = 2, 3 from the spare bits: (w0 & 0x8..) >> 3 |
//                         (w1 & 0x8..) >> 2 | (w2 & 0x8..) >> 1.
// (Moving the shifts to integer multiply-adds on the FMA pipe was measured slower: longer dependency latency.)
__device__ __forceinline__ void cb3k_dequant_chunk(uint32_t w0, uint32_t w1, uint32_t w2, const Codebook& cg,
                                                   const Codebook& ch, uint32_t (&a)[4][4]) {
  const uint32_t g01 = w0 & 0x77777777u;
  const uint32_t g23 = w1 & 0x77777777u;
  const uint32_t h01 = w2 & 0x77777777u;
  const uint32_t h23 = ((w0 >> 3) & 0x11111111u) | ((w1 >> 2) & 0x22222222u) | ((w2 >> 1) & 0x44444444u);
  const uint32_t sg[4] = {g01, g01 >> 16, g23, g23 >> 16};
  const uint32_t sh[4] = {h01, h01 >> 16, h23, h23 >> 16};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    uint32_t lo = prmt(cg.la, cg.lb, sg[s]);
    uint32_t hi = prmt(cg.ha, cg.hb, sg[s]);
    a[s][0] = prmt(lo, hi, 0x5140u);
    a[s][2] = prmt(lo, hi, 0x7362u);
    lo = prmt(ch.la, ch.lb, sh[s]);
    hi = prmt(ch.ha, ch.hb, sh[s]);
    a[s][1] = prmt(lo, hi, 0x5140u);
    a[s][3] = prmt(lo, hi, 0x7362u);
  }
}

// 4 signed bytes of q -> exact floats, without the conversion unit: byte ^ 0x80 placed in the mantissa of 2^23
// gives 2^23 + 128 + b, and one subtraction of 2^23 + 128 leaves b.
__device__ __forceinline__ void w8_bytes_to_f32(uint32_t q, float (&f)[4]) {
  const uint32_t qx = q ^ 0x80808080u;
  constexpr float kBias = 8388736.0f;  // 2^23 + 128
  f[0] = __uint_as_float(prmt(qx, 0x4B000000u, 0x7540u)) - kBias;
  f[1] = __uint_as_float(prmt(qx, 0x4B000000u, 0x7541u)) - kBias;
  f[2] = __uint_as_float(prmt(qx, 0x4B000000u, 0x7542u)) - kBias;
  f[3] = __uint_as_float(prmt(qx, 0x4B000000u, 0x7543u)) - kBias;
}

// One chunk of one W8K matrix: qg/qh = this lane's 16 int8 of rows g and g+8 (4 words each) -> bf16 fragments
// of bf16(f32(q) * s) (quant8.py:94). Scales: per row (sg, sh) when kscale == nullptr, else per input from
// kscale[0..15] (this lane's 16 inputs of the chunk).
__device__ __forceinline__ void w8k_dequant_chunk(const uint4& qg, const uint4& qh, float sg, float sh,
                                                  const float* kscale, uint32_t (&a)[4][4]) {
  const uint32_t g[4] = {qg.x, qg.y, qg.z, qg.w};
  const uint32_t h[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    float fg[4], fh[4];
    w8_bytes_to_f32(g[s], fg);
    w8_bytes_to_f32(h[s], fh);
    if (kscale == nullptr) {
      a[s][0] = pack_bf16x2(fg[0] * sg, fg[1] * sg);
      a[s][2] = pack_bf16x2(fg[2] * sg, fg[3] * sg);
      a[s][1] = pack_bf16x2(fh[0] * sh, fh[1] * sh);
      a[s][3] = pack_bf16x2(fh[2] * sh, fh[3] * sh);
    } else {
      const float k0 = kscale[4 * s], k1 = kscale[4 * s + 1], k2 = kscale[4 * s + 2], k3 = kscale[4 * s + 3];
      a[s][0] = pack_bf16x2(fg[0] * k0, fg[1] * k1);
      a[s][2] = pack_bf16x2(fg[2] * k2, fg[3] * k3);
      a[s][1] = pack_bf16x2(fh[0] * k0, fh[1] * k1);
      a[s][3] = pack_bf16x2(fh[2] * k2, fh[3] * k3);
    }
  }
}

// X8 rows: one CTA per row. The row's largest |x| sets the factor: X = rint(x 2^t), largest |X| in [2^13, 2^14);
// digits d1 = (X + 128) >> 8, d0 = X - 256 d1 (both int8): x = 2^-t (256 d1 + d0).
__device__ inline void split_x_row(const uint16_t* __restrict__ xr, int K, uint8_t* __restrict__ out,
                                   float* __restrict__ scale, float* red) {
  float mx = 0.f;
  for (int i = threadIdx.x; i < K; i += blockDim.x)
    mx = fmaxf(mx, fabsf(__uint_as_float((uint32_t)xr[i] << 16)));
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();   // red is reused by the next row
  const int sh = shift_for(mx, 14);
  if (threadIdx.x == 0) *scale = ldexpf(1.f, -sh);
  for (int i = 2 * threadIdx.x; i < K; i += 2 * blockDim.x) {
    uint32_t dig[2][2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int X = __float2int_rn(ldexpf(__uint_as_float((uint32_t)xr[i + e] << 16), sh));
      const int d1 = (X + 128) >> 8;
      dig[e][1] = (uint32_t)d1 & 0xffu;
      dig[e][0] = (uint32_t)(X - 256 * d1) & 0xffu;
    }
    const int ks = i / kStageK, c = (i % kStageK) / kChunkK, q = i % kChunkK;
    uint8_t* o = out + (size_t)ks * kX8StageBytes + c * 128 + q;
    *reinterpret_cast<uint16_t*>(o) = (uint16_t)(dig[0][0] | (dig[1][0] << 8));
    *reinterpret_cast<uint16_t*>(o + 64) = (uint16_t)(dig[0][1] | (dig[1][1] << 8));
  }
}

__host__ __device__ inline size_t unit_offset(int e, int rb, int ks, int w, int m, int RB, int KS, int nmat,
                                              int unit_bytes) {
  return (((((size_t)e * RB + rb) * KS + ks) * kWarpsPerBlock + w) * nmat + m) * (size_t)unit_bytes;
}

__host__ __device__ inline size_t cb_offset_words(int e, int rb, int w, int m, int r16, int RB, int nmat) {
  return ((((size_t)e * RB + rb) * kWarpsPerBlock + w) * nmat + m) * 64 + (size_t)r16 * 4;
}

// Byte offset of the CB8 block of (expert e, 64-row block rb).
__host__ __device__ inline size_t cb8_block_offset(int e, int rb, int RB, int nmat) {
  return ((size_t)e * RB + rb) * nmat * kCb8BlockBytes;
}

}  // namespace cbmoe
