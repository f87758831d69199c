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

struct Codebook {
  uint32_t la, lb, ha, hb;
};

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

__host__ __device__ inline size_t unit_offset(int e, int rb, int ks, int w, int m, int RB, int KS, int nmat,
                                              int unit_bytes) {
  return (((((size_t)e * RB + rb) * KS + ks) * kWarpsPerBlock + w) * nmat + m) * (size_t)unit_bytes;
}

__host__ __device__ inline size_t cb_offset_words(int e, int rb, int w, int m, int r16, int RB, int nmat) {
  return ((((size_t)e * RB + rb) * kWarpsPerBlock + w) * nmat + m) * 64 + (size_t)r16 * 4;
}

}  // namespace cbmoe
