// Int8 tensor-core layout ("IQ8") of the reference's IQ2_S and IQ3_S expert tables, and the per-lane arithmetic of
// the kernels that read it (iq8.cu). Host and device code: a host test harness compiles this same source.
//
// An exact transcode at load time: every weight of a raw GGUF block is d * k * v with d the block's f16 scale, k a
// small odd integer per group (IQ2_S: (1 + 2s) / 8 per 16 weights, since d (0.5 + s) 0.25 = d (1 + 2s) / 8; IQ3_S:
// 1 + 2s per 32 weights) and v a signed integer grid value times its sign (IQ2_S: +-8, +-25, +-43; IQ3_S: the odd
// values +-1 .. +-15). The layout keeps v as a per-weight code, k as a byte per group and d as f32 per block row:
//   IQ2_S: code = 3 bits (0, 1, 2 = 8, 25, 43; +4 = negative), looked up with `prmt` in a fixed 8-byte table;
//   IQ3_S: code = 4 bits u with v = 2u - 15, so the int8 MMA takes u directly (sum of v x = 2 sum u x - 15 sum x).
// The products v * x (x in X8 digits) sum exactly in int32; k multiplies each group's int32 partial; d and the
// token factor multiply once per 256-weight block in fp32. The reference computes each weight exactly in fp32
// (iqquant.py:108-134: d * (0.5 + s) * 0.25 * grid and d * (1 + 2s) * grid are exact products), so the only
// difference is the order of the fp32 sums.
//
// Per (expert, 64-row block, 256-input stage): 4 warp units of 16 rows, lane-major, kLaneWords 32-bit words per lane.
// Lane (g = lane / 4, t = lane % 4) holds rows g and g + 8:
//   IQ2_S (m16n8k16 steps, one per 16-weight group: step j of chunk c = group 4c + j): per chunk c three words
//     w0 = sel(g, 0) | sel(g, 1) << 16, w1 = sel(g, 2) | sel(g, 3) << 16, w2 = sel(g + 8, 0) | sel(g + 8, 1) << 16,
//     with sel(r, j) the 4 codes of row r at inputs 64c + 16j + 4t + b (b = 0..3, nibble b) in bits 0-2 of each
//     nibble, and sel(g + 8, 2) | sel(g + 8, 3) << 16 spread over the spare bit 3 of every nibble (bit i of its
//     nibble n in bit 3 of nibble n of word i).
//   IQ3_S (m16n8k32 steps, one per 32-weight group: step h of chunk c = group 2c + h): per chunk c four words
//     W(h, r) for h = 0, 1 and r = g, g + 8: byte b of (W & 0x0F0F0F0F) is the code of input 64c + 32h + 4t + b,
//     byte b of ((W >> 4) & 0x0F0F0F0F) that of input 64c + 32h + 16 + 4t + b.
// Activations: X8 rows (two base-256 digits per input, one factor per row), stored per 64-input chunk in the order
// the B fragments want: storage byte s of a chunk's digit plane holds input iq8_perm<T>(s) of the chunk.
#pragma once
#include <cstdint>

#include "iqlane.cuh"

namespace cbmoe {

template <int T>
struct Iq8Fmt;
template <>
struct Iq8Fmt<CBMOE_GGML_IQ2_S> {
  static constexpr int kLaneWords = 12;   // per lane per stage
  static constexpr int kGroups = 16;      // scale groups per 256 weights
};
template <>
struct Iq8Fmt<CBMOE_GGML_IQ3_S> {
  static constexpr int kLaneWords = 16;
  static constexpr int kGroups = 8;
};

template <int T>
constexpr bool iq8_supported() {
  return T == CBMOE_GGML_IQ2_S || T == CBMOE_GGML_IQ3_S;
}

// Bytes of one matrix's transcoded table: units [E][RB][KS][4][32][kLaneWords] u32 | group factors
// [E][rows][KS][kGroups] u8 | block scales [E][rows][KS] f32 (each part 256-byte aligned).
struct Iq8Sizes {
  size_t units, groups, scales, total;
};
template <int T>
__host__ __device__ inline Iq8Sizes iq8_sizes(int E, int rows, int K) {
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const size_t blocks = (size_t)E * rows * (K / 256);
  Iq8Sizes s;
  s.units = up(blocks * 8 * Iq8Fmt<T>::kLaneWords);   // 32 lanes x kLaneWords words cover 16 block rows
  s.groups = up(blocks * Iq8Fmt<T>::kGroups);
  s.scales = up(blocks * 4);
  s.total = s.units + s.groups + s.scales;
  return s;
}

// Input (within a 64-input chunk) that storage byte s of an X8 digit plane holds, per format.
template <int T>
__host__ __device__ __forceinline__ int iq8_perm(int s) {
  const int t = s >> 4;
  if constexpr (T == CBMOE_GGML_IQ2_S) {
    const int j = (s >> 2) & 3, b = s & 3;   // s = 16t + 4j + b  <-  input 16j + 4t + b
    return 16 * j + 4 * t + b;
  } else {
    const int h = (s >> 3) & 1, r = (s >> 2) & 1, b = s & 3;   // s = 16t + 8h + 4r + b  <-  32h + 16r + 4t + b
    return 32 * h + 16 * r + 4 * t + b;
  }
}

// Code of weight p (0..255) of one raw block; false when the grid value is not one the code can hold.
template <int T>
__host__ __device__ __forceinline__ bool iq8_code_at(const uint8_t* __restrict__ blk, const float* table, int p,
                                                     uint32_t& code) {
  if constexpr (T == CBMOE_GGML_IQ2_S) {
    const int g = p >> 3, k = p & 7;
    const int idx = blk[2 + g] | (((blk[66 + g / 4] >> (2 * (g % 4))) & 3) << 8);
    const float gv = table[idx * 8 + k];
    const uint32_t neg = (blk[34 + g] >> k) & 1u;
    const uint32_t mag = gv == 8.f ? 0u : gv == 25.f ? 1u : gv == 43.f ? 2u : 3u;
    code = mag | (neg << 2);
    return mag != 3u;
  } else {
    const int G = p >> 2, q = p & 3;
    const int idx = blk[2 + G] | (((blk[66 + G / 8] >> (G % 8)) & 1) << 8);
    const float gv = table[idx * 4 + q];
    const int v = ((blk[74 + p / 8] >> (p % 8)) & 1) ? -(int)gv : (int)gv;
    const bool ok = gv >= 1.f && gv <= 15.f && (float)(int)gv == gv && ((int)gv & 1);
    code = (uint32_t)((v + 15) / 2) & 15u;
    return ok;
  }
}

// Integer group factor k of group m (IQ2_S: 1 + 2s of 16-weight group m; IQ3_S: 1 + 2s of 32-weight group m).
template <int T>
__host__ __device__ __forceinline__ uint32_t iq8_group_factor(const uint8_t* __restrict__ blk, int m) {
  if constexpr (T == CBMOE_GGML_IQ2_S) return 1u + 2u * ((blk[74 + m / 2] >> (4 * (m % 2))) & 15u);
  else return 1u + 2u * ((blk[106 + m / 2] >> (4 * (m % 2))) & 15u);
}

// Scale of the block's int32 sums: d / 8 (IQ2_S) or d (IQ3_S), exact in fp32.
template <int T>
__host__ __device__ __forceinline__ float iq8_block_scale(const uint8_t* __restrict__ blk) {
  const float d = f16_at(blk);
  return T == CBMOE_GGML_IQ2_S ? d * 0.125f : d;
}

// The kLaneWords words of lane `lane` for one stage of one warp: blk_g / blk_h = the raw blocks of rows g and g + 8
// at this stage. Returns false if some grid value has no code.
template <int T>
__host__ __device__ inline bool iq8_lane_words(const uint8_t* blk_g, const uint8_t* blk_h, const float* table,
                                               int lane, uint32_t* words) {
  const int t = lane & 3;
  bool ok = true;
  for (int c = 0; c < 4; ++c) {
    if constexpr (T == CBMOE_GGML_IQ2_S) {
      uint32_t sel[2][4];
      for (int rr = 0; rr < 2; ++rr)
        for (int j = 0; j < 4; ++j) {
          uint32_t s = 0;
          for (int b = 0; b < 4; ++b) {
            uint32_t code;
            ok &= iq8_code_at<T>(rr ? blk_h : blk_g, table, 64 * c + 16 * j + 4 * t + b, code);
            s |= code << (4 * b);
          }
          sel[rr][j] = s;
        }
      uint32_t w0 = sel[0][0] | (sel[0][1] << 16), w1 = sel[0][2] | (sel[0][3] << 16);
      uint32_t w2 = sel[1][0] | (sel[1][1] << 16);
      const uint32_t h23 = sel[1][2] | (sel[1][3] << 16);
      for (int n = 0; n < 8; ++n) {
        const uint32_t nib = (h23 >> (4 * n)) & 7u;
        w0 |= (nib & 1u) << (4 * n + 3);
        w1 |= ((nib >> 1) & 1u) << (4 * n + 3);
        w2 |= ((nib >> 2) & 1u) << (4 * n + 3);
      }
      words[3 * c] = w0;
      words[3 * c + 1] = w1;
      words[3 * c + 2] = w2;
    } else {
      for (int h = 0; h < 2; ++h)
        for (int rr = 0; rr < 2; ++rr) {
          uint32_t w = 0;
          for (int b = 0; b < 4; ++b) {
            uint32_t lo, hi;
            ok &= iq8_code_at<T>(rr ? blk_h : blk_g, table, 64 * c + 32 * h + 4 * t + b, lo);
            ok &= iq8_code_at<T>(rr ? blk_h : blk_g, table, 64 * c + 32 * h + 16 + 4 * t + b, hi);
            w |= lo << (8 * b);
            w |= hi << (8 * b + 4);
          }
          words[4 * c + 2 * h + rr] = w;
        }
    }
  }
  return ok;
}

// Byte permute (PTX prmt, default mode) with the host stand-in the harness uses.
__host__ __device__ __forceinline__ uint32_t iq8_prmt(uint32_t a, uint32_t b, uint32_t sel) {
#ifdef __CUDA_ARCH__
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
#else
  const uint64_t src = (uint64_t)a | ((uint64_t)b << 32);
  uint32_t d = 0;
  for (int i = 0; i < 4; ++i) {
    const uint32_t n = (sel >> (4 * i)) & 15u;
    uint32_t byte = (uint32_t)(src >> (8 * (n & 7))) & 255u;
    if (n & 8) byte = (byte & 128u) ? 255u : 0u;
    d |= byte << (8 * i);
  }
  return d;
#endif
}

// IQ2_S code table (bytes of the int8 values 8, 25, 43, 0, -8, -25, -43, 0).
constexpr uint32_t kIq2TabLo = 0x002B1908u;
constexpr uint32_t kIq2TabHi = 0x00D5E7F8u;

// IQ2_S: the 3 words of a chunk -> A fragments of its 4 k16 steps, rows g (ag) and g + 8 (ah).
__host__ __device__ __forceinline__ void iq8_frag_iq2(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t (&ag)[4],
                                                      uint32_t (&ah)[4]) {
  const uint32_t g01 = w0 & 0x77777777u, g23 = w1 & 0x77777777u, h01 = w2 & 0x77777777u;
  const uint32_t h23 = ((w0 >> 3) & 0x11111111u) | ((w1 >> 2) & 0x22222222u) | ((w2 >> 1) & 0x44444444u);
  ag[0] = iq8_prmt(kIq2TabLo, kIq2TabHi, g01);
  ag[1] = iq8_prmt(kIq2TabLo, kIq2TabHi, g01 >> 16);
  ag[2] = iq8_prmt(kIq2TabLo, kIq2TabHi, g23);
  ag[3] = iq8_prmt(kIq2TabLo, kIq2TabHi, g23 >> 16);
  ah[0] = iq8_prmt(kIq2TabLo, kIq2TabHi, h01);
  ah[1] = iq8_prmt(kIq2TabLo, kIq2TabHi, h01 >> 16);
  ah[2] = iq8_prmt(kIq2TabLo, kIq2TabHi, h23);
  ah[3] = iq8_prmt(kIq2TabLo, kIq2TabHi, h23 >> 16);
}

// IQ3_S: the 2 words of a k32 step (rows g, g + 8) -> its A fragment {a0, a1, a2, a3} of 4-bit codes as bytes.
__host__ __device__ __forceinline__ void iq8_frag_iq3(uint32_t wg, uint32_t wh, uint32_t (&a)[4]) {
  a[0] = wg & 0x0F0F0F0Fu;
  a[1] = wh & 0x0F0F0F0Fu;
  a[2] = (wg >> 4) & 0x0F0F0F0Fu;
  a[3] = (wh >> 4) & 0x0F0F0F0Fu;
}

}  // namespace cbmoe
