// Per-lane dequant of the reference's GGUF expert formats: weights 8*lane .. 8*lane+7 of one 256-weight block, in
// fp32 with every product (and Q2_K's difference) rounded once, in the reference's order (iqquant.py:108-146 for
// the IQ formats, :200-226 for the K-quants of its MTP layer; gguf-py computes the same values). Host and device
// code: the GPU kernels (iq.cu) and a host test harness compile this same source.
//   IQ2_S  (82 B)  lane = group of 8: 10-bit grid index (qs byte | 2 bits of qh), sign byte, 4-bit scale of its 16
//                  weights; w = ((d * (0.5 + s)) * 0.25) * grid[idx][k], negated where the sign bit is set.
//   IQ3_S  (110 B) lane = groups 2 lane, 2 lane + 1 of 4: 9-bit index (qs byte | 1 bit of qh), sign byte lane, 4-bit
//                  scale of its 32 weights; w = (d * (1 + 2s)) * grid[idx][k], sign as above.
//   IQ4_XS (136 B) lane = 8 weights of sub-block lane/4 (32 weights): low nibbles for the first 16, high for the rest;
//                  w = (d * (scale - 32)) * kvalues[nibble], scale = 4 low bits | 2 high bits << 4.
//   Q2_K   (84 B)  weight 128n + 32s + l = (qs[32n + l] >> 2s) & 3, scale byte 8n + 2s + l/16 (low nibble x d,
//                  high nibble x dmin at bytes 80 / 82): w = (d * sc) * q - dmin * m.
//   Q3_K   (110 B) weight 128n + 32s + l: q = ((qs[32 + 32n + l] >> 2s) & 3) - 4 unless bit 4n + s of hmask[l];
//                  the 6-bit scale m = 8n + 2s + l/16 from the 12 scale bytes; w = (d * (scale - 32)) * q.
// The lookup tables are the caller's (fp32): IQ2_S [1024][8], IQ3_S [512][4], IQ4_XS [16]; the K-quants have none.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "cbmoe.h"

namespace cbmoe {

template <int T>
struct IqFmt;
template <>
struct IqFmt<CBMOE_GGML_IQ2_S> {
  static constexpr int kBytes = 82, kEntries = 1024, kWidth = 8;
};
template <>
struct IqFmt<CBMOE_GGML_IQ3_S> {
  static constexpr int kBytes = 110, kEntries = 512, kWidth = 4;
};
template <>
struct IqFmt<CBMOE_GGML_IQ4_XS> {
  static constexpr int kBytes = 136, kEntries = 16, kWidth = 1;
};
template <>
struct IqFmt<CBMOE_GGML_Q2_K> {
  static constexpr int kBytes = 84, kEntries = 0, kWidth = 0;
};
template <>
struct IqFmt<CBMOE_GGML_Q3_K> {
  static constexpr int kBytes = 110, kEntries = 0, kWidth = 0;
};

// One rounding per operation on both sides (the host harness is built without contraction as well).
__host__ __device__ __forceinline__ float iq_mul(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
__host__ __device__ __forceinline__ float iq_sub(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}

__host__ __device__ __forceinline__ float f16_at(const uint8_t* p) {
  const unsigned short bits = (unsigned short)(p[0] | (p[1] << 8));
  return __half2float(__ushort_as_half(bits));
}

__host__ __device__ __forceinline__ float with_sign(float v, unsigned sign_byte, int k) {
  return ((sign_byte >> k) & 1u) ? -v : v;
}

// W consecutive table values (a grid row: 16-byte aligned in the kernels' shared-memory copy, so one or two
// 16-byte loads there).
template <int W>
__host__ __device__ __forceinline__ void grid_row(const float* row, float (&out)[W]) {
#ifdef __CUDA_ARCH__
#pragma unroll
  for (int i = 0; i < W / 4; ++i) {
    const float4 q = reinterpret_cast<const float4*>(row)[i];
    out[4 * i] = q.x;
    out[4 * i + 1] = q.y;
    out[4 * i + 2] = q.z;
    out[4 * i + 3] = q.w;
  }
#else
  for (int i = 0; i < W; ++i) out[i] = row[i];
#endif
}

template <int T>
__host__ __device__ __forceinline__ void iq_lane8(const uint8_t* __restrict__ blk, int lane, const float* table,
                                                  float (&v)[8]) {
  if constexpr (T == CBMOE_GGML_IQ2_S) {
    const float d = f16_at(blk);
    const int g = lane;
    const int idx = blk[2 + g] | (((blk[66 + g / 4] >> (2 * (g % 4))) & 3) << 8);
    const int s = (blk[74 + g / 4] >> (4 * ((g / 2) % 2))) & 15;
    const unsigned sg = blk[34 + g];
    const float db = iq_mul(iq_mul(d, 0.5f + (float)s), 0.25f);
    float gr[8];
    grid_row<8>(table + idx * 8, gr);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = with_sign(iq_mul(db, gr[k]), sg, k);
  } else if constexpr (T == CBMOE_GGML_IQ3_S) {
    const float d = f16_at(blk);
    const int m = lane / 4;   // 32-weight scale group
    const int s = (blk[106 + m / 2] >> (4 * (m % 2))) & 15;
    const float db = iq_mul(d, (float)(1 + 2 * s));
    const unsigned sg = blk[74 + lane];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int G = 2 * lane + h;
      const int idx = blk[2 + G] | (((blk[66 + G / 8] >> (G % 8)) & 1) << 8);
      float gr[4];
      grid_row<4>(table + idx * 4, gr);
#pragma unroll
      for (int q = 0; q < 4; ++q) v[4 * h + q] = with_sign(iq_mul(db, gr[q]), sg, 4 * h + q);
    }
  } else if constexpr (T == CBMOE_GGML_IQ4_XS) {
    const float d = f16_at(blk);
    const int i = lane / 4, q = (lane % 4) * 8;   // sub-block, first position inside it
    const int sh = blk[2] | (blk[3] << 8);
    const int sc = (((blk[4 + i / 2] >> (4 * (i % 2))) & 15) | (((sh >> (2 * i)) & 3) << 4)) - 32;
    const float dl = iq_mul(d, (float)sc);
    const uint8_t* qs = blk + 8 + 16 * i + (q & 15);
    const int shift = q >= 16 ? 4 : 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = iq_mul(dl, table[(qs[j] >> shift) & 15]);
  } else {
    // K-quants: lane covers half n = lane / 16, shift s = (lane % 16) / 4, positions l = 8 (lane % 4) .. + 7
    const int n = lane / 16, s = (lane % 16) / 4, l0 = 8 * (lane % 4);
    const int m = 8 * n + 2 * s + l0 / 16;   // scale index (16 weights each)
    if constexpr (T == CBMOE_GGML_Q2_K) {
      const int sc = blk[m];
      const float dl = iq_mul(f16_at(blk + 80), (float)(sc & 15));
      const float ml = iq_mul(f16_at(blk + 82), (float)(sc >> 4));
      const uint8_t* qs = blk + 16 + 32 * n + l0;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = iq_sub(iq_mul(dl, (float)((qs[j] >> (2 * s)) & 3)), ml);
    } else {
      const uint8_t* sc12 = blk + 96;
      const int lo = (sc12[m % 8] >> (4 * (m / 8))) & 15;
      const int hi = (sc12[8 + m % 4] >> (2 * (m / 4))) & 3;
      const float dl = iq_mul(f16_at(blk + 108), (float)((lo | (hi << 4)) - 32));
      const uint8_t* qs = blk + 32 + 32 * n + l0;
      const int bit = 4 * n + s;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = ((qs[j] >> (2 * s)) & 3) - (((blk[l0 + j] >> bit) & 1) ? 0 : 4);
        v[j] = iq_mul(dl, (float)q);
      }
    }
  }
}

}  // namespace cbmoe
