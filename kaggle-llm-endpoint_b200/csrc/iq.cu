// llama.cpp IQ expert formats (the reference's real GLM-5.3-Flash tables): dequant of raw GGUF blocks on the GPU.
// Counterpart of the reference's iqquant.dequant_rows / dequant_iq2_s / dequant_iq3_s / dequant_iq4_xs
// (engine/glm53/iqquant.py:108-146, 230-235) and planes.dequant_planes (planes.py:183-196), in fp32, bit for bit:
// the same products in the same order, each rounded once (no fused multiply-add).
//
// One warp per 256-weight block, lane l producing weights 8l .. 8l+7 (two 16-byte stores):
//   IQ2_S  (82 B)  lane l = group l of 8: 10-bit grid index (qs byte | 2 bits of qh), sign byte, 4-bit scale of
//                  its 16 weights; w = ((d * (0.5 + s)) * 0.25) * grid[idx][k], negated where the sign bit is set.
//   IQ3_S  (110 B) lane l = groups 2l, 2l+1 of 4: 9-bit index (qs byte | 1 bit of qh), sign byte l, 4-bit scale of
//                  its 32 weights; w = (d * (1 + 2s)) * grid[idx][k], sign as above.
//   IQ4_XS (136 B) lane l = 8 weights of sub-block l/4 (32 weights): low nibbles for the first 16, high for the rest;
//                  w = (d * (scale - 32)) * kvalues[nibble], scale = 4 low bits | 2 high bits << 4.
// The lookup tables are the caller's (fp32, from gguf-py's grids): IQ2_S [1024][8], IQ3_S [512][4], IQ4_XS [16].
#include <cuda_fp16.h>

#include "layout.cuh"
#include "profile.cuh"

namespace cbmoe {

namespace {

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

__device__ __forceinline__ float f16_at(const uint8_t* p) {
  const unsigned short bits = (unsigned short)(p[0] | (p[1] << 8));
  return __half2float(__ushort_as_half(bits));
}

__device__ __forceinline__ float with_sign(float v, unsigned sign_byte, int k) {
  return ((sign_byte >> k) & 1u) ? -v : v;
}

template <int T>
__global__ void iq_dequant_kernel(const uint8_t* __restrict__ blocks, long long n_blocks,
                                  const float* __restrict__ table, float* __restrict__ out) {
  constexpr int BB = IqFmt<T>::kBytes;
  const int lane = threadIdx.x & 31;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long b = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < n_blocks; b += warps) {
    const uint8_t* blk = blocks + b * BB;
    const float d = f16_at(blk);
    float v[8];
    if constexpr (T == CBMOE_GGML_IQ2_S) {
      const int g = lane;
      const int idx = blk[2 + g] | (((blk[66 + g / 4] >> (2 * (g % 4))) & 3) << 8);
      const int s = (blk[74 + g / 4] >> (4 * ((g / 2) % 2))) & 15;
      const unsigned sg = blk[34 + g];
      const float db = __fmul_rn(__fmul_rn(d, 0.5f + (float)s), 0.25f);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = with_sign(__fmul_rn(db, table[idx * 8 + k]), sg, k);
    } else if constexpr (T == CBMOE_GGML_IQ3_S) {
      const int m = lane / 4;   // 32-weight scale group
      const int s = (blk[106 + m / 2] >> (4 * (m % 2))) & 15;
      const float db = __fmul_rn(d, (float)(1 + 2 * s));
      const unsigned sg = blk[74 + lane];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int G = 2 * lane + h;
        const int idx = blk[2 + G] | (((blk[66 + G / 8] >> (G % 8)) & 1) << 8);
#pragma unroll
        for (int p = 0; p < 4; ++p) v[4 * h + p] = with_sign(__fmul_rn(db, table[idx * 4 + p]), sg, 4 * h + p);
      }
    } else {
      const int i = lane / 4, q = (lane % 4) * 8;   // sub-block, first position inside it
      const int sh = blk[2] | (blk[3] << 8);
      const int sc = (((blk[4 + i / 2] >> (4 * (i % 2))) & 15) | (((sh >> (2 * i)) & 3) << 4)) - 32;
      const float dl = __fmul_rn(d, (float)sc);
      const uint8_t* qs = blk + 8 + 16 * i + (q & 15);
      const int shift = q >= 16 ? 4 : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(dl, table[(qs[j] >> shift) & 15]);
    }
    float4* o = reinterpret_cast<float4*>(out + b * 256 + 8 * lane);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

template <int T>
int launch_iq(const void* blocks, long long n_blocks, const float* table, float* out, cudaStream_t s) {
  long long grid = (n_blocks + 7) / 8;   // 8 warps per CTA, one block each
  const long long cap = (long long)num_sms() * 16;
  if (grid > cap) grid = cap;
  prof_begin(kProfOther, s);
  iq_dequant_kernel<T><<<(int)grid, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), n_blocks, table, out);
  prof_end(kProfOther, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

}  // namespace

}  // namespace cbmoe

using namespace cbmoe;

extern "C" size_t cbmoe_iq_block_bytes(int ggml_type) {
  switch (ggml_type) {
    case CBMOE_GGML_IQ2_S: return IqFmt<CBMOE_GGML_IQ2_S>::kBytes;
    case CBMOE_GGML_IQ3_S: return IqFmt<CBMOE_GGML_IQ3_S>::kBytes;
    case CBMOE_GGML_IQ4_XS: return IqFmt<CBMOE_GGML_IQ4_XS>::kBytes;
    default: return 0;
  }
}

extern "C" int cbmoe_iq_table_shape(int ggml_type, int* entries, int* width) {
  if (!entries || !width) return CBMOE_ERR_INVALID;
  switch (ggml_type) {
    case CBMOE_GGML_IQ2_S: *entries = IqFmt<CBMOE_GGML_IQ2_S>::kEntries; *width = IqFmt<CBMOE_GGML_IQ2_S>::kWidth; break;
    case CBMOE_GGML_IQ3_S: *entries = IqFmt<CBMOE_GGML_IQ3_S>::kEntries; *width = IqFmt<CBMOE_GGML_IQ3_S>::kWidth; break;
    case CBMOE_GGML_IQ4_XS: *entries = IqFmt<CBMOE_GGML_IQ4_XS>::kEntries; *width = IqFmt<CBMOE_GGML_IQ4_XS>::kWidth; break;
    default: return CBMOE_ERR_UNSUPPORTED;
  }
  return CBMOE_OK;
}

extern "C" int cbmoe_iq_dequant(int ggml_type, const void* blocks, long long n_blocks, const float* table, float* out,
                                cudaStream_t stream) {
  if (cbmoe_iq_block_bytes(ggml_type) == 0) return CBMOE_ERR_UNSUPPORTED;
  if (n_blocks < 0) return CBMOE_ERR_INVALID;
  if (n_blocks == 0) return CBMOE_OK;
  if (!blocks || !table || !out || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(table) & 3))
    return CBMOE_ERR_INVALID;
  switch (ggml_type) {
    case CBMOE_GGML_IQ2_S: return launch_iq<CBMOE_GGML_IQ2_S>(blocks, n_blocks, table, out, stream);
    case CBMOE_GGML_IQ3_S: return launch_iq<CBMOE_GGML_IQ3_S>(blocks, n_blocks, table, out, stream);
    default: return launch_iq<CBMOE_GGML_IQ4_XS>(blocks, n_blocks, table, out, stream);
  }
}
