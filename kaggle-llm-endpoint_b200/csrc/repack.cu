// Load-time repack of the expert tables into the kernel layouts (layout.cuh), and the dequant-to-dense kernels
// that check them bit-for-bit against the oracle. Plays the role of the reference's load-time planar repack
// (resident.py:48-60 pack_chip_planes -> planes.py:136-170 pack_planes) and of its XLA dequant
// (planes.py:196-291 dequant_planes, quant8.py:91-99 dequant_tree).
#include "layout.cuh"

namespace cbmoe {
namespace {

// Index j of one CB3 row (little-endian 3-bit stream).
__device__ __forceinline__ uint32_t cb3_get(const uint32_t* row, int j) {
  const int bit = 3 * j;
  const int w = bit >> 5, off = bit & 31;
  uint32_t v = row[w] >> off;
  if (off > 29) v |= row[w + 1] << (32 - off);
  return v & 7u;
}

__global__ void cb3k_repack_idx_kernel(const uint32_t* __restrict__ idx0, const uint32_t* __restrict__ idx1,
                                       int nmat, int E, int rows, int K, uint32_t* __restrict__ out) {
  const int RB = rows / kRowsPerBlock, KS = K / kStageK;
  const long long total = (long long)E * RB * KS * kWarpsPerBlock * nmat * 32;
  const int wpr = K * 3 / 32;
  for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
       tid += (long long)gridDim.x * blockDim.x) {
    long long r = tid;
    const int lane = r % 32; r /= 32;
    const int m = r % nmat; r /= nmat;
    const int w = r % kWarpsPerBlock; r /= kWarpsPerBlock;
    const int ks = r % KS; r /= KS;
    const int rb = r % RB; r /= RB;
    const int e = (int)r;
    const int g = lane >> 2, t = lane & 3;
    const int row_g = rb * kRowsPerBlock + w * kRowsPerWarp + g;
    const uint32_t* src = (m == 0) ? idx0 : idx1;
    const uint32_t* rg = src + ((size_t)e * rows + row_g) * wpr;
    const uint32_t* rh = rg + (size_t)8 * wpr;
    uint32_t words[12];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int kb = ks * kStageK + c * kChunkK + 16 * t;
      uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t qg = cb3_get(rg, kb + 4 * s + i);
          const uint32_t qh = cb3_get(rh, kb + 4 * s + i);
          const int n = 4 * (s & 1) + i;
          if (s < 2) {
            w0 |= qg << (4 * n);
            w2 |= qh << (4 * n);
          } else {
            w1 |= qg << (4 * n);
            w0 |= (qh & 1u) << (4 * n + 3);
            w1 |= ((qh >> 1) & 1u) << (4 * n + 3);
            w2 |= ((qh >> 2) & 1u) << (4 * n + 3);
          }
        }
      }
      words[3 * c] = w0;
      words[3 * c + 1] = w1;
      words[3 * c + 2] = w2;
    }
    uint32_t* dst = out + unit_offset(e, rb, ks, w, m, RB, KS, nmat, kCb3kUnitBytes) / 4 + lane * 12;
#pragma unroll
    for (int i = 0; i < 12; ++i) dst[i] = words[i];
  }
}

__global__ void cb3k_repack_cb_kernel(const uint16_t* __restrict__ cb0, const uint16_t* __restrict__ cb1, int nmat,
                                      int E, int rows, uint32_t* __restrict__ out) {
  const int RB = rows / kRowsPerBlock;
  const long long total = (long long)E * rows * nmat;
  for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
       tid += (long long)gridDim.x * blockDim.x) {
    long long r = tid;
    const int r16 = r % 16; r /= 16;
    const int m = r % nmat; r /= nmat;
    const int w = r % kWarpsPerBlock; r /= kWarpsPerBlock;
    const int rb = r % RB; r /= RB;
    const int e = (int)r;
    const int row = rb * kRowsPerBlock + w * kRowsPerWarp + r16;
    const uint16_t* c = ((m == 0) ? cb0 : cb1) + ((size_t)e * rows + row) * 8;
    uint32_t la = 0, lb = 0, ha = 0, hb = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      la |= (uint32_t)(c[i] & 0xFF) << (8 * i);
      lb |= (uint32_t)(c[4 + i] & 0xFF) << (8 * i);
      ha |= (uint32_t)(c[i] >> 8) << (8 * i);
      hb |= (uint32_t)(c[4 + i] >> 8) << (8 * i);
    }
    uint32_t* dst = out + cb_offset_words(e, rb, w, m, r16, RB, nmat);
    dst[0] = la;
    dst[1] = lb;
    dst[2] = ha;
    dst[3] = hb;
  }
}

// Writes the 16 bf16 of fragment rows (g or g+8) for one chunk, from the dequantized fragments, to dense rows.
__device__ __forceinline__ void store_frag_rows(const uint32_t (&a)[4][4], uint16_t* row_g, uint16_t* row_h) {
  uint32_t* pg = reinterpret_cast<uint32_t*>(row_g);
  uint32_t* ph = reinterpret_cast<uint32_t*>(row_h);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    pg[2 * s] = a[s][0];
    pg[2 * s + 1] = a[s][2];
    ph[2 * s] = a[s][1];
    ph[2 * s + 1] = a[s][3];
  }
}

__global__ void cb3k_dequant_kernel(const uint32_t* __restrict__ idx_k, const uint32_t* __restrict__ cb_k, int nmat,
                                    int E, int rows, int K, uint16_t* __restrict__ out) {
  const int RB = rows / kRowsPerBlock, KS = K / kStageK;
  const long long total = (long long)E * RB * KS * kWarpsPerBlock * nmat * 32;
  for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
       tid += (long long)gridDim.x * blockDim.x) {
    long long r = tid;
    const int lane = r % 32; r /= 32;
    const int m = r % nmat; r /= nmat;
    const int w = r % kWarpsPerBlock; r /= kWarpsPerBlock;
    const int ks = r % KS; r /= KS;
    const int rb = r % RB; r /= RB;
    const int e = (int)r;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t* cbw = cb_k + cb_offset_words(e, rb, w, m, 0, RB, nmat);
    const Codebook cg{cbw[4 * g], cbw[4 * g + 1], cbw[4 * g + 2], cbw[4 * g + 3]};
    const Codebook ch{cbw[4 * (g + 8)], cbw[4 * (g + 8) + 1], cbw[4 * (g + 8) + 2], cbw[4 * (g + 8) + 3]};
    const uint32_t* src = idx_k + unit_offset(e, rb, ks, w, m, RB, KS, nmat, kCb3kUnitBytes) / 4 + lane * 12;
    const int row_g = rb * kRowsPerBlock + w * kRowsPerWarp + g;
    uint16_t* base = out + (((size_t)m * E + e) * rows) * K;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t a[4][4];
      cb3k_dequant_chunk(src[3 * c], src[3 * c + 1], src[3 * c + 2], cg, ch, a);
      const int kb = ks * kStageK + c * kChunkK + 16 * t;
      store_frag_rows(a, base + (size_t)row_g * K + kb, base + (size_t)(row_g + 8) * K + kb);
    }
  }
}

// W8K: one thread per (rb, ks, w, m, c, h, lane) 16-byte group; q is [K, rows] ("[in, out]") int8.
__global__ void w8k_repack_kernel(const int8_t* __restrict__ q0, const int8_t* __restrict__ q1, int nmat, int K,
                                  int rows, uint4* __restrict__ out) {
  const int RB = rows / kRowsPerBlock, KS = K / kStageK;
  const long long total = (long long)RB * KS * kWarpsPerBlock * nmat * 4 * 2 * 32;
  for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
       tid += (long long)gridDim.x * blockDim.x) {
    long long r = tid;
    const int lane = r % 32; r /= 32;
    const int h = r % 2; r /= 2;
    const int c = r % 4; r /= 4;
    const int m = r % nmat; r /= nmat;
    const int w = r % kWarpsPerBlock; r /= kWarpsPerBlock;
    const int ks = r % KS; r /= KS;
    const int rb = (int)r;
    const int g = lane >> 2, t = lane & 3;
    const int row = rb * kRowsPerBlock + w * kRowsPerWarp + g + 8 * h;
    const int kb = ks * kStageK + c * kChunkK + 16 * t;
    const int8_t* src = (m == 0) ? q0 : q1;
    uint32_t v[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i / 4] |= (uint32_t)(uint8_t)src[(size_t)(kb + i) * rows + row] << (8 * (i % 4));
    const size_t unit = unit_offset(0, rb, ks, w, m, RB, KS, nmat, kW8kUnitBytes) / 16;
    out[unit + (c * 2 + h) * 32 + lane] = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

__global__ void w8k_dequant_kernel(const uint4* __restrict__ qk, const float* __restrict__ s0,
                                   const float* __restrict__ s1, int scale_axis, int nmat, int rows, int K,
                                   uint16_t* __restrict__ out) {
  const int RB = rows / kRowsPerBlock, KS = K / kStageK;
  const long long total = (long long)RB * KS * kWarpsPerBlock * nmat * 4 * 32;
  for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
       tid += (long long)gridDim.x * blockDim.x) {
    long long r = tid;
    const int lane = r % 32; r /= 32;
    const int c = r % 4; r /= 4;
    const int m = r % nmat; r /= nmat;
    const int w = r % kWarpsPerBlock; r /= kWarpsPerBlock;
    const int ks = r % KS; r /= KS;
    const int rb = (int)r;
    const int g = lane >> 2, t = lane & 3;
    const int row_g = rb * kRowsPerBlock + w * kRowsPerWarp + g;
    const int kb = ks * kStageK + c * kChunkK + 16 * t;
    const float* s = (m == 0) ? s0 : s1;
    const size_t unit = unit_offset(0, rb, ks, w, m, RB, KS, nmat, kW8kUnitBytes) / 16;
    const uint4 qg = qk[unit + (c * 2 + 0) * 32 + lane];
    const uint4 qh = qk[unit + (c * 2 + 1) * 32 + lane];
    uint32_t a[4][4];
    if (scale_axis == 1) {
      w8k_dequant_chunk(qg, qh, s[row_g], s[row_g + 8], nullptr, a);
    } else {
      w8k_dequant_chunk(qg, qh, 0.f, 0.f, s + kb, a);
    }
    uint16_t* base = out + (size_t)m * rows * K;
    store_frag_rows(a, base + (size_t)row_g * K + kb, base + (size_t)(row_g + 8) * K + kb);
  }
}

int grid_for(long long total, int threads) {
  long long b = (total + threads - 1) / threads;
  const long long cap = (long long)num_sms() * 32;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace cbmoe

using namespace cbmoe;

extern "C" size_t cbmoe_cb3k_idx_bytes(int E, int rows, int K, int nmat) {
  if (E <= 0 || rows <= 0 || K <= 0 || nmat < 1 || nmat > 2) return 0;
  return (size_t)E * rows * K * nmat * 3 / 8;
}

extern "C" size_t cbmoe_cb3k_cb_bytes(int E, int rows, int nmat) {
  if (E <= 0 || rows <= 0 || nmat < 1 || nmat > 2) return 0;
  return (size_t)E * rows * nmat * 16;
}

static bool cb3k_shape_ok(int nmat, int E, int rows, int K) {
  return E > 0 && rows > 0 && K > 0 && rows % kRowsPerBlock == 0 && K % kStageK == 0 && (nmat == 1 || nmat == 2);
}

namespace cbmoe {
namespace {

// CB8 tables of one row from its CB3K codebook words (layout.cuh): T = rint(v 2^s), the largest |v| 2^s in
// [2^14, 2^15) (at most 255 * 2^7 for bf16 entries, so T fits 16 bits); hi = T >> 8, lo = T & 255; row factor 2^-s.
// A row of zeros (or of non-finite entries) gets s = 0.
__global__ void cb8_build_kernel(const uint32_t* __restrict__ cbk, int nmat, int E, int rows,
                                 uint8_t* __restrict__ out) {
  const long long total = (long long)E * rows * nmat;
  for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
       tid += (long long)gridDim.x * blockDim.x) {
    // tid = (((e*RB + rb)*4 + w)*nmat + m)*16 + r16: the CB3K codebook order
    const long long blk = tid / (kRowsPerBlock * nmat);   // e*RB + rb
    const int in_blk = (int)(tid % (kRowsPerBlock * nmat));   // (w*nmat + m)*16 + r16
    const uint32_t* wds = cbk + tid * 4;
    float v[8];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = (wds[i >> 2] >> (8 * (i & 3))) & 0xffu;
      const uint32_t hi = (wds[2 + (i >> 2)] >> (8 * (i & 3))) & 0xffu;
      v[i] = __uint_as_float(((hi << 8) | lo) << 16);
      mx = fmaxf(mx, fabsf(v[i]));
    }
    const int sh = shift_for(mx, 15);
    uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int T = __float2int_rn(ldexpf(v[i], sh));
      hw[i >> 2] |= ((uint32_t)(T >> 8) & 0xffu) << (8 * (i & 3));
      lw[i >> 2] |= ((uint32_t)T & 0xffu) << (8 * (i & 3));
    }
    uint8_t* b = out + blk * (size_t)nmat * kCb8BlockBytes;
    *reinterpret_cast<uint4*>(b + (size_t)in_blk * 16) = make_uint4(hw[0], hw[1], lw[0], lw[1]);
    reinterpret_cast<float*>(b + (size_t)nmat * kRowsPerBlock * 16)[in_blk] = ldexpf(1.f, -sh);
  }
}

}  // namespace
}  // namespace cbmoe

extern "C" size_t cbmoe_cb8_bytes(int E, int rows, int nmat) {
  if (E <= 0 || rows <= 0 || rows % cbmoe::kRowsPerBlock || nmat < 1 || nmat > 2) return 0;
  return (size_t)E * rows * nmat * cbmoe::kCb8RowBytes;
}

extern "C" int cbmoe_cb8_build(const void* cb_k, int nmat, int E, int rows, void* cb8, cudaStream_t stream) {
  if (!cb3k_shape_ok(nmat, E, rows, cbmoe::kStageK) || !cb_k || !cb8 || !aligned16(cb_k) || !aligned16(cb8))
    return CBMOE_ERR_INVALID;
  const long long n = (long long)E * rows * nmat;
  cbmoe::cb8_build_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint32_t*>(cb_k), nmat, E, rows,
                                                                  static_cast<uint8_t*>(cb8));
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

extern "C" int cbmoe_cb3k_repack(const uint32_t* idx0, const uint16_t* cb0, const uint32_t* idx1,
                                 const uint16_t* cb1, int nmat, int E, int rows, int K, void* idx_k, void* cb_k,
                                 cudaStream_t stream) {
  if (!cb3k_shape_ok(nmat, E, rows, K) || !idx0 || !cb0 || !idx_k || !cb_k) return CBMOE_ERR_INVALID;
  if (nmat == 2 && (!idx1 || !cb1)) return CBMOE_ERR_INVALID;
  if (!aligned16(idx_k) || !aligned16(cb_k)) return CBMOE_ERR_INVALID;
  const long long n_idx = (long long)E * (rows / kRowsPerBlock) * (K / kStageK) * kWarpsPerBlock * nmat * 32;
  cb3k_repack_idx_kernel<<<grid_for(n_idx, 256), 256, 0, stream>>>(idx0, idx1, nmat, E, rows, K,
                                                                     static_cast<uint32_t*>(idx_k));
  CBMOE_CUDA_TRY(cudaGetLastError());
  const long long n_cb = (long long)E * rows * nmat;
  cb3k_repack_cb_kernel<<<grid_for(n_cb, 256), 256, 0, stream>>>(cb0, cb1, nmat, E, rows,
                                                                   static_cast<uint32_t*>(cb_k));
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

extern "C" int cbmoe_cb3k_dequant(const void* idx_k, const void* cb_k, int nmat, int E, int rows, int K,
                                  uint16_t* out, cudaStream_t stream) {
  if (!cb3k_shape_ok(nmat, E, rows, K) || !idx_k || !cb_k || !out) return CBMOE_ERR_INVALID;
  const long long n = (long long)E * (rows / kRowsPerBlock) * (K / kStageK) * kWarpsPerBlock * nmat * 32;
  cb3k_dequant_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint32_t*>(idx_k),
                                                              static_cast<const uint32_t*>(cb_k), nmat, E, rows, K,
                                                              out);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

extern "C" size_t cbmoe_w8k_bytes(int rows, int K, int nmat) {
  if (rows <= 0 || K <= 0 || nmat < 1 || nmat > 2) return 0;
  return (size_t)rows * K * nmat;
}

extern "C" int cbmoe_w8k_repack(const int8_t* q0, const int8_t* q1, int nmat, int K, int rows, void* qk,
                                cudaStream_t stream) {
  if (!cb3k_shape_ok(nmat, 1, rows, K) || !q0 || !qk || (nmat == 2 && !q1) || !aligned16(qk))
    return CBMOE_ERR_INVALID;
  const long long n = (long long)(rows / kRowsPerBlock) * (K / kStageK) * kWarpsPerBlock * nmat * 4 * 2 * 32;
  w8k_repack_kernel<<<grid_for(n, 256), 256, 0, stream>>>(q0, q1, nmat, K, rows, static_cast<uint4*>(qk));
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

extern "C" int cbmoe_w8k_dequant(const void* qk, const float* s0, const float* s1, int scale_axis, int nmat,
                                 int rows, int K, uint16_t* out, cudaStream_t stream) {
  if (!cb3k_shape_ok(nmat, 1, rows, K) || !qk || !s0 || !out || (nmat == 2 && !s1) ||
      (scale_axis != 0 && scale_axis != 1) || !aligned16(qk))
    return CBMOE_ERR_INVALID;
  const long long n = (long long)(rows / kRowsPerBlock) * (K / kStageK) * kWarpsPerBlock * nmat * 4 * 32;
  w8k_dequant_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint4*>(qk), s0, s1, scale_axis,
                                                             nmat, rows, K, out);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}
