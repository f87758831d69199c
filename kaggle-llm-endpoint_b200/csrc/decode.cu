// Decode / small-batch expert kernels: fused dequant + tensor-core matvec over the kernel layouts (layout.cuh).
//
// Counterpart of the reference's moe_matvec Pallas kernel (pallas_moe.py:238-307) and of `_apply_kernel`'s
// gate/up -> swiglu -> down composition (resident.py:110-120), with two changes of design for B200:
//   * work is per (expert pass, 64-row block), not per slot: a pass is up to 8*NT tokens routed to one expert, so
//     an expert's weights stream from HBM once per pass instead of once per (token, slot) pair;
//   * the weights never leave registers in dense form: a producer warp streams 256-input stages of packed bits
//     into shared memory with bulk async copies (mbarrier pipeline, NSTAGE deep); four consumer warps turn them
//     into bf16 tensor-core fragments with byte permutes (CB3K) or int8 -> fp32 * scale -> bf16 (W8K) and
//     multiply them with mma.sync m16n8k16 against the pass's tokens, accumulating in fp32.
// Persistent grid: gridDim = SMs x resident CTAs; CTA b takes items b, b + gridDim, ... of (pass, row block).
// Epilogues: SWIGLU (gate+up -> h stored as bf16 hi + bf16 lo, so the down matvec sees h to ~16 mantissa bits),
// STORE (fp32 rows), COMBINE (shared-expert down + the routed slots' weighted sum -> bf16 layer output).
#include "decode.cuh"
#include "profile.cuh"

namespace cbmoe {

template <int FMT, int NMAT, int NT, int HILO, int NSTAGE>
struct DecodeSmem {
  static constexpr int kUnit = Fmt<FMT>::kUnitBytes;
  static constexpr int kWBytes = kConsumerWarps * NMAT * kUnit;
  static constexpr int kBCopy = kStageK * 2 * (HILO ? 2 : 1);  // bytes of one token row per stage
  static constexpr int kBRow = kBCopy + 16;                    // padded: conflict-free fragment loads
  static constexpr int kBBytes = NT * 8 * kBRow;
  static constexpr int kStage = kWBytes + kBBytes;
  static constexpr int kBarBytes = 128;
  static constexpr int kTotal = kBarBytes + NSTAGE * kStage;
};

struct PassInfo {
  int e, row0, cnt;
};

__device__ __forceinline__ PassInfo get_pass(const DecodeParams& p, int pass, int pass_tokens) {
  if (p.pass_expert == nullptr) {
    const int row0 = pass * pass_tokens;
    return {0, row0, min(pass_tokens, p.N - row0)};
  }
  return {p.pass_expert[pass], p.pass_row0[pass], p.pass_cnt[pass]};
}

__device__ __forceinline__ int count_items(const DecodeParams& p, int pass_tokens) {
  const int np = (p.pass_expert == nullptr) ? (p.N + pass_tokens - 1) / pass_tokens : *p.n_pass;
  return np * p.RB;
}

// The kernel proper; HILO is a template argument so the B staging size is a compile-time constant.
template <int FMT, int NMAT, int NT, int EPI, int HILO, int NSTAGE>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel_t(const DecodeParams p) {
  using SM = DecodeSmem<FMT, NMAT, NT, HILO, NSTAGE>;
  constexpr int kPassTokens = NT * 8;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  uint8_t* stages = smem + SM::kBarBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int n_items = count_items(p, kPassTokens);
  const int RB = p.RB, KS = p.KS;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------------------------------ producer
    int st = 0;
    uint32_t ph = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int pass = item / RB, rb = item % RB;
      const PassInfo pi = get_pass(p, pass, kPassTokens);
      if (pi.e < 0 || pi.e >= p.E) continue;  // consumers skip the same item
      int brow = -1;
      if (lane < pi.cnt) brow = p.tok_row ? p.tok_row[pi.row0 + lane] : pi.row0 + lane;
      const int n_copies = __popc(__ballot_sync(0xffffffffu, brow >= 0));
      for (int ks = 0; ks < KS; ++ks) {
        bool ok = true;
        if (lane == 0) {
          ok = mbar_wait(&empty[st], ph ^ 1);
          if (ok) mbar_arrive_expect_tx(&full[st], SM::kWBytes + n_copies * SM::kBCopy);
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) return;
        uint8_t* sw = stages + st * SM::kStage;
        if (lane == 0) {
          const uint8_t* src = p.wq + unit_offset(pi.e, rb, ks, 0, 0, RB, KS, NMAT, SM::kUnit);
          bulk_g2s(sw, src, SM::kWBytes, &full[st]);
        }
        if (lane < pi.cnt && brow >= 0) {
          const uint16_t* src = p.b + (size_t)brow * (p.K * (HILO ? 2 : 1)) + (size_t)ks * kStageK * (HILO ? 2 : 1);
          bulk_g2s(sw + SM::kWBytes + lane * SM::kBRow, src, SM::kBCopy, &full[st]);
        }
        if (++st == NSTAGE) {
          st = 0;
          ph ^= 1;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  int st = 0;
  uint32_t ph = 0;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int pass = item / RB, rb = item % RB;
    const PassInfo pi = get_pass(p, pass, kPassTokens);
    if (pi.e < 0 || pi.e >= p.E) continue;
    const int rowbase = rb * kRowsPerBlock + warp * kRowsPerWarp;

    Codebook cbg[NMAT], cbh[NMAT];
    float sg[NMAT], sh[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      if constexpr (FMT == kFmtCB3) {
        const uint4* c4 = reinterpret_cast<const uint4*>(p.cb + cb_offset_words(pi.e, rb, warp, m, 0, RB, NMAT));
        const uint4 a = c4[g], b = c4[g + 8];
        cbg[m] = {a.x, a.y, a.z, a.w};
        cbh[m] = {b.x, b.y, b.z, b.w};
        sg[m] = sh[m] = 0.f;
      } else {
        const float* s = (m == 0) ? p.s0 : p.s1;
        sg[m] = (p.scale_axis == 1) ? s[rowbase + g] : 0.f;
        sh[m] = (p.scale_axis == 1) ? s[rowbase + g + 8] : 0.f;
        cbg[m] = cbh[m] = {0, 0, 0, 0};
      }
    }

    float acc[NMAT][NT][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][n][i] = 0.f;

    for (int ks = 0; ks < KS; ++ks) {
      if (!mbar_wait(&full[st], ph)) return;
      const uint8_t* sw = stages + st * SM::kStage;
      const uint8_t* sb = sw + SM::kWBytes;

      uint32_t wd[NMAT][12];
      if constexpr (FMT == kFmtCB3) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          const uint8_t* u = sw + (warp * NMAT + m) * SM::kUnit + lane * 48;
#pragma unroll
          for (int v = 0; v < 3; ++v) {
            const uint4 q = lds128(u + 16 * v);
            wd[m][4 * v] = q.x;
            wd[m][4 * v + 1] = q.y;
            wd[m][4 * v + 2] = q.z;
            wd[m][4 * v + 3] = q.w;
          }
        }
      }

#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t bf[NT][8];
        uint32_t bl[NT][HILO ? 8 : 1];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (n * 8 < pi.cnt) {
            const uint8_t* r = sb + (n * 8 + g) * SM::kBRow + c * 128 + 32 * t;
            const uint4 x0 = lds128(r), x1 = lds128(r + 16);
            bf[n][0] = x0.x; bf[n][1] = x0.y; bf[n][2] = x0.z; bf[n][3] = x0.w;
            bf[n][4] = x1.x; bf[n][5] = x1.y; bf[n][6] = x1.z; bf[n][7] = x1.w;
            if constexpr (HILO) {
              const uint4 y0 = lds128(r + 512), y1 = lds128(r + 528);
              bl[n][0] = y0.x; bl[n][1] = y0.y; bl[n][2] = y0.z; bl[n][3] = y0.w;
              bl[n][4] = y1.x; bl[n][5] = y1.y; bl[n][6] = y1.z; bl[n][7] = y1.w;
            }
          }
        }
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          uint32_t a[4][4];
          if constexpr (FMT == kFmtCB3) {
            cb3k_dequant_chunk(wd[m][3 * c], wd[m][3 * c + 1], wd[m][3 * c + 2], cbg[m], cbh[m], a);
          } else {
            const uint8_t* u = sw + (warp * NMAT + m) * SM::kUnit;
            const uint4 qg = lds128(u + ((c * 2 + 0) * 32 + lane) * 16);
            const uint4 qh = lds128(u + ((c * 2 + 1) * 32 + lane) * 16);
            const float* ksc = nullptr;
            if (p.scale_axis == 0) ksc = ((m == 0) ? p.s0 : p.s1) + ks * kStageK + c * kChunkK + 16 * t;
            w8k_dequant_chunk(qg, qh, sg[m], sh[m], ksc, a);
          }
#pragma unroll
          for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              if (n * 8 < pi.cnt) {
                mma_bf16(acc[m][n], a[s], bf[n][2 * s], bf[n][2 * s + 1]);
                if constexpr (HILO) mma_bf16(acc[m][n], a[s], bl[n][2 * s], bl[n][2 * s + 1]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (++st == NSTAGE) {
        st = 0;
        ph ^= 1;
      }
    }

    // ------------------------------------------------------------------------------------------ epilogue
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = n * 8 + 2 * t + (i & 1);
        const int r = rowbase + g + ((i & 2) ? 8 : 0);
        if (j >= pi.cnt) continue;
        const int row = pi.row0 + j;
        if constexpr (EPI == kEpiSwiglu) {
          const float h = swiglu_clamped(acc[0][n][i], acc[NMAT - 1][n][i], p.limit);
          const __nv_bfloat16 hi = __float2bfloat16_rn(h);
          const __nv_bfloat16 lo = __float2bfloat16_rn(h - __bfloat162float(hi));
          uint16_t* dst = p.h_out + (size_t)row * (2 * p.rows) + (r / kStageK) * (2 * kStageK) + (r % kStageK);
          dst[0] = *reinterpret_cast<const uint16_t*>(&hi);
          dst[kStageK] = *reinterpret_cast<const uint16_t*>(&lo);
        } else if constexpr (EPI == kEpiStore) {
          p.y_out[(size_t)row * p.rows + r] = acc[0][n][i];
        } else {
          float v = acc[0][n][i];
          if (p.y_sorted != nullptr) {
            for (int q = 0; q < p.topk; ++q) {
              const int rs = p.row_slot[row * p.topk + q];
              if (rs >= 0) v += p.wts[row * p.topk + q] * p.y_sorted[(size_t)rs * p.rows + r];
            }
          }
          const __nv_bfloat16 o = __float2bfloat16_rn(v);
          p.out_bf16[(size_t)row * p.rows + r] = *reinterpret_cast<const uint16_t*>(&o);
        }
      }
    }
  }
}

// Routed-only combine: y[n][r] = sum_j w[n][j] * y_sorted[row_slot[n][j]][r] (einsum "nkd,nk->nd").
__global__ void combine_kernel(const float* __restrict__ y_sorted, const int* __restrict__ row_slot,
                               const float* __restrict__ wts, int N, int topk, int H, float* __restrict__ y) {
  const long long total = (long long)N * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / H), r = (int)(i % H);
    float v = 0.f;
    for (int q = 0; q < topk; ++q) {
      const int rs = row_slot[n * topk + q];
      if (rs >= 0) v += wts[n * topk + q] * y_sorted[(size_t)rs * H + r];
    }
    y[i] = v;
  }
}

// ------------------------------------------------------------------------------------------------ launch
template <int FMT, int NMAT, int NT, int EPI, int HILO, int NSTAGE>
int launch_decode_t(const DecodeParams& p, int kind, cudaStream_t stream) {
  using SM = DecodeSmem<FMT, NMAT, NT, HILO, NSTAGE>;
  auto kern = decode_kernel_t<FMT, NMAT, NT, EPI, HILO, NSTAGE>;
  static int grid = 0;
  if (grid == 0) {
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kTotal));
    int per_sm = 0;
    CBMOE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecodeThreads, SM::kTotal));
    grid = num_sms() * (per_sm > 0 ? per_sm : 1);
  }
  prof_begin(kind, stream);
  kern<<<grid, kDecodeThreads, SM::kTotal, stream>>>(p);
  prof_end(kind, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

constexpr int kStagesCB3 = 4;
constexpr int kStagesW8 = 3;

template <int FMT, int NMAT, int EPI, int HILO>
int launch_decode_nt(const DecodeParams& p, int nt, int kind, cudaStream_t stream) {
  constexpr int NS = (FMT == kFmtCB3) ? kStagesCB3 : kStagesW8;
  switch (nt) {
    case 1: return launch_decode_t<FMT, NMAT, 1, EPI, HILO, NS>(p, kind, stream);
    case 2: return launch_decode_t<FMT, NMAT, 2, EPI, HILO, NS>(p, kind, stream);
    default: return launch_decode_t<FMT, NMAT, 4, EPI, HILO, NS>(p, kind, stream);
  }
}

int launch_combine(const float* y_sorted, const int* row_slot, const float* wts, int N, int topk, int H, float* y,
                   cudaStream_t stream) {
  const long long total = (long long)N * H;
  int blocks = (int)((total + 255) / 256);
  if (blocks > num_sms() * 8) blocks = num_sms() * 8;
  if (blocks < 1) blocks = 1;
  prof_begin(kProfCombine, stream);
  combine_kernel<<<blocks, 256, 0, stream>>>(y_sorted, row_slot, wts, N, topk, H, y);
  prof_end(kProfCombine, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

// Explicit entry points used by capi.cu.
int decode_cb3_gateup(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtCB3, 2, kEpiSwiglu, 0>(p, nt, kProfCb3GateUp, s);
}
int decode_cb3_down(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtCB3, 1, kEpiStore, 1>(p, nt, kProfCb3Down, s);
}
int decode_cb3_single(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtCB3, 1, kEpiStore, 0>(p, nt, kProfCb3Single, s);
}
int decode_w8_gateup(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtW8, 2, kEpiSwiglu, 0>(p, nt, kProfW8GateUp, s);
}
int decode_w8_down_combine(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtW8, 1, kEpiCombine, 1>(p, nt, kProfW8DownCombine, s);
}
int decode_w8_single(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtW8, 1, kEpiStore, 0>(p, nt, kProfW8Single, s);
}

}  // namespace cbmoe
