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
  static constexpr int kAuxBytes = NMAT * 1024;                // codebooks (CB3K) or scales (W8K) of the item
  static constexpr int kBCopy = kStageK * 2 * (HILO ? 2 : 1);  // bytes of one token row per stage
  static constexpr int kBRow = kBCopy + 16;                    // padded: conflict-free fragment loads
  static constexpr int kBBytes = NT * 8 * kBRow;
  static constexpr int kStage = kWBytes + kAuxBytes + kBBytes;
  static constexpr int kBarBytes = ((16 + 32) * NSTAGE + 127) / 128 * 128;   // barriers + stage headers
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
  return np * p.RB * p.KQ;
}

// Auxiliary bytes the producer copies into a stage: the item's codebooks (CB3K) or row scales (W8K
// per-output-channel) on the item's first stage, the stage's input scales (W8K per-input-row) on every stage.
template <int FMT, int NMAT>
__device__ __forceinline__ int aux_bytes(const DecodeParams& p, bool first) {
  if constexpr (FMT == kFmtCB3) return first ? NMAT * 1024 : 0;
  else return p.scale_axis == 1 ? (first ? NMAT * kRowsPerBlock * 4 : 0) : NMAT * kStageK * 4;
}

// What the producer tells the consumers about the stage it filled (written before the stage's full-barrier
// arrive, which releases it). item < 0 ends the consumers' loop.
struct StageHdr {
  int item, e, row0, cnt;
  int rb, kq, ks, flags;  // flags: 1 = first stage of the item, 2 = last stage of the item
};

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32)); }

// Sum over token `row`'s routed slots of w * y_sorted[slot row][r]. The slot rows and weights are loaded first and
// the (up to 16 at a time) y loads issued together, so the epilogue waits for two memory round trips, not 2k.
__device__ __forceinline__ float routed_sum(const DecodeParams& p, int row, int r) {
  float v = 0.f;
  for (int q0 = 0; q0 < p.topk; q0 += 16) {
    int rs[16];
    float wt[16], y[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const bool in = q0 + q < p.topk;
      rs[q] = in ? p.row_slot[row * p.topk + q0 + q] : -1;
      wt[q] = in ? p.wts[row * p.topk + q0 + q] : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 16; ++q) y[q] = rs[q] >= 0 ? p.y_sorted[(size_t)rs[q] * p.rows + r] : 0.f;
#pragma unroll
    for (int q = 0; q < 16; ++q) v += wt[q] * y[q];
  }
  return v;
}

// The kernel proper; HILO is a template argument so the B staging size is a compile-time constant.
//   producer warp: takes items (pass, 64-row block, K split) from the next-item counter (or round-robin), and for
//                  each of the item's 256-input stages fills a ring slot: header, weights, aux, the pass's B rows;
//   consumer warps: dequantize + MMA per stage, then the item's epilogue; with K splits, each split stores its
//                  partial sums and the last split to arrive adds them up and runs the epilogue.
template <int FMT, int NMAT, int NT, int EPI, int HILO, int NSTAGE>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel_t(const DecodeParams p) {
  using SM = DecodeSmem<FMT, NMAT, NT, HILO, NSTAGE>;
  constexpr int kPassTokens = NT * 8;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NSTAGE;
  StageHdr* hdr = reinterpret_cast<StageHdr*>(smem + 16 * NSTAGE);
  uint8_t* stages = smem + SM::kBarBytes;
  __shared__ int s_flag;

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
  const int RB = p.RB, KS = p.KS, KQ = p.KQ;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------------------------------ producer
    int st = 0;
    uint32_t ph = 0;
    int iter = 0;
    for (;;) {
      int item = 0;
      if (lane == 0) item = p.sched ? atomicAdd(p.sched, 1) : (int)blockIdx.x + iter * (int)gridDim.x;
      item = __shfl_sync(0xffffffffu, item, 0);
      ++iter;
      if (item >= n_items) {
        bool ok = true;
        if (lane == 0) {
          ok = mbar_wait_sleepy(&empty[st], ph ^ 1);
          if (ok) {
            hdr[st].item = -1;
            mbar_arrive(&full[st]);
          }
        }
        return;
      }
      const int kq = item % KQ, rest = item / KQ;
      const int rb = rest % RB, pass = rest / RB;
      const PassInfo pi = get_pass(p, pass, kPassTokens);
      if (pi.e < 0 || pi.e >= p.E || pi.cnt <= 0) continue;
      int brow = -1;
      if (lane < pi.cnt) brow = p.tok_row ? p.tok_row[pi.row0 + lane] : pi.row0 + lane;
      const int n_copies = __popc(__ballot_sync(0xffffffffu, brow >= 0));
      const int ks0 = kq * KS / KQ, ks1 = (kq + 1) * KS / KQ;
      for (int ks = ks0; ks < ks1; ++ks) {
        const bool first = ks == ks0;
        const int aux = aux_bytes<FMT, NMAT>(p, first);
        bool ok = true;
        if (lane == 0) {
          ok = mbar_wait_sleepy(&empty[st], ph ^ 1);
          if (ok) {
            hdr[st] = {item, pi.e, pi.row0, pi.cnt, rb, kq, ks, (first ? 1 : 0) | (ks == ks1 - 1 ? 2 : 0)};
            mbar_arrive_expect_tx(&full[st], SM::kWBytes + aux + n_copies * SM::kBCopy);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) return;
        uint8_t* sw = stages + st * SM::kStage;
        uint8_t* sa = sw + SM::kWBytes;
        if (lane == 0) {
          const uint8_t* src = p.wq + unit_offset(pi.e, rb, ks, 0, 0, RB, KS, NMAT, SM::kUnit);
          bulk_g2s(sw, src, SM::kWBytes, &full[st]);
        }
        if (aux > 0 && lane < NMAT) {
          if constexpr (FMT == kFmtCB3) {
            if (lane == 0) bulk_g2s(sa, p.cb + cb_offset_words(pi.e, rb, 0, 0, 0, RB, NMAT), aux, &full[st]);
          } else {
            const float* sc = (lane == 0) ? p.s0 : p.s1;
            const int per = aux / NMAT;
            const float* src = (p.scale_axis == 1) ? sc + rb * kRowsPerBlock : sc + ks * kStageK;
            bulk_g2s(sa + lane * per, src, per, &full[st]);
          }
        }
        if (brow >= 0) {
          const uint16_t* src = p.b + (size_t)brow * (p.K * (HILO ? 2 : 1)) + (size_t)ks * kStageK * (HILO ? 2 : 1);
          bulk_g2s(sw + SM::kWBytes + SM::kAuxBytes + lane * SM::kBRow, src, SM::kBCopy, &full[st]);
        }
        if (++st == NSTAGE) {
          st = 0;
          ph ^= 1;
        }
      }
    }
  }

  // -------------------------------------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  int st = 0;
  uint32_t ph = 0;
  Codebook cbg[NMAT], cbh[NMAT];
  float sg[NMAT], sh[NMAT];
  float acc[NMAT][NT][4];
  for (;;) {
    if (!mbar_wait(&full[st], ph)) return;
    const StageHdr h = hdr[st];
    if (h.item < 0) return;
    const uint8_t* sw = stages + st * SM::kStage;
    const uint8_t* sa = sw + SM::kWBytes;
    const uint8_t* sb = sa + SM::kAuxBytes;

    if (h.flags & 1) {
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        if constexpr (FMT == kFmtCB3) {
          const uint4 ca = lds128(sa + ((warp * NMAT + m) * 16 + g) * 16);
          const uint4 cb = lds128(sa + ((warp * NMAT + m) * 16 + g + 8) * 16);
          cbg[m] = {ca.x, ca.y, ca.z, ca.w};
          cbh[m] = {cb.x, cb.y, cb.z, cb.w};
          sg[m] = sh[m] = 0.f;
        } else {
          const float* sc = reinterpret_cast<const float*>(sa) + m * kRowsPerBlock + warp * kRowsPerWarp;
          sg[m] = (p.scale_axis == 1) ? sc[g] : 0.f;
          sh[m] = (p.scale_axis == 1) ? sc[g + 8] : 0.f;
          cbg[m] = cbh[m] = {0, 0, 0, 0};
        }
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[m][n][i] = 0.f;
      }
    }

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
        if (n == 0 || n * 8 < h.cnt) {   // a pass has at least one token
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
          if (p.scale_axis == 0) ksc = reinterpret_cast<const float*>(sa) + m * kStageK + c * kChunkK + 16 * t;
          w8k_dequant_chunk(qg, qh, sg[m], sh[m], ksc, a);
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            if (n == 0 || n * 8 < h.cnt) {
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
    if (!(h.flags & 2)) continue;

    // ---------------------------------------------------------------------------------- item epilogue
    const int rowbase = h.rb * kRowsPerBlock + warp * kRowsPerWarp;
    if (KQ > 1) {
      // store this split's partial sums; the last split to arrive reduces them and runs the epilogue
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = n * 8 + 2 * t + (i & 1);
            const int r = rowbase + g + ((i & 2) ? 8 : 0);
            if (j < h.cnt)
              p.part[(((size_t)h.kq * p.part_rows + h.row0 + j) * NMAT + m) * p.rows + r] = acc[m][n][i];
          }
      __threadfence();
      consumer_bar();
      if (threadIdx.x == 0) {
        const int slot = (h.item / KQ);
        s_flag = (atomicAdd(&p.done[slot], 1) == KQ - 1) ? 1 : 0;
        if (s_flag) p.done[slot] = 0;   // every split has arrived: ready for the next launch
      }
      consumer_bar();
      if (!s_flag) continue;
      __threadfence();
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = n * 8 + 2 * t + (i & 1);
            const int r = rowbase + g + ((i & 2) ? 8 : 0);
            float v = 0.f;
            if (j < h.cnt)
              for (int q = 0; q < KQ; ++q)
                v += __ldcg(&p.part[(((size_t)q * p.part_rows + h.row0 + j) * NMAT + m) * p.rows + r]);
            acc[m][n][i] = v;
          }
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = n * 8 + 2 * t + (i & 1);
        const int r = rowbase + g + ((i & 2) ? 8 : 0);
        if (j >= h.cnt) continue;
        const int row = h.row0 + j;
        if constexpr (EPI == kEpiSwiglu) {
          const float hv = swiglu_clamped(acc[0][n][i], acc[NMAT - 1][n][i], p.limit);
          const __nv_bfloat16 hi = __float2bfloat16_rn(hv);
          const __nv_bfloat16 lo = __float2bfloat16_rn(hv - __bfloat162float(hi));
          uint16_t* dst = p.h_out + (size_t)row * (2 * p.rows) + (r / kStageK) * (2 * kStageK) + (r % kStageK);
          dst[0] = *reinterpret_cast<const uint16_t*>(&hi);
          dst[kStageK] = *reinterpret_cast<const uint16_t*>(&lo);
        } else if constexpr (EPI == kEpiStore) {
          p.y_out[(size_t)row * p.rows + r] = acc[0][n][i];
        } else {
          float v = acc[0][n][i];
          if (p.y_sorted != nullptr) v += routed_sum(p, row, r);
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
    for (int q0 = 0; q0 < topk; q0 += 8) {
      int rs[8];
      float wt[8], yy[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool in = q0 + q < topk;
        rs[q] = in ? row_slot[n * topk + q0 + q] : -1;
        wt[q] = in ? wts[n * topk + q0 + q] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) yy[q] = rs[q] >= 0 ? y_sorted[(size_t)rs[q] * H + r] : 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) v += wt[q] * yy[q];
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

#ifndef CBMOE_STAGES_CB3
#define CBMOE_STAGES_CB3 3
#endif
constexpr int kStagesCB3 = CBMOE_STAGES_CB3;
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
