// Grouped expert GEMM on tcgen05 tensor cores: the prefill / large-batch path. Counterpart of the reference's
// moe_ragged_gateup / moe_ragged_down Pallas kernels (pallas_moe.py:622-755) and of the int8 dense projections
// (quant8.dequant_tree + dot, quant8.py:91-99).
//
//   D[w, t] = sum_k W_e[w, k] * X[t, k]     w: 128 weight rows of expert e (tcgen05 M = 128)
//                                           t: up to TN sorted token rows routed to e (tcgen05 N): 256 for the
//                                              routed CB3 passes, 128 / 256 for the int8 projections
// A 128 x 16 slice of A costs the tensor core about as long whatever N (up to 256) it meets, so the widest pass
// that the accumulators allow does the most work per dequantized tile.
// The weights are dequantized ONCE per (pass, 128-row tile) straight into the tensor core's shared-memory
// operand layout; the tokens come in by TMA. One CTA per SM, 11 warps:
//   warp 0       packed-weight producer: bulk copies of CB3K / W8K bits (+ codebooks / scales) into a ring
//   warp 1       TMEM owner and MMA issuer (one thread): tcgen05.mma kind::f16, fp32 accumulators in TMEM
//   warp 2       token producer: 2-D TMA loads of 128 x 64 bf16 tiles (128-byte swizzle)
//   warps 3-6    dequant: packed bits -> bf16 A tiles (the decode kernels' register dequant) -> shared memory
//   warps 7-10   epilogue: tcgen05.ld of the accumulators -> SwiGLU (gate/up) or store -> bf16 rows
// Barriers: per MMA stage full (4 dequant warps + token TMA) / empty (MMA commit); per packed slot full / empty;
// tmem_full / tmem_empty (MMA commit / 4 epilogue warps) per accumulator buffer: two buffers where they fit TMEM,
// so the epilogue of one item overlaps the MMAs of the next (gate/up with 256-token passes has one). Every wait is bounded; a role that gives up sets
// CBMOE_DEVERR_TIMEOUT and falls through to the final barrier, after which warp 1 frees TMEM.
// Items (pass, 128-row tile) are dealt round-robin to the persistent CTAs. No multicast anywhere.
#include <cudaTypedefs.h>
#include <mutex>

#include "grouped.cuh"
#include "profile.cuh"
#include "umma.cuh"

namespace cbmoe {

namespace {

constexpr int kGrpThreads = 11 * 32;
constexpr int kWarpPk = 0, kWarpMma = 1, kWarpTok = 2, kWarpDq0 = 3, kWarpEpi0 = 7;

template <int FMT, int NMAT, int TN>
struct GrpCfg {
  static constexpr int kGK = (FMT == kFmtCB3) ? kStageK : kChunkK;      // K per packed slot
  static constexpr int kChunks = kGK / kChunkK;                          // MMA stages per packed slot
  // packed slot: the tile's 8 units (2 row blocks x 4 warps) x NMAT, then aux
  static constexpr int kUnitSlice = (FMT == kFmtCB3) ? kCb3kUnitBytes : 1024;
  static constexpr int kPkData = 2 * kWarpsPerBlock * NMAT * kUnitSlice;
  static constexpr int kPkAux = (FMT == kFmtCB3) ? 2 * NMAT * 1024 : NMAT * kGrpTileM * 4;
  static constexpr int kPkBytes = kPkData + kPkAux;
  // CB3: one slot covers 4 MMA stages and the dequant warps free it as soon as its bits are in registers;
  // W8: one slot per MMA stage, so several are in flight
  static constexpr int kNpk = (FMT == kFmtCB3) ? 1 : 3;
  static constexpr int kATile = kGrpTileM * 128;                         // 16 KB: 128 rows x 64 bf16
  static constexpr int kBTile = TN * 128;                                // 16 / 32 KB
  static constexpr int kStage = NMAT * kATile + kBTile;
  static constexpr int kNStage = (FMT == kFmtW8) ? ((NMAT == 2 || TN == 256) ? 3 + (TN == 256) : 5)
                                                 : (TN == 256 ? (NMAT == 2 ? 3 : 4) : (NMAT == 2 ? 4 : 6));
  static constexpr int kAccCols = NMAT * TN;                             // one accumulator buffer
  // Two buffers (the epilogue of one item overlaps the MMAs of the next) where they fit the 512 TMEM columns;
  // gate/up with 256-token passes has one, so its epilogue and the next item's MMAs take turns.
  static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccBufs * kAccCols;
  static_assert(kAccCols <= 512, "TMEM budget");
  static constexpr int kBarOff = kNStage * kStage + kNpk * kPkBytes;
  static constexpr int kSmem = 1024 + kBarOff + 256;                     // +1024: manual 1 KB alignment
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

struct ItemInfo {
  int e, row0, cnt, rt;
};

template <int TN>
__device__ __forceinline__ int grp_n_items(const GroupedParams& p) {
  const int np = p.pass_expert ? *p.n_pass : (p.N + TN - 1) / TN;
  return np * (p.rows / kGrpTileM);
}

template <int TN>
__device__ __forceinline__ ItemInfo grp_item(const GroupedParams& p, int item) {
  const int RT = p.rows / kGrpTileM;
  const int pass = item / RT, rt = item % RT;
  if (p.pass_expert == nullptr) {
    const int row0 = pass * TN;
    return {0, row0, min(TN, p.N - row0), rt};
  }
  return {p.pass_expert[pass], p.pass_row0[pass], p.pass_cnt[pass], rt};
}

__device__ __forceinline__ bool item_ok(const GroupedParams& p, const ItemInfo& it) {
  return it.e >= 0 && it.e < p.E && it.cnt > 0;
}

template <int FMT, int NMAT, int EPI, int TN>
__global__ void __launch_bounds__(kGrpThreads, 1) grouped_kernel(const GroupedParams p,
                                                                 const __grid_constant__ CUtensorMap tmap_b) {
  using C = GrpCfg<FMT, NMAT, TN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* packed = smem + C::kNStage * C::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = full + C::kNStage;
  uint64_t* pk_full = empty + C::kNStage;
  uint64_t* pk_empty = pk_full + C::kNpk;
  uint64_t* tm_full = pk_empty + C::kNpk;     // [2]
  uint64_t* tm_empty = tm_full + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tm_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kNStage; ++s) {
      mbar_init(&full[s], kWarpsPerBlock + 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < C::kNpk; ++s) {
      mbar_init(&pk_full[s], 1);
      mbar_init(&pk_empty[s], kWarpsPerBlock);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], kWarpsPerBlock);
    }
    fence_mbar_init();
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, C::kTmemCols);
  if (warp == kWarpTok && lane == 0) prefetch_tmap(&tmap_b);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int n_items = grp_n_items<TN>(p);
  const int RB = p.rows / kRowsPerBlock, KS256 = p.K / kStageK, KS64 = p.K / kChunkK;
  const int KG = p.K / C::kGK;

  if (warp == kWarpPk) {
    // -------------------------------------------------------------------------- packed-weight producer
    int ps = 0;
    uint32_t pph = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const ItemInfo it = grp_item<TN>(p, item);
      if (!item_ok(p, it)) continue;
      for (int kg = 0; kg < KG; ++kg) {
        const bool first = kg == 0;
        int aux = 0;
        if constexpr (FMT == kFmtCB3) aux = first ? C::kPkAux : 0;
        else aux = (p.scale_axis == 1) ? (first ? NMAT * kGrpTileM * 4 : 0) : NMAT * kChunkK * 4;
        bool ok = true;
        if (lane == 0) {
          ok = mbar_wait_sleepy(&pk_empty[ps], pph ^ 1);
          if (ok) mbar_arrive_expect_tx(&pk_full[ps], C::kPkData + aux);
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) goto done;
        uint8_t* slot = packed + ps * C::kPkBytes;
        if constexpr (FMT == kFmtCB3) {
          if (lane < 2) {   // one 6 KB x NMAT run per row block
            const int rb = 2 * it.rt + lane;
            bulk_g2s(slot + lane * (C::kPkData / 2),
                     p.wq + unit_offset(it.e, rb, kg, 0, 0, RB, KS256, NMAT, kCb3kUnitBytes), C::kPkData / 2,
                     &pk_full[ps]);
            if (first)
              bulk_g2s(slot + C::kPkData + lane * NMAT * 1024, p.cb + cb_offset_words(it.e, rb, 0, 0, 0, RB, NMAT),
                       NMAT * 1024, &pk_full[ps]);
          }
        } else {
          // 8 units x NMAT slices of 1 KB: chunk kg % 4 of the unit holding stage kg / 4
          if (lane < 8 * NMAT) {
            const int u = lane / NMAT, m = lane % NMAT;
            const int rb = 2 * it.rt + u / kWarpsPerBlock, w = u % kWarpsPerBlock;
            const uint8_t* src = p.wq + unit_offset(0, rb, kg / 4, w, m, RB, KS256, NMAT, kW8kUnitBytes) + (kg % 4) * 1024;
            bulk_g2s(slot + (u * NMAT + m) * 1024, src, 1024, &pk_full[ps]);
          }
          if (aux > 0 && lane >= 16 && lane < 16 + NMAT) {
            const int m = lane - 16;
            const float* sc = m == 0 ? p.s0 : p.s1;
            const int per = aux / NMAT;
            const float* src = (p.scale_axis == 1) ? sc + it.rt * kGrpTileM : sc + kg * kChunkK;
            bulk_g2s(slot + C::kPkData + m * per, src, per, &pk_full[ps]);
          }
        }
        if (++ps == C::kNpk) {
          ps = 0;
          pph ^= 1;
        }
      }
    }
  } else if (warp == kWarpTok) {
    // --------------------------------------------------------------------------------- token producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const ItemInfo it = grp_item<TN>(p, item);
        if (!item_ok(p, it)) continue;
        for (int ks = 0; ks < KS64; ++ks) {
          if (!mbar_wait_sleepy(&empty[st], ph ^ 1)) goto done;
          mbar_arrive_expect_tx(&full[st], C::kBTile);
          tma_load_2d(stages + st * C::kStage + NMAT * C::kATile, &tmap_b, ks * kChunkK, it.row0, &full[st]);
          if (++st == C::kNStage) {
            st = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0, local = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const ItemInfo it = grp_item<TN>(p, item);
        if (!item_ok(p, it)) continue;
        const int n = (it.cnt + 15) & ~15;
        const uint32_t idesc = idesc_bf16_m128(n);
        const int buf = (int)(local % C::kAccBufs);
        const uint32_t acc = tmem + buf * C::kAccCols;
        if (!mbar_wait(&tm_empty[buf], ((local / C::kAccBufs) & 1) ^ 1)) goto done;
        tc_fence_after();
        for (int ks = 0; ks < KS64; ++ks) {
          if (!mbar_wait(&full[st], ph)) goto done;
          tc_fence_after();
          const uint32_t sbase = smem_addr(stages + st * C::kStage);
          const uint64_t bdesc = sw128_desc(sbase + NMAT * C::kATile);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
              const uint64_t adesc = sw128_desc(sbase + m * C::kATile);
              umma_bf16(acc + m * TN, adesc + 2 * kk, bdesc + 2 * kk, idesc, (ks | kk) != 0);
            }
          }
          umma_commit(&empty[st]);
          if (++st == C::kNStage) {
            st = 0;
            ph ^= 1;
          }
        }
        umma_commit(&tm_full[buf]);
        ++local;
      }
    }
  } else if (warp < kWarpEpi0) {
    // ---------------------------------------------------------------------------------------- dequant
    const int d = warp - kWarpDq0;
    const int g = lane >> 2, t = lane & 3;
    int st = 0, ps = 0;
    uint32_t ph = 0, pph = 0;
    Codebook cbg[2][NMAT], cbh[2][NMAT];
    float sg[2][NMAT], sh[2][NMAT];
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const ItemInfo it = grp_item<TN>(p, item);
      if (!item_ok(p, it)) continue;
      for (int kg = 0; kg < KG; ++kg) {
        if (!mbar_wait(&pk_full[ps], pph)) goto done;
        const uint8_t* slot = packed + ps * C::kPkBytes;
        const uint8_t* aux = slot + C::kPkData;
        uint32_t wd[2][NMAT][12];
        uint4 q8[2][NMAT][2];
        float ksc[NMAT][16];
#pragma unroll
        for (int uu = 0; uu < 2; ++uu) {
          const int u = 2 * d + uu, rbsel = u / kWarpsPerBlock, w = u % kWarpsPerBlock;
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            if constexpr (FMT == kFmtCB3) {
              if (kg == 0) {
                const uint8_t* cbp = aux + rbsel * NMAT * 1024 + ((w * NMAT + m) * 16) * 16;
                const uint4 ca = lds128(cbp + g * 16), cb = lds128(cbp + (g + 8) * 16);
                cbg[uu][m] = {ca.x, ca.y, ca.z, ca.w};
                cbh[uu][m] = {cb.x, cb.y, cb.z, cb.w};
              }
              const uint8_t* src = slot + rbsel * (C::kPkData / 2) + (w * NMAT + m) * kCb3kUnitBytes + lane * 48;
#pragma unroll
              for (int v = 0; v < 3; ++v) {
                const uint4 q = lds128(src + 16 * v);
                wd[uu][m][4 * v] = q.x;
                wd[uu][m][4 * v + 1] = q.y;
                wd[uu][m][4 * v + 2] = q.z;
                wd[uu][m][4 * v + 3] = q.w;
              }
            } else {
              const uint8_t* src = slot + (u * NMAT + m) * 1024;
              q8[uu][m][0] = lds128(src + (0 * 32 + lane) * 16);
              q8[uu][m][1] = lds128(src + (1 * 32 + lane) * 16);
              if (p.scale_axis == 1) {
                if (kg == 0) {
                  const float* sc = reinterpret_cast<const float*>(aux) + m * kGrpTileM + u * kRowsPerWarp;
                  sg[uu][m] = sc[g];
                  sh[uu][m] = sc[g + 8];
                }
              }
            }
          }
        }
        if constexpr (FMT == kFmtW8) {
          if (p.scale_axis == 0) {
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
              for (int i = 0; i < 16; ++i)
                ksc[m][i] = reinterpret_cast<const float*>(aux)[m * kChunkK + 16 * t + i];
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&pk_empty[ps]);
        if (++ps == C::kNpk) {
          ps = 0;
          pph ^= 1;
        }
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          if (!mbar_wait(&empty[st], ph ^ 1)) goto done;
          uint8_t* sA = stages + st * C::kStage;
#pragma unroll
          for (int uu = 0; uu < 2; ++uu) {
            const int u = 2 * d + uu;
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
              uint32_t a[4][4];
              if constexpr (FMT == kFmtCB3) {
                cb3k_dequant_chunk(wd[uu][m][3 * c], wd[uu][m][3 * c + 1], wd[uu][m][3 * c + 2], cbg[uu][m],
                                   cbh[uu][m], a);
              } else {
                w8k_dequant_chunk(q8[uu][m][0], q8[uu][m][1], sg[uu][m], sh[uu][m],
                                  p.scale_axis == 0 ? ksc[m] : nullptr, a);
              }
              uint8_t* tile = sA + m * C::kATile;
              const int rg = u * kRowsPerWarp + g, rh = rg + 8;
              const uint4 g0 = make_uint4(a[0][0], a[0][2], a[1][0], a[1][2]);
              const uint4 g1 = make_uint4(a[2][0], a[2][2], a[3][0], a[3][2]);
              const uint4 h0 = make_uint4(a[0][1], a[0][3], a[1][1], a[1][3]);
              const uint4 h1 = make_uint4(a[2][1], a[2][3], a[3][1], a[3][3]);
              *reinterpret_cast<uint4*>(tile + sw128_off(rg, 2 * t)) = g0;
              *reinterpret_cast<uint4*>(tile + sw128_off(rg, 2 * t + 1)) = g1;
              *reinterpret_cast<uint4*>(tile + sw128_off(rh, 2 * t)) = h0;
              *reinterpret_cast<uint4*>(tile + sw128_off(rh, 2 * t + 1)) = h1;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[st]);
          if (++st == C::kNStage) {
            st = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else {
    // --------------------------------------------------------------------------------------- epilogue
    const int q = warp & 3;              // TMEM lane quadrant this warp may read
    uint32_t local = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const ItemInfo it = grp_item<TN>(p, item);
      if (!item_ok(p, it)) continue;
      const int buf = (int)(local % C::kAccBufs);
      if (!mbar_wait(&tm_full[buf], (local / C::kAccBufs) & 1)) goto done;
      tc_fence_after();
      const int wrow = it.rt * kGrpTileM + 32 * q + lane;
      const uint32_t tbase = tmem + buf * C::kAccCols + ((uint32_t)(32 * q) << 16);
      const int n = (it.cnt + 15) & ~15;
      for (int c0 = 0; c0 < n; c0 += 16) {
        float v0[16], v1[16];
        tmem_ld16(tbase + c0, v0);
        if constexpr (NMAT == 2) tmem_ld16(tbase + TN + c0, v1);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c0 + j < it.cnt) {
            float v = v0[j];
            if constexpr (EPI == kGrpEpiSwiglu) v = swiglu_clamped(v0[j], v1[j], p.limit);
            if constexpr (EPI == kGrpEpiStoreF32) {
              p.out_f32[(size_t)(it.row0 + c0 + j) * p.rows + wrow] = v;
            } else {
              const __nv_bfloat16 o = __float2bfloat16_rn(v);
              p.out[(size_t)(it.row0 + c0 + j) * p.rows + wrow] = *reinterpret_cast<const uint16_t*>(&o);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tm_empty[buf]);
      ++local;
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// bf16 matrix [rows][K] (row stride K*2 bytes): 64 x 128 boxes, 128-byte swizzle, zero fill out of bounds.
int make_token_map(CUtensorMap* map, const void* base, int K, int rows, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return CBMOE_ERR_CUDA;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kChunkK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CBMOE_OK : CBMOE_ERR_CUDA;
}

template <int FMT, int NMAT, int EPI, int TN>
int launch_grouped(const GroupedParams& p, const void* b, int b_rows, int kind, cudaStream_t stream) {
  using C = GrpCfg<FMT, NMAT, TN>;
  if (p.rows % kGrpTileM || p.K % kStageK || b_rows <= 0 || (reinterpret_cast<uintptr_t>(b) & 15))
    return CBMOE_ERR_INVALID;
  CUtensorMap map;
  int rc = make_token_map(&map, b, p.K, b_rows, TN);
  if (rc) return rc;
  auto kern = grouped_kernel<FMT, NMAT, EPI, TN>;
  static PerDevice s_attr;
  long long set = 0;
  rc = per_device(s_attr, [&](long long& v) -> int {
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    v = 1;
    return CBMOE_OK;
  }, &set);
  if (rc) return rc;
  prof_begin(kind, stream);
  kern<<<num_sms(), kGrpThreads, C::kSmem, stream>>>(p, map);
  prof_end(kind, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

// xs[r] = x[tok_row[r]] (zero rows where tok_row < 0): 16-byte copies
__global__ void gather_rows_kernel(const uint4* __restrict__ x, int H16, const int* __restrict__ tok_row, int rows,
                                   uint4* __restrict__ xs) {
  const long long total = (long long)rows * H16;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / H16), c = (int)(i % H16);
    const int t = tok_row[r];
    xs[i] = t >= 0 ? x[(size_t)t * H16 + c] : make_uint4(0, 0, 0, 0);
  }
}

// out[n][r] = add[n][r] + sum_j w[n][j] * y_sorted[row_slot[n][j]][r], y_sorted / add bf16; fp32 or bf16 out.
// One thread per 8 consecutive outputs (16-byte loads of the bf16 rows).
__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__global__ void combine_bf16_kernel(const uint16_t* __restrict__ y_sorted, const int* __restrict__ row_slot,
                                    const float* __restrict__ wts, int N, int topk, int H,
                                    const uint16_t* __restrict__ add, const float* __restrict__ add_f32,
                                    float* __restrict__ out_f32, uint16_t* __restrict__ out_bf16) {
  const int H8 = H / 8;
  const long long total = (long long)N * H8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / H8), c8 = (int)(i % H8);
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int q0 = 0; q0 < topk; q0 += 8) {
      int rs[8];
      float wt[8];
      uint4 yv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool in = q0 + q < topk;
        rs[q] = in ? row_slot[n * topk + q0 + q] : -1;
        wt[q] = in ? wts[n * topk + q0 + q] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        yv[q] = rs[q] >= 0 ? reinterpret_cast<const uint4*>(y_sorted + (size_t)rs[q] * H)[c8] : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float f[8];
        bf16x8_to_f32(yv[q], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] += wt[q] * f[e];
      }
    }
    if (add != nullptr) {
      float f[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(add + (size_t)n * H)[c8], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += f[e];
    }
    if (add_f32 != nullptr) {
      const float4* a = reinterpret_cast<const float4*>(add_f32 + (size_t)n * H + (size_t)c8 * 8);
      const float4 a0 = a[0], a1 = a[1];
      v[0] += a0.x; v[1] += a0.y; v[2] += a0.z; v[3] += a0.w;
      v[4] += a1.x; v[5] += a1.y; v[6] += a1.z; v[7] += a1.w;
    }
    const size_t o = (size_t)n * H + (size_t)c8 * 8;
    if (out_f32 != nullptr) {
      reinterpret_cast<float4*>(out_f32 + o)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(out_f32 + o)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (out_bf16 != nullptr)
      *reinterpret_cast<uint4*>(out_bf16 + o) =
          make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

int grid_of(long long total) {
  long long b = (total + 255) / 256;
  const long long cap = (long long)num_sms() * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

int grouped_cb3_gateup(const GroupedParams& p, const void* b, int b_rows, int tn, cudaStream_t s) {
  if (tn == 128) return launch_grouped<kFmtCB3, 2, kGrpEpiSwiglu, 128>(p, b, b_rows, kProfGrpCb3GateUp, s);
  if (tn == 256) return launch_grouped<kFmtCB3, 2, kGrpEpiSwiglu, 256>(p, b, b_rows, kProfGrpCb3GateUp, s);
  return CBMOE_ERR_INVALID;
}
int grouped_cb3_down(const GroupedParams& p, const void* b, int b_rows, int tn, cudaStream_t s) {
  if (tn == 128) return launch_grouped<kFmtCB3, 1, kGrpEpiStore, 128>(p, b, b_rows, kProfGrpCb3Down, s);
  if (tn == 256) return launch_grouped<kFmtCB3, 1, kGrpEpiStore, 256>(p, b, b_rows, kProfGrpCb3Down, s);
  return CBMOE_ERR_INVALID;
}
int grouped_w8_gateup(const GroupedParams& p, const void* b, int b_rows, cudaStream_t s) {
  return launch_grouped<kFmtW8, 2, kGrpEpiSwiglu, 128>(p, b, b_rows, kProfGrpW8GateUp, s);
}
int grouped_w8_store(const GroupedParams& p, const void* b, int b_rows, cudaStream_t s) {
  return launch_grouped<kFmtW8, 1, kGrpEpiStore, 256>(p, b, b_rows, kProfGrpW8Store, s);
}
int grouped_w8_store_f32(const GroupedParams& p, const void* b, int b_rows, cudaStream_t s) {
  return launch_grouped<kFmtW8, 1, kGrpEpiStoreF32, 256>(p, b, b_rows, kProfGrpW8Store, s);
}

int launch_gather_rows(const uint16_t* x, int H, const int* tok_row, int rows, uint16_t* xs, cudaStream_t s) {
  const int H16 = H / 8;
  prof_begin(kProfOther, s);
  gather_rows_kernel<<<grid_of((long long)rows * H16), 256, 0, s>>>(reinterpret_cast<const uint4*>(x), H16, tok_row,
                                                                     rows, reinterpret_cast<uint4*>(xs));
  prof_end(kProfOther, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

int launch_combine_bf16(const uint16_t* y_sorted, const int* row_slot, const float* wts, int N, int topk, int H,
                        const uint16_t* add_bf16, float* out_f32, uint16_t* out_bf16, cudaStream_t s,
                        const float* add_f32) {
  prof_begin(kProfCombine, s);
  combine_bf16_kernel<<<grid_of((long long)N * H / 8), 256, 0, s>>>(y_sorted, row_slot, wts, N, topk, H, add_bf16,
                                                                 add_f32, out_f32, out_bf16);
  prof_end(kProfCombine, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

}  // namespace cbmoe
