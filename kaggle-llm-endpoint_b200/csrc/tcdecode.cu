// Decode / medium-batch routed experts on tcgen05: the CB3 weights are dequantized in registers (the decode
// kernels' byte-permute dequant over the CB3K layout) and stored straight into TMEM, where the tensor core reads
// them as operand A; the tokens are operand B in shared memory (TMA); fp32 accumulators live in TMEM. Counterpart
// of the reference's moe_matvec Pallas kernel (pallas_moe.py:238-307) and of `_apply_kernel`'s gate/up -> swiglu
// -> down composition (resident.py:110-120).
//
// Why: with mma.sync the dequant and the MMAs share the consumer warps' issue slots, and every 8 tokens of a pass
// beyond the first cost about 0.6 of a whole weight pass. Here the dequant warps issue nothing but the lookup
// arithmetic and one TMEM store per 64-input chunk; the contraction runs asynchronously on the tensor core, so a
// pass of 16, 32 or 64 tokens costs the same ALU work as a pass of one.
//
//   D[w, t] = sum_k W_e[w, k] * X[t, k]    w: 128 weight rows (tcgen05 M)    t: <= TN tokens of one pass (N)
//
// One CTA per SM (all 512 TMEM columns), 14 warps:
//   warp 0       producer: tickets, stage headers, bulk copies of the packed bits (+ codebooks), TMA token tiles
//   warp 1       TMEM owner and MMA issuer (one thread): tcgen05.mma kind::f16, A from TMEM, B from shared memory
//   warps 2-9    dequant: warp w owns the 16-row unit 2*(w%4) + (w-2)/4 of the tile, i.e. TMEM lanes of its
//                quarter w%4; packed bits -> bf16 fragments -> tcgen05.st.16x256b (16 lanes x 32 columns per chunk)
//   warps 10-13  epilogue: tcgen05.ld of the accumulators -> SwiGLU (gate/up, hi + lo bf16 planes) or fp32 store
// The fragment a dequant lane holds (rows g and g+8, inputs 16t+4s .. +3 of each chunk, layout.cuh) lands in
// TMEM column 8s + 2t (+1) of MMA slice s; so the 16 inputs of slice s are {16a + 4s + b}, and the token operand
// holds every 64-input chunk in the same order (tc_perm64): the gather writes x that way and the gate/up
// epilogue writes h that way.
// Rings: packed stages (256 inputs) full/empty, token stages full/empty, TMEM A chunks (64 inputs) full/empty,
// two accumulator buffers full/empty, segment headers for the epilogue full/empty. Work: tickets from a counter,
// whole items (pass, 128-row tile) first, then the last items cut into pieces of the 256-input stages whose
// partial sums the last-arriving piece adds up in order. Every wait is bounded; a role that gives up sets
// CBMOE_DEVERR_TIMEOUT and falls through to the final barrier, after which warp 1 frees TMEM. No multicast.
#include <cudaTypedefs.h>
#include <mutex>

#include "tcdecode.cuh"
#include "profile.cuh"
#include "umma.cuh"

namespace cbmoe {

namespace {

constexpr int kTcWarps = 14;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcWarpProd = 0, kTcWarpMma = 1, kTcWarpDq0 = 2, kTcWarpEpi0 = 10;
constexpr int kTcTmemCols = 512;
constexpr int kTcLookahead = 3;        // the next ticket is taken this many stages before the segment's end
constexpr int kTcMinSmem = 116 * 1024; // keeps a second CTA (and a second 512-column TMEM allocation) off the SM

template <int NMAT, int TN>
struct TcCfg {
  static constexpr bool kHilo = NMAT == 1;                               // down: h as hi + lo planes
  static constexpr int kPkData = 2 * kWarpsPerBlock * NMAT * kCb3kUnitBytes;   // 8 units x NMAT per stage
  static constexpr int kPkAux = 2 * NMAT * 1024;                         // codebooks of the tile's 128 rows
  static constexpr int kPkBytes = kPkData + kPkAux;
  static constexpr int kNpk = 3;
  static constexpr int kBBox = TN * 128;                                 // TN rows x 64 bf16, 128B swizzle
  static constexpr int kBPlane = 4 * kBBox;                              // one 256-input stage
  static constexpr int kBBytes = (kHilo ? 2 : 1) * kBPlane;
  static constexpr int kNb = kBBytes >= 32 * 1024 ? 2 : 3;
  static constexpr int kAccCols = NMAT * TN;                             // one accumulator buffer
  static constexpr int kAChunk = 32 * NMAT;                              // TMEM columns of one 64-input chunk
  static constexpr int kNaFit = (kTcTmemCols - 2 * kAccCols) / kAChunk;
  static constexpr int kNa = kNaFit > 8 ? 8 : kNaFit;
  static constexpr int kAOff = 2 * kAccCols;
  static constexpr int kPkOff = kNb * kBBytes;
  static constexpr int kHdrOff = kPkOff + kNpk * kPkBytes;
  static constexpr int kHdrs = kNpk + kNb + 4;
  static constexpr int kBarOff = kHdrOff + kHdrs * 32;
  static constexpr int kBars = 2 * (kNpk + kNb + kNa + 2 + 4);
  static constexpr int kSmemUsed = 1024 + kBarOff + kBars * 8 + 16;
  static constexpr int kSmem = kSmemUsed > kTcMinSmem ? kSmemUsed : kTcMinSmem;
  static_assert(kNa >= 2, "TMEM budget");
  static_assert(kBBytes % 1024 == 0 && kPkBytes % 16 == 0, "alignment of the rings");
  static_assert(kSmemUsed <= 227 * 1024, "shared memory budget");
};

// What the producer tells the other roles about a stage (or, in the header ring, a segment). item < 0 ends a role.
struct TcHdr {
  int item, e, row0, cnt, rt, piece, nseg, flags;   // flags: 1 = first stage of the segment, 2 = last
};

struct TcSched {
  int n_whole, n_tail, Q, KS;
  __device__ int tickets() const { return n_whole + n_tail * Q; }
  __device__ void decode(int t, int& item, int& ks0, int& ks1, int& piece) const {
    if (t < n_whole) {
      item = t;
      ks0 = 0;
      ks1 = KS;
      piece = -1;
      return;
    }
    const int u = t - n_whole;
    item = n_whole + u / Q;
    piece = u % Q;
    ks0 = piece * KS / Q;
    ks1 = (piece + 1) * KS / Q;
  }
};

__device__ __forceinline__ TcSched tc_schedule(const TcParams& p, int n_items) {
  TcSched s;
  s.KS = p.K / kStageK;
  s.Q = s.KS < kTcPieces ? s.KS : kTcPieces;
  int tail = 0;
  if (p.part != nullptr && s.Q > 1) {
    tail = (int)gridDim.x / 2 > 1 ? (int)gridDim.x / 2 : 1;
    if (tail > p.tail_items) tail = p.tail_items;
    if (tail > n_items) tail = n_items;
  }
  s.n_tail = tail;
  s.n_whole = n_items - tail;
  if (tail == 0) s.Q = 1;
  return s;
}

template <int NMAT, int TN>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_decode_kernel(const TcParams p, const __grid_constant__ CUtensorMap map0,
                     const __grid_constant__ CUtensorMap map1) {
  using C = TcCfg<NMAT, TN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bring = smem;
  uint8_t* packed = smem + C::kPkOff;
  TcHdr* pk_hdr = reinterpret_cast<TcHdr*>(smem + C::kHdrOff);
  TcHdr* b_hdr = pk_hdr + C::kNpk;
  TcHdr* ihdr = b_hdr + C::kNb;
  uint64_t* pk_full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* pk_empty = pk_full + C::kNpk;
  uint64_t* b_full = pk_empty + C::kNpk;
  uint64_t* b_empty = b_full + C::kNb;
  uint64_t* a_full = b_empty + C::kNb;
  uint64_t* a_empty = a_full + C::kNa;
  uint64_t* acc_full = a_empty + C::kNa;     // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* ih_full = acc_empty + 2;         // [4]
  uint64_t* ih_empty = ih_full + 4;          // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ih_empty + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kNpk; ++i) {
      mbar_init(&pk_full[i], 1);
      mbar_init(&pk_empty[i], 8);
    }
    for (int i = 0; i < C::kNb; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < C::kNa; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&ih_full[i], 1);
      mbar_init(&ih_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == kTcWarpMma) tmem_alloc(tmem_slot, kTcTmemCols);
  if (warp == kTcWarpProd && lane == 0) {
    prefetch_tmap(&map0);
    if constexpr (C::kHilo) prefetch_tmap(&map1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int RT = p.rows / kTcTileM, RB = p.rows / kRowsPerBlock, KS = p.K / kStageK;
  const int n_items = *p.n_pass * RT;
  const TcSched sc = tc_schedule(p, n_items);
  const int n_tickets = sc.tickets();

  if (warp == kTcWarpProd) {
    // ------------------------------------------------------------------------------------------- producer
    int ps = 0, bs = 0, ih = 0;
    uint32_t pph = 0, bph = 0, ihph = 0;
    bool ok = true;
    int tk = 0;
    if (lane == 0) tk = atomicAdd(p.sched, 1);
    tk = __shfl_sync(0xffffffffu, tk, 0);
    while (ok && tk < n_tickets) {
      int item = 0, ks0 = 0, ks1 = 0, piece = -1;
      sc.decode(tk, item, ks0, ks1, piece);
      const int pass = item / RT, rt = item - pass * RT;
      const int e = p.pass_expert[pass], row0 = p.pass_row0[pass], cnt = p.pass_cnt[pass];
      const int nseg = piece < 0 ? 1 : sc.Q;
      int pending = 0;
      if (e < 0 || e >= p.E || cnt <= 0 || cnt > TN) {   // not produced by the routing plan; skipped
        if (lane == 0) pending = atomicAdd(p.sched, 1);
        tk = __shfl_sync(0xffffffffu, pending, 0);
        continue;
      }
      const int look = ks1 - kTcLookahead > ks0 ? ks1 - kTcLookahead : ks0;
      if (lane == 0) {
        ok = mbar_wait_sleepy(&ih_empty[ih], ihph ^ 1);
        if (ok) {
          ihdr[ih] = TcHdr{item, e, row0, cnt, rt, piece, nseg, 0};
          mbar_arrive(&ih_full[ih]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (++ih == 4) {
        ih = 0;
        ihph ^= 1;
      }
      for (int ks = ks0; ks < ks1; ++ks) {
        const bool first = ks == ks0;
        const TcHdr h{item, e, row0, cnt, rt, piece, nseg, (first ? 1 : 0) | (ks == ks1 - 1 ? 2 : 0)};
        uint8_t* pk = packed + ps * C::kPkBytes;
        if (lane == 0) {
          ok = mbar_wait_sleepy(&pk_empty[ps], pph ^ 1);
          if (ok) {
            pk_hdr[ps] = h;
            mbar_arrive_expect_tx(&pk_full[ps], C::kPkData + (first ? C::kPkAux : 0));
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        if (lane < 2) {   // one contiguous run of 4 units x NMAT per 64-row block, + its codebooks
          const int rb = 2 * rt + lane;
          bulk_g2s(pk + lane * (C::kPkData / 2),
                   p.wq + unit_offset(e, rb, ks, 0, 0, RB, KS, NMAT, kCb3kUnitBytes), C::kPkData / 2,
                   &pk_full[ps]);
          if (first)
            bulk_g2s(pk + C::kPkData + lane * NMAT * 1024, p.cb + cb_offset_words(e, rb, 0, 0, 0, RB, NMAT),
                     NMAT * 1024, &pk_full[ps]);
        }
        if (++ps == C::kNpk) {
          ps = 0;
          pph ^= 1;
        }
        uint8_t* bslot = bring + bs * C::kBBytes;
        if (lane == 0) {
          ok = mbar_wait_sleepy(&b_empty[bs], bph ^ 1);
          if (ok) {
            b_hdr[bs] = h;
            mbar_arrive_expect_tx(&b_full[bs], C::kBBytes);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_2d(bslot + c * C::kBBox, &map0, ks * kStageK + c * kChunkK, row0, &b_full[bs]);
            if constexpr (C::kHilo) {
#pragma unroll
              for (int c = 0; c < 4; ++c)
                tma_load_2d(bslot + C::kBPlane + c * C::kBBox, &map1, ks * kStageK + c * kChunkK, row0,
                            &b_full[bs]);
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        if (++bs == C::kNb) {
          bs = 0;
          bph ^= 1;
        }
        if (ks == look && lane == 0) pending = atomicAdd(p.sched, 1);
      }
      tk = __shfl_sync(0xffffffffu, pending, 0);
    }
    if (ok && lane == 0) {   // end marks for the three consumers
      if (mbar_wait_sleepy(&pk_empty[ps], pph ^ 1)) {
        pk_hdr[ps].item = -1;
        mbar_arrive(&pk_full[ps]);
      }
      if (mbar_wait_sleepy(&b_empty[bs], bph ^ 1)) {
        b_hdr[bs].item = -1;
        mbar_arrive(&b_full[bs]);
      }
      if (mbar_wait_sleepy(&ih_empty[ih], ihph ^ 1)) {
        ihdr[ih].item = -1;
        mbar_arrive(&ih_full[ih]);
      }
    }
  } else if (warp == kTcWarpMma) {
    // ----------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int bs = 0, ai = 0;
      uint32_t bph = 0, aph = 0, nacc = 0;
      uint32_t acc = tmem, idesc = idesc_bf16_m128(16);
      for (;;) {
        if (!mbar_wait(&b_full[bs], bph)) break;
        const TcHdr h = b_hdr[bs];
        if (h.item < 0) break;
        tc_fence_after();
        const bool first = (h.flags & 1) != 0;
        if (first) {
          const uint32_t buf = nacc & 1;
          if (!mbar_wait(&acc_empty[buf], ((nacc >> 1) & 1) ^ 1)) break;
          tc_fence_after();
          acc = tmem + buf * C::kAccCols;
          idesc = idesc_bf16_m128((h.cnt + 15) & ~15);
        }
        const uint32_t bbase = smem_addr(bring + bs * C::kBBytes);
        bool ok = true;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          if (!mbar_wait(&a_full[ai], aph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t abase = tmem + C::kAOff + ai * C::kAChunk;
          const uint64_t bd = sw128_desc(bbase + c * C::kBBox);
#pragma unroll
          for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
              const uint32_t a = abase + m * 32 + 8 * s;
              umma_bf16_ts(acc + m * TN, a, bd + 2 * s, idesc, (first && c == 0 && s == 0) ? 0u : 1u);
              if constexpr (C::kHilo) {
                const uint64_t bl = sw128_desc(bbase + C::kBPlane + c * C::kBBox);
                umma_bf16_ts(acc + m * TN, a, bl + 2 * s, idesc, 1u);
              }
            }
          }
          umma_commit(&a_empty[ai]);
          if (++ai == C::kNa) {
            ai = 0;
            aph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&b_empty[bs]);
        if (++bs == C::kNb) {
          bs = 0;
          bph ^= 1;
        }
        if (h.flags & 2) {
          umma_commit(&acc_full[nacc & 1]);
          ++nacc;
        }
      }
    }
  } else if (warp < kTcWarpEpi0) {
    // --------------------------------------------------------------------------------------------- dequant
    const int q = warp & 3;                          // TMEM lane quarter this warp may write
    const int u = 2 * q + ((warp - kTcWarpDq0) >> 2);   // 16-row unit of the tile = TMEM lanes 16u .. 16u+15
    const int rbsel = u >> 2, wu = u & 3;            // 64-row block of the tile, unit inside the block
    const int g = lane >> 2;
    const uint32_t lanes = (uint32_t)(16 * u) << 16;
    Codebook cbg[NMAT], cbh[NMAT];
    int ps = 0, ai = 0;
    uint32_t pph = 0, aph = 0;
    for (;;) {
      if (!mbar_wait(&pk_full[ps], pph)) break;
      const TcHdr h = pk_hdr[ps];
      if (h.item < 0) break;
      const uint8_t* slot = packed + ps * C::kPkBytes;
      if (h.flags & 1) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          const uint8_t* cbp = slot + C::kPkData + rbsel * NMAT * 1024 + ((wu * NMAT + m) * 16) * 16;
          const uint4 ca = lds128(cbp + g * 16), cb = lds128(cbp + (g + 8) * 16);
          cbg[m] = {ca.x, ca.y, ca.z, ca.w};
          cbh[m] = {cb.x, cb.y, cb.z, cb.w};
        }
      }
      uint32_t wd[NMAT][12];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const uint8_t* src = slot + rbsel * (C::kPkData / 2) + (wu * NMAT + m) * kCb3kUnitBytes + lane * 48;
#pragma unroll
        for (int v = 0; v < 3; ++v) {
          const uint4 w4 = lds128(src + 16 * v);
          wd[m][4 * v] = w4.x;
          wd[m][4 * v + 1] = w4.y;
          wd[m][4 * v + 2] = w4.z;
          wd[m][4 * v + 3] = w4.w;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pk_empty[ps]);
      if (++ps == C::kNpk) {
        ps = 0;
        pph ^= 1;
      }
      bool ok = true;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[NMAT][16];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          uint32_t a[4][4];
          cb3k_dequant_chunk(wd[m][3 * c], wd[m][3 * c + 1], wd[m][3 * c + 2], cbg[m], cbh[m], a);
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            r[m][4 * s] = a[s][0];
            r[m][4 * s + 1] = a[s][2];
            r[m][4 * s + 2] = a[s][1];
            r[m][4 * s + 3] = a[s][3];
          }
        }
        if (!mbar_wait(&a_empty[ai], aph ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int m = 0; m < NMAT; ++m) tmem_st_16x256b_x4(tmem + lanes + C::kAOff + ai * C::kAChunk + m * 32, r[m]);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[ai]);
        if (++ai == C::kNa) {
          ai = 0;
          aph ^= 1;
        }
      }
      if (!ok) break;
    }
  } else {
    // -------------------------------------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may read
    const int rloc = 32 * q + lane;         // tile row = TMEM lane
    int ih = 0;
    uint32_t ihph = 0, nacc = 0;
    for (;;) {
      if (!mbar_wait(&ih_full[ih], ihph)) break;
      const TcHdr H = ihdr[ih];
      __syncwarp();
      if (lane == 0) mbar_arrive(&ih_empty[ih]);
      if (++ih == 4) {
        ih = 0;
        ihph ^= 1;
      }
      if (H.item < 0) break;
      const uint32_t buf = nacc & 1;
      if (!mbar_wait(&acc_full[buf], (nacc >> 1) & 1)) break;
      tc_fence_after();
      const int r = H.rt * kTcTileM + rloc;   // output row of the matrix
      const uint32_t tb = tmem + buf * C::kAccCols + ((uint32_t)(32 * q) << 16);
      const int n = (H.cnt + 15) & ~15;
      const size_t slot_base =
          H.nseg > 1 ? (((size_t)(H.item - sc.n_whole) * sc.Q + H.piece) * TN) * NMAT * kTcTileM : 0;
      auto emit = [&](int j, float v0, float v1) {
        const size_t row = (size_t)(H.row0 + j);
        if constexpr (NMAT == 2) {
          const float hv = swiglu_clamped(v0, v1, p.limit);
          const __nv_bfloat16 hi = __float2bfloat16_rn(hv);
          const __nv_bfloat16 lo = __float2bfloat16_rn(hv - __bfloat162float(hi));
          const size_t col = (size_t)((r & ~63) | tc_perm64(r & 63));
          p.h_out[row * p.rows + col] = *reinterpret_cast<const uint16_t*>(&hi);
          p.h_out[p.h_plane + row * p.rows + col] = *reinterpret_cast<const uint16_t*>(&lo);
        } else {
          p.y_out[row * p.rows + r] = v0;
        }
      };
      for (int c0 = 0; c0 < n; c0 += 16) {
        float v0[16], v1[16];
        tmem_ld16(tb + c0, v0);
        if constexpr (NMAT == 2) tmem_ld16(tb + TN + c0, v1);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c0 + j >= H.cnt) continue;
          if (H.nseg == 1) {
            emit(c0 + j, v0[j], NMAT == 2 ? v1[j] : 0.f);
          } else {
            float* sl = p.part + slot_base + (size_t)(c0 + j) * NMAT * kTcTileM + rloc;
            sl[0] = v0[j];
            if constexpr (NMAT == 2) sl[kTcTileM] = v1[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      ++nacc;
      if (H.nseg > 1) {
        // This warp's rows of the piece are stored; the warp whose arrival completes the item (per quarter) adds
        // the pieces' slots up in piece order and runs the epilogue for those rows.
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          int* ctr = p.done + (size_t)(H.item - sc.n_whole) * 4 + q;
          last = atomicAdd(ctr, 1) == H.nseg - 1;
          if (last) *ctr = 0;   // ready for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          const size_t item_base = ((size_t)(H.item - sc.n_whole) * sc.Q) * TN * NMAT * kTcTileM;
          for (int j = 0; j < H.cnt; ++j) {
            float v0 = 0.f, v1 = 0.f;
            for (int pq = 0; pq < H.nseg; ++pq) {
              const float* sl = p.part + item_base + ((size_t)pq * TN + j) * NMAT * kTcTileM + rloc;
              v0 += __ldcg(sl);
              if constexpr (NMAT == 2) v1 += __ldcg(sl + kTcTileM);
            }
            emit(j, v0, v1);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

// xs[r][chunk order] = x[tok_row[r]] with each chunk's 16 groups of 4 inputs permuted (tc_perm64 moves groups of
// 4 consecutive inputs together: position group 4s + a holds input group 4a + s). 8-byte copies.
__global__ void gather_perm_kernel(const uint2* __restrict__ x, int H4, const int* __restrict__ tok_row, int rows,
                                   uint2* __restrict__ xs) {
  const long long total = (long long)rows * H4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / H4), gd = (int)(i % H4);
    const int within = gd & 15;
    const int gs = (gd & ~15) | ((within & 3) << 2) | (within >> 2);
    const int t = tok_row[r];
    xs[i] = t >= 0 ? x[(size_t)t * H4 + gs] : make_uint2(0, 0);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tc_encode_fn() {
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

// bf16 matrix [rows][K]: boxes of 64 inputs x box_rows rows, 128-byte swizzle, zero fill out of bounds.
int tc_token_map(CUtensorMap* map, const void* base, int K, int rows, int box_rows) {
  auto fn = tc_encode_fn();
  if (fn == nullptr) return CBMOE_ERR_CUDA;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kChunkK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS ? CBMOE_OK : CBMOE_ERR_CUDA;
}

template <int NMAT, int TN>
int launch_tc_t(const TcParams& p, const void* b0, const void* b1, int b_rows, int kind, cudaStream_t stream) {
  using C = TcCfg<NMAT, TN>;
  if (p.rows % kTcTileM || p.K % kStageK || b_rows <= 0 || p.sched == nullptr || (p.part && !p.done) ||
      (reinterpret_cast<uintptr_t>(b0) & 15) || (C::kHilo && (reinterpret_cast<uintptr_t>(b1) & 15)))
    return CBMOE_ERR_INVALID;
  CUtensorMap m0, m1;
  int rc = tc_token_map(&m0, b0, p.K, b_rows, TN);
  if (rc) return rc;
  rc = tc_token_map(&m1, C::kHilo ? b1 : b0, p.K, b_rows, TN);
  if (rc) return rc;
  auto kern = tc_decode_kernel<NMAT, TN>;
  static bool attr = false;
  if (!attr) {
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    attr = true;
  }
  int grid = num_sms();
  if (p.grid_cap > 0 && p.grid_cap < grid) grid = p.grid_cap;
  prof_begin(kind, stream);
  kern<<<grid, kTcThreads, C::kSmem, stream>>>(p, m0, m1);
  prof_end(kind, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

template <int NMAT>
int launch_tc(const TcParams& p, const void* b0, const void* b1, int b_rows, int tn, int kind, cudaStream_t s) {
  switch (tn) {
    case 16: return launch_tc_t<NMAT, 16>(p, b0, b1, b_rows, kind, s);
    case 32: return launch_tc_t<NMAT, 32>(p, b0, b1, b_rows, kind, s);
    case 64: return launch_tc_t<NMAT, 64>(p, b0, b1, b_rows, kind, s);
    default: return CBMOE_ERR_INVALID;
  }
}

}  // namespace

int tc_pass_tokens(long long S, int E) {
  const long long per = E > 0 ? (S + E - 1) / E : S;
  return per <= 8 ? 16 : (per <= 24 ? 32 : 64);
}

size_t tc_part_bytes(int tail_items, int tn, int nmat) {
  return (size_t)tail_items * kTcPieces * tn * nmat * kTcTileM * sizeof(float);
}

int tc_tail_items(long long items) {
  const long long half = num_sms() / 2;
  return (int)(items < half ? items : half);
}

int launch_gather_perm(const uint16_t* x, int H, const int* tok_row, int rows, uint16_t* xs, cudaStream_t s) {
  if (H % kChunkK || (reinterpret_cast<uintptr_t>(x) & 7) || (reinterpret_cast<uintptr_t>(xs) & 7))
    return CBMOE_ERR_INVALID;
  const int H4 = H / 4;
  const long long total = (long long)rows * H4;
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  prof_begin(kProfOther, s);
  gather_perm_kernel<<<(int)blocks, 256, 0, s>>>(reinterpret_cast<const uint2*>(x), H4, tok_row, rows,
                                                 reinterpret_cast<uint2*>(xs));
  prof_end(kProfOther, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

int tc_cb3_gateup(const TcParams& p, const uint16_t* xs, int xs_rows, int tn, cudaStream_t s) {
  return launch_tc<2>(p, xs, nullptr, xs_rows, tn, kProfCb3GateUp, s);
}

int tc_cb3_down(const TcParams& p, const uint16_t* h_hi, const uint16_t* h_lo, int h_rows, int tn, cudaStream_t s) {
  return launch_tc<1>(p, h_hi, h_lo, h_rows, tn, kProfCb3Down, s);
}

}  // namespace cbmoe
