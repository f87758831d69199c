// Decode / small-batch expert kernels: fused dequant + tensor-core matvec over the kernel layouts (layout.cuh).
//
// Counterpart of the reference's moe_matvec Pallas kernel (pallas_moe.py:238-307) and of `_apply_kernel`'s
// gate/up -> swiglu -> down composition (resident.py:110-120), with two changes of design for B200:
//   * work is per (expert pass, 64-row block), not per slot: a pass is a few tokens routed to one expert, so an
//     expert's weights stream from HBM once per pass instead of once per (token, slot) pair;
//   * the weights never leave registers in dense form: a producer warp streams 256-input stages of packed bits
//     into shared memory with bulk async copies (mbarrier pipeline, NSTAGE deep); four consumer warps turn them
//     into tensor-core fragments in registers and multiply them against the pass's tokens:
//       CB8 (default for CB3 layers): byte-table lookups into int8 hi / lo digits of the 16-bit fixed-point
//         codebook, mma.sync m16n8k32 int8 against X8 (gate/up) or H8 (down) activation digits, exact int32 sums;
//       W8I: the stored int8 leaves as the int8 A fragments (the shared expert at small batches, the int8 lm_head);
//       CB3 / W8: bf16 fragments (byte permutes of the bf16 codebooks; int8 -> fp32 * scale -> bf16) and
//         mma.sync m16n8k16 bf16, fp32 accumulation (layers without CB8 tables, or many tokens per expert).
// Persistent grid: gridDim = SMs x resident CTAs, work handed out by tickets, the last partial wave of long items
// cut into pieces. Epilogues: SWIGLU (gate+up -> h as H8 digit rows, or bf16 hi + lo), STORE (f32 or bf16 rows).
// The layer's weighted sum of the slots (+ the shared expert) is combine_kernel.
#include "decode.cuh"
#include "profile.cuh"

namespace cbmoe {

// The CB8 kernels' template format value (kFmtCB8 is the tables' format id; the kernels are built once, with the
// selector arithmetic on the ALU pipe).
constexpr int kFmtCB8A = 3;
template <>
struct Fmt<kFmtCB8A> {
  static constexpr int kUnitBytes = kCb3kUnitBytes;
};
template <int FMT>
constexpr bool is_cb8() { return FMT == kFmtCB8 || FMT == kFmtCB8A; }
// Formats multiplied on the int8 tensor-core MMA against split activations (X8 / H8 rows): CB8 (table lookups into
// int8 / uint8 bytes) and W8I (the stored int8 weights as they are).
template <int FMT>
constexpr bool is_split() { return is_cb8<FMT>() || FMT == kFmtW8I; }

template <int FMT, int NMAT, int NT, int HILO, int NSTAGE>
struct DecodeSmem {
  static constexpr bool kCb8 = is_split<FMT>();
  static constexpr int kUnit = Fmt<FMT>::kUnitBytes;
  static constexpr int kWBytes = kConsumerWarps * NMAT * kUnit;
  // codebooks (CB3K), tables + row factors (CB8) or scales (W8K) of the item
  static constexpr int kAuxBytes = NMAT * (kCb8 ? kCb8BlockBytes : 1024);
  // bytes of one B row per stage: bf16 (x, or h as hi + lo), X8 or H8
  static constexpr int kBCopy = kCb8 ? (HILO ? kH8StageBytes : kX8StageBytes) : kStageK * 2 * (HILO ? 2 : 1);
  static constexpr int kBRow = kBCopy + 16;                    // padded: conflict-free fragment loads
  // B rows of a pass: 8 tokens per column tile (bf16); CB8: 4 tokens (X8, hi and lo columns) or 2 slots (H8, 4
  // part columns) per tile
  static constexpr int kTokPerTile = kCb8 ? (HILO ? 2 : 4) : 8;
  static constexpr int kPassTokens = NT * kTokPerTile;
  static constexpr int kBBytes = kPassTokens * kBRow;
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
  return np * p.RB;
}

// Work distribution. An item is (pass, 64-row block): KS stages of weights for the pass's tokens. CTAs take work
// from a shared ticket counter, so the CTAs that start late (their SM still busy with another kernel) or run slow
// simply take less. Tickets first hand out whole items; the last n_tail items are cut into Q pieces of ~KS/Q stages
// each, so the grid runs out of work within a fraction of an item. A piece stores its partial sums in the item's
// slot q; the piece that arrives last on the item's counter adds the Q slots up in order (deterministic) and runs
// the epilogue. Without partial-sum space (part == nullptr) every item is whole.
struct Schedule {
  int n_items, n_whole, n_tail, Q, KS;
  __device__ int tickets() const { return n_whole + n_tail * Q; }
  // ticket -> item, stage range, piece (-1: whole item)
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

// Which items are cut: a cut item pays for partial sums, a device-wide fence and a last-arriver reduction
// (measured: cutting the last half-grid of items of a config-1 launch cost 10% of the kernel), so only the items of
// a partial last wave are cut, only when that wave is at most half full and an item is long (>= 12 stages: for the
// 6-stage items of the config-1 down kernel the cut cost more than the imbalance it removed); with fewer items than
// CTAs every item is cut (small batches: the pieces spread over the grid).
__device__ __forceinline__ Schedule make_schedule(const DecodeParams& p, int n_items) {
  Schedule sc;
  sc.n_items = n_items;
  sc.KS = p.KS;
  sc.Q = p.KS < kDecodePieces ? p.KS : kDecodePieces;
  int tail = 0;
  if (p.part != nullptr && p.done != nullptr && sc.Q > 1 && n_items > 0) {
    const int G = (int)gridDim.x;
    const int rem = n_items % G;
    tail = n_items < G ? n_items : (rem <= G / 2 && p.KS >= 12 ? rem : 0);
    if (tail > p.tail_items) tail = p.tail_items;
  }
  sc.n_tail = tail;
  sc.n_whole = n_items - tail;
  if (tail == 0) sc.Q = 1;
  return sc;
}

// Auxiliary bytes the producer copies into a stage: the item's codebooks (CB3K) or row scales (W8K
// per-output-channel) on the item's first stage, the stage's input scales (W8K per-input-row) on every stage.
template <int FMT, int NMAT>
__device__ __forceinline__ int aux_bytes(const DecodeParams& p, bool first) {
  if constexpr (FMT == kFmtCB3) return first ? NMAT * 1024 : 0;
  else if constexpr (is_cb8<FMT>()) return first ? NMAT * kCb8BlockBytes : 0;
  else return p.scale_axis == 1 ? (first ? NMAT * kRowsPerBlock * 4 : 0) : NMAT * kStageK * 4;
}

// What the producer tells the consumers about the stage it filled (written before the stage's full-barrier
// arrive, which releases it). item < 0 ends the consumers' loop.
struct StageHdr {
  int item, e, row0, cnt;
  int rb, kq, ks, flags;  // kq: the segment's partial-sum slot; flags: 1 = first stage of the segment,
                          // 2 = last stage of the segment, bits 8+: segments of the item (1 = whole)
};

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32)); }

// The kernel proper; HILO is a template argument so the B staging size is a compile-time constant.
//   producer warp: walks the CTA's stage range item by item (pass, 64-row block) and for each 256-input stage
//                  fills a ring slot: header, weights, aux, the pass's B rows;
//   consumer warps: dequantize + MMA per stage, then the segment's epilogue (whole item) or partial sums (cut
//                  item, finished by its last-arriving segment).
#ifndef CBMOE_DECODE_MINB_NT1
#define CBMOE_DECODE_MINB_NT1 1
#endif
// Resident CTAs the CB8 kernels are compiled for: 4 per SM for the smallest tiles (1 token tile with X8 rows, 2
// slot tiles with H8 rows: 96 registers, no spills), 3 above.
#ifndef CBMOE_CB8_MINB_SMALL
#define CBMOE_CB8_MINB_SMALL 4
#endif
template <int FMT, int NT, int HILO>
constexpr int decode_min_blocks() {
  if constexpr (is_split<FMT>()) return (NT == (HILO ? 2 : 1)) ? CBMOE_CB8_MINB_SMALL : 3;
  return NT == 1 ? CBMOE_DECODE_MINB_NT1 : 1;
}

template <int FMT, int NMAT, int NT, int EPI, int HILO, int NSTAGE>
__global__ void __launch_bounds__(kDecodeThreads, decode_min_blocks<FMT, NT, HILO>())
    decode_kernel_t(const DecodeParams p) {
  using SM = DecodeSmem<FMT, NMAT, NT, HILO, NSTAGE>;
  constexpr bool kCb8 = SM::kCb8;          // split activations, int8 MMA (CB8 or W8I)
  constexpr bool kW8I = FMT == kFmtW8I;
  constexpr int kPassTokens = SM::kPassTokens;
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
  griddep_wait();   // the plan / the previous expert kernel's output is complete past this point

  const int n_items = count_items(p, kPassTokens);
  const int RB = p.RB, KS = p.KS;
  const Schedule sc = make_schedule(p, n_items);
  const int n_tickets = sc.tickets();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------------------------------ producer
    // Items are taken one ahead: the next item's number (a ticket from the shared counter) and its pass record
    // (expert, first row, count) are requested before the current item's stages are issued, and the next item's
    // B rows right after its first stage, so their global-memory round trips overlap the current item's copies.
    int st = 0;
    uint32_t ph = 0;
    int iter = 0;
    auto take = [&]() -> int {   // meaningful in lane 0 only
      int tk = 0;
      if (lane == 0) tk = p.sched ? atomicAdd(p.sched, 1) : (int)blockIdx.x + iter * (int)gridDim.x;
      ++iter;
      return tk;
    };
    auto pass_of = [&](int it) -> PassInfo { return get_pass(p, it / RB, kPassTokens); };
    auto b_row = [&](const PassInfo& q) -> int {
      if (lane >= q.cnt || q.cnt <= 0) return -1;
      return p.tok_row ? p.tok_row[q.row0 + lane] : q.row0 + lane;
    };
    // The next ticket is taken kLookahead stages before the current one's last stage is issued, its pass record
    // read one stage later and its B rows one more, so their round trips overlap the copies; taking it later than
    // that would stall the ring, earlier would commit this CTA to more work while others may run dry.
    constexpr int kLookahead = 3;
    int tk = __shfl_sync(0xffffffffu, take(), 0);
    int item = 0, ks0 = 0, ks1 = 0, piece = -1;
    PassInfo pi{-1, 0, 0};
    int brow = -1;
    if (tk < n_tickets) {
      sc.decode(tk, item, ks0, ks1, piece);
      pi = pass_of(item);
      brow = b_row(pi);
    }
    while (tk < n_tickets) {
      int pending = 0, tn = 0;
      int item_n = 0, ks0_n = 0, ks1_n = 0, piece_n = -1;
      PassInfo pn{-1, 0, 0};
      bool has_n = false;
      int brow_n = -1;
      int next_step = 0;   // 0: take the ticket, 1: read its pass record, 2: its B rows, 3: done
      auto advance = [&]() {
        if (next_step == 0) {
          pending = take();
        } else if (next_step == 1) {
          tn = __shfl_sync(0xffffffffu, pending, 0);
          has_n = tn < n_tickets;
          if (has_n) {
            sc.decode(tn, item_n, ks0_n, ks1_n, piece_n);
            pn = pass_of(item_n);
          }
        } else if (next_step == 2) {
          if (has_n) brow_n = b_row(pn);
        }
        ++next_step;
      };
      const int rb = item % RB;
      const int nseg = piece < 0 ? 1 : sc.Q;
      if (pi.e >= 0 && pi.e < p.E && pi.cnt > 0) {
        const int n_copies = __popc(__ballot_sync(0xffffffffu, brow >= 0));
        for (int ks = ks0; ks < ks1; ++ks) {
          const bool first = ks == ks0;
          const int aux = aux_bytes<FMT, NMAT>(p, first);
          bool ok = true;
          if (lane == 0) {
            ok = mbar_wait_sleepy(&empty[st], ph ^ 1);
            if (ok) {
              hdr[st] = {item, pi.e, pi.row0, pi.cnt, rb, piece < 0 ? 0 : piece, ks,
                         (first ? 1 : 0) | (ks == ks1 - 1 ? 2 : 0) | (nseg << 8)};
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
            } else if constexpr (kCb8 && !kW8I) {
              if (lane == 0) bulk_g2s(sa, p.cb8 + cb8_block_offset(pi.e, rb, RB, NMAT), aux, &full[st]);
            } else {
              const float* scl = (lane == 0) ? p.s0 : p.s1;
              const int per = aux / NMAT;
              const float* src = (p.scale_axis == 1) ? scl + rb * kRowsPerBlock : scl + ks * kStageK;
              bulk_g2s(sa + lane * per, src, per, &full[st]);
            }
          }
          if (brow >= 0) {
            const void* src;
            if constexpr (kCb8)
              src = p.b8 + ((size_t)brow * KS + ks) * SM::kBCopy;
            else
              src = p.b + (size_t)brow * (p.K * (HILO ? 2 : 1)) + (size_t)ks * kStageK * (HILO ? 2 : 1);
            bulk_g2s(sw + SM::kWBytes + SM::kAuxBytes + lane * SM::kBRow, src, SM::kBCopy, &full[st]);
          }
          if (++st == NSTAGE) {
            st = 0;
            ph ^= 1;
          }
          if (ks >= ks1 - kLookahead && next_step < 3) advance();
        }
      }
      while (next_step < 3) advance();
      tk = tn;
      item = item_n;
      ks0 = ks0_n;
      ks1 = ks1_n;
      piece = piece_n;
      pi = pn;
      brow = brow_n;
    }
    if (lane == 0 && mbar_wait_sleepy(&empty[st], ph ^ 1)) {
      hdr[st].item = -1;
      mbar_arrive(&full[st]);
    }
    if (lane == 0) griddep_launch();   // no more copies from this CTA: the next kernel may start being placed
    return;
  }

  // -------------------------------------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  int st = 0;
  uint32_t ph = 0;
  Codebook cbg[NMAT], cbh[NMAT];
  Cb8 c8g[NMAT], c8h[NMAT];
  float sg[NMAT], sh[NMAT];   // W8K row scales; CB8 row factors
  // Few accumulator tiles per warp (NT * NMAT <= 2) make a long chain of dependent MMAs per stage; a second set
  // (odd MMA steps, the h-lo products with HILO, or the lo-part products of CB8) halves it and is added in before
  // the epilogue. (CB8 accumulates in int32: over the item with X8 rows, per chunk with H8 rows.)
  constexpr int kAccSets = (NT * NMAT <= 2 && !kCb8) ? 2 : 1;
  // Token (or slot) of a column of this lane's accumulator tile n, register i: bf16 tiles hold 8 tokens (columns
  // 2t, 2t+1 = two tokens); CB8 X8 tiles 4 tokens (columns 2t, 2t+1 = hi and lo of token t); CB8 H8 tiles 2 slots
  // (columns 2t, 2t+1 = two of the 4 parts of slot t/2). Partial sums are kept per column, j = n*8 + 2t + (i&1).
  auto col_tok = [&](int n, int i) -> int {
    if constexpr (!kCb8) return n * 8 + 2 * t + (i & 1);
    else if constexpr (HILO) return n * 2 + (t >> 1);
    else return n * 4 + t;
  };
  __shared__ float s_hmax[kConsumerWarps][8];   // CB8 SwiGLU epilogue: per-warp |h| maxima of each token
  float acc[NMAT][NT][4];
  float acc_b[kAccSets > 1 ? NMAT : 1][NT][4];
  // CB8 with X8 rows: exact int32 sums of the hi-byte and lo-byte products over the item (converted to acc, as
  // 256 hi + lo, when the segment ends)
  int ci_hi[kCb8 && !HILO ? NMAT : 1][NT][4], ci_lo[kCb8 && !HILO ? NMAT : 1][NT][4];

  // Epilogue of one item from acc (the item's full sums).
  auto epilogue = [&](const StageHdr& e) {
    const int rowbase = e.rb * kRowsPerBlock + warp * kRowsPerWarp;
    if constexpr (kCb8) {
      if constexpr (EPI == kEpiStore && HILO) {
        // down (H8 rows): the 4 part columns of a slot are spread over lane pairs (t, t^1)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          float vg = acc[0][n][0] + acc[0][n][1], vh = acc[0][n][2] + acc[0][n][3];
          vg += __shfl_xor_sync(0xffffffffu, vg, 1);
          vh += __shfl_xor_sync(0xffffffffu, vh, 1);
          const int j = col_tok(n, 0);
          if ((t & 1) || j >= e.cnt) continue;
          float* y = p.y_out + (size_t)(e.row0 + j) * p.rows + rowbase + g;
          y[0] = vg;
          y[8] = vh;
        }
      } else {
        // X8 rows: token t's low-digit column and high-digit column (x 256), times the token's factor (the sums
        // already carry the row factors)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int j = col_tok(n, 0);
          float fx = 0.f;
          if (j < e.cnt) fx = p.b8_scale[p.tok_row ? p.tok_row[e.row0 + j] : e.row0 + j];
          const float g0 = (acc[0][n][0] + acc[0][n][1] * 256.f) * fx;
          const float h0 = (acc[0][n][2] + acc[0][n][3] * 256.f) * fx;
          if constexpr (EPI == kEpiStore) {
            if (j < e.cnt) {
              const size_t o = (size_t)(e.row0 + j) * p.rows + rowbase + g;
              if (p.y_bf16 != nullptr) {
                const __nv_bfloat16 b0 = __float2bfloat16_rn(g0), b1 = __float2bfloat16_rn(h0);
                p.y_bf16[o] = *reinterpret_cast<const uint16_t*>(&b0);
                p.y_bf16[o + 8] = *reinterpret_cast<const uint16_t*>(&b1);
              } else {
                p.y_out[o] = g0;
                p.y_out[o + 8] = h0;
              }
            }
          } else {
            // SwiGLU, then h as 4 signed base-256 digits with one factor per (token, 64-row block): the block's
            // largest |h| times 2^u in [2^28, 2^29)
            const float g1 = (acc[NMAT - 1][n][0] + acc[NMAT - 1][n][1] * 256.f) * fx;
            const float h1 = (acc[NMAT - 1][n][2] + acc[NMAT - 1][n][3] * 256.f) * fx;
            float hg = 0.f, hh = 0.f;
            if (j < e.cnt) {
              hg = swiglu_clamped(g0, g1, p.limit);
              hh = swiglu_clamped(h0, h1, p.limit);
            }
            float mx = fmaxf(fabsf(hg), fabsf(hh));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            consumer_bar();   // the previous item's readers are done with s_hmax
            if (g == 0) s_hmax[warp][n * 4 + t] = mx;
            consumer_bar();
            mx = fmaxf(fmaxf(s_hmax[0][n * 4 + t], s_hmax[1][n * 4 + t]),
                       fmaxf(s_hmax[2][n * 4 + t], s_hmax[3][n * 4 + t]));
            if (j >= e.cnt) continue;
            const int u = shift_for(mx, 29);
            const int ksd = p.rows / kStageK;
            uint8_t* stage8 = p.h8_out + ((size_t)(e.row0 + j) * ksd + (e.rb >> 2)) * kH8StageBytes;
            uint8_t* row8 = stage8 + (e.rb & 3) * 256 + warp * kRowsPerWarp + g;
            int vg = __float2int_rn(ldexpf(hg, u)), vh = __float2int_rn(ldexpf(hh, u));
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int dg = (q < 3) ? (int)(int8_t)(vg & 0xff) : vg;   // balanced digits; the last one takes the rest
              const int dh = (q < 3) ? (int)(int8_t)(vh & 0xff) : vh;
              row8[q * 64] = (uint8_t)dg;
              row8[q * 64 + 8] = (uint8_t)dh;
              vg = (vg - dg) >> 8;
              vh = (vh - dh) >> 8;
            }
            if (warp == 0 && g == 0) *reinterpret_cast<float*>(stage8 + 1024 + (e.rb & 3) * 4) = ldexpf(1.f, -u);
          }
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = n * 8 + 2 * t + (i & 1);
          const int r = rowbase + g + ((i & 2) ? 8 : 0);
          if (j >= e.cnt) continue;
          const int row = e.row0 + j;
          if constexpr (EPI == kEpiSwiglu) {
            const float hv = swiglu_clamped(acc[0][n][i], acc[NMAT - 1][n][i], p.limit);
            const __nv_bfloat16 hi = __float2bfloat16_rn(hv);
            const __nv_bfloat16 lo = __float2bfloat16_rn(hv - __bfloat162float(hi));
            uint16_t* dst = p.h_out + (size_t)row * (2 * p.rows) + (r / kStageK) * (2 * kStageK) + (r % kStageK);
            dst[0] = *reinterpret_cast<const uint16_t*>(&hi);
            dst[kStageK] = *reinterpret_cast<const uint16_t*>(&lo);
          } else {
            p.y_out[(size_t)row * p.rows + r] = acc[0][n][i];
          }
        }
      }
    }
  };
  // Tail items cut into pieces (Schedule, above): a piece's partial sums go to the item's slot q when it ends;
  // its arrival on the item's counter (fence + atomic) is counted after the next stage, and the atomic's result is
  // read when the next piece or item ends (or when the consumers stop), so no global round trip stalls the MMAs.
  // The last arriver adds the Q slots up and runs the epilogue.
  constexpr int kSlotFloats = NT * 8 * NMAT * kRowsPerBlock;   // columns x matrices x rows
  int pend_state = 0;   // 0: nothing pending, 1: partials stored, 2: arrival counted (ticket in thread 0)
  StageHdr pend{};
  int ticket = 0;
  auto slot_at = [&](int item, int q, int j, int m, int rl) -> size_t {
    return ((size_t)(item - sc.n_whole) * sc.Q + q) * kSlotFloats + ((size_t)j * NMAT + m) * kRowsPerBlock + rl;
  };
  auto count_arrival = [&]() {
    __threadfence();
    consumer_bar();
    if (threadIdx.x == 0) ticket = atomicAdd(&p.done[pend.item], 1);
    pend_state = 2;
  };
  auto resolve = [&]() {
    const int nseg = pend.flags >> 8;
    if (threadIdx.x == 0) {
      s_flag = (ticket == nseg - 1) ? 1 : 0;
      if (s_flag) p.done[pend.item] = 0;   // every segment has arrived: ready for the next launch
    }
    consumer_bar();
    pend_state = 0;
    if (!s_flag) return;
    __threadfence();
    const int rl0 = warp * kRowsPerWarp + g;
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = n * 8 + 2 * t + (i & 1);
          const int rl = rl0 + ((i & 2) ? 8 : 0);
          float v = 0.f;
          if (col_tok(n, i) < pend.cnt)
            for (int q = 0; q < nseg; ++q) v += __ldcg(&p.part[slot_at(pend.item, q, j, m, rl)]);
          acc[m][n][i] = v;
        }
    epilogue(pend);
  };

  for (;;) {
    if (!mbar_wait(&full[st], ph)) return;
    const StageHdr h = hdr[st];
    if (h.item < 0) {
      if (pend_state == 1) count_arrival();
      if (pend_state == 2) resolve();
      return;
    }
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
        } else if constexpr (kCb8 && !kW8I) {
          const uint4 ca = lds128(sa + ((warp * NMAT + m) * 16 + g) * 16);
          const uint4 cb = lds128(sa + ((warp * NMAT + m) * 16 + g + 8) * 16);
          c8g[m] = {ca.x, ca.y, ca.z, ca.w};
          c8h[m] = {cb.x, cb.y, cb.z, cb.w};
          const float* rf = reinterpret_cast<const float*>(sa + NMAT * 1024) + (warp * NMAT + m) * 16;
          sg[m] = rf[g];
          sh[m] = rf[g + 8];
        } else {
          const float* sc = reinterpret_cast<const float*>(sa) + m * kRowsPerBlock + warp * kRowsPerWarp;
          sg[m] = (p.scale_axis == 1) ? sc[g] : 0.f;
          sh[m] = (p.scale_axis == 1) ? sc[g + 8] : 0.f;
          cbg[m] = cbh[m] = {0, 0, 0, 0};
        }
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[m][n][i] = 0.f;
            if constexpr (kAccSets > 1) acc_b[m][n][i] = 0.f;
            if constexpr (kCb8 && !HILO) ci_hi[m][n][i] = ci_lo[m][n][i] = 0;
          }
      }
    }

    uint32_t wd[NMAT][12];
    if constexpr (FMT == kFmtCB3 || (kCb8 && !kW8I)) {
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

    if constexpr (kCb8) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        // B fragments: column g of tile n = token n*4 + g/2, part g%2 (X8) or slot n*2 + g/4, part g%4 (H8);
        // one 16-byte load gives both k32 steps (x, y: step 0; z, w: step 1)
        uint4 bx[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (n == 0 || n * SM::kTokPerTile < h.cnt) {
            const int brow = n * SM::kTokPerTile + (HILO ? (g >> 2) : (g >> 1));
            const int part = HILO ? (g & 3) : (g & 1);
            bx[n] = lds128(sb + brow * SM::kBRow + c * (HILO ? 256 : 128) + part * 64 + 16 * t);
          }
        }
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          uint32_t ah[2][4], al[2][4];
          if constexpr (kW8I) {
            // the lane's 16 stored int8 weights of rows g and g+8 in this chunk: 8 per k32 step, as the fragment wants
            const uint8_t* u = sw + (warp * NMAT + m) * SM::kUnit;
            const uint4 qg = lds128(u + ((c * 2 + 0) * 32 + lane) * 16);
            const uint4 qh = lds128(u + ((c * 2 + 1) * 32 + lane) * 16);
            ah[0][0] = qg.x; ah[0][1] = qh.x; ah[0][2] = qg.y; ah[0][3] = qh.y;
            ah[1][0] = qg.z; ah[1][1] = qh.z; ah[1][2] = qg.w; ah[1][3] = qh.w;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              if (!(n == 0 || n * SM::kTokPerTile < h.cnt)) continue;
              if constexpr (HILO) {
                // H8 rows: this chunk's exact products, times the factor of the chunk and of the digit column
                int dh[4] = {0, 0, 0, 0};
                mma_i8<false>(dh, ah[0], bx[n].x, bx[n].y);
                mma_i8<false>(dh, ah[1], bx[n].z, bx[n].w);
                const float F = *reinterpret_cast<const float*>(sb + (n * 2 + (t >> 1)) * SM::kBRow + 1024 + 4 * c);
                const float f0 = (t & 1) ? F * 65536.f : F, f1 = f0 * 256.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][n][i] += (float)dh[i] * ((i & 1) ? f1 : f0);
              } else {
                mma_i8<false>(ci_hi[m][n], ah[0], bx[n].x, bx[n].y);
                mma_i8<false>(ci_hi[m][n], ah[1], bx[n].z, bx[n].w);
              }
            }
          } else {
            cb8_dequant_chunk(wd[m][3 * c], wd[m][3 * c + 1], wd[m][3 * c + 2], c8g[m], c8h[m], ah, al);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              if (!(n == 0 || n * SM::kTokPerTile < h.cnt)) continue;
              if constexpr (HILO) {
                // this chunk's exact products (T = 256 hi + lo), then times the factor of the chunk and of the part
                // (digit p of the slot's h: 256^p)
                int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0};
                mma_i8<false>(dh, ah[0], bx[n].x, bx[n].y);
                mma_i8<true>(dl, al[0], bx[n].x, bx[n].y);
                mma_i8<false>(dh, ah[1], bx[n].z, bx[n].w);
                mma_i8<true>(dl, al[1], bx[n].z, bx[n].w);
                const float F = *reinterpret_cast<const float*>(sb + (n * 2 + (t >> 1)) * SM::kBRow + 1024 + 4 * c);
                const float f0 = (t & 1) ? F * 65536.f : F, f1 = f0 * 256.f;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  acc[m][n][i] += (float)(dh[i] * 256 + dl[i]) * ((i & 1) ? f1 : f0);
              } else {
                mma_i8<false>(ci_hi[m][n], ah[0], bx[n].x, bx[n].y);
                mma_i8<true>(ci_lo[m][n], al[0], bx[n].x, bx[n].y);
                mma_i8<false>(ci_hi[m][n], ah[1], bx[n].z, bx[n].w);
                mma_i8<true>(ci_lo[m][n], al[1], bx[n].z, bx[n].w);
              }
            }
          }
        }
      }
    } else {
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
              if constexpr (kAccSets > 1) {
                if constexpr (HILO) {
                  mma_bf16(acc[m][n], a[s], bf[n][2 * s], bf[n][2 * s + 1]);
                  mma_bf16(acc_b[m][n], a[s], bl[n][2 * s], bl[n][2 * s + 1]);
                } else {
                  mma_bf16((s & 1) ? acc_b[m][n] : acc[m][n], a[s], bf[n][2 * s], bf[n][2 * s + 1]);
                }
              } else {
                mma_bf16(acc[m][n], a[s], bf[n][2 * s], bf[n][2 * s + 1]);
                if constexpr (HILO) mma_bf16(acc[m][n], a[s], bl[n][2 * s], bl[n][2 * s + 1]);
              }
            }
          }
        }
      }
    }
    }   // bf16 formats
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (++st == NSTAGE) {
      st = 0;
      ph ^= 1;
    }
    if (pend_state == 1) count_arrival();
    if (!(h.flags & 2)) continue;

    // ---------------------------------------------------------------------------------- item epilogue
    // CB8: the segment's sums times the row factors now, while they are the item's: a cut item's epilogue runs
    // later (in its last-arriving piece), after this warp may have loaded the next item's.
    if constexpr (kCb8) {
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float v = HILO  ? acc[m][n][i]
                            : kW8I ? (float)ci_hi[m][n][i]
                                   : (float)ci_hi[m][n][i] * 256.f + (float)ci_lo[m][n][i];
            acc[m][n][i] = v * ((i & 2) ? sh[m] : sg[m]);
          }
    }
    if constexpr (kAccSets > 1) {
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[m][n][i] += acc_b[m][n][i];
    }
    if ((h.flags >> 8) > 1) {
      const int rl0 = warp * kRowsPerWarp + g;
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = n * 8 + 2 * t + (i & 1);
            if (col_tok(n, i) < h.cnt) p.part[slot_at(h.item, h.kq, j, m, rl0 + ((i & 2) ? 8 : 0))] = acc[m][n][i];
          }
      if (pend_state == 2) resolve();   // the previous segment's; acc is free again
      pend = h;
      pend_state = 1;
      continue;
    }
    epilogue(h);
  }
}

// Weighted sum of the routed slots' outputs (einsum "nkd,nk->nd"), plus an optional f32 addend (the shared
// expert's output): out[n][r] = sum_j w[n][j] * y_sorted[row_slot[n][j]][r] (+ add[n][r]), written as f32 and/or
// bf16. Four consecutive r per thread; the slot rows, weights and slot outputs each take one memory round trip.
__global__ void combine_kernel(const float* __restrict__ y_sorted, const int* __restrict__ row_slot,
                               const float* __restrict__ wts, int N, int topk, int H, const float* __restrict__ add,
                               float* __restrict__ out_f32, uint16_t* __restrict__ out_bf16) {
  griddep_wait();
  griddep_launch();
  const int H4 = H / 4;
  const long long total = (long long)N * H4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / H4), c4 = (int)(i % H4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q0 = 0; q0 < topk; q0 += 8) {
      int rs[8];
      float wt[8];
      float4 yv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool in = q0 + q < topk;
        rs[q] = in ? row_slot[n * topk + q0 + q] : -1;
        wt[q] = in ? wts[n * topk + q0 + q] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        yv[q] = rs[q] >= 0 ? reinterpret_cast<const float4*>(y_sorted + (size_t)rs[q] * H)[c4]
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v.x += wt[q] * yv[q].x;
        v.y += wt[q] * yv[q].y;
        v.z += wt[q] * yv[q].z;
        v.w += wt[q] * yv[q].w;
      }
    }
    if (add != nullptr) {
      const float4 a = reinterpret_cast<const float4*>(add + (size_t)n * H)[c4];
      v.x += a.x;
      v.y += a.y;
      v.z += a.z;
      v.w += a.w;
    }
    const size_t o = (size_t)n * H4 + c4;
    if (out_f32 != nullptr) reinterpret_cast<float4*>(out_f32)[o] = v;
    if (out_bf16 != nullptr) {
      uint2 pk;
      pk.x = pack_bf16x2(v.x, v.y);
      pk.y = pack_bf16x2(v.z, v.w);
      reinterpret_cast<uint2*>(out_bf16)[o] = pk;
    }
  }
}

// ------------------------------------------------------------------------------------------------ launch
template <int FMT, int NMAT, int NT, int EPI, int HILO, int NSTAGE>
int launch_decode_t(const DecodeParams& p, int kind, cudaStream_t stream) {
  using SM = DecodeSmem<FMT, NMAT, NT, HILO, NSTAGE>;
  auto kern = decode_kernel_t<FMT, NMAT, NT, EPI, HILO, NSTAGE>;
  static PerDevice s_grid;
  long long grid = 0;
  int rc = per_device(s_grid, [&](long long& v) -> int {
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kTotal));
    int per_sm = 0;
    CBMOE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecodeThreads, SM::kTotal));
    v = (long long)num_sms() * (per_sm > 0 ? per_sm : 1);
    return CBMOE_OK;
  }, &grid);
  if (rc) return rc;
  const int g = (p.grid_cap > 0 && p.grid_cap < grid) ? p.grid_cap : (int)grid;
  prof_begin(kind, stream);
  CBMOE_CUDA_TRY(launch_pdl(kern, dim3(g), dim3(kDecodeThreads), SM::kTotal, stream, p));
  prof_end(kind, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

#ifndef CBMOE_STAGES_CB3
#define CBMOE_STAGES_CB3 3
#endif
#ifndef CBMOE_STAGES_NT1
#define CBMOE_STAGES_NT1 3
#endif
constexpr int kStagesCB3 = CBMOE_STAGES_CB3;
constexpr int kStagesW8 = 2;   // the W8 kernels run beside the routed ones (side stream): small footprint

template <int FMT, int NMAT, int EPI, int HILO>
int launch_decode_nt(const DecodeParams& p, int nt, int kind, cudaStream_t stream) {
  constexpr int NS = (FMT == kFmtCB3) ? kStagesCB3 : kStagesW8;
  switch (nt) {
    case 1: return launch_decode_t<FMT, NMAT, 1, EPI, HILO, CBMOE_STAGES_NT1>(p, kind, stream);
    case 2: return launch_decode_t<FMT, NMAT, 2, EPI, HILO, NS>(p, kind, stream);
    default: return launch_decode_t<FMT, NMAT, 4, EPI, HILO, NS>(p, kind, stream);
  }
}

int launch_combine(const float* y_sorted, const int* row_slot, const float* wts, int N, int topk, int H,
                   const float* add, float* out_f32, uint16_t* out_bf16, cudaStream_t stream) {
  const long long total = (long long)N * (H / 4);
  int blocks = (int)((total + 255) / 256);
  if (blocks > num_sms() * 8) blocks = num_sms() * 8;
  if (blocks < 1) blocks = 1;
  prof_begin(kProfCombine, stream);
  CBMOE_CUDA_TRY(launch_pdl(combine_kernel, dim3(blocks), dim3(256), 0, stream, y_sorted, row_slot, wts, N, topk, H,
                            add, out_f32, out_bf16));
  prof_end(kProfCombine, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

// Ring stages of the CB8 kernels: 3 with X8 rows (a gate+up stage is 17-19 KB), 4 with H8 rows (down: 12-16 KB),
// so that the resident CTAs fit the SM's shared memory.
#ifndef CBMOE_STAGES_CB8_X8
#define CBMOE_STAGES_CB8_X8 3
#endif
#ifndef CBMOE_STAGES_CB8_H8
#define CBMOE_STAGES_CB8_H8 4
#endif
template <int FMT, int NMAT, int EPI, int HILO>
int launch_cb8_nt(const DecodeParams& p, int nt, int kind, cudaStream_t stream) {
  constexpr int NS = HILO ? CBMOE_STAGES_CB8_H8 : CBMOE_STAGES_CB8_X8;
  if constexpr (HILO != 0) {   // slot tiles of 2: 2 or 4 tiles (passes of up to 4 or 8 slots)
    if (nt <= 2) return launch_decode_t<FMT, NMAT, 2, EPI, HILO, NS>(p, kind, stream);
    return launch_decode_t<FMT, NMAT, 4, EPI, HILO, NS>(p, kind, stream);
  } else {                     // token tiles of 4: 1 or 2 tiles (passes of up to 4 or 8 tokens)
    if (nt <= 1) return launch_decode_t<FMT, NMAT, 1, EPI, HILO, NS>(p, kind, stream);
    return launch_decode_t<FMT, NMAT, 2, EPI, HILO, NS>(p, kind, stream);
  }
}

int decode_cb8_gateup(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_cb8_nt<kFmtCB8A, 2, kEpiSwiglu, 0>(p, nt, kProfCb3GateUp, s);
}
int decode_cb8_down(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_cb8_nt<kFmtCB8A, 1, kEpiStore, 1>(p, nt, kProfCb3Down, s);
}
int decode_w8i_logits(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_cb8_nt<kFmtW8I, 1, kEpiStore, 0>(p, nt, kProfW8Single, s);
}
int decode_w8i_gateup(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_cb8_nt<kFmtW8I, 2, kEpiSwiglu, 0>(p, nt, kProfW8GateUp, s);
}
int decode_w8i_down(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_cb8_nt<kFmtW8I, 1, kEpiStore, 1>(p, nt, kProfW8Down, s);
}
int decode_cb8_single(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_cb8_nt<kFmtCB8A, 1, kEpiStore, 0>(p, nt, kProfCb3Single, s);
}

__global__ void split_x_kernel(const uint16_t* __restrict__ x, int N, int K, uint8_t* __restrict__ x8,
                               float* __restrict__ scale) {
  __shared__ float red[32];
  griddep_wait();
  griddep_launch();
  for (int r = blockIdx.x; r < N; r += gridDim.x)
    split_x_row(x + (size_t)r * K, K, x8 + (size_t)r * (K / kStageK) * kX8StageBytes, scale + r, red);
}

int launch_split_x(const uint16_t* x, int N, int K, uint8_t* x8, float* scale, cudaStream_t stream) {
  if (N <= 0) return CBMOE_OK;
  const int blocks = N < num_sms() * 4 ? N : num_sms() * 4;
  prof_begin(kProfOther, stream);
  CBMOE_CUDA_TRY(launch_pdl(split_x_kernel, dim3(blocks), dim3(256), 0, stream, x, N, K, x8, scale));
  prof_end(kProfOther, stream);
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
int decode_w8_down_store(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtW8, 1, kEpiStore, 1>(p, nt, kProfW8Down, s);
}
int decode_w8_single(const DecodeParams& p, int nt, cudaStream_t s) {
  return launch_decode_nt<kFmtW8, 1, kEpiStore, 0>(p, nt, kProfW8Single, s);
}

}  // namespace cbmoe
