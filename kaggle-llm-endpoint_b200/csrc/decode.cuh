// Parameters and entry points of the decode / small-batch expert kernels (decode.cu).
#pragma once
#include "layout.cuh"

namespace cbmoe {

constexpr int kEpiSwiglu = 0;
constexpr int kEpiStore = 1;
constexpr int kConsumerWarps = kWarpsPerBlock;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;

struct DecodeParams {
  const uint8_t* wq;        // weights in unit layout (CB3K index bits or W8K int8)
  const uint32_t* cb;       // CB3K codebooks
  const uint8_t* cb8;       // CB8 tables + row factors (layout.cuh)
  const float* s0;          // W8K scales, matrix 0 / 1
  const float* s1;
  int scale_axis;
  int rows, K, RB, KS;
  const uint16_t* b;        // B operand rows (bf16): [*, K], or hi/lo interleaved [*, 2K] when b_hilo
  int b_hilo;
  const uint8_t* b8;        // CB8: B rows as X8 ([*][K/256][512 B]) or, for down, H8 ([*][K/256][1040 B])
  const float* b8_scale;    // CB8 with X8 rows: the factor of each B row
  const int* tok_row;       // sorted row -> B row; nullptr: B row = sorted row
  const int* pass_expert;   // nullptr: one expert (0) and passes over rows 0..N-1
  const int* pass_row0;
  const int* pass_cnt;
  const int* n_pass;
  int N;
  int E;
  float limit;
  uint16_t* h_out;          // SWIGLU: [sorted row][2*rows] (per 256 block: hi 256 | lo 256)
  uint8_t* h8_out;          // CB8 SWIGLU: H8 rows [sorted row][rows/256][1040 B]
  float* y_out;             // STORE: [row][rows]
  uint16_t* y_bf16;         // STORE with X8 rows: bf16 [row][rows] instead of y_out (the int8 lm_head)
  // work distribution (decode.cu, Schedule): tickets over whole items, then over pieces of the tail items
  int grid_cap;             // CTAs to launch at most (0: the resident grid)
  int* sched;               // [0] = ticket counter, zero at launch (nullptr: static round-robin over tickets)
  int tail_items;           // tail items the partial-sum space holds
  int* done;                // arrival counter per item [passes x RB], zero at launch, reset by the last arriver
  float* part;              // partial sums of the tail items' pieces, [tail_items][Q][8*NT][NMAT][64] f32
                            // (nullptr: every item whole)
};

constexpr int kDecodePieces = 4;   // pieces per tail item (at most; KS if smaller)

// Partial-sum space of one decode launch (DecodeParams::part).
inline size_t decode_part_bytes(int tail_items, int nt, int nmat) {
  return (size_t)tail_items * kDecodePieces * (8 * nt) * nmat * kRowsPerBlock * sizeof(float);
}

// CB8 (int8-digit) kernels: nt = token tiles of 4 (gate/up, single; 1 or 2) or slot tiles of 2 (down; 2 or 4).
int decode_cb8_gateup(const DecodeParams& p, int nt, cudaStream_t s);
int decode_cb8_down(const DecodeParams& p, int nt, cudaStream_t s);
int decode_cb8_single(const DecodeParams& p, int nt, cudaStream_t s);
// int8 leaves (W8K, per-output-column scales) times X8 rows, bf16 out: the int8 lm_head (nt: token tiles of 4).
int decode_w8i_logits(const DecodeParams& p, int nt, cudaStream_t s);
// The int8 shared expert (W8K leaves, per-output-channel scales) on the int8 MMA: gate/up on X8 rows with the
// SwiGLU epilogue writing H8 rows, down on those H8 rows storing f32. No dequant arithmetic: the stored leaves are
// the MMA's A fragments.
int decode_w8i_gateup(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8i_down(const DecodeParams& p, int nt, cudaStream_t s);
// X8 rows of N bf16 rows of K inputs (K % 256 == 0): x8 [N][K/256][512 B], scale [N].
int launch_split_x(const uint16_t* x, int N, int K, uint8_t* x8, float* scale, cudaStream_t stream);
int decode_cb3_gateup(const DecodeParams& p, int nt, cudaStream_t s);
int decode_cb3_down(const DecodeParams& p, int nt, cudaStream_t s);
int decode_cb3_single(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8_gateup(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8_single(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8_down_store(const DecodeParams& p, int nt, cudaStream_t s);
int launch_combine(const float* y_sorted, const int* row_slot, const float* wts, int N, int topk, int H,
                   const float* add, float* out_f32, uint16_t* out_bf16, cudaStream_t stream);
// The routing plan; with x8 != nullptr the same launch also writes the X8 rows of x [N_x][K] (extra CTAs).
struct SplitX {
  const uint16_t* x = nullptr;
  int N = 0, K = 0;
  uint8_t* x8 = nullptr;
  float* scale = nullptr;
};
int launch_route_plan(const int32_t* idx, const float* w, int T, int k, int E, int tm, int pass_tokens,
                      int32_t* plan, cudaStream_t stream, int* zero = nullptr, int n_zero = 0,
                      const SplitX* split = nullptr);

}  // namespace cbmoe
