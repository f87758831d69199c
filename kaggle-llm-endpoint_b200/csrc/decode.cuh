// Parameters and entry points of the decode / small-batch expert kernels (decode.cu).
#pragma once
#include "layout.cuh"

namespace cbmoe {

constexpr int kEpiSwiglu = 0;
constexpr int kEpiStore = 1;
constexpr int kEpiCombine = 2;
constexpr int kConsumerWarps = kWarpsPerBlock;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;

struct DecodeParams {
  const uint8_t* wq;        // weights in unit layout (CB3K index bits or W8K int8)
  const uint32_t* cb;       // CB3K codebooks
  const float* s0;          // W8K scales, matrix 0 / 1
  const float* s1;
  int scale_axis;
  int rows, K, RB, KS;
  const uint16_t* b;        // B operand rows (bf16): [*, K], or hi/lo interleaved [*, 2K] when b_hilo
  int b_hilo;
  const int* tok_row;       // sorted row -> B row; nullptr: B row = sorted row
  const int* pass_expert;   // nullptr: one expert (0) and passes over rows 0..N-1
  const int* pass_row0;
  const int* pass_cnt;
  const int* n_pass;
  int N;
  int E;
  float limit;
  uint16_t* h_out;          // SWIGLU: [sorted row][2*rows] (per 256 block: hi 256 | lo 256)
  float* y_out;             // STORE: [row][rows]
  const float* y_sorted;    // COMBINE: routed slot outputs [sorted row][rows] (nullptr: none)
  const int* row_slot;      //          sorted row of slot (n, j), [N, topk]
  const float* wts;         //          routing weights [N, topk]
  int topk;
  uint16_t* out_bf16;       //          [N][rows]
  // work distribution
  int KQ;                   // K splits per (pass, row block): 1, or > 1 with partial sums + last-arriver epilogue
  int* sched;               // [0] = next-item counter, zero at launch (nullptr: static round-robin over items)
  int* done;                // KQ > 1: arrival counter per (pass, row block), zero at launch, reset by the last
  float* part;              // KQ > 1: partial sums [KQ][part_rows][NMAT][rows]
  int part_rows;
};

int decode_cb3_gateup(const DecodeParams& p, int nt, cudaStream_t s);
int decode_cb3_down(const DecodeParams& p, int nt, cudaStream_t s);
int decode_cb3_single(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8_gateup(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8_down_combine(const DecodeParams& p, int nt, cudaStream_t s);
int decode_w8_single(const DecodeParams& p, int nt, cudaStream_t s);
int launch_combine(const float* y_sorted, const int* row_slot, const float* wts, int N, int topk, int H, float* y,
                   cudaStream_t stream);
int launch_route_plan(const int32_t* idx, const float* w, int T, int k, int E, int tm, int pass_tokens,
                      int32_t* plan, cudaStream_t stream, int* zero = nullptr, int n_zero = 0);

}  // namespace cbmoe
