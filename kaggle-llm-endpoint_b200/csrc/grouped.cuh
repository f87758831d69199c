// Parameters and entry points of the grouped (prefill / large-batch) expert GEMMs on tcgen05 (grouped.cu).
#pragma once
#include <cuda.h>

#include "layout.cuh"

namespace cbmoe {

constexpr int kGrpEpiSwiglu = 0;   // NMAT = 2: out = bf16(swiglu_clamped(gate, up))
constexpr int kGrpEpiStore = 1;    // NMAT = 1: out = bf16(acc)
constexpr int kGrpEpiStoreF32 = 2; // NMAT = 1: out_f32 = acc
constexpr int kGrpTileM = 128;     // weight rows per tile (tcgen05 M)
// Token rows per routed CB3 pass (tcgen05 N). A 128 x 16 slice of weights costs the tensor core about as long for
// N = 16 as for N = 256, so experts with many rows take 256-row passes; with few rows (a pass holds them all
// either way) 128-row passes keep two accumulator buffers for gate/up, so the epilogue overlaps the next item.
constexpr int kGrpTileN = 256;
inline int grp_pass_tokens(long long S, int E) { return E > 0 && S > 128LL * E ? 256 : 128; }

struct GroupedParams {
  const uint8_t* wq;       // CB3K index bits or W8K int8, unit layout (layout.cuh)
  const uint32_t* cb;      // CB3K codebooks
  const float* s0;         // W8K scales (matrix 0 / 1)
  const float* s1;
  int scale_axis;
  int rows, K;             // weight rows per expert (multiple of 128) and inputs (multiple of 256)
  const int* pass_expert;  // sorted-row passes of <= 256 rows of one expert (nullptr: dense, passes over N rows)
  const int* pass_row0;
  const int* pass_cnt;
  const int* n_pass;
  int N;                   // dense: token rows
  int E;
  float limit;
  uint16_t* out;           // bf16 [row][rows]: row = pass_row0 + token index
  float* out_f32;          // kGrpEpiStoreF32
};

// tn: token rows per pass of the routing plan (128 or 256).
int grouped_cb3_gateup(const GroupedParams& p, const void* b, int b_rows, int tn, cudaStream_t s);
int grouped_cb3_down(const GroupedParams& p, const void* b, int b_rows, int tn, cudaStream_t s);
int grouped_w8_gateup(const GroupedParams& p, const void* b, int b_rows, cudaStream_t s);
int grouped_w8_store(const GroupedParams& p, const void* b, int b_rows, cudaStream_t s);
int grouped_w8_store_f32(const GroupedParams& p, const void* b, int b_rows, cudaStream_t s);
int launch_gather_rows(const uint16_t* x, int H, const int* tok_row, int rows, uint16_t* xs, cudaStream_t s);
int launch_combine_bf16(const uint16_t* y_sorted, const int* row_slot, const float* wts, int N, int topk, int H,
                        const uint16_t* add_bf16, float* out_f32, uint16_t* out_bf16, cudaStream_t s,
                        const float* add_f32 = nullptr);

}  // namespace cbmoe
