// Parameters and entry points of the tcgen05 decode kernels (tcdecode.cu): the routed CB3 experts of small and
// medium batches (up to 64 tokens per expert pass), dequantized into TMEM and contracted on the tensor cores.
#pragma once
#include "layout.cuh"

namespace cbmoe {

constexpr int kTcTileM = 128;   // weight rows per item (tcgen05 M)
constexpr int kTcPieces = 4;    // pieces a tail item is cut into (at most; the 256-input stages if fewer)

struct TcParams {
  const uint8_t* wq;        // CB3K index bits (unit layout, layout.cuh)
  const uint32_t* cb;       // CB3K codebooks
  int rows, K;              // weight rows per expert (multiple of 128), inputs (multiple of 256)
  const int* pass_expert;   // passes of <= TN sorted rows of one expert (routing plan)
  const int* pass_row0;
  const int* pass_cnt;
  const int* n_pass;
  int E;
  float limit;
  uint16_t* h_out;          // gate/up: SwiGLU output as two bf16 planes [plane][sorted row][rows] (hi, then
  size_t h_plane;           //   lo = bf16(h - hi)), inputs of every 64-wide chunk in tc_perm64 order
  float* y_out;             // down: fp32 [sorted row][rows]
  int* sched;               // ticket counter, zero at launch
  int* done;                // arrival counters of the tail items (4 per item: one per TMEM lane quarter), zero at
                            //   launch; the last arriver resets its counter
  float* part;              // partial sums of the tail items' pieces (nullptr: every item whole)
  int tail_items;           // tail items `part` holds
  int grid_cap;             // CTAs to launch at most (0: one per SM)
};

// Order of the 64 inputs of a chunk in the token operand: position 16s + 4a + b holds input 16a + 4s + b (the
// order in which the dequant's register fragments land in TMEM). The map is its own inverse.
__host__ __device__ constexpr int tc_perm64(int k) { return (((k >> 2) & 3) << 4) | ((k >> 4) << 2) | (k & 3); }

// Token rows per pass for S real slots over E experts.
int tc_pass_tokens(long long S, int E);
size_t tc_part_bytes(int tail_items, int tn, int nmat);
int tc_tail_items(long long items);

// xs[r] = x[tok_row[r]] with every 64-input chunk in tc_perm64 order (zero rows where tok_row < 0).
int launch_gather_perm(const uint16_t* x, int H, const int* tok_row, int rows, uint16_t* xs, cudaStream_t s);
// Gate/up + SwiGLU over the gathered tokens xs [xs_rows][K] -> p.h_out.
int tc_cb3_gateup(const TcParams& p, const uint16_t* xs, int xs_rows, int tn, cudaStream_t s);
// Down over the two h planes [h_rows][K] (hi, lo) -> p.y_out.
int tc_cb3_down(const TcParams& p, const uint16_t* h_hi, const uint16_t* h_lo, int h_rows, int tn, cudaStream_t s);

}  // namespace cbmoe
