// Internal interface between the C-ABI files (capi.cu, ep.cu): workspace layouts and the routed-expert kernel
// sequences of one layer call. Not part of the public ABI.
#pragma once
#include "decode.cuh"
#include "grouped.cuh"

namespace cbmoe {
namespace lyr {

struct PlanLayoutHost {
  int64_t off[14];
};

// Workspace of the decode path (layout documented at decode_workspace in capi.cu).
struct DecodeWorkspace {
  size_t plan, x8, x8s, h, y, hs, ys, xs8, xs8s, done, part_gu, part_dn, part_sgu, part_sdn, total;
  int cb8;                                    // routed experts on the CB8 (int8-digit) kernels
  int nt, nt_dn;                              // column tiles of the routed gate/up and down kernels
  int nt_s, Rp, P, Ps, RB_gu, RB_dn;
  int tail_gu, tail_dn, tail_sgu, tail_sdn;   // partial-sum space of each launch, in tail items
  int n_zero_routed, n_zero_shared;           // arrival counters (words)
  PlanLayoutHost L;
};

// Resident CTAs per SM of the decode kernels are at most this (their shared memory bounds it).
constexpr int kDecodeMaxCtasPerSm = 4;

struct GroupedWorkspace {
  size_t plan, xs, h, y, hs, sy, total;
  int Rp;
  int tn;                                     // token rows per routed pass (grp_pass_tokens)
  PlanLayoutHost L;
};

struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

// CTAs of the shared-expert kernels, which run on the side stream beside the routed kernels: few enough to leave
// the routed kernels most of the GPU, enough to finish well within them.
#ifndef CBMOE_SIDE_CTAS
#define CBMOE_SIDE_CTAS 48
#endif
constexpr int kSideCtas = CBMOE_SIDE_CTAS;
// Token rows above which the int8 kernels (cbmoe_w8_linear, the shared expert) run the tcgen05 GEMM instead of
// the decode kernel.
constexpr int kW8DecodeMaxTokens = 64;

// Shared expert of one layer call on the side stream (forked after the caller's prior work on `stream`, its
// counters zeroed there first): gate/up (x -> hs, SwiGLU) then down (hs -> ys f32), by the decode kernels up to
// kW8DecodeMaxTokens tokens and the tensor-core kernels above. The caller joins `side->join` before reading ys.
// grid_cap: CTAs of the decode kernels (kSideCtas beside routed kernels; 0: the whole GPU).
int shared_side(const cbmoe_shared* sh, const uint16_t* x, int N, int H, int I, float limit, uint8_t* ws,
                const DecodeWorkspace& W, SideStream* side, cudaStream_t stream, int grid_cap = kSideCtas);

size_t align_up(size_t v);
PlanLayoutHost host_plan_layout(int T, int k, int E, int tm, int pass_tokens);
int decode_nt(int N);
int decode_nt_routed(int N, int k, int E);
// slots_hint: the slots expected to be real when N*k counts empty ones too (< 0: N*k); picks the token tile.
// cb8: the experts carry CB8 tables (cbmoe_experts.gateup_cb8 / down_cb8), so the CB8 kernels run.
DecodeWorkspace decode_workspace(int E, int H, int I, int N, int k, long long slots_hint, int cb8);
GroupedWorkspace grouped_workspace(int E, int H, int I, int N, int k);
int pick_path(int N, int k, int path);
bool aligned16(const void* p);
bool experts_ok(const cbmoe_experts* ex);
bool has_cb8(const cbmoe_experts* ex);
bool shared_ok(const cbmoe_shared* sh);
DecodeParams base_params();
int side_stream(SideStream** out);
int routed_decode(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w, int k,
                  float limit, uint8_t* ws, const DecodeWorkspace& W, cudaStream_t stream);
int routed_grouped(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w, int k,
                   float limit, uint8_t* ws, const GroupedWorkspace& W, cudaStream_t stream);

}  // namespace lyr

// Peer-memory transport of the expert-parallel layer (ep_peer.cu).
struct EpPeer;
bool ep_peer_matches(const EpPeer* pe, int nranks, int rank, int H, int cap);
bool ep_peer_poisoned(const EpPeer* pe);
// Dispatch in two launches: the rows into the peers' memory (send), then the wait for every peer's rows (wait);
// the caller may queue independent work on other streams between the two.
int ep_peer_dispatch_send(EpPeer* pe, const uint16_t* x, int H, const int32_t* slot_pos, int S, int k,
                          const int32_t* send_meta, cudaStream_t stream);
int ep_peer_dispatch_wait(EpPeer* pe, cudaStream_t stream);
int ep_peer_return(EpPeer* pe, const void* y_sorted, bool bf16, const int32_t* row_slot, const int32_t* recv_meta,
                   int R, int H, cudaStream_t stream);
uint16_t* ep_peer_in_x(EpPeer* pe);
int32_t* ep_peer_in_meta(EpPeer* pe);
void* ep_peer_in_y(EpPeer* pe);

// Int8 tensor-core kernels of the IQ2_S / IQ3_S expert tables (iq8.cu).
bool iq8_type(int ggml_type);
size_t iq8_table_bytes(int ggml_type, int E, int rows, int K);
// R rows of K inputs (bf16, or f32 when f32) -> X8 rows in ggml_type's storage order + one factor per row.
int iq8_split(int ggml_type, const void* x, bool f32, int R, int K, uint8_t* x8, float* scale, cudaStream_t s);
// The same for h = swiglu_clamped(g, u, limit) of f32 rows g, u (h itself is not stored).
int iq8_swiglu_split(int ggml_type, const float* g, const float* u, float limit, int R, int K, uint8_t* x8,
                     float* scale, cudaStream_t s);
// out[sorted row][rows] = W_e x8[row] over a routing plan's passes (of up to 8 rows); tok_row maps a sorted row to
// its X8 row (nullptr: itself).
int iq8_matvec(int ggml_type, const void* table8, int E, int rows, int K, const int32_t* pass_expert,
               const int32_t* pass_row0, const int32_t* pass_cnt, const int32_t* n_pass, const int32_t* tok_row,
               const uint8_t* x8, const float* x8_scale, float* out, int kind, cudaStream_t s);
}  // namespace cbmoe
