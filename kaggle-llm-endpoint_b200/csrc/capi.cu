// C-ABI entry points of the expert layer (include/cbmoe.h): argument checks, workspace carving and the kernel
// sequence of one call. The drop-in boundary is ResidentFetch.apply (resident.py:100-108) and moe_dense below the
// router (model.py:840-856).
#include <cstdio>
#include <mutex>

#include "decode.cuh"
#include "grouped.cuh"
#include "layer.cuh"

namespace cbmoe {

__device__ int g_device_errors = 0;

namespace lyr {
thread_local int t_last_cuda_error = 0;

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }


PlanLayoutHost host_plan_layout(int T, int k, int E, int tm, int pass_tokens) {
  PlanLayoutHost L;
  cbmoe_plan_layout(T, k, E, tm, pass_tokens, L.off);
  return L;
}

// Token tiles (of 8) per pass of the decode kernels. Shared expert: every token goes to the one expert, so by N.
int decode_nt(int N) { return N <= 8 ? 1 : (N <= 16 ? 2 : 4); }
// Routed experts: by the average slots per expert (an expert with more tokens than a pass takes several passes;
// larger passes cost shared memory, occupancy and MMA issue slots on every item). Measured on one B200 at 12.8
// slots per expert (20-80 experts): 16-token passes 1.8x faster than 32-token ones, 1.1-1.3x faster than 8-token
// ones; at 6.4 slots per expert 8-token passes 1.1x faster than 16-token ones, 2.1x than 32-token ones.
int decode_nt_routed(int N, int k, int E) {
  const long long S = (long long)N * k;
#ifndef CBMOE_NT1_SLOTS_PER_EXPERT
#define CBMOE_NT1_SLOTS_PER_EXPERT 2
#endif
#ifndef CBMOE_NT2_SLOTS_PER_EXPERT
#define CBMOE_NT2_SLOTS_PER_EXPERT 16
#endif
  return S <= (long long)CBMOE_NT1_SLOTS_PER_EXPERT * E ? 1
                                                        : (S <= (long long)CBMOE_NT2_SLOTS_PER_EXPERT * E ? 2 : 4);
}

// Workspace of the decode path:
//   plan | x8 (N x H/256 x 512 B: the tokens as X8 rows, CB8 tables only) | x8 factors (N f32) |
//   h (the SwiGLU output of the routed slots: Rp x 2I bf16 (hi, lo) for the bf16 kernels, Rp x I/256 x 1040 B H8
//   rows for the CB8 ones) | y_sorted (Rp x H f32) | h_shared (N x 2I bf16, or N x I/256 x 1040 B H8 rows) |
//   y_shared (N x H f32) | the shared expert's own X8 rows of x (N x H x 2 B) and factors (N f32) |
//   scheduling words: routed [gate/up tickets, down tickets, gate/up arrival counters, down arrival counters]
//                     (zeroed by the plan kernel), shared [the same] (zeroed by a memset on the side stream) |
//   partial sums of the tail items' pieces of the routed gate/up, routed down, shared gate/up, shared down.

// Tail items a decode launch cuts into pieces: at most half its resident grid (the kernel takes the same bound).
int decode_tail_items(long long items) {
  const long long half = (long long)num_sms() * kDecodeMaxCtasPerSm / 2;
  return (int)(items < half ? items : half);
}

// Token tiles of the CB8 gate/up kernel (4 tokens each) by the average slots per expert; its passes hold 4 * nt
// rows, and the down kernel takes the same passes in tiles of 2 slots (2 * nt tiles).
int cb8_nt_routed(long long S, int E) { return S <= 2LL * E ? 1 : 2; }

// The CB8 kernels up to 4 slots per expert on average, the bf16 ones above: per token tile the CB8 kernels do 2
// (gate/up) or 8 (down) int8 MMAs per 32 inputs where the bf16 ones do 2 and 4 per 16 for twice the tokens, so the
// table lookups they save stop paying once passes fill several tiles (measured on one B200, 160 experts at 12.8
// slots each, 16-token passes: CB8 gate/up 589 us, down 682 us; the grouped GEMMs 506 and 362 us).
bool use_cb8(long long S, int E, int cb8) { return cb8 && S <= 4LL * E; }

DecodeWorkspace decode_workspace(int E, int H, int I, int N, int k, long long slots_hint, int cb8) {
  DecodeWorkspace w;
  const long long S_real = slots_hint >= 0 ? (slots_hint < N ? slots_hint : N) : (long long)N * k;
  cb8 = use_cb8(S_real, E, cb8) ? 1 : 0;
  w.cb8 = cb8;
  if (cb8) {
    w.nt = cb8_nt_routed(S_real, E);
    w.nt_dn = 2 * w.nt;
  } else {
    w.nt = slots_hint >= 0 ? decode_nt_routed((int)S_real, 1, E) : decode_nt_routed(N, k, E);
    w.nt_dn = w.nt;
  }
  w.nt_s = decode_nt(N);
  const int pt = cb8 ? 4 * w.nt : 8 * w.nt;
  w.L = host_plan_layout(N, k, E, 1, pt);
  w.Rp = (int)(w.L.off[8] - w.L.off[7]);
  w.P = (int)(w.L.off[11] - w.L.off[10]);
  w.Ps = (N + 8 * w.nt_s - 1) / (8 * w.nt_s);   // shared-expert passes
  w.RB_gu = I / kRowsPerBlock;
  w.RB_dn = H / kRowsPerBlock;
  w.tail_gu = decode_tail_items((long long)w.P * w.RB_gu);
  w.tail_dn = decode_tail_items((long long)w.P * w.RB_dn);
  w.n_zero_routed = 2 + w.P * (w.RB_gu + w.RB_dn);
  w.tail_sgu = decode_tail_items((long long)w.Ps * w.RB_gu);
  w.tail_sdn = decode_tail_items((long long)w.Ps * w.RB_dn);
  w.n_zero_shared = 2 + w.Ps * (w.RB_gu + w.RB_dn);
  const size_t h_bf16 = (size_t)w.Rp * 2 * I * 2, h_h8 = (size_t)w.Rp * (I / kStageK) * kH8StageBytes;
  w.plan = 0;
  w.x8 = align_up((size_t)w.L.off[13] * 4);
  w.x8s = w.x8 + align_up((size_t)N * H * 2);
  w.h = w.x8s + align_up((size_t)N * 4);
  w.y = w.h + align_up(h_bf16 > h_h8 ? h_bf16 : h_h8);
  const size_t hs_bf16 = (size_t)N * 2 * I * 2, hs_h8 = (size_t)N * (I / kStageK) * kH8StageBytes;
  w.hs = w.y + align_up((size_t)w.Rp * H * 4);
  w.ys = w.hs + align_up(hs_bf16 > hs_h8 ? hs_bf16 : hs_h8);
  w.xs8 = w.ys + align_up((size_t)N * H * 4);
  w.xs8s = w.xs8 + align_up((size_t)N * H * 2);
  w.done = w.xs8s + align_up((size_t)N * 4);
  w.part_gu = w.done + align_up((size_t)(w.n_zero_routed + w.n_zero_shared) * 4);
  w.part_dn = w.part_gu + align_up(decode_part_bytes(w.tail_gu, w.nt, 2));
  w.part_sgu = w.part_dn + align_up(decode_part_bytes(w.tail_dn, w.nt_dn, 1));
  w.part_sdn = w.part_sgu + align_up(decode_part_bytes(w.tail_sgu, w.nt_s, 2));
  w.total = w.part_sdn + align_up(decode_part_bytes(w.tail_sdn, w.nt_s, 1));
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool experts_ok(const cbmoe_experts* ex) {
  return ex && ex->E > 0 && ex->E <= 1024 && ex->H > 0 && ex->I > 0 && ex->H % kStageK == 0 &&
         ex->I % kStageK == 0 && ex->gateup_idx && ex->gateup_cb && ex->down_idx && ex->down_cb &&
         aligned16(ex->gateup_idx) && aligned16(ex->down_idx) && aligned16(ex->gateup_cb) && aligned16(ex->down_cb) &&
         (ex->gateup_cb8 == nullptr) == (ex->down_cb8 == nullptr) && aligned16(ex->gateup_cb8) &&
         aligned16(ex->down_cb8);
}

bool has_cb8(const cbmoe_experts* ex) { return ex->gateup_cb8 != nullptr && ex->down_cb8 != nullptr; }

DecodeParams base_params() {
  DecodeParams p{};
  p.E = 1;
  return p;
}

bool shared_ok(const cbmoe_shared* sh) {
  return sh && sh->gateup_q && sh->gate_s && sh->up_s && sh->down_q && sh->down_s &&
         (sh->scale_axis == 0 || sh->scale_axis == 1) && aligned16(sh->gateup_q) && aligned16(sh->down_q) &&
         aligned16(sh->gate_s) && aligned16(sh->up_s) && aligned16(sh->down_s);
}

// Per host thread and device: a second stream and two events, so the shared expert's gate/up (independent of
// the routing) runs concurrently with the routed experts: fork after the caller's prior work, join before the
// shared down + combine. Created on first use; stream-ordered, so the sequence also records into a graph capture.
thread_local SideStream t_side[64];

int side_stream(SideStream** out) {
  int dev = 0;
  CBMOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CBMOE_ERR_UNSUPPORTED;
  SideStream& ss = t_side[dev];
  if (ss.s == nullptr) {
    CBMOE_CUDA_TRY(cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking));
    CBMOE_CUDA_TRY(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming));
    CBMOE_CUDA_TRY(cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming));
  }
  *out = &ss;
  return CBMOE_OK;
}

// Plan + routed gate/up + routed down into the workspace (y_sorted f32, rows in plan order).
int routed_decode(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w, int k,
                  float limit, uint8_t* ws, const DecodeWorkspace& W, cudaStream_t stream) {
  int32_t* plan = reinterpret_cast<int32_t*>(ws + W.plan);
  int* done = reinterpret_cast<int*>(ws + W.done);
  float* ys = reinterpret_cast<float*>(ws + W.y);
  if (W.cb8 && !has_cb8(ex)) return CBMOE_ERR_INVALID;   // workspace sized for tables the call does not have
  if (W.cb8) {
    uint8_t* x8 = ws + W.x8;
    float* x8s = reinterpret_cast<float*>(ws + W.x8s);
    uint8_t* h8 = ws + W.h;
    SplitX sx;
    sx.x = x;
    sx.N = N;
    sx.K = ex->H;
    sx.x8 = x8;
    sx.scale = x8s;
    int rc = launch_route_plan(idx, w, N, k, ex->E, 1, 4 * W.nt, plan, stream, done, W.n_zero_routed, &sx);
    if (rc) return rc;
    DecodeParams p = base_params();
    p.wq = static_cast<const uint8_t*>(ex->gateup_idx);
    p.cb8 = static_cast<const uint8_t*>(ex->gateup_cb8);
    p.rows = ex->I;
    p.K = ex->H;
    p.RB = ex->I / kRowsPerBlock;
    p.KS = ex->H / kStageK;
    p.b8 = x8;
    p.b8_scale = x8s;
    p.tok_row = plan + W.L.off[7];
    p.pass_expert = plan + W.L.off[10];
    p.pass_row0 = plan + W.L.off[11];
    p.pass_cnt = plan + W.L.off[12];
    p.n_pass = plan + W.L.off[5];
    p.N = N;
    p.E = ex->E;
    p.limit = limit;
    p.h8_out = h8;
    p.sched = done;
    p.tail_items = W.tail_gu;
    p.done = done + 2;
    p.part = reinterpret_cast<float*>(ws + W.part_gu);
    rc = decode_cb8_gateup(p, W.nt, stream);
    if (rc) return rc;
    DecodeParams d = p;
    d.wq = static_cast<const uint8_t*>(ex->down_idx);
    d.cb8 = static_cast<const uint8_t*>(ex->down_cb8);
    d.rows = ex->H;
    d.K = ex->I;
    d.RB = ex->H / kRowsPerBlock;
    d.KS = ex->I / kStageK;
    d.b8 = h8;
    d.b8_scale = nullptr;
    d.tok_row = nullptr;
    d.h8_out = nullptr;
    d.y_out = ys;
    d.sched = done + 1;
    d.tail_items = W.tail_dn;
    d.done = done + 2 + W.P * W.RB_gu;
    d.part = reinterpret_cast<float*>(ws + W.part_dn);
    return decode_cb8_down(d, W.nt_dn, stream);
  }

  int rc = launch_route_plan(idx, w, N, k, ex->E, 1, 8 * W.nt, plan, stream, done, W.n_zero_routed);
  if (rc) return rc;
  uint16_t* h = reinterpret_cast<uint16_t*>(ws + W.h);
  DecodeParams p = base_params();
  p.wq = static_cast<const uint8_t*>(ex->gateup_idx);
  p.cb = static_cast<const uint32_t*>(ex->gateup_cb);
  p.rows = ex->I;
  p.K = ex->H;
  p.RB = ex->I / kRowsPerBlock;
  p.KS = ex->H / kStageK;
  p.b = x;
  p.b_hilo = 0;
  p.tok_row = plan + W.L.off[7];
  p.pass_expert = plan + W.L.off[10];
  p.pass_row0 = plan + W.L.off[11];
  p.pass_cnt = plan + W.L.off[12];
  p.n_pass = plan + W.L.off[5];
  p.N = N;
  p.E = ex->E;
  p.limit = limit;
  p.h_out = h;
  p.sched = done;
  p.tail_items = W.tail_gu;
  p.done = done + 2;
  p.part = reinterpret_cast<float*>(ws + W.part_gu);
  rc = decode_cb3_gateup(p, W.nt, stream);
  if (rc) return rc;

  DecodeParams d = p;
  d.wq = static_cast<const uint8_t*>(ex->down_idx);
  d.cb = static_cast<const uint32_t*>(ex->down_cb);
  d.rows = ex->H;
  d.K = ex->I;
  d.RB = ex->H / kRowsPerBlock;
  d.KS = ex->I / kStageK;
  d.b = h;
  d.b_hilo = 1;
  d.tok_row = nullptr;
  d.h_out = nullptr;
  d.y_out = ys;
  d.sched = done + 1;
  d.tail_items = W.tail_dn;
  d.done = done + 2 + W.P * W.RB_gu;
  d.part = reinterpret_cast<float*>(ws + W.part_dn);
  return decode_cb3_down(d, W.nt, stream);
}

int shared_side(const cbmoe_shared* sh, const uint16_t* x, int N, int H, int I, float limit, uint8_t* ws,
                const DecodeWorkspace& W, SideStream* side, cudaStream_t stream, int grid_cap) {
  CBMOE_CUDA_TRY(cudaEventRecord(side->fork, stream));
  CBMOE_CUDA_TRY(cudaStreamWaitEvent(side->s, side->fork, 0));
  int* done_sh = reinterpret_cast<int*>(ws + W.done) + W.n_zero_routed;
  CBMOE_CUDA_TRY(cudaMemsetAsync(done_sh, 0, (size_t)W.n_zero_shared * 4, side->s));
  uint16_t* hs = reinterpret_cast<uint16_t*>(ws + W.hs);
  if (N > kW8DecodeMaxTokens && H % kGrpTileM == 0 && I % kGrpTileM == 0) {
    // Enough tokens for the tensor-core kernels (h as plain bf16 [N][I] in the same region).
    cudaStream_t ss = side->s;
    GroupedParams g{};
    g.wq = static_cast<const uint8_t*>(sh->gateup_q);
    g.s0 = sh->gate_s;
    g.s1 = sh->up_s;
    g.scale_axis = sh->scale_axis;
    g.rows = I;
    g.K = H;
    g.N = N;
    g.E = 1;
    g.limit = limit;
    g.out = hs;
    int rc = grouped_w8_gateup(g, x, N, ss);
    if (rc) return rc;
    GroupedParams gd{};
    gd.wq = static_cast<const uint8_t*>(sh->down_q);
    gd.s0 = sh->down_s;
    gd.scale_axis = sh->scale_axis;
    gd.rows = H;
    gd.K = I;
    gd.N = N;
    gd.E = 1;
    gd.out_f32 = reinterpret_cast<float*>(ws + W.ys);
    rc = grouped_w8_store_f32(gd, hs, N, ss);
    if (rc) return rc;
    CBMOE_CUDA_TRY(cudaEventRecord(side->join, side->s));
    return CBMOE_OK;
  }

  if (W.cb8 && sh->scale_axis == 1 && N <= 8) {
    // int8 MMA on the stored leaves (no dequant arithmetic, so the side stream takes fewer SM cycles from the routed
    // kernels; config 1: CB8 gate+up 102 -> 92 us inside the layer): x split into its own X8 rows here, gate/up ->
    // SwiGLU -> H8 rows, down -> ys. Whole items only (cutting the 24 gate/up items into pieces over the 48 CTAs
    // measured slower: 132 us against 93, on the critical path). Up to one 8-token pass: its token tiles hold 4
    // tokens, so at 64 tokens it would stream the weights 8 times (measured slower there than the bf16 kernels'
    // 32-token passes).
    uint8_t* xs8 = ws + W.xs8;
    float* xs8s = reinterpret_cast<float*>(ws + W.xs8s);
    uint8_t* hs8 = ws + W.hs;
    int rc = launch_split_x(x, N, H, xs8, xs8s, side->s);
    if (rc) return rc;
    const int nt = N <= 4 ? 1 : 2;
    DecodeParams p = base_params();
    p.wq = static_cast<const uint8_t*>(sh->gateup_q);
    p.s0 = sh->gate_s;
    p.s1 = sh->up_s;
    p.scale_axis = 1;
    p.rows = I;
    p.K = H;
    p.RB = I / kRowsPerBlock;
    p.KS = H / kStageK;
    p.b8 = xs8;
    p.b8_scale = xs8s;
    p.N = N;
    p.limit = limit;
    p.h8_out = hs8;
    p.grid_cap = grid_cap;
    p.sched = done_sh;
    rc = decode_w8i_gateup(p, nt, side->s);
    if (rc) return rc;
    DecodeParams d = base_params();
    d.wq = static_cast<const uint8_t*>(sh->down_q);
    d.s0 = sh->down_s;
    d.scale_axis = 1;
    d.rows = H;
    d.K = I;
    d.RB = H / kRowsPerBlock;
    d.KS = I / kStageK;
    d.b8 = hs8;
    d.N = N;
    d.y_out = reinterpret_cast<float*>(ws + W.ys);
    d.grid_cap = grid_cap;
    d.sched = done_sh + 1;
    rc = decode_w8i_down(d, 2 * nt, side->s);
    if (rc) return rc;
    CBMOE_CUDA_TRY(cudaEventRecord(side->join, side->s));
    return CBMOE_OK;
  }

  DecodeParams p = base_params();
  p.wq = static_cast<const uint8_t*>(sh->gateup_q);
  p.s0 = sh->gate_s;
  p.s1 = sh->up_s;
  p.scale_axis = sh->scale_axis;
  p.rows = I;
  p.K = H;
  p.RB = I / kRowsPerBlock;
  p.KS = H / kStageK;
  p.b = x;
  p.N = N;
  p.limit = limit;
  p.h_out = hs;
  p.grid_cap = grid_cap;
  p.sched = done_sh;
  p.tail_items = W.tail_sgu;
  p.done = done_sh + 2;
  p.part = reinterpret_cast<float*>(ws + W.part_sgu);
  int rc = decode_w8_gateup(p, W.nt_s, side->s);
  if (rc) return rc;

  DecodeParams d = base_params();
  d.wq = static_cast<const uint8_t*>(sh->down_q);
  d.s0 = sh->down_s;
  d.scale_axis = sh->scale_axis;
  d.rows = H;
  d.K = I;
  d.RB = H / kRowsPerBlock;
  d.KS = I / kStageK;
  d.b = hs;
  d.b_hilo = 1;
  d.N = N;
  d.y_out = reinterpret_cast<float*>(ws + W.ys);
  d.grid_cap = grid_cap;
  d.sched = done_sh + 1;
  d.tail_items = W.tail_sdn;
  d.done = done_sh + 2 + W.Ps * W.RB_gu;
  d.part = reinterpret_cast<float*>(ws + W.part_sdn);
  rc = decode_w8_down_store(d, W.nt_s, side->s);
  if (rc) return rc;
  CBMOE_CUDA_TRY(cudaEventRecord(side->join, side->s));
  return CBMOE_OK;
}

// Slots (N*k) above which CBMOE_PATH_AUTO takes the grouped tensor-core path.
#ifndef CBMOE_GROUPED_MIN_SLOTS
#define CBMOE_GROUPED_MIN_SLOTS 1024
#endif
constexpr int kGroupedMinSlots = CBMOE_GROUPED_MIN_SLOTS;

int pick_path(int N, int k, int path) {
  if (path != CBMOE_PATH_AUTO) return path;
  return (long long)N * k > kGroupedMinSlots ? CBMOE_PATH_GROUPED : CBMOE_PATH_DECODE;
}

// Workspace of the grouped path: plan | xs (Rp x H bf16, tokens gathered in expert order) | h (Rp x I bf16) |
// y_sorted (Rp x H bf16) | shared h (N x I bf16) | shared down (N x H bf16).

GroupedWorkspace grouped_workspace(int E, int H, int I, int N, int k) {
  GroupedWorkspace w;
  w.tn = grp_pass_tokens((long long)N * k, E);
  w.L = host_plan_layout(N, k, E, 1, w.tn);
  w.Rp = (int)(w.L.off[8] - w.L.off[7]);
  w.plan = 0;
  w.xs = align_up((size_t)w.L.off[13] * 4);
  w.h = w.xs + align_up((size_t)w.Rp * H * 2);
  w.y = w.h + align_up((size_t)w.Rp * I * 2);
  w.hs = w.y + align_up((size_t)w.Rp * H * 2);
  w.sy = w.hs + align_up((size_t)N * I * 2);
  w.total = w.sy + align_up((size_t)N * H * 2);
  return w;
}

// Plan + gather + grouped gate/up + grouped down into the workspace (y_sorted bf16, rows in expert order).
int routed_grouped(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w, int k,
                   float limit, uint8_t* ws, const GroupedWorkspace& W, cudaStream_t stream) {
  int32_t* plan = reinterpret_cast<int32_t*>(ws + W.plan);
  int rc = launch_route_plan(idx, w, N, k, ex->E, 1, W.tn, plan, stream);
  if (rc) return rc;
  uint16_t* xs = reinterpret_cast<uint16_t*>(ws + W.xs);
  uint16_t* h = reinterpret_cast<uint16_t*>(ws + W.h);
  uint16_t* ys = reinterpret_cast<uint16_t*>(ws + W.y);
  rc = launch_gather_rows(x, ex->H, plan + W.L.off[7], W.Rp, xs, stream);
  if (rc) return rc;
  GroupedParams p{};
  p.wq = static_cast<const uint8_t*>(ex->gateup_idx);
  p.cb = static_cast<const uint32_t*>(ex->gateup_cb);
  p.rows = ex->I;
  p.K = ex->H;
  p.pass_expert = plan + W.L.off[10];
  p.pass_row0 = plan + W.L.off[11];
  p.pass_cnt = plan + W.L.off[12];
  p.n_pass = plan + W.L.off[5];
  p.E = ex->E;
  p.limit = limit;
  p.out = h;
  rc = grouped_cb3_gateup(p, xs, W.Rp, W.tn, stream);
  if (rc) return rc;
  GroupedParams d = p;
  d.wq = static_cast<const uint8_t*>(ex->down_idx);
  d.cb = static_cast<const uint32_t*>(ex->down_cb);
  d.rows = ex->H;
  d.K = ex->I;
  d.out = ys;
  return grouped_cb3_down(d, h, W.Rp, W.tn, stream);
}

}  // namespace lyr
using namespace lyr;

void set_last_cuda_error(cudaError_t e) { t_last_cuda_error = (int)e; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("CBMOE_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace cbmoe

using namespace cbmoe;

extern "C" int cbmoe_version(void) { return 1; }

extern "C" const char* cbmoe_status_string(int status) {
  switch (status) {
    case CBMOE_OK: return "ok";
    case CBMOE_ERR_INVALID: return "invalid argument";
    case CBMOE_ERR_CUDA: return "CUDA error";
    case CBMOE_ERR_WORKSPACE: return "workspace too small";
    case CBMOE_ERR_UNSUPPORTED: return "unsupported";
    case CBMOE_ERR_NCCL: return "NCCL error";
    case CBMOE_ERR_DEVICE: return "device-side error";
    default: return "unknown status";
  }
}

extern "C" int cbmoe_last_cuda_error(void) { return t_last_cuda_error; }

extern "C" int cbmoe_num_sms(void) { return num_sms(); }

extern "C" int cbmoe_device_errors(int clear, int* out_host) {
  if (!out_host) return CBMOE_ERR_INVALID;
  CBMOE_CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  CBMOE_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_errors, sizeof(int)));
  *out_host = v;
  if (clear) {
    const int zero = 0;
    CBMOE_CUDA_TRY(cudaMemcpyToSymbol(g_device_errors, &zero, sizeof(int)));
  }
  return CBMOE_OK;
}

extern "C" size_t cbmoe_workspace_bytes(const cbmoe_experts* ex, int N, int k, int path) {
  if (!ex || N < 0 || k <= 0 || ex->E <= 0) return 0;
  if (path != CBMOE_PATH_AUTO && path != CBMOE_PATH_DECODE && path != CBMOE_PATH_GROUPED) return 0;
  if (pick_path(N, k, path) == CBMOE_PATH_GROUPED) return grouped_workspace(ex->E, ex->H, ex->I, N, k).total;
  return decode_workspace(ex->E, ex->H, ex->I, N, k, -1, has_cb8(ex)).total;
}

static int check_common(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w,
                        int k, int path) {
  if (!experts_ok(ex) || N < 0 || k <= 0 || k > 64) return CBMOE_ERR_INVALID;
  if (N > 0 && (!x || !idx || !w || !aligned16(x))) return CBMOE_ERR_INVALID;
  if (path != CBMOE_PATH_AUTO && path != CBMOE_PATH_DECODE && path != CBMOE_PATH_GROUPED) return CBMOE_ERR_INVALID;
  if (pick_path(N, k, path) == CBMOE_PATH_GROUPED && (ex->I % kGrpTileM || ex->H % kGrpTileM || N > (1 << 24)))
    return CBMOE_ERR_UNSUPPORTED;
  return CBMOE_OK;
}

extern "C" int cbmoe_experts_apply(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx,
                                   const float* w, int k, float limit, int path, float* y, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
  int rc = check_common(ex, x, N, idx, w, k, path);
  if (rc) return rc;
  if (N > 0 && (!y || !aligned16(y))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (pick_path(N, k, path) == CBMOE_PATH_GROUPED) {
    const GroupedWorkspace G = grouped_workspace(ex->E, ex->H, ex->I, N, k);
    if (!workspace || workspace_bytes < G.total) return CBMOE_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    rc = routed_grouped(ex, x, N, idx, w, k, limit, ws, G, stream);
    if (rc) return rc;
    const int32_t* plan = reinterpret_cast<const int32_t*>(ws + G.plan);
    return launch_combine_bf16(reinterpret_cast<const uint16_t*>(ws + G.y), plan + G.L.off[9], w, N, k, ex->H,
                               nullptr, y, nullptr, stream);
  }
  const DecodeWorkspace W = decode_workspace(ex->E, ex->H, ex->I, N, k, -1, has_cb8(ex));
  if (!workspace || workspace_bytes < W.total) return CBMOE_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  rc = routed_decode(ex, x, N, idx, w, k, limit, ws, W, stream);
  if (rc) return rc;
  const int32_t* plan = reinterpret_cast<const int32_t*>(ws + W.plan);
  return launch_combine(reinterpret_cast<const float*>(ws + W.y), plan + W.L.off[9], w, N, k, ex->H, nullptr, y,
                        nullptr, stream);
}

extern "C" int cbmoe_moe_layer(const cbmoe_experts* ex, const cbmoe_shared* sh, const uint16_t* x, int N,
                               const int32_t* idx, const float* w, int k, float limit, int path, uint16_t* out,
                               void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int rc = check_common(ex, x, N, idx, w, k, path);
  if (rc) return rc;
  if (!shared_ok(sh) || (N > 0 && (!out || !aligned16(out)))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (pick_path(N, k, path) == CBMOE_PATH_GROUPED) {
    const GroupedWorkspace G = grouped_workspace(ex->E, ex->H, ex->I, N, k);
    if (!workspace || workspace_bytes < G.total) return CBMOE_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    rc = routed_grouped(ex, x, N, idx, w, k, limit, ws, G, stream);
    if (rc) return rc;
    uint16_t* hs = reinterpret_cast<uint16_t*>(ws + G.hs);
    uint16_t* sy = reinterpret_cast<uint16_t*>(ws + G.sy);
    GroupedParams p{};
    p.wq = static_cast<const uint8_t*>(sh->gateup_q);
    p.s0 = sh->gate_s;
    p.s1 = sh->up_s;
    p.scale_axis = sh->scale_axis;
    p.rows = ex->I;
    p.K = ex->H;
    p.N = N;
    p.E = 1;
    p.limit = limit;
    p.out = hs;
    rc = grouped_w8_gateup(p, x, N, stream);
    if (rc) return rc;
    GroupedParams d = p;
    d.wq = static_cast<const uint8_t*>(sh->down_q);
    d.s0 = sh->down_s;
    d.s1 = nullptr;
    d.rows = ex->H;
    d.K = ex->I;
    d.out = sy;
    rc = grouped_w8_store(d, hs, N, stream);
    if (rc) return rc;
    const int32_t* plan = reinterpret_cast<const int32_t*>(ws + G.plan);
    return launch_combine_bf16(reinterpret_cast<const uint16_t*>(ws + G.y), plan + G.L.off[9], w, N, k, ex->H, sy,
                               nullptr, out, stream);
  }
  const DecodeWorkspace W = decode_workspace(ex->E, ex->H, ex->I, N, k, -1, has_cb8(ex));
  if (!workspace || workspace_bytes < W.total) return CBMOE_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  SideStream* side = nullptr;
  rc = side_stream(&side);
  if (rc) return rc;
  rc = shared_side(sh, x, N, ex->H, ex->I, limit, ws, W, side, stream);
  if (rc) return rc;
  rc = routed_decode(ex, x, N, idx, w, k, limit, ws, W, stream);
  CBMOE_CUDA_TRY(cudaStreamWaitEvent(stream, side->join, 0));   // join even when a routed launch failed
  if (rc) return rc;
  const int32_t* plan = reinterpret_cast<const int32_t*>(ws + W.plan);
  return launch_combine(reinterpret_cast<const float*>(ws + W.y), plan + W.L.off[9], w, N, k, ex->H,
                        reinterpret_cast<const float*>(ws + W.ys), nullptr, out, stream);
}

extern "C" size_t cbmoe_matvec_workspace_bytes(int N) { return N >= 0 ? 0 : 0; }

extern "C" int cbmoe_cb3_matvec(const void* idx_k, const void* cb_k, int rows, int K, const uint16_t* x, int N,
                                float* y, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!idx_k || !cb_k || rows <= 0 || K <= 0 || rows % kRowsPerBlock || K % kStageK || N < 0) return CBMOE_ERR_INVALID;
  if (N > 0 && (!x || !y || !aligned16(x) || !aligned16(idx_k) || !aligned16(cb_k))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  DecodeParams p = base_params();
  p.wq = static_cast<const uint8_t*>(idx_k);
  p.cb = static_cast<const uint32_t*>(cb_k);
  p.rows = rows;
  p.K = K;
  p.RB = rows / kRowsPerBlock;
  p.KS = K / kStageK;
  p.b = x;
  p.N = N;
  p.y_out = y;
  return decode_cb3_single(p, decode_nt(N), stream);
}

extern "C" size_t cbmoe_cb8_matvec_workspace_bytes(int N, int K) {
  if (N < 0 || K <= 0 || K % kStageK) return 0;
  return align_up((size_t)N * K * 2) + align_up((size_t)N * 4);
}

extern "C" int cbmoe_cb8_matvec(const void* idx_k, const void* cb8, int rows, int K, const uint16_t* x, int N,
                                float* y, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!idx_k || !cb8 || rows <= 0 || K <= 0 || rows % kRowsPerBlock || K % kStageK || K > 65536 || N < 0)
    return CBMOE_ERR_INVALID;
  if (N > 0 && (!x || !y || !aligned16(x) || !aligned16(idx_k) || !aligned16(cb8))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (!workspace || workspace_bytes < cbmoe_cb8_matvec_workspace_bytes(N, K) || !aligned16(workspace))
    return CBMOE_ERR_WORKSPACE;
  uint8_t* x8 = static_cast<uint8_t*>(workspace);
  float* xs = reinterpret_cast<float*>(x8 + align_up((size_t)N * K * 2));
  int rc = launch_split_x(x, N, K, x8, xs, stream);
  if (rc) return rc;
  DecodeParams p = base_params();
  p.wq = static_cast<const uint8_t*>(idx_k);
  p.cb8 = static_cast<const uint8_t*>(cb8);
  p.rows = rows;
  p.K = K;
  p.RB = rows / kRowsPerBlock;
  p.KS = K / kStageK;
  p.b8 = x8;
  p.b8_scale = xs;
  p.N = N;
  p.y_out = y;
  return decode_cb8_single(p, N <= 4 ? 1 : 2, stream);
}

extern "C" int cbmoe_w8_logits(const void* qk, const float* s, int rows, int K, const uint16_t* x, int N,
                               uint16_t* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!qk || !s || rows <= 0 || K <= 0 || rows % kRowsPerBlock || K % kStageK || K > 65536 || N < 0 ||
      !aligned16(s))
    return CBMOE_ERR_INVALID;
  if (N > 0 && (!x || !out || !aligned16(x) || !aligned16(qk))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (!workspace || workspace_bytes < cbmoe_cb8_matvec_workspace_bytes(N, K) || !aligned16(workspace))
    return CBMOE_ERR_WORKSPACE;
  uint8_t* x8 = static_cast<uint8_t*>(workspace);
  float* xs = reinterpret_cast<float*>(x8 + align_up((size_t)N * K * 2));
  int rc = launch_split_x(x, N, K, x8, xs, stream);
  if (rc) return rc;
  DecodeParams p = base_params();
  p.wq = static_cast<const uint8_t*>(qk);
  p.s0 = s;
  p.scale_axis = 1;
  p.rows = rows;
  p.K = K;
  p.RB = rows / kRowsPerBlock;
  p.KS = K / kStageK;
  p.b8 = x8;
  p.b8_scale = xs;
  p.N = N;
  p.y_bf16 = out;
  return decode_w8i_logits(p, N <= 4 ? 1 : 2, stream);
}

extern "C" int cbmoe_w8_linear(const void* qk, const float* s, int scale_axis, int rows, int K, const uint16_t* x,
                               int N, float* y, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!qk || !s || rows <= 0 || K <= 0 || rows % kRowsPerBlock || K % kStageK || N < 0 ||
      (scale_axis != 0 && scale_axis != 1) || !aligned16(s))
    return CBMOE_ERR_INVALID;
  if (N > 0 && (!x || !y || !aligned16(x) || !aligned16(qk))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (N > kW8DecodeMaxTokens && rows % kGrpTileM == 0) {
    GroupedParams g{};
    g.wq = static_cast<const uint8_t*>(qk);
    g.s0 = s;
    g.scale_axis = scale_axis;
    g.rows = rows;
    g.K = K;
    g.N = N;
    g.E = 1;
    g.out_f32 = y;
    return grouped_w8_store_f32(g, x, N, stream);
  }
  DecodeParams p = base_params();
  p.wq = static_cast<const uint8_t*>(qk);
  p.s0 = s;
  p.scale_axis = scale_axis;
  p.rows = rows;
  p.K = K;
  p.RB = rows / kRowsPerBlock;
  p.KS = K / kStageK;
  p.b = x;
  p.N = N;
  p.y_out = y;
  return decode_w8_single(p, decode_nt(N), stream);
}

// ------------------------------------------------------------------------------------------------------
// cbmoe_experts_apply_noalloc: cbmoe_experts_apply for callers that cannot allocate device memory.
//
// The other entry points take a caller-provided workspace. Some callers cannot provide one: an inference
// engine that carves all device memory up front with its own allocator and hands a plugin only the buffers it
// owns, a plugin host that forbids allocation inside its execute callback, or host code that must not block on
// cudaMalloc (which can synchronize the device). This entry point keeps its scratch in a file-scope device array
// instead. The array is part of the library image: every GPU that loads the library holds
// kNoAllocScratchBytes (48 MiB) of device memory for it until the process exits, whether or not this entry point
// is ever called. Requests that need more scratch than that are rejected with CBMOE_ERR_WORKSPACE.
//
// In host code the name `g_noalloc_scratch` is only a host-side stand-in for the device array, not its device
// address, so it is never handed to a kernel. The first call on each device, with that device current, looks
// the address up with cudaGetSymbolAddress (return code checked) and caches it per device; make that first call
// before any stream capture begins. Every call on a device shares the one array, which keeps whatever the last
// call left in it: calls that overlap on the GPU (different streams with no ordering between them) race on it.
// Nothing in the array has to start at zero: the routing-plan kernel writes every plan field before it is read,
// and the expert kernels write every h / y row before a later kernel reads it.
namespace {
constexpr size_t kNoAllocScratchBytes = CBMOE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {nullptr};
}  // namespace

extern "C" int cbmoe_experts_apply_noalloc(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx,
                                           const float* w, int k, float limit, float* y, cudaStream_t stream) {
  int rc = check_common(ex, x, N, idx, w, k, CBMOE_PATH_DECODE);
  if (rc) return rc;
  if (N > 0 && (!y || !aligned16(y))) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  const DecodeWorkspace W = decode_workspace(ex->E, ex->H, ex->I, N, k, -1, has_cb8(ex));
  if (W.total > kNoAllocScratchBytes) return CBMOE_ERR_WORKSPACE;   // request needs more than the fixed array
  int dev = 0;
  CBMOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CBMOE_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
      void* p = nullptr;
      CBMOE_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      g_noalloc_addr[dev] = p;
    }
    scratch = g_noalloc_addr[dev];
  }
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  rc = routed_decode(ex, x, N, idx, w, k, limit, ws, W, stream);
  if (rc) return rc;
  const int32_t* plan = reinterpret_cast<const int32_t*>(ws + W.plan);
  return launch_combine(reinterpret_cast<const float*>(ws + W.y), plan + W.L.off[9], w, N, k, ex->H, nullptr, y,
                        nullptr, stream);
}
