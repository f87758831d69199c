// Device routing plan: pallas_moe.ragged_plan (pallas_moe.py:564-592) plus the per-expert pass lists the decode
// kernels walk. One CTA: a stable counting sort of the T*k (token, slot) pairs by expert.
//   pass A  each warp counts its contiguous slot range per expert (warp match_any, no atomics)
//   scan    per-expert totals -> padded row starts, block starts, pass starts, active list (warp scans)
//   pass C  each warp re-walks its range; a slot's sorted row = its expert's row start + the slots of that expert
//           in earlier warps + earlier slots in this warp: the same order as a stable argsort.
#include "decode.cuh"
#include "profile.cuh"

namespace cbmoe {

constexpr int kPlanWarps = 16;
constexpr int kPlanThreads = kPlanWarps * 32;
constexpr int kPlanMaxExperts = 1024;
constexpr int kPlanMaxChunks = 160;      // CTAs of the multi-CTA plan (large T*k)
constexpr int kPlanChunkSlots = 512;     // slots per CTA of the multi-CTA plan
constexpr int kPlanBigSlots = 4096;      // above this many slots the multi-CTA plan runs

struct PlanLayout {
  int64_t off[14];
};

__host__ __device__ inline PlanLayout plan_layout(int T, int k, int E, int tm, int pass_tokens) {
  const int64_t S = (int64_t)T * k;
  const int64_t G = (S + tm - 1) / tm + E;
  const int64_t Rp = G * tm;
  const int64_t P = (S + pass_tokens - 1) / pass_tokens + E;
  auto up4 = [](int64_t v) { return (v + 3) & ~int64_t(3); };
  PlanLayout L;
  L.off[0] = 0;
  L.off[1] = up4(E);
  L.off[2] = L.off[1] + up4(E);
  L.off[3] = L.off[2] + up4(E);
  L.off[4] = L.off[3] + 1;
  L.off[5] = L.off[4] + 1;
  L.off[6] = up4(L.off[5] + 1);
  L.off[7] = L.off[6] + up4(G);
  L.off[8] = L.off[7] + up4(Rp);
  L.off[9] = L.off[8] + up4(Rp);
  L.off[10] = L.off[9] + up4(S);
  L.off[11] = L.off[10] + up4(P);
  L.off[12] = L.off[11] + up4(P);
  L.off[13] = L.off[12] + up4(P) + (int64_t)kPlanMaxChunks * E;   // + scratch: per-chunk expert counts
  return L;
}

namespace {

// Exclusive warp scan of v; returns the prefix and writes the warp total to *total.
__device__ __forceinline__ int warp_exclusive_scan(int v, int* total) {
  const int lane = threadIdx.x & 31;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  *total = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

// CTA 0 builds the plan; CTAs 1.. (when split.x8 is set) write the X8 rows of split.x, which the expert kernels
// after the plan read (independent work sharing the launch).
__global__ void __launch_bounds__(kPlanThreads) route_plan_kernel(const int32_t* __restrict__ idx,
                                                                  const float* __restrict__ wts, int T, int k, int E,
                                                                  int tm, int pass_tokens, int32_t* __restrict__ plan,
                                                                  PlanLayout L, int* __restrict__ zero, int n_zero,
                                                                  SplitX split) {
  griddep_wait();     // the previous layer's kernels may still read the plan buffer until here
  griddep_launch();
  if (blockIdx.x > 0) {
    __shared__ float s_red[32];
    const int KS = split.K / kStageK;
    for (int r = blockIdx.x - 1; r < split.N; r += gridDim.x - 1)
      split_x_row(split.x + (size_t)r * split.K, split.K, split.x8 + (size_t)r * KS * kX8StageBytes, split.scale + r,
                  s_red);
    return;
  }
  extern __shared__ int sm[];
  int* cnt = sm;                               // [kPlanWarps][E]
  int* counts = cnt + kPlanWarps * E;          // [E]
  int* ends = counts + E;                      // [E] block end (exclusive) per expert
  __shared__ int s_tot[4];
  __shared__ int s_chunk[4][32];

  const int S = T * k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_warp = ((S + kPlanWarps - 1) / kPlanWarps + 31) & ~31;
  const int beg = warp * per_warp;
  const int end = min(S, beg + per_warp);

  for (int i = threadIdx.x; i < kPlanWarps * E; i += kPlanThreads) cnt[i] = 0;
  for (int i = threadIdx.x; i < n_zero; i += kPlanThreads) zero[i] = 0;   // scheduling words of the next kernels
  __syncthreads();

  // pass A: per-warp per-expert counts
  for (int base = beg; base < end; base += 32) {
    const int s = base + lane;
    int e = (s < end) ? idx[s] : -1;
    if (s < end && e >= E) {          // negative ids are empty slots; ids past E are errors
      atomicOr(&g_device_errors, CBMOE_DEVERR_INDEX);
      e = -1;
    }
    if (e < 0) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
  }
  __syncthreads();

  int32_t* counts_g = plan + L.off[0];
  int32_t* row_start = plan + L.off[1];
  int32_t* act = plan + L.off[2];
  int32_t* pass_expert = plan + L.off[10];
  int32_t* pass_row0 = plan + L.off[11];
  int32_t* pass_cnt = plan + L.off[12];
  const int P = (int)(L.off[11] - L.off[10]);

  // per-expert totals
  for (int e = threadIdx.x; e < E; e += kPlanThreads) {
    int c = 0;
    for (int w = 0; w < kPlanWarps; ++w) c += cnt[w * E + e];
    counts[e] = c;
  }
  __syncthreads();

  // scans over experts, 32 experts per chunk, chunks spread over the warps: (1) per-chunk totals
  const int n_chunks = (E + 31) / 32;
  for (int q = warp; q < n_chunks; q += kPlanWarps) {
    const int e = q * 32 + lane;
    const int c = (e < E) ? counts[e] : 0;
    const int nb = (c + tm - 1) / tm;
    const int np = (c + pass_tokens - 1) / pass_tokens;
    int t_rows, t_blocks, t_pass, t_act;
    warp_exclusive_scan(nb * tm, &t_rows);
    warp_exclusive_scan(nb, &t_blocks);
    warp_exclusive_scan(np, &t_pass);
    warp_exclusive_scan(c > 0 ? 1 : 0, &t_act);
    if (lane == 0) {
      s_chunk[0][q] = t_rows;
      s_chunk[1][q] = t_blocks;
      s_chunk[2][q] = t_pass;
      s_chunk[3][q] = t_act;
    }
  }
  __syncthreads();
  // (2) every warp scans the chunk totals itself, then finishes its own chunks
  int c_rows, c_blocks, c_pass, c_act, tot_rows, tot_blocks, tot_pass, tot_act;
  {
    const bool in = lane < n_chunks;
    c_rows = warp_exclusive_scan(in ? s_chunk[0][lane] : 0, &tot_rows);
    c_blocks = warp_exclusive_scan(in ? s_chunk[1][lane] : 0, &tot_blocks);
    c_pass = warp_exclusive_scan(in ? s_chunk[2][lane] : 0, &tot_pass);
    c_act = warp_exclusive_scan(in ? s_chunk[3][lane] : 0, &tot_act);
  }
  for (int q = warp; q < n_chunks; q += kPlanWarps) {
    const int e = q * 32 + lane;
    const int c = (e < E) ? counts[e] : 0;
    const int nb = (c + tm - 1) / tm;
    const int np = (c + pass_tokens - 1) / pass_tokens;
    int dummy;
    const int x_rows = warp_exclusive_scan(nb * tm, &dummy) + __shfl_sync(0xffffffffu, c_rows, q);
    const int x_blocks = warp_exclusive_scan(nb, &dummy) + __shfl_sync(0xffffffffu, c_blocks, q);
    const int x_pass = warp_exclusive_scan(np, &dummy) + __shfl_sync(0xffffffffu, c_pass, q);
    const int x_act = warp_exclusive_scan(c > 0 ? 1 : 0, &dummy) + __shfl_sync(0xffffffffu, c_act, q);
    if (e < E) {
      counts_g[e] = c;
      row_start[e] = x_rows;
      ends[e] = x_blocks + nb;
      if (c > 0) act[x_act] = e;
      for (int p = 0; p < np; ++p) {
        pass_expert[x_pass + p] = e;
        pass_row0[x_pass + p] = x_rows + p * pass_tokens;
        pass_cnt[x_pass + p] = min(pass_tokens, c - p * pass_tokens);
      }
      // this expert's per-warp counts -> per-warp starting rows
      int run = x_rows;
      for (int w = 0; w < kPlanWarps; ++w) {
        const int v = cnt[w * E + e];
        cnt[w * E + e] = run;
        run += v;
      }
    }
  }
  if (threadIdx.x == 0) {
    s_tot[0] = tot_act;
    s_tot[1] = tot_blocks;
    s_tot[2] = tot_pass;
    plan[L.off[3]] = tot_act;
    plan[L.off[4]] = tot_blocks;
    plan[L.off[5]] = tot_pass;
  }
  // padding rows and unused list entries
  const int Rp = (int)(L.off[8] - L.off[7]);
  int32_t* tok_row = plan + L.off[7];
  float* w_row = reinterpret_cast<float*>(plan + L.off[8]);
  for (int r = threadIdx.x; r < Rp; r += kPlanThreads) {
    tok_row[r] = -1;
    w_row[r] = 0.f;
  }
  __syncthreads();
  for (int i = s_tot[0] + threadIdx.x; i < E; i += kPlanThreads) act[i] = -1;
  for (int i = s_tot[2] + threadIdx.x; i < P; i += kPlanThreads) {
    pass_expert[i] = -1;
    pass_row0[i] = 0;
    pass_cnt[i] = 0;
  }

  // pass C: stable placement
  int32_t* row_slot = plan + L.off[9];
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int base = beg; base < end; base += 32) {
    const int s = base + lane;
    int e = (s < end) ? idx[s] : -1;
    if (e >= E || e < 0) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int pos = -1;
    if (e >= 0) {
      pos = cnt[warp * E + e] + __popc(peers & lt_mask);
      tok_row[pos] = s / k;
      w_row[pos] = wts[s];
    }
    if (s < end) row_slot[s] = pos;
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }

  // block -> expert (first expert whose block range ends after the block; blocks past n_blocks repeat the last)
  const int G = (int)(L.off[7] - L.off[6]);
  int32_t* blk_expert = plan + L.off[6];
  const int n_blocks = s_tot[1];
  auto find = [&](int g) {
    int lo = 0, hi = E;  // first e with ends[e] > g
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (ends[mid] > g) hi = mid; else lo = mid + 1;
    }
    return min(lo, E - 1);
  };
  const int last = find(max(n_blocks - 1, 0));
  for (int g = threadIdx.x; g < G; g += kPlanThreads) blk_expert[g] = (g < n_blocks) ? find(g) : last;
}


// ------------------------------------------------------------------------------------ multi-CTA variant
// The same stable expert sort for large T*k, in three launches: per-chunk counts (one CTA per 512-slot chunk),
// one CTA of scans (expert starts, per-chunk bases, lists, blocks), and a stable placement per chunk.
constexpr int kPlanCtaWarps = 8;

__device__ __forceinline__ void chunk_warp_counts(const int32_t* idx, int beg, int end, int E, int* cnt, int warp,
                                                  int lane, bool flag_errors) {
  for (int base = beg; base < end; base += 32) {
    const int s = base + lane;
    int e = (s < end) ? idx[s] : -1;
    if (s < end && e >= E) {          // negative ids are empty slots; ids past E are errors
      if (flag_errors) atomicOr(&g_device_errors, CBMOE_DEVERR_INDEX);
      e = -1;
    }
    if (e < 0) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
  }
}

__global__ void __launch_bounds__(kPlanCtaWarps * 32) plan_count_kernel(const int32_t* __restrict__ idx, int S, int E,
                                                                        int32_t* __restrict__ chunk_cnt) {
  extern __shared__ int cnt[];  // [kPlanCtaWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * kPlanChunkSlots;
  const int per = kPlanChunkSlots / kPlanCtaWarps;
  for (int i = threadIdx.x; i < kPlanCtaWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  chunk_warp_counts(idx, c0 + warp * per, min(S, c0 + (warp + 1) * per), E, cnt, warp, lane, true);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0;
    for (int w = 0; w < kPlanCtaWarps; ++w) t += cnt[w * E + e];
    chunk_cnt[blockIdx.x * E + e] = t;
  }
}

__global__ void __launch_bounds__(kPlanThreads) plan_scan_kernel(int T, int k, int E, int tm, int pass_tokens,
                                                                 int n_chunks, int32_t* __restrict__ plan,
                                                                 PlanLayout L, int32_t* __restrict__ chunk_cnt,
                                                                 int* __restrict__ zero, int n_zero) {
  extern __shared__ int sm[];
  int* counts = sm;        // [E]
  int* ends = sm + E;      // [E]
  int* bases = sm + 2 * E; // [E] first sorted row of each expert
  __shared__ int s_tot[4];
  __shared__ int s_chunk[4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < n_zero; i += kPlanThreads) zero[i] = 0;
  // per-expert totals; chunk counts -> exclusive prefix over chunks (relative to the expert's first row). One warp
  // per expert, one chunk per lane: the loads are issued together instead of as a chain of dependent round trips.
  constexpr int kMaxGroups = (kPlanMaxChunks + 31) / 32;
  for (int e = warp; e < E; e += kPlanWarps) {
    int v[kMaxGroups];
#pragma unroll
    for (int gi = 0; gi < kMaxGroups; ++gi) {
      const int c = gi * 32 + lane;
      v[gi] = c < n_chunks ? chunk_cnt[c * E + e] : 0;
    }
    int carry = 0;
#pragma unroll
    for (int gi = 0; gi < kMaxGroups; ++gi) {
      const int c = gi * 32 + lane;
      int tot;
      const int ex = warp_exclusive_scan(v[gi], &tot);
      if (c < n_chunks) chunk_cnt[c * E + e] = carry + ex;
      carry += tot;
    }
    if (lane == 0) counts[e] = carry;
  }
  __syncthreads();
  int32_t* counts_g = plan + L.off[0];
  int32_t* row_start = plan + L.off[1];
  int32_t* act = plan + L.off[2];
  int32_t* pass_expert = plan + L.off[10];
  int32_t* pass_row0 = plan + L.off[11];
  int32_t* pass_cnt = plan + L.off[12];
  const int P = (int)(L.off[11] - L.off[10]);
  const int n_ech = (E + 31) / 32;
  for (int q = warp; q < n_ech; q += kPlanWarps) {
    const int e = q * 32 + lane;
    const int c = (e < E) ? counts[e] : 0;
    const int nb = (c + tm - 1) / tm;
    const int np = (c + pass_tokens - 1) / pass_tokens;
    int t_rows, t_blocks, t_pass, t_act;
    warp_exclusive_scan(nb * tm, &t_rows);
    warp_exclusive_scan(nb, &t_blocks);
    warp_exclusive_scan(np, &t_pass);
    warp_exclusive_scan(c > 0 ? 1 : 0, &t_act);
    if (lane == 0) {
      s_chunk[0][q] = t_rows;
      s_chunk[1][q] = t_blocks;
      s_chunk[2][q] = t_pass;
      s_chunk[3][q] = t_act;
    }
  }
  __syncthreads();
  int c_rows, c_blocks, c_pass, c_act, tot_rows, tot_blocks, tot_pass, tot_act;
  {
    const bool in = lane < n_ech;
    c_rows = warp_exclusive_scan(in ? s_chunk[0][lane] : 0, &tot_rows);
    c_blocks = warp_exclusive_scan(in ? s_chunk[1][lane] : 0, &tot_blocks);
    c_pass = warp_exclusive_scan(in ? s_chunk[2][lane] : 0, &tot_pass);
    c_act = warp_exclusive_scan(in ? s_chunk[3][lane] : 0, &tot_act);
  }
  for (int q = warp; q < n_ech; q += kPlanWarps) {
    const int e = q * 32 + lane;
    const int c = (e < E) ? counts[e] : 0;
    const int nb = (c + tm - 1) / tm;
    const int np = (c + pass_tokens - 1) / pass_tokens;
    int dummy;
    const int x_rows = warp_exclusive_scan(nb * tm, &dummy) + __shfl_sync(0xffffffffu, c_rows, q);
    const int x_blocks = warp_exclusive_scan(nb, &dummy) + __shfl_sync(0xffffffffu, c_blocks, q);
    const int x_pass = warp_exclusive_scan(np, &dummy) + __shfl_sync(0xffffffffu, c_pass, q);
    const int x_act = warp_exclusive_scan(c > 0 ? 1 : 0, &dummy) + __shfl_sync(0xffffffffu, c_act, q);
    if (e < E) {
      counts_g[e] = c;
      row_start[e] = x_rows;
      ends[e] = x_blocks + nb;
      if (c > 0) act[x_act] = e;
      for (int p = 0; p < np; ++p) {
        pass_expert[x_pass + p] = e;
        pass_row0[x_pass + p] = x_rows + p * pass_tokens;
        pass_cnt[x_pass + p] = min(pass_tokens, c - p * pass_tokens);
      }
    }
    if (e < E) bases[e] = x_rows;
  }
  __syncthreads();
  // absolute chunk bases: one warp per expert, one chunk per lane
  for (int e = warp; e < E; e += kPlanWarps) {
    const int base = bases[e];
    for (int c = lane; c < n_chunks; c += 32) chunk_cnt[c * E + e] += base;
  }
  if (threadIdx.x == 0) {
    s_tot[0] = tot_act;
    s_tot[1] = tot_blocks;
    s_tot[2] = tot_pass;
    plan[L.off[3]] = tot_act;
    plan[L.off[4]] = tot_blocks;
    plan[L.off[5]] = tot_pass;
  }
  const int Rp = (int)(L.off[8] - L.off[7]);
  int32_t* tok_row = plan + L.off[7];
  float* w_row = reinterpret_cast<float*>(plan + L.off[8]);
  for (int r = threadIdx.x; r < Rp; r += kPlanThreads) {
    tok_row[r] = -1;
    w_row[r] = 0.f;
  }
  __syncthreads();
  for (int i = s_tot[0] + threadIdx.x; i < E; i += kPlanThreads) act[i] = -1;
  for (int i = s_tot[2] + threadIdx.x; i < P; i += kPlanThreads) {
    pass_expert[i] = -1;
    pass_row0[i] = 0;
    pass_cnt[i] = 0;
  }
  const int G = (int)(L.off[7] - L.off[6]);
  int32_t* blk_expert = plan + L.off[6];
  const int n_blocks = s_tot[1];
  auto find = [&](int g) {
    int lo = 0, hi = E;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (ends[mid] > g) hi = mid; else lo = mid + 1;
    }
    return min(lo, E - 1);
  };
  const int last = find(max(n_blocks - 1, 0));
  for (int g = threadIdx.x; g < G; g += kPlanThreads) blk_expert[g] = (g < n_blocks) ? find(g) : last;
}

__global__ void __launch_bounds__(kPlanCtaWarps * 32) plan_place_kernel(const int32_t* __restrict__ idx,
                                                                        const float* __restrict__ wts, int S, int k,
                                                                        int E, int32_t* __restrict__ plan, PlanLayout L,
                                                                        const int32_t* __restrict__ chunk_base) {
  extern __shared__ int cnt[];  // [kPlanCtaWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * kPlanChunkSlots;
  const int per = kPlanChunkSlots / kPlanCtaWarps;
  const int beg = c0 + warp * per, end = min(S, c0 + (warp + 1) * per);
  for (int i = threadIdx.x; i < kPlanCtaWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  chunk_warp_counts(idx, beg, end, E, cnt, warp, lane, false);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = chunk_base[blockIdx.x * E + e];
    for (int w = 0; w < kPlanCtaWarps; ++w) {
      const int v = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += v;
    }
  }
  __syncthreads();
  int32_t* tok_row = plan + L.off[7];
  float* w_row = reinterpret_cast<float*>(plan + L.off[8]);
  int32_t* row_slot = plan + L.off[9];
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int base = beg; base < end; base += 32) {
    const int s = base + lane;
    int e = (s < end) ? idx[s] : -1;
    if (e >= E || e < 0) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int pos = -1;
    if (e >= 0) {
      pos = cnt[warp * E + e] + __popc(peers & lt_mask);
      tok_row[pos] = s / k;
      w_row[pos] = wts[s];
    }
    if (s < end) row_slot[s] = pos;
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

}  // namespace

size_t plan_smem_bytes(int E) { return (size_t)(kPlanWarps + 2) * E * sizeof(int); }

int launch_route_plan(const int32_t* idx, const float* w, int T, int k, int E, int tm, int pass_tokens,
                      int32_t* plan, cudaStream_t stream, int* zero, int n_zero, const SplitX* split) {
  const PlanLayout L = plan_layout(T, k, E, tm, pass_tokens);
  const size_t smem = plan_smem_bytes(E);
  static PerDevice s_attr;
  long long set = 0;
  const int arc = per_device(s_attr, [&](long long& v) -> int {
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)plan_smem_bytes(kPlanMaxExperts)));
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(plan_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kPlanCtaWarps * kPlanMaxExperts * 4));
    CBMOE_CUDA_TRY(cudaFuncSetAttribute(plan_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kPlanCtaWarps * kPlanMaxExperts * 4));
    v = 1;
    return CBMOE_OK;
  }, &set);
  if (arc) return arc;
  const long long S = (long long)T * k;
  const int n_chunks = (int)((S + kPlanChunkSlots - 1) / kPlanChunkSlots);
  SplitX sx{};
  if (split != nullptr && split->x8 != nullptr && split->N > 0) sx = *split;
  if (S > kPlanBigSlots && n_chunks <= kPlanMaxChunks) {
    if (sx.x8 != nullptr) {
      const int rc = launch_split_x(sx.x, sx.N, sx.K, sx.x8, sx.scale, stream);
      if (rc) return rc;
    }
    int32_t* chunk = plan + L.off[12] + ((L.off[11] - L.off[10] + 3) & ~3);   // scratch after the pass lists
    const size_t csmem = (size_t)kPlanCtaWarps * E * 4;
    prof_begin(kProfPlan, stream);
    plan_count_kernel<<<n_chunks, kPlanCtaWarps * 32, csmem, stream>>>(idx, (int)S, E, chunk);
    plan_scan_kernel<<<1, kPlanThreads, 3 * E * 4, stream>>>(T, k, E, tm, pass_tokens, n_chunks, plan, L, chunk, zero,
                                                             n_zero);
    plan_place_kernel<<<n_chunks, kPlanCtaWarps * 32, csmem, stream>>>(idx, w, (int)S, k, E, plan, L, chunk);
    prof_end(kProfPlan, stream);
    prof_add_launches(2);
    CBMOE_CUDA_TRY(cudaGetLastError());
    return CBMOE_OK;
  }
  prof_begin(kProfPlan, stream);
  int blocks = 1;
  if (sx.x8 != nullptr) blocks += sx.N < num_sms() * 2 ? sx.N : num_sms() * 2;
  CBMOE_CUDA_TRY(launch_pdl(route_plan_kernel, dim3(blocks), dim3(kPlanThreads), smem, stream, idx, w, T, k, E, tm,
                            pass_tokens, plan, L, zero, n_zero, sx));
  prof_end(kProfPlan, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

}  // namespace cbmoe

extern "C" int cbmoe_plan_layout(int T, int k, int E, int tm, int pass_tokens, int64_t* offsets14_host) {
  if (T < 0 || k <= 0 || E <= 0 || E > cbmoe::kPlanMaxExperts || tm <= 0 || pass_tokens <= 0 || !offsets14_host)
    return CBMOE_ERR_INVALID;
  const cbmoe::PlanLayout L = cbmoe::plan_layout(T, k, E, tm, pass_tokens);
  for (int i = 0; i < 14; ++i) offsets14_host[i] = L.off[i];
  return CBMOE_OK;
}

extern "C" int cbmoe_route_plan(const int32_t* idx, const float* w, int T, int k, int E, int tm, int pass_tokens,
                                void* plan, size_t plan_bytes, cudaStream_t stream) {
  if (T < 0 || k <= 0 || E <= 0 || E > cbmoe::kPlanMaxExperts || tm <= 0 || pass_tokens <= 0 || !plan ||
      (T > 0 && (!idx || !w)))
    return CBMOE_ERR_INVALID;
  const cbmoe::PlanLayout L = cbmoe::plan_layout(T, k, E, tm, pass_tokens);
  if (plan_bytes < (size_t)L.off[13] * 4) return CBMOE_ERR_WORKSPACE;
  return cbmoe::launch_route_plan(idx, w, T, k, E, tm, pass_tokens, static_cast<int32_t*>(plan), stream, nullptr, 0);
}
