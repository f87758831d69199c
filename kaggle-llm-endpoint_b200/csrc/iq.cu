// The reference's GGUF expert formats (llama.cpp IQ2_S / IQ3_S / IQ4_XS, and Q2_K / Q3_K of its MTP layer): dequant
// of raw GGUF blocks on the GPU and the routed experts straight from those tables. The per-lane arithmetic is
// iqlane.cuh (shared with a host test harness).
// Counterpart of the reference's iqquant.dequant_rows and dequant_* (engine/glm53/iqquant.py:108-146, 200-235) and
// planes.dequant_planes (planes.py:183-196), in fp32, bit for bit: the same products in the same order, each rounded
// once (no fused multiply-add). One warp per 256-weight block, lane l producing weights 8l .. 8l+7 (iq_lane8, two
// 16-byte stores). The lookup tables are the caller's (fp32, gguf-py's grids): IQ2_S [1024][8], IQ3_S [512][4],
// IQ4_XS [16]; the K-quants need none.
#include <cuda_fp16.h>

#include "iqlane.cuh"
#include "layer.cuh"
#include "profile.cuh"

namespace cbmoe {

namespace {

template <int T>
__global__ void iq_dequant_kernel(const uint8_t* __restrict__ blocks, long long n_blocks,
                                  const float* __restrict__ table, float* __restrict__ out) {
  constexpr int BB = IqFmt<T>::kBytes;
  constexpr int TAB = IqFmt<T>::kEntries * IqFmt<T>::kWidth;   // 0: no lookup table (K-quants)
  __shared__ __align__(16) float tab[TAB > 0 ? TAB : 4];         // grid rows 16-byte aligned for iq_lane8
  for (int i = threadIdx.x; i < TAB; i += blockDim.x) tab[i] = table[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long b = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < n_blocks; b += warps) {
    float v[8];
    iq_lane8<T>(blocks + b * BB, lane, tab, v);
    float4* o = reinterpret_cast<float4*>(out + b * 256 + 8 * lane);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

template <int T>
int launch_iq(const void* blocks, long long n_blocks, const float* table, float* out, cudaStream_t s) {
  long long grid = (n_blocks + 7) / 8;   // 8 warps per CTA, one block each
  const long long cap = (long long)num_sms() * 16;
  if (grid > cap) grid = cap;
  prof_begin(kProfOther, s);
  iq_dequant_kernel<T><<<(int)grid, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), n_blocks, table, out);
  prof_end(kProfOther, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

// ------------------------------------------------------------------------------------------ fused expert path
// The decode composition of resident.py:110-120 (`_apply_kernel`: gate/up -> swiglu_clamped -> down -> weighted sum
// of the slots) over raw GGUF IQ tables, computing in fp32 as the reference's moe_matvec does
// (pallas_moe.py:238-307: on-the-fly dequant, fp32 products and sums). Rows of the routing plan are grouped in
// passes of up to kIqPassTokens slots of one expert; an item is (pass, kIqRows consecutive weight rows), one warp
// per item: for every 256-weight block, each lane loads its 8 inputs of every token of the pass once (registers),
// then dequantizes its 8 weights of each of the item's rows (iq_lane8, the table in shared memory) and multiply-adds
// them into one fp32 partial per (row, token); warp sums give the outputs. The rows of an item share the input
// loads, and their dequant chains are independent (instruction-level parallelism).
//   gate, up: x = the slots' token rows (bf16, through the plan's row -> token map) -> g, u fp32 [sorted row][I]
//   h = swiglu_clamped(g, u) (elementwise, into g's buffer)
//   down:     x = h (fp32 sorted rows) -> y fp32 [sorted row][H]; combine_kernel sums the slots.
constexpr int kIqPassTokens = 8;
constexpr int kIqRows = 4;   // weight rows per item (rows are multiples of 256)

struct IqMatParams {
  const uint8_t* w;          // raw blocks [E][rows][K / 256][block bytes]
  const float* table;        // the format's lookup table (global; copied to shared memory per CTA)
  int rows, K, E;
  const int* pass_expert;
  const int* pass_row0;
  const int* pass_cnt;
  const int* n_pass;
  const uint16_t* x;         // gate/up: bf16 token rows [N][K]
  const int* tok_row;        //   sorted row -> token
  const float* h;            // down: fp32 SwiGLU rows [sorted row][K]
  float* out;                // fp32 [sorted row][rows]
};

__device__ __forceinline__ void bf16x8(const uint4& q, float (&f)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// PT: tokens held in registers at a time (2 for small passes: more warps per SM; 8 for full ones); a pass of more
// tokens is walked in chunks of PT, each chunk dequantizing the weights again.
template <int T, int H_IN, int PT>
__global__ void __launch_bounds__(256, PT <= 2 ? 3 : 1) iq_matvec_kernel(const IqMatParams p) {
  constexpr int BB = IqFmt<T>::kBytes;
  constexpr int TAB = IqFmt<T>::kEntries * IqFmt<T>::kWidth;   // 0: no lookup table (K-quants)
  __shared__ __align__(16) float tab[TAB > 0 ? TAB : 4];
  for (int i = threadIdx.x; i < TAB; i += blockDim.x) tab[i] = p.table[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nblk = p.K / 256;
  const int groups = p.rows / kIqRows;
  const long long items = (long long)(*p.n_pass) * groups;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
    const int pass = (int)(it / groups), r0 = (int)(it % groups) * kIqRows;
    const int e = p.pass_expert[pass], row0_pass = p.pass_row0[pass];
    const int cnt_pass = min(p.pass_cnt[pass], kIqPassTokens);
    if (e < 0 || e >= p.E || cnt_pass <= 0) continue;
    const uint8_t* wrow = p.w + ((size_t)e * p.rows + r0) * nblk * BB;
    const size_t row_stride = (size_t)nblk * BB;
    for (int c0 = 0; c0 < cnt_pass; c0 += PT) {
      const int row0 = row0_pass + c0, cnt = min(PT, cnt_pass - c0);
      const uint16_t* xr[PT];
      const float* hr[PT];
#pragma unroll
      for (int t = 0; t < PT; ++t) {
        const int tt = t < cnt ? t : 0;
        xr[t] = H_IN ? nullptr : p.x + (size_t)p.tok_row[row0 + tt] * p.K + 8 * lane;
        hr[t] = H_IN ? p.h + (size_t)(row0 + tt) * p.K + 8 * lane : nullptr;
      }
      float acc[kIqRows][PT];
#pragma unroll
      for (int r = 0; r < kIqRows; ++r)
#pragma unroll
        for (int t = 0; t < PT; ++t) acc[r][t] = 0.f;
      for (int b = 0; b < nblk; ++b) {
        float xv[PT][8];
#pragma unroll
        for (int t = 0; t < PT; ++t) {
          if (t < cnt) {
            if constexpr (H_IN) {
              const float4 h0 = __ldg(reinterpret_cast<const float4*>(hr[t] + b * 256));
              const float4 h1 = __ldg(reinterpret_cast<const float4*>(hr[t] + b * 256) + 1);
              xv[t][0] = h0.x; xv[t][1] = h0.y; xv[t][2] = h0.z; xv[t][3] = h0.w;
              xv[t][4] = h1.x; xv[t][5] = h1.y; xv[t][6] = h1.z; xv[t][7] = h1.w;
            } else {
              bf16x8(__ldg(reinterpret_cast<const uint4*>(xr[t] + b * 256)), xv[t]);
            }
          }
        }
#pragma unroll
        for (int r = 0; r < kIqRows; ++r) {
          float v[8];
          iq_lane8<T>(wrow + r * row_stride + (size_t)b * BB, lane, tab, v);
#pragma unroll
          for (int t = 0; t < PT; ++t) {
            if (t < cnt) {
              float a = acc[r][t];
#pragma unroll
              for (int j = 0; j < 8; ++j) a = fmaf(v[j], xv[t][j], a);
              acc[r][t] = a;
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < PT; ++t) {
        if (t >= cnt) break;
#pragma unroll
        for (int r = 0; r < kIqRows; ++r) {
          float a = acc[r][t];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
          if (lane == r) p.out[(size_t)(row0 + t) * p.rows + r0 + r] = a;
        }
      }
    }
  }
}

// g[i] = swiglu_clamped(g[i], u[i], limit) over n elements (fp32, in place).
__global__ void iq_swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, long long n, float limit) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    g[i] = swiglu_clamped(g[i], u[i], limit);
}

template <int H_IN, int PT>
void launch_iq_matvec_pt(int type, const IqMatParams& p, int grid, cudaStream_t s) {
  switch (type) {
    case CBMOE_GGML_IQ2_S: iq_matvec_kernel<CBMOE_GGML_IQ2_S, H_IN, PT><<<grid, 256, 0, s>>>(p); break;
    case CBMOE_GGML_IQ3_S: iq_matvec_kernel<CBMOE_GGML_IQ3_S, H_IN, PT><<<grid, 256, 0, s>>>(p); break;
    case CBMOE_GGML_IQ4_XS: iq_matvec_kernel<CBMOE_GGML_IQ4_XS, H_IN, PT><<<grid, 256, 0, s>>>(p); break;
    case CBMOE_GGML_Q2_K: iq_matvec_kernel<CBMOE_GGML_Q2_K, H_IN, PT><<<grid, 256, 0, s>>>(p); break;
    default: iq_matvec_kernel<CBMOE_GGML_Q3_K, H_IN, PT><<<grid, 256, 0, s>>>(p); break;
  }
}

// small: the passes average at most 2 tokens (the 2-token register variant, 3 CTAs per SM)
template <int H_IN>
int launch_iq_matvec(int type, const IqMatParams& p, long long max_items, bool small, int kind, cudaStream_t s) {
  long long grid = (max_items / kIqRows + 7) / 8;
  const long long cap = (long long)num_sms() * (small ? 3 : 1);
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  prof_begin(kind, s);
  if (small) launch_iq_matvec_pt<H_IN, 2>(type, p, (int)grid, s);
  else launch_iq_matvec_pt<H_IN, kIqPassTokens>(type, p, (int)grid, s);
  prof_end(kind, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

// Workspace: plan | g (Rp x I f32) | u | y (Rp x H f32) | X8 rows of x for the gate matrix's int8 kernel (N x H x 2
// B) and factors | the same for up when its format differs | X8 rows of h for the down matrix's (Rp x I x 2 B) and
// factors (each X8 region only when that matrix has its int8 layout).
struct IqWorkspace {
  lyr::PlanLayoutHost L;
  int Rp, P;
  size_t plan, g, u, y, xg8, xg8s, xu8, xu8s, h8, h8s, total;
};

bool use_iq8(int type, const void* table8) { return table8 != nullptr && iq8_type(type); }

IqWorkspace iq_workspace(const cbmoe_iq_experts* ex, int N, int k) {
  IqWorkspace w;
  w.L = lyr::host_plan_layout(N, k, ex->E, 1, kIqPassTokens);
  w.Rp = (int)(w.L.off[8] - w.L.off[7]);
  w.P = (int)(w.L.off[11] - w.L.off[10]);
  w.plan = 0;
  w.g = lyr::align_up((size_t)w.L.off[13] * 4);
  w.u = w.g + lyr::align_up((size_t)w.Rp * ex->I * 4);
  w.y = w.u + lyr::align_up((size_t)w.Rp * ex->I * 4);
  size_t o = w.y + lyr::align_up((size_t)w.Rp * ex->H * 4);
  const bool g8 = use_iq8(ex->gate_type, ex->gate8), u8 = use_iq8(ex->up_type, ex->up8);
  const bool u8_own = u8 && !(g8 && ex->gate_type == ex->up_type);
  w.xg8 = o;
  w.xg8s = w.xg8 + (g8 ? lyr::align_up((size_t)N * ex->H * 2) : 0);
  w.xu8 = w.xg8s + (g8 ? lyr::align_up((size_t)N * 4) : 0);
  w.xu8s = w.xu8 + (u8_own ? lyr::align_up((size_t)N * ex->H * 2) : 0);
  w.h8 = w.xu8s + (u8_own ? lyr::align_up((size_t)N * 4) : 0);
  const bool d8 = use_iq8(ex->down_type, ex->down8);
  w.h8s = w.h8 + (d8 ? lyr::align_up((size_t)w.Rp * ex->I * 2) : 0);
  w.total = w.h8s + (d8 ? lyr::align_up((size_t)w.Rp * 4) : 0);
  return w;
}

bool iq_has_table(int t) { return t == CBMOE_GGML_IQ2_S || t == CBMOE_GGML_IQ3_S || t == CBMOE_GGML_IQ4_XS; }

bool iq_experts_ok(const cbmoe_iq_experts* ex) {
  auto ok_type = [](int t) { return cbmoe_iq_block_bytes(t) != 0; };
  return ex && ex->E > 0 && ex->E <= 1024 && ex->H > 0 && ex->I > 0 && ex->H % 256 == 0 && ex->I % 256 == 0 &&
         ok_type(ex->gate_type) && ok_type(ex->up_type) && ok_type(ex->down_type) && ex->gate && ex->up &&
         ex->down && (ex->gate_table || !iq_has_table(ex->gate_type)) &&
         (ex->up_table || !iq_has_table(ex->up_type)) && (ex->down_table || !iq_has_table(ex->down_type)) &&
         !(reinterpret_cast<uintptr_t>(ex->gate8) & 255) && !(reinterpret_cast<uintptr_t>(ex->up8) & 255) &&
         !(reinterpret_cast<uintptr_t>(ex->down8) & 255);
}

}  // namespace

}  // namespace cbmoe

using namespace cbmoe;

extern "C" size_t cbmoe_iq_workspace_bytes(const cbmoe_iq_experts* ex, int N, int k) {
  if (!iq_experts_ok(ex) || N < 0 || k <= 0 || k > 64) return 0;
  return iq_workspace(ex, N, k).total;
}

extern "C" int cbmoe_iq_experts_apply(const cbmoe_iq_experts* ex, const uint16_t* x, int N, const int32_t* idx,
                                      const float* w, int k, float limit, float* y, void* workspace,
                                      size_t workspace_bytes, cudaStream_t stream) {
  if (!iq_experts_ok(ex) || N < 0 || k <= 0 || k > 64) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (!x || !idx || !w || !y || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return CBMOE_ERR_INVALID;
  const IqWorkspace W = iq_workspace(ex, N, k);
  if (!workspace || workspace_bytes < W.total) return CBMOE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return CBMOE_ERR_INVALID;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* plan = reinterpret_cast<int32_t*>(ws + W.plan);
  int rc = launch_route_plan(idx, w, N, k, ex->E, 1, kIqPassTokens, plan, stream);
  if (rc) return rc;
  float* g = reinterpret_cast<float*>(ws + W.g);
  float* u = reinterpret_cast<float*>(ws + W.u);
  float* ys = reinterpret_cast<float*>(ws + W.y);
  IqMatParams p{};
  p.rows = ex->I;
  p.K = ex->H;
  p.E = ex->E;
  p.pass_expert = plan + W.L.off[10];
  p.pass_row0 = plan + W.L.off[11];
  p.pass_cnt = plan + W.L.off[12];
  p.n_pass = plan + W.L.off[5];
  p.x = x;
  p.tok_row = plan + W.L.off[7];
  const long long items_gu = (long long)W.P * ex->I, items_dn = (long long)W.P * ex->H;
  const bool small = (long long)N * k <= 2LL * ex->E;
  const int32_t* n_pass = plan + W.L.off[5];
  // gate and up: the int8 kernels on X8 rows of x where the matrix has its int8 layout, else the fp32 kernel
  const bool g8 = use_iq8(ex->gate_type, ex->gate8), u8 = use_iq8(ex->up_type, ex->up8);
  uint8_t* xg8 = ws + W.xg8;
  float* xg8s = reinterpret_cast<float*>(ws + W.xg8s);
  uint8_t* xu8 = (g8 && ex->gate_type == ex->up_type) ? xg8 : ws + W.xu8;
  float* xu8s = (g8 && ex->gate_type == ex->up_type) ? xg8s : reinterpret_cast<float*>(ws + W.xu8s);
  if (g8) {
    rc = iq8_split(ex->gate_type, x, false, N, ex->H, xg8, xg8s, stream);
    if (!rc) rc = iq8_matvec(ex->gate_type, ex->gate8, ex->E, ex->I, ex->H, p.pass_expert, p.pass_row0, p.pass_cnt,
                             n_pass, p.tok_row, xg8, xg8s, g, kProfIqGateUp, stream);
  } else {
    p.w = static_cast<const uint8_t*>(ex->gate);
    p.table = ex->gate_table;
    p.out = g;
    rc = launch_iq_matvec<0>(ex->gate_type, p, items_gu, small, kProfIqGateUp, stream);
  }
  if (rc) return rc;
  if (u8) {
    if (xu8 != xg8) rc = iq8_split(ex->up_type, x, false, N, ex->H, xu8, xu8s, stream);
    if (!rc) rc = iq8_matvec(ex->up_type, ex->up8, ex->E, ex->I, ex->H, p.pass_expert, p.pass_row0, p.pass_cnt,
                             n_pass, p.tok_row, xu8, xu8s, u, kProfIqGateUp, stream);
  } else {
    p.w = static_cast<const uint8_t*>(ex->up);
    p.table = ex->up_table;
    p.out = u;
    rc = launch_iq_matvec<0>(ex->up_type, p, items_gu, small, kProfIqGateUp, stream);
  }
  if (rc) return rc;
  if (use_iq8(ex->down_type, ex->down8)) {
    // SwiGLU and the split of h into X8 digits in one pass over the rows (h itself is not stored)
    uint8_t* h8 = ws + W.h8;
    float* h8s = reinterpret_cast<float*>(ws + W.h8s);
    rc = iq8_swiglu_split(ex->down_type, g, u, limit, W.Rp, ex->I, h8, h8s, stream);
    if (!rc) rc = iq8_matvec(ex->down_type, ex->down8, ex->E, ex->H, ex->I, p.pass_expert, p.pass_row0, p.pass_cnt,
                             n_pass, nullptr, h8, h8s, ys, kProfIqDown, stream);
  } else {
    const long long n = (long long)W.Rp * ex->I;
    long long blocks = (n + 255) / 256;
    if (blocks > (long long)num_sms() * 8) blocks = (long long)num_sms() * 8;
    prof_begin(kProfIqGateUp, stream);
    iq_swiglu_kernel<<<(int)blocks, 256, 0, stream>>>(g, u, n, limit);
    prof_end(kProfIqGateUp, stream);
    CBMOE_CUDA_TRY(cudaGetLastError());
    IqMatParams d = p;
    d.w = static_cast<const uint8_t*>(ex->down);
    d.table = ex->down_table;
    d.rows = ex->H;
    d.K = ex->I;
    d.x = nullptr;
    d.tok_row = nullptr;
    d.h = g;
    d.out = ys;
    rc = launch_iq_matvec<1>(ex->down_type, d, items_dn, small, kProfIqDown, stream);
  }
  if (rc) return rc;
  return launch_combine(ys, plan + W.L.off[9], w, N, k, ex->H, nullptr, y, nullptr, stream);
}

extern "C" size_t cbmoe_iq_block_bytes(int ggml_type) {
  switch (ggml_type) {
    case CBMOE_GGML_IQ2_S: return IqFmt<CBMOE_GGML_IQ2_S>::kBytes;
    case CBMOE_GGML_IQ3_S: return IqFmt<CBMOE_GGML_IQ3_S>::kBytes;
    case CBMOE_GGML_IQ4_XS: return IqFmt<CBMOE_GGML_IQ4_XS>::kBytes;
    case CBMOE_GGML_Q2_K: return IqFmt<CBMOE_GGML_Q2_K>::kBytes;
    case CBMOE_GGML_Q3_K: return IqFmt<CBMOE_GGML_Q3_K>::kBytes;
    default: return 0;
  }
}

extern "C" int cbmoe_iq_table_shape(int ggml_type, int* entries, int* width) {
  if (!entries || !width) return CBMOE_ERR_INVALID;
  switch (ggml_type) {
    case CBMOE_GGML_IQ2_S: *entries = IqFmt<CBMOE_GGML_IQ2_S>::kEntries; *width = IqFmt<CBMOE_GGML_IQ2_S>::kWidth; break;
    case CBMOE_GGML_IQ3_S: *entries = IqFmt<CBMOE_GGML_IQ3_S>::kEntries; *width = IqFmt<CBMOE_GGML_IQ3_S>::kWidth; break;
    case CBMOE_GGML_IQ4_XS: *entries = IqFmt<CBMOE_GGML_IQ4_XS>::kEntries; *width = IqFmt<CBMOE_GGML_IQ4_XS>::kWidth; break;
    case CBMOE_GGML_Q2_K:
    case CBMOE_GGML_Q3_K: *entries = 0; *width = 0; break;
    default: return CBMOE_ERR_UNSUPPORTED;
  }
  return CBMOE_OK;
}

extern "C" int cbmoe_iq_dequant(int ggml_type, const void* blocks, long long n_blocks, const float* table, float* out,
                                cudaStream_t stream) {
  if (cbmoe_iq_block_bytes(ggml_type) == 0) return CBMOE_ERR_UNSUPPORTED;
  if (n_blocks < 0) return CBMOE_ERR_INVALID;
  if (n_blocks == 0) return CBMOE_OK;
  if (!blocks || !out || (reinterpret_cast<uintptr_t>(out) & 15) || (iq_has_table(ggml_type) && !table) ||
      (reinterpret_cast<uintptr_t>(table) & 3))
    return CBMOE_ERR_INVALID;
  switch (ggml_type) {
    case CBMOE_GGML_IQ2_S: return launch_iq<CBMOE_GGML_IQ2_S>(blocks, n_blocks, table, out, stream);
    case CBMOE_GGML_IQ3_S: return launch_iq<CBMOE_GGML_IQ3_S>(blocks, n_blocks, table, out, stream);
    case CBMOE_GGML_IQ4_XS: return launch_iq<CBMOE_GGML_IQ4_XS>(blocks, n_blocks, table, out, stream);
    case CBMOE_GGML_Q2_K: return launch_iq<CBMOE_GGML_Q2_K>(blocks, n_blocks, table, out, stream);
    default: return launch_iq<CBMOE_GGML_Q3_K>(blocks, n_blocks, table, out, stream);
  }
}
