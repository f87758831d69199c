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
  const int lane = threadIdx.x & 31;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long b = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < n_blocks; b += warps) {
    float v[8];
    iq_lane8<T>(blocks + b * BB, lane, table, v);
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
// passes of up to kIqPassTokens slots of one expert; an item is (pass, weight row), one warp per item: each lane
// dequantizes its 8 weights of every 256-weight block of the row once (iq_lane8, the table in shared memory) and
// multiply-adds them into one fp32 partial per token of the pass; a warp sum gives the row's outputs.
//   gate, up: x = the slots' token rows (bf16, through the plan's row -> token map) -> g, u fp32 [sorted row][I]
//   h = swiglu_clamped(g, u) (elementwise, into g's buffer)
//   down:     x = h (fp32 sorted rows) -> y fp32 [sorted row][H]; combine_kernel sums the slots.
constexpr int kIqPassTokens = 8;

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

template <int T, int H_IN>
__global__ void __launch_bounds__(256) iq_matvec_kernel(const IqMatParams p) {
  constexpr int BB = IqFmt<T>::kBytes;
  constexpr int TAB = IqFmt<T>::kEntries * IqFmt<T>::kWidth;   // 0: no lookup table (K-quants)
  __shared__ float tab[TAB > 0 ? TAB : 1];
  for (int i = threadIdx.x; i < TAB; i += blockDim.x) tab[i] = p.table[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nblk = p.K / 256;
  const long long items = (long long)(*p.n_pass) * p.rows;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
    const int pass = (int)(it / p.rows), r = (int)(it % p.rows);
    const int e = p.pass_expert[pass], row0 = p.pass_row0[pass];
    const int cnt = min(p.pass_cnt[pass], kIqPassTokens);
    if (e < 0 || e >= p.E || cnt <= 0) continue;
    const uint8_t* wrow = p.w + ((size_t)e * p.rows + r) * nblk * BB;
    int tok[kIqPassTokens];
#pragma unroll
    for (int t = 0; t < kIqPassTokens; ++t) tok[t] = (!H_IN && t < cnt) ? p.tok_row[row0 + t] : 0;
    float acc[kIqPassTokens];
#pragma unroll
    for (int t = 0; t < kIqPassTokens; ++t) acc[t] = 0.f;
    for (int b = 0; b < nblk; ++b) {
      float v[8];
      iq_lane8<T>(wrow + (size_t)b * BB, lane, tab, v);
      const int k0 = b * 256 + 8 * lane;
#pragma unroll
      for (int t = 0; t < kIqPassTokens; ++t) {
        if (t >= cnt) break;
        float xv[8];
        if constexpr (H_IN) {
          const float* hp = p.h + (size_t)(row0 + t) * p.K + k0;
          const float4 h0 = *reinterpret_cast<const float4*>(hp), h1 = *reinterpret_cast<const float4*>(hp + 4);
          xv[0] = h0.x; xv[1] = h0.y; xv[2] = h0.z; xv[3] = h0.w;
          xv[4] = h1.x; xv[5] = h1.y; xv[6] = h1.z; xv[7] = h1.w;
        } else {
          bf16x8(*reinterpret_cast<const uint4*>(p.x + (size_t)tok[t] * p.K + k0), xv);
        }
        float a = acc[t];
#pragma unroll
        for (int j = 0; j < 8; ++j) a = fmaf(v[j], xv[j], a);
        acc[t] = a;
      }
    }
#pragma unroll
    for (int t = 0; t < kIqPassTokens; ++t) {
      if (t >= cnt) break;
      float a = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) p.out[(size_t)(row0 + t) * p.rows + r] = a;
    }
  }
}

// g[i] = swiglu_clamped(g[i], u[i], limit) over n elements (fp32, in place).
__global__ void iq_swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, long long n, float limit) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    g[i] = swiglu_clamped(g[i], u[i], limit);
}

template <int H_IN>
int launch_iq_matvec(int type, const IqMatParams& p, long long max_items, int kind, cudaStream_t s) {
  long long grid = (max_items + 7) / 8;
  const long long cap = (long long)num_sms() * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  prof_begin(kind, s);
  switch (type) {
    case CBMOE_GGML_IQ2_S: iq_matvec_kernel<CBMOE_GGML_IQ2_S, H_IN><<<(int)grid, 256, 0, s>>>(p); break;
    case CBMOE_GGML_IQ3_S: iq_matvec_kernel<CBMOE_GGML_IQ3_S, H_IN><<<(int)grid, 256, 0, s>>>(p); break;
    case CBMOE_GGML_IQ4_XS: iq_matvec_kernel<CBMOE_GGML_IQ4_XS, H_IN><<<(int)grid, 256, 0, s>>>(p); break;
    case CBMOE_GGML_Q2_K: iq_matvec_kernel<CBMOE_GGML_Q2_K, H_IN><<<(int)grid, 256, 0, s>>>(p); break;
    default: iq_matvec_kernel<CBMOE_GGML_Q3_K, H_IN><<<(int)grid, 256, 0, s>>>(p); break;
  }
  prof_end(kind, s);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

struct IqWorkspace {
  lyr::PlanLayoutHost L;
  int Rp, P;
  size_t plan, g, u, y, total;
};

IqWorkspace iq_workspace(const cbmoe_iq_experts* ex, int N, int k) {
  IqWorkspace w;
  w.L = lyr::host_plan_layout(N, k, ex->E, 1, kIqPassTokens);
  w.Rp = (int)(w.L.off[8] - w.L.off[7]);
  w.P = (int)(w.L.off[11] - w.L.off[10]);
  w.plan = 0;
  w.g = lyr::align_up((size_t)w.L.off[13] * 4);
  w.u = w.g + lyr::align_up((size_t)w.Rp * ex->I * 4);
  w.y = w.u + lyr::align_up((size_t)w.Rp * ex->I * 4);
  w.total = w.y + lyr::align_up((size_t)w.Rp * ex->H * 4);
  return w;
}

bool iq_has_table(int t) { return t == CBMOE_GGML_IQ2_S || t == CBMOE_GGML_IQ3_S || t == CBMOE_GGML_IQ4_XS; }

bool iq_experts_ok(const cbmoe_iq_experts* ex) {
  auto ok_type = [](int t) { return cbmoe_iq_block_bytes(t) != 0; };
  return ex && ex->E > 0 && ex->E <= 1024 && ex->H > 0 && ex->I > 0 && ex->H % 256 == 0 && ex->I % 256 == 0 &&
         ok_type(ex->gate_type) && ok_type(ex->up_type) && ok_type(ex->down_type) && ex->gate && ex->up &&
         ex->down && (ex->gate_table || !iq_has_table(ex->gate_type)) &&
         (ex->up_table || !iq_has_table(ex->up_type)) && (ex->down_table || !iq_has_table(ex->down_type));
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
  p.w = static_cast<const uint8_t*>(ex->gate);
  p.table = ex->gate_table;
  p.out = g;
  rc = launch_iq_matvec<0>(ex->gate_type, p, items_gu, kProfIqGateUp, stream);
  if (rc) return rc;
  p.w = static_cast<const uint8_t*>(ex->up);
  p.table = ex->up_table;
  p.out = u;
  rc = launch_iq_matvec<0>(ex->up_type, p, items_gu, kProfIqGateUp, stream);
  if (rc) return rc;
  {
    const long long n = (long long)W.Rp * ex->I;
    long long blocks = (n + 255) / 256;
    if (blocks > (long long)num_sms() * 8) blocks = (long long)num_sms() * 8;
    prof_begin(kProfIqGateUp, stream);
    iq_swiglu_kernel<<<(int)blocks, 256, 0, stream>>>(g, u, n, limit);
    prof_end(kProfIqGateUp, stream);
    CBMOE_CUDA_TRY(cudaGetLastError());
  }
  IqMatParams d = p;
  d.w = static_cast<const uint8_t*>(ex->down);
  d.table = ex->down_table;
  d.rows = ex->H;
  d.K = ex->I;
  d.x = nullptr;
  d.tok_row = nullptr;
  d.h = g;
  d.out = ys;
  rc = launch_iq_matvec<1>(ex->down_type, d, items_dn, kProfIqDown, stream);
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
