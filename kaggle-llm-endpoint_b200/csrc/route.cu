// MoE router, fused: logits -> sigmoid -> + bias -> top-k -> normalize -> scale in one kernel. Counterpart of the
// reference's moe_route (engine/glm53/model.py:798-808, n_group == 1), which produces the (idx, w) the expert path
// takes:
//   logits = f32(x) @ f32(W);  s = sigmoid(logits);  idx = top_k(s + bias, k) (largest first, the lower expert
//   index first among equal choices);  w = s[idx];  norm_topk: w /= (sum w + 1e-20);  w *= scaling.
// One CTA per 8 tokens, 8 warps: warp q multiplies the 8 tokens' inputs [q*D/8, (q+1)*D/8) against W (bf16 [D][E],
// row-major; lane owns experts lane + 32j, so every warp load of a W row segment is contiguous) with the tokens'
// inputs staged in shared memory; the partial logits meet in shared memory, then warp t sums them for token t and
// selects its top k with k rounds of a warp-wide argmax. fp32 throughout (the sum order differs from the
// reference's dot, so only near-equal choices can come out in a different order).
#include "layout.cuh"
#include "profile.cuh"

namespace cbmoe {

namespace {

constexpr int kRouteTok = 8;         // tokens per CTA
constexpr int kRouteWarps = 8;
constexpr int kRouteMaxE = 256;      // 8 experts per lane
constexpr int kRouteMaxK = 32;

// a beats b: larger choice, or equal choice and lower expert index
__device__ __forceinline__ bool route_better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

__global__ void __launch_bounds__(kRouteWarps * 32)
    route_kernel(const uint16_t* __restrict__ x, int N, int D, const uint16_t* __restrict__ W,
                 const float* __restrict__ bias, int E, int k, int norm_topk, float scaling, int32_t* __restrict__ idx,
                 float* __restrict__ wout) {
  extern __shared__ float route_smem[];
  float* part = route_smem;                                   // [warps][tokens][E]
  uint16_t* xs = reinterpret_cast<uint16_t*>(part + kRouteWarps * kRouteTok * E);   // [tokens][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kRouteTok;
  const int nt = min(kRouteTok, N - n0);
  for (int i = threadIdx.x; i < kRouteTok * D; i += blockDim.x) {
    const int t = i / D, d = i % D;
    xs[i] = t < nt ? x[(size_t)(n0 + t) * D + d] : (uint16_t)0;
  }
  __syncthreads();

  const int EJ = (E + 31) / 32;
  float acc[kRouteTok][8];
#pragma unroll
  for (int t = 0; t < kRouteTok; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[t][j] = 0.f;
  const int dpw = (D + kRouteWarps - 1) / kRouteWarps;
  const int d0 = warp * dpw, d1 = min(D, d0 + dpw);
  for (int d = d0; d < d1; ++d) {
    float xv[kRouteTok];
#pragma unroll
    for (int t = 0; t < kRouteTok; ++t) xv[t] = __uint_as_float((uint32_t)xs[t * D + d] << 16);
    const uint16_t* wr = W + (size_t)d * E;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane + 32 * j;
      if (j < EJ && e < E) {
        const float wv = __uint_as_float((uint32_t)__ldg(wr + e) << 16);
#pragma unroll
        for (int t = 0; t < kRouteTok; ++t) acc[t][j] = fmaf(xv[t], wv, acc[t][j]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kRouteTok; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane + 32 * j;
      if (j < EJ && e < E) part[(warp * kRouteTok + t) * E + e] = acc[t][j];
    }
  __syncthreads();

  // warp t: token n0 + t
  const int t = warp;
  if (t >= nt) return;
  float sc[8], ch[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane + 32 * j;
    sc[j] = 0.f;
    ch[j] = -INFINITY;
    if (j < EJ && e < E) {
      float lg = 0.f;
      for (int q = 0; q < kRouteWarps; ++q) lg += part[(q * kRouteTok + t) * E + e];
      sc[j] = 1.0f / (1.0f + expf(-lg));
      ch[j] = sc[j] + bias[e];
    }
  }
  int my_idx = -1;     // lane r < k keeps the r-th choice
  float my_w = 0.f, sum = 0.f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY, bs = 0.f;
    int be = 0x7fffffff, bj = -1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane + 32 * j;
      if (j < EJ && e < E && ch[j] != -INFINITY && route_better(ch[j], e, bv, be)) {
        bv = ch[j];
        be = e;
        bs = sc[j];
        bj = j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      if (route_better(ov, oe, bv, be)) {
        bv = ov;
        be = oe;
        bs = os;
      }
    }
    // every lane now holds the winner (be, bs); its owner takes it out of the running
    if (bj >= 0 && lane + 32 * bj == be) ch[bj] = -INFINITY;
    if (lane == r) {
      my_idx = be;
      my_w = bs;
    }
    sum += bs;
  }
  if (lane < k) {
    float wv = my_w;
    if (norm_topk) wv = wv / (sum + 1e-20f);
    idx[(size_t)(n0 + t) * k + lane] = my_idx;
    wout[(size_t)(n0 + t) * k + lane] = wv * scaling;
  }
}

}  // namespace

}  // namespace cbmoe

using namespace cbmoe;

extern "C" int cbmoe_route(const uint16_t* x, int N, int D, const uint16_t* router_w, const float* bias, int E, int k,
                           int norm_topk, float scaling, int32_t* idx, float* w, cudaStream_t stream) {
  if (N < 0 || D <= 0 || E <= 0 || E > kRouteMaxE || k <= 0 || k > kRouteMaxK || k > E) return CBMOE_ERR_INVALID;
  if (N == 0) return CBMOE_OK;
  if (!x || !router_w || !bias || !idx || !w) return CBMOE_ERR_INVALID;
  const size_t smem = (size_t)kRouteWarps * kRouteTok * E * sizeof(float) + (size_t)kRouteTok * D * sizeof(uint16_t);
  if (smem > 200 * 1024) return CBMOE_ERR_UNSUPPORTED;   // D up to ~8000 at E = 256
  if (smem > 48 * 1024) {   // the largest size the kernel may be given, once per device
    static PerDevice s_attr;
    long long set = 0;
    const int rc = per_device(s_attr, [&](long long& v) -> int {
      CBMOE_CUDA_TRY(cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      v = 1;
      return CBMOE_OK;
    }, &set);
    if (rc) return rc;
  }
  const int blocks = (N + kRouteTok - 1) / kRouteTok;
  prof_begin(kProfOther, stream);
  route_kernel<<<blocks, kRouteWarps * 32, smem, stream>>>(x, N, D, router_w, bias, E, k, norm_topk, scaling, idx, w);
  prof_end(kProfOther, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}
