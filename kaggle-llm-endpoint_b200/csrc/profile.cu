// Launch accounting and optional per-kernel CUDA-event timing (host side only).
// Every kernel launcher calls prof_begin / prof_end around its launch. The launch counter always runs; when timing
// is enabled each launch is bracketed by a pair of events recorded on the launching stream, and
// cbmoe_profile_read() sums their elapsed times per kernel kind.
#include <mutex>
#include <vector>

#include "profile.cuh"
#include "common.cuh"

namespace cbmoe {
namespace {

struct Pending {
  int kind;
  cudaEvent_t a, b;
};

std::mutex g_mu;
bool g_enabled = false;
long long g_launches = 0;
std::vector<cudaEvent_t> g_pool;
std::vector<Pending> g_pending;
double g_ms[kProfKinds] = {0};
long long g_count[kProfKinds] = {0};
thread_local Pending t_open{-1, nullptr, nullptr};

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

}  // namespace

void prof_begin(int kind, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (kind != kProfExchange) ++g_launches;   // an exchange is NCCL's work, not a launch of this library
  if (!g_enabled) return;
  t_open = {kind, take_event(), take_event()};
  cudaEventRecord(t_open.a, s);
}

void prof_add_launches(int n) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_launches += n;
}

void prof_end(int kind, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_enabled || t_open.kind != kind) return;
  cudaEventRecord(t_open.b, s);
  g_pending.push_back(t_open);
  t_open = {-1, nullptr, nullptr};
}

}  // namespace cbmoe

using namespace cbmoe;

extern "C" long long cbmoe_launch_count(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  return g_launches;
}

extern "C" int cbmoe_profile_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_enabled = enable != 0;
  return CBMOE_OK;
}

extern "C" int cbmoe_profile_read(int reset, double* ms_host, long long* count_host, int n_kinds) {
  if (!ms_host || !count_host || n_kinds < kProfKinds) return CBMOE_ERR_INVALID;
  std::lock_guard<std::mutex> lk(g_mu);
  for (const Pending& p : g_pending) {
    if (cudaEventSynchronize(p.b) != cudaSuccess) return CBMOE_ERR_CUDA;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, p.a, p.b) != cudaSuccess) return CBMOE_ERR_CUDA;
    g_ms[p.kind] += ms;
    g_count[p.kind] += 1;
    g_pool.push_back(p.a);
    g_pool.push_back(p.b);
  }
  g_pending.clear();
  for (int i = 0; i < kProfKinds; ++i) {
    ms_host[i] = g_ms[i];
    count_host[i] = g_count[i];
    if (reset) {
      g_ms[i] = 0;
      g_count[i] = 0;
    }
  }
  return CBMOE_OK;
}

// ------------------------------------------------------------------------------------------------ self-test
namespace cbmoe {
namespace {
// One CTA waits, through the kernels' own bounded wait, on an mbarrier phase that nothing completes. The wait
// gives up after limit_ns, records CBMOE_DEVERR_TIMEOUT and the kernel returns: the path every ring wait takes
// when a producer or a peer never delivers.
__global__ void wait_selftest_kernel(unsigned long long limit_ns, int* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) *gave_up = mbar_wait(&bar, 0, limit_ns) ? 0 : 1;
}
}  // namespace
}  // namespace cbmoe

extern "C" int cbmoe_selftest_wait_timeout(long long limit_ns, int* gave_up_device, cudaStream_t stream) {
  if (limit_ns <= 0 || limit_ns > 10000000000LL || !gave_up_device) return CBMOE_ERR_INVALID;
  cbmoe::prof_begin(cbmoe::kProfOther, stream);
  cbmoe::wait_selftest_kernel<<<1, 32, 0, stream>>>((unsigned long long)limit_ns, gave_up_device);
  cbmoe::prof_end(cbmoe::kProfOther, stream);
  return cudaGetLastError() == cudaSuccess ? CBMOE_OK : CBMOE_ERR_CUDA;
}
