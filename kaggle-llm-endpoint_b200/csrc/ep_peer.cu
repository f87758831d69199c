// Peer-memory transport of the expert-parallel layer: the dispatch and the return go straight into the other GPUs'
// memory over NVLink instead of through NCCL send/recv.
//
// Every rank holds one buffer, mapped into every other rank's address space with CUDA IPC at set-up:
//   in_x    [nranks][cap][H] bf16   token rows sent to this rank, by source rank
//   in_meta [nranks][cap]    int32  their local expert ids (-1: unused row)
//   in_y    [nranks][cap][H]        expert outputs of this rank's slots, by the rank that computed them: f32
//                                   rows from the decode kernels, bf16 rows (packed) from the grouped ones
//   flag_x  [nranks], flag_y [nranks]  sequence numbers: source s sets flag_x[s] / flag_y[s] to the call's number
//                                   once all its writes for that call are visible
//   ctr     grid-completion counters of this rank's dispatch and return kernels
// One layer call: the dispatch kernel writes each kept slot's token row and every (peer, row) id into the peers'
// in_x / in_meta, and its last CTA raises flag_x on every peer; a one-CTA wait kernel on the receiver spins
// (bounded, %globaltimer) until every source's flag_x reached the call's number; the local experts read in_x; the
// return kernel writes each received row's output into its source's in_y and raises flag_y; the source waits on
// flag_y and combines from in_y. Writes are plain stores through peer pointers, made visible with a system-scope
// fence before the flag's release store; the receiver reads the flag with an acquire load. No multicast.
// Reuse of the buffers across calls is ordered by the calls themselves: a source writes call t+1's rows only after
// it has all of call t's outputs back, which every receiver sends only after it has finished reading call t's rows.
#include <cstring>
#include <vector>
#include <nccl.h>

#include "layer.cuh"
#include "profile.cuh"

namespace cbmoe {

constexpr int kPeerMax = 8;   // GPUs of one NVLink node

struct PeerPtrs {
  uint8_t* base[kPeerMax];
};

struct EpPeer {
  int nranks = 0, rank = 0, cap = 0, H = 0;
  size_t off_x = 0, off_meta = 0, off_y = 0, off_fx = 0, off_fy = 0, off_ctr = 0, off_poison = 0, bytes = 0;
  uint8_t* own = nullptr;
  PeerPtrs peers{};
  uint32_t seq = 0;
  // Poison: a wait kernel that gave up sets the device word (in this rank's own buffer, which the transport's
  // kernels read: an L2 hit) and its mirror in mapped pinned host memory (written only then, never read by a
  // kernel: a read of host memory from every thread would cross PCIe). From then on the transport's kernels write
  // nothing to peers and wait for nothing, and cbmoe_ep_layer returns CBMOE_ERR_DEVICE (it reads the host mirror
  // without synchronizing) until the peer is destroyed and set up again.
  volatile int* poison_host = nullptr;
  int* poison_mirror = nullptr;   // device address of poison_host
  int* poison_dev = nullptr;      // own + off_poison
};

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The CTA that finishes last raises flag[rank] on every peer (flags at byte offset off_flag of each peer buffer).
__device__ __forceinline__ void signal_peers(uint32_t* ctr, const PeerPtrs& peers, int nranks, int rank,
                                             size_t off_flag, uint32_t seq) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < nranks; ++d)
        st_release_sys(reinterpret_cast<uint32_t*>(peers.base[d] + off_flag) + rank, seq);
      *ctr = 0;   // ready for the next call (this kernel's CTAs are all past their increment)
    }
  }
}

__device__ __forceinline__ bool poisoned(const int* poison) {
  return *reinterpret_cast<const volatile int*>(poison) != 0;
}

// Token rows of the kept slots -> in_x[rank][pos] of their destination; all (peer, row) ids -> in_meta[rank][..].
__global__ void ep_dispatch_kernel(const uint4* __restrict__ x, int H16, const int32_t* __restrict__ slot_pos,
                                   int S, int k, const int32_t* __restrict__ send_meta, int nranks, int rank,
                                   int cap, PeerPtrs peers, size_t off_x, size_t off_meta, size_t off_flag,
                                   uint32_t* ctr, uint32_t seq, const int* poison) {
  if (poisoned(poison)) return;   // an earlier wait gave up: the peers' buffers are no longer in step
  const long long rows_work = (long long)S * H16;
  const long long total = rows_work + (long long)nranks * cap;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < rows_work) {
      const int s = (int)(i / H16), c = (int)(i % H16);
      const int pos = slot_pos[s];
      if (pos < 0) continue;
      const int d = pos / cap, row = pos % cap;
      uint4* dst = reinterpret_cast<uint4*>(peers.base[d] + off_x) + ((size_t)rank * cap + row) * H16;
      dst[c] = x[(size_t)(s / k) * H16 + c];
    } else {
      const int m = (int)(i - rows_work);
      const int d = m / cap, row = m % cap;
      reinterpret_cast<int32_t*>(peers.base[d] + off_meta)[(size_t)rank * cap + row] = send_meta[m];
    }
  }
  signal_peers(ctr, peers, nranks, rank, off_flag, seq);
}

// Outputs of the received rows (row r = source r / cap, position r % cap) -> in_y[rank][position] of the source.
// y_sorted rows are those of this rank's routing plan: row_slot[r] (one slot per received row).
template <typename T>
__global__ void ep_return_kernel(const T* __restrict__ y_sorted, const int32_t* __restrict__ row_slot,
                                 const int32_t* __restrict__ recv_meta, int R, int H, int cap, int nranks, int rank,
                                 PeerPtrs peers, size_t off_y, size_t off_flag, uint32_t* ctr, uint32_t seq,
                                 const int* poison) {
  if (poisoned(poison)) return;
  const int H16 = H * (int)sizeof(T) / 16;
  const size_t row_stride = (size_t)H * sizeof(T);   // packed [nranks][cap][H] rows of T
  const long long total = (long long)R * H16;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / H16), c = (int)(i % H16);
    if (recv_meta[r] < 0) continue;
    const int sr = row_slot[r];
    if (sr < 0) continue;
    const int src = r / cap, pos = r % cap;
    uint4* dst = reinterpret_cast<uint4*>(peers.base[src] + off_y + ((size_t)rank * cap + pos) * row_stride);
    dst[c] = reinterpret_cast<const uint4*>(y_sorted + (size_t)sr * H)[c];
  }
  signal_peers(ctr, peers, nranks, rank, off_flag, seq);
}

// One CTA: wait until every source's flag reached seq (bounded; on expiry CBMOE_DEVERR_TIMEOUT, the poison word
// is set and the kernel returns). A poisoned transport waits for nothing.
__global__ void ep_wait_kernel(const uint32_t* flags, int nranks, uint32_t seq, int* poison, int* poison_mirror) {
  const int t = threadIdx.x;
  if (t < nranks && !poisoned(poison)) {
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(flags + t) - seq) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(&g_device_errors, CBMOE_DEVERR_TIMEOUT);
        *reinterpret_cast<volatile int*>(poison) = 1;
        *reinterpret_cast<volatile int*>(poison_mirror) = 1;
        __threadfence_system();
        break;
      }
      if (poisoned(poison)) break;   // another waiter of this call gave up
      __nanosleep(64);
    }
  }
  __syncthreads();
}

int grid_for(long long work) {
  long long b = (work + 255) / 256;
  const long long cap = (long long)num_sms() * 4;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

size_t ep_peer_capacity(const EpPeer* pe) { return pe ? (size_t)pe->cap : 0; }

int ep_peer_dispatch_send(EpPeer* pe, const uint16_t* x, int H, const int32_t* slot_pos, int S, int k,
                          const int32_t* send_meta, cudaStream_t stream) {
  ++pe->seq;
  const int H16 = H / 8;
  uint32_t* ctr = reinterpret_cast<uint32_t*>(pe->own + pe->off_ctr);
  prof_begin(kProfExchange, stream);
  ep_dispatch_kernel<<<grid_for((long long)S * H16 + (long long)pe->nranks * pe->cap), 256, 0, stream>>>(
      reinterpret_cast<const uint4*>(x), H16, slot_pos, S, k, send_meta, pe->nranks, pe->rank, pe->cap, pe->peers,
      pe->off_x, pe->off_meta, pe->off_fx, ctr, pe->seq, pe->poison_dev);
  prof_add_launches(1);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

int ep_peer_dispatch_wait(EpPeer* pe, cudaStream_t stream) {
  ep_wait_kernel<<<1, 64, 0, stream>>>(reinterpret_cast<const uint32_t*>(pe->own + pe->off_fx), pe->nranks, pe->seq,
                                       pe->poison_dev, pe->poison_mirror);
  prof_end(kProfExchange, stream);
  prof_add_launches(1);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

int ep_peer_return(EpPeer* pe, const void* y_sorted, bool bf16, const int32_t* row_slot, const int32_t* recv_meta,
                   int R, int H, cudaStream_t stream) {
  uint32_t* ctr = reinterpret_cast<uint32_t*>(pe->own + pe->off_ctr) + 1;
  const long long work = (long long)R * H * (bf16 ? 2 : 4) / 16;
  prof_begin(kProfExchange, stream);
  if (bf16)
    ep_return_kernel<uint16_t><<<grid_for(work), 256, 0, stream>>>(
        static_cast<const uint16_t*>(y_sorted), row_slot, recv_meta, R, H, pe->cap, pe->nranks, pe->rank, pe->peers,
        pe->off_y, pe->off_fy, ctr, pe->seq, pe->poison_dev);
  else
    ep_return_kernel<float><<<grid_for(work), 256, 0, stream>>>(
        static_cast<const float*>(y_sorted), row_slot, recv_meta, R, H, pe->cap, pe->nranks, pe->rank, pe->peers,
        pe->off_y, pe->off_fy, ctr, pe->seq, pe->poison_dev);
  ep_wait_kernel<<<1, 64, 0, stream>>>(reinterpret_cast<const uint32_t*>(pe->own + pe->off_fy), pe->nranks, pe->seq,
                                       pe->poison_dev, pe->poison_mirror);
  prof_end(kProfExchange, stream);
  prof_add_launches(2);
  CBMOE_CUDA_TRY(cudaGetLastError());
  return CBMOE_OK;
}

uint16_t* ep_peer_in_x(EpPeer* pe) { return reinterpret_cast<uint16_t*>(pe->own + pe->off_x); }
int32_t* ep_peer_in_meta(EpPeer* pe) { return reinterpret_cast<int32_t*>(pe->own + pe->off_meta); }
void* ep_peer_in_y(EpPeer* pe) { return pe->own + pe->off_y; }
bool ep_peer_matches(const EpPeer* pe, int nranks, int rank, int H, int cap) {
  return pe && pe->nranks == nranks && pe->rank == rank && pe->H == H && cap == pe->cap;
}
bool ep_peer_poisoned(const EpPeer* pe) { return pe && pe->poison_host && *pe->poison_host != 0; }

}  // namespace cbmoe

using namespace cbmoe;

// What every rank contributes to the set-up all-gather: its (H, capacity, nranks) and its buffer's IPC handle.
// Every rank sees every record, so every rank reaches the same verdict on a mismatch.
struct PeerRecord {
  int32_t H, cap, nranks, magic;
  cudaIpcMemHandle_t handle;
};
constexpr int32_t kPeerMagic = 0x63626d65;   // "cbme"

extern "C" int cbmoe_ep_peer_init(void* comm_v, int nranks, int rank, int H, int capacity, cudaStream_t stream,
                                  void** peer_out) {
  if (!comm_v || !peer_out || nranks < 1 || nranks > kPeerMax || rank < 0 || rank >= nranks || H <= 0 || H % 8 ||
      capacity <= 0)
    return CBMOE_ERR_INVALID;
  *peer_out = nullptr;
  ncclComm_t comm = static_cast<ncclComm_t>(comm_v);
  EpPeer* pe = new EpPeer();
  pe->nranks = nranks;
  pe->rank = rank;
  pe->cap = capacity;
  pe->H = H;
  const size_t rows = (size_t)nranks * capacity;
  pe->off_x = 0;
  pe->off_meta = lyr::align_up(rows * H * 2);
  pe->off_y = pe->off_meta + lyr::align_up(rows * 4);
  pe->off_fx = pe->off_y + lyr::align_up(rows * H * 4);
  pe->off_fy = pe->off_fx + 256;
  pe->off_ctr = pe->off_fy + 256;
  pe->off_poison = pe->off_ctr + 256;
  pe->bytes = pe->off_poison + 256;
  int rc = CBMOE_OK;
  uint8_t* records_dev = nullptr;
  std::vector<PeerRecord> records(nranks);
  PeerRecord mine{};
  mine.H = H;
  mine.cap = capacity;
  mine.nranks = nranks;
  mine.magic = kPeerMagic;
  void* poison = nullptr;
  if (cudaMalloc(&pe->own, pe->bytes) != cudaSuccess || cudaMemset(pe->own, 0, pe->bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(&mine.handle, pe->own) != cudaSuccess ||
      cudaHostAlloc(&poison, sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
      cudaMalloc(&records_dev, records.size() * sizeof(PeerRecord)) != cudaSuccess ||
      cudaMemcpy(records_dev + (size_t)rank * sizeof(PeerRecord), &mine, sizeof(mine), cudaMemcpyHostToDevice) !=
          cudaSuccess) {
    rc = CBMOE_ERR_CUDA;
  }
  if (poison) {
    pe->poison_host = static_cast<volatile int*>(poison);
    *pe->poison_host = 0;
    if (!rc && cudaHostGetDevicePointer(reinterpret_cast<void**>(&pe->poison_mirror), poison, 0) != cudaSuccess)
      rc = CBMOE_ERR_CUDA;
  }
  if (pe->own) pe->poison_dev = reinterpret_cast<int*>(pe->own + pe->off_poison);   // zeroed with the buffer
  // Every rank takes part in the all-gather even when its own set-up failed (the others would wait for it); a
  // failed rank contributes a zeroed record, which the others reject as a mismatch.
  if (records_dev && ncclAllGather(records_dev + (size_t)rank * sizeof(PeerRecord), records_dev,
                                   sizeof(PeerRecord), ncclUint8, comm, stream) != ncclSuccess)
    rc = rc ? rc : CBMOE_ERR_NCCL;
  if (records_dev && (cudaStreamSynchronize(stream) != cudaSuccess ||
                      cudaMemcpy(records.data(), records_dev, records.size() * sizeof(PeerRecord),
                                 cudaMemcpyDeviceToHost) != cudaSuccess))
    rc = rc ? rc : CBMOE_ERR_CUDA;
  // Equal (H, capacity) on every rank: a sender computes its peers' row addresses from its own capacity.
  for (int d = 0; d < nranks && !rc; ++d)
    if (records[d].magic != kPeerMagic || records[d].H != H || records[d].cap != capacity ||
        records[d].nranks != nranks)
      rc = CBMOE_ERR_INVALID;
  for (int d = 0; d < nranks && !rc; ++d) {
    if (d == rank) {
      pe->peers.base[d] = pe->own;
      continue;
    }
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, records[d].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) rc = CBMOE_ERR_CUDA;
    pe->peers.base[d] = static_cast<uint8_t*>(p);
  }
  if (records_dev) cudaFree(records_dev);
  if (rc) {
    for (int d = 0; d < nranks; ++d)
      if (d != rank && pe->peers.base[d]) cudaIpcCloseMemHandle(pe->peers.base[d]);
    if (pe->own) cudaFree(pe->own);
    if (poison) cudaFreeHost(poison);
    delete pe;
    return rc;
  }
  *peer_out = pe;
  return CBMOE_OK;
}

extern "C" int cbmoe_ep_peer_destroy(void* peer_v) {
  EpPeer* pe = static_cast<EpPeer*>(peer_v);
  if (!pe) return CBMOE_ERR_INVALID;
  int rc = CBMOE_OK;
  for (int d = 0; d < pe->nranks; ++d)
    if (d != pe->rank && pe->peers.base[d] && cudaIpcCloseMemHandle(pe->peers.base[d]) != cudaSuccess)
      rc = CBMOE_ERR_CUDA;
  if (pe->own && cudaFree(pe->own) != cudaSuccess) rc = CBMOE_ERR_CUDA;
  if (pe->poison_host && cudaFreeHost(const_cast<int*>(pe->poison_host)) != cudaSuccess) rc = CBMOE_ERR_CUDA;
  delete pe;
  return rc;
}
