// Expert parallelism over the GPUs of one node: the routed experts are sharded by expert id (rank r holds experts
// [r*E/n, (r+1)*E/n)), every rank keeps its own tokens and a replica of the shared expert, and one layer call is
//   1. route   (one CTA) each (token, slot) gets its destination rank and a stable position among that rank's
//              slots; slots beyond `capacity` per peer are dropped and flagged (CBMOE_DEVERR_CAPACITY)
//   2. pack    the token rows into a per-peer send buffer (capacity rows per peer) + local expert ids
//   3. NCCL    send/recv of rows and ids with every peer (grouped, on the caller's stream, over NVLink)
//   4. compute the local experts on the received rows (each row = one slot, weight 1): the decode or grouped path
//   5. NCCL    the fp32 expert outputs go back to their source ranks
//   6. combine shared-expert down + sum_j w[t, j] * returned row (the decode COMBINE epilogue), bf16 out
// The shared expert's gate/up runs on a side stream while steps 1-5 run. The reference has no expert parallelism
// (it shards moe_inter over chips and psums, engine.py:129-176, model.py:855); the layer output is defined to be
// the single-GPU layer's output (model.py:840-856).
#include <mutex>
#include <nccl.h>

#include "layer.cuh"
#include "profile.cuh"

namespace cbmoe {
namespace {

constexpr int kEpThreads = 1024;

// One CTA: destination rank and stable per-destination position of every slot.
__global__ void __launch_bounds__(kEpThreads) ep_route_kernel(const int32_t* __restrict__ idx, int S, int E_total,
                                                              int E_loc, int nranks, int cap,
                                                              int32_t* __restrict__ send_meta,
                                                              int32_t* __restrict__ slot_pos, float* __restrict__ ones,
                                                              int R) {
  __shared__ int run[64];   // per-destination running count (nranks <= 64)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int i = threadIdx.x; i < nranks * cap; i += blockDim.x) send_meta[i] = -1;
  for (int i = threadIdx.x; i < R; i += blockDim.x) ones[i] = 1.f;
  if (threadIdx.x < 64) run[threadIdx.x] = 0;
  __syncthreads();
  __shared__ int wcnt[32][64];   // per warp and destination: slots of this chunk
  const unsigned lt = (1u << lane) - 1u;
  for (int base = 0; base < S; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int e = (s < S) ? idx[s] : -1;
    if (s < S && e >= E_total) {
      atomicOr(&g_device_errors, CBMOE_DEVERR_INDEX);
      e = -1;
    }
    const int d = e >= 0 ? e / E_loc : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int rank_in_warp = __popc(peers & lt);
    for (int i = threadIdx.x; i < 32 * 64; i += blockDim.x) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    if (d >= 0 && lane == __ffs(peers) - 1) wcnt[warp][d] = __popc(peers);
    __syncthreads();
    if (s < S) {
      int pos = -1;
      if (d >= 0) {
        int before = run[d];
        for (int w2 = 0; w2 < warp; ++w2) before += wcnt[w2][d];
        pos = before + rank_in_warp;
        if (pos < cap) {
          send_meta[d * cap + pos] = e - d * E_loc;
          pos = d * cap + pos;
        } else {
          atomicOr(&g_device_errors, CBMOE_DEVERR_CAPACITY);
          pos = -1;
        }
      }
      slot_pos[s] = pos;
    }
    __syncthreads();
    if (threadIdx.x < nranks) {
      int add = 0;
      for (int w2 = 0; w2 < nwarps; ++w2) add += wcnt[w2][threadIdx.x];
      run[threadIdx.x] += add;
    }
    __syncthreads();
  }
}

// send_x[slot_pos[s]] = x[s / k] for every kept slot (16-byte copies).
__global__ void ep_pack_kernel(const uint4* __restrict__ x, int H16, const int32_t* __restrict__ slot_pos, int S,
                               int k, uint4* __restrict__ send_x) {
  const long long total = (long long)S * H16;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int s = (int)(i / H16), c = (int)(i % H16);
    const int pos = slot_pos[s];
    if (pos >= 0) send_x[(size_t)pos * H16 + c] = x[(size_t)(s / k) * H16 + c];
  }
}

struct EpWorkspace {
  size_t send_x, recv_x, send_meta, recv_meta, slot_pos, ones, y_recv, y_back, sub_local, sub_recv, total;
  int R;
  lyr::DecodeWorkspace Wl;     // local tokens: shared-expert regions
  int recv_path;
  lyr::DecodeWorkspace Wr;     // received rows, decode path
  lyr::GroupedWorkspace Gr;    // received rows, grouped path
};

EpWorkspace ep_workspace(int E_loc, int H, int I, int N_local, int k, int nranks, int cap, int path, int cb8) {
  using lyr::align_up;
  EpWorkspace w;
  w.R = nranks * cap;
  w.send_x = 0;
  w.recv_x = w.send_x + align_up((size_t)w.R * H * 2);
  w.send_meta = w.recv_x + align_up((size_t)w.R * H * 2);
  w.recv_meta = w.send_meta + align_up((size_t)w.R * 4);
  w.slot_pos = w.recv_meta + align_up((size_t)w.R * 4);
  w.ones = w.slot_pos + align_up((size_t)N_local * k * 4);
  w.y_recv = w.ones + align_up((size_t)w.R * 4);
  w.y_back = w.y_recv + align_up((size_t)w.R * H * 4);
  w.sub_local = w.y_back + align_up((size_t)w.R * H * 4);
  // shared-expert regions only; with CB8 tables a one-pass batch (<= 8 local tokens) gets the int8-MMA shared
  // expert, as on one GPU
  w.Wl = lyr::decode_workspace(E_loc, H, I, N_local, k, -1, cb8);
  w.sub_recv = w.sub_local + align_up(w.Wl.total);
  // The receive buffer holds up to R rows, but a rank expects about its own slot count (N_local * k) of real
  // ones: AUTO chooses the kernels by that. From 8 rows per local expert on, the tensor-core GEMMs, except where
  // the rank holds 32 or more experts with at most 16 rows each: there the decode kernels (the bf16 ones at that
  // load: 16-token passes) are faster (measured on one B200 at 12.8 rows per expert, routed part: 40 experts 253 us
  // decode vs 279 us grouped, 80 experts 436 vs 489 us; 20 experts 167 vs 159 us).
  const long long expect = (long long)N_local * k;
  const bool grouped_ok = H % kGrpTileM == 0 && I % kGrpTileM == 0;
  if (path == CBMOE_PATH_GROUPED && grouped_ok) {
    w.recv_path = CBMOE_PATH_GROUPED;
  } else if (path == CBMOE_PATH_DECODE || !grouped_ok) {
    w.recv_path = CBMOE_PATH_DECODE;
  } else {
    const bool decode_wide = E_loc >= 32 && expect <= 16LL * E_loc;
    w.recv_path = (expect >= 8LL * E_loc && !decode_wide) ? CBMOE_PATH_GROUPED : CBMOE_PATH_DECODE;
  }
  size_t rb = 0;
  if (w.recv_path == CBMOE_PATH_GROUPED) {
    w.Gr = lyr::grouped_workspace(E_loc, H, I, w.R, 1);
    rb = w.Gr.total;
  } else {
    w.Wr = lyr::decode_workspace(E_loc, H, I, w.R, 1, expect, cb8);
    rb = w.Wr.total;
  }
  w.total = w.sub_recv + align_up(rb);
  return w;
}

int nccl_rc(ncclResult_t r) { return r == ncclSuccess ? CBMOE_OK : CBMOE_ERR_NCCL; }

// rows[p*cap .. (p+1)*cap) go to peer p; recv[p*cap ..) come from peer p. Self traffic is a device copy.
int exchange(ncclComm_t comm, int nranks, int rank, const void* send, void* recv, size_t count_per_peer,
             ncclDataType_t type, size_t elem_bytes, cudaStream_t stream) {
  const size_t bytes = count_per_peer * elem_bytes;
  if (ncclGroupStart() != ncclSuccess) return CBMOE_ERR_NCCL;
  for (int p = 0; p < nranks; ++p) {
    if (p == rank) continue;
    int rc = nccl_rc(ncclSend(static_cast<const uint8_t*>(send) + p * bytes, count_per_peer, type, p, comm, stream));
    if (!rc) rc = nccl_rc(ncclRecv(static_cast<uint8_t*>(recv) + p * bytes, count_per_peer, type, p, comm, stream));
    if (rc) {
      ncclGroupEnd();
      return rc;
    }
  }
  if (ncclGroupEnd() != ncclSuccess) return CBMOE_ERR_NCCL;
  CBMOE_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(recv) + rank * bytes,
                                 static_cast<const uint8_t*>(send) + rank * bytes, bytes, cudaMemcpyDeviceToDevice,
                                 stream));
  return CBMOE_OK;
}

bool ep_args_ok(void* comm, int nranks, int rank, const cbmoe_experts* local, int E_total, int N_local, int k,
                int cap) {
  return comm && nranks >= 1 && nranks <= 64 && rank >= 0 && rank < nranks && lyr::experts_ok(local) &&
         E_total == local->E * nranks && N_local >= 0 && k > 0 && k <= 64 && cap > 0;
}

}  // namespace
}  // namespace cbmoe

using namespace cbmoe;

extern "C" int cbmoe_ep_unique_id(uint8_t* id128_host) {
  if (!id128_host) return CBMOE_ERR_INVALID;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return CBMOE_ERR_NCCL;
  static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
  memcpy(id128_host, &id, 128);
  return CBMOE_OK;
}

extern "C" int cbmoe_ep_comm_init(const uint8_t* id128_host, int nranks, int rank, void** comm_out) {
  if (!id128_host || !comm_out || nranks < 1 || rank < 0 || rank >= nranks) return CBMOE_ERR_INVALID;
  ncclUniqueId id;
  memcpy(&id, id128_host, 128);
  ncclComm_t comm = nullptr;
  if (ncclCommInitRank(&comm, nranks, id, rank) != ncclSuccess) return CBMOE_ERR_NCCL;
  *comm_out = comm;
  return CBMOE_OK;
}

extern "C" int cbmoe_ep_comm_destroy(void* comm) {
  if (!comm) return CBMOE_ERR_INVALID;
  return ncclCommDestroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? CBMOE_OK : CBMOE_ERR_NCCL;
}

extern "C" size_t cbmoe_ep_workspace_bytes(const cbmoe_experts* local, int N_local, int k, int nranks, int capacity,
                                           int path) {
  if (!local || local->E <= 0 || N_local < 0 || k <= 0 || nranks < 1 || capacity <= 0) return 0;
  if (path != CBMOE_PATH_AUTO && path != CBMOE_PATH_DECODE && path != CBMOE_PATH_GROUPED) return 0;
  return ep_workspace(local->E, local->H, local->I, N_local, k, nranks, capacity, path, lyr::has_cb8(local)).total;
}

extern "C" int cbmoe_ep_layer(void* comm_v, int nranks, int rank, const cbmoe_experts* local, int E_total,
                              const cbmoe_shared* sh, const uint16_t* x, int N_local, const int32_t* idx,
                              const float* w, int k, float limit, int capacity, int path, void* peer_v,
                              uint16_t* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!ep_args_ok(comm_v, nranks, rank, local, E_total, N_local, k, capacity) || !lyr::shared_ok(sh))
    return CBMOE_ERR_INVALID;
  if (path != CBMOE_PATH_AUTO && path != CBMOE_PATH_DECODE && path != CBMOE_PATH_GROUPED) return CBMOE_ERR_INVALID;
  if (N_local > 0 && (!x || !idx || !w || !out || !lyr::aligned16(x) || !lyr::aligned16(out)))
    return CBMOE_ERR_INVALID;
  ncclComm_t comm = static_cast<ncclComm_t>(comm_v);
  const int E_loc = local->E, H = local->H, I = local->I;
  EpPeer* pe = static_cast<EpPeer*>(peer_v);
  if (pe && !ep_peer_matches(pe, nranks, rank, H, capacity)) return CBMOE_ERR_INVALID;
  if (ep_peer_poisoned(pe)) return CBMOE_ERR_DEVICE;   // a wait of an earlier call gave up
  const EpWorkspace W = ep_workspace(E_loc, H, I, N_local, k, nranks, capacity, path, lyr::has_cb8(local));
  if (!workspace || workspace_bytes < W.total) return CBMOE_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* send_x = reinterpret_cast<uint16_t*>(ws + W.send_x);
  uint16_t* recv_x = pe ? ep_peer_in_x(pe) : reinterpret_cast<uint16_t*>(ws + W.recv_x);
  int32_t* send_meta = reinterpret_cast<int32_t*>(ws + W.send_meta);
  int32_t* recv_meta = pe ? ep_peer_in_meta(pe) : reinterpret_cast<int32_t*>(ws + W.recv_meta);
  int32_t* slot_pos = reinterpret_cast<int32_t*>(ws + W.slot_pos);
  float* ones = reinterpret_cast<float*>(ws + W.ones);
  float* y_recv = reinterpret_cast<float*>(ws + W.y_recv);
  float* y_back = pe ? static_cast<float*>(ep_peer_in_y(pe)) : reinterpret_cast<float*>(ws + W.y_back);
  uint8_t* wl = ws + W.sub_local;
  uint8_t* wr = ws + W.sub_recv;
  const int S = N_local * k;
  int rc = CBMOE_OK;

  // shared expert of the local tokens on the side stream (gate/up, down -> ys), beside the dispatch and the local
  // experts; joined before the final combine. (Measured: joining it before the local experts, with the decode
  // kernels on the whole GPU, is slower at 32-64 tokens per rank: those kernels outlast the dispatch; forking it
  // after this rank's rows are sent, on the whole GPU, slowed the routed kernels that follow the wait: config 4 at
  // 2 / 4 / 8 GPUs 128k / 173k / 205k tok/s against 135k / 200k / 209k with the 48-CTA side stream; running it on
  // this stream between the send and the wait, on the whole GPU, measured slower again: config 4 at 2 / 8 GPUs
  // 109k / 184k, the weak-scaling line 68k / 276k against 80k / 319k: its decode kernels outlast the wait.)
  lyr::SideStream* side = nullptr;
  rc = lyr::side_stream(&side);
  if (rc) return rc;
  if (N_local > 0) {
    rc = lyr::shared_side(sh, x, N_local, H, I, limit, wl, W.Wl, side, stream);
    if (rc) return rc;
  }

  // 1-2. route + pack
  prof_begin(kProfOther, stream);
  ep_route_kernel<<<1, kEpThreads, 0, stream>>>(idx, S, E_total, E_loc, nranks, capacity, send_meta, slot_pos, ones,
                                                W.R);
  prof_end(kProfOther, stream);
  CBMOE_CUDA_TRY(cudaGetLastError());
  if (pe) {   // 2-3. rows straight into the destinations' memory
    rc = ep_peer_dispatch_send(pe, x, H, slot_pos, S, k, send_meta, stream);
    if (!rc) rc = ep_peer_dispatch_wait(pe, stream);
    if (rc) goto join;
  }
  if (S > 0 && !pe) {
    prof_begin(kProfOther, stream);
    const long long total = (long long)S * (H / 8);
    int blocks = (int)((total + 255) / 256);
    if (blocks > num_sms() * 8) blocks = num_sms() * 8;
    ep_pack_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(x), H / 8, slot_pos, S, k,
                                               reinterpret_cast<uint4*>(send_x));
    prof_end(kProfOther, stream);
    CBMOE_CUDA_TRY(cudaGetLastError());
  }
  // 3. dispatch
  if (!pe) {
    prof_begin(kProfExchange, stream);
    rc = exchange(comm, nranks, rank, send_x, recv_x, (size_t)capacity * H, ncclBfloat16, 2, stream);
    if (!rc) rc = exchange(comm, nranks, rank, send_meta, recv_meta, (size_t)capacity, ncclInt32, 4, stream);
    prof_end(kProfExchange, stream);
  }
  if (rc) goto join;
  // 4. local experts on the received rows (one slot per row, weight 1); the grouped kernels' slot outputs are
  // bf16, and go back as bf16
  if (W.recv_path == CBMOE_PATH_GROUPED) {
    rc = lyr::routed_grouped(local, recv_x, W.R, recv_meta, ones, 1, limit, wr, W.Gr, stream);
    if (!rc) {
      const int32_t* plan = reinterpret_cast<const int32_t*>(wr + W.Gr.plan);
      if (pe)   // 4-5. outputs straight into the sources' memory
        rc = ep_peer_return(pe, wr + W.Gr.y, true, plan + W.Gr.L.off[9], recv_meta, W.R, H, stream);
      else
        rc = launch_combine_bf16(reinterpret_cast<const uint16_t*>(wr + W.Gr.y), plan + W.Gr.L.off[9], ones, W.R, 1,
                                 H, nullptr, nullptr, reinterpret_cast<uint16_t*>(y_recv), stream);
    }
  } else {
    rc = lyr::routed_decode(local, recv_x, W.R, recv_meta, ones, 1, limit, wr, W.Wr, stream);
    if (!rc) {
      const int32_t* plan = reinterpret_cast<const int32_t*>(wr + W.Wr.plan);
      if (pe)
        rc = ep_peer_return(pe, wr + W.Wr.y, false, plan + W.Wr.L.off[9], recv_meta, W.R, H, stream);
      else
        rc = launch_combine(reinterpret_cast<const float*>(wr + W.Wr.y), plan + W.Wr.L.off[9], ones, W.R, 1, H,
                            nullptr, y_recv, nullptr, stream);
    }
  }
  if (rc || pe) goto join;
  // 5. return the expert outputs
  prof_begin(kProfExchange, stream);
  if (W.recv_path == CBMOE_PATH_GROUPED)
    rc = exchange(comm, nranks, rank, y_recv, y_back, (size_t)capacity * H, ncclBfloat16, 2, stream);
  else
    rc = exchange(comm, nranks, rank, y_recv, y_back, (size_t)capacity * H, ncclFloat32, 4, stream);
  prof_end(kProfExchange, stream);
join:
  if (N_local > 0) CBMOE_CUDA_TRY(cudaStreamWaitEvent(stream, side->join, 0));
  if (rc || N_local == 0) return rc;
  // 6. weighted sum of the returned rows + the shared expert
  const float* ys = reinterpret_cast<const float*>(wl + W.Wl.ys);
  if (W.recv_path == CBMOE_PATH_GROUPED)
    return launch_combine_bf16(reinterpret_cast<const uint16_t*>(y_back), slot_pos, w, N_local, k, H, nullptr, nullptr,
                               out, stream, ys);
  return launch_combine(y_back, slot_pos, w, N_local, k, H, ys, nullptr, out, stream);
}
