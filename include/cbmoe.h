/* cbmoe: B200 (sm_100a) kernels for the codebook-quantized MoE expert path of the GLM engine in
 * shallmall/kaggle-llm-endpoint. C ABI: plain pointers and sizes, no C++ or torch types.
 *
 * Conventions for every entry point:
 *   - returns CBMOE_OK (0) or a negative CBMOE_ERR_* status; never throws, never aborts;
 *   - pointer arguments are DEVICE pointers unless the name ends in _host;
 *   - work is enqueued on `stream` (stream-ordered, asynchronous); nothing synchronizes unless documented;
 *   - tables and buffers are owned by the caller; no compute path allocates device memory (the set-up calls
 *     cbmoe_ep_comm_init and cbmoe_ep_peer_init do, and cbmoe_ep_peer_destroy frees what the latter took);
 *   - bf16 tensors are passed as uint16_t bit patterns;
 *   - kernels never trap: a device-side problem (a wait that ran out, an expert id out of range) sets a bit
 *     that cbmoe_device_errors() reports.
 * Reference paths below are relative to launcher/glm53-flash/engine/glm53/ in the reference repository.
 */
#ifndef CBMOE_H
#define CBMOE_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CBMOE_OK 0
#define CBMOE_ERR_INVALID (-1)     /* bad argument: shape, alignment, null pointer */
#define CBMOE_ERR_CUDA (-2)        /* a CUDA call failed: see cbmoe_last_cuda_error() */
#define CBMOE_ERR_WORKSPACE (-3)   /* workspace smaller than the *_workspace_bytes() query */
#define CBMOE_ERR_UNSUPPORTED (-4) /* valid request this build does not implement */
#define CBMOE_ERR_NCCL (-5)        /* an NCCL call failed */
#define CBMOE_ERR_DEVICE (-6)      /* a kernel recorded a device-side error (cbmoe_device_errors) */

#define CBMOE_DEVERR_TIMEOUT 1     /* a bounded spin-wait gave up */
#define CBMOE_DEVERR_INDEX 2       /* an expert id >= E was routed (the slot is skipped); ids < 0 are empty slots */
#define CBMOE_DEVERR_CAPACITY 4    /* expert parallel: more slots for one peer than the capacity (extra dropped) */

#define CBMOE_PATH_AUTO 0          /* decode kernel for small batches, grouped tensor-core GEMM otherwise */
#define CBMOE_PATH_DECODE 1        /* fused dequant matvec (resident.py:110-120 `_apply_kernel`) */
#define CBMOE_PATH_GROUPED 2       /* grouped dequant GEMM (resident.py:144-165 `_apply_ragged_kernel`) */

/* ---------------------------------------------------------------------------------------------- library */
int cbmoe_version(void);
const char* cbmoe_status_string(int status);
/* The cudaError_t of the last CBMOE_ERR_CUDA returned on this thread. */
int cbmoe_last_cuda_error(void);
/* Synchronizes the device, writes the OR of device error bits to *out_host, and clears them when clear != 0. */
int cbmoe_device_errors(int clear, int* out_host);
/* SM count of the current device (what the persistent kernels size their grids by). */
int cbmoe_num_sms(void);
/* Kernels this library has launched in this process (host-side counter). */
long long cbmoe_launch_count(void);
/* No counterpart in the reference. Self-test of the kernels' bounded waits: one CTA waits on a barrier phase that
 * nothing completes, gives up after limit_ns (0 < limit_ns <= 10 s), records CBMOE_DEVERR_TIMEOUT in
 * cbmoe_device_errors and writes 1 to *gave_up_device (device int). The context stays usable afterwards. */
int cbmoe_selftest_wait_timeout(long long limit_ns, int* gave_up_device, cudaStream_t stream);
/* Per-kernel CUDA-event timing: when enabled, every launch is bracketed by two events on its stream.
 * cbmoe_profile_read synchronizes on the recorded events and writes, per kernel kind (n_kinds >= 16 slots:
 * 0 plan, 1 CB3 gate/up, 2 CB3 down, 3 CB3 single, 4 int8 gate/up, 5 int8 down, 6 int8 single, 7 combine,
 * 8 other, 9-12 grouped CB3 gate/up, CB3 down, int8 gate/up, int8 store, 13 expert-parallel exchange), the
 * summed milliseconds and launch counts; reset != 0 clears them. */
int cbmoe_profile_enable(int enable);
int cbmoe_profile_read(int reset, double* ms_host, long long* count_host, int n_kinds);

/* ------------------------------------------------------------------------------------ CB3 kernel layout
 * CB3 (benchmark format): per matrix W [rows, K], 3-bit indices packed little-endian into uint32 (index j at
 * bits 3j..3j+2 of the row's bit stream, K*3/32 words per row) and one 8-entry bf16 codebook per row.
 * The kernels read a load-time repack of it, "CB3K": the same 3 bits per weight and 16 bytes of codebook per
 * row, reordered so that each lane of a decode warp reads its tensor-core fragment bits with 16-byte loads and
 * every 256-input stage of a 64-row block is one contiguous bulk copy. nmat = 2 interleaves gate and up so one
 * stage carries both. Requirements: rows % 64 == 0, K % 256 == 0.
 * Replaces the load-time planar repack pack_chip_planes / planes.pack_planes (resident.py:48-60,
 * planes.py:136-170). */
size_t cbmoe_cb3k_idx_bytes(int E, int rows, int K, int nmat);
size_t cbmoe_cb3k_cb_bytes(int E, int rows, int nmat);
/* idx0/cb0 = matrix 0 (gate or the only matrix), idx1/cb1 = matrix 1 (up; NULL when nmat == 1):
 * idx [E, rows, K*3/32] uint32, cb [E, rows, 8] bf16. Output idx_k / cb_k sized by the two queries. */
int cbmoe_cb3k_repack(const uint32_t* idx0, const uint16_t* cb0, const uint32_t* idx1, const uint16_t* cb1,
                      int nmat, int E, int rows, int K, void* idx_k, void* cb_k, cudaStream_t stream);
/* Dequantize a CB3K table with the kernels' own register dequant -> bf16 [nmat, E, rows, K]
 * (planes.dequant_planes, planes.py:196-291: the bit-exactness check of layout + dequant). */
int cbmoe_cb3k_dequant(const void* idx_k, const void* cb_k, int nmat, int E, int rows, int K, uint16_t* out,
                       cudaStream_t stream);
/* CB8: the decode kernels' form of the CB3K codebooks (same index bits), built at load time alongside them
 * (part of the same load-time repack, resident.py:48-60). Per row, the 8 entries as 16-bit fixed point
 * T = rint(v 2^s) (the largest magnitude times 2^s in [2^14, 2^15)) in two byte tables, hi = T >> 8 (int8) and
 * lo = T & 255 (uint8), and the factor 2^-s: 20 bytes per row, laid out per (expert, 64-row block) as the CB3K
 * codebooks are. T is exact for entries within 2^7 of the row's largest magnitude and within 2^-15 of that
 * largest magnitude below it. With these tables the decode path multiplies int8 digits on the tensor cores with
 * exact int32 sums (activations as two base-256 digits per element with one factor per token, exact for bf16
 * within 2^6 of the token's largest; the SwiGLU output as four, with one factor per 64 inputs), which halves the
 * table lookups per weight of the bf16 kernels. cb_k: a CB3K codebook table. */
size_t cbmoe_cb8_bytes(int E, int rows, int nmat);
int cbmoe_cb8_build(const void* cb_k, int nmat, int E, int rows, void* cb8, cudaStream_t stream);

/* ----------------------------------------------------------------------------------- int8 kernel layout
 * int8 weight-only leaves as quant8.quantize_array makes them (quant8.py:26-32): q int8 [K_in, rows_out]
 * ("[in, out]"), scales fp32 per output column (scale_axis 1, [rows_out]) or per input row (scale_axis 0,
 * [K_in]). "W8K" is the same bytes transposed to output-row-major fragment order; nmat = 2 interleaves gate and
 * up. Requirements: rows % 64 == 0, K % 256 == 0. */
size_t cbmoe_w8k_bytes(int rows, int K, int nmat);
int cbmoe_w8k_repack(const int8_t* q0, const int8_t* q1, int nmat, int K, int rows, void* qk, cudaStream_t stream);
/* bf16(f32(q) * s) -> bf16 [nmat, rows, K] (quant8.dequant_tree, quant8.py:91-99), for the bit-exactness check. */
int cbmoe_w8k_dequant(const void* qk, const float* s0, const float* s1, int scale_axis, int nmat, int rows, int K,
                      uint16_t* out, cudaStream_t stream);

/* --------------------------------------------------------------------------------------- routing plan
 * pallas_moe.ragged_plan (pallas_moe.py:564-592) on the device: the T*k (token, slot) pairs sorted by expert
 * (stable) into tm-row blocks, plus the lists the decode kernels walk. All int32 except w_row (fp32).
 * Layout of the plan buffer, offsets in 4-byte words from cbmoe_plan_layout (index: field):
 *   0 counts[E]  1 row_start[E] (first sorted row of each expert)  2 act[E] (active experts, ascending)
 *   3 n_act[1]  4 n_blocks[1]  5 n_pass[1]  6 blk_expert[G]  7 tok_row[Rp] (-1 = padding)  8 w_row[Rp]
 *   9 row_slot[T*k]  10 pass_expert[P]  11 pass_row0[P]  12 pass_cnt[P]  13 total words
 * G = ceil(T*k/tm) + E, Rp = G*tm, P = ceil(T*k/pass_tokens) + E. A "pass" is up to pass_tokens consecutive
 * sorted rows of one expert: the decode kernels stream an expert's weights once per pass. */
int cbmoe_plan_layout(int T, int k, int E, int tm, int pass_tokens, int64_t* offsets14_host);
int cbmoe_route_plan(const int32_t* idx, const float* w, int T, int k, int E, int tm, int pass_tokens, void* plan,
                     size_t plan_bytes, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------ the layer */
typedef struct cbmoe_experts {
  int E, H, I;                 /* routed experts, hidden size, expert intermediate size */
  const void* gateup_idx;      /* CB3K nmat = 2 (gate, up), rows = I, K = H */
  const void* gateup_cb;
  const void* down_idx;        /* CB3K nmat = 1, rows = H, K = I */
  const void* down_cb;
  const void* gateup_cb8;      /* CB8 tables of gateup_cb / down_cb (cbmoe_cb8_build), both or neither: with them */
  const void* down_cb8;        /* the decode path runs the int8-digit kernels, without them the bf16 ones */
} cbmoe_experts;

typedef struct cbmoe_shared {
  const void* gateup_q;        /* W8K nmat = 2 (gate, up), rows = I, K = H */
  const float* gate_s;
  const float* up_s;
  const void* down_q;          /* W8K nmat = 1, rows = H, K = I */
  const float* down_s;
  int scale_axis;              /* 1: per output channel (benchmark configs), 0: per input row */
} cbmoe_shared;

/* Workspace bytes for cbmoe_experts_apply / cbmoe_moe_layer with N tokens and top-k routing. */
size_t cbmoe_workspace_bytes(const cbmoe_experts* ex, int N, int k, int path);

/* ResidentFetch.apply (resident.py:100-108): x bf16 [N, H], idx int32 [N, k] in [0, E) (negative = empty slot),
 * w fp32 [N, k] ->
 * y fp32 [N, H] = sum_j w[n, j] * down_e(swiglu_clamped(gate_e x_n, up_e x_n, limit)), e = idx[n, j]. */
int cbmoe_experts_apply(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w,
                        int k, float limit, int path, float* y, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream);

/* No counterpart in the reference. cbmoe_experts_apply for callers that cannot allocate device memory (an
 * engine whose allocator owns all device memory and passes only its own buffers, a plugin host that forbids
 * allocation inside execute, host code that must not block on cudaMalloc). Same inputs and output as
 * cbmoe_experts_apply on the decode path, but no workspace argument: scratch lives in a fixed device array of
 * CBMOE_NOALLOC_SCRATCH_BYTES inside the library, held on every GPU that loads the library until exit. Returns
 * CBMOE_ERR_WORKSPACE when the request needs more scratch than that (e.g. 160 experts, hidden 5120,
 * intermediate 1536, top-8: up to 64 tokens fit). The first call on a device looks up the array's device address
 * (make it before any stream capture). All calls on a device share the array: calls that overlap on the GPU race.
 * Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
#define CBMOE_NOALLOC_SCRATCH_BYTES (48u << 20)
int cbmoe_experts_apply_noalloc(const cbmoe_experts* ex, const uint16_t* x, int N, const int32_t* idx,
                                const float* w, int k, float limit, float* y, cudaStream_t stream);

/* moe_dense below the router (model.py:840-856): routed experts + int8 shared expert (model.py:125-127),
 * out bf16 [N, H]. */
int cbmoe_moe_layer(const cbmoe_experts* ex, const cbmoe_shared* sh, const uint16_t* x, int N, const int32_t* idx,
                    const float* w, int k, float limit, int path, uint16_t* out, void* workspace,
                    size_t workspace_bytes, cudaStream_t stream);

/* One CB3K matrix times N activation rows (pallas_moe.moe_matvec with every slot on expert 0,
 * pallas_moe.py:238-307): x bf16 [N, K] -> y fp32 [N, rows]. Workspace: cbmoe_matvec_workspace_bytes. */
size_t cbmoe_matvec_workspace_bytes(int N);
int cbmoe_cb3_matvec(const void* idx_k, const void* cb_k, int rows, int K, const uint16_t* x, int N, float* y,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* cbmoe_cb3_matvec on CB8 tables (cbmoe_cb8_build): the same product through the int8-digit decode kernel. The
 * workspace (cbmoe_cb8_matvec_workspace_bytes, 16-byte aligned) holds the split activations. K <= 65536. */
size_t cbmoe_cb8_matvec_workspace_bytes(int N, int K);
int cbmoe_cb8_matvec(const void* idx_k, const void* cb8, int rows, int K, const uint16_t* x, int N, float* y,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* int8 weight-only linear (quant8.dequant_tree + the consuming dot, quant8.py:91-99): x bf16 [N, K] ->
 * y fp32 [N, rows] = x @ bf16(q * s). Workspace: cbmoe_matvec_workspace_bytes. */
int cbmoe_w8_linear(const void* qk, const float* s, int scale_axis, int rows, int K, const uint16_t* x, int N,
                    float* y, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* The int8 lm_head (engine.py:345-351 `_logits_local` with int8 columns): logits bf16 [N, rows] =
 * bf16(f32(x @ q) * s), the scale applied after the dot, per output column: q int8 [K, rows] as quantize_array makes
 * it with per-column scales s fp32 [rows] (scale_axis 1), in the W8K layout (cbmoe_w8k_repack, nmat 1); x bf16
 * [N, K]. The stored int8 weights are multiplied as they are against x split into two int8 digits per element
 * (exact int32 sums; exact for bf16 within 2^6 of the token's largest |x|). Workspace:
 * cbmoe_cb8_matvec_workspace_bytes(N, K), 16-byte aligned. K <= 65536. */
int cbmoe_w8_logits(const void* qk, const float* s, int rows, int K, const uint16_t* x, int N, uint16_t* out,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* -------------------------------------------------------------------------------- expert parallelism
 * Routed experts sharded by id over the ranks of one node (rank r holds experts [r*E/n, (r+1)*E/n)); tokens stay on
 * their rank; the shared expert is replicated. The reference shards moe_inter instead (engine.py:129-176) and
 * psums the partials (model.py:855); the EP layer's output equals the single-GPU layer's (model.py:840-856).
 * Communicator: rank 0 calls cbmoe_ep_unique_id, the 128 bytes reach every rank out of band, each rank calls
 * cbmoe_ep_comm_init (NCCL, blocking). cbmoe_ep_layer is stream-ordered on `stream` (NCCL send/recv included);
 * `capacity` = rows per peer in each direction: a rank sends at most `capacity` slots to one peer, the rest are
 * dropped and flagged CBMOE_DEVERR_CAPACITY (N_local * k is always enough). local: this rank's E/n experts. */
int cbmoe_ep_unique_id(uint8_t* id128_host);
int cbmoe_ep_comm_init(const uint8_t* id128_host, int nranks, int rank, void** comm_out);
int cbmoe_ep_comm_destroy(void* comm);
size_t cbmoe_ep_workspace_bytes(const cbmoe_experts* local, int N_local, int k, int nranks, int capacity, int path);
/* path: kernels for the received rows (CBMOE_PATH_DECODE, CBMOE_PATH_GROUPED, or CBMOE_PATH_AUTO: grouped from 8
 * expected rows per local expert, N_local * k >= 8 * local->E). */
int cbmoe_ep_layer(void* comm, int nranks, int rank, const cbmoe_experts* local, int E_total, const cbmoe_shared* sh,
                   const uint16_t* x, int N_local, const int32_t* idx, const float* w, int k, float limit,
                   int capacity, int path, void* peer, uint16_t* out, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream);
/* Peer-memory transport for cbmoe_ep_layer (peer != NULL there): the dispatch and the return are written straight
 * into the other GPUs' memory over NVLink (CUDA IPC mappings) instead of NCCL send/recv; every wait on a peer is
 * bounded (CBMOE_DEVERR_TIMEOUT). Collective: every rank calls cbmoe_ep_peer_init with the same H and capacity
 * (nranks <= 8, one process per GPU of one node); cbmoe_ep_layer then requires that capacity. Destroy after all
 * ranks are past their last layer call (e.g. after a barrier). */
int cbmoe_ep_peer_init(void* comm, int nranks, int rank, int H, int capacity, cudaStream_t stream, void** peer_out);
int cbmoe_ep_peer_destroy(void* peer);

/* MoE router, fused (replaces moe_route, engine/glm53/model.py:798-808, n_group == 1): x bf16 [N][D], router_w bf16
 * [D][E] (x @ router_w), bias fp32 [E] -> idx int32 [N][k], w fp32 [N][k]: logits in fp32, s = sigmoid(logits),
 * idx = top k of s + bias (largest first; the lower expert index first among equal choices), w = s[idx],
 * normalized to sum 1 when norm_topk (w / (sum + 1e-20)), times scaling. E <= 256, k <= 32, k <= E. */
int cbmoe_route(const uint16_t* x, int N, int D, const uint16_t* router_w, const float* bias, int E, int k,
                int norm_topk, float scaling, int32_t* idx, float* w, cudaStream_t stream);

/* ---- llama.cpp IQ expert formats (the reference's real GLM-5.3-Flash tables) ----------------------------------
 * Raw GGUF blocks of 256 weights, identified by their ggml_type numbers. Replaces iqquant.dequant_rows
 * (engine/glm53/iqquant.py:230-235; the per-format dequant at :108-146): blocks [n_blocks][block bytes] ->
 * out fp32 [n_blocks][256], bit for bit the reference's and gguf-py's values. `table` (device, fp32) is the
 * format's lookup table as gguf-py defines it: IQ2_S grid [1024][8], IQ3_S grid [512][4], IQ4_XS the 16 IQ4_NL
 * levels (cbmoe_iq_table_shape gives entries x width); Q2_K and Q3_K have none (0 x 0, table may be NULL).
 * out 16-byte aligned. */
#define CBMOE_GGML_Q2_K 10                                      /* the reference's MTP-layer experts */
#define CBMOE_GGML_Q3_K 11
#define CBMOE_GGML_IQ3_S 21
#define CBMOE_GGML_IQ2_S 22
#define CBMOE_GGML_IQ4_XS 23
size_t cbmoe_iq_block_bytes(int ggml_type);          /* 84 / 110 / 110 / 82 / 136; 0 if not one of the five here */
int cbmoe_iq_table_shape(int ggml_type, int* entries, int* width);
int cbmoe_iq_dequant(int ggml_type, const void* blocks, long long n_blocks, const float* table, float* out,
                     cudaStream_t stream);

/* The int8 tensor-core layout of an IQ2_S or IQ3_S matrix [E][rows][K/256][block bytes] (rows multiple of 64):
 * an exact load-time transcode (each weight d * k * v as a per-weight code of the signed grid value v, a byte per
 * group for k, f32 per block for d), which cbmoe_iq_experts_apply uses for that matrix when given. No counterpart
 * in the reference (its TPU kernel reads the GGUF planes directly). cbmoe_iq8_bytes: size of `out` (0 for other
 * formats); cbmoe_iq8_build: out 256-byte aligned; synchronizes `stream`; CBMOE_ERR_UNSUPPORTED if the table holds
 * a grid value the code cannot (IQ2_S: other than 8, 25, 43; IQ3_S: other than the odd values 1..15). */
size_t cbmoe_iq8_bytes(int ggml_type, int E, int rows, int K);
int cbmoe_iq8_build(int ggml_type, const void* raw, const float* table, int E, int rows, int K, void* out,
                    cudaStream_t stream);

/* Routed experts on raw GGUF IQ tables: ResidentFetch.apply with IQ qtypes (resident.py:100-120 over
 * pallas_moe.moe_matvec, pallas_moe.py:238-307), per-matrix formats as in the reference's qtypes. Tables as in
 * the GGUF: [E][rows][K/256][block bytes], gate/up rows = I over K = H, down rows = H over K = I (H, I multiples
 * of 256); tables[] = each matrix's lookup table (see cbmoe_iq_dequant). g, u = W x, h = swiglu_clamped(g, u,
 * limit), y = sum_k w * (W_down h), y fp32 [N][H], 16-byte aligned. A matrix with its int8 layout (gate8 / up8 /
 * down8, from cbmoe_iq8_build; NULL: none) runs on the int8 tensor cores against its input split into two int8
 * digits per element (exact int32 sums, the input to within 2^-14 of its row's largest); the others compute in
 * fp32 like the reference. */
typedef struct {
  int E, H, I;
  int gate_type, up_type, down_type;              /* CBMOE_GGML_IQ2_S / IQ3_S / IQ4_XS / Q2_K / Q3_K */
  const void* gate;
  const void* up;
  const void* down;
  const float* gate_table;
  const float* up_table;
  const float* down_table;
  const void* gate8;                              /* cbmoe_iq8_build output of each matrix, or NULL */
  const void* up8;
  const void* down8;
} cbmoe_iq_experts;
size_t cbmoe_iq_workspace_bytes(const cbmoe_iq_experts* ex, int N, int k);
int cbmoe_iq_experts_apply(const cbmoe_iq_experts* ex, const uint16_t* x, int N, const int32_t* idx, const float* w,
                           int k, float limit, float* y, void* workspace, size_t workspace_bytes, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* CBMOE_H */
