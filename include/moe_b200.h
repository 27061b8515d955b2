/*
 * moe_b200.h -- C ABI of libmoe_b200, the sm_100a MoE token packing and
 * dispatch library.
 *
 * Conventions
 *  - Every pointer argument is a device pointer unless its comment says
 *    "host".  All device buffers are owned by the caller.
 *  - Token rows are opaque 16-bit words (fp16 or bf16); `dtype` matters only
 *    where arithmetic happens (combine, FFN): MOE_B200_F16 or MOE_B200_BF16.
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream).  Work is
 *    enqueued asynchronously; no entry point blocks the host unless its
 *    comment says so.
 *  - Return value: MOE_B200_OK or a host-detected error (bad argument, short
 *    workspace, CUDA launch failure).  Errors the device detects while running
 *    (an assignment outside [0, E), a bounded wait that ran out) are recorded
 *    in the workspace and read with moe_b200_workspace_status().
 *
 * Reference interfaces replaced (paths within feiyang-cmu/15618-final):
 *  - moe_b200_pack* replace moe::IScatter::workspace_bytes / run
 *    (include/moe/scatter.cuh:37, :48-53) and the strategies behind them
 *    (src/scatter/scatter_{atomic,sort,warp,vec,csort}.cu); the output
 *    contract is moe::cpu_scatter's (src/common/cpu_reference.cpp:12-51).
 *  - moe_b200_unpermute replaces the app-local unpack_combine_kernel +
 *    f32_to_f16_kernel pair (apps/bench_e2e.cu:136-152, launched :304-312).
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum moe_b200_status {
    MOE_B200_OK = 0,
    MOE_B200_ERR_INVALID_ARG = 1,      /* bad size, null pointer, misaligned */
    MOE_B200_ERR_WORKSPACE = 2,        /* workspace null or too small */
    MOE_B200_ERR_UNSUPPORTED = 3,      /* shape outside the supported limits */
    MOE_B200_ERR_CUDA = 4,             /* a CUDA call or launch failed */
    /* device-side conditions, reported by moe_b200_workspace_status() as bits */
    MOE_B200_DEV_BAD_ASSIGNMENT = 0x10, /* some assignment was outside [0, E) */
    MOE_B200_DEV_WAIT_TIMEOUT = 0x20,   /* a bounded cross-CTA wait gave up */
    MOE_B200_DEV_BAD_WEIGHTS = 0x40     /* router weights not prepared for this d / E / dtype */
};

enum moe_b200_dtype { MOE_B200_F16 = 0, MOE_B200_BF16 = 1 };

/* Limits of the packing kernels. */
#define MOE_B200_MAX_EXPERTS 1024

/* Library version (major*10000 + minor*100 + patch). */
int moe_b200_version(void);

/* Static description of a status code. */
const char* moe_b200_status_string(int status);

/* Human-readable text of the last host-side error on this thread ("" if none). */
const char* moe_b200_last_error(void);

/* ---------------------------------------------------------------- pack ---- */

/* Scratch bytes moe_b200_pack needs for T tokens, K slots each, E experts.
 * Replaces moe::IScatter::workspace_bytes (include/moe/scatter.cuh:37).     */
size_t moe_b200_pack_workspace_bytes(int T, int K, int E);

/* Zero-fill a workspace before its first use (enqueued on `stream`).  Every
 * moe_b200_pack call leaves the workspace zero-filled again, so this is needed
 * once per allocation, not per call.                                        */
int moe_b200_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Pack token rows by expert, stably: within each expert the rows keep
 * ascending (t, k) order, exactly as moe::cpu_scatter
 * (src/common/cpu_reference.cpp:12-51) produces them.  Replaces
 * moe::IScatter::run (include/moe/scatter.cuh:48-53).
 *   emb            [T, d]    16-bit rows (read only)
 *   asgn           [T, K]    expert of slot (t, k), in [0, E)
 *   wts            [T, K]    routing weight of slot (t, k); may be NULL when
 *                            packed_weights is NULL
 *   packed         [T*K, d]  out: packed[p] = emb[perm[p]]; may be NULL: then
 *                            only the indices are produced (no row copy, emb
 *                            unused) for moe_b200_grouped_swiglu_gather
 *   packed_weights [T*K]     out: weight of packed row p (may be NULL)
 *   perm           [T*K]     out: source token of packed row p
 *   expert_count   [E]       out: rows per expert
 *   expert_start   [E+1]     out: exclusive prefix of expert_count; [E] = T*K
 *   slot_pos       [T*K]     out (may be NULL): packed row of slot (t, k), the
 *                            inverse of perm that moe_b200_unpermute reads
 *   workspace      moe_b200_pack_workspace_bytes(T, K, E) bytes, zero-filled
 *                  once with moe_b200_workspace_init.
 * Concurrent calls must use distinct workspaces.                            */
int moe_b200_pack(const void* emb, const int32_t* asgn, const float* wts,
                  int T, int K, int E, int d,
                  void* packed, float* packed_weights, int32_t* perm,
                  int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Synchronise `stream`, then read and clear the device-side condition bits
 * (MOE_B200_DEV_*) recorded in `workspace`; *device_status = 0 means clean. */
int moe_b200_workspace_status(void* workspace, size_t workspace_bytes, void* stream,
                              int* device_status /* host */);

/* Scratch bytes built into the library for moe_b200_pack_noalloc, per device. */
#define MOE_B200_NOALLOC_SCRATCH_BYTES (4u << 20)

/* moe_b200_pack for callers that cannot allocate device memory.  This entry
 * point has no counterpart in the reference.  Some callers own only their
 * inputs and outputs: a plugin inside a host framework that hands out device
 * memory from its own pool and forbids direct cudaMalloc, or a thin FFI
 * binding with no allocator of its own.  Here the scratch is a 4 MiB array
 * built into the library (every GPU that loads the library holds it until
 * exit); the caller passes only inputs and outputs, with the same meaning as
 * in moe_b200_pack.  Shapes whose scratch (moe_b200_pack_workspace_bytes)
 * exceeds MOE_B200_NOALLOC_SCRATCH_BYTES are rejected with
 * MOE_B200_ERR_WORKSPACE (e.g. T*K above ~1M slots).
 *  - The first call on each device, made with that device current, looks up
 *    the array's address (a host-side lookup, nothing is enqueued); make that
 *    first call before any stream capture.  The address is remembered per
 *    device: after cudaDeviceReset it is stale, so do not call this entry
 *    point on a device the process has reset.
 *  - Every call clears the part of the array that must start at zero on its
 *    own stream before its kernels run.
 *  - All calls on a device share the array: calls that overlap on the GPU
 *    race and must be serialised by the caller.
 *  - Device-side conditions (MOE_B200_DEV_*) are not reported by this entry
 *    point.  No cudaMalloc, cudaFree or allocating routine is called.       */
int moe_b200_pack_noalloc(const void* emb, const int32_t* asgn, const float* wts,
                          int T, int K, int E, int d,
                          void* packed, float* packed_weights, int32_t* perm,
                          int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                          void* stream);

/* Synchronise `stream`, then read and clear the device-side condition bits
 * (MOE_B200_DEV_*) that workspace-less kernels (unpermute, grouped FFN) of the
 * current device recorded; *device_status = 0 means clean.  New: the
 * reference reports nothing from the device.                               */
int moe_b200_device_status(void* stream, int* device_status /* host */);

/* ------------------------------------------------------------ combine ---- */

/* Weighted unpermute + top-K combine:
 *   out[t, :] = round16( sum_{k=0..K-1} packed_weights[p] * y[p, :] ),
 *   p = slot_pos[t*K + k],  accumulated in fp32 in ascending k.
 * Replaces unpack_combine_kernel + f32_to_f16_kernel (apps/bench_e2e.cu:136-152).
 *   y [T*K, d] 16-bit expert outputs in packed order; out [T, d] 16-bit.    */
int moe_b200_unpermute(const void* y, const float* packed_weights, const int32_t* slot_pos,
                       int T, int K, int d, int dtype, void* out, void* stream);

/* -------------------------------------------------------------- router ---- */

/* Router: gate GEMM + softmax over all E experts + top-K, one kernel on the
 * tcgen05 tensor cores with the logits kept on chip:
 *   logit[t, e] = sum_i emb[t, i] * w_gate[i, e]               (fp32)
 *   p[t, e]     = expf(logit - max_e logit) / sum_e expf(...)  (ascending e)
 *   assignments[t, k], weights[t, k] = the K largest p[t, :] in descending
 *   order, ties to the lower expert index; weights are the softmax
 *   probabilities themselves (not renormalised over K).
 * Replaces fused_route_kernel (apps/bench_e2e.cu:95-130) and the unfused
 * gate_kernel / softmax_kernel / topk_kernel chain (apps/bench_e2e.cu:51-93),
 * same argument meaning (w_gate [d, E] fp32, row i = input feature i).
 *
 * The fp32 gate weights are prepared once (moe_b200_router_prepare) into a
 * caller-allocated buffer of moe_b200_router_weights_bytes(d, E, dtype)
 * bytes: transposed to K-major and split into 16-bit pieces of the
 * embeddings' type whose sum is w_gate to 22 (fp16, 2 pieces, power-of-two
 * pre-scaled) or 24 (bf16, 3 pieces) significant bits, so the tensor cores
 * take the embeddings unconverted and the logits keep fp32 accuracy.
 * Limits: d a multiple of 8; 1 <= E <= 256 (fp16) or 128 (bf16);
 * 1 <= K <= min(8, E).  Pointers 16-byte aligned.                           */
size_t moe_b200_router_weights_bytes(int d, int E, int dtype);
int moe_b200_router_prepare(const float* w_gate, int d, int E, int dtype, void* packed_weights,
                            void* stream);
int moe_b200_route(const void* emb, int T, int d, int E, int K, int dtype, const void* packed_weights,
                   int32_t* assignments, float* weights, void* stream);

/* ---------------------------------------------------------- expert FFN ---- */

/* Grouped SwiGLU expert FFN on packed rows, on the tcgen05 tensor cores:
 *   h[r] = silu(x[r] . Wg[e]^T) * (x[r] . Wu[e]^T),   y[r] = h[r] . Wd[e]^T
 * for each row r of segment s (rows [seg_start[s], seg_start[s+1])), with
 * e = seg_expert[s] (seg_expert NULL: e = s, e.g. seg_start = expert_start
 * from moe_b200_pack).  fp32 accumulation; h and y rounded once to dtype.
 *   x          [rows, d]       packed rows (16-bit, dtype)
 *   w_gate_up  [E, 2*I, d]     row j < I: gate column j; row I + j: up column j
 *   w_down     [E, d, I]       row c: output column c over the I inner features
 *   h          [rows, I]       out: the SwiGLU intermediate
 *   y          [rows, d]       out: expert outputs, in packed order
 * d and I multiples of 16; all pointers 16-byte aligned; nseg <= 1024.
 * Replaces the per-expert cublasHgemm loop (apps/bench_e2e.cu:274-301,
 * apps/bench_prefill.cu:854-884) and the CUTLASS sm80 GemmGrouped FFN
 * (apps/bench_prefill.cu:68-202, 812-852), which have no activation and need
 * the expert counts on the host.  Device-side conditions are reported by
 * moe_b200_device_status().                                                 */
int moe_b200_grouped_swiglu(const void* x, const int32_t* seg_start, const int32_t* seg_expert,
                            int nseg, int rows, int d, int I, int E,
                            const void* w_gate_up, const void* w_down, int dtype,
                            void* h, void* y, void* stream);

/* Gathered form (no packed copy of the rows): packed row r is
 * x_tokens[row_token[r]], row_token = perm from moe_b200_pack (which may then
 * run with packed = NULL).  The gate/up GEMM fetches its A rows from
 * x_tokens [T, d] with TMA tile::gather4 loads (4 token rows per load); all
 * other arguments and results as moe_b200_grouped_swiglu.  The reference's
 * attempt at the same idea is apps/bench_blocksparse.cu:197-231.           */
int moe_b200_grouped_swiglu_gather(const void* x_tokens, int T, const int32_t* row_token,
                                   const int32_t* seg_start, const int32_t* seg_expert, int nseg,
                                   int rows, int d, int I, int E, const void* w_gate_up,
                                   const void* w_down, int dtype, void* h, void* y, void* stream);

/* The reference's expert, activation-free, on the same grouped tcgen05
 * kernel:  mid[r] = round16(x[r] . Wup[e]^T),  y[r] = round16(mid[r] . Wdown[e]^T),
 * fp32 accumulation, for each row r of segment s (e = seg_expert[s], or s).
 *   w_up   [E, F, d]   K-major up-projection (row j = inner feature j)
 *   w_down [E, d, F]   K-major down-projection (row c = output column c)
 *   mid    [rows, F]   out: the intermediate; y [rows, d] out
 * d and F multiples of 16; pointers 16-byte aligned; nseg <= 1024.
 * Replaces the per-expert cublasHgemm up/down loop (apps/bench_e2e.cu:274-301,
 * apps/bench_prefill.cu:854-884), which needs the expert counts on the host;
 * that loop's d_ffn is F.  Device-side conditions: moe_b200_device_status(). */
int moe_b200_grouped_ffn(const void* x, const int32_t* seg_start, const int32_t* seg_expert,
                         int nseg, int rows, int d, int F, int E, const void* w_up,
                         const void* w_down, int dtype, void* mid, void* y, void* stream);

/* One-time conversion of the reference's expert weights into the layout
 * above: w1 [E, d, F] (the reference's d_W1, row-major B of mid = A . W1,
 * apps/bench_e2e.cu:281-292) -> w_up [E, F, d]; w2 [E, F, d] (d_W2) ->
 * w_down [E, d, F].  16-bit words, enqueued on `stream`; E <= 65535.        */
int moe_b200_ffn_weights_from_reference(const void* w1, const void* w2, int E, int d, int F,
                                        void* w_up, void* w_down, void* stream);

/* ----------------------------------------------------- expert parallel ---- */

/* Exchange layout of rank `rank` among `nranks` expert-parallel ranks, on the
 * device.  Experts are owned in contiguous ranges: rank g owns
 * [expert_first[g], expert_first[g+1]) (host array, nranks+1 entries, may be
 * uneven).  all_counts [nranks, E]: every rank's expert_count (one all-gather).
 *   send_counts [nranks]  rows of this rank's packed buffer for rank g -- the
 *                         packed buffer is already the rank-major send buffer
 *   recv_counts [nranks]  rows received from rank g
 *   seg_start   [nranks*L + 1], seg_expert [nranks*L]  (L = local experts):
 *                         the receive buffer's segments, sender-major then
 *                         local-expert-major; seg_expert is the local expert
 *                         index, as moe_b200_grouped_swiglu expects.
 * Replaces the host-side offset computation after a D2H copy
 * (apps/bench_prefill.cu:768-788) and the per-round host FFN problem list
 * (apps/bench_prefill.cu:812-852).  nranks <= 64.                          */
int moe_b200_ep_layout(const int32_t* all_counts, int nranks, int E, int rank,
                       const int32_t* expert_first /* host */, int32_t* seg_start,
                       int32_t* seg_expert, int32_t* send_counts, int32_t* recv_counts,
                       void* stream);

/* ------------------------------ fused expert parallel over peer memory ---- */

/* One process per GPU.  A context owns this rank's symmetric region (receive
 * rows for up to nranks*max_tokens*K rows with each row's return address,
 * back rows, counts inbox, epoch flags), which the peers map through CUDA
 * IPC.  Lifecycle:
 *   moe_b200_ep_create -> moe_b200_ep_ipc_handle (64 bytes) -> exchange the
 *   handles between the ranks (any host channel) -> moe_b200_ep_connect with
 *   all nranks handles in rank order -> steps -> barrier -> moe_b200_ep_destroy.
 * A step, with the same epoch on every rank (1, 2, 3, ...), enqueued on one
 * stream and never blocking the host:
 *   moe_b200_ep_dispatch         route/scan (whose last tile publishes the
 *                                 counts to every peer), then store every
 *                                 token row straight into the receive buffer
 *                                 of the rank owning its expert
 *   moe_b200_ep_receive           wait for all senders' rows; segment
 *                                 table of the receive buffer, which is
 *                                 expert-major: one segment per local expert,
 *                                 this rank's own rows of the H replicated
 *                                 experts first, then the L' non-replicated
 *                                 ones holding every sender's rows
 *                                 (seg_start L'+H+1 entries, seg_expert L'+H);
 *                                 any expert kernel may read them after it
 *   moe_b200_ep_ffn_return        grouped SwiGLU on the received rows: the
 *                                 gate/up GEMM starts on the replicated
 *                                 segments and waits for the senders' rows
 *                                 before the others; the down-GEMM stores
 *                                 every row straight into the sender's back
 *                                 buffer, at the return address the dispatch
 *                                 stored beside it
 *     or moe_b200_ep_return_identity   (identity expert; waits for the
 *                                 senders' rows itself)
 *   moe_b200_ep_combine           wait for all returns; weighted unpermute
 * or all of it with one call, moe_b200_ep_step.
 * Replaces the reference's AllGather -> D2H -> host offsets -> grouped
 * ncclSend/ncclRecv dispatch and combine (apps/bench_prefill.cu:768-807,
 * 889-906).  Waits are bounded by timeout_ms and report
 * MOE_B200_DEV_WAIT_TIMEOUT through moe_b200_device_status().              */
int moe_b200_ep_create(int nranks, int rank, int E, int K, int d, int max_tokens,
                       const int32_t* expert_first /* host, nranks+1 */, int timeout_ms,
                       void** ctx /* host, out */);
int moe_b200_ep_destroy(void* ctx);
/* Replicated experts (no reference counterpart; the reference partitions the
 * experts contiguously, apps/bench_prefill.cu:361): every rank holds its own
 * copy of experts[0..n-1], and rows routed to them stay on their rank (no
 * NVLink traffic); the other experts keep their owner ranks.  Call before
 * the first step with the same set on every rank.  The rank's local expert
 * weights (moe_b200_ep_ffn_return) are then ordered as
 * moe_b200_ep_local_experts lists them: the non-replicated experts of its
 * range, then the replicated ones, each ascending.  Returns the count;
 * experts_out (host, may be NULL) receives the global ids.                 */
int moe_b200_ep_set_replicated(void* ctx, const int32_t* experts /* host */, int n);
int moe_b200_ep_local_experts(void* ctx, int32_t* experts_out /* host, may be NULL */);
int moe_b200_ep_ipc_handle(void* ctx, void* handle /* host, 64 bytes out */);
int moe_b200_ep_connect(void* ctx, const void* handles /* host, nranks*64 bytes */);
void* moe_b200_ep_recv_rows(void* ctx);
void* moe_b200_ep_back_rows(void* ctx);
int64_t moe_b200_ep_recv_capacity(void* ctx);
int moe_b200_ep_dispatch(void* ctx, uint64_t epoch, const void* emb, const int32_t* asgn,
                         const float* wts, int T, float* packed_weights, int32_t* perm,
                         int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                         void* workspace, size_t workspace_bytes, void* stream);
int moe_b200_ep_receive(void* ctx, uint64_t epoch, int32_t* seg_start, int32_t* seg_expert,
                        void* stream);
int moe_b200_ep_return_identity(void* ctx, uint64_t epoch, const int32_t* seg_start, void* stream);
int moe_b200_ep_ffn_return(void* ctx, uint64_t epoch, const int32_t* seg_start,
                           const int32_t* seg_expert, int I, const void* w_gate_up,
                           const void* w_down, int dtype, void* h, void* stream);
int moe_b200_ep_combine(void* ctx, uint64_t epoch, const float* packed_weights,
                        const int32_t* slot_pos, int T, int dtype, void* out, void* stream);

/* One whole step in one call: dispatch -> receive -> expert -> combine with
 * the next epoch (moe_b200_ep_epoch(ctx) + 1), four kernel launches for the
 * identity expert (w_gate_up = w_down = NULL; I and h unused; its return
 * kernel waits for the senders itself) and six for the grouped SwiGLU
 * (w_gate_up / w_down / h as moe_b200_ep_ffn_return; its receive waits for
 * the counts only and the gate/up GEMM for the senders' rows, after the
 * replicated experts' local rows).  The segment table lives in the context.  Arguments otherwise as the stage
 * calls; out [T, d] receives the combined rows.  Replaces one round of
 * apps/bench_prefill.cu:768-906 (count all-gather, host offsets, dispatch
 * AllToAllv, per-expert GEMMs, combine AllToAllv).                        */
int moe_b200_ep_step(void* ctx, const void* emb, const int32_t* asgn, const float* wts, int T,
                     int I, const void* w_gate_up, const void* w_down, int dtype, void* h,
                     float* packed_weights, int32_t* perm, int32_t* expert_count,
                     int32_t* expert_start, int32_t* slot_pos, void* workspace,
                     size_t workspace_bytes, void* out, void* stream);
/* Largest epoch enqueued on this context so far (0 before the first step). */
uint64_t moe_b200_ep_epoch(void* ctx);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* MOE_B200_H */
