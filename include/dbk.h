/* dbk.h - C ABI of the decodebench_b200 fused decode kernels (sm_100a).
 *
 * Every entry point:
 *   - takes device pointers, sizes and a cudaStream_t passed as void*; an output
 *     pointer may also be pinned host memory (its unified address): the kernel
 *     then writes the result there directly, with no separate copy-out;
 *   - allocates nothing and never synchronises (safe inside CUDA-graph capture);
 *     scratch space is a caller-owned workspace sized by dbk_workspace_bytes();
 *   - returns 0 on success, a negative DBK_E* code for a rejected argument, or a
 *     positive cudaError_t value when a CUDA call fails.
 *
 * The reference (animeshsri14/Decodebench) launches its kernels through one
 * by-value struct, `KernelArgs` (validation/include/decodebench_val/kernel_args.h:24-103),
 * with geometry chosen by its harness (validation/src/bench/bench_variant.cu:376-387,
 * :562-575, :758-770) and host checks that exit(1) (bench_variant.cu:60-70, :324-331,
 * :689-700). These entry points replace that struct with one call per fused
 * operation; the checks become DBK_E* return codes.
 */
#ifndef DBK_H_
#define DBK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DBK_ABI_VERSION 1

/* Element type of activations, weights, caches and outputs. */
typedef enum { DBK_F16 = 0, DBK_BF16 = 1 } dbk_dtype;

/* Argument errors (negative). Positive values are cudaError_t. */
#define DBK_OK 0
#define DBK_ENULL (-1)        /* a required pointer is NULL                         */
#define DBK_ESHAPE (-2)       /* a size is out of the supported range                */
#define DBK_EALIGN (-3)       /* a pointer or row is not 16-byte aligned             */
#define DBK_EWORKSPACE (-4)   /* workspace missing or smaller than dbk_workspace_bytes */
#define DBK_EDTYPE (-5)       /* unknown dtype                                        */
#define DBK_EDEVICE (-6)      /* the current device is not sm_100                     */

/* Operation ids for dbk_workspace_bytes(). */
typedef enum {
  DBK_OP_RMSNORM_GEMV = 0,
  DBK_OP_GATEUP_SWIGLU = 1,
  DBK_OP_GEMV = 2
} dbk_op;

/* ABI version compiled into the library (== DBK_ABI_VERSION). */
int dbk_abi_version(void);

/* Static description of a status code. */
const char* dbk_status_string(int status);

/* First error a kernel recorded after giving up a bounded wait (0 = none), and
 * clear it. Synchronises the current device. */
int dbk_take_device_error(void);

/* Poll budget of every bounded wait in this library's kernels, for the current
 * device (0 restores the default of 1<<24 polls, seconds). No counterpart in
 * the reference: the reference's kernels have no bounded waits. A smaller
 * budget lets a test make a wait give up quickly; set it only while no kernel
 * of this library is running on the device. Synchronous. */
int dbk_set_spin_limit(uint32_t polls);

/* Test hook (no counterpart in the reference): launches one CTA that runs the
 * library's bounded wait on an event that never happens -- which = 0: an
 * mbarrier nobody arrives at (records 1, "stage never filled"); which = 1: a
 * peer flag nobody raises (records 5, "peer signal missing"). The kernel gives
 * up after the spin budget, records the code for dbk_take_device_error and
 * returns, leaving the context usable. */
int dbk_test_bounded_wait(int which, void* stream);

/* Workspace bytes a GEMV-family operation needs (0 if none):
 *   op = DBK_OP_RMSNORM_GEMV | DBK_OP_GATEUP_SWIGLU | DBK_OP_GEMV,
 *   sizes (batch, d_in, d_out or d_ff).
 * A workspace must be zero-filled once before its first use (e.g. cudaMemset
 * right after allocation); every kernel leaves it zero-filled again, so one
 * workspace serves any number of calls ordered on one stream. */
size_t dbk_workspace_bytes(int op, int64_t batch, int64_t d_in, int64_t d_out);

/* Workspace bytes of dbk_flashdecode for the given sizes (same zero-fill rule). */
size_t dbk_flashdecode_workspace_bytes(int batch, int n_q_heads, int n_kv_heads, int max_len,
                                       int split_tokens);

/* F1: y[b, :] = W @ (x[b, :] * rsqrt(mean(x[b, :]^2) + eps) * gamma)
 *   x [batch, d_in], gamma [d_in], W [d_out, d_in] row-major, y [batch, d_out].
 *   fp32 accumulation; normalisation folded into the GEMV.
 * Replaces fused f1_kernel (validation/src/kernels/fused/f1.cu:18-84, launched at
 * bench_variant.cu:379-387) and the Python stages rmsnorm + gemv
 * (src/decodebench/demos/llama_decode.py:36-43).
 * batch 1..8: streaming kernel (mma.sync; CUDA cores when d_in % 16 != 0), no workspace;
 * batch 9..256: tcgen05 tensor cores (needs workspace).
 * Ordering (programmatic dependent launch, all GEMV entry points): W is
 * streamed while the preceding kernel in the stream may still run; x, gamma
 * and residual are read, and y written, after it has completed. Weights are
 * not written during decode; if they are, by the immediately preceding dbk_*
 * call, put an event between or set DBK_PDL=0. */
int dbk_rmsnorm_gemv(const void* x, const void* gamma, const void* W, void* y,
                     int batch, int d_in, int d_out, float eps, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* F2: h[b, j] = silu(x[b, :] . Wg[j, :]) * (x[b, :] . Wu[j, :])
 *   optionally with an RMSNorm prologue on x when gamma != NULL.
 *   x [batch, d_in], Wg, Wu [d_ff, d_in], h [batch, d_ff].
 * Replaces fused f2_kernel (validation/src/kernels/fused/f2.cu:17-76, launched at
 * bench_variant.cu:562-575) and the Python stages gate, up, swiglu
 * (src/decodebench/demos/llama_decode.py:77-87). */
int dbk_gateup_swiglu(const void* x, const void* gamma, const void* Wg, const void* Wu,
                      void* h, int batch, int d_in, int d_ff, float eps, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Plain GEMV / thin GEMM: y[b, :] = W @ x[b, :] (+ residual[b, :] when not NULL).
 * Replaces the unfused gemv_kernel role (validation/src/kernels/unfused/gemv.cu:15-48)
 * and F.linear (llama_decode.py:41-43); used for the MLP down projection. */
int dbk_gemv(const void* x, const void* W, const void* residual, void* y,
             int batch, int d_in, int d_out, int dtype,
             void* workspace, size_t workspace_bytes, void* stream);

/* Decode MLP block in ONE persistent launch (batch 1..4):
 *   h = silu(Wg x') * (Wu x'), x' = x or, when gamma is not NULL, RMSNorm(x);
 *   y = Wd h (+ residual when not NULL).
 * x, residual, y [batch, d_model]; Wg, Wu [d_ff, d_model]; Wd [d_model, d_ff];
 * h [batch, d_ff] is written (the intermediate activation, caller-owned).
 * One CTA per SM computes its rows of h, meets the other CTAs at a grid-wide
 * barrier (bounded wait; two counters in `workspace`), then its rows of y,
 * while the down weights stream in behind the gate/up weights without a
 * kernel boundary. Bit-identical to dbk_gateup_swiglu followed by dbk_gemv.
 * workspace: >= dbk_mlp_block_workspace_bytes() bytes, zero-filled before the
 * first call (every call leaves it zero); one per call that may run
 * concurrently. All CTAs must be resident at once: do not run it beside a
 * kernel that holds SMs until this one finishes. DBK_ESHAPE unless
 * d_model % 16 == 0, d_ff % 16 == 0, SM count <= d_model <= 4096,
 * d_ff >= SM count and every phase's activation stage fits in shared memory
 * (with three weight-ring stages up to batch * d_ff of about 16,000, with two
 * up to about 49,000). Replaces the f2_kernel launch plus the down-projection
 * launch (validation/src/kernels/fused/f2.cu:17-76, bench_variant.cu:562-575;
 * src/decodebench/demos/llama_decode.py:77-87) with one launch. */
int dbk_mlp_block(const void* x, const void* gamma, const void* Wg, const void* Wu,
                  const void* Wd, const void* residual, void* h, void* y, int batch,
                  int d_model, int d_ff, float eps, int dtype, void* workspace,
                  size_t workspace_bytes, void* stream);
size_t dbk_mlp_block_workspace_bytes(void);

/* The rest of a decode layer after attention, in ONE persistent launch:
 *   h_attn = Wo attn + x;  y = dbk_mlp_block(h_attn, gamma, Wg, Wu, Wd, residual = h_attn).
 * attn [batch, d_attn] (the attention output, heads concatenated); Wo
 * [d_model, d_attn]; h_attn and h are written (caller-owned). Two grid-wide
 * barriers; the Wg/Wu and Wd streams start behind Wo's. Bit-identical to
 * dbk_gemv(attn, Wo, x) followed by dbk_mlp_block. Same rules as
 * dbk_mlp_block, plus d_attn % 16 == 0. No counterpart in the reference (its
 * demos stop at single stages, src/decodebench/demos/llama_decode.py). */
int dbk_oproj_mlp_block(const void* attn, const void* Wo, const void* x, const void* gamma,
                        const void* Wg, const void* Wu, const void* Wd, void* h_attn, void* h,
                        void* y, int batch, int d_attn, int d_model, int d_ff, float eps,
                        int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* F4: split-KV FlashDecode, one query token per sequence.
 *   q   [batch, n_q_heads, head_dim]
 *   out [batch, n_q_heads, head_dim]
 *   Contiguous cache (page_table == NULL):
 *       k_cache, v_cache [batch, n_kv_heads, max_len, head_dim]
 *   Paged cache (page_table != NULL, int32 [batch, max_pages_per_seq]):
 *       k_cache, v_cache [num_pages, n_kv_heads, page_size, head_dim]
 *   seq_lens: int32 [batch] on the device, or NULL (every sequence has max_len).
 *   q head h reads kv head h / (n_q_heads / n_kv_heads) (GQA; MHA when equal).
 *   scale multiplies q.k (1/sqrt(head_dim) for standard attention).
 *   split_tokens: tokens per split-KV work item (multiple of 64), 0 = automatic.
 * Replaces f4_partial_kernel + f4_reduce_kernel (validation/src/kernels/fused/f4.cu:173-319,
 * launched at bench_variant.cu:758-763) and the Python stages scores, softmax,
 * weighted_v (llama_decode.py:120-134). head_dim 128 only.
 * Ordering (programmatic dependent launch): q, and each sequence's newest K/V
 * row (the one a preceding dbk_qkv_rope_append writes), are read, and out and
 * the workspace written, only after every earlier kernel in the stream has
 * completed. seq_lens, the page table and the rest of the cache
 * are read earlier, while the preceding kernel may still run. That matters
 * only when the preceding kernel is one of this library's (other kernels never
 * release their dependents early): such a call may write the newest token's
 * K/V but not older slots, seq_lens or the page table; otherwise put an event
 * or any other kernel between, or set DBK_PDL=0. */
int dbk_flashdecode(const void* q, const void* k_cache, const void* v_cache,
                    const int32_t* page_table, const int32_t* seq_lens, void* out,
                    int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_len,
                    int page_size, int max_pages_per_seq, float scale, int split_tokens,
                    int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* dbk_flashdecode without a caller workspace, for callers that cannot allocate
 * device memory (for example a plugin inside a host process whose own
 * allocator owns the GPU, so it may not call cudaMalloc or a framework
 * allocator). No counterpart in the reference: it is an addition of this
 * library. Same arguments and results as dbk_flashdecode (automatic split), but
 * the scratch comes from a 2 MiB array compiled into the library and held on
 * every GPU that loads it until the process exits. Sizes whose workspace
 * (dbk_flashdecode_workspace_bytes) exceeds 2 MiB return DBK_EWORKSPACE.
 * The first call in each CUDA context (a device's primary context, or a
 * context the host made current) looks up the array's device address in that
 * context and should come before any stream capture. All calls share the array: calls that
 * overlap on the GPU race. Allocates nothing. */
int dbk_flashdecode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                            const int32_t* page_table, const int32_t* seq_lens, void* out,
                            int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_len,
                            int page_size, int max_pages_per_seq, float scale, int dtype,
                            void* stream);

/* QKV projection + RoPE + KV-cache append for one decode token (batch 1..8):
 *   qkv = Wqkv x'  (x' = RMSNorm(x) * gamma when gamma != NULL, else x; eps)
 *   q, k get rotary embedding at position positions[b] (rotate-half / NeoX
 *   pairing: dims i and i + head_dim/2, angle positions[b] * inv_freq[i]);
 *   q -> q_out [batch, n_q_heads, head_dim]; k and v are written into the cache
 *   slot positions[b]: paged (page_table != NULL, int32 [batch, max_pages]):
 *   k_cache/v_cache [pages, n_kv_heads, page_size, head_dim]; contiguous
 *   (page_table == NULL): [batch, n_kv_heads, page_size (= max_len), head_dim].
 *   A position outside the cache writes q only.
 * Wqkv [(n_q_heads + 2 n_kv_heads) * head_dim, d_in]: the q heads, the k heads,
 * then the v heads; inside each q and k head the rows are pair-interleaved
 * (row 2i = dim i, row 2i + 1 = dim i + head_dim/2; decodebench_b200.ops
 * .interleave_rope_rows builds it from the usual layout once); v rows in
 * natural order. inv_freq: fp32 [head_dim/2] on the device (e.g. theta^(-2i/D)).
 * fp32 arithmetic, one rounding per output. This is the step before
 * dbk_flashdecode in a decode layer; the reference has no such stage (README.md:106
 * lists multi-output stages such as a QKV split or RoPE as unsupported). */
int dbk_qkv_rope_append(const void* x, const void* gamma, const void* Wqkv,
                        const int32_t* positions, const float* inv_freq, void* q_out,
                        void* k_cache, void* v_cache, const int32_t* page_table, int batch,
                        int d_in, int n_q_heads, int n_kv_heads, int head_dim, int page_size,
                        int max_pages_per_seq, float eps, int dtype, void* stream);

/* fp8 weights (batch 1..8): W8 holds e4m3 bytes (OCP FP8, torch.float8_e4m3fn),
 * row-major [d_out, d_in], with one fp32 scale per row: the weight is
 * scale[r] * W8[r, k]. Same operations and argument rules as dbk_gemv,
 * dbk_rmsnorm_gemv and dbk_gateup_swiglu, with d_in % 32 == 0, x and y fp16 or
 * bf16 (dtype), fp32 accumulation; the activation is used in fp16 (hi + lo
 * parts), so |x * gamma| must stay below 65504. The activation is staged in
 * shared memory: batch * d_in up to about 22,000 (DBK_ESHAPE beyond). Half the weight bytes of the
 * 16-bit entry points, for an HBM-bound decode step. No counterpart in the
 * reference (README.md:118 lists quantization as out of its scope). */
int dbk_gemv_fp8(const void* x, const void* W8, const float* w_scale, const void* residual,
                 void* y, int batch, int d_in, int d_out, int dtype, void* stream);
int dbk_rmsnorm_gemv_fp8(const void* x, const void* gamma, const void* W8, const float* w_scale,
                         void* y, int batch, int d_in, int d_out, float eps, int dtype,
                         void* stream);
int dbk_gateup_swiglu_fp8(const void* x, const void* gamma, const void* Wg8, const float* g_scale,
                          const void* Wu8, const float* u_scale, void* h, int batch, int d_in,
                          int d_ff, float eps, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Shard-boundary all-gather over NVLink peer memory (multi-GPU, one process
 * per GPU). No counterpart in the reference, which is single-GPU: it replaces
 * the ncclAllGather that ends each sharded op (weight rows or kv heads split
 * over the GPUs of one node). Setup, once per process group:
 *   1. every rank: dbk_comm_alloc(capacity, world, &buf, record)  (cudaMalloc +
 *      CUDA IPC handle; set-up time only, like a communicator's creation);
 *   2. exchange the DBK_COMM_RECORD_BYTES records (rank order) out of band;
 *   3. every rank: dbk_comm_open(rank, world, buf, records, &comm).
 * Then dbk_allgather(comm, ...) on every rank, in the same order with the same
 * sizes; teardown: dbk_comm_close on every rank, then dbk_comm_free.
 * Ranks must be on different GPUs (dbk_comm_open returns DBK_EDEVICE
 * otherwise). Waits on peers are bounded; a wait that gives up records a
 * device error (dbk_take_device_error) and the kernel returns. */
#define DBK_COMM_RECORD_BYTES 128
typedef struct dbk_comm dbk_comm;

/* Bytes of the comm buffer for `capacity_per_rank` bytes per block and `world` ranks. */
size_t dbk_comm_buffer_bytes(size_t capacity_per_rank, int world);

/* Allocates and zero-fills this rank's comm buffer on the current device and
 * writes its DBK_COMM_RECORD_BYTES-byte record (IPC handle, GPU uuid, sizes). */
int dbk_comm_alloc(size_t capacity_per_rank, int world, void** buf_out, void* record_out);

/* Maps every peer's buffer; `records` holds world records in rank order. */
int dbk_comm_open(int rank, int world, void* local_buf, const void* records, dbk_comm** out);
int dbk_comm_close(dbk_comm* comm);
int dbk_comm_free(void* buf);

/* All-gather of equal blocks: this rank's block is `rows` rows of `row_bytes`
 * bytes, `src_ld` bytes apart at `src`; rank p's row i is written to
 *   out + p * out_block + i * out_ld
 * on every rank (so [world][block] when out_block = block bytes, or blocks side
 * by side in each row of [rows][world * row] when out_ld = world * row_bytes and
 * out_block = row_bytes). row_bytes, the strides and both pointers must be
 * 16-byte multiples; rows * row_bytes <= capacity_per_rank. Stream-ordered,
 * no host synchronisation. Replaces ncclAllGather(src, out, ...) at the shard
 * boundary. */
int dbk_allgather(dbk_comm* comm, const void* src, void* out, int rows, size_t row_bytes,
                  size_t src_ld, size_t out_ld, size_t out_block, void* stream);

/* Sharded GEMVs with the all-gather fused in (batch 1..8, one process per GPU).
 * Each rank holds d_local rows of the weights (its output columns) and writes
 * the gathered result y_full [batch][world * d_local] on every rank, rank p's
 * columns at [p * d_local, (p + 1) * d_local). The exchange happens inside the
 * GEMV kernel: every CTA stores its output rows straight into the peers' comm
 * buffers, then waits (bounded) only for the CTA with the same index on each
 * peer. Replaces "dbk_rmsnorm_gemv / dbk_gateup_swiglu / dbk_gemv followed by
 * ncclAllGather" in a column-sharded decode (no counterpart in the single-GPU
 * reference). residual_full (may be NULL) has y_full's layout; the local
 * columns are read. Same argument rules as the unsharded entry points, plus
 * batch * d_local * elem_size <= the comm's capacity; DBK_ESHAPE when the
 * shape needs the CUDA-core variant (d_in % 16 != 0) or batch > 8. Every rank
 * must make the same calls in the same order, interleaved in the same way with
 * dbk_allgather. */
int dbk_rmsnorm_gemv_allgather(dbk_comm* comm, const void* x, const void* gamma, const void* W,
                               void* y_full, int batch, int d_in, int d_local, float eps,
                               int dtype, void* stream);
int dbk_gateup_swiglu_allgather(dbk_comm* comm, const void* x, const void* gamma,
                                const void* Wg, const void* Wu, void* h_full, int batch,
                                int d_in, int d_local, float eps, int dtype, void* stream);
int dbk_gemv_allgather(dbk_comm* comm, const void* x, const void* W, const void* residual_full,
                       void* y_full, int batch, int d_in, int d_local, int dtype, void* stream);

/* Stream-ordered copy by a kernel, for a decode step's small inputs and outputs
 * (a few KB): dst and src may each be device memory or pinned host memory
 * (cudaHostAlloc / torch pin_memory, reached through its unified address), not
 * pageable memory (DBK_EDEVICE). Both 16-byte aligned (DBK_EALIGN otherwise).
 * Lower fixed latency than a copy-engine transfer at these sizes, and it keeps
 * the programmatic-dependent-launch chain: a following library kernel starts
 * streaming its weights while the input is still arriving. A copy into host
 * memory is visible to the host once the stream's work has completed. No
 * counterpart in the reference (whose harness uses cudaMemcpy). */
int dbk_copy(void* dst, const void* src, size_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DBK_H_ */
