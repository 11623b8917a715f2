/* pkb200.h - C ABI of libpkb200.so, the B200 (sm_100a) kernel library that
 * replaces the reference's kernels/generated/<op>.cu launch entry points.
 *
 * Conventions shared by every entry point:
 *   - bf16 tensors are raw 16-bit brain-float values (the reference's pk_bf16 /
 *     __nv_bfloat16, kernels/template/kernel_common.h:42-60), row-major.
 *   - The caller allocates and owns every device buffer; outputs are sized by
 *     the caller. Inputs are not modified unless stated (the KV cache of the
 *     append entry is written in place).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream),
 *     as in the reference's launch_* functions. Launches are asynchronous.
 *     Entry points may be called from several host threads and streams at
 *     once; one-time per-device set-up is serialised inside the library. The
 *     persistent GEMM's dynamic tile schedule takes one of 4096 per-device
 *     counters per launch, so at most 4096 GEMM launches may be in flight
 *     (enqueued, not finished) on one device at a time.
 *   - Return value: 0 on success, otherwise a cudaError_t value
 *     (cudaErrorInvalidValue = 1 for a rejected shape/pointer). The reference's
 *     void launch_* functions only print on error (kernel_common.h:160-167);
 *     the C++ symbols below keep that behaviour and forward to these.
 *
 * The reference's own C++ entry points (mangled, pk_bf16 = __nv_bfloat16) are
 * exported unchanged by the same library and declared at the bottom for C++
 * callers (cuda_run_main.cpp:59-71 and bench_cuda.cpp:50-58 link against them).
 */
#ifndef PKB200_H
#define PKB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library version string ("pkb200 <major>.<minor> sm_100a"). */
const char* pkb200_version(void);

/* y = bf16( x / sqrt(mean(x^2) + eps) [* weight] ) over the last axis.
 * Replaces launch_rmsnorm (kernels/generated/rmsnorm.cu:106-108). weight may be NULL. */
int pkb200_rmsnorm(const void* input, const void* weight, void* output, int rows, int cols,
                   float eps, void* stream);

/* Exact erf GELU over n elements. Replaces launch_gelu (gelu.cu:56). */
int pkb200_gelu(const void* input, void* output, long long n, void* stream);

/* Row softmax over the last axis, fp32 math, bf16 out (golden.py:75-80).
 * Replaces launch_softmax (kernels/generated/softmax.cu), which the
 * reference's cuda_run_main.cpp:64 declares. */
int pkb200_softmax(const void* input, void* output, int rows, int cols, void* stream);

/* C = bf16(A @ B); A [M,K], B [K,N]. Replaces launch_matmul (matmul.cu:78-79). */
int pkb200_matmul(const void* A, const void* B, void* C, int M, int N, int K, void* stream);

/* C = fp32(A @ B) (no rounding): the partial sums a tensor-parallel rank feeds
 * to the all-reduce. New; no reference counterpart (the reference has no TP). */
int pkb200_matmul_f32out(const void* A, const void* B, float* C, int M, int N, int K,
                         void* stream);

/* C = bf16(rmsnorm(X; gamma, eps) @ W). gamma may be NULL (the reference kernel
 * has no gamma: fused_rmsnorm_matmul.cu:110-112). Replaces
 * launch_fused_rmsnorm_matmul (fused_rmsnorm_matmul.cu:114-116); the gamma
 * argument follows golden.fused_rmsnorm_matmul (tests/golden/golden.py:96-100).
 * Uses a library-owned device workspace of M*K bf16 for the normalised rows. */
int pkb200_fused_rmsnorm_matmul(const void* X, const void* W, const void* gamma, void* out,
                                int M, int N, int K, float eps, void* stream);

/* Same result as pkb200_fused_rmsnorm_matmul, but this entry point allocates
 * no device memory at all. It is for callers that cannot call cudaMalloc on
 * the calling thread: code running while a CUDA graph is being captured,
 * real-time or embedded hosts that forbid allocation after start-up, and
 * plugins whose host application owns all memory. The normalised rows go to
 * a fixed 16 MiB scratch array compiled into the library (each GPU that loads
 * the library holds it until the process exits), so M*K must not exceed
 * 8,388,608 elements; larger shapes return cudaErrorInvalidValue with a
 * message on stderr. The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture. All calls share the one array: calls
 * whose work overlaps on the GPU (different streams, or different host
 * threads) race on it and must be serialised by the caller.
 * This entry point has no counterpart in the reference. */
int pkb200_fused_rmsnorm_matmul_noalloc(const void* X, const void* W, const void* gamma,
                                        void* out, int M, int N, int K, float eps, void* stream);

/* out = bf16(gelu(bf16(bf16(A @ B) + bias))). Replaces launch_fused_matmul_bias_gelu
 * (fused_matmul_bias_gelu.cu:104-106). */
int pkb200_fused_matmul_bias_gelu(const void* A, const void* B, const void* bias, void* out,
                                  int M, int N, int K, void* stream);

/* out = bf16(bf16(bf16(A @ B) + bias) + resid); resid [M,N]. The MLP's second
 * GEMM with the residual add (golden.add/bias, tests/golden/golden.py:48-55) in
 * its epilogue; the reference has no kernel for this add. */
int pkb200_matmul_bias_residual(const void* A, const void* B, const void* bias,
                                const void* resid, void* out, int M, int N, int K, void* stream);

/* Tensor-parallel GEMM2 that moves its partial sums to their owners itself.
 * Row block r of this rank's fp32 partial A @ B is stored (TMA bulk stores of
 * 32x32 tiles, over NVLink for peers) into slot src_rank of peer_slots[r], an fp32
 * [world][M/world][N] buffer owned by rank r. After all ranks synchronise, each
 * owner runs pkb200_reduce_slots_bias_residual on its buffer.
 * world <= 8; M % world == 0 and (M / world) % 32 == 0; K, N multiples of 8.
 * New; no reference counterpart. */
int pkb200_matmul_peer_store_f32(const void* A, const void* B, float* const* peer_slots,
                                 int world, int src_rank, int M, int N, int K, void* stream);

/* out[rows,N] = bf16(bf16(bf16(sum over the world slots) + bias) + resid), slots
 * being the [world][rows][N] fp32 buffer filled by pkb200_matmul_peer_store_f32.
 * New; no reference counterpart. */
int pkb200_reduce_slots_bias_residual(const float* slots, int world, int rows, int N,
                                      const void* bias, const void* resid, void* out,
                                      void* stream);

/* out = bf16(bf16(bf16(Y) + bias) + resid) for an fp32 Y [M,N] (the all-reduced
 * tensor-parallel partial sums). */
int pkb200_bias_residual_f32(const float* Y, const void* bias, const void* resid, void* out,
                             int M, int N, void* stream);

/* Tile schedule of the persistent tcgen05 GEMM: 1 (default) = each CTA takes
 * its next tile from a per-launch atomic counter, so CTAs that start late
 * (SMs held by a concurrent kernel such as a collective) take fewer tiles;
 * 0 = fixed stride over the tiles by CTA index. Results are identical. */
int pkb200_set_gemm_schedule(int dynamic);

/* Stream memory operations for the copy-engine tensor-parallel exchange (new;
 * the reference has no multi-GPU path): `stream` waits until the 32-bit word
 * at `addr` (device memory of this GPU) is >= `value`, cyclically compared;
 * or writes `value` to `addr` in stream order. Both run on the GPU's front end
 * and hold no SM. */
int pkb200_stream_wait_value32(void* stream, const void* addr, unsigned int value);
int pkb200_stream_write_value32(void* stream, void* addr, unsigned int value);

/* Copy-engine tensor-parallel MLP exchange (new; the reference has no
 * multi-GPU path). W1 is column-split and W2 row-split over `world` ranks.
 * pkb200_tp_ce_mlp_block runs, in `chunks` row chunks on `stream`, GEMM1
 * (xn = rmsnorm(x; gamma) [M, d] times this rank's W1 shard [d, ffn_shard],
 * + b1, erf-GELU; into h_ws, bf16 [M/chunks, ffn_shard]) and GEMM2 (h times the
 * W2 shard [ffn_shard, d] into fp32 partials); pkb200_tp_ce_mlp_step takes
 * GEMM1's output h [M, ffn_shard] instead and runs GEMM2 alone in chunks.
 * After each chunk's GEMM2 the copy engines push every fp32 partial row block
 * to the rank that owns it (slots), the owner sums the slots in rank order
 * with the b2 + residual epilogue into its gather buffer and pushes those
 * bf16 rows into every peer's gather buffer (all NVLink traffic is writes);
 * once all of a chunk has landed it is copied into `out` [M, d] on every rank.
 * Each chunk's exchange overlaps the next chunk's GEMMs.
 * Buffers (peer pointers in this process's address space, e.g. from
 * pkb200_ipc_alloc / pkb200_ipc_open): slots[p] fp32 [chunks][world][M/chunks/world][d],
 * rows[p] bf16 [M][d] (gather buffer), flags[p] uint32 [2][chunks][world]
 * zeroed before first use, on every rank; y32 fp32 [M, d] and epoch_src
 * uint32 [2*8+2] local to this rank. `epoch` increases by 1 per step from 1.
 * pkb200_tp_ce_wait waits on the host for the last step, at most
 * `timeout_ms`; when a peer has not delivered by then it releases this rank's
 * waits, marks the plan failed and returns cudaErrorTimeout (the context
 * stays usable; create a new plan after the failure). */
/* Peer mappings without multicast: device memory this library allocates
 * (zeroed) with its 64-byte CUDA IPC handle, opened by the peer processes;
 * used for the copy-engine exchange's slots, rows and flags. */
int pkb200_ipc_alloc(size_t bytes, void** ptr, void* handle64);
int pkb200_ipc_open(const void* handle64, void** ptr);
int pkb200_ipc_close(void* ptr);
int pkb200_free(void* ptr);
/* One copy-engine copy in stream order (cudaMemcpyAsync, direction inferred
 * from the pointers; a peer pointer from pkb200_ipc_open is fine). */
int pkb200_copy_async(void* dst, const void* src, size_t bytes, void* stream);
int pkb200_tp_ce_create(int world, int rank, int M, int d, int chunks, int per_peer_streams,
                        float* y32, float* const* slots, void* const* rows,
                        unsigned int* const* flags, unsigned int* epoch_src, void** plan_out);
int pkb200_tp_ce_destroy(void* plan);
int pkb200_tp_ce_mlp_step(void* plan, const void* h, const void* w2, int ffn_shard,
                          const void* b2, const void* x, void* out, unsigned int epoch,
                          void* stream);
int pkb200_tp_ce_mlp_block(void* plan, const void* xn, const void* w1, const void* b1,
                           const void* w2, int ffn_shard, const void* b2, const void* x,
                           void* out, void* h_ws, unsigned int epoch, void* stream);
int pkb200_tp_ce_wait(void* plan, int timeout_ms);
/* Number of exchange streams (push, pull, reduce and land) the last step
 * joined back into the caller's stream: 2*(world-1)+2 with one push/pull
 * stream per peer, 4 with one shared pair. */
int pkb200_tp_ce_joined_streams(void* plan, int* count);

/* out = rmsnorm(bf16(x + resid); weight, eps) over the last axis
 * (golden.fused_residual_rmsnorm, tests/golden/golden.py:108-112): the residual
 * add + next-layer norm that follows the MLP. sum_out (nullable) receives the
 * rounded sum, the new residual stream. New entry point (the reference has the
 * fusion pass FuseResidualRmsnorm but no kernel for it). */
int pkb200_fused_residual_rmsnorm(const void* x, const void* resid, const void* weight,
                                  void* out, void* sum_out, int rows, int cols, float eps,
                                  void* stream);

/* [Q|K|V] = X @ W_qkv (golden.qkv_projection, golden.py:120-136) with the
 * split and head reshape done in the GEMM epilogue: X [B*S, H*Dh], W_qkv
 * [H*Dh, 3*H*Dh]; Q, K, V are written in the [B, H, S, Dh] layout the attention
 * entry points take (the golden returns [B, S, H, Dh]; same values). Dh % 8 == 0.
 * New entry point. */
int pkb200_qkv_projection(const void* X, const void* W_qkv, void* Q, void* K, void* V, int B,
                          int S, int H, int Dh, void* stream);

/* C = bf16(A @ (Wq * scale[n])); A bf16 [M,K], Wq int8 [K,N], scale fp32 [N].
 * Replaces launch_matmul_int8 (kernels/generated/matmul_int8.cu:97-98). */
int pkb200_matmul_int8(const void* A, const int8_t* Wq, const float* scale, void* C, int M,
                       int N, int K, void* stream);

/* fp8 weight path (fmt 0 = e4m3fn, 1 = e5m2). The reference only simulates
 * fp8 weights (tests/golden/quant_golden.py:116-125, matmul_fp8_sim;
 * kernels/cpu/matmul_quant.cpp:130-160 and its `fp8sim` mode :207-236);
 * these entry points keep the weights in HBM as one byte per element.
 * pkb200_quantize_fp8: W bf16 [n] -> fp8 codes [n], round-to-nearest-even,
 *   saturating like the reference's fp8_round (matmul_quant.cpp:130-150).
 * pkb200_dequantize_fp8: fp8 codes [n] -> bf16 [n] (exact).
 * pkb200_matmul_fp8: C = bf16(A @ fp8(W)); A bf16 [M,K], Wf8 codes [K,N].
 * pkb200_matmul_fp8_sim: the reference's simulated path with bf16 W [K,N]
 *   (round onto the fp8 grid, then matmul); same result as quantize + matmul_fp8. */
int pkb200_quantize_fp8(const void* W, uint8_t* Wf8, long long n, int fmt, void* stream);
int pkb200_dequantize_fp8(const uint8_t* Wf8, void* W, long long n, int fmt, void* stream);
int pkb200_matmul_fp8(const void* A, const uint8_t* Wf8, void* C, int M, int N, int K, int fmt,
                      void* stream);
int pkb200_matmul_fp8_sim(const void* A, const void* W, void* C, int M, int N, int K, int fmt,
                          void* stream);

/* Bytes of device workspace pkb200_mlp_block / pkb200_mlp_block_int8 need. */
size_t pkb200_mlp_block_workspace_size(int M, int d, int ffn);

/* Y = X + (GELU(rmsnorm(X;gamma,eps) @ W1 + b1) @ W2 + b2), every op rounded to
 * bf16 as the golden composes it (golden.py:48-100; tests/e2e/conftest.py:104-107;
 * examples/mlp_block.mlir semantics with the biases BASELINE adds).
 * X,Y [M,d]; gamma [d]; W1 [d,ffn]; b1 [ffn]; W2 [ffn,d]; b2 [d].
 * workspace: caller-owned device memory of pkb200_mlp_block_workspace_size bytes. */
int pkb200_mlp_block(const void* X, const void* gamma, const void* W1, const void* b1,
                     const void* W2, const void* b2, void* Y, int M, int d, int ffn, float eps,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Same chain with int8 weight-only W1/W2 and fp32 per-output-channel scales
 * (quant_golden.matmul_int8 semantics, tests/golden/quant_golden.py:91-101). */
int pkb200_mlp_block_int8(const void* X, const void* gamma, const int8_t* W1q,
                          const float* s1, const void* b1, const int8_t* W2q, const float* s2,
                          const void* b2, void* Y, int M, int d, int ffn, float eps,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Causal (or full) scaled-dot-product prefill attention. Q/O [B,H,S_q,D],
 * K/V [B,H,S_kv,D]. Row i sees keys j <= S_kv - S_q + i when causal != 0.
 * Replaces launch_attention_prefill (kernels/generated/attention_prefill.cu:169-172). */
int pkb200_attention_prefill(const void* Q, const void* K, const void* V, void* O, int B,
                             int H, int S_q, int S_kv, int D, float scale, int causal,
                             void* stream);

/* out [B,H,S_cache+S_new,D] = concat(cache, new_rows) along the sequence axis
 * (out-of-place). Replaces launch_kv_cache_update (kv_cache_update.cu:67-69). */
int pkb200_kv_cache_update(const void* cache, const void* new_rows, void* out, int B, int H,
                           int S_cache, int S_new, int D, void* stream);

/* Fused KV append + prefill attention over a preallocated cache:
 *   Kcache/Vcache [B,H,S_max,D] hold S_cache valid rows; K_new/V_new [B,H,S_q,D]
 *   are written in place into rows [S_cache, S_cache+S_q) and Q attends to the
 *   S_cache+S_q keys (golden.fused_kv_append_attention, golden.py:139-172, with the
 *   causal offset of attention_prefill.cu:103). Rows >= S_cache+S_q stay untouched.
 * Requires S_cache + S_q <= S_max. */
int pkb200_attention_prefill_kv_append(const void* Q, const void* K_new, const void* V_new,
                                       void* K_cache, void* V_cache, void* O, int B, int H,
                                       int S_q, int S_cache, int S_max, int D, float scale,
                                       int causal, void* stream);

/* Caps the grid of the persistent tensor-core GEMM at max_ctas CTAs (one per
 * SM); 0 restores the default of one CTA per SM. Process-wide. The GEMM holds
 * every SM it is given until it finishes, so a tensor-parallel caller that
 * wants NCCL kernels to run beside it (overlapping communication) leaves some
 * SMs free this way. New; no reference counterpart. */
int pkb200_set_gemm_max_ctas(int max_ctas);

/* ---- runtime: device detection and the tuning cache (lib/Runtime/
 * DeviceDetect.cpp:62-69, KernelCache.cpp:83-100 semantics; cache files in
 * the reference's tuning/schema.json format, version 1). */

/* Writes this device's arch name ("sm_100" on B200). */
int pkb200_device_arch(char* buf, size_t cap);

/* Loads a tuning-cache JSON file, replacing the current cache. Returns the
 * number of entries, or -1 with a message in err for an unreadable file or any
 * schema error (a malformed cache is never silently ignored). Only entries with
 * validated == true and gpu == this device's arch are ever served. */
int pkb200_tuning_load(const char* path, char* err, size_t err_cap);
int pkb200_tuning_clear(void);

/* The tensor-core GEMM config a launch of `op` at (M,N,K) would use, as the
 * cache's seven `best` fields in schema order (block_m, block_n, block_k,
 * num_warps, vector_width, unroll, shared_memory_stages). Returns 0 for the
 * default config, 1 for a cache hit, 2 while a config is forced, -1 for an
 * unknown op. Ops: matmul, fused_rmsnorm_matmul, fused_matmul_bias_gelu,
 * matmul_bias_residual, matmul_int8, matmul_f32out, matmul_peer_store_f32. */
int pkb200_gemm_select(const char* op, int M, int N, int K, int* cfg7);

/* Forces every tensor-core GEMM launch to `cfg7` (for the autotuner); NULL
 * returns to cache/default selection. cudaErrorInvalidValue for a config with
 * no compiled variant. */
int pkb200_set_gemm_config(const int* cfg7);

/* The config of the most recent tensor-core GEMM launch. */
int pkb200_last_gemm_config(int* cfg7);

/* Failure-detection self test: launches one warp that waits on an mbarrier
 * nothing will complete, with a wait limit of limit_cycles SM clocks (at most
 * the kernels' own ~2 s limit). The bounded wait gives up, the kernel returns
 * normally and *code receives the error word it recorded (6 = self-test
 * timeout); the CUDA context stays usable. New; no reference counterpart. */
int pkb200_selftest_wait_timeout(long long limit_cycles, int* code);

/* ---- serving engine ABI. The reference's Modal app binds
 *   int polykernel_fused_mlp_block(float* in, float* out, int M, int N, int K)
 * through ctypes (modal/app.py:206-215, 795, 836) but no library in the
 * reference implements it. Here: pkb200_engine_load_mlp copies one MLP block's
 * bf16 weights (host pointers; gamma may be NULL) to the current device; then
 * polykernel_fused_mlp_block runs that block on host fp32 rows: in [M,K] and
 * out [M,N] with K == N == d, rounded to bf16 on the way in (RNE) and widened
 * on the way out. Returns 0, 2 if no weights are loaded, or a cudaError_t. */
int pkb200_engine_load_mlp(const void* gamma, const void* w1, const void* b1, const void* w2,
                           const void* b2, int d, int ffn, float eps);
int polykernel_fused_mlp_block(float* in, float* out, int M, int N, int K);

/* Reads (and clears) the device-side error word that bounded waits inside the
 * tensor-core kernels set on timeout (0 = none). Synchronises the device. */
int pkb200_device_error(int* code);

/* The MLP block followed by the next layer's RMSNorm (new; the survey's "next"
 * row f1, golden.fused_residual_rmsnorm, golden.py:108-112): Y = the MLP block
 * output (the residual stream, as pkb200_mlp_block) and
 * Yn = bf16(Y / sqrt(mean(Y^2) + eps_next) * gamma_next) (gamma_next may be
 * NULL). GEMM2's epilogue also writes each row's partial sums of squares of the
 * rounded Y, so the normalisation is one elementwise pass over Y with no row
 * reduction. Workspace: pkb200_mlp_block_rmsnorm_next_workspace_size bytes. */
size_t pkb200_mlp_block_rmsnorm_next_workspace_size(int M, int d, int ffn);
int pkb200_mlp_block_rmsnorm_next(const void* X, const void* gamma, const void* W1,
                                  const void* b1, const void* W2, const void* b2,
                                  const void* gamma_next, void* Y, void* Yn, int M, int d, int ffn,
                                  float eps, float eps_next, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Number of tensor-core attention CTAs, since load on the current device, that
 * recomputed their query rows with the exact fp32 row routine because a V
 * tile held values the fp16 P.V pass cannot carry exactly (|v| >= 2^16,
 * inf/NaN, or a tile of values all below 2^-6 with some below 2^-17).
 * Synchronises the device. */
int pkb200_attention_exact_ctas(unsigned long long* count);

/* Counters of which implementation each entry point took since load:
 * out[0] tcgen05 GEMM launches, out[1] SIMT GEMM launches,
 * out[2] tcgen05 attention launches, out[3] SIMT attention launches,
 * out[4] other kernels. Returns the number of counters written (<= n). */
int pkb200_path_counters(long long* out, int n);

#ifdef __cplusplus
} /* extern "C" */

/* ---- reference-compatible C++ entry points (same names, argument order and
 * void return as kernels/generated/<op>.cu; errors are printed to stderr). */
#include <cuda_bf16.h>
void launch_rmsnorm(const __nv_bfloat16* input, const __nv_bfloat16* weight,
                    __nv_bfloat16* output, int rows, int cols, float epsilon, void* stream);
void launch_gelu(const __nv_bfloat16* input, __nv_bfloat16* output, int n, void* stream);
void launch_softmax(const __nv_bfloat16* input, __nv_bfloat16* output, int rows, int cols,
                    void* stream);
void launch_matmul(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M,
                   int N, int K, void* stream);
void launch_fused_rmsnorm_matmul(const __nv_bfloat16* input, const __nv_bfloat16* weight,
                                 __nv_bfloat16* output, int M, int N, int K, float epsilon,
                                 void* stream);
void launch_fused_matmul_bias_gelu(const __nv_bfloat16* a, const __nv_bfloat16* b,
                                   const __nv_bfloat16* bias, __nv_bfloat16* output, int M,
                                   int N, int K, void* stream);
void launch_attention_prefill(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                              const __nv_bfloat16* V, __nv_bfloat16* O, int B, int H, int S_q,
                              int S_kv, int D, float scale, int causal, void* stream);
void launch_kv_cache_update(const __nv_bfloat16* cache, const __nv_bfloat16* new_rows,
                            __nv_bfloat16* out, int B, int H, int S_cache, int S_new, int D,
                            void* stream);
void launch_matmul_int8(const __nv_bfloat16* A, const int8_t* Wq, const float* scale,
                        __nv_bfloat16* C, int M, int N, int K, void* stream);

/* Additive entries in the same style (new; the reference composes these
 * chains from the kernels above and golden primitives, tests/e2e/conftest.py:
 * 104-107): RMSNorm with gamma fused into the GEMM (golden.py:96-100), the
 * whole MLP block and its int8 weight-only variant (library-owned workspace),
 * and prefill attention appending the new K/V rows in place into a
 * preallocated [B, H, S_max, D] cache. */
void launch_fused_rmsnorm_matmul_gamma(const __nv_bfloat16* input, const __nv_bfloat16* weight,
                                       const __nv_bfloat16* gamma, __nv_bfloat16* output, int M,
                                       int N, int K, float epsilon, void* stream);
void launch_mlp_block(const __nv_bfloat16* X, const __nv_bfloat16* gamma,
                      const __nv_bfloat16* W1, const __nv_bfloat16* b1, const __nv_bfloat16* W2,
                      const __nv_bfloat16* b2, __nv_bfloat16* Y, int M, int d, int ffn, float eps,
                      void* stream);
void launch_mlp_block_int8(const __nv_bfloat16* X, const __nv_bfloat16* gamma,
                           const int8_t* W1q, const float* s1, const __nv_bfloat16* b1,
                           const int8_t* W2q, const float* s2, const __nv_bfloat16* b2,
                           __nv_bfloat16* Y, int M, int d, int ffn, float eps, void* stream);
void launch_attention_prefill_kv_append(const __nv_bfloat16* Q, const __nv_bfloat16* K_new,
                                        const __nv_bfloat16* V_new, __nv_bfloat16* K_cache,
                                        __nv_bfloat16* V_cache, __nv_bfloat16* O, int B, int H,
                                        int S_q, int S_cache, int S_max, int D, float scale,
                                        int causal, void* stream);
#endif

#endif /* PKB200_H */
