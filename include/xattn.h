/*
 * xattn.h -- C ABI of the B200 (sm_100a) cross-attention library `kernels.so`.
 *
 * O = softmax(Q K^T / sqrt(D)) V for Q[B][N_latent][D], K,V[B][N_input][D], row-major,
 * contiguous, device pointers owned by the caller.  Every launch is asynchronous on
 * `stream` (NULL = legacy default stream) and runs on the current device.
 *
 * Part 1 repeats, symbol for symbol and argument for argument, the entry points the
 * upstream project's ctypes wrapper binds (satyam19k/fast-cuda-cross-attention,
 * cuda_wrappers.py:83-175), so that project's cuda_wrappers.py, benchmark.py and
 * benchmark_batching.py load this library unchanged.  Like upstream they return void;
 * launch errors surface through cudaGetLastError() of the shared CUDA runtime (the
 * library links libcudart dynamically), and host-side argument errors through
 * xattn_last_error().
 *
 * Part 2 is new API: status-returning variants, caller-owned split partials, the bf16
 * multi-head entry, the pieces of the multi-GPU N_input merge, and diagnostics.
 */
#ifndef XATTN_H_
#define XATTN_H_

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- Part 1: upstream ABI */

/* Replaces launch_naive_kernel (kernel_naive.cu:68-89; bound at cuda_wrappers.py:83-94).
 * Same result as launch_optimized_kernel: all four fp32 names share one kernel family.  */
void launch_naive_kernel(const float* Q, const float* K, const float* V, float* output,
                         int batch_size, int N_latent, int N_input, int dim,
                         cudaStream_t stream);

/* Replaces launch_parallel_kernel (kernel_warp_parallel.cu:113-139; cuda_wrappers.py:96-107).
 * No shared-memory design limit: any N_input is accepted.                               */
void launch_parallel_kernel(const float* Q, const float* K, const float* V, float* output,
                            int batch_size, int N_latent, int N_input, int dim,
                            cudaStream_t stream);

/* Replaces launch_tiled_kernel (kernel_tiled.cu:169-186; cuda_wrappers.py:109-120).     */
void launch_tiled_kernel(const float* Q, const float* K, const float* V, float* output,
                         int batch_size, int N_latent, int N_input, int dim,
                         cudaStream_t stream);

/* Replaces launch_optimized_kernel (kernel_vectorized.cu:198-215; cuda_wrappers.py:122-133).
 * fp32 in/out, tcgen05 kind::tf32 tensor cores with fp32 accumulation; picks a key split
 * on its own when batch_size * N_latent is too small to fill the GPU (library-owned
 * workspace, allocated once per device and stream and grown on demand).
 * CUDA graphs: after one call on the device outside any capture (its one-time set-up),
 * calls can be captured on any stream; a workspace that captured work used is never
 * freed (it is retired, not freed, when the stream's workspace grows), so a graph stays
 * valid after later, larger calls.  Replays share that workspace with calls on the
 * stream the graph was captured on: order them on one stream.                          */
void launch_optimized_kernel(const float* Q, const float* K, const float* V, float* output,
                             int batch_size, int N_latent, int N_input, int dim,
                             cudaStream_t stream);

/* Replaces launch_wmma_kernel (kernel_wmma.cu:139-154; cuda_wrappers.py:136-146).
 * fp16 Q (already multiplied by 1/sqrt(dim) by the caller, cuda_wrappers.py:635-640),
 * fp16 K, V; fp32 output.  Any N_latent / N_input (upstream needs multiples of 16).
 * dim in {256, 512, 768}: tcgen05 kind::f16 tensor cores; other multiples of 64: the
 * fp16 values widened (exactly) to fp32 for the TF32 kernels.                           */
void launch_wmma_kernel(const __half* Q, const __half* K, const __half* V, float* output,
                        int batch_size, int N_latent, int N_input, int dim,
                        cudaStream_t stream);

/* Replaces launch_splitk_kernel (kernel_splitk.cu:238-251; cuda_wrappers.py:149-161).
 * Split s covers keys [s*c, min((s+1)*c, N_input)) with c = ceil(N_input/num_splits)
 * (kernel_splitk.cu:59-61).  Caller-owned scratch in the upstream layout:
 *   po [B][N_latent][num_splits][dim], pm, pl [B][N_latent][num_splits]  (fp32)
 * pm = max scaled score of the split (natural-log units), pl = sum exp(s - pm),
 * po = sum exp(s - pm) v; empty splits hold pm = -FLT_MAX, pl = 0, po = 0.
 * The merge divides by L exactly (upstream adds 1e-6, kernel_splitk.cu:225).           */
void launch_splitk_kernel(const float* Q, const float* K, const float* V, float* output,
                          float* po, float* pm, float* pl, int batch_size, int N_latent,
                          int N_input, int dim, int num_splits, cudaStream_t stream);

/* Replaces launch_wmma_splitk_kernel (kernel_wmma_splitk.cu:201-219; cuda_wrappers.py:164-175).
 * fp16 inputs as launch_wmma_kernel; split chunk rounded up to a multiple of 16 keys
 * (kernel_wmma_splitk.cu:52); scratch layout as launch_splitk_kernel.                  */
void launch_wmma_splitk_kernel(const __half* Q, const __half* K, const __half* V,
                               float* output, float* po, float* pm, float* pl, int batch_size,
                               int N_latent, int N_input, int dim, int num_splits,
                               cudaStream_t stream);

/* ---------------------------------------------------------------- Part 2: new API */

/* Status codes returned by the xattn_* functions and by xattn_last_error(). */
#define XATTN_OK 0
#define XATTN_ERR_ARG 1        /* negative size, null pointer, bad alignment           */
#define XATTN_ERR_LAUNCH 2     /* a kernel launch failed (see cudaGetLastError)         */
#define XATTN_ERR_NOMEM 3      /* the library workspace could not be grown              */
#define XATTN_ERR_DEVICE 4     /* a device wait timed out (see xattn_status)            */
#define XATTN_ERR_TOO_LARGE 5  /* the problem needs more scratch than the fixed array    */

/* Status-returning form of launch_optimized_kernel (no counterpart upstream).          */
int xattn_fp32(const float* Q, const float* K, const float* V, float* output, int batch_size,
               int N_latent, int N_input, int dim, cudaStream_t stream);

/* Unnormalised partial (m, l, O) of the keys this call sees, written with num_splits = 1
 * in the launch_splitk_kernel layout: po [B][N_latent][dim], pm, pl [B][N_latent].
 * Building block of the multi-GPU N_input split (no counterpart upstream).              */
int xattn_fp32_partial(const float* Q, const float* K, const float* V, float* po, float* pm,
                       float* pl, int batch_size, int N_latent, int N_input, int dim,
                       cudaStream_t stream);

/* Log-sum-exp merge of split partials into output (the combine half of
 * launch_splitk_kernel, kernel_splitk.cu:186-236), rows = B * N_latent.                 */
int xattn_combine(const float* po, const float* pm, const float* pl, float* output,
                  long long rows, int dim, int num_splits, cudaStream_t stream);

/* Multi-GPU N_input split merge, run on every rank between NCCL collectives:
 *   pack:     ol[r] = [po[r][0..dim), pl[r]]                     ([rows][dim+1] fp32)
 *   (all-reduce MAX of pm -> m_glob)
 *   rescale:  ol[r] *= exp(pm[r] - m_glob[r])
 *   (all-reduce SUM of ol)
 *   finalize: output[r] = ol[r][0..dim) / ol[r][dim]                                    */
int xattn_lse_pack(const float* po, const float* pl, float* ol, long long rows, int dim,
                   cudaStream_t stream);
int xattn_lse_rescale(float* ol, const float* pm, const float* m_glob, long long rows, int dim,
                      cudaStream_t stream);
int xattn_lse_finalize(const float* ol, float* output, long long rows, int dim,
                       cudaStream_t stream);

/* Multi-head bf16 cross attention (no counterpart upstream): Q [B][N_latent][H*dh],
 * K, V [B][N_input][H*dh], heads contiguous inside each row, per-head scale 1/sqrt(dh),
 * fp32 accumulation, bf16 output [B][N_latent][H*dh].  dh in {64, 96, 128} with 16-byte
 * aligned pointers runs on the tcgen05 kind::f16 kernel; other head sizes on the generic
 * CUDA-core kernel.                                                                    */
int xattn_bf16_mha(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                   __nv_bfloat16* output, int batch_size, int N_latent, int N_input,
                   int heads, int head_dim, cudaStream_t stream);

/* Plan of an xattn_fp32 / launch_optimized_kernel call on the current device for aligned
 * pointers: returns the number of kernels the call launches (1, or 2 with a key split
 * and its merge) and stores the key-split count in *num_splits (may be NULL).          */
int xattn_plan_fp32(int batch_size, int N_latent, int N_input, int dim, int* num_splits);

/* Split-K attention that allocates nothing.  No counterpart in the upstream project.
 *
 * Same key-split rule, kernels, result and tolerance as launch_splitk_kernel, but the caller
 * passes only Q, K, V and the output: the (m, l, O) partials live in one scratch array
 * compiled into the library (32 MiB plus 768 bytes of alignment room, held by every GPU
 * that loads the library until the process exits).  It is meant for callers that may not allocate device memory during a call:
 * programs that hand the whole GPU to their own memory pool at start-up, where an extra
 * cudaMalloc would fail or fragment that pool, and latency-critical loops that cannot
 * afford the device-wide synchronisation a cudaMalloc / cudaFree can cause.  (The
 * automatic split of launch_optimized_kernel grows a library workspace with cudaMalloc;
 * launch_splitk_kernel needs caller-allocated scratch.)
 *
 * Limit: batch_size * N_latent * num_splits * (dim + 2) floats <= 8,388,608 (32 MiB);
 * larger problems return XATTN_ERR_TOO_LARGE without launching anything.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  Every call on a device uses
 * the same array and leaves the last call's partials in it; nothing in it has to start at
 * zero (every partial a call reads, that call writes first).  Calls whose kernels overlap
 * on the GPU (different streams, or different host threads without ordering) race on the
 * array: order them on one stream.                                                      */
int xattn_splitk_noalloc(const float* Q, const float* K, const float* V, float* output,
                         int batch_size, int N_latent, int N_input, int dim, int num_splits,
                         cudaStream_t stream);

/* ---- Multi-GPU N_input split over peer memory (no counterpart upstream; the single-GPU
 * combine it generalises is kernel_splitk.cu:186-236).  One process per GPU of one node.
 *
 * Each rank allocates one exchange buffer with xattn_ipc_alloc, sends the 64-byte handle to
 * the other ranks (any host channel) and maps theirs with xattn_ipc_open (CUDA IPC over
 * NVLink; no multicast object).  The buffer layout for `rows` = B * N_latent rows of `dim`
 * floats comes from xattn_peer_layout (offsets in floats: pm, pl, po, out).  Per call, a
 * rank writes its partial (m, l, O) over its keys into pm / pl / po of its own buffer
 * (xattn_fp32_partial) and then calls xattn_peer_merge with every rank's mapped base
 * pointer (its own at index `rank`) and an epoch that grows by one per call (first call:
 * 1).  That one kernel waits until every rank's partials are written, merges its share
 * of the rows reading every rank's partials over NVLink, writes the merged rows into the
 * out region of every rank, and waits until every rank has done the same: when it
 * completes, out holds all rows on every rank and the buffers may be reused.  All ranks
 * must call it with the same rows, dim and epoch.  A rank that never arrives makes the
 * others give up after the device wait bound (status XATTN_ERR_DEVICE via xattn_status,
 * device code 9).  rank = -1 merges all rows of n_ranks buffers of this GPU in one launch
 * without barriers (single-process use and tests).                                      */
#define XATTN_IPC_HANDLE_BYTES 64
int xattn_ipc_alloc(size_t bytes, void** ptr, void* handle);
int xattn_ipc_open(const void* handle, void** ptr);
int xattn_ipc_close(void* ptr);
int xattn_ipc_free(void* ptr);
long long xattn_peer_layout(long long rows, int dim, long long* offsets);
int xattn_peer_merge(void* const* bases, int n_ranks, int rank, long long rows, int dim,
                     unsigned int epoch, cudaStream_t stream);

/* Host-side status of the most recent call on this thread (XATTN_* code).              */
int xattn_last_error(void);

/* Device status word: 0, or the code of the first bounded device wait that gave up.
 * Synchronises the current device.  clear != 0 resets it to 0.                          */
int xattn_status(int clear);

/* Options for tests and tuning.  key 1 = path: 0 auto, 1 tensor-core kernels only
 * (no automatic key split), 2 CUDA-core generic kernel.  key 2 = forced number of key
 * splits for the automatic fp32 path (0 = heuristic).  key 3 = device wait bound in
 * microseconds (default 2,000,000).  key 4 = TF32 truncation-bias compensation of the
 * tensor-core fp32 path (the tensor cores truncate fp32 operands to 10 mantissa bits):
 * 1 (default) measures, per work item, the least-squares relative truncation e_Q, e_K,
 * e_V of a sample of the inputs and scales the scores by (1 + e_Q + e_K) and the output
 * by (1 + e_V) -- exactly no compensation for inputs already exact in TF32 (widened bf16
 * or fp16, small integers); 2 applies the fixed constants for random mantissas,
 * e = 2^-11 / (2 ln 2) per operand, whatever the inputs; 0 turns it off.  key 5 = fp32 tensor-core kernel: 0 auto, 1 the
 * two-CTA kernel, 2 the four-CTA pair kernel (where the shape allows it).  key 6 = accurate
 * fp32 mode: 1 makes the non-split fp32 entries compute with 3xTF32 on the tensor cores
 * (two 3xTF32 GEMMs around an exact row softmax; max|dO| <= 1e-5 * max|O|; workspace of
 * 2 B N_latent N_input + B N_latent D + 2 B N_input D floats), 0 (default) the fused TF32
 * kernels.  Returns the previous value.                                                 */
int xattn_set_option(int key, int value);

/* Runs a kernel that waits on an mbarrier nothing will ever arrive on, with the wait
 * bound set to `bound_us`; returns the device status it produced (expected: the
 * injected-timeout code 99) and clears it.  Exercises the give-up path of every
 * bounded wait without faulting or hanging the GPU.                                    */
int xattn_selftest_timeout(int bound_us);

/* Library version: major * 10000 + minor * 100 + patch.                               */
int xattn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* XATTN_H_ */
