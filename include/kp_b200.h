/*
 * kp_b200.h -- C ABI of the B200 (sm_100a) kernels behind torch.ops.kp.*.
 *
 * Each entry point replaces one host launcher of kernelpilot's csrc/launchers.h
 * (cited per function) with the same argument order and meaning: an integer
 * `variant` (the optimisation stage, highest = tuned B200 kernel), an element type,
 * plain device pointers, int64 sizes and the raw cudaStream_t as `void*`.
 * Differences from the reference launchers:
 *   - extern "C", no C++ types, usable from ctypes / cffi / any FFI;
 *   - failures return a non-zero status instead of throwing std::runtime_error
 *     (csrc/compat.h:28-36); kpb_last_error() gives the message;
 *   - KPB_BF16 joins the reference's DType::F32 = 0 / DType::F16 = 1
 *     (csrc/launchers.h:10), with the same numeric values;
 *   - attention_causal is new (the reference has only non-causal attention).
 * Every call is asynchronous on `stream` (never synchronises), reads its inputs
 * and writes only its outputs and, where stated, a caller-provided workspace.
 */
#ifndef KP_B200_H
#define KP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types: kp::DType values (csrc/launchers.h:10) plus bf16 */
#define KPB_F32 0
#define KPB_F16 1
#define KPB_BF16 2

/* status codes */
#define KPB_OK 0
#define KPB_EINVAL 1       /* bad argument: variant, dtype, size, null pointer, alignment */
#define KPB_EUNSUPPORTED 2 /* valid request this build has no kernel for */
#define KPB_ECUDA 3        /* a CUDA runtime call or kernel launch failed */

/* Message of the last failed call on this thread ("" if none). */
const char* kpb_last_error(void);

/* ABI version (major*100 + minor). */
int kpb_version(void);

/* Number of variants of an op ("vector_add", "reduce_sum", "softmax", "matmul",
 * "layernorm", "attention", "attention_causal"), or -1 for an unknown name. Mirrors
 * check_variant's counts (csrc/bindings.cpp:30-33, :77, :111). */
int kpb_num_variants(const char* op);

/* Error bits that kernels on the current device recorded since the last call
 * (bit 0 = a bounded wait inside a kernel gave up), then cleared. No counterpart in
 * the reference, whose kernels have no waits. Synchronous; for tests and health
 * checks, not hot paths. */
int kpb_device_errors(unsigned* bits);

/* ---- elementwise add: replaces kp::vector_add (csrc/launchers.h:12-13) ----
 * c[i] = a[i] + b[i] for i < n, added in fp32 and rounded to the dtype. a, b, c must
 * be element-aligned; the fast variant needs no further alignment. */
int kpb_vector_add(int variant, int dtype, const void* a, const void* b, void* c, int64_t n,
                   void* stream);

/* ---- full sum: replaces kp::reduce_sum (csrc/launchers.h:14-15) ----
 * out[0] = sum of x[0..n) accumulated in fp32. Unlike the reference, `out` need not
 * be zero-initialised: it is overwritten (a zeroed `out` gives the same result).
 * The result is deterministic: per-CTA partials are combined in a fixed order.
 * kpb_reduce_sum takes its partials buffer from a stream-ordered pool the library
 * keeps per device (allocated and freed on `stream`; the pool keeps its memory
 * between calls); kpb_reduce_sum_ws takes it from the caller instead. */
int kpb_reduce_sum(int variant, int dtype, const void* x, float* out, int64_t n,
                   void* stream);
size_t kpb_reduce_sum_workspace_bytes(int variant, int64_t n);
int kpb_reduce_sum_ws(int variant, int dtype, const void* x, float* out, int64_t n,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- full sum without allocation: no counterpart in the reference ----
 * Same result as kpb_reduce_sum(2, ...) (the persistent kernel), for callers that may
 * not allocate device memory when they call (a fixed start-up budget, memory owned by
 * another allocator, no allocation after initialisation). The per-CTA partials live
 * in a 16 KB array built into the library (held by every GPU that loads it until
 * exit); calls needing more than 4096 partials are rejected with KPB_EINVAL. The
 * first call on a device looks up the array's address: make it before any stream
 * capture. All calls on a device share the array, so calls that overlap on the GPU
 * race; order them on one stream. No cudaMalloc/cudaFree or allocating library call
 * is made. */
int kpb_reduce_sum_noalloc(int dtype, const void* x, float* out, int64_t n, void* stream);

/* ---- full sum over the GPUs of one node, exchange in the kernel: replaces the
 * all_reduce step of the data-parallel reduction (the reference has no multi-GPU
 * code; on one GPU its reduction ends in atomicAdd, csrc/kernels/reduction.hip:86) ----
 * One process per GPU, each holding its shard of the vector. Once per process:
 * kpb_peer_sum_create exports this rank's small exchange buffer as a CUDA IPC handle
 * (kpb_peer_sum_handle_bytes() bytes); the caller gathers every rank's handle in rank
 * order (any host-side all_gather) and passes them to kpb_peer_sum_connect. Then every
 * rank calls kpb_peer_sum_run the same number of times, in the same order, all calls
 * of a rank on one stream: each call reduces the local shard (the persistent kernel;
 * partials in the caller's workspace of kpb_peer_sum_workspace_bytes(n) bytes) and
 * its one-CTA finishing kernel stores the local sum into every rank's buffer over
 * NVLink, waits (bounded) for the other ranks' sums and writes out[0] = sum over
 * ranks in rank order: the same bits on every rank. The call number is kept in device
 * memory and advanced by the kernel, so a CUDA graph holding the call can be replayed
 * (every rank replaying the same number of times). A rank that never arrives makes
 * the others set the timeout bit of kpb_device_errors(), write NaN and mark their
 * exchange out of step; from then on every call writes NaN at once.
 * kpb_peer_sum_status (synchronous) reports that mark. Call kpb_peer_sum_destroy only
 * once every rank's calls have completed (a device synchronise and a barrier across
 * the ranks), since the peers store into this rank's buffer. At most 8 ranks; all on
 * one node with peer access (NVLink/NVSwitch). */
typedef struct kpb_peer_sum kpb_peer_sum;
size_t kpb_peer_sum_handle_bytes(void);
int kpb_peer_sum_create(int rank, int world, void* ipc_handle_out, kpb_peer_sum** out);
int kpb_peer_sum_connect(kpb_peer_sum* ps, const void* all_handles);
size_t kpb_peer_sum_workspace_bytes(int64_t n);
int kpb_peer_sum_run(kpb_peer_sum* ps, int dtype, const void* x, float* out, int64_t n,
                     void* workspace, size_t workspace_bytes, void* stream);
int kpb_peer_sum_status(kpb_peer_sum* ps, int* out_of_step);
int kpb_peer_sum_destroy(kpb_peer_sum* ps);

/* ---- row softmax: replaces kp::softmax (csrc/launchers.h:17-18) ----
 * y = softmax(x) over the last dimension of a contiguous (M, N) matrix;
 * fp32 math for every dtype; M, N < 2^31. */
int kpb_softmax(int variant, int dtype, const void* x, void* y, int64_t M, int64_t N,
                void* stream);

/* ---- GEMM: replaces kp::matmul (csrc/launchers.h:20-22) ----
 * C = A @ B, row-major A (M, K), B (K, N), C (M, N); fp32 accumulation, output in
 * the input dtype; K == 0 writes zeros. kpb_matmul obtains any staging buffer it
 * needs (a 16-byte-aligned copy of B when N*elem is not a multiple of 16) from
 * the library's stream-ordered pool; kpb_matmul_ws takes it from the caller. */
int kpb_matmul(int variant, int dtype, const void* A, const void* B, void* C, int64_t M,
               int64_t N, int64_t K, void* stream);
size_t kpb_matmul_workspace_bytes(int variant, int dtype, int64_t M, int64_t N, int64_t K);
int kpb_matmul_ws(int variant, int dtype, const void* A, const void* B, void* C, int64_t M,
                  int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ---- LayerNorm: replaces kp::layernorm (csrc/launchers.h:25-27) ----
 * y = (x - mean) / sqrt(var + eps) * w + b over the last dimension of a contiguous
 * (M, N) matrix; w, b have N elements; biased variance; fp32 statistics for every
 * dtype; M, N < 2^31. eps is used as given (the reference does not check it). */
int kpb_layernorm(int variant, int dtype, const void* x, const void* w, const void* b, void* y,
                  int64_t M, int64_t N, float eps, void* stream);

/* ---- attention forward: replaces kp::attention (csrc/launchers.h:28-30) ----
 * o = softmax(q k^T / sqrt(D)) v on contiguous (BH, S, D) q, k, v, o;
 * fp32 softmax statistics; D <= 256, BH < 65536 (csrc/bindings.cpp:109). */
int kpb_attention(int variant, int dtype, const void* q, const void* k, const void* v,
                  void* o, int64_t BH, int64_t S, int64_t D, void* stream);

/* ---- causal attention forward: new; same contract with key j > query i masked ---- */
int kpb_attention_causal(int variant, int dtype, const void* q, const void* k,
                         const void* v, void* o, int64_t BH, int64_t S, int64_t D,
                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KP_B200_H */
