/*
 * q3xk.h -- C ABI of the B200 (sm_100a) packed-weight matrix kernels.
 *
 * This is the thin launcher layer under the qwen3x backend interface
 * (internal.h:11-34 of qwen3x): plain pointers and sizes, no C++ or torch
 * types, so ctypes, cgo or a C++ backend can bind it directly.
 *
 * Conventions
 *   - All data pointers are DEVICE pointers unless a comment says otherwise.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *   - Every entry point returns a q3xk_status and never aborts; argument
 *     errors are detected on the host before any launch.
 *   - Activations, outputs and logits are FP32, as in the reference
 *     (README.md:83-86 of qwen3x).
 *
 * Device matrix layout ("row records").  The reference keeps model.bin's
 * packed blocks (34-byte Q8_0, 18-byte Q4_0; q8.h:10-15, q4.h:29-42) as they
 * are, which leaves them 2-byte aligned.  Here each row is one 16-byte-aligned
 * record, built once at upload by q3xk_repack():
 *   Q8_0: cols bytes of (q XOR 0x80), element k at byte k, then the row's
 *         cols/32 FP16 scales, padded to a multiple of 8 scales.
 *   Q4_0: cols/2 bytes: the 16 nibble bytes of each block unchanged (element
 *         i<16 = low nibble of byte i, i>=16 = high nibble of byte i-16), then
 *         the scales as above.
 *   BF16: cols*2 bytes, padded to 16 bytes.
 * Expert pools (MoE) are `experts` such matrices back to back.
 */
#ifndef Q3XK_H
#define Q3XK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3XK_ABI_VERSION 1

#if defined(__GNUC__)
#define Q3XK_API __attribute__((visibility("default")))
#else
#define Q3XK_API
#endif

typedef enum q3xk_status {
    Q3XK_OK = 0,
    Q3XK_EINVAL = 1,       /* bad shape, type, pointer or size */
    Q3XK_EUNSUPPORTED = 2, /* valid request this build does not implement */
    Q3XK_ECUDA = 3,        /* a CUDA runtime call or launch failed */
    Q3XK_EALIGN = 4,       /* a pointer or stride breaks the layout's alignment */
    Q3XK_ETIMEOUT = 5,     /* a bounded device-side wait gave up */
    Q3XK_EWORKSPACE = 6    /* caller-provided workspace too small */
} q3xk_status;

/* Matches q3x_model::MatrixType (model_config.h:16-20). */
typedef enum q3xk_matrix_type {
    Q3XK_BF16 = 0,
    Q3XK_Q8_0 = 1,
    Q3XK_Q4_0 = 2
} q3xk_matrix_type;

/* One device matrix (or expert pool) in row-record layout. */
typedef struct q3xk_matrix {
    void* data;            /* device pointer, 256-byte aligned */
    int64_t row_stride;    /* bytes between row records, multiple of 16 */
    int64_t expert_stride; /* bytes between expert matrices (rows*row_stride) */
    int32_t type;          /* q3xk_matrix_type */
    int32_t rows;          /* output features per expert */
    int32_t cols;          /* input features (K); multiple of 32 if quantized */
    int32_t experts;       /* 1 for a plain matrix */
} q3xk_matrix;

/* Human-readable name of a status code (static string). */
Q3XK_API const char* q3xk_status_string(int status);
Q3XK_API int q3xk_abi_version(void);

/*
 * Size of a matrix in model.bin's packed format.  Replaces
 * q3x_cpu::quantized_bytes (arch/cpu.cpp:161-179) with the same rules:
 * Q8_0/Q4_0 only, rows > 0, cols > 0, cols % 32 == 0, overflow-checked;
 * returns Q3XK_EINVAL and leaves *bytes untouched otherwise.
 */
Q3XK_API int q3xk_quantized_bytes(int type, int rows, int cols, size_t* bytes);

/*
 * Fill row_stride/expert_stride/type/rows/cols/experts of *m (data is left
 * as is) and the device bytes the row-record layout needs.  Replaces the
 * pointer binding of Model::load (engine.cu:2007-2026 `take`).
 */
Q3XK_API int q3xk_matrix_layout(int type, int rows, int cols, int experts,
                       q3xk_matrix* m, size_t* device_bytes);

/*
 * Build the row-record layout in m->data from `packed`, a DEVICE copy of the
 * matrix exactly as stored in model.bin (all experts, back to back).
 * Replaces the whole-file cudaMemcpy of Model::load (engine.cu:2074-2079),
 * after which the reference kernels read the 34/18-byte blocks in place.
 */
Q3XK_API int q3xk_repack(const q3xk_matrix* m, const void* packed, void* stream);

/*
 * Decode GEMV: y[rows] = W x (accumulate = 0) or y[rows] += W x
 * (accumulate != 0).  x: cols FP32, y: rows FP32, both 16-byte aligned; x
 * and y must not overlap.  CUDA cores only (HBM-bound).
 * Replaces engine.cu:1531-1561 mv()/mv_add() (kernels mv_q8_kernel,
 * mv_add_q8_kernel, mv_q4_kernel, mv_add_q4_kernel, mv_kernel at
 * engine.cu:519-612) and, for the CPU engine, q3x_cpu::try_mv
 * (arch/cpu.cpp:192-226) as called from engine.cpp:207-212.
 */
Q3XK_API int q3xk_gemv(const q3xk_matrix* w, const float* x, float* y, int accumulate,
              void* stream);

/*
 * Input transforms for the _ex GEMVs: the elementwise pass that produces a
 * GEMV's input in the reference is applied while the GEMV stages x, so the
 * intermediate vector is never written.  No counterpart in the reference
 * (which runs these as separate loops / kernels); each follows its formula:
 *   RMS        x[k] * rsqrt(mean(x^2) + 1e-6) * w[k], w = 1 + w'     engine.cpp:231-236
 *   GATED_RMS  per group of `group` elements:
 *              x[k] * (rsqrt(mean_g(x^2) + 1e-6) * w[k % group] * silu(z[k]))
 *                                                                 engine.cpp:237-242
 *   SWIGLU     x holds [g | u] pairs of width `group` (one pair per segment):
 *              silu(g[i]) * u[i], times seg_weights[s] when given  engine.cpp:374, :415-416
 * Limits: GATED_RMS needs cols % group == 0 and cols / group <= 64 (plain
 * GEMV only); SWIGLU's group must equal the matrix's cols.
 */
typedef enum q3xk_xform_kind {
    Q3XK_XFORM_NONE = 0,
    Q3XK_XFORM_RMS = 1,
    Q3XK_XFORM_GATED_RMS = 2,
    Q3XK_XFORM_SWIGLU = 3
} q3xk_xform_kind;

typedef struct q3xk_xform {
    int32_t kind;             /* q3xk_xform_kind */
    int32_t group;            /* GATED_RMS group size; SWIGLU pair width */
    const float* w;           /* RMS: 1 + w' [cols]; GATED_RMS: norm [group] */
    const float* z;           /* GATED_RMS: gate [cols] */
    const float* seg_weights; /* SWIGLU: one weight per segment, or NULL */
} q3xk_xform;

/* q3xk_gemv / q3xk_expert_gemv_rows / q3xk_expert_gemv_segments with an
 * input transform (xf may be NULL = none). */
Q3XK_API int q3xk_gemv_ex(const q3xk_matrix* w, const float* x, float* y, int accumulate,
                          const q3xk_xform* xf, void* stream);
Q3XK_API int q3xk_expert_gemv_rows_ex(const q3xk_matrix* pool, const int* ids, int slots, const float* x,
                                      float* y, int accumulate, const q3xk_xform* xf, void* stream);
Q3XK_API int q3xk_expert_gemv_segments_ex(const q3xk_matrix* pool, const int* ids, int slots,
                                          const float* x, float* y, int accumulate, const q3xk_xform* xf,
                                          void* stream);

/*
 * GEMV of one expert of a pool: y = W[expert] x.  `expert` is a host int.
 * Replaces engine.cpp:214-224 expert_mv.
 */
Q3XK_API int q3xk_expert_gemv(const q3xk_matrix* w, int expert, const float* x, float* y,
                     int accumulate, void* stream);

/*
 * Grouped expert GEMVs over an expert pool (MoE decode), expert ids read on
 * the device so a whole layer stays inside one CUDA graph:
 *   rows:     y[s * pool->rows + r] (+)= W[ids[s]][r] . x          (s < slots)
 *   segments: y[r] (+)= sum_s W[ids[s]][r] . x[s * cols .. (s+1) * cols)
 * `ids` (int32) and x, y are device pointers; slots <= 16 for segments.
 * An id < 0 skips its slot (expert parallelism: an expert held by another
 * GPU): rows leaves that slot's y rows untouched and reads none of its
 * weights; segments adds nothing for it and never reads that segment of x
 * as data.  With every slot skipped, segments writes y = 0 (or leaves y).
 * Replace expert_gate_up_q4_kernel (rows) and expert_down_weighted_q4_kernel
 * (segments, weights folded into x; engine.cu:1186-1250) and the CPU loop of
 * engine.cpp:412-420.
 */
Q3XK_API int q3xk_expert_gemv_rows(const q3xk_matrix* pool, const int* ids, int slots, const float* x,
                                   float* y, int accumulate, void* stream);
Q3XK_API int q3xk_expert_gemv_segments(const q3xk_matrix* pool, const int* ids, int slots,
                                       const float* x, float* y, int accumulate, void* stream);

/*
 * Router of one token (engine.cpp:377-405; replaces router_top_k_kernel,
 * engine.cu:1153-1184): softmax over logits[0..experts), greedy top_k
 * (strict '>', the lowest id wins a tie), weights renormalised over the
 * selected slots.  With with_shared != 0, logits[experts] is the shared-expert
 * gate and slot top_k gets id `experts` and weight sigmoid(logit)
 * (engine.cpp:427-429).  One warp; experts <= 512, top_k <= 8.
 */
Q3XK_API int q3xk_router_topk(const float* logits, int experts, int top_k, int with_shared, int* ids,
                              float* weights, void* stream);

/* out[s][i] = w[s] * silu(g) * u with [g | u] = gate_up[s] (w may be NULL);
 * engine.cpp:415-416, :424-425. */
Q3XK_API int q3xk_swiglu(const float* gate_up, const float* weights, int slots, int width, float* out,
                         void* stream);

/* First index of the maximum of values[0..n) into *out_index (device int);
 * replaces the host scan of state_argmax (engine.cu:2339-2350). */
Q3XK_API int q3xk_argmax_workspace_bytes(size_t* bytes);
Q3XK_API int q3xk_argmax(const float* values, int n, int* out_index, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Prefill dequant-GEMM on tcgen05: Y[T, rows] = X[T, cols] W^T (accumulate =
 * 0) or Y += X W^T, all row-major FP32 (Y[t][r] at t * rows + r).  Q8_0/Q4_0
 * only; cols % 32 == 0.  FP32 accumulation in tensor memory; X is scaled per
 * token by a power of two.  Two precisions:
 *   Q3XK_GEMM_SPLIT (q3xk_gemm's): X and d*q each as two FP16 planes (hi +
 *     residual; d*q is split exactly), three MMAs per K-step: FP32-grade,
 *     error ~1e-7 of sum_k |w x|.
 *   Q3XK_GEMM_FP16: X and d*q rounded to FP16, one MMA per K-step: error
 *     ~1e-4 of sum_k |w x|, about 1.5x the throughput.
 * `workspace` is a caller-owned DEVICE buffer of
 * q3xk_gemm_workspace_bytes(T, cols) bytes, 256-byte aligned (either
 * precision).
 * Replaces engine.cu:1568-1597 batch_mv (batch_mv_q8_kernel, engine.cu:751-
 * 839) and adds the Q4_0 prefill the reference asserts on (engine.cu:1580).
 */
#define Q3XK_GEMM_SPLIT 0
#define Q3XK_GEMM_FP16 1
Q3XK_API int q3xk_gemm_workspace_bytes(int T, int cols, size_t* bytes);
Q3XK_API int q3xk_gemm(const q3xk_matrix* w, const float* x, int T, float* y, int accumulate,
                       void* workspace, size_t workspace_bytes, void* stream);
Q3XK_API int q3xk_gemm_ex(const q3xk_matrix* w, const float* x, int T, float* y, int accumulate,
                          int precision, void* workspace, size_t workspace_bytes, void* stream);
/* Device error word of the GEMM kernels (bit 0: a bounded wait gave up). */
Q3XK_API int q3xk_gemm_device_error(int* flags);

/*
 * Synchronous GEMV on HOST vectors, the contract of q3x_cpu::try_mv
 * (arch/cpu.cpp:192-226): y_host is complete when the call returns.  The
 * matrix stays resident on the device; x_host (cols floats) goes up and
 * y_host (rows floats) comes back on `stream` (pinned host memory makes the
 * copies asynchronous DMA).  `workspace` is a caller-owned DEVICE buffer of
 * at least (cols + rows) * 4 bytes, 16-byte aligned: nothing is allocated.
 */
Q3XK_API int q3xk_try_mv_host(const q3xk_matrix* w, const float* x_host, float* y_host,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * q3xk_try_mv_host without a workspace: no allocation at any time.  For
 * callers that cannot hand over device memory -- code written against the
 * reference's q3x_cpu::try_mv(w, type, rows, cols, x, y), whose signature has
 * no workspace argument, and FFI hosts that hold no CUDA allocator -- and that
 * should not pay a cudaMalloc/cudaFree (an implicit device synchronisation)
 * on every matvec.  No counterpart in the reference.
 *
 * x and y are staged in a fixed device array inside libq3xk.so of 4 MiB per
 * device: cols rounded up to 4, plus rows, must not exceed 1048576 floats,
 * otherwise Q3XK_EWORKSPACE is returned before any CUDA call.  The first call
 * on a device (the current one) looks the array's address up with
 * cudaGetSymbolAddress; make it before any stream capture.  The address is
 * kept per device and CUDA context: after cudaDeviceReset (a new context) the
 * next call looks it up again.  The array is
 * shared: calls whose work overlaps on the GPU (other streams or host threads
 * on the same device) race on it, so run them one at a time.  Nothing in it
 * needs to start at zero: each call overwrites the x and y it reads.
 */
Q3XK_API int q3xk_try_mv_host_noalloc(const q3xk_matrix* w, const float* x_host, float* y_host,
                                      void* stream);

/*
 * Device-side error word of the current device: bit 0 = a wait inside the
 * dequant-GEMM's pipeline (TMA producer, dequantisers, MMA issuer or
 * epilogue, each on an mbarrier) gave up.  The GEMVs have no device-side
 * waits.  Every such wait is bounded (about one second); on a timeout the
 * kernel sets the bit and its CTA leaves its tile loop, so the context stays
 * usable.  Reading synchronises the device; clearing resets the word.
 * (The peer all-reduce has an error word per State: q3xb_state_tp_error.)
 */
Q3XK_API int q3xk_device_error(int* flags);
Q3XK_API int q3xk_clear_device_error(void);

/*
 * One-shot all-reduce of a short vector over peer memory (decode-sized:
 * n <= 5120 floats, up to 8 ranks), the collective of the multi-GPU backend's
 * decode step: y[0..n) += the sum over ranks of partial[0..n), added in rank
 * order, so every rank gets bit-identical results.  bases[r] = rank r's
 * buffer of q3xk_peer_buffer_bytes(n_max) bytes (this rank's own one, zeroed
 * before first use, and the peers' mapped with CUDA IPC); seq = a device int,
 * zero at first, advanced by each call; err = a device int.  Each rank waits
 * for the others' flags at most timeout_s seconds (0 < timeout_s <= 60);
 * then it sets *err = 1, leaves y alone and returns, and every later call
 * with *err set returns at once.  No counterpart in the reference
 * (single-GPU backends only).
 */
Q3XK_API size_t q3xk_peer_buffer_bytes(int n_max);
Q3XK_API int q3xk_peer_allreduce_add(void* const* bases, int rank, int world, int n_max, int* seq,
                                     const float* partial, float* y, int n, int* err, double timeout_s,
                                     void* stream);

/*
 * Kernel family of the plain Q8_0 / Q4_0 GEMVs (q3xk_gemv, q3xk_gemv_ex
 * without a transform, q3xk_expert_gemv, q3xk_try_mv_host*):
 *   0  automatic (default): the shared-memory ring kernel where its staging
 *      fits (x prescaled plus a ~140-210 KB ring per SM; 24 warps per CTA
 *      for Q8_0 matrices of up to one 4-row group per warp, else 16), else
 *      the register one
 *   1  register batches (128-bit loads held in registers)
 *   2  ring, 16 warps per CTA     3  ring, 24 warps per CTA (20 for Q4_0)
 * Process-wide; meant for tests and measurements that compare the families
 * on the same inputs.  Results of every family meet the same parity bar.
 * No counterpart in the reference.
 */
Q3XK_API int q3xk_gemv_set_family(int family);

/* Number of kernel launches the calls above made since the last reset
 * (host-side counter used by the benchmark's gpu_launches report). */
Q3XK_API uint64_t q3xk_launch_count(void);
Q3XK_API void q3xk_reset_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
