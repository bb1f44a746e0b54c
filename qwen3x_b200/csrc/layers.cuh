// layers.cuh -- launchers of the decoder's non-matrix steps (layers.cu).
#pragma once

#include "common.cuh"

namespace q3xk {

// Offsets inside a DeltaNet projection row [qkv (DQKV) | z (DO) | a (VH) | b (VH)].
struct DeltaDims {
    int KH, VH, KD, VD;
    int z_off, a_off, b_off;
};

// Attention projection row [q+gate (2 AH AD) | k (KVH AD) | v (KVH AD)].
struct AttnDims {
    int AH, KVH, AD, RD;
};

// Repack `src_rows` packed rows of [gate (half) | up (half)] matrices (one
// per 2*half source rows, counted from row_offset) into m's rows with the
// SwiGLU interleave g(2j) g(2j+1) u(2j) u(2j+1) (layout.cu).
int repack_swiglu(const q3xk_matrix* m, const void* packed, int64_t src_rows, int half, int row_offset,
                  cudaStream_t s);

// GEMV whose epilogue applies SwiGLU to the interleaved rows: y[i] =
// (w[slot] *) silu(g_i) * u_i, rows/2 outputs (gemv.cu).  ids/rows mode when
// ids != nullptr (MoE gate|up of the selected experts; w per slot).
int gemv_swiglu(const q3xk_matrix* w, const float* x, float* y, const int* ids, int slots, const float* slot_w,
                const q3xk_xform* xf, cudaStream_t s);

int launch_embed(const q3xk_matrix& m, const int* tokens, int T, float* out, cudaStream_t s);
int launch_rms(const float* x, const float* w1, int n, int T, float* out, cudaStream_t s);
int launch_conv(float* proj, int64_t proj_stride, int T, int channels, const float* w, int CK, float* hist,
                cudaStream_t s);
// norm == nullptr: write the raw delta-rule output (the gated RMS is then
// applied by the consumer, q3xk_gemv_ex with Q3XK_XFORM_GATED_RMS).
// conv_w/hist given (T = 1, CK = 4): the causal conv runs inside the kernel
// on the raw projections (no launch_conv before it); group_count is a device
// int[KH], zero between launches (the kernel leaves it zero).
int launch_delta(const float* proj, int64_t proj_stride, int T, const DeltaDims& dd, const float* alog,
                 const float* dt, const float* norm, float* state, float* out, int64_t out_stride,
                 cudaStream_t s, const float* conv_w = nullptr, float* hist = nullptr, int CK = 0,
                 int* group_count = nullptr);
// Chunked gated DeltaNet over T > 1 tokens (delta.cu): same results as
// launch_delta with a norm, in parallel over 64-token chunks.  q | k | v come
// from `qkv` (the conv output, launch_conv_prefill), a, b, z from `proj`.
// `work` holds delta_chunked_workspace_bytes(T, VH) bytes.
size_t delta_chunked_workspace_bytes(int T, int VH);
int launch_delta_chunked(const float* qkv, int64_t qkv_stride, const float* proj, int64_t proj_stride, int T,
                         const DeltaDims& dd, const float* alog, const float* dt, const float* norm, float* state,
                         float* out, int64_t out_stride, float* work, cudaStream_t s);
// Causal conv1d + SiLU over T tokens, out of place (out[t][c], stride
// `channels`), parallel over 64-token segments; updates the history.
int launch_conv_prefill(const float* proj, int64_t proj_stride, int T, int channels, const float* w, int CK,
                        float* hist, float* out, cudaStream_t s);
int launch_attention(float* proj, int64_t proj_stride, int T, const AttnDims& ad, const float* qn1,
                     const float* kn1, const int* pos, float* kcache, float* vcache, int capacity, float* part,
                     int split_len, float* out, int64_t out_stride, cudaStream_t s);
int launch_ffn_swiglu(const float* proj, int64_t proj_stride, int T, int I, float* out, cudaStream_t s);
int launch_advance(int* pos, int by, cudaStream_t s);

}  // namespace q3xk
