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
// y = W RMSNorm(x) (weights w1 = 1 + w') on the ring GEMV, which also writes
// RMSNorm(x) to xout for the kernels after it (MoE decode: router logits, then
// the experts read xout).  Q3XK_EUNSUPPORTED when the ring kernel cannot take
// the shape (the caller then runs the norm as its own kernel).
int gemv_rms_out(const q3xk_matrix* w, const float* x, const float* w1, float* y, float* xout, cudaStream_t s);

// ---- dequant-GEMM internals (gemm.cu) --------------------------------------------
// Expert-grouped tiles: X rows [xoff[e], xoff[e+1]) multiply expert e of a
// pool; tile_off[e] = first tile of expert e (tiles_w * ceil(count/64) each),
// tile_off[groups] = total.  Device arrays.
struct GemmGroups {
    int groups;
    const int* xoff;
    const int* tile_off;
};
// X (FP32 [T][K]) -> FP16 with a per-row power-of-two scale (tok_scale = 2^-s);
// x16lo != nullptr also gets the residual plane fp16(x 2^s - x16);
// counters != nullptr: zeroes the GEMM's split-K counters too.
int launch_x_to_f16(const float* x, int T, int K, __half* x16, __half* x16lo, float* tok_scale, cudaStream_t s,
                    int* counters = nullptr);
// Split-K scratch of a plain (non-grouped) GEMM call: partials and per-tile
// arrival counters (zero before the call, left zero after it).
struct GemmSplitWs {
    float* part;
    int* counters;
};
// Y[T][N] (+)= X16 W^T * tok_scale on tcgen05; `groups` selects the expert-grouped tiles
// (then W is a pool of groups experts and T the packed row count).  x16lo !=
// nullptr selects the split precision (X = x16 + x16lo, three MMAs per K-step).
// splitws != nullptr allows split-K for few-token calls.
int gemm_f16(const q3xk_matrix* w, const __half* x16, const __half* x16lo, const float* tok_scale, int T, float* y,
             int accumulate, const GemmGroups* groups, int bn_hint, cudaStream_t s,
             const GemmSplitWs* splitws = nullptr);
size_t gemm_grouped_tile_width();
// Resets the GEMM's device error word (bounded mbarrier waits that gave up).
int gemm_clear_error();

// MoE FFN over T prompt tokens on tcgen05 (moe.cu): router for all tokens,
// device top-k, pairs grouped by expert, grouped gate|up GEMM, weighted
// SwiGLU, grouped down GEMM, per-token sum of the slots added to hidden.
struct MoePrefillArgs {
    const q3xk_matrix* router;   // BF16 [E+1][H] (router rows + shared gate)
    const q3xk_matrix* gate_up;  // pool [E+1][2I][H], SwiGLU-interleaved rows
    const q3xk_matrix* down;     // pool [E+1][H][I]
    int experts, top_k, T;
    // Expert parallelism: the pools hold experts [e0, e0 + local) and the
    // shared expert at index `local`; shared_id = local where this GPU runs
    // the shared expert, else -1.  One GPU: e0 = 0, local = shared_id = E.
    int e0, local, shared_id;
    const float* x;  // RMSNorm(hidden) [T][H]
    float* hidden;   // [T][H]: += MoE output (accumulate = 1) or = (0)
    int accumulate;
    // work (device): sizes for P = T * (top_k + 1) pairs
    float* logits;       // [T][E+1]
    int* ids;            // [T][S]
    float* weights;      // [T][S]
    int *xoff, *tile_gu, *tile_dn;  // [E+2]
    int* pos;            // [P]
    int* pair_token;     // [P]
    float* pair_weight;  // [P]
    // FP16 planes: split precision keeps a residual plane after each
    // (x16 + T*H, x16g + P*H, h16 + P*I), FP16 precision only the first.
    __half* x16;         // [2][T][H]
    float* scale;        // [T]
    __half* x16g;        // [2][P][H]
    float* scale_g;      // [P]
    float* gu;           // [P][2I]
    __half* h16;         // [2][P][I]
    float* scale_h;      // [P]
    float* out;          // [P][H]
    bool split;          // split precision in the expert GEMMs
};
int moe_prefill(const MoePrefillArgs& a, cudaStream_t s);
// Top-k routing of T tokens (router_topk_kernel) with the expert-parallel id
// mapping of MoePrefillArgs (e0, local, shared_id).
int router_topk(const float* logits, int experts, int top_k, int T, int e0, int local, int shared_id, int* ids,
                float* weights, cudaStream_t s);

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
