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

int launch_embed(const q3xk_matrix& m, const int* tokens, int T, float* out, cudaStream_t s);
int launch_rms(const float* x, const float* w1, int n, int T, float* out, cudaStream_t s);
int launch_conv(float* proj, int64_t proj_stride, int T, int channels, const float* w, int CK, float* hist,
                cudaStream_t s);
int launch_delta(const float* proj, int64_t proj_stride, int T, const DeltaDims& dd, const float* alog,
                 const float* dt, const float* norm, float* state, float* out, int64_t out_stride,
                 cudaStream_t s);
int launch_attention(float* proj, int64_t proj_stride, int T, const AttnDims& ad, const float* qn1,
                     const float* kn1, const int* pos, float* kcache, float* vcache, int capacity, float* part,
                     int split_len, float* out, int64_t out_stride, cudaStream_t s);
int launch_ffn_swiglu(const float* proj, int64_t proj_stride, int T, int I, float* out, cudaStream_t s);
int launch_advance(int* pos, int by, cudaStream_t s);

}  // namespace q3xk
