// moe.cu -- MoE routing and the small kernels around the grouped expert GEMVs.
//
// The reference routes one token with a single-threaded kernel
// (router_top_k_kernel<<<1,1>>>, engine.cu:1153-1184) and runs the routed
// experts as expert_gate_up_q4_kernel / expert_swiglu_kernel /
// expert_down_weighted_q4_kernel (engine.cu:1186-1250).  Here:
//   router_topk   one warp: softmax, greedy top-k (strict '>', lowest id wins
//                 a tie, engine.cpp:377-405), renormalised weights, and the
//                 shared-expert gate sigmoid(l) as an extra slot;
//   swiglu        h[s] = w_s * silu(g_s) * u_s, the weighted input of the
//                 segment-gather down projection (q3xk_expert_gemv_segments);
//   argmax        first index of the maximum (engine.cpp:601-605), computed
//                 on the device instead of copying 248320 logits to the host.
#include <float.h>

#include "common.cuh"

namespace q3xk {
namespace {

constexpr int kMaxPerLane = 16;  // experts <= 512


__global__ void __launch_bounds__(32) router_topk_kernel(const float* __restrict__ logits, int experts, int top_k,
                                                         int with_shared, int* __restrict__ ids,
                                                         float* __restrict__ weights) {
    griddep_wait();
    griddep_launch_dependents();
    const int lane = threadIdx.x;
    float p[kMaxPerLane];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = lane + 32 * j;
        p[j] = e < experts ? logits[e] : -INFINITY;
        mx = fmaxf(mx, p[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = lane + 32 * j;
        p[j] = e < experts ? expf(p[j] - mx) : 0.f;
        total += p[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) p[j] = p[j] / total;

    uint32_t used = 0;  // bit j: expert lane + 32 j already selected
    float selected_total = 0.f;
    float chosen_p[8];
    int chosen_id[8];
    for (int slot = 0; slot < top_k; ++slot) {
        float bv = -1.f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int e = lane + 32 * j;
            if (e < experts && !((used >> j) & 1u) && p[j] > bv) { bv = p[j]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if ((bi & 31) == lane) used |= 1u << (bi >> 5);
        chosen_p[slot] = bv;
        chosen_id[slot] = bi;
        selected_total += bv;  // slot order, as the reference
    }
    if (lane == 0) {
        for (int slot = 0; slot < top_k; ++slot) {
            ids[slot] = chosen_id[slot];
            weights[slot] = chosen_p[slot] / selected_total;
        }
        if (with_shared) {
            ids[top_k] = experts;  // the shared expert is stored as expert `experts` of each pool
            weights[top_k] = sigmoid_ref(logits[experts]);
        }
    }
}

// h[s][i] = w[s] * silu(g[s][i]) * u[s][i]; gate_up[s] = [g (width) | u (width)].
__global__ void swiglu_kernel(const float* __restrict__ gate_up, const float* __restrict__ w, int slots, int width,
                              float* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    const int64_t n = (int64_t)slots * width;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int s = (int)(t / width), i = (int)(t - (int64_t)s * width);
        const float g = gate_up[(int64_t)s * 2 * width + i];
        const float u = gate_up[(int64_t)s * 2 * width + width + i];
        const float h = g * sigmoid_ref(g) * u;  // engine.cpp:191 silu, then * up
        out[t] = w ? w[s] * h : h;
    }
}

struct ArgBest {
    float v;
    int i;
};

__device__ __forceinline__ ArgBest better(ArgBest a, ArgBest b) {
    // std::max_element: the first index of the largest value.
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ __forceinline__ ArgBest block_best(ArgBest b) {
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest other{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
        b = better(b, other);
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[w] = b.v; si[w] = b.i; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        b = lane < nw ? ArgBest{sv[lane], si[lane]} : ArgBest{-INFINITY, 0x7fffffff};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ArgBest other{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
            b = better(b, other);
        }
    }
    return b;
}

__global__ void __launch_bounds__(512) argmax_partial_kernel(const float* __restrict__ v, int n,
                                                             ArgBest* __restrict__ part) {
    griddep_wait();
    griddep_launch_dependents();
    ArgBest b{-INFINITY, 0x7fffffff};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        b = better(b, ArgBest{v[i], i});
    b = block_best(b);
    if (threadIdx.x == 0) part[blockIdx.x] = b;
}

__global__ void __launch_bounds__(512) argmax_final_kernel(const ArgBest* __restrict__ part, int parts,
                                                           int* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    ArgBest b{-INFINITY, 0x7fffffff};
    for (int i = threadIdx.x; i < parts; i += blockDim.x) b = better(b, part[i]);
    b = block_best(b);
    if (threadIdx.x == 0) *out = b.i == 0x7fffffff ? 0 : b.i;
}

constexpr int kArgmaxParts = 148;

}  // namespace
}  // namespace q3xk

using namespace q3xk;

extern "C" {

int q3xk_router_topk(const float* logits, int experts, int top_k, int with_shared, int* ids, float* weights,
                     void* stream) {
    if (!logits || !ids || !weights || experts <= 0 || experts > 32 * kMaxPerLane || top_k <= 0 ||
        top_k > 8 || top_k > experts)
        return Q3XK_EINVAL;
    const cudaError_t e = launch_pdl(router_topk_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                                     logits, experts, top_k, with_shared ? 1 : 0, ids, weights);
    if (e != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int q3xk_swiglu(const float* gate_up, const float* weights, int slots, int width, float* out, void* stream) {
    if (!gate_up || !out || slots <= 0 || width <= 0) return Q3XK_EINVAL;
    const int64_t n = (int64_t)slots * width;
    const int blocks = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
    const cudaError_t e = launch_pdl(swiglu_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                                     gate_up, weights, slots, width, out);
    if (e != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int q3xk_argmax_workspace_bytes(size_t* bytes) {
    if (!bytes) return Q3XK_EINVAL;
    *bytes = sizeof(ArgBest) * kArgmaxParts;
    return Q3XK_OK;
}

int q3xk_argmax(const float* values, int n, int* out_index, void* workspace, size_t workspace_bytes,
                void* stream) {
    if (!values || !out_index || n <= 0) return Q3XK_EINVAL;
    if (!workspace || workspace_bytes < sizeof(ArgBest) * kArgmaxParts) return Q3XK_EWORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ArgBest* part = static_cast<ArgBest*>(workspace);
    if (launch_pdl(argmax_partial_kernel, dim3(kArgmaxParts), dim3(512), 0, s, values, n, part) != cudaSuccess)
        return Q3XK_ECUDA;
    if (launch_pdl(argmax_final_kernel, dim3(1), dim3(512), 0, s, (const ArgBest*)part, kArgmaxParts, out_index) !=
        cudaSuccess)
        return Q3XK_ECUDA;
    count_launch(2);
    return Q3XK_OK;
}

}  // extern "C"
