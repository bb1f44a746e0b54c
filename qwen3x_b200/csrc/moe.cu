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
#include "layers.cuh"

namespace q3xk {
namespace {

constexpr int kMaxPerLane = 16;  // experts <= 512


// Expert parallelism: the ids written are local to the rank's pool -- a
// routed expert e becomes e - e0 when e0 <= e < e0 + local, else -1 (not on
// this rank); the shared slot gets shared_id (-1: another rank runs it).  One
// GPU: e0 = 0, local = experts, shared_id = experts.
__global__ void __launch_bounds__(32) router_topk_kernel(const float* __restrict__ logits, int experts, int top_k,
                                                         int with_shared, int* __restrict__ ids,
                                                         float* __restrict__ weights, int e0, int local,
                                                         int shared_id) {
    griddep_wait();
    griddep_launch_dependents();
    // one token per block: block b reads row b of [T][experts + with_shared] logits
    logits += (int64_t)blockIdx.x * (experts + with_shared);
    ids += (int64_t)blockIdx.x * (top_k + with_shared);
    weights += (int64_t)blockIdx.x * (top_k + with_shared);
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
            const int e = chosen_id[slot] - e0;
            ids[slot] = e >= 0 && e < local ? e : -1;
            weights[slot] = chosen_p[slot] / selected_total;
        }
        if (with_shared) {
            ids[top_k] = shared_id;  // the shared expert is stored after the routed ones of each pool
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

// ---- MoE over a prompt: routing for all tokens, grouping by expert ------------

// logits[t][e] = router row e . x_t for T tokens (BF16 row records, FP32):
// a register-tiled FP32 GEMM on CUDA cores.  CTA = 64 tokens x 64 router rows,
// 256 threads with 4 x 4 outputs each; K in steps of 32 staged in shared
// memory, transposed ([k][token], [k][row]), BF16 widened to FP32.  Each
// output is one fmaf chain over k in ascending order.
constexpr int kRtT = 64, kRtE = 64, kRtK = 32, kRtPad = 4;

__global__ void __launch_bounds__(256) router_gemm_kernel(const uint8_t* __restrict__ w, int64_t row_stride,
                                                          int rows, int H, const float* __restrict__ x, int T,
                                                          float* __restrict__ logits) {
    __shared__ __align__(16) float xs[kRtK][kRtT + kRtPad];
    __shared__ __align__(16) float ws[kRtK][kRtE + kRtPad];
    griddep_wait();
    griddep_launch_dependents();
    const int t0 = blockIdx.x * kRtT, e0 = blockIdx.y * kRtE;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;  // rows 4tx.., tokens 4ty..
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int k0 = 0; k0 < H; k0 += kRtK) {
#pragma unroll
        for (int r = 0; r < kRtT * kRtK / 4 / 256; ++r) {  // 64 tokens x 8 float4
            const int i = tid + 256 * r, tt = i >> 3, kq = i & 7;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + tt < T) v = *reinterpret_cast<const float4*>(x + (int64_t)(t0 + tt) * H + k0 + 4 * kq);
            xs[4 * kq][tt] = v.x;
            xs[4 * kq + 1][tt] = v.y;
            xs[4 * kq + 2][tt] = v.z;
            xs[4 * kq + 3][tt] = v.w;
        }
        {  // 64 rows x 4 uint4 (8 BF16 each)
            const int ee = tid >> 2, kq = tid & 3;
            uint4 q = make_uint4(0u, 0u, 0u, 0u);
            if (e0 + ee < rows)
                q = __ldg(reinterpret_cast<const uint4*>(w + (int64_t)(e0 + ee) * row_stride + (k0 + 8 * kq) * 2));
            const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                ws[8 * kq + 2 * c][ee] = __uint_as_float(u[c] << 16);
                ws[8 * kq + 2 * c + 1][ee] = __uint_as_float(u[c] & 0xFFFF0000u);
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kRtK; ++k) {
            const float4 a = *reinterpret_cast<const float4*>(&xs[k][4 * ty]);
            const float4 b = *reinterpret_cast<const float4*>(&ws[k][4 * tx]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + 4 * ty + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + 4 * tx + j;
            if (e < rows) logits[(int64_t)t * rows + e] = acc[i][j];
        }
    }
}

// Groups the (token, slot) pairs by expert (pairs with id < 0 are left out,
// pos = -1).  One CTA.  Outputs: xoff[E+1]
// (first packed row of each expert), tile_off_a/b[E+1] (first GEMM tile of each
// expert for two GEMMs with tiles_a / tiles_b weight-row tiles), pos[T*S]
// (packed row of each pair), pair_token[P], pair_weight[P].  Positions inside
// an expert depend on arrival order; every packed row is computed
// independently, so results do not.
__global__ void __launch_bounds__(1024) moe_group_kernel(const int* __restrict__ ids, const float* __restrict__ wts,
                                                         int pairs, int S, int experts, int tiles_a, int tiles_b,
                                                         int bn, int* __restrict__ xoff, int* __restrict__ tile_a,
                                                         int* __restrict__ tile_b, int* __restrict__ pos,
                                                         int* __restrict__ pair_token, float* __restrict__ pair_weight) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ int gsm[];
    int* count = gsm;             // [experts]
    int* cursor = gsm + experts;  // [experts]
    for (int e = threadIdx.x; e < experts; e += blockDim.x) count[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < pairs; i += blockDim.x)
        if (ids[i] >= 0) atomicAdd(&count[ids[i]], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int x = 0, ta = 0, tb = 0;
        for (int e = 0; e < experts; ++e) {
            xoff[e] = x;
            tile_a[e] = ta;
            tile_b[e] = tb;
            cursor[e] = x;
            const int tt = (count[e] + bn - 1) / bn;
            x += count[e];
            ta += tiles_a * tt;
            tb += tiles_b * tt;
        }
        xoff[experts] = x;
        tile_a[experts] = ta;
        tile_b[experts] = tb;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
        if (ids[i] < 0) {  // expert on another rank
            pos[i] = -1;
            continue;
        }
        const int p = atomicAdd(&cursor[ids[i]], 1);
        pos[i] = p;
        pair_token[p] = i / S;
        pair_weight[p] = wts[i];
    }
}

// x16g[p] = x16[pair_token[p]], scale_g[p] = scale[pair_token[p]] (K halves per
// row) for the *pairs grouped rows; with lo planes (split precision) the
// residual row too.
__global__ void __launch_bounds__(256) gather_rows_kernel(const __half* __restrict__ x16,
                                                          const __half* __restrict__ x16lo,
                                                          const float* __restrict__ scale,
                                                          const int* __restrict__ pair_token,
                                                          const int* __restrict__ pairs, int K,
                                                          __half* __restrict__ x16g, __half* __restrict__ x16glo,
                                                          float* __restrict__ scale_g) {
    griddep_wait();
    griddep_launch_dependents();
    const int p = blockIdx.x;
    if (p >= *pairs) return;
    const int t = pair_token[p];
    const uint4* src = reinterpret_cast<const uint4*>(x16 + (int64_t)t * K);
    uint4* dst = reinterpret_cast<uint4*>(x16g + (int64_t)p * K);
    for (int i = threadIdx.x; i < K / 8; i += blockDim.x) dst[i] = src[i];
    if (x16lo) {
        const uint4* srcl = reinterpret_cast<const uint4*>(x16lo + (int64_t)t * K);
        uint4* dstl = reinterpret_cast<uint4*>(x16glo + (int64_t)p * K);
        for (int i = threadIdx.x; i < K / 8; i += blockDim.x) dstl[i] = srcl[i];
    }
    if (threadIdx.x == 0) scale_g[p] = scale[t];
}

// Per packed row p: h = w_p * silu(g) * u over the interleaved gate|up row
// (g(2j) g(2j+1) u(2j) u(2j+1)), then FP16 with a per-row power-of-two scale
// (as x_to_f16_kernel) for the down GEMM, plus the residual plane when
// h16lo != nullptr.  I <= 1024.
__global__ void __launch_bounds__(256) swiglu_f16_kernel(const float* __restrict__ gu, const float* __restrict__ pw,
                                                         const int* __restrict__ pairs, int I,
                                                         __half* __restrict__ h16, __half* __restrict__ h16lo,
                                                         float* __restrict__ scale) {
    griddep_wait();
    griddep_launch_dependents();
    const int p = blockIdx.x;
    if (p >= *pairs) return;
    const float* row = gu + (int64_t)p * 2 * I;
    const float wt = pw[p];
    float h[4];
    uint32_t emax = 0;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int i = threadIdx.x + 256 * a;
        h[a] = 0.f;
        if (i < I) {
            const int c = (i >> 1) * 4 + (i & 1);
            const float g = row[c], u = row[c + 2];
            h[a] = wt * (g * sigmoid_ref(g) * u);
            emax = max(emax, (__float_as_uint(h[a]) >> 23) & 0xFFu);
        }
    }
    __shared__ uint32_t red[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = emax;
    __syncthreads();
    emax = 0;
    for (int i = 0; i < 8; ++i) emax = max(emax, red[i]);
    const int E = emax == 0xFFu ? 0 : (int)emax - 127;
    const int sh = min(100, max(-100, 14 - E));
    const float up = __uint_as_float((uint32_t)(sh + 127) << 23);
    if (threadIdx.x == 0) scale[p] = __uint_as_float((uint32_t)(127 - sh) << 23);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int i = threadIdx.x + 256 * a;
        if (i < I) {
            const float v = h[a] * up;
            const __half hv = __float2half_rn(v);
            h16[(int64_t)p * I + i] = hv;
            if (h16lo) h16lo[(int64_t)p * I + i] = __float2half_rn(v - __half2float(hv));
        }
    }
}

// hidden[t] (+)= sum over the slots s run here (pos >= 0, in slot order) of
// out[pos[t*S + s]].
__global__ void __launch_bounds__(256) moe_combine_kernel(const float* __restrict__ out, const int* __restrict__ pos,
                                                          int S, int H, float* __restrict__ hidden, int accumulate) {
    griddep_wait();
    griddep_launch_dependents();
    const int t = blockIdx.x;
    const int* pt = pos + (int64_t)t * S;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
        float acc = 0.f;
        for (int sl = 0; sl < S; ++sl) {
            const int p = pt[sl];
            if (p >= 0) acc += out[(int64_t)p * H + j];
        }
        float* h = hidden + (int64_t)t * H + j;
        *h = accumulate ? *h + acc : acc;
    }
}

}  // namespace

int router_topk(const float* logits, int experts, int top_k, int T, int e0, int local, int shared_id, int* ids,
                float* weights, cudaStream_t s) {
    if (launch_pdl(router_topk_kernel, dim3(T), dim3(32), 0, s, logits, experts, top_k, 1, ids, weights, e0, local,
                   shared_id) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int moe_prefill(const MoePrefillArgs& a, cudaStream_t s) {
    // router over all experts (+ shared gate); grouping over the local pool
    const int T = a.T, S = a.top_k + 1, E1 = a.local + 1, P = T * S, R1 = a.experts + 1;
    const int H = a.gate_up->cols, I = a.down->cols;
    if (I > 1024 || a.gate_up->rows != 2 * I || a.down->rows != H) return Q3XK_EUNSUPPORTED;
    // 1. router logits (+ shared gate) for every token, then top-k per token
    if (H % kRtK || (a.router->row_stride & 15)) return Q3XK_EUNSUPPORTED;
    if (launch_pdl(router_gemm_kernel, dim3((T + kRtT - 1) / kRtT, (R1 + kRtE - 1) / kRtE), dim3(256), 0, s,
                   (const uint8_t*)a.router->data, a.router->row_stride, R1, H, a.x, T, a.logits) != cudaSuccess)
        return Q3XK_ECUDA;
    if (launch_pdl(router_topk_kernel, dim3(T), dim3(32), 0, s, (const float*)a.logits, a.experts, a.top_k, 1,
                   a.ids, a.weights, a.e0, a.local, a.shared_id) != cudaSuccess)
        return Q3XK_ECUDA;
    // 2. group the pairs by expert
    const int bn = (int)gemm_grouped_tile_width();
    const int tiles_a = (a.gate_up->rows + 127) / 128, tiles_b = (a.down->rows + 127) / 128;
    if (launch_pdl(moe_group_kernel, dim3(1), dim3(1024), (size_t)2 * E1 * sizeof(int), s, (const int*)a.ids,
                   (const float*)a.weights, P, S, E1, tiles_a, tiles_b, bn, a.xoff, a.tile_gu, a.tile_dn, a.pos,
                   a.pair_token, a.pair_weight) != cudaSuccess)
        return Q3XK_ECUDA;
    // 3. FP16 rows per token (+ residual planes), gathered per pair
    __half* x16lo = a.split ? a.x16 + (size_t)T * H : nullptr;
    __half* x16glo = a.split ? a.x16g + (size_t)P * H : nullptr;
    __half* h16lo = a.split ? a.h16 + (size_t)P * I : nullptr;
    int st = launch_x_to_f16(a.x, T, H, a.x16, x16lo, a.scale, s);
    if (st != Q3XK_OK) return st;
    const int* grouped = a.xoff + E1;  // pairs run on this GPU (device)
    if (launch_pdl(gather_rows_kernel, dim3(P), dim3(256), 0, s, (const __half*)a.x16, (const __half*)x16lo,
                   (const float*)a.scale, (const int*)a.pair_token, grouped, H, a.x16g, x16glo,
                   a.scale_g) != cudaSuccess)
        return Q3XK_ECUDA;
    // 4. gate|up of every pair on its expert, weighted SwiGLU -> FP16, down
    const GemmGroups ggu{E1, a.xoff, a.tile_gu}, gdn{E1, a.xoff, a.tile_dn};
    st = gemm_f16(a.gate_up, a.x16g, x16glo, a.scale_g, P, a.gu, 0, &ggu, 0, s);
    if (st != Q3XK_OK) return st;
    if (launch_pdl(swiglu_f16_kernel, dim3(P), dim3(256), 0, s, (const float*)a.gu, (const float*)a.pair_weight,
                   grouped, I, a.h16, h16lo, a.scale_h) != cudaSuccess)
        return Q3XK_ECUDA;
    st = gemm_f16(a.down, a.h16, h16lo, a.scale_h, P, a.out, 0, &gdn, 0, s);
    if (st != Q3XK_OK) return st;
    // 5. add each token's slots into its hidden row, in slot order
    if (launch_pdl(moe_combine_kernel, dim3(T), dim3(256), 0, s, (const float*)a.out, (const int*)a.pos, S, H,
                   a.hidden, a.accumulate) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch(7);
    return Q3XK_OK;
}

}  // namespace q3xk

using namespace q3xk;

extern "C" {

int q3xk_router_topk(const float* logits, int experts, int top_k, int with_shared, int* ids, float* weights,
                     void* stream) {
    if (!logits || !ids || !weights || experts <= 0 || experts > 32 * kMaxPerLane || top_k <= 0 ||
        top_k > 8 || top_k > experts)
        return Q3XK_EINVAL;
    const cudaError_t e = launch_pdl(router_topk_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                                     logits, experts, top_k, with_shared ? 1 : 0, ids, weights, 0, experts, experts);
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
