// delta.cu -- gated DeltaNet over a prompt in chunks (prefill, T > 1).
//
// The reference runs the delta rule one token at a time (engine.cpp:274-320):
//   S <- a_t S;  u_t = b_t (v_t - S^T k_t);  S <- S + k_t u_t^T;  o_t = S^T q_t
// with a_t = exp(g_t), g_t = -exp(A_log) softplus(a_t + dt_bias), b_t =
// sigmoid(b_t).  Over a chunk of C tokens starting from state S0, with
// G_t = g_1 + ... + g_t and Gam_tj = exp(G_t - G_j), this is exactly
//   (I + A) U = beta V - diag(beta exp(G)) K S0,  A_tj = beta_t Gam_tj k_t.k_j (j < t)
//   O  = diag(exp(G)) Q S0 + tril(Q K^T o Gam) U
//   S' = exp(G_C) S0 + (diag(exp(G_C - G)) K)^T U
// (the chunked / "WY" form of the delta rule).  U = U' - W S0 with
// U' = (I + A)^-1 beta V and W = (I + A)^-1 diag(beta exp(G)) K, both by
// forward substitution.  Two kernels:
//   delta_prep  one CTA per (chunk, head), all chunks in parallel: q/k
//               l2-norms, beta, G, A, U', W, M = tril(Q K^T o Gam), Q~, K~;
//   delta_scan  one CTA per (head, 32-column block of S), chunks in order:
//               U = U' - W S, O = Q~ S + M U, S = exp(G_C) S + K~^T U,
//               the next chunk's blocks loading (cp.async) meanwhile.
// The output is the raw o; gated_rms_kernel applies the gated RMS after.
#include "layers.cuh"

namespace q3xk {
namespace {

constexpr int kC = 64;            // chunk length
constexpr int kD = 128;           // KD = VD
constexpr int kLd = kD + 4;       // padded smem row (floats)
constexpr int kCols = 32;         // S columns per scan CTA
constexpr float kEps = 1e-6f;     // engine.cpp:27
// Workspace block of one (head, chunk), laid out for the scan's register
// tiles: Q~^T [kD][kC], W^T [kD][kC], K~ [kC][kD], U' [kC][kD], M^T [kC][kC], gamma.
constexpr int64_t kBlockFloats = 4 * kC * kD + kC * kC + 4;
constexpr int kOffQT = 0, kOffWT = kC * kD, kOffK = 2 * kC * kD, kOffU = 3 * kC * kD, kOffMT = 4 * kC * kD,
              kOffGamma = 4 * kC * kD + kC * kC;

__device__ __forceinline__ float sigm(float x) { return sigmoid_ref(x); }
__device__ __forceinline__ float softplus_ref(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__device__ __forceinline__ float* block_ptr(float* work, int head, int chunk, int nchunks) {
    return work + ((int64_t)head * nchunks + chunk) * kBlockFloats;
}

// ---- prep: one CTA per (chunk, head), 256 threads --------------------------------
__global__ void __launch_bounds__(256) delta_prep_kernel(const float* __restrict__ qkv, int64_t qkv_stride,
                                                         const float* __restrict__ proj, int64_t proj_stride, int T,
                                                         DeltaDims dd, const float* __restrict__ alog,
                                                         const float* __restrict__ dt, float* __restrict__ work) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ __align__(16) float sm[];
    float* Ks = sm;                 // [kC][kLd] normalised k
    float* Qs = Ks + kC * kLd;      // [kC][kLd] normalised, scaled q; later W
    float* Vs = Qs + kC * kLd;      // [kC][kLd] v; later U'
    float* As = Vs + kC * kLd;      // [kC][kC + 1]
    float* G = As + kC * (kC + 1);  // [kC] cumulative log decay
    float* beta = G + kC;           // [kC]
    float* gl = beta + kC;          // [kC] per-token log decay
    const int chunk = blockIdx.x, head = blockIdx.y, nchunks = gridDim.x;
    const int t0 = chunk * kC, n = min(kC, T - t0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qk_head = head / (dd.VH / dd.KH);
    float* out = block_ptr(work, head, chunk, nchunks);

    // 1. load q, k, v rows; l2-normalise q and k per token (warp per token)
    for (int i = warp; i < kC; i += 8) {
        float q[4], k[4], v[4];
        const bool live = i < n;
        const float* crow = qkv + (int64_t)(t0 + i) * qkv_stride;  // conv output: q | k | v
        const float* row = proj + (int64_t)(t0 + i) * proj_stride;  // a, b
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = lane + 32 * e;
            q[e] = live ? crow[qk_head * kD + d] : 0.f;
            k[e] = live ? crow[dd.KH * kD + qk_head * kD + d] : 0.f;
            v[e] = live ? crow[2 * dd.KH * kD + head * kD + d] : 0.f;
        }
        float qs = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
        float ks = k[0] * k[0] + k[1] * k[1] + k[2] * k[2] + k[3] * k[3];
        qs = warp_sum(qs);
        ks = warp_sum(ks);
        // engine.cpp:246-251: q, k l2-normalised, q divided by sqrt(KD)
        const float qscale = 1.0f / sqrtf(qs + kEps), kscale = 1.0f / sqrtf(ks + kEps);
        const float root = sqrtf((float)kD);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = lane + 32 * e;
            Qs[i * kLd + d] = q[e] * qscale / root;
            Ks[i * kLd + d] = k[e] * kscale;
            Vs[i * kLd + d] = v[e];
        }
        if (lane == 0) {
            float b = 0.f, g = 0.f;
            if (live) {
                b = sigm(row[dd.b_off + head]);
                g = -expf(alog[head]) * softplus_ref(row[dd.a_off + head] + dt[head]);
            }
            beta[i] = b;
            gl[i] = g;
        }
    }
    __syncthreads();
    if (tid == 0) {  // cumulative log decay within the chunk
        float acc = 0.f;
        for (int i = 0; i < kC; ++i) {
            acc += gl[i];
            G[i] = acc;
        }
    }
    __syncthreads();

    // 2. A (strictly lower) and M (lower incl. diagonal) from 128-long dots
    float* Mo = out + kOffMT;
    for (int e = tid; e < kC * kC; e += 256) {
        const int i = e / kC, j = e % kC;
        float a = 0.f, m = 0.f;
        if (j <= i && i < n) {
            const float4* ki = reinterpret_cast<const float4*>(Ks + i * kLd);
            const float4* kj = reinterpret_cast<const float4*>(Ks + j * kLd);
            const float4* qi = reinterpret_cast<const float4*>(Qs + i * kLd);
            float dk = 0.f, dq = 0.f;
#pragma unroll 8
            for (int d = 0; d < kD / 4; ++d) {
                const float4 x = kj[d], y = ki[d], z = qi[d];
                dk += y.x * x.x + y.y * x.y + y.z * x.z + y.w * x.w;
                dq += z.x * x.x + z.y * x.y + z.z * x.z + z.w * x.w;
            }
            const float gam = expf(G[i] - G[j]);
            m = dq * gam;
            if (j < i) a = beta[i] * gam * dk;
        }
        As[i * (kC + 1) + j] = a;
        Mo[j * kC + i] = m;  // M^T
    }
    // Q~ = exp(G) q, K~ = exp(G_last - G) k, straight to the workspace
    const float Glast = G[n - 1];
    for (int e = tid; e < kC * kD; e += 256) {
        const int i = e / kD, d = e % kD;
        out[kOffK + e] = i < n ? expf(Glast - G[i]) * Ks[i * kLd + d] : 0.f;  // K~
        const int dt_ = e / kC, it = e % kC;
        out[kOffQT + e] = it < n ? expf(G[it]) * Qs[it * kLd + dt_] : 0.f;     // Q~^T
    }
    if (tid == 0) out[kOffGamma] = expf(Glast);
    __syncthreads();

    // 3. forward substitution: rows t of U' (in Vs) and W (in Qs), in order
    //    U'_t = beta_t v_t - sum_{j<t} A_tj U'_j;  W_t = beta_t e^{G_t} k_t - sum_{j<t} A_tj W_j
    const int col = tid & (kD - 1);
    const bool is_w = tid >= kD;
    float* X = is_w ? Qs : Vs;
    for (int t = 0; t < n; ++t) {
        float acc = is_w ? beta[t] * expf(G[t]) * Ks[t * kLd + col] : beta[t] * Vs[t * kLd + col];
        const float* arow = As + t * (kC + 1);
        for (int j = 0; j < t; ++j) acc -= arow[j] * X[j * kLd + col];
        X[t * kLd + col] = acc;
        __syncthreads();
    }
    for (int e = tid; e < kC * kD; e += 256) {
        const int i = e / kD, d = e % kD;
        out[kOffU + e] = i < n ? Vs[i * kLd + d] : 0.f;  // U'
        const int dt_ = e / kC, it = e % kC;
        out[kOffWT + e] = it < n ? Qs[it * kLd + dt_] : 0.f;  // W^T
    }
}

// ---- scan: one CTA per (head, 32-column block), chunks in order ----------------
// Register tiles: U and O as 4 rows x 2 columns per thread, S as 4 x 4.  The
// chunk blocks stream in with cp.async: W^T, Q~^T and M^T of chunk c + 1 are in
// flight while chunk c computes (two buffers each), and K~ of chunk c while its
// U and O phases run.
__device__ __forceinline__ void cp_async16(float* smem, const float* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void copy_async(float* dst, const float* src, int n4) {
    for (int e = threadIdx.x; e < n4; e += 256) cp_async16(dst + 4 * e, src + 4 * e);
}

__global__ void __launch_bounds__(256) delta_scan_kernel(const float* __restrict__ work, int T,
                                                         float* __restrict__ state /*[VH][KD][VD]*/,
                                                         float* __restrict__ out, int64_t out_stride) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ __align__(16) float sm[];
    float* S = sm;                       // [kD][kCols]
    float* U = S + kD * kCols;           // [kC][kCols]
    float* Kb = U + kC * kCols;          // K~ [kC][kD] of the current chunk
    float* Wbase = Kb + kC * kD;         // W^T [kD][kC], two buffers
    float* Qbase = Wbase + 2 * kC * kD;  // Q~^T [kD][kC], two buffers
    float* Mbase = Qbase + 2 * kC * kD;  // M^T [kC][kC], two buffers
    const int head = blockIdx.x, cb = blockIdx.y;
    const int nchunks = (T + kC - 1) / kC;
    const int tid = threadIdx.x;
    const int i0 = 4 * (tid & 15), c0 = 2 * (tid >> 4);  // U / O tile
    const int r0 = 4 * (tid & 31), c4 = 4 * (tid >> 5);  // S tile
    float* st = state + (int64_t)head * kD * kD + cb * kCols;
    for (int e = tid; e < kD * kCols; e += 256) S[e] = st[(e / kCols) * kD + e % kCols];
    auto block_of = [&](int chunk) { return work + ((int64_t)head * nchunks + chunk) * kBlockFloats; };
    auto issue_wqm = [&](int chunk, int par) {
        const float* blk = block_of(chunk);
        copy_async(Wbase + par * kC * kD, blk + kOffWT, kC * kD / 4);
        copy_async(Qbase + par * kC * kD, blk + kOffQT, kC * kD / 4);
        copy_async(Mbase + par * kC * kC, blk + kOffMT, kC * kC / 4);
    };
    issue_wqm(0, 0);
    cp_async_commit();

    for (int chunk = 0; chunk < nchunks; ++chunk) {
        const float* blk = block_of(chunk);
        const int par = chunk & 1, t0 = chunk * kC, n = min(kC, T - t0);
        const float* A1 = Wbase + par * kC * kD;
        const float* A2 = Qbase + par * kC * kD;
        const float* Ms = Mbase + par * kC * kC;
        cp_async_wait<0>();  // this chunk's W^T, Q~^T, M^T have landed
        __syncthreads();     // ... for every thread; the previous chunk is done with Kb and the other buffers
        copy_async(Kb, blk + kOffK, kC * kD / 4);
        cp_async_commit();
        if (chunk + 1 < nchunks) issue_wqm(chunk + 1, par ^ 1);
        cp_async_commit();
        // U = U' - W S
        float u[4][2];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const float2 up = *reinterpret_cast<const float2*>(blk + kOffU + (i0 + a) * kD + cb * kCols + c0);
            u[a][0] = up.x;
            u[a][1] = up.y;
        }
#pragma unroll 4
        for (int r = 0; r < kD; ++r) {
            const float4 w = *reinterpret_cast<const float4*>(A1 + r * kC + i0);
            const float2 sv = *reinterpret_cast<const float2*>(S + r * kCols + c0);
            u[0][0] -= w.x * sv.x; u[0][1] -= w.x * sv.y;
            u[1][0] -= w.y * sv.x; u[1][1] -= w.y * sv.y;
            u[2][0] -= w.z * sv.x; u[2][1] -= w.z * sv.y;
            u[3][0] -= w.w * sv.x; u[3][1] -= w.w * sv.y;
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) *reinterpret_cast<float2*>(U + (i0 + a) * kCols + c0) = make_float2(u[a][0], u[a][1]);
        __syncthreads();
        // O = Q~ S + M U
        float o[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll 4
        for (int r = 0; r < kD; ++r) {
            const float4 q = *reinterpret_cast<const float4*>(A2 + r * kC + i0);
            const float2 sv = *reinterpret_cast<const float2*>(S + r * kCols + c0);
            o[0][0] += q.x * sv.x; o[0][1] += q.x * sv.y;
            o[1][0] += q.y * sv.x; o[1][1] += q.y * sv.y;
            o[2][0] += q.z * sv.x; o[2][1] += q.z * sv.y;
            o[3][0] += q.w * sv.x; o[3][1] += q.w * sv.y;
        }
#pragma unroll 4
        for (int j = 0; j < kC; ++j) {
            const float4 mm = *reinterpret_cast<const float4*>(Ms + j * kC + i0);
            const float2 uv = *reinterpret_cast<const float2*>(U + j * kCols + c0);
            o[0][0] += mm.x * uv.x; o[0][1] += mm.x * uv.y;
            o[1][0] += mm.y * uv.x; o[1][1] += mm.y * uv.y;
            o[2][0] += mm.z * uv.x; o[2][1] += mm.z * uv.y;
            o[3][0] += mm.w * uv.x; o[3][1] += mm.w * uv.y;
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
            if (i0 + a < n)
                *reinterpret_cast<float2*>(out + (int64_t)(t0 + i0 + a) * out_stride + head * kD + cb * kCols + c0) =
                    make_float2(o[a][0], o[a][1]);
        cp_async_wait<1>();  // K~ of this chunk has landed (the next chunk's blocks may still be in flight)
        __syncthreads();
        // S = gamma S + K~^T U
        const float gam = blk[kOffGamma];
        float sacc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const float4 sv = *reinterpret_cast<const float4*>(S + (r0 + a) * kCols + c4);
            sacc[a][0] = gam * sv.x; sacc[a][1] = gam * sv.y; sacc[a][2] = gam * sv.z; sacc[a][3] = gam * sv.w;
        }
#pragma unroll 4
        for (int j = 0; j < kC; ++j) {
            const float4 kk = *reinterpret_cast<const float4*>(Kb + j * kD + r0);
            const float4 uv = *reinterpret_cast<const float4*>(U + j * kCols + c4);
            const float kr[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                sacc[a][0] += kr[a] * uv.x; sacc[a][1] += kr[a] * uv.y;
                sacc[a][2] += kr[a] * uv.z; sacc[a][3] += kr[a] * uv.w;
            }
        }
        __syncthreads();  // every thread has read S (U and O phases) before it changes
#pragma unroll
        for (int a = 0; a < 4; ++a)
            *reinterpret_cast<float4*>(S + (r0 + a) * kCols + c4) =
                make_float4(sacc[a][0], sacc[a][1], sacc[a][2], sacc[a][3]);
    }
    cp_async_wait<0>();
    __syncthreads();
    for (int e = tid; e < kD * kCols; e += 256) st[(e / kCols) * kD + e % kCols] = S[e];
}

// o <- o * rsqrt(mean o^2 + eps) * norm * silu(z) per (token, head) row of VD
// (engine.cpp:237-242); one warp per row.
__global__ void __launch_bounds__(256) gated_rms_kernel(float* __restrict__ out, int64_t out_stride, int T, int VH,
                                                        const float* __restrict__ proj, int64_t proj_stride,
                                                        int z_off, const float* __restrict__ norm) {
    griddep_wait();
    griddep_launch_dependents();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= T * VH) return;
    const int t = row / VH, h = row % VH;
    float* o = out + (int64_t)t * out_stride + h * kD;
    const float* z = proj + (int64_t)t * proj_stride + z_off + h * kD;
    float v[4], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        v[e] = o[lane + 32 * e];
        ss += v[e] * v[e];
    }
    ss = warp_sum(ss);
    const float scale = 1.0f / sqrtf(ss / (float)kD + kEps);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float zz = z[lane + 32 * e];
        o[lane + 32 * e] = v[e] * (scale * norm[lane + 32 * e] * (zz * sigmoid_ref(zz)));
    }
}

constexpr size_t kPrepSmem = (size_t)(3 * kC * kLd + kC * (kC + 1) + 3 * kC) * 4;
constexpr size_t kScanSmem = (size_t)(kD * kCols + kC * kCols + 5 * kC * kD + 2 * kC * kC) * 4;  // 216 KB
static_assert(kScanSmem <= 227 * 1024, "scan shared memory");

}  // namespace

size_t delta_chunked_workspace_bytes(int T, int VH) {
    const int64_t nchunks = (T + kC - 1) / kC;
    return (size_t)(VH * nchunks * kBlockFloats) * 4;
}

int launch_delta_chunked(const float* qkv, int64_t qkv_stride, const float* proj, int64_t proj_stride, int T,
                         const DeltaDims& dd, const float* alog, const float* dt, const float* norm, float* state,
                         float* out, int64_t out_stride, float* work, cudaStream_t s) {
    if (dd.KD != kD || dd.VD != kD || dd.VH % dd.KH || T < 1 || !work || !norm) return Q3XK_EUNSUPPORTED;
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(delta_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrepSmem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(delta_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScanSmem) !=
                cudaSuccess)
            return Q3XK_ECUDA;
        configured = true;
    }
    const int nchunks = (T + kC - 1) / kC;
    if (launch_pdl(delta_prep_kernel, dim3(nchunks, dd.VH), dim3(256), kPrepSmem, s, qkv, qkv_stride, proj,
                   proj_stride, T, dd, alog, dt, work) != cudaSuccess)
        return Q3XK_ECUDA;
    if (launch_pdl(delta_scan_kernel, dim3(dd.VH, kD / kCols), dim3(256), kScanSmem, s, (const float*)work, T, state,
                   out, out_stride) != cudaSuccess)
        return Q3XK_ECUDA;
    if (launch_pdl(gated_rms_kernel, dim3((T * dd.VH + 7) / 8), dim3(256), 0, s, out, out_stride, T, dd.VH, proj,
                   proj_stride, dd.z_off, norm) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch(3);
    return Q3XK_OK;
}

}  // namespace q3xk
