// layers.cu -- the non-matrix steps of the hybrid decoder's forward.
//
// These surround the packed-weight matrix path (gemv.cu, gemm.cu, moe.cu)
// and follow the reference CPU forward's formulas (engine.cpp:181-369); each
// kernel names the function it restates.  All state and activations are FP32
// as in the reference.  Positions are read from device memory (`pos`) so a
// whole decode step can live in one CUDA graph.
#include "layers.cuh"
#include "stream.cuh"

namespace q3xk {
namespace {

constexpr float kEps = 1e-6f;          // engine.cpp:27
constexpr float kTheta = 10000000.0f;  // engine.cpp:27

// engine.cpp:187-192
__device__ __forceinline__ float sigmoidf_ref(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}
__device__ __forceinline__ float siluf_ref(float x) { return x * sigmoidf_ref(x); }
__device__ __forceinline__ float softplusf_ref(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) s += red[i];
    return s;
}

// ---- embedding: one decoded row per token (engine.cpp:195-200, arch/cpu.cpp:55-90)
__global__ void embed_kernel(const uint8_t* __restrict__ w, int64_t row_stride, int64_t qbytes, int type, int cols,
                             const int* __restrict__ tokens, int T, float* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    const int t = blockIdx.y;
    if (t >= T) return;
    const uint8_t* rec = w + (int64_t)tokens[t] * row_stride;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < cols; k += gridDim.x * blockDim.x) {
        float v;
        if (type == Q3XK_BF16) {
            v = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(rec)[k] << 16);
        } else {
            const float d = f16_bits_to_float(reinterpret_cast<const uint16_t*>(rec + qbytes)[k >> 5]);
            if (type == Q3XK_Q8_0) {
                v = d * (float)(int8_t)(rec[k] ^ 0x80);
            } else {
                const int blk = k >> 5, i = k & 31;
                const uint8_t b = rec[blk * 16 + (i & 15)];
                v = d * (float)((i < 16 ? (b & 15) : (b >> 4)) - 8);
            }
        }
        out[(int64_t)t * cols + k] = v;
    }
}

// ---- RMSNorm with a precomputed (1 + w) (engine.cpp:231-236)
__global__ void __launch_bounds__(256) rms_kernel(const float* __restrict__ x, const float* __restrict__ w1, int n,
                                                  float* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ float red[8];
    const float* xr = x + (int64_t)blockIdx.x * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) ss += xr[i] * xr[i];
    ss = block_sum<256>(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)n + kEps);
    float* o = out + (int64_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += 256) o[i] = xr[i] * scale * w1[i];
}

// The same sums in the same order for n <= 256 * PER, with the row held in
// registers: the norm weights are loaded before the dependency wait, and all
// of a thread's loads of x are in flight at once (a decode row is one CTA, so
// its time is load latency).
template <int PER>
__global__ void __launch_bounds__(256) rms_reg_kernel(const float* __restrict__ x, const float* __restrict__ w1,
                                                      int n, float* __restrict__ out) {
    __shared__ float red[8];
    const int tid = threadIdx.x;
    float wv[PER], xv[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = tid + 256 * j;
        wv[j] = i < n ? __ldg(w1 + i) : 0.f;
    }
    griddep_wait();
    griddep_launch_dependents();
    const float* xr = x + (int64_t)blockIdx.x * n;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = tid + 256 * j;
        xv[j] = i < n ? xr[i] : 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
        if (tid + 256 * j < n) ss += xv[j] * xv[j];
    ss = block_sum<256>(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)n + kEps);
    float* o = out + (int64_t)blockIdx.x * n;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = tid + 256 * j;
        if (i < n) o[i] = xv[j] * scale * wv[j];
    }
}

// ---- causal conv1d over T tokens with SiLU and history (engine.cpp:264-273).
// proj[t][c] for c < channels is replaced by the activated conv output.  One
// thread per channel; KC is the kernel width when known at compile time
// (0: runtime `CK`, at most 9).
template <int KC>
__global__ void conv_kernel(float* __restrict__ proj, int64_t proj_stride, int T, int channels,
                            const float* __restrict__ w /*[channels][CK]*/, int CK_rt, float* __restrict__ hist) {
    griddep_wait();
    griddep_launch_dependents();
    const int CK = KC ? KC : CK_rt;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    float h[KC ? KC : 8], wc[KC ? KC + 1 : 9];
    float* hc = hist + (int64_t)c * (CK - 1);
#pragma unroll
    for (int i = 0; i < (KC ? KC - 1 : 8); ++i)
        if (i < CK - 1) h[i] = hc[i];
#pragma unroll
    for (int i = 0; i < (KC ? KC : 9); ++i)
        if (i < CK) wc[i] = w[(int64_t)c * CK + i];
    constexpr int kTile = 16;  // tokens whose inputs are loaded before any is written back
    for (int t0 = 0; t0 < T; t0 += kTile) {
        float xs[kTile];
#pragma unroll
        for (int i = 0; i < kTile; ++i) xs[i] = t0 + i < T ? proj[(int64_t)(t0 + i) * proj_stride + c] : 0.f;
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            if (t0 + i >= T) break;  // T is uniform: no divergence
            const float x = xs[i];
            float sum = x * wc[CK - 1];
#pragma unroll
            for (int j = 0; j < (KC ? KC - 1 : 8); ++j)
                if (j < CK - 1) sum += h[j] * wc[j];
#pragma unroll
            for (int j = 0; j < (KC ? KC - 2 : 7); ++j)
                if (j < CK - 2) h[j] = h[j + 1];
            h[CK - 2] = x;
            xs[i] = siluf_ref(sum);
        }
#pragma unroll
        for (int i = 0; i < kTile; ++i)
            if (t0 + i < T) proj[(int64_t)(t0 + i) * proj_stride + c] = xs[i];
    }
#pragma unroll
    for (int i = 0; i < (KC ? KC - 1 : 8); ++i)
        if (i < CK - 1) hc[i] = h[i];
}

// ---- the same conv over a prompt, out of place: CTA = (128 channels, 64-token
// segment).  A segment's history is the raw input of the CK-1 tokens before it
// (or the stored history for the first segment, whose CTA also writes the new
// history).
constexpr int kConvSeg = 64;
__global__ void __launch_bounds__(128) conv_prefill_kernel(const float* __restrict__ proj, int64_t proj_stride, int T,
                                                           int channels, const float* __restrict__ w,
                                                           float* __restrict__ hist, float* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int CK = 4;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int t0 = blockIdx.y * kConvSeg, t1 = min(T, t0 + kConvSeg);
    if (c >= channels) return;
    float h[CK - 1], wc[CK];
#pragma unroll
    for (int i = 0; i < CK; ++i) wc[i] = w[(int64_t)c * CK + i];
#pragma unroll
    for (int i = 0; i < CK - 1; ++i) {
        const int t = t0 - (CK - 1) + i;  // token whose raw input is history slot i
        h[i] = t >= 0 ? proj[(int64_t)t * proj_stride + c] : hist[(int64_t)c * (CK - 1) + (t + (CK - 1))];
    }
    constexpr int kTile = 16;
    for (int tb = t0; tb < t1; tb += kTile) {
        float xs[kTile];
#pragma unroll
        for (int i = 0; i < kTile; ++i) xs[i] = tb + i < t1 ? proj[(int64_t)(tb + i) * proj_stride + c] : 0.f;
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            if (tb + i >= t1) break;
            const float x = xs[i];
            float sum = x * wc[CK - 1];
#pragma unroll
            for (int j = 0; j < CK - 1; ++j) sum += h[j] * wc[j];
#pragma unroll
            for (int j = 0; j < CK - 2; ++j) h[j] = h[j + 1];
            h[CK - 2] = x;
            out[(int64_t)(tb + i) * channels + c] = siluf_ref(sum);
        }
    }
    // The first segment's CTA alone reads the stored history, so it alone
    // writes the new one: the raw inputs of the last CK-1 tokens.
    if (blockIdx.y == 0) {
#pragma unroll
        for (int i = 0; i < CK - 1; ++i)
            hist[(int64_t)c * (CK - 1) + i] = t1 == T ? h[i] : proj[(int64_t)(T - (CK - 1) + i) * proj_stride + c];
    }
}

// ---- gated DeltaNet, one head per CTA, T tokens in order (engine.cpp:274-320).
// 512 threads: thread (v = tid % 128, g = tid / 128) keeps state rows
// 32g..32g+31 of column v in registers for the whole chunk.
constexpr int kDeltaThreads = 512;
// conv_w != nullptr (T = 1 only): the causal conv + SiLU of this head's q, k
// and v channels (engine.cpp:264-273) is computed here from the raw
// projections and the history `hist`, which it updates.  The q/k channels are
// shared by the VH/KH heads of a key group: each of their CTAs reads the old
// history, counts itself in group_count[key head], and the last one to arrive
// writes the new history and resets the count to zero.
__global__ void __launch_bounds__(kDeltaThreads) delta_kernel(const float* __restrict__ proj, int64_t proj_stride,
                                                              int T, DeltaDims dd, const float* __restrict__ alog,
                                                              const float* __restrict__ dt,
                                                              const float* __restrict__ norm,
                                                              float* __restrict__ state /*[VH][KD][VD]*/,
                                                              float* __restrict__ out, int64_t out_stride,
                                                              const float* __restrict__ conv_w,
                                                              float* __restrict__ hist,
                                                              int* __restrict__ group_count) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int KD = 128, VD = 128, G = kDeltaThreads / VD, RG = KD / G;  // rows per group
    constexpr int CK = 4;
    const int head = blockIdx.x;
    const int tid = threadIdx.x, v = tid % VD, g = tid / VD;
    __shared__ float qs[KD], ks[KD], vs[VD], part[G][VD], red[kDeltaThreads / 32], scal[4], cx[3 * KD];
    float S[RG];
    float* st = state + (int64_t)head * KD * VD;
#pragma unroll
    for (int r = 0; r < RG; ++r) S[r] = st[(int64_t)(g * RG + r) * VD + v];
    const int qk_head = head / (dd.VH / dd.KH);
    const float qscale = sqrtf((float)KD);
    if (conv_w) {
        // threads 0..127: q channel, 128..255: k channel, 256..383: v channel
        const int part_ = tid / KD, d = tid % KD;
        const int c = part_ == 0 ? qk_head * KD + d : part_ == 1 ? dd.KH * KD + qk_head * KD + d
                                                                : 2 * dd.KH * KD + head * VD + d;
        float x = 0.f, h[CK - 1];
        if (tid < 3 * KD) {
            x = proj[c];
            float w[CK];
#pragma unroll
            for (int i = 0; i < CK - 1; ++i) h[i] = hist[(int64_t)c * (CK - 1) + i];
#pragma unroll
            for (int i = 0; i < CK; ++i) w[i] = conv_w[(int64_t)c * CK + i];
            float sum = x * w[CK - 1];
#pragma unroll
            for (int i = 0; i < CK - 1; ++i) sum += h[i] * w[i];
            cx[tid] = siluf_ref(sum);
        }
        __syncthreads();  // every read of the old history of this CTA is done
        if (tid == 0) {
            __threadfence();
            const int ratio = dd.VH / dd.KH;
            const int prev = atomicAdd(group_count + qk_head, 1);
            scal[2] = prev == ratio - 1 ? 1.f : 0.f;
            if (prev == ratio - 1) group_count[qk_head] = 0;
        }
        __syncthreads();
        const bool write_qk = scal[2] != 0.f;
        if (tid < 3 * KD && (part_ == 2 || write_qk)) {
#pragma unroll
            for (int i = 0; i < CK - 2; ++i) hist[(int64_t)c * (CK - 1) + i] = h[i + 1];
            hist[(int64_t)c * (CK - 1) + CK - 2] = x;
        }
    }
    for (int t = 0; t < T; ++t) {
        const float* row = proj + (int64_t)t * proj_stride;
        // q, k: the GQA key head's slices of the conv output; l2-normalised (engine.cpp:246-251)
        float qv = 0.f, kv = 0.f;
        if (tid < KD) {
            qv = conv_w ? cx[tid] : row[qk_head * KD + tid];
            kv = conv_w ? cx[KD + tid] : row[dd.KH * KD + qk_head * KD + tid];
        }
        const float qss = block_sum<kDeltaThreads>(tid < KD ? qv * qv : 0.f, red);
        const float kss = block_sum<kDeltaThreads>(tid < KD ? kv * kv : 0.f, red);
        if (tid < KD) {
            qs[tid] = qv * (1.0f / sqrtf(qss + kEps)) / qscale;
            ks[tid] = kv * (1.0f / sqrtf(kss + kEps));
        }
        if (tid < VD) vs[tid] = conv_w ? cx[2 * KD + tid] : row[2 * dd.KH * KD + head * VD + tid];
        if (tid == 0) {
            const float a = row[dd.a_off + head], b = row[dd.b_off + head];
            scal[0] = sigmoidf_ref(b);                                     // beta
            scal[1] = expf(-expf(alog[head]) * softplusf_ref(a + dt[head]));  // exp(decay)
        }
        __syncthreads();
        const float beta = scal[0], gdecay = scal[1];
        // S <- decay * S; pred = k^T S
        float p = 0.f;
#pragma unroll
        for (int r = 0; r < RG; ++r) {
            S[r] *= gdecay;
            p += ks[g * RG + r] * S[r];
        }
        part[g][v] = p;
        __syncthreads();
        float pred = 0.f;
#pragma unroll
        for (int i = 0; i < G; ++i) pred += part[i][v];
        const float dv = vs[v] - pred;
        // S += k (beta (v - pred)); o = q^T S
        float o = 0.f;
#pragma unroll
        for (int r = 0; r < RG; ++r) {
            S[r] += ks[g * RG + r] * beta * dv;
            o += qs[g * RG + r] * S[r];
        }
        __syncthreads();
        part[g][v] = o;
        __syncthreads();
        float ov = 0.f;
        if (tid < VD) {
#pragma unroll
            for (int i = 0; i < G; ++i) ov += part[i][tid];
        }
        if (norm) {
            // gated RMS: o * rsqrt(mean o^2 + eps) * norm * silu(z) (engine.cpp:237-242)
            const float oss = block_sum<kDeltaThreads>(tid < VD ? ov * ov : 0.f, red);
            if (tid < VD) {
                const float scale = 1.0f / sqrtf(oss / (float)VD + kEps);
                const float z = row[dd.z_off + head * VD + tid];
                out[(int64_t)t * out_stride + head * VD + tid] = ov * (scale * norm[tid] * siluf_ref(z));
            }
        } else if (tid < VD) {
            out[(int64_t)t * out_stride + head * VD + tid] = ov;  // gated RMS left to the out projection
        }
        __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < RG; ++r) st[(int64_t)(g * RG + r) * VD + v] = S[r];
}

// ---- attention inputs (engine.cpp:327-346): per token, q/gate split, RMS of
// q and k with (1 + w), partial RoPE, K/V appended to the cache at pos + t.
__global__ void __launch_bounds__(256) attn_prep_kernel(float* __restrict__ proj, int64_t proj_stride,
                                                        AttnDims ad, const float* __restrict__ qn1,
                                                        const float* __restrict__ kn1, const int* __restrict__ pos,
                                                        float* __restrict__ kcache, float* __restrict__ vcache) {
    griddep_wait();
    griddep_launch_dependents();
    const int t = blockIdx.x, h = blockIdx.y;  // h < AH: query head; AH <= h < AH + KVH: key head
    const int AD = ad.AD, RD = ad.RD;
    float* row = proj + (int64_t)t * proj_stride;
    const int position = *pos + t;
    const bool is_q = h < ad.AH;
    float* x = is_q ? row + (int64_t)h * 2 * AD : row + 2 * ad.AH * AD + (int64_t)(h - ad.AH) * AD;
    const float* w1 = is_q ? qn1 : kn1;
    __shared__ float red[8], buf[512];
    float ss = 0.f;
    for (int i = threadIdx.x; i < AD; i += 256) ss += x[i] * x[i];
    ss = block_sum<256>(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)AD + kEps);
    for (int i = threadIdx.x; i < AD; i += 256) buf[i] = x[i] * scale * w1[i];
    __syncthreads();
    for (int i = threadIdx.x; i < AD; i += 256) {
        float v = buf[i];
        if (i < RD) {
            const int half = RD / 2, j = i < half ? i : i - half;
            const float angle = (float)position / powf(kTheta, 2.0f * (float)j / (float)RD);
            const float c = cosf(angle), s = sinf(angle);
            v = i < half ? buf[i] * c - buf[i + half] * s : buf[i] * c + buf[i - half] * s;
        }
        if (is_q) {
            x[i] = v;
        } else {
            const int64_t off = ((int64_t)position * ad.KVH + (h - ad.AH)) * AD + i;
            kcache[off] = v;
            vcache[off] = row[2 * ad.AH * AD + (int64_t)ad.KVH * AD + (int64_t)(h - ad.AH) * AD + i];
        }
    }
}

// ---- causal attention, split over keys (engine.cpp:347-367).  CTA = (key
// split, kv head, token): each warp walks keys j = split0 + w, + 8, ... for all
// G query heads of the kv head with an online softmax; partial (m, l, o) per
// split go to `part`, merged by attn_merge_kernel.
constexpr int kAttnWarps = 8;
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(const float* __restrict__ proj,
                                                                     int64_t proj_stride, AttnDims ad,
                                                                     const int* __restrict__ pos,
                                                                     const float* __restrict__ kcache,
                                                                     const float* __restrict__ vcache,
                                                                     int split_len, float* __restrict__ part) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int kMaxG = 8, kPerLane = 8;  // AD = 256 = 32 lanes x 8
    const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
    const int nsplit = gridDim.x, G = ad.AH / ad.KVH, AD = ad.AD;
    const int last = *pos + t;  // keys 0..last
    const int j0 = split * split_len, j1 = min(last + 1, j0 + split_len);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* row = proj + (int64_t)t * proj_stride;
    const float inv = 1.0f / sqrtf((float)AD);
    float q[kMaxG][kPerLane], o[kMaxG][kPerLane], m[kMaxG], l[kMaxG];
#pragma unroll
    for (int gi = 0; gi < kMaxG; ++gi) {
        m[gi] = -INFINITY;
        l[gi] = 0.f;
#pragma unroll
        for (int e = 0; e < kPerLane; ++e) {
            o[gi][e] = 0.f;
            q[gi][e] = gi < G ? row[(int64_t)(kvh * G + gi) * 2 * AD + lane * kPerLane + e] : 0.f;
        }
    }
    for (int j = j0 + warp; j < j1; j += kAttnWarps) {
        const float* kr = kcache + ((int64_t)j * ad.KVH + kvh) * AD + lane * kPerLane;
        const float* vr = vcache + ((int64_t)j * ad.KVH + kvh) * AD + lane * kPerLane;
        float kv[kPerLane], vv[kPerLane];
        *reinterpret_cast<float4*>(kv) = *reinterpret_cast<const float4*>(kr);
        *reinterpret_cast<float4*>(kv + 4) = *reinterpret_cast<const float4*>(kr + 4);
        *reinterpret_cast<float4*>(vv) = *reinterpret_cast<const float4*>(vr);
        *reinterpret_cast<float4*>(vv + 4) = *reinterpret_cast<const float4*>(vr + 4);
#pragma unroll
        for (int gi = 0; gi < kMaxG; ++gi) {
            if (gi >= G) break;
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < kPerLane; ++e) d += q[gi][e] * kv[e];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            const float s = d * inv;
            const float mn = fmaxf(m[gi], s);
            const float corr = expf(m[gi] - mn), p = expf(s - mn);
            l[gi] = l[gi] * corr + p;
#pragma unroll
            for (int e = 0; e < kPerLane; ++e) o[gi][e] = o[gi][e] * corr + p * vv[e];
            m[gi] = mn;
        }
    }
    // merge the 8 warps in shared memory
    __shared__ float sm[kAttnWarps][kMaxG], sl[kAttnWarps][kMaxG];
    __shared__ float so[kAttnWarps][256];
#pragma unroll
    for (int gi = 0; gi < kMaxG; ++gi) {
        if (gi < G) {  // uniform over the CTA
            if (lane == 0) {
                sm[warp][gi] = m[gi];
                sl[warp][gi] = l[gi];
            }
#pragma unroll
            for (int e = 0; e < kPerLane; ++e) so[warp][lane * kPerLane + e] = o[gi][e];
            __syncthreads();
            if (warp == 0) {
                float M = -INFINITY;
                for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm[w][gi]);
                float L = 0.f, acc[kPerLane] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int w = 0; w < kAttnWarps; ++w) {
                    const float c = sm[w][gi] == -INFINITY ? 0.f : expf(sm[w][gi] - M);
                    L += sl[w][gi] * c;
#pragma unroll
                    for (int e = 0; e < kPerLane; ++e) acc[e] += so[w][lane * kPerLane + e] * c;
                }
                // part[t][h][split] = {m, l, o[AD]}
                float* dst = part + (((int64_t)t * ad.AH + kvh * G + gi) * nsplit + split) * (AD + 2);
                if (lane == 0) {
                    dst[0] = M;
                    dst[1] = L;
                }
#pragma unroll
                for (int e = 0; e < kPerLane; ++e) dst[2 + lane * kPerLane + e] = acc[e];
            }
            __syncthreads();
        }
    }
}

// ---- decode attention (T = 1): CTA = (128-key split, kv head), 8 warps of 16
// keys.  Each warp streams 4 keys at a time (K and V rows, 8 KB) into its own
// two-stage shared-memory ring with cp.async, so its next keys are in flight
// while it computes; lanes own 8 of the 256 dims.  Partials (m, l, o) per
// (split, query head) go to `part` for attn_merge_kernel, as attn_split_kernel.
constexpr int kDecSplit = 128, kDecKeys = 4, kDecWarps = 8;
constexpr size_t kDecSmem = (size_t)kDecWarps * 2 * kDecKeys * 2 * 256 * 4;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

template <int kMaxG>  // query heads per kv head, at most
__global__ void __launch_bounds__(kDecWarps * 32) attn_decode_kernel(const float* __restrict__ proj, AttnDims ad,
                                                                     const int* __restrict__ pos,
                                                                     const float* __restrict__ kcache,
                                                                     const float* __restrict__ vcache,
                                                                     float* __restrict__ part) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ __align__(16) float dsm[];
    constexpr int kPer = 8;
    const int split = blockIdx.x, kvh = blockIdx.y, nsplit = gridDim.x;
    const int G = ad.AH / ad.KVH, AD = 256;
    const int last = *pos;  // keys 0..last (the new key is already in the cache)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w0 = split * kDecSplit + warp * (kDecSplit / kDecWarps);
    const int w1 = min(last + 1, w0 + kDecSplit / kDecWarps);
    float* ring = dsm + warp * (2 * kDecKeys * 2 * AD);  // [stage][key][K | V][256]
    const float inv = 1.0f / sqrtf((float)AD);
    float q[kMaxG][kPer], o[kMaxG][kPer], m[kMaxG], l[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            o[g][e] = 0.f;
            q[g][e] = g < G ? proj[(int64_t)(kvh * G + g) * 2 * AD + lane * kPer + e] : 0.f;
        }
    }
    auto issue = [&](int stage, int j0) {
#pragma unroll
        for (int kk = 0; kk < kDecKeys; ++kk) {
            const int j = j0 + kk;
            if (j < w1) {
                const int64_t off = ((int64_t)j * ad.KVH + kvh) * AD;
                float* dk = ring + (stage * kDecKeys + kk) * 2 * AD;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    cp_async16(dk + (lane + 32 * c) * 4, kcache + off + (lane + 32 * c) * 4);
                    cp_async16(dk + AD + (lane + 32 * c) * 4, vcache + off + (lane + 32 * c) * 4);
                }
            }
        }
        cp_async_commit();
    };
    if (w0 < w1) {
        issue(0, w0);
        issue(1, w0 + kDecKeys);
        int stage = 0;
        for (int j0 = w0; j0 < w1; j0 += kDecKeys, stage ^= 1) {
            cp_async_wait<1>();
            __syncwarp();
            const float* base = ring + stage * kDecKeys * 2 * AD;
#pragma unroll
            for (int kk = 0; kk < kDecKeys; ++kk) {
                if (j0 + kk >= w1) break;
                const float* kr = base + kk * 2 * AD + lane * kPer;
                const float4 k0 = *reinterpret_cast<const float4*>(kr);
                const float4 k1 = *reinterpret_cast<const float4*>(kr + 4);
                const float4 v0 = *reinterpret_cast<const float4*>(kr + AD);
                const float4 v1 = *reinterpret_cast<const float4*>(kr + AD + 4);
                const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
                const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int g = 0; g < kMaxG; ++g) {
                    if (g >= G) break;
                    float d = 0.f;
#pragma unroll
                    for (int e = 0; e < kPer; ++e) d += q[g][e] * kv[e];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
                    const float sc = d * inv;
                    const float mn = fmaxf(m[g], sc);
                    const float corr = expf(m[g] - mn), p = expf(sc - mn);
                    l[g] = l[g] * corr + p;
#pragma unroll
                    for (int e = 0; e < kPer; ++e) o[g][e] = o[g][e] * corr + p * vv[e];
                    m[g] = mn;
                }
            }
            __syncwarp();  // the stage is free again
            issue(stage, j0 + 2 * kDecKeys);
        }
        cp_async_wait<0>();
    }
    // merge the warps of the CTA per query head (shared memory reuses the ring)
    __syncthreads();
    float* sm_m = dsm;                         // [kDecWarps][kMaxG]
    float* sm_l = sm_m + kDecWarps * kMaxG;    // [kDecWarps][kMaxG]
    float* sm_o = sm_l + kDecWarps * kMaxG;    // [kDecWarps][256]
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;  // uniform over the CTA
        if (lane == 0) {
            sm_m[warp * kMaxG + g] = m[g];
            sm_l[warp * kMaxG + g] = l[g];
        }
#pragma unroll
        for (int e = 0; e < kPer; ++e) sm_o[warp * AD + lane * kPer + e] = o[g][e];
        __syncthreads();
        if (warp == 0) {
            float M = -INFINITY;
            for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, sm_m[w * kMaxG + g]);
            float L = 0.f, acc[kPer] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int w = 0; w < kDecWarps; ++w) {
                const float mw = sm_m[w * kMaxG + g];
                const float cw = mw == -INFINITY ? 0.f : expf(mw - M);
                L += sm_l[w * kMaxG + g] * cw;
#pragma unroll
                for (int e = 0; e < kPer; ++e) acc[e] += sm_o[w * AD + lane * kPer + e] * cw;
            }
            float* dst = part + ((int64_t)(kvh * G + g) * nsplit + split) * (AD + 2);
            if (lane == 0) {
                dst[0] = M;
                dst[1] = L;
            }
#pragma unroll
            for (int e = 0; e < kPer; ++e) dst[2 + lane * kPer + e] = acc[e];
        }
        __syncthreads();
    }
}

// Merge of the key splits of one (token, query head): softmax weights of the
// splits once in shared memory, then one output dim per thread (AD <= 256).
__global__ void __launch_bounds__(256) attn_merge_kernel(const float* __restrict__ part, int nsplit,
                                                         const float* __restrict__ proj, int64_t proj_stride,
                                                         AttnDims ad, float* __restrict__ out,
                                                         int64_t out_stride) {
    griddep_wait();
    griddep_launch_dependents();
    __shared__ float cw[256], red[8];
    const int t = blockIdx.x, h = blockIdx.y, AD = ad.AD;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t stride = AD + 2;
    const float* p = part + ((int64_t)t * ad.AH + h) * nsplit * stride;
    float mx = -INFINITY;
    for (int sp = tid; sp < nsplit; sp += 256) mx = fmaxf(mx, p[sp * stride]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) M = fmaxf(M, red[w]);
    __syncthreads();
    float Lp = 0.f, acc = 0.f;
    for (int s0 = 0; s0 < nsplit; s0 += 256) {
        const int sp = s0 + tid;
        float c = 0.f;
        if (sp < nsplit) {
            const float ms = p[sp * stride];
            c = ms == -INFINITY ? 0.f : expf(ms - M);
            Lp += c * p[sp * stride + 1];
        }
        cw[tid] = c;
        __syncthreads();
        const int n = min(256, nsplit - s0);
        if (tid < AD) {
            const float* col = p + (int64_t)s0 * stride + 2 + tid;
#pragma unroll 4
            for (int k = 0; k < n; ++k) acc += col[k * stride] * cw[k];
        }
        __syncthreads();
    }
    Lp = warp_sum(Lp);
    if (lane == 0) red[warp] = Lp;
    __syncthreads();
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) L += red[w];
    if (tid < AD) {
        const float gate = proj[(int64_t)t * proj_stride + (int64_t)h * 2 * AD + AD + tid];
        out[(int64_t)t * out_stride + (int64_t)h * AD + tid] = acc / L * sigmoidf_ref(gate);
    }
}

// ---- causal attention for a prompt (T > 1): flash-style tiles on CUDA cores.
// CTA = 64 query tokens of one query head; 64-key tiles of K and V stream
// through shared memory with an online softmax (engine.cpp:347-367 computes
// the same softmax(q.k / sqrt(AD)) V per token); the output is already gated
// by sigmoid(gate) (engine.cpp:368).  Thread (ty, tx) of 16 x 16 owns query
// rows 4ty..4ty+3: scores for keys tx + 16i, output dims 4tx + 64j; products
// accumulate with packed FFMA2.
constexpr int kFBQ = 64, kFBK = 64, kFD = 256, kFLd = kFD + 4, kFPd = kFBK + 4;
constexpr size_t kFlashSmem = (size_t)(2 * kFBQ * kFLd + kFBK * kFD + kFBQ * kFPd) * 4;

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__global__ void __launch_bounds__(256) attn_prefill_kernel(const float* __restrict__ proj, int64_t proj_stride, int T,
                                                           AttnDims ad, const int* __restrict__ pos,
                                                           const float* __restrict__ kcache,
                                                           const float* __restrict__ vcache, float* __restrict__ out,
                                                           int64_t out_stride) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ __align__(16) float fsm[];
    float* Qs = fsm;                 // [kFBQ][kFLd]
    float* Ks = Qs + kFBQ * kFLd;    // [kFBK][kFLd]
    float* Vs = Ks + kFBK * kFLd;    // [kFBK][kFD]
    float* Ps = Vs + kFBK * kFD;     // [kFBQ][kFPd]
    const int qt = blockIdx.x, h = blockIdx.y;
    const int G = ad.AH / ad.KVH, kvh = h / G;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int t0 = qt * kFBQ;
    const int pos0 = *pos;
    const int rows = min(kFBQ, T - t0);
    const int last_key = pos0 + t0 + rows - 1;
    const float inv = 1.0f / sqrtf((float)kFD);
    // Q tile (already RMS-normalised and rotated by attn_prep_kernel)
    for (int e = tid; e < kFBQ * kFD / 4; e += 256) {
        const int r = e / (kFD / 4), d4 = e % (kFD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows)
            v = reinterpret_cast<const float4*>(proj + (int64_t)(t0 + r) * proj_stride + (int64_t)h * 2 * kFD)[d4];
        reinterpret_cast<float4*>(Qs + r * kFLd)[d4] = v;
    }
    const int r0 = ty * 4;
    float m[4], l[4];
    float2 o[4][8];  // row a, dims 4tx + 64j (+0,1 | +2,3)
    int qpos[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -INFINITY;
        l[a] = 0.f;
        qpos[a] = pos0 + t0 + r0 + a;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[a][j] = make_float2(0.f, 0.f);
    }
    for (int k0 = 0; k0 <= last_key; k0 += kFBK) {
        __syncthreads();  // previous tile consumed
        for (int e = tid; e < kFBK * kFD / 4; e += 256) {
            const int r = e / (kFD / 4), d4 = e % (kFD / 4);
            const int j = k0 + r;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (j <= last_key) {
                const int64_t off = ((int64_t)j * ad.KVH + kvh) * kFD;
                kv = reinterpret_cast<const float4*>(kcache + off)[d4];
                vv = reinterpret_cast<const float4*>(vcache + off)[d4];
            }
            reinterpret_cast<float4*>(Ks + r * kFLd)[d4] = kv;
            reinterpret_cast<float4*>(Vs + r * kFD)[d4] = vv;
        }
        __syncthreads();
        // S = Q K^T: rows r0 + a, keys tx + 16 i; sc[a][i/2] packs keys (i, i+1)
        float2 sc[4][2];
#pragma unroll
        for (int a = 0; a < 4; ++a) sc[a][0] = sc[a][1] = make_float2(0.f, 0.f);
#pragma unroll 2
        for (int d4 = 0; d4 < kFD / 4; ++d4) {
            float4 q[4], k[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) q[a] = reinterpret_cast<const float4*>(Qs + (r0 + a) * kFLd)[d4];
#pragma unroll
            for (int i = 0; i < 4; ++i) k[i] = reinterpret_cast<const float4*>(Ks + (tx + 16 * i) * kFLd)[d4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int ip = 0; ip < 2; ++ip) {
                    const float4 ka = k[2 * ip], kb = k[2 * ip + 1];
                    float2 acc = sc[a][ip];
                    acc = ffma2(make_float2(q[a].x, q[a].x), make_float2(ka.x, kb.x), acc);
                    acc = ffma2(make_float2(q[a].y, q[a].y), make_float2(ka.y, kb.y), acc);
                    acc = ffma2(make_float2(q[a].z, q[a].z), make_float2(ka.z, kb.z), acc);
                    acc = ffma2(make_float2(q[a].w, q[a].w), make_float2(ka.w, kb.w), acc);
                    sc[a][ip] = acc;
                }
        }
        // online softmax per row over this tile (16 threads share a row)
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float s4[4] = {sc[a][0].x, sc[a][0].y, sc[a][1].x, sc[a][1].y};
            float tmax = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = k0 + tx + 16 * i;
                s4[i] = j <= qpos[a] ? s4[i] * inv : -INFINITY;
                tmax = fmaxf(tmax, s4[i]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mn = fmaxf(m[a], tmax);
            const float corr = mn == -INFINITY ? 1.f : expf(m[a] - mn);
            float psum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pv = s4[i] == -INFINITY ? 0.f : expf(s4[i] - mn);
                psum += pv;
                Ps[(r0 + a) * kFPd + tx + 16 * i] = pv;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[a] = l[a] * corr + psum;
            m[a] = mn;
            const float2 c2 = make_float2(corr, corr);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[a][j] = __fmul2_rn(o[a][j], c2);
        }
        __syncwarp();  // a row's probabilities come from the 16 threads of its half-warp
        // O += P V
#pragma unroll 2
        for (int j4 = 0; j4 < kFBK / 4; ++j4) {
            float4 p[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) p[a] = reinterpret_cast<const float4*>(Ps + (r0 + a) * kFPd)[j4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int key = 4 * j4 + jj;
                float4 v[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) v[c] = reinterpret_cast<const float4*>(Vs + key * kFD)[tx + 16 * c];
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float pa = jj == 0 ? p[a].x : jj == 1 ? p[a].y : jj == 2 ? p[a].z : p[a].w;
                    const float2 p2 = make_float2(pa, pa);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        o[a][2 * c] = ffma2(p2, make_float2(v[c].x, v[c].y), o[a][2 * c]);
                        o[a][2 * c + 1] = ffma2(p2, make_float2(v[c].z, v[c].w), o[a][2 * c + 1]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int r = r0 + a;
        if (r >= rows) continue;
        const float* gate = proj + (int64_t)(t0 + r) * proj_stride + (int64_t)h * 2 * kFD + kFD;
        float* dst = out + (int64_t)(t0 + r) * out_stride + (int64_t)h * kFD;
        const float invl = 1.0f / l[a];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int d = 4 * tx + 64 * c;
            const float4 g = *reinterpret_cast<const float4*>(gate + d);
            float4 res;
            res.x = o[a][2 * c].x * invl * sigmoidf_ref(g.x);
            res.y = o[a][2 * c].y * invl * sigmoidf_ref(g.y);
            res.z = o[a][2 * c + 1].x * invl * sigmoidf_ref(g.z);
            res.w = o[a][2 * c + 1].y * invl * sigmoidf_ref(g.w);
            *reinterpret_cast<float4*>(dst + d) = res;
        }
    }
}

// dense FFN SwiGLU over T tokens: out[t][i] = silu(g_i) * u_i; proj[t] holds
// the gate|up rows interleaved in fours, g(2j) g(2j+1) u(2j) u(2j+1).
__global__ void ffn_swiglu_kernel(const float* __restrict__ proj, int64_t proj_stride, int T, int I,
                                  float* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    const int64_t n = (int64_t)T * I;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = k / I, i = k - t * I;
        const int64_t c = (i >> 1) * 4 + (i & 1);
        const float g = proj[t * proj_stride + c], u = proj[t * proj_stride + c + 2];
        out[k] = siluf_ref(g) * u;  // engine.cpp:374
    }
}

__global__ void advance_kernel(int* pos, int by) {
    griddep_wait();
    griddep_launch_dependents();
    *pos += by;
}

}  // namespace

// ---- launchers -----------------------------------------------------------------

int launch_embed(const q3xk_matrix& m, const int* tokens, int T, float* out, cudaStream_t s) {
    const dim3 grid((m.cols + 255) / 256, T);
    if (launch_pdl(embed_kernel, grid, dim3(256), 0, s, (const uint8_t*)m.data, m.row_stride,
                   quant_bytes(m.type, m.cols), m.type, m.cols, tokens, T, out) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int launch_rms(const float* x, const float* w1, int n, int T, float* out, cudaStream_t s) {
    cudaError_t e;
    if (n <= 256 * 8)
        e = launch_pdl(rms_reg_kernel<8>, dim3(T), dim3(256), 0, s, x, w1, n, out);
    else if (n <= 256 * 16)
        e = launch_pdl(rms_reg_kernel<16>, dim3(T), dim3(256), 0, s, x, w1, n, out);
    else if (n <= 256 * 24)
        e = launch_pdl(rms_reg_kernel<24>, dim3(T), dim3(256), 0, s, x, w1, n, out);
    else
        e = launch_pdl(rms_kernel, dim3(T), dim3(256), 0, s, x, w1, n, out);
    if (e != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int launch_conv(float* proj, int64_t proj_stride, int T, int channels, const float* w, int CK, float* hist,
                cudaStream_t s) {
    if (CK < 2 || CK > 9) return Q3XK_EUNSUPPORTED;
    const dim3 grid((channels + 127) / 128);
    const cudaError_t e = CK == 4 ? launch_pdl(conv_kernel<4>, grid, dim3(128), 0, s, proj, proj_stride, T, channels,
                                               w, CK, hist)
                                  : launch_pdl(conv_kernel<0>, grid, dim3(128), 0, s, proj, proj_stride, T, channels,
                                               w, CK, hist);
    if (e != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int launch_conv_prefill(const float* proj, int64_t proj_stride, int T, int channels, const float* w, int CK,
                        float* hist, float* out, cudaStream_t s) {
    if (CK != 4) return Q3XK_EUNSUPPORTED;
    const dim3 grid((channels + 127) / 128, (T + kConvSeg - 1) / kConvSeg);
    if (launch_pdl(conv_prefill_kernel, grid, dim3(128), 0, s, proj, proj_stride, T, channels, w, hist, out) !=
        cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int launch_delta(const float* proj, int64_t proj_stride, int T, const DeltaDims& dd, const float* alog,
                 const float* dt, const float* norm, float* state, float* out, int64_t out_stride,
                 cudaStream_t s, const float* conv_w, float* hist, int CK, int* group_count) {
    if (dd.KD != 128 || dd.VD != 128 || dd.VH % dd.KH) return Q3XK_EUNSUPPORTED;
    if (conv_w && (T != 1 || CK != 4 || !hist || !group_count)) return Q3XK_EUNSUPPORTED;
    if (launch_pdl(delta_kernel, dim3(dd.VH), dim3(kDeltaThreads), 0, s, proj, proj_stride, T, dd, alog, dt, norm,
                   state, out, out_stride, conv_w, hist, group_count) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int launch_attention(float* proj, int64_t proj_stride, int T, const AttnDims& ad, const float* qn1,
                     const float* kn1, const int* pos, float* kcache, float* vcache, int capacity, float* part,
                     int split_len, float* out, int64_t out_stride, cudaStream_t s) {
    if (ad.AD != 256 || ad.AH % ad.KVH || ad.AH / ad.KVH > 8 || ad.RD > ad.AD) return Q3XK_EUNSUPPORTED;
    if (launch_pdl(attn_prep_kernel, dim3(T, ad.AH + ad.KVH), dim3(256), 0, s, proj, proj_stride, ad, qn1, kn1, pos,
                   kcache, vcache) != cudaSuccess)
        return Q3XK_ECUDA;
    if (T > 1) {
        static bool configured = false;
        if (!configured) {
            if (cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kFlashSmem) != cudaSuccess)
                return Q3XK_ECUDA;
            configured = true;
        }
        if (launch_pdl(attn_prefill_kernel, dim3((T + kFBQ - 1) / kFBQ, ad.AH), dim3(256), kFlashSmem, s,
                       (const float*)proj, proj_stride, T, ad, pos, (const float*)kcache, (const float*)vcache, out,
                       out_stride) != cudaSuccess)
            return Q3XK_ECUDA;
        count_launch(2);
        return Q3XK_OK;
    }
    if (T == 1 && split_len == kDecSplit) {
        static bool dec_configured = false;
        if (!dec_configured) {
            if (cudaFuncSetAttribute(attn_decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kDecSmem) != cudaSuccess ||
                cudaFuncSetAttribute(attn_decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kDecSmem) != cudaSuccess)
                return Q3XK_ECUDA;
            dec_configured = true;
        }
        const int nsplit = (capacity + kDecSplit - 1) / kDecSplit;
        const int G = ad.AH / ad.KVH;
        const cudaError_t e =
            G <= 4 ? launch_pdl(attn_decode_kernel<4>, dim3(nsplit, ad.KVH), dim3(kDecWarps * 32), kDecSmem, s,
                                (const float*)proj, ad, pos, (const float*)kcache, (const float*)vcache, part)
                   : launch_pdl(attn_decode_kernel<8>, dim3(nsplit, ad.KVH), dim3(kDecWarps * 32), kDecSmem, s,
                                (const float*)proj, ad, pos, (const float*)kcache, (const float*)vcache, part);
        if (e != cudaSuccess) return Q3XK_ECUDA;
        if (launch_pdl(attn_merge_kernel, dim3(T, ad.AH), dim3(256), 0, s, (const float*)part, nsplit,
                       (const float*)proj, proj_stride, ad, out, out_stride) != cudaSuccess)
            return Q3XK_ECUDA;
        count_launch(3);
        return Q3XK_OK;
    }
    const int nsplit = (capacity + split_len - 1) / split_len;
    if (launch_pdl(attn_split_kernel, dim3(nsplit, ad.KVH, T), dim3(kAttnWarps * 32), 0, s, (const float*)proj,
                   proj_stride, ad, pos, (const float*)kcache, (const float*)vcache, split_len, part) != cudaSuccess)
        return Q3XK_ECUDA;
    if (launch_pdl(attn_merge_kernel, dim3(T, ad.AH), dim3(256), 0, s, (const float*)part, nsplit,
                   (const float*)proj, proj_stride, ad, out, out_stride) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch(3);
    return Q3XK_OK;
}

int launch_ffn_swiglu(const float* proj, int64_t proj_stride, int T, int I, float* out, cudaStream_t s) {
    const int64_t n = (int64_t)T * I;
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    if (launch_pdl(ffn_swiglu_kernel, dim3(blocks), dim3(256), 0, s, proj, proj_stride, T, I, out) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int launch_advance(int* pos, int by, cudaStream_t s) {
    if (launch_pdl(advance_kernel, dim3(1), dim3(1), 0, s, pos, by) != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

}  // namespace q3xk
