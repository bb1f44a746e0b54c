// gemv.cu -- decode GEMV y = W x (and y += W x) on CUDA cores, sm_100a.
//
// Replaces the reference's one-CTA-per-row kernels with 1-byte loads and a
// per-element FP16 decode (engine.cu:546-612).  Decode GEMV is HBM-bound
// (~1.9 flop/B for Q8_0).  Two kernel families share the dequant arithmetic
// below: the ring kernel (gemv_ring_kernel, further down), which stages the
// weight stream through shared-memory rings filled by cp.async and is the
// default for plain Q8_0 / Q4_0 / BF16 GEMVs, and the register kernel
// (gemv_kernel), used for expert gathers and input transforms other than
// RMSNorm.  The register kernel is built around bytes in flight:
//
//  * Every CTA owns a contiguous, balanced range of rows (+-1 row), so all
//    SMs stream the same number of bytes.  Inside a CTA, thread t owns one
//    16-byte "unit" column (Q8_0: 16 weights, Q4_0: one 32-weight block,
//    BF16: 8 weights) and
//    kRows rows of a row group; a row's units are spread over the threads,
//    so every thread works on every row group (no imbalance within a CTA).
//  * Weights are read once with 128-bit L1::no_allocate loads, double
//    buffered in registers: the next row group's loads are in flight while
//    the current one is dequantised.  Measured on B200, plain vector loads
//    stream a 53 MB matrix faster than cp.async.bulk staging.
//  * x is prescaled once per CTA into shared memory, per unit, by a power of
//    two chosen from the unit's largest |x|.  A Q8_0 byte (stored as q+128)
//    or a Q4_0 nibble masked in place is then used directly as the float
//    n * 2^(pos-149) (exact; FP32 subnormals are kept), so the dequant costs
//    one LOP3 and half a packed FFMA2 per weight and no offset subtraction;
//    sum(n x) is rescaled once per unit and the +128 / +8 offsets removed
//    with the unit's sum of x.  Units whose x holds non-finite values or
//    magnitudes >= 2^104 use an exact "2^23 + n" PRMT decode instead.
//  * A row's partial sums meet in a warp butterfly, then in shared memory in
//    a fixed order: results are deterministic.
//  * Programmatic dependent launch: the first row group's weights are
//    requested before griddepcontrol.wait, i.e. while the previous kernel in
//    the stream is still finishing; x and y are only touched after it.
#include <mutex>
#include <type_traits>

#include <cuda.h>

#include "common.cuh"
#include "layers.cuh"

namespace q3xk {
namespace {

#ifndef Q3XK_GEMV_PDL
#define Q3XK_GEMV_PDL 1
#endif
#ifndef Q3XK_GEMV_MIN_BLOCKS
#define Q3XK_GEMV_MIN_BLOCKS 3
#endif
// CTAs per SM of the double-buffered kernels (two register batches per warp),
// used when a matrix has too few rows to fill the GPU without a K split.
constexpr int kDbBlocks = 2;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 4;  // rows per warp

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}
__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
    uint16_t r;
    asm("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

struct GemvParams {
    const uint8_t* w;  // first row record
    const float* x;
    float* y;
    int64_t row_stride;
    int64_t qbytes;  // quantised bytes per row (scales follow)
    int rows, cols;
    int accumulate;
    int units;   // 16-byte units per (virtual) row
    int ksplit;  // warps sharing a row group (1, 2, 4 or 8), each on a slice of K
    // Expert gathers (MoE): `ids` (device) picks experts of a pool whose
    // matrices are `expert_stride` bytes apart.
    // An id < 0 skips its slot: rows of a skipped slot are neither read nor
    // written (row gather); a skipped segment adds nothing (segment gather).
    const int* ids;
    int64_t expert_stride;
    int rows_per_expert;  // row gather: virtual row r = expert ids[r / rpe], row r % rpe
    int units_per_seg;    // segment gather: unit u reads expert ids[u / ups]
    // Input transform applied while x is staged (q3xk_xform): x_eff = f(x).
    int xform;
    const float* xw;   // RMS: (1 + w)[cols]; gated RMS: norm[group]
    const float* xz;   // gated RMS: gate z[cols]
    const float* xsw;  // SwiGLU: per-segment weights (or null)
    int xgroup;        // gated RMS: group size; SwiGLU: width W of [g | u] pairs
    // Epilogue: 1 = SwiGLU over interleaved rows (g g u u per 4-row group),
    // y[row / 2 + {0,1}] = (ew[slot] *) silu(g) * u.
    int epi;
    const float* ew;
    // Ring kernel: when set, CTA 0 also writes the transformed x here (the
    // RMSNorm output that later kernels of a decode step read).
    float* xout;
};

constexpr int kMaxXGroups = 64;
constexpr float kXEps = 1e-6f;  // engine.cpp:27

// Row addressing modes of the GEMV kernel.
enum GemvMode { kPlain = 0, kRowGather = 1, kSegGather = 2 };
constexpr int kMaxSegments = 16;

// Per-type geometry and arithmetic.  A unit's x values reach dot() as
// kChunks float4 in slot order; `gg` = {g, gs}: g = 2^(149-P) rescales
// sum(n x) on the fast path, gs = -offset * sum(x).
template <int TYPE>
struct Codec;

template <>
struct Codec<Q3XK_Q8_0> {
    // 16 weights (half a block, 16 bytes) per unit; two units share a scale.
    static constexpr int kCols = 16, kVecs = 1, kChunks = 4, kUnitsPerBlock = 2, kBatch = 2;
    static constexpr float kOffset = 128.f;
    // x slot k holds element k (byte k): byte position k % 4 of word k / 4;
    // positions 0..2 are masked in place (bit 8k), position 3 after >> 24.
    __device__ static int shift(int k) { return (k & 3) == 1 ? 8 : (k & 3) == 2 ? 16 : 0; }
    __device__ static int element(int k) { return k; }

    template <bool FAST>
    __device__ __forceinline__ static float dot(const uint4* q, const float4* x, float2 gg) {
        const uint32_t w[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
        float2 a = f2(0.f, 0.f), b = f2(0.f, 0.f);
        if (FAST) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a = __ffma2_rn(f2(bits_f(w[j] & 0xFFu), bits_f(w[j] & 0xFF00u)), f2(x[j].x, x[j].y), a);
                b = __ffma2_rn(f2(bits_f(w[j] & 0xFF0000u), bits_f(w[j] >> 24)), f2(x[j].z, x[j].w), b);
            }
            return fmaf((a.x + a.y) + (b.x + b.y), gg.x, gg.y);
        }
        const float2 off = f2(-8388736.0f, -8388736.0f);  // 2^23 + 128
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 v01 = __fadd2_rn(f2(byte_as_magic_float<0>(w[j]), byte_as_magic_float<1>(w[j])), off);
            const float2 v23 = __fadd2_rn(f2(byte_as_magic_float<2>(w[j]), byte_as_magic_float<3>(w[j])), off);
            a = __ffma2_rn(v01, f2(x[j].x, x[j].y), a);
            b = __ffma2_rn(v23, f2(x[j].z, x[j].w), b);
        }
        return (a.x + a.y) + (b.x + b.y);
    }
};

// Q4_0: word j of the 16-byte unit holds bytes 4j..4j+3; nibble position p
// (bits 4p..4p+3) is element 4j + p/2, +16 for odd p (q4.h:31-36).  x slot
// 8j + p holds that element; positions 0..5 are masked in place, 6 and 7
// after >> 8 (so they sit at bits 16 and 20).
template <>
struct Codec<Q3XK_Q4_0> {
    static constexpr int kCols = 32, kVecs = 1, kChunks = 8, kUnitsPerBlock = 1, kBatch = 1;
    static constexpr float kOffset = 8.f;
    __device__ static int shift(int k) {
        const int p = k & 7;
        return p < 6 ? 4 * p : 4 * p - 8;
    }
    __device__ static int element(int k) {
        const int j = k >> 3, p = k & 7;
        return 4 * j + (p >> 1) + (p & 1) * 16;
    }

    template <bool FAST>
    __device__ __forceinline__ static float dot(const uint4* q, const float4* x, float2 gg) {
        const uint32_t w[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
        float2 a = f2(0.f, 0.f), b = f2(0.f, 0.f);
        if (FAST) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 x0 = x[2 * j], x1 = x[2 * j + 1];
                const uint32_t h = w[j] >> 8;
                a = __ffma2_rn(f2(bits_f(w[j] & 0xFu), bits_f(w[j] & 0xF0u)), f2(x0.x, x0.y), a);
                b = __ffma2_rn(f2(bits_f(w[j] & 0xF00u), bits_f(w[j] & 0xF000u)), f2(x0.z, x0.w), b);
                a = __ffma2_rn(f2(bits_f(w[j] & 0xF0000u), bits_f(w[j] & 0xF00000u)), f2(x1.x, x1.y), a);
                b = __ffma2_rn(f2(bits_f(h & 0xF0000u), bits_f(h & 0xF00000u)), f2(x1.z, x1.w), b);
            }
            return fmaf((a.x + a.y) + (b.x + b.y), gg.x, gg.y);
        }
        const float2 off = f2(-8388616.0f, -8388616.0f);  // 2^23 + 8
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 x0 = x[2 * j], x1 = x[2 * j + 1];  // (lo0 hi0 lo1 hi1) (lo2 hi2 lo3 hi3)
            const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
            const float2 l01 = __fadd2_rn(f2(byte_as_magic_float<0>(lo), byte_as_magic_float<1>(lo)), off);
            const float2 l23 = __fadd2_rn(f2(byte_as_magic_float<2>(lo), byte_as_magic_float<3>(lo)), off);
            const float2 h01 = __fadd2_rn(f2(byte_as_magic_float<0>(hi), byte_as_magic_float<1>(hi)), off);
            const float2 h23 = __fadd2_rn(f2(byte_as_magic_float<2>(hi), byte_as_magic_float<3>(hi)), off);
            a = __ffma2_rn(l01, f2(x0.x, x0.z), a);
            b = __ffma2_rn(l23, f2(x1.x, x1.z), b);
            a = __ffma2_rn(h01, f2(x0.y, x0.w), a);
            b = __ffma2_rn(h23, f2(x1.y, x1.w), b);
        }
        return (a.x + a.y) + (b.x + b.y);
    }
};

template <>
struct Codec<Q3XK_BF16> {
    static constexpr int kCols = 8, kVecs = 1, kChunks = 2, kUnitsPerBlock = 1, kBatch = 2;
    static constexpr float kOffset = 0.f;
    __device__ static int shift(int) { return 0; }
    __device__ static int element(int k) { return k; }

    template <bool FAST>
    __device__ __forceinline__ static float dot(const uint4* q, const float4* x, float2) {
        const uint32_t w[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
        float2 a = __ffma2_rn(f2(bits_f(w[0] << 16), bits_f(w[0] & 0xFFFF0000u)), f2(x[0].x, x[0].y), f2(0.f, 0.f));
        float2 b = __ffma2_rn(f2(bits_f(w[1] << 16), bits_f(w[1] & 0xFFFF0000u)), f2(x[0].z, x[0].w), f2(0.f, 0.f));
        a = __ffma2_rn(f2(bits_f(w[2] << 16), bits_f(w[2] & 0xFFFF0000u)), f2(x[1].x, x[1].y), a);
        b = __ffma2_rn(f2(bits_f(w[3] << 16), bits_f(w[3] & 0xFFFF0000u)), f2(x[1].z, x[1].w), b);
        return (a.x + a.y) + (b.x + b.y);
    }
};

// Unit u's 16-byte chunk j lives at chunk swz(u, j) of the unit's slot, so the
// 8 lanes of a quarter warp (consecutive units) hit 8 different bank groups.
template <int TYPE>
__device__ __forceinline__ int swz(int u, int j) {
    return (j + u) & (Codec<TYPE>::kChunks - 1);
}

// Warp-level work: kRows consecutive rows and one of `ksplit` interleaved
// slices of their units; the warp's lanes walk the slice with a stride of 32
// units and load Codec::kBatch units per lane and row at once.
template <int TYPE>
struct Batch {
    static constexpr int kBatch = Codec<TYPE>::kBatch;
    uint4 q[kBatch][kRows];
    uint16_t d[kBatch][kRows];
};

// Unit index of batch b, entry i, for a warp on slice ks of ksplit.
__device__ __forceinline__ int unit_of(int lane, int b, int i, int kbatch, int ks, int ksplit) {
    return lane + 32 * ((b * kbatch + i) * ksplit + ks);
}

template <int TYPE, int KS, int MODE>
__device__ __forceinline__ void load_batch(Batch<TYPE>& bt, const GemvParams& p,
                                           const uint8_t* const* rec, int lane, int b, int ks,
                                           const int64_t* seg_off) {
    constexpr int kBatch = Codec<TYPE>::kBatch;
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
        int u = unit_of(lane, b, i, kBatch, ks, KS);
        if (u < p.units) {
            int64_t off = 0;
            if (MODE == kSegGather) {  // unit u of segment u / ups, at that expert's row
                const int seg = u / p.units_per_seg;
                off = seg_off[seg];
                u -= seg * p.units_per_seg;
            }
            if (MODE == kSegGather && off < 0) {  // skipped segment: zero weights (its x is zero too)
#pragma unroll
                for (int j = 0; j < kRows; ++j) {
                    bt.q[i][j] = make_uint4(0u, 0u, 0u, 0u);
                    bt.d[i][j] = 0;
                }
                continue;
            }
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                bt.q[i][j] = ldg_stream(rec[j] + off + (int64_t)u * 16);
                if (TYPE != Q3XK_BF16)
                    bt.d[i][j] = ldg_u16(rec[j] + off + p.qbytes + 2 * (u / Codec<TYPE>::kUnitsPerBlock));
            }
        }
    }
}

// Returns this warp's partial sum of row (b4 ? 2 : 0) + (b3 ? 1 : 0) in lanes
// 0, 8, 16 and 24 (transposed butterfly over the 4 rows).
template <int TYPE, bool FAST, int KS, int MODE, bool DB>
__device__ __forceinline__ float warp_rows(const GemvParams& p, const uint8_t* const* rec, int lane,
                                           int ks, Batch<TYPE>& A, const float4* xs4,
                                           const float2* gg, const int64_t* seg_off) {
    using C = Codec<TYPE>;
    constexpr int kC = C::kChunks;
    constexpr int kBatch = C::kBatch;
    float acc[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j) acc[j] = 0.f;
    const int span = 32 * kBatch * KS;
    const int nb = (p.units + span - 1) / span;  // batches per row group and slice
    auto compute = [&](const Batch<TYPE>& X, int b) {
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int u = unit_of(lane, b, i, kBatch, ks, KS);
            if (u < p.units) {
                float4 xr[kC];
#pragma unroll
                for (int j = 0; j < kC; ++j) xr[j] = xs4[u * kC + swz<TYPE>(u, j)];
                const float2 gu = gg[u];
#pragma unroll
                for (int j = 0; j < kRows; ++j) {
                    const float dv = C::template dot<FAST>(&X.q[i][j], xr, gu);
                    if (TYPE == Q3XK_BF16) acc[j] += dv;
                    else acc[j] = fmaf(f16_bits_to_float(X.d[i][j]), dv, acc[j]);
                }
            }
        }
    };
    if (DB) {
        // two register batches: the next one is in flight while this one is used
        Batch<TYPE> B;
        for (int b = 0; b < nb; b += 2) {
            if (b + 1 < nb) load_batch<TYPE, KS, MODE>(B, p, rec, lane, b + 1, ks, seg_off);
            compute(A, b);
            if (b + 2 < nb) load_batch<TYPE, KS, MODE>(A, p, rec, lane, b + 2, ks, seg_off);
            if (b + 1 < nb) compute(B, b + 1);
        }
    } else {
        for (int b = 0; b < nb; ++b) {
            if (b > 0) load_batch<TYPE, KS, MODE>(A, p, rec, lane, b, ks, seg_off);
            compute(A, b);
        }
    }
    const bool b4 = lane & 16, b3 = lane & 8;
    float k0 = b4 ? acc[2] : acc[0], k1 = b4 ? acc[3] : acc[1];
    const float s0 = b4 ? acc[0] : acc[2], s1 = b4 ? acc[1] : acc[3];
    k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
    k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
    float k = b3 ? k1 : k0;
    k += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}

// Writes elements [u N, u N + N) of the transformed input vector, in natural
// order, to dst (the unit's own slot of the staging area), 4 at a time:
//   RMS        x * scale * w1                 (engine.cpp:231-236, w1 = 1 + w')
//   gated RMS  x * (scale_g * norm * silu(z)) (engine.cpp:237-242), per group
//   SwiGLU     [wt_s *] silu(g) * u           (engine.cpp:374, :415-416)
template <int N>
__device__ __forceinline__ void stage_x(const GemvParams& p, int u, float* dst, const float* xstat) {
    const int e0 = u * N;  // every group / pair width is a multiple of N
    if (p.xform == Q3XK_XFORM_SWIGLU) {
        const int seg = e0 / p.xgroup;
        const float* g = p.x + e0 + seg * p.xgroup;  // g of pair `seg`; u follows at + W
        const float wt = p.xsw ? __ldg(p.xsw + seg) : 1.f;
#pragma unroll 2
        for (int i = 0; i < N / 4; ++i) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(g) + i);
            const float4 b = __ldg(reinterpret_cast<const float4*>(g + p.xgroup) + i);
            float4 h = make_float4(a.x * sigmoid_ref(a.x) * b.x, a.y * sigmoid_ref(a.y) * b.y,
                                   a.z * sigmoid_ref(a.z) * b.z, a.w * sigmoid_ref(a.w) * b.w);
            if (p.xsw) h = make_float4(wt * h.x, wt * h.y, wt * h.z, wt * h.w);
            reinterpret_cast<float4*>(dst)[i] = h;
        }
    } else if (p.xform == Q3XK_XFORM_RMS) {
        const float scale = xstat[0];
#pragma unroll 2
        for (int i = 0; i < N / 4; ++i) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p.x + e0) + i);
            const float4 w = __ldg(reinterpret_cast<const float4*>(p.xw + e0) + i);
            reinterpret_cast<float4*>(dst)[i] =
                make_float4(a.x * scale * w.x, a.y * scale * w.y, a.z * scale * w.z, a.w * scale * w.w);
        }
    } else {  // gated RMS
        const int g = e0 / p.xgroup, k0 = e0 - g * p.xgroup;
        const float scale = xstat[g];
#pragma unroll 2
        for (int i = 0; i < N / 4; ++i) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p.x + e0) + i);
            const float4 z = __ldg(reinterpret_cast<const float4*>(p.xz + e0) + i);
            const float4 n = __ldg(reinterpret_cast<const float4*>(p.xw + k0) + i);
            reinterpret_cast<float4*>(dst)[i] = make_float4(
                a.x * (scale * n.x * (z.x * sigmoid_ref(z.x))), a.y * (scale * n.y * (z.y * sigmoid_ref(z.y))),
                a.z * (scale * n.z * (z.z * sigmoid_ref(z.z))), a.w * (scale * n.w * (z.w * sigmoid_ref(z.w))));
        }
    }
}

// Elements [u N, u N + N) of the GEMV input: straight from x, or (XF) from
// the unit's staging slot that stage_x filled.
template <int N, bool XF>
__device__ __forceinline__ void unit_x(const GemvParams& p, int u, float (&v)[N], const float4* slot) {
    const float4* src = XF ? slot : reinterpret_cast<const float4*>(p.x + (int64_t)u * N);
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
        const float4 t = XF ? src[i] : __ldg(src + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
}

// Statistics of the input transform, once per CTA into xstat (shared):
// RMS: xstat[0] = 1 / sqrt(mean(x^2) + eps); gated RMS: the same per group.
__device__ __forceinline__ void x_stats(const GemvParams& p, float* xstat, float* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (p.xform == Q3XK_XFORM_RMS) {
        float ss = 0.f;
        for (int k = tid * 4; k < p.cols; k += kThreads * 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(p.x + k));
            ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int w = 0; w < kWarps; ++w) t += red[w];
            xstat[0] = 1.0f / sqrtf(t / (float)p.cols + kXEps);
        }
    } else if (p.xform == Q3XK_XFORM_GATED_RMS) {
        const int G = p.xgroup, groups = p.cols / G;
        for (int g = warp; g < groups; g += kWarps) {
            float ss = 0.f;
            for (int k = lane; k < G; k += 32) {
                const float t = __ldg(p.x + (int64_t)g * G + k);
                ss += t * t;
            }
            ss = warp_sum(ss);
            if (lane == 0) xstat[g] = 1.0f / sqrtf(ss / (float)G + kXEps);
        }
    }
    __syncthreads();
}

// Rows of pass `it` for the warp's row group: row0, live, rec[].
template <int MODE>
__device__ __forceinline__ void pass_rows(const GemvParams& p, int gb, int ge, int it, int gpc, int group,
                                          const uint8_t** rec, int& row0, bool& live) {
    const int gi = gb + it * gpc + group;
    live = gi < ge;
    row0 = gi * kRows;
    bool any = false;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        const int row = min(row0 + j, p.rows - 1);
        if (MODE == kRowGather) {
            const int e = p.ids[row / p.rows_per_expert];  // < 0: skipped slot (row 0 stands in)
            any |= e >= 0;
            rec[j] = e < 0 ? p.w
                           : p.w + (int64_t)e * p.expert_stride + (int64_t)(row % p.rows_per_expert) * p.row_stride;
        } else {
            rec[j] = p.w + (int64_t)row * p.row_stride;
        }
    }
    if (MODE == kRowGather) live = live && any;
}

// False for a row of a skipped slot (row gather), whose output is left as it is.
template <int MODE>
__device__ __forceinline__ bool row_kept(const GemvParams& p, int row) {
    return MODE != kRowGather || __ldg(p.ids + row / p.rows_per_expert) >= 0;
}

// The CTA's passes over its row groups [gb, ge): dot products, then the
// epilogue (y write / accumulate / SwiGLU), K slices combined in shared memory.
template <int TYPE, bool FAST, int KS, int MODE, bool DB>
__device__ __forceinline__ void gemv_passes(const GemvParams& p, const uint8_t** rec, Batch<TYPE>& A,
                                            const float4* xs4, const float2* gg, float* part,
                                            const int64_t* seg_off, int gb, int ge, int passes, int row0,
                                            bool live) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ks = warp % KS, group = warp / KS;
    constexpr int groups_per_cta = kWarps / KS;
    const int r = (lane & 16 ? 2 : 0) + (lane & 8 ? 1 : 0);
    for (int it = 0; it < passes; ++it) {
        if (it > 0) {
            pass_rows<MODE>(p, gb, ge, it, groups_per_cta, group, rec, row0, live);
            if (live) load_batch<TYPE, KS, MODE>(A, p, rec, lane, 0, ks, seg_off);
        }
        const float k = live ? warp_rows<TYPE, FAST, KS, MODE, DB>(p, rec, lane, ks, A, xs4, gg, seg_off) : 0.f;
        if (KS == 1) {
            if (p.epi) {
                const float u = __shfl_down_sync(0xffffffffu, k, 16);  // lanes 0, 8 <- rows 2, 3
                if ((lane == 0 || lane == 8) && live && row0 < p.rows && row_kept<MODE>(p, row0)) {
                    float h = k * sigmoid_ref(k) * u;
                    if (p.ew) h = __ldg(p.ew + row0 / p.rows_per_expert) * h;
                    p.y[row0 / 2 + (lane >> 3)] = h;
                }
            } else if ((lane & 7) == 0 && live && row0 + r < p.rows && row_kept<MODE>(p, row0 + r)) {
                float* yp = p.y + row0 + r;
                *yp = p.accumulate ? *yp + k : k;
            }
            continue;
        }
        // Slices of a row group meet in shared memory, added in slice order.
        if ((lane & 7) == 0) part[warp * kRows + r] = k;
        __syncthreads();
        const int gbase = gb + it * groups_per_cta;
        if (p.epi) {
            if (tid < groups_per_cta * 2) {
                const int g = tid / 2, rr = tid % 2;
                const int grow = (gbase + g) * kRows;
                if (gbase + g < ge && grow < p.rows && row_kept<MODE>(p, grow)) {
                    float vg = 0.f, vu = 0.f;
#pragma unroll
                    for (int sl = 0; sl < KS; ++sl) {
                        vg += part[(g * KS + sl) * kRows + rr];
                        vu += part[(g * KS + sl) * kRows + rr + 2];
                    }
                    float h = vg * sigmoid_ref(vg) * vu;
                    if (p.ew) h = __ldg(p.ew + grow / p.rows_per_expert) * h;
                    p.y[grow / 2 + rr] = h;
                }
            }
        } else if (tid < groups_per_cta * kRows) {
            const int g = tid / kRows, rr = tid % kRows;
            const int row = (gbase + g) * kRows + rr;
            if (gbase + g < ge && row < p.rows && row_kept<MODE>(p, row)) {
                float v = 0.f;
#pragma unroll
                for (int sl = 0; sl < KS; ++sl) v += part[(g * KS + sl) * kRows + rr];
                p.y[row] = p.accumulate ? p.y[row] + v : v;
            }
        }
        __syncthreads();  // part[] is reused by the next pass
    }
}

// XF: the input transform is compiled in (p.xform may be non-zero).
// DB: two register batches per warp (kDbBlocks CTAs per SM instead of 3).
template <int TYPE, int KS, int MODE, bool XF, bool DB>
__global__ void __launch_bounds__(kThreads, DB ? kDbBlocks : Q3XK_GEMV_MIN_BLOCKS) gemv_kernel(const GemvParams p) {
    using C = Codec<TYPE>;
    static_assert(kRows == 4, "the transposed row reduction is written for 4 rows");
    extern __shared__ __align__(16) float smem[];
    float4* xs4 = reinterpret_cast<float4*>(smem);                              // units * kChunks
    float2* gg = reinterpret_cast<float2*>(smem + (size_t)p.units * C::kCols);  // units
    float* part = reinterpret_cast<float*>(gg + p.units);                      // kWarps * kRows

    griddep_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ks = warp % KS;                 // K slice of this warp
    constexpr int groups_per_cta = kWarps / KS;  // row groups per CTA and pass
    const int group = warp / KS;
    // This CTA's balanced share of the row groups (4 rows each): [gb, ge).
    const int64_t gt = (p.rows + kRows - 1) / kRows;
    const int gb = (int)(blockIdx.x * gt / gridDim.x), ge = (int)((blockIdx.x + 1) * gt / gridDim.x);
    const int passes = (ge - gb + groups_per_cta - 1) / groups_per_cta;  // uniform over the CTA
    __shared__ int64_t seg_off[kMaxSegments];
    const uint8_t* rec[kRows];
    Batch<TYPE> A;
    int row0 = 0;
    bool live = false;
    if (MODE == kPlain) {
        pass_rows<MODE>(p, gb, ge, 0, groups_per_cta, group, rec, row0, live);
        // The first batch of weights is requested before waiting on the previous kernel.
        if (live) load_batch<TYPE, KS, MODE>(A, p, rec, lane, 0, ks, seg_off);
        griddep_wait();  // x and (when accumulating) y may be written by the previous kernel
    } else {
        griddep_wait();  // the expert ids come from the previous kernel
        if (MODE == kSegGather) {
            if (tid < p.units / p.units_per_seg) {
                const int e = p.ids[tid];
                seg_off[tid] = e < 0 ? -1 : (int64_t)e * p.expert_stride;  // -1: skipped segment
            }
            __syncthreads();
        }
        pass_rows<MODE>(p, gb, ge, 0, groups_per_cta, group, rec, row0, live);
        if (live) load_batch<TYPE, KS, MODE>(A, p, rec, lane, 0, ks, seg_off);
    }

    __shared__ float xstat[XF ? kMaxXGroups : 1], xred[kWarps];
    if (XF && (p.xform == Q3XK_XFORM_RMS || p.xform == Q3XK_XFORM_GATED_RMS)) x_stats(p, xstat, xred);

    // Prescale x per unit into shared memory (16-byte chunks, swizzled).
    int slow = 0;
    for (int u = tid; u < p.units; u += kThreads) {
        float v[C::kCols];
        if (XF) stage_x<C::kCols>(p, u, reinterpret_cast<float*>(xs4 + u * C::kChunks), xstat);
        unit_x<C::kCols, XF>(p, u, v, xs4 + u * C::kChunks);
        if (MODE == kSegGather && seg_off[u / p.units_per_seg] < 0)
#pragma unroll
            for (int k = 0; k < C::kCols; ++k) v[k] = 0.f;
        int P = 0;
        float2 gu = f2(1.f, 0.f);
        if (TYPE != Q3XK_BF16) {
            uint32_t emax = 0;
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < C::kCols; ++k) {
                emax = max(emax, (__float_as_uint(v[k]) >> 23) & 0xFFu);
                sum += v[k];
            }
            // Exponents up to 103 keep every prescaled value finite.
            slow |= (emax == 0xFFu || (int)emax - 127 > 103) ? 1 : 0;
            P = min(127, max(23, 126 - ((int)emax - 127)));
            gu = f2(pow2f(149 - P), -C::kOffset * sum);
        }
#pragma unroll
        for (int j = 0; j < C::kChunks; ++j) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int kk = 4 * j + e;
                o[e] = TYPE == Q3XK_BF16 ? v[kk] : v[C::element(kk)] * pow2f(P - C::shift(kk));
            }
            xs4[u * C::kChunks + swz<TYPE>(u, j)] = make_float4(o[0], o[1], o[2], o[3]);
        }
        gg[u] = gu;
    }
    const int any_slow = __syncthreads_or(slow);
    if (any_slow) {
        // Exact fallback for the whole CTA: unscaled x in the same slot order.
        for (int u = tid; u < p.units; u += kThreads) {
            float v[C::kCols];
            if (XF) stage_x<C::kCols>(p, u, reinterpret_cast<float*>(xs4 + u * C::kChunks), xstat);
            unit_x<C::kCols, XF>(p, u, v, xs4 + u * C::kChunks);
            if (MODE == kSegGather && seg_off[u / p.units_per_seg] < 0)
#pragma unroll
                for (int k = 0; k < C::kCols; ++k) v[k] = 0.f;
#pragma unroll
            for (int j = 0; j < C::kChunks; ++j)
                xs4[u * C::kChunks + swz<TYPE>(u, j)] =
                    make_float4(v[C::element(4 * j)], v[C::element(4 * j + 1)],
                                v[C::element(4 * j + 2)], v[C::element(4 * j + 3)]);
        }
        __syncthreads();
    }
    if (any_slow)
        gemv_passes<TYPE, false, KS, MODE, DB>(p, rec, A, xs4, gg, part, seg_off, gb, ge, passes, row0, live);
    else
        gemv_passes<TYPE, true, KS, MODE, DB>(p, rec, A, xs4, gg, part, seg_off, gb, ge, passes, row0, live);
}

// ---- Ring-staged GEMV (plain row addressing, Q8_0 / Q4_0 / BF16) -----------
//
// The weight stream goes through a per-warp ring of shared-memory stages
// filled with cp.async (16 bytes per copy, no registers held while in
// flight), and each ring is filled before griddepcontrol.wait: while the
// previous kernel finishes and x is prescaled, ~200 KB per SM are already on
// their way.  Measured on B200, a 53.5 MB read staged this way takes 7.9 us
// per launch in a chain (6.7 TB/s) against 9.2 us for register-held loads.
//
// One CTA per SM with RW warps (16-24: enough eligible warps to hide the
// shared-memory and FMA latencies of the dequant).  The CTA owns a balanced
// range of 4-row groups; warp w takes groups w, w + RW, ...  A group's K runs
// through the ring in stages of 64 units (two 16-byte units per lane and
// row, each copied by that lane itself from a coalesced 512-byte span), so a
// warp's stages run back to back across its groups.  A stage holds the 4
// rows' quants [row][half][lane] and then their scales (copied by the first
// lanes, read after __syncwarp).  x is prescaled once per CTA into shared
// memory, unit by unit, with the chunks of a unit permuted so that 8
// consecutive units hit 8 different bank groups; an RMSNorm of x (the
// decode norms) is applied while staging it, its statistics computed once
// per CTA.  Arithmetic per unit is the register kernel's (Codec::dot, one FMA
// of the unit's scale into the row sum -- BF16 rows have no scales; the row
// sums meet in the same butterfly).  Deterministic.
constexpr int kUPL = 2;  // 16-byte units per lane and row in a stage

template <int TYPE>
struct RingGeo {
    using C = Codec<TYPE>;
    // scale bytes per row and stage (BF16 rows carry none)
    static constexpr int kSB = TYPE == Q3XK_BF16 ? 0 : 64 * kUPL / C::kUnitsPerBlock;
    static constexpr int kSPieces = kSB / 16;                   // 16-byte scale copies per row
    static constexpr int kQBytes = kRows * kUPL * 512;          // quants of a stage
    static constexpr int kStage = kQBytes + kRows * kSB;
    static_assert(kRows * kSPieces <= 32, "scale copies must fit one warp");
    // float4 slot of chunk j of unit u in the x area (the permutation depends
    // only on u mod 8, i.e. on the lane)
    __device__ static int xslot(int u, int j) {
        return C::kChunks == 2 ? u * 2 + (j ^ ((u >> 2) & 1))
             : C::kChunks == 4 ? u * 4 + (j ^ ((u >> 1) & 3)) : u * 8 + (j ^ (u & 7));
    }
};

template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async16_s(uint32_t saddr, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gmem) : "memory");
}

// Issue side of a warp's ring: the next stage to copy (its group, its stage
// within the group, its slot) and this lane's running source pointers into
// the group's 4 row records.  FULL: K is a whole number of stages, so no
// copy needs a bounds check.
template <int TYPE, int RW, int S, bool FULL>
struct RingIssue {
    using G = RingGeo<TYPE>;
    const uint8_t* q[kRows];  // this lane's first unit of the next stage, per row
    const uint8_t* sc;        // this lane's scale piece of the next stage (lanes < 4 * kSPieces)
    uint32_t dq, ds;          // shared addresses of the same in slot 0
    int grp, c, slot, t;

    __device__ __forceinline__ void set_rows(const GemvParams& p, int gb, int warp, int lane) {
        const int row0 = (gb + warp + RW * grp) * kRows;
#pragma unroll
        for (int j = 0; j < kRows; ++j)
            q[j] = p.w + (int64_t)min(row0 + j, p.rows - 1) * p.row_stride + lane * 16;
        const int js = (lane / G::kSPieces) & (kRows - 1), pc = lane % G::kSPieces;
        sc = p.w + (int64_t)min(row0 + js, p.rows - 1) * p.row_stride + p.qbytes + pc * 16;
    }
    __device__ __forceinline__ void init(const GemvParams& p, uint8_t* wring, int gb, int warp, int lane, int ng) {
        grp = c = slot = t = 0;
        const uint32_t base = (uint32_t)__cvta_generic_to_shared(wring);
        dq = base + lane * 16;
        ds = base + G::kQBytes + (lane / G::kSPieces) * G::kSB + (lane % G::kSPieces) * 16;
        if (ng > 0) set_rows(p, gb, warp, lane);
    }
    // Copies the next stage (if any) into its slot and commits one group of copies.
    __device__ __forceinline__ void issue(const GemvParams& p, int gb, int warp, int lane, int ng, int nst,
                                          int total, int nblocks) {
        if (t < total) {
            const uint32_t off = (uint32_t)slot * G::kStage;
#pragma unroll
            for (int h = 0; h < kUPL; ++h) {
                if (FULL || c * 32 * kUPL + h * 32 + lane < p.units) {
#pragma unroll
                    for (int j = 0; j < kRows; ++j) cp_async16_s(dq + off + (j * kUPL + h) * 512, q[j] + h * 512);
                }
            }
            if (lane < kRows * G::kSPieces && (FULL || (c * G::kSB + (lane % G::kSPieces) * 16) / 2 < nblocks))
                cp_async16_s(ds + off, sc);
#pragma unroll
            for (int j = 0; j < kRows; ++j) q[j] += 512 * kUPL;
            sc += G::kSB;
            ++t;
            slot = slot + 1 == S ? 0 : slot + 1;
            if (++c == nst) {
                c = 0;
                if (++grp < ng) set_rows(p, gb, warp, lane);
            }
        }
        cp_async_commit();
    }
};

template <int TYPE, int RW, int S, bool FULL, bool FAST>
__device__ __forceinline__ void ring_main(const GemvParams& p, RingIssue<TYPE, RW, S, FULL>& is, const float4* xs4,
                                          const float2* gg, uint8_t* wring, int gb, int warp, int lane, int ng,
                                          int nst, int total, int nblocks) {
    using C = Codec<TYPE>;
    using G = RingGeo<TYPE>;
    float acc[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j) acc[j] = 0.f;
    // x chunk offsets of this lane's units (the permutation repeats every 8 units)
    int xo[C::kChunks];
#pragma unroll
    for (int k = 0; k < C::kChunks; ++k) xo[k] = G::xslot(lane, k);
    int c = 0, grp = 0, slot = 0;
#pragma unroll 1
    for (int t = 0; t < total; ++t) {
        cp_async_wait<S - 1>();
        __syncwarp();
        const uint8_t* st = wring + slot * G::kStage;
#pragma unroll
        for (int h = 0; h < kUPL; ++h) {
            const int u = c * 32 * kUPL + h * 32;  // this lane's unit is u + lane
            if (FULL || u + lane < p.units) {
                const float4* xu = xs4 + u * C::kChunks;
                float4 xr[C::kChunks];
#pragma unroll
                for (int k = 0; k < C::kChunks; ++k) xr[k] = xu[xo[k]];
                const float2 gu = gg[u + lane];
                const int sidx = (h * 32 + lane) / C::kUnitsPerBlock;  // the unit's scale within the stage
#pragma unroll
                for (int j = 0; j < kRows; ++j) {
                    const uint4 qv = *reinterpret_cast<const uint4*>(st + (j * kUPL + h) * 512 + lane * 16);
                    if (TYPE == Q3XK_BF16) {
                        acc[j] += C::template dot<FAST>(&qv, xr, gu);
                    } else {
                        const float d = f16_bits_to_float(
                            *reinterpret_cast<const uint16_t*>(st + G::kQBytes + j * G::kSB + sidx * 2));
                        acc[j] = fmaf(d, C::template dot<FAST>(&qv, xr, gu), acc[j]);
                    }
                }
            }
        }
        __syncwarp();  // every lane has read this slot (scales included) before it is refilled
        is.issue(p, gb, warp, lane, ng, nst, total, nblocks);
        slot = slot + 1 == S ? 0 : slot + 1;
        if (++c == nst) {  // group done: 4 row sums meet in the transposed butterfly
            c = 0;
            const int row0 = (gb + warp + RW * grp) * kRows;
            ++grp;
            const bool b4 = lane & 16, b3 = lane & 8;
            float k0 = b4 ? acc[2] : acc[0], k1 = b4 ? acc[3] : acc[1];
            const float s0 = b4 ? acc[0] : acc[2], s1 = b4 ? acc[1] : acc[3];
            k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
            k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
            float k = b3 ? k1 : k0;
            k += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
            k += __shfl_xor_sync(0xffffffffu, k, 4);
            k += __shfl_xor_sync(0xffffffffu, k, 2);
            k += __shfl_xor_sync(0xffffffffu, k, 1);
            if (p.epi) {
                const float uu = __shfl_down_sync(0xffffffffu, k, 16);  // lanes 0, 8 <- rows 2, 3
                if ((lane == 0 || lane == 8) && row0 < p.rows) p.y[row0 / 2 + (lane >> 3)] = k * sigmoid_ref(k) * uu;
            } else {
                const int r = (lane & 16 ? 2 : 0) + (lane & 8 ? 1 : 0);
                if ((lane & 7) == 0 && row0 + r < p.rows) {
                    float* yp = p.y + row0 + r;
                    *yp = p.accumulate ? *yp + k : k;
                }
            }
#pragma unroll
            for (int j = 0; j < kRows; ++j) acc[j] = 0.f;
        }
    }
}

template <int TYPE, int RW, int S, bool FULL>
__global__ void __launch_bounds__(RW * 32, 1) gemv_ring_kernel(const GemvParams p) {
    using C = Codec<TYPE>;
    using G = RingGeo<TYPE>;
    extern __shared__ __align__(128) uint8_t rsm[];
    const int nblocks = p.cols / kBlock;
    float4* xs4 = reinterpret_cast<float4*>(rsm);                                      // units * kChunks
    float2* gg = reinterpret_cast<float2*>(rsm + (size_t)p.units * C::kCols * 4);      // units
    uint8_t* ring = rsm + (size_t)p.units * C::kCols * 4 + (((size_t)p.units * 8 + 127) & ~(size_t)127);

    griddep_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t gt = (p.rows + kRows - 1) / kRows;
    const int gb = (int)(blockIdx.x * gt / gridDim.x), ge = (int)((blockIdx.x + 1) * gt / gridDim.x);
    const int ng = ge - gb > warp ? (ge - gb - warp + RW - 1) / RW : 0;  // this warp's groups
    const int nst = (p.units + 32 * kUPL - 1) / (32 * kUPL);              // stages per group
    const int total = ng * nst;
    uint8_t* const wring = ring + (size_t)warp * S * G::kStage;

    RingIssue<TYPE, RW, S, FULL> is;
    is.init(p, wring, gb, warp, lane, ng);
#pragma unroll 1
    for (int t = 0; t < S; ++t) is.issue(p, gb, warp, lane, ng, nst, total, nblocks);
    griddep_wait();  // x and (when accumulating) y may be written by the previous kernel

    // RMSNorm of x applied while staging it (p.xform == RMS): x * scale * w1,
    // scale = 1 / sqrt(mean(x^2) + eps) (engine.cpp:231-236), the statistics
    // from one pass over x by the whole CTA.
    float rscale = 1.f;
    if (p.xform == Q3XK_XFORM_RMS) {
        __shared__ float red[RW];
        float ss = 0.f;
        for (int k = tid * 4; k < p.cols; k += RW * 32 * 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(p.x + k));
            ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < RW; ++w) tot += red[w];
        rscale = 1.0f / sqrtf(tot / (float)p.cols + kXEps);
    }
    auto load_unit = [&](int u, float (&v)[C::kCols]) {
        unit_x<C::kCols, false>(p, u, v, nullptr);
        if (p.xform == Q3XK_XFORM_RMS) {
            const float4* w4 = reinterpret_cast<const float4*>(p.xw + (int64_t)u * C::kCols);
#pragma unroll
            for (int i = 0; i < C::kCols / 4; ++i) {
                const float4 w = __ldg(w4 + i);
                v[4 * i] = v[4 * i] * rscale * w.x;
                v[4 * i + 1] = v[4 * i + 1] * rscale * w.y;
                v[4 * i + 2] = v[4 * i + 2] * rscale * w.z;
                v[4 * i + 3] = v[4 * i + 3] * rscale * w.w;
            }
        }
    };

    // Prescale x per unit (as the register kernel does); BF16 rows use x as it
    // is.  CTA 0 also hands the transformed x to later kernels (p.xout).
    int slow = 0;
    for (int u = tid; u < p.units; u += RW * 32) {
        float v[C::kCols];
        load_unit(u, v);
        if (p.xout && blockIdx.x == 0) {
#pragma unroll
            for (int i = 0; i < C::kCols / 4; ++i)
                reinterpret_cast<float4*>(p.xout + (int64_t)u * C::kCols)[i] =
                    make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
        if (TYPE == Q3XK_BF16) {
#pragma unroll
            for (int j = 0; j < C::kChunks; ++j)
                xs4[G::xslot(u, j)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            continue;
        }
        uint32_t emax = 0;
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < C::kCols; ++k) {
            emax = max(emax, (__float_as_uint(v[k]) >> 23) & 0xFFu);
            sum += v[k];
        }
        slow |= (emax == 0xFFu || (int)emax - 127 > 103) ? 1 : 0;
        const int P = min(127, max(23, 126 - ((int)emax - 127)));
#pragma unroll
        for (int j = 0; j < C::kChunks; ++j) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = v[C::element(4 * j + e)] * pow2f(P - C::shift(4 * j + e));
            xs4[G::xslot(u, j)] = make_float4(o[0], o[1], o[2], o[3]);
        }
        gg[u] = f2(pow2f(149 - P), -C::kOffset * sum);
    }
    const int any_slow = __syncthreads_or(slow);
    if (any_slow) {  // exact decode for the whole CTA: unscaled x in the same slots
        for (int u = tid; u < p.units; u += RW * 32) {
            float v[C::kCols];
            load_unit(u, v);
#pragma unroll
            for (int j = 0; j < C::kChunks; ++j)
                xs4[G::xslot(u, j)] = make_float4(v[C::element(4 * j)], v[C::element(4 * j + 1)],
                                                  v[C::element(4 * j + 2)], v[C::element(4 * j + 3)]);
        }
        __syncthreads();
        ring_main<TYPE, RW, S, FULL, false>(p, is, xs4, gg, wring, gb, warp, lane, ng, nst, total, nblocks);
    } else {
        ring_main<TYPE, RW, S, FULL, true>(p, is, xs4, gg, wring, gb, warp, lane, ng, nst, total, nblocks);
    }
    cp_async_wait<0>();
}

// Kernel family for plain GEMVs: 0 = automatic, 1 = register batches, 2 / 3 =
// ring with 16 / 24 warps (q3xk_gemv_set_family; tests run every family on
// the same inputs).
int g_gemv_family = 0;
constexpr size_t kRingSmemMax = 227 * 1024 - 256;  // dynamic; the kernel's static arrays take the rest

int sm_count_cached() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            count = 148;
    }
    return count;
}

// Split K over the warps of a CTA only when the matrix has too few rows to
// fill the GPU: the smallest split (1, 2, 4) whose grid keeps at least half
// of the resident CTA slots busy.  Every CTA prescales all of x, so small
// CTAs (large splits) pay that prologue over fewer rows.
int choose_ksplit(int rows, int units, int slots) {
    for (int ks = 1; ks <= 4; ks *= 2) {
        if (ks > 1 && units < 32 * ks) return ks / 2;
        const int64_t per = (int64_t)(kWarps / ks) * kRows;
        const int64_t ctas = (rows + per - 1) / per;
        const int64_t waves = (ctas + slots - 1) / slots;
        if (2 * ctas >= waves * slots) return ks;
    }
    return 4;
}

template <int TYPE>
size_t smem_bytes(const GemvParams& p) {
    return (size_t)p.units * Codec<TYPE>::kCols * 4 + (size_t)p.units * 8 + kWarps * kRows * 4;
}

template <int TYPE, int KS, int MODE, bool XF, bool DB>
int launch_ks(const GemvParams& p, size_t smem, cudaStream_t s) {
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        if (cudaFuncSetAttribute(gemv_kernel<TYPE, KS, MODE, XF, DB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024) != cudaSuccess)
            return Q3XK_ECUDA;
        configured = 200 * 1024;
    }
    // One CTA per resident slot (or per row group when there are fewer), each
    // with a balanced share of the row groups: every SM streams the same bytes.
    const int64_t groups = (p.rows + kRows - 1) / kRows;
    const int64_t slots = (int64_t)sm_count_cached() * (DB ? kDbBlocks : Q3XK_GEMV_MIN_BLOCKS);
    const int64_t grid = groups < slots ? groups : slots;
#if Q3XK_GEMV_PDL
    const cudaError_t e =
        launch_pdl(gemv_kernel<TYPE, KS, MODE, XF, DB>, dim3((unsigned)grid), dim3(kThreads), smem, s, p);
#else
    gemv_kernel<TYPE, KS, MODE, XF, DB><<<(unsigned)grid, kThreads, smem, s>>>(p);
    const cudaError_t e = cudaGetLastError();
#endif
    return e == cudaSuccess ? Q3XK_OK : Q3XK_ECUDA;
}

template <int TYPE, int MODE, bool XF, bool DB>
int launch_xf(const GemvParams& p, size_t smem, cudaStream_t s) {
    switch (p.ksplit) {
    case 1: return launch_ks<TYPE, 1, MODE, XF, DB>(p, smem, s);
    case 2: return launch_ks<TYPE, 2, MODE, XF, DB>(p, smem, s);
    case 4: return launch_ks<TYPE, 4, MODE, XF, DB>(p, smem, s);
    default: return launch_ks<TYPE, 8, MODE, XF, DB>(p, smem, s);
    }
}

// Kernel family: when the matrix needs a K split to fill the GPU (few rows),
// the double-buffered kernels (fewer, longer-lived warps with two batches in
// flight) stream faster; with enough rows the single-buffered ones at 3 CTAs
// per SM avoid a second wave.  Measured on B200 (Q8_0, us): 4096x4096 6.9 vs
// 5.6 double-buffered, 4096x12288 19.2 vs 15.3; 12352x4096 12.0 vs 16.1.
// Ring-kernel launch: one CTA per SM (fewer for small matrices); returns
// Q3XK_EUNSUPPORTED when the shape's shared memory does not fit.
template <int TYPE>
size_t ring_smem(const GemvParams& p, int rw, int stages) {
    return (size_t)p.units * Codec<TYPE>::kCols * 4 + (((size_t)p.units * 8 + 127) & ~(size_t)127) +
           (size_t)rw * stages * RingGeo<TYPE>::kStage;
}

// Ring-kernel launch: one CTA per SM (fewer for small matrices).
template <int TYPE, int RW, int S>
int launch_ring(const GemvParams& p, cudaStream_t s) {
    const size_t smem = ring_smem<TYPE>(p, RW, S);
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(gemv_ring_kernel<TYPE, RW, S, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRingSmemMax) != cudaSuccess ||
            cudaFuncSetAttribute(gemv_ring_kernel<TYPE, RW, S, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRingSmemMax) != cudaSuccess)
            return Q3XK_ECUDA;
        configured = true;
    }
    const int64_t groups = (p.rows + kRows - 1) / kRows;
    const int64_t sms = sm_count_cached();
    const int64_t grid = groups < sms ? groups : sms;
    const cudaError_t e =
        p.units % (32 * kUPL) == 0
            ? launch_pdl(gemv_ring_kernel<TYPE, RW, S, true>, dim3((unsigned)grid), dim3(RW * 32), smem, s, p)
            : launch_pdl(gemv_ring_kernel<TYPE, RW, S, false>, dim3((unsigned)grid), dim3(RW * 32), smem, s, p);
    return e == cudaSuccess ? Q3XK_OK : Q3XK_ECUDA;
}

// The deepest ring (stages per warp, up to SMAX) whose shared memory fits in
// `cap` next to x; Q3XK_EUNSUPPORTED when even two stages do not fit.
template <int TYPE, int RW, int SMAX>
int launch_ring_depth(const GemvParams& p, cudaStream_t s) {
    if (SMAX >= 4 && ring_smem<TYPE>(p, RW, 4) <= kRingSmemMax) return launch_ring<TYPE, RW, 4>(p, s);
    if (SMAX >= 3 && ring_smem<TYPE>(p, RW, 3) <= kRingSmemMax) return launch_ring<TYPE, RW, 3>(p, s);
    if (ring_smem<TYPE>(p, RW, 2) <= kRingSmemMax) return launch_ring<TYPE, RW, 2>(p, s);
    return Q3XK_EUNSUPPORTED;
}

template <int TYPE>
int launch_ring_family(const GemvParams& p, cudaStream_t s) {
    switch (g_gemv_family) {
    case 3: {
        const int st = launch_ring_depth<TYPE, 24, 2>(p, s);
        if (st != Q3XK_EUNSUPPORTED) return st;
        return launch_ring_depth<TYPE, 20, 2>(p, s);
    }
    case 2: return launch_ring_depth<TYPE, 16, 3>(p, s);
    default: {
        // Measured on B200 (us): Q8_0 12288x4096 10.1 with 24 warps vs 10.9
        // with 16 (one 4-row group per warp), 248320x4096 169 vs 165; Q4_0
        // 12288x4096 10.3 vs 9.5, 248320x2048 60.4 vs 54.3.
        const int64_t groups = (p.rows + kRows - 1) / kRows;
        if (TYPE == Q3XK_Q8_0 && groups <= 24 * (int64_t)sm_count_cached()) {
            const int st = launch_ring_depth<TYPE, 24, 2>(p, s);
            if (st != Q3XK_EUNSUPPORTED) return st;
        }
        return launch_ring_depth<TYPE, 16, 3>(p, s);
    }
    }
}

template <int TYPE, int MODE>
int launch(GemvParams p, cudaStream_t s) {
    if (MODE == kPlain && (!p.xform || p.xform == Q3XK_XFORM_RMS) && g_gemv_family != 1) {
        const int st = launch_ring_family<TYPE>(p, s);
        if (st != Q3XK_EUNSUPPORTED) return st;
    }
    if (p.xout) return Q3XK_EUNSUPPORTED;  // the normalised-x output is the ring kernel's
    const size_t smem = smem_bytes<TYPE>(p);
    if (smem > 200 * 1024) return Q3XK_EUNSUPPORTED;
    if (p.xform) return launch_xf<TYPE, MODE, true, false>(p, smem, s);
    if (MODE != kRowGather && p.ksplit > 1) {
        p.ksplit = choose_ksplit(p.rows, p.units, sm_count_cached() * kDbBlocks);
        return launch_xf<TYPE, MODE, false, true>(p, smem, s);
    }
    return launch_xf<TYPE, MODE, false, false>(p, smem, s);
}

template <int MODE>
int launch_type(int type, const GemvParams& p, cudaStream_t s) {
    switch (type) {
    case Q3XK_Q8_0: return launch<Q3XK_Q8_0, MODE>(p, s);
    case Q3XK_Q4_0: return launch<Q3XK_Q4_0, MODE>(p, s);
    default: return launch<Q3XK_BF16, MODE>(p, s);
    }
}

int unit_cols(int type) { return type == Q3XK_Q4_0 ? 32 : type == Q3XK_Q8_0 ? 16 : 8; }

int check_matrix(const q3xk_matrix* m) {
    if (!m || !m->data || m->rows <= 0 || m->cols <= 0) return Q3XK_EINVAL;
    if (m->row_stride != row_record_bytes(m->type, m->cols)) return Q3XK_EINVAL;
    if (m->type != Q3XK_BF16 && m->type != Q3XK_Q8_0 && m->type != Q3XK_Q4_0) return Q3XK_EINVAL;
    if (m->type != Q3XK_BF16 && m->cols % kBlock) return Q3XK_EINVAL;
    if (m->type == Q3XK_BF16 && m->cols % 8) return Q3XK_EUNSUPPORTED;
    return Q3XK_OK;
}

GemvParams base_params(const q3xk_matrix* m, const uint8_t* base, const float* x, float* y, int accumulate) {
    GemvParams p{};
    p.w = base;
    p.x = x;
    p.y = y;
    p.row_stride = m->row_stride;
    p.qbytes = quant_bytes(m->type, m->cols);
    p.rows = m->rows;
    p.cols = m->cols;
    p.accumulate = accumulate ? 1 : 0;
    p.units = m->cols / unit_cols(m->type);
    p.expert_stride = m->expert_stride;
    return p;
}

// Validates `xf` for a matrix of `cols` inputs (per segment) and fills p.
int set_xform(GemvParams& p, const q3xk_xform* xf, int cols, int mode) {
    if (!xf || xf->kind == Q3XK_XFORM_NONE) return Q3XK_OK;
    switch (xf->kind) {
    case Q3XK_XFORM_RMS:
        if (!xf->w || mode == kSegGather) return Q3XK_EINVAL;
        break;
    case Q3XK_XFORM_GATED_RMS:
        if (!xf->w || !xf->z || xf->group <= 0 || xf->group % 32 || cols % xf->group) return Q3XK_EINVAL;
        if (cols / xf->group > kMaxXGroups || mode != kPlain) return Q3XK_EUNSUPPORTED;
        break;
    case Q3XK_XFORM_SWIGLU:
        if (xf->group != cols) return Q3XK_EINVAL;
        if (mode == kRowGather) return Q3XK_EUNSUPPORTED;
        break;
    default:
        return Q3XK_EINVAL;
    }
    if (((uintptr_t)xf->w & 15) || ((uintptr_t)xf->z & 15)) return Q3XK_EALIGN;
    p.xform = xf->kind;
    p.xgroup = xf->group;
    p.xw = xf->w;
    p.xz = xf->z;
    p.xsw = xf->seg_weights;
    return Q3XK_OK;
}

int gemv_impl(const q3xk_matrix* m, const uint8_t* base, const float* x, float* y,
              int accumulate, cudaStream_t s, const q3xk_xform* xf = nullptr) {
    int st = check_matrix(m);
    if (st != Q3XK_OK || !base || !x || !y) return Q3XK_EINVAL;
    if (((uintptr_t)base & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 3)) return Q3XK_EALIGN;
    GemvParams p = base_params(m, base, x, y, accumulate);
    st = set_xform(p, xf, m->cols, kPlain);
    if (st != Q3XK_OK) return st;
    p.ksplit = choose_ksplit(p.rows, p.units, sm_count_cached() * Q3XK_GEMV_MIN_BLOCKS);
    st = launch_type<kPlain>(m->type, p, s);
    if (st != Q3XK_OK) return st;
    count_launch();
    return last_launch_status();
}

}  // namespace

int gemv_rms_out(const q3xk_matrix* m, const float* x, const float* w1, float* y, float* xout, cudaStream_t s) {
    int st = check_matrix(m);
    if (st != Q3XK_OK || !x || !w1 || !y || !xout) return Q3XK_EINVAL;
    if (((uintptr_t)m->data & 15) || ((uintptr_t)x & 15) || ((uintptr_t)w1 & 15) || ((uintptr_t)xout & 15) ||
        ((uintptr_t)y & 3))
        return Q3XK_EALIGN;
    GemvParams p = base_params(m, static_cast<const uint8_t*>(m->data), x, y, 0);
    q3xk_xform xf{};
    xf.kind = Q3XK_XFORM_RMS;
    xf.w = w1;
    st = set_xform(p, &xf, m->cols, kPlain);
    if (st != Q3XK_OK) return st;
    p.xout = xout;
    p.ksplit = 1;
    st = launch_type<kPlain>(m->type, p, s);
    if (st != Q3XK_OK) return st;
    count_launch();
    return last_launch_status();
}

int gemv_swiglu(const q3xk_matrix* m, const float* x, float* y, const int* ids, int slots, const float* slot_w,
                const q3xk_xform* xf, cudaStream_t s) {
    int st = check_matrix(m);
    if (st != Q3XK_OK || !x || !y || m->rows % 4) return Q3XK_EINVAL;
    if (((uintptr_t)m->data & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 3)) return Q3XK_EALIGN;
    GemvParams p = base_params(m, static_cast<const uint8_t*>(m->data), x, y, 0);
    st = set_xform(p, xf, m->cols, ids ? kRowGather : kPlain);
    if (st != Q3XK_OK) return st;
    p.epi = 1;
    p.rows_per_expert = m->rows;
    if (ids) {
        if (slots <= 0 || m->expert_stride != m->row_stride * m->rows) return Q3XK_EINVAL;
        p.ids = ids;
        p.rows = m->rows * slots;
        p.ew = slot_w;
    }
    p.ksplit = choose_ksplit(p.rows, p.units, sm_count_cached() * Q3XK_GEMV_MIN_BLOCKS);
    st = ids ? launch_type<kRowGather>(m->type, p, s) : launch_type<kPlain>(m->type, p, s);
    if (st != Q3XK_OK) return st;
    count_launch();
    return last_launch_status();
}

}  // namespace q3xk

using namespace q3xk;

extern "C" {

int q3xk_gemv(const q3xk_matrix* w, const float* x, float* y, int accumulate, void* stream) {
    if (!w) return Q3XK_EINVAL;
    return gemv_impl(w, static_cast<const uint8_t*>(w->data), x, y, accumulate,
                     static_cast<cudaStream_t>(stream));
}

int q3xk_expert_gemv(const q3xk_matrix* w, int expert, const float* x, float* y,
                     int accumulate, void* stream) {
    if (!w || expert < 0 || expert >= w->experts) return Q3XK_EINVAL;
    if (w->expert_stride != w->row_stride * w->rows) return Q3XK_EINVAL;
    const uint8_t* base = static_cast<const uint8_t*>(w->data) + (int64_t)expert * w->expert_stride;
    return gemv_impl(w, base, x, y, accumulate, static_cast<cudaStream_t>(stream));
}

int q3xk_gemv_ex(const q3xk_matrix* w, const float* x, float* y, int accumulate, const q3xk_xform* xf,
                 void* stream) {
    if (!w) return Q3XK_EINVAL;
    return gemv_impl(w, static_cast<const uint8_t*>(w->data), x, y, accumulate,
                     static_cast<cudaStream_t>(stream), xf);
}

int q3xk_expert_gemv_rows(const q3xk_matrix* pool, const int* ids, int slots, const float* x, float* y,
                          int accumulate, void* stream) {
    return q3xk_expert_gemv_rows_ex(pool, ids, slots, x, y, accumulate, nullptr, stream);
}

int q3xk_expert_gemv_rows_ex(const q3xk_matrix* pool, const int* ids, int slots, const float* x, float* y,
                             int accumulate, const q3xk_xform* xf, void* stream) {
    int st = check_matrix(pool);
    if (st != Q3XK_OK || !ids || !x || !y || slots <= 0) return Q3XK_EINVAL;
    if (pool->expert_stride != pool->row_stride * pool->rows) return Q3XK_EINVAL;
    if (((uintptr_t)pool->data & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 3)) return Q3XK_EALIGN;
    GemvParams p = base_params(pool, static_cast<const uint8_t*>(pool->data), x, y, accumulate);
    st = set_xform(p, xf, pool->cols, kRowGather);
    if (st != Q3XK_OK) return st;
    p.ids = ids;
    p.rows_per_expert = pool->rows;
    p.rows = pool->rows * slots;
    p.ksplit = choose_ksplit(p.rows, p.units, sm_count_cached() * Q3XK_GEMV_MIN_BLOCKS);
    st = launch_type<kRowGather>(pool->type, p, static_cast<cudaStream_t>(stream));
    if (st != Q3XK_OK) return st;
    count_launch();
    return last_launch_status();
}

int q3xk_expert_gemv_segments(const q3xk_matrix* pool, const int* ids, int slots, const float* x, float* y,
                              int accumulate, void* stream) {
    return q3xk_expert_gemv_segments_ex(pool, ids, slots, x, y, accumulate, nullptr, stream);
}

int q3xk_expert_gemv_segments_ex(const q3xk_matrix* pool, const int* ids, int slots, const float* x, float* y,
                                 int accumulate, const q3xk_xform* xf, void* stream) {
    int st = check_matrix(pool);
    if (st != Q3XK_OK || !ids || !x || !y || slots <= 0) return Q3XK_EINVAL;
    if (slots > kMaxSegments) return Q3XK_EUNSUPPORTED;
    if (pool->expert_stride != pool->row_stride * pool->rows) return Q3XK_EINVAL;
    if (((uintptr_t)pool->data & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 3)) return Q3XK_EALIGN;
    GemvParams p = base_params(pool, static_cast<const uint8_t*>(pool->data), x, y, accumulate);
    st = set_xform(p, xf, pool->cols, kSegGather);
    if (st != Q3XK_OK) return st;
    p.ids = ids;
    p.units_per_seg = p.units;
    p.units = p.units * slots;
    p.cols = pool->cols * slots;
    p.ksplit = choose_ksplit(p.rows, p.units, sm_count_cached() * Q3XK_GEMV_MIN_BLOCKS);
    st = launch_type<kSegGather>(pool->type, p, static_cast<cudaStream_t>(stream));
    if (st != Q3XK_OK) return st;
    count_launch();
    return last_launch_status();
}

int q3xk_try_mv_host(const q3xk_matrix* w, const float* x_host, float* y_host, void* workspace,
                     size_t workspace_bytes, void* stream) {
    if (!w || !x_host || !y_host || !workspace || w->rows <= 0 || w->cols <= 0)
        return Q3XK_EINVAL;
    const size_t x_bytes = (size_t)w->cols * 4, y_off = (x_bytes + 15) & ~(size_t)15;
    const size_t need = y_off + (size_t)w->rows * 4;
    if (workspace_bytes < need) return Q3XK_EWORKSPACE;
    if ((uintptr_t)workspace & 15) return Q3XK_EALIGN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* xd = static_cast<float*>(workspace);
    float* yd = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + y_off);
    if (cudaMemcpyAsync(xd, x_host, x_bytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return Q3XK_ECUDA;
    const int st = gemv_impl(w, static_cast<const uint8_t*>(w->data), xd, yd, 0, s);
    if (st != Q3XK_OK) return st;
    if (cudaMemcpyAsync(y_host, yd, (size_t)w->rows * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return Q3XK_ECUDA;
    return cuda_status(cudaStreamSynchronize(s));
}

}  // extern "C"

// ---- q3xk_try_mv_host_noalloc: q3xk_try_mv_host with a fixed scratch ---------------
//
// The staging copies of x and y live in this module's own device array instead
// of a caller workspace.  Its device address is looked up with
// cudaGetSymbolAddress on the first call made with a device current and kept
// in g_static_scratch together with the CUDA context it belongs to; a call
// made under another context of that device (after cudaDeviceReset, or a
// driver-API context) looks it up again.  Nothing is allocated at any time.
namespace q3xk {
namespace {

constexpr size_t kStaticScratchFloats = (size_t)1 << 20;  // 4 MiB: x (cols) + y (rows) floats
constexpr int kMaxScratchDevices = 64;

static __device__ __align__(256) float g_mv_scratch[kStaticScratchFloats];

struct ScratchEntry {
    CUcontext ctx;
    float* ptr;
};

std::mutex g_scratch_mutex;
ScratchEntry g_static_scratch[kMaxScratchDevices] = {};

// The driver's cuCtxGetCurrent, through the runtime (the library does not
// link libcuda, so it also loads on machines without a GPU driver).
using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent ctx_get_current() {
    static CtxGetCurrent fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrent>(p);
    }
    return fn;
}

// Address of g_mv_scratch in the current device's current context.
int static_scratch(float** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q3XK_ECUDA;
    if (dev < 0 || dev >= kMaxScratchDevices) return Q3XK_EUNSUPPORTED;
    CUcontext ctx = nullptr;
    const CtxGetCurrent get = ctx_get_current();
    if (!get || cudaFree(nullptr) != cudaSuccess || get(&ctx) != CUDA_SUCCESS || !ctx) return Q3XK_ECUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchEntry& e = g_static_scratch[dev];
    if (!e.ptr || e.ctx != ctx) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_mv_scratch) != cudaSuccess || !p) return Q3XK_ECUDA;
        e.ptr = static_cast<float*>(p);
        e.ctx = ctx;
    }
    *out = e.ptr;
    return Q3XK_OK;
}

}  // namespace
}  // namespace q3xk

extern "C" {

int q3xk_try_mv_host_noalloc(const q3xk_matrix* w, const float* x_host, float* y_host, void* stream) {
    if (!w || !x_host || !y_host || w->rows <= 0 || w->cols <= 0) return Q3XK_EINVAL;
    const size_t y_off = ((size_t)w->cols + 3) & ~(size_t)3;  // y starts 16-byte aligned
    if (y_off + (size_t)w->rows > kStaticScratchFloats) return Q3XK_EWORKSPACE;
    float* scratch = nullptr;
    const int st0 = static_scratch(&scratch);
    if (st0 != Q3XK_OK) return st0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* xd = scratch;
    float* yd = scratch + y_off;
    if (cudaMemcpyAsync(xd, x_host, (size_t)w->cols * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return Q3XK_ECUDA;
    const int st = gemv_impl(w, static_cast<const uint8_t*>(w->data), xd, yd, 0, s);
    if (st != Q3XK_OK) return st;
    if (cudaMemcpyAsync(y_host, yd, (size_t)w->rows * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return Q3XK_ECUDA;
    return cuda_status(cudaStreamSynchronize(s));
}

// The GEMVs have no device-side waits: the word is the dequant-GEMM's.
int q3xk_device_error(int* flags) {
    if (!flags) return Q3XK_EINVAL;
    if (cudaDeviceSynchronize() != cudaSuccess) return Q3XK_ECUDA;
    return q3xk_gemm_device_error(flags);
}

int q3xk_clear_device_error(void) { return gemm_clear_error(); }

int q3xk_gemv_set_family(int family) {
    if (family < 0 || family > 3) return Q3XK_EINVAL;
    g_gemv_family = family;
    return Q3XK_OK;
}

}  // extern "C"
