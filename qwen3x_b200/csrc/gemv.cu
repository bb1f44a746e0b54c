// gemv.cu -- decode GEMV y = W x (and y += W x) on CUDA cores, sm_100a.
//
// Replaces the reference's one-CTA-per-row kernels with 1-byte loads and a
// per-element FP16 decode (engine.cu:546-612).  Decode GEMV is HBM-bound
// (≈1.9 flop/B for Q8_0), so the design goal is bytes in flight, not FLOPs:
//   * each warp owns R consecutive rows and walks K in 16-byte lane units
//     (Q8_0: 16 weights, Q4_0: 32 weights = one block, BF16: 8 weights);
//   * UB units per lane and row are loaded (128-bit, L1::no_allocate) before
//     any is consumed, so a CTA keeps 8 warps x 32 lanes x UB x R x 16 B of
//     weights in flight;
//   * the R rows share each x load, which keeps L1 traffic for x at 4/R bytes
//     per weight;
//   * dequant is exact and branch-free: PRMT turns a byte (or a nibble after
//     one LOP3) into the float 2^23 + value, one packed f32x2 add removes the
//     offset, one packed f32x2 FMA accumulates (Blackwell FFMA2);
//   * a block's FP16 scale multiplies the block's inner sum, as in
//     arch/cpu.cpp:64-73, and the lanes' partial sums meet in a warp shuffle.
#include "common.cuh"

namespace q3xk {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// Inner sum of one Q8_0 half block (16 weights = one 16-byte unit).
__device__ __forceinline__ float q8_unit_dot(const uint4 q, const float4 xa, const float4 xb,
                                             const float4 xc, const float4 xd) {
    const float2 off = f2(-8388736.0f, -8388736.0f);  // 2^23 + 128 (offset binary)
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#define Q8_WORD(W, X)                                                                     \
    {                                                                                     \
        const float2 v01 = __fadd2_rn(f2(byte_as_magic_float<0>(W), byte_as_magic_float<1>(W)), off); \
        const float2 v23 = __fadd2_rn(f2(byte_as_magic_float<2>(W), byte_as_magic_float<3>(W)), off); \
        a0 = __ffma2_rn(v01, f2(X.x, X.y), a0);                                           \
        a1 = __ffma2_rn(v23, f2(X.z, X.w), a1);                                           \
    }
    Q8_WORD(q.x, xa)
    Q8_WORD(q.y, xb)
    Q8_WORD(q.z, xc)
    Q8_WORD(q.w, xd)
#undef Q8_WORD
    return (a0.x + a0.y) + (a1.x + a1.y);
}

// Inner sum of one Q4_0 block (32 weights = one 16-byte unit).  Byte i holds
// element i (low nibble) and element i + 16 (high nibble), q4.h:31-36.
__device__ __forceinline__ float q4_unit_dot(const uint4 q, const float4* xs) {
    const float2 off = f2(-8388616.0f, -8388616.0f);  // 2^23 + 8
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = words[j] & 0x0F0F0F0Fu;
        const uint32_t hi = (words[j] >> 4) & 0x0F0F0F0Fu;
        const float4 xl = xs[j], xh = xs[4 + j];
        const float2 l01 = __fadd2_rn(f2(byte_as_magic_float<0>(lo), byte_as_magic_float<1>(lo)), off);
        const float2 l23 = __fadd2_rn(f2(byte_as_magic_float<2>(lo), byte_as_magic_float<3>(lo)), off);
        const float2 h01 = __fadd2_rn(f2(byte_as_magic_float<0>(hi), byte_as_magic_float<1>(hi)), off);
        const float2 h23 = __fadd2_rn(f2(byte_as_magic_float<2>(hi), byte_as_magic_float<3>(hi)), off);
        a0 = __ffma2_rn(l01, f2(xl.x, xl.y), a0);
        a1 = __ffma2_rn(l23, f2(xl.z, xl.w), a1);
        a0 = __ffma2_rn(h01, f2(xh.x, xh.y), a0);
        a1 = __ffma2_rn(h23, f2(xh.z, xh.w), a1);
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
}

// BF16 unit: 8 weights; bf16 -> f32 is a 16-bit shift.
__device__ __forceinline__ float bf16_unit_dot(const uint4 q, const float4 xa, const float4 xb) {
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#define BF_WORD(W, X0, X1, ACC) \
    ACC = __ffma2_rn(f2(__uint_as_float((W) << 16), __uint_as_float((W) & 0xFFFF0000u)), f2(X0, X1), ACC);
    BF_WORD(q.x, xa.x, xa.y, a0)
    BF_WORD(q.y, xa.z, xa.w, a1)
    BF_WORD(q.z, xb.x, xb.y, a0)
    BF_WORD(q.w, xb.z, xb.w, a1)
#undef BF_WORD
    return (a0.x + a0.y) + (a1.x + a1.y);
}

template <int TYPE, int R, int UB>
__global__ void __launch_bounds__(kThreads)
gemv_kernel(const uint8_t* __restrict__ w, int64_t row_stride, int rows, int cols,
            const float* __restrict__ x, float* __restrict__ y, int accumulate) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kWarps + warp) * R;
    if (row0 >= rows) return;
    const int64_t qbytes = quant_bytes(TYPE, cols);
    const int units = (int)((TYPE == Q3XK_BF16 ? (int64_t)cols * 2 : qbytes) / 16);
    const uint8_t* rec[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rec[r] = w + (int64_t)min(row0 + r, rows - 1) * row_stride;

    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;

    for (int base = lane; base < units; base += 32 * UB) {
        uint4 q[UB][R];
        float d[UB][R];
#pragma unroll
        for (int i = 0; i < UB; ++i) {
            const int u = base + 32 * i;
            if (u < units) {
#pragma unroll
                for (int r = 0; r < R; ++r) q[i][r] = ld_stream_v4(rec[r] + (int64_t)u * 16);
                if (TYPE != Q3XK_BF16) {
                    const int blk = TYPE == Q3XK_Q8_0 ? (u >> 1) : u;
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        d[i][r] = f16_bits_to_float(ld_nc_u16(rec[r] + qbytes + 2 * blk));
                }
            }
        }
#pragma unroll
        for (int i = 0; i < UB; ++i) {
            const int u = base + 32 * i;
            if (u < units) {
                if (TYPE == Q3XK_Q8_0) {
                    const float4* xp = reinterpret_cast<const float4*>(x) + (int64_t)u * 4;
                    const float4 xa = __ldg(xp), xb = __ldg(xp + 1), xc = __ldg(xp + 2),
                                 xd = __ldg(xp + 3);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        acc[r] = fmaf(d[i][r], q8_unit_dot(q[i][r], xa, xb, xc, xd), acc[r]);
                } else if (TYPE == Q3XK_Q4_0) {
                    const float4* xp = reinterpret_cast<const float4*>(x) + (int64_t)u * 8;
                    float4 xs[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) xs[k] = __ldg(xp + k);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        acc[r] = fmaf(d[i][r], q4_unit_dot(q[i][r], xs), acc[r]);
                } else {
                    const float4* xp = reinterpret_cast<const float4*>(x) + (int64_t)u * 2;
                    const float4 xa = __ldg(xp), xb = __ldg(xp + 1);
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r] += bf16_unit_dot(q[i][r], xa, xb);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
    if (lane < R) {
        float v = acc[0];
#pragma unroll
        for (int r = 1; r < R; ++r)
            if (lane == r) v = acc[r];
        const int row = row0 + lane;
        if (row < rows) y[row] = accumulate ? y[row] + v : v;
    }
}

template <int TYPE, int R>
void launch_rows(const q3xk_matrix* m, const uint8_t* base, const float* x, float* y,
                 int accumulate, cudaStream_t s) {
    const int rows_per_cta = kWarps * R;
    const unsigned grid = (unsigned)((m->rows + rows_per_cta - 1) / rows_per_cta);
    constexpr int UB = TYPE == Q3XK_Q4_0 ? 2 : 2;
    gemv_kernel<TYPE, R, UB><<<grid, kThreads, 0, s>>>(base, m->row_stride, m->rows, m->cols, x,
                                                      y, accumulate);
}

template <int TYPE>
void launch_type(const q3xk_matrix* m, const uint8_t* base, const float* x, float* y,
                 int accumulate, cudaStream_t s, int sm_count) {
    // Enough CTAs to fill every SM at least twice; more rows per warp when the
    // matrix is tall, so each x load serves several rows.
    const int target = 2 * sm_count;
    if ((m->rows + 31) / 32 >= target)
        launch_rows<TYPE, 4>(m, base, x, y, accumulate, s);
    else if ((m->rows + 15) / 16 >= target)
        launch_rows<TYPE, 2>(m, base, x, y, accumulate, s);
    else
        launch_rows<TYPE, 1>(m, base, x, y, accumulate, s);
}

int sm_count_cached() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return 148;
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            count = 148;
    }
    return count;
}

int gemv_impl(const q3xk_matrix* m, const uint8_t* base, const float* x, float* y,
              int accumulate, cudaStream_t s) {
    if (!m || !base || !x || !y || m->rows <= 0 || m->cols <= 0) return Q3XK_EINVAL;
    if (m->row_stride != row_record_bytes(m->type, m->cols)) return Q3XK_EINVAL;
    if (((uintptr_t)base & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 3)) return Q3XK_EALIGN;
    const int sms = sm_count_cached();
    switch (m->type) {
    case Q3XK_Q8_0:
        if (m->cols % kBlock) return Q3XK_EINVAL;
        launch_type<Q3XK_Q8_0>(m, base, x, y, accumulate, s, sms);
        break;
    case Q3XK_Q4_0:
        if (m->cols % kBlock) return Q3XK_EINVAL;
        launch_type<Q3XK_Q4_0>(m, base, x, y, accumulate, s, sms);
        break;
    case Q3XK_BF16:
        if (m->cols % 8) return Q3XK_EUNSUPPORTED;
        launch_type<Q3XK_BF16>(m, base, x, y, accumulate, s, sms);
        break;
    default:
        return Q3XK_EINVAL;
    }
    count_launch();
    return last_launch_status();
}

}  // namespace
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
