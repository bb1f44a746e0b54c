// common.cuh -- shared device helpers for the q3xk kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q3xk.h"

namespace q3xk {

constexpr int kBlock = 32;        // weights per Q8_0/Q4_0 block (q8.h:8, q4.h:8)
constexpr int kQ8PackedBytes = 34;  // q8.h:15
constexpr int kQ4PackedBytes = 18;  // q4.h:27

// Host-side launch accounting (q3xk_launch_count).
void count_launch(int n = 1);

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? Q3XK_OK : Q3XK_ECUDA; }

inline int last_launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? Q3XK_OK : Q3XK_ECUDA;
}

// The reference's sigmoid (engine.cpp:187-191): same branches, CUDA's expf.
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}

// Bytes of the quantised part of one row record.
__host__ __device__ inline int64_t quant_bytes(int type, int cols) {
    return type == Q3XK_Q8_0 ? (int64_t)cols : type == Q3XK_Q4_0 ? (int64_t)cols / 2
                                                                 : (int64_t)cols * 2;
}
// Scale entries per row, padded to a multiple of 8 (16 bytes).
__host__ __device__ inline int scale_slots(int cols) { return ((cols / kBlock) + 7) & ~7; }

__host__ __device__ inline int64_t row_record_bytes(int type, int cols) {
    if (type == Q3XK_BF16) return ((int64_t)cols * 2 + 15) & ~(int64_t)15;
    return quant_bytes(type, cols) + (int64_t)scale_slots(cols) * 2;
}

// ---- device helpers -------------------------------------------------------

// Streaming 128-bit load that bypasses L1 allocation: weights are read once.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float f16_bits_to_float(uint16_t bits) {
    return __half2float(__ushort_as_half(bits));
}

// Byte k (0..3) of w as the float 2^23 + byte (exact): PRMT places the byte
// in the low mantissa bits under the exponent byte 0x4B.
template <int K>
__device__ __forceinline__ float byte_as_magic_float(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | K));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace q3xk

namespace q3xk {

// Programmatic dependent launch (sm_90+).  A kernel launched with the
// programmatic-serialization attribute may start while its predecessor in
// the stream is still running; griddep_wait() blocks until the predecessor
// has completed and its writes are visible.  Everything a kernel reads that
// an earlier kernel may write (activations, outputs it accumulates into)
// must be read after griddep_wait(); immutable weights may be read before.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with the programmatic stream serialization attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace q3xk
