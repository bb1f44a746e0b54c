// layout.cu -- sizes, the row-record device layout and the upload repack.
//
// model.bin stores each matrix as packed blocks (q8.h:10-15, q4.h:29-42)
// that the reference binds in place (engine.cu:2007-2026) and reads with
// 1-byte loads.  Here the blocks are split once, on the device, into
// 16-byte-aligned row records so every kernel can use 128-bit loads and TMA.
#include <atomic>
#include <limits>

#include "common.cuh"

namespace q3xk {

static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

namespace {

// Destination row of source row r.  half == 0: r.  half == I > 0: the rows
// of [gate (I) | up (I)] matrices (one per 2I source rows, r counted from
// row_offset) are interleaved in fours, g(2j) g(2j+1) u(2j) u(2j+1), so that a
// GEMV warp's 4-row group holds both operands of two SwiGLU outputs.
__device__ __forceinline__ int64_t dest_row(int64_t r, int64_t half, int64_t row_offset) {
    if (half == 0) return r;
    r += row_offset;
    const int64_t e = r / (2 * half), i = r - e * 2 * half;
    const int64_t up = i >= half, k = up ? i - half : i;
    return e * 2 * half + (k >> 1) * 4 + 2 * up + (k & 1);
}

// One thread per packed block.  Q8_0 quants are stored as q XOR 0x80 (offset
// binary) so the kernels can turn a byte into an exact float with one PRMT.
__global__ void repack_q8_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ out,
                                 int64_t total_rows, int blocks_per_row, int64_t row_stride,
                                 int64_t quant_bytes, int pad_slots, int64_t half = 0, int64_t row_offset = 0) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total_rows * blocks_per_row) return;
    const int64_t row = t / blocks_per_row;
    const int blk = (int)(t - row * blocks_per_row);
    const uint16_t* src = reinterpret_cast<const uint16_t*>(packed + t * kQ8PackedBytes);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        q[i] = ((uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16)) ^ 0x80808080u;
    uint8_t* rec = out + dest_row(row, half, row_offset) * row_stride;
    uint4* dst = reinterpret_cast<uint4*>(rec + (int64_t)blk * kBlock);
    dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
    dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
    uint16_t* scales = reinterpret_cast<uint16_t*>(rec + quant_bytes);
    scales[blk] = src[0];
    if (blk == blocks_per_row - 1)
        for (int i = blocks_per_row; i < pad_slots; ++i) scales[i] = 0;
}

__global__ void repack_q4_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ out,
                                 int64_t total_rows, int blocks_per_row, int64_t row_stride,
                                 int64_t quant_bytes, int pad_slots, int64_t half = 0, int64_t row_offset = 0) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total_rows * blocks_per_row) return;
    const int64_t row = t / blocks_per_row;
    const int blk = (int)(t - row * blocks_per_row);
    const uint16_t* src = reinterpret_cast<const uint16_t*>(packed + t * kQ4PackedBytes);
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
    uint8_t* rec = out + dest_row(row, half, row_offset) * row_stride;
    *reinterpret_cast<uint4*>(rec + (int64_t)blk * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    uint16_t* scales = reinterpret_cast<uint16_t*>(rec + quant_bytes);
    scales[blk] = src[0];
    if (blk == blocks_per_row - 1)
        for (int i = blocks_per_row; i < pad_slots; ++i) scales[i] = 0;
}

// BF16 rows: copy, zero the tail padding.  One thread per 2-byte slot.
__global__ void repack_bf16_kernel(const uint16_t* __restrict__ packed, uint8_t* __restrict__ out,
                                   int64_t total_rows, int cols, int64_t row_stride, int64_t half = 0,
                                   int64_t row_offset = 0) {
    const int slots = (int)(row_stride / 2);
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total_rows * slots) return;
    const int64_t row = t / slots;
    const int c = (int)(t - row * slots);
    uint16_t* rec = reinterpret_cast<uint16_t*>(out + dest_row(row, half, row_offset) * row_stride);
    rec[c] = c < cols ? packed[row * cols + c] : (uint16_t)0;
}

}  // namespace

int repack_swiglu(const q3xk_matrix* m, const void* packed, int64_t src_rows, int half, int row_offset,
                  cudaStream_t s) {
    if (!m || !m->data || !packed || src_rows <= 0 || half <= 0 || (half & 1)) return Q3XK_EINVAL;
    if (m->row_stride != row_record_bytes(m->type, m->cols)) return Q3XK_EINVAL;
    const int threads = 256;
    if (m->type == Q3XK_BF16) {
        const int64_t n = src_rows * (m->row_stride / 2);
        repack_bf16_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, s>>>(
            static_cast<const uint16_t*>(packed), static_cast<uint8_t*>(m->data), src_rows, m->cols, m->row_stride,
            half, row_offset);
    } else {
        const int bpr = m->cols / kBlock;
        const int64_t n = src_rows * bpr;
        const unsigned grid = (unsigned)((n + threads - 1) / threads);
        if (m->type == Q3XK_Q8_0)
            repack_q8_kernel<<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(packed),
                                                      static_cast<uint8_t*>(m->data), src_rows, bpr, m->row_stride,
                                                      quant_bytes(m->type, m->cols), scale_slots(m->cols), half,
                                                      row_offset);
        else
            repack_q4_kernel<<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(packed),
                                                      static_cast<uint8_t*>(m->data), src_rows, bpr, m->row_stride,
                                                      quant_bytes(m->type, m->cols), scale_slots(m->cols), half,
                                                      row_offset);
    }
    count_launch();
    return last_launch_status();
}

}  // namespace q3xk

using namespace q3xk;

extern "C" {

const char* q3xk_status_string(int status) {
    switch (status) {
    case Q3XK_OK: return "ok";
    case Q3XK_EINVAL: return "invalid argument";
    case Q3XK_EUNSUPPORTED: return "unsupported";
    case Q3XK_ECUDA: return "CUDA error";
    case Q3XK_EALIGN: return "misaligned pointer or stride";
    case Q3XK_ETIMEOUT: return "device wait timed out";
    case Q3XK_EWORKSPACE: return "workspace too small";
    default: return "unknown status";
    }
}

int q3xk_abi_version(void) { return Q3XK_ABI_VERSION; }

uint64_t q3xk_launch_count(void) { return g_launches.load(); }
void q3xk_reset_launch_count(void) { g_launches.store(0); }

// arch/cpu.cpp:161-179, same acceptance rules.
int q3xk_quantized_bytes(int type, int rows, int cols, size_t* bytes) {
    size_t block_bytes;
    if (type == Q3XK_Q8_0) block_bytes = kQ8PackedBytes;
    else if (type == Q3XK_Q4_0) block_bytes = kQ4PackedBytes;
    else return Q3XK_EINVAL;
    if (!bytes || rows <= 0 || cols <= 0 || cols % kBlock != 0) return Q3XK_EINVAL;
    const size_t blocks = (size_t)cols / kBlock;
    const size_t maximum = std::numeric_limits<size_t>::max();
    if (blocks > maximum / block_bytes) return Q3XK_EINVAL;
    const size_t rb = blocks * block_bytes;
    if ((size_t)rows > maximum / rb) return Q3XK_EINVAL;
    *bytes = (size_t)rows * rb;
    return Q3XK_OK;
}

int q3xk_matrix_layout(int type, int rows, int cols, int experts, q3xk_matrix* m,
                       size_t* device_bytes) {
    if (!m || rows <= 0 || cols <= 0 || experts <= 0) return Q3XK_EINVAL;
    if (type != Q3XK_BF16 && type != Q3XK_Q8_0 && type != Q3XK_Q4_0) return Q3XK_EINVAL;
    if (type != Q3XK_BF16 && cols % kBlock) return Q3XK_EINVAL;
    const int64_t stride = row_record_bytes(type, cols);
    const int64_t per_expert = stride * rows;
    if (per_expert / rows != stride || (per_expert * experts) / experts != per_expert)
        return Q3XK_EINVAL;
    m->row_stride = stride;
    m->expert_stride = per_expert;
    m->type = type;
    m->rows = rows;
    m->cols = cols;
    m->experts = experts;
    if (device_bytes) *device_bytes = (size_t)(per_expert * experts);
    return Q3XK_OK;
}

int q3xk_repack(const q3xk_matrix* m, const void* packed, void* stream) {
    if (!m || !m->data || !packed || m->rows <= 0 || m->cols <= 0 || m->experts <= 0)
        return Q3XK_EINVAL;
    if (m->row_stride != row_record_bytes(m->type, m->cols) ||
        m->expert_stride != m->row_stride * m->rows)
        return Q3XK_EINVAL;
    if (((uintptr_t)m->data & 15) || ((uintptr_t)packed & 1)) return Q3XK_EALIGN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t total_rows = (int64_t)m->rows * m->experts;
    const int threads = 256;
    if (m->type == Q3XK_BF16) {
        const int64_t n = total_rows * (m->row_stride / 2);
        repack_bf16_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, s>>>(
            static_cast<const uint16_t*>(packed), static_cast<uint8_t*>(m->data), total_rows,
            m->cols, m->row_stride);
    } else {
        if (m->cols % kBlock) return Q3XK_EINVAL;
        const int bpr = m->cols / kBlock;
        const int64_t n = total_rows * bpr;
        const unsigned grid = (unsigned)((n + threads - 1) / threads);
        if (m->type == Q3XK_Q8_0)
            repack_q8_kernel<<<grid, threads, 0, s>>>(
                static_cast<const uint8_t*>(packed), static_cast<uint8_t*>(m->data), total_rows,
                bpr, m->row_stride, quant_bytes(m->type, m->cols), scale_slots(m->cols));
        else if (m->type == Q3XK_Q4_0)
            repack_q4_kernel<<<grid, threads, 0, s>>>(
                static_cast<const uint8_t*>(packed), static_cast<uint8_t*>(m->data), total_rows,
                bpr, m->row_stride, quant_bytes(m->type, m->cols), scale_slots(m->cols));
        else
            return Q3XK_EINVAL;
    }
    count_launch();
    return last_launch_status();
}

}  // extern "C"
