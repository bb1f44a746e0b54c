// gemm.cu -- prefill dequant-GEMM  Y[T, N] (+)= X[T, K] * W[N, K]^T  on tcgen05.
//
// Replaces the reference's CUDA-core batch_mv_q8_kernel (engine.cu:751-839)
// and adds the Q4_0 prefill the reference lacks (engine.cu:1580-1581 asserts).
//
//  * X (FP32) is first converted to FP16 with a per-token power-of-two scale
//    (x * 2^s_t has its largest magnitude in [2^14, 2^15)), so FP16 cannot
//    overflow whatever the activations' range; the epilogue multiplies by
//    2^-s_t exactly.
//  * Two precisions.  FP16: one MMA per K-step on fp16(x) and fp16(d*q).
//    SPLIT (the default of q3xk_gemm): both operands carry a second FP16
//    plane, x = x_hi + x_lo (x_lo = fp16(x - x_hi), ~22 significant bits in
//    all) and d*q = w_hi + w_lo exactly (w_lo = fma(q, d, -w_hi) in FP16:
//    the residual of an 11-bit x 8-bit product always fits), and the MMAs
//    accumulate w_hi x_hi + w_hi x_lo + w_lo x_hi in FP32 (two MMAs per
//    16-wide K-step: w_hi against [x_hi; x_lo] stacked as one 2 BN-token
//    operand, then w_lo against x_hi).  The
//    dropped w_lo x_lo term is ~2^-22 of the product, so the result is
//    FP32-grade (the reference's per-token FP32 matvec, engine.cpp:580-583,
//    rounds at ~2^-24 per add).
//  * One tcgen05.mma tile is 128 weight rows (M, operand A) x 128 tokens (N,
//    operand B) x 16 K, FP16 x FP16 -> FP32 accumulated in tensor memory.
//    Operands are K-major in the 128-byte-swizzled layout: B (X16) arrives by
//    TMA, A is dequantised from the row-record layout by kDqWarps warps straight into
//    that layout (value = fp16(d * q), one rounding of the exact product).
//  * Warp roles: 0 TMA producer, 1 MMA issuer (one thread) and TMEM owner,
//    2..1+kDqWarps dequantisers, then 4 epilogue warps (TMEM -> registers -> Y).
//    A ring of raw-weight stages (TMA), a ring of operand stages and two TMEM
//    accumulators let the loads, the dequant, the MMAs and the epilogue of
//    consecutive tiles overlap.  Persistent CTAs walk the work units; every
//    mbarrier wait is bounded.
//  * Few tokens (T <= 64): token tiles of 16 or 64, a deeper raw ring, and,
//    when the tiles cannot fill the SMs, split-K: a work unit is one K segment
//    of a tile (segments are whole raw stages), its FP32 partial goes to the
//    workspace, and the last unit of a tile to finish (an atomic counter per
//    tile) adds the segments in segment order and writes Y -- deterministic,
//    one launch.
#include <cuda.h>

#include "layers.cuh"
#include "tc.cuh"

namespace q3xk {
namespace {

#ifndef Q3XK_GEMM_DQ_WARPS
#define Q3XK_GEMM_DQ_WARPS 8
#endif
#ifndef Q3XK_GEMM_STAGES
#define Q3XK_GEMM_STAGES 3
#endif
#ifndef Q3XK_GEMM_RAW_STAGES
#define Q3XK_GEMM_RAW_STAGES 2
#endif

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // K per stage: 64 FP16 = one 128-byte swizzle row
constexpr int kAcc = 2;  // TMEM accumulator buffers
constexpr int kDqWarps = Q3XK_GEMM_DQ_WARPS;   // dequantiser warps
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kEpiWarp0 = 2 + kDqWarps;        // first of 4 epilogue warps
constexpr int kThreads = (kEpiWarp0 + 4) * 32;
static_assert(kDqThreads <= 256 && 256 % kDqThreads == 0, "dequant work split");
constexpr int kTileBytesW = BM * BK * 2;   // 16 KB
// Raw weights are staged by TMA RAWK columns (4 MMA K-steps) at a time:
// quants (Q8_0: 256 B per row, Q4_0: 128 B) and the 8 FP16 scales of the
// 256 columns (16 B per row).
constexpr int RAWK = 256;
constexpr int kKPerRaw = RAWK / BK;        // MMA K-steps per raw stage
constexpr int kRawQuantBytes = BM * RAWK;  // sized for Q8_0 (Q4_0 uses half)
constexpr int kRawScaleBytes = BM * 16;
constexpr int kRawBytes = kRawQuantBytes + kRawScaleBytes;
// Split-K bounds: work units (tiles x segments) per call, so the partials
// fit a fixed part of the workspace, and per-tile counters.
constexpr int kMaxSplitUnits = 320;
constexpr int kMaxSplit = 8;
constexpr int kSplitMaxBN = 64;
constexpr int kCounterInts = 1024;
constexpr size_t kPartBytes = (size_t)kMaxSplitUnits * BM * kSplitMaxBN * 4;

__device__ int g_gemm_error;

struct GemmParams {
    const uint8_t* w;  // row records
    int64_t row_stride;
    int64_t qbytes;
    int N, K, T;
    const float* tok_scale;  // [T] 2^-s_t
    float* y;
    int accumulate;
    int tiles_w, tiles_t, ksteps;
    // Split-K (ksplit > 1, plain mode only): unit u = tile u / ksplit, K
    // segment u % ksplit of nraw raw stages; partials [unit][BM][BN] in
    // `part`, arrival counters per tile in `counters` (zero between calls).
    int ksplit, nraw;
    float* part;
    int* counters;
    // Expert-grouped mode (groups > 0): X rows [xoff[e], xoff[e+1]) use expert
    // e of the pool (weight rows e*N ..), their tiles are [tile_off[e],
    // tile_off[e+1]) of the tile space; both arrays live on the device.
    int groups;
    const int* xoff;
    const int* tile_off;
};

// One tile of work: weight rows (TMA row of the pool), output columns, X/Y rows.
struct TileCoord {
    int w_row, n0, x_row, t_valid;
};

template <int BN>
__device__ __forceinline__ TileCoord tile_coord(const GemmParams& p, int tile) {
    if (!p.groups) {
        const int wt = tile / p.tiles_t, tt = tile % p.tiles_t;
        return {wt * BM, wt * BM, tt * BN, min(BN, p.T - tt * BN)};
    }
    int lo = 0, hi = p.groups;  // largest e with tile_off[e] <= tile
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(p.tile_off + mid) <= tile) lo = mid;
        else hi = mid;
    }
    const int x0 = __ldg(p.xoff + lo), count = __ldg(p.xoff + lo + 1) - x0;
    const int tt_e = (count + BN - 1) / BN;
    const int local = tile - __ldg(p.tile_off + lo);
    const int wt = local / tt_e, tt = local % tt_e;
    return {lo * p.N + wt * BM, wt * BM, x0 + tt * BN, min(BN, count - tt * BN)};
}

// Work units: tiles (x K segments under split-K).
template <int BN>
__device__ __forceinline__ int unit_count(const GemmParams& p) {
    return p.groups ? __ldg(p.tile_off + p.groups) : p.tiles_w * p.tiles_t * p.ksplit;
}

// First K-step of segment s (whole raw stages; segment ksplit ends at ksteps).
__device__ __forceinline__ int seg_begin(const GemmParams& p, int s) {
    return s >= p.ksplit ? p.ksteps : min(p.ksteps, (s * p.nraw / p.ksplit) * kKPerRaw);
}

// Per token-tile-width geometry: BN tokens per tile = MMA N (16, 64, 128,
// 256).  SPLIT stages hold two planes of each operand (hi, lo), so they get
// fewer stages and at most 128 tokens.
// Three rings per shape, within the 227 KB of shared memory: dequantised
// weights (kStages x planes x 16 KB), X tiles (kXStages x planes x BN x 128 B,
// loaded by their own producer thread, so an X tile's TMA round trip is not
// in the weight ring's recycle loop) and raw weights (kRaw x 34 KB):
//            FP16                          SPLIT
//   BN 256   A 3, X 3, raw 2  (212 KB)     -
//   BN 128   A 3, X 3, raw 3  (198 KB)     A 2, X 2, raw 2  (196 KB)
//   BN  64   A 3, X 4, raw 4  (216 KB)     A 2, X 3, raw 3  (214 KB)
//   BN  16   A 3, X 8, raw 4  (200 KB)     A 2, X 8, raw 3  (198 KB)
// Narrow token tiles are weight-streaming bound: they get the deeper raw and
// X rings.
template <int BN, bool SPLIT>
struct TileN {
    static_assert(!SPLIT || BN <= 128, "split stages hold at most 128 tokens");
    static constexpr int kTileBytesX = BN * BK * 2;  // one plane
    static constexpr int kPlanes = SPLIT ? 2 : 1;
    static constexpr int kStageX = kPlanes * kTileBytesX;
    static constexpr int kStageW = kPlanes * kTileBytesW;
    static constexpr int kStages = SPLIT ? 2 : Q3XK_GEMM_STAGES;
    static constexpr int kXStages = BN == 16 ? 8 : BN == 64 ? (SPLIT ? 3 : 4) : SPLIT ? 2 : Q3XK_GEMM_STAGES;
    static constexpr int kRaw = BN == 256 ? Q3XK_GEMM_RAW_STAGES
                                : BN == 128 ? (SPLIT ? 2 : 3)
                                : SPLIT ? 3 : 4;
    // SPLIT: an accumulator is 2 BN columns wide, [w_hi x_hi + w_lo x_hi | w_hi x_lo]:
    // the hi and lo X planes sit back to back in shared memory, so one MMA
    // with N = 2 BN reads w_hi once for both, and a second (N = BN) adds
    // w_lo x_hi into the first half; the epilogue adds the two halves.
    static constexpr int kAccCols = kPlanes * BN;
    static constexpr uint32_t kTmemCols = kAcc * kAccCols < 32 ? 32 : kAcc * kAccCols;  // power of 2 >= 32
    static constexpr uint32_t kIdesc = f16_idesc(BM, BN, 0);
    static constexpr uint32_t kIdescWide = f16_idesc(BM, kAccCols, 0);
    static constexpr size_t kSmem = 1024 /* alignment slack */ + (size_t)kXStages * kStageX +
                                    (size_t)kStages * kStageW + (size_t)kRaw * kRawBytes +
                                    (size_t)(2 * kStages + 2 * kXStages + 2 * kAcc + 2 * kRaw) * 8 + 16;
    static_assert(kSmem <= 232448, "shared memory per CTA");
    static_assert(BN % 16 == 0 && BN >= 16 && kAccCols <= 256, "MMA N for M = 128");
    static_assert(kTmemCols <= 512, "tensor memory columns");
};

// ---- X -> FP16 with a per-token power-of-two scale -----------------------------

// x16lo != nullptr: also the residual plane, x16lo = fp16(x * 2^s - x16) (the
// subtraction is exact in FP32).
// counters != nullptr: block 0 also zeroes the split-K arrival counters that
// the following GEMM uses (they are left at zero by every GEMM, but the
// caller's workspace starts out undefined).
// One token per CTA of kXThreads threads; the token's values stay in
// registers between the exponent pass and the conversion (K <= kXThreads * 4 *
// kXVecs = 20480; longer rows are read again for the conversion).
constexpr int kXThreads = 1024, kXVecs = 5;
__global__ void __launch_bounds__(kXThreads) x_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ x16,
                                                             __half* __restrict__ x16lo, float* __restrict__ tok_scale,
                                                             int K, int* __restrict__ counters) {
    griddep_wait();
    griddep_launch_dependents();
    const int t = blockIdx.x;
    if (counters && t == 0)
        for (int i = threadIdx.x; i < kCounterInts; i += blockDim.x) counters[i] = 0;
    const float* row = x + (int64_t)t * K;
    const bool held = K <= kXThreads * 4 * kXVecs;
    float4 v[kXVecs];
    uint32_t emax = 0;
    auto upd = [&](const float4& a) {
        emax = max(emax, max(max((__float_as_uint(a.x) >> 23) & 0xFFu, (__float_as_uint(a.y) >> 23) & 0xFFu),
                             max((__float_as_uint(a.z) >> 23) & 0xFFu, (__float_as_uint(a.w) >> 23) & 0xFFu)));
    };
    if (held) {
#pragma unroll
        for (int i = 0; i < kXVecs; ++i) {
            const int k = (threadIdx.x + i * kXThreads) * 4;
            v[i] = k < K ? *reinterpret_cast<const float4*>(row + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            upd(v[i]);
        }
    } else {
        for (int k = threadIdx.x * 4; k < K; k += kXThreads * 4) upd(*reinterpret_cast<const float4*>(row + k));
    }
    __shared__ uint32_t red[kXThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = emax;
    __syncthreads();
    emax = 0;
    for (int i = 0; i < kXThreads / 32; ++i) emax = max(emax, red[i]);
    // Largest |x| < 2^(E+1): scale by 2^(14-E) so it lands in [2^14, 2^15).
    const int E = emax == 0xFFu ? 0 : (int)emax - 127;  // inf/nan stay inf/nan
    const int s = min(100, max(-100, 14 - E));
    const float up = __uint_as_float((uint32_t)(s + 127) << 23);
    if (threadIdx.x == 0) tok_scale[t] = __uint_as_float((uint32_t)(127 - s) << 23);
    __half2* out = reinterpret_cast<__half2*>(x16 + (int64_t)t * K);
    __half2* lo = x16lo ? reinterpret_cast<__half2*>(x16lo + (int64_t)t * K) : nullptr;
    auto put = [&](int k, const float4& a) {
        const float a0 = a.x * up, a1 = a.y * up, a2 = a.z * up, a3 = a.w * up;
        const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
        out[k / 2] = h01;
        out[k / 2 + 1] = h23;
        if (lo) {
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            lo[k / 2] = __floats2half2_rn(a0 - f01.x, a1 - f01.y);
            lo[k / 2 + 1] = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
        }
    };
    if (held) {
#pragma unroll
        for (int i = 0; i < kXVecs; ++i) {
            const int k = (threadIdx.x + i * kXThreads) * 4;
            if (k < K) put(k, v[i]);
        }
    } else {
        for (int k = threadIdx.x * 4; k < K; k += kXThreads * 4) put(k, *reinterpret_cast<const float4*>(row + k));
    }
}

// ---- dequantisation into the SW128 K-major layout ------------------------------

// Byte offset of 16-byte chunk c (8 FP16 along K) of row m in a 128-byte-row
// SWIZZLE_128B tile: chunks are XOR-swizzled with the row index mod 8.
__device__ __forceinline__ uint32_t sw128_off(int m, int c) {
    return (uint32_t)(m * 128 + ((c ^ (m & 7)) << 4));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two exact FP16 weights q (as half2) times the scale: hi = fp16(d*q); with a
// residual plane also r = fma(q, d, -hi), one rounding of a value that always
// fits FP16 (an 11-bit scale times a <= 8-bit integer leaves at most 8 bits
// below hi's rounding point), so hi + r == d*q exactly.
__device__ __forceinline__ void mul_split(__half2 q, __half2 d2, uint32_t& hi, uint32_t* r) {
    const __half2 h = __hmul2(q, d2);
    hi = h2u(h);
    if (r) *r = h2u(__hfma2(q, d2, __hneg2(h)));
}

// 4 bytes of offset-binary Q8 (q + 128) -> 4 FP16 d*q (two half2), and the
// residuals when r != nullptr (r[0], r[1]).
__device__ __forceinline__ void q8_word(uint32_t w, __half2 d2, uint32_t& o01, uint32_t& o23, uint32_t* r) {
    const __half2 bias = u2h(0x64806480u);  // 1024 + 128 in both halves
    const __half2 h01 = __hsub2(u2h(__byte_perm(w, 0x64646464u, 0x4140)), bias);  // exact q
    const __half2 h23 = __hsub2(u2h(__byte_perm(w, 0x64646464u, 0x4342)), bias);
    mul_split(h01, d2, o01, r);
    mul_split(h23, d2, o23, r ? r + 1 : nullptr);
}

// Two Q4 bytes (b0 in byte 0, b1 in byte 2 of `x`) -> low and high nibbles as
// exact FP16 (n - 8), multiplied by d (residuals into rl / rh when given).
__device__ __forceinline__ void q4_pair(uint32_t x, __half2 d2, uint32_t& lo, uint32_t& hi, uint32_t* rl,
                                        uint32_t* rh) {
    const __half2 lo_h = __hsub2(u2h((x & 0x000F000Fu) | 0x64006400u), u2h(0x64086408u));  // 1024+n - 1032
    // (x & 0xF0) | 0x6400 = 1024 + 16 n; /16 - 72 = n - 8 (exact, one rounding)
    const __half2 hi_h = __hfma2(u2h((x & 0x00F000F0u) | 0x64006400u), u2h(0x2C002C00u) /* 1/16 */,
                                 u2h(0xD480D480u) /* -72 */);
    mul_split(lo_h, d2, lo, rl);
    mul_split(hi_h, d2, hi, rh);
}

template <int TYPE>
struct Dequant;

// Q8_0: a stage row segment is 64 bytes (4 raw chunks of 16 weights); thread
// d handles raw chunks d, d+128, d+256, d+384 of the 128x4 chunk grid.
template <>
struct Dequant<Q3XK_Q8_0> {
    static constexpr int kPerThread = 512 / kDqThreads;  // 128 rows x 4 raw chunks
    static constexpr int kRawRow = RAWK;  // quant bytes per staged row
    // raw: [128 rows][256 B] quants, then [128 rows][8] FP16 scales.
    // kk: which 64-column K-step of the 256-column raw stage.  SPLIT: the
    // residual plane goes to dst + kTileBytesW in the same layout.
    template <bool SPLIT>
    __device__ static void run(const uint8_t* raw, uint8_t* dst, int d, int kk) {
        const uint16_t* scales = reinterpret_cast<const uint16_t*>(raw + kRawQuantBytes);
#pragma unroll
        for (int i = 0; i < kPerThread; ++i) {
            const int idx = d + kDqThreads * i;
            const int m = idx >> 2, c = idx & 3;  // row in tile, 16-byte raw chunk
            const int col = kk * BK + 16 * c;     // column within the raw stage
            const uint4 q = *reinterpret_cast<const uint4*>(raw + m * kRawRow + col);
            const __half2 d2 = __half2half2(__ushort_as_half(scales[m * 8 + (col >> 5)]));
            uint4 o0, o1;
            uint32_t r[8];
            q8_word(q.x, d2, o0.x, o0.y, SPLIT ? r + 0 : nullptr);
            q8_word(q.y, d2, o0.z, o0.w, SPLIT ? r + 2 : nullptr);
            q8_word(q.z, d2, o1.x, o1.y, SPLIT ? r + 4 : nullptr);
            q8_word(q.w, d2, o1.z, o1.w, SPLIT ? r + 6 : nullptr);
            *reinterpret_cast<uint4*>(dst + sw128_off(m, 2 * c)) = o0;
            *reinterpret_cast<uint4*>(dst + sw128_off(m, 2 * c + 1)) = o1;
            if (SPLIT) {
                *reinterpret_cast<uint4*>(dst + kTileBytesW + sw128_off(m, 2 * c)) = make_uint4(r[0], r[1], r[2], r[3]);
                *reinterpret_cast<uint4*>(dst + kTileBytesW + sw128_off(m, 2 * c + 1)) =
                    make_uint4(r[4], r[5], r[6], r[7]);
            }
        }
    }
};

// Q4_0: a stage row segment is 2 blocks = 32 bytes (2 raw chunks of 32
// weights); element i < 16 of a block is the low nibble of byte i, i >= 16
// the high nibble of byte i - 16 (q4.h:31-36).
template <>
struct Dequant<Q3XK_Q4_0> {
    static constexpr int kPerThread = 256 / kDqThreads;  // 128 rows x 2 blocks
    static constexpr int kRawRow = RAWK / 2;
    template <bool SPLIT>
    __device__ static void run(const uint8_t* raw, uint8_t* dst, int d, int kk) {
        const uint16_t* scales = reinterpret_cast<const uint16_t*>(raw + kRawQuantBytes);
#pragma unroll
        for (int i = 0; i < kPerThread; ++i) {
            const int idx = d + kDqThreads * i;
            const int m = idx >> 1, b = idx & 1;  // row in tile, block within the K-step
            const int blk = kk * 2 + b;           // block within the raw stage
            const uint4 q = *reinterpret_cast<const uint4*>(raw + m * kRawRow + 16 * blk);
            const __half2 d2 = __half2half2(__ushort_as_half(scales[m * 8 + blk]));
            uint32_t l[8], h[8], rl[8], rh[8];
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // bytes (4j, 4j+1) and (4j+2, 4j+3) -> elements in order
                q4_pair(__byte_perm(w[j], 0u, 0x5150), d2, l[2 * j], h[2 * j], SPLIT ? rl + 2 * j : nullptr,
                        SPLIT ? rh + 2 * j : nullptr);
                q4_pair(__byte_perm(w[j], 0u, 0x5352), d2, l[2 * j + 1], h[2 * j + 1],
                        SPLIT ? rl + 2 * j + 1 : nullptr, SPLIT ? rh + 2 * j + 1 : nullptr);
            }
            const int c0 = 4 * b;  // 16-byte FP16 chunk of element 32b within the K-step
            *reinterpret_cast<uint4*>(dst + sw128_off(m, c0)) = make_uint4(l[0], l[1], l[2], l[3]);
            *reinterpret_cast<uint4*>(dst + sw128_off(m, c0 + 1)) = make_uint4(l[4], l[5], l[6], l[7]);
            *reinterpret_cast<uint4*>(dst + sw128_off(m, c0 + 2)) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(dst + sw128_off(m, c0 + 3)) = make_uint4(h[4], h[5], h[6], h[7]);
            if (SPLIT) {
                uint8_t* lo = dst + kTileBytesW;
                *reinterpret_cast<uint4*>(lo + sw128_off(m, c0)) = make_uint4(rl[0], rl[1], rl[2], rl[3]);
                *reinterpret_cast<uint4*>(lo + sw128_off(m, c0 + 1)) = make_uint4(rl[4], rl[5], rl[6], rl[7]);
                *reinterpret_cast<uint4*>(lo + sw128_off(m, c0 + 2)) = make_uint4(rh[0], rh[1], rh[2], rh[3]);
                *reinterpret_cast<uint4*>(lo + sw128_off(m, c0 + 3)) = make_uint4(rh[4], rh[5], rh[6], rh[7]);
            }
        }
    }
};

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, int* cta_err) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicOr(&g_gemm_error, 1);
    atomicExch(cta_err, 1);
    return false;
}

// Named barrier 1 over the 4 epilogue warps; the _and form returns whether
// every participating thread passed `ok` (so the warps leave together).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool epi_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)ok)
        : "memory");
    return r != 0;
}

// Accumulator columns [c0, c0 + 32) (16-token tiles: [c0, c0 + 16)) of this
// warp's lanes as floats; SPLIT adds the second half (column + BN).
template <int BN, bool SPLIT>
__device__ __forceinline__ void tmem_cols(uint32_t taddr, float (&v)[32]) {
    constexpr int W = BN >= 32 ? 32 : 16;
    uint32_t r[32], h[32];
    if constexpr (W == 32) {
        tmem_ld32(taddr, r);
        if (SPLIT) tmem_ld32(taddr + BN, h);
    } else {
        uint32_t a[16], b[16];
        tmem_ld16(taddr, a);
        if (SPLIT) tmem_ld16(taddr + BN, b);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            r[j] = a[j];
            h[j] = SPLIT ? b[j] : 0u;
        }
    }
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = SPLIT ? __uint_as_float(r[j]) + __uint_as_float(h[j]) : __uint_as_float(r[j]);
}

// K-steps [k0, k1) of unit `unit`.
__device__ __forceinline__ void unit_ksteps(const GemmParams& p, int unit, int& k0, int& k1) {
    if (p.ksplit > 1) {
        const int s = unit % p.ksplit;
        k0 = seg_begin(p, s);
        k1 = seg_begin(p, s + 1);
    } else {
        k0 = 0;
        k1 = p.ksteps;
    }
}

template <int TYPE, int BN, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xlomap,
            const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap smap, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    using G = TileN<BN, SPLIT>;
    constexpr int kTileBytesX = G::kTileBytesX;
    constexpr int kStageX = G::kStageX, kStageW = G::kStageW, kStages = G::kStages, kRaw = G::kRaw;
    constexpr int kXStages = G::kXStages;
    constexpr uint32_t kTmemCols = G::kTmemCols;
    constexpr uint32_t kIdesc = G::kIdesc, kIdescWide = G::kIdescWide;
    constexpr int kAccCols = G::kAccCols;
    uint8_t* sx = smem;                                // kXStages x planes x BN x 128 B (hi, then lo)
    uint8_t* sw = smem + kXStages * kStageX;           // kStages x planes x 16 KB (hi, then lo)
    uint8_t* sraw = sw + kStages * kStageW;            // kRaw x (32 + 2) KB
    uint64_t* bars = reinterpret_cast<uint64_t*>(sraw + kRaw * kRawBytes);
    uint64_t* full = bars;                 // weight stage: every dequant warp arrived
    uint64_t* empty = full + kStages;      // weight stage: its MMAs are done
    uint64_t* xfull = empty + kStages;     // X stage: bytes landed
    uint64_t* xempty = xfull + kXStages;   // X stage: its MMAs are done
    uint64_t* acc_full = xempty + kXStages;
    uint64_t* acc_empty = acc_full + kAcc;
    uint64_t* raw_full = acc_empty + kAcc;
    uint64_t* raw_empty = raw_full + kRaw;
    uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(raw_empty + kRaw);
    int* cta_err = reinterpret_cast<int*>(tmem_base_p + 1);
    int* last_flag = cta_err + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kDqWarps);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kXStages; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], 1);
        }
        for (int b = 0; b < kAcc; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        for (int r = 0; r < kRaw; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], kDqWarps);
        }
        *cta_err = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_base_p, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_p;
    griddep_launch_dependents();
    // X16, the scales, the counters, Y and (grouped) the tile table come from
    // earlier kernels.  The raw-weight producer of a plain GEMM reads none of
    // them (weights are immutable, its tiles are arithmetic on the
    // parameters), so it starts streaming while the previous kernel -- the X
    // conversion -- is still running.
    if (!(warp == 0 && lane == 0 && !p.groups)) griddep_wait();
    const int units = unit_count<BN>(p);
    const int S = p.groups ? 1 : p.ksplit;

    if (warp == 0) {
        // ---------------- TMA producers ----------------
        // Lane 0 streams the raw weight stages, lane 1 the X tiles: separate
        // threads, so the raw ring runs as far ahead as its own depth allows
        // instead of waiting on the (shallower) operand ring.
        if (lane == 0) {
            const int qdiv = TYPE == Q3XK_Q4_0 ? 2 : 1;  // quant bytes per column
            const uint32_t raw_tx = (uint32_t)(BM * (RAWK / qdiv) + kRawScaleBytes);
            int rit = 0;
            for (int unit = blockIdx.x; unit < units && !*(volatile int*)cta_err; unit += gridDim.x) {
                const TileCoord tc = tile_coord<BN>(p, unit / S);
                int k0, k1;
                unit_ksteps(p, unit, k0, k1);
                bool ok = true;
                for (int ks = k0; ks < k1; ks += kKPerRaw, ++rit) {
                    const int r = rit % kRaw;
                    if (rit >= kRaw && !wait_or_flag(&raw_empty[r], ((rit / kRaw) - 1) & 1, cta_err)) {
                        ok = false;
                        break;
                    }
                    uint8_t* dst = sraw + r * kRawBytes;
                    mbar_arrive_expect_tx(&raw_full[r], raw_tx);
                    tma_load_2d(dst, &qmap, ks * BK / qdiv, tc.w_row, &raw_full[r]);
                    tma_load_2d(dst + kRawQuantBytes, &smap, ks * BK / 32, tc.w_row, &raw_full[r]);
                }
                if (!ok) break;
            }
        } else if (lane == 1) {
            int it = 0;
            for (int unit = blockIdx.x; unit < units && !*(volatile int*)cta_err; unit += gridDim.x) {
                const TileCoord tc = tile_coord<BN>(p, unit / S);
                int k0, k1;
                unit_ksteps(p, unit, k0, k1);
                bool ok = true;
                for (int ks = k0; ks < k1; ++ks, ++it) {
                    const int s = it % kXStages;
                    if (it >= kXStages && !wait_or_flag(&xempty[s], ((it / kXStages) - 1) & 1, cta_err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&xfull[s], kStageX);
                    tma_load_2d(sx + s * kStageX, &xmap, ks * BK, tc.x_row, &xfull[s]);
                    if (SPLIT) tma_load_2d(sx + s * kStageX + kTileBytesX, &xlomap, ks * BK, tc.x_row, &xfull[s]);
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0, lt = 0;
            for (int unit = blockIdx.x; unit < units && !*(volatile int*)cta_err; unit += gridDim.x, ++lt) {
                int k0, k1;
                unit_ksteps(p, unit, k0, k1);
                const int b = lt % kAcc;
                if (lt >= kAcc && !wait_or_flag(&acc_empty[b], ((lt / kAcc) - 1) & 1, cta_err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * kAccCols;
                bool ok = true;
                for (int ks = k0; ks < k1; ++ks, ++it) {
                    const int s = it % kStages, sxi = it % kXStages;
                    if (!wait_or_flag(&xfull[sxi], (it / kXStages) & 1, cta_err) ||
                        !wait_or_flag(&full[s], (it / kStages) & 1, cta_err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sw + s * kStageW), b0 = smem_u32(sx + sxi * kStageX);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ah = sw128_desc(a0 + kk * 32), bh = sw128_desc(b0 + kk * 32);
                        // SPLIT: B = [x_hi; x_lo] (2 BN rows) -> both halves of the accumulator
                        umma_f16(d_tmem, ah, bh, kIdescWide, (ks > k0 || kk) ? 1u : 0u);
                        if (SPLIT)  // + w_lo x_hi into the first half
                            umma_f16(d_tmem, sw128_desc(a0 + kTileBytesW + kk * 32), bh, kIdesc, 1u);
                    }
                    umma_commit(&empty[s]);     // weight stage s free once these MMAs finish
                    umma_commit(&xempty[sxi]);  // and X stage sxi
                }
                if (!ok) break;
                umma_commit(&acc_full[b]);
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------- dequantisers ----------------
        const int d = threadIdx.x - 64;
        int it = 0, rit = 0;
        for (int unit = blockIdx.x; unit < units && !*(volatile int*)cta_err; unit += gridDim.x) {
            int k0, k1;
            unit_ksteps(p, unit, k0, k1);
            bool ok = true;
            for (int ks = k0; ks < k1; ++ks, ++it) {
                const int kk = (ks - k0) % kKPerRaw;
                const int r = rit % kRaw;
                if (kk == 0) {
                    int good = 1;
                    if (lane == 0) good = wait_or_flag(&raw_full[r], (rit / kRaw) & 1, cta_err);
                    good = __shfl_sync(0xffffffffu, good, 0);
                    if (!good) {
                        ok = false;
                        break;
                    }
                }
                const int s = it % kStages;
                if (it >= kStages) {
                    int good = 1;
                    if (lane == 0) good = wait_or_flag(&empty[s], ((it / kStages) - 1) & 1, cta_err);
                    good = __shfl_sync(0xffffffffu, good, 0);
                    if (!good) {
                        ok = false;
                        break;
                    }
                }
                Dequant<TYPE>::template run<SPLIT>(sraw + r * kRawBytes, sw + s * kStageW, d, kk);
                fence_proxy_async_smem();  // generic-proxy writes -> tensor core reads
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                if (kk == kKPerRaw - 1 || ks == k1 - 1) {
                    if (lane == 0) mbar_arrive(&raw_empty[r]);
                    ++rit;
                }
            }
            if (!ok) break;
        }
    } else {
        // ---------------- epilogue (TMEM -> Y, or -> split-K partial) ----------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int m = 32 * q + lane;  // row of the tile
        int lt = 0;
        for (int unit = blockIdx.x; unit < units; unit += gridDim.x, ++lt) {
            const int tile = unit / S;
            const TileCoord tc = tile_coord<BN>(p, tile);
            const int b = lt % kAcc;
            int good = 1;
            if (lane == 0) good = wait_or_flag(&acc_full[b], (lt / kAcc) & 1, cta_err);
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!epi_all(good)) break;  // all 4 warps leave together
            tc_fence_after();
            const int n = tc.n0 + m;
            if (S == 1) {
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float r[32];
                    tmem_cols<BN, SPLIT>(tmem + ((uint32_t)(32 * q) << 16) + b * kAccCols + c0, r);
#pragma unroll
                    for (int j = 0; j < (BN < 32 ? BN : 32); ++j) {
                        if (c0 + j < tc.t_valid && n < p.N) {
                            const int t = tc.x_row + c0 + j;
                            const float v = r[j] * __ldg(&p.tok_scale[t]);
                            float* yp = p.y + (int64_t)t * p.N + n;
                            *yp = p.accumulate ? *yp + v : v;
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[b]);
                continue;
            }
            // split-K: this segment's raw accumulators -> part[unit][m][c]
            float* mine = p.part + (size_t)unit * BM * BN + (size_t)m * BN;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float r[32];
                tmem_cols<BN, SPLIT>(tmem + ((uint32_t)(32 * q) << 16) + b * kAccCols + c0, r);
#pragma unroll
                for (int j = 0; j < (BN < 32 ? BN : 32); j += 4)
                    __stcg(reinterpret_cast<float4*>(mine + c0 + j), make_float4(r[j], r[j + 1], r[j + 2], r[j + 3]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);  // TMEM reusable; the partial is in memory
            __threadfence();
            epi_sync();
            if (warp == kEpiWarp0 && lane == 0) *last_flag = atomicAdd(&p.counters[tile], 1) == S - 1;
            epi_sync();
            if (*(volatile int*)last_flag) {
                // every segment of this tile has landed: add them in segment order,
                // 8 columns at a time with every segment's loads in flight at once
                __threadfence();
                const float* base = p.part + (size_t)tile * S * BM * BN + (size_t)m * BN;
#pragma unroll 1
                for (int c0 = 0; c0 < BN && c0 < tc.t_valid; c0 += 8) {
                    float4 a[kMaxSplit][2];
#pragma unroll
                    for (int sg = 0; sg < kMaxSplit; ++sg)
                        if (sg < S) {
                            const float4* src = reinterpret_cast<const float4*>(base + (size_t)sg * BM * BN + c0);
                            a[sg][0] = __ldcg(src);
                            a[sg][1] = __ldcg(src + 1);
                        }
                    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int sg = 0; sg < kMaxSplit; ++sg)
                        if (sg < S) {
                            v[0] += a[sg][0].x; v[1] += a[sg][0].y; v[2] += a[sg][0].z; v[3] += a[sg][0].w;
                            v[4] += a[sg][1].x; v[5] += a[sg][1].y; v[6] += a[sg][1].z; v[7] += a[sg][1].w;
                        }
                    if (n < p.N) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (c0 + j < tc.t_valid) {
                                const int t = tc.x_row + c0 + j;
                                const float r = v[j] * __ldg(&p.tok_scale[t]);
                                float* yp = p.y + (int64_t)t * p.N + n;
                                *yp = p.accumulate ? *yp + r : r;
                            }
                        }
                    }
                }
                epi_sync();
                if (warp == kEpiWarp0 && lane == 0) p.counters[tile] = 0;  // ready for the next call
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

int sm_count() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            count = 148;
    }
    return count;
}

}  // namespace

int launch_x_to_f16(const float* x, int T, int K, __half* x16, __half* x16lo, float* tok_scale, cudaStream_t s,
                    int* counters) {
    if (K % 8) return Q3XK_EINVAL;  // TMA row stride of X16 must be a multiple of 16 bytes
    if (launch_pdl(x_to_f16_kernel, dim3(T), dim3(kXThreads), 0, s, x, x16, x16lo, tok_scale, K, counters) !=
        cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

namespace {

using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemmParams);

struct KernSlot {
    Kern fn;
    size_t smem;
    bool configured;
};

template <int TYPE, int BN, bool SPLIT>
constexpr KernSlot slot_of() {
    return KernSlot{gemm_kernel<TYPE, BN, SPLIT>, TileN<BN, SPLIT>::kSmem, false};
}

constexpr int kBNs[4] = {16, 64, 128, 256};
int bn_index(int bn) { return bn == 16 ? 0 : bn == 64 ? 1 : bn == 128 ? 2 : 3; }

// [type: Q8_0, Q4_0][BN: 16, 64, 128, 256][FP16, SPLIT]; split has no 256-token tile.
KernSlot g_kernels[2][4][2] = {
    {{slot_of<Q3XK_Q8_0, 16, false>(), slot_of<Q3XK_Q8_0, 16, true>()},
     {slot_of<Q3XK_Q8_0, 64, false>(), slot_of<Q3XK_Q8_0, 64, true>()},
     {slot_of<Q3XK_Q8_0, 128, false>(), slot_of<Q3XK_Q8_0, 128, true>()},
     {slot_of<Q3XK_Q8_0, 256, false>(), KernSlot{nullptr, 0, false}}},
    {{slot_of<Q3XK_Q4_0, 16, false>(), slot_of<Q3XK_Q4_0, 16, true>()},
     {slot_of<Q3XK_Q4_0, 64, false>(), slot_of<Q3XK_Q4_0, 64, true>()},
     {slot_of<Q3XK_Q4_0, 128, false>(), slot_of<Q3XK_Q4_0, 128, true>()},
     {slot_of<Q3XK_Q4_0, 256, false>(), KernSlot{nullptr, 0, false}}},
};

bool encode_x_map(EncodeTiled enc, CUtensorMap* map, const __half* x16, int T, int K, int bn) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {BK, (cuuint32_t)bn};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x16), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K segments per tile when the tiles alone leave SMs idle: the count that
// minimises (waves of units) x (raw stages per segment), with a small charge
// for the partials' round trip; bounded by kMaxSplit, by the raw stages of a
// row and by the workspace's kMaxSplitUnits.
int choose_ksplit(int tiles, int nraw, int sms) {
    if (tiles >= sms) return 1;
    int best = 1;
    double best_cost = 1e30;
    for (int S = 1; S <= kMaxSplit && S <= nraw && tiles * S <= kMaxSplitUnits; ++S) {
        const int waves = (tiles * S + sms - 1) / sms;
        const double cost = (double)waves * ((nraw + S - 1) / S) + (S > 1 ? 0.5 : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = S;
        }
    }
    return best;
}

}  // namespace

int gemm_f16(const q3xk_matrix* w, const __half* x16, const __half* x16lo, const float* tok_scale, int T, float* y,
             int accumulate, const GemmGroups* groups, int bn_hint, cudaStream_t s, const GemmSplitWs* splitws) {
    const int K = w->cols;
    const bool split = x16lo != nullptr;
    if (K % 8 || ((uintptr_t)x16 & 15) || ((uintptr_t)x16lo & 15) || ((uintptr_t)w->data & 15)) return Q3XK_EALIGN;
    // Token tile = MMA N: the smallest of 16/64/128/256 that covers T, else
    // 256 (split precision: at most 128; grouped: 64).
    int bn = groups ? 64 : bn_hint ? bn_hint : T <= 16 ? 16 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
    if (split && bn > 128) bn = 128;
    if (bn != 16 && bn != 64 && bn != 128 && bn != 256) return Q3XK_EINVAL;
    EncodeTiled enc = encode_fn();
    if (!enc) return Q3XK_ECUDA;
    CUtensorMap map, lomap;
    if (!encode_x_map(enc, &map, x16, T, K, bn)) return Q3XK_ECUDA;
    if (!encode_x_map(enc, &lomap, split ? x16lo : x16, T, K, bn)) return Q3XK_ECUDA;

    // Raw weights: the quant bytes of every row record (uint8, [rows][qbytes])
    // and the scales ([rows][cols/32] FP16), both with the record stride; a
    // pool is one tensor of experts * rows rows.
    const int64_t qbytes = quant_bytes(w->type, K);
    const int64_t all_rows = (int64_t)w->rows * (groups ? w->experts : 1);
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap qmap, smap;
    {
        const cuuint64_t qd[2] = {(cuuint64_t)qbytes, (cuuint64_t)all_rows};
        const cuuint64_t qs[1] = {(cuuint64_t)w->row_stride};
        const cuuint32_t qb[2] = {(cuuint32_t)(w->type == Q3XK_Q4_0 ? RAWK / 2 : RAWK), BM};
        if (enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->data, qd, qs, qb, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return Q3XK_ECUDA;
        const cuuint64_t sd[2] = {(cuuint64_t)(K / kBlock), (cuuint64_t)all_rows};
        const cuuint32_t sb[2] = {8, BM};
        if (enc(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, static_cast<uint8_t*>(w->data) + qbytes, sd, qs, sb, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return Q3XK_ECUDA;
    }

    GemmParams p{};
    p.w = static_cast<const uint8_t*>(w->data);
    p.row_stride = w->row_stride;
    p.qbytes = qbytes;
    p.N = w->rows;
    p.K = K;
    p.T = T;
    p.tok_scale = tok_scale;
    p.y = y;
    p.accumulate = accumulate ? 1 : 0;
    p.tiles_w = (w->rows + BM - 1) / BM;
    p.tiles_t = (T + bn - 1) / bn;
    p.ksteps = (K + BK - 1) / BK;
    p.nraw = (p.ksteps + kKPerRaw - 1) / kKPerRaw;
    p.ksplit = 1;
    if (groups) {
        p.groups = groups->groups;
        p.xoff = groups->xoff;
        p.tile_off = groups->tile_off;
    } else if (splitws && bn <= kSplitMaxBN) {
        p.ksplit = choose_ksplit(p.tiles_w * p.tiles_t, p.nraw, sm_count());
        if (p.ksplit > 1) {
            if (p.tiles_w * p.tiles_t > kCounterInts) return Q3XK_EUNSUPPORTED;  // cannot happen: tiles < SMs
            p.part = splitws->part;
            p.counters = splitws->counters;
        }
    }
    KernSlot& ks = g_kernels[w->type == Q3XK_Q8_0 ? 0 : 1][bn_index(bn)][split ? 1 : 0];
    if (!ks.fn) return Q3XK_EUNSUPPORTED;
    if (!ks.configured) {
        if (cudaFuncSetAttribute(ks.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ks.smem) != cudaSuccess)
            return Q3XK_ECUDA;
        ks.configured = true;
    }
    // grouped: the tile count is only known on the device -> one CTA per SM
    const int units = groups ? sm_count() : p.tiles_w * p.tiles_t * p.ksplit;
    const int grid = units < sm_count() ? units : sm_count();
    const cudaError_t e1 = launch_pdl(ks.fn, dim3(grid), dim3(kThreads), ks.smem, s, map, lomap, qmap, smap, p);
    if (e1 != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return last_launch_status();
}

size_t gemm_grouped_tile_width() { return 64; }

int gemm_clear_error() {
    const int zero = 0;
    return cuda_status(cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof zero));
}

namespace {

// Workspace of one call: two FP16 planes of X (hi, lo), each 256-byte
// aligned, the token scales, the split-K counters, then the split-K partials.
struct WsLayout {
    size_t plane, scale_off, counter_off, part_off, total;
};
WsLayout ws_layout(int T, int K) {
    WsLayout l;
    l.plane = ((size_t)T * K * 2 + 255) & ~(size_t)255;
    l.scale_off = 2 * l.plane;
    l.counter_off = l.scale_off + (((size_t)T * 4 + 255) & ~(size_t)255);
    l.part_off = l.counter_off + (size_t)kCounterInts * 4;
    l.total = l.part_off + kPartBytes;
    return l;
}

}  // namespace

}  // namespace q3xk

using namespace q3xk;

extern "C" {

int q3xk_gemm_workspace_bytes(int T, int K, size_t* bytes) {
    if (!bytes || T <= 0 || K <= 0) return Q3XK_EINVAL;
    *bytes = ws_layout(T, K).total;
    return Q3XK_OK;
}

int q3xk_gemm_ex(const q3xk_matrix* w, const float* x, int T, float* y, int accumulate, int precision,
                 void* workspace, size_t workspace_bytes, void* stream) {
    if (!w || !w->data || !x || !y || T <= 0 || w->rows <= 0 || w->cols <= 0) return Q3XK_EINVAL;
    if (precision != Q3XK_GEMM_SPLIT && precision != Q3XK_GEMM_FP16) return Q3XK_EINVAL;
    if (w->type != Q3XK_Q8_0 && w->type != Q3XK_Q4_0) return Q3XK_EUNSUPPORTED;
    if (w->cols % kBlock || w->row_stride != row_record_bytes(w->type, w->cols)) return Q3XK_EINVAL;
    const WsLayout l = ws_layout(T, w->cols);
    if (!workspace || workspace_bytes < l.total) return Q3XK_EWORKSPACE;
    if (((uintptr_t)workspace & 255) || ((uintptr_t)x & 15) || ((uintptr_t)w->data & 15) || ((uintptr_t)y & 3))
        return Q3XK_EALIGN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int K = w->cols;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __half* x16 = reinterpret_cast<__half*>(ws);
    __half* x16lo = precision == Q3XK_GEMM_SPLIT ? reinterpret_cast<__half*>(ws + l.plane) : nullptr;
    float* tok_scale = reinterpret_cast<float*>(ws + l.scale_off);
    const GemmSplitWs sw{reinterpret_cast<float*>(ws + l.part_off), reinterpret_cast<int*>(ws + l.counter_off)};
    const int st = launch_x_to_f16(x, T, K, x16, x16lo, tok_scale, s, sw.counters);
    if (st != Q3XK_OK) return st;
    return gemm_f16(w, x16, x16lo, tok_scale, T, y, accumulate, nullptr, 0, s, &sw);
}

int q3xk_gemm(const q3xk_matrix* w, const float* x, int T, float* y, int accumulate, void* workspace,
              size_t workspace_bytes, void* stream) {
    return q3xk_gemm_ex(w, x, T, y, accumulate, Q3XK_GEMM_SPLIT, workspace, workspace_bytes, stream);
}

int q3xk_gemm_device_error(int* flags) {
    if (!flags) return Q3XK_EINVAL;
    return cuda_status(cudaMemcpyFromSymbol(flags, g_gemm_error, sizeof(int)));
}

}  // extern "C"
