// engine.cu -- the qwen3x backend on one B200: model.bin load, state, forward.
//
// Implements q3x_backend (internal.h:11-34) and its C mirror (q3x_backend.h).
// The forward follows the reference CPU engine (engine.cpp:406-458) layer by
// layer, with every matrix product on the packed-weight path:
//   T == 1   q3xk_gemv (CUDA cores, HBM-bound; residual adds fused as y += W x)
//   T >  1   q3xk_gemm (tcgen05 dequant-GEMM) for Q8_0/Q4_0 models
//   MoE      router GEMV -> device top-k -> grouped expert GEMVs over pools
//            that hold the shared expert as one more expert (engine.cpp:406-430)
//   logits   rms of the last token -> lm_head GEMV; argmax on the device.
// Matrices that read the same input are stored as one matrix (row
// concatenation), so a DeltaNet layer reads its input once for qkv|z|a|b,
// attention once for q|k|v, the FFN once for gate|up.
//
// Device layout: one arena holds every weight (row-record matrices, FP32
// norms with the 1 + w' folded in); a State owns the recurrent arena (conv
// history + DeltaNet memory of every DeltaNet layer, as engine.cpp:126-160),
// the KV cache, the logits and chunk-sized work buffers.  Positions live in
// device memory, so a decode step (count 1, logits) is one CUDA graph replay.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>
#include <thread>
#include <vector>

#include "layers.cuh"
#include "q3x_backend.h"
#include "tp.cuh"

namespace q3xk {
namespace {

constexpr int kMaxContext = 262144;                 // model_config.h:13
constexpr size_t kHeaderSize = 8 + 16 * 4;          // model_config.h:10-12
constexpr int kEndOfText = 248044, kImEnd = 248046;  // engine.cpp:28
constexpr int kChunk = 2048;                        // prefill tokens per pass
constexpr int kMaxBatch = 16;                       // sequences per batched decode step
constexpr size_t kAlign = 256;

struct Config {
    uint32_t id;
    const char* name;
    int V, H, I, N, AI, AH, KVH, AD, RD, KH, VH, KD, VD, CK;
    int experts, top_k, shared_I;
    int matrix_type;
    bool tied;
};

// model_config.h:59-101 (registered IDs) plus the IDs this build adds: a
// Q8_0 27B-shaped model and three small test models with the real head sizes.
const Config kConfigs[] = {
    {800, "Qwen3.5-0.8B", 248320, 1024, 3584, 24, 4, 8, 2, 256, 64, 16, 16, 128, 128, 4, 0, 0, 0, Q3XK_BF16, true},
    {4000, "Qwen3.5-4B", 248320, 2560, 9216, 32, 4, 16, 4, 256, 64, 16, 32, 128, 128, 4, 0, 0, 0, Q3XK_BF16, true},
    {9000, "Qwen3.5-9B", 248320, 4096, 12288, 32, 4, 16, 4, 256, 64, 16, 32, 128, 128, 4, 0, 0, 0, Q3XK_Q8_0, false},
    {36035, "Qwen3.6-35B-A3B", 248320, 2048, 512, 40, 4, 16, 2, 256, 64, 16, 32, 128, 128, 4, 256, 8, 512,
     Q3XK_Q4_0, false},
    {38027, "Qwen3.8-27B", 248320, 5120, 17408, 64, 4, 24, 4, 256, 64, 16, 48, 128, 128, 4, 0, 0, 0, Q3XK_Q4_0,
     false},
    {27008, "27B-shaped Q8_0", 248320, 5120, 17408, 64, 4, 24, 4, 256, 64, 16, 48, 128, 128, 4, 0, 0, 0, Q3XK_Q8_0,
     false},
    {9091, "test dense Q8_0", 4096, 512, 1024, 8, 4, 2, 1, 256, 64, 2, 4, 128, 128, 4, 0, 0, 0, Q3XK_Q8_0, false},
    {9092, "test dense Q4_0", 4096, 512, 1024, 4, 4, 2, 1, 256, 64, 2, 4, 128, 128, 4, 0, 0, 0, Q3XK_Q4_0, false},
    {35091, "test MoE Q4_0", 4096, 512, 128, 4, 4, 2, 1, 256, 64, 2, 4, 128, 128, 4, 16, 4, 128, Q3XK_Q4_0, false},
};

const Config* config_for_id(uint32_t id) {
    for (const Config& c : kConfigs)
        if (c.id == id) return &c;
    return nullptr;
}

uint32_t header_field(const uint8_t* file, int i) {
    uint32_t v;
    std::memcpy(&v, file + 8 + 4 * (size_t)i, 4);
    return v;
}

// model_config.h:107-133
bool header_matches(const uint8_t* file, const Config& c) {
    const uint32_t expect[16] = {c.id,         (uint32_t)c.V,   (uint32_t)c.H,   (uint32_t)c.I,  (uint32_t)c.N,
                                 (uint32_t)c.AI, (uint32_t)c.AH,  (uint32_t)c.KVH, (uint32_t)c.AD, (uint32_t)c.RD,
                                 (uint32_t)c.KH, (uint32_t)c.VH,  (uint32_t)c.KD,  (uint32_t)c.VD, (uint32_t)c.CK,
                                 (uint32_t)kMaxContext};
    for (int i = 0; i < 16; ++i)
        if (header_field(file, i) != expect[i]) return false;
    return true;
}

bool is_delta(const Config& c, int layer) { return layer % c.AI != c.AI - 1; }

float bf16_to_float(uint16_t b) {
    const uint32_t bits = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

struct Layer {
    bool delta = false;
    float* in_norm = nullptr;  // 1 + w'
    float* post_norm = nullptr;
    q3xk_matrix in_proj{};  // delta: [qkv | z | a | b]; attention: [q+gate | k | v]
    q3xk_matrix out{};      // delta.out / attention.out
    float *conv = nullptr, *alog = nullptr, *dt = nullptr, *dnorm = nullptr;  // DeltaNet
    float *qn1 = nullptr, *kn1 = nullptr;                                     // attention
    q3xk_matrix gate_up{};  // FFN gate|up, rows interleaved g g u u (repack_swiglu);
                            // MoE pool [experts + 1][2I] the same way (shared expert last)
    q3xk_matrix down{};     // FFN down; MoE pool [experts + 1][H]
    q3xk_matrix router{};   // MoE: BF16 [experts + 1][H] = router rows + shared gate row
};

// Share of one rank (world = 1: everything).  Dense models, tensor
// parallelism -- column-parallel (split output rows): DeltaNet q/k by key
// head, v/z/a/b by value head, attention q+gate by query head, k/v by KV head
// (replicated when there are fewer KV heads than ranks), FFN gate/up by
// intermediate row, lm_head by vocabulary row; row-parallel (split input
// columns, partial sums all-reduced): DeltaNet out, attention out, FFN down.
// MoE models, expert parallelism -- the routed experts [e0, e0 + el) of every
// layer, everything else (router and shared expert included) replicated; each
// rank adds the slots it runs into a partial sum that is all-reduced.
// lc = the rank's dims (lc.experts stays the routed total).
struct Shard {
    int rank = 0, world = 1;
    int kh0 = 0, vh0 = 0, ah0 = 0, kv0 = 0, i0 = 0, v0 = 0;
    bool ep = false;
    int e0 = 0, el = 0;
    Config lc{};
};

// Pool index of the shared expert where this rank runs it, else -1: under
// expert parallelism the shared expert of layer i runs on rank i % world.
int shared_slot(const Shard& sh, int layer) { return layer % sh.world == sh.rank ? sh.el : -1; }

const char* make_shard(const Config& c, int rank, int world, Shard& sh) {
    sh = Shard{};
    sh.rank = rank;
    sh.world = world;
    sh.lc = c;
    sh.el = c.experts;
    if (world < 1 || rank < 0 || rank >= world) return "invalid tensor-parallel rank";
    if (world == 1) return nullptr;
    if (c.experts) {
        if (c.experts % world) return "the experts do not split over the expert-parallel ranks";
        sh.ep = true;
        sh.el = c.experts / world;
        sh.e0 = rank * sh.el;
        return nullptr;
    }
    if (c.KH % world || c.VH % world || c.AH % world || c.V % world || c.I % world || (c.I / world) % 32)
        return "model shape does not split over the tensor-parallel ranks";
    const int ahn = c.AH / world, G = c.AH / c.KVH;
    int kvn = 0;
    if (c.KVH % world == 0) {
        kvn = c.KVH / world;
        sh.kv0 = rank * kvn;
    } else if (world % c.KVH == 0 && G % ahn == 0) {
        kvn = 1;  // the rank's query heads share one KV head, replicated on its group of ranks
        sh.kv0 = rank * ahn / G;
    } else {
        return "model shape does not split over the tensor-parallel ranks";
    }
    sh.kh0 = rank * (c.KH / world);
    sh.vh0 = rank * (c.VH / world);
    sh.ah0 = rank * ahn;
    sh.i0 = rank * (c.I / world);
    sh.v0 = rank * (c.V / world);
    sh.lc.KH = c.KH / world;
    sh.lc.VH = c.VH / world;
    sh.lc.AH = ahn;
    sh.lc.KVH = kvn;
    sh.lc.I = c.I / world;
    sh.lc.V = c.V / world;
    return nullptr;
}

// Bytes of `cols` packed columns of one model.bin row.
size_t row_bytes(int type, int cols) {
    return type == Q3XK_BF16 ? (size_t)cols * 2
                             : (size_t)cols / kBlock * (type == Q3XK_Q8_0 ? kQ8PackedBytes : kQ4PackedBytes);
}

}  // namespace
}  // namespace q3xk

using namespace q3xk;

namespace q3x_backend {

struct Model {
    const Config* config = nullptr;
    int device = 0;
    int fd = -1;
    size_t file_size = 0;
    const uint8_t* file = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    q3xk_matrix embedding{}, lm_head{};
    float* final_norm = nullptr;
    std::vector<q3xk::Layer> layer;
    int P = 0;       // widest in_proj / gate_up (dense) row count
    int mix = 0;     // widest mixer output (DO, AS, I)
    int maxcols = 0; // widest matrix input
    Shard shard;     // this rank's share (world = 1 unless created for tensor parallelism)

    ~Model() {
        if (arena) {
            cudaSetDevice(device);
            cudaFree(arena);
        }
        if (file) munmap(const_cast<uint8_t*>(file), file_size);
        if (fd >= 0) close(fd);
    }
    bool load(const char* path, int rank, int world, const char** error);
};

struct State {
    Model* model = nullptr;
    const Config* c = nullptr;
    int device = 0;
    int capacity = 0, position = 0, checkpoint_position = 0;
    cudaStream_t stream = nullptr;
    // recurrent arena: per DeltaNet layer conv history [DQKV][CK-1] then memory [VH][KD][VD]
    float* recurrent = nullptr;
    float* checkpoint_recurrent = nullptr;
    size_t recurrent_floats = 0;
    std::vector<float*> conv, memory, kcache, vcache;
    float* kv = nullptr;
    float *logits = nullptr, *checkpoint_logits = nullptr;
    int* pos = nullptr;        // device position
    int* tokens = nullptr;     // device tokens of the current chunk
    int* argmax_out = nullptr;
    void* argmax_ws = nullptr;
    size_t argmax_ws_bytes = 0;
    float *hidden = nullptr, *normed = nullptr, *proj = nullptr, *mix = nullptr, *part = nullptr;
    float *rlogits = nullptr, *rweights = nullptr, *hbuf = nullptr;
    float* delta_work = nullptr;  // chunked DeltaNet workspace (prefill)
    float* qkv = nullptr;         // conv output q | k | v of a prefill pass [chunk][DQKV]
    MoePrefillArgs moe{};         // work buffers of the grouped MoE prompt path
    int* rids = nullptr;
    int* group_count = nullptr;  // [KH] arrival counts of the fused-conv delta kernel (kept zero)
    void* gemm_ws = nullptr;
    size_t gemm_ws_bytes = 0;
    int split_len = 0;
    int rank = 0, world = 1;
    bool tp = false;               // tensor parallelism (dense model, world > 1)
    bool ep = false;               // expert parallelism (MoE model, world > 1)
    void* comm = nullptr;          // NCCL communicator (world > 1)
    float* partial = nullptr;      // row-parallel partial sums [chunk][H] (world > 1)
    float* full_logits = nullptr;  // gathered logits [V] (world > 1)
    float* best = nullptr;         // [world][2] (value, index) of each rank's argmax
    void* peer_buf = nullptr;      // own one-shot all-reduce buffer (CUDA IPC exported)
    void* peer_bases[8] = {};      // every rank's buffer, mapped (own one included)
    bool peer_ready = false;       // decode all-reduces go over peer memory
    int* peer_seq = nullptr;       // call counter of the peer all-reduce
    int* tp_err = nullptr;         // set by a peer all-reduce that gave up waiting
    int* tp_err_host = nullptr;    // pinned copy of tp_err, refreshed after every forward
    double peer_timeout_s = 1.0;   // bound of the peer all-reduce's wait for a peer
    bool use_graphs = true;
    bool exact_prefill = false;  // T > 1 through per-token GEMVs instead of the GEMM
    int gemm_precision = Q3XK_GEMM_SPLIT;  // prompt GEMMs: split (FP32-grade) or FP16
    int chunk = 0;               // tokens per forward pass (work buffers hold `chunk_capacity`)
    int chunk_capacity = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    cudaEvent_t batch_event = nullptr;  // orders this state's stream against a batched step it joins
    float* batch_logits = nullptr;      // [chunk][V] lm_head output of a batched step this state leads
    uint64_t uid = 0;                   // unique per State of the process (never reused)
    // the batched step this State leads, captured as a graph for one set of States
    cudaGraphExec_t batch_exec = nullptr;
    std::vector<uint64_t> batch_key;
    std::vector<void*> allocations;

    ~State() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (graph_exec) cudaGraphExecDestroy(graph_exec);
        if (graph) cudaGraphDestroy(graph);
        if (batch_exec) cudaGraphExecDestroy(batch_exec);
        for (int r = 0; r < world && r < 8; ++r)
            if (peer_ready && r != rank && peer_bases[r]) cudaIpcCloseMemHandle(peer_bases[r]);
        for (void* p : allocations) cudaFree(p);
        if (tp_err_host) cudaFreeHost(tp_err_host);
        if (batch_event) cudaEventDestroy(batch_event);
        tp_comm_destroy(comm);
        if (stream) cudaStreamDestroy(stream);
    }
    template <typename T>
    bool alloc(T** p, size_t count) {
        void* raw = nullptr;
        if (cudaMalloc(&raw, count * sizeof(T) > 0 ? count * sizeof(T) : 16) != cudaSuccess) return false;
        allocations.push_back(raw);
        *p = static_cast<T*>(raw);
        return true;
    }
};

}  // namespace q3x_backend

using q3x_backend::Model;
using q3x_backend::State;

namespace q3xk {
namespace {

// engine.cpp:461-477 `take`: 64-byte aligned tensors in a fixed order.
struct Cursor {
    const uint8_t* file;
    size_t size, pos;
    const char* error = nullptr;
    const uint8_t* take(size_t bytes) {
        if (error) return nullptr;
        const size_t pad = (64 - pos % 64) % 64;
        if (pos > size || pad > size - pos) {
            error = "truncated model.bin";
            return nullptr;
        }
        pos += pad;
        if (bytes > size - pos) {
            error = "truncated model.bin";
            return nullptr;
        }
        const uint8_t* r = file + pos;
        pos += bytes;
        return r;
    }
};

// Builds the device copy of the model.  Pass 0 only sizes the arena; pass 1
// carves it and uploads (matrices through a device staging buffer and
// q3xk_repack, small vectors converted to FP32 on the host).
struct Loader {
    Model& m;
    const Config& c;
    int pass = 0;
    size_t used = 0;
    uint8_t* staging = nullptr;
    size_t staging_bytes = 0;
    cudaStream_t stream = nullptr;
    int status = Q3XK_OK;
    std::vector<float> host;
    std::vector<uint8_t> gather;
    // Host -> device copies of the file's bytes go through two pinned buffers:
    // host threads copy chunk i into one while the DMA of chunk i - 1 runs from
    // the other (pageable copies from the mmap are staged by the driver and do
    // not overlap with anything).
    static constexpr size_t kPinChunk = (size_t)64 << 20;
    static constexpr int kCopyThreads = 8;
    uint8_t* pinned[2] = {nullptr, nullptr};
    cudaEvent_t pin_free[2] = {nullptr, nullptr};
    int pin_next = 0;

    bool open_pinned() {
        for (int i = 0; i < 2; ++i) {
            if (cudaHostAlloc(reinterpret_cast<void**>(&pinned[i]), kPinChunk, cudaHostAllocDefault) != cudaSuccess ||
                cudaEventCreateWithFlags(&pin_free[i], cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                close_pinned();
                return false;
            }
        }
        return true;
    }
    void close_pinned() {
        for (int i = 0; i < 2; ++i) {
            if (pin_free[i]) cudaEventSynchronize(pin_free[i]), cudaEventDestroy(pin_free[i]);
            if (pinned[i]) cudaFreeHost(pinned[i]);
            pinned[i] = nullptr;
            pin_free[i] = nullptr;
        }
    }
    // dst (device) <- bytes of src (host) on `stream`.
    bool h2d(void* dst, const uint8_t* src, size_t bytes) {
        if (!pinned[0]) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream) == cudaSuccess;
        for (size_t off = 0; off < bytes; off += kPinChunk) {
            const size_t len = bytes - off < kPinChunk ? bytes - off : kPinChunk;
            const int b = pin_next;
            pin_next ^= 1;
            if (cudaEventSynchronize(pin_free[b]) != cudaSuccess) return false;  // its last DMA is done
            uint8_t* buf = pinned[b];
            const uint8_t* from = src + off;
            if (len < ((size_t)4 << 20)) {
                std::memcpy(buf, from, len);
            } else {
                std::thread workers[kCopyThreads];
                const size_t part = (len + kCopyThreads - 1) / kCopyThreads;
                for (int t = 0; t < kCopyThreads; ++t) {
                    const size_t a = (size_t)t * part, e = a + part < len ? a + part : len;
                    if (a < e) workers[t] = std::thread([=] { std::memcpy(buf + a, from + a, e - a); });
                }
                for (auto& w : workers)
                    if (w.joinable()) w.join();
            }
            if (cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, buf, len, cudaMemcpyHostToDevice, stream) !=
                    cudaSuccess ||
                cudaEventRecord(pin_free[b], stream) != cudaSuccess)
                return false;
        }
        return true;
    }

    uint8_t* carve(size_t bytes) {
        const size_t at = used;
        used += align_up(bytes);
        return pass == 0 ? nullptr : m.arena + at;
    }
    // A matrix (or pool) of `rows` x `cols` per expert in row-record layout.
    q3xk_matrix matrix(int type, int rows, int cols, int experts) {
        q3xk_matrix w{};
        size_t bytes = 0;
        if (q3xk_matrix_layout(type, rows, cols, experts, &w, &bytes) != Q3XK_OK) {
            status = Q3XK_EINVAL;
            return w;
        }
        w.data = carve(bytes);
        return w;
    }
    // Rows [row0, row0 + rows) of expert `e` of w, as a matrix of its own.
    static q3xk_matrix view(const q3xk_matrix& w, int e, int row0, int rows) {
        q3xk_matrix v = w;
        v.data = static_cast<uint8_t*>(w.data) + (size_t)e * w.expert_stride + (size_t)row0 * w.row_stride;
        v.rows = rows;
        v.experts = 1;
        v.expert_stride = (int64_t)rows * w.row_stride;
        return v;
    }
    // Repack `experts` consecutive packed matrices of the file into dst.
    void upload(const q3xk_matrix& dst, const uint8_t* src, int experts) {
        if (pass == 0 || status != Q3XK_OK) return;
        size_t bytes = 0;
        if (dst.type == Q3XK_BF16)
            bytes = (size_t)dst.rows * dst.cols * 2 * experts;
        else if (q3xk_quantized_bytes(dst.type, dst.rows, dst.cols, &bytes) == Q3XK_OK)
            bytes *= experts;
        if (bytes > staging_bytes) {
            status = Q3XK_EINVAL;
            return;
        }
        q3xk_matrix d = dst;
        d.experts = experts;
        if (!h2d(staging, src, bytes)) {
            status = Q3XK_ECUDA;
            return;
        }
        const int st = q3xk_repack(&d, staging, stream);
        if (st != Q3XK_OK) status = st;
    }
    // Packed [gate | up] rows (src_rows of them, counted from row_offset) into
    // dst with the SwiGLU row interleave (repack_swiglu).
    void upload_swiglu(const q3xk_matrix& dst, const uint8_t* src, int64_t src_rows, int half, int row_offset) {
        if (pass == 0 || status != Q3XK_OK) return;
        size_t bytes = 0;
        if (dst.type == Q3XK_BF16)
            bytes = (size_t)src_rows * dst.cols * 2;
        else if (q3xk_quantized_bytes(dst.type, 1, dst.cols, &bytes) == Q3XK_OK)
            bytes *= (size_t)src_rows;
        if (bytes > staging_bytes) {
            status = Q3XK_EINVAL;
            return;
        }
        if (!h2d(staging, src, bytes)) {
            status = Q3XK_ECUDA;
            return;
        }
        const int st = repack_swiglu(&dst, staging, src_rows, half, row_offset, stream);
        if (st != Q3XK_OK) status = st;
    }
    void need_staging(int type, int rows, int cols) {
        size_t b = 0;
        if (type == Q3XK_BF16)
            b = (size_t)rows * cols * 2;
        else
            q3xk_quantized_bytes(type, rows, cols, &b);
        if (b > staging_bytes) staging_bytes = b;
    }
    // FP32 device vector from n values of the file: BF16 (plus `add`) or FP32.
    float* vec(const uint8_t* src, int n, bool bf16, float add) {
        float* d = reinterpret_cast<float*>(carve((size_t)n * 4));
        if (pass == 0 || status != Q3XK_OK || !src) return d;
        host.resize(n);
        for (int i = 0; i < n; ++i) {
            if (bf16) {
                uint16_t b;
                std::memcpy(&b, src + 2 * (size_t)i, 2);
                host[i] = add + bf16_to_float(b);
            } else {
                std::memcpy(&host[i], src + 4 * (size_t)i, 4);
            }
        }
        // synchronous: the host vector is reused
        if (cudaMemcpy(d, host.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) status = Q3XK_ECUDA;
        return d;
    }

    // Columns [c0, c0 + cn) of a packed rows x K matrix (row-parallel shard):
    // gathered row by row on the host, then repacked into dst.
    void upload_cols(const q3xk_matrix& dst, const uint8_t* src, int rows, int K, int c0, int cn) {
        if (pass == 0 || status != Q3XK_OK || !src) return;
        const size_t full = row_bytes(dst.type, K), rb = row_bytes(dst.type, cn), off = row_bytes(dst.type, c0);
        if ((size_t)rows * rb > staging_bytes) {
            status = Q3XK_EINVAL;
            return;
        }
        gather.resize((size_t)rows * rb);
        for (int r = 0; r < rows; ++r) std::memcpy(gather.data() + (size_t)r * rb, src + (size_t)r * full + off, rb);
        if (!h2d(staging, gather.data(), gather.size())) {
            status = Q3XK_ECUDA;
            return;
        }
        const int st = q3xk_repack(&dst, staging, stream);
        if (st != Q3XK_OK) status = st;
    }
    // FP32 device vector of the listed row ranges (each `per` values wide) of
    // a BF16 file tensor.
    float* vec_rows(const uint8_t* src, const int (*ranges)[2], int nranges, int per) {
        int n = 0;
        for (int i = 0; i < nranges; ++i) n += ranges[i][1] * per;
        float* d = reinterpret_cast<float*>(carve((size_t)n * 4));
        if (pass == 0 || status != Q3XK_OK || !src) return d;
        host.resize(n);
        int k = 0;
        for (int i = 0; i < nranges; ++i)
            for (int r = 0; r < ranges[i][1] * per; ++r) {
                uint16_t b;
                std::memcpy(&b, src + 2 * ((size_t)ranges[i][0] * per + r), 2);
                host[k++] = bf16_to_float(b);
            }
        if (cudaMemcpy(d, host.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) status = Q3XK_ECUDA;
        return d;
    }

    // One walk over the file (engine.cpp:488-557), keeping this rank's share.
    // Returns the cursor error.
    const char* walk() {
        const Shard& sh = m.shard;
        const Config& L = sh.lc;
        const int type = c.matrix_type;
        const int AS = c.AH * c.AD, KVW = c.KVH * c.AD, DO = c.VH * c.VD, DQKV = 2 * c.KH * c.KD + DO;
        const int ASl = L.AH * L.AD, KVWl = L.KVH * L.AD, DOl = L.VH * L.VD, DQKVl = 2 * L.KH * L.KD + DOl;
        const int E = c.experts;
        Cursor cur{m.file, m.file_size, kHeaderSize};
        auto packed = [&](int t, int rows, int cols) -> const uint8_t* {
            size_t b = 0;
            if (t == Q3XK_BF16)
                b = (size_t)rows * cols * 2;
            else if (q3xk_quantized_bytes(t, rows, cols, &b) != Q3XK_OK && !cur.error)
                cur.error = "invalid quantized matrix layout";
            if (pass == 0) need_staging(t, rows, cols);
            return cur.take(b);
        };
        // row r0 of a packed matrix with `cols` columns (nullptr stays nullptr)
        auto at_row = [&](const uint8_t* p, int cols, int r0) -> const uint8_t* {
            return p ? p + (size_t)r0 * row_bytes(type, cols) : nullptr;
        };
        m.embedding = matrix(type, c.V, c.H, 1);
        upload(m.embedding, packed(type, c.V, c.H), 1);
        if (c.tied) {
            m.lm_head = view(m.embedding, 0, sh.v0, L.V);
        } else {
            m.lm_head = matrix(type, L.V, c.H, 1);
            upload(m.lm_head, at_row(packed(type, c.V, c.H), c.H, sh.v0), 1);
        }
        m.final_norm = vec(cur.take((size_t)c.H * 2), c.H, true, 1.0f);
        m.layer.assign(c.N, Layer{});
        for (int i = 0; i < c.N; ++i) {
            Layer& l = m.layer[i];
            l.delta = is_delta(c, i);
            l.in_norm = vec(cur.take((size_t)c.H * 2), c.H, true, 1.0f);
            if (l.delta) {
                l.in_proj = matrix(type, DQKVl + DOl + 2 * L.VH, c.H, 1);
                const uint8_t* qkv = packed(type, DQKV, c.H);
                upload(view(l.in_proj, 0, 0, L.KH * c.KD), at_row(qkv, c.H, sh.kh0 * c.KD), 1);
                upload(view(l.in_proj, 0, L.KH * c.KD, L.KH * c.KD), at_row(qkv, c.H, c.KH * c.KD + sh.kh0 * c.KD), 1);
                upload(view(l.in_proj, 0, 2 * L.KH * c.KD, DOl), at_row(qkv, c.H, 2 * c.KH * c.KD + sh.vh0 * c.VD), 1);
                upload(view(l.in_proj, 0, DQKVl, DOl), at_row(packed(type, DO, c.H), c.H, sh.vh0 * c.VD), 1);
                upload(view(l.in_proj, 0, DQKVl + DOl, L.VH), at_row(packed(type, c.VH, c.H), c.H, sh.vh0), 1);
                upload(view(l.in_proj, 0, DQKVl + DOl + L.VH, L.VH), at_row(packed(type, c.VH, c.H), c.H, sh.vh0),
                       1);
                const int ranges[3][2] = {{sh.kh0 * c.KD, L.KH * c.KD},
                                          {c.KH * c.KD + sh.kh0 * c.KD, L.KH * c.KD},
                                          {2 * c.KH * c.KD + sh.vh0 * c.VD, DOl}};
                l.conv = vec_rows(cur.take((size_t)DQKV * c.CK * 2), ranges, 3, c.CK);
                const uint8_t* alog = cur.take((size_t)c.VH * 4);
                l.alog = vec(alog ? alog + (size_t)sh.vh0 * 4 : nullptr, L.VH, false, 0.0f);
                const uint8_t* dt = cur.take((size_t)c.VH * 2);
                l.dt = vec(dt ? dt + (size_t)sh.vh0 * 2 : nullptr, L.VH, true, 0.0f);
                l.dnorm = vec(cur.take((size_t)c.VD * 4), c.VD, false, 0.0f);
                l.out = matrix(type, c.H, DOl, 1);
                upload_cols(l.out, packed(type, c.H, DO), c.H, DO, sh.vh0 * c.VD, DOl);
            } else {
                l.in_proj = matrix(type, 2 * ASl + 2 * KVWl, c.H, 1);
                upload(view(l.in_proj, 0, 0, 2 * ASl), at_row(packed(type, 2 * AS, c.H), c.H, sh.ah0 * 2 * c.AD), 1);
                upload(view(l.in_proj, 0, 2 * ASl, KVWl), at_row(packed(type, KVW, c.H), c.H, sh.kv0 * c.AD), 1);
                upload(view(l.in_proj, 0, 2 * ASl + KVWl, KVWl), at_row(packed(type, KVW, c.H), c.H, sh.kv0 * c.AD),
                       1);
                l.qn1 = vec(cur.take((size_t)c.AD * 2), c.AD, true, 1.0f);
                l.kn1 = vec(cur.take((size_t)c.AD * 2), c.AD, true, 1.0f);
                l.out = matrix(type, c.H, ASl, 1);
                upload_cols(l.out, packed(type, c.H, AS), c.H, AS, sh.ah0 * c.AD, ASl);
            }
            l.post_norm = vec(cur.take((size_t)c.H * 2), c.H, true, 1.0f);
            if (E) {
                // router: all experts; pools: this rank's experts [e0, e0 + El), shared expert at El
                const int El = sh.el;
                l.router = matrix(Q3XK_BF16, E + 1, c.H, 1);
                upload(view(l.router, 0, 0, E), packed(Q3XK_BF16, E, c.H), 1);
                l.gate_up = matrix(type, 2 * c.I, c.H, El + 1);
                upload_swiglu(l.gate_up, at_row(packed(type, E * 2 * c.I, c.H), c.H, sh.e0 * 2 * c.I),
                              (int64_t)El * 2 * c.I, c.I, 0);
                l.down = matrix(type, c.H, c.I, El + 1);
                upload(view(l.down, 0, 0, c.H), at_row(packed(type, E * c.H, c.I), c.I, sh.e0 * c.H), El);
                upload_swiglu(view(l.gate_up, El, 0, 2 * c.I), packed(type, c.shared_I, c.H), c.I, c.I, 0);
                upload_swiglu(view(l.gate_up, El, 0, 2 * c.I), packed(type, c.shared_I, c.H), c.I, c.I, c.I);
                upload(view(l.down, El, 0, c.H), packed(type, c.H, c.shared_I), 1);
                upload(view(l.router, 0, E, 1), packed(Q3XK_BF16, 1, c.H), 1);
            } else {
                l.gate_up = matrix(type, 2 * L.I, c.H, 1);
                upload_swiglu(l.gate_up, at_row(packed(type, c.I, c.H), c.H, sh.i0), L.I, L.I, 0);
                upload_swiglu(l.gate_up, at_row(packed(type, c.I, c.H), c.H, sh.i0), L.I, L.I, L.I);
                l.down = matrix(type, c.H, L.I, 1);
                upload_cols(l.down, packed(type, c.H, c.I), c.H, c.I, sh.i0, L.I);
            }
        }
        if (!cur.error && cur.pos != m.file_size) cur.error = "model.bin size does not match schema";
        return cur.error;
    }
};

}  // namespace
}  // namespace q3xk

namespace q3x_backend {

// engine.cpp:480-559: same checks and error strings, then the device upload.
bool Model::load(const char* path, int rank, int world, const char** error) {
    auto fail = [&](const char* message) {
        *error = message;
        return false;
    };
    fd = open(path, O_RDONLY);
    struct stat info {};
    if (fd < 0) return fail("cannot open model.bin");
    if (fstat(fd, &info) || info.st_size < (off_t)kHeaderSize) return fail("bad model.bin");
    file_size = (size_t)info.st_size;
    void* mapped = mmap(nullptr, file_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (mapped == MAP_FAILED) return fail("mmap model.bin failed");
    file = static_cast<const uint8_t*>(mapped);
    if (std::memcmp(file, "Q3XMODL\0", 8) != 0) return fail("wrong model.bin magic");
    config = config_for_id(header_field(file, 0));
    if (!config) return fail("unsupported Qwen model ID");
    if (!header_matches(file, *config)) return fail("Qwen model.bin header mismatch");
    const Config& c = *config;
    if (const char* e = make_shard(c, rank, world, shard)) return fail(e);
    if (c.experts && c.shared_I != c.I) return fail("unsupported MoE shape (shared_I != I)");
    if (c.experts && (c.experts > 512 || c.top_k > 8)) return fail("unsupported MoE shape");

    Loader ld{*this, c};
    ld.pass = 0;
    if (const char* e = ld.walk()) return fail(e);
    if (ld.status != Q3XK_OK) return fail("invalid quantized matrix layout");
    arena_bytes = ld.used;
    if (cudaGetDevice(&device) != cudaSuccess) return fail("no CUDA device");
    if (cudaMalloc(reinterpret_cast<void**>(&arena), arena_bytes) != cudaSuccess) {
        arena = nullptr;
        return fail("cannot allocate device memory for the model");
    }
    if (cudaMalloc(reinterpret_cast<void**>(&ld.staging), ld.staging_bytes) != cudaSuccess)
        return fail("cannot allocate the upload staging buffer");
    cudaStreamCreateWithFlags(&ld.stream, cudaStreamNonBlocking);
    madvise(mapped, file_size, MADV_SEQUENTIAL);
    ld.open_pinned();  // without pinned memory the copies stay pageable
    ld.pass = 1;
    ld.used = 0;
    const char* e = ld.walk();
    const cudaError_t se = cudaStreamSynchronize(ld.stream);
    ld.close_pinned();
    cudaStreamDestroy(ld.stream);
    cudaFree(ld.staging);
    if (e) return fail(e);
    if (ld.status != Q3XK_OK || se != cudaSuccess) return fail("model upload to the device failed");

    const Config& L = shard.lc;
    const int AS = L.AH * L.AD, KVW = L.KVH * L.AD, DO = L.VH * L.VD, DQKV = 2 * L.KH * L.KD + DO;
    P = DQKV + DO + 2 * L.VH;
    if (2 * AS + 2 * KVW > P) P = 2 * AS + 2 * KVW;
    if (!L.experts && 2 * L.I > P) P = 2 * L.I;
    mix = DO > AS ? DO : AS;
    if (L.I > mix) mix = L.I;
    maxcols = L.H > mix ? L.H : mix;
    return true;
}

}  // namespace q3x_backend

namespace q3xk {
namespace {

#define Q3XB_TRY(expr)                  \
    do {                                \
        const int q3xb_st = (expr);     \
        if (q3xb_st != Q3XK_OK) return q3xb_st; \
    } while (0)

// Up to this many tokens a matrix is applied as one ring GEMV per token: the
// GEMV streams 53.5 MB in 10.2 us, the few-token dequant-GEMM takes ~39 us at
// any T <= 16 (its TMA weight stream and split-K reduction set the floor).
constexpr int kGemvTokens = 3;

int mm(State& s, const q3xk_matrix& w, const float* X, int T, float* Y, int accumulate) {
    if (T == 1) return q3xk_gemv(&w, X, Y, accumulate, s.stream);
    // no BF16 GEMM / FP32-exact mode / few tokens: one GEMV per token
    if (w.type == Q3XK_BF16 || s.exact_prefill || T <= kGemvTokens) {
        for (int t = 0; t < T; ++t)
            Q3XB_TRY(q3xk_gemv(&w, X + (size_t)t * w.cols, Y + (size_t)t * w.rows, accumulate, s.stream));
        return Q3XK_OK;
    }
    return q3xk_gemm_ex(&w, X, T, Y, accumulate, s.gemm_precision, s.gemm_ws, s.gemm_ws_bytes, s.stream);
}

q3xk_xform rms_xf(const float* w1) {
    q3xk_xform xf{};
    xf.kind = Q3XK_XFORM_RMS;
    xf.w = w1;
    return xf;
}

// RMSNorm feeding a Q8_0 / Q4_0 decode GEMV runs in the GEMV's staging of x
// (the ring GEMV's one CTA per SM computes the statistics in its prologue):
// 9B-shaped decode measured 2.30 ms/token with the norms as their own
// kernels.  The register GEMV family (BF16 router, MoE row gathers) keeps
// the separate kernel: there every one of ~450 CTAs recomputed the
// statistics (2.88 -> 3.20 ms/token when fused).
#ifndef Q3XB_FUSE_RMS
#define Q3XB_FUSE_RMS 1
#endif
#ifndef Q3XB_FUSE_GATED
#define Q3XB_FUSE_GATED 0
#endif

// Input of a decode GEMV that reads RMSNorm(x) (engine.cpp:231-236): with
// `fuse` (and Q3XB_FUSE_RMS) the GEMV normalises x while staging it (*xf is
// set), else the norm runs as its own kernel into `normed` (returned).
int rms_input(State& s, const float* x, const float* w1, int n, q3xk_xform* xf, const float** in, bool fuse) {
    if (Q3XB_FUSE_RMS && fuse) {
        *xf = rms_xf(w1);
        *in = x;
        return Q3XK_OK;
    }
    *xf = q3xk_xform{};
    *in = s.normed;
    return launch_rms(x, w1, n, 1, s.normed, s.stream);
}

// y[0..T*H) += the sum over ranks of s.partial[0..T*H) (row-parallel
// projections, expert-parallel MoE).  Decode: one-shot all-reduce over NVLink
// peer memory once the peers' buffers are open, else NCCL.
int allreduce_add(State& s, float* y, int T) {
    const int H = s.c->H;
    if (T == 1 && s.peer_ready)
        return tp_peer_allreduce_add(s.peer_bases, s.rank, s.world, H, s.peer_seq, s.partial, y, H, s.tp_err,
                                     s.peer_timeout_s, s.stream);
    return tp_allreduce_add(s.comm, s.partial, y, (int64_t)T * H, s.stream);
}

// MoE FFN of token t (engine.cpp:406-430): router logits (+ the shared-expert
// gate as one more row) from RMS(hidden_t), device top-k, gate|up rows of the
// selected experts with the weighted SwiGLU in their epilogue, then the down
// projections of all slots added to hidden_t.
//
// Expert parallelism: the slots whose expert lives on another rank get id -1
// (skipped by both GEMVs); this rank's slots are summed into s.partial, and
// the partial sums of all ranks are all-reduced into hidden_t.
int moe_token(State& s, const Config& c, const Layer& l, int t, int layer) {
    const cudaStream_t st = s.stream;
    const Shard& sh = s.model->shard;
    const int S = c.top_k + 1;  // routed slots + the shared expert
    float* h = s.hidden + (size_t)t * c.H;
    q3xk_xform xr{};
    const float* in = s.normed;
    // RMSNorm in the router GEMV's prologue, which also leaves the normalised
    // hidden state in s.normed for the expert GEMVs; else its own kernel.
    int rs = Q3XB_FUSE_RMS ? gemv_rms_out(&l.router, h, l.post_norm, s.rlogits, s.normed, st) : Q3XK_EUNSUPPORTED;
    if (rs == Q3XK_EUNSUPPORTED) {
        Q3XB_TRY(rms_input(s, h, l.post_norm, c.H, &xr, &in, false));
        rs = q3xk_gemv_ex(&l.router, in, s.rlogits, 0, &xr, st);
    }
    Q3XB_TRY(rs);
    Q3XB_TRY(router_topk(s.rlogits, c.experts, c.top_k, 1, sh.e0, sh.el, shared_slot(sh, layer), s.rids, s.rweights,
                         st));
    Q3XB_TRY(gemv_swiglu(&l.gate_up, in, s.hbuf, s.rids, S, s.rweights, &xr, st));
    if (!s.ep) return q3xk_expert_gemv_segments(&l.down, s.rids, S, s.hbuf, h, 1, st);
    Q3XB_TRY(q3xk_expert_gemv_segments(&l.down, s.rids, S, s.hbuf, s.partial, 0, st));
    return allreduce_add(s, h, 1);
}

// One decode token (T = 1): every elementwise step that feeds a GEMV is
// fused into that GEMV's staging of x (RMSNorm, DeltaNet gated RMS, SwiGLU);
// residual adds are the GEMVs' accumulate.
// out = W x for a row-parallel projection: y += W x on one GPU; with
// tensor parallelism the rank's partial sum is all-reduced into y.
int row_parallel(State& s, const q3xk_matrix& w, const float* x, int T, float* y) {
    if (!s.tp) return mm(s, w, x, T, y, 1);
    Q3XB_TRY(mm(s, w, x, T, s.partial, 0));
    return allreduce_add(s, y, T);
}

int forward_token(Model& m, State& s, bool logits) {
    const Config& c = m.shard.lc;
    const cudaStream_t st = s.stream;
    const int DO = c.VH * c.VD, DQKV = 2 * c.KH * c.KD + DO, AS = c.AH * c.AD;
    Q3XB_TRY(launch_embed(m.embedding, s.tokens, 1, s.hidden, st));
    int di = 0, ai = 0;
    for (int i = 0; i < c.N; ++i) {
        const Layer& l = m.layer[i];
        const int P = l.in_proj.rows;
        q3xk_xform xin;
        const float* in = nullptr;
        Q3XB_TRY(rms_input(s, s.hidden, l.in_norm, c.H, &xin, &in, l.in_proj.type != Q3XK_BF16));
        Q3XB_TRY(q3xk_gemv_ex(&l.in_proj, in, s.proj, 0, &xin, st));
        if (l.delta) {
            const DeltaDims dd{c.KH, c.VH, c.KD, c.VD, DQKV, DQKV + DO, DQKV + DO + c.VH};
            // the conv runs inside the delta kernel (CK = 4); the gated RMS in the out
            // projection's staging of x (Q3XB_FUSE_GATED) or in the delta kernel
            const bool fuse_conv = c.CK == 4;
            if (!fuse_conv) Q3XB_TRY(launch_conv(s.proj, P, 1, DQKV, l.conv, c.CK, s.conv[di], st));
            Q3XB_TRY(launch_delta(s.proj, P, 1, dd, l.alog, l.dt, Q3XB_FUSE_GATED ? nullptr : l.dnorm, s.memory[di],
                                  s.mix, DO, st, fuse_conv ? l.conv : nullptr, fuse_conv ? s.conv[di] : nullptr,
                                  c.CK, s.group_count));
            q3xk_xform xg{};
            if (Q3XB_FUSE_GATED) {
                xg.kind = Q3XK_XFORM_GATED_RMS;
                xg.group = c.VD;
                xg.w = l.dnorm;
                xg.z = s.proj + DQKV;
            }
            if (!s.tp || xg.kind != Q3XK_XFORM_NONE)
                Q3XB_TRY(q3xk_gemv_ex(&l.out, s.mix, s.hidden, 1, &xg, st));
            else
                Q3XB_TRY(row_parallel(s, l.out, s.mix, 1, s.hidden));
            ++di;
        } else {
            const AttnDims ad{c.AH, c.KVH, c.AD, c.RD};
            Q3XB_TRY(launch_attention(s.proj, P, 1, ad, l.qn1, l.kn1, s.pos, s.kcache[ai], s.vcache[ai], s.capacity,
                                      s.part, s.split_len, s.mix, AS, st));
            Q3XB_TRY(row_parallel(s, l.out, s.mix, 1, s.hidden));
            ++ai;
        }
        if (c.experts) {
            Q3XB_TRY(moe_token(s, c, l, 0, i));
        } else {
            q3xk_xform xpost;
            const float* pin = nullptr;
            Q3XB_TRY(rms_input(s, s.hidden, l.post_norm, c.H, &xpost, &pin, l.gate_up.type != Q3XK_BF16));
            Q3XB_TRY(gemv_swiglu(&l.gate_up, pin, s.mix, nullptr, 0, nullptr, &xpost, st));
            Q3XB_TRY(row_parallel(s, l.down, s.mix, 1, s.hidden));
        }
    }
    if (logits) {
        q3xk_xform xf;
        const float* fin = nullptr;
        Q3XB_TRY(rms_input(s, s.hidden, m.final_norm, c.H, &xf, &fin, m.lm_head.type != Q3XK_BF16));
        Q3XB_TRY(q3xk_gemv_ex(&m.lm_head, fin, s.logits, 0, &xf, st));
    }
    return launch_advance(s.pos, 1, st);
}

// One pass over T <= chunk tokens already in s.tokens (engine.cpp:431-458).
#ifndef Q3XB_FUSED_DECODE
#define Q3XB_FUSED_DECODE 1
#endif

int forward_chunk(Model& m, State& s, int T, bool logits) {
    if (Q3XB_FUSED_DECODE && T == 1 && !s.exact_prefill) return forward_token(m, s, logits);
    const Config& c = m.shard.lc;
    const cudaStream_t st = s.stream;
    const int H = c.H, DO = c.VH * c.VD, DQKV = 2 * c.KH * c.KD + DO, AS = c.AH * c.AD;
    Q3XB_TRY(launch_embed(m.embedding, s.tokens, T, s.hidden, st));
    int di = 0, ai = 0;
    for (int i = 0; i < c.N; ++i) {
        const Layer& l = m.layer[i];
        Q3XB_TRY(launch_rms(s.hidden, l.in_norm, H, T, s.normed, st));
        const int P = l.in_proj.rows;
        Q3XB_TRY(mm(s, l.in_proj, s.normed, T, s.proj, 0));
        if (l.delta) {
            const DeltaDims dd{c.KH, c.VH, c.KD, c.VD, DQKV, DQKV + DO, DQKV + DO + c.VH};
            if (c.CK == 4) {
                Q3XB_TRY(launch_conv_prefill(s.proj, P, T, DQKV, l.conv, c.CK, s.conv[di], s.qkv, st));
                Q3XB_TRY(launch_delta_chunked(s.qkv, DQKV, s.proj, P, T, dd, l.alog, l.dt, l.dnorm, s.memory[di],
                                              s.mix, DO, s.delta_work, st));
            } else {
                Q3XB_TRY(launch_conv(s.proj, P, T, DQKV, l.conv, c.CK, s.conv[di], st));
                Q3XB_TRY(launch_delta_chunked(s.proj, P, s.proj, P, T, dd, l.alog, l.dt, l.dnorm, s.memory[di],
                                              s.mix, DO, s.delta_work, st));
            }
            Q3XB_TRY(row_parallel(s, l.out, s.mix, T, s.hidden));
            ++di;
        } else {
            const AttnDims ad{c.AH, c.KVH, c.AD, c.RD};
            Q3XB_TRY(launch_attention(s.proj, P, T, ad, l.qn1, l.kn1, s.pos, s.kcache[ai], s.vcache[ai], s.capacity,
                                      s.part, s.split_len, s.mix, AS, st));
            Q3XB_TRY(row_parallel(s, l.out, s.mix, T, s.hidden));
            ++ai;
        }
        if (c.experts && !s.exact_prefill) {
            // grouped expert GEMMs on tcgen05 for the whole pass
            Q3XB_TRY(launch_rms(s.hidden, l.post_norm, H, T, s.normed, st));
            MoePrefillArgs a = s.moe;
            a.router = &l.router;
            a.gate_up = &l.gate_up;
            a.down = &l.down;
            a.experts = c.experts;
            a.top_k = c.top_k;
            a.T = T;
            a.e0 = m.shard.e0;
            a.local = m.shard.el;
            a.shared_id = shared_slot(m.shard, i);
            a.x = s.normed;
            a.hidden = s.ep ? s.partial : s.hidden;
            a.accumulate = s.ep ? 0 : 1;
            a.split = s.gemm_precision == Q3XK_GEMM_SPLIT;
            Q3XB_TRY(moe_prefill(a, st));
            if (s.ep) Q3XB_TRY(allreduce_add(s, s.hidden, T));
        } else if (c.experts) {
            for (int t = 0; t < T; ++t) Q3XB_TRY(moe_token(s, c, l, t, i));
        } else {
            Q3XB_TRY(launch_rms(s.hidden, l.post_norm, H, T, s.normed, st));
            Q3XB_TRY(mm(s, l.gate_up, s.normed, T, s.proj, 0));
            Q3XB_TRY(launch_ffn_swiglu(s.proj, 2 * c.I, T, c.I, s.mix, st));
            Q3XB_TRY(row_parallel(s, l.down, s.mix, T, s.hidden));
        }
    }
    if (logits) {
        const q3xk_xform xf = rms_xf(m.final_norm);
        Q3XB_TRY(q3xk_gemv_ex(&m.lm_head, s.hidden + (size_t)(T - 1) * H, s.logits, 0, &xf, st));
    }
    return launch_advance(s.pos, T, st);
}

// One decode step of n independent sequences (batched decode): sequence b
// is states[b], fed tokens[b].  Every matrix is read once for all n tokens
// (the dequant-GEMM over T = n, few-token tiles with split-K); the
// recurrent and attention steps run per sequence on its own state (DeltaNet
// memory and conv history, KV cache, position); MoE layers route all n
// tokens together through the grouped expert GEMMs.  Work buffers are the
// lead state's (states[0]), whose stream runs the step; the other states'
// streams are joined before and after with events.  Equivalent to
// state_forward(states[b], &tokens[b], 1, true) for every b, up to the
// rounding of the split-precision GEMM (FP32-grade) against the GEMV.
int forward_batch(Model& m, State** states, int n) {
    State& L = *states[0];
    const Config& c = m.shard.lc;
    const cudaStream_t st = L.stream;
    const int H = c.H, DO = c.VH * c.VD, DQKV = 2 * c.KH * c.KD + DO, AS = c.AH * c.AD;
    Q3XB_TRY(launch_embed(m.embedding, L.tokens, n, L.hidden, st));
    int di = 0, ai = 0;
    for (int i = 0; i < c.N; ++i) {
        const Layer& l = m.layer[i];
        Q3XB_TRY(launch_rms(L.hidden, l.in_norm, H, n, L.normed, st));
        const int P = l.in_proj.rows;
        Q3XB_TRY(mm(L, l.in_proj, L.normed, n, L.proj, 0));
        if (l.delta) {
            const DeltaDims dd{c.KH, c.VH, c.KD, c.VD, DQKV, DQKV + DO, DQKV + DO + c.VH};
            for (int b = 0; b < n; ++b) {
                State& s = *states[b];
                float* pb = L.proj + (size_t)b * P;
                if (c.CK == 4) {
                    Q3XB_TRY(launch_delta(pb, P, 1, dd, l.alog, l.dt, l.dnorm, s.memory[di], L.mix + (size_t)b * DO, DO,
                                          st, l.conv, s.conv[di], c.CK, s.group_count));
                } else {
                    Q3XB_TRY(launch_conv(pb, P, 1, DQKV, l.conv, c.CK, s.conv[di], st));
                    Q3XB_TRY(launch_delta(pb, P, 1, dd, l.alog, l.dt, l.dnorm, s.memory[di], L.mix + (size_t)b * DO,
                                          DO, st));
                }
            }
            ++di;
        } else {
            const AttnDims ad{c.AH, c.KVH, c.AD, c.RD};
            for (int b = 0; b < n; ++b) {
                State& s = *states[b];
                Q3XB_TRY(launch_attention(L.proj + (size_t)b * P, P, 1, ad, l.qn1, l.kn1, s.pos, s.kcache[ai],
                                          s.vcache[ai], s.capacity, s.part, s.split_len, L.mix + (size_t)b * AS, AS,
                                          st));
            }
            ++ai;
        }
        // the n mixer outputs are dense rows of the out projection's width
        Q3XB_TRY(mm(L, l.out, L.mix, n, L.hidden, 1));
        Q3XB_TRY(launch_rms(L.hidden, l.post_norm, H, n, L.normed, st));
        if (c.experts) {
            MoePrefillArgs a = L.moe;
            a.router = &l.router;
            a.gate_up = &l.gate_up;
            a.down = &l.down;
            a.experts = c.experts;
            a.top_k = c.top_k;
            a.T = n;
            a.e0 = m.shard.e0;
            a.local = m.shard.el;
            a.shared_id = shared_slot(m.shard, i);
            a.x = L.normed;
            a.hidden = L.hidden;
            a.accumulate = 1;
            a.split = L.gemm_precision == Q3XK_GEMM_SPLIT;
            Q3XB_TRY(moe_prefill(a, st));
        } else {
            Q3XB_TRY(mm(L, l.gate_up, L.normed, n, L.proj, 0));
            Q3XB_TRY(launch_ffn_swiglu(L.proj, 2 * c.I, n, c.I, L.mix, st));
            Q3XB_TRY(mm(L, l.down, L.mix, n, L.hidden, 1));
        }
    }
    Q3XB_TRY(launch_rms(L.hidden, m.final_norm, H, n, L.normed, st));
    Q3XB_TRY(mm(L, m.lm_head, L.normed, n, L.batch_logits, 0));
    for (int b = 0; b < n; ++b) {
        State& s = *states[b];
        if (cudaMemcpyAsync(s.logits, L.batch_logits + (size_t)b * c.V, (size_t)c.V * 4, cudaMemcpyDeviceToDevice,
                            st) != cudaSuccess)
            return Q3XK_ECUDA;
        Q3XB_TRY(launch_advance(s.pos, 1, st));
    }
    return Q3XK_OK;
}

int capture_decode_graph(Model& m, State& s) {
    if (cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeRelaxed) != cudaSuccess) return Q3XK_ECUDA;
    const int st = forward_chunk(m, s, 1, true);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s.stream, &g);
    if (st != Q3XK_OK || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return st != Q3XK_OK ? st : Q3XK_ECUDA;
    }
    if (cudaGraphInstantiate(&s.graph_exec, g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        s.graph_exec = nullptr;
        return Q3XK_ECUDA;
    }
    s.graph = g;
    return Q3XK_OK;
}

void set_error(char* err, size_t errlen, const char* fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

State* create_state(Model* model, int context, const char* nccl_id, char* err, size_t errlen) {
    if (!model || !model->config || context <= 0 || context > kMaxContext) {
        set_error(err, errlen, "state_create model=%p context=%d", static_cast<void*>(model), context);
        return nullptr;
    }
    if (cudaSetDevice(model->device) != cudaSuccess) {
        set_error(err, errlen, "cannot select the model's device");
        return nullptr;
    }
    std::unique_ptr<State> s(new (std::nothrow) State());
    if (!s) return nullptr;
    static std::atomic<uint64_t> next_uid{1};
    s->uid = next_uid.fetch_add(1);
    const Config& c = model->shard.lc;  // this rank's dims
    s->model = model;
    s->c = &c;
    s->device = model->device;
    s->capacity = context;
    s->rank = model->shard.rank;
    s->world = model->shard.world;
    s->ep = model->shard.ep;
    s->tp = s->world > 1 && !s->ep;
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_error(err, errlen, "cannot create a CUDA stream");
        return nullptr;
    }
    const int DO = c.VH * c.VD, DQKV = 2 * c.KH * c.KD + DO;
    const size_t conv = (size_t)DQKV * (c.CK - 1), memory = (size_t)c.VH * c.KD * c.VD;
    const size_t cache = (size_t)context * c.KVH * c.AD;
    const int attn_layers = c.N / c.AI, delta_layers = c.N - attn_layers;
    const int chunk = context < kChunk ? context : kChunk;
    s->chunk = s->chunk_capacity = chunk;
    s->recurrent_floats = (size_t)delta_layers * (conv + memory);
    s->split_len = 128;  // decode attention: 128-key splits (attn_decode_kernel)
    const int nsplit = (context + s->split_len - 1) / s->split_len;
    bool ok = s->alloc(&s->recurrent, s->recurrent_floats) && s->alloc(&s->checkpoint_recurrent, s->recurrent_floats) &&
              s->alloc(&s->kv, (size_t)attn_layers * 2 * cache) && s->alloc(&s->logits, c.V) &&
              s->alloc(&s->checkpoint_logits, c.V) && s->alloc(&s->pos, 1) && s->alloc(&s->tokens, chunk) &&
              s->alloc(&s->argmax_out, 1) && s->alloc(&s->group_count, c.KH > 0 ? c.KH : 1) &&
              s->alloc(&s->hidden, (size_t)chunk * c.H) &&
              s->alloc(&s->normed, (size_t)chunk * c.H) && s->alloc(&s->proj, (size_t)chunk * model->P) &&
              s->alloc(&s->mix, (size_t)chunk * model->mix) &&
              s->alloc(&s->part, (size_t)c.AH * nsplit * (c.AD + 2));  // decode attention partials
    if (ok && c.experts) {
        const int S = c.top_k + 1;
        ok = s->alloc(&s->rlogits, c.experts + 1) && s->alloc(&s->rweights, S) && s->alloc(&s->rids, S) &&
             s->alloc(&s->hbuf, (size_t)S * c.I);
    }
    if (ok && c.experts && chunk > 1) {
        const int S = c.top_k + 1, E1 = c.experts + 1;
        const size_t P = (size_t)chunk * S;
        MoePrefillArgs& a = s->moe;
        ok = s->alloc(&a.logits, (size_t)chunk * E1) && s->alloc(&a.ids, P) && s->alloc(&a.weights, P) &&
             s->alloc(&a.xoff, E1 + 1) && s->alloc(&a.tile_gu, E1 + 1) && s->alloc(&a.tile_dn, E1 + 1) &&
             s->alloc(&a.pos, P) && s->alloc(&a.pair_token, P) && s->alloc(&a.pair_weight, P) &&
             s->alloc(&a.x16, 2 * (size_t)chunk * c.H) && s->alloc(&a.scale, chunk) &&
             s->alloc(&a.x16g, 2 * P * c.H) && s->alloc(&a.scale_g, P) && s->alloc(&a.gu, P * 2 * c.I) &&
             s->alloc(&a.h16, 2 * P * c.I) &&
             s->alloc(&a.scale_h, P) && s->alloc(&a.out, P * c.H);
    }
    if (ok && s->world > 1) {
        uint8_t* pb = nullptr;
        ok = s->alloc(&s->partial, (size_t)chunk * c.H) && s->alloc(&s->full_logits, model->config->V) &&
             s->alloc(&s->best, 2 * (size_t)s->world + 2) && s->alloc(&pb, tp_peer_buffer_bytes(c.H)) &&
             s->alloc(&s->peer_seq, 1) && s->alloc(&s->tp_err, 1);
        s->peer_buf = pb;
        if (ok)
            ok = cudaMemset(pb, 0, tp_peer_buffer_bytes(c.H)) == cudaSuccess &&
                 cudaMemset(s->peer_seq, 0, 4) == cudaSuccess && cudaMemset(s->tp_err, 0, 4) == cudaSuccess &&
                 cudaHostAlloc(reinterpret_cast<void**>(&s->tp_err_host), sizeof(int), cudaHostAllocDefault) ==
                     cudaSuccess;
        if (ok) *s->tp_err_host = 0;
    }
    if (ok && chunk > 1 && delta_layers > 0)
        ok = s->alloc(&s->delta_work, delta_chunked_workspace_bytes(chunk, c.VH) / 4) &&
             s->alloc(&s->qkv, (size_t)chunk * DQKV);
    if (ok) {
        q3xk_argmax_workspace_bytes(&s->argmax_ws_bytes);
        uint8_t* ws = nullptr;
        ok = s->alloc(&ws, s->argmax_ws_bytes);
        s->argmax_ws = ws;
    }
    if (ok && chunk > 1) {
        q3xk_gemm_workspace_bytes(chunk, model->maxcols, &s->gemm_ws_bytes);
        uint8_t* ws = nullptr;
        ok = s->alloc(&ws, s->gemm_ws_bytes);
        s->gemm_ws = ws;
    }
    if (!ok) {
        set_error(err, errlen, "State allocation failed model=%s context=%d", c.name, context);
        return nullptr;
    }
    if (s->world > 1) {
        if (!nccl_id) {
            set_error(err, errlen, "tensor-parallel state needs a communicator id");
            return nullptr;
        }
        if (const char* why = nccl_load()) {
            set_error(err, errlen, "%s", why);
            return nullptr;
        }
        if (tp_comm_create(nccl_id, s->rank, s->world, &s->comm) != Q3XK_OK) {
            set_error(err, errlen, "NCCL communicator creation failed (%s)", tp_last_error());
            return nullptr;
        }
    }
    float* r = s->recurrent;
    float* kv = s->kv;
    for (int i = 0; i < c.N; ++i) {
        if (is_delta(c, i)) {
            s->conv.push_back(r);
            r += conv;
            s->memory.push_back(r);
            r += memory;
        } else {
            s->kcache.push_back(kv);
            kv += cache;
            s->vcache.push_back(kv);
            kv += cache;
        }
    }
    // engine.cpp:156-159 reset; logits start at zero as well
    if (cudaMemsetAsync(s->recurrent, 0, s->recurrent_floats * 4, s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->pos, 0, 4, s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->group_count, 0, sizeof(int) * (c.KH > 0 ? c.KH : 1), s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->logits, 0, (size_t)c.V * 4, s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->checkpoint_logits, 0, (size_t)c.V * 4, s->stream) != cudaSuccess ||
        cudaStreamSynchronize(s->stream) != cudaSuccess) {
        set_error(err, errlen, "State initialisation failed");
        return nullptr;
    }
    return s.release();
}

// Status of the peer all-reduces so far, as last copied to the host: a peer
// that never published within the bound leaves this State out of step with
// its peers for good (Q3XK_ETIMEOUT from every later call).  Exact once the
// state's stream has been synchronised.
int peer_status(const State* s) {
    return s->tp_err_host && *(volatile int*)s->tp_err_host ? Q3XK_ETIMEOUT : Q3XK_OK;
}

int state_forward_impl(Model* m, State* s, const int* tokens, int count, bool logits) {
    if (!m || !s || !tokens || count <= 0 || s->model != m) return Q3XK_EINVAL;
    Q3XB_TRY(peer_status(s));
    const Config& c = *m->config;
    for (int i = 0; i < count; ++i)
        if (tokens[i] < 0 || tokens[i] >= c.V) return Q3XK_EINVAL;
    if (count > s->capacity - s->position) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    const int chunk = s->chunk;
    for (int done = 0; done < count;) {
        const int T = count - done < chunk ? count - done : chunk;
        const bool last = done + T == count;
        if (cudaMemcpyAsync(s->tokens, tokens + done, (size_t)T * 4, cudaMemcpyHostToDevice, s->stream) !=
            cudaSuccess)
            return Q3XK_ECUDA;
        if (T == 1 && last && logits && s->use_graphs) {
            if (!s->graph_exec) Q3XB_TRY(capture_decode_graph(*m, *s));
            if (cudaGraphLaunch(s->graph_exec, s->stream) != cudaSuccess) return Q3XK_ECUDA;
        } else {
            Q3XB_TRY(forward_chunk(*m, *s, T, logits && last));
        }
        s->position += T;
        done += T;
    }
    if (s->tp_err_host &&
        cudaMemcpyAsync(s->tp_err_host, s->tp_err, 4, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
        return Q3XK_ECUDA;
    return Q3XK_OK;
}

// Checks and stream joins around forward_batch.
int state_forward_batch_impl(Model* m, State** states, const int* tokens, int n) {
    if (!m || !states || !tokens || n < 1 || n > kMaxBatch) return Q3XK_EINVAL;
    const Config& c = *m->config;
    for (int b = 0; b < n; ++b) {
        State* s = states[b];
        if (!s || s->model != m || tokens[b] < 0 || tokens[b] >= c.V || s->position + 1 > s->capacity)
            return Q3XK_EINVAL;
        for (int q = 0; q < b; ++q)
            if (states[q] == s) return Q3XK_EINVAL;  // a sequence appears once per step
        Q3XB_TRY(peer_status(s));
    }
    State& L = *states[0];
    if (L.world > 1) return Q3XK_EUNSUPPORTED;  // batched decode runs on one GPU
    if (n > L.chunk_capacity) return Q3XK_EINVAL;
    if (m->layer.empty() || c.V <= 0) return Q3XK_EINVAL;
    if (cudaSetDevice(L.device) != cudaSuccess) return Q3XK_ECUDA;
    if (!L.batch_logits && !L.alloc(&L.batch_logits, (size_t)kMaxBatch * c.V)) return Q3XK_ECUDA;
    // the other sequences' queued work comes first, their later work after the step
    for (int b = 1; b < n; ++b) {
        State& s = *states[b];
        if (!s.batch_event && cudaEventCreateWithFlags(&s.batch_event, cudaEventDisableTiming) != cudaSuccess)
            return Q3XK_ECUDA;
        if (cudaEventRecord(s.batch_event, s.stream) != cudaSuccess ||
            cudaStreamWaitEvent(L.stream, s.batch_event, 0) != cudaSuccess)
            return Q3XK_ECUDA;
    }
    if (cudaMemcpyAsync(L.tokens, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, L.stream) != cudaSuccess)
        return Q3XK_ECUDA;
    if (L.use_graphs) {
        // replay the step captured for exactly this list of States (positions
        // live on the device, so one capture serves every later step)
        std::vector<uint64_t> key(n);
        for (int b = 0; b < n; ++b) key[b] = states[b]->uid;
        if (!L.batch_exec || L.batch_key != key) {
            if (L.batch_exec) {
                cudaGraphExecDestroy(L.batch_exec);
                L.batch_exec = nullptr;
            }
            if (cudaStreamBeginCapture(L.stream, cudaStreamCaptureModeRelaxed) != cudaSuccess) return Q3XK_ECUDA;
            const int st = forward_batch(*m, states, n);
            cudaGraph_t g = nullptr;
            const cudaError_t e = cudaStreamEndCapture(L.stream, &g);
            if (st != Q3XK_OK || e != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                cudaGetLastError();
                return st != Q3XK_OK ? st : Q3XK_ECUDA;
            }
            const cudaError_t ie = cudaGraphInstantiate(&L.batch_exec, g, 0);
            cudaGraphDestroy(g);
            if (ie != cudaSuccess) {
                L.batch_exec = nullptr;
                return Q3XK_ECUDA;
            }
            L.batch_key = key;
        }
        if (cudaGraphLaunch(L.batch_exec, L.stream) != cudaSuccess) return Q3XK_ECUDA;
    } else {
        Q3XB_TRY(forward_batch(*m, states, n));
    }
    if (n > 1) {
        if (!L.batch_event && cudaEventCreateWithFlags(&L.batch_event, cudaEventDisableTiming) != cudaSuccess)
            return Q3XK_ECUDA;
        if (cudaEventRecord(L.batch_event, L.stream) != cudaSuccess) return Q3XK_ECUDA;
        for (int b = 1; b < n; ++b)
            if (cudaStreamWaitEvent(states[b]->stream, L.batch_event, 0) != cudaSuccess) return Q3XK_ECUDA;
    }
    for (int b = 0; b < n; ++b) states[b]->position += 1;
    return Q3XK_OK;
}

int checkpoint_copy(State* s, bool save) {
    if (!s) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    float* rd = save ? s->checkpoint_recurrent : s->recurrent;
    float* rs = save ? s->recurrent : s->checkpoint_recurrent;
    float* ld = save ? s->checkpoint_logits : s->logits;
    float* ls = save ? s->logits : s->checkpoint_logits;
    if (cudaMemcpyAsync(rd, rs, s->recurrent_floats * 4, cudaMemcpyDeviceToDevice, s->stream) != cudaSuccess ||
        cudaMemcpyAsync(ld, ls, (size_t)s->c->V * 4, cudaMemcpyDeviceToDevice, s->stream) != cudaSuccess)
        return Q3XK_ECUDA;
    if (save) {
        s->checkpoint_position = s->position;
    } else {
        // engine.cpp:591-600
        if (s->checkpoint_position < 0 || s->checkpoint_position > s->capacity) return Q3XK_EINVAL;
        s->position = s->checkpoint_position;
        if (cudaMemcpyAsync(s->pos, &s->position, 4, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
            return Q3XK_ECUDA;
        if (cudaStreamSynchronize(s->stream) != cudaSuccess) return Q3XK_ECUDA;  // &position is host memory
    }
    return Q3XK_OK;
}

int reset_impl(State* s) {
    if (!s) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    s->position = 0;
    if (cudaMemsetAsync(s->recurrent, 0, s->recurrent_floats * 4, s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->pos, 0, 4, s->stream) != cudaSuccess)
        return Q3XK_ECUDA;
    return Q3XK_OK;
}

int argmax_impl(const State* s, int* token) {
    if (!s || !token) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    Q3XB_TRY(q3xk_argmax(s->logits, s->c->V, s->argmax_out, s->argmax_ws, s->argmax_ws_bytes, s->stream));
    if (s->tp) {
        // every rank's (value, global index), gathered; the first maximum wins
        float* mine = s->best + 2 * s->world;
        Q3XB_TRY(tp_pack_best(s->logits, s->argmax_out, s->model->shard.v0, mine, s->stream));
        Q3XB_TRY(tp_allgather(s->comm, mine, s->best, 2, s->stream));
        std::vector<float> all(2 * (size_t)s->world);
        if (cudaMemcpyAsync(all.data(), s->best, all.size() * 4, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess ||
            cudaStreamSynchronize(s->stream) != cudaSuccess)
            return Q3XK_ECUDA;
        Q3XB_TRY(peer_status(s));
        int bi = 0;
        for (int r = 1; r < s->world; ++r)
            if (all[2 * r] > all[2 * bi] || (all[2 * r] == all[2 * bi] && all[2 * r + 1] < all[2 * bi + 1])) bi = r;
        *token = (int)all[2 * bi + 1];
        return Q3XK_OK;
    }
    if (cudaMemcpyAsync(token, s->argmax_out, 4, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess ||
        cudaStreamSynchronize(s->stream) != cudaSuccess)
        return Q3XK_ECUDA;
    return peer_status(s);
}

int copy_logits_impl(const State* s, float* out) {
    if (!s || !out) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    if (s->tp) {  // vocabulary shards in rank order
        Q3XB_TRY(tp_allgather(s->comm, s->logits, s->full_logits, s->c->V, s->stream));
        if (cudaMemcpyAsync(out, s->full_logits, (size_t)s->c->V * s->world * 4, cudaMemcpyDeviceToHost,
                            s->stream) != cudaSuccess ||
            cudaStreamSynchronize(s->stream) != cudaSuccess)
            return Q3XK_ECUDA;
        return peer_status(s);
    }
    if (cudaMemcpyAsync(out, s->logits, (size_t)s->c->V * 4, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess ||
        cudaStreamSynchronize(s->stream) != cudaSuccess)
        return Q3XK_ECUDA;
    return peer_status(s);
}

// Waits until the state's stream has drained; then the peer-wait status.
int drain(const State* s) {
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess) return Q3XK_ECUDA;
    return peer_status(s);
}

// The reference's Q3X_ASSERT: report, then abort (internal.h:70-80).
[[noreturn]] void fatal(const char* what, int status) {
    std::fprintf(stderr, "q3x_backend: %s failed: %s\n", what, q3xk_status_string(status));
    std::abort();
}

}  // namespace
}  // namespace q3xk

// ---- q3x_backend (C++) ------------------------------------------------------------

namespace q3x_backend {

Model* model_create_shard(const char* path, int rank, int world, char* err, size_t errlen) {
    std::unique_ptr<Model> model(new (std::nothrow) Model());
    const char* message = nullptr;
    if (!model || !path || !model->load(path, rank, world, &message)) {
        if (err && errlen) std::snprintf(err, errlen, "%s", message ? message : "allocation failed");
        return nullptr;
    }
    if (err && errlen) err[0] = '\0';
    return model.release();
}
Model* model_create(const char* path, char* err, size_t errlen) { return model_create_shard(path, 0, 1, err, errlen); }
void model_destroy(Model* model) { delete model; }

State* state_create(Model* model, int context_size) {
    char err[256];
    State* s = create_state(model, context_size, nullptr, err, sizeof err);
    if (!s) {
        std::fprintf(stderr, "q3x_backend: %s\n", err);
        std::abort();
    }
    return s;
}
void state_destroy(State* state) { delete state; }
void state_reset(State* state) {
    const int st = reset_impl(state);
    if (st != Q3XK_OK) fatal("state_reset", st);
}
// state_forward returns once the step's work is done, as the reference's CUDA
// backend does (arch/cuda/engine.cu:2307, a stream synchronize at the end), so
// callers that sequence or time calls by the wall clock (the runtime's
// --bench, its logs) see the same behaviour.  The C mirror (q3xb_*) stays
// stream-ordered; q3xb_state_synchronize waits there.
void state_forward(Model* model, State* state, const int* tokens, int count, bool compute_logits) {
    int st = state_forward_impl(model, state, tokens, count, compute_logits);
    if (st == Q3XK_OK) st = drain(state);
    if (st != Q3XK_OK) fatal("state_forward", st);
}
void state_checkpoint_save(State* state) {
    const int st = checkpoint_copy(state, true);
    if (st != Q3XK_OK) fatal("state_checkpoint_save", st);
}
void state_checkpoint_restore(State* state) {
    const int st = checkpoint_copy(state, false);
    if (st != Q3XK_OK) fatal("state_checkpoint_restore", st);
}
int state_argmax(const State* state) {
    if (!state) return -1;
    int token = -1;
    const int st = argmax_impl(state, &token);
    if (st != Q3XK_OK) fatal("state_argmax", st);
    return token;
}
void state_copy_logits(const State* state, float* output) {
    const int st = copy_logits_impl(state, output);
    if (st != Q3XK_OK) fatal("state_copy_logits", st);
}
void state_forward_batch(Model* model, State* const* states, const int* tokens, int count) {
    int st = state_forward_batch_impl(model, const_cast<State**>(states), tokens, count);
    for (int i = 0; st == Q3XK_OK && i < count; ++i) st = drain(states[i]);
    if (st != Q3XK_OK) fatal("state_forward_batch", st);
}
uint32_t model_id(const Model* model) { return model->config->id; }
int vocab_size() { return 248320; }
int max_context() { return kMaxContext; }
bool token_is_stop(int token) { return token == kEndOfText || token == kImEnd; }

}  // namespace q3x_backend

// ---- C ABI --------------------------------------------------------------------------

extern "C" {

q3xb_model* q3xb_model_create(const char* path, char* err, size_t errlen) {
    return reinterpret_cast<q3xb_model*>(q3x_backend::model_create(path, err, errlen));
}
void q3xb_model_destroy(q3xb_model* model) { delete reinterpret_cast<Model*>(model); }
uint32_t q3xb_model_id(const q3xb_model* model) {
    return model ? reinterpret_cast<const Model*>(model)->config->id : 0;
}
int q3xb_model_config(const q3xb_model* model, int* f) {
    if (!model || !f) return Q3XK_EINVAL;
    const Config& c = *reinterpret_cast<const Model*>(model)->config;
    const int v[21] = {(int)c.id, c.V,  c.H,  c.I,  c.N,  c.AI,      c.AH,  c.KVH,        c.AD,        c.RD, c.KH,
                       c.VH,      c.KD, c.VD, c.CK, kMaxContext, c.experts, c.top_k, c.shared_I, c.matrix_type,
                       (int)c.tied};
    std::memcpy(f, v, sizeof v);
    return Q3XK_OK;
}
size_t q3xb_model_device_bytes(const q3xb_model* model) {
    return model ? reinterpret_cast<const Model*>(model)->arena_bytes : 0;
}
q3xb_state* q3xb_state_create(q3xb_model* model, int context_size, char* err, size_t errlen) {
    return reinterpret_cast<q3xb_state*>(
        create_state(reinterpret_cast<Model*>(model), context_size, nullptr, err, errlen));
}
q3xb_model* q3xb_model_create_tp(const char* path, int rank, int world, char* err, size_t errlen) {
    return reinterpret_cast<q3xb_model*>(q3x_backend::model_create_shard(path, rank, world, err, errlen));
}
int q3xb_tp_unique_id(char* id) { return tp_unique_id(id); }
q3xb_state* q3xb_state_create_tp(q3xb_model* model, int context_size, const char* nccl_id, char* err,
                                 size_t errlen) {
    return reinterpret_cast<q3xb_state*>(
        create_state(reinterpret_cast<Model*>(model), context_size, nccl_id, err, errlen));
}
static void shard_fields(const Shard& sh, int* f) {
    const int v[16] = {sh.rank,   sh.world,  sh.kh0,   sh.vh0,    sh.ah0,  sh.kv0,  sh.i0, sh.v0,
                       sh.lc.KH, sh.lc.VH, sh.lc.AH, sh.lc.KVH, sh.lc.I, sh.lc.V, sh.e0, sh.el};
    std::memcpy(f, v, sizeof v);
}
int q3xb_state_ipc_handle(const q3xb_state* state, char* handle64) {
    const State* s = reinterpret_cast<const State*>(state);
    if (!s || !handle64 || s->world < 2 || !s->peer_buf) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, s->peer_buf) != cudaSuccess) return Q3XK_ECUDA;
    static_assert(sizeof(h) == 64, "IPC handle size");
    std::memcpy(handle64, &h, sizeof h);
    return Q3XK_OK;
}
int q3xb_state_ipc_open(q3xb_state* state, const char* handles) {
    State* s = reinterpret_cast<State*>(state);
    if (!s || !handles || s->world < 2 || s->world > 8 || s->peer_ready) return Q3XK_EINVAL;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    for (int r = 0; r < s->world; ++r) {
        if (r == s->rank) {
            s->peer_bases[r] = s->peer_buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handles + 64 * (size_t)r, sizeof h);
        if (cudaIpcOpenMemHandle(&s->peer_bases[r], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != s->rank && s->peer_bases[q]) cudaIpcCloseMemHandle(s->peer_bases[q]);
            return Q3XK_ECUDA;
        }
    }
    s->peer_ready = true;
    return Q3XK_OK;
}
int q3xb_state_set_peer_timeout(q3xb_state* state, double seconds) {
    State* s = reinterpret_cast<State*>(state);
    if (!s || !(seconds > 0.0) || seconds > 60.0) return Q3XK_EINVAL;
    if (s->graph_exec) return Q3XK_EUNSUPPORTED;  // the captured decode step keeps the bound it was made with
    s->peer_timeout_s = seconds;
    return Q3XK_OK;
}
int q3xb_state_tp_error(const q3xb_state* state, int* flags) {
    const State* s = reinterpret_cast<const State*>(state);
    if (!s || !flags) return Q3XK_EINVAL;
    *flags = 0;
    if (!s->tp_err) return Q3XK_OK;
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    return cudaMemcpy(flags, s->tp_err, 4, cudaMemcpyDeviceToHost) == cudaSuccess ? Q3XK_OK : Q3XK_ECUDA;
}
int q3xb_model_shard(const q3xb_model* model, int* fields16) {
    if (!model || !fields16) return Q3XK_EINVAL;
    shard_fields(reinterpret_cast<const Model*>(model)->shard, fields16);
    return Q3XK_OK;
}
int q3xb_tp_plan(uint32_t model_id, int rank, int world, int* fields16, char* err, size_t errlen) {
    const Config* c = config_for_id(model_id);
    if (!c || !fields16) {
        set_error(err, errlen, "unsupported Qwen model ID");
        return Q3XK_EINVAL;
    }
    Shard sh;
    if (const char* e = make_shard(*c, rank, world, sh)) {
        set_error(err, errlen, "%s", e);
        return Q3XK_EUNSUPPORTED;
    }
    shard_fields(sh, fields16);
    return Q3XK_OK;
}
void q3xb_state_destroy(q3xb_state* state) { delete reinterpret_cast<State*>(state); }
int q3xb_state_reset(q3xb_state* state) { return reset_impl(reinterpret_cast<State*>(state)); }
int q3xb_state_forward(q3xb_model* model, q3xb_state* state, const int* tokens, int count, int compute_logits) {
    return state_forward_impl(reinterpret_cast<Model*>(model), reinterpret_cast<State*>(state), tokens, count,
                              compute_logits != 0);
}
int q3xb_state_checkpoint_save(q3xb_state* state) { return checkpoint_copy(reinterpret_cast<State*>(state), true); }
int q3xb_state_forward_batch(q3xb_model* model, q3xb_state* const* states, const int* tokens, int count) {
    return state_forward_batch_impl(reinterpret_cast<Model*>(model),
                                    reinterpret_cast<State**>(const_cast<q3xb_state**>(states)), tokens, count);
}
int q3xb_state_checkpoint_restore(q3xb_state* state) {
    return checkpoint_copy(reinterpret_cast<State*>(state), false);
}
int q3xb_state_argmax(const q3xb_state* state, int* token) {
    return argmax_impl(reinterpret_cast<const State*>(state), token);
}
int q3xb_state_copy_logits(const q3xb_state* state, float* output) {
    return copy_logits_impl(reinterpret_cast<const State*>(state), output);
}
int q3xb_state_position(const q3xb_state* state) {
    return state ? reinterpret_cast<const State*>(state)->position : -1;
}
int q3xb_state_synchronize(const q3xb_state* state) {
    if (!state) return Q3XK_EINVAL;
    const State* s = reinterpret_cast<const State*>(state);
    if (cudaSetDevice(s->device) != cudaSuccess) return Q3XK_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess) return Q3XK_ECUDA;
    return peer_status(s);
}
void* q3xb_state_stream(const q3xb_state* state) {
    return state ? static_cast<void*>(reinterpret_cast<const State*>(state)->stream) : nullptr;
}
int q3xb_state_set_exact_prefill(q3xb_state* state, int enabled) {
    if (!state) return Q3XK_EINVAL;
    reinterpret_cast<State*>(state)->exact_prefill = enabled != 0;
    return Q3XK_OK;
}
int q3xb_state_set_prefill_precision(q3xb_state* state, int precision) {
    if (!state || (precision != Q3XK_GEMM_SPLIT && precision != Q3XK_GEMM_FP16)) return Q3XK_EINVAL;
    reinterpret_cast<State*>(state)->gemm_precision = precision;
    return Q3XK_OK;
}
int q3xb_state_set_prefill_chunk(q3xb_state* state, int tokens) {
    if (!state) return Q3XK_EINVAL;
    State* s = reinterpret_cast<State*>(state);
    if (tokens < 1 || tokens > s->chunk_capacity) return Q3XK_EINVAL;
    s->chunk = tokens;
    return Q3XK_OK;
}
int q3xb_state_set_graphs(q3xb_state* state, int enabled) {
    if (!state) return Q3XK_EINVAL;
    reinterpret_cast<State*>(state)->use_graphs = enabled != 0;
    return Q3XK_OK;
}

}  // extern "C"
