// tp.cu -- NCCL, loaded at run time, and the peer-memory all-reduce for the
// multi-GPU backend.
//
// Row-parallel projections (tensor parallelism: attention/DeltaNet out, FFN
// down) and the MoE layer (expert parallelism: the slots a rank runs) leave a
// partial [T][H] sum on every rank; tp_allreduce_add sums the partials with
// one ncclAllReduce on the state's stream (capturable in the decode graph) and
// adds the result into the replicated residual stream.
#include <dlfcn.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <nccl.h>

#include "tp.cuh"

namespace q3xk {
namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};
char g_last_error[160] = "";

NcclApi g_nccl;
std::mutex g_nccl_mutex;
const char* g_nccl_error = nullptr;
bool g_nccl_tried = false;

__global__ void add_kernel(float* __restrict__ hidden, const float* __restrict__ partial, int64_t n) {
    griddep_wait();
    griddep_launch_dependents();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        hidden[i] += partial[i];
}

__global__ void pack_best_kernel(const float* __restrict__ logits, const int* __restrict__ idx, int v0,
                                 float* __restrict__ out) {
    griddep_wait();
    const int i = *idx;
    out[0] = logits[i];
    out[1] = (float)(i + v0);  // exact: vocabulary indices < 2^24
}

// ---- one-shot all-reduce over NVLink peer memory (decode-sized vectors) ------
//
// Every rank owns a PeerBuf in its own HBM, mapped into the other ranks with
// CUDA IPC:  data[2][n_max] (this rank's partial, by phase)  flags[2][kMaxRanks]
// (flags[phase][r] = the sequence number rank r has published).  A call with
// sequence s (phase s & 1):
//   1. copy the local partial into data[phase] of the own buffer;
//   2. fence (system scope), then store s into flags[phase][rank] of every
//      peer's buffer;
//   3. wait until the own flags[phase][r] == s for every rank r -- bounded:
//      after ~1 s the kernel sets the error word and returns;
//   4. y[j] += sum over r = 0..world-1, in rank order, of data_r[phase][j]
//      (peer loads over NVLink), so every rank gets bit-identical sums.
// Two phases make the reuse safe: a rank reaches call s + 2 only after every
// peer has published s + 1, i.e. finished reading the phase of call s.
constexpr int kMaxRanks = 8;
constexpr int kPerThread = 5;  // vectors up to 5 x 1024 floats (H <= 5120)

struct PeerArgs {
    float* data[kMaxRanks];  // data[2][n_max] of every rank (own one included)
    int* flags[kMaxRanks];   // flags[2][kMaxRanks] of every rank
    int rank, world, n_max;
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(1024) peer_allreduce_kernel(PeerArgs a, int* __restrict__ seq_ptr,
                                                              const float* __restrict__ partial,
                                                              float* __restrict__ y, int n,
                                                              int* __restrict__ err, uint64_t limit_ns) {
    griddep_wait();
    __shared__ int s_ok;
    // A rank whose earlier call gave up is out of step with its peers: every
    // later call returns at once, leaving y alone, with the error word kept.
    if (*(volatile int*)err) return;
    const int seq = *seq_ptr + 1, phase = seq & 1;
    float* mine = a.data[a.rank] + (int64_t)phase * a.n_max;
    {
        float v[kPerThread];
#pragma unroll
        for (int k = 0; k < kPerThread; ++k) {
            const int j = threadIdx.x + k * 1024;
            v[k] = j < n ? partial[j] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < kPerThread; ++k) {
            const int j = threadIdx.x + k * 1024;
            if (j < n) mine[j] = v[k];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int r = 0; r < a.world; ++r) st_release_sys(a.flags[r] + phase * kMaxRanks + a.rank, seq);
        s_ok = 1;
    }
    __syncthreads();
    if (threadIdx.x < a.world) {  // one thread per source rank
        const int* f = a.flags[a.rank] + phase * kMaxRanks + threadIdx.x;
        const uint64_t start = global_ns();
        int n_try = 0;
        while (ld_acquire_sys(f) != seq) {
            if ((++n_try & 63) == 0 && global_ns() - start > limit_ns) {
                atomicExch(err, 1);
                s_ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;
    // every load of every rank is issued before the first use (peer loads
    // cost ~1 us each over NVLink), then the sums are taken in rank order
    float t[kMaxRanks][kPerThread];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
        if (r < a.world) {
            const float* src = a.data[r] + (int64_t)phase * a.n_max;
#pragma unroll
            for (int k = 0; k < kPerThread; ++k) {
                const int j = threadIdx.x + k * 1024;
                t[r][k] = j < n ? src[j] : 0.f;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
        const int j = threadIdx.x + k * 1024;
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
            if (r < a.world) acc += t[r][k];
        if (j < n) y[j] += acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) *seq_ptr = seq;
}

}  // namespace

size_t tp_peer_buffer_bytes(int n_max) {
    return ((size_t)2 * n_max * 4 + 255) / 256 * 256 + 2 * kMaxRanks * sizeof(int);
}

int tp_peer_allreduce_add(void* const* bases, int rank, int world, int n_max, int* seq, const float* partial,
                          float* y, int n, int* err, double timeout_s, cudaStream_t s) {
    if (world < 1 || rank < 0 || rank >= world || n < 0 || !(timeout_s > 0.0) || timeout_s > 60.0)
        return Q3XK_EINVAL;
    if (world > kMaxRanks || n > n_max || n > kPerThread * 1024) return Q3XK_EUNSUPPORTED;
    for (int r = 0; r < world; ++r)
        if (!bases[r]) return Q3XK_EINVAL;
    PeerArgs a{};
    const size_t data_bytes = ((size_t)2 * n_max * 4 + 255) / 256 * 256;
    for (int r = 0; r < world; ++r) {
        a.data[r] = static_cast<float*>(bases[r]);
        a.flags[r] = reinterpret_cast<int*>(static_cast<uint8_t*>(bases[r]) + data_bytes);
    }
    a.rank = rank;
    a.world = world;
    a.n_max = n_max;
    const uint64_t limit_ns = (uint64_t)(timeout_s * 1e9);
    if (launch_pdl(peer_allreduce_kernel, dim3(1), dim3(1024), 0, s, a, seq, partial, y, n, err, limit_ns) !=
        cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int tp_pack_best(const float* logits, const int* idx, int v0, float* out2, cudaStream_t s) {
    if (launch_pdl(pack_best_kernel, dim3(1), dim3(1), 0, s, logits, idx, v0, out2) != cudaSuccess) return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

const char* nccl_load() {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl_tried) return g_nccl_error;
    g_nccl_tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy torch loaded, if any
    if (!h) {
        const char* path = std::getenv("Q3XK_NCCL_LIBRARY");
        h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) return g_nccl_error = "libnccl.so.2 not found (set Q3XK_NCCL_LIBRARY)";
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
    g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(h, "ncclAllGather"));
    g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.comm_destroy || !g_nccl.all_reduce ||
        !g_nccl.all_gather)
        return g_nccl_error = "libnccl.so.2 lacks a needed symbol";
    return nullptr;
}

int tp_unique_id(char id[kNcclIdBytes]) {
    static_assert(sizeof(ncclUniqueId) == kNcclIdBytes, "NCCL id size");
    if (!id) return Q3XK_EINVAL;
    if (nccl_load()) return Q3XK_EUNSUPPORTED;
    ncclUniqueId u;
    if (g_nccl.get_unique_id(&u) != ncclSuccess) return Q3XK_ECUDA;
    std::memcpy(id, &u, sizeof u);
    return Q3XK_OK;
}

int tp_comm_create(const char id[kNcclIdBytes], int rank, int world, void** comm) {
    if (!id || !comm || world < 1 || rank < 0 || rank >= world) return Q3XK_EINVAL;
    if (nccl_load()) return Q3XK_EUNSUPPORTED;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    ncclComm_t c = nullptr;
    const ncclResult_t r = g_nccl.comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) {
        std::snprintf(g_last_error, sizeof g_last_error, "ncclCommInitRank: %s",
                      g_nccl.error_string ? g_nccl.error_string(r) : "error");
        return Q3XK_ECUDA;
    }
    *comm = c;
    return Q3XK_OK;
}

const char* tp_last_error() { return g_last_error; }

void tp_comm_destroy(void* comm) {
    if (comm && !nccl_load()) g_nccl.comm_destroy(static_cast<ncclComm_t>(comm));
}

int tp_allreduce_add(void* comm, float* partial, float* hidden, int64_t n, cudaStream_t s) {
    if (g_nccl.all_reduce(partial, partial, (size_t)n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), s) !=
        ncclSuccess)
        return Q3XK_ECUDA;
    const int blocks = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
    if (launch_pdl(add_kernel, dim3(blocks), dim3(256), 0, s, hidden, (const float*)partial, n) != cudaSuccess)
        return Q3XK_ECUDA;
    count_launch();
    return Q3XK_OK;
}

int tp_allgather(void* comm, const float* in, float* out, int64_t n, cudaStream_t s) {
    if (g_nccl.all_gather(in, out, (size_t)n, ncclFloat32, static_cast<ncclComm_t>(comm), s) != ncclSuccess)
        return Q3XK_ECUDA;
    return Q3XK_OK;
}

}  // namespace q3xk

using namespace q3xk;

extern "C" {

size_t q3xk_peer_buffer_bytes(int n_max) { return n_max > 0 ? tp_peer_buffer_bytes(n_max) : 0; }

int q3xk_peer_allreduce_add(void* const* bases, int rank, int world, int n_max, int* seq, const float* partial,
                            float* y, int n, int* err, double timeout_s, void* stream) {
    if (!bases || !seq || !partial || !y || !err || n_max <= 0) return Q3XK_EINVAL;
    return tp_peer_allreduce_add(bases, rank, world, n_max, seq, partial, y, n, err, timeout_s,
                                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
