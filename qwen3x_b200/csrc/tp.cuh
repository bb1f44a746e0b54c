// tp.cuh -- tensor and expert parallelism across GPUs: the collectives the
// backend makes (NCCL, and a peer-memory all-reduce for decode).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2: the copy torch already
// loaded, or the path in Q3XK_NCCL_LIBRARY), so libq3xk.so itself does not
// depend on it and single-GPU use never touches it.
#pragma once

#include "common.cuh"

namespace q3xk {

constexpr int kNcclIdBytes = 128;

// The NCCL library (nullptr with a reason if it cannot be loaded).
const char* nccl_load();
// A new communicator id (rank 0 creates it, every rank receives the bytes).
int tp_unique_id(char id[kNcclIdBytes]);
// Communicator of `world` ranks (collective: every rank calls it).
int tp_comm_create(const char id[kNcclIdBytes], int rank, int world, void** comm);
void tp_comm_destroy(void* comm);
// Message of the last failed NCCL call.
const char* tp_last_error();
// hidden[0..n) += allreduce_sum(partial[0..n)) (partial is overwritten).
int tp_allreduce_add(void* comm, float* partial, float* hidden, int64_t n, cudaStream_t s);
// One-shot all-reduce of decode-sized vectors over peer memory (tp.cu):
// bases[r] = rank r's buffer of tp_peer_buffer_bytes(n_max) bytes (own one
// included, the others mapped with CUDA IPC), flags zeroed at creation; `seq`
// a device int (zero-initialised, identical call sequence on every rank);
// `err` a device int set to 1 if a peer did not publish within timeout_s
// seconds (then y is left alone, and every later call with err set returns at
// once).  y[0..n) += sum over ranks of partial[0..n), bit-identical on every
// rank.
size_t tp_peer_buffer_bytes(int n_max);
int tp_peer_allreduce_add(void* const* bases, int rank, int world, int n_max, int* seq, const float* partial,
                          float* y, int n, int* err, double timeout_s, cudaStream_t s);
// out2 = {logits[*idx], *idx + v0} (a rank's argmax in global numbering).
int tp_pack_best(const float* logits, const int* idx, int v0, float* out2, cudaStream_t s);
// out[world * n] = concatenation of every rank's in[n] (floats).
int tp_allgather(void* comm, const float* in, float* out, int64_t n, cudaStream_t s);

}  // namespace q3xk
