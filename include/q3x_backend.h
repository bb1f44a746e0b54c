/*
 * q3x_backend.h -- the qwen3x compute-backend interface, implemented on B200.
 *
 * Part 1 (C++) is the reference's opaque backend API with the same names,
 * signatures and semantics (internal.h:11-34, namespace q3x_backend), so the
 * reference's runtime.cpp (Session, CLI, HTTP server) links against this
 * library in place of engine.cpp / arch/cuda/engine.cu.  As in the reference,
 * invalid arguments are fatal (the reference's Q3X_ASSERT reports and aborts).
 *
 * Part 2 (C) is the same operations as a C ABI with status codes instead of
 * aborts, for FFI callers (Python ctypes in this repository's tests and
 * benchmark).  Statuses are q3xk_status values (q3xk.h).
 *
 * One Model and its States live on the device that is current when
 * model_create is called; every later call sets that device itself.
 */
#ifndef Q3X_BACKEND_H
#define Q3X_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#include "q3xk.h"

#ifdef __cplusplus
namespace q3x_backend {

struct Model;
struct State;

/* internal.h:16-17; model.bin is mmapped, checked (magic, registered model
 * ID, header fields, schema size; the reference's error strings) and its
 * matrices uploaded once in the device row-record layout. */
Q3XK_API Model* model_create(const char* path, char* err, size_t errlen);
Q3XK_API void model_destroy(Model* model);

/* internal.h:19-30.  state_forward (and state_forward_batch) return once the
 * step's device work has finished, as the reference's CUDA backend does
 * (arch/cuda/engine.cu:2307); the C mirror below is stream-ordered instead. */
Q3XK_API State* state_create(Model* model, int context_size);
Q3XK_API void state_destroy(State* state);
Q3XK_API void state_reset(State* state);
Q3XK_API void state_forward(Model* model, State* state, const int* tokens, int count, bool compute_logits);
Q3XK_API void state_checkpoint_save(State* state);
Q3XK_API void state_checkpoint_restore(State* state);
Q3XK_API int state_argmax(const State* state);
Q3XK_API void state_copy_logits(const State* state, float* output);
Q3XK_API uint32_t model_id(const Model* model);

/* Batched decode (no counterpart in the reference, which advances one State
 * per call): one token for each of `count` (1..16) distinct States of the
 * same model, each computing its logits -- the same as state_forward(
 * states[b], &tokens[b], 1, true) for every b, with every matrix read once
 * for all of them.  Runs on states[0]'s stream (the others' streams are
 * joined before and after); one GPU. */
Q3XK_API void state_forward_batch(Model* model, State* const* states, const int* tokens, int count);

/* internal.h:32-34 (constants of the registered Qwen family). */
Q3XK_API int vocab_size();
Q3XK_API int max_context();
Q3XK_API bool token_is_stop(int token);

}  // namespace q3x_backend

extern "C" {
#endif

typedef struct q3xb_model q3xb_model;
typedef struct q3xb_state q3xb_state;

/* Model handles: NULL on failure with the reason in err. */
Q3XK_API q3xb_model* q3xb_model_create(const char* path, char* err, size_t errlen);
Q3XK_API void q3xb_model_destroy(q3xb_model* model);
Q3XK_API uint32_t q3xb_model_id(const q3xb_model* model);
/* The 16 header fields of the model's configuration followed by experts,
 * top_k, shared_I, matrix_type, tied (21 ints). */
Q3XK_API int q3xb_model_config(const q3xb_model* model, int* fields21);
/* Device bytes the model's weights occupy. */
Q3XK_API size_t q3xb_model_device_bytes(const q3xb_model* model);

/* State: context_size in 1..262144.  NULL on failure (err filled). */
Q3XK_API q3xb_state* q3xb_state_create(q3xb_model* model, int context_size, char* err, size_t errlen);
Q3XK_API void q3xb_state_destroy(q3xb_state* state);
Q3XK_API int q3xb_state_reset(q3xb_state* state);
/* tokens: host int32[count]; returns once the work is queued on the
 * state's stream (logits/argmax calls synchronise). */
Q3XK_API int q3xb_state_forward(q3xb_model* model, q3xb_state* state, const int* tokens, int count,
                                int compute_logits);
/* state_forward_batch of part 1 (tokens: host int32[count]). */
Q3XK_API int q3xb_state_forward_batch(q3xb_model* model, q3xb_state* const* states, const int* tokens, int count);
Q3XK_API int q3xb_state_checkpoint_save(q3xb_state* state);
Q3XK_API int q3xb_state_checkpoint_restore(q3xb_state* state);
Q3XK_API int q3xb_state_argmax(const q3xb_state* state, int* token);
Q3XK_API int q3xb_state_copy_logits(const q3xb_state* state, float* output);
Q3XK_API int q3xb_state_position(const q3xb_state* state);
/* Blocks until the state's queued work is done; returns its CUDA status. */
Q3XK_API int q3xb_state_synchronize(const q3xb_state* state);
/* The CUDA stream the state's work runs on (cudaStream_t). */
Q3XK_API void* q3xb_state_stream(const q3xb_state* state);
/* 1 = decode steps (count 1 with logits) replay one captured CUDA graph
 * (default); 0 = launch them one by one. */
Q3XK_API int q3xb_state_set_graphs(q3xb_state* state, int enabled);
/* 1 = prompts (count > 1) run every matrix through the CUDA-core GEMV, one
 * token at a time, with the decode path's FP32 accuracy; 0 (default) = the
 * tcgen05 dequant-GEMM. */
Q3XK_API int q3xb_state_set_exact_prefill(q3xb_state* state, int enabled);
/* Precision of the prompt GEMMs (q3xk.h): Q3XK_GEMM_SPLIT (default; split
 * FP16 operands, FP32-grade logits) or Q3XK_GEMM_FP16 (one FP16 MMA per
 * K-step: faster, logits within ~3e-3). */
Q3XK_API int q3xb_state_set_prefill_precision(q3xb_state* state, int precision);
/* Tokens per forward pass of a prompt, 1..min(context, 2048) (the default is
 * the maximum; the work buffers are sized for it at state creation). */
Q3XK_API int q3xb_state_set_prefill_chunk(q3xb_state* state, int tokens);

/*
 * Tensor parallelism (one process per GPU, dense models): each rank loads its
 * share of model.bin (column-parallel q/k/v/z/a/b, q+gate, gate/up and
 * lm_head rows; row-parallel out/down columns, partial sums all-reduced with
 * NCCL) and owns a State whose collectives run on the state's stream.
 * MoE models take expert parallelism through the same calls: each rank loads
 * the routed experts [e0, e0 + experts/world) of every layer and replicates
 * everything else; a token's MoE output is the all-reduced sum of the slots
 * each rank runs (the shared expert of layer i runs on rank i % world), and
 * logits/argmax are local (every rank holds the full lm_head).  Rank 0
 * makes a communicator id with q3xb_tp_unique_id and every rank passes the
 * same 128 bytes to q3xb_state_create_tp; an id bootstraps one communicator,
 * so every State needs a fresh one.  state_forward, state_argmax and
 * state_copy_logits are collective: every rank calls them in the same order.
 * No counterpart in the reference (single-GPU backends only).
 */
Q3XK_API q3xb_model* q3xb_model_create_tp(const char* path, int rank, int world, char* err, size_t errlen);
Q3XK_API int q3xb_tp_unique_id(char* id128);
Q3XK_API q3xb_state* q3xb_state_create_tp(q3xb_model* model, int context_size, const char* id128, char* err,
                                          size_t errlen);
/* Decode all-reduces over NVLink peer memory instead of NCCL (one kernel, one
 * round of flags): every rank exports its buffer (64-byte CUDA IPC handle),
 * the handles are exchanged in rank order, and every rank opens the others'.
 * Without this step the state uses NCCL for every all-reduce. */
Q3XK_API int q3xb_state_ipc_handle(const q3xb_state* state, char* handle64);
Q3XK_API int q3xb_state_ipc_open(q3xb_state* state, const char* handles_world_x_64);
/* 1 if a peer all-reduce gave up waiting for a peer, else 0 (synchronous).
 * A rank whose wait ran out is out of step with its peers for good: its
 * later all-reduces return at once, and state_forward, state_argmax,
 * state_copy_logits and q3xb_state_synchronize report Q3XK_ETIMEOUT (the C++
 * q3x_backend calls abort, as the reference's Q3X_ASSERT does) -- from the
 * first of them that runs after the failed step's work has finished. */
Q3XK_API int q3xb_state_tp_error(const q3xb_state* state, int* flags);
/* Bound of the peer all-reduce's wait for a peer, in seconds (0 < s <= 60,
 * default 1).  Set it before the first decode step: the captured decode
 * graph keeps the bound it was made with (Q3XK_EUNSUPPORTED afterwards). */
Q3XK_API int q3xb_state_set_peer_timeout(q3xb_state* state, double seconds);
/* The rank's share: rank, world, first key/value/query/KV head, first
 * intermediate row, first vocabulary row, the local KH, VH, AH, KVH, I, V,
 * then the first routed expert and the local routed-expert count (MoE). */
Q3XK_API int q3xb_model_shard(const q3xb_model* model, int* fields16);
/* The same plan for a registered model ID without loading anything. */
Q3XK_API int q3xb_tp_plan(uint32_t model_id, int rank, int world, int* fields16, char* err, size_t errlen);

#ifdef __cplusplus
}  // extern "C"
#endif

#endif /* Q3X_BACKEND_H */
