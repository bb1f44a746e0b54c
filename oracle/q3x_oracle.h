/*
 * q3x_oracle.h -- CPU restatement of qwen3x's packed-weight matrix path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in qwen3x_b200/csrc: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs load it.  The product
 * path never calls into it and has no CPU fallback.
 *
 * Every function restates one reference routine (paths are relative to the
 * qwen3x source tree) and keeps its FP32 operation order, so that on the
 * same inputs the results are bit-identical to the reference's scalar build
 * (pinned by tests/test_oracle_golden.py against fixtures produced by the
 * reference itself, see tests/golden/make_golden.py).
 */
#ifndef Q3X_ORACLE_H
#define Q3X_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* model_config.h:16-20 */
enum { Q3XO_BF16 = 0, Q3XO_Q8_0 = 1, Q3XO_Q4_0 = 2 };

/* arch/cpu.cpp:31-52 -- IEEE binary16 -> binary32, subnormals included. */
float q3xo_f16(uint16_t bits);
/* Round-to-nearest-even binary32 -> binary16 (numpy astype('<f2')). */
uint16_t q3xo_f32_to_f16(float value);
/* engine.cpp:181-186 */
float q3xo_bf16(uint16_t bits);

/* arch/cpu.cpp:161-179: 1 on success, 0 (bytes untouched) otherwise. */
int q3xo_quantized_bytes(uint32_t type, int rows, int cols, size_t* bytes);

/* arch/cpu.cpp:64-73 and :91-101 (q4.h:31-36 nibble order). */
float q3xo_dot_q8_0(const void* blocks, const float* x, int n);
float q3xo_dot_q4_0(const void* blocks, const float* x, int n);
/* engine.cpp:201-205 -- scalar BF16 dot (the engine's baseline). */
float q3xo_dot_bf16(const uint16_t* w, const float* x, int n);

/* arch/cpu.cpp:55-63, :81-90 -- one decoded row. */
int q3xo_embed(const void* w, uint32_t type, int cols, int token, float* out);

/*
 * arch/cpu.cpp:192-226 + engine.cpp:207-212: y[rows] = W[rows,cols] x.
 * Rows are independent, so `threads` > 1 splits the rows across pthreads and
 * gives bit-identical results.  Returns 0 on success, -1 on a bad type/shape.
 */
int q3xo_mv(const void* w, uint32_t type, int rows, int cols,
            const float* x, float* y, int threads);

/*
 * engine.cpp:580-583: the reference prefill is a per-token loop over mv, so
 * Y[T,rows] is T independent matvecs (row-major output [token][row]).
 */
int q3xo_gemm(const void* w, uint32_t type, int rows, int cols,
              const float* X, int T, float* Y, int threads);

/* engine.cpp:214-224: expert e of a contiguous W[experts,rows,cols]. */
int q3xo_expert_mv(const void* w, uint32_t type, int experts, int rows,
                   int cols, int expert, const float* x, float* y);

/* engine.cpp:377-405: softmax, greedy top-k (strict '>', lowest id wins a
 * tie), renormalised over the selected slots.  probabilities[experts] holds
 * the softmax with the selected entries renormalised in place. */
int q3xo_router_top_k(const float* logits, int experts, int top_k,
                      int* ids, float* probabilities);

/* engine.cpp:406-430: one MoE FFN for one token, out[H] (overwritten).
 * router and shared_scale are BF16; the expert pools and the shared expert
 * use `type`.  ids/weights (may be NULL) receive the routing decision. */
int q3xo_moe(const uint16_t* router, const void* gate_up, const void* down,
             const void* shared_gate, const void* shared_up,
             const void* shared_down, const uint16_t* shared_scale,
             uint32_t type, int experts, int top_k, int H, int I,
             int shared_I, const float* input, float* out,
             int* ids, float* weights);

/* engine.cpp:601-605: first index of the maximum (std::max_element). */
int q3xo_argmax(const float* logits, int n);

/* scripts/pack_weights.py:299-318 (Q8_0) and :321-343 (ggml Q4_0): BF16
 * source bits -> packed blocks.  Returns 0, or -1 on non-finite input. */
int q3xo_quantize_q8_0(const uint16_t* bf16, size_t count, void* blocks);
int q3xo_quantize_q4_0(const uint16_t* bf16, size_t count, void* blocks);

#ifdef __cplusplus
}
#endif
#endif
