// ref_shim.cpp -- C entry points over the UNMODIFIED qwen3x CPU engine.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with the reference's own engine.cpp and arch/cpu.cpp, where they lie in
// the reference source tree, into oracle/_ref/libq3xref_*.so.  It is used to
// pin the C restatement (q3x_oracle.c), to make golden fixtures, and as the
// timed CPU baseline (bench.py --impl reference).  Nothing here is product
// code: the reference sources are compiled, never copied.
//
// The reference's own tests reach engine internals the same way, by
// including engine.cpp into the test translation unit (tests/q4_cpu_test.cpp:10).
#include "engine.cpp"

#include <cstdarg>
#include <thread>
#include <vector>

// internal.h declares these; the reference defines them in log.cpp on top of
// spdlog.  The oracle only needs assertion reports on stderr.
namespace q3x_internal {
void report_assertion(const char* expression, const char* file, int line,
                      const char* format, ...) {
    std::fprintf(stderr, "reference assertion failed: %s at %s:%d: ", expression, file, line);
    va_list args;
    va_start(args, format);
    std::vfprintf(stderr, format, args);
    va_end(args);
    std::fputc('\n', stderr);
}
void logf(q3x_log_level, const char*, int, const char*, ...) {}
}  // namespace q3x_internal

namespace {

size_t linear_bytes(q3x_model::MatrixType type, int rows, int cols) {
    size_t bytes = static_cast<size_t>(rows) * cols * sizeof(q3x_backend::BF16);
    if (type != q3x_model::MATRIX_BF16) q3x_cpu::quantized_bytes(type, rows, cols, &bytes);
    return bytes;
}

}  // namespace

extern "C" {

int q3xref_has_avx512() {
#if defined(__AVX512F__) && defined(__AVX512BW__)
    return 1;
#else
    return 0;
#endif
}

int q3xref_quantized_bytes(uint32_t type, int rows, int cols, size_t* bytes) {
    return q3x_cpu::quantized_bytes(static_cast<q3x_model::MatrixType>(type), rows, cols, bytes) ? 1 : 0;
}

// q3x_cpu::try_mv as is: 1 when it handled the matrix, 0 when it declined.
int q3xref_try_mv(const void* w, uint32_t type, int rows, int cols, const float* x, float* y) {
    return q3x_cpu::try_mv(w, static_cast<q3x_model::MatrixType>(type), rows, cols, x, y) ? 1 : 0;
}

int q3xref_try_embed(const void* w, uint32_t type, int cols, int token, float* out) {
    return q3x_cpu::try_embed(w, static_cast<q3x_model::MatrixType>(type), cols, token, out) ? 1 : 0;
}

// engine.cpp's mv() (try_mv, else the BF16 baseline) on row slices spread over
// `threads` std::threads.  Rows are independent, so the bytes of y are those
// of one single-threaded call.
int q3xref_mv(const void* w, uint32_t type, int rows, int cols, const float* x, float* y,
              int threads) {
    const auto t = static_cast<q3x_model::MatrixType>(type);
    if (rows <= 0 || cols <= 0) return -1;
    const size_t row_bytes = linear_bytes(t, 1, cols);
    auto run = [&](int row0, int row1) {
        if (row1 <= row0) return;
        q3x_backend::Linear slice {static_cast<const uint8_t*>(w) + row_bytes * row0,
                                   row1 - row0, cols, t};
        q3x_backend::mv(slice, x, y + row0);
    };
    if (threads <= 1) { run(0, rows); return 0; }
    if (threads > rows) threads = rows;
    std::vector<std::thread> pool;
    pool.reserve(threads);
    for (int i = 1; i < threads; ++i)
        pool.emplace_back(run, static_cast<int>(1LL * rows * i / threads),
                          static_cast<int>(1LL * rows * (i + 1) / threads));
    run(0, static_cast<int>(1LL * rows / threads));
    for (auto& th : pool) th.join();
    return 0;
}

int q3xref_router_top_k(const float* logits, int experts, int top_k, int* ids, float* probabilities) {
    q3x_backend::router_top_k(logits, experts, top_k, ids, probabilities);
    return 0;
}

// engine.cpp:406-430 for one token.  Work sizes come from a ModelConfig whose
// delta value width equals H, so Work::delta_output can hold an expert output.
int q3xref_moe(const uint16_t* router, const void* gate_up, const void* down,
               const void* shared_gate, const void* shared_up, const void* shared_down,
               const uint16_t* shared_scale, uint32_t type, int experts, int top_k,
               int H, int I, int shared_I, const float* input, float* out,
               int* ids, float* weights) {
    if (shared_I > I) return -1;
    const auto t = static_cast<q3x_model::MatrixType>(type);
    const q3x_model::ModelConfig config {
        1, "oracle-moe", 1, H, I, 1,
        1, 1, 1, 1, 0, 1, 1, 1, H, 4,
        experts, top_k, shared_I, t, false,
    };
    q3x_backend::MoeWeights moe {
        {router, experts, H, q3x_model::MATRIX_BF16},
        {gate_up, experts, 2 * I, H, t},
        {down, experts, H, I, t},
        {shared_gate, shared_I, H, t},
        {shared_up, shared_I, H, t},
        {shared_down, H, shared_I, t},
        {shared_scale, 1, H, q3x_model::MATRIX_BF16},
    };
    q3x_backend::Work work(config);
    q3x_backend::moe(moe, input, work, out, config);
    for (int slot = 0; slot < top_k; ++slot) {
        if (ids) ids[slot] = work.expert_ids[slot];
        if (weights) weights[slot] = work.router_probs[work.expert_ids[slot]];
    }
    return 0;
}

// The full reference CPU forward (q3x_backend interface, internal.h:16-32).
void* q3xref_model_create(const char* path, char* err, size_t errlen) {
    return q3x_backend::model_create(path, err, errlen);
}
void q3xref_model_destroy(void* model) {
    q3x_backend::model_destroy(static_cast<q3x_backend::Model*>(model));
}
void* q3xref_state_create(void* model, int context) {
    return q3x_backend::state_create(static_cast<q3x_backend::Model*>(model), context);
}
void q3xref_state_destroy(void* state) {
    q3x_backend::state_destroy(static_cast<q3x_backend::State*>(state));
}
void q3xref_state_reset(void* state) {
    q3x_backend::state_reset(static_cast<q3x_backend::State*>(state));
}
void q3xref_state_forward(void* model, void* state, const int* tokens, int count, int logits) {
    q3x_backend::state_forward(static_cast<q3x_backend::Model*>(model),
                               static_cast<q3x_backend::State*>(state), tokens, count, logits != 0);
}
int q3xref_state_argmax(void* state) {
    return q3x_backend::state_argmax(static_cast<q3x_backend::State*>(state));
}
void q3xref_state_copy_logits(void* state, float* out) {
    q3x_backend::state_copy_logits(static_cast<q3x_backend::State*>(state), out);
}
void q3xref_state_checkpoint_save(void* state) {
    q3x_backend::state_checkpoint_save(static_cast<q3x_backend::State*>(state));
}
void q3xref_state_checkpoint_restore(void* state) {
    q3x_backend::state_checkpoint_restore(static_cast<q3x_backend::State*>(state));
}
uint32_t q3xref_model_id(void* model) {
    return q3x_backend::model_id(static_cast<q3x_backend::Model*>(model));
}

}  // extern "C"
