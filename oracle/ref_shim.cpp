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

// ---------------------------------------------------------------------------
// Custom-shape models for the parity tests.  Model::load only accepts the
// registered model IDs (model_config.h:104-113); the tests also use small
// models with the real head sizes.  This binds a model.bin written for a
// caller-given ModelConfig with the same tensor walk as Model::load
// (engine.cpp:481-559), then the unmodified reference forward runs on it.
namespace {

bool load_custom(q3x_backend::Model& m, const char* path, const q3x_model::ModelConfig* cfg,
                 const char** error) {
    using namespace q3x_backend;
    auto fail = [&](const char* message) { *error = message; return false; };
    m.fd = open(path, O_RDONLY);
    struct stat info {};
    if (m.fd < 0) return fail("cannot open model.bin");
    if (fstat(m.fd, &info) || info.st_size < static_cast<off_t>(q3x_model::HEADER_SIZE))
        return fail("bad model.bin");
    m.file_size = static_cast<size_t>(info.st_size);
    m.file = static_cast<const uint8_t*>(mmap(nullptr, m.file_size, PROT_READ, MAP_PRIVATE, m.fd, 0));
    if (m.file == MAP_FAILED) { m.file = nullptr; return fail("mmap model.bin failed"); }
    if (std::memcmp(m.file, "Q3XMODL\0", 8) != 0) return fail("wrong model.bin magic");
    if (!q3x_model::header_matches(m.file, m.file_size, *cfg)) return fail("Qwen model.bin header mismatch");
    m.config = cfg;
    const auto& c = *cfg;
    size_t cursor = q3x_model::HEADER_SIZE;
    const int AS = c.AH * c.AD, KVW = c.KVH * c.AD;
    const int DO = c.VH * c.VD, DQKV = 2 * c.KH * c.KD + DO;
    auto linear = [&](int rows, int cols, q3x_model::MatrixType type) {
        if (type == q3x_model::MATRIX_BF16)
            return Linear {take<BF16>(m.file, m.file_size, cursor, static_cast<size_t>(rows) * cols, error),
                           rows, cols, type};
        size_t bytes = 0;
        if (!*error && !q3x_cpu::quantized_bytes(type, rows, cols, &bytes)) *error = "invalid quantized matrix layout";
        return Linear {take<uint8_t>(m.file, m.file_size, cursor, bytes, error), rows, cols, type};
    };
    auto model_linear = [&](int rows, int cols) { return linear(rows, cols, c.matrix_type); };
    auto expert = [&](int rows, int cols) {
        const Linear all = model_linear(c.experts * rows, cols);
        return ExpertLinear {all.w, c.experts, rows, cols, all.type};
    };
    m.layer.reset(new (std::nothrow) Layer[c.N]);
    if (!m.layer) return fail("cannot allocate model layer table");
    m.embedding = model_linear(c.V, c.H);
    m.lm_head = c.tied_embeddings ? m.embedding : model_linear(c.V, c.H);
    m.final_norm = take<BF16>(m.file, m.file_size, cursor, c.H, error);
    for (int i = 0; i < c.N; ++i) {
        Layer& l = m.layer[i];
        l.input_norm = take<BF16>(m.file, m.file_size, cursor, c.H, error);
        if (i % c.AI != c.AI - 1) {
            l.delta.qkv = model_linear(DQKV, c.H); l.delta.z = model_linear(DO, c.H);
            l.delta.a = model_linear(c.VH, c.H); l.delta.b = model_linear(c.VH, c.H);
            l.delta.conv = take<BF16>(m.file, m.file_size, cursor, static_cast<size_t>(DQKV) * c.CK, error);
            l.delta.alog = take<FP32>(m.file, m.file_size, cursor, c.VH, error);
            l.delta.dt = take<BF16>(m.file, m.file_size, cursor, c.VH, error);
            l.delta.norm = take<FP32>(m.file, m.file_size, cursor, c.VD, error);
            l.delta.out = model_linear(c.H, DO);
        } else {
            l.attention.q = model_linear(2 * AS, c.H); l.attention.k = model_linear(KVW, c.H);
            l.attention.v = model_linear(KVW, c.H);
            l.attention.qnorm = take<BF16>(m.file, m.file_size, cursor, c.AD, error);
            l.attention.knorm = take<BF16>(m.file, m.file_size, cursor, c.AD, error);
            l.attention.out = model_linear(c.H, AS);
        }
        l.post_norm = take<BF16>(m.file, m.file_size, cursor, c.H, error);
        if (c.experts) {
            l.moe.router = linear(c.experts, c.H, q3x_model::MATRIX_BF16);
            l.moe.gate_up = expert(2 * c.I, c.H);
            l.moe.down = expert(c.H, c.I);
            l.moe.shared_gate = model_linear(c.shared_I, c.H);
            l.moe.shared_up = model_linear(c.shared_I, c.H);
            l.moe.shared_down = model_linear(c.H, c.shared_I);
            l.moe.shared_scale = linear(1, c.H, q3x_model::MATRIX_BF16);
        } else {
            l.gate = model_linear(c.I, c.H);
            l.up = model_linear(c.I, c.H); l.down = model_linear(c.H, c.I);
        }
    }
    if (*error) return false;
    if (cursor != m.file_size) return fail("model.bin size does not match schema");
    return true;
}

}  // namespace

extern "C" {

// fields: id V H I N AI AH KVH AD RD KH VH KD VD CK experts top_k shared_I matrix_type tied
void* q3xref_model_create_custom(const char* path, const int* f, char* err, size_t errlen) {
    auto* cfg = new q3x_model::ModelConfig {
        static_cast<uint32_t>(f[0]), "custom", f[1], f[2], f[3], f[4], f[5], f[6], f[7], f[8], f[9],
        f[10], f[11], f[12], f[13], f[14], f[15], f[16], f[17],
        static_cast<q3x_model::MatrixType>(f[18]), f[19] != 0,
    };
    std::unique_ptr<q3x_backend::Model> model(new (std::nothrow) q3x_backend::Model());
    const char* message = nullptr;
    if (!model || !load_custom(*model, path, cfg, &message)) {
        if (err && errlen) std::snprintf(err, errlen, "%s", message ? message : "allocation failed");
        return nullptr;
    }
    if (err && errlen) err[0] = '\0';
    return model.release();
}

}  // extern "C"
