// TEST INFRASTRUCTURE ONLY -- the parity checker, never shipped or measured as the product.
//
// extern "C" shim over the reference CPU engine (astrowar/MiniCPM5.cpp), linked
// against the unmodified reference sources by oracle/Makefile.  It exposes the
// reference's own hot-path entry points to ctypes:
//   * MiniCPM5Engine::init_kv_cache / load_model / forward   (src/model.cpp:17-242)
//   * quantize_row_q8_K_avx2                                  (src/ops/ops_avx2.cpp:85-144)
//   * gemv_{q4,q6}_K_q8_K_avx2                                (src/ops/ops_avx2.cpp:278-298)
//   * gemv_{q4,q6}_K_avx2 (fp32 input, ties-to-even quantise) (src/ops/ops_avx2.cpp:470-476)
//   * gemv_qkv_*_avx2, gemv_gate_up_q4_K_q8_K_avx2            (src/ops/ops_avx2.cpp:320-460)
//   * gemv_q8_0                                               (src/ops/ops.cpp:58-79)
//   * rmsnorm, rmsnorm_and_quantize_q8k, swiglu_and_quantize_q8k, apply_rope,
//     execute_attention, get_embedding                        (src/ops/ops.cpp:468-765)
//   * quantize_row_q8_K_scalar, dot_row_q{4,6}_K_q8_K_scalar  (src/ops/ops_scalar_optimized.cpp)
#include <cstring>
#include <string>
#include <vector>

#include "model.h"
#include "ops.h"
#include "ops_internal.h"

#if defined(_OPENMP)
#include <omp.h>
#endif

// Defined with external linkage in the reference sources but not declared in a header.
void gemv_q8_0(const char* matrix_weights, const float* x, float* out, int num_rows, int num_cols);
void quantize_row_q8_K_scalar(const float* x, block_q8_K* y, int n);
float dot_row_q4_K_q8_K_scalar(const block_q4_K* w, const block_q8_K* xq, int num_blocks);
float dot_row_q6_K_q8_K_scalar(const block_q6_K* w, const block_q8_K* xq, int num_blocks);

namespace {
Tensor f32_tensor(const float* w, int n) {
    Tensor t;
    t.name = "w";
    t.type_str = "F32";
    t.dims = {static_cast<uint64_t>(n)};
    t.data_ptr = reinterpret_cast<const char*>(w);
    t.size_bytes = static_cast<uint64_t>(n) * 4;
    return t;
}
Tensor mat_tensor(const void* w, const char* type, int rows, int cols) {
    Tensor t;
    t.name = "m";
    t.type_str = type;
    t.dims = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
    t.data_ptr = reinterpret_cast<const char*>(w);
    return t;
}
struct RefEngine {
    MiniCPM5Engine eng;
    int max_seq = 0;
};
}  // namespace

extern "C" {

int ref_omp_threads() {
#if defined(_OPENMP)
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void* ref_engine_create(const char* path, int max_seq) {
    auto* e = new RefEngine();
    e->max_seq = max_seq;
    e->eng.init_kv_cache(max_seq);
    if (!e->eng.load_model(std::string(path), false)) {
        delete e;
        return nullptr;
    }
    return e;
}

void ref_engine_destroy(void* h) { delete static_cast<RefEngine*>(h); }

// logits_out may be null; returns the greedy argmax (lowest index on ties).
int ref_forward(void* h, int token, int pos, float* logits_out) {
    auto* e = static_cast<RefEngine*>(h);
    const std::vector<float>& lg = e->eng.forward(token, pos, e->max_seq);
    if (logits_out) std::memcpy(logits_out, lg.data(), lg.size() * sizeof(float));
    int best = 0;
    for (int i = 1; i < static_cast<int>(lg.size()); ++i)
        if (lg[i] > lg[best]) best = i;
    return best;
}

void ref_quantize_row_q8k_avx2(const float* x, void* y, int n) {
    quantize_row_q8_K_avx2(x, static_cast<block_q8_K*>(y), n);
}
void ref_quantize_row_q8k_scalar(const float* x, void* y, int n) {
    quantize_row_q8_K_scalar(x, static_cast<block_q8_K*>(y), n);
}
void ref_gemv_q4k_q8k(const void* w, const void* xq, float* out, int rows, int cols) {
    gemv_q4_K_q8_K_avx2(static_cast<const char*>(w), static_cast<const block_q8_K*>(xq), out, rows, cols);
}
void ref_gemv_q6k_q8k(const void* w, const void* xq, float* out, int rows, int cols) {
    gemv_q6_K_q8_K_avx2(static_cast<const char*>(w), static_cast<const block_q8_K*>(xq), out, rows, cols);
}
void ref_gemv_q4k_f32(const void* w, const float* x, float* out, int rows, int cols) {
    gemv_q4_K_avx2(static_cast<const char*>(w), x, out, rows, cols);
}
void ref_gemv_q6k_f32(const void* w, const float* x, float* out, int rows, int cols) {
    gemv_q6_K_avx2(static_cast<const char*>(w), x, out, rows, cols);
}
void ref_gemv_q8_0(const void* w, const float* x, float* out, int rows, int cols) {
    gemv_q8_0(static_cast<const char*>(w), x, out, rows, cols);
}
float ref_dot_row_q4k_scalar(const void* w, const void* xq, int nb) {
    return dot_row_q4_K_q8_K_scalar(static_cast<const block_q4_K*>(w), static_cast<const block_q8_K*>(xq), nb);
}
float ref_dot_row_q6k_scalar(const void* w, const void* xq, int nb) {
    return dot_row_q6_K_q8_K_scalar(static_cast<const block_q6_K*>(w), static_cast<const block_q8_K*>(xq), nb);
}
void ref_gemv_qkv(const void* wq, const void* wk, const void* wv, int v_is_q6k, const void* xq,
                  float* q, float* k, float* v, int q_rows, int kv_rows, int cols) {
    auto* x = static_cast<const block_q8_K*>(xq);
    if (v_is_q6k)
        gemv_qkv_q4_q4_q6_q8_K_avx2(static_cast<const char*>(wq), static_cast<const char*>(wk),
                                    static_cast<const char*>(wv), x, q, k, v, q_rows, kv_rows, cols);
    else
        gemv_qkv_q4_K_q8_K_avx2(static_cast<const char*>(wq), static_cast<const char*>(wk),
                                static_cast<const char*>(wv), x, q, k, v, q_rows, kv_rows, cols);
}
void ref_gemv_gate_up(const void* wg, const void* wu, const void* xq, float* g, float* u, int rows, int cols) {
    gemv_gate_up_q4_K_q8_K_avx2(static_cast<const char*>(wg), static_cast<const char*>(wu),
                                static_cast<const block_q8_K*>(xq), g, u, rows, cols);
}
void ref_rmsnorm(float* out, const float* x, const float* w, int n) {
    std::vector<float> o(n), xv(x, x + n);
    rmsnorm(o, xv, f32_tensor(w, n));
    std::memcpy(out, o.data(), n * sizeof(float));
}
void ref_rmsnorm_quantize_q8k(void* out, const float* x, const float* w, int n) {
    std::vector<float> xv(x, x + n);
    rmsnorm_and_quantize_q8k(static_cast<block_q8_K*>(out), xv, f32_tensor(w, n));
}
void ref_swiglu_quantize_q8k(void* out, const float* g, const float* u, int n) {
    std::vector<float> gv(g, g + n), uv(u, u + n);
    swiglu_and_quantize_q8k(static_cast<block_q8_K*>(out), gv, uv);
}
void ref_apply_rope(float* vec, int n, int pos, int head_idx, int head_dim, float base) {
    std::vector<float> v(vec, vec + n);
    apply_rope(v, pos, head_idx, head_dim, base);
    std::memcpy(vec, v.data(), n * sizeof(float));
}
// kcache/vcache: [max_seq][n_kv*head_dim] fp32, updated in place at pos.
void ref_attention(float* out, const float* q, const float* k, const float* v, float* kcache, float* vcache,
                   int pos, int max_seq, int n_head, int n_kv, int head_dim) {
    const int kvd = n_kv * head_dim;
    std::vector<float> o(n_head * head_dim), qv(q, q + n_head * head_dim), kv_(k, k + kvd), vv(v, v + kvd);
    KVCacheLayer layer;
    layer.k.assign(kcache, kcache + static_cast<size_t>(max_seq) * kvd);
    layer.v.assign(vcache, vcache + static_cast<size_t>(max_seq) * kvd);
    execute_attention(o, qv, kv_, vv, layer, pos, max_seq, n_head, n_kv, head_dim);
    std::memcpy(out, o.data(), o.size() * sizeof(float));
    std::memcpy(kcache, layer.k.data(), layer.k.size() * sizeof(float));
    std::memcpy(vcache, layer.v.data(), layer.v.size() * sizeof(float));
}
void ref_get_embedding(float* out, const void* w, const char* type, int token, int dim, int vocab) {
    std::vector<float> o(dim);
    get_embedding(o, mat_tensor(w, type, vocab, dim), token);
    std::memcpy(out, o.data(), dim * sizeof(float));
}
float ref_silu(float x) { return silu(x); }

}  // extern "C"
