// Host side of the engine: GGUF load into one HBM arena, KV cache, RoPE table, the
// decode-kernel launch, and the C ABI of include/mcpm.h.
//
// Reference counterpart: MiniCPM5Engine (include/model.h:37-70, src/model.cpp:17-242).
// The reference reads the whole file into one host buffer and points tensors into it by
// absolute offset; here the tensor bytes are uploaded unchanged into one device
// allocation at the same relative offsets (base = first tensor byte).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>
#include <utility>
#include <initializer_list>

#include <cuda_fp16.h>

#include "../../include/mcpm.h"
#include "gguf.h"
#include "mcpm_device.cuh"
#include "mcpm_internal.h"

using namespace mcpm;

namespace {
// Control words, one small device allocation (mirrored into pinned host memory).
enum { CTL_ARGMAX = 0, CTL_TOKEN = 1, CTL_ERR = 2, CTL_BAR = 4, CTL_CNT = 8, CTL_WORDS = 16 };

const char* LAYER_NAMES[9] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
                              "attn_norm", "ffn_norm"};
}  // namespace

struct mcpm_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    int n_sm = 0;
    int n_ctas = 0;
    int req_ctas = 0;
    int batch_gemm = 0;   // MCPM_GEMM_MMA / MCPM_GEMM_TCGEN05
    int sched = 0;        // decode schedule option bits (mcpm_config::sched)
    int kv_f16 = 0;       // mcpm_config::kv_type == MCPM_KV_F16: kc / vc / b_kc / b_vc hold fp16 rows
    size_t kv_elt() const { return kv_f16 ? sizeof(__half) : sizeof(float); }
    // address of cache element `idx` (in elements) of a K or V array of this engine's element type
    uint8_t* kv_at(float* base, size_t idx) const { return reinterpret_cast<uint8_t*>(base) + idx * kv_elt(); }
    bool loaded = false;
    GGUFFile gguf;
    uint8_t* arena = nullptr;
    uint64_t arena_base = 0, arena_bytes = 0;
    std::vector<LayerDev> layers;
    LayerDev* d_layers = nullptr;
    int n_layer = 0, n_vocab = 0;
    float rope_base = 5000000.0f;
    const uint8_t* embd = nullptr;
    int embd_type = 0;
    const float* out_norm = nullptr;
    const uint8_t* lm = nullptr;
    int lm_type = 0;
    float *kc = nullptr, *vc = nullptr;
    int max_seq = 0;
    float2* rope = nullptr;
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *att_part = nullptr, *logits = nullptr;
    unsigned long long* xll = nullptr;   // residual stream with per-element epochs
    unsigned long long* qll = nullptr;   // q, K row, V row with per-element epochs
    unsigned long long* attw = nullptr;  // combined attention with per-element epochs
    float* am_val = nullptr;
    int* am_idx = nullptr;
    uint8_t* att_q8k = nullptr;
    int* ctl = nullptr;       // device control words
    int* ctl_host = nullptr;  // pinned mirror
    unsigned long long* trace = nullptr;   // phase timestamps when tracing is on
    // batched decode: b_n independent sequences, each with its own KV cache of b_max_seq positions
    int b_n = 0, b_max_seq = 0;
    float *b_kc = nullptr, *b_vc = nullptr, *b_x = nullptr, *b_y = nullptr, *b_q = nullptr;
    float *b_part = nullptr, *b_att = nullptr, *b_logits = nullptr;
    float2* b_rope = nullptr;
    int8_t* b_aqs = nullptr;
    float* b_ad = nullptr;
    int16_t* b_abs = nullptr;
    int *b_tokens = nullptr, *b_pos = nullptr, *b_argmax = nullptr;
    std::vector<int> b_pos_host;   // positions of the next step
    // batched prefill: row buffers for BATCH_MAX prompt positions of the engine's own sequence
    float *p_x = nullptr, *p_y = nullptr, *p_q = nullptr, *p_part = nullptr, *p_att = nullptr, *p_logits = nullptr;
    int8_t* p_aqs = nullptr;
    float* p_ad = nullptr;
    int16_t* p_abs = nullptr;
    int *p_tokens = nullptr, *p_pos = nullptr, *p_argmax = nullptr;
    // tcgen05 batched GEMM scratch (group partials, row-tile counters), shared by batch and prefill
    float* g_part = nullptr;
    unsigned* g_cnt = nullptr;
};

namespace {

mcpm_status cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return MCPM_OK;
    if (e == cudaErrorMemoryAllocation) return MCPM_OUT_OF_MEMORY;
    std::fprintf(stderr, "[mcpm] CUDA error: %s\n", cudaGetErrorString(e));
    return MCPM_CUDA_ERROR;
}

#define MCPM_CUDA(call)                                  \
    do {                                                 \
        const mcpm_status st__ = cuda_status((call));    \
        if (st__ != MCPM_OK) return st__;                \
    } while (0)

template <typename T>
void free_dev(T*& p) {
    if (p) cudaFree(const_cast<void*>(reinterpret_cast<const void*>(p)));
    p = nullptr;
}

void free_kv(mcpm_engine* e) {
    free_dev(e->kc);
    free_dev(e->vc);
    free_dev(e->rope);
    e->max_seq = 0;
}

void free_batch(mcpm_engine* e) {
    for (float** b : {&e->b_kc, &e->b_vc, &e->b_x, &e->b_y, &e->b_q, &e->b_part, &e->b_att, &e->b_logits}) free_dev(*b);
    free_dev(e->b_rope);
    free_dev(e->b_aqs);
    free_dev(e->b_ad);
    free_dev(e->b_abs);
    free_dev(e->b_tokens);
    free_dev(e->b_pos);
    free_dev(e->b_argmax);
    e->b_n = e->b_max_seq = 0;
    e->b_pos_host.clear();
}

void free_prefill(mcpm_engine* e) {
    for (float** b : {&e->p_x, &e->p_y, &e->p_q, &e->p_part, &e->p_att, &e->p_logits}) free_dev(*b);
    free_dev(e->p_aqs);
    free_dev(e->p_ad);
    free_dev(e->p_abs);
    free_dev(e->p_tokens);
    free_dev(e->p_pos);
    free_dev(e->p_argmax);
}

// Scratch of the tcgen05 batched GEMM, allocated on first use (counters zeroed).
mcpm_status ensure_gemm_scratch(mcpm_engine* e) {
    if (e->batch_gemm != MCPM_GEMM_TCGEN05 || e->g_part) return MCPM_OK;
    cudaError_t err = cudaMalloc(&e->g_part, batch_gemm_scratch_floats(e->n_vocab) * sizeof(float));
    if (err == cudaSuccess) err = cudaMalloc(&e->g_cnt, batch_gemm_counters(e->n_vocab) * sizeof(unsigned));
    if (err == cudaSuccess) err = cudaMemset(e->g_cnt, 0, batch_gemm_counters(e->n_vocab) * sizeof(unsigned));
    if (err != cudaSuccess) {
        free_dev(e->g_part);
        free_dev(e->g_cnt);
    }
    return cuda_status(err);
}

void free_model(mcpm_engine* e) {
    free_prefill(e);
    free_dev(e->g_part);
    free_dev(e->g_cnt);
    free_dev(e->arena);
    free_dev(e->d_layers);
    free_dev(e->x);
    free_dev(e->q);
    free_dev(e->att);
    free_dev(e->h);
    free_dev(e->xll);
    free_dev(e->qll);
    free_dev(e->attw);
    free_dev(e->att_part);
    free_dev(e->logits);
    free_dev(e->am_val);
    free_dev(e->am_idx);
    free_dev(e->att_q8k);
    e->layers.clear();
    e->loaded = false;
}

}  // namespace

// RoPE factors: theta_i = base^(-(i * (1/head_dim))), angle = theta * pos, (cos, sin)
// from the C library (the reference build's pow(base, -(i/head_dim)) / cosf / sinf,
// ops.cpp:502-516).  The CPU restatement computes the same table.
__attribute__((noinline)) void mcpm::rope_row(int pos, float base, float2* out) {
    const float inv = 1.0f / static_cast<float>(HEAD_DIM);
    for (int i = 0; i < HEAD_DIM; i += 2) {
        const float theta = powf(base, -(static_cast<float>(i) * inv));
        const float ang = theta * static_cast<float>(pos);
        const float c = cosf(ang);
        const float s = sinf(ang);
        out[i / 2] = make_float2(c, s);
    }
}

namespace {

// Largest per-CTA byte counts of the decode kernel's weight phases for n CTAs.
bool phases_fit(const mcpm_engine* e, int n, std::string& why) {
    auto ceil_div = [](int a, int b) { return (a + b - 1) / b; };
    int rb_qkv = 0, rb_o = 0, rb_gu = 0, rb_d = 0;
    for (const auto& L : e->layers) {
        rb_qkv = std::max({rb_qkv, row_bytes(L.tq, N_EMBD), row_bytes(L.tk, N_EMBD), row_bytes(L.tv, N_EMBD)});
        rb_o = std::max(rb_o, row_bytes(L.to, N_EMBD));
        rb_gu = std::max(rb_gu, row_bytes(L.tg, N_EMBD) + row_bytes(L.tu, N_EMBD));
        rb_d = std::max(rb_d, row_bytes(L.td, N_FF));
    }
    // QKV: the exact cost-weighted split of every layer (three 16-byte aligned segments)
    int qkv_rows = 0;
    long long qkv_bytes = 0;
    for (const auto& L : e->layers)
        for (int c = 0; c < n; ++c) {
            const int a = 2 * qkv_pair_boundary(L.tq, L.tk, L.tv, c, n), b = 2 * qkv_pair_boundary(L.tq, L.tk, L.tv, c + 1, n);
            qkv_rows = std::max(qkv_rows, b - a);
            const int lo[3] = {0, N_EMBD, N_EMBD + KV_DIM}, hi[3] = {N_EMBD, N_EMBD + KV_DIM, QKV_ROWS};
            const int ty[3] = {L.tq, L.tk, L.tv};
            long long bytes = 0;
            for (int i = 0; i < 3; ++i) {
                const int rows = std::max(0, std::min(b, hi[i]) - std::max(a, lo[i]));
                bytes += (static_cast<long long>(rows) * row_bytes(ty[i], N_EMBD) + 15) / 16 * 16;
            }
            qkv_bytes = std::max(qkv_bytes, bytes);
        }
    (void)rb_qkv;
    const int gu_rows = ceil_div(N_FF, n), od_rows = ceil_div(N_EMBD, n);
    const long long need[4] = {qkv_bytes, (long long)od_rows * rb_o, (long long)gu_rows * rb_gu + 16,
                               (long long)od_rows * rb_d};
    for (long long b : need)
        if (b > WBUF_BYTES) {
            why = "decode grid of " + std::to_string(n) + " CTAs needs " + std::to_string(b) +
                  " B per weight buffer (limit " + std::to_string(WBUF_BYTES) + ")";
            return false;
        }
    if (qkv_rows > ROWVAL_FLOATS || gu_rows > 128) {
        why = "too few CTAs for the row buffers";
        return false;
    }
    return true;
}

mcpm_status reset_ctl(mcpm_engine* e) {
    MCPM_CUDA(cudaMemsetAsync(e->ctl, 0, CTL_WORDS * sizeof(int), e->stream));
    // the launch sequence restarts, so no epoch of an aborted launch may remain
    if (e->xll) MCPM_CUDA(cudaMemsetAsync(e->xll, 0, XLL_COPIES * N_EMBD * sizeof(unsigned long long), e->stream));
    if (e->qll) MCPM_CUDA(cudaMemsetAsync(e->qll, 0, (N_EMBD + 2 * KV_DIM) * sizeof(unsigned long long), e->stream));
    if (e->attw)
        MCPM_CUDA(cudaMemsetAsync(e->attw, 0, ATTW_COPIES * N_EMBD * sizeof(unsigned long long), e->stream));
    if (e->att_part) MCPM_CUDA(cudaMemsetAsync(e->att_part, 0, ATT_PART_FLOATS * sizeof(float), e->stream));   // headers
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    return MCPM_OK;
}

mcpm_status check_ctl(mcpm_engine* e) {
    MCPM_CUDA(cudaMemcpyAsync(e->ctl_host, e->ctl, 4 * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    const unsigned err = static_cast<unsigned>(e->ctl_host[CTL_ERR]);
    if (err) {
        reset_ctl(e);   // barrier words may be mid-count after an aborted launch
        if (err & ERR_BAD_TOKEN) return MCPM_BAD_TOKEN;
        return MCPM_TIMEOUT;
    }
    return MCPM_OK;
}

DecodeParams make_params(const mcpm_engine* e, int token, int pos, int write_logits) {
    DecodeParams p{};
    p.layers = e->d_layers;
    p.arena = e->arena;
    p.n_layer = e->n_layer;
    p.embd = e->embd;
    p.embd_type = e->embd_type;
    p.out_norm = e->out_norm;
    p.lm = e->lm;
    p.lm_type = e->lm_type;
    p.n_vocab = e->n_vocab;
    p.kc = e->kc;
    p.vc = e->vc;
    p.max_seq = e->max_seq;
    p.rope = e->rope;
    p.x = e->x;
    p.q = e->q;
    p.att = e->att;
    p.att_q8k = e->att_q8k;
    p.h = e->h;
    p.xll = e->xll;
    p.qll = e->qll;
    p.attw = e->attw;
    p.att_part = e->att_part;
    p.logits = e->logits;
    p.am_val = e->am_val;
    p.am_idx = e->am_idx;
    p.argmax_out = e->ctl + CTL_ARGMAX;
    p.token_dev = e->ctl + CTL_TOKEN;
    p.err = reinterpret_cast<unsigned*>(e->ctl + CTL_ERR);
    p.bar = reinterpret_cast<unsigned*>(e->ctl + CTL_BAR);
    p.cnt = reinterpret_cast<unsigned*>(e->ctl + CTL_CNT);
    p.trace = e->trace;
    p.sched = e->sched;
    p.kv_f16 = e->kv_f16;
    p.blk_order = e->batch_gemm == MCPM_GEMM_TCGEN05;
    p.token = token;
    p.pos = pos;
    p.write_logits = write_logits;
    return p;
}

mcpm_status launch(mcpm_engine* e, int token, int pos, int write_logits) {
    if (!e || !e->loaded || !e->kc) return MCPM_NOT_LOADED;
    if (pos < 0 || pos >= e->max_seq) return MCPM_CTX_OVERFLOW;
    if (token >= e->n_vocab) return MCPM_BAD_TOKEN;
    MCPM_CUDA(cudaSetDevice(e->device));
    const DecodeParams p = make_params(e, token, pos, write_logits);
    MCPM_CUDA(launch_decode(p, e->n_ctas, e->stream));
    return MCPM_OK;
}

}  // namespace

extern "C" {

const char* mcpm_status_string(mcpm_status s) {
    switch (s) {
        case MCPM_OK: return "ok";
        case MCPM_BAD_ARG: return "bad argument";
        case MCPM_BAD_FILE: return "bad or unsupported model file";
        case MCPM_UNSUPPORTED_TYPE: return "unsupported tensor type";
        case MCPM_CTX_OVERFLOW: return "position beyond the KV cache";
        case MCPM_CUDA_ERROR: return "CUDA error";
        case MCPM_NCCL_ERROR: return "NCCL error";
        case MCPM_TIMEOUT: return "device wait timed out";
        case MCPM_OUT_OF_MEMORY: return "out of device memory";
        case MCPM_BAD_TOKEN: return "token id out of range";
        case MCPM_NOT_LOADED: return "model or KV cache not loaded";
    }
    return "unknown status";
}

mcpm_status mcpm_engine_create(const mcpm_config* cfg, mcpm_engine** out) {
    if (!cfg || !out) return MCPM_BAD_ARG;
    *out = nullptr;
    if (cfg->max_seq < 0 || cfg->max_seq > MAX_SEQ || cfg->n_ctas < 0) return MCPM_BAD_ARG;
    if (cfg->batch_gemm != MCPM_GEMM_MMA && cfg->batch_gemm != MCPM_GEMM_TCGEN05) return MCPM_BAD_ARG;
    if (cfg->kv_type != MCPM_KV_F32 && cfg->kv_type != MCPM_KV_F16) return MCPM_BAD_ARG;
    int ndev = 0;
    MCPM_CUDA(cudaGetDeviceCount(&ndev));
    if (cfg->device < 0 || cfg->device >= ndev) return MCPM_BAD_ARG;
    auto e = std::make_unique<mcpm_engine>();
    e->device = cfg->device;
    e->req_ctas = cfg->n_ctas;
    e->batch_gemm = cfg->batch_gemm;
    e->sched = cfg->sched;
    e->kv_f16 = cfg->kv_type == MCPM_KV_F16;
    e->max_seq = 0;
    MCPM_CUDA(cudaSetDevice(e->device));
    MCPM_CUDA(cudaDeviceGetAttribute(&e->n_sm, cudaDevAttrMultiProcessorCount, e->device));
    int coop = 0;
    MCPM_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, e->device));
    if (!coop) return MCPM_CUDA_ERROR;
    MCPM_CUDA(decode_prepare());
    const int per_sm = decode_max_ctas_per_sm();
    if (per_sm < 1) return MCPM_CUDA_ERROR;
    e->n_ctas = e->n_sm;   // one persistent CTA per SM
    if (cfg->n_ctas > 0) e->n_ctas = std::min(cfg->n_ctas, e->n_sm * per_sm);
    MCPM_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    MCPM_CUDA(cudaMalloc(&e->ctl, CTL_WORDS * sizeof(int)));
    MCPM_CUDA(cudaMallocHost(&e->ctl_host, CTL_WORDS * sizeof(int)));
    const mcpm_status st = reset_ctl(e.get());
    if (st != MCPM_OK) return st;
    e->max_seq = cfg->max_seq;   // allocated at load
    *out = e.release();
    return MCPM_OK;
}

mcpm_status mcpm_load_gguf(mcpm_engine* e, const char* path) {
    if (!e || !path) return MCPM_BAD_ARG;
    MCPM_CUDA(cudaSetDevice(e->device));
    free_model(e);
    GGUFFile g;
    const std::string why = gguf_read(path, g);
    if (!why.empty()) {
        std::fprintf(stderr, "[mcpm] %s\n", why.c_str());
        return MCPM_BAD_FILE;
    }
    auto find = [&](const std::string& name) -> const GGUFTensor* {
        for (const auto& t : g.tensors)
            if (t.name == name) return &t;
        return nullptr;
    };
    int n_layer = 0;
    while (find("blk." + std::to_string(n_layer) + ".attn_q.weight")) ++n_layer;
    const GGUFTensor* emb = find("token_embd.weight");
    const GGUFTensor* onorm = find("output_norm.weight");
    const GGUFTensor* out = find("output.weight");
    if (n_layer == 0 || n_layer > MAX_LAYERS || !emb || !onorm || !out) {
        std::fprintf(stderr, "[mcpm] missing MiniCPM5 tensors in %s\n", path);
        return MCPM_BAD_FILE;
    }
    auto dims_are = [](const GGUFTensor* t, uint64_t c, uint64_t r) {
        return t->dims.size() >= 1 && t->dims[0] == c && (r == 0 ? t->dims.size() == 1 : t->dims.size() == 2 && t->dims[1] == r);
    };
    const uint64_t vocab = emb->dims.size() == 2 ? emb->dims[1] : 0;
    if (!dims_are(emb, N_EMBD, vocab) || !dims_are(out, N_EMBD, vocab) || !dims_are(onorm, N_EMBD, 0) || vocab == 0 ||
        vocab > (1u << 30)) {
        std::fprintf(stderr, "[mcpm] unexpected embedding / output shapes\n");
        return MCPM_BAD_FILE;
    }
    if (emb->type != GGML_Q4_K || (out->type != GGML_Q4_K && out->type != GGML_Q6_K) || onorm->type != GGML_F32) {
        std::fprintf(stderr, "[mcpm] embedding/output types %u/%u not handled by the decode kernel\n", emb->type,
                     out->type);
        return MCPM_UNSUPPORTED_TYPE;
    }
    // Arena: [first tensor byte, end of file) uploaded unchanged.
    uint64_t lo = ~0ull, hi = 0;
    for (const auto& t : g.tensors) {
        if (!t.nbytes) continue;
        lo = std::min(lo, t.offset);
        hi = std::max(hi, t.offset + t.nbytes);
    }
    e->arena_base = lo;
    e->arena_bytes = hi - lo;
    if (e->arena_bytes >= (1ull << 32)) {   // the decode kernel addresses tensors by 32-bit arena offsets
        std::fprintf(stderr, "[mcpm] weight arena of %llu bytes exceeds 4 GiB\n", (unsigned long long)e->arena_bytes);
        return MCPM_UNSUPPORTED_TYPE;
    }
    MCPM_CUDA(cudaMalloc(&e->arena, e->arena_bytes + 256));
    {
        std::unique_ptr<FILE, int (*)(FILE*)> f(std::fopen(path, "rb"), &std::fclose);
        if (!f) return MCPM_BAD_FILE;
        const size_t CH = 64ull << 20;
        uint8_t* pin[2] = {nullptr, nullptr};
        MCPM_CUDA(cudaMallocHost(&pin[0], CH));
        MCPM_CUDA(cudaMallocHost(&pin[1], CH));
        cudaEvent_t ev[2];
        cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming);
        cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming);
        std::fseek(f.get(), static_cast<long>(lo), SEEK_SET);
        uint64_t done = 0;
        int k = 0;
        bool io_ok = true;
        while (done < e->arena_bytes) {
            const size_t n = static_cast<size_t>(std::min<uint64_t>(CH, e->arena_bytes - done));
            cudaEventSynchronize(ev[k]);
            if (std::fread(pin[k], 1, n, f.get()) != n) {
                io_ok = false;
                break;
            }
            cudaMemcpyAsync(e->arena + done, pin[k], n, cudaMemcpyHostToDevice, e->stream);
            cudaEventRecord(ev[k], e->stream);
            done += n;
            k ^= 1;
        }
        cudaStreamSynchronize(e->stream);
        cudaEventDestroy(ev[0]);
        cudaEventDestroy(ev[1]);
        cudaFreeHost(pin[0]);
        cudaFreeHost(pin[1]);
        if (!io_ok) return MCPM_BAD_FILE;
        MCPM_CUDA(cudaGetLastError());
    }
    auto dev = [&](const GGUFTensor* t) { return e->arena + (t->offset - lo); };
    e->layers.assign(n_layer, LayerDev{});
    for (int l = 0; l < n_layer; ++l) {
        const GGUFTensor* t[9];
        for (int i = 0; i < 9; ++i) {
            t[i] = find("blk." + std::to_string(l) + "." + LAYER_NAMES[i] + ".weight");
            if (!t[i]) {
                std::fprintf(stderr, "[mcpm] layer %d lacks %s\n", l, LAYER_NAMES[i]);
                return MCPM_BAD_FILE;
            }
        }
        const bool shapes = dims_are(t[0], N_EMBD, N_EMBD) && dims_are(t[1], N_EMBD, KV_DIM) &&
                            dims_are(t[2], N_EMBD, KV_DIM) && dims_are(t[3], N_EMBD, N_EMBD) &&
                            dims_are(t[4], N_EMBD, N_FF) && dims_are(t[5], N_EMBD, N_FF) &&
                            dims_are(t[6], N_FF, N_EMBD) && dims_are(t[7], N_EMBD, 0) && dims_are(t[8], N_EMBD, 0);
        if (!shapes) {
            std::fprintf(stderr, "[mcpm] layer %d has unexpected shapes\n", l);
            return MCPM_BAD_FILE;
        }
        for (int i = 0; i < 7; ++i)
            if (t[i]->type != GGML_Q4_K && t[i]->type != GGML_Q6_K) {
                std::fprintf(stderr, "[mcpm] layer %d %s has type %u (decode kernel: Q4_K / Q6_K)\n", l,
                             LAYER_NAMES[i], t[i]->type);
                return MCPM_UNSUPPORTED_TYPE;
            }
        if (t[7]->type != GGML_F32 || t[8]->type != GGML_F32) return MCPM_UNSUPPORTED_TYPE;
        LayerDev& L = e->layers[l];
        L.wq = dev(t[0]), L.wk = dev(t[1]), L.wv = dev(t[2]), L.wo = dev(t[3]);
        L.wg = dev(t[4]), L.wu = dev(t[5]), L.wd = dev(t[6]);
        L.attn_norm = reinterpret_cast<const float*>(dev(t[7]));
        L.ffn_norm = reinterpret_cast<const float*>(dev(t[8]));
        L.tq = t[0]->type, L.tk = t[1]->type, L.tv = t[2]->type, L.to = t[3]->type;
        L.tg = t[4]->type, L.tu = t[5]->type, L.td = t[6]->type;
    }
    for (const auto& t : g.tensors)
        if ((t.offset - lo) % 16) return MCPM_BAD_FILE;   // TMA copies need 16-byte aligned rows
    e->n_layer = n_layer;
    e->n_vocab = static_cast<int>(vocab);
    e->embd = dev(emb);
    e->embd_type = emb->type;
    e->out_norm = reinterpret_cast<const float*>(dev(onorm));
    e->lm = dev(out);
    e->lm_type = out->type;
    auto fb = g.f_kv.find("minicpm5.rope.freq_base");
    if (fb != g.f_kv.end()) e->rope_base = static_cast<float>(fb->second);
    std::string why2;
    if (!phases_fit(e, e->n_ctas, why2)) {
        std::fprintf(stderr, "[mcpm] %s\n", why2.c_str());
        return MCPM_UNSUPPORTED_TYPE;
    }
    MCPM_CUDA(cudaMalloc(&e->d_layers, sizeof(LayerDev) * n_layer));
    MCPM_CUDA(cudaMemcpy(e->d_layers, e->layers.data(), sizeof(LayerDev) * n_layer, cudaMemcpyHostToDevice));
    MCPM_CUDA(cudaMalloc(&e->x, N_EMBD * 4));
    MCPM_CUDA(cudaMalloc(&e->q, N_EMBD * 4));
    MCPM_CUDA(cudaMalloc(&e->att, N_EMBD * 4));
    MCPM_CUDA(cudaMalloc(&e->h, N_FF * 4));
    MCPM_CUDA(cudaMalloc(&e->xll, XLL_COPIES * N_EMBD * sizeof(unsigned long long)));
    MCPM_CUDA(cudaMemset(e->xll, 0, XLL_COPIES * N_EMBD * sizeof(unsigned long long)));
    MCPM_CUDA(cudaMalloc(&e->qll, (N_EMBD + 2 * KV_DIM) * sizeof(unsigned long long)));
    MCPM_CUDA(cudaMemset(e->qll, 0, (N_EMBD + 2 * KV_DIM) * sizeof(unsigned long long)));
    MCPM_CUDA(cudaMalloc(&e->attw, ATTW_COPIES * N_EMBD * sizeof(unsigned long long)));
    MCPM_CUDA(cudaMemset(e->attw, 0, ATTW_COPIES * N_EMBD * sizeof(unsigned long long)));
    MCPM_CUDA(cudaMalloc(&e->att_part, ATT_PART_FLOATS * sizeof(float)));
    MCPM_CUDA(cudaMemset(e->att_part, 0, ATT_PART_FLOATS * sizeof(float)));
    MCPM_CUDA(cudaMalloc(&e->logits, sizeof(float) * e->n_vocab));
    MCPM_CUDA(cudaMalloc(&e->am_val, sizeof(float) * e->n_ctas));
    MCPM_CUDA(cudaMalloc(&e->am_idx, sizeof(int) * e->n_ctas));
    MCPM_CUDA(cudaMalloc(&e->att_q8k, Q8K_BYTES * (N_EMBD / 256)));
    MCPM_CUDA(cudaMemset(e->logits, 0, sizeof(float) * e->n_vocab));
    e->gguf = std::move(g);
    e->loaded = true;
    if (e->max_seq > 0) return mcpm_init_kv(e, e->max_seq);
    return MCPM_OK;
}

mcpm_status mcpm_init_kv(mcpm_engine* e, int max_seq) {
    if (!e) return MCPM_BAD_ARG;
    if (max_seq <= 0 || max_seq > MAX_SEQ) return MCPM_BAD_ARG;
    if (!e->loaded) {
        e->max_seq = max_seq;   // applied at load
        return MCPM_OK;
    }
    MCPM_CUDA(cudaSetDevice(e->device));
    free_kv(e);
    const size_t n = static_cast<size_t>(e->n_layer) * max_seq * KV_DIM;
    MCPM_CUDA(cudaMalloc(&e->kc, n * e->kv_elt()));
    MCPM_CUDA(cudaMalloc(&e->vc, n * e->kv_elt()));
    MCPM_CUDA(cudaMemset(e->kc, 0, n * e->kv_elt()));
    MCPM_CUDA(cudaMemset(e->vc, 0, n * e->kv_elt()));
    std::vector<float2> table(static_cast<size_t>(max_seq) * (HEAD_DIM / 2));
    for (int p = 0; p < max_seq; ++p) rope_row(p, e->rope_base, table.data() + static_cast<size_t>(p) * (HEAD_DIM / 2));
    MCPM_CUDA(cudaMalloc(&e->rope, table.size() * sizeof(float2)));
    MCPM_CUDA(cudaMemcpy(e->rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice));
    e->max_seq = max_seq;
    return MCPM_OK;
}

mcpm_status mcpm_forward(mcpm_engine* e, int token, int pos, float* logits_out, int* argmax_out) {
    if (!e) return MCPM_BAD_ARG;
    mcpm_status st = launch(e, token, pos, logits_out != nullptr);
    if (st != MCPM_OK) return st;
    if (logits_out)
        MCPM_CUDA(cudaMemcpyAsync(logits_out, e->logits, sizeof(float) * e->n_vocab, cudaMemcpyDeviceToHost, e->stream));
    st = check_ctl(e);
    if (st != MCPM_OK) return st;
    if (argmax_out) *argmax_out = e->ctl_host[CTL_ARGMAX];
    return MCPM_OK;
}

mcpm_status mcpm_forward_async(mcpm_engine* e, int token, int pos, int write_logits) {
    return launch(e, token, pos, write_logits);
}

mcpm_status mcpm_sync(mcpm_engine* e) {
    if (!e) return MCPM_BAD_ARG;
    MCPM_CUDA(cudaSetDevice(e->device));
    return check_ctl(e);
}

const float* mcpm_logits_device(mcpm_engine* e) { return e ? e->logits : nullptr; }
const int* mcpm_argmax_device(mcpm_engine* e) { return e ? e->ctl + CTL_ARGMAX : nullptr; }

mcpm_status mcpm_read_x(mcpm_engine* e, float* x_host) {
    if (!e || !x_host) return MCPM_BAD_ARG;
    if (!e->loaded) return MCPM_NOT_LOADED;
    MCPM_CUDA(cudaSetDevice(e->device));
    MCPM_CUDA(cudaMemcpyAsync(x_host, e->x, N_EMBD * 4, cudaMemcpyDeviceToHost, e->stream));
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    return MCPM_OK;
}

mcpm_status mcpm_read_kv(mcpm_engine* e, int layer, int pos, float* k_host, float* v_host) {
    if (!e || !k_host || !v_host) return MCPM_BAD_ARG;
    if (!e->loaded || !e->kc) return MCPM_NOT_LOADED;
    if (layer < 0 || layer >= e->n_layer || pos < 0 || pos >= e->max_seq) return MCPM_BAD_ARG;
    MCPM_CUDA(cudaSetDevice(e->device));
    const size_t off = (static_cast<size_t>(layer) * e->max_seq + pos) * KV_DIM;
    if (!e->kv_f16) {
        MCPM_CUDA(cudaMemcpyAsync(k_host, e->kc + off, KV_DIM * 4, cudaMemcpyDeviceToHost, e->stream));
        MCPM_CUDA(cudaMemcpyAsync(v_host, e->vc + off, KV_DIM * 4, cudaMemcpyDeviceToHost, e->stream));
        MCPM_CUDA(cudaStreamSynchronize(e->stream));
        return MCPM_OK;
    }
    std::vector<__half> h(2 * KV_DIM);   // fp16 rows widen exactly to fp32
    MCPM_CUDA(cudaMemcpyAsync(h.data(), e->kv_at(e->kc, off), KV_DIM * 2, cudaMemcpyDeviceToHost, e->stream));
    MCPM_CUDA(cudaMemcpyAsync(h.data() + KV_DIM, e->kv_at(e->vc, off), KV_DIM * 2, cudaMemcpyDeviceToHost, e->stream));
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < KV_DIM; ++i) k_host[i] = __half2float(h[i]), v_host[i] = __half2float(h[KV_DIM + i]);
    return MCPM_OK;
}

mcpm_status mcpm_write_kv(mcpm_engine* e, int layer, int pos0, int n_pos, const float* k_host, const float* v_host) {
    if (!e || !k_host || !v_host) return MCPM_BAD_ARG;
    if (!e->loaded || !e->kc) return MCPM_NOT_LOADED;
    if (layer < 0 || layer >= e->n_layer || pos0 < 0 || n_pos < 0 || pos0 > e->max_seq - n_pos) return MCPM_BAD_ARG;
    MCPM_CUDA(cudaSetDevice(e->device));
    const size_t off = (static_cast<size_t>(layer) * e->max_seq + pos0) * KV_DIM;
    const size_t n = static_cast<size_t>(n_pos) * KV_DIM;
    if (!e->kv_f16) {
        MCPM_CUDA(cudaMemcpyAsync(e->kc + off, k_host, n * 4, cudaMemcpyHostToDevice, e->stream));
        MCPM_CUDA(cudaMemcpyAsync(e->vc + off, v_host, n * 4, cudaMemcpyHostToDevice, e->stream));
        MCPM_CUDA(cudaStreamSynchronize(e->stream));
        return MCPM_OK;
    }
    std::vector<__half> h(2 * n);   // rounded to nearest-even, as the decode step rounds the rows it writes
    for (size_t i = 0; i < n; ++i) h[i] = __float2half_rn(k_host[i]), h[n + i] = __float2half_rn(v_host[i]);
    MCPM_CUDA(cudaMemcpyAsync(e->kv_at(e->kc, off), h.data(), n * 2, cudaMemcpyHostToDevice, e->stream));
    MCPM_CUDA(cudaMemcpyAsync(e->kv_at(e->vc, off), h.data() + n, n * 2, cudaMemcpyHostToDevice, e->stream));
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    return MCPM_OK;
}

// Session snapshot: positions [0, n_pos) of every layer, [layer][K then V][pos][KV_DIM] fp32.
size_t mcpm_kv_snapshot_bytes(mcpm_engine* e, int n_pos) {
    if (!e || !e->loaded || n_pos < 0) return 0;
    return static_cast<size_t>(e->n_layer) * 2 * n_pos * KV_DIM * e->kv_elt();
}

namespace {
mcpm_status kv_copy(mcpm_engine* e, int n_pos, void* host, size_t bytes, bool to_host) {
    if (!e || !host || n_pos < 0) return MCPM_BAD_ARG;
    if (!e->loaded || !e->kc) return MCPM_NOT_LOADED;
    if (n_pos > e->max_seq) return MCPM_CTX_OVERFLOW;
    const size_t per = static_cast<size_t>(n_pos) * KV_DIM * e->kv_elt();
    if (bytes < static_cast<size_t>(e->n_layer) * 2 * per) return MCPM_BAD_ARG;
    MCPM_CUDA(cudaSetDevice(e->device));
    uint8_t* h = static_cast<uint8_t*>(host);
    for (int l = 0; l < e->n_layer; ++l) {   // one copy per layer and per K / V
        const size_t lo = static_cast<size_t>(l) * e->max_seq * KV_DIM;
        uint8_t* dev[2] = {e->kv_at(e->kc, lo), e->kv_at(e->vc, lo)};
        for (int kv = 0; kv < 2; ++kv) {
            uint8_t* hp = h + (2 * static_cast<size_t>(l) + kv) * per;
            if (to_host)
                MCPM_CUDA(cudaMemcpyAsync(hp, dev[kv], per, cudaMemcpyDeviceToHost, e->stream));
            else
                MCPM_CUDA(cudaMemcpyAsync(dev[kv], hp, per, cudaMemcpyHostToDevice, e->stream));
        }
    }
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    return MCPM_OK;
}
}  // namespace

mcpm_status mcpm_kv_snapshot(mcpm_engine* e, int n_pos, void* host, size_t bytes) {
    return kv_copy(e, n_pos, host, bytes, true);
}

mcpm_status mcpm_kv_restore(mcpm_engine* e, int n_pos, const void* host, size_t bytes) {
    return kv_copy(e, n_pos, const_cast<void*>(host), bytes, false);
}

mcpm_status mcpm_model_dims(mcpm_engine* e, int dims[6]) {
    if (!e || !dims) return MCPM_BAD_ARG;
    if (!e->loaded) return MCPM_NOT_LOADED;
    dims[0] = e->n_layer, dims[1] = N_EMBD, dims[2] = N_FF, dims[3] = N_HEAD, dims[4] = N_HEAD_KV;
    dims[5] = e->n_vocab;
    return MCPM_OK;
}

mcpm_status mcpm_trace_enable(mcpm_engine* e, int enable) {
    if (!e) return MCPM_BAD_ARG;
    MCPM_CUDA(cudaSetDevice(e->device));
    if (enable && !e->trace) {
        MCPM_CUDA(cudaMalloc(&e->trace, TRACE_WORDS * sizeof(unsigned long long)));
        MCPM_CUDA(cudaMemset(e->trace, 0, TRACE_WORDS * sizeof(unsigned long long)));
    } else if (!enable) {
        MCPM_CUDA(cudaStreamSynchronize(e->stream));
        free_dev(e->trace);
    }
    return MCPM_OK;
}

mcpm_status mcpm_trace_read(mcpm_engine* e, unsigned long long* out, int n) {
    if (!e || !out || n <= 0) return MCPM_BAD_ARG;
    if (!e->trace) return MCPM_NOT_LOADED;
    MCPM_CUDA(cudaSetDevice(e->device));
    MCPM_CUDA(cudaMemcpyAsync(out, e->trace, sizeof(unsigned long long) * std::min(n, TRACE_WORDS),
                              cudaMemcpyDeviceToHost, e->stream));
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    return MCPM_OK;
}

void* mcpm_engine_stream(mcpm_engine* e) { return e ? reinterpret_cast<void*>(e->stream) : nullptr; }
int mcpm_engine_n_ctas(mcpm_engine* e) { return e ? e->n_ctas : 0; }

void mcpm_engine_destroy(mcpm_engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    free_batch(e);
    free_kv(e);
    free_model(e);
    free_dev(e->ctl);
    free_dev(e->trace);
    if (e->ctl_host) cudaFreeHost(e->ctl_host);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

// ------------------------------------------------------------------ sampler
namespace {
struct SampleWorkspace {
    int n = 0;
    float* staged = nullptr;   // host logits copied in by mcpm_sample_top_p_host
    float* p = nullptr;
    uint32_t* gk = nullptr;
    int* gi = nullptr;
    int* out = nullptr;
};
SampleWorkspace g_sample_ws[64];

mcpm_status sample_workspace(int n, SampleWorkspace*& ws) {
    int dev = 0;
    MCPM_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return MCPM_BAD_ARG;
    ws = &g_sample_ws[dev];
    if (ws->n < n) {
        free_dev(ws->staged);
        free_dev(ws->p);
        free_dev(ws->gk);
        free_dev(ws->gi);
        free_dev(ws->out);
        ws->n = 0;
        MCPM_CUDA(cudaMalloc(&ws->staged, sizeof(float) * n));
        MCPM_CUDA(cudaMalloc(&ws->p, sizeof(float) * n));
        MCPM_CUDA(cudaMalloc(&ws->gk, sizeof(uint32_t) * 2 * n));
        MCPM_CUDA(cudaMalloc(&ws->gi, sizeof(int) * 2 * n));
        MCPM_CUDA(cudaMalloc(&ws->out, sizeof(int) * 2));
        ws->n = n;
    }
    return MCPM_OK;
}
}  // namespace

mcpm_status mcpm_sample_top_p(const float* logits, int n, float temperature, float top_p, float r, int* out,
                              void* stream) {
    if (!logits || !out || n <= 0 || n > (1 << 20)) return MCPM_BAD_ARG;
    SampleWorkspace* ws = nullptr;
    mcpm_status st = sample_workspace(n, ws);
    if (st != MCPM_OK) return st;
    return cuda_status(launch_sample_top_p(logits, n, temperature, top_p, r, out, ws->p, ws->gk, ws->gi,
                                           static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_sample_top_p_host(const float* logits, int n, float temperature, float top_p, float r,
                                   int* token_out) {
    if (!logits || !token_out || n <= 0 || n > (1 << 20)) return MCPM_BAD_ARG;
    SampleWorkspace* ws = nullptr;
    mcpm_status st = sample_workspace(n, ws);
    if (st != MCPM_OK) return st;
    MCPM_CUDA(cudaMemcpy(ws->staged, logits, sizeof(float) * n, cudaMemcpyHostToDevice));
    MCPM_CUDA(launch_sample_top_p(ws->staged, n, temperature, top_p, r, ws->out, ws->p, ws->gk, ws->gi, nullptr));
    MCPM_CUDA(cudaMemcpy(token_out, ws->out, sizeof(int), cudaMemcpyDeviceToHost));
    return MCPM_OK;
}

mcpm_status mcpm_rope_kv_append(float* q, float* k, const float* v, float* kcache, float* vcache, int pos, int max_seq,
                                float rope_base, void* stream) {
    if (!q || !k || !v || !kcache || !vcache || max_seq <= 0 || !(rope_base > 0.0f)) return MCPM_BAD_ARG;
    if (pos < 0 || pos >= max_seq) return MCPM_CTX_OVERFLOW;
    return cuda_status(op_rope_kv_append(q, k, v, kcache, vcache, pos, rope_base, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_sample(mcpm_engine* e, float temperature, float top_p, float r, int* token_out) {
    if (!e) return MCPM_BAD_ARG;
    if (!e->loaded) return MCPM_NOT_LOADED;
    MCPM_CUDA(cudaSetDevice(e->device));
    SampleWorkspace* ws = nullptr;
    mcpm_status st = sample_workspace(e->n_vocab, ws);
    if (st != MCPM_OK) return st;
    MCPM_CUDA(launch_sample_top_p(e->logits, e->n_vocab, temperature, top_p, r, ws->out, ws->p, ws->gk, ws->gi,
                                  e->stream));
    MCPM_CUDA(cudaMemcpyAsync(e->ctl + CTL_TOKEN, ws->out, sizeof(int), cudaMemcpyDeviceToDevice, e->stream));
    if (token_out) {
        MCPM_CUDA(cudaMemcpyAsync(token_out, ws->out, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
        MCPM_CUDA(cudaStreamSynchronize(e->stream));
    }
    return MCPM_OK;
}

// ------------------------------------------------------------------ batched decode
mcpm_status mcpm_batch_init(mcpm_engine* e, int n_seq, int max_seq) {
    if (!e || n_seq <= 0 || n_seq > BATCH_MAX || max_seq <= 0 || max_seq > MAX_SEQ) return MCPM_BAD_ARG;
    if (!e->loaded) return MCPM_NOT_LOADED;
    MCPM_CUDA(cudaSetDevice(e->device));
    MCPM_CUDA(cudaStreamSynchronize(e->stream));
    free_batch(e);
    if (const mcpm_status st = ensure_gemm_scratch(e); st != MCPM_OK) return st;
    const size_t kv = static_cast<size_t>(n_seq) * e->n_layer * max_seq * KV_DIM;
    auto alloc = [&](auto** ptr, size_t bytes) -> cudaError_t {
        cudaError_t err = cudaMalloc(reinterpret_cast<void**>(ptr), bytes);
        if (err == cudaSuccess) err = cudaMemset(*ptr, 0, bytes);
        return err;
    };
    const size_t ns = n_seq;
    cudaError_t err = cudaSuccess;
    for (auto& [ptr, bytes] : std::initializer_list<std::pair<float**, size_t>>{
             {&e->b_kc, kv * e->kv_elt()}, {&e->b_vc, kv * e->kv_elt()}, {&e->b_x, ns * N_EMBD * 4}, {&e->b_y, ns * 2 * N_FF * 4},
             {&e->b_q, ns * N_EMBD * 4}, {&e->b_part, ns * ATT_PART_FLOATS * 4}, {&e->b_att, ns * N_EMBD * 4},
             {&e->b_logits, ns * e->n_vocab * 4}})
        if (err == cudaSuccess) err = alloc(ptr, bytes);
    if (err == cudaSuccess) err = alloc(&e->b_aqs, ns * (N_FF / 256) * 256);
    if (err == cudaSuccess) err = alloc(&e->b_ad, ns * (N_FF / 256) * 4);
    if (err == cudaSuccess) err = alloc(&e->b_abs, ns * (N_FF / 256) * 16 * 2);
    if (err == cudaSuccess) err = alloc(&e->b_tokens, ns * 4);
    if (err == cudaSuccess) err = alloc(&e->b_pos, ns * 4);
    if (err == cudaSuccess) err = alloc(&e->b_argmax, ns * 4);
    if (err == cudaSuccess) {
        std::vector<float2> table(static_cast<size_t>(max_seq) * (HEAD_DIM / 2));
        for (int p = 0; p < max_seq; ++p) rope_row(p, e->rope_base, table.data() + static_cast<size_t>(p) * (HEAD_DIM / 2));
        err = cudaMalloc(&e->b_rope, table.size() * sizeof(float2));
        if (err == cudaSuccess)
            err = cudaMemcpy(e->b_rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice);
    }
    if (err != cudaSuccess) {
        free_batch(e);
        return cuda_status(err);
    }
    e->b_n = n_seq;
    e->b_max_seq = max_seq;
    e->b_pos_host.assign(n_seq, 0);
    return MCPM_OK;
}

mcpm_status mcpm_batch_step_async(mcpm_engine* e, const int* tokens, const int* pos) {
    if (!e) return MCPM_BAD_ARG;
    if (!e->loaded || e->b_n == 0) return MCPM_NOT_LOADED;
    const int n = e->b_n;
    if (tokens)
        for (int i = 0; i < n; ++i)
            if (tokens[i] < 0 || tokens[i] >= e->n_vocab) return MCPM_BAD_TOKEN;
    std::vector<int> next = pos ? std::vector<int>(pos, pos + n) : e->b_pos_host;
    int max_pos = 0;
    for (int i = 0; i < n; ++i) {
        if (next[i] < 0 || next[i] >= e->b_max_seq) return MCPM_CTX_OVERFLOW;
        max_pos = std::max(max_pos, next[i]);
    }
    MCPM_CUDA(cudaSetDevice(e->device));
    if (tokens) MCPM_CUDA(cudaMemcpyAsync(e->b_tokens, tokens, n * sizeof(int), cudaMemcpyHostToDevice, e->stream));
    if (pos) MCPM_CUDA(cudaMemcpyAsync(e->b_pos, pos, n * sizeof(int), cudaMemcpyHostToDevice, e->stream));
    BatchLaunch b{};
    b.n_seq = n, b.max_seq = e->b_max_seq, b.n_layer = e->n_layer, b.n_vocab = e->n_vocab, b.lm_type = e->lm_type;
    b.max_pos = max_pos, b.chain = 1, b.n_sm = e->n_sm, b.tcgen05 = e->batch_gemm == MCPM_GEMM_TCGEN05;
    b.kv_f16 = e->kv_f16;
    b.gemm_part = e->g_part, b.gemm_cnt = e->g_cnt, b.trace = e->trace;
    b.layers = e->layers.data(), b.embd = e->embd, b.out_norm = e->out_norm, b.lm = e->lm, b.rope = e->b_rope;
    b.kc = e->b_kc, b.vc = e->b_vc, b.x = e->b_x, b.y = e->b_y, b.q = e->b_q, b.att_part = e->b_part;
    b.att = e->b_att, b.logits = e->b_logits, b.aqs = e->b_aqs, b.ad = e->b_ad, b.abs = e->b_abs;
    b.tokens = e->b_tokens, b.pos = e->b_pos, b.argmax = e->b_argmax;
    b.err = reinterpret_cast<unsigned*>(e->ctl + CTL_ERR);
    MCPM_CUDA(launch_batch_step(b, e->stream));
    for (int i = 0; i < n; ++i) next[i] += 1;   // the argmax kernel advances the device copy the same way
    e->b_pos_host = next;
    return MCPM_OK;
}

// ------------------------------------------------------------------ batched prefill
mcpm_status mcpm_prefill(mcpm_engine* e, const int* tokens, int n, int pos0, float* logits_out, int* argmax_out) {
    if (!e || !tokens || n <= 0 || pos0 < 0) return MCPM_BAD_ARG;
    if (!e->loaded || !e->kc) return MCPM_NOT_LOADED;
    if (pos0 + n > e->max_seq) return MCPM_CTX_OVERFLOW;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= e->n_vocab) return MCPM_BAD_TOKEN;
    MCPM_CUDA(cudaSetDevice(e->device));
    if (!e->p_x) {   // row buffers of BATCH_MAX positions, kept until the model is unloaded
        const size_t ns = BATCH_MAX;
        auto alloc = [&](auto** ptr, size_t bytes) { return cudaMalloc(reinterpret_cast<void**>(ptr), bytes); };
        cudaError_t err = cudaSuccess;
        for (auto& [ptr, bytes] : std::initializer_list<std::pair<float**, size_t>>{
                 {&e->p_x, ns * N_EMBD * 4}, {&e->p_y, ns * 2 * N_FF * 4}, {&e->p_q, ns * N_EMBD * 4},
                 {&e->p_part, ns * ATT_PART_FLOATS * 4}, {&e->p_att, ns * N_EMBD * 4},
                 {&e->p_logits, ns * e->n_vocab * 4}})
            if (err == cudaSuccess) err = alloc(ptr, bytes);
        if (err == cudaSuccess) err = alloc(&e->p_aqs, ns * (N_FF / 256) * 256);
        if (err == cudaSuccess) err = alloc(&e->p_ad, ns * (N_FF / 256) * 4);
        if (err == cudaSuccess) err = alloc(&e->p_abs, ns * (N_FF / 256) * 16 * 2);
        if (err == cudaSuccess) err = alloc(&e->p_tokens, ns * 4);
        if (err == cudaSuccess) err = alloc(&e->p_pos, ns * 4);
        if (err == cudaSuccess) err = alloc(&e->p_argmax, ns * 4);
        if (err != cudaSuccess) {
            free_prefill(e);
            return cuda_status(err);
        }
    }
    if (const mcpm_status st = ensure_gemm_scratch(e); st != MCPM_OK) return st;
    std::vector<int> pos(BATCH_MAX);
    for (int done = 0; done < n;) {
        const int m = std::min(BATCH_MAX, n - done);
        const bool last = done + m == n;
        for (int i = 0; i < m; ++i) pos[i] = pos0 + done + i;
        MCPM_CUDA(cudaMemcpyAsync(e->p_tokens, tokens + done, m * sizeof(int), cudaMemcpyHostToDevice, e->stream));
        MCPM_CUDA(cudaMemcpyAsync(e->p_pos, pos.data(), m * sizeof(int), cudaMemcpyHostToDevice, e->stream));
        BatchLaunch b{};
        b.n_seq = m, b.max_seq = e->max_seq, b.n_layer = e->n_layer, b.n_vocab = e->n_vocab, b.lm_type = e->lm_type;
        b.max_pos = pos[m - 1], b.chain = 0, b.n_sm = e->n_sm, b.tcgen05 = e->batch_gemm == MCPM_GEMM_TCGEN05;
        b.shared_kv = 1, b.skip_lm = last ? 0 : 1, b.kv_f16 = e->kv_f16;
        b.gemm_part = e->g_part, b.gemm_cnt = e->g_cnt;
        b.layers = e->layers.data(), b.embd = e->embd, b.out_norm = e->out_norm, b.lm = e->lm, b.rope = e->rope;
        b.kc = e->kc, b.vc = e->vc, b.x = e->p_x, b.y = e->p_y, b.q = e->p_q, b.att_part = e->p_part;
        b.att = e->p_att, b.aqs = e->p_aqs, b.ad = e->p_ad, b.abs = e->p_abs;
        b.logits = e->p_logits;   // [m][n_vocab]: the LM head runs on the last chunk only
        b.tokens = e->p_tokens, b.pos = e->p_pos, b.argmax = e->p_argmax;
        b.err = reinterpret_cast<unsigned*>(e->ctl + CTL_ERR);
        MCPM_CUDA(launch_batch_step(b, e->stream));
        done += m;
        if (last) {
            // the last position's logits and greedy token, where a decode step leaves them, so
            // mcpm_sample / mcpm_forward(token < 0) continue from the prompt
            MCPM_CUDA(cudaMemcpyAsync(e->logits, e->p_logits + static_cast<size_t>(m - 1) * e->n_vocab,
                                      static_cast<size_t>(e->n_vocab) * 4, cudaMemcpyDeviceToDevice, e->stream));
            MCPM_CUDA(cudaMemcpyAsync(e->ctl + CTL_ARGMAX, e->p_argmax + (m - 1), sizeof(int), cudaMemcpyDeviceToDevice,
                                      e->stream));
            MCPM_CUDA(cudaMemcpyAsync(e->ctl + CTL_TOKEN, e->p_argmax + (m - 1), sizeof(int), cudaMemcpyDeviceToDevice,
                                      e->stream));
        }
    }
    if (logits_out)
        MCPM_CUDA(cudaMemcpyAsync(logits_out, e->logits, static_cast<size_t>(e->n_vocab) * 4, cudaMemcpyDeviceToHost,
                                  e->stream));
    if (argmax_out) MCPM_CUDA(cudaMemcpyAsync(argmax_out, e->ctl + CTL_ARGMAX, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    return check_ctl(e);
}

mcpm_status mcpm_batch_read(mcpm_engine* e, float* logits, int* argmax) {
    if (!e) return MCPM_BAD_ARG;
    if (!e->loaded || e->b_n == 0) return MCPM_NOT_LOADED;
    MCPM_CUDA(cudaSetDevice(e->device));
    const size_t n = e->b_n;
    if (logits)
        MCPM_CUDA(cudaMemcpyAsync(logits, e->b_logits, n * e->n_vocab * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
    if (argmax) MCPM_CUDA(cudaMemcpyAsync(argmax, e->b_argmax, n * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    return check_ctl(e);
}

// ------------------------------------------------------------------ ops
namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool gemv_shape_ok(int type, const void* w, int rows, int cols) {
    if ((type != GGML_Q4_K && type != GGML_Q6_K) || rows <= 0 || cols <= 0 || cols % 256 || cols > 6144) return false;
    if (type == GGML_Q6_K && cols % 2048) return false;   // 16-byte aligned rows for TMA
    return aligned16(w);
}
}  // namespace

mcpm_status mcpm_quantize_q8k(const float* x, void* y, int n, int rounding, void* stream) {
    if (!x || !y || n <= 0 || n % 256 || (rounding != MCPM_ROUND_EVEN && rounding != MCPM_ROUND_AWAY) || !aligned16(x))
        return MCPM_BAD_ARG;
    return cuda_status(op_quantize_q8k(x, y, n, rounding, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_gemv_q8_0_f32(const void* w, const float* x, float* y, int rows, int cols, void* stream) {
    if (!w || !x || !y || rows <= 0 || cols <= 0 || cols % 256 != 0 || cols > 8192) return MCPM_BAD_ARG;
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return MCPM_BAD_ARG;
    return cuda_status(op_gemv_q8_0(w, x, y, rows, cols, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_gemv_q8k(int type, const void* w, const void* xq, float* y, int rows, int cols, void* stream) {
    if (!w || !xq || !y) return MCPM_BAD_ARG;
    if (type != GGML_Q4_K && type != GGML_Q6_K) return MCPM_UNSUPPORTED_TYPE;
    if (!gemv_shape_ok(type, w, rows, cols)) return MCPM_BAD_ARG;
    return cuda_status(op_gemv_q8k(type, w, xq, y, nullptr, nullptr, rows, cols, 0, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_gemv_q8k_block(int type, const void* w, const void* xq, float* y, int rows, int cols, void* stream) {
    if (!w || !xq || !y) return MCPM_BAD_ARG;
    if (type != GGML_Q4_K && type != GGML_Q6_K) return MCPM_UNSUPPORTED_TYPE;
    if (!gemv_shape_ok(type, w, rows, cols) || (cols != 2048 && cols != 6144)) return MCPM_BAD_ARG;
    return cuda_status(op_gemv_q8k(type, w, xq, y, nullptr, nullptr, rows, cols, 1, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_gemv_blocksums(int type, const void* w, const void* xq, int32_t* isum, int32_t* aux, int rows,
                                int cols, void* stream) {
    if (!w || !xq || !isum || !aux) return MCPM_BAD_ARG;
    if (type != GGML_Q4_K && type != GGML_Q6_K) return MCPM_UNSUPPORTED_TYPE;
    if (!gemv_shape_ok(type, w, rows, cols)) return MCPM_BAD_ARG;
    return cuda_status(op_gemv_q8k(type, w, xq, nullptr, isum, aux, rows, cols, 0, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_gemv_gate_up_q8k(const void* wg, const void* wu, const void* xq, float* gate, float* up, int rows,
                                  int cols, void* stream) {
    mcpm_status st = mcpm_gemv_q8k(GGML_Q4_K, wg, xq, gate, rows, cols, stream);
    if (st != MCPM_OK) return st;
    return mcpm_gemv_q8k(GGML_Q4_K, wu, xq, up, rows, cols, stream);
}

mcpm_status mcpm_rmsnorm_q8k(const float* x, const float* w, void* out, int n, float eps, void* stream) {
    if (!x || !w || !out || n != 2048) return MCPM_BAD_ARG;
    return cuda_status(op_rmsnorm_q8k(x, w, out, eps, static_cast<cudaStream_t>(stream)));
}

mcpm_status mcpm_swiglu_q8k(const float* gate, const float* up, void* out, int n, void* stream) {
    if (!gate || !up || !out || n <= 0 || n % 256) return MCPM_BAD_ARG;
    return cuda_status(op_swiglu_q8k(gate, up, out, n, static_cast<cudaStream_t>(stream)));
}

// Attention workspace (chunk records, Q8_K sink), one per device, allocated on first use
// and kept until exit.
namespace {
struct AttWorkspace {
    float* part = nullptr;
    uint8_t* q8k = nullptr;
};
AttWorkspace g_att_ws[64];
}  // namespace

mcpm_status mcpm_attention(const float* q, const float* k, const float* v, float* kcache, float* vcache, int pos,
                           int max_seq, float* out, void* out_q8k, void* stream) {
    if (!q || !k || !v || !kcache || !vcache || !out || !aligned16(q) || !aligned16(kcache) || !aligned16(vcache))
        return MCPM_BAD_ARG;
    if (max_seq <= 0 || max_seq > MAX_SEQ) return MCPM_BAD_ARG;
    if (pos < 0 || pos >= max_seq) return MCPM_CTX_OVERFLOW;
    int dev = 0;
    MCPM_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return MCPM_BAD_ARG;
    AttWorkspace& ws = g_att_ws[dev];
    if (!ws.part) {
        MCPM_CUDA(cudaMalloc(&ws.part, ATT_PART_FLOATS * sizeof(float)));
        MCPM_CUDA(cudaMalloc(&ws.q8k, (N_EMBD / 256) * Q8K_BYTES));
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return cuda_status(launch_attention(q, k, v, kcache, vcache, pos, max_seq, out,
                                        out_q8k ? static_cast<uint8_t*>(out_q8k) : ws.q8k, ws.part, s));
}

mcpm_status mcpm_gemv_q8k_timed(int type, const void* w, int n_copies, const void* xq, float* y, int rows, int cols,
                                int order, int reps, float* ms_per_launch, void* stream) {
    if (!w || !xq || !y || !ms_per_launch || n_copies <= 0 || reps <= 0) return MCPM_BAD_ARG;
    if (!gemv_shape_ok(type, w, rows, cols)) return MCPM_BAD_ARG;
    if (order != MCPM_ORDER_AVX2 && order != MCPM_ORDER_BLOCK) return MCPM_BAD_ARG;
    if (order == MCPM_ORDER_BLOCK && cols != 2048 && cols != 6144) return MCPM_BAD_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t stride = static_cast<size_t>(rows) * row_bytes(type, cols);
    cudaEvent_t a, b;
    MCPM_CUDA(cudaEventCreate(&a));
    MCPM_CUDA(cudaEventCreate(&b));
    MCPM_CUDA(op_gemv_q8k(type, w, xq, y, nullptr, nullptr, rows, cols, order, s));   // warm-up
    MCPM_CUDA(cudaEventRecord(a, s));
    for (int i = 0; i < reps; ++i)
        MCPM_CUDA(op_gemv_q8k(type, static_cast<const uint8_t*>(w) + (i % n_copies) * stride, xq, y, nullptr, nullptr,
                              rows, cols, order, s));
    MCPM_CUDA(cudaEventRecord(b, s));
    MCPM_CUDA(cudaEventSynchronize(b));
    float ms = 0.0f;
    MCPM_CUDA(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    *ms_per_launch = ms / reps;
    return MCPM_OK;
}

}  // extern "C"
