// Internal declarations shared by the decode kernel (mcpm_decode.cu), the op kernels
// (mcpm_ops.cu) and the host engine (mcpm_engine.cu).
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace mcpm {

constexpr int N_EMBD = 2048, N_FF = 6144, N_HEAD = 16, N_HEAD_KV = 2, HEAD_DIM = 128, KV_DIM = 256;
constexpr int QKV_ROWS = N_EMBD + 2 * KV_DIM;   // 2560 combined rows of the fused QKV GEMV
constexpr int MAX_LAYERS = 64;

// Decode kernel geometry.
constexpr int DEC_THREADS = 512;
constexpr int WBUF_BYTES = 98304;          // one weight buffer (two per CTA)
constexpr int WBUF_SLACK = 128;            // readable tail after each buffer (unaligned Q6_K reads)
constexpr int MAX_TASKS = 512;             // (row, super-block) tasks per GEMV pass
constexpr int ROWVAL_FLOATS = 256;
constexpr int LM_SLOTS = 2;                 // LM head: a ring of stages laid over both weight buffers
constexpr int LM_SLOT_STRIDE = WBUF_BYTES + WBUF_SLACK;   // bytes per stage slot
constexpr int LM_SLOT_BYTES = LM_SLOT_STRIDE - WBUF_SLACK;   // weight bytes per stage (the rest: readable tail)
static_assert(LM_SLOTS * LM_SLOT_STRIDE <= 2 * (WBUF_BYTES + WBUF_SLACK), "LM ring inside the weight buffers");
constexpr int ATT_MAX_CHUNKS = 64;         // attention chunks per head (chunk = 32*ceil(n/2048))
constexpr int ATT_PART_STRIDE = 4 + HEAD_DIM;   // m, l, 2 pad, o[128]: o 16-byte aligned
constexpr int ATT_PART_O = 4;
constexpr int BATCH_MAX = 64;            // sequences of one batched-decode engine
constexpr int ATTW_COPIES = 8;           // copies of the combined attention: CTA c polls copy c % 8
constexpr int XLL_COPIES = 1;            // copies of the published residual: CTA c polls copy c % 8
constexpr int ATT_SC_STRIDE = 256;         // chunk-length bound: 32*ceil(MAX_SEQ/2048)
constexpr int MAX_SEQ = 16384;
constexpr int TRACE_WORDS = 3400;         // 2 + 2*(5*layers+1) phase marks, detail marks from 650, per-CTA from 720
constexpr int TRACE_DETAIL = 650;         // sub-step marks of layer 1: 650 + 10*phase + step
constexpr int TRACE_CTA = 720;            // layer-1 barrier k, CTA c: arrival 720 + 148k + c, release 1460 + 148k + c, SM id 2200 + c,
                                          // QKV sub-steps m = 0..2 of layer 1 at 2400 + 148m + c
constexpr int TRACE_GEMV = 2848;          // layer-1 GEMV marks of CTA 0 (pass 1, pass 2, entry): O, D, gate, QKV
constexpr int TRACE_POLL = 2960;          // per CTA: residual poll done, gate/up norm of layer 1 (+0), QKV norm of layer 2 (+148)
constexpr int TRACE_GEMM = 3260;          // batched tcgen05 GEMM of layer 1's gate/up: CTA 0's first unit (28 marks)

// QKV row pairs [0, 1280) (Q pairs, then K, then V) are split over the CTAs in proportion
// to their GEMV cost: a Q6_K row costs about 1.6 Q4_K rows (unaligned 210-byte blocks), so
// CTAs holding Q6_K V rows get fewer of them and every CTA reaches the barrier together.
__host__ __device__ inline int qkv_row_cost(int type) { return type == 14 ? 16 : 10; }
__host__ __device__ inline int qkv_pair_boundary(int tq, int tk, int tv, int c, int ncta) {
    const long long cq = qkv_row_cost(tq), ck = qkv_row_cost(tk), cv = qkv_row_cost(tv);
    const int nq = N_EMBD / 2, nk = KV_DIM / 2, nv = KV_DIM / 2;
    const long long total = cq * nq + ck * nk + cv * nv;
    const long long t = total * c / ncta;
    if (t <= cq * nq) return static_cast<int>(t / cq);
    if (t <= cq * nq + ck * nk) return nq + static_cast<int>((t - cq * nq) / ck);
    const int pv = nq + nk + static_cast<int>((t - cq * nq - ck * nk) / cv);
    return pv < nq + nk + nv ? pv : nq + nk + nv;
}

// Decode schedule options (DecodeParams::sched, mcpm_config::sched bits).
constexpr int SCHED_L2_PREFETCH = 1;   // L2 prefetch of the next layer's weight rows (measured slower: off)
constexpr int SCHED_ATT_COMBINERS = 2; // head-pair combiners at every context length (default: above 16 chunks)
constexpr int SCHED_EARLY_GU = 4;      // gate/up rows copied during attention (default: after it; measured
                                       // slower, the copy delays the q/K/V hand-off)

struct LayerDev {
    const uint8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *attn_norm, *ffn_norm;
    int tq, tk, tv, to, tg, tu, td;
};

struct DecodeParams {
    const LayerDev* layers;
    const uint8_t* arena;   // base of the weight arena (LayerDev pointers point into it)
    int n_layer;
    const uint8_t* embd;
    int embd_type;
    const float* out_norm;
    const uint8_t* lm;
    int lm_type;
    int n_vocab;
    float* kc;          // [n_layer][max_seq][KV_DIM] of fp32, or of fp16 when kv_f16 (cast before indexing)
    float* vc;
    int max_seq;
    const float2* rope; // [max_seq][HEAD_DIM/2] (cos, sin)
    float* x;           // residual stream [N_EMBD]
    float* q;           // rotated queries [N_EMBD]
    float* att;         // attention output [N_EMBD] (fp32, for inspection)
    uint8_t* att_q8k;   // attention output as 8 block_q8_K
    float* h;           // SwiGLU output [N_FF]
    unsigned long long* xll;   // residual stream published per element as (epoch << 32) | fp32 bits
                               // [XLL_COPIES][N_EMBD]
    unsigned long long* qll;   // rotated q [N_EMBD] then this position's K and V rows [2*KV_DIM], same encoding;
                               // null outside the decode kernel (q and the cache are then final)
    float* att_part;    // [N_HEAD][ATT_MAX_CHUNKS][ATT_PART_STRIDE]: epoch-tagged (m, l) header, o[128]
    unsigned long long* attw;   // combined attention [ATTW_COPIES][N_EMBD], epoch-tagged (decode kernel, > 16 chunks)
    int8_t* att_qs;     // optional split Q8_K output of combine_pair (batched decode): values [8][256],
    float* att_d;       //   scales [8], block sums [8][16]; null: block_q8_K blocks in att_q8k
    int16_t* att_bs;
    float* logits;      // [n_vocab]
    float* am_val;      // per-CTA argmax partials
    int* am_idx;
    int* argmax_out;
    int* token_dev;     // token id for the next step (greedy chaining)
    unsigned* bar;      // grid barrier {count, base}, [2] launch sequence (epochs of xll)
    unsigned* cnt;      // [2] argmax counter
    unsigned* err;      // error bits
    unsigned long long* trace;   // optional: CTA 0 phase timestamps (2 per phase + 2)
    int sched;          // SCHED_* option bits
    int blk_order;      // GEMVs in the block order (warp per row, exact block sums, one fma per block in
                        // groups of four); 0: the reference's eight-lane AVX2 order
    int kv_f16;         // kc / vc hold fp16 rows (their element offsets are the same)
    int token;          // < 0: read *token_dev
    int pos;
    int write_logits;
};

// RoPE (cos, sin) factors of one position: HEAD_DIM / 2 pairs (host, C library functions).
void rope_row(int pos, float base, float2* out);

size_t decode_smem_bytes();
cudaError_t decode_prepare();
cudaError_t launch_decode(const DecodeParams& p, int n_ctas, cudaStream_t stream);
int decode_max_ctas_per_sm();

// Standalone attention (mcpm_decode.cu): appends k/v at pos, then split-KV attention with
// the decode kernel's numerics.  part: ATT_PART_FLOATS floats, cnt: 3 zeroed words.
constexpr size_t ATT_PART_FLOATS = static_cast<size_t>(N_HEAD) * ATT_MAX_CHUNKS * ATT_PART_STRIDE;
// Scratch of the tcgen05 batched GEMM (128-row tiles, groups of 4 blocks, 64 sequences): the
// group partials of the widest launch (units = row tiles x groups) and one counter per row tile.
inline size_t batch_gemm_units(int n_vocab) {
    auto tiles = [](int rows) { return static_cast<size_t>((rows + 127) / 128); };
    size_t u = 2 * tiles(n_vocab);                                         // LM head, 8 blocks per row
    u = std::max(u, 2 * (2 * tiles(N_FF)));                                // gate + up
    u = std::max(u, (N_FF / 256 / 4) * tiles(N_EMBD));                     // down, 24 blocks per row
    u = std::max(u, 2 * (tiles(N_EMBD) + 2 * tiles(KV_DIM)));              // q, k, v
    return u;
}
inline size_t batch_gemm_scratch_floats(int n_vocab) { return batch_gemm_units(n_vocab) * 64 * 128; }
inline size_t batch_gemm_counters(int n_vocab) { return batch_gemm_units(n_vocab); }
// Batched decode (n_seq independent sequences): one step of every sequence.
struct BatchLaunch {
    int n_seq, max_seq, n_layer, n_vocab, lm_type, max_pos, chain, n_sm;
    int tcgen05;              // GEMMs on k_b_gemm_tc (batched block order) instead of the mma.sync
                              // kernels (the batch-1 decode's eight-lane order)
    float* gemm_part;         // k_b_gemm_tc scratch: batch_gemm_scratch_floats(n_vocab) floats
    unsigned* gemm_cnt;       // k_b_gemm_tc tile counters: batch_gemm_counters(n_vocab) zeroed words
    unsigned long long* trace;   // optional: TRACE_GEMM marks of one GEMM launch
    int shared_kv;            // every row is a position of ONE sequence: one cache [n_layer][max_seq][KV_DIM]
                              // (batched prefill: row i attends to positions 0 .. pos[i], causal)
    int skip_lm;              // no LM head / argmax (prefill chunks before the last)
    int kv_f16;               // the cache holds fp16 rows (mcpm_config::kv_type MCPM_KV_F16)
    const LayerDev* layers;   // host array; weight pointers are device pointers
    const uint8_t* embd;
    const float* out_norm;
    const uint8_t* lm;
    const float2* rope;
    float *kc, *vc, *x, *y, *q, *att_part, *att, *logits;   // [n_seq][...] device buffers
    int8_t* aqs;
    float* ad;
    int16_t* abs;
    int *tokens, *pos, *argmax;
    unsigned* err;
};
cudaError_t launch_batch_step(const BatchLaunch& b, cudaStream_t stream);

cudaError_t launch_sample_top_p(const float* logits, int n, float temperature, float top_p, float r, int* out, float* p,
                                uint32_t* gk, int* gi, cudaStream_t stream);

// Attention of one tensor-parallel rank: units of KV groups g0 .. g0+ng-1, combine of head
// pairs b0 .. b0+nb-1; p.pos is taken from pos_dev on the device.
cudaError_t launch_tp_attention(const DecodeParams& p, const int* pos_dev, int g0, int ng, int b0, int nb,
                                cudaStream_t stream);

cudaError_t launch_attention(const float* q, const float* k, const float* v, float* kc, float* vc, int pos, int max_seq,
                             float* out, uint8_t* out_q8k, float* part, cudaStream_t stream);

// Standalone op launchers (mcpm_ops.cu).
cudaError_t op_quantize_q8k(const float* x, void* y, int n, int rounding, cudaStream_t s);
cudaError_t op_gemv_q8_0(const void* w, const float* x, float* y, int rows, int cols, cudaStream_t s);
cudaError_t op_gemv_q8k(int type, const void* w, const void* xq, float* y, int32_t* isum, int32_t* aux, int rows,
                        int cols, int blk_order, cudaStream_t s);
cudaError_t op_rmsnorm_q8k(const float* x, const float* w, void* out, float eps, cudaStream_t s);
cudaError_t op_swiglu_q8k(const float* g, const float* u, void* out, int n, cudaStream_t s);
cudaError_t op_rope_kv_append(float* q, float* k, const float* v, float* kc, float* vc, int pos, float base,
                              cudaStream_t s);

}  // namespace mcpm
