// Tensor-parallel batch-1 decode of an all-Q8_0 MiniCPM5 model: one engine per GPU, one
// process (or thread) per GPU, Megatron partition.
//
// Reference counterpart: MiniCPM5Engine::forward (src/model.cpp:142-242) with every matrix
// Q8_0, i.e. matmul -> gemv_q8_0 (ops.cpp:58-79) for all projections, rmsnorm (ops.cpp:468-481)
// on fp32, apply_rope (ops.cpp:502-516), execute_attention (ops.cpp:537-628), silu
// (ops.cpp:447-449) and the Q8_0 embedding row d*q.  The reference itself has no tensor
// parallelism and cannot run this model (its fused QKV / Gate+Up / Q8_K paths do not handle
// Q8_0), so the C restatement's all-Q8_0 forward is the oracle.
//
// Partition of rank r of N (N = 1, 2, 4, 8): query heads [16r/N, 16(r+1)/N); the KV head
// those heads use (both at N = 1; at N = 4, 8 each GPU recomputes its KV head's 128 K and
// 128 V rows and keeps its own copy of that head's cache); FFN rows [6144r/N, 6144(r+1)/N);
// vocabulary rows [V r/N, V(r+1)/N).  QKV, Gate+Up and the LM head are split by rows
// (output), o_proj and down by columns (input), so each of those two yields a partial sum
// of all 2048 outputs that the ranks exchange.
//
// One token is a fixed sequence of kernels on the engine's stream, captured once as a CUDA
// graph; token, position and step counter live in device memory (TPCtl):
//   layer l  QKV      prologue: residual += exchanged down partials of layer l-1 (layer 0:
//                     the embedding row), RMSNorm; epilogue: RoPE on q and k, q to the query
//                     buffer, k and v into the KV cache at pos
//            attention split-KV units of the rank's KV head(s), combine of its head pairs
//            o_proj   partial sums over the rank's heads -> exchange
//            Gate+Up  prologue: residual += exchanged o_proj partials, RMSNorm
//            down     prologue: SwiGLU of the rank's FFN rows; partial sums -> exchange
//   LM head  prologue: residual += exchanged down partials, output RMSNorm; fused argmax of
//            the rank's vocabulary rows -> exchange of (value, index); a one-warp kernel
//            picks the token (highest value, lowest index on ties), logs it, advances pos.
// Exchange (N > 1), selected per engine:
//   P2P   each GEMV row's partial sum is stored, tagged with the step's epoch in the same
//         64-bit word, into this rank's slot of every rank's receive buffer (CUDA IPC
//         mappings, plain stores over NVLink); the consuming kernel's prologue polls each
//         slot for the epoch (bounded wait) and adds the slots in rank order, so every rank
//         forms the same residual.  No separate collective launch and no flag round trip.
//   NCCL  plain partial sums, ncclAllReduce (sum, fp32) in place after o_proj and down,
//         ncclAllGather of the argmax pairs (NCCL loaded at run time with dlopen).
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/mcpm.h"
#include "gguf.h"
#include "mcpm_device.cuh"
#include "mcpm_internal.h"
#include "mcpm_q80.cuh"

using namespace mcpm;

namespace {

constexpr int TP_MAX_WORLD = 8;
constexpr int PRO_PLAIN = 0, PRO_NORM = 1, PRO_SWIGLU = 2;
constexpr int EPI_STORE = 0, EPI_ROPE = 1, EPI_PUBLISH = 2, EPI_ARGMAX = 3;
constexpr unsigned STEP_ARGMAX = 255;
// Waits on other GPUs: the ranks launch independently, so allow for host-side skew
// (mcpm_tp_config::peer_wait_us, default 5 s).  Once one wait of the engine has timed out
// (ERR_TIMEOUT in the control word), every later wait gives up at once, so a rank that
// stopped costs one bound, not one per exchange.
constexpr unsigned DEFAULT_PEER_WAIT_US = 5000000u;

struct TPCtl {
    int token;         // input token of the next step
    int pos;           // its position
    unsigned seq;      // steps run so far + 1: epoch of the exchanged values (seq << 8 | step)
    unsigned err;      // ERR_* bits
    unsigned am_cnt;   // LM-head CTAs whose argmax partial is stored
    unsigned wait_us;  // bound of every wait for another rank's values
    unsigned pad[2];
};

struct TPGemv {
    const uint8_t* w;   // weight shard [rows][nb * 34 B]
    int rows, nb, pro, epi;
    TPCtl* ctl;
    // prologue
    const float* x;      // PLAIN: input; SWIGLU: gate [nb*32] then up [nb*32]; NORM: residual before the add
    float* x_next;       // NORM: residual after the add (written by CTA 0)
    const float* norm;   // NORM: RMSNorm weight
    const uint8_t* embd; // NORM: non-null -> residual = Q8_0 embedding row of ctl->token
    int n_vocab;
    const float* red;                  // NORM: summed partials to add (one rank or NCCL); null: none
    const unsigned long long* slots;   // NORM (P2P): receive slots [world][N_EMBD] to add
    int world, red_step;
    // epilogue
    float* y;                                  // STORE, ARGMAX: row values
    unsigned long long* pub[TP_MAX_WORLD];     // PUBLISH: this rank's slot in every rank's receive buffer
    int pub_step;
    float *q, *kc, *vc;                        // ROPE: query buffer, cache rows of this layer (+ KV column offset)
    const float2* rope;
    int nq, nkv, max_seq;
    float* am_val;                             // ARGMAX: per-CTA partials
    int* am_idx;
    int vocab_off;
    unsigned long long* am_pub[TP_MAX_WORLD];  // ARGMAX (P2P): (value, index) slot in every rank's buffer
    float* am_local;                           // ARGMAX (one rank, NCCL): (value, index bits)
    unsigned long long* wait_ns;               // optional: CTA 0's wait for the exchanged partials
};

__device__ __forceinline__ void st_epoch_sys(unsigned long long* p, float v, unsigned epoch) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_epoch2_sys(const unsigned long long* p) {
    ulonglong2 w;
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}
// n2 pairs of epoch-tagged values (16-byte aligned) written by any GPU, polled until all
// carry `epoch`; false (and ERR_TIMEOUT) after ctl->wait_us, or at once when an earlier wait
// of this engine timed out.
template <int N2>
__device__ __forceinline__ bool load_epoch_sys(const unsigned long long* src, unsigned epoch, float (&v)[2 * N2],
                                               TPCtl* ctl) {
    unsigned* err = &ctl->err;
    ulonglong2 w[N2];
    auto ready = [&]() {
        bool r = true;
#pragma unroll
        for (int i = 0; i < N2; ++i) r &= (w[i].x >> 32) == epoch && (w[i].y >> 32) == epoch;
        return r;
    };
#pragma unroll
    for (int i = 0; i < N2; ++i) w[i] = ld_epoch2_sys(src + 2 * i);
    if (!ready()) {
        const uint64_t t0 = globaltimer();
        const unsigned long long limit = 1000ull * ctl->wait_us;
        do {
            __nanosleep(32);
#pragma unroll
            for (int i = 0; i < N2; ++i) w[i] = ld_epoch2_sys(src + 2 * i);
            if (ready()) break;
            if ((ld_relaxed_u32(err) & ERR_TIMEOUT) || globaltimer() - t0 > limit) {
                atomicOr(err, ERR_TIMEOUT);
                return false;
            }
        } while (true);
    }
#pragma unroll
    for (int i = 0; i < N2; ++i) {
        v[2 * i] = __uint_as_float(static_cast<unsigned>(w[i].x));
        v[2 * i + 1] = __uint_as_float(static_cast<unsigned>(w[i].y));
    }
    return true;
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// s.xs <- the GEMV input (see TPGemv).  false (whole CTA) when an exchanged slot timed out.
__device__ bool tp_prologue(const TPGemv& g, const Q80Smem& s, unsigned seq) {
    const int tid = threadIdx.x, cols = g.nb * 32;
    if (g.pro == PRO_PLAIN) {
        for (int i = tid; i < cols / 4; i += blockDim.x)
            *reinterpret_cast<float4*>(s.xs + q80_xpos(4 * i)) = reinterpret_cast<const float4*>(g.x)[i];
        return true;
    }
    if (g.pro == PRO_SWIGLU) {   // silu(g)*u (ops.cpp:447-449), h stays fp32 for the Q8_0 down
        for (int i = tid; i < cols; i += blockDim.x) s.xs[q80_xpos(i)] = canon_silu_mul(g.x[i], g.x[cols + i]);
        return true;
    }
    // PRO_NORM: 512 threads x 4 consecutive elements of the residual
    float* xin = reinterpret_cast<float*>(s.part);   // scratch until pass 1
    const int i0 = 4 * tid;
    float v[4];
    bool ok = true;
    if (g.embd) {   // get_embedding for a Q8_0 row: d * q
        int token = g.ctl->token;
        if (token < 0 || token >= g.n_vocab) {
            if (tid == 0) atomicOr(&g.ctl->err, ERR_BAD_TOKEN);
            token = 0;
        }
        const uint8_t* blk = g.embd + (static_cast<size_t>(token) * (N_EMBD / 32) + (i0 >> 5)) * Q8_0_BYTES;
        const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
        const int8_t* qs = reinterpret_cast<const int8_t*>(blk + 2) + (i0 & 31);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __fmul_rn(d, static_cast<float>(qs[k]));
    } else {
        const float4 xv = *reinterpret_cast<const float4*>(g.x + i0);
        v[0] = xv.x, v[1] = xv.y, v[2] = xv.z, v[3] = xv.w;
        float r[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        bool add = false;
        if (g.slots) {   // partials of every rank, summed in rank order
            const unsigned e = (seq << 8) | static_cast<unsigned>(g.red_step);
            const uint64_t t0 = (g.wait_ns && blockIdx.x == 0 && tid == 0) ? globaltimer() : 0;
            ok = load_epoch_sys<2>(g.slots + i0, e, r, g.ctl);
            for (int k = 1; k < g.world && ok; ++k) {
                float t[4];
                ok = load_epoch_sys<2>(g.slots + static_cast<size_t>(k) * N_EMBD + i0, e, t, g.ctl);
#pragma unroll
                for (int j = 0; j < 4; ++j) r[j] = __fadd_rn(r[j], t[j]);
            }
            if (g.wait_ns && blockIdx.x == 0 && tid == 0) atomicAdd(g.wait_ns, globaltimer() - t0);
            add = true;
        } else if (g.red) {
            const float4 rv = *reinterpret_cast<const float4*>(g.red + i0);
            r[0] = rv.x, r[1] = rv.y, r[2] = rv.z, r[3] = rv.w;
            add = true;
        }
        if (add) {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __fadd_rn(v[k], r[k]);
        }
    }
    if (__syncthreads_or(!ok)) return false;
    reinterpret_cast<float4*>(xin)[tid] = make_float4(v[0], v[1], v[2], v[3]);
    if (blockIdx.x == 0 && g.x_next) reinterpret_cast<float4*>(g.x_next)[tid] = make_float4(v[0], v[1], v[2], v[3]);
    __syncthreads();
    float xv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = tid < 256 ? xin[tid + 256 * i] : 0.0f;
    const float ss = sumsq_2048(xv, s.scratch);
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(N_EMBD)), 1e-6f)));
    const float4 wv = *reinterpret_cast<const float4*>(g.norm + i0);
    const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __fmul_rn(__fmul_rn(v[k], w4[k]), rms);
    *reinterpret_cast<float4*>(s.xs + q80_xpos(i0)) = make_float4(o[0], o[1], o[2], o[3]);
    return true;
}

// One Q8_0 GEMV of the token sequence with its prologue and epilogue (TPGemv).  Row ranges
// are pair-aligned (RoPE pairs stay inside one CTA's stage).  Launched as a programmatic
// dependent: the weight copies start before the preceding kernel has finished.
__global__ void __launch_bounds__(Q80_THREADS, 1) k_tp_gemv(const TPGemv g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const Q80Smem s(smem_raw);
    __shared__ int last_cta;
    const int tid = threadIdx.x;
    const int pairs = g.rows >> 1;
    const int r0 = 2 * static_cast<int>((static_cast<long long>(pairs) * blockIdx.x) / gridDim.x);
    const int r1 = 2 * static_cast<int>((static_cast<long long>(pairs) * (blockIdx.x + 1)) / gridDim.x);
    const int sr = max(2, q80_pick_stage(g.nb, 2 * ((pairs + gridDim.x - 1) / gridDim.x)) & ~1);
    if (tid == 0) q80_start(g.w, r0, r1, g.nb, sr, s);
    grid_dep_launch();
    grid_dep_wait();   // activations, control words and outputs of earlier kernels from here on
    const unsigned seq = g.ctl->seq;
    if (!tp_prologue(g, s, seq)) {   // an exchanged slot timed out: drain the copies in flight
        q80_run(g.w, r0, r1, g.nb, sr, s, &g.ctl->err, [&](int, float, float) {});
        return;
    }
    __syncthreads();
    unsigned* err = &g.ctl->err;
    if (g.epi == EPI_STORE) {
        q80_run(g.w, r0, r1, g.nb, sr, s, err, [&](int r, float v, float) { g.y[r] = v; });
    } else if (g.epi == EPI_PUBLISH) {
        const unsigned e = (seq << 8) | static_cast<unsigned>(g.pub_step);
        q80_run(g.w, r0, r1, g.nb, sr, s, err, [&](int r, float v, float) {
            for (int k = 0; k < g.world; ++k) st_epoch_sys(g.pub[k] + r, v, e);
        });
    } else if (g.epi == EPI_ROPE) {
        const int pos = g.ctl->pos;
        if (pos < 0 || pos >= g.max_seq) {   // the host bounds pos; never write outside the cache
            if (tid == 0) atomicOr(err, ERR_BAD_ARG);
            q80_run(g.w, r0, r1, g.nb, sr, s, err, [&](int, float, float) {});   // drain the copies in flight
            return;
        }
        float* kdst = g.kc + static_cast<size_t>(pos) * KV_DIM;
        float* vdst = g.vc + static_cast<size_t>(pos) * KV_DIM;
        const float2* cs = g.rope + static_cast<size_t>(pos) * (HEAD_DIM / 2);
        q80_run(g.w, r0, r1, g.nb, sr, s, err, [&](int R, float v, float vp) {
            if (R < g.nq + g.nkv) {   // rotated pair (interleaved, with the build's FMA contraction)
                const float2 c = __ldg(cs + ((R & (HEAD_DIM - 1)) >> 1));
                const bool odd = R & 1;
                const float v0 = odd ? vp : v, v1 = odd ? v : vp;
                const float o = odd ? __fmaf_rn(c.y, v0, __fmul_rn(c.x, v1)) : __fmaf_rn(c.x, v0, -__fmul_rn(c.y, v1));
                if (R < g.nq)
                    g.q[R] = o;
                else
                    kdst[R - g.nq] = o;
            } else {
                vdst[R - g.nq - g.nkv] = v;
            }
        });
    } else {   // EPI_ARGMAX: logits slice and this CTA's (max, lowest index)
        float bv = -__int_as_float(0x7f800000);
        int bi = 0x7fffffff;
        if (!q80_run(g.w, r0, r1, g.nb, sr, s, err, [&](int r, float v, float) {
                g.y[r] = v;
                if (better(v, r, bv, bi)) bv = v, bi = r;
            }))
            return;
        for (int o = 16; o >= 1; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
        }
        int* sidx = reinterpret_cast<int*>(s.scratch + 32);
        if ((tid & 31) == 0) s.scratch[tid >> 5] = bv, sidx[tid >> 5] = bi;
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
                if (better(s.scratch[w], sidx[w], s.scratch[0], sidx[0])) s.scratch[0] = s.scratch[w], sidx[0] = sidx[w];
            g.am_val[blockIdx.x] = s.scratch[0];
            g.am_idx[blockIdx.x] = sidx[0];
            __threadfence();
            last_cta = atomicAdd(&g.ctl->am_cnt, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (last_cta && tid == 0) {   // every CTA's partial is visible (fence before its count)
            __threadfence();
            float v = ld_cg_f32(g.am_val);
            int i = __ldcg(g.am_idx);
            for (int c = 1; c < static_cast<int>(gridDim.x); ++c) {
                const float cv = ld_cg_f32(g.am_val + c);
                const int ci = __ldcg(g.am_idx + c);
                if (better(cv, ci, v, i)) v = cv, i = ci;
            }
            i = i == 0x7fffffff ? 0 : i + g.vocab_off;
            if (g.am_pub[0]) {
                const unsigned e = (seq << 8) | STEP_ARGMAX;
                for (int k = 0; k < g.world; ++k) {
                    st_epoch_sys(g.am_pub[k], v, e);
                    st_epoch_sys(g.am_pub[k] + 1, __int_as_float(i), e);
                }
            } else {
                g.am_local[0] = v;
                g.am_local[1] = __int_as_float(i);
            }
            g.ctl->am_cnt = 0;
        }
    }
}

// The token of the step: best (value, index) over the ranks; logs it and advances pos and
// the step counter.  One warp.
__global__ void k_tp_pick(TPCtl* ctl, int world, const unsigned long long* am_slots, const float* gathered, int* log,
                          int max_seq) {
    grid_dep_wait();
    const int lane = threadIdx.x;
    const unsigned seq = ctl->seq;
    const int pos = ctl->pos;
    float bv = -__int_as_float(0x7f800000);
    int bi = 0x7fffffff;
    bool ok = true;
    if (lane < world) {
        if (am_slots) {
            float v[2];
            ok = load_epoch_sys<1>(am_slots + 2 * lane, (seq << 8) | STEP_ARGMAX, v, ctl);
            bv = v[0], bi = __float_as_int(v[1]);
        } else {
            bv = gathered[2 * lane], bi = __float_as_int(gathered[2 * lane + 1]);
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    if (lane == 0) {
        if (ok) {
            ctl->token = bi;
            if (pos >= 0 && pos < max_seq) log[pos] = bi;
        }
        ctl->pos = pos + 1;
        ctl->seq = seq + 1;
    }
}

// ---- NCCL, resolved at run time (the process may already hold torch's copy).
struct NcclId {
    char internal[128];
};
struct NcclApi {
    void* h = nullptr;
    int (*get_unique_id)(NcclId*) = nullptr;
    int (*comm_init_rank)(void**, int, NcclId, int) = nullptr;
    int (*all_reduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
    int (*all_gather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
    int (*comm_destroy)(void*) = nullptr;
    const char* (*error_string)(int) = nullptr;
};
constexpr int NCCL_FLOAT32 = 7, NCCL_SUM = 0;

NcclApi* nccl() {
    static NcclApi api;
    static bool tried = false;
    if (tried) return api.h ? &api : nullptr;
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        std::fprintf(stderr, "[mcpm] libnccl.so.2 not found: %s\n", dlerror());
        return nullptr;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.comm_init_rank || !api.all_reduce || !api.all_gather || !api.comm_destroy ||
        !api.error_string) {
        std::fprintf(stderr, "[mcpm] libnccl.so.2 lacks an entry point\n");
        return nullptr;
    }
    api.h = h;
    return &api;
}

}  // namespace

struct mcpm_tp {
    int device = 0, rank = 0, world = 1, max_seq = 0, comm = MCPM_TP_P2P, use_graph = 1;
    unsigned wait_us = DEFAULT_PEER_WAIT_US;
    cudaStream_t stream = nullptr;
    int n_sm = 0;
    bool loaded = false, connected = false;
    int n_layer = 0, n_vocab = 0, vocab_lo = 0, vocab_hi = 0;
    int hq = 0, h0 = 0, g0 = 0, ng = 0, f0 = 0, nf = 0;
    float rope_base = 5000000.0f;
    struct Layer {
        const uint8_t *wqkv, *wo, *wgu, *wd;
        const float *anorm, *fnorm;
    };
    std::vector<Layer> layers;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    const uint8_t *embd = nullptr, *lm = nullptr;
    const float* onorm = nullptr;
    TPCtl* ctl = nullptr;
    TPCtl* ctl_host = nullptr;   // pinned
    int* tok_log = nullptr;
    float *kc = nullptr, *vc = nullptr;
    float2* rope = nullptr;
    float *x0 = nullptr, *x1 = nullptr, *q = nullptr, *att = nullptr, *att_part = nullptr, *gu = nullptr;
    float *red_o = nullptr, *red_d = nullptr, *logits = nullptr, *am_val = nullptr, *am_local = nullptr;
    float* gathered = nullptr;
    int* am_idx = nullptr;
    uint8_t* att_q8k = nullptr;
    unsigned long long* recv = nullptr;   // [2][world][N_EMBD] partials (o_proj, down), [world][2] argmax
    unsigned long long* peer_recv[TP_MAX_WORLD] = {};
    unsigned long long* wait_ns = nullptr;   // profiling: CTA 0's waits for exchanged partials
    bool profile = false;
    void* nccl_comm = nullptr;
    cudaGraphExec_t graph = nullptr;
    int pos_next = 0;   // host mirror of ctl->pos
};

namespace {

mcpm_status cuda_st(cudaError_t e) {
    if (e == cudaSuccess) return MCPM_OK;
    if (e == cudaErrorMemoryAllocation) return MCPM_OUT_OF_MEMORY;
    std::fprintf(stderr, "[mcpm] CUDA error: %s\n", cudaGetErrorString(e));
    return MCPM_CUDA_ERROR;
}
#define TP_CUDA(call)                                  \
    do {                                               \
        const mcpm_status st__ = cuda_st((call));      \
        if (st__ != MCPM_OK) return st__;              \
    } while (0)

mcpm_status nccl_st(int r) {
    if (r == 0) return MCPM_OK;
    NcclApi* api = nccl();
    std::fprintf(stderr, "[mcpm] NCCL error %d: %s\n", r, api ? api->error_string(r) : "?");
    return MCPM_NCCL_ERROR;
}

template <typename T>
void free_dev(T*& p) {
    if (p) cudaFree(const_cast<void*>(reinterpret_cast<const void*>(p)));
    p = nullptr;
}

constexpr size_t kv_elems(int n_layer, int max_seq) { return static_cast<size_t>(n_layer) * max_seq * KV_DIM; }

// Exchange slots of kind k (0 = o_proj, 1 = down) in a receive buffer.
unsigned long long* slot_base(unsigned long long* buf, int world, int kind) {
    return buf + static_cast<size_t>(kind) * world * N_EMBD;
}

TPGemv gemv_base(const mcpm_tp* t) {
    TPGemv g{};
    g.ctl = t->ctl;
    g.world = t->world;
    g.n_vocab = t->n_vocab;
    g.wait_ns = t->profile ? t->wait_ns : nullptr;
    return g;
}

bool p2p(const mcpm_tp* t) { return t->world > 1 && t->comm == MCPM_TP_P2P; }
bool use_nccl(const mcpm_tp* t) { return t->world > 1 && t->comm == MCPM_TP_NCCL; }

// Residual add source of a NORM prologue: partials of kind `kind` at exchange step `step`.
void set_red(const mcpm_tp* t, TPGemv& g, int kind, int step) {
    if (p2p(t)) {
        g.slots = slot_base(t->recv, t->world, kind);
        g.red_step = step;
    } else {
        g.red = kind == 0 ? t->red_o : t->red_d;
    }
}
// Output of a row-split GEMV: partials of kind `kind` at exchange step `step`.
void set_publish(const mcpm_tp* t, TPGemv& g, int kind, int step) {
    if (p2p(t)) {
        g.epi = EPI_PUBLISH;
        for (int k = 0; k < t->world; ++k) g.pub[k] = slot_base(t->peer_recv[k], t->world, kind) + t->rank * N_EMBD;
        g.pub_step = step;
    } else {
        g.epi = EPI_STORE;
        g.y = kind == 0 ? t->red_o : t->red_d;
    }
}

// Launch as a programmatic dependent of the preceding kernel in the stream.
template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

cudaError_t launch_gemv(const mcpm_tp* t, const TPGemv& g, cudaStream_t s) {
    const int grid = std::min(t->n_sm, g.rows / 2);
    return launch_pdl(k_tp_gemv, dim3(grid), dim3(Q80_THREADS), q80_smem_bytes(), s, g);
}

// Events around each collective (profiling runs, eager launches only).
struct CommTimer {
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>>* ev = nullptr;
    void begin(cudaStream_t s) {
        if (!ev) return;
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, s);
        ev->push_back({a, b});
    }
    void end(cudaStream_t s) {
        if (ev) cudaEventRecord(ev->back().second, s);
    }
};

// The kernels (and collectives) of one token on stream s.
mcpm_status enqueue_token(mcpm_tp* t, cudaStream_t s, CommTimer ct = {}) {
    const int nq = t->hq * HEAD_DIM, nkv = t->ng * HEAD_DIM;
    NcclApi* api = use_nccl(t) ? nccl() : nullptr;
    if (use_nccl(t) && !api) return MCPM_NCCL_ERROR;
    for (int l = 0; l < t->n_layer; ++l) {
        const mcpm_tp::Layer& L = t->layers[l];
        const size_t lay = static_cast<size_t>(l) * t->max_seq * KV_DIM;
        TPGemv a = gemv_base(t);   // QKV
        a.w = L.wqkv, a.rows = nq + 2 * nkv, a.nb = N_EMBD / 32, a.pro = PRO_NORM;
        a.embd = l == 0 ? t->embd : nullptr;
        a.x = t->x0, a.x_next = t->x1, a.norm = L.anorm;
        if (l > 0) set_red(t, a, 1, 2 * (l - 1) + 1);
        a.epi = EPI_ROPE, a.q = t->q + t->h0 * HEAD_DIM;
        a.kc = t->kc + lay + t->g0 * HEAD_DIM, a.vc = t->vc + lay + t->g0 * HEAD_DIM;
        a.rope = t->rope, a.nq = nq, a.nkv = nkv, a.max_seq = t->max_seq;
        TP_CUDA(launch_gemv(t, a, s));
        DecodeParams p{};   // attention of the rank's KV head(s) and head pairs
        p.q = t->q, p.kc = t->kc + lay, p.vc = t->vc + lay, p.max_seq = t->max_seq;
        p.att = t->att, p.att_q8k = t->att_q8k, p.att_part = t->att_part;
        p.err = &t->ctl->err;
        TP_CUDA(launch_tp_attention(p, &t->ctl->pos, t->g0, t->ng, t->h0 / 2, t->hq / 2, s));
        TPGemv o = gemv_base(t);   // o_proj over the rank's heads
        o.w = L.wo, o.rows = N_EMBD, o.nb = t->hq * HEAD_DIM / 32, o.pro = PRO_PLAIN;
        o.x = t->att + t->h0 * HEAD_DIM;
        set_publish(t, o, 0, 2 * l);
        TP_CUDA(launch_gemv(t, o, s));
        if (api) {
            ct.begin(s);
            const mcpm_status st = nccl_st(api->all_reduce(t->red_o, t->red_o, N_EMBD, NCCL_FLOAT32, NCCL_SUM,
                                                           t->nccl_comm, s));
            ct.end(s);
            if (st != MCPM_OK) return st;
        }
        TPGemv gu = gemv_base(t);   // Gate+Up rows of the rank's FFN slice
        gu.w = L.wgu, gu.rows = 2 * t->nf, gu.nb = N_EMBD / 32, gu.pro = PRO_NORM;
        gu.x = t->x1, gu.x_next = t->x0, gu.norm = L.fnorm;
        set_red(t, gu, 0, 2 * l);
        gu.epi = EPI_STORE, gu.y = t->gu;
        TP_CUDA(launch_gemv(t, gu, s));
        TPGemv d = gemv_base(t);   // down over the slice
        d.w = L.wd, d.rows = N_EMBD, d.nb = t->nf / 32, d.pro = PRO_SWIGLU, d.x = t->gu;
        set_publish(t, d, 1, 2 * l + 1);
        TP_CUDA(launch_gemv(t, d, s));
        if (api) {
            ct.begin(s);
            const mcpm_status st = nccl_st(api->all_reduce(t->red_d, t->red_d, N_EMBD, NCCL_FLOAT32, NCCL_SUM,
                                                           t->nccl_comm, s));
            ct.end(s);
            if (st != MCPM_OK) return st;
        }
    }
    TPGemv lm = gemv_base(t);   // LM head rows of the rank's vocabulary slice + argmax
    lm.w = t->lm, lm.rows = t->vocab_hi - t->vocab_lo, lm.nb = N_EMBD / 32, lm.pro = PRO_NORM;
    lm.x = t->x0, lm.x_next = t->x1, lm.norm = t->onorm;
    set_red(t, lm, 1, 2 * (t->n_layer - 1) + 1);
    lm.epi = EPI_ARGMAX, lm.y = t->logits, lm.am_val = t->am_val, lm.am_idx = t->am_idx, lm.vocab_off = t->vocab_lo;
    if (p2p(t)) {
        for (int k = 0; k < t->world; ++k)
            lm.am_pub[k] = slot_base(t->peer_recv[k], t->world, 2) + 2 * t->rank;
    } else {
        lm.am_local = t->am_local;
    }
    TP_CUDA(launch_gemv(t, lm, s));
    if (api) {
        ct.begin(s);
        const mcpm_status st = nccl_st(api->all_gather(t->am_local, t->gathered, 2, NCCL_FLOAT32, t->nccl_comm, s));
        ct.end(s);
        if (st != MCPM_OK) return st;
    }
    TP_CUDA(launch_pdl(k_tp_pick, dim3(1), dim3(32), 0, s, t->ctl, t->world,
                       static_cast<const unsigned long long*>(p2p(t) ? slot_base(t->recv, t->world, 2) : nullptr),
                       static_cast<const float*>(use_nccl(t) ? t->gathered : t->am_local), t->tok_log, t->max_seq));
    return MCPM_OK;
}

mcpm_status ensure_graph(mcpm_tp* t) {
    if (t->graph || !t->use_graph) return MCPM_OK;
    cudaGraph_t g = nullptr;
    TP_CUDA(cudaStreamBeginCapture(t->stream, cudaStreamCaptureModeThreadLocal));
    const mcpm_status st = enqueue_token(t, t->stream);
    const cudaError_t ce = cudaStreamEndCapture(t->stream, &g);
    if (st != MCPM_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    TP_CUDA(ce);
    const cudaError_t ie = cudaGraphInstantiate(&t->graph, g, 0);
    cudaGraphDestroy(g);
    TP_CUDA(ie);
    return MCPM_OK;
}

mcpm_status run_token(mcpm_tp* t) {
    if (t->use_graph) {
        TP_CUDA(cudaGraphLaunch(t->graph, t->stream));
        return MCPM_OK;
    }
    return enqueue_token(t, t->stream);
}

mcpm_status check_err(mcpm_tp* t) {
    TP_CUDA(cudaMemcpyAsync(t->ctl_host, t->ctl, sizeof(TPCtl), cudaMemcpyDeviceToHost, t->stream));
    TP_CUDA(cudaStreamSynchronize(t->stream));
    const unsigned err = t->ctl_host->err;
    if (err) {
        TP_CUDA(cudaMemsetAsync(&t->ctl->err, 0, sizeof(unsigned), t->stream));
        TP_CUDA(cudaStreamSynchronize(t->stream));
        if (err & ERR_BAD_TOKEN) return MCPM_BAD_TOKEN;
        if (err & ERR_BAD_ARG) return MCPM_CTX_OVERFLOW;
        return MCPM_TIMEOUT;
    }
    return MCPM_OK;
}

void free_all(mcpm_tp* t) {
    if (t->graph) cudaGraphExecDestroy(t->graph);
    t->graph = nullptr;
    for (int k = 0; k < TP_MAX_WORLD; ++k) {
        if (t->peer_recv[k] && t->peer_recv[k] != t->recv) cudaIpcCloseMemHandle(t->peer_recv[k]);
        t->peer_recv[k] = nullptr;
    }
    free_dev(t->arena);
    free_dev(t->kc);
    free_dev(t->vc);
    free_dev(t->rope);
    for (float** b : {&t->x0, &t->x1, &t->q, &t->att, &t->att_part, &t->gu, &t->red_o, &t->red_d, &t->logits,
                      &t->am_val, &t->am_local, &t->gathered})
        free_dev(*b);
    free_dev(t->am_idx);
    free_dev(t->att_q8k);
    free_dev(t->recv);
    free_dev(t->tok_log);
    t->layers.clear();
    t->loaded = false;
}

// Read-only mapping of the model file.
struct MappedFile {
    uint8_t* p = nullptr;
    size_t n = 0;
    ~MappedFile() {
        if (p) munmap(p, n);
    }
    bool open(const char* path) {
        const int fd = ::open(path, O_RDONLY);
        if (fd < 0) return false;
        struct stat st;
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            return false;
        }
        n = static_cast<size_t>(st.st_size);
        void* m = mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) return false;
        p = static_cast<uint8_t*>(m);
        return true;
    }
};

}  // namespace

extern "C" {

mcpm_status mcpm_tp_nccl_id(void* id128) {
    if (!id128) return MCPM_BAD_ARG;
    NcclApi* api = nccl();
    if (!api) return MCPM_NCCL_ERROR;
    NcclId id;
    const mcpm_status st = nccl_st(api->get_unique_id(&id));
    if (st != MCPM_OK) return st;
    std::memcpy(id128, id.internal, sizeof(id.internal));
    return MCPM_OK;
}

mcpm_status mcpm_tp_create(const mcpm_tp_config* cfg, mcpm_tp** out) {
    if (!cfg || !out) return MCPM_BAD_ARG;
    *out = nullptr;
    const int w = cfg->world;
    if (!(w == 1 || w == 2 || w == 4 || w == 8) || cfg->rank < 0 || cfg->rank >= w) return MCPM_BAD_ARG;
    if (cfg->max_seq <= 0 || cfg->max_seq > MAX_SEQ || cfg->peer_wait_us < 0) return MCPM_BAD_ARG;
    if (cfg->comm != MCPM_TP_P2P && cfg->comm != MCPM_TP_NCCL) return MCPM_BAD_ARG;
    int ndev = 0;
    TP_CUDA(cudaGetDeviceCount(&ndev));
    if (cfg->device < 0 || cfg->device >= ndev) return MCPM_BAD_ARG;
    auto t = std::make_unique<mcpm_tp>();
    t->device = cfg->device, t->rank = cfg->rank, t->world = w, t->max_seq = cfg->max_seq, t->comm = cfg->comm;
    t->wait_us = cfg->peer_wait_us > 0 ? static_cast<unsigned>(cfg->peer_wait_us) : DEFAULT_PEER_WAIT_US;
    t->use_graph = cfg->eager ? 0 : 1;
    TP_CUDA(cudaSetDevice(t->device));
    TP_CUDA(cudaDeviceGetAttribute(&t->n_sm, cudaDevAttrMultiProcessorCount, t->device));
    TP_CUDA(cudaFuncSetAttribute(k_tp_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(q80_smem_bytes())));
    TP_CUDA(cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking));
    TP_CUDA(cudaMallocHost(&t->ctl_host, sizeof(TPCtl)));
    t->hq = N_HEAD / w, t->h0 = t->rank * t->hq;
    t->g0 = w == 1 ? 0 : t->h0 / (N_HEAD / N_HEAD_KV);
    t->ng = w == 1 ? N_HEAD_KV : 1;
    t->nf = N_FF / w, t->f0 = t->rank * t->nf;
    *out = t.release();
    return MCPM_OK;
}

mcpm_status mcpm_tp_load_gguf(mcpm_tp* t, const char* path) {
    if (!t || !path) return MCPM_BAD_ARG;
    TP_CUDA(cudaSetDevice(t->device));
    free_all(t);
    t->connected = false;
    GGUFFile g;
    const std::string why = gguf_read(path, g);
    if (!why.empty()) {
        std::fprintf(stderr, "[mcpm] %s\n", why.c_str());
        return MCPM_BAD_FILE;
    }
    MappedFile mf;
    if (!mf.open(path) || mf.n < g.file_size) return MCPM_BAD_FILE;
    auto find = [&](const std::string& name) -> const GGUFTensor* {
        for (const auto& x : g.tensors)
            if (x.name == name) return &x;
        return nullptr;
    };
    auto is = [](const GGUFTensor* x, uint32_t type, uint64_t c, uint64_t r) {
        return x && x->type == type && x->dims.size() >= 1 && x->dims[0] == c &&
               (r == 0 ? x->dims.size() == 1 : x->dims.size() == 2 && x->dims[1] == r);
    };
    int n_layer = 0;
    while (find("blk." + std::to_string(n_layer) + ".attn_q.weight")) ++n_layer;
    const GGUFTensor* emb = find("token_embd.weight");
    const GGUFTensor* out = find("output.weight");
    const GGUFTensor* onorm = find("output_norm.weight");
    const uint64_t vocab = emb && emb->dims.size() == 2 ? emb->dims[1] : 0;
    if (n_layer == 0 || n_layer > MAX_LAYERS || vocab == 0 || vocab > (1u << 30) || !onorm ||
        !is(onorm, GGML_F32, N_EMBD, 0)) {
        std::fprintf(stderr, "[mcpm] missing MiniCPM5 tensors in %s\n", path);
        return MCPM_BAD_FILE;
    }
    if (!is(emb, GGML_Q8_0, N_EMBD, vocab) || !is(out, GGML_Q8_0, N_EMBD, vocab)) {
        std::fprintf(stderr, "[mcpm] tensor-parallel engine: embedding and output must be Q8_0\n");
        return MCPM_UNSUPPORTED_TYPE;
    }
    static const char* NAMES[9] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
                                   "attn_norm", "ffn_norm"};
    const uint64_t C[9] = {N_EMBD, N_EMBD, N_EMBD, N_EMBD, N_EMBD, N_EMBD, N_FF, N_EMBD, N_EMBD};
    const uint64_t R[9] = {N_EMBD, KV_DIM, KV_DIM, N_EMBD, N_FF, N_FF, N_EMBD, 0, 0};
    std::vector<std::array<const GGUFTensor*, 9>> lt(n_layer);
    for (int l = 0; l < n_layer; ++l)
        for (int i = 0; i < 9; ++i) {
            const GGUFTensor* x = find("blk." + std::to_string(l) + "." + NAMES[i] + ".weight");
            if (!x) return MCPM_BAD_FILE;
            if (!is(x, i < 7 ? GGML_Q8_0 : GGML_F32, C[i], R[i])) {
                std::fprintf(stderr, "[mcpm] tensor-parallel engine: layer %d %s must be %s with the MiniCPM5 shape\n",
                             l, NAMES[i], i < 7 ? "Q8_0" : "F32");
                return MCPM_UNSUPPORTED_TYPE;
            }
            lt[l][i] = x;
        }
    for (const auto& x : g.tensors)
        if (x.offset + x.nbytes > mf.n) return MCPM_BAD_FILE;
    t->n_layer = n_layer;
    t->n_vocab = static_cast<int>(vocab);
    const int vpairs = t->n_vocab / 2;
    t->vocab_lo = 2 * static_cast<int>(static_cast<long long>(vpairs) * t->rank / t->world);
    t->vocab_hi = t->rank == t->world - 1 ? t->n_vocab
                                          : 2 * static_cast<int>(static_cast<long long>(vpairs) * (t->rank + 1) / t->world);
    if ((t->vocab_hi - t->vocab_lo) % 2) return MCPM_UNSUPPORTED_TYPE;   // pair-aligned rows (even vocabulary)
    auto fb = g.f_kv.find("minicpm5.rope.freq_base");
    if (fb != g.f_kv.end()) t->rope_base = static_cast<float>(fb->second);

    // Shard layout in one arena (each piece 256-byte aligned).
    const size_t RB = N_EMBD / 32 * Q8_0_BYTES;                     // 2176 B per 2048-column row
    const size_t ob = static_cast<size_t>(t->hq) * HEAD_DIM / 32 * Q8_0_BYTES;   // o_proj shard row
    const size_t db = static_cast<size_t>(t->nf) / 32 * Q8_0_BYTES;             // down shard row
    const int nq = t->hq * HEAD_DIM, nkv = t->ng * HEAD_DIM;
    auto al = [](size_t n) { return (n + 255) / 256 * 256; };
    const size_t sz_qkv = al((nq + 2 * nkv) * RB), sz_o = al(N_EMBD * ob), sz_gu = al(2 * t->nf * RB),
                 sz_d = al(N_EMBD * db), sz_norm = al(N_EMBD * 4);
    const size_t per_layer = sz_qkv + sz_o + sz_gu + sz_d + 2 * sz_norm;
    const size_t sz_emb = al(static_cast<size_t>(t->n_vocab) * RB);
    const size_t sz_lm = al(static_cast<size_t>(t->vocab_hi - t->vocab_lo) * RB);
    t->arena_bytes = per_layer * n_layer + sz_emb + sz_lm + sz_norm;
    TP_CUDA(cudaMalloc(&t->arena, t->arena_bytes));
    std::vector<uint8_t> stage;
    size_t off = 0;
    auto put = [&](const uint8_t* src, size_t n, size_t reserve) -> mcpm_status {
        const cudaError_t e = cudaMemcpy(t->arena + off, src, n, cudaMemcpyHostToDevice);
        off += reserve;
        return cuda_st(e);
    };
    auto rows_of = [&](const GGUFTensor* x, size_t r0, size_t nr, size_t rb) {
        return mf.p + x->offset + r0 * rb;   // rows [r0, r0 + nr) are contiguous
    };
    auto gather_cols = [&](const GGUFTensor* x, size_t rows, size_t rb, size_t c0b, size_t cb) {
        stage.resize(rows * cb);
        for (size_t r = 0; r < rows; ++r) std::memcpy(stage.data() + r * cb, mf.p + x->offset + r * rb + c0b, cb);
        return stage.data();
    };
    t->layers.assign(n_layer, mcpm_tp::Layer{});
    for (int l = 0; l < n_layer; ++l) {
        mcpm_tp::Layer& L = t->layers[l];
        const auto& x = lt[l];
        L.wqkv = t->arena + off;
        stage.resize((nq + 2 * nkv) * RB);
        std::memcpy(stage.data(), rows_of(x[0], t->h0 * HEAD_DIM, nq, RB), nq * RB);
        std::memcpy(stage.data() + nq * RB, rows_of(x[1], t->g0 * HEAD_DIM, nkv, RB), nkv * RB);
        std::memcpy(stage.data() + (nq + nkv) * RB, rows_of(x[2], t->g0 * HEAD_DIM, nkv, RB), nkv * RB);
        mcpm_status st = put(stage.data(), stage.size(), sz_qkv);
        if (st != MCPM_OK) return st;
        L.wo = t->arena + off;
        st = put(gather_cols(x[3], N_EMBD, RB, static_cast<size_t>(t->h0) * HEAD_DIM / 32 * Q8_0_BYTES, ob),
                 N_EMBD * ob, sz_o);
        if (st != MCPM_OK) return st;
        L.wgu = t->arena + off;
        stage.resize(2 * t->nf * RB);
        std::memcpy(stage.data(), rows_of(x[4], t->f0, t->nf, RB), t->nf * RB);
        std::memcpy(stage.data() + t->nf * RB, rows_of(x[5], t->f0, t->nf, RB), t->nf * RB);
        st = put(stage.data(), stage.size(), sz_gu);
        if (st != MCPM_OK) return st;
        L.wd = t->arena + off;
        const size_t rbd = N_FF / 32 * Q8_0_BYTES;
        st = put(gather_cols(x[6], N_EMBD, rbd, static_cast<size_t>(t->f0) / 32 * Q8_0_BYTES, db), N_EMBD * db, sz_d);
        if (st != MCPM_OK) return st;
        L.anorm = reinterpret_cast<const float*>(t->arena + off);
        st = put(mf.p + x[7]->offset, N_EMBD * 4, sz_norm);
        if (st != MCPM_OK) return st;
        L.fnorm = reinterpret_cast<const float*>(t->arena + off);
        st = put(mf.p + x[8]->offset, N_EMBD * 4, sz_norm);
        if (st != MCPM_OK) return st;
    }
    t->embd = t->arena + off;
    mcpm_status st = put(mf.p + emb->offset, static_cast<size_t>(t->n_vocab) * RB, sz_emb);
    if (st != MCPM_OK) return st;
    t->lm = t->arena + off;
    st = put(rows_of(out, t->vocab_lo, t->vocab_hi - t->vocab_lo, RB),
             static_cast<size_t>(t->vocab_hi - t->vocab_lo) * RB, sz_lm);
    if (st != MCPM_OK) return st;
    t->onorm = reinterpret_cast<const float*>(t->arena + off);
    st = put(mf.p + onorm->offset, N_EMBD * 4, sz_norm);
    if (st != MCPM_OK) return st;

    // State and activations.
    const size_t kv = kv_elems(n_layer, t->max_seq);
    TP_CUDA(cudaMalloc(&t->kc, kv * 4));
    TP_CUDA(cudaMalloc(&t->vc, kv * 4));
    TP_CUDA(cudaMemset(t->kc, 0, kv * 4));
    TP_CUDA(cudaMemset(t->vc, 0, kv * 4));
    std::vector<float2> table(static_cast<size_t>(t->max_seq) * (HEAD_DIM / 2));
    for (int p = 0; p < t->max_seq; ++p) rope_row(p, t->rope_base, table.data() + static_cast<size_t>(p) * (HEAD_DIM / 2));
    TP_CUDA(cudaMalloc(&t->rope, table.size() * sizeof(float2)));
    TP_CUDA(cudaMemcpy(t->rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice));
    for (float** b : {&t->x0, &t->x1, &t->q, &t->att, &t->red_o, &t->red_d}) {
        TP_CUDA(cudaMalloc(b, N_EMBD * 4));
        TP_CUDA(cudaMemset(*b, 0, N_EMBD * 4));   // q: the heads of other ranks stay 0
    }
    TP_CUDA(cudaMalloc(&t->att_part, ATT_PART_FLOATS * 4));
    TP_CUDA(cudaMemset(t->att_part, 0, ATT_PART_FLOATS * 4));
    TP_CUDA(cudaMalloc(&t->att_q8k, Q8K_BYTES * (N_EMBD / 256)));
    TP_CUDA(cudaMalloc(&t->gu, 2 * t->nf * 4));
    TP_CUDA(cudaMalloc(&t->logits, static_cast<size_t>(t->vocab_hi - t->vocab_lo) * 4));
    TP_CUDA(cudaMalloc(&t->am_val, t->n_sm * 4));
    TP_CUDA(cudaMalloc(&t->am_idx, t->n_sm * 4));
    TP_CUDA(cudaMalloc(&t->am_local, 2 * 4));
    TP_CUDA(cudaMalloc(&t->gathered, 2 * TP_MAX_WORLD * 4));
    TP_CUDA(cudaMalloc(&t->tok_log, t->max_seq * 4));
    TP_CUDA(cudaMemset(t->tok_log, 0xff, t->max_seq * 4));
    const size_t recv_words = static_cast<size_t>(2) * t->world * N_EMBD + 2 * t->world;
    TP_CUDA(cudaMalloc(&t->recv, recv_words * 8));
    TP_CUDA(cudaMemset(t->recv, 0, recv_words * 8));
    if (!t->ctl) TP_CUDA(cudaMalloc(&t->ctl, sizeof(TPCtl)));
    if (!t->wait_ns) TP_CUDA(cudaMalloc(&t->wait_ns, sizeof(unsigned long long)));
    TPCtl c{};
    c.seq = 1;
    c.wait_us = t->wait_us;
    TP_CUDA(cudaMemcpy(t->ctl, &c, sizeof(TPCtl), cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemset(t->wait_ns, 0, sizeof(unsigned long long)));
    t->peer_recv[t->rank] = t->recv;
    t->pos_next = 0;
    t->loaded = true;
    t->connected = t->world == 1;
    return MCPM_OK;
}

mcpm_status mcpm_tp_ipc_handle(mcpm_tp* t, void* handle64) {
    if (!t || !handle64) return MCPM_BAD_ARG;
    if (!t->loaded) return MCPM_NOT_LOADED;
    TP_CUDA(cudaSetDevice(t->device));
    cudaIpcMemHandle_t h;
    static_assert(sizeof(h) == 64, "IPC handle size");
    TP_CUDA(cudaIpcGetMemHandle(&h, t->recv));
    std::memcpy(handle64, &h, sizeof(h));
    return MCPM_OK;
}

mcpm_status mcpm_tp_connect(mcpm_tp* t, const void* nccl_id128, const void* ipc_handles) {
    if (!t) return MCPM_BAD_ARG;
    if (!t->loaded) return MCPM_NOT_LOADED;
    TP_CUDA(cudaSetDevice(t->device));
    if (t->world == 1) {
        t->connected = true;
        return MCPM_OK;
    }
    if (t->comm == MCPM_TP_NCCL) {
        if (!nccl_id128) return MCPM_BAD_ARG;
        NcclApi* api = nccl();
        if (!api) return MCPM_NCCL_ERROR;
        NcclId id;
        std::memcpy(id.internal, nccl_id128, sizeof(id.internal));
        const mcpm_status st = nccl_st(api->comm_init_rank(&t->nccl_comm, t->world, id, t->rank));
        if (st != MCPM_OK) return st;
    } else {
        if (!ipc_handles) return MCPM_BAD_ARG;
        for (int k = 0; k < t->world; ++k) {
            if (k == t->rank) continue;
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t*>(ipc_handles) + 64 * k, 64);
            void* p = nullptr;
            TP_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
            t->peer_recv[k] = static_cast<unsigned long long*>(p);
        }
    }
    t->connected = true;
    return MCPM_OK;
}

mcpm_status mcpm_tp_forward(mcpm_tp* t, int token, int pos, float* logits_slice, int* next_token) {
    if (!t) return MCPM_BAD_ARG;
    if (!t->loaded || !t->connected) return MCPM_NOT_LOADED;
    if (token >= t->n_vocab) return MCPM_BAD_TOKEN;
    TP_CUDA(cudaSetDevice(t->device));
    if (token >= 0) {
        if (pos < 0 || pos >= t->max_seq) return MCPM_CTX_OVERFLOW;
        int tp[2] = {token, pos};
        TP_CUDA(cudaMemcpyAsync(t->ctl, tp, sizeof(tp), cudaMemcpyHostToDevice, t->stream));
        t->pos_next = pos;
    } else if (t->pos_next >= t->max_seq) {
        return MCPM_CTX_OVERFLOW;
    }
    mcpm_status st = ensure_graph(t);
    if (st != MCPM_OK) return st;
    st = run_token(t);
    if (st != MCPM_OK) return st;
    t->pos_next += 1;
    if (logits_slice)
        TP_CUDA(cudaMemcpyAsync(logits_slice, t->logits, static_cast<size_t>(t->vocab_hi - t->vocab_lo) * 4,
                                cudaMemcpyDeviceToHost, t->stream));
    st = check_err(t);
    if (st != MCPM_OK) return st;
    if (next_token) *next_token = t->ctl_host->token;
    return MCPM_OK;
}

mcpm_status mcpm_tp_generate_async(mcpm_tp* t, int n) {
    if (!t || n < 0) return MCPM_BAD_ARG;
    if (!t->loaded || !t->connected) return MCPM_NOT_LOADED;
    if (t->pos_next + n > t->max_seq) return MCPM_CTX_OVERFLOW;
    TP_CUDA(cudaSetDevice(t->device));
    mcpm_status st = ensure_graph(t);
    if (st != MCPM_OK) return st;
    for (int i = 0; i < n; ++i) {
        st = run_token(t);
        if (st != MCPM_OK) return st;
    }
    t->pos_next += n;
    return MCPM_OK;
}

mcpm_status mcpm_tp_sync(mcpm_tp* t) {
    if (!t) return MCPM_BAD_ARG;
    TP_CUDA(cudaSetDevice(t->device));
    return check_err(t);
}

mcpm_status mcpm_tp_read_tokens(mcpm_tp* t, int pos0, int n, int* tokens) {
    if (!t || !tokens || pos0 < 0 || n < 0 || pos0 + n > t->max_seq) return MCPM_BAD_ARG;
    if (!t->loaded) return MCPM_NOT_LOADED;
    TP_CUDA(cudaSetDevice(t->device));
    TP_CUDA(cudaMemcpyAsync(tokens, t->tok_log + pos0, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, t->stream));
    return check_err(t);
}

mcpm_status mcpm_tp_info(mcpm_tp* t, int info[8]) {
    if (!t || !info) return MCPM_BAD_ARG;
    if (!t->loaded) return MCPM_NOT_LOADED;
    info[0] = t->n_layer, info[1] = t->n_vocab, info[2] = t->vocab_lo, info[3] = t->vocab_hi;
    info[4] = t->h0, info[5] = t->hq, info[6] = t->f0, info[7] = t->nf;
    return MCPM_OK;
}

mcpm_status mcpm_tp_reset(mcpm_tp* t) {
    if (!t) return MCPM_BAD_ARG;
    if (!t->loaded) return MCPM_NOT_LOADED;
    TP_CUDA(cudaSetDevice(t->device));
    TP_CUDA(cudaStreamSynchronize(t->stream));
    const size_t kv = kv_elems(t->n_layer, t->max_seq);
    TP_CUDA(cudaMemsetAsync(t->kc, 0, kv * 4, t->stream));
    TP_CUDA(cudaMemsetAsync(t->vc, 0, kv * 4, t->stream));
    TP_CUDA(cudaMemsetAsync(t->tok_log, 0xff, t->max_seq * 4, t->stream));
    // Step counter back to 1 and the receive slots cleared: after a timeout the ranks may have
    // run different numbers of steps, and values of an earlier step must not match a new epoch.
    // Every rank resets between steps (none in flight) before any rank steps again.
    TPCtl c{};
    c.seq = 1;
    c.wait_us = t->wait_us;
    TP_CUDA(cudaMemcpyAsync(t->ctl, &c, sizeof(TPCtl), cudaMemcpyHostToDevice, t->stream));
    if (t->recv) {
        const size_t recv_words = static_cast<size_t>(2) * t->world * N_EMBD + 2 * t->world;
        TP_CUDA(cudaMemsetAsync(t->recv, 0, recv_words * 8, t->stream));
    }
    TP_CUDA(cudaStreamSynchronize(t->stream));
    t->pos_next = 0;
    return MCPM_OK;
}

mcpm_status mcpm_tp_profile(mcpm_tp* t, int n, float* ms_token, float* ms_comm) {
    if (!t || n <= 0 || !ms_token || !ms_comm) return MCPM_BAD_ARG;
    if (!t->loaded || !t->connected) return MCPM_NOT_LOADED;
    if (t->pos_next + n > t->max_seq) return MCPM_CTX_OVERFLOW;
    TP_CUDA(cudaSetDevice(t->device));
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
    CommTimer ct;
    if (use_nccl(t)) ct.ev = &ev;
    t->profile = true;
    TP_CUDA(cudaMemsetAsync(t->wait_ns, 0, sizeof(unsigned long long), t->stream));
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, t->stream);
    mcpm_status st = MCPM_OK;
    for (int i = 0; i < n && st == MCPM_OK; ++i) st = enqueue_token(t, t->stream, ct);   // eager launches
    cudaEventRecord(b, t->stream);
    t->profile = false;
    const mcpm_status st2 = check_err(t);
    float total = 0.0f, comm = 0.0f;
    cudaEventElapsedTime(&total, a, b);
    for (auto& e : ev) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e.first, e.second);
        comm += ms;
        cudaEventDestroy(e.first);
        cudaEventDestroy(e.second);
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (st != MCPM_OK) return st;
    if (st2 != MCPM_OK) return st2;
    if (p2p(t)) {
        unsigned long long ns = 0;
        TP_CUDA(cudaMemcpy(&ns, t->wait_ns, sizeof(ns), cudaMemcpyDeviceToHost));
        comm = static_cast<float>(ns * 1e-6);
    }
    t->pos_next += n;
    *ms_token = total / n;
    *ms_comm = comm / n;
    return MCPM_OK;
}

void* mcpm_tp_stream(mcpm_tp* t) { return t ? reinterpret_cast<void*>(t->stream) : nullptr; }

void mcpm_tp_destroy(mcpm_tp* t) {
    if (!t) return;
    cudaSetDevice(t->device);
    if (t->stream) cudaStreamSynchronize(t->stream);
    free_all(t);
    if (t->nccl_comm) {
        NcclApi* api = nccl();
        if (api) api->comm_destroy(t->nccl_comm);
    }
    free_dev(t->ctl);
    free_dev(t->wait_ns);
    if (t->ctl_host) cudaFreeHost(t->ctl_host);
    if (t->stream) cudaStreamDestroy(t->stream);
    delete t;
}

}  // extern "C"
