// Persistent decode kernel: one cooperative launch computes one token of
// MiniCPM5Engine::forward (reference src/model.cpp:142-242) on every SM.
//
// Per layer five phases separated by a grid barrier:
//   QKV  : RMSNorm -> Q8_K (every CTA, redundantly), fused Q/K/V GEMV over this CTA's
//          row pairs, RoPE on Q/K pairs, K/V appended to the cache at `pos`
//          (ops.cpp:676-723, ops_avx2.cpp:320-374, ops.cpp:502-516, 557-563)
//   ATT  : split-KV attention, chunk partials + last-CTA combine + Q8_K (ties-to-even)
//          quantisation of the attention output (ops.cpp:537-628, ops_avx2.cpp:85-144)
//   O    : o_proj GEMV + residual add (model.cpp:198-203)
//   GU   : RMSNorm -> Q8_K, gate/up GEMV, SwiGLU (ops_avx2.cpp:444-460, ops.cpp:725-765)
//   D    : SwiGLU output -> Q8_K (every CTA), down GEMV + residual (model.cpp:220-225)
// then the LM head (final RMSNorm, Q8_K ties-to-even, GEMV, greedy argmax).
//
// Weights move with TMA bulk copies (cp.async.bulk into this CTA's own shared memory) into two shared
// buffers; the copy for weight phase w+1 is issued when phase w starts, so HBM keeps
// streaming through the grid barriers.  All waits are bounded (~1 s) and report
// ERR_TIMEOUT instead of hanging.
#include "mcpm_device.cuh"
#include "mcpm_gemv_bo.cuh"
#include "mcpm_internal.h"
#include <algorithm>
#include <initializer_list>

namespace mcpm {
namespace {

// Per-layer fields the phases read on their critical path, copied to shared memory at
// kernel start: a field read from global memory costs a full L2 round trip there
// (the L1 is almost all carved out for shared memory).
struct LayerMeta {
    uint32_t w[7];                  // arena offsets of wq, wk, wv, wo, wg, wu, wd
    uint32_t attn_norm, ffn_norm;   // arena offsets of the norm weights
    uint8_t tq, tk, tv, to, tg, tu, td, pad;
    int16_t qkv0, qkv1;             // this CTA's rows of the combined [Q; K; V] (cost-weighted split)
};
// This CTA's rows of the 2048-row (o_proj, down) and 6144-row (gate/up) phases.
struct CtaRows {
    int od0, od1, gu0, gu1;
};
__device__ __forceinline__ const float* meta_f32(const DecodeParams& p, uint32_t off) {
    return reinterpret_cast<const float*>(p.arena + off);
}

// GEMV partials and the staged fp32 activation share one scratch region.
constexpr int SCRATCH_BYTES = MAX_TASKS * PART_WORDS * 4 > N_EMBD * 4 ? MAX_TASKS * PART_WORDS * 4 : N_EMBD * 4;

// Dynamic shared memory of the decode kernel (and of k_attention, launched with the same
// size): fixed offsets from one base, so no pointer to it is held in a register.
extern __shared__ __align__(1024) uint8_t smem_raw[];
constexpr int SM_WBUF0 = 0;
constexpr int SM_WBUF1 = WBUF_BYTES + WBUF_SLACK;
constexpr int SM_XQ = 2 * (WBUF_BYTES + WBUF_SLACK);
constexpr int SM_SCRATCH = SM_XQ + ((static_cast<int>(sizeof(XQSmem)) + 127) & ~127);
constexpr int SM_ROWVAL = SM_SCRATCH + SCRATCH_BYTES;
constexpr int SM_RED = SM_ROWVAL + ROWVAL_FLOATS * 4;
constexpr int SM_WBAR = SM_RED + 32 * 4;
constexpr int SM_LMBAR = SM_WBAR + 8 * 8;
constexpr int SM_FLAG = SM_LMBAR + 4 * 8;
constexpr int SM_ROWS = SM_FLAG + 16;
constexpr int SM_META = SM_ROWS + 16;
constexpr int SM_BYTES = SM_META + MAX_LAYERS * static_cast<int>(sizeof(LayerMeta));

struct Smem {
    __device__ uint8_t* wbuf(int i) const { return smem_raw + (i ? SM_WBUF1 : SM_WBUF0); }
    __device__ XQSmem* xq() const { return reinterpret_cast<XQSmem*>(smem_raw + SM_XQ); }
    __device__ int* part() const { return reinterpret_cast<int*>(smem_raw + SM_SCRATCH); }   // GEMV scratch
    __device__ float* xs() const { return reinterpret_cast<float*>(smem_raw + SM_SCRATCH); }  // same storage
    __device__ float* rowval() const { return reinterpret_cast<float*>(smem_raw + SM_ROWVAL); }
    __device__ float* red() const { return reinterpret_cast<float*>(smem_raw + SM_RED); }      // 32 floats
    __device__ uint64_t* wbar() const { return reinterpret_cast<uint64_t*>(smem_raw + SM_WBAR); }   // [2][4]
    __device__ uint64_t* lmbar() const { return reinterpret_cast<uint64_t*>(smem_raw + SM_LMBAR); } // [4]
    __device__ CtaRows* rows() const { return reinterpret_cast<CtaRows*>(smem_raw + SM_ROWS); }
    __device__ LayerMeta* meta() const { return reinterpret_cast<LayerMeta*>(smem_raw + SM_META); }   // [n_layer]
    __device__ int* flags() const { return reinterpret_cast<int*>(smem_raw + SM_FLAG); }   // [0]: early_gu
};

__device__ __forceinline__ void split_range(int n, int cta, int ncta, int& a, int& b) {
    a = static_cast<int>((static_cast<long long>(n) * cta) / ncta);
    b = static_cast<int>((static_cast<long long>(n) * (cta + 1)) / ncta);
}

// Row layout of weight phase `kind` for this CTA inside its buffer.
struct PhaseLayout {
    int row0[3], nrows[3];
    uint32_t off[3], bytes[3];
};

__device__ __forceinline__ uint32_t align16(uint32_t v) { return (v + 15u) & ~15u; }

// Row splits are precomputed at kernel start (CtaRows, LayerMeta::qkv0/1): the 64-bit
// divisions they need would otherwise sit on every phase's critical path.
__device__ PhaseLayout phase_layout(const LayerMeta& L, const CtaRows& cr, int kind) {
    PhaseLayout pl;
#pragma unroll
    for (int i = 0; i < 3; ++i) pl.row0[i] = pl.nrows[i] = 0, pl.off[i] = pl.bytes[i] = 0;
    int a, b;
    if (kind == 0) {   // QKV: row pairs of the combined [Q; K; V] rows, cost-weighted split
        a = L.qkv0;
        b = L.qkv1;
        const int lo[3] = {0, N_EMBD, N_EMBD + KV_DIM}, hi[3] = {N_EMBD, N_EMBD + KV_DIM, QKV_ROWS};
        const int types[3] = {L.tq, L.tk, L.tv};
        uint32_t off = 0;
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            const int s = max(a, lo[i]), e = min(b, hi[i]);
            pl.row0[i] = max(0, s - lo[i]);
            pl.nrows[i] = max(0, e - s);
            pl.off[i] = off;
            pl.bytes[i] = pl.nrows[i] * row_bytes(types[i], N_EMBD);
            off = align16(off + pl.bytes[i]);
        }
    } else if (kind == 1 || kind == 3) {   // O, D: 2048 output rows
        a = cr.od0;
        b = cr.od1;
        pl.row0[0] = a;
        pl.nrows[0] = b - a;
        pl.bytes[0] = (b - a) * (kind == 1 ? row_bytes(L.to, N_EMBD) : row_bytes(L.td, N_FF));
    } else {   // GU: gate rows then up rows
        a = cr.gu0;
        b = cr.gu1;
        pl.row0[0] = pl.row0[1] = a;
        pl.nrows[0] = pl.nrows[1] = b - a;
        pl.bytes[0] = (b - a) * row_bytes(L.tg, N_EMBD);
        pl.off[1] = align16(pl.bytes[0]);
        pl.bytes[1] = (b - a) * row_bytes(L.tu, N_EMBD);
    }
    return pl;
}

__device__ const uint8_t* phase_src(const DecodeParams& p, const LayerMeta& M, int kind, int i) {
    const int k = kind == 0 ? i : kind == 1 ? 3 : kind == 2 ? 4 + i : 6;
    return p.arena + M.w[k];
}

__device__ int phase_type(const LayerMeta& L, int kind, int i) {
    if (kind == 0) return i == 0 ? L.tq : i == 1 ? L.tk : L.tv;
    if (kind == 1) return L.to;
    if (kind == 2) return i == 0 ? L.tg : L.tu;
    return L.td;
}

__device__ int phase_cols(int kind) { return kind == 3 ? N_FF : N_EMBD; }

// Thread 0 only: arm the four barriers of buffer (wp & 1) and issue weight phase `wp`.
// `half`: -1 issues the whole phase; 0 / 1 issue the first / second half of the rows of a
// single-segment phase (down), on barriers 0 / 3, so its copy can be spread over time.
__device__ void issue_weight_phase(const DecodeParams& p, const Smem& s, int wp, int cta, int ncta, int half = -1) {
    const int buf = wp & 1;
    uint64_t* bars = s.wbar() + 4 * buf;
    const int l = wp >> 2, kind = wp & 3;
    const LayerMeta& M = s.meta()[l];
    const PhaseLayout pl = phase_layout(M, *s.rows(), kind);
    const uint64_t pol = l2_evict_first_policy();
    if (half >= 0) {   // down: rows [0, n/2) on barrier 0, [n/2, n) on barrier 3
        const int rb = row_bytes(phase_type(M, kind, 0), phase_cols(kind));
        const int n0 = pl.nrows[0] / 2, a = half ? n0 : 0, n = half ? pl.nrows[0] - n0 : n0;
        const uint32_t bytes = static_cast<uint32_t>(n) * rb;
        uint64_t* bar = &bars[half ? 3 : 0];
        mbar_expect_tx(bar, bytes);
        if (bytes)
            bulk_g2s_stream(s.wbuf(buf) + static_cast<size_t>(a) * rb,
                            phase_src(p, M, kind, 0) + static_cast<size_t>(pl.row0[0] + a) * rb, bytes, bar, pol);
        if (half == 0) {
            mbar_expect_tx(&bars[1], 0);
            mbar_expect_tx(&bars[2], 0);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        mbar_expect_tx(&bars[i], pl.bytes[i]);
        if (pl.bytes[i]) {
            const int rb = row_bytes(phase_type(M, kind, i), phase_cols(kind));
            bulk_g2s_stream(s.wbuf(buf) + pl.off[i], phase_src(p, M, kind, i) + static_cast<size_t>(pl.row0[i]) * rb,
                            pl.bytes[i], &bars[i], pol);
        }
    }
    mbar_expect_tx(&bars[3], 0);
}

// LM-head ring: stage st covers rows [r0 + st*SR, ...) of this CTA's vocabulary range.
struct LmPlan {
    int r0, r1, sr, nstages, rb, nb;
};
__device__ LmPlan lm_plan(const DecodeParams& p, int cta, int ncta) {
    LmPlan q;
    split_range(p.n_vocab, cta, ncta, q.r0, q.r1);
    q.rb = row_bytes(p.lm_type, N_EMBD);
    q.nb = N_EMBD / 256;
    q.sr = min(LM_SLOT_BYTES / q.rb, MAX_TASKS / q.nb);
    q.nstages = (q.r1 - q.r0 + q.sr - 1) / q.sr;
    return q;
}
__device__ uint8_t* lm_slot(const Smem& s, int slot) { return s.wbuf(0) + slot * LM_SLOT_STRIDE; }
__device__ void issue_lm_stage(const DecodeParams& p, const Smem& s, const LmPlan& q, int st) {
    const int slot = st % LM_SLOTS;
    const int a = q.r0 + st * q.sr, n = min(q.sr, q.r1 - a);
    const uint32_t bytes = n > 0 ? static_cast<uint32_t>(n) * q.rb : 0;
    mbar_expect_tx(&s.lmbar()[slot], bytes);
    if (bytes) bulk_g2s_stream(lm_slot(s, slot), p.lm + static_cast<size_t>(a) * q.rb, bytes, &s.lmbar()[slot], l2_evict_first_policy());
}

// Bounded grid barrier (all CTAs co-resident: cooperative launch).  A monotonic arrival
// counter: barrier i of a launch completes when the counter reaches base + (i+1)*ncta, so
// the last arrival costs one fire-and-forget release-add and the waiters one acquire poll.
// `base` (bar[1]) is advanced by CTA 0 after the launch's last barrier; the host zeroes both
// words after an error.  While waiting, thread 0 runs `during` (issues the next TMA copies).
// Only thread 0 touches global memory here: its acquire plus the closing bar.red order the
// other CTAs' writes before every thread's later reads.  The error word is read relaxed,
// in the shadow of the poll; an error raised during this wait is seen at the next barrier
// (or by the bounded waits).
struct BarState {
    unsigned base;
    unsigned idx;
};

template <typename F>
__device__ bool grid_barrier(const DecodeParams& p, BarState& bs, F&& during) {
    __syncthreads();
    int bad = 0;
    if (threadIdx.x == 0) {
        red_release_add_u32(p.bar, 1u);
        const unsigned e = ld_relaxed_u32(p.err);
        during();
        const unsigned target = bs.base + (bs.idx + 1) * gridDim.x;
        if (static_cast<int>(ld_acquire_u32(p.bar) - target) < 0) {
            const uint64_t t0 = globaltimer();
            while (static_cast<int>(ld_acquire_u32(p.bar) - target) < 0) {
                if (globaltimer() - t0 > 1000000000ull) {
                    atomicOr(p.err, ERR_TIMEOUT);
                    bad = 1;
                    break;
                }
            }
        }
        bad |= e != 0;
    }
    ++bs.idx;
    return __syncthreads_or(bad) == 0;
}

// Trace: CTA 0 records when phase `ph` finished its own work (slot 2+2ph) and when the
// barrier after it released (slot 3+2ph).
__device__ __forceinline__ void trace_mark(const DecodeParams& p, int slot) {
    if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) p.trace[slot] = globaltimer();
}

// Sub-step marks inside the phases of layer 1 (phase kind ph: 0 QKV .. 4 D, 5 LM).
__device__ __forceinline__ void trace_step(const DecodeParams& p, int l, int ph, int step) {
    if (l == 1) trace_mark(p, TRACE_DETAIL + 10 * ph + step);
    if (l == 1 && ph == 0 && step <= 3 && p.trace && threadIdx.x == 0 && blockIdx.x < 148)
        p.trace[2400 + 148 * (step - 1) + blockIdx.x] = globaltimer();
}

// GEMV of a decode phase over rows staged in this CTA's shared memory: rows [0, R0) at w0 and
// [R0, R) at w1 (same type), in the engine's order -- the block order (exact block sums, one fma
// per block in groups of four) or the reference's eight-lane AVX2 order.
__device__ __forceinline__ void dec_gemv(const DecodeParams& p, const Smem& s, int type, const uint8_t* w0, int R0,
                                         const uint8_t* w1, int R, int nb, float* out, unsigned long long* tr) {
    if (p.blk_order)
        gemv_bo2(type, w0, R0, w1, R, nb, *s.xq(), s.part(), SCRATCH_BYTES / 4, out);
    else
        gemv_rows2(type, w0, R0, w1, R, nb, *s.xq(), s.part(), MAX_TASKS, out, tr);
}

// Thread that issues weight copies and prefetches at the end of o_proj and down: outside
// warps 0-7, which poll the epoch-tagged residual in the following norm.
constexpr int ISSUE_THREAD = 256;

// Per-CTA marks of layer 1 for boundaries without a grid barrier (k as in traced_barrier:
// 0 QKV, 2 o_proj, 4 down): `rel` 0 when the phase finished, 1 when its consumer's wait ended.
__device__ __forceinline__ void trace_cta(const DecodeParams& p, int l, int k, int rel) {
    if (p.trace && l == 1 && threadIdx.x == 0 && blockIdx.x < 148)
        p.trace[TRACE_CTA + 740 * rel + 148 * k + blockIdx.x] = globaltimer();
}

template <typename F>
__device__ bool traced_barrier(const DecodeParams& p, BarState& bs, int ph, F&& during) {
    trace_mark(p, 2 + 2 * ph);
    const bool per_cta = p.trace && threadIdx.x == 0 && ph >= 5 && ph < 10 && blockIdx.x < 148;
    if (per_cta) {
        p.trace[TRACE_CTA + 148 * (ph - 5) + blockIdx.x] = globaltimer();
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        p.trace[TRACE_CTA + 1480 + blockIdx.x] = smid;
    }
    const bool ok = grid_barrier(p, bs, during);
    if (per_cta) p.trace[TRACE_CTA + 740 + 148 * (ph - 5) + blockIdx.x] = globaltimer();
    trace_mark(p, 3 + 2 * ph);
    return ok;
}

// Thread 0: L2 prefetch of the K/V rows (both KV heads, contiguous) of this CTA's
// attention chunk of layer l; the row at pos is written later by the QKV phase.
template <typename KT>
__device__ void prefetch_attention(const DecodeParams& p, int l, int cta) {
    const int n = p.pos + 1, P = 32 * ((n + 2047) / 2048), C = (n + P - 1) / P;
    if (cta >= 2 * C) return;
    const int c = cta % C, t0 = c * P, t1 = min(t0 + P, n);
    const size_t off = (static_cast<size_t>(l) * p.max_seq + t0) * KV_DIM;
    const uint32_t bytes = static_cast<uint32_t>(t1 - t0) * KV_DIM * sizeof(KT);
    bulk_prefetch_l2(reinterpret_cast<const KT*>(p.kc) + off, bytes);
    bulk_prefetch_l2(reinterpret_cast<const KT*>(p.vc) + off, bytes);
}

// L2 prefetch of layer l's two norm weight vectors (8 KB each), by CTA 0 only.
__device__ void prefetch_norms(const DecodeParams& p, const Smem& s, int l, int cta) {
    if (cta != 0) return;
    bulk_prefetch_l2(meta_f32(p, s.meta()[l].attn_norm), N_EMBD * 4);
    bulk_prefetch_l2(meta_f32(p, s.meta()[l].ffn_norm), N_EMBD * 4);
}

// L2 prefetch of this CTA's rows of layer l's weight phases kind0..3, fire and forget (each CTA
// fetches its own rows): their shared-memory copies, one layer later, then read L2.
__device__ __noinline__ void prefetch_layer_l2(const DecodeParams& p, const Smem& s, int l, int kind0) {
    if (!(p.sched & SCHED_L2_PREFETCH)) return;
    const LayerMeta& M = s.meta()[l];
    for (int kind = kind0; kind < 4; ++kind) {
        const PhaseLayout pl = phase_layout(M, *s.rows(), kind);
        for (int i = 0; i < 3; ++i) {
            if (pl.bytes[i] == 0) continue;
            const int rb = row_bytes(phase_type(M, kind, i), phase_cols(kind));
            bulk_prefetch_l2(phase_src(p, M, kind, i) + static_cast<size_t>(pl.row0[i]) * rb, pl.bytes[i]);
        }
    }
}

// Weight copies into shared memory are issued while a GEMV computes, never in front of a
// handoff: on an SM whose TMA copy is in flight, the loads of a handoff (epoch polls, the
// attention partials, h) queue behind the copy's bytes.  Phase w+1's copy goes into the
// buffer of phase w-1 when phase w's weights have arrived; gate/up (buffer 0) goes when
// attention is done (its copy during attention delayed the q/K/V hand-off more than it
// saved).  With SCHED_EARLY_GU it goes right after the QKV GEMV, which needs the attention
// scratch out of buffer 0: behind o_proj's rows in buffer 1 (`early_gu`, contexts up to 2048
// positions; longer contexts stage more K/V rows and keep buffer 0).
constexpr int ATT_B1_OFF = 28672;   // attention scratch offset inside buffer 1
static_assert(ATT_B1_OFF + (32 * HEAD_DIM + 8 * 32 + 32 + 8 * HEAD_DIM + HEAD_DIM) * 4 <= WBUF_BYTES,
              "32-position unit scratch behind o_proj's rows");
static_assert(ATT_B1_OFF + (2 * ATT_MAX_CHUNKS * HEAD_DIM + 6 * ATT_MAX_CHUNKS + 4 + 256) * 4 <= WBUF_BYTES,
              "head-pair combine scratch behind o_proj's rows");
constexpr int COPY_THREAD = DEC_THREADS - 1;   // last warp: the fewest GEMV tasks

// Weight phase wp (after the last layer: the LM head's first stage) into its buffer; the
// fence orders this CTA's generic-proxy writes to the buffer (attention scratch) before it.
__device__ __forceinline__ void issue_copy(const DecodeParams& p, const Smem& s, int wp, int cta, int ncta) {
    fence_proxy_async_smem();
    if (wp < 4 * p.n_layer) {
        issue_weight_phase(p, s, wp, cta, ncta);
    } else {
        const LmPlan q = lm_plan(p, cta, ncta);
        issue_lm_stage(p, s, q, 0);
    }
}

// Waits for this CTA's part of weight phase wp; false on timeout.
__device__ bool wait_weights(const DecodeParams& p, const Smem& s, int wp) {
    const int buf = wp & 1;
    const uint32_t parity = (wp >> 1) & 1;
    bool ok = true;
    for (int i = 0; i < 4; ++i) ok &= mbar_wait(&s.wbar()[4 * buf + i], parity, p.err);
    return !__syncthreads_or(!ok);   // one decision for the whole CTA
}

// ------------------------------------------------------------- activation prologues
// xs <- embedding row of `token` (get_embedding, ops.cpp:631-673; Q4_K rows).
__device__ void embed_row(const uint8_t* embd, int token, float* xs) {
    const int tid = threadIdx.x;
    if (tid < 256) {
        const int b = tid >> 5, l = tid & 31;   // block b, elements 8l .. 8l+7
        const uint8_t* blk = embd + (static_cast<size_t>(token) * (N_EMBD / 256) + b) * Q4K_BYTES;
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk);
        const float d = h2f(w0), dmin = h2f(w0 >> 16);
        const int j = (8 * l) >> 6, i0 = (8 * l) & 63;   // 64-element chunk, offset inside it
        const bool hi = i0 >= 32;
        const uint8_t* q = blk + 4;
        const int sub = 2 * j + (hi ? 1 : 0);
        int sc, mn;
        if (sub < 4) {
            sc = q[sub] & 63;
            mn = q[sub + 4] & 63;
        } else {
            sc = (q[sub + 4] & 15) | ((q[sub - 4] >> 6) << 4);
            mn = (q[sub + 4] >> 4) | ((q[sub] >> 6) << 4);
        }
        const float d1 = __fmul_rn(d, static_cast<float>(sc)), m1 = __fmul_rn(dmin, static_cast<float>(mn));
        const uint8_t* qs = blk + 16 + 32 * j + (i0 & 31);
        for (int k = 0; k < 8; ++k) {
            const int nib = hi ? (qs[k] >> 4) : (qs[k] & 15);
            xs[256 * b + 8 * l + k] = __fsub_rn(__fmul_rn(d1, static_cast<float>(nib)), m1);
        }
    }
}

// Q8_K block `blk` of s.xq() from the warp's 256 values (lane l: a = y[8l..8l+3], b = y[8l+4..8l+7]).
template <bool AWAY>
__device__ __forceinline__ void quant_xq(float4 a, float4 b, XQSmem* xq, int blk) {
    const float y[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    quant_block_warp<AWAY>(y, xq->qs[blk], &xq->d[blk], xq->bsums[blk]);
}

// Reads x[tid + 256 i] (i < 8) from epoch-tagged words, polling until every word carries
// `epoch` (written by the phase that produced x).  False after the 1 s bound.
__device__ bool load8_epoch(const unsigned long long* src, unsigned epoch, int tid, float (&xv)[8], unsigned* err) {
    unsigned long long w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = ld_epoch(src + tid + 256 * i);
    unsigned pending = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) pending |= static_cast<unsigned>((w[i] >> 32) != epoch) << i;
    if (pending) {
        const uint64_t t0 = globaltimer();
        while (pending) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (pending & (1u << i)) w[i] = ld_epoch(src + tid + 256 * i);
            pending = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) pending |= static_cast<unsigned>((w[i] >> 32) != epoch) << i;
            if (pending && globaltimer() - t0 > 1000000000ull) {
                atomicOr(err, ERR_TIMEOUT);
                return false;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = __uint_as_float(static_cast<unsigned>(w[i]));
    return true;
}

// xq <- Q8_K of (x * w) * rms(x), canonical order; rounding per template argument.
// SRC: X_SMEM (x already staged in s.xs()), X_EPOCH (x published by the previous phase as
// epoch-tagged words in p.xll; x is staged in s.xs()).  False (for the whole CTA) when the
// wait for x timed out.
enum { X_SMEM = 1, X_EPOCH = 2 };
template <bool AWAY, int SRC>
__device__ bool norm_quant(const DecodeParams& p, const float* x, unsigned epoch, const float* w, const Smem& s,
                           int trace_slot = -1) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float4 w0 = make_float4(0.f, 0.f, 0.f, 0.f), w1 = w0;
    if (warp < N_EMBD / 256) {   // norm weights first: independent of x
        w0 = __ldg(reinterpret_cast<const float4*>(w + 256 * warp + 8 * lane));
        w1 = __ldg(reinterpret_cast<const float4*>(w + 256 * warp + 8 * lane + 4));
    }
    float* red = s.red();
    bool ok = true;
    if (tid < 256) {
        float xv[8];
        if (SRC == X_EPOCH) {
            ok = load8_epoch(p.xll + (blockIdx.x % XLL_COPIES) * N_EMBD, epoch, tid, xv, p.err);
#pragma unroll
            for (int i = 0; i < 8; ++i) s.xs()[tid + 256 * i] = xv[i];
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] = x[tid + 256 * i];
        }
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = __fmaf_rn(xv[i], xv[i], a);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) red[warp] = a;
    }
    if (__syncthreads_or(!ok)) return false;
    if (trace_slot >= 0 && p.trace && threadIdx.x == 0 && blockIdx.x < 148) p.trace[trace_slot + blockIdx.x] = globaltimer();
    if (warp < N_EMBD / 256) {
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3])),
                                   __fadd_rn(__fadd_rn(red[4], red[5]), __fadd_rn(red[6], red[7])));
        const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(N_EMBD)), 1e-6f)));
        const float4 xa = *reinterpret_cast<const float4*>(s.xs() + 256 * warp + 8 * lane);
        const float4 xc = *reinterpret_cast<const float4*>(s.xs() + 256 * warp + 8 * lane + 4);
        const float xb[8] = {xa.x, xa.y, xa.z, xa.w, xc.x, xc.y, xc.z, xc.w};
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float y[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = __fmul_rn(__fmul_rn(xb[k], wv[k]), rms);
        quant_xq<AWAY>(make_float4(y[0], y[1], y[2], y[3]), make_float4(y[4], y[5], y[6], y[7]), s.xq(), warp);
    }
    __syncthreads();
    return true;
}

// Epoch of layer l's q and K/V rows in p.qll (own buffer, so the same numbering is free).
__device__ __forceinline__ unsigned qkv_epoch(unsigned seq, int l) { return (seq << 8) | static_cast<unsigned>(l + 1); }

// Epoch of the residual published by layer l's o_proj (k = 2l+1) or down (k = 2l+2) in
// launch `seq` (24 bits, never 0 after the host zeroes the words).
__device__ __forceinline__ unsigned x_epoch(unsigned seq, int k) { return (seq << 8) | static_cast<unsigned>(k); }

// Epoch of layer l's attention records (chunk headers in p.att_part, combined values in
// p.attw).  The standalone attention op uses seq = 1.
__device__ __forceinline__ unsigned att_epoch(unsigned seq, int l) { return (seq << 8) | static_cast<unsigned>(l); }

// Chunk record [head][chunk] in p.att_part: a 16-byte header of two epoch-tagged words
// (chunk max m, chunk sum l), then o[128].  Up to DIST_COMBINE_MAX chunks a grid barrier
// separates the records from their readers; beyond, the head-pair combiners poll the
// headers, which are then written after the record's o values with a fence in between.
__device__ __forceinline__ unsigned long long* att_header(const DecodeParams& p, int h, int c) {
    return reinterpret_cast<unsigned long long*>(p.att_part + (static_cast<size_t>(h) * ATT_MAX_CHUNKS + c) *
                                                                  ATT_PART_STRIDE);
}

// ------------------------------------------------------------------------ phases
template <typename KT>
__device__ bool phase_qkv(const DecodeParams& p, const Smem& s, int l, int token, int cta, int ncta, unsigned seq) {
    const LayerMeta& L = s.meta()[l];
    const int a = L.qkv0, b = L.qkv1;   // same split as phase_layout
    // this thread's RoPE factors (pair pr = threadIdx.x), fetched before the norm
    const int pr0 = threadIdx.x, R0 = a + 2 * pr0;
    float2 cs0 = make_float2(0.0f, 0.0f);
    if (pr0 < (b - a) / 2 && R0 < N_EMBD + KV_DIM)
        cs0 = __ldg(p.rope + static_cast<size_t>(p.pos) * (HEAD_DIM / 2) + ((R0 & (HEAD_DIM - 1)) >> 1));
    if (threadIdx.x == ISSUE_THREAD && l + 1 < p.n_layer) prefetch_layer_l2(p, s, l + 1, 0);
    if (l == 0) {
        embed_row(p.embd, token, s.xs());
        __syncthreads();
        if (cta == 0)
            for (int i = threadIdx.x; i < N_EMBD; i += blockDim.x) p.x[i] = s.xs()[i];
        norm_quant<true, X_SMEM>(p, s.xs(), 0, meta_f32(p, L.attn_norm), s);
    } else {
        if (!norm_quant<true, X_EPOCH>(p, nullptr, x_epoch(seq, 2 * l), meta_f32(p, L.attn_norm), s,
                                       l == 2 ? TRACE_POLL + 148 : -1))
            return false;
        trace_mark(p, 3 + 2 * (5 * (l - 1) + 4));
        trace_cta(p, l - 1, 4, 1);
    }
    trace_step(p, l, 0, 1);
    if (!wait_weights(p, s, 4 * l)) return false;
    if (threadIdx.x == COPY_THREAD) issue_copy(p, s, 4 * l + 1, cta, ncta);   // o_proj rows: buffer 1
    trace_step(p, l, 0, 2);
    const PhaseLayout pl = phase_layout(L, *s.rows(), 0);
    const int lo[3] = {0, N_EMBD, N_EMBD + KV_DIM};
    float* rv = s.rowval();
    // A CTA's rows span at most two of Q, K, V; two spans of one type (Q and K, or K and V rows
    // of the same quantisation) run as one GEMV call: their outputs are adjacent in rv.
    bool done_next = false;   // segment i was taken by the call of segment i-1
#pragma unroll
    for (int i = 0; i < 3; ++i) {   // unrolled: PhaseLayout stays in registers
        if (done_next) {
            done_next = false;
            continue;
        }
        if (pl.nrows[i] == 0) continue;   // uniform across the CTA
        const int base = lo[i] + pl.row0[i] - a;
        const int ti = phase_type(L, 0, i);
        if (i < 2 && pl.nrows[i + 1] > 0 && phase_type(L, 0, i + 1) == ti) {
            dec_gemv(p, s, ti, s.wbuf(0) + pl.off[i], pl.nrows[i], s.wbuf(0) + pl.off[i + 1],
                     pl.nrows[i] + pl.nrows[i + 1], N_EMBD / 256, rv + base, nullptr);
            done_next = true;
            continue;
        }
        dec_gemv(p, s, ti, s.wbuf(0) + pl.off[i], pl.nrows[i], s.wbuf(0) + pl.off[i], pl.nrows[i], N_EMBD / 256,
                 rv + base, (p.trace && l == 1 && cta == 0 && i == 0) ? p.trace + TRACE_GEMV + 9 : nullptr);
    }
    trace_step(p, l, 0, 3);
    __syncthreads();   // buffer 0 read by every GEMV above
    if (threadIdx.x == COPY_THREAD && s.flags()[0]) issue_copy(p, s, 4 * l + 2, cta, ncta);   // gate/up: buffer 0
    // RoPE on Q/K pairs (interleaved, ops.cpp:502-516 with the build's FMA contraction),
    // then Q to the query buffer and K/V into the cache at pos (ops.cpp:557-563).
    // K and V as the cache stores them (fp16 rows: rounded once here, and the attention units
    // read this launch's rows from the epoch-tagged copies in the same rounded form)
    KT* kdst = reinterpret_cast<KT*>(p.kc) + (static_cast<size_t>(l) * p.max_seq + p.pos) * KV_DIM;
    KT* vdst = reinterpret_cast<KT*>(p.vc) + (static_cast<size_t>(l) * p.max_seq + p.pos) * KV_DIM;
    for (int pr = threadIdx.x; pr < (b - a) / 2; pr += blockDim.x) {
        const int R = a + 2 * pr;
        const float v0 = rv[2 * pr], v1 = rv[2 * pr + 1];
        if (R < N_EMBD + KV_DIM) {
            const float2 c = pr == pr0 ? cs0 : __ldg(p.rope + static_cast<size_t>(p.pos) * (HEAD_DIM / 2) +
                                                     ((R & (HEAD_DIM - 1)) >> 1));
            float r0 = __fmaf_rn(c.x, v0, -__fmul_rn(c.y, v1));
            float r1 = __fmaf_rn(c.y, v0, __fmul_rn(c.x, v1));
            if (R < N_EMBD) {
                p.q[R] = r0;
                p.q[R + 1] = r1;
            } else {
                r0 = kv_round<KT>(r0);
                r1 = kv_round<KT>(r1);
                kdst[R - N_EMBD] = KvElt<KT>::put(r0);
                kdst[R - N_EMBD + 1] = KvElt<KT>::put(r1);
            }
            st_epoch(p.qll + R, r0, qkv_epoch(seq, l));
            st_epoch(p.qll + R + 1, r1, qkv_epoch(seq, l));
        } else {
            const float w0 = kv_round<KT>(v0), w1 = kv_round<KT>(v1);
            vdst[R - N_EMBD - KV_DIM] = KvElt<KT>::put(w0);
            vdst[R - N_EMBD - KV_DIM + 1] = KvElt<KT>::put(w1);
            st_epoch(p.qll + R, w0, qkv_epoch(seq, l));
            st_epoch(p.qll + R + 1, w1, qkv_epoch(seq, l));
        }
    }
    return true;
}

// Chunk counts up to DIST_COMBINE_MAX are combined by every CTA in the o_proj prologue
// (no atomics, no serial combiner); longer contexts use the head-pair combiners.
constexpr int DIST_COMBINE_MAX = 16;

__device__ __forceinline__ int attn_chunks(int n) {
    const int P = 32 * ((n + 2047) / 2048);
    return (n + P - 1) / P;
}

// Decode kernel with more than DIST_COMBINE_MAX chunks (or any number, with the
// SCHED_ATT_COMBINERS option): head-pair combiners, no grid barrier after attention.
__device__ __forceinline__ bool att_flagged(const DecodeParams& p) {
    return p.attw != nullptr && ((p.sched & SCHED_ATT_COMBINERS) || attn_chunks(p.pos + 1) > DIST_COMBINE_MAX);
}

// Unit tail: the (m, l) headers of the chunk's 8 heads (stat[0..7] maxima, stat[8..15]
// sums), after every o value of the chunk.  Called by all threads after their o stores.
// Without a grid barrier to follow (combiners poll), the headers wait for a CTA barrier and
// a fence; with one they are stored right away.
__device__ __forceinline__ void publish_headers(const DecodeParams& p, const float* stat, int g, int c, int l,
                                                unsigned seq, bool flagged) {
    const int tid = threadIdx.x;
    if (flagged) __syncthreads();
    if (tid < 8) {
        unsigned long long* hdr = att_header(p, 8 * g + tid, c);
        const unsigned long long e = static_cast<unsigned long long>(att_epoch(seq, l)) << 32;
        if (flagged) {
            __threadfence();
            st_epoch(hdr, stat[tid], static_cast<unsigned>(e >> 32));
            st_epoch(hdr + 1, stat[8 + tid], static_cast<unsigned>(e >> 32));
        } else {   // a grid barrier orders them: plain stores
            __stcg(reinterpret_cast<ulonglong2*>(hdr),
                   make_ulonglong2(e | __float_as_uint(stat[tid]), e | __float_as_uint(stat[8 + tid])));
        }
    }
    if (!flagged) __syncthreads();
}

// One attention unit of at most 32 positions (chunk length P = 32, contexts up to 2048):
// the 8 query heads of KV head g against positions [t0, t0+np).  q and K go straight from
// L2 into registers (one round trip), V streams into shared memory meanwhile (cp.async).
// Thread (warp w, group G = lane/8, j = lane%8): heads 2G, 2G+1 x positions t0+2w, t0+2w+1,
// dims 4j + 32i + c of each dot, then the butterfly v += v^4, v += v^2, v += v^1 (the
// canonical 8-lane q.k split).
// Same numerics as the general path below: scores, chunk max, exp, position-ordered
// sum and fma chains, partials [head][chunk][m, l, o[128]].
// In the decode kernel (p.qll set) q and this position's K/V rows are read from their
// epoch-tagged copies, so no grid barrier separates the QKV phase from attention.
template <typename KT>
__device__ void attention_unit32(const DecodeParams& p, float* scratch, int l, int g, int c, int t0, int np,
                                 unsigned seq, bool flagged) {
    using E = KvElt<KT>;
    constexpr int CPR = HEAD_DIM / E::PER16;   // 16-byte copies per cache row
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, j = lane & 7, G = lane >> 3;
    KT* vb = reinterpret_cast<KT*>(scratch);            // [32][128] V rows of the chunk (a float-sized slot)
    float* sc = scratch + 32 * HEAD_DIM;                // [8][32] scores -> probabilities
    float* stat = sc + 8 * 32;                          // m[8], l[8]
    float* qsm = stat + 32;                             // [8][128] q of the group (epoch path)
    float* krow = qsm + 8 * HEAD_DIM;                   // [128] K row at pos (epoch path)
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HEAD_DIM)));
    const KT* kl = reinterpret_cast<const KT*>(p.kc) + static_cast<size_t>(l) * p.max_seq * KV_DIM + g * HEAD_DIM;
    const KT* vl = reinterpret_cast<const KT*>(p.vc) + static_cast<size_t>(l) * p.max_seq * KV_DIM + g * HEAD_DIM;
    const bool epoch_in = p.qll != nullptr;
    const int cur = epoch_in && t0 + np - 1 == p.pos ? np - 1 : -1;   // chunk row published this launch
    const int ncache = cur >= 0 ? np - 1 : np;                         // rows read from the cache
    for (int i = tid; i < ncache * CPR; i += blockDim.x)
        cp_async16(vb + E::PER16 * i, vl + static_cast<size_t>(t0 + i / CPR) * KV_DIM + E::PER16 * (i % CPR));
    cp_async_commit();
    const int tA = 2 * warp, tB = tA + 1;
    const bool va = tA < np, vbv = tB < np;
    const KT* kA = kl + static_cast<size_t>(t0 + (va && tA != cur ? tA : 0)) * KV_DIM + 4 * j;
    const KT* kB = kl + static_cast<size_t>(t0 + (vbv && tB != cur ? tB : 0)) * KV_DIM + 4 * j;
    float4 qa[4], qb[4], ka[4], kb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {   // cached K rows first: their loads overlap the waits below
        ka[i] = E::ld4(kA + 32 * i);
        kb[i] = E::ld4(kB + 32 * i);
    }
    if (epoch_in) {
        const unsigned ep = qkv_epoch(seq, l);
        bool ok = true;
        if (tid < 256) {
            float4 v;
            ok = load4_epoch(p.qll + 8 * g * HEAD_DIM + 4 * tid, ep, v, p.err);
            reinterpret_cast<float4*>(qsm)[tid] = v;
        } else if (cur >= 0 && tid < 256 + 32) {
            float4 v;
            ok = load4_epoch(p.qll + N_EMBD + g * HEAD_DIM + 4 * (tid - 256), ep, v, p.err);
            reinterpret_cast<float4*>(krow)[tid - 256] = v;
        } else if (cur >= 0 && tid < 256 + 64) {
            float4 v;
            ok = load4_epoch(p.qll + N_EMBD + KV_DIM + g * HEAD_DIM + 4 * (tid - 288), ep, v, p.err);
            E::st4(vb + cur * HEAD_DIM + 4 * (tid - 288), v);
        }
        if (__syncthreads_or(!ok)) {
            cp_async_wait_all();
            return;   // ERR_TIMEOUT is set; the next grid barrier stops every CTA
        }
        trace_mark(p, 3 + 2 * (5 * l));   // inputs of this unit published
        const float* q0 = qsm + (2 * G) * HEAD_DIM + 4 * j;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qa[i] = *reinterpret_cast<const float4*>(q0 + 32 * i);
            qb[i] = *reinterpret_cast<const float4*>(q0 + HEAD_DIM + 32 * i);
            if (tA == cur) ka[i] = *reinterpret_cast<const float4*>(krow + 4 * j + 32 * i);
            if (tB == cur) kb[i] = *reinterpret_cast<const float4*>(krow + 4 * j + 32 * i);
        }
    } else {
        const float* q0 = p.q + (8 * g + 2 * G) * HEAD_DIM + 4 * j;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qa[i] = ld_cg_f4(q0 + 32 * i);
            qb[i] = ld_cg_f4(q0 + HEAD_DIM + 32 * i);
        }
    }
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // (h0,tA) (h0,tB) (h1,tA) (h1,tB)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        d[0] = __fmaf_rn(qa[i].x, ka[i].x, d[0]);
        d[0] = __fmaf_rn(qa[i].y, ka[i].y, d[0]);
        d[0] = __fmaf_rn(qa[i].z, ka[i].z, d[0]);
        d[0] = __fmaf_rn(qa[i].w, ka[i].w, d[0]);
        d[1] = __fmaf_rn(qa[i].x, kb[i].x, d[1]);
        d[1] = __fmaf_rn(qa[i].y, kb[i].y, d[1]);
        d[1] = __fmaf_rn(qa[i].z, kb[i].z, d[1]);
        d[1] = __fmaf_rn(qa[i].w, kb[i].w, d[1]);
        d[2] = __fmaf_rn(qb[i].x, ka[i].x, d[2]);
        d[2] = __fmaf_rn(qb[i].y, ka[i].y, d[2]);
        d[2] = __fmaf_rn(qb[i].z, ka[i].z, d[2]);
        d[2] = __fmaf_rn(qb[i].w, ka[i].w, d[2]);
        d[3] = __fmaf_rn(qb[i].x, kb[i].x, d[3]);
        d[3] = __fmaf_rn(qb[i].y, kb[i].y, d[3]);
        d[3] = __fmaf_rn(qb[i].z, kb[i].z, d[3]);
        d[3] = __fmaf_rn(qb[i].w, kb[i].w, d[3]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        d[e] = __fadd_rn(d[e], __shfl_xor_sync(0xffffffffu, d[e], 4));
        d[e] = __fadd_rn(d[e], __shfl_xor_sync(0xffffffffu, d[e], 2));
        d[e] = __fadd_rn(d[e], __shfl_xor_sync(0xffffffffu, d[e], 1));
    }
    trace_step(p, l, 1, 3);   // thread 0's K rows have arrived
    if (j == 0) {
        if (va) sc[(2 * G) * 32 + tA] = __fmul_rn(d[0], scale), sc[(2 * G + 1) * 32 + tA] = __fmul_rn(d[2], scale);
        if (vbv) sc[(2 * G) * 32 + tB] = __fmul_rn(d[1], scale), sc[(2 * G + 1) * 32 + tB] = __fmul_rn(d[3], scale);
    }
    __syncthreads();
    trace_step(p, l, 1, 1);
    if (warp < 8) {   // chunk max, probabilities, position-ordered sum (warp = head)
        float v = lane < np ? sc[warp * 32 + lane] : -__int_as_float(0x7f800000);
        float m = v;
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float pr = lane < np ? canon_expf(__fsub_rn(v, m)) : 0.0f;
        if (lane < np) sc[warp * 32 + lane] = pr;
        float sum = pr;   // canonical chunk sum: lane sums (one position each here), then a butterfly
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        if (lane == 0) stat[warp] = m, stat[8 + warp] = sum;
    }
    if (warp == 0) trace_step(p, l, 1, 5);
    cp_async_wait_all();
    __syncthreads();
    trace_step(p, l, 1, 6);
    float acc0 = 0.0f, acc1 = 0.0f;   // o[h][dd] = fma chain over positions
    const int h0 = tid >> 7, h1 = h0 + 4, dd = tid & 127;
    for (int t = 0; t < np; t += 4) {   // four positions per step: loads first, chain in order
        const float4 s0 = *reinterpret_cast<const float4*>(sc + h0 * 32 + t);
        const float4 s1 = *reinterpret_cast<const float4*>(sc + h1 * 32 + t);
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = t + k < np ? E::get(vb[(t + k) * HEAD_DIM + dd]) : 0.0f;
        const float a0[4] = {s0.x, s0.y, s0.z, s0.w}, a1[4] = {s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (t + k < np) {
                acc0 = __fmaf_rn(a0[k], v[k], acc0);
                acc1 = __fmaf_rn(a1[k], v[k], acc1);
            }
        }
    }
    trace_step(p, l, 1, 7);
    float* pa0 = p.att_part + (static_cast<size_t>(8 * g + h0) * ATT_MAX_CHUNKS + c) * ATT_PART_STRIDE;
    float* pa1 = p.att_part + (static_cast<size_t>(8 * g + h1) * ATT_MAX_CHUNKS + c) * ATT_PART_STRIDE;
    __stcg(pa0 + ATT_PART_O + dd, acc0);
    __stcg(pa1 + ATT_PART_O + dd, acc1);
    publish_headers(p, stat, g, c, l, seq, flagged);
    trace_step(p, l, 1, 2);
}

// One attention unit of a chunk longer than 32 positions (contexts above 2048): the 8 query
// heads of KV head g against positions [t0, t0+np), np <= 256.  Cached K rows stream into
// shared memory with cp.async, up to ATT_BIG_ROWS rows per round trip, while q and this
// launch's K/V rows are polled from their epoch-tagged copies (no grid barrier after the QKV
// phase); then the V rows through the same buffer.
// Warp w: head pair w&3 (q in registers), positions (w>>2)*4 + group + 16i; lane j of an
// 8-lane group owns dims 4j + 32i + c of each dot (the canonical 8-lane split).  Same
// numerics as attention_unit32.
constexpr int ATT_BIG_ROWS = 160;   // one round trip per chunk up to 10240 positions (chunk 160)
// q, K/V rows, scores, stat, this launch's K and V rows
static_assert((8 * HEAD_DIM + ATT_BIG_ROWS * HEAD_DIM + 8 * ATT_SC_STRIDE + 16 + 2 * HEAD_DIM) * sizeof(float) <=
                  WBUF_BYTES,
              "attention scratch exceeds weight buffer 0");
// combine_pair: chunk o vectors of two heads, maxima, sums, weights, 1/L, output
static_assert((2 * ATT_MAX_CHUNKS * HEAD_DIM + 6 * ATT_MAX_CHUNKS + 4 + 256) * sizeof(float) <= WBUF_BYTES,
              "combine scratch exceeds weight buffer 0");
template <typename KT>
__device__ void attention_unit_big(const DecodeParams& p, float* scratch, int l, int g, int c, int t0, int np,
                                   unsigned seq, bool flagged) {
    using E = KvElt<KT>;
    constexpr int CPR = HEAD_DIM / E::PER16;   // 16-byte copies per cache row
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, j = lane & 7, G = lane >> 3;
    float* qh = scratch;                                // [8][128]
    KT* kv = reinterpret_cast<KT*>(qh + 8 * HEAD_DIM);  // [ATT_BIG_ROWS][128] K, then V rows (float-sized slot)
    float* sc = qh + 8 * HEAD_DIM + ATT_BIG_ROWS * HEAD_DIM;   // [8][ATT_SC_STRIDE] scores -> probabilities
    float* stat = sc + 8 * ATT_SC_STRIDE;               // m[8], l[8]
    float* krow = stat + 16;                            // [128] K row at pos (epoch path)
    float* vrow = krow + HEAD_DIM;                      // [128] V row at pos (epoch path)
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HEAD_DIM)));
    const KT* kl = reinterpret_cast<const KT*>(p.kc) + static_cast<size_t>(l) * p.max_seq * KV_DIM + g * HEAD_DIM;
    const KT* vl = reinterpret_cast<const KT*>(p.vc) + static_cast<size_t>(l) * p.max_seq * KV_DIM + g * HEAD_DIM;
    const bool epoch_in = p.qll != nullptr;
    const int cur = epoch_in && t0 + np - 1 == p.pos ? np - 1 : -1;   // chunk row published this launch
    // Stages the cache rows of [s0, s0+ns) into kv and returns their count; the row
    // published this launch (the chunk's last) is copied in from krow / vrow instead.
    auto stage = [&](const KT* src, int s0, int ns) {
        const int nc = cur >= s0 && cur < s0 + ns ? ns - 1 : ns;   // cur is the chunk's last row
        for (int i = tid; i < nc * CPR; i += blockDim.x)
            cp_async16(kv + E::PER16 * i, src + static_cast<size_t>(t0 + s0 + i / CPR) * KV_DIM + E::PER16 * (i % CPR));
        cp_async_commit();
        return nc;
    };
    const int hp = warp & 3, ps = warp >> 2;
    for (int s0 = 0; s0 < np; s0 += ATT_BIG_ROWS) {   // scores
        const int ns = min(ATT_BIG_ROWS, np - s0);
        const int nc = stage(kl, s0, ns);
        if (s0 == 0) {   // q of the group (and this launch's K/V rows) while the cache rows load
            bool ok = true;
            if (epoch_in) {
                const unsigned ep = qkv_epoch(seq, l);
                float4 v;
                if (tid < 256) {
                    ok = load4_epoch(p.qll + 8 * g * HEAD_DIM + 4 * tid, ep, v, p.err);
                    reinterpret_cast<float4*>(qh)[tid] = v;
                } else if (cur >= 0 && tid < 256 + 32) {
                    ok = load4_epoch(p.qll + N_EMBD + g * HEAD_DIM + 4 * (tid - 256), ep, v, p.err);
                    reinterpret_cast<float4*>(krow)[tid - 256] = v;
                } else if (cur >= 0 && tid < 256 + 64) {
                    ok = load4_epoch(p.qll + N_EMBD + KV_DIM + g * HEAD_DIM + 4 * (tid - 288), ep, v, p.err);
                    reinterpret_cast<float4*>(vrow)[tid - 288] = v;
                }
            } else if (tid < 256) {
                reinterpret_cast<float4*>(qh)[tid] = ld_cg_f4(p.q + 8 * g * HEAD_DIM + 4 * tid);
            }
            if (__syncthreads_or(!ok)) {
                cp_async_wait_all();
                return;   // ERR_TIMEOUT is set; every waiter downstream times out too
            }
            trace_mark(p, 3 + 2 * (5 * l));   // inputs of this unit published
        }
        if (nc < ns && tid < 32) E::st4(kv + nc * HEAD_DIM + 4 * tid, reinterpret_cast<float4*>(krow)[tid]);
        cp_async_wait_all();
        __syncthreads();
        if (s0 == 0) trace_step(p, l, 1, 4);
        float4 qa[4], qb[4];   // reloaded per round: registers stay free between rounds
        const float* q0 = qh + (2 * hp) * HEAD_DIM + 4 * j;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qa[i] = *reinterpret_cast<const float4*>(q0 + 32 * i);
            qb[i] = *reinterpret_cast<const float4*>(q0 + HEAD_DIM + 32 * i);
        }
        // positions ta = base + G, tb = ta + 16 for heads a = 2hp, b = 2hp+1: four dots per
        // lane group; the 8-lane butterfly runs reduce-scatter (a lane sends the value its
        // partner keeps), the same additions as v += shfl_xor(v, 4 / 2 / 1) on each dot.
        for (int base = ps * 4; base < ns; base += 32) {   // warp-uniform trip count
            const int ta = base + G, tb = ta + 16;
            const KT* ka = kv + min(ta, ns - 1) * HEAD_DIM + 4 * j;
            const KT* kb = kv + min(tb, ns - 1) * HEAD_DIM + 4 * j;
            float aa = 0.0f, ba = 0.0f, ab = 0.0f, bb = 0.0f;   // (head a|b, position ta|tb)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 x = E::sm4(ka + 32 * i);
                const float4 y = E::sm4(kb + 32 * i);
                aa = __fmaf_rn(qa[i].x, x.x, aa);
                aa = __fmaf_rn(qa[i].y, x.y, aa);
                aa = __fmaf_rn(qa[i].z, x.z, aa);
                aa = __fmaf_rn(qa[i].w, x.w, aa);
                ba = __fmaf_rn(qb[i].x, x.x, ba);
                ba = __fmaf_rn(qb[i].y, x.y, ba);
                ba = __fmaf_rn(qb[i].z, x.z, ba);
                ba = __fmaf_rn(qb[i].w, x.w, ba);
                ab = __fmaf_rn(qa[i].x, y.x, ab);
                ab = __fmaf_rn(qa[i].y, y.y, ab);
                ab = __fmaf_rn(qa[i].z, y.z, ab);
                ab = __fmaf_rn(qa[i].w, y.w, ab);
                bb = __fmaf_rn(qb[i].x, y.x, bb);
                bb = __fmaf_rn(qb[i].y, y.y, bb);
                bb = __fmaf_rn(qb[i].z, y.z, bb);
                bb = __fmaf_rn(qb[i].w, y.w, bb);
            }
            const bool lo4 = j < 4;   // keeps head a
            const float r1 = __shfl_xor_sync(0xffffffffu, lo4 ? ba : aa, 4);
            const float r2 = __shfl_xor_sync(0xffffffffu, lo4 ? bb : ab, 4);
            const float X = __fadd_rn(lo4 ? aa : ba, r1);   // position ta
            const float Y = __fadd_rn(lo4 ? ab : bb, r2);   // position tb
            const bool lo2 = (j & 2) == 0;                  // keeps ta
            const float r3 = __shfl_xor_sync(0xffffffffu, lo2 ? Y : X, 2);
            float Z = __fadd_rn(lo2 ? X : Y, r3);
            Z = __fadd_rn(Z, __shfl_xor_sync(0xffffffffu, Z, 1));
            const int t = lo2 ? ta : tb;
            if ((j & 1) == 0 && t < ns) sc[(2 * hp + (lo4 ? 0 : 1)) * ATT_SC_STRIDE + s0 + t] = __fmul_rn(Z, scale);
        }
        __syncthreads();   // kv is overwritten next
    }
    trace_step(p, l, 1, 1);
    if (warp < 8) {   // chunk max, probabilities, canonical chunk sum (warp = head); np <= 256
        float* sh = sc + warp * ATT_SC_STRIDE;
        float x[ATT_SC_STRIDE / 32];
        float m = -__int_as_float(0x7f800000);
#pragma unroll
        for (int k = 0; k < ATT_SC_STRIDE / 32; ++k) {
            x[k] = lane + 32 * k < np ? sh[lane + 32 * k] : 0.0f;
            if (lane + 32 * k < np) m = fmaxf(m, x[k]);
        }
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float sum = 0.0f;   // lane sum over t = lane (mod 32) in position order
#pragma unroll
        for (int k = 0; k < ATT_SC_STRIDE / 32; ++k) {
            if (lane + 32 * k < np) {
                const float e = canon_expf(__fsub_rn(x[k], m));
                sh[lane + 32 * k] = e;
                sum = __fadd_rn(sum, e);
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        if (lane == 0) stat[warp] = m, stat[8 + warp] = sum;
    }
    // o[h][d] = fma chain over positions: threads 0-127 own heads 4hq..4hq+3 x dims 2dp, 2dp+1
    // (float2 V rows, float4 probabilities): the fewest shared-memory wavefronts per position.
    const int hq = (tid >> 6) & 1, dp = tid & 63;
    float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
    trace_step(p, l, 1, 8);
    for (int s0 = 0; s0 < np; s0 += ATT_BIG_ROWS) {
        const int ns = min(ATT_BIG_ROWS, np - s0);
        const int nc = stage(vl, s0, ns);
        if (nc < ns && tid < 32) E::st4(kv + nc * HEAD_DIM + 4 * tid, reinterpret_cast<float4*>(vrow)[tid]);
        cp_async_wait_all();
        __syncthreads();   // V rows, and (first round) the probabilities
        if (s0 == 0) trace_step(p, l, 1, 9);
        if (tid < 128) {
            const float* pr = sc + 4 * hq * ATT_SC_STRIDE + s0;
            const KT* vr = kv + 2 * dp;
            int tt = 0;
#pragma unroll 2
            for (; tt + 4 <= ns; tt += 4) {
                float4 pw[4];
                float2 v[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) pw[h] = *reinterpret_cast<const float4*>(pr + h * ATT_SC_STRIDE + tt);
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = E::sm2(vr + (tt + k) * HEAD_DIM);
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const float w[4] = {pw[h].x, pw[h].y, pw[h].z, pw[h].w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc[h][0] = __fmaf_rn(w[k], v[k].x, acc[h][0]);
                        acc[h][1] = __fmaf_rn(w[k], v[k].y, acc[h][1]);
                    }
                }
            }
            for (; tt < ns; ++tt) {
                const float2 v = E::sm2(vr + tt * HEAD_DIM);
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const float w = pr[h * ATT_SC_STRIDE + tt];
                    acc[h][0] = __fmaf_rn(w, v.x, acc[h][0]);
                    acc[h][1] = __fmaf_rn(w, v.y, acc[h][1]);
                }
            }
        }
        __syncthreads();
    }
    trace_step(p, l, 1, 3);
    if (tid < 128) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float* pa = p.att_part + (static_cast<size_t>(8 * g + 4 * hq + h) * ATT_MAX_CHUNKS + c) * ATT_PART_STRIDE +
                        ATT_PART_O + 2 * dp;
            __stcg(reinterpret_cast<float2*>(pa), make_float2(acc[h][0], acc[h][1]));
        }
    }
    publish_headers(p, stat, g, c, l, seq, flagged);
    trace_step(p, l, 1, 2);
}

// Combiner of head pair b (heads 2b, 2b+1: one Q8_K block of the attention output) for
// contexts of more than DIST_COMBINE_MAX chunks.  Waits for the chunk headers of its two
// heads, stages their o vectors in shared memory (one round trip), then
//   M = max_c m_c, w_c = exp(m_c - M), L = fma chain of w_c*l_c over c, o = fma chain of
//   w_c*o_c over c, out = o * (1/L)
// (ops.cpp:590-611 restated per chunk), and writes p.att, the Q8_K block b of p.att_q8k
// and, in the decode kernel (p.attw set), the epoch-tagged values o_proj waits for.
__device__ bool combine_pair(const DecodeParams& p, float* scratch, int l, int b, unsigned seq) {
    const int n = p.pos + 1, C = attn_chunks(n);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned e = att_epoch(seq, l);
    float* po = scratch;                                // [2][ATT_MAX_CHUNKS][128] chunk o vectors
    float* msm = po + 2 * ATT_MAX_CHUNKS * HEAD_DIM;    // [2][ATT_MAX_CHUNKS] chunk maxima
    float* lsm = msm + 2 * ATT_MAX_CHUNKS;              // [2][ATT_MAX_CHUNKS] chunk sums
    float* wts = lsm + 2 * ATT_MAX_CHUNKS;              // [2][ATT_MAX_CHUNKS] exp(m_c - M)
    float* inv = wts + 2 * ATT_MAX_CHUNKS;              // [2] (+2 pad)
    float* ab = inv + 4;                                // [256]
    if (p.trace && l == 1 && tid == 0) p.trace[2880 + 4 * b + 0] = globaltimer();
    // one thread per (head, chunk) header, then the o vectors in one round trip
    bool ok = true;
    if (tid < 2 * C) {
        const int hh = tid & 1, c = tid >> 1;
        float m = 0.0f, lv = 0.0f;
        ok = load2_epoch(att_header(p, 2 * b + hh, c), e, m, lv, p.err);
        msm[hh * ATT_MAX_CHUNKS + c] = m;
        lsm[hh * ATT_MAX_CHUNKS + c] = lv;
        fence_acq_rel_gpu();   // the header is seen before its o vector is read
    }
    if (!__syncthreads_and(ok)) return false;
    for (int i = tid; i < 2 * C * 32; i += blockDim.x) {
        const int hh = i / (32 * C), r = i - hh * 32 * C, c = r >> 5, f = r & 31;
        cp_async16(po + (hh * ATT_MAX_CHUNKS + c) * HEAD_DIM + 4 * f,
                   p.att_part + (static_cast<size_t>(2 * b + hh) * ATT_MAX_CHUNKS + c) * ATT_PART_STRIDE + ATT_PART_O +
                       4 * f);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    if (p.trace && l == 1 && tid == 0) p.trace[2880 + 4 * b + 1] = globaltimer();
    const bool tr0 = p.trace && l == 1 && b == 0 && tid == 0;
    if (tr0) p.trace[2940] = clock64(), p.trace[2941] = globaltimer();
    if (warp < 2) {   // warp = head of the pair: M, w_c, and the chunk-ordered L chain
        const float* mh = msm + warp * ATT_MAX_CHUNKS;
        float m0 = lane < C ? mh[lane] : -__int_as_float(0x7f800000);
        const float m1 = lane + 32 < C ? mh[lane + 32] : -__int_as_float(0x7f800000);
        float M = fmaxf(m0, m1);
        for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (tr0) p.trace[2942] = clock64();
        if (lane < C) wts[warp * ATT_MAX_CHUNKS + lane] = canon_expf(__fsub_rn(m0, M));
        if (lane + 32 < C) wts[warp * ATT_MAX_CHUNKS + lane + 32] = canon_expf(__fsub_rn(m1, M));
        __syncwarp();
        if (tr0) p.trace[2943] = clock64();
        if (lane == 0) {   // chunk-ordered chain; loads hoisted (fixed trip count, predicated)
            const float* wh = wts + warp * ATT_MAX_CHUNKS;
            const float* lh = lsm + warp * ATT_MAX_CHUNKS;
            float Ls = 0.0f;
#pragma unroll 16
            for (int c = 0; c < ATT_MAX_CHUNKS; ++c)
                if (c < C) Ls = __fmaf_rn(wh[c], lh[c], Ls);
            inv[warp] = __fdiv_rn(1.0f, Ls);
        }
        if (tr0) p.trace[2944] = clock64();
    }
    __syncthreads();
    if (tr0) p.trace[2945] = clock64(), p.trace[2946] = globaltimer();
    if (p.trace && l == 1 && tid == 0) p.trace[2880 + 4 * b + 2] = globaltimer();
    if (tid < 2 * HEAD_DIM) {
        const int hh = tid >> 7, dd = tid & 127;
        const float* w = wts + hh * ATT_MAX_CHUNKS;
        const float* o = po + hh * ATT_MAX_CHUNKS * HEAD_DIM + dd;
        float O = 0.0f;   // chunk-ordered chain; loads hoisted (fixed trip count, predicated)
#pragma unroll 16
        for (int c = 0; c < ATT_MAX_CHUNKS; ++c)
            if (c < C) O = __fmaf_rn(w[c], o[c * HEAD_DIM], O);
        const float out = __fmul_rn(O, inv[hh]);
        ab[tid] = out;
        if (p.attw) {   // one copy per group of polling CTAs (fewer pollers per L2 line)
#pragma unroll
            for (int r = 0; r < ATTW_COPIES; ++r) st_epoch(p.attw + r * N_EMBD + 256 * b + tid, out, e);
        }
        p.att[256 * b + tid] = out;
    }
    if (p.trace && l == 1 && tid == 0) p.trace[2912 + b] = globaltimer();   // published (thread 0's value)
    __syncthreads();
    if (warp == 0) {   // Q8_K block b, ties-to-even (quantize_row_q8_K_avx2)
        float y[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = ab[8 * lane + k];
        if (p.att_qs) {
            quant_block_warp<false, true>(y, p.att_qs + 256 * b, p.att_d + b, p.att_bs + 16 * b);   // lane-major
        } else {
            uint8_t* blk = p.att_q8k + static_cast<size_t>(b) * Q8K_BYTES;
            quant_block_warp<false>(y, reinterpret_cast<int8_t*>(blk + 4), reinterpret_cast<float*>(blk),
                                    reinterpret_cast<int16_t*>(blk + 260));
        }
    }
    if (p.trace && l == 1 && tid == 0) p.trace[2880 + 4 * b + 3] = globaltimer();
    __syncthreads();   // po / ab reused by the caller
    return true;
}

// Attention of layer l: units (KV group g, chunk c) over the CTAs, then, for more than
// DIST_COMBINE_MAX chunks in the decode kernel, the head-pair combiners on the last CTAs
// (usually CTAs without a unit).  Shorter contexts are combined in the o_proj prologue;
// the standalone op combines in k_att_combine.
template <typename KT>
__device__ bool phase_attention(const DecodeParams& p, const Smem& s, float* scratch, int l, int cta, int ncta,
                                unsigned seq) {
    const int n = p.pos + 1;
    const int P = 32 * ((n + 2047) / 2048);
    const int C = (n + P - 1) / P;
    const bool flagged = att_flagged(p);
    for (int item = cta; item < 2 * C; item += ncta) {
        const int g = item / C, c = item % C;
        const int t0 = c * P, t1 = min(t0 + P, n), np = t1 - t0;
        __syncthreads();
        if (P == 32)
            attention_unit32<KT>(p, scratch, l, g, c, t0, np, seq, flagged);
        else
            attention_unit_big<KT>(p, scratch, l, g, c, t0, np, seq, flagged);
    }
    if (flagged) {
        for (int b = ncta - 1 - cta; b < N_EMBD / 256; b += ncta) {
            __syncthreads();
            if (!combine_pair(p, scratch, l, b, seq)) return false;
        }
    }
    return true;
}

// Up to DIST_COMBINE_MAX chunks: every CTA combines the attention chunks of all 16 heads
// (same operations and order as combine_pair) and quantises the result ties-to-even
// straight into s.xq().
__device__ void combine_attention(const DecodeParams& p, const Smem& s, int l, int cta) {
    // warp = head h, lane = dims 4*lane .. 4*lane+3: the chunk weights of a head never leave
    // its warp, so loads, max, exp, the L chain and the O chains run without a CTA barrier.
    const int n = p.pos + 1, C = attn_chunks(n);
    const int tid = threadIdx.x, lane = tid & 31, h = tid >> 5;
    float* ab = s.xs();   // [2048]
    const float* ph = p.att_part + static_cast<size_t>(h) * ATT_MAX_CHUNKS * ATT_PART_STRIDE;
    // lane c < C: chunk c's header (m, l), final after the grid barrier: plain loads issued
    // with the o vectors (one round trip)
    const float2 ml = lane < C ? make_float2(ph[lane * ATT_PART_STRIDE], ph[lane * ATT_PART_STRIDE + 2])
                               : make_float2(0.f, 0.f);   // low halves of the two header words
    float4 v[DIST_COMBINE_MAX];
#pragma unroll
    for (int cc = 0; cc < DIST_COMBINE_MAX; ++cc)
        v[cc] = cc < C ? ld_cg_f4(ph + cc * ATT_PART_STRIDE + ATT_PART_O + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    float M = lane < C ? ml.x : -__int_as_float(0x7f800000);
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (h == 0) trace_step(p, l, 2, 3);   // chunk headers loaded
    const float wv = lane < C ? canon_expf(__fsub_rn(ml.x, M)) : 0.0f;
    float Ls = 0.0f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int cc = 0; cc < DIST_COMBINE_MAX; ++cc) {
        if (cc < C) {
            const float w = __shfl_sync(0xffffffffu, wv, cc);
            Ls = __fmaf_rn(w, __shfl_sync(0xffffffffu, ml.y, cc), Ls);
            O.x = __fmaf_rn(w, v[cc].x, O.x);
            O.y = __fmaf_rn(w, v[cc].y, O.y);
            O.z = __fmaf_rn(w, v[cc].z, O.z);
            O.w = __fmaf_rn(w, v[cc].w, O.w);
        }
    }
    const float inv = __fdiv_rn(1.0f, Ls);
    const float4 out = make_float4(__fmul_rn(O.x, inv), __fmul_rn(O.y, inv), __fmul_rn(O.z, inv), __fmul_rn(O.w, inv));
    *reinterpret_cast<float4*>(ab + 128 * h + 4 * lane) = out;
    if (cta == 0) *reinterpret_cast<float4*>(p.att + 128 * h + 4 * lane) = out;
    if (h == 0) trace_step(p, l, 2, 4);
    __syncthreads();
    trace_step(p, l, 2, 6);
    if (h < N_EMBD / 256) {
        const float4 a = *reinterpret_cast<const float4*>(ab + 256 * h + 8 * lane);
        const float4 b = *reinterpret_cast<const float4*>(ab + 256 * h + 8 * lane + 4);
        quant_xq<false>(a, b, s.xq(), h);
    }
    __syncthreads();
}

// o_proj input for contexts combined by the head-pair combiners: the 2048 epoch-tagged
// attention values (polled), quantized here to Q8_K ties-to-even, one block per warp --
// the same bytes as the combiners' p.att_q8k blocks.
__device__ bool load_att_epoch(const DecodeParams& p, const Smem& s, unsigned epoch) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    bool ok = true;
    if (warp < N_EMBD / 256) {
        float y[8];
        ok = load8c_epoch(p.attw + (blockIdx.x % ATTW_COPIES) * N_EMBD + 256 * warp + 8 * lane, epoch, y, p.err);
        if (p.trace && blockIdx.x == 0 && lane == 0 && epoch == (epoch & ~0xffu) + 1) p.trace[2920 + warp] = globaltimer();
        quant_xq<false>(make_float4(y[0], y[1], y[2], y[3]), make_float4(y[4], y[5], y[6], y[7]), s.xq(), warp);
    }
    return __syncthreads_and(ok);
}

__device__ bool phase_o(const DecodeParams& p, const Smem& s, int l, int cta, int ncta, unsigned seq) {
    const LayerMeta& L = s.meta()[l];
    const PhaseLayout pl = phase_layout(L, *s.rows(), 1);
    const int r0 = pl.row0[0], n = pl.nrows[0];
    const float xr = threadIdx.x < n ? __ldcg(p.x + r0 + threadIdx.x) : 0.0f;   // residual rows, early
    if (!att_flagged(p)) {
        combine_attention(p, s, l, cta);
    } else if (trace_step(p, l, 2, 5), !load_att_epoch(p, s, att_epoch(seq, l))) {
        return false;
    }
    trace_step(p, l, 2, 1);
    if (!wait_weights(p, s, 4 * l + 1)) return false;
    trace_step(p, l, 2, 2);
    dec_gemv(p, s, L.to, s.wbuf(1), n, s.wbuf(1), n, N_EMBD / 256, s.rowval(),
             (p.trace && l == 1 && cta == 0) ? p.trace + TRACE_GEMV + 0 : nullptr);
    if (threadIdx.x < n) {
        const float xn = __fadd_rn(xr, s.rowval()[threadIdx.x]);
        p.x[r0 + threadIdx.x] = xn;
#pragma unroll
        for (int r = 0; r < XLL_COPIES; ++r) st_epoch(p.xll + r * N_EMBD + r0 + threadIdx.x, xn, x_epoch(seq, 2 * l + 1));
    }
    trace_cta(p, l, 2, 0);
    return true;
}

__device__ bool phase_gu(const DecodeParams& p, const Smem& s, int l, int cta, int ncta, unsigned seq) {
    const LayerMeta& L = s.meta()[l];
    if (!norm_quant<true, X_EPOCH>(p, nullptr, x_epoch(seq, 2 * l + 1), meta_f32(p, L.ffn_norm), s,
                                   l == 1 ? TRACE_POLL : -1))
        return false;
    trace_mark(p, 3 + 2 * (5 * l + 2));
    trace_cta(p, l, 2, 1);
    trace_step(p, l, 3, 1);
    if (!wait_weights(p, s, 4 * l + 2)) return false;
    if (threadIdx.x == COPY_THREAD) issue_copy(p, s, 4 * l + 3, cta, ncta);   // down rows: buffer 1
    trace_step(p, l, 3, 2);
    const PhaseLayout pl = phase_layout(L, *s.rows(), 2);
    const int n = pl.nrows[0];
    float* rv = s.rowval();
    unsigned long long* tr = (p.trace && l == 1 && cta == 0) ? p.trace + TRACE_GEMV + 6 : nullptr;
    if (L.tg == L.tu) {   // gate rows then up rows in one pass: rv[0, n) gate, rv[n, 2n) up
        dec_gemv(p, s, L.tg, s.wbuf(0) + pl.off[0], n, s.wbuf(0) + pl.off[1], 2 * n, N_EMBD / 256, rv, tr);
        trace_step(p, l, 3, 3);
    } else {
        dec_gemv(p, s, L.tg, s.wbuf(0) + pl.off[0], n, s.wbuf(0) + pl.off[0], n, N_EMBD / 256, rv, tr);
        trace_step(p, l, 3, 3);
        dec_gemv(p, s, L.tu, s.wbuf(0) + pl.off[1], n, s.wbuf(0) + pl.off[1], n, N_EMBD / 256, rv + n, nullptr);
    }
    trace_step(p, l, 3, 4);
    for (int r = threadIdx.x; r < n; r += blockDim.x) p.h[pl.row0[0] + r] = canon_silu_mul(rv[r], rv[n + r]);
    return true;
}

// down + residual; the new residual rows are published as epoch-tagged words (k = 2l+2);
// then the next layer's K/V and norm prefetches (or the LM head's second stage).
template <typename KT>
__device__ bool phase_down(const DecodeParams& p, const Smem& s, int l, int cta, int ncta, unsigned seq,
                           const LmPlan& lmq) {
    const LayerMeta& L = s.meta()[l];
    const PhaseLayout pl = phase_layout(L, *s.rows(), 3);
    const int r0 = pl.row0[0], n = pl.nrows[0];
    const float xr = threadIdx.x < n ? __ldcg(p.x + r0 + threadIdx.x) : 0.0f;   // residual rows, early
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    {   // Q8_K of h straight from L2: warp w quantises blocks w and w+16 (24 blocks), both loads first
        static_assert(N_FF / 256 <= 2 * (DEC_THREADS / 32), "two h blocks per warp");
        const int b0 = warp, b1 = warp + (DEC_THREADS >> 5);
        const bool two = b1 < N_FF / 256;
        const float4 a0 = ld_cg_f4(p.h + 256 * b0 + 8 * lane);
        const float4 c0 = ld_cg_f4(p.h + 256 * b0 + 8 * lane + 4);
        float4 a1 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = a1;
        if (two) {
            a1 = ld_cg_f4(p.h + 256 * b1 + 8 * lane);
            c1 = ld_cg_f4(p.h + 256 * b1 + 8 * lane + 4);
        }
        quant_xq<true>(a0, c0, s.xq(), b0);
        if (warp == 0) trace_step(p, l, 4, 3);   // h loaded, first block quantised
        if (two) quant_xq<true>(a1, c1, s.xq(), b1);
    }
    __syncthreads();
    trace_step(p, l, 4, 1);
    if (!wait_weights(p, s, 4 * l + 3)) return false;
    if (threadIdx.x == COPY_THREAD) issue_copy(p, s, 4 * l + 4, cta, ncta);   // next QKV rows or LM stage 0: buffer 0
    trace_step(p, l, 4, 2);
    dec_gemv(p, s, L.td, s.wbuf(1), n, s.wbuf(1), n, N_FF / 256, s.rowval(),
             (p.trace && l == 1 && cta == 0) ? p.trace + TRACE_GEMV + 3 : nullptr);
    if (threadIdx.x < n) {
        const float xn = __fadd_rn(xr, s.rowval()[threadIdx.x]);
        p.x[r0 + threadIdx.x] = xn;
#pragma unroll
        for (int r = 0; r < XLL_COPIES; ++r) st_epoch(p.xll + r * N_EMBD + r0 + threadIdx.x, xn, x_epoch(seq, 2 * l + 2));
    }
    trace_cta(p, l, 4, 0);
    if (threadIdx.x == ISSUE_THREAD) {
        if (l + 1 == p.n_layer) {
            fence_proxy_async_smem();
            for (int st = 1; st < LM_SLOTS; ++st) issue_lm_stage(p, s, lmq, st);   // slots after stage 0's lie
                                                                                  // over buffer 1, free now
        } else {
            prefetch_attention<KT>(p, l + 1, cta);
            prefetch_norms(p, s, l + 1, cta);
        }
    }
    return true;
}

__device__ void phase_lm(const DecodeParams& p, const Smem& s, int cta, int ncta, unsigned seq) {
    const LmPlan q = lm_plan(p, cta, ncta);
    if (!norm_quant<false, X_EPOCH>(p, nullptr, x_epoch(seq, 2 * p.n_layer), p.out_norm, s)) return;
    trace_mark(p, 3 + 2 * (5 * (p.n_layer - 1) + 4));
    trace_step(p, 1, 5, 1);   // rmsnorm (ops.cpp:468-481) + quantize_row_q8_K_avx2
    float best = -__int_as_float(0x7f800000);
    int besti = 0x7fffffff;
    int nan0 = 0;
    for (int st = 0; st < q.nstages; ++st) {
        const int slot = st % LM_SLOTS;
        const bool ok = mbar_wait(&s.lmbar()[slot], (st / LM_SLOTS) & 1, p.err);
        if (__syncthreads_or(!ok)) return;
        const int a = q.r0 + st * q.sr, n = min(q.sr, q.r1 - a);
        float* lg = p.logits;
        const int wl = p.write_logits;
        dec_gemv(p, s, p.lm_type, lm_slot(s, slot), n, lm_slot(s, slot), n, q.nb, s.rowval(), nullptr);
        if (threadIdx.x < n) {
            const int row = a + threadIdx.x;
            const float v = s.rowval()[threadIdx.x];
            if (wl) lg[row] = v;
            if (row == 0 && v != v) nan0 = 1;
            if (v > best || (v == best && row < besti)) best = v, besti = row;
        }
        if (threadIdx.x == 0 && st + LM_SLOTS < q.nstages) issue_lm_stage(p, s, q, st + LM_SLOTS);
        if (st < 4) trace_step(p, 1, 5, 2 + st);
    }
    trace_step(p, 1, 5, 6);
    // CTA argmax (lowest index on ties; NaN never wins; a NaN logit 0 forces 0 like the
    // reference's `if (lg[i] > lg[best])` scan)
    float* red = s.red();
    int* redi = reinterpret_cast<int*>(s.rowval());
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ob > best || (ob == best && oi < besti)) best = ob, besti = oi;
    }
    nan0 = __any_sync(0xffffffffu, nan0);
    if (lane == 0) red[warp] = best, redi[warp] = besti, redi[32 + warp] = nan0;
    __syncthreads();
    if (threadIdx.x == 0) {
        int anynan = 0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
            if (red[w] > best || (red[w] == best && redi[w] < besti)) best = red[w], besti = redi[w];
            anynan |= redi[32 + w];
        }
        p.am_val[cta] = best;
        p.am_idx[cta] = anynan ? -1 : besti;
        __threadfence();
        const unsigned old = atomicAdd(&p.cnt[2], 1u);
        if (old == gridDim.x - 1) {
            __threadfence();
            atomicExch(&p.cnt[2], 0u);
            float bv = -__int_as_float(0x7f800000);
            int bi = 0x7fffffff;
            bool n0 = false;
            for (int c = 0; c < static_cast<int>(gridDim.x); ++c) {
                const float v = __ldcg(p.am_val + c);
                const int i = __ldcg(p.am_idx + c);
                if (i < 0) {
                    n0 = true;
                    continue;
                }
                if (v > bv || (v == bv && i < bi)) bv = v, bi = i;
            }
            const int result = (n0 || bi == 0x7fffffff) ? 0 : bi;
            *p.argmax_out = result;
            *p.token_dev = result;
        }
    }
}

template <typename KT>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(const DecodeParams p) {
    const Smem s;
    if (threadIdx.x == 0) {
        CtaRows cr;
        split_range(N_EMBD, blockIdx.x, gridDim.x, cr.od0, cr.od1);
        split_range(N_FF, blockIdx.x, gridDim.x, cr.gu0, cr.gu1);
        *s.rows() = cr;
    }
    for (int i = threadIdx.x; i < p.n_layer; i += blockDim.x) {
        const LayerDev& L = p.layers[i];
        LayerMeta m;
        const uint8_t* const wp[7] = {L.wq, L.wk, L.wv, L.wo, L.wg, L.wu, L.wd};
#pragma unroll
        for (int k = 0; k < 7; ++k) m.w[k] = static_cast<uint32_t>(wp[k] - p.arena);
        m.attn_norm = static_cast<uint32_t>(reinterpret_cast<const uint8_t*>(L.attn_norm) - p.arena);
        m.ffn_norm = static_cast<uint32_t>(reinterpret_cast<const uint8_t*>(L.ffn_norm) - p.arena);
        m.tq = static_cast<uint8_t>(L.tq), m.tk = static_cast<uint8_t>(L.tk), m.tv = static_cast<uint8_t>(L.tv);
        m.to = static_cast<uint8_t>(L.to), m.tg = static_cast<uint8_t>(L.tg), m.tu = static_cast<uint8_t>(L.tu);
        m.td = static_cast<uint8_t>(L.td), m.pad = 0;
        m.qkv0 = static_cast<int16_t>(2 * qkv_pair_boundary(L.tq, L.tk, L.tv, blockIdx.x, gridDim.x));
        m.qkv1 = static_cast<int16_t>(2 * qkv_pair_boundary(L.tq, L.tk, L.tv, blockIdx.x + 1, gridDim.x));
        s.meta()[i] = m;
    }
    __syncthreads();

    const int cta = blockIdx.x, ncta = gridDim.x;
    const int token = p.token >= 0 ? p.token : *reinterpret_cast<volatile int*>(p.token_dev);
    if (token < 0 || token >= p.n_vocab) {
        if (threadIdx.x == 0) atomicOr(p.err, ERR_BAD_TOKEN);
        return;
    }
    BarState bs;
    bs.base = *reinterpret_cast<volatile unsigned*>(p.bar + 1);
    unsigned seq = (*reinterpret_cast<volatile unsigned*>(p.bar + 2) + 1u) & 0xffffffu;   // epochs of xll
    if (seq == 0) seq = 1;
    bs.idx = 0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 8; ++i) mbar_init(&s.wbar()[i], 1);
        for (int i = 0; i < 4; ++i) mbar_init(&s.lmbar()[i], 1);
        fence_mbar_init();
        issue_weight_phase(p, s, 0, cta, ncta);
        prefetch_layer_l2(p, s, 0, 1);
        prefetch_attention<KT>(p, 0, cta);
        prefetch_norms(p, s, 0, cta);
    }
    __syncthreads();
    trace_mark(p, 0);
    const LmPlan lmq = lm_plan(p, cta, ncta);
    const bool flagged = att_flagged(p);
    // flags[0] (early_gu, SCHED_EARLY_GU): the attention scratch fits behind this CTA's o_proj
    // rows in buffer 1 (every layer), so gate/up is copied into buffer 0 during attention.
    if (threadIdx.x == 0) {
        int ob = 0;
        for (int l = 0; l < p.n_layer; ++l) ob = max(ob, row_bytes(s.meta()[l].to, N_EMBD));
        s.flags()[0] = (p.sched & SCHED_EARLY_GU) && p.pos + 1 <= 2048 && (s.rows()->od1 - s.rows()->od0) * ob <= ATT_B1_OFF;
    }
    __syncthreads();
    for (int l = 0; l < p.n_layer; ++l) {
        if (!phase_qkv<KT>(p, s, l, token, cta, ncta, seq)) return;
        // attention units wait on the q/K/V epochs themselves: no grid barrier
        trace_mark(p, 2 + 2 * (5 * l));
        if (!phase_attention<KT>(p, s, reinterpret_cast<float*>(s.flags()[0] ? s.wbuf(1) + ATT_B1_OFF : s.wbuf(0)), l,
                                 cta, ncta, seq))
            return;
        if (flagged) {   // no grid barrier: o_proj waits for the combiners' epoch-tagged values
            __syncthreads();   // the attention scratch is free once this CTA's units are done
            if (threadIdx.x == COPY_THREAD && !s.flags()[0]) issue_copy(p, s, 4 * l + 2, cta, ncta);
            trace_mark(p, 2 + 2 * (5 * l + 1));
            trace_mark(p, 3 + 2 * (5 * l + 1));
        } else if (!traced_barrier(p, bs, 5 * l + 1, [&] {
                       if (!s.flags()[0]) issue_copy(p, s, 4 * l + 2, cta, ncta);
                   })) {
            return;
        }
        // o_proj -> gate/up and down -> next QKV exchange the residual through epoch-tagged
        // words: no grid barrier (every consumer needs all of x, which orders all reuse).
        if (!phase_o(p, s, l, cta, ncta, seq)) return;
        trace_mark(p, 2 + 2 * (5 * l + 2));
        if (!phase_gu(p, s, l, cta, ncta, seq)) return;
        if (!traced_barrier(p, bs, 5 * l + 3, [&] {
                if (l + 1 == p.n_layer && cta == 0) bulk_prefetch_l2(p.out_norm, N_EMBD * 4);
            }))
            return;
        if (!phase_down<KT>(p, s, l, cta, ncta, seq, lmq)) return;
        trace_mark(p, 2 + 2 * (5 * l + 4));
    }
    if (cta == 0 && threadIdx.x == 0) {
        p.bar[1] = bs.base + bs.idx * gridDim.x;   // next launch's barrier base
        p.bar[2] = seq;                            // next launch uses seq + 1
    }
    phase_lm(p, s, cta, ncta, seq);
    trace_mark(p, 2 + 2 * (5 * p.n_layer));
}

// ---- standalone attention op (execute_attention, ops.cpp:537-628): K/V append at pos,
// then the same split-KV chunks and combine as the decode kernel's attention phase.

__global__ void k_kv_append(const float* __restrict__ k, const float* __restrict__ v, float* kc, float* vc, int pos) {
    const int i = threadIdx.x;
    if (i < KV_DIM) {
        kc[static_cast<size_t>(pos) * KV_DIM + i] = k[i];
        vc[static_cast<size_t>(pos) * KV_DIM + i] = v[i];
    }
}

__global__ void __launch_bounds__(DEC_THREADS, 1) k_attention(const DecodeParams p) {
    const Smem s;
    phase_attention<float>(p, s, reinterpret_cast<float*>(s.wbuf(0)), 0, blockIdx.x, gridDim.x, 1u);
}

// Standalone op: head pair blockIdx.x of the chunks written by k_attention (stream order).
__global__ void __launch_bounds__(DEC_THREADS, 1) k_att_combine(const DecodeParams p) {
    const Smem s;
    combine_pair(p, reinterpret_cast<float*>(s.wbuf(0)), 0, blockIdx.x, 1u);
}

#include "mcpm_batch.cuh"

// Tensor-parallel attention (one rank's KV group(s) and head pairs).  The position is read
// from device memory so a whole token can be captured in one CUDA graph; the grid covers the
// largest chunk count of the cache and units past the current one return at once.
__global__ void __launch_bounds__(DEC_THREADS, 1) k_tp_att_units(DecodeParams p, const int* pos, int g0) {
    grid_dep_launch();
    grid_dep_wait();
    p.pos = *pos;
    const int n = p.pos + 1, P = 32 * ((n + 2047) / 2048), C = (n + P - 1) / P;
    const int c = blockIdx.x, g = g0 + blockIdx.y;
    if (c >= C) return;
    const Smem sm;
    const int t0 = c * P, np = min(t0 + P, n) - t0;
    if (P == 32)
        attention_unit32<float>(p, reinterpret_cast<float*>(sm.wbuf(0)), 0, g, c, t0, np, 1u, false);
    else
        attention_unit_big<float>(p, reinterpret_cast<float*>(sm.wbuf(0)), 0, g, c, t0, np, 1u, false);
}

__global__ void __launch_bounds__(DEC_THREADS, 1) k_tp_att_combine(DecodeParams p, const int* pos, int b0) {
    grid_dep_launch();
    grid_dep_wait();
    p.pos = *pos;
    const Smem sm;
    combine_pair(p, reinterpret_cast<float*>(sm.wbuf(0)), 0, b0 + blockIdx.x, 1u);
}

}  // namespace

cudaError_t launch_tp_attention(const DecodeParams& p, const int* pos_dev, int g0, int ng, int b0, int nb,
                                cudaStream_t stream) {
    static int prepared_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (prepared_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(k_tp_att_units, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_BYTES);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_tp_att_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_BYTES);
        if (e != cudaSuccess) return e;
        prepared_dev = dev;
    }
    const int cmax = std::min(ATT_MAX_CHUNKS, (p.max_seq + 31) / 32);   // most chunks of any length <= max_seq
    cudaLaunchAttribute attr[1];   // programmatic dependents of the preceding kernel
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = SM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(cmax, ng);
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_tp_att_units, p, pos_dev, g0);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(nb);
    return cudaLaunchKernelEx(&cfg, k_tp_att_combine, p, pos_dev, b0);
}

size_t decode_smem_bytes() { return SM_BYTES; }

cudaError_t decode_prepare() {
    cudaError_t e = cudaFuncSetAttribute(k_decode<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(decode_smem_bytes()));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_decode<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(decode_smem_bytes()));
}

int decode_max_ctas_per_sm() {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_decode<float>, DEC_THREADS, decode_smem_bytes()) !=
        cudaSuccess)
        return 0;
    return n;
}

// One batched decode step (every sequence one token), as a sequence of stream-ordered
// launches: per layer QKV GEMM, RoPE + K/V append, attention units, head-pair combine,
// o_proj GEMM, residual + norm, gate/up GEMM, SwiGLU, down GEMM, residual + norm; then the
// LM head GEMM and the per-sequence argmax.
cudaError_t launch_batch_step(const BatchLaunch& b, cudaStream_t stream) {
    static int prepared_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr int UNIT_SMEM_BIG = 98304, COMBINE_SMEM = 68608;
    if (prepared_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(k_b_att_units<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, UNIT_SMEM_BIG);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_b_att_units<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, UNIT_SMEM_BIG);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_b_att_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, COMBINE_SMEM);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_b_gemm8, cudaFuncAttributeMaxDynamicSharedMemorySize, GA_BYTES);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_b_gemm24, cudaFuncAttributeMaxDynamicSharedMemorySize, GB_BYTES);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_b_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TB_BYTES);
        if (e != cudaSuccess) return e;
        prepared_dev = dev;
    }
    static_assert((2 * ATT_MAX_CHUNKS * HEAD_DIM + 6 * ATT_MAX_CHUNKS + 4 + 256) * 4 <= COMBINE_SMEM, "combine smem");
    static_assert((8 * HEAD_DIM + ATT_BIG_ROWS * HEAD_DIM + 8 * ATT_SC_STRIDE + 16 + 2 * HEAD_DIM) * 4 <= UNIT_SMEM_BIG,
                  "unit smem");
    BStepArgs a{};
    a.n_seq = b.n_seq, a.max_seq = b.max_seq, a.n_layer = b.n_layer, a.n_vocab = b.n_vocab;
    a.kv_seq_stride = b.shared_kv ? 0 : static_cast<size_t>(b.n_layer) * b.max_seq * KV_DIM;
    a.kc = b.kc, a.vc = b.vc, a.x = b.x, a.y = b.y, a.q = b.q, a.att_part = b.att_part, a.att = b.att;
    a.logits = b.logits, a.aqs = b.aqs, a.ad = b.ad, a.abs = b.abs;
    a.tokens = b.tokens, a.pos = b.pos, a.argmax = b.argmax, a.embd = b.embd, a.rope = b.rope, a.err = b.err;
    const int n = b.n_seq;
    const int nmax = b.max_pos + 1, Pmax = 32 * ((nmax + 2047) / 2048), Cmax = (nmax + Pmax - 1) / Pmax;
    const int unit_smem = Pmax == 32 ? 24576 : UNIT_SMEM_BIG;
    const bool gemm_kind = b.tcgen05 != 0;
    auto gemm = [&](std::initializer_list<BGemmSeg> segs, int nb, float* y, int y_stride,
                    unsigned long long* trace = nullptr) {
        BGemmArgs g{};
        g.trace = trace;
        const int rows_per_tile = gemm_kind ? TB_M : BG_ROWS;
        int tiles = 0, i = 0;
        for (BGemmSeg sg : segs) {
            sg.tile0 = tiles;
            tiles += (sg.rows + rows_per_tile - 1) / rows_per_tile;
            g.seg[i++] = sg;
        }
        g.nseg = i, g.ntiles = tiles, g.nb = nb;
        g.aqs = b.aqs, g.ad = b.ad, g.abs = b.abs, g.y = y, g.y_stride = y_stride, g.n_seq = n, g.err = b.err;
        if (gemm_kind) {
            g.part = b.gemm_part, g.cnt = b.gemm_cnt;
            const int units = tiles * (nb / TB_G);
            k_b_gemm_tc<<<std::min(units, b.n_sm), TB_CTA_THREADS, TB_BYTES, stream>>>(g);
            return;
        }
        if (nb == 8)
            k_b_gemm8<<<std::min(tiles, b.n_sm), BG_THREADS, GA_BYTES, stream>>>(g);
        else
            k_b_gemm24<<<std::min(tiles, b.n_sm), BG_THREADS, GB_BYTES, stream>>>(g);
    };
    a.norm = b.layers[0].attn_norm;
    k_b_embed<<<n, 256, 0, stream>>>(a);
    for (int l = 0; l < b.n_layer; ++l) {
        const LayerDev& L = b.layers[l];
        gemm({{L.wq, L.tq, N_EMBD, 0, 0}, {L.wk, L.tk, KV_DIM, N_EMBD, 0}, {L.wv, L.tv, KV_DIM, N_EMBD + KV_DIM, 0}},
             N_EMBD / 256, b.y, 2 * N_FF);
        if (b.kv_f16) {
            k_b_rope_kv<__half><<<n, 256, 0, stream>>>(a, l);
            k_b_att_units<__half><<<dim3(n, 2 * Cmax), DEC_THREADS, unit_smem, stream>>>(a, l);
        } else {
            k_b_rope_kv<float><<<n, 256, 0, stream>>>(a, l);
            k_b_att_units<float><<<dim3(n, 2 * Cmax), DEC_THREADS, unit_smem, stream>>>(a, l);
        }
        k_b_att_combine<<<dim3(n, N_EMBD / 256), DEC_THREADS, COMBINE_SMEM, stream>>>(a, l);
        gemm({{L.wo, L.to, N_EMBD, 0, 0}}, N_EMBD / 256, b.y, 2 * N_FF);
        a.norm = L.ffn_norm;
        k_b_res_norm<true><<<n, 256, 0, stream>>>(a);
        gemm({{L.wg, L.tg, N_FF, 0, 0}, {L.wu, L.tu, N_FF, N_FF, 0}}, N_EMBD / 256, b.y, 2 * N_FF,
             l == 1 && b.trace ? b.trace + TRACE_GEMM : nullptr);
        k_b_swiglu<<<dim3(n, N_FF / 256 / 8), 256, 0, stream>>>(a);
        gemm({{L.wd, L.td, N_EMBD, 0, 0}}, N_FF / 256, b.y, 2 * N_FF);
        if (l + 1 < b.n_layer) {
            a.norm = b.layers[l + 1].attn_norm;
            k_b_res_norm<true><<<n, 256, 0, stream>>>(a);
        } else {
            a.norm = b.out_norm;
            k_b_res_norm<false><<<n, 256, 0, stream>>>(a);
        }
    }
    if (!b.skip_lm) {
        gemm({{b.lm, b.lm_type, b.n_vocab, 0, 0}}, N_EMBD / 256, b.logits, b.n_vocab);
        k_b_argmax<<<n, 1024, 0, stream>>>(a, b.chain);
    }
    return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeParams& p, int n_ctas, cudaStream_t stream) {
    void* args[] = {const_cast<DecodeParams*>(&p)};
    const void* fn = p.kv_f16 ? reinterpret_cast<const void*>(&k_decode<__half>) : reinterpret_cast<const void*>(&k_decode<float>);
    return cudaLaunchCooperativeKernel(fn, dim3(n_ctas), dim3(DEC_THREADS), args,
                                       decode_smem_bytes(), stream);
}

}  // namespace mcpm

namespace mcpm {
cudaError_t launch_attention(const float* q, const float* k, const float* v, float* kc, float* vc, int pos, int max_seq,
                             float* out, uint8_t* out_q8k, float* part, cudaStream_t stream) {
    k_kv_append<<<1, KV_DIM, 0, stream>>>(k, v, kc, vc, pos);
    DecodeParams p{};
    p.q = const_cast<float*>(q);
    p.kc = kc;
    p.vc = vc;
    p.max_seq = max_seq;
    p.pos = pos;
    p.att = out;
    p.att_q8k = out_q8k;
    p.att_part = part;
    static int prepared_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (prepared_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_BYTES);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_att_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_BYTES);
        if (e != cudaSuccess) return e;
        prepared_dev = dev;
    }
    const int n = pos + 1, P = 32 * ((n + 2047) / 2048), C = (n + P - 1) / P;
    k_attention<<<2 * C, DEC_THREADS, SM_BYTES, stream>>>(p);   // chunk records (headers with epoch 1<<8)
    k_att_combine<<<N_EMBD / 256, DEC_THREADS, SM_BYTES, stream>>>(p);
    return cudaGetLastError();
}
}  // namespace mcpm
