// Batched decode (config 3): n_seq <= 64 independent sequences advance one token per step.
// Included by mcpm_decode.cu inside its anonymous namespace: the attention units, the
// head-pair combine, the Q8_K quantiser and the canonical exp / SiLU are the decode kernel's
// own device functions, so every sequence's logits equal a batch-1 decode of that sequence
// bit for bit (MiniCPM5Engine::forward, src/model.cpp:142-242, once per sequence).
//
// Activations between GEMMs are Q8_K blocks split into arrays per sequence: values
// [seq][B_NBA][256] int8, scales [seq][B_NBA] fp32, block sums [seq][B_NBA][16] int16.
//
// GEMM (k_b_gemm): a CTA owns 16 weight rows x 64 sequences; warp w owns sequences
// 8w..8w+7.  Per 256-weight block the reference's AVX2 row kernel keeps eight int32 lane
// partials (ops_avx2.cpp:153-196 Q4_K, :201-276 Q6_K): lane k sums the elements 32s + 4k + t
// (s = 0..7 sub-blocks, t = 0..3) times their sub-block scale.  The block is staged with its
// K dimension permuted lane-major (position 32k + 4s + t), so lane k is the contiguous K range
// [32k, 32k+32): one m16n8k32 int8 MMA per lane.  The weight operand is w' = scale x q split
// as w' = 64*hi + lo (hi = w' >> 6, lo = w' & 63, both int8), so lane_k = 64*(hi.x) + (lo.x)
// exactly, from two MMAs.  The fp32 epilogue then runs the batch-1 GEMV's chain per (row,
// sequence): acc[k] = fma(xd*d, lane_k, acc[k]) over blocks, the fused min chain, and the
// hsum_f32_8 tree.

constexpr int B_NBA = N_FF / 256;   // activation blocks per sequence (24)
constexpr int BG_ROWS = 16;         // GEMM tile rows
constexpr int BG_SEQ = BATCH_MAX;   // GEMM tile sequences (64)
constexpr int BG_STRIDE = 272;      // smem bytes per staged 256-byte row (+16: conflict-free fragment loads)
constexpr int BG_THREADS = 256;

struct BGemmSeg {
    const uint8_t* w;
    int type, rows, out_off, tile0;
};
struct BGemmArgs {
    BGemmSeg seg[3];
    int nseg, ntiles, nb;
    const int8_t* aqs;
    const float* ad;
    const int16_t* abs;
    float* y;
    int y_stride, n_seq;
};

// smem layout of k_b_gemm
constexpr int BGS_AHI = 0;
constexpr int BGS_ALO = BGS_AHI + BG_ROWS * BG_STRIDE;
constexpr int BGS_X = BGS_ALO + BG_ROWS * BG_STRIDE;
constexpr int BGS_XD = BGS_X + BG_SEQ * BG_STRIDE;       // float [64]
constexpr int BGS_PAIR = BGS_XD + BG_SEQ * 4;             // int [64][8] bsums[2g] + bsums[2g+1]
constexpr int BGS_BS = BGS_PAIR + BG_SEQ * 8 * 4;         // int16 [64][16]
constexpr int BGS_RD = BGS_BS + BG_SEQ * 16 * 2;          // float [16] d
constexpr int BGS_RM = BGS_RD + BG_ROWS * 4;              // float [16] dmin
constexpr int BGS_MN = BGS_RM + BG_ROWS * 4;              // uint8 [16][8] Q4_K mins / int8 [16][16] Q6_K scales
constexpr int BGS_BYTES = BGS_MN + BG_ROWS * 16;

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Raw loads of one block for this thread's share (row r, sub-block s, half of it), taken one
// block ahead so their latency overlaps the MMAs of the current block.
struct BRaw {
    uint4 x[4];        // activation chunks c = tid + 256 j
    float xd;          // tid < 64: scale of sequence tid
    uint4 bs;          // tid < 128: 8 block sums of sequence tid/2
    uint32_t w[9];     // weight bytes of (r, s, half)
};

template <int TYPE>
__device__ __forceinline__ void bg_load(const BGemmArgs& a, const uint8_t* w, int rows, int row0, int nb, int b,
                                        BRaw& raw) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = tid + BG_THREADS * j, q = c >> 4, m = c & 15;
        raw.x[j] = q < a.n_seq ? __ldcg(reinterpret_cast<const uint4*>(a.aqs + (static_cast<size_t>(q) * B_NBA + b) * 256) + m)
                               : make_uint4(0u, 0u, 0u, 0u);
    }
    raw.xd = tid < a.n_seq ? __ldcg(a.ad + static_cast<size_t>(tid) * B_NBA + b) : 0.0f;
    raw.bs = tid < 2 * a.n_seq
                 ? __ldcg(reinterpret_cast<const uint4*>(a.abs + (static_cast<size_t>(tid >> 1) * B_NBA + b) * 16) + (tid & 1))
                 : make_uint4(0u, 0u, 0u, 0u);
    const int r = tid >> 4, s = (tid >> 1) & 7, half = tid & 1;
    const int grow = row0 + r;
#pragma unroll
    for (int i = 0; i < 9; ++i) raw.w[i] = 0u;
    if (grow >= rows) return;
    if (TYPE == GGML_Q4_K) {
        const uint8_t* blk = w + (static_cast<size_t>(grow) * nb + b) * Q4K_BYTES;
        const uint4 head = __ldg(reinterpret_cast<const uint4*>(blk));                                  // d, dmin, scales
        const uint4 qv = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * (s >> 1) + 16 * half));   // 16 nibble pairs
        raw.w[0] = head.x, raw.w[1] = head.y, raw.w[2] = head.z, raw.w[3] = head.w;
        raw.w[4] = qv.x, raw.w[5] = qv.y, raw.w[6] = qv.z, raw.w[7] = qv.w;
    } else {   // Q6_K blocks are 210 bytes: 2-byte aligned loads
        const uint8_t* blk = w + (static_cast<size_t>(grow) * nb + b) * Q6K_BYTES;
        const int h = s >> 2, kk = s & 3;
        const uint16_t* ql = reinterpret_cast<const uint16_t*>(blk + 64 * h + 32 * (kk & 1) + 16 * half);
        const uint16_t* qh = reinterpret_cast<const uint16_t*>(blk + 128 + 32 * h + 16 * half);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            raw.w[i] = static_cast<uint32_t>(__ldg(ql + 2 * i)) | (static_cast<uint32_t>(__ldg(ql + 2 * i + 1)) << 16);
            raw.w[4 + i] = static_cast<uint32_t>(__ldg(qh + 2 * i)) | (static_cast<uint32_t>(__ldg(qh + 2 * i + 1)) << 16);
        }
        raw.w[8] = static_cast<uint32_t>(blk[192 + 2 * s + half]) |
                   (static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(blk + 208))) << 16);   // scale, d
    }
}

// Registers -> shared memory: activations permuted lane-major, weights dequantised into the
// hi / lo int8 operands, row and sequence metadata.
template <int TYPE>
__device__ __forceinline__ void bg_store(const BRaw& raw, uint8_t* sm) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = tid + BG_THREADS * j, q = c >> 4, m = c & 15, s = m >> 1;
        const uint32_t wv[4] = {raw.x[j].x, raw.x[j].y, raw.x[j].z, raw.x[j].w};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {   // word kk holds elements 32s + 4k + t, k = 4(m&1) + kk
            const int k = 4 * (m & 1) + kk;
            *reinterpret_cast<uint32_t*>(sm + BGS_X + q * BG_STRIDE + 32 * k + 4 * s) = wv[kk];
        }
    }
    if (tid < BG_SEQ) reinterpret_cast<float*>(sm + BGS_XD)[tid] = raw.xd;
    if (tid < 2 * BG_SEQ) {
        const int q = tid >> 1, h = tid & 1;
        const uint32_t bw[4] = {raw.bs.x, raw.bs.y, raw.bs.z, raw.bs.w};
        int16_t* bs = reinterpret_cast<int16_t*>(sm + BGS_BS) + 16 * q + 8 * h;
        int* pair = reinterpret_cast<int*>(sm + BGS_PAIR) + 8 * q + 4 * h;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int lo = static_cast<int16_t>(bw[i] & 0xffffu), hi = static_cast<int16_t>(bw[i] >> 16);
            bs[2 * i] = static_cast<int16_t>(lo);
            bs[2 * i + 1] = static_cast<int16_t>(hi);
            pair[i] = lo + hi;
        }
    }
    const int r = tid >> 4, s = (tid >> 1) & 7, half = tid & 1;
    uint32_t hw[4], lw[4];
    if (TYPE == GGML_Q4_K) {
        // byte i of the 12 packed scale bytes (raw.w[1..3]), selected without indexing registers
        auto sc8 = [&](int i) -> int {
            const uint32_t wd = i < 4 ? raw.w[1] : i < 8 ? raw.w[2] : raw.w[3];
            return static_cast<int>((wd >> (8 * (i & 3))) & 0xffu);
        };
        int sc, mn;   // get_scale_min_k4 (include/ops.h:67-75)
        if (s < 4) {
            sc = sc8(s) & 63;
            mn = sc8(s + 4) & 63;
        } else {
            sc = (sc8(s + 4) & 15) | ((sc8(s - 4) >> 6) << 4);
            mn = (sc8(s + 4) >> 4) | ((sc8(s) >> 6) << 4);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t qb = raw.w[4 + kk];   // bytes for elements i = 16 half + 4kk + t
            uint32_t h4 = 0u, l4 = 0u;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int byte = (qb >> (8 * t)) & 0xff;
                const int q = (s & 1) ? (byte >> 4) : (byte & 15);
                const int wq = sc * q;
                h4 |= static_cast<uint32_t>((wq >> 6) & 0xff) << (8 * t);
                l4 |= static_cast<uint32_t>(wq & 63) << (8 * t);
            }
            hw[kk] = h4, lw[kk] = l4;
        }
        if (half == 0) sm[BGS_MN + 8 * r + s] = static_cast<uint8_t>(mn);
        if (s == 0 && half == 0) {
            reinterpret_cast<float*>(sm + BGS_RD)[r] = h2f(raw.w[0]);
            reinterpret_cast<float*>(sm + BGS_RM)[r] = h2f(raw.w[0] >> 16);
        }
    } else {
        const int scale = static_cast<int8_t>(raw.w[8] & 0xff);
        const int kk6 = s & 3;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t h4 = 0u, l4 = 0u;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int e = 4 * kk + t;   // element l = 16 half + e of quarter kk6 of half s>>2
                const int qlb = (raw.w[e >> 2] >> (8 * (e & 3))) & 0xff;
                const int qhb = (raw.w[4 + (e >> 2)] >> (8 * (e & 3))) & 0xff;
                const int lo4 = (kk6 & 2) ? (qlb >> 4) : (qlb & 15);
                const int q6 = lo4 | (((qhb >> (2 * kk6)) & 3) << 4);
                const int wq = scale * q6;
                h4 |= static_cast<uint32_t>((wq >> 6) & 0xff) << (8 * t);
                l4 |= static_cast<uint32_t>(wq & 63) << (8 * t);
            }
            hw[kk] = h4, lw[kk] = l4;
        }
        reinterpret_cast<int8_t*>(sm + BGS_MN)[16 * r + 2 * s + half] = static_cast<int8_t>(scale);
        if (s == 0 && half == 0) reinterpret_cast<float*>(sm + BGS_RD)[r] = h2f(raw.w[8] >> 16);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {   // lane k = 4 half + kk, permuted position 32k + 4s
        const int k = 4 * half + kk;
        *reinterpret_cast<uint32_t*>(sm + BGS_AHI + r * BG_STRIDE + 32 * k + 4 * s) = hw[kk];
        *reinterpret_cast<uint32_t*>(sm + BGS_ALO + r * BG_STRIDE + 32 * k + 4 * s) = lw[kk];
    }
}

template <int TYPE, int NB>
__device__ void bg_tile(const BGemmArgs& a, const BGemmSeg& sg, int row0, uint8_t* sm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const bool active = 8 * warp < a.n_seq;   // warp-uniform
    float acc[4][8], acc_min[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        acc_min[e] = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[e][k] = 0.0f;
    }
    BRaw raw;
    bg_load<TYPE>(a, sg.w, sg.rows, row0, NB, 0, raw);
    for (int b = 0; b < NB; ++b) {
        bg_store<TYPE>(raw, sm);
        __syncthreads();
        if (b + 1 < NB) bg_load<TYPE>(a, sg.w, sg.rows, row0, NB, b + 1, raw);
        if (active) {
            const float* xd = reinterpret_cast<const float*>(sm + BGS_XD);
            const float* rd = reinterpret_cast<const float*>(sm + BGS_RD);
            const int rr[4] = {g, g, g + 8, g + 8};
            const int qq[4] = {8 * warp + 2 * t, 8 * warp + 2 * t + 1, 8 * warp + 2 * t, 8 * warp + 2 * t + 1};
            float ds[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) ds[e] = __fmul_rn(xd[qq[e]], rd[rr[e]]);
            if (TYPE == GGML_Q4_K) {   // min term: minsum = sum_g mins[g] * (bsums[2g] + bsums[2g+1])
                const float* rm = reinterpret_cast<const float*>(sm + BGS_RM);
                const int* pair = reinterpret_cast<const int*>(sm + BGS_PAIR);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint8_t* mn = sm + BGS_MN + 8 * rr[e];
                    const int* pr = pair + 8 * qq[e];
                    int ms = 0;
#pragma unroll
                    for (int gg = 0; gg < 8; ++gg) ms += static_cast<int>(mn[gg]) * pr[gg];
                    acc_min[e] = __fmaf_rn(-__fmul_rn(xd[qq[e]], rm[rr[e]]), __int2float_rn(ms), acc_min[e]);
                }
            }
            const uint8_t* ah = sm + BGS_AHI + g * BG_STRIDE + 4 * t;
            const uint8_t* al = sm + BGS_ALO + g * BG_STRIDE + 4 * t;
            const uint8_t* xb = sm + BGS_X + (8 * warp + g) * BG_STRIDE + 4 * t;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t fa_h[4] = {*reinterpret_cast<const uint32_t*>(ah + 32 * k),
                                          *reinterpret_cast<const uint32_t*>(ah + 8 * BG_STRIDE + 32 * k),
                                          *reinterpret_cast<const uint32_t*>(ah + 32 * k + 16),
                                          *reinterpret_cast<const uint32_t*>(ah + 8 * BG_STRIDE + 32 * k + 16)};
                const uint32_t fa_l[4] = {*reinterpret_cast<const uint32_t*>(al + 32 * k),
                                          *reinterpret_cast<const uint32_t*>(al + 8 * BG_STRIDE + 32 * k),
                                          *reinterpret_cast<const uint32_t*>(al + 32 * k + 16),
                                          *reinterpret_cast<const uint32_t*>(al + 8 * BG_STRIDE + 32 * k + 16)};
                const uint32_t fb[2] = {*reinterpret_cast<const uint32_t*>(xb + 32 * k),
                                        *reinterpret_cast<const uint32_t*>(xb + 32 * k + 16)};
                int ch[4], cl[4];
                mma_s8(ch, fa_h, fb);
                mma_s8(cl, fa_l, fb);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    int lv = ch[e] * 64 + cl[e];
                    if (TYPE == GGML_Q6_K) {   // -32 * (bsums[2k] * sc[2k] + bsums[2k+1] * sc[2k+1])
                        const int16_t* bs = reinterpret_cast<const int16_t*>(sm + BGS_BS) + 16 * qq[e];
                        const int8_t* sc = reinterpret_cast<const int8_t*>(sm + BGS_MN) + 16 * rr[e];
                        lv -= 32 * (bs[2 * k] * sc[2 * k] + bs[2 * k + 1] * sc[2 * k + 1]);
                    }
                    acc[e][k] = __fmaf_rn(ds[e], __int2float_rn(lv), acc[e][k]);
                }
            }
        }
        __syncthreads();
    }
    if (!active) return;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int row = row0 + (e < 2 ? g : g + 8), q = 8 * warp + 2 * t + (e & 1);
        if (row >= sg.rows || q >= a.n_seq) continue;
        const float* v = acc[e];   // hsum_f32_8 (ops_avx2.cpp:43-48)
        float r = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[4]), __fadd_rn(v[2], v[6])),
                            __fadd_rn(__fadd_rn(v[1], v[5]), __fadd_rn(v[3], v[7])));
        if (TYPE == GGML_Q4_K) r = __fadd_rn(r, acc_min[e]);
        a.y[static_cast<size_t>(q) * a.y_stride + sg.out_off + row] = r;
    }
}

__global__ void __launch_bounds__(BG_THREADS, 2) k_b_gemm(const BGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smg[];
    for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
        // segment by value (a runtime index into the parameter array would copy it to local memory)
        const BGemmSeg sg = (a.nseg > 2 && tile >= a.seg[2].tile0) ? a.seg[2]
                            : (a.nseg > 1 && tile >= a.seg[1].tile0) ? a.seg[1]
                                                                     : a.seg[0];
        const int row0 = (tile - sg.tile0) * BG_ROWS;
        if (sg.type == GGML_Q4_K) {
            if (a.nb == 8)
                bg_tile<GGML_Q4_K, 8>(a, sg, row0, smg);
            else
                bg_tile<GGML_Q4_K, 24>(a, sg, row0, smg);
        } else {
            if (a.nb == 8)
                bg_tile<GGML_Q6_K, 8>(a, sg, row0, smg);
            else
                bg_tile<GGML_Q6_K, 24>(a, sg, row0, smg);
        }
    }
}

// RMSNorm + Q8_K of one sequence (norm_quant's arithmetic: per-thread fma chains over
// x[tid + 256 i], warp butterflies, an 8-leaf tree; y = (x * w) * rms) for a 256-thread CTA.
template <bool AWAY>
__device__ void b_norm_quant(const float* xs, const float* w, int8_t* qs, float* d, int16_t* bs) {
    __shared__ float red[8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a = __fmaf_rn(xs[tid + 256 * i], xs[tid + 256 * i], a);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) red[warp] = a;
    __syncthreads();
    const float ss = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3])),
                               __fadd_rn(__fadd_rn(red[4], red[5]), __fadd_rn(red[6], red[7])));
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(N_EMBD)), 1e-6f)));
    float y[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
        y[k] = __fmul_rn(__fmul_rn(xs[256 * warp + 8 * lane + k], __ldg(w + 256 * warp + 8 * lane + k)), rms);
    quant_block_warp<AWAY>(y, qs + 256 * warp, d + warp, bs + 16 * warp);
    __syncthreads();
}

struct BStepArgs {
    int n_seq, max_seq, n_layer;
    float *kc, *vc, *x, *y, *q, *att_part, *att, *logits;
    int8_t* aqs;
    float* ad;
    int16_t* abs;
    int *tokens, *pos, *argmax;
    const uint8_t* embd;
    const float2* rope;
    const float* norm;   // this launch's norm weights
    int n_vocab;
    unsigned* err;
};

__device__ __forceinline__ size_t b_kv_off(const BStepArgs& a, int s, int l) {
    return (static_cast<size_t>(s) * a.n_layer + l) * a.max_seq * KV_DIM;
}

// Layer-0 input: embedding row of each sequence's token, then RMSNorm + Q8_K (ties away).
__global__ void __launch_bounds__(256) k_b_embed(const BStepArgs a) {
    __shared__ __align__(16) float xs[N_EMBD];
    const int s = blockIdx.x;
    embed_row(a.embd, a.tokens[s], xs);
    __syncthreads();
    for (int i = threadIdx.x; i < N_EMBD; i += blockDim.x) a.x[static_cast<size_t>(s) * N_EMBD + i] = xs[i];
    b_norm_quant<true>(xs, a.norm, a.aqs + static_cast<size_t>(s) * B_NBA * 256, a.ad + static_cast<size_t>(s) * B_NBA,
                       a.abs + static_cast<size_t>(s) * B_NBA * 16);
}

// x += y (residual, model.cpp:201-203 / :223-225), then RMSNorm + Q8_K for the next GEMM
// (ties away for QKV / gate-up, ties to even before the LM head).
template <bool AWAY>
__global__ void __launch_bounds__(256) k_b_res_norm(const BStepArgs a) {
    __shared__ __align__(16) float xs[N_EMBD];
    const int s = blockIdx.x;
    float* x = a.x + static_cast<size_t>(s) * N_EMBD;
    const float* y = a.y + static_cast<size_t>(s) * 2 * N_FF;
    for (int i = threadIdx.x; i < N_EMBD; i += blockDim.x) {
        const float v = __fadd_rn(x[i], y[i]);
        x[i] = v;
        xs[i] = v;
    }
    __syncthreads();
    b_norm_quant<AWAY>(xs, a.norm, a.aqs + static_cast<size_t>(s) * B_NBA * 256, a.ad + static_cast<size_t>(s) * B_NBA,
                       a.abs + static_cast<size_t>(s) * B_NBA * 16);
}

// RoPE on q and k (interleaved pairs, as in phase_qkv), q to its buffer, K/V into the
// sequence's cache at its position.
__global__ void __launch_bounds__(256) k_b_rope_kv(const BStepArgs a, int l) {
    const int s = blockIdx.x, pos = a.pos[s];
    const float* y = a.y + static_cast<size_t>(s) * 2 * N_FF;
    float* kdst = a.kc + b_kv_off(a, s, l) + static_cast<size_t>(pos) * KV_DIM;
    float* vdst = a.vc + b_kv_off(a, s, l) + static_cast<size_t>(pos) * KV_DIM;
    for (int pr = threadIdx.x; pr < (N_EMBD + 2 * KV_DIM) / 2; pr += blockDim.x) {
        const int R = 2 * pr;
        const float v0 = y[R], v1 = y[R + 1];
        if (R < N_EMBD + KV_DIM) {
            const float2 c = __ldg(a.rope + static_cast<size_t>(pos) * (HEAD_DIM / 2) + ((R & (HEAD_DIM - 1)) >> 1));
            const float r0 = __fmaf_rn(c.x, v0, -__fmul_rn(c.y, v1));
            const float r1 = __fmaf_rn(c.y, v0, __fmul_rn(c.x, v1));
            if (R < N_EMBD) {
                a.q[static_cast<size_t>(s) * N_EMBD + R] = r0;
                a.q[static_cast<size_t>(s) * N_EMBD + R + 1] = r1;
            } else {
                kdst[R - N_EMBD] = r0;
                kdst[R - N_EMBD + 1] = r1;
            }
        } else {
            vdst[R - N_EMBD - KV_DIM] = v0;
            vdst[R - N_EMBD - KV_DIM + 1] = v1;
        }
    }
}

__device__ DecodeParams b_att_params(const BStepArgs& a, int s) {
    DecodeParams p{};
    p.q = a.q + static_cast<size_t>(s) * N_EMBD;
    p.kc = a.kc + b_kv_off(a, s, 0);
    p.vc = a.vc + b_kv_off(a, s, 0);
    p.max_seq = a.max_seq;
    p.pos = a.pos[s];
    p.att_part = a.att_part + static_cast<size_t>(s) * ATT_PART_FLOATS;
    p.att = a.att + static_cast<size_t>(s) * N_EMBD;
    p.att_qs = a.aqs + static_cast<size_t>(s) * B_NBA * 256;
    p.att_d = a.ad + static_cast<size_t>(s) * B_NBA;
    p.att_bs = a.abs + static_cast<size_t>(s) * B_NBA * 16;
    p.err = a.err;
    return p;
}

// Attention units of every sequence: blockIdx.x = sequence, blockIdx.y = (KV group, chunk).
__global__ void __launch_bounds__(DEC_THREADS, 1) k_b_att_units(const BStepArgs a, int l) {
    const int s = blockIdx.x, item = blockIdx.y;
    const int n = a.pos[s] + 1, P = 32 * ((n + 2047) / 2048), C = (n + P - 1) / P;
    if (item >= 2 * C) return;
    const DecodeParams p = b_att_params(a, s);
    const Smem sm;
    const int g = item / C, c = item % C, t0 = c * P, np = min(t0 + P, n) - t0;
    if (P == 32)
        attention_unit32(p, sm, l, g, c, t0, np, 1u, false);
    else
        attention_unit_big(p, sm, l, g, c, t0, np, 1u, false);
}

// Head-pair combine of every sequence: blockIdx.x = sequence, blockIdx.y = head pair.  The
// Q8_K (ties to even) of the result is the o_proj input.
__global__ void __launch_bounds__(DEC_THREADS, 1) k_b_att_combine(const BStepArgs a, int l) {
    const DecodeParams p = b_att_params(a, blockIdx.x);
    const Smem sm;
    combine_pair(p, sm, l, blockIdx.y, 1u);
}

// h = silu(gate) * up (canon_silu_mul), Q8_K ties away, 24 blocks per sequence.
__global__ void __launch_bounds__(256) k_b_swiglu(const BStepArgs a) {
    const int s = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* y = a.y + static_cast<size_t>(s) * 2 * N_FF;
    for (int b = warp; b < N_FF / 256; b += 8) {
        float h[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = 256 * b + 8 * lane + k;
            h[k] = canon_silu_mul(y[i], y[N_FF + i]);
        }
        quant_block_warp<true>(h, a.aqs + (static_cast<size_t>(s) * B_NBA + b) * 256,
                               a.ad + static_cast<size_t>(s) * B_NBA + b, a.abs + (static_cast<size_t>(s) * B_NBA + b) * 16);
    }
}

// Greedy token per sequence over its logits (lowest index on ties; NaN never wins; a NaN
// logit 0 gives 0, like phase_lm); with `chain`, the token feeds the next step at pos + 1.
__global__ void __launch_bounds__(1024) k_b_argmax(const BStepArgs a, int chain) {
    __shared__ float bv[32];
    __shared__ int bi[32], bn[32];
    const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* lg = a.logits + static_cast<size_t>(s) * a.n_vocab;
    float best = -__int_as_float(0x7f800000);
    int besti = 0x7fffffff, nan0 = 0;
    for (int i = tid; i < a.n_vocab; i += blockDim.x) {
        const float v = lg[i];
        if (i == 0 && v != v) nan0 = 1;
        if (v > best || (v == best && i < besti)) best = v, besti = i;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ob > best || (ob == best && oi < besti)) best = ob, besti = oi;
    }
    nan0 = __any_sync(0xffffffffu, nan0);
    if (lane == 0) bv[warp] = best, bi[warp] = besti, bn[warp] = nan0;
    __syncthreads();
    if (tid == 0) {
        int anynan = 0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
            if (bv[w] > best || (bv[w] == best && bi[w] < besti)) best = bv[w], besti = bi[w];
            anynan |= bn[w];
        }
        const int r = (anynan || besti == 0x7fffffff) ? 0 : besti;
        a.argmax[s] = r;
        if (chain) {
            a.tokens[s] = r;
            a.pos[s] = a.pos[s] + 1;
        }
    }
}
