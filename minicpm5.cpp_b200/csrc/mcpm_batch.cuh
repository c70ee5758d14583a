// Batched decode (config 3): n_seq <= 64 independent sequences advance one token per step.
// Included by mcpm_decode.cu inside its anonymous namespace: the attention units, the
// head-pair combine, the Q8_K quantiser and the canonical exp / SiLU are the decode kernel's
// own device functions, so every sequence's logits equal a batch-1 decode of that sequence
// bit for bit (MiniCPM5Engine::forward, src/model.cpp:142-242, once per sequence).
//
// Activations between GEMMs are Q8_K blocks split into arrays per sequence: values
// [seq][B_NBA][256] int8 (stored lane-major by their producers, see below), scales
// [seq][B_NBA] fp32, block sums [seq][B_NBA][16] int16.
//
// GEMMs (k_b_gemm8 / k_b_gemm24): a tile is 16 weight rows x 64 sequences; warp w owns
// sequences 8w..8w+7.  Per 256-weight block the reference's AVX2 row kernel keeps eight int32 lane
// partials (ops_avx2.cpp:153-196 Q4_K, :201-276 Q6_K): lane k sums the elements 32s + 4k + t
// (s = 0..7 sub-blocks, t = 0..3) times their sub-block scale.  The block is staged with its
// K dimension permuted lane-major (position 32k + 4s + t), so lane k is the contiguous K range
// [32k, 32k+32): one m16n8k32 int8 MMA per lane.  The weight operand is w' = scale x q split
// as w' = 64*hi + lo (hi = w' >> 6, lo = w' & 63, both int8), so lane_k = 64*(hi.x) + (lo.x)
// exactly, from two MMAs.  The fp32 epilogue then runs the batch-1 GEMV's chain per (row,
// sequence): acc[k] = fma(xd*d, lane_k, acc[k]) over blocks, the fused min chain, and the
// hsum_f32_8 tree.

constexpr int B_NBA = N_FF / 256;          // activation blocks per sequence (24)
constexpr int BG_ROWS = 16;                // GEMM tile rows
constexpr int BG_SEQ = BATCH_MAX;          // GEMM tile sequences (64)
constexpr int BG_STRIDE = 272;             // smem bytes per staged 256-byte block row (+16: conflict-free fragments)
constexpr int BG_THREADS = 256;
constexpr int BG_WROW8 = 8 * Q6K_BYTES;    // smem bytes per staged weight row of an 8-block matrix
constexpr int BG_WROW24 = 24 * Q6K_BYTES;  // ... of a 24-block matrix

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
    unsigned* err;   // k_b_gemm_tc: ERR_TIMEOUT when an MMA completion never arrives
    float* part;     // k_b_gemm_tc: group partials, [tile][group][64][128] fp32
    unsigned* cnt;   // k_b_gemm_tc: one counter per row tile, zero between launches
    unsigned long long* trace;   // k_b_gemm_tc, optional: globaltimer marks of CTA 0's first unit
};

// k_b_gemm8 (8 blocks per row: QKV, o_proj, gate/up, LM head): the activations of every
// sequence stay resident; weight tiles are double-buffered.
constexpr int GA_X = 0;                                   // [8][64][272] activation values
constexpr int GA_XD = GA_X + 8 * BG_SEQ * BG_STRIDE;      // float [8][64] scales
constexpr int GA_XB = GA_XD + 8 * BG_SEQ * 4;             // int16 [8][64][16] block sums
constexpr int GA_W = GA_XB + 8 * BG_SEQ * 32;             // 2 x [16][BG_WROW8] raw weight rows
constexpr int GA_A = GA_W + 2 * BG_ROWS * BG_WROW8;       // hi [16][272], lo [16][272]
constexpr int GA_RM = GA_A + 2 * BG_ROWS * BG_STRIDE;     // d [16], dmin [16], mins / scales [16][16]
constexpr int GA_BYTES = GA_RM + BG_ROWS * (8 + 16);
// k_b_gemm24 (24 blocks per row: down): the tile's weight rows stay resident; activation
// blocks stream through a 3-slot ring.
constexpr int GB_W = 0;                                                // [16][BG_WROW24]
constexpr int GB_SLOT = BG_SEQ * BG_STRIDE + BG_SEQ * 4 + BG_SEQ * 32;   // values, scales, block sums
constexpr int GB_X = GB_W + BG_ROWS * BG_WROW24;
constexpr int GB_A = GB_X + 3 * GB_SLOT;
constexpr int GB_RM = GB_A + 2 * BG_ROWS * BG_STRIDE;
constexpr int GB_BYTES = GB_RM + BG_ROWS * (8 + 16);

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ BGemmSeg bg_seg(const BGemmArgs& a, int tile) {   // by value: no local copy of a.seg
    return (a.nseg > 2 && tile >= a.seg[2].tile0) ? a.seg[2] : (a.nseg > 1 && tile >= a.seg[1].tile0) ? a.seg[1] : a.seg[0];
}

// Activation block b of every sequence (already lane-major) -> xs [64][272], xd [64],
// xb [64][16]; zeros beyond n_seq.
__device__ void bg_stage_x(const BGemmArgs& a, int b, uint8_t* xs, float* xd, int16_t* xb) {
    const int tid = threadIdx.x;
    for (int i = tid; i < BG_SEQ * 16; i += BG_THREADS) {
        const int q = i >> 4, m = i & 15;
        uint8_t* dst = xs + q * BG_STRIDE + 16 * m;
        if (q < a.n_seq)
            cp_async16(dst, a.aqs + (static_cast<size_t>(q) * B_NBA + b) * 256 + 16 * m);
        else
            *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
    for (int i = tid; i < BG_SEQ * 2; i += BG_THREADS) {
        const int q = i >> 1, h = i & 1;
        int16_t* dst = xb + 16 * q + 8 * h;
        if (q < a.n_seq)
            cp_async16(dst, a.abs + (static_cast<size_t>(q) * B_NBA + b) * 16 + 8 * h);
        else
            *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
    if (tid < BG_SEQ) {
        if (tid < a.n_seq)
            cp_async4(xd + tid, a.ad + static_cast<size_t>(tid) * B_NBA + b);
        else
            xd[tid] = 0.0f;
    }
}

// Weight rows row0 .. row0+15 of a segment (all nb blocks) -> dst [16][wrow]; zeros past the end.
__device__ void bg_stage_w(const BGemmSeg& sg, int row0, int nb, uint8_t* dst, int wrow) {
    const int rb = row_bytes(sg.type, 256 * nb), nch = rb >> 4;
    for (int i = threadIdx.x; i < BG_ROWS * nch; i += BG_THREADS) {
        const int r = i / nch, c = i - r * nch;
        uint8_t* d = dst + r * wrow + 16 * c;
        if (row0 + r < sg.rows)
            cp_async16(d, sg.w + static_cast<size_t>(row0 + r) * rb + 16 * c);
        else
            *reinterpret_cast<uint4*>(d) = make_uint4(0u, 0u, 0u, 0u);
    }
}

// Block b of the staged rows -> the hi / lo int8 operands (lane-major) and the row metadata.
// Thread (r, s, half): row r, sub-block s, elements 16 half .. 16 half + 15 of it.  Four
// elements at a time in two words of 16-bit lanes (elements t, t+2 and t+1, t+3):
// w' = sc * q stays below 2^16 per lane (Q4_K: 63 * 15; Q6_K: W = q (sc + 128) + 8192 - 128 q,
// i.e. sc * q + 8192 in [128, 24257], so hi = (W >> 6) - 128 and lo = W & 63 exactly).
__device__ __forceinline__ void bg_pack(uint32_t wa, uint32_t wb, int bias_hi, uint32_t& h4, uint32_t& l4) {
    // wa: elements 0 / 2, wb: 1 / 3 (16-bit lanes) -> bytes 0..3
    uint32_t ha = (wa >> 6) & 0x00ff00ffu, hb = (wb >> 6) & 0x00ff00ffu;
    if (bias_hi) ha ^= 0x00800080u, hb ^= 0x00800080u;
    h4 = __byte_perm(ha, hb, 0x6240);
    l4 = __byte_perm(wa & 0x003f003fu, wb & 0x003f003fu, 0x6240);
}

template <int TYPE>
__device__ __forceinline__ void bg_dequant(const uint8_t* w, int wrow, int b, uint8_t* ahi, uint8_t* alo, uint8_t* rm) {
    const int tid = threadIdx.x, r = tid >> 4, s = (tid >> 1) & 7, half = tid & 1;
    uint32_t hw[4], lw[4];
    if (TYPE == GGML_Q4_K) {
        const uint8_t* blk = w + r * wrow + b * Q4K_BYTES;
        const uint4 head = *reinterpret_cast<const uint4*>(blk);   // d, dmin, 12 packed scale bytes
        const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (s >> 1) + 16 * half);
        auto sc8 = [&](int i) -> int {   // byte i of the packed scales, selected without register indexing
            const uint32_t wd = i < 4 ? head.y : i < 8 ? head.z : head.w;
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
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t nib = (s & 1) ? (qw[kk] >> 4) & 0x0f0f0f0fu : qw[kk] & 0x0f0f0f0fu;
            const uint32_t wa = __byte_perm(nib, 0u, 0x4240) * static_cast<uint32_t>(sc);
            const uint32_t wb = __byte_perm(nib, 0u, 0x4341) * static_cast<uint32_t>(sc);
            bg_pack(wa, wb, 0, hw[kk], lw[kk]);
        }
        if (half == 0)   // min m[s] twice in a 16-bit word (dp2a operand)
            reinterpret_cast<uint16_t*>(rm + 8 * BG_ROWS)[8 * r + s] = static_cast<uint16_t>(mn * 0x0101);
        if (s == 0 && half == 0) {
            reinterpret_cast<float*>(rm)[r] = h2f(head.x);
            reinterpret_cast<float*>(rm)[BG_ROWS + r] = h2f(head.x >> 16);
        }
    } else {   // Q6_K: 210-byte blocks, 2-byte aligned
        const uint8_t* blk = w + r * wrow + b * Q6K_BYTES;
        const int h = s >> 2, kk6 = s & 3;
        const uint16_t* ql = reinterpret_cast<const uint16_t*>(blk + 64 * h + 32 * (kk6 & 1) + 16 * half);
        const uint16_t* qh = reinterpret_cast<const uint16_t*>(blk + 128 + 32 * h + 16 * half);
        const int scale = static_cast<int8_t>(blk[192 + 2 * s + half]);
        const uint32_t sc1 = static_cast<uint32_t>(scale + 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t lq = static_cast<uint32_t>(ql[2 * kk]) | (static_cast<uint32_t>(ql[2 * kk + 1]) << 16);
            const uint32_t hq = static_cast<uint32_t>(qh[2 * kk]) | (static_cast<uint32_t>(qh[2 * kk + 1]) << 16);
            const uint32_t lo4 = (kk6 & 2) ? (lq >> 4) & 0x0f0f0f0fu : lq & 0x0f0f0f0fu;
            const uint32_t q6 = lo4 | (((hq >> (2 * kk6)) & 0x03030303u) << 4);   // four values 0..63
            const uint32_t qa = __byte_perm(q6, 0u, 0x4240), qb = __byte_perm(q6, 0u, 0x4341);
            const uint32_t wa = qa * sc1 + 0x20002000u - (qa << 7), wb = qb * sc1 + 0x20002000u - (qb << 7);
            bg_pack(wa, wb, 1, hw[kk], lw[kk]);
        }
        reinterpret_cast<int8_t*>(rm + 8 * BG_ROWS)[16 * r + 2 * s + half] = static_cast<int8_t>(scale);
        if (s == 0 && half == 0) reinterpret_cast<float*>(rm)[r] = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {   // lane k = 4 half + kk, permuted position 32k + 4s
        const int k = 4 * half + kk;
        *reinterpret_cast<uint32_t*>(ahi + r * BG_STRIDE + 32 * k + 4 * s) = hw[kk];
        *reinterpret_cast<uint32_t*>(alo + r * BG_STRIDE + 32 * k + 4 * s) = lw[kk];
    }
}

// signed dp2a: two int16 of a times the low / high two int8 of b, plus c
__device__ __forceinline__ int dp2lo(uint32_t a, uint32_t b, int c) {
    return __dp2a_lo(static_cast<int>(a), static_cast<int>(b), c);
}
__device__ __forceinline__ int dp2hi(uint32_t a, uint32_t b, int c) {
    return __dp2a_hi(static_cast<int>(a), static_cast<int>(b), c);
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}

// One block: two MMAs per AVX2 lane and the batch-1 GEMV's fp32 chains for this thread's
// four (row, sequence) pairs: rows g, g+8 x sequences 8w + 2t, 8w + 2t + 1.  Fragments come
// from ldmatrix (int8 m16n8k32 operands have the b16 8x8 layout); the Q6_K lane offset and
// the Q4_K min sum are dp2a dot products of block-sum pairs with scale bytes.
template <int TYPE>
__device__ __forceinline__ void bg_block(const uint8_t* xs, const float* xd, const int16_t* xb, const uint8_t* ahi,
                                         const uint8_t* alo, const uint8_t* rm, float (&acc)[4][8], float (&acc_min)[4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int q0 = 8 * warp + 2 * t;
    const float* rd = reinterpret_cast<const float*>(rm);
    const float xd0 = xd[q0], xd1 = xd[q0 + 1];
    const float d0 = rd[g], d1 = rd[g + 8];
    const float ds[4] = {__fmul_rn(xd0, d0), __fmul_rn(xd1, d0), __fmul_rn(xd0, d1), __fmul_rn(xd1, d1)};
    // block sums of the two sequences as int16 pairs: word k = (bsums[2k], bsums[2k+1])
    const uint4 b0a = *reinterpret_cast<const uint4*>(xb + 16 * q0), b0b = *reinterpret_cast<const uint4*>(xb + 16 * q0 + 8);
    const uint4 b1a = *reinterpret_cast<const uint4*>(xb + 16 * (q0 + 1)),
                b1b = *reinterpret_cast<const uint4*>(xb + 16 * (q0 + 1) + 8);
    const uint32_t bw0[8] = {b0a.x, b0a.y, b0a.z, b0a.w, b0b.x, b0b.y, b0b.z, b0b.w};
    const uint32_t bw1[8] = {b1a.x, b1a.y, b1a.z, b1a.w, b1b.x, b1b.y, b1b.z, b1b.w};
    const uint4 sr0 = *reinterpret_cast<const uint4*>(rm + 8 * BG_ROWS + 16 * g);        // row g: Q6_K scales /
    const uint4 sr1 = *reinterpret_cast<const uint4*>(rm + 8 * BG_ROWS + 16 * (g + 8));  // Q4_K doubled mins
    const uint32_t sw0[4] = {sr0.x, sr0.y, sr0.z, sr0.w}, sw1[4] = {sr1.x, sr1.y, sr1.z, sr1.w};
    if (TYPE == GGML_Q4_K) {   // minsum = sum_g mins[g] * (bsums[2g] + bsums[2g+1])
        int ms[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ms[0] = dp2hi(bw0[2 * j + 1], sw0[j], dp2lo(bw0[2 * j], sw0[j], ms[0]));
            ms[1] = dp2hi(bw1[2 * j + 1], sw0[j], dp2lo(bw1[2 * j], sw0[j], ms[1]));
            ms[2] = dp2hi(bw0[2 * j + 1], sw1[j], dp2lo(bw0[2 * j], sw1[j], ms[2]));
            ms[3] = dp2hi(bw1[2 * j + 1], sw1[j], dp2lo(bw1[2 * j], sw1[j], ms[3]));
        }
        const float m0 = rd[BG_ROWS + g], m1 = rd[BG_ROWS + g + 8];
        const float dm[4] = {-__fmul_rn(xd0, m0), -__fmul_rn(xd1, m0), -__fmul_rn(xd0, m1), -__fmul_rn(xd1, m1)};
#pragma unroll
        for (int e = 0; e < 4; ++e) acc_min[e] = __fmaf_rn(dm[e], __int2float_rn(ms[e]), acc_min[e]);
    }
    // ldmatrix row addresses: A rows (lane & 7) + 8 ((lane >> 3) & 1), K half lane >> 4;
    // B sequence rows lane & 7, K half (lane >> 3) & 1
    const int ar = (lane & 7) + 8 * ((lane >> 3) & 1), ak = 16 * (lane >> 4);
    const uint8_t* pah = ahi + ar * BG_STRIDE + ak;
    const uint8_t* pal = alo + ar * BG_STRIDE + ak;
    const uint8_t* pb = xs + (8 * warp + (lane & 7)) * BG_STRIDE + 16 * ((lane >> 3) & 1);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t fh[4], fl[4], fb[2];
        ldsm_x4(fh, pah + 32 * k);
        ldsm_x4(fl, pal + 32 * k);
        ldsm_x2(fb, pb + 32 * k);
        int ch[4], cl[4];
        mma_s8(ch, fh, fb);
        mma_s8(cl, fl, fb);
        int lv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) lv[e] = ch[e] * 64 + cl[e];
        if (TYPE == GGML_Q6_K) {   // -32 * (bsums[2k] * sc[2k] + bsums[2k+1] * sc[2k+1])
            const uint32_t s0 = sw0[k >> 1], s1 = sw1[k >> 1];
            if (k & 1) {
                lv[0] -= 32 * dp2hi(bw0[k], s0, 0), lv[1] -= 32 * dp2hi(bw1[k], s0, 0);
                lv[2] -= 32 * dp2hi(bw0[k], s1, 0), lv[3] -= 32 * dp2hi(bw1[k], s1, 0);
            } else {
                lv[0] -= 32 * dp2lo(bw0[k], s0, 0), lv[1] -= 32 * dp2lo(bw1[k], s0, 0);
                lv[2] -= 32 * dp2lo(bw0[k], s1, 0), lv[3] -= 32 * dp2lo(bw1[k], s1, 0);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e][k] = __fmaf_rn(ds[e], __int2float_rn(lv[e]), acc[e][k]);
    }
}

template <int TYPE>
__device__ __forceinline__ void bg_store_out(const BGemmArgs& a, const BGemmSeg& sg, int row0, const float (&acc)[4][8],
                                             const float (&acc_min)[4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
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

template <int TYPE, int NB>
__device__ void bg_tile(const BGemmArgs& a, const BGemmSeg& sg, int row0, const uint8_t* w, int wrow, uint8_t* xs0,
                        int xs_step, float* xd0, int16_t* xb0, uint8_t* sm_a, uint8_t* rm, bool ring) {
    const bool active = 8 * (threadIdx.x >> 5) < a.n_seq;   // warp-uniform
    float acc[4][8], acc_min[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        acc_min[e] = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[e][k] = 0.0f;
    }
    for (int b = 0; b < NB; ++b) {
        const int slot = ring ? b % 3 : b;
        if (ring) {   // block b's activations are the oldest group but one in flight
            cp_async_wait_group<1>();
            __syncthreads();
        }
        bg_dequant<TYPE>(w, wrow, b, sm_a, sm_a + BG_ROWS * BG_STRIDE, rm);
        __syncthreads();
        if (active)
            bg_block<TYPE>(xs0 + slot * xs_step, xd0 + slot * (ring ? GB_SLOT / 4 : BG_SEQ),
                           reinterpret_cast<const int16_t*>(reinterpret_cast<const uint8_t*>(xb0) + slot * (ring ? GB_SLOT : BG_SEQ * 32)),
                           sm_a, sm_a + BG_ROWS * BG_STRIDE, rm, acc, acc_min);
        __syncthreads();
        if (ring) {   // block b+2 into the slot block b-1 used
            if (b + 2 < NB) {
                uint8_t* sl = xs0 + ((b + 2) % 3) * xs_step;
                bg_stage_x(a, b + 2, sl, reinterpret_cast<float*>(sl + BG_SEQ * BG_STRIDE),
                           reinterpret_cast<int16_t*>(sl + BG_SEQ * BG_STRIDE + BG_SEQ * 4));
            }
            cp_async_commit();
        }
    }
    if (active) bg_store_out<TYPE>(a, sg, row0, acc, acc_min);
}

__global__ void __launch_bounds__(BG_THREADS, 1) k_b_gemm8(const BGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smg[];
    for (int b = 0; b < 8; ++b)
        bg_stage_x(a, b, smg + GA_X + b * BG_SEQ * BG_STRIDE, reinterpret_cast<float*>(smg + GA_XD) + b * BG_SEQ,
                   reinterpret_cast<int16_t*>(smg + GA_XB) + b * BG_SEQ * 16);
    cp_async_commit();
    int tile = blockIdx.x;
    if (tile < a.ntiles) {
        const BGemmSeg sg = bg_seg(a, tile);
        bg_stage_w(sg, (tile - sg.tile0) * BG_ROWS, 8, smg + GA_W, BG_WROW8);
    }
    cp_async_commit();
    for (int it = 0; tile < a.ntiles; tile += gridDim.x, ++it) {
        const int nxt = tile + gridDim.x;
        if (nxt < a.ntiles) {   // next tile's rows into the other buffer (read last by tile it-1)
            const BGemmSeg sn = bg_seg(a, nxt);
            bg_stage_w(sn, (nxt - sn.tile0) * BG_ROWS, 8, smg + GA_W + ((it + 1) & 1) * BG_ROWS * BG_WROW8, BG_WROW8);
        }
        cp_async_commit();
        cp_async_wait_group<1>();   // activations and this tile's rows landed
        __syncthreads();
        const BGemmSeg sg = bg_seg(a, tile);
        const int row0 = (tile - sg.tile0) * BG_ROWS;
        const uint8_t* w = smg + GA_W + (it & 1) * BG_ROWS * BG_WROW8;
        if (sg.type == GGML_Q4_K)
            bg_tile<GGML_Q4_K, 8>(a, sg, row0, w, BG_WROW8, smg + GA_X, BG_SEQ * BG_STRIDE,
                                  reinterpret_cast<float*>(smg + GA_XD), reinterpret_cast<int16_t*>(smg + GA_XB),
                                  smg + GA_A, smg + GA_RM, false);
        else
            bg_tile<GGML_Q6_K, 8>(a, sg, row0, w, BG_WROW8, smg + GA_X, BG_SEQ * BG_STRIDE,
                                  reinterpret_cast<float*>(smg + GA_XD), reinterpret_cast<int16_t*>(smg + GA_XB),
                                  smg + GA_A, smg + GA_RM, false);
    }
    cp_async_wait_all();
}

__global__ void __launch_bounds__(BG_THREADS, 1) k_b_gemm24(const BGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smg[];
    for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
        const BGemmSeg sg = bg_seg(a, tile);
        const int row0 = (tile - sg.tile0) * BG_ROWS;
        bg_stage_w(sg, row0, 24, smg + GB_W, BG_WROW24);
        cp_async_commit();
        for (int b = 0; b < 2; ++b) {
            uint8_t* sl = smg + GB_X + b * GB_SLOT;
            bg_stage_x(a, b, sl, reinterpret_cast<float*>(sl + BG_SEQ * BG_STRIDE),
                       reinterpret_cast<int16_t*>(sl + BG_SEQ * BG_STRIDE + BG_SEQ * 4));
            cp_async_commit();
        }
        if (sg.type == GGML_Q4_K)
            bg_tile<GGML_Q4_K, 24>(a, sg, row0, smg + GB_W, BG_WROW24, smg + GB_X, GB_SLOT,
                                   reinterpret_cast<float*>(smg + GB_X + BG_SEQ * BG_STRIDE),
                                   reinterpret_cast<int16_t*>(smg + GB_X + BG_SEQ * BG_STRIDE + BG_SEQ * 4), smg + GB_A,
                                   smg + GB_RM, true);
        else
            bg_tile<GGML_Q6_K, 24>(a, sg, row0, smg + GB_W, BG_WROW24, smg + GB_X, GB_SLOT,
                                   reinterpret_cast<float*>(smg + GB_X + BG_SEQ * BG_STRIDE),
                                   reinterpret_cast<int16_t*>(smg + GB_X + BG_SEQ * BG_STRIDE + BG_SEQ * 4), smg + GB_A,
                                   smg + GB_RM, true);
        cp_async_wait_all();
        __syncthreads();
    }
}

#include "mcpm_batch_tc.cuh"

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
    quant_block_warp<AWAY, true>(y, qs + 256 * warp, d + warp, bs + 16 * warp);
    __syncthreads();
}

struct BStepArgs {
    int n_seq, max_seq, n_layer;
    size_t kv_seq_stride;   // floats between two rows' caches; 0: every row one sequence's cache (prefill)
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
    return static_cast<size_t>(s) * a.kv_seq_stride + static_cast<size_t>(l) * a.max_seq * KV_DIM;
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
    float xv[8], yv[8];   // every load before any store (x and y could alias for the compiler)
#pragma unroll
    for (int k = 0; k < 8; ++k) xv[k] = __ldcg(x + threadIdx.x + 256 * k), yv[k] = __ldcg(y + threadIdx.x + 256 * k);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float v = __fadd_rn(xv[k], yv[k]);
        x[threadIdx.x + 256 * k] = v;
        xs[threadIdx.x + 256 * k] = v;
    }
    __syncthreads();
    b_norm_quant<AWAY>(xs, a.norm, a.aqs + static_cast<size_t>(s) * B_NBA * 256, a.ad + static_cast<size_t>(s) * B_NBA,
                       a.abs + static_cast<size_t>(s) * B_NBA * 16);
}

// RoPE on q and k (interleaved pairs, as in phase_qkv), q to its buffer, K/V into the
// sequence's cache at its position.
template <typename KT>
__global__ void __launch_bounds__(256) k_b_rope_kv(const BStepArgs a, int l) {
    const int s = blockIdx.x, pos = a.pos[s];
    const float* y = a.y + static_cast<size_t>(s) * 2 * N_FF;
    KT* kdst = reinterpret_cast<KT*>(a.kc) + b_kv_off(a, s, l) + static_cast<size_t>(pos) * KV_DIM;
    KT* vdst = reinterpret_cast<KT*>(a.vc) + b_kv_off(a, s, l) + static_cast<size_t>(pos) * KV_DIM;
    constexpr int NPAIR = (N_EMBD + 2 * KV_DIM) / 2, PER = NPAIR / 256;   // 5 pairs per thread
    static_assert(NPAIR % 256 == 0, "pairs per thread");
    float2 vv[PER], cc[PER];   // every load before any store
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int R = 2 * (threadIdx.x + 256 * j);
        vv[j] = __ldcg(reinterpret_cast<const float2*>(y + R));
        cc[j] = __ldg(a.rope + static_cast<size_t>(pos) * (HEAD_DIM / 2) + ((R & (HEAD_DIM - 1)) >> 1));
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int R = 2 * (threadIdx.x + 256 * j);
        const float v0 = vv[j].x, v1 = vv[j].y;
        if (R < N_EMBD + KV_DIM) {
            const float2 c = cc[j];
            const float r0 = __fmaf_rn(c.x, v0, -__fmul_rn(c.y, v1));
            const float r1 = __fmaf_rn(c.y, v0, __fmul_rn(c.x, v1));
            if (R < N_EMBD) {
                a.q[static_cast<size_t>(s) * N_EMBD + R] = r0;
                a.q[static_cast<size_t>(s) * N_EMBD + R + 1] = r1;
            } else {
                kdst[R - N_EMBD] = KvElt<KT>::put(r0);
                kdst[R - N_EMBD + 1] = KvElt<KT>::put(r1);
            }
        } else {
            vdst[R - N_EMBD - KV_DIM] = KvElt<KT>::put(v0);
            vdst[R - N_EMBD - KV_DIM + 1] = KvElt<KT>::put(v1);
        }
    }
}

template <typename KT>
__device__ DecodeParams b_att_params(const BStepArgs& a, int s) {
    DecodeParams p{};
    p.q = a.q + static_cast<size_t>(s) * N_EMBD;
    p.kc = reinterpret_cast<float*>(reinterpret_cast<KT*>(a.kc) + b_kv_off(a, s, 0));
    p.vc = reinterpret_cast<float*>(reinterpret_cast<KT*>(a.vc) + b_kv_off(a, s, 0));
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
// Two CTAs per SM (64 registers, no spills; shared memory 2 x 24 KB, or 2 x 96 KB for chunks
// longer than 32): thousands of short units, so the second CTA hides the first one's loads.
template <typename KT>
__global__ void __launch_bounds__(DEC_THREADS, 2) k_b_att_units(const BStepArgs a, int l) {
    const int s = blockIdx.x, item = blockIdx.y;
    const int n = a.pos[s] + 1, P = 32 * ((n + 2047) / 2048), C = (n + P - 1) / P;
    if (item >= 2 * C) return;
    const DecodeParams p = b_att_params<KT>(a, s);
    const Smem sm;
    const int g = item / C, c = item % C, t0 = c * P, np = min(t0 + P, n) - t0;
    if (P == 32)
        attention_unit32<KT>(p, reinterpret_cast<float*>(sm.wbuf(0)), l, g, c, t0, np, 1u, false);
    else
        attention_unit_big<KT>(p, reinterpret_cast<float*>(sm.wbuf(0)), l, g, c, t0, np, 1u, false);
}

// Head-pair combine of every sequence: blockIdx.x = sequence, blockIdx.y = head pair.  The
// Q8_K (ties to even) of the result is the o_proj input.
__global__ void __launch_bounds__(DEC_THREADS, 1) k_b_att_combine(const BStepArgs a, int l) {
    const DecodeParams p = b_att_params<float>(a, blockIdx.x);   // the combine reads no cache row
    const Smem sm;
    combine_pair(p, reinterpret_cast<float*>(sm.wbuf(0)), l, blockIdx.y, 1u);
}

// h = silu(gate) * up (canon_silu_mul), Q8_K ties away: one warp per 256-element block
// (blockIdx.y selects blocks 8y .. 8y+7 of sequence blockIdx.x).
__global__ void __launch_bounds__(256) k_b_swiglu(const BStepArgs a) {
    const int s = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, b = 8 * blockIdx.y + warp;
    const float* y = a.y + static_cast<size_t>(s) * 2 * N_FF + 256 * b + 8 * lane;
    const float4 g0 = __ldcg(reinterpret_cast<const float4*>(y)), g1 = __ldcg(reinterpret_cast<const float4*>(y + 4));
    const float4 u0 = __ldcg(reinterpret_cast<const float4*>(y + N_FF)),
                 u1 = __ldcg(reinterpret_cast<const float4*>(y + N_FF + 4));
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float h[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] = canon_silu_mul(g[k], u[k]);
    quant_block_warp<true, true>(h, a.aqs + (static_cast<size_t>(s) * B_NBA + b) * 256, a.ad + static_cast<size_t>(s) * B_NBA + b,
                           a.abs + (static_cast<size_t>(s) * B_NBA + b) * 16);
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
