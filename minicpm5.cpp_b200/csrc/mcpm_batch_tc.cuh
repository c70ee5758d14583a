// Batched GEMM on the 5th-generation tensor cores (mcpm_config::batch_gemm = MCPM_GEMM_TCGEN05,
// the default for batched decode and prompt prefill).  Included by mcpm_decode.cu after
// mcpm_batch.cuh, inside its anonymous namespace.
//
// Products (the reference's K-quant dot, ops_avx2.cpp:153-276, per 256-weight block): the
// block's integer sum is exact on the tensor cores and the fp32 scaling is one FMA per
// (row, sequence, block):
//   isum = sum over the 256 elements of w' * x, w' = sub-block scale * q (Q4_K) or
//          scale * (q - 32) (Q6_K; the -32 enters as -32 * sum_s scale_s * bsums_s)
//   acc  = fma(xd * d, (float) isum, acc)                      over the blocks of a group
//   accm = fma(-(xd * dmin), (float) minsum, accm)             (Q4_K)
//   g    = acc + accm (Q4_K) or acc (Q6_K)
//   y    = ((g_0 + g_1) + g_2) + ...                          over the groups in order
// with groups of TB_G = 4 consecutive blocks (2 groups for 2048-wide rows, 6 for 6144).  This
// is the batched path's own canonical order (restated as ORC_ORDER_BATCH in the C
// restatement): its integer block sums equal the reference's, its fp32 rounding differs from
// the batch-1 eight-lane chains by a few ulps.
//
// Tile: 128 weight rows x 64 sequences x one group.  Per block the CTA dequantises the rows
// into two int8 operands w' = 64 * hi + lo (hi, lo in int8: tc_dequant's arithmetic), one
// thread issues 16 tcgen05.mma (kind::i8, M = 128, N = 64, K = 32; the eight K = 32 slices of
// the block accumulate into one int32 accumulator for hi and one for lo), and the epilogue of
// the previous block (tcgen05.ld of its accumulators, the other TMEM buffer) runs while the
// MMAs execute.  The groups of a row tile run on different CTAs: each writes its g to a
// scratch buffer, and the last to finish (a per-tile counter) adds the groups in order and
// stores y.
constexpr int TB_M = 128, TB_N = 64, TB_THREADS = 512, TB_G = 4, TB_COLS = 256;
constexpr int TB_A_LBO = (TB_M / 8) * 128;                // K-half stride of a weight operand (2048 B)
constexpr int TB_B_LBO = (TB_N / 8) * 128;                // K-half stride of the activation operand (1024 B)
constexpr int TB_AHI = 0;                                 // [16 K-halves][16 row groups][8][16] int8
constexpr int TB_ALO = TB_AHI + 16 * TB_A_LBO;
constexpr int TB_BX = TB_ALO + 16 * TB_A_LBO;             // 2 x [16 K-halves][8 seq groups][8][16] int8
constexpr int TB_XD = TB_BX + 2 * 16 * TB_B_LBO;          // 3 x float [64]
constexpr int TB_XB = TB_XD + 3 * TB_N * 4;               // 3 x int16 [64][16]
constexpr int TB_RM_BYTES = TB_M * 8 + TB_M * 16;         // float d [128], dmin [128]; 16 B of mins / scales per row
constexpr int TB_RM = TB_XB + 3 * TB_N * 32;              // 2 x row metadata
constexpr int TB_RAW_STRIDE = 432;                        // bytes per row of a staged block pair (>= 2 x 210, 16 | 432)
constexpr int TB_RAW = TB_RM + 2 * TB_RM_BYTES;           // 2 x [128 rows][TB_RAW_STRIDE]: the group's two block pairs
constexpr int TB_BAR = TB_RAW + 2 * TB_M * TB_RAW_STRIDE; // mbarrier, TMEM base address, last-CTA flag
constexpr int TB_BYTES = TB_BAR + 16;
// instruction descriptor: S32 accumulator, S8 x S8, both K-major, N = 64, M = 128
constexpr uint32_t TB_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(TB_N >> 3) << 17) |
                              (static_cast<uint32_t>(TB_M >> 4) << 24);
static_assert(TB_BYTES <= 232448 && TB_BX % 1024 == 0 && TB_RM % 16 == 0 && TB_RAW % 16 == 0 && TB_BAR % 8 == 0,
              "k_b_gemm_tc layout");
static_assert(BATCH_MAX <= TB_N, "one sequence tile holds every sequence of a batch");

// Scratch of the group partials: [tile][group][64 sequences][128 rows] fp32, and one
// counter per row tile (zero between launches: the last CTA of a tile resets it).
__host__ __device__ constexpr size_t tb_scratch_floats(int ntiles, int ngroups) {
    return static_cast<size_t>(ntiles) * ngroups * TB_N * TB_M;
}

__device__ __forceinline__ uint64_t tc_desc(const void* p, uint32_t lbo, uint32_t sbo) {   // SWIZZLE_NONE, version 1
    return static_cast<uint64_t>((smem_u32(p) & 0x3ffffu) >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16) |
           (static_cast<uint64_t>(sbo >> 4) << 32) | (1ull << 46);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D (+)= A x B; `accumulate` 0 overwrites the accumulator
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Activation block b of sequences 0..63 -> operand buffer b & 1 (K-major core matrices; the
// values are already lane-major), scales and block sums -> slot b % 3; zeros beyond n_seq.
__device__ void tb_stage_x(const BGemmArgs& a, int b, uint8_t* smt) {
    const int tid = threadIdx.x;
    uint8_t* bx = smt + TB_BX + (b & 1) * 16 * TB_B_LBO;
#pragma unroll
    for (int i = 0; i < 2; ++i) {   // 64 sequences x 16 chunks: two per thread
        const int t = tid + TB_THREADS * i, q = t >> 4, c = t & 15;
        uint8_t* dst = bx + c * TB_B_LBO + (q >> 3) * 128 + (q & 7) * 16;
        if (q < a.n_seq)
            cp_async16(dst, a.aqs + (static_cast<size_t>(q) * B_NBA + b) * 256 + 16 * c);
        else
            *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
    const int slot = b % 3;
    if (tid < 2 * TB_N) {
        const int q = tid >> 1, h = tid & 1;
        int16_t* dst = reinterpret_cast<int16_t*>(smt + TB_XB + slot * TB_N * 32) + 16 * q + 8 * h;
        if (q < a.n_seq)
            cp_async16(dst, a.abs + (static_cast<size_t>(q) * B_NBA + b) * 16 + 8 * h);
        else
            *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    } else if (tid < 3 * TB_N) {
        const int q = tid - 2 * TB_N;
        float* dst = reinterpret_cast<float*>(smt + TB_XD + slot * TB_N * 4) + q;
        if (q < a.n_seq)
            cp_async4(dst, a.ad + static_cast<size_t>(q) * B_NBA + b);
        else
            *dst = 0.0f;
    }
}

// Blocks 2p, 2p+1 of rows row0 .. row0+127 -> raw buffer `buf` (Q4_K: 288 B per row in 16-byte
// copies; Q6_K: 420 B per row, 4-byte copies).  Rows past the segment are skipped.
template <int TYPE>
__device__ __forceinline__ void tb_stage_raw(const BGemmSeg& sg, int row0, int nb, int p, int buf, uint8_t* smt) {
    constexpr int BYTES = TYPE == GGML_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    const size_t rb = static_cast<size_t>(nb) * BYTES;
    uint8_t* dst0 = smt + TB_RAW + buf * TB_M * TB_RAW_STRIDE;
    const int nr = min(TB_M, sg.rows - row0);
    if (TYPE == GGML_Q4_K) {
        constexpr int NCH = 2 * BYTES / 16;   // 18
        for (int i = threadIdx.x; i < nr * NCH; i += TB_THREADS) {
            const int r = i / NCH, c = i - r * NCH;
            cp_async16(dst0 + r * TB_RAW_STRIDE + 16 * c,
                       sg.w + static_cast<size_t>(row0 + r) * rb + static_cast<size_t>(p) * 2 * BYTES + 16 * c);
        }
    } else {
        constexpr int NCH = 2 * BYTES / 4;    // 105
        for (int i = threadIdx.x; i < nr * NCH; i += TB_THREADS) {
            const int r = i / NCH, c = i - r * NCH;
            cp_async4(dst0 + r * TB_RAW_STRIDE + 4 * c,
                      sg.w + static_cast<size_t>(row0 + r) * rb + static_cast<size_t>(p) * 2 * BYTES + 4 * c);
        }
    }
}

// Block b of the staged rows (raw buffer (b >> 1) & 1: the group's first or second pair) ->
// the hi / lo int8 operands (lane-major K, bg_dequant's arithmetic) and row metadata buffer
// b & 1.  Task (r, s, half): row r, sub-block s, elements 16 half .. 16 half + 15.  Rows past
// the segment are left stale: their outputs are never stored.
template <int TYPE>
__device__ __forceinline__ void tb_dequant(const BGemmSeg& sg, int row0, int b, uint8_t* smt) {
    constexpr int BYTES = TYPE == GGML_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    const uint8_t* raw = smt + TB_RAW + ((b >> 1) & 1) * TB_M * TB_RAW_STRIDE + (b & 1) * BYTES;
    uint8_t* rm = smt + TB_RM + (b & 1) * TB_RM_BYTES;
    float* rd = reinterpret_cast<float*>(rm);
    uint8_t* rms = rm + 8 * TB_M;
#pragma unroll 1
    for (int task = threadIdx.x; task < TB_M * 16; task += TB_THREADS) {
        const int r = task >> 4, s = (task >> 1) & 7, half = task & 1;
        if (row0 + r >= sg.rows) continue;
        const uint8_t* blk = raw + r * TB_RAW_STRIDE;
        uint32_t hw[4], lw[4];
        if (TYPE == GGML_Q4_K) {
            const uint4 head = *reinterpret_cast<const uint4*>(blk);   // d, dmin, 12 packed scale bytes
            const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (s >> 1) + 16 * half);
            auto sc8 = [&](int i) -> int {
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
            if (half == 0) reinterpret_cast<uint16_t*>(rms + 16 * r)[s] = static_cast<uint16_t>(mn * 0x0101);
            if (s == 0 && half == 0) {
                rd[r] = h2f(head.x);
                rd[TB_M + r] = h2f(head.x >> 16);
            }
        } else {
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
                const uint32_t q6 = lo4 | (((hq >> (2 * kk6)) & 0x03030303u) << 4);
                const uint32_t qa = __byte_perm(q6, 0u, 0x4240), qb = __byte_perm(q6, 0u, 0x4341);
                const uint32_t wa = qa * sc1 + 0x20002000u - (qa << 7), wb = qb * sc1 + 0x20002000u - (qb << 7);
                bg_pack(wa, wb, 1, hw[kk], lw[kk]);
            }
            reinterpret_cast<int8_t*>(rms + 16 * r)[2 * s + half] = static_cast<int8_t>(scale);
            if (s == 0 && half == 0) rd[r] = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {   // lane k = 4 half + kk: K bytes 32k + 4s .. +3 -> K-half 2k + (s >> 2)
            const int k = 4 * half + kk;
            const int off = (2 * k + (s >> 2)) * TB_A_LBO + (r >> 3) * 128 + (r & 7) * 16 + 4 * (s & 3);
            *reinterpret_cast<uint32_t*>(smt + TB_AHI + off) = hw[kk];
            *reinterpret_cast<uint32_t*>(smt + TB_ALO + off) = lw[kk];
        }
    }
}

// Epilogue of block b for this thread's row (TMEM lane) and its 16 sequences: the block's
// integer sums from the two accumulators of TMEM buffer b & 1, then the fp32 chains.
template <int TYPE>
__device__ __forceinline__ void tb_epilogue(const uint8_t* smt, uint32_t tmem, int b, int re, int qd, int part,
                                            float (&acc)[16], float (&accm)[16]) {
    const uint8_t* rm = smt + TB_RM + (b & 1) * TB_RM_BYTES;
    const float* rd = reinterpret_cast<const float*>(rm);
    const uint4 mw = *reinterpret_cast<const uint4*>(rm + 8 * TB_M + 16 * re);
    const uint32_t msw[4] = {mw.x, mw.y, mw.z, mw.w};
    const int slot = b % 3;
    const float* xd = reinterpret_cast<const float*>(smt + TB_XD + slot * TB_N * 4) + 16 * part;
    const uint4* xb = reinterpret_cast<const uint4*>(smt + TB_XB + slot * TB_N * 32) + 2 * 16 * part;
    const float d = rd[re], dmin = TYPE == GGML_Q4_K ? rd[TB_M + re] : 0.0f;
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * qd) << 16) + (b & 1) * 128 + 16 * part;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t hv[8], lv[8];
        tc_ld8(tl + 8 * h, hv);
        tc_ld8(tl + 64 + 8 * h, lv);
        tc_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            const int j = 8 * h + jj;
            const uint4 b0 = xb[2 * j], b1 = xb[2 * j + 1];   // bsums pairs (0,1) .. (14,15)
            const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            int v = static_cast<int>(hv[jj]) * 64 + static_cast<int>(lv[jj]);
            const float xdj = xd[j];
            if (TYPE == GGML_Q4_K) {   // minsum = sum_g mins[g] * (bsums[2g] + bsums[2g+1])
                int ms = 0;
#pragma unroll
                for (int g = 0; g < 4; ++g) ms = dp2hi(bw[2 * g + 1], msw[g], dp2lo(bw[2 * g], msw[g], ms));
                accm[j] = __fmaf_rn(-__fmul_rn(xdj, dmin), __int2float_rn(ms), accm[j]);
            } else {   // -32 * sum_s scale_s * bsums_s
                int o = 0;
#pragma unroll
                for (int w = 0; w < 8; ++w) o = (w & 1) ? dp2hi(bw[w], msw[w >> 1], o) : dp2lo(bw[w], msw[w >> 1], o);
                v -= 32 * o;
            }
            acc[j] = __fmaf_rn(__fmul_rn(xdj, d), __int2float_rn(v), acc[j]);
        }
    }
}

// One work unit: rows row0 .. row0+127 of segment sg, blocks 4 grp .. 4 grp + 3.  Writes y
// (one group per row) or this group's partial, then, as the tile's last group, y.  false
// when an MMA completion timed out (the CTA stops; the error word is set).
template <int TYPE>
__device__ bool tb_unit(const BGemmArgs& a, const BGemmSeg& sg, int mt, int row0, int grp, int ngrp, uint32_t tmem,
                        uint64_t* bar, uint32_t& phase, uint8_t* smt) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, qd = warp & 3, part = warp >> 2;
    const int re = 32 * qd + lane;                  // this thread's tile row (TMEM lane)
    const bool live = 16 * part < a.n_seq;          // warp-uniform: this warp's sequences exist
    const int b0 = TB_G * grp;
    float acc[16], accm[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = accm[j] = 0.0f;
    tb_stage_raw<TYPE>(sg, row0, a.nb, 2 * grp, 0, smt);
    tb_stage_raw<TYPE>(sg, row0, a.nb, 2 * grp + 1, 1, smt);
    tb_stage_x(a, b0, smt);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    bool ok = true;
    for (int b = b0; b < b0 + TB_G; ++b) {
        tb_dequant<TYPE>(sg, row0, b, smt);
        fence_proxy_async_smem();   // operands written by the generic proxy -> visible to the tensor cores
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint8_t* bx = smt + TB_BX + (b & 1) * 16 * TB_B_LBO;
            const uint32_t dh = tmem + (b & 1) * 128, dl = dh + 64;
#pragma unroll
            for (int k = 0; k < 8; ++k) {   // the block's eight K = 32 slices into one accumulator each
                const uint64_t bd = tc_desc(bx + 2 * k * TB_B_LBO, TB_B_LBO, 128);
                tc_mma(dh, tc_desc(smt + TB_AHI + 2 * k * TB_A_LBO, TB_A_LBO, 128), bd, TB_IDESC, k);
                tc_mma(dl, tc_desc(smt + TB_ALO + 2 * k * TB_A_LBO, TB_A_LBO, 128), bd, TB_IDESC, k);
            }
            tc_commit(bar);
        }
        if (b + 1 < b0 + TB_G) tb_stage_x(a, b + 1, smt);   // next activation block, other buffer / slot
        cp_async_commit();
        if (b > b0 && live) tb_epilogue<TYPE>(smt, tmem, b - 1, re, qd, part, acc, accm);
        ok = __all_sync(0xffffffffu, mbar_wait(bar, phase, a.err));   // warp-uniform: tcgen05.ld is .aligned
        phase ^= 1u;
        tc_fence_after();
        cp_async_wait_all();
        tc_fence_before();
        if (!__syncthreads_and(ok)) return false;   // operands and the older accumulators free
    }
    tc_fence_after();
    if (live) tb_epilogue<TYPE>(smt, tmem, b0 + TB_G - 1, re, qd, part, acc, accm);
    const int row = row0 + re;
    const bool row_ok = row < sg.rows;
    float g[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) g[j] = TYPE == GGML_Q4_K ? __fadd_rn(acc[j], accm[j]) : acc[j];
    if (ngrp == 1) {
        if (live && row_ok)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int q = 16 * part + j;
                if (q < a.n_seq) a.y[static_cast<size_t>(q) * a.y_stride + sg.out_off + row] = g[j];
            }
        return true;
    }
    // partial of this group -> scratch; the tile's last group adds them in group order
    float* sc = a.part + (static_cast<size_t>(mt) * ngrp) * TB_N * TB_M;
    if (live)
#pragma unroll
        for (int j = 0; j < 16; ++j) __stcg(sc + (static_cast<size_t>(grp) * TB_N + 16 * part + j) * TB_M + re, g[j]);
    __threadfence();
    __syncthreads();
    unsigned* last = reinterpret_cast<unsigned*>(smt + TB_BAR + 12);
    if (tid == 0) {
        const unsigned prev = atomicAdd(a.cnt + mt, 1u);
        *last = prev == static_cast<unsigned>(ngrp - 1);
        if (prev == static_cast<unsigned>(ngrp - 1)) a.cnt[mt] = 0u;   // ready for the next launch
        __threadfence();
    }
    __syncthreads();
    if (*last && live && row_ok) {
#pragma unroll 1
        for (int j = 0; j < 16; ++j) {
            const int q = 16 * part + j;
            if (q >= a.n_seq) break;
            float r = __ldcg(sc + static_cast<size_t>(q) * TB_M + re);
            for (int t = 1; t < ngrp; ++t) r = __fadd_rn(r, __ldcg(sc + (static_cast<size_t>(t) * TB_N + q) * TB_M + re));
            a.y[static_cast<size_t>(q) * a.y_stride + sg.out_off + row] = r;
        }
    }
    __syncthreads();   // `last` is rewritten by the next unit
    return true;
}

// L2 prefetch of a unit's weight bytes (its rows' four blocks; 128-byte lines over the CTA).
__device__ __forceinline__ void tb_prefetch_unit(const BGemmArgs& a, int u, int ngrp) {
    if (u >= a.ntiles * ngrp) return;
    const int mt = u / ngrp, grp = u - mt * ngrp;
    const BGemmSeg sg = bg_seg(a, mt);
    const int row0 = (mt - sg.tile0) * TB_M, nr = min(TB_M, sg.rows - row0);
    const int bytes = sg.type == GGML_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    const size_t rb = static_cast<size_t>(a.nb) * bytes, gb = static_cast<size_t>(TB_G) * bytes;
    const int lines = static_cast<int>((gb + 127) / 128) + 1;   // a group's span, any alignment
    for (int i = threadIdx.x; i < nr * lines; i += TB_THREADS) {
        const int r = i / lines, c = i - r * lines;
        const uint8_t* base = sg.w + static_cast<size_t>(row0 + r) * rb + static_cast<size_t>(grp) * gb;
        const uint8_t* line = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(base) & ~uintptr_t(127)) + 128 * c;
        if (line < base + gb) asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
}

// Persistent: CTA c takes units c, c + grid, ...; unit u = (row tile u / ngrp, group u % ngrp).
// One CTA per SM (512 threads at up to 128 registers fill the register file); 256 TMEM columns.
__global__ void __launch_bounds__(TB_THREADS, 1) k_b_gemm_tc(const BGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smt[];
    const int tid = threadIdx.x, warp = tid >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smt + TB_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smt + TB_BAR + 8);
    const int ngrp = a.nb / TB_G, units = a.ntiles * ngrp;
    if (static_cast<int>(blockIdx.x) >= units) return;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(TB_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 32) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    tb_prefetch_unit(a, blockIdx.x, ngrp);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        tb_prefetch_unit(a, u + gridDim.x, ngrp);
        const int mt = u / ngrp, grp = u - mt * ngrp;
        const BGemmSeg sg = bg_seg(a, mt);
        const int row0 = (mt - sg.tile0) * TB_M;
        ok = sg.type == GGML_Q4_K ? tb_unit<GGML_Q4_K>(a, sg, mt, row0, grp, ngrp, tmem, bar, phase, smt)
                                  : tb_unit<GGML_Q6_K>(a, sg, mt, row0, grp, ngrp, tmem, bar, phase, smt);
    }
    cp_async_wait_all();
    if (!ok && tid == 0) mbar_wait(bar, phase ^ 1u, nullptr);   // a late completion: let the MMAs drain
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TB_COLS) : "memory");
}
