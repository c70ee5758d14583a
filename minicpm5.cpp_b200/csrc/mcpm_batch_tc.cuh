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
// into two int8 operands with w' = F * A1 + A2 exactly: Q4_K A1 = q * (sc >> 3), A2 = q * (sc & 7),
// F = 8 (both <= 105: one multiply per four packed weights); Q6_K the 64-based split
// w' = 64 * hi + lo of bg_pack, F = 64.  One thread issues 18 tcgen05.mma (kind::i8, M = 128,
// N = 64): the block's eight K = 32 slices into one int32 accumulator per operand, and the
// min / offset term as two more products of the row's 16 min (Q4_K, each repeated for its two
// block sums) or scale (Q6_K) bytes with the low (biased by -128) and high bytes of the
// sequences' 16 block sums.  Pipeline, per block: the MMAs of block b run while the CTA
// dequantises block b + 1 into the other operand buffer and runs the epilogue of block b - 1
// (tcgen05.ld of the other TMEM buffer); the raw rows of block b + 2 and the activations of
// block b + 1 are copied in meanwhile.  Buffers rotate with a per-CTA block counter, so the
// next work unit's first block is staged during this unit's last ones.  The groups of a row
// tile run on different CTAs: each writes its g to a scratch buffer, and the last to finish
// (a per-tile counter) adds the groups in order and stores y.
constexpr int TB_M = 128, TB_N = 64, TB_THREADS = 512, TB_G = 4, TB_COLS = 512;
constexpr int TB_CTA_THREADS = TB_THREADS + 32;           // 16 compute warps + the MMA warp
constexpr int TB_MAX_GROUPS = 6;                          // groups of a 6144-wide row
constexpr int TB_A_LBO = (TB_M / 8) * 128;                // K-half stride of a weight operand (2048 B)
constexpr int TB_B_LBO = (TB_N / 8) * 128;                // K-half stride of the activation operand (1024 B)
constexpr int TB_A_BYTES = 2 * 16 * TB_A_LBO;             // A1 then A2: [16 K-halves][16 row groups][8][16] int8 each
constexpr int TB_A = 0;                                   // 2 x operand pair (block counter parity)
constexpr int TB_BX = TB_A + 2 * TB_A_BYTES;              // 2 x [16 K-halves][8 seq groups][8][16] int8
constexpr int TB_XD = TB_BX + 2 * 16 * TB_B_LBO;          // 3 x float [64]
constexpr int TB_XB = TB_XD + 3 * TB_N * 4;               // 3 x int16 [64][16]
constexpr int TB_RM_BYTES = TB_M * 8 + TB_M * 16;         // float d, dmin [128]; min / scale operand rows [128][16]
constexpr int TB_RM = TB_XB + 3 * TB_N * 32;              // 3 x row metadata
constexpr int TB_BS = TB_RM + 3 * TB_RM_BYTES;            // 2 x {low bytes, high bytes} of the block sums: [8][8][16] each
constexpr int TB_ZERO = TB_BS + 2 * 2 * TB_B_LBO;         // 2048 zero bytes: second K-half of the min operands
constexpr int TB_RAW_Q4 = 144, TB_RAW_Q6 = 216;           // raw row stride of one staged block (Q6_K: 212 aligned bytes)
constexpr int TB_RAW = TB_ZERO + 2048;                    // [128 rows][stride]: one block's raw rows
constexpr int TB_BAR = TB_RAW + TB_M * TB_RAW_Q6;         // MMA-done mbarrier, TMEM base address, last-CTA flag,
constexpr int TB_BYTES = TB_BAR + 24;                     // operand mbarrier
// TMEM buffer u (block counter parity): A1 at 256 u, A2 at 256 u + 64, min low at + 128, min high at + 192
// instruction descriptor: S32 accumulator, S8 x S8, both K-major, N = 64, M = 128
constexpr uint32_t TB_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(TB_N >> 3) << 17) |
                              (static_cast<uint32_t>(TB_M >> 4) << 24);
static_assert(TB_BYTES <= 232448 && TB_BX % 1024 == 0 && TB_RM % 16 == 0 && TB_BS % 16 == 0 && TB_ZERO % 16 == 0 &&
                  TB_RAW % 16 == 0 && TB_BAR % 8 == 0,
              "k_b_gemm_tc layout");
static_assert(BATCH_MAX <= TB_N, "one sequence tile holds every sequence of a batch");

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
// Barrier of the 16 compute warps (the MMA warp never joins it); the _and form reduces a predicate.
__device__ __forceinline__ void tb_sync() { asm volatile("bar.sync 1, %0;" ::"n"(TB_THREADS) : "memory"); }
__device__ __forceinline__ bool tb_sync_and(bool p) {
    uint32_t r;
    asm volatile("{\n .reg .pred q, o;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred o, 1, %2, q;\n selp.u32 %0, 1, 0, o;\n}"
                 : "=r"(r)
                 : "r"(static_cast<uint32_t>(p)), "n"(TB_THREADS)
                 : "memory");
    return r != 0;
}
// Operands of the next block are in shared memory: every compute thread fences its writes for
// the tensor cores, then one lane per warp arrives on the operand barrier (16 arrivals).
__device__ __forceinline__ void tb_operands_ready(uint64_t* opbar) {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(opbar)) : "memory");
}

// Activation block b of sequences 0..63 -> operand buffer it & 1 (K-major core matrices; the
// values are already lane-major), scales and block sums -> slot it % 3; zeros beyond n_seq.
__device__ void tb_stage_x(const BGemmArgs& a, int b, int it, uint8_t* smt) {
    const int tid = threadIdx.x;
    uint8_t* bx = smt + TB_BX + (it & 1) * 16 * TB_B_LBO;
#pragma unroll
    for (int i = 0; i < 2; ++i) {   // 64 sequences x 16 chunks: two per thread
        const int t = tid + TB_THREADS * i, q = t >> 4, c = t & 15;
        uint8_t* dst = bx + c * TB_B_LBO + (q >> 3) * 128 + (q & 7) * 16;
        if (q < a.n_seq)
            cp_async16(dst, a.aqs + (static_cast<size_t>(q) * B_NBA + b) * 256 + 16 * c);
        else
            *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
    const int slot = it % 3;
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

// Block b of rows row0 .. row0+127 -> the raw buffer.  Q4_K: the 144 bytes in 16-byte copies
// (16-byte aligned in the file).  Q6_K: blocks are 2-byte aligned, so the 212 bytes of the
// 4-byte aligned span holding the block (it starts (b & 1) * 2 bytes in) in 4-byte copies;
// the span never leaves the row.  Rows past the segment are skipped.
template <int TYPE>
__device__ __forceinline__ void tb_stage_raw1(const BGemmSeg& sg, int row0, int nb, int b, uint8_t* smt) {
    uint8_t* dst0 = smt + TB_RAW;
    const int nr = min(TB_M, sg.rows - row0);
    if (TYPE == GGML_Q4_K) {
        const size_t rb = static_cast<size_t>(nb) * Q4K_BYTES;
        for (int i = threadIdx.x; i < nr * 9; i += TB_THREADS) {
            const int r = i / 9, c = i - r * 9;
            cp_async16(dst0 + r * TB_RAW_Q4 + 16 * c,
                       sg.w + static_cast<size_t>(row0 + r) * rb + static_cast<size_t>(b) * Q4K_BYTES + 16 * c);
        }
    } else {
        const size_t rb = static_cast<size_t>(nb) * Q6K_BYTES;
        const size_t start = static_cast<size_t>(b) * Q6K_BYTES - (b & 1) * 2;
        for (int i = threadIdx.x; i < nr * 53; i += TB_THREADS) {
            const int r = i / 53, c = i - r * 53;
            cp_async4(dst0 + r * TB_RAW_Q6 + 4 * c, sg.w + static_cast<size_t>(row0 + r) * rb + start + 4 * c);
        }
    }
}
__device__ __forceinline__ void tb_stage_raw1_any(const BGemmSeg& sg, int row0, int nb, int b, uint8_t* smt) {
    if (sg.type == GGML_Q4_K)
        tb_stage_raw1<GGML_Q4_K>(sg, row0, nb, b, smt);
    else
        tb_stage_raw1<GGML_Q6_K>(sg, row0, nb, b, smt);
}

// Block sums of activation slot it % 3 -> the low (minus 128) and high byte operands of
// buffer it & 1 (threads 384..511: sequence q, half hh).
__device__ __forceinline__ void tb_build_bs(int it, uint8_t* smt) {
    const int i = static_cast<int>(threadIdx.x) - (TB_THREADS - 2 * TB_N);
    if (i < 0) return;
    const int q = i >> 1, hh = i & 1;
    const uint4 v = *reinterpret_cast<const uint4*>(smt + TB_XB + (it % 3) * TB_N * 32 + 32 * q + 16 * hh);
    uint8_t* lo = smt + TB_BS + (it & 1) * 2 * TB_B_LBO + (q >> 3) * 128 + (q & 7) * 16 + 8 * hh;
    *reinterpret_cast<uint2*>(lo) =   // s = 256 hi + lo = 256 hi + (lo - 128) + 128: all operands signed
        make_uint2(__byte_perm(v.x, v.y, 0x6420) ^ 0x80808080u, __byte_perm(v.z, v.w, 0x6420) ^ 0x80808080u);
    *reinterpret_cast<uint2*>(lo + TB_B_LBO) = make_uint2(__byte_perm(v.x, v.y, 0x7531), __byte_perm(v.z, v.w, 0x7531));
}

// Block b's staged raw rows -> operand pair it & 1 (lane-major K) and row metadata slot
// it % 3 (d, dmin and the min / scale operand rows), in one pass; the caller fences and
// publishes them with a barrier.  Rows past the segment are left stale: their outputs are
// never stored.
template <int TYPE>
__device__ __forceinline__ void tb_dequant(const BGemmSeg& sg, int row0, int b, int it, uint8_t* smt) {
    const int tid = threadIdx.x;
    uint8_t* ao = smt + TB_A + (it & 1) * TB_A_BYTES;   // A1 at +0, A2 at + 16 K-halves
    uint8_t* rm = smt + TB_RM + (it % 3) * TB_RM_BYTES;
    float* rd = reinterpret_cast<float*>(rm);
    uint32_t* mrow = reinterpret_cast<uint32_t*>(rm + 8 * TB_M);   // [128][4] words
    if (TYPE == GGML_Q4_K) {   // task (row r, sub-blocks 4jj .. 4jj+3, lanes 4kh .. 4kh+3): one 16-byte K chunk per lane
        const int r = tid & (TB_M - 1), jj = (tid >> 7) & 1, kh = tid >> 8;
        if (row0 + r >= sg.rows) return;
        const uint8_t* blk = smt + TB_RAW + r * TB_RAW_Q4;
        const uint4 head = *reinterpret_cast<const uint4*>(blk);   // d, dmin, 12 packed scale bytes
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 64 * jj + 16 * kh);        // group 2jj, lanes 4kh..
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 16 + 64 * jj + 32 + 16 * kh);   // group 2jj+1
        auto sb = [&](int i) -> uint32_t {   // scale byte i (0..11)
            const uint32_t w = i < 4 ? head.y : i < 8 ? head.z : head.w;
            return (w >> (8 * (i & 3))) & 0xffu;
        };
        uint32_t sc[4], mn[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {   // get_scale_min_k4 (include/ops.h:67-75) of sub-block 4jj + e
            const int s = 4 * jj + e;
            if (jj == 0) {
                sc[e] = sb(s) & 63;
                mn[e] = sb(s + 4) & 63;
            } else {
                sc[e] = (sb(s + 4) & 15) | ((sb(s - 4) >> 6) << 4);
                mn[e] = (sb(s + 4) >> 4) | ((sb(s) >> 6) << 4);
            }
        }
        if (kh == 0) {   // block sums 8jj .. 8jj+7 pair with the mins of their sub-blocks
            mrow[4 * r + 2 * jj] = mn[0] * 0x0101u | (mn[1] * 0x0101u) << 16;
            mrow[4 * r + 2 * jj + 1] = mn[2] * 0x0101u | (mn[3] * 0x0101u) << 16;
            if (jj == 0) {
                rd[r] = h2f(head.x);
                rd[TB_M + r] = h2f(head.x >> 16);
            }
        }
        const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wb[4] = {qb.x, qb.y, qb.z, qb.w};
        uint32_t hi[4], lo[4];   // sc >> 3 and sc & 7 of the four sub-blocks
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[e] = sc[e] >> 3, lo[e] = sc[e] & 7u;
        uint8_t* dst = ao + jj * TB_A_LBO + (r >> 3) * 128 + (r & 7) * 16;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {   // lane k = 4kh + kk: K bytes 32k + 16jj + 4e + t, e = sub-block 4jj + e
            const int k = 4 * kh + kk;
            const uint32_t m0 = wa[kk] & 0x0f0f0f0fu, m1 = (wa[kk] >> 4) & 0x0f0f0f0fu;
            const uint32_t m2 = wb[kk] & 0x0f0f0f0fu, m3 = (wb[kk] >> 4) & 0x0f0f0f0fu;
            *reinterpret_cast<uint4*>(dst + 2 * k * TB_A_LBO) = make_uint4(m0 * hi[0], m1 * hi[1], m2 * hi[2], m3 * hi[3]);
            *reinterpret_cast<uint4*>(dst + (16 + 2 * k) * TB_A_LBO) =
                make_uint4(m0 * lo[0], m1 * lo[1], m2 * lo[2], m3 * lo[3]);
        }
    } else {   // tasks (row r, sub-block s, half): bg_pack's 64-based split of sc * q
#pragma unroll 1
        for (int task = tid; task < TB_M * 16; task += TB_THREADS) {
            const int r = task & (TB_M - 1), sh = task >> 7, s = sh >> 1, half = sh & 1;
            if (row0 + r >= sg.rows) continue;
            const uint8_t* blk = smt + TB_RAW + r * TB_RAW_Q6 + (b & 1) * 2;
            if (sh == 0) {   // the row's 16 scales (operand of the offset products) and d
                const uint16_t* sp = reinterpret_cast<const uint16_t*>(blk + 192);   // 2-byte aligned
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    mrow[4 * r + g] = static_cast<uint32_t>(sp[2 * g]) | (static_cast<uint32_t>(sp[2 * g + 1]) << 16);
                rd[r] = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
            }
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
                uint32_t h4, l4;
                bg_pack(wa, wb, 1, h4, l4);
                const int k = 4 * half + kk;   // lane k: K bytes 32k + 4s .. +3 -> K-half 2k + (s >> 2)
                const int off = (2 * k + (s >> 2)) * TB_A_LBO + (r >> 3) * 128 + (r & 7) * 16 + 4 * (s & 3);
                *reinterpret_cast<uint32_t*>(ao + off) = h4;
                *reinterpret_cast<uint32_t*>(ao + 16 * TB_A_LBO + off) = l4;
            }
        }
    }
}

// Epilogue of the block of counter it for this thread's row (TMEM lane) and its 16 sequences:
// the block's integer sums from TMEM buffer it & 1, then the fp32 chains.
template <int TYPE>
__device__ __forceinline__ void tb_epilogue(const uint8_t* smt, uint32_t tmem, int it, int re, int qd, int part,
                                            float (&acc)[16], float (&accm)[16]) {
    const float* rd = reinterpret_cast<const float*>(smt + TB_RM + (it % 3) * TB_RM_BYTES);
    const float* xd = reinterpret_cast<const float*>(smt + TB_XD + (it % 3) * TB_N * 4) + 16 * part;
    const float d = rd[re], dmin = TYPE == GGML_Q4_K ? rd[TB_M + re] : 0.0f;
    const uint4 mw = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(rd) + 8 * TB_M + 16 * re);
    // the low bytes' -128 bias: 128 * the sum of the row's 16 operand bytes
    const int m128 = 128 * __dp4a(static_cast<int>(mw.w), 0x01010101,
                                  __dp4a(static_cast<int>(mw.z), 0x01010101,
                                         __dp4a(static_cast<int>(mw.y), 0x01010101, __dp4a(static_cast<int>(mw.x), 0x01010101, 0))));
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * qd) << 16) + (it & 1) * 256 + 16 * part;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t a1[8], a2[8], ml[8], mh[8];
        tc_ld8(tl + 8 * h, a1);
        tc_ld8(tl + 64 + 8 * h, a2);
        tc_ld8(tl + 128 + 8 * h, ml);
        tc_ld8(tl + 192 + 8 * h, mh);
        tc_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            const int j = 8 * h + jj;
            const int ms = static_cast<int>(mh[jj]) * 256 + static_cast<int>(ml[jj]) + m128;   // sum_i m_i * bsums_i
            const float xdj = xd[j];
            int v;
            if (TYPE == GGML_Q4_K) {
                v = static_cast<int>(a1[jj]) * 8 + static_cast<int>(a2[jj]);
                accm[j] = __fmaf_rn(-__fmul_rn(xdj, dmin), __int2float_rn(ms), accm[j]);
            } else {
                v = static_cast<int>(a1[jj]) * 64 + static_cast<int>(a2[jj]) - 32 * ms;
            }
            acc[j] = __fmaf_rn(__fmul_rn(xdj, d), __int2float_rn(v), acc[j]);
        }
    }
}

// The 18 MMAs of the block of counter it (thread 0): the eight K = 32 slices of A1 and A2 into
// TMEM buffer it & 1, then the min / offset products with the low and high bytes of the block sums.
__device__ __forceinline__ void tb_issue(uint8_t* smt, uint32_t tmem, int it, uint64_t* bar) {
    tc_fence_after();
    const uint32_t d0 = tmem + (it & 1) * 256;
    // descriptors of slice 0; slice k starts 2k K-halves further (the 16-byte address field
    // of the descriptor stays below 2^14 for any shared-memory offset)
    const uint8_t* ao = smt + TB_A + (it & 1) * TB_A_BYTES;
    const uint64_t bd0 = tc_desc(smt + TB_BX + (it & 1) * 16 * TB_B_LBO, TB_B_LBO, 128);
    const uint64_t a1d0 = tc_desc(ao, TB_A_LBO, 128), a2d0 = tc_desc(ao + 16 * TB_A_LBO, TB_A_LBO, 128);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint64_t bd = bd0 + static_cast<uint64_t>((2 * k * TB_B_LBO) >> 4);
        const uint64_t ak = static_cast<uint64_t>((2 * k * TB_A_LBO) >> 4);
        tc_mma(d0, a1d0 + ak, bd, TB_IDESC, k);
        tc_mma(d0 + 64, a2d0 + ak, bd, TB_IDESC, k);
    }
    const uint8_t* am = smt + TB_RM + (it % 3) * TB_RM_BYTES + 8 * TB_M;   // [128][16]: K-half 0; K-half 1 zero
    const uint8_t* bl = smt + TB_BS + (it & 1) * 2 * TB_B_LBO;
    const uint8_t* zero = smt + TB_ZERO;
    const uint64_t ad = tc_desc(am, static_cast<uint32_t>(zero - am), 128);
    tc_mma(d0 + 128, ad, tc_desc(bl, static_cast<uint32_t>(zero - bl), 128), TB_IDESC, 0);
    tc_mma(d0 + 192, ad, tc_desc(bl + TB_B_LBO, static_cast<uint32_t>(zero - (bl + TB_B_LBO)), 128), TB_IDESC, 0);
    tc_commit(bar);
}

// A CTA's next work unit, whose first block is staged during this unit.
struct TbNext {
    BGemmSeg sg;
    int row0, grp, valid;
};

// One work unit: rows row0 .. row0+127 of segment sg, blocks 4 grp .. 4 grp + 3, at block
// counter `it` (advanced by 4).  `staged`: the raw rows and activations of the unit's first
// block were copied in during the previous unit; `nx`: the CTA's next unit, whose first block
// is staged during this one.  Writes y (one group per row) or this group's partial and then,
// as the tile's last group, y.  false when an MMA completion timed out (the CTA stops; the
// error word is set).
template <int TYPE>
__device__ bool tb_unit(const BGemmArgs& a, const BGemmSeg& sg, int mt, int row0, int grp, int ngrp, bool staged,
                        const TbNext& nx, uint32_t tmem, uint64_t* bar, uint64_t* opbar, uint32_t& phase, int& it,
                        uint8_t* smt) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, qd = warp & 3, part = warp >> 2;
    const int re = 32 * qd + lane;                  // this thread's tile row (TMEM lane)
    const bool live = 16 * part < a.n_seq;          // warp-uniform: this warp's sequences exist
    const int b0 = TB_G * grp;
    unsigned long long* tr = (a.trace && !staged && blockIdx.x == 0 && tid == 0) ? a.trace : nullptr;
    if (tr) tr[0] = globaltimer();
    float acc[16], accm[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = accm[j] = 0.0f;
    if (!staged) {
        tb_stage_raw1<TYPE>(sg, row0, a.nb, b0, smt);
        tb_stage_x(a, b0, it, smt);
        cp_async_commit();
    }
    cp_async_wait_all();
    tb_sync();
    tb_build_bs(it, smt);
    tb_dequant<TYPE>(sg, row0, b0, it, smt);
    tb_operands_ready(opbar);   // the MMA warp issues block b0
    tb_sync();                  // the raw buffer is free
    tb_stage_raw1<TYPE>(sg, row0, a.nb, b0 + 1, smt);
    cp_async_commit();          // group R(b0 + 1)
    if (tr) tr[1] = globaltimer();
    bool ok = true;
    for (int i = 0; i < TB_G; ++i) {
        const int b = b0 + i, cur = it + i;
        if (tr) tr[2 + 6 * i] = globaltimer();
        // activations of the next block (this unit's, else the next unit's first): buffer / slot cur + 1
        if (i + 1 < TB_G)
            tb_stage_x(a, b + 1, cur + 1, smt);
        else if (nx.valid)
            tb_stage_x(a, TB_G * nx.grp, cur + 1, smt);
        cp_async_commit();      // group X(cur + 1)
        if (i + 1 < TB_G) {     // block b + 1 while the MMAs of block b run
            cp_async_wait_group<1>();   // R(b + 1): every group but X(cur + 1)
            tb_sync();
            if (tr) tr[3 + 6 * i] = globaltimer();
            tb_dequant<TYPE>(sg, row0, b + 1, cur + 1, smt);
            tb_sync();          // the raw buffer is free
            if (i + 2 < TB_G)
                tb_stage_raw1<TYPE>(sg, row0, a.nb, b + 2, smt);
            else if (nx.valid)
                tb_stage_raw1_any(nx.sg, nx.row0, a.nb, TB_G * nx.grp, smt);
            cp_async_commit();  // group R(b + 2)
        }
        if (tr) tr[4 + 6 * i] = globaltimer();
        if (i > 0 && live) tb_epilogue<TYPE>(smt, tmem, cur - 1, re, qd, part, acc, accm);
        if (tr) tr[5 + 6 * i] = globaltimer();
        ok = __all_sync(0xffffffffu, mbar_wait(bar, phase, a.err));   // warp-uniform: tcgen05.ld is .aligned
        phase ^= 1u;
        tc_fence_after();
        if (!tb_sync_and(ok)) return false;
        if (tr) tr[6 + 6 * i] = globaltimer();
        if (i + 1 < TB_G) {
            cp_async_wait_group<1>();   // X(cur + 1) (the raw rows of block b + 2 may stay in flight)
            tb_sync();
            tb_build_bs(cur + 1, smt);
            tb_operands_ready(opbar);   // block cur + 1: operands written, the epilogue of cur - 1 done
        }
        if (tr) tr[7 + 6 * i] = globaltimer();
    }
    tc_fence_after();
    if (live) tb_epilogue<TYPE>(smt, tmem, it + TB_G - 1, re, qd, part, acc, accm);
    tc_fence_before();
    it += TB_G;
    if (tr) tr[26] = globaltimer();
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
    tb_sync();   // the CTA's partial stores happen before thread 0's fence (cumulative) and count
    unsigned* last = reinterpret_cast<unsigned*>(smt + TB_BAR + 12);
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.cnt + mt, 1u);
        *last = prev == static_cast<unsigned>(ngrp - 1);
        if (prev == static_cast<unsigned>(ngrp - 1)) a.cnt[mt] = 0u;   // ready for the next launch
        __threadfence();   // the other groups' partials are read after their counts
    }
    tb_sync();
    if (*last && live && row_ok) {   // every load of four sequences in flight at once, then the ordered sums
        static_assert(TB_MAX_GROUPS * TB_G == B_NBA, "groups of the widest row");
#pragma unroll 1
        for (int j0 = 0; j0 < 16; j0 += 4) {
            float v[4][TB_MAX_GROUPS];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                for (int t = 0; t < TB_MAX_GROUPS; ++t)
                    v[jj][t] = t < ngrp ? __ldcg(sc + (static_cast<size_t>(t) * TB_N + 16 * part + j0 + jj) * TB_M + re)
                                        : 0.0f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int q = 16 * part + j0 + jj;
                float r = v[jj][0];
#pragma unroll
                for (int t = 1; t < TB_MAX_GROUPS; ++t)
                    if (t < ngrp) r = __fadd_rn(r, v[jj][t]);
                if (q < a.n_seq) a.y[static_cast<size_t>(q) * a.y_stride + sg.out_off + row] = r;
            }
        }
    }
    tb_sync();   // `last` is rewritten by the next unit
    if (tr) tr[27] = globaltimer();
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
// Warps 0-15 stage, dequantise and run the epilogues; warp 16 only issues the MMAs of each
// block once the compute warps report its operands (operand mbarrier), so the tensor cores
// work on block b while the compute warps prepare block b + 1.  One CTA per SM, so the
// 512-column TMEM allocation never waits for another CTA.
__global__ void __launch_bounds__(TB_CTA_THREADS, 1) k_b_gemm_tc(const BGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smt[];
    const int tid = threadIdx.x, warp = tid >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smt + TB_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smt + TB_BAR + 8);
    uint64_t* opbar = reinterpret_cast<uint64_t*>(smt + TB_BAR + 16);
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
        mbar_init(opbar, TB_THREADS / 32);
        fence_mbar_init();
    }
    if (tid < TB_THREADS) reinterpret_cast<uint32_t*>(smt + TB_ZERO)[tid] = 0u;   // zero K-half of the min operands
    tb_prefetch_unit(a, blockIdx.x, ngrp);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const int my_units = (units - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
    if (warp == TB_THREADS / 32) {   // the MMA warp
        if (tid == TB_THREADS) {
            int issued = 0;
            bool ok = true;
            for (; issued < my_units * TB_G; ++issued) {
                if (!mbar_wait(opbar, static_cast<uint32_t>(issued) & 1u, a.err)) {
                    ok = false;
                    break;
                }
                tb_issue(smt, tmem, issued, bar);
            }
            if (issued > 0) mbar_wait(bar, static_cast<uint32_t>(issued - 1) & 1u, ok ? a.err : nullptr);   // drained
        }
        __syncwarp();
    } else {
        uint32_t phase = 0;
        bool ok = true;
        auto unit_at = [&](int u, TbNext& t) {
            t.valid = u < units;
            if (!t.valid) return;
            const int mt = u / ngrp;
            t.grp = u - mt * ngrp;
            t.sg = bg_seg(a, mt);
            t.row0 = (mt - t.sg.tile0) * TB_M;
        };
        TbNext cur, nx;
        unit_at(blockIdx.x, cur);
        int it = 0;             // blocks processed by this CTA: operand / TMEM buffer parity, metadata slot
        bool staged = false;    // the current unit's first block already copied in
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            tb_prefetch_unit(a, u + gridDim.x, ngrp);
            unit_at(u + gridDim.x, nx);
            const int mt = u / ngrp;
            ok = cur.sg.type == GGML_Q4_K
                     ? tb_unit<GGML_Q4_K>(a, cur.sg, mt, cur.row0, cur.grp, ngrp, staged, nx, tmem, bar, opbar, phase, it, smt)
                     : tb_unit<GGML_Q6_K>(a, cur.sg, mt, cur.row0, cur.grp, ngrp, staged, nx, tmem, bar, opbar, phase, it, smt);
            staged = nx.valid;
            cur = nx;
        }
        cp_async_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TB_COLS) : "memory");
}
