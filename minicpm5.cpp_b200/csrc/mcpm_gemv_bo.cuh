// GEMV over Q4_K / Q6_K rows staged in shared memory, in the block order: every (row,
// super-block) integer sum is exact (the integers of dot_row_q*_K_q8_K_scalar,
// src/ops/ops_scalar_optimized.cpp:139-404), scaled by one fp32 fma per block and accumulated in
// groups of four blocks:
//   acc  = fma(xd*d, isum, acc)              (Q6_K: isum minus its 32*sum(sc*bsums) offset)
//   accm = fma(-(xd*dmin), minsum, accm)     (Q4_K only)
//   g    = acc + accm per group of 4 blocks;  row = ((g0 + g1) + g2) + ...
// This is the order of the tcgen05 batched GEMM and of the C restatement's ORC_ORDER_BATCH, so a
// sequence decoded token by token and one prefilled in batches give the same bits.
//
// Pass 1 (integer sums): each (row, super-block) task is split over S adjacent threads (S = 1, 2
// or 4: the largest that keeps every task of the pass to one per thread), thread k of a task
// taking quarters k*4/S .. (k+1)*4/S - 1:
//   Q4_K quarter j: qs bytes [32j, 32j+32): low nibbles against x[64j, 64j+32), high nibbles
//                   against x[64j+32, 64j+64) (sub-blocks 2j, 2j+1);
//   Q6_K quarter j = 2h + lh: the four 16-element sub-blocks 8h + 2kk + lh (kk = 0..3).
// The parts are added with xor shuffles (exact integers); isum, minsum and the fp16 scale bits of
// each task go to shared memory.  Pass 2: one thread per row runs the fp32 chain.
#pragma once
#include "mcpm_device.cuh"

namespace mcpm {

constexpr int GEMV_BO_LG = -1;   // log2 of the threads per task; -1: the largest that fits the CTA
constexpr int BO_WORDS = 3;   // per (row, block): isum, minsum (Q4_K), fp16 scale bits (Q4_K: d | dmin << 16)

__device__ __forceinline__ int dp2a_lo_ss(int a, int b, int c) {   // c + a.h0*b.b0 + a.h1*b.b1, signed
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_ss(int a, int b, int c) {   // c + a.h0*b.b2 + a.h1*b.b3, signed
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_lo_su(int a, uint32_t b, int c) {   // signed 16-bit pairs, unsigned bytes
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_su(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Q4_K quarter j of one super-block: 16*(sc[2j]*lo + sc[2j+1]*hi) (|.| < 2^27) and
// mn[2j]*P[2j] + mn[2j+1]*P[2j+1] (P = bsum pairs of the 32-element sub-blocks).
__device__ __forceinline__ void q4k_qtr(const uint8_t* blk, const uint4& hdr, const XQSmem& xq, int b, int j, int& s16,
                                        int& m) {
    const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
    const int4* xp = reinterpret_cast<const int4*>(xq.qs[b] + 64 * j);
    int lo = 0, hi = 0;   // hi carries 16 * (high-nibble dot): the nibbles are masked in place
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 q = qp[c];
        const int4 xl = xp[c], xh = xp[2 + c];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        const int a[4] = {xl.x, xl.y, xl.z, xl.w}, e[4] = {xh.x, xh.y, xh.z, xh.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            lo = dp4a_us(w[k] & 0x0f0f0f0fu, a[k], lo);
            hi = dp4a_us(w[k] & 0xf0f0f0f0u, e[k], hi);
        }
    }
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    uint32_t scw, mnw;
    if (j < 2) {   // sub-blocks 0..3: sc = scales[s] & 63, mn = scales[s+4] & 63
        scw = s0 & 0x3f3f3f3fu;
        mnw = s1 & 0x3f3f3f3fu;
    } else {       // sub-blocks 4..7: low nibbles of scales[s+4], top bits of scales[s-4] / scales[s]
        scw = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
        mnw = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    }
    const uint32_t sh = 16 * (j & 1);
    scw >>= sh;
    mnw >>= sh;
    s16 = (static_cast<int>(scw & 0xffu) << 4) * lo + static_cast<int>((scw >> 8) & 0xffu) * hi;
    const int* bs = reinterpret_cast<const int*>(xq.bsums[b]);   // int16 pairs: sub-block s = word s
    const int p0 = bs[2 * j], p1 = bs[2 * j + 1];
    const int P = ((static_cast<int16_t>(p0 & 0xffff) + (p0 >> 16)) & 0xffff) |
                  ((static_cast<int16_t>(p1 & 0xffff) + (p1 >> 16)) << 16);   // |P| <= 4064: int16 pairs
    m = dp2a_lo_su(P, mnw, 0);
}

// Q6_K quarter j = 2h + lh: sum over its four sub-blocks of sc * (dot - 32*bsum).  Blocks are 210
// bytes (2-byte aligned): words are read aligned and funnel-shifted, at most 4 bytes past the
// block (callers keep the tail readable).
__device__ __forceinline__ int q6k_qtr(const uint32_t* base, uint32_t sh, const XQSmem& xq, int b, int j) {
    const int h = j >> 1, lh = j & 1;
    const int ia = 16 * h + 4 * lh, ib = ia + 8, ih = 32 + 8 * h + 4 * lh;
    uint32_t A[5], B[5], H[5];
#pragma unroll
    for (int t = 0; t < 5; ++t) {
        A[t] = base[ia + t];
        B[t] = base[ib + t];
        H[t] = base[ih + t];
    }
    const int8_t* xb = xq.qs[b] + 128 * h + 16 * lh;
    const int4 x0 = *reinterpret_cast<const int4*>(xb), x1 = *reinterpret_cast<const int4*>(xb + 32);
    const int4 x2 = *reinterpret_cast<const int4*>(xb + 64), x3 = *reinterpret_cast<const int4*>(xb + 96);
    const int xa[4] = {x0.x, x0.y, x0.z, x0.w}, xc[4] = {x1.x, x1.y, x1.z, x1.w};
    const int xe[4] = {x2.x, x2.y, x2.z, x2.w}, xf[4] = {x3.x, x3.y, x3.z, x3.w};
    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t a = __funnelshift_r(A[t], A[t + 1], sh), c = __funnelshift_r(B[t], B[t + 1], sh);
        const uint32_t hh = __funnelshift_r(H[t], H[t + 1], sh);
        d0 = dp4a_us((a & 0x0f0f0f0fu) | ((hh << 4) & 0x30303030u), xa[t], d0);
        d1 = dp4a_us((c & 0x0f0f0f0fu) | ((hh << 2) & 0x30303030u), xc[t], d1);
        d2 = dp4a_us(((a >> 4) & 0x0f0f0f0fu) | (hh & 0x30303030u), xe[t], d2);
        d3 = dp4a_us(((c >> 4) & 0x0f0f0f0fu) | ((hh >> 2) & 0x30303030u), xf[t], d3);
    }
    // scales[8h + 2kk + lh]: bytes lh, lh+2 of the words at byte 192 + 8h and 196 + 8h
    const uint32_t w0 = __funnelshift_r(base[48 + 2 * h], base[49 + 2 * h], sh) >> (8 * lh);
    const uint32_t w1 = __funnelshift_r(base[49 + 2 * h], base[50 + 2 * h], sh) >> (8 * lh);
    const uint32_t sc4 = __byte_perm(w0, w1, 0x6420);   // (sc kk0, sc kk1, sc kk2, sc kk3)
    const int16_t* q = xq.bsums[b] + 8 * h + lh;       // bsums of sub-blocks 8h + 2kk + lh
    const int bp0 = (q[0] & 0xffff) | (static_cast<int>(q[2]) << 16);
    const int bp1 = (q[4] & 0xffff) | (static_cast<int>(q[6]) << 16);
    const int s = sbyte(sc4, 0) * d0 + sbyte(sc4, 1) * d1 + sbyte(sc4, 2) * d2 + sbyte(sc4, 3) * d3;
    const int off = dp2a_lo_ss(bp0, static_cast<int>(sc4), dp2a_hi_ss(bp1, static_cast<int>(sc4), 0));
    return s - 32 * off;
}

// Rows [0, R0) at w0 and [R0, R) at w1 (same TYPE, NB super-blocks per row, rows contiguous in
// shared memory) -> out[r].  part: part_words ints of scratch (BO_WORDS per task, whole rows per
// pass).  Must be called by all threads of the CTA; out is visible to every thread on return.
// Not inlined: one copy per (TYPE, NB) serves every phase.
template <int TYPE, int NB>
__device__ __noinline__ void gemv_bo_t(const uint8_t* w0, int R0, const uint8_t* w1, int R, const XQSmem& xq,
                                       int* part, int part_words, float* out) {
    constexpr int RB = TYPE == GGML_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int mt = (part_words / BO_WORDS / NB) * NB;   // whole rows per pass
    for (int t0 = 0; t0 < R * NB; t0 += mt) {
        const int ntask = min(mt, R * NB - t0);
        const int lg = GEMV_BO_LG >= 0 ? GEMV_BO_LG : 4 * ntask <= nthr ? 2 : 2 * ntask <= nthr ? 1 : 0;   // log2 of S
        const int S = 1 << lg, per = 4 >> lg;                                // threads per task, quarters each
        for (int u = tid; u < ntask * S; u += nthr) {   // a task's S threads are adjacent lanes of one warp
            const int t = u >> lg, k = u & (S - 1);
            const int task = t0 + t, row = task / NB, b = task - row * NB;
            const uint8_t* blk = row < R0 ? w0 + static_cast<size_t>(task) * RB
                                          : w1 + static_cast<size_t>(task - R0 * NB) * RB;
            int is = 0, ms = 0;
            uint32_t dd;
            if (TYPE == GGML_Q4_K) {
                const uint4 hdr = *reinterpret_cast<const uint4*>(blk);   // d|dmin, scales[0..11]
                for (int q = 0; q < per; ++q) {
                    int s16, m;
                    q4k_qtr(blk, hdr, xq, b, k * per + q, s16, m);
                    is += s16;
                    ms += m;
                }
                dd = hdr.x;
            } else {
                const uintptr_t addr = reinterpret_cast<uintptr_t>(blk);
                const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
                const uint32_t sh = static_cast<uint32_t>(addr & 3) * 8;
                for (int q = 0; q < per; ++q) is += q6k_qtr(base, sh, xq, b, k * per + q);
                dd = __funnelshift_r(base[52], base[53], sh) & 0xffffu;
            }
            if (lg) {
                const unsigned grp = ((1u << S) - 1u) << (tid & 31 & ~(S - 1));   // this task's S lanes
                for (int o = 1; o < S; o <<= 1) {
                    is += __shfl_xor_sync(grp, is, o);
                    if (TYPE == GGML_Q4_K) ms += __shfl_xor_sync(grp, ms, o);
                }
            }
            if (k == 0) {
                int* dst = part + t * BO_WORDS;
                dst[0] = TYPE == GGML_Q4_K ? (is >> 4) : is;   // Q4_K: exact, a multiple of 16
                dst[1] = ms;
                dst[2] = static_cast<int>(dd);
            }
        }
        __syncthreads();
        // pass 2: one thread per row, the block-order chain
        const int r_begin = t0 / NB, nrows = ntask / NB;
        for (int r = tid; r < nrows; r += nthr) {
            const int* src = part + r * NB * BO_WORDS;
            float row_v = 0.0f;
#pragma unroll
            for (int g0 = 0; g0 < NB; g0 += 4) {
                float acc = 0.0f, accm = 0.0f;
#pragma unroll
                for (int bb = g0; bb < g0 + 4; ++bb) {
                    const float xd = xq.d[bb];
                    const uint32_t dd = static_cast<uint32_t>(src[bb * BO_WORDS + 2]);
                    acc = __fmaf_rn(__fmul_rn(xd, h2f(dd)), __int2float_rn(src[bb * BO_WORDS]), acc);
                    if (TYPE == GGML_Q4_K)
                        accm = __fmaf_rn(-__fmul_rn(xd, h2f(dd >> 16)), __int2float_rn(src[bb * BO_WORDS + 1]), accm);
                }
                const float gv = TYPE == GGML_Q4_K ? __fadd_rn(acc, accm) : acc;
                row_v = g0 == 0 ? gv : __fadd_rn(row_v, gv);
            }
            out[r_begin + r] = row_v;
        }
        __syncthreads();
    }
}

// Dispatch on the weight type and the row length (8 or 24 super-blocks).  Rows [0, R0) at w0 and,
// optionally, rows [R0, R) of a second matrix of the same type at w1 (gate and up in one pass).
__device__ __forceinline__ void gemv_bo2(int type, const uint8_t* w0, int R0, const uint8_t* w1, int R, int nb,
                                         const XQSmem& xq, int* part, int part_words, float* out) {
    if (type == GGML_Q4_K) {
        if (nb == 8)
            gemv_bo_t<GGML_Q4_K, 8>(w0, R0, w1, R, xq, part, part_words, out);
        else
            gemv_bo_t<GGML_Q4_K, 24>(w0, R0, w1, R, xq, part, part_words, out);
    } else {
        if (nb == 8)
            gemv_bo_t<GGML_Q6_K, 8>(w0, R0, w1, R, xq, part, part_words, out);
        else
            gemv_bo_t<GGML_Q6_K, 24>(w0, R0, w1, R, xq, part, part_words, out);
    }
}
__device__ __forceinline__ void gemv_bo(int type, const uint8_t* w, int R, int nb, const XQSmem& xq, int* part,
                                        int part_words, float* out) {
    gemv_bo2(type, w, R, w, R, nb, xq, part, part_words, out);
}

}  // namespace mcpm
