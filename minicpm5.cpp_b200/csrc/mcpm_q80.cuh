// Q8_0 x fp32 GEMV (gemv_q8_0, ops.cpp:58-79) shared by the standalone op (mcpm_ops.cu)
// and the tensor-parallel engine (mcpm_tp.cu).
//
// Evaluation order of the reference build: per 32-block eight lanes k with
// A_k = fma(q_k, x_k, q_{k+8} x_{k+8}), B_k = fma(q_{k+16}, x_{k+16}, q_{k+24} x_{k+24}),
// v_k = B_k + A_k, then the pairs (k, k+4), (k, k+2), (k, k+1); row = fma(fp16 d, local, row)
// over the blocks in order.  A CTA streams its row range through a 3-slot TMA ring; pass 1
// gives one thread per (row, block) its local sum, then one thread per row runs the block
// chain while the rest of the CTA moves on to the next stage.
#pragma once
#include "mcpm_device.cuh"

namespace mcpm {

constexpr int Q80_SLOTS = 3;
constexpr int Q80_SLOT_BYTES = 40960;
constexpr int Q80_SLOT_STRIDE = Q80_SLOT_BYTES + 128;   // readable tail for the funnel-shifted reads
constexpr int Q80_MAX_TASKS = 1536;
constexpr int Q80_MAX_COLS = 8192;
constexpr int Q80_THREADS = 512;

constexpr int Q80_PART = 1536;   // (local, d) pairs of one stage, per buffer

// Shared-memory carve-up of one Q8_0 GEMV CTA.
struct Q80Smem {
    uint8_t* ring;   // [Q80_SLOTS][Q80_SLOT_STRIDE] weight stages
    float* xs;       // [Q80_MAX_COLS] activations (swizzled, q80_xpos)
    float2* part;    // [2][Q80_PART] (local, d) per (row, block) of the last two stages
    uint64_t* bars;  // [Q80_SLOTS]
    float* scratch;  // [64] reductions
    __device__ explicit Q80Smem(uint8_t* base) {
        ring = base;
        xs = reinterpret_cast<float*>(ring + Q80_SLOTS * Q80_SLOT_STRIDE);
        part = reinterpret_cast<float2*>(xs + Q80_MAX_COLS);
        bars = reinterpret_cast<uint64_t*>(part + 2 * Q80_PART);
        scratch = reinterpret_cast<float*>(bars + Q80_SLOTS + 1);
    }
};
constexpr size_t q80_smem_bytes() {
    return static_cast<size_t>(Q80_SLOTS) * Q80_SLOT_STRIDE + Q80_MAX_COLS * 4 + 2 * Q80_PART * 8 +
           (Q80_SLOTS + 1) * 8 + 64 * 4;
}

// Activations sit in shared memory swizzled per 32-block: the 4-float chunk j of block b
// at 32 b + 4 (j ^ (b & 7)), so the eight lanes of a quarter warp, which read the same chunk
// of eight consecutive blocks, hit eight different bank groups.
__device__ __forceinline__ int q80_xpos(int i) {
    const int b = i >> 5, j = (i >> 2) & 7;
    return (b << 5) | ((j ^ (b & 7)) << 2) | (i & 3);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE round-to-nearest operations per
// instruction, each lane rounded exactly as the scalar operation).
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// int8 lanes k, k+1 of w as exact floats: (q + 128) is a low byte of w ^ 0x80 (two's
// complement), 0x4B0000xx is 2^23 + q + 128, and subtracting 2^23 + 128 is exact.
__device__ __forceinline__ unsigned long long q80_i8f2(uint32_t wx, int k) {
    const uint32_t lo = __byte_perm(wx, 0x4B000000u, 0x7640u | static_cast<uint32_t>(k));
    const uint32_t hi = __byte_perm(wx, 0x4B000000u, 0x7640u | static_cast<uint32_t>(k + 1));
    return f2_add(f2_pack(__uint_as_float(lo), __uint_as_float(hi)), f2_pack(-8388736.0f, -8388736.0f));
}

// Local sum of 32-block b (34 bytes at blk: fp16 d, 32 int8) against the swizzled
// activations xsw; d returned apart.  Lanes k, k+1 of the reference's eight-lane order are
// computed as one f32x2 pair at every step, so every lane sees the same operations in the
// same order as the scalar form.
__device__ __forceinline__ float q80_block_local(const uint8_t* blk, const float* xsw, int b, float& d) {
    d = h2f(*reinterpret_cast<const uint16_t*>(blk));
    const uintptr_t qa = reinterpret_cast<uintptr_t>(blk + 2);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(qa & 3) * 8;
    unsigned long long q[16], xv[16];   // element pairs (2m, 2m+1)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = __funnelshift_r(base[i], base[i + 1], sh) ^ 0x80808080u;
        q[2 * i] = q80_i8f2(w, 0);
        q[2 * i + 1] = q80_i8f2(w, 2);
    }
    const float* xb = xsw + 32 * b;
    const int sw = b & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = *reinterpret_cast<const float4*>(xb + 4 * (i ^ sw));
        xv[2 * i] = f2_pack(f.x, f.y);
        xv[2 * i + 1] = f2_pack(f.z, f.w);
    }
    unsigned long long v[4];   // (v_k, v_k+1), k = 0, 2, 4, 6
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const unsigned long long A = f2_fma(q[m], xv[m], f2_mul(q[m + 4], xv[m + 4]));       // lanes 2m, 2m+1 (+8)
        const unsigned long long B = f2_fma(q[m + 8], xv[m + 8], f2_mul(q[m + 12], xv[m + 12]));   // (+16, +24)
        v[m] = f2_add(B, A);
    }
    const unsigned long long c01 = f2_add(v[2], v[0]);   // (v4 + v0, v5 + v1)
    const unsigned long long c23 = f2_add(v[3], v[1]);   // (v6 + v2, v7 + v3)
    const float2 t = f2_unpack(f2_add(c23, c01));         // (c2 + c0, c3 + c1)
    return __fadd_rn(t.y, t.x);
}

// Rows per stage for nb blocks per row: one slot of weights, and the (local, d) pairs of a
// stage at a padded row stride of nb + 2 (16-byte aligned rows that start 4 banks apart).
__host__ __device__ constexpr int q80_stage_rows(int nb) {
    return (Q80_SLOT_BYTES / (nb * Q8_0_BYTES) < Q80_PART / (nb + 2) ? Q80_SLOT_BYTES / (nb * Q8_0_BYTES)
                                                                          : Q80_PART / (nb + 2));
}
// Rows per stage for a CTA range of at most `rows` rows: at least three stages where the
// range allows (the first copies overlap the first compute), at most q80_stage_rows(nb).
__host__ __device__ constexpr int q80_pick_stage(int nb, int rows) {
    const int third = (rows + 2) / 3;
    const int want = third < 1 ? 1 : third;
    return want < q80_stage_rows(nb) ? want : q80_stage_rows(nb);
}

// Rows [r0, r1) of w (nb blocks per row, nb % 8 == 0), `sr` rows per stage (at most
// q80_stage_rows(nb)).  q80_start (thread 0) initialises the ring and issues the first
// copies: weights only, so it may run before the producer of the activations has finished.
__device__ __forceinline__ void q80_issue(const uint8_t* __restrict__ w, int r0, int r1, int nb, int sr,
                                          const Q80Smem& s, int st) {
    const int rb = nb * Q8_0_BYTES, slot = st % Q80_SLOTS, a = r0 + st * sr, n = min(sr, r1 - a);
    const uint32_t bytes = static_cast<uint32_t>(n) * rb;
    mbar_expect_tx(&s.bars[slot], bytes);
    bulk_g2s(s.ring + slot * Q80_SLOT_STRIDE, w + static_cast<size_t>(a) * rb, bytes, &s.bars[slot]);
}
__device__ __forceinline__ void q80_start(const uint8_t* __restrict__ w, int r0, int r1, int nb, int sr,
                                          const Q80Smem& s) {
    for (int i = 0; i < Q80_SLOTS; ++i) mbar_init(&s.bars[i], 1);
    fence_mbar_init();
    const int nstages = (r1 - r0 + sr - 1) / sr;
    for (int st = 0; st < min(nstages, Q80_SLOTS); ++st) q80_issue(w, r0, r1, nb, sr, s, st);
}

// Streams the stages against the swizzled s.xs (filled and synchronised by the caller after
// q80_start).  Per stage: every thread takes (row, block) tasks (pass 1), one barrier, then
// the last ceil(n/32) warps each own a row -- row r of the stage at thread
// blockDim - 32 ceil(n/32) + r -- and run its block chain while the other warps start the
// next stage's pass 1 (the pairs alternate between two buffers).  row(i, v, v_pair) gets the
// row index, its value and the value of row i ^ 1 (the neighbouring lane); stage ranges are
// assumed pair-aligned where v_pair is used.  Returns false (uniformly) when a weight wait
// timed out; the values are then garbage and ERR_TIMEOUT is raised.
template <class Row>
__device__ bool q80_run(const uint8_t* __restrict__ w, int r0, int r1, int nb, int sr, const Q80Smem& s,
                        unsigned* err, Row row) {
    const int tid = threadIdx.x;
    const int nstages = (r1 - r0 + sr - 1) / sr;
    bool ok = true;
    for (int st = 0; st < nstages; ++st) {
        const int slot = st % Q80_SLOTS, a = r0 + st * sr, n = min(sr, r1 - a);
        const uint8_t* sw = s.ring + slot * Q80_SLOT_STRIDE;
        float2* part = s.part + (st & 1) * Q80_PART;
        ok &= mbar_wait(&s.bars[slot], (st / Q80_SLOTS) & 1, err);
        for (int t = tid; t < n * nb; t += blockDim.x) {
            const int r = t / nb, b = t - r * nb;
            float d;
            const float local = q80_block_local(sw + static_cast<size_t>(t) * Q8_0_BYTES, s.xs, b, d);
            part[r * (nb + 2) + b] = make_float2(local, d);
        }
        __syncthreads();   // pairs complete; the slot is free
        if (tid == 0 && st + Q80_SLOTS < nstages) q80_issue(w, r0, r1, nb, sr, s, st + Q80_SLOTS);
        const int cw0 = static_cast<int>(blockDim.x) - 32 * ((n + 31) / 32);
        if (tid >= cw0) {   // whole warps: the row's block chain, in block order
            const int r = tid - cw0;
            float acc = 0.0f;
            if (r < n) {
                const float4* pr = reinterpret_cast<const float4*>(part + r * (nb + 2));
                for (int b = 0; b < nb / 2; b += 4) {
                    float4 ld[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) ld[k] = pr[b + k];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc = __fmaf_rn(ld[k].y, ld[k].x, acc);
                        acc = __fmaf_rn(ld[k].w, ld[k].z, acc);
                    }
                }
            }
            const float pair = __shfl_xor_sync(0xffffffffu, acc, 1);
            if (r < n) row(a + r, acc, pair);
        }
    }
    return __syncthreads_and(ok);
}

}  // namespace mcpm
