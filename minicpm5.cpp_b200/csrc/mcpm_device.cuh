// Device-side building blocks of the MiniCPM5 decode path for sm_100a.
//
// Numerics: every fp32 operation whose result is compared bit-for-bit with the CPU
// restatement (oracle/mcpm_oracle.c) is written with an explicit rounding intrinsic
// (__fadd_rn, __fmul_rn, __fmaf_rn, __fdiv_rn, __fsqrt_rn) so the compiler cannot
// contract or reorder it.  The GEMV accumulation follows the reference's AVX2 kernels
// (src/ops/ops_avx2.cpp:153-276) lane for lane, which makes GEMV outputs identical to
// the reference for identical Q8_K inputs.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace mcpm {

// ---------------------------------------------------------------- block formats
// Byte layouts of reference include/ops.h:33-65 (kept unchanged in HBM).
constexpr int QK_K = 256;
constexpr int Q4K_BYTES = 144;   // fp16 d, fp16 dmin, scales[12], qs[128]
constexpr int Q6K_BYTES = 210;   // ql[128], qh[64], scales[16] (int8), fp16 d
constexpr int Q8_0_BYTES = 34;   // fp16 d, qs[32]
constexpr int Q8K_BYTES = 292;   // f32 d, qs[256], int16 bsums[16]
constexpr int GGML_F32 = 0, GGML_Q8_0 = 8, GGML_Q4_K = 12, GGML_Q6_K = 14;

// Error bits written to the engine's device error word.
constexpr unsigned ERR_TIMEOUT = 1u, ERR_BAD_TOKEN = 2u, ERR_BAD_ARG = 4u;

__host__ __device__ constexpr int row_bytes(int type, int cols) {
    return type == GGML_Q4_K ? cols / 256 * Q4K_BYTES
         : type == GGML_Q6_K ? cols / 256 * Q6K_BYTES
         : type == GGML_Q8_0 ? cols / 32 * Q8_0_BYTES : cols * 4;
}
__host__ __device__ constexpr int block_bytes(int type) {
    return type == GGML_Q4_K ? Q4K_BYTES : type == GGML_Q6_K ? Q6K_BYTES : Q8_0_BYTES;
}

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses before its later
// async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bulk global->shared copy (TMA, no tensor map, this CTA's shared memory only).  dst, src 16-byte aligned,
// bytes a multiple of 16; completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Same copy, tagged evict-first in L2: streamed-once weights must not push the kernel's
// code, the activations and the KV cache out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// L2 prefetch of a global range (TMA unit, fire and forget).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// 16-byte global->shared copy (LDGSTS, L2 only); completes at cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// 4-byte global->shared copy (LDGSTS through L1).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Waits until at most N of this thread's committed cp.async groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// 16-byte L2 load that the compiler keeps in program order (issued where written).
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_cg_f32(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
// Programmatic dependent launch: wait until the preceding kernel in the stream has finished
// and its writes are visible (returns at once without a programmatic dependency), and allow
// the next kernel to start launching its CTAs.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Epoch-tagged element (value + epoch in one naturally aligned 64-bit word, which is
// single-copy atomic): the consumer's load is also its synchronisation, with no fence on
// the producer side and no separate flag round trip.
__device__ __forceinline__ void st_epoch(unsigned long long* p, float v, unsigned epoch) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_epoch(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ ulonglong2 ld_epoch2(const unsigned long long* p) {   // each element atomic
    ulonglong2 w;
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}
// Four consecutive epoch-tagged values (16-byte aligned), polled until all carry `epoch`;
// false (and ERR_TIMEOUT raised) after 1 s.
__device__ __forceinline__ bool load4_epoch(const unsigned long long* src, unsigned epoch, float4& v, unsigned* err) {
    ulonglong2 a = ld_epoch2(src), b = ld_epoch2(src + 2);
    auto ready = [&]() {
        return (a.x >> 32) == epoch && (a.y >> 32) == epoch && (b.x >> 32) == epoch && (b.y >> 32) == epoch;
    };
    if (!ready()) {
        const uint64_t t0 = globaltimer();
        do {
            a = ld_epoch2(src);
            b = ld_epoch2(src + 2);
            if (!ready() && globaltimer() - t0 > 1000000000ull) {
                atomicOr(err, ERR_TIMEOUT);
                return false;
            }
        } while (!ready());
    }
    v = make_float4(__uint_as_float(static_cast<unsigned>(a.x)), __uint_as_float(static_cast<unsigned>(a.y)),
                    __uint_as_float(static_cast<unsigned>(b.x)), __uint_as_float(static_cast<unsigned>(b.y)));
    return true;
}
// Two consecutive epoch-tagged values (16-byte aligned), polled until both carry `epoch`;
// false (and ERR_TIMEOUT raised) after 1 s.
__device__ __forceinline__ bool load2_epoch(const unsigned long long* src, unsigned epoch, float& a, float& b,
                                            unsigned* err) {
    ulonglong2 w = ld_epoch2(src);
    if ((w.x >> 32) != epoch || (w.y >> 32) != epoch) {
        const uint64_t t0 = globaltimer();
        do {
            w = ld_epoch2(src);
            if (((w.x >> 32) != epoch || (w.y >> 32) != epoch) && globaltimer() - t0 > 1000000000ull) {
                if (err) atomicOr(err, ERR_TIMEOUT);
                return false;
            }
        } while ((w.x >> 32) != epoch || (w.y >> 32) != epoch);
    }
    a = __uint_as_float(static_cast<unsigned>(w.x));
    b = __uint_as_float(static_cast<unsigned>(w.y));
    return true;
}
// Eight consecutive epoch-tagged values (16-byte aligned), polled until all carry `epoch`.
__device__ __forceinline__ bool load8c_epoch(const unsigned long long* src, unsigned epoch, float (&y)[8],
                                             unsigned* err) {
    ulonglong2 w[4];
    auto pending = [&]() {
        unsigned m = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            m |= static_cast<unsigned>((w[i].x >> 32) != epoch) | static_cast<unsigned>((w[i].y >> 32) != epoch);
        return m != 0;
    };
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = ld_epoch2(src + 2 * i);
    if (pending()) {
        const uint64_t t0 = globaltimer();
        do {
            __nanosleep(64);   // back off: many CTAs poll the same lines
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = ld_epoch2(src + 2 * i);
            if (pending() && globaltimer() - t0 > 1000000000ull) {
                if (err) atomicOr(err, ERR_TIMEOUT);
                return false;
            }
        } while (pending());
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        y[2 * i] = __uint_as_float(static_cast<unsigned>(w[i].x));
        y[2 * i + 1] = __uint_as_float(static_cast<unsigned>(w[i].y));
    }
    return true;
}
// Acquire side of a flag handshake: loads after it see what the flag's writer published.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_u32(const unsigned* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u32(unsigned* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_u32(unsigned* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}
// signed / unsigned byte i (0..3) of w
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return static_cast<int>(w << (24 - 8 * i)) >> 24; }
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (w >> (8 * i)) & 0xff; }

// Bounded wait on an mbarrier phase.  Returns false (and sets ERR_TIMEOUT in *err when err
// is given) after ~1 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > 1000000000ull) {
            if (err) atomicOr(err, ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------- K/V cache elements
// The cache holds fp32 rows (the reference's KVCacheLayer) or, as an option, fp16 rows: a
// value enters the cache rounded to nearest-even half precision and is read back exactly, so
// every later operation sees the same float as the C restatement's fp16 option.
__device__ __forceinline__ float4 half4_to_float4(uint2 u) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
template <typename KT>
struct KvElt;
template <>
struct KvElt<float> {
    static constexpr int PER16 = 4;   // elements per 16-byte copy
    __device__ static float4 ld4(const float* p) { return ld_cg_f4(p); }   // global, through L2
    __device__ static float4 sm4(const float* p) { return *reinterpret_cast<const float4*>(p); }
    __device__ static float2 sm2(const float* p) { return *reinterpret_cast<const float2*>(p); }
    __device__ static float get(float v) { return v; }
    __device__ static float put(float v) { return v; }
    __device__ static void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
};
template <>
struct KvElt<__half> {
    static constexpr int PER16 = 8;
    __device__ static float4 ld4(const __half* p) {
        uint2 u;
        asm volatile("ld.global.cg.v2.u32 {%0, %1}, [%2];" : "=r"(u.x), "=r"(u.y) : "l"(p));
        return half4_to_float4(u);
    }
    __device__ static float4 sm4(const __half* p) { return half4_to_float4(*reinterpret_cast<const uint2*>(p)); }
    __device__ static float2 sm2(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }
    __device__ static float get(__half v) { return __half2float(v); }
    __device__ static __half put(float v) { return __float2half_rn(v); }
    __device__ static void st4(__half* p, float4 v) {   // values already half-representable
        const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&a);
        u.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = u;
    }
};
// The float a value becomes once stored in a cache of element type KT.
template <typename KT>
__device__ __forceinline__ float kv_round(float v) {
    return KvElt<KT>::get(KvElt<KT>::put(v));
}

// ---------------------------------------------------------------- canonical scalar math
// exp(x): k = rint(x*log2e), two-constant Cody-Waite reduction, degree-7 Taylor
// polynomial in Horner form, 2^k applied as two exact power-of-two factors.
// Identical operation sequence to orc_expf (oracle/mcpm_oracle.c).
__device__ __forceinline__ float canon_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.972084045410156f) return 0.0f;
    const float kf = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = __fmaf_rn(-kf, 0.693145751953125f, x);
    r = __fmaf_rn(-kf, 1.428606765330187045e-06f, r);
    float p = 1.98412701138295233250e-04f;
    p = __fmaf_rn(p, r, 1.38888892251998186111e-03f);
    p = __fmaf_rn(p, r, 8.33333376795053482056e-03f);
    p = __fmaf_rn(p, r, 4.16666679084300994873e-02f);
    p = __fmaf_rn(p, r, 1.66666671633720397949e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int k = static_cast<int>(kf);
    const int k1 = k / 2, k2 = k - k1;
    return __fmul_rn(__fmul_rn(p, __int_as_float((k1 + 127) << 23)), __int_as_float((k2 + 127) << 23));
}

// silu(g)*u as the reference build evaluates it (reciprocal, then products); an
// overflowing exp(-g) yields NaN like the build's Newton-refined reciprocal estimate.
__device__ __forceinline__ float canon_silu_mul(float g, float u) {
    const float y = __fadd_rn(1.0f, canon_expf(-g));
    const float r = isinf(y) ? __int_as_float(0x7fc00000) : __fdiv_rn(1.0f, y);
    return __fmul_rn(__fmul_rn(g, r), u);
}

// lround + clamp as inlined by the reference build (ops.cpp:717); NaN/huge -> -127.
// Branch-free: the conversion truncates and saturates, the clamp is integer min/max, and
// values outside the build's 64-bit conversion range (and NaN) select -127.
__device__ __forceinline__ int quant_away(float v) {
    const float a = __fadd_rn(v, copysignf(0.4999999701976776f, v));
    const bool ok = a < 9223372036854775808.0f && a >= -9223372036854775808.0f;
    const int t = min(max(__float2int_rz(a), -127), 127);
    return ok ? t : -127;
}
// _mm256_cvtps_epi32 (ties-to-even; NaN and |v| >= 2^31 give INT_MIN) + clamp
// (ops_avx2.cpp:118-121).  Branch-free, as quant_away.
__device__ __forceinline__ int quant_even(float v) {
    const bool ok = v < 2147483648.0f && v >= -2147483648.0f;
    const int t = min(max(__float2int_rn(v), -127), 127);
    return ok ? t : -127;
}

// ---------------------------------------------------------------- activation staging
// Q8_K activation in shared memory: qs rows padded to 272 B so that lanes reading
// different blocks at the same offset hit different bank groups.
constexpr int XQ_STRIDE = 272;
constexpr int XQ_MAX_BLOCKS = 24;
struct XQSmem {
    int8_t qs[XQ_MAX_BLOCKS][XQ_STRIDE];
    float d[XQ_MAX_BLOCKS];
    int16_t bsums[XQ_MAX_BLOCKS][16];
};

// Quantise one 256-block held by a full warp (lane l holds y[8l .. 8l+7]) into the
// canonical Q8_K block.  Block amax follows the reference build's NaN-sensitive
// eight-lane maximum (orc_block_amax); d = amax*(1/127); mul = 127/amax.
// Writes qs/d/bsums through the supplied pointers (shared or global, 4-byte aligned).
template <bool AWAY, bool PERM = false>
__device__ __forceinline__ void quant_block_warp(const float (&y)[8], int8_t* qs_out, float* d_out,
                                                 int16_t* bsums_out) {
    const int lane = threadIdx.x & 31;
    bool nan = false;
    unsigned mine = 0u;   // largest |y| of this lane, as bits (ordered like the values)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        nan |= y[k] != y[k];
        mine = max(mine, __float_as_uint(fabsf(y[k])));
    }
    float amax;
    if (!__any_sync(0xffffffffu, nan)) {   // no NaN: every lane order gives the plain maximum
        amax = __uint_as_float(__reduce_max_sync(0xffffffffu, mine));
    } else {
        float accs[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float e = fabsf(y[k]);
            const unsigned nanmask = __ballot_sync(0xffffffffu, e != e);
            const int last = nanmask ? 31 - __clz(nanmask) : -1;
            const unsigned bits = (lane > last) ? __float_as_uint(e) : 0u;
            const unsigned mx = __reduce_max_sync(0xffffffffu, bits);
            accs[k] = (last == 31) ? __int_as_float(0x7fc00000) : __uint_as_float(mx);
        }
        float m[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) m[i] = (accs[i + 4] > accs[i]) ? accs[i + 4] : accs[i];
        const float n0 = (m[2] > m[0]) ? m[2] : m[0];
        const float n1 = (m[3] > m[1]) ? m[3] : m[1];
        amax = (n1 > n0) ? n1 : n0;
    }
    int q[8];
    if (amax == 0.0f || amax != amax) {
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = 0;
        if (lane == 0) *d_out = 0.0f;
    } else {
        const float mul = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float v = __fmul_rn(y[k], mul);
            q[k] = AWAY ? quant_away(v) : quant_even(v);
        }
        if (lane == 0) *d_out = __fmul_rn(amax, 1.0f / 127.0f);
    }
    const uint32_t w0 = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
    const uint32_t w1 = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
    if (PERM) {   // lane-major order of the batched GEMM: element 32s + 4k + t at 32k + 4s + t
        *reinterpret_cast<uint32_t*>(qs_out + 64 * (lane & 3) + 4 * (lane >> 2)) = w0;
        *reinterpret_cast<uint32_t*>(qs_out + 64 * (lane & 3) + 32 + 4 * (lane >> 2)) = w1;
    } else {
        uint32_t* qw = reinterpret_cast<uint32_t*>(qs_out + 8 * lane);
        qw[0] = w0;
        qw[1] = w1;
    }
    int s = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if ((lane & 1) == 0) bsums_out[lane >> 1] = static_cast<int16_t>(s);
}

// Canonical sum of squares of x[0..2047] by the first 256 threads of the block (lane l
// = fma chain over x[l + 256 i], 32-lane butterfly, warps combined as
// ((w0+w1)+(w2+w3))+((w4+w5)+(w6+w7))).  xv[i] = x[tid + 256 i] already loaded.
// `red` is 8 floats of shared scratch.  Result valid in all threads after return.
__device__ __forceinline__ float sumsq_2048(const float (&xv)[8], float* red) {
    const int tid = threadIdx.x;
    if (tid < 256) {
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = __fmaf_rn(xv[i], xv[i], a);
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, s));
        if ((tid & 31) == 0) red[tid >> 5] = a;
    }
    __syncthreads();
    const float r = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3])),
                              __fadd_rn(__fadd_rn(red[4], red[5]), __fadd_rn(red[6], red[7])));
    __syncthreads();
    return r;
}

// ---------------------------------------------------------------- GEMV pass 1
// Integer partial sums of one (row, super-block) task, split into the eight AVX2
// accumulator lanes of the reference kernels:
//   Q4_K lane k: sum_j sc[2j]*sum_{i=4k}^{4k+3} lo(qs[32j+i])*x[64j+i]
//                     + sc[2j+1]*sum hi(qs[32j+i])*x[64j+32+i]        (ops_avx2.cpp:168-181)
//   Q6_K lane k: sum over the four quarters of both halves for l in [4k, 4k+4), minus
//                32*(bsums[2k]*sc[2k] + bsums[2k+1]*sc[2k+1])          (ops_avx2.cpp:225-270)
// minsum: Q4_K sum_g mn[g]*(bsums[2g]+bsums[2g+1]); Q6_K the total -32 offset.
struct Partials {
    int k[8];
    int minsum;
};

__device__ __forceinline__ void q4k_task(const uint8_t* blk, const XQSmem& xq, int b, Partials& out) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);   // d|dmin, scales[0..11]
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    const uint32_t sc_lo = s0 & 0x3f3f3f3fu;                                       // sc[0..3]
    const uint32_t sc_hi = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);         // sc[4..7]
    const uint32_t mn_lo = s1 & 0x3f3f3f3fu;                                       // mn[0..3]
    const uint32_t mn_hi = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);  // mn[4..7]
    const uint4* qs = reinterpret_cast<const uint4*>(blk + 16);
    const uint4* xs = reinterpret_cast<const uint4*>(xq.qs[b]);
#pragma unroll
    for (int k = 0; k < 8; ++k) out.k[k] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t scw = j < 2 ? sc_lo : sc_hi;
        const int sa = ubyte(scw, 2 * (j & 1)), sb = ubyte(scw, 2 * (j & 1) + 1);
        const uint4 w0 = qs[2 * j], w1 = qs[2 * j + 1];            // qs[32j .. 32j+31]
        const uint4 xl0 = xs[4 * j], xl1 = xs[4 * j + 1];          // x[64j .. 64j+31]
        const uint4 xh0 = xs[4 * j + 2], xh1 = xs[4 * j + 3];      // x[64j+32 .. 64j+63]
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const int xl[8] = {(int)xl0.x, (int)xl0.y, (int)xl0.z, (int)xl0.w, (int)xl1.x, (int)xl1.y, (int)xl1.z, (int)xl1.w};
        const int xh[8] = {(int)xh0.x, (int)xh0.y, (int)xh0.z, (int)xh0.w, (int)xh1.x, (int)xh1.y, (int)xh1.z, (int)xh1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int lo = dp4a_us(w[k] & 0x0f0f0f0fu, xl[k], 0);
            const int hi = dp4a_us((w[k] >> 4) & 0x0f0f0f0fu, xh[k], 0);
            out.k[k] += sa * lo + sb * hi;
        }
    }
    const int* bs = reinterpret_cast<const int*>(xq.bsums[b]);   // 8 words of int16 pairs
    int m = 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const int pair = bs[g];
        const int sx = static_cast<int>(static_cast<int16_t>(pair & 0xffff)) + (pair >> 16);
        m += ubyte(g < 4 ? mn_lo : mn_hi, g & 3) * sx;
    }
    out.minsum = m;
}

// Q6_K super-blocks sit at any 2-byte alignment: words are read aligned and funnel-shifted
// (reads at most 4 bytes past the block, which callers keep readable).
__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint32_t* base, int i, uint32_t sh) {
    return __funnelshift_r(base[i], base[i + 1], sh);
}

__device__ __forceinline__ void q6k_task(const uint8_t* blk, const XQSmem& xq, int b, Partials& out) {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(blk);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(addr & 3) * 8;
    uint32_t scw[4];   // scales: bytes 192..207 -> words 48..51
#pragma unroll
    for (int i = 0; i < 4; ++i) scw[i] = ld_u32_unaligned(base, 48 + i, sh);
    const int* bs = reinterpret_cast<const int*>(xq.bsums[b]);
    int off = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int pair = bs[k];
        const int b0 = static_cast<int>(static_cast<int16_t>(pair & 0xffff)), b1 = pair >> 16;
        const int o = b0 * sbyte(scw[k >> 1], 2 * (k & 1)) + b1 * sbyte(scw[k >> 1], 2 * (k & 1) + 1);
        out.k[k] = -32 * o;
        off += o;
    }
    out.minsum = 32 * off;
    const uint4* xs = reinterpret_cast<const uint4*>(xq.qs[b]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint4 xv[8];   // x[128h .. 128h+127]; quarter kk covers words 8kk .. 8kk+7
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[i] = xs[8 * h + i];
        const int* xw = reinterpret_cast<const int*>(xv);
        const uint32_t sw = scw[2 * h], sw2 = scw[2 * h + 1];
#pragma unroll
        for (int t = 0; t < 8; ++t) {   // t = AVX2 lane: l in [4t, 4t+4)
            const uint32_t A = ld_u32_unaligned(base, 16 * h + t, sh);        // ql[64h + 4t]
            const uint32_t B = ld_u32_unaligned(base, 16 * h + 8 + t, sh);    // ql[64h + 32 + 4t]
            const uint32_t H = ld_u32_unaligned(base, 32 + 8 * h + t, sh);    // qh[32h + 4t]
            const uint32_t q0 = (A & 0x0f0f0f0fu) | ((H << 4) & 0x30303030u);
            const uint32_t q1 = (B & 0x0f0f0f0fu) | ((H << 2) & 0x30303030u);
            const uint32_t q2 = ((A >> 4) & 0x0f0f0f0fu) | (H & 0x30303030u);
            const uint32_t q3 = ((B >> 4) & 0x0f0f0f0fu) | ((H >> 2) & 0x30303030u);
            const int si = (t >= 4) ? 1 : 0;   // scale index 8h + 2kk + (l >= 16)
            const int sc0 = sbyte(sw, si), sc1 = sbyte(sw, 2 + si), sc2 = sbyte(sw2, si), sc3 = sbyte(sw2, 2 + si);
            int acc = out.k[t];
            acc += sc0 * dp4a_us(q0, xw[t], 0);
            acc += sc1 * dp4a_us(q1, xw[8 + t], 0);
            acc += sc2 * dp4a_us(q2, xw[16 + t], 0);
            acc += sc3 * dp4a_us(q3, xw[24 + t], 0);
            out.k[t] = acc;
        }
    }
}

// fp16 super-block scale(s) of a task: Q4_K -> (d, dmin); Q6_K -> (d, 0).
__device__ __forceinline__ void block_scales(int type, const uint8_t* blk, float& d, float& dmin) {
    if (type == GGML_Q4_K) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(blk);
        d = h2f(w);
        dmin = h2f(w >> 16);
    } else {
        const uintptr_t addr = reinterpret_cast<uintptr_t>(blk) + 208;
        const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
        d = h2f(__funnelshift_r(base[0], base[1], static_cast<uint32_t>(addr & 3) * 8));
        dmin = 0.0f;
    }
}

// ---------------------------------------------------------------- GEMV over staged rows
// Rows [0, R) of one or two matrices of the same TYPE and NB super-blocks per row, staged
// contiguously in shared memory: rows [0, R0) at w0, rows [R0, R) at w1.  Pass 1, one
// (row, block) task per thread (q4k_task / q6k_task): the task's integer partials split into the
// eight AVX2 lanes, its min term (Q4_K) or offset (Q6_K), and the two fp32 scale products
// dx = xd*d and dm = -(xd*dmin) go to `part` (PART_WORDS words per task).  Pass 2: lane k of
// a row group loads every operand of its chain, then runs the reference's fp32 accumulator
// chain for AVX2 lane k over the blocks (acc = fma(dx, isum_k, acc); Q4_K also
// acc_min = fma(dm, minsum, acc_min)); the eight lanes are reduced with hsum_f32_8's tree
// (a butterfly over lane bits 2, 1, 0) and the min term is added.  Row r's value goes to
// out[r] (shared memory), visible to every thread on return.  Not inlined: one copy per
// (TYPE, NB) serves every phase.  Must be called by all threads of the CTA (contains
// __syncthreads).
constexpr int PART_WORDS = 11;   // k0..k7, minsum, dx, dm (odd stride: conflict-free stores)

template <int TYPE, int NB>
__device__ __noinline__ void gemv_rows_t(const uint8_t* w0, int R0, const uint8_t* w1, int R, const XQSmem& xq,
                                         int* part, int max_tasks, float* out, unsigned long long* tr) {
    constexpr int RB = TYPE == GGML_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int mt = (max_tasks / NB) * NB;   // whole rows per chunk
    for (int t0 = 0; t0 < R * NB; t0 += mt) {
        const int ntask = min(mt, R * NB - t0);
        for (int t = tid; t < ntask; t += nthr) {
            const int task = t0 + t, row = task / NB, b = task - row * NB;
            const uint8_t* blk = row < R0 ? w0 + static_cast<size_t>(task) * RB
                                          : w1 + static_cast<size_t>(task - R0 * NB) * RB;
            Partials pt;
            if (TYPE == GGML_Q4_K)
                q4k_task(blk, xq, b, pt);
            else
                q6k_task(blk, xq, b, pt);
            float d, dmin;
            block_scales(TYPE, blk, d, dmin);
            const float xd = xq.d[b];
            int* dst = part + t * PART_WORDS;
#pragma unroll
            for (int k = 0; k < 8; ++k) dst[k] = pt.k[k];
            dst[8] = pt.minsum;
            dst[9] = __float_as_int(__fmul_rn(xd, d));
            dst[10] = __float_as_int(-__fmul_rn(xd, dmin));
        }
        __syncthreads();
        if (tr && tid == 0) tr[0] = globaltimer();
        // pass 2: one 8-lane group per row; trip count uniform per warp for the shuffles
        const int r_begin = t0 / NB, total = (ntask / NB) * 8;
        for (int base = tid & ~31; base < total; base += nthr) {
            const int g = base + (tid & 31);
            const bool valid = g < total;
            const int r = valid ? (g >> 3) : 0, k = g & 7;
            const int* src = part + r * NB * PART_WORDS;
            float dx[NB], iv[NB], dm[NB], im[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                dx[b] = __int_as_float(src[b * PART_WORDS + 9]);
                iv[b] = __int2float_rn(src[b * PART_WORDS + k]);
                if (TYPE == GGML_Q4_K) {
                    dm[b] = __int_as_float(src[b * PART_WORDS + 10]);
                    im[b] = __int2float_rn(src[b * PART_WORDS + 8]);
                }
            }
            float acc = 0.0f, acc_min = 0.0f;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                acc = __fmaf_rn(dx[b], iv[b], acc);
                if (TYPE == GGML_Q4_K) acc_min = __fmaf_rn(dm[b], im[b], acc_min);
            }
            acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
            acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
            acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
            if (valid && k == 0) out[r_begin + r] = TYPE == GGML_Q4_K ? __fadd_rn(acc, acc_min) : acc;
        }
        __syncthreads();
        if (tr && tid == 0) tr[1] = globaltimer();
    }
}

// Dispatch on the weight type (Q4_K / Q6_K) and the row length (8 or 24 super-blocks).
// Rows [0, R0) at w0 and, optionally, rows [R0, R) of a second matrix of the same type at
// w1 (gate and up in one pass).  `tr` (optional): thread 0 stores globaltimer after pass 1
// (tr[0]) and pass 2 (tr[1]).
__device__ __forceinline__ void gemv_rows2(int type, const uint8_t* w0, int R0, const uint8_t* w1, int R, int nb,
                                           const XQSmem& xq, int* part, int max_tasks, float* out,
                                           unsigned long long* tr = nullptr) {
    if (type == GGML_Q4_K) {
        if (nb == 8)
            gemv_rows_t<GGML_Q4_K, 8>(w0, R0, w1, R, xq, part, max_tasks, out, tr);
        else
            gemv_rows_t<GGML_Q4_K, 24>(w0, R0, w1, R, xq, part, max_tasks, out, tr);
    } else {
        if (nb == 8)
            gemv_rows_t<GGML_Q6_K, 8>(w0, R0, w1, R, xq, part, max_tasks, out, tr);
        else
            gemv_rows_t<GGML_Q6_K, 24>(w0, R0, w1, R, xq, part, max_tasks, out, tr);
    }
}
__device__ __forceinline__ void gemv_rows(int type, const uint8_t* w, int R, int nb, const XQSmem& xq, int* part,
                                          int max_tasks, float* out, unsigned long long* tr = nullptr) {
    gemv_rows2(type, w, R, w, R, nb, xq, part, max_tasks, out, tr);
}

}  // namespace mcpm
