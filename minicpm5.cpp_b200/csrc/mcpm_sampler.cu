// Device top-p sampler (Sampler::sample, src/sampler.cpp:8-72) in its canonical form:
//   v = logits * (1/T) when T > 0 and T != 1; M = max(-1e9, max v); e = canon_expf(v - M);
//   S = blocked sum of e (index order); p = e / S;
//   0 < top_p < 1: order by p descending, index ascending; keep the shortest prefix whose
//   blocked running sum reaches top_p (C = that running value); q = p / C;
//   otherwise: all tokens in index order, q = p;
//   token = first kept position whose blocked running sum of q is >= r, else the last kept.
// Blocked sums over a[0..m): 1024 ranges of L = ceil(m/1024) positions; range c runs
// sequentially from E_c, the sequential prefix of the range totals (each range total summed
// from 0).  The C restatement (orc_sample_top_p) computes the same numbers bit for bit.
//
// One CTA of 1024 threads.  The top-p candidates are located with a 16-bit histogram of
// the probability bits (its approximate sums only choose how much to sort), compacted in
// index order, and sorted with a stable LSD radix sort in shared memory; flat distributions
// whose top-p set exceeds SP_CAP positions take the same sort through global memory.
#include <cstdint>

#include "mcpm_device.cuh"
#include "mcpm_internal.h"

namespace mcpm {
namespace {

constexpr int SP_THREADS = 1024;
constexpr int SP_CAP = 8192;   // candidates sorted in shared memory

// smem layout
constexpr int SPS_T = 0;                          // float [1024] range totals
constexpr int SPS_E = SPS_T + 4 * SP_THREADS;     // float [1025] range prefixes
constexpr int SPS_RED = SPS_E + 4 * (SP_THREADS + 8);   // 64 words scratch
constexpr int SPS_HIST = SPS_RED + 4 * 64;        // int [256] counts, float [256] sums
constexpr int SPS_CNT = SPS_HIST + 8 * 256;       // int [16][1024] radix counts / scan
constexpr int SPS_K = SPS_CNT + 4 * 16 * SP_THREADS;   // uint32 [2][SP_CAP]
constexpr int SPS_I = SPS_K + 8 * SP_CAP;         // int [2][SP_CAP]
constexpr int SPS_BYTES = SPS_I + 8 * SP_CAP;

struct SampleArgs {
    const float* logits;
    int n;
    float temp, top_p, r;
    int* out;      // [0] token, [1] kept count
    float* p;      // [n] scratch
    uint32_t* gk;  // [2][n] global sort buffers
    int* gi;
};

__device__ float block_max(float v, float* red) {   // `o > v` semantics: NaN never wins
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o >= 1; o >>= 1) {
        const float x = __shfl_xor_sync(0xffffffffu, v, o);
        v = x > v ? x : v;
    }
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < SP_THREADS / 32; ++w) m = red[w] > m ? red[w] : m;
    __syncthreads();
    return m;
}

__device__ int block_min_int(int v, int* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o >= 1; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    int m = red[0];
    for (int w = 1; w < SP_THREADS / 32; ++w) m = min(m, red[w]);
    __syncthreads();
    return m;
}

__device__ int block_sum_int(int v, int* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    int s = 0;
    for (int w = 0; w < SP_THREADS / 32; ++w) s += red[w];
    __syncthreads();
    return s;
}

// Exclusive scan of a[0 .. 16 * 1024) in place (16 consecutive entries per thread).
__device__ void block_scan16(int* a, int* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int v[16], s = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v[i] = s;
        s += a[16 * tid + i];
    }
    int x = s;   // inclusive warp scan of thread totals
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) red[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = red[lane];
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        red[lane] = w;   // inclusive over warps
    }
    __syncthreads();
    const int base = (warp ? red[warp - 1] : 0) + x - s;
#pragma unroll
    for (int i = 0; i < 16; ++i) a[16 * tid + i] = base + v[i];
    __syncthreads();
}

// Stable ascending LSD radix sort (8 passes of 4 bits) of (k, i)[0..m) by `nthr` threads,
// each owning a contiguous range; ping-pong between (k0, i0) and (k1, i1); the result ends
// in (k0, i0).  cnt: shared [16][1024].
__device__ void radix_sort(uint32_t* k0, int* i0, uint32_t* k1, int* i1, int m, int nthr, int* cnt, int* red) {
    const int tid = threadIdx.x;
    const bool part = tid < nthr;
    const int L = (m + nthr - 1) / nthr, b = min(m, tid * L), e = min(m, b + L);
    for (int pass = 0; pass < 8; ++pass) {
        const uint32_t* ks = (pass & 1) ? k1 : k0;
        const int* is = (pass & 1) ? i1 : i0;
        uint32_t* kd = (pass & 1) ? k0 : k1;
        int* id = (pass & 1) ? i0 : i1;
        const int sh = 4 * pass;
        for (int d = 0; d < 16; ++d) cnt[d * SP_THREADS + tid] = 0;
        if (part)
            for (int k = b; k < e; ++k) ++cnt[((ks[k] >> sh) & 15) * SP_THREADS + tid];
        __syncthreads();
        block_scan16(cnt, red);   // digit-major, thread-minor: stable order
        if (part)
            for (int k = b; k < e; ++k) {
                const uint32_t key = ks[k];
                const int pos = cnt[((key >> sh) & 15) * SP_THREADS + tid]++;
                kd[pos] = key;
                id[pos] = is[k];
            }
        __syncthreads();
    }
}

// Blocked running sums over f(0..m) (f: position -> value, read twice): returns, via
// `hit`, the first position whose running value satisfies pred, and its running value.
template <typename F, typename P>
__device__ void blocked_first(int m, F f, P pred, float* T, float* E, int* red, int& hit, float& hit_val,
                              float& last_val) {
    const int tid = threadIdx.x, L = (m + SP_THREADS - 1) / SP_THREADS;
    const int b = min(m, tid * L), e = min(m, b + L);
    float t = 0.0f;
    for (int k = b; k < e; ++k) t = __fadd_rn(t, f(k));
    T[tid] = t;
    __syncthreads();
    if (tid == 0) {   // sequential prefix of the range totals
        float s = 0.0f;
        for (int c = 0; c < SP_THREADS; ++c) {
            E[c] = s;
            s = __fadd_rn(s, T[c]);
        }
    }
    __syncthreads();
    float cur = E[tid];
    int mine = 0x7fffffff;
    float mv = 0.0f;
    for (int k = b; k < e; ++k) {
        cur = __fadd_rn(cur, f(k));
        if (mine == 0x7fffffff && pred(cur)) mine = k, mv = cur;
    }
    if (b < e && e == m) reinterpret_cast<float*>(red)[40] = cur;   // running value at m - 1
    const int first = block_min_int(mine, red);
    if (first != 0x7fffffff && mine == first) reinterpret_cast<float*>(red)[41] = mv;
    __syncthreads();
    hit = first;
    hit_val = reinterpret_cast<float*>(red)[41];
    last_val = reinterpret_cast<float*>(red)[40];
    __syncthreads();
}

__global__ void __launch_bounds__(SP_THREADS, 1) k_sample_top_p(const SampleArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    float* T = reinterpret_cast<float*>(sm + SPS_T);
    float* E = reinterpret_cast<float*>(sm + SPS_E);
    int* red = reinterpret_cast<int*>(sm + SPS_RED);
    int* hcnt = reinterpret_cast<int*>(sm + SPS_HIST);
    float* hsum = reinterpret_cast<float*>(sm + SPS_HIST + 4 * 256);
    int* cnt = reinterpret_cast<int*>(sm + SPS_CNT);
    uint32_t* ck = reinterpret_cast<uint32_t*>(sm + SPS_K);
    int* ci = reinterpret_cast<int*>(sm + SPS_I);
    const int n = a.n, tid = threadIdx.x;
    const bool apply = a.temp != 1.0f && a.temp > 0.0f;
    const float inv_temp = a.temp > 0.0f ? __fdiv_rn(1.0f, a.temp) : 1.0f;
    auto val = [&](int i) { return apply ? __fmul_rn(a.logits[i], inv_temp) : a.logits[i]; };
    // max and e
    float m = -1e9f;
    for (int i = tid; i < n; i += SP_THREADS) {
        const float v = val(i);
        m = v > m ? v : m;
    }
    const float M = block_max(m, reinterpret_cast<float*>(red));
    for (int i = tid; i < n; i += SP_THREADS) a.p[i] = canon_expf(__fsub_rn(val(i), M));
    __syncthreads();
    int hit;
    float hv, S;
    blocked_first(n, [&](int k) { return a.p[k]; }, [](float) { return false; }, T, E, red, hit, hv, S);
    for (int i = tid; i < n; i += SP_THREADS) a.p[i] = __fdiv_rn(a.p[i], S);
    __syncthreads();
    int token, kept = n;
    if (a.top_p > 0.0f && a.top_p < 1.0f) {
        // threshold on the probability bits holding (approximately) top_p + 1e-3 of the mass
        const float target = a.top_p + 1e-3f;
        uint32_t prefix = 0u;
        int above = 0;
        float above_sum = 0.0f;
        bool all = false;
        for (int pass = 0; pass < 2 && !all; ++pass) {
            const int sh = pass ? 16 : 24;
            for (int i = tid; i < 256; i += SP_THREADS) hcnt[i] = 0, hsum[i] = 0.0f;
            __syncthreads();
            for (int i = tid; i < n; i += SP_THREADS) {
                const uint32_t kb = __float_as_uint(a.p[i]);
                if (pass == 0 || (kb >> 24) == (prefix >> 24)) {
                    atomicAdd(&hcnt[(kb >> sh) & 255], 1);
                    atomicAdd(&hsum[(kb >> sh) & 255], a.p[i]);
                }
            }
            __syncthreads();
            if (tid == 0) {
                int bin = -1;
                for (int d = 255; d >= 0; --d) {
                    above += hcnt[d];
                    above_sum += hsum[d];
                    if (above_sum >= target) {
                        bin = d;
                        break;
                    }
                }
                red[50] = bin;
            }
            __syncthreads();
            const int bin = red[50];
            if (bin < 0) {
                all = true;   // the histogram never reached the target: every position is a candidate
            } else {
                prefix |= static_cast<uint32_t>(bin) << sh;
                if (tid == 0) {   // back off to the bin's start for the next refinement
                    above -= hcnt[bin];
                    above_sum -= hsum[bin];
                }
            }
            __syncthreads();
        }
        const uint32_t tau = all ? 0u : prefix;
        // count and compact the candidates in index order
        const int L = (n + SP_THREADS - 1) / SP_THREADS, b = min(n, tid * L), e = min(n, b + L);
        int mine = 0;
        for (int i = b; i < e; ++i) mine += __float_as_uint(a.p[i]) >= tau;
        const int count = block_sum_int(mine, red);
        for (int attempt = 0; attempt < 2; ++attempt) {
            const bool in_smem = attempt == 0 && count <= SP_CAP;
            if (attempt == 0 && !in_smem) continue;
            const uint32_t t = attempt == 0 ? tau : 0u;
            const int mcount = attempt == 0 ? count : n;
            uint32_t* k0 = in_smem ? ck : a.gk;
            int* i0 = in_smem ? ci : a.gi;
            uint32_t* k1 = in_smem ? ck + SP_CAP : a.gk + n;
            int* i1 = in_smem ? ci + SP_CAP : a.gi + n;
            // exclusive position of this thread's range among the candidates
            int c = 0;
            for (int i = b; i < e; ++i) c += __float_as_uint(a.p[i]) >= t;
            for (int d = 0; d < 16; ++d) cnt[16 * tid + d] = d == 0 ? c : 0;
            __syncthreads();
            block_scan16(cnt, red);
            int pos = cnt[16 * tid];
            for (int i = b; i < e; ++i) {
                const uint32_t kb = __float_as_uint(a.p[i]);
                if (kb >= t) k0[pos] = ~kb, i0[pos] = i, ++pos;   // ascending ~bits = descending p
            }
            __syncthreads();
            radix_sort(k0, i0, k1, i1, mcount, in_smem ? 256 : SP_THREADS, cnt, red);
            // shortest prefix whose blocked running sum (ranges of the full n) reaches top_p
            const float tp = a.top_p;
            int K = -1;
            float C = 0.0f;
            {
                // ranges over n positions; positions >= mcount lie beyond the candidates
                const int Ln = (n + SP_THREADS - 1) / SP_THREADS;
                const int rb = min(mcount, tid * Ln), re = min(mcount, tid * Ln + Ln);
                float tt = 0.0f;
                for (int k = rb; k < re; ++k) tt = __fadd_rn(tt, __uint_as_float(~k0[k]));
                T[tid] = tt;
                __syncthreads();
                if (tid == 0) {
                    float s = 0.0f;
                    for (int q = 0; q < SP_THREADS; ++q) {
                        E[q] = s;
                        s = __fadd_rn(s, T[q]);
                    }
                }
                __syncthreads();
                float cur = E[tid];
                int first = 0x7fffffff;
                float fv = 0.0f;
                for (int k = rb; k < re; ++k) {
                    cur = __fadd_rn(cur, __uint_as_float(~k0[k]));
                    if (first == 0x7fffffff && cur >= tp) first = k, fv = cur;
                }
                if (rb < re && re == mcount) reinterpret_cast<float*>(red)[40] = cur;
                const int f = block_min_int(first, red);
                if (f != 0x7fffffff && first == f) reinterpret_cast<float*>(red)[41] = fv;
                __syncthreads();
                if (f != 0x7fffffff) {
                    K = f + 1;
                    C = reinterpret_cast<float*>(red)[41];
                } else if (mcount == n) {
                    K = n;
                    C = reinterpret_cast<float*>(red)[40];
                }
                // A cut inside a range that extends past the candidates is still exact: its
                // prefix comes from complete earlier ranges and its running values before the
                // cut from candidate positions only.  A miss means the candidates were too
                // few (approximate histogram sums): retry with every position.
                __syncthreads();
            }
            if (K < 0) continue;
            // walk: first kept position whose blocked running sum of p / C is >= r
            blocked_first(K, [&](int k) { return __fdiv_rn(__uint_as_float(~k0[k]), C); },
                          [&](float cur) { return a.r <= cur; }, T, E, red, hit, hv, S);
            token = i0[hit != 0x7fffffff ? hit : K - 1];
            kept = K;
            break;
        }
    } else {
        blocked_first(n, [&](int k) { return a.p[k]; }, [&](float cur) { return a.r <= cur; }, T, E, red, hit, hv, S);
        token = hit != 0x7fffffff ? hit : n - 1;
    }
    if (tid == 0) {
        a.out[0] = token;
        a.out[1] = kept;
    }
}

}  // namespace

cudaError_t launch_sample_top_p(const float* logits, int n, float temperature, float top_p, float r, int* out, float* p,
                                uint32_t* gk, int* gi, cudaStream_t stream) {
    static int prepared_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (prepared_dev != dev) {
        const cudaError_t e = cudaFuncSetAttribute(k_sample_top_p, cudaFuncAttributeMaxDynamicSharedMemorySize, SPS_BYTES);
        if (e != cudaSuccess) return e;
        prepared_dev = dev;
    }
    SampleArgs a{logits, n, temperature, top_p, r, out, p, gk, gi};
    k_sample_top_p<<<1, SP_THREADS, SPS_BYTES, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace mcpm
