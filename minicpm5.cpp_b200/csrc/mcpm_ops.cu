// Standalone kernels behind the op entry points of include/mcpm.h: Q8_K quantisation,
// quantised GEMV (and its integer block sums), RMSNorm->Q8_K and SwiGLU->Q8_K.  They use
// the same device functions as the decode kernel, so the per-op parity tests cover the
// decode path's arithmetic.
#include "mcpm_device.cuh"
#include "mcpm_gemv_bo.cuh"
#include "mcpm_internal.h"
#include "mcpm_q80.cuh"

namespace mcpm {
namespace {

constexpr int OP_THREADS = 512;
constexpr int RING_SLOTS = 4;
constexpr int SLOT_BYTES = 49152;
constexpr int SLOT_STRIDE = SLOT_BYTES + 128;   // readable tail for unaligned Q6_K reads

__global__ void k_quantize_q8k(const float* __restrict__ x, uint8_t* __restrict__ y, int nblocks, int away) {
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;   // whole warp
    const int lane = threadIdx.x & 31;
    const float4 a = *reinterpret_cast<const float4*>(x + 256 * b + 8 * lane);
    const float4 c = *reinterpret_cast<const float4*>(x + 256 * b + 8 * lane + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    uint8_t* blk = y + static_cast<size_t>(b) * Q8K_BYTES;
    if (away)
        quant_block_warp<true>(v, reinterpret_cast<int8_t*>(blk + 4), reinterpret_cast<float*>(blk),
                               reinterpret_cast<int16_t*>(blk + 260));
    else
        quant_block_warp<false>(v, reinterpret_cast<int8_t*>(blk + 4), reinterpret_cast<float*>(blk),
                                reinterpret_cast<int16_t*>(blk + 260));
}

__global__ void k_swiglu_q8k(const float* __restrict__ g, const float* __restrict__ u, uint8_t* __restrict__ y,
                             int nblocks) {
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const int lane = threadIdx.x & 31;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = canon_silu_mul(g[256 * b + 8 * lane + k], u[256 * b + 8 * lane + k]);
    uint8_t* blk = y + static_cast<size_t>(b) * Q8K_BYTES;
    quant_block_warp<true>(v, reinterpret_cast<int8_t*>(blk + 4), reinterpret_cast<float*>(blk),
                           reinterpret_cast<int16_t*>(blk + 260));
}

// n == 2048, one CTA of 256 threads.
__global__ void k_rmsnorm_q8k(const float* __restrict__ x, const float* __restrict__ w, uint8_t* __restrict__ y,
                              float eps) {
    __shared__ float red[8];
    const int tid = threadIdx.x;
    float xv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = x[tid + 256 * i];
    const float ss = sumsq_2048(xv, red);
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 2048.0f), eps)));
    const int warp = tid >> 5, lane = tid & 31;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int i = 256 * warp + 8 * lane + k;
        v[k] = __fmul_rn(__fmul_rn(x[i], w[i]), rms);
    }
    uint8_t* blk = y + static_cast<size_t>(warp) * Q8K_BYTES;
    quant_block_warp<true>(v, reinterpret_cast<int8_t*>(blk + 4), reinterpret_cast<float*>(blk),
                           reinterpret_cast<int16_t*>(blk + 260));
}

// Quantised GEMV: each CTA streams a contiguous row range through a 4-slot TMA ring.
// isum/aux != null selects the block-sum probe (integer partials only).
__global__ void __launch_bounds__(OP_THREADS, 1)
    k_gemv(int type, const uint8_t* __restrict__ w, const uint8_t* __restrict__ xq_g, float* __restrict__ y,
           int32_t* __restrict__ isum, int32_t* __restrict__ aux, int rows, int nb, int blk_order, unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* ring = smem_raw;
    XQSmem* xq = reinterpret_cast<XQSmem*>(ring + RING_SLOTS * SLOT_STRIDE);
    int* part = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(xq) + ((sizeof(XQSmem) + 127) & ~size_t(127)));
    float* rowval = reinterpret_cast<float*>(part + MAX_TASKS * PART_WORDS);
    uint64_t* bars = reinterpret_cast<uint64_t*>(rowval + MAX_TASKS);

    const int tid = threadIdx.x;
    const int rb = row_bytes(type, nb * 256);
    const int sr = min(SLOT_BYTES / rb, MAX_TASKS / nb);
    const int r0 = static_cast<int>((static_cast<long long>(rows) * blockIdx.x) / gridDim.x);
    const int r1 = static_cast<int>((static_cast<long long>(rows) * (blockIdx.x + 1)) / gridDim.x);
    const int nstages = (r1 - r0 + sr - 1) / sr;

    for (int i = tid; i < nb * 64; i += blockDim.x) {
        const int b = i >> 6, wd = i & 63;
        reinterpret_cast<uint32_t*>(xq->qs[b])[wd] =
            reinterpret_cast<const uint32_t*>(xq_g + static_cast<size_t>(b) * Q8K_BYTES + 4)[wd];
    }
    for (int i = tid; i < nb * 8; i += blockDim.x) {
        const int b = i >> 3, wd = i & 7;
        reinterpret_cast<uint32_t*>(xq->bsums[b])[wd] =
            reinterpret_cast<const uint32_t*>(xq_g + static_cast<size_t>(b) * Q8K_BYTES + 260)[wd];
    }
    if (tid < nb) xq->d[tid] = *reinterpret_cast<const float*>(xq_g + static_cast<size_t>(tid) * Q8K_BYTES);
    auto issue = [&](int st) {
        const int slot = st % RING_SLOTS, a = r0 + st * sr, n = min(sr, r1 - a);
        const uint32_t bytes = static_cast<uint32_t>(n) * rb;
        mbar_expect_tx(&bars[slot], bytes);
        bulk_g2s(ring + slot * SLOT_STRIDE, w + static_cast<size_t>(a) * rb, bytes, &bars[slot]);
    };
    if (tid == 0) {
        for (int i = 0; i < RING_SLOTS; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
        for (int st = 0; st < min(nstages, RING_SLOTS); ++st) issue(st);
    }
    __syncthreads();
    for (int st = 0; st < nstages; ++st) {
        const int slot = st % RING_SLOTS, a = r0 + st * sr, n = min(sr, r1 - a);
        const uint8_t* sw = ring + slot * SLOT_STRIDE;
        const bool ok = mbar_wait(&bars[slot], (st / RING_SLOTS) & 1, err);
        if (__syncthreads_or(!ok)) return;
        if (isum) {
            const int bb = block_bytes(type);
            for (int t = tid; t < n * nb; t += blockDim.x) {
                Partials pp;
                if (type == GGML_Q4_K)
                    q4k_task(sw + static_cast<size_t>(t) * bb, *xq, t % nb, pp);
                else
                    q6k_task(sw + static_cast<size_t>(t) * bb, *xq, t % nb, pp);
                int tot = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) tot += pp.k[k];
                const size_t o = static_cast<size_t>(a) * nb + t;
                isum[o] = type == GGML_Q6_K ? tot + pp.minsum : tot;
                aux[o] = pp.minsum;
            }
            __syncthreads();
        } else {
            if (blk_order)
                gemv_bo(type, sw, n, nb, *xq, part, MAX_TASKS * PART_WORDS, rowval);
            else
                gemv_rows(type, sw, n, nb, *xq, part, MAX_TASKS, rowval);
            if (tid < n) y[a + tid] = rowval[tid];
        }
        if (tid == 0 && st + RING_SLOTS < nstages) issue(st + RING_SLOTS);
    }
}

// ---- Q8_0 x fp32 GEMV (mcpm_q80.cuh): each CTA streams a contiguous row range.
__global__ void __launch_bounds__(Q80_THREADS, 1)
    k_gemv_q8_0(const uint8_t* __restrict__ w, const float* __restrict__ x, float* __restrict__ y, int rows, int nb,
                unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const Q80Smem s(smem_raw);
    const int tid = threadIdx.x, cols = nb * 32;
    const int sr = q80_pick_stage(nb, (rows + gridDim.x - 1) / gridDim.x);
    const int r0 = (rows * blockIdx.x) / gridDim.x, r1 = (rows * (blockIdx.x + 1)) / gridDim.x;
    if (tid == 0) q80_start(w, r0, r1, nb, sr, s);
    for (int i = tid; i < cols / 4; i += blockDim.x)
        *reinterpret_cast<float4*>(s.xs + q80_xpos(4 * i)) = reinterpret_cast<const float4*>(x)[i];
    __syncthreads();
    q80_run(w, r0, r1, nb, sr, s, err, [&](int r, float v, float) { y[r] = v; });
}

size_t gemv_q8_0_smem_bytes() { return q80_smem_bytes(); }

size_t gemv_smem_bytes() {
    return RING_SLOTS * SLOT_STRIDE + ((sizeof(XQSmem) + 127) & ~size_t(127)) + MAX_TASKS * PART_WORDS * 4 +
           MAX_TASKS * 4 + RING_SLOTS * 8;
}

int g_num_sms = 0;

}  // namespace

cudaError_t op_gemv_q8_0(const void* w, const float* x, float* y, int rows, int cols, cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool prepared[64] = {};
    static unsigned* d_err[64] = {};
    static int n_sms[64] = {};
    if (dev >= 64) return cudaErrorInvalidDevice;
    if (!prepared[dev]) {
        e = cudaFuncSetAttribute(k_gemv_q8_0, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(gemv_q8_0_smem_bytes()));
        if (e != cudaSuccess) return e;
        cudaDeviceGetAttribute(&n_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        e = cudaMalloc(&d_err[dev], sizeof(unsigned));
        if (e != cudaSuccess) return e;
        cudaMemset(d_err[dev], 0, sizeof(unsigned));
        prepared[dev] = true;
    }
    const int grid = rows < n_sms[dev] ? rows : n_sms[dev];
    k_gemv_q8_0<<<grid, Q80_THREADS, gemv_q8_0_smem_bytes(), s>>>(static_cast<const uint8_t*>(w), x, y, rows, cols / 32,
                                                                  d_err[dev]);
    return cudaGetLastError();
}

cudaError_t op_quantize_q8k(const float* x, void* y, int n, int rounding, cudaStream_t s) {
    const int nblocks = n / 256;
    k_quantize_q8k<<<(nblocks + 7) / 8, 256, 0, s>>>(x, static_cast<uint8_t*>(y), nblocks, rounding);
    return cudaGetLastError();
}

cudaError_t op_swiglu_q8k(const float* g, const float* u, void* out, int n, cudaStream_t s) {
    const int nblocks = n / 256;
    k_swiglu_q8k<<<(nblocks + 7) / 8, 256, 0, s>>>(g, u, static_cast<uint8_t*>(out), nblocks);
    return cudaGetLastError();
}

namespace {
// RoPE factors of one position (host C library, the same table the decode engine uses).
struct RopeRow {
    float2 cs[HEAD_DIM / 2];
};

// apply_rope (ops.cpp:502-516) on the 16 query heads and 2 key heads, pair (2i, 2i+1) of a
// head rotated by factor i, with the reference build's contraction (one fma per output), then
// the K and V rows written at `pos` of the cache (execute_attention, ops.cpp:557-563).
__global__ void k_rope_kv_append(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                                 float* __restrict__ kc, float* __restrict__ vc, int pos, const RopeRow rr) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;   // pair index over [q pairs; k pairs]
    constexpr int QP = N_EMBD / 2, KP = KV_DIM / 2;
    if (t < QP + KP) {
        float* vec = t < QP ? q + 2 * t : k + 2 * (t - QP);
        const int i = (t < QP ? t : t - QP) & (HEAD_DIM / 2 - 1);
        const float2 c = rr.cs[i];
        const float v0 = vec[0], v1 = vec[1];
        const float r0 = __fmaf_rn(c.x, v0, -__fmul_rn(c.y, v1));
        const float r1 = __fmaf_rn(c.y, v0, __fmul_rn(c.x, v1));
        vec[0] = r0;
        vec[1] = r1;
        if (t >= QP) {
            float* kd = kc + static_cast<size_t>(pos) * KV_DIM + 2 * (t - QP);
            kd[0] = r0;
            kd[1] = r1;
        }
    }
    if (t < KV_DIM) vc[static_cast<size_t>(pos) * KV_DIM + t] = v[t];
}
}  // namespace

cudaError_t op_rope_kv_append(float* q, float* k, const float* v, float* kc, float* vc, int pos, float base,
                              cudaStream_t s) {
    RopeRow rr;
    rope_row(pos, base, rr.cs);
    constexpr int pairs = N_EMBD / 2 + KV_DIM / 2;
    k_rope_kv_append<<<(pairs + 255) / 256, 256, 0, s>>>(q, k, v, kc, vc, pos, rr);
    return cudaGetLastError();
}

cudaError_t op_rmsnorm_q8k(const float* x, const float* w, void* out, float eps, cudaStream_t s) {
    k_rmsnorm_q8k<<<1, 256, 0, s>>>(x, w, static_cast<uint8_t*>(out), eps);
    return cudaGetLastError();
}

cudaError_t op_gemv_q8k(int type, const void* w, const void* xq, float* y, int32_t* isum, int32_t* aux, int rows,
                        int cols, int blk_order, cudaStream_t s) {
    static bool prepared = false;
    static unsigned* d_err = nullptr;
    if (!prepared) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(gemv_smem_bytes()));
        if (e != cudaSuccess) return e;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        e = cudaMalloc(&d_err, sizeof(unsigned));
        if (e != cudaSuccess) return e;
        cudaMemset(d_err, 0, sizeof(unsigned));
        prepared = true;
    }
    const int nb = cols / 256;
    const int grid = rows < g_num_sms ? rows : g_num_sms;
    k_gemv<<<grid, OP_THREADS, gemv_smem_bytes(), s>>>(type, static_cast<const uint8_t*>(w),
                                                        static_cast<const uint8_t*>(xq), y, isum, aux, rows, nb, blk_order,
                                                        d_err);
    return cudaGetLastError();
}

}  // namespace mcpm
