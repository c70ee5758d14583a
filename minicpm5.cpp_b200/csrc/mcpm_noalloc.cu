// mcpm_attention_noalloc: the GQA attention op for callers that cannot allocate device
// memory.
//
// Some hosts embed the engine where cudaMalloc is not available to them: code that runs
// while a CUDA graph is being captured on the device it owns, plug-ins whose host process
// owns every allocation through its own pool, and real-time loops that must not touch the
// allocator after start-up.  mcpm_attention obtains its split-KV workspace with cudaMalloc
// on its first call; this variant uses a fixed workspace that lives in this library's
// static device memory instead, so no call ever allocates.
//
// The workspace below is the chunk records of 16 query heads x 64 chunks (a 16-byte
// header and 128 floats each, 540,672 bytes) and a Q8_K sink: enough for any context up
// to MAX_SEQ = 16384 positions.  Every GPU that loads the library holds it until the
// process exits.  All calls on a device share it, so calls that overlap on the GPU race
// and must be serialised by the caller (one stream, or events).
#include <cstdio>
#include <mutex>

#include "../../include/mcpm.h"
#include "mcpm_device.cuh"
#include "mcpm_internal.h"

using namespace mcpm;

namespace {

static __device__ __align__(256) float g_att_part[ATT_PART_FLOATS];
static __device__ __align__(256) uint8_t g_att_q8k[(N_EMBD / 256) * Q8K_BYTES];

// Device addresses of the arrays above, looked up once per device.  In host code the
// array names are host-side stand-ins, never device addresses.
struct ScratchAddr {
    bool ready = false;
    float* part = nullptr;
    uint8_t* q8k = nullptr;
};
ScratchAddr g_addr[64];
std::mutex g_addr_mu;   // host threads making their first call on one device at the same time

mcpm_status setup_scratch(int dev) {
    std::lock_guard<std::mutex> lock(g_addr_mu);
    ScratchAddr& a = g_addr[dev];
    if (a.ready) return MCPM_OK;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&a.part), g_att_part) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&a.q8k), g_att_q8k) != cudaSuccess) {
        std::fprintf(stderr, "[mcpm] mcpm_attention_noalloc: cudaGetSymbolAddress failed on device %d\n", dev);
        return MCPM_CUDA_ERROR;
    }
    a.ready = true;
    return MCPM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" mcpm_status mcpm_attention_noalloc(const float* q, const float* k, const float* v, float* kcache,
                                              float* vcache, int pos, int max_seq, float* out, void* out_q8k,
                                              void* stream) {
    if (!q || !k || !v || !kcache || !vcache || !out || !aligned16(q) || !aligned16(kcache) || !aligned16(vcache))
        return MCPM_BAD_ARG;
    // Same checks in the same order as mcpm_attention, so both ops return the same status
    // for the same arguments: the cache size first, then the position.
    if (max_seq <= 0) return MCPM_BAD_ARG;
    if (max_seq > MAX_SEQ) {
        std::fprintf(stderr,
                     "[mcpm] mcpm_attention_noalloc: cache of %d positions exceeds the fixed workspace limit of %d "
                     "positions\n",
                     max_seq, MAX_SEQ);
        return MCPM_BAD_ARG;
    }
    if (pos < 0 || pos >= max_seq) return MCPM_CTX_OVERFLOW;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MCPM_CUDA_ERROR;
    const mcpm_status st = setup_scratch(dev);
    if (st != MCPM_OK) return st;
    const ScratchAddr& a = g_addr[dev];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = launch_attention(q, k, v, kcache, vcache, pos, max_seq, out,
                                           out_q8k ? static_cast<uint8_t*>(out_q8k) : a.q8k, a.part, s);
    return e == cudaSuccess ? MCPM_OK : MCPM_CUDA_ERROR;
}
