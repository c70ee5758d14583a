/* mcpm.h -- C ABI of the B200 MiniCPM5 decode engine.
 *
 * Drop-in boundary for the reference's hot path (astrowar/MiniCPM5.cpp):
 *   engine : class MiniCPM5Engine           include/model.h:37-70, src/model.cpp:17-242
 *   ops    : quantised GEMV / norm / SwiGLU include/ops.h:113-160, src/ops/ops_internal.h:15-54
 * Plain pointers and sizes only.  Every function returns an mcpm_status; nothing throws
 * across the ABI and nothing is silently zero-filled (the reference prints a warning and
 * fills outputs with 0 / 0.001 on unsupported input, src/ops/ops.cpp:281-289, 341-348).
 *
 * Device-pointer functions take a CUDA stream as `void*` (NULL = legacy default stream)
 * and are asynchronous with respect to the host.  Engine functions are synchronous
 * unless their name ends in _async.
 */
#ifndef MCPM_H
#define MCPM_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MCPM_OK = 0,
    MCPM_BAD_ARG = 1,          /* null pointer, size not a multiple of the block, ... */
    MCPM_BAD_FILE = 2,         /* unreadable / truncated / malformed GGUF, wrong architecture */
    MCPM_UNSUPPORTED_TYPE = 3, /* tensor type the path does not handle */
    MCPM_CTX_OVERFLOW = 4,     /* pos >= max_seq (reference: warning + stale output, ops.cpp:550-553) */
    MCPM_CUDA_ERROR = 5,
    MCPM_NCCL_ERROR = 6,
    MCPM_TIMEOUT = 7,          /* a bounded device-side wait gave up */
    MCPM_OUT_OF_MEMORY = 8,
    MCPM_BAD_TOKEN = 9,        /* token id outside [0, n_vocab) */
    MCPM_NOT_LOADED = 10       /* engine call before mcpm_load_gguf / mcpm_init_kv */
} mcpm_status;

const char* mcpm_status_string(mcpm_status s);

/* ------------------------------------------------------------------ engine */
typedef struct mcpm_engine mcpm_engine;

enum { MCPM_GEMM_TCGEN05 = 0, MCPM_GEMM_MMA = 1 };
typedef struct {
    int device;      /* CUDA device ordinal */
    int max_seq;     /* KV-cache positions (reference init_kv_cache(max_seq_len), model.cpp:17-24); <= 16384 */
    int n_ctas;      /* persistent CTAs of the decode kernel; 0 = one per SM */
    int batch_gemm;  /* the engine's GEMV order and batched GEMM, for decode (mcpm_forward), batched decode
                        (mcpm_batch_*) and prompt prefill (mcpm_prefill): MCPM_GEMM_TCGEN05 (0, the
                        default and the faster) computes every (row, super-block) integer sum exactly and
                        scales it with one fp32 fma per block in groups of four blocks -- the decode
                        kernel's GEMVs and the 5th-generation tensor-core GEMM of batched decode and
                        prefill; MCPM_GEMM_MMA (1) keeps the reference's eight-lane AVX2 order
                        (dot_row_q*_K_q8_K_avx2) -- the decode kernel's eight-lane GEMVs and int8
                        mma.sync batched GEMMs.  Either way a prefilled prompt gives the same bits as
                        one mcpm_forward per position, and the two orders differ by a few ulps per row */
    int sched;       /* decode schedule options, for measurement: MCPM_SCHED_L2_PREFETCH (1) prefetches each
                        layer's weight rows into L2 one layer ahead; MCPM_SCHED_ATT_COMBINERS (2) combines
                        the attention chunks on 8 head-pair CTAs at every context length (by default only
                        above 16 chunks; below, every CTA combines all heads); MCPM_SCHED_EARLY_GU (4) copies
                        the gate/up rows during attention instead of after it; every option gives the
                        same results */
    int kv_type;     /* KV-cache element type: MCPM_KV_F32 (0, the reference's std::vector<float> cache,
                        model.h:66-67) or MCPM_KV_F16 (1: K and V rounded to fp16 when written, half the
                        cache bytes; the attention reads them back exactly and computes in fp32) */
    int reserved[2];
} mcpm_config;
enum { MCPM_SCHED_L2_PREFETCH = 1, MCPM_SCHED_ATT_COMBINERS = 2, MCPM_SCHED_EARLY_GU = 4 };
enum { MCPM_KV_F32 = 0, MCPM_KV_F16 = 1 };

/* Creates an engine bound to cfg->device (MiniCPM5Engine constructor + init_kv_cache). */
mcpm_status mcpm_engine_create(const mcpm_config* cfg, mcpm_engine** out);
/* Parses the GGUF header, checks the MiniCPM5 tensor set, uploads every tensor's bytes
 * unchanged into one HBM arena, builds the RoPE table and allocates the KV cache.
 * Replaces MiniCPM5Engine::load_model (model.cpp:33-133). */
mcpm_status mcpm_load_gguf(mcpm_engine* e, const char* path);
/* (Re)allocates and zeroes the fp32 KV cache, layout [layer][pos][kv_head][head_dim]
 * (reference KVCacheLayer, include/ops.h:147-150; init_kv_cache, model.cpp:17-24). */
mcpm_status mcpm_init_kv(mcpm_engine* e, int max_seq);
/* One decode step: embeds `token` at position `pos`, runs every layer, appends K/V at
 * pos.  logits_out (host, n_vocab floats) and argmax_out (host) are optional.  Replaces
 * MiniCPM5Engine::forward(token_id, pos, max_seq_len) (model.cpp:142-242); the greedy
 * argmax (lowest index on ties) is computed on the device.  token < 0 uses the argmax
 * that the previous step left on the device. */
mcpm_status mcpm_forward(mcpm_engine* e, int token, int pos, float* logits_out, int* argmax_out);
/* Asynchronous decode step on the engine's stream.  token < 0 reads the token id that the
 * previous step's argmax left on the device (greedy chaining without a host round trip).
 * write_logits = 0 skips the logits store.  Errors surface at the next mcpm_sync. */
mcpm_status mcpm_forward_async(mcpm_engine* e, int token, int pos, int write_logits);
mcpm_status mcpm_sync(mcpm_engine* e);
/* Device pointers of the last step's logits (n_vocab floats) and argmax (one int). */
const float* mcpm_logits_device(mcpm_engine* e);
const int* mcpm_argmax_device(mcpm_engine* e);
/* Internal state for parity checks: residual x (n_embd floats), one K and V row (widened to
 * fp32 from an fp16 cache). */
mcpm_status mcpm_read_x(mcpm_engine* e, float* x_host);
mcpm_status mcpm_read_kv(mcpm_engine* e, int layer, int pos, float* k_host, float* v_host);
/* Writes n_pos K and V rows ([n_pos][n_head_kv * head_dim] floats each) of one layer from
 * position pos0: restores a saved cache, or seeds one for a parity check of a late step.
 * An fp16 cache stores them rounded to nearest-even, as a decode step rounds its own rows. */
mcpm_status mcpm_write_kv(mcpm_engine* e, int layer, int pos0, int n_pos, const float* k_host, const float* v_host);
/* Session snapshot and restore (multi-turn sessions; the reference re-renders and
 * re-prefills the whole conversation every turn, src/chat_session.cpp:126-160).  A snapshot
 * holds the KV rows of positions [0, n_pos) of every layer, mcpm_kv_snapshot_bytes(e, n_pos)
 * bytes laid out [layer][K, V][pos][256] in the cache's element type (fp32, or fp16 with
 * kv_type MCPM_KV_F16; host memory).  After mcpm_kv_restore(e, n_pos, ...) -- into this engine
 * or another one with the same model, kv_type and max_seq >= n_pos -- decoding
 * or mcpm_prefill from position n_pos continues the session exactly as it was (the next step
 * depends only on the cache rows below its position and on its token).  Synchronous. */
size_t mcpm_kv_snapshot_bytes(mcpm_engine* e, int n_pos);
mcpm_status mcpm_kv_snapshot(mcpm_engine* e, int n_pos, void* host, size_t bytes);
mcpm_status mcpm_kv_restore(mcpm_engine* e, int n_pos, const void* host, size_t bytes);
/* Batched decode (the reference's forward once per sequence, for n_seq independent
 * sequences in lockstep).  mcpm_batch_init allocates a KV cache of max_seq positions for
 * each of n_seq <= 64 sequences (zeroed; positions restart at 0).  mcpm_batch_step_async
 * advances every sequence by one token on the engine's stream: tokens (host, n_seq ids) or
 * NULL for each sequence's previous greedy token; pos (host, n_seq) or NULL for the
 * previous positions + 1.  mcpm_batch_read waits and copies the last step's logits
 * ([n_seq][n_vocab], optional) and greedy tokens ([n_seq], optional). */
mcpm_status mcpm_batch_init(mcpm_engine* e, int n_seq, int max_seq);
/* Batched prefill of the engine's own sequence: positions pos0 .. pos0+n-1 of `tokens` (host,
 * n ids) in chunks of up to 64 positions, each chunk one batched step whose rows share the
 * engine's KV cache (row i attends to positions 0 .. pos0+i, causal), so every K/V row and
 * the last position's logits equal n calls of mcpm_forward bit for bit (the reference
 * prefills token by token, src/chat_session.cpp:154-160).  logits_out (host, n_vocab) and
 * argmax_out (host) receive the last position's logits and greedy token; the device keeps
 * them as a decode step would, so mcpm_sample and mcpm_forward(token < 0, pos0 + n) continue
 * from the prompt.  Synchronous.  Row buffers for 64 positions are allocated on the first
 * call and kept until the model is unloaded. */
mcpm_status mcpm_prefill(mcpm_engine* e, const int* tokens, int n, int pos0, float* logits_out, int* argmax_out);
mcpm_status mcpm_batch_step_async(mcpm_engine* e, const int* tokens, const int* pos);
mcpm_status mcpm_batch_read(mcpm_engine* e, float* logits, int* argmax);
/* Top-p sampling on the device (Sampler::sample, src/sampler.cpp:8-72): logits (device,
 * n <= 1048576 floats), temperature (applied when > 0 and != 1), top_p (truncation when in
 * (0, 1)), r: the uniform draw in [0, 1) (the reference draws it from mt19937 seeded by
 * random_device; here the caller supplies it).  out (device, 2 ints): the token and the number
 * of tokens kept.  Fixed canonical order (ties by index, blocked fp32 sums) shared with the C
 * restatement.  A per-device workspace is allocated on the first call. */
mcpm_status mcpm_sample_top_p(const float* logits, int n, float temperature, float top_p, float r, int* out,
                              void* stream);
/* Sampler::sample (src/sampler.cpp:8-72) on host logits: copies the n floats to the
 * device and runs mcpm_sample_top_p there (same canonical order, same draw r); writes the
 * token to *token_out (host).  Synchronous, on the current device. */
mcpm_status mcpm_sample_top_p_host(const float* logits, int n, float temperature, float top_p, float r,
                                   int* token_out);
/* Samples the last decode step's logits (the step must have written them) and makes the
 * token the next step's input (forward with token < 0).  token_out (host) is optional. */
mcpm_status mcpm_sample(mcpm_engine* e, float temperature, float top_p, float r, int* token_out);
/* n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab of the loaded model. */
mcpm_status mcpm_model_dims(mcpm_engine* e, int dims[6]);
/* Phase trace (no reference counterpart; the reference only times whole loops,
 * chat_session.cpp:152-187): when enabled, each decode step records globaltimer
 * nanoseconds on CTA 0 -- [0] kernel start, then per phase i (5 per layer: QKV, attention,
 * o_proj, gate/up, down) [2+2i] = its own work done, [3+2i] = grid barrier released, and
 * [2+2*(5*n_layer)] = LM head done.  mcpm_trace_read copies up to n words. */
mcpm_status mcpm_trace_enable(mcpm_engine* e, int enable);
mcpm_status mcpm_trace_read(mcpm_engine* e, unsigned long long* out, int n);
/* The engine's CUDA stream (cudaStream_t) and decode grid size. */
void* mcpm_engine_stream(mcpm_engine* e);
int mcpm_engine_n_ctas(mcpm_engine* e);
void mcpm_engine_destroy(mcpm_engine* e);

/* ------------------------------------------------------------------ tensor-parallel engine
 * Batch-1 decode of an all-Q8_0 model over `world` GPUs (1, 2, 4 or 8), one engine per GPU
 * (one process or host thread each).  The reference has no multi-GPU path; this is the
 * Megatron partition of MiniCPM5Engine::forward (model.cpp:142-242) with every projection
 * gemv_q8_0 (ops.cpp:58-79): QKV, Gate+Up and the LM head split by output rows, o_proj and
 * down by input columns, their partial sums exchanged between the ranks after each of the
 * two (84 exchanges per token for 42 layers), and the greedy argmax reduced over the ranks'
 * vocabulary slices.  Every rank returns the same token.
 * Setup: rank 0 makes an NCCL id (MCPM_TP_NCCL) or every rank makes an IPC handle of its
 * receive buffer after loading (MCPM_TP_P2P); the caller distributes them (any host
 * channel) and every rank calls mcpm_tp_connect with the full set. */
typedef struct mcpm_tp mcpm_tp;
enum { MCPM_TP_P2P = 0, MCPM_TP_NCCL = 1 };
typedef struct {
    int device;    /* CUDA device of this rank */
    int rank;      /* 0 .. world-1 */
    int world;     /* 1, 2, 4 or 8 */
    int max_seq;   /* KV-cache positions, <= 16384 */
    int comm;      /* MCPM_TP_P2P: epoch-tagged partial sums stored into every rank's receive
                      buffer over CUDA IPC and summed in rank order by the consuming kernel;
                      MCPM_TP_NCCL: ncclAllReduce / ncclAllGather (libnccl.so.2 at run time) */
    int eager;     /* 0: each token is one CUDA graph launch; 1: kernels launched one by one */
    int peer_wait_us; /* bound of every device-side wait for another rank's values, microseconds
                         (0: 5 s); a wait that runs out fails the step with MCPM_TIMEOUT */
    int reserved[1];
} mcpm_tp_config;
/* 128-byte NCCL unique id (rank 0, MCPM_TP_NCCL). */
mcpm_status mcpm_tp_nccl_id(void* id128);
mcpm_status mcpm_tp_create(const mcpm_tp_config* cfg, mcpm_tp** out);
/* Loads this rank's shards of an all-Q8_0 MiniCPM5 GGUF (MCPM_UNSUPPORTED_TYPE for other
 * mixes) and allocates its KV cache; the embedding and norms are replicated. */
mcpm_status mcpm_tp_load_gguf(mcpm_tp* t, const char* path);
/* 64-byte cudaIpcMemHandle_t of this rank's receive buffer (MCPM_TP_P2P, after load). */
mcpm_status mcpm_tp_ipc_handle(mcpm_tp* t, void* handle64);
/* nccl_id128: rank 0's id (MCPM_TP_NCCL); ipc_handles: world x 64 bytes in rank order
 * (MCPM_TP_P2P).  A single-GPU engine needs neither. */
mcpm_status mcpm_tp_connect(mcpm_tp* t, const void* nccl_id128, const void* ipc_handles);
/* One decode step on every rank (each rank calls it with the same arguments): token at pos,
 * or token < 0 for the previous step's greedy token at the next position.  logits_slice
 * (host, optional) receives this rank's vocabulary rows [lo, hi) (mcpm_tp_info);
 * next_token (host, optional) the greedy token over the whole vocabulary. */
mcpm_status mcpm_tp_forward(mcpm_tp* t, int token, int pos, float* logits_slice, int* next_token);
/* n greedy steps chained on the device after the last step, without host round trips;
 * mcpm_tp_read_tokens (which waits) returns the tokens, logged by the position whose step
 * produced them.  Errors surface at mcpm_tp_sync / mcpm_tp_read_tokens. */
mcpm_status mcpm_tp_generate_async(mcpm_tp* t, int n);
mcpm_status mcpm_tp_sync(mcpm_tp* t);
mcpm_status mcpm_tp_read_tokens(mcpm_tp* t, int pos0, int n, int* tokens);
/* n_layer, n_vocab, vocabulary rows [lo, hi), first query head and head count, first FFN
 * row and row count of this rank. */
mcpm_status mcpm_tp_info(mcpm_tp* t, int info[8]);
/* Zeroes the KV cache and the token log; positions restart at 0.  Also restarts the step
 * counter that tags exchanged values and clears this rank's receive slots, which is how the
 * ranks recover after MCPM_TIMEOUT: every rank calls mcpm_tp_reset between steps, and no rank
 * steps again before all have reset (a host-side barrier). */
mcpm_status mcpm_tp_reset(mcpm_tp* t);
/* n greedy steps launched kernel by kernel with timing: ms_token = mean device time per
 * step; ms_comm = per step, the device time of the NCCL collectives (MCPM_TP_NCCL) or the
 * time CTA 0 of the consuming kernels waited for the exchanged partials (MCPM_TP_P2P). */
mcpm_status mcpm_tp_profile(mcpm_tp* t, int n, float* ms_token, float* ms_comm);
/* The engine's CUDA stream (cudaStream_t). */
void* mcpm_tp_stream(mcpm_tp* t);
void mcpm_tp_destroy(mcpm_tp* t);

/* ------------------------------------------------------------------ ops (device pointers)
 * Block layouts are the reference's: block_q4_K 144 B, block_q6_K 210 B, block_q8_0 34 B,
 * block_q8_K 292 B (include/ops.h:33-65).  `type` is the ggml type id (12 = Q4_K,
 * 14 = Q6_K).  `rows` x `cols` is the matrix shape (GGUF dims[1] x dims[0]); weight
 * pointers must be 16-byte aligned and cols <= 6144 (Q6_K: cols % 2048 == 0).
 */
enum { MCPM_ROUND_EVEN = 0, MCPM_ROUND_AWAY = 1 };

/* fp32 -> Q8_K.  MCPM_ROUND_EVEN: quantize_row_q8_K_avx2 (ops_avx2.cpp:85-144);
 * MCPM_ROUND_AWAY: the lround quantisers of ops.cpp:702-722.  n % 256 == 0. */
mcpm_status mcpm_quantize_q8k(const float* x, void* y, int n, int rounding, void* stream);
/* y = W xq for Q4_K / Q6_K weights: gemv_q4_K_q8_K_avx2 / gemv_q6_K_q8_K_avx2
 * (ops_avx2.cpp:278-298) behind matmul_q8k (ops.cpp:317-349); bit-identical results. */
mcpm_status mcpm_gemv_q8k(int type, const void* w, const void* xq, float* y, int rows, int cols, void* stream);
/* The same product in the engine's default block order (no reference counterpart: the order of
 * the decode kernel's GEMVs and of the tcgen05 batched GEMM when mcpm_config::batch_gemm is
 * MCPM_GEMM_TCGEN05).  Each (row, super-block) integer sum is exact -- the integers of
 * dot_row_q{4,6}_K_q8_K_scalar (ops_scalar_optimized.cpp:139-404) -- and is scaled by one fp32 fma
 * per block, acc = fma(xd*d, isum, acc) and, for Q4_K, accm = fma(-(xd*dmin), minsum, accm), over
 * groups of four consecutive blocks; a row is ((g0 + g1) + g2) + ... with g = acc + accm.
 * cols == 2048 or 6144. */
mcpm_status mcpm_gemv_q8k_block(int type, const void* w, const void* xq, float* y, int rows, int cols, void* stream);
/* y = W x for Q8_0 weights and fp32 activations: gemv_q8_0 (ops.cpp:58-79) behind matmul
 * (ops.cpp:264-290); bit-identical to the reference build (its -ffast-math AVX2 evaluation
 * order: eight lanes per 32-block, pairwise lane reduction, one fma per block along the row).
 * cols % 256 == 0, cols <= 8192, w and x 16-byte aligned. */
mcpm_status mcpm_gemv_q8_0_f32(const void* w, const float* x, float* y, int rows, int cols, void* stream);
/* Integer block sums of the same product, [rows][cols/256] each: Q4_K isum = sum_j sc_j*dot_j,
 * aux = sum_g mn_g*(bsums[2g]+bsums[2g+1]); Q6_K isum = sum sc*q*x over unsigned q,
 * aux = 32*sum_g sc_g*bsums_g (dot_row_q{4,6}_K_q8_K_scalar, ops_scalar_optimized.cpp:139-404). */
mcpm_status mcpm_gemv_blocksums(int type, const void* w, const void* xq, int32_t* isum, int32_t* aux, int rows,
                                int cols, void* stream);
/* gate = Wg xq, up = Wu xq (gemv_gate_up_q4_K_q8_K_avx2, ops_avx2.cpp:444-460). */
mcpm_status mcpm_gemv_gate_up_q8k(const void* wg, const void* wu, const void* xq, float* gate, float* up, int rows,
                                  int cols, void* stream);
/* rmsnorm_and_quantize_q8k (ops.cpp:676-723); n == 2048. */
mcpm_status mcpm_rmsnorm_q8k(const float* x, const float* w, void* out, int n, float eps, void* stream);
/* swiglu_and_quantize_q8k (ops.cpp:725-765); n % 256 == 0. */
mcpm_status mcpm_swiglu_q8k(const float* gate, const float* up, void* out, int n, void* stream);
/* RoPE and the K/V append of one decode step (apply_rope, ops.cpp:502-516, on the 16 query
 * heads and 2 key heads; the KV write of execute_attention, ops.cpp:557-563): q[2048] and
 * k[256] are rotated in place (interleaved pairs, theta_i = rope_base^(-2i/128), angle
 * pos*theta_i; factors from the host C library, as the engine's table), then k and v are
 * written to row pos of kcache / vcache ([max_seq][256] fp32).  Device pointers; pos must
 * lie in [0, max_seq) (MCPM_CTX_OVERFLOW).  Bit-identical to the decode kernel's QKV epilogue. */
mcpm_status mcpm_rope_kv_append(float* q, float* k, const float* v, float* kcache, float* vcache, int pos, int max_seq,
                                float rope_base, void* stream);
/* GQA decode attention for one layer (execute_attention, ops.cpp:537-628): writes k, v
 * (256 floats each, already rotated) into kcache/vcache ([max_seq][256] fp32) at pos,
 * then out[16*128] = softmax(q.K^T / sqrt(128)) V over positions 0..pos, 8 query heads
 * per KV head, split into chunks of 32*ceil((pos+1)/2048) positions.  out_q8k (optional,
 * 8 block_q8_K) receives out quantised ties-to-even, the o_proj input.  max_seq <= 16384.
 * Uses a per-device workspace the library allocates on the first call; calls that
 * overlap on the GPU share it and race. */
mcpm_status mcpm_attention(const float* q, const float* k, const float* v, float* kcache, float* vcache, int pos,
                           int max_seq, float* out, void* out_q8k, void* stream);
/* Same computation and results as mcpm_attention, for callers that cannot allocate device
 * memory (code running inside someone else's graph capture, hosts that own every
 * allocation, loops that must not call the allocator).  No counterpart in the reference.
 * The split-KV workspace is a fixed 540,672-byte array in the library's static device
 * memory (held by every GPU that loads the library until exit), so contexts are limited to
 * pos + 1 <= 16384 and max_seq <= 16384 (MCPM_BAD_ARG beyond).  No call allocates; the
 * first call on a device looks up the workspace address, so make it before any stream
 * capture.  All calls on a device share the workspace: calls that overlap on the GPU race. */
mcpm_status mcpm_attention_noalloc(const float* q, const float* k, const float* v, float* kcache, float* vcache,
                                   int pos, int max_seq, float* out, void* out_q8k, void* stream);
/* GEMV throughput probe: `reps` launches of mcpm_gemv_q8k (order MCPM_ORDER_AVX2) or
 * mcpm_gemv_q8k_block (MCPM_ORDER_BLOCK) rotating over `n_copies` weight copies laid out back to
 * back from `w` (stride rows*row_bytes), so successive launches miss in L2; writes the mean device
 * time per launch in milliseconds. */
enum { MCPM_ORDER_AVX2 = 0, MCPM_ORDER_BLOCK = 1 };
mcpm_status mcpm_gemv_q8k_timed(int type, const void* w, int n_copies, const void* xq, float* y, int rows, int cols,
                                int order, int reps, float* ms_per_launch, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MCPM_H */
