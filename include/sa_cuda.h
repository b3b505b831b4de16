/*
 * sa_cuda.h -- C ABI of libsa_cuda.so, the B200 (sm_100a) implementation of
 * streaming-attention's hot path: online-softmax block attention and the
 * Qwen3 forward it drives.
 *
 * Plain C: opaque handles, raw pointers, sizes and int status codes.  No C++
 * or torch types cross this boundary.  Each entry point names the reference
 * interface it replaces (path:line inside the reference project).
 *
 * Conventions
 *  - Every call returns SA_OK (0) or a negative SA_ERR_* code; the message of
 *    the last failure on the calling thread is returned by sa_last_error().
 *  - Pointers are device pointers unless SA_HOST_PTRS is set in `flags`; then
 *    inputs are read from and outputs written to host memory (pinned memory
 *    gives full PCIe bandwidth) and the call returns after the result is on
 *    the host.
 *  - Device-pointer calls are asynchronous on the context's stream
 *    (sa_ctx_stream); sa_ctx_synchronize() waits for them and reports any
 *    asynchronous CUDA error.
 *  - A context is bound to one GPU and is not thread-safe; distinct contexts
 *    may be used concurrently from different threads.
 *  - Results are deterministic run to run: split counts depend only on the
 *    shape and the GPU's SM count.
 */
#ifndef SA_CUDA_H
#define SA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define SA_OK            0
#define SA_ERR_ARG      -1   /* bad shape, null pointer, misalignment      */
#define SA_ERR_CUDA     -2   /* a CUDA runtime call failed                 */
#define SA_ERR_OOM      -3   /* device or pinned allocation failed         */
#define SA_ERR_TIMEOUT  -4   /* a bounded device-side wait expired         */
#define SA_ERR_NCCL     -5   /* a collective failed                        */
#define SA_ERR_RANGE    -6   /* index out of range (token id, cache slot)  */
#define SA_ERR_FULL     -7   /* KV cache full (kv_cache.h:109-111)         */

/* ---- element types ------------------------------------------------------ */
#define SA_F32   0
#define SA_BF16  1

/* ---- flags -------------------------------------------------------------- */
#define SA_HOST_PTRS   1u    /* pointers are host memory; call is blocking */
/* Decode attention (sa_attn_decode, _partial, _sp) with device pointers: K
 * and V are not written by any kernel still running when the call is issued
 * (e.g. a KV cache appended by earlier steps or by a memory copy).  The
 * kernel is then launched as a programmatic dependent of the stream's
 * previous kernel and streams its first K/V stages while that kernel
 * finishes; q and every output are read / written only after it completed. */
#define SA_KV_STATIC   2u

typedef struct sa_ctx sa_ctx;

/* Message of the last failed call on this thread ("" if none). */
const char* sa_last_error(void);

/* Library version string. */
const char* sa_version(void);

/* Number of CUDA devices visible to the process (0 without a GPU). */
int sa_device_count(int* out);

/* Create a context on `device` with its own non-blocking stream. */
int sa_ctx_create(int device, sa_ctx** out);
/* Destroy a context (synchronises its stream first). */
int sa_ctx_destroy(sa_ctx* ctx);
/* Issue device-pointer calls on a caller-owned stream (a cudaStream_t)
 * instead of the context's own.  NULL selects CUDA's legacy default stream
 * (stream 0); to go back to the context's own stream pass the handle that
 * sa_ctx_stream returned before the first sa_ctx_set_stream call. */
int sa_ctx_set_stream(sa_ctx* ctx, void* stream);
/* The stream device-pointer calls are issued on (a cudaStream_t). */
void* sa_ctx_stream(sa_ctx* ctx);
/* Wait for all work on the context's stream; returns SA_ERR_CUDA with the
 * CUDA error text on an asynchronous failure. */
int sa_ctx_synchronize(sa_ctx* ctx);
/* Number of SMs of the context's GPU (148 on B200). */
int sa_ctx_num_sms(sa_ctx* ctx);

/* ======================================================================== */
/* Decode (single-query) streaming attention                                 */
/* ======================================================================== */

/*
 * Multi-head GQA decode attention for one query token.
 *
 *   q    [hq, d]                     element type `dtype`
 *   k, v head h at k + h*kv_head_stride (elements), rows of d elements,
 *        T rows: [hkv, T(+pad), d]   element type `dtype`
 *   out  [hq, d] fp32
 *
 * out[h] = softmax(scale * q[h] . K[h/(hq/hkv)]^T) V[h/(hq/hkv)]
 *
 * With hq = hkv = 1 and scale = 1 this is streaming_attention_serial /
 * streaming_attention_omp / naive_attention_serial of
 * attention/src/attention.h:27-208 (which apply no 1/sqrt(d) scale).  With
 * hq = 16, hkv = 8 and scale = 1/sqrt(d) it is the decode attention of
 * qwen3_decoder_layer_with_cache (tensor_cpp/src/qwen3_ops.cpp:860-900:
 * repeat_kv + ops::self_attention over the cache).
 *
 * `block` is the reference's online-softmax block size (64 or 128); it must be
 * > 0 but does not change the result beyond fp32 rounding -- the GPU tiles the
 * sequence its own way.  T = 0 yields zeros (as the reference's serial path).
 * Requirements: d in {64, 128, 256}; hq % hkv == 0 and hq/hkv in {1,2,4,8};
 * k, v and kv_head_stride*elt 16-byte aligned.
 * The call keeps its (m, l, O) split partials in context scratch memory, so
 * two calls on one context must not overlap on different streams.
 */
int sa_attn_decode(sa_ctx* ctx, int dtype, const void* q, const void* k, const void* v,
                   long long kv_head_stride, int T, int d, int hq, int hkv, int block,
                   float scale, float* out, unsigned flags);

/*
 * Same attention, returning the un-finalised online-softmax state so that
 * several KV shards (e.g. one per GPU) can be merged with sa_attn_merge.
 *   m_out, l_out [hq]   running max and normaliser (reference: PartialResult,
 *                       attention/src/streaming_omp.cpp:12-16; m=-inf, l=1
 *                       for an empty shard)
 *   o_out [hq, d]       output normalised by l (process_blocks_serial,
 *                       streaming_omp.cpp:53-89)
 * Replaces the rank-local part of streaming_attention_mpi_simple
 * (attention/src/streaming_mpi.cpp:252-292).
 */
int sa_attn_decode_partial(sa_ctx* ctx, int dtype, const void* q, const void* k,
                           const void* v, long long kv_head_stride, int T, int d, int hq,
                           int hkv, int block, float scale, float* m_out, float* l_out,
                           float* o_out, unsigned flags);

/*
 * Merge n_parts partial states, part-major:
 *   m, l [n_parts, hq];  o [n_parts, hq, d];  out [hq, d] fp32.
 * Optional m_out/l_out [hq] (may be NULL) receive the merged state.
 * The associative merge of merge_partial_results
 * (attention/src/streaming_omp.cpp:27-48) used by rank 0 at
 * streaming_mpi.cpp:295-305.  All pointers device unless SA_HOST_PTRS.
 */
int sa_attn_merge(sa_ctx* ctx, int n_parts, int hq, int d, const float* m, const float* l,
                  const float* o, float* out, float* m_out, float* l_out, unsigned flags);

/* ======================================================================== */
/* Sequence-parallel decode over several GPUs                                */
/* ======================================================================== */

/*
 * The KV sequence is split over `world` ranks (1..8), one GPU per rank, each
 * holding a contiguous slice in rank order -- the partition of
 * streaming_attention_mpi_simple (attention/src/streaming_mpi.cpp:252-309).
 * Each rank's sa_attn_decode_sp launch reduces its slice to per-head (m, l, O)
 * states, and the CTA that finishes each KV head stores those states into
 * every rank's exchange buffer over NVLink and merges all ranks' states in
 * rank order (merge_partial_results, streaming_omp.cpp:27-48): one launch per
 * rank, no collective library, and the result on EVERY rank (the reference
 * returns it on rank 0 only and zeros elsewhere, streaming_mpi.cpp:306-308).
 *
 * sa_sp_create: this rank's exchange object on the context's GPU, for calls
 *   with hq <= max_hq and d <= max_d (d in {64, 128, 256}).
 * sa_sp_handle: SA_SP_HANDLE_BYTES bytes naming this rank's exchange buffer
 *   (a CUDA IPC handle and the GPU's UUID), to be sent to every rank over any
 *   host channel.
 * sa_sp_connect: the world handles in rank order; maps the other ranks'
 *   buffers.  Ranks on one GPU are rejected (SA_ERR_ARG): the launches wait
 *   for one another and must run on different GPUs.
 * sa_sp_connect_local: the same for `n` ranks of ONE process (one sa_sp per
 *   GPU, sps[i] rank i): enables peer access and links the buffers directly.
 * sa_attn_decode_sp: sa_attn_decode_partial's arguments for this rank's
 *   slice (T_local rows, may be 0), q identical on every rank.  out [hq, d]
 *   (and m_out / l_out [hq] if non-NULL) receive the merged result of the
 *   whole sequence on every rank.  Every rank must make the same calls, with
 *   the same hq / hkv / d, in the same order; calls on one rank must not
 *   overlap on different streams.  A rank that does not take part makes the
 *   others' waits expire after a few seconds (NaN in out, SA_ERR_TIMEOUT at
 *   their next synchronising call).  SA_HOST_PTRS is accepted (staged,
 *   blocking).
 */
#define SA_SP_HANDLE_BYTES 128
typedef struct sa_sp sa_sp;
int sa_sp_create(sa_ctx* ctx, int rank, int world, int max_hq, int max_d, sa_sp** out);
int sa_sp_handle(sa_sp* sp, void* handle);
int sa_sp_connect(sa_sp* sp, const void* handles);
int sa_sp_connect_local(sa_sp* const* sps, int n);
int sa_sp_destroy(sa_sp* sp);
int sa_attn_decode_sp(sa_sp* sp, int dtype, const void* q, const void* k, const void* v,
                      long long kv_head_stride, int T_local, int d, int hq, int hkv, int block,
                      float scale, float* out, float* m_out, float* l_out, unsigned flags);

/* ======================================================================== */
/* Causal prefill attention (tensor cores)                                   */
/* ======================================================================== */

/*
 * Causal multi-head GQA attention for Sq query tokens against Skv keys.
 *   q   [Sq,  hq  heads, d]  bf16, token stride q_tok_stride (elements)
 *   k,v [Skv, hkv heads, d]  bf16, token stride kv_tok_stride
 *   out [Sq,  hq  heads, d]  fp32 (SA_F32) or bf16 (SA_BF16), token stride
 *                            o_tok_stride
 * Query i (global position q_pos0 + i) sees keys 0 .. q_pos0 + i; the usual
 * prefill is q_pos0 = 0, Skv = Sq; a chunk of a longer prompt (sequence
 * parallelism, chunked prefill) passes its offset and the keys before it.
 * out = softmax(scale * q k^T + causal mask) v, computed with bf16 operands
 * and fp32 accumulation on tcgen05 tensor cores.
 * Replaces ops::self_attention with create_causal_mask
 * (tensor_cpp/src/ops.cpp:514-641, qwen3_ops.cpp:240-259) and
 * self_attention_streaming_blockwise (ops.cpp:1027-1112,1383-1450) after
 * repeat_kv (qwen3_ops.cpp:194-234).  Requirements: d = 128; hq a multiple
 * of hkv; q_pos0 + Sq <= Skv; device pointers (16-byte aligned, token strides
 * multiples of 8 elements).
 */
int sa_attn_prefill(sa_ctx* ctx, const void* q, const void* k, const void* v, int Sq, int Skv,
                    int q_pos0, int d, int hq, int hkv, long long q_tok_stride,
                    long long kv_tok_stride, float scale, void* out, int out_dtype,
                    long long o_tok_stride, unsigned flags);

/* ======================================================================== */
/* Sequence-parallel causal prefill (one rank per GPU)                       */
/* ======================================================================== */

/*
 * The causal prefill of S tokens with the sequence split over `world` ranks
 * (1..8), one GPU each, in the load-balanced zig-zag order: the sequence is
 * cut into 2 x world chunks of C = S / (2 world) tokens and rank r holds
 * chunks r and 2 world - 1 - r -- the sequence strategy of
 * attention_sequence_online_softmax (tensor_cpp/include/tensor_cpp/ops_mpi.h:326,
 * ops_mpi.cpp:1000-1212), computing the causal attention that strategy stands
 * for (its statistics all-reduce mixes positions).
 *
 * sa_spp_create: this rank's object on the context's GPU for sequences of up
 *   to max_seq tokens with hkv <= 8 KV heads of d = 128 (two K/V buffers of
 *   max_seq x hkv x 128 bf16 each, shared with the other ranks).
 * sa_spp_handle / sa_spp_connect / sa_spp_connect_local / sa_spp_destroy:
 *   as the sa_sp_* functions (SA_SPP_HANDLE_BYTES per handle; one GPU per
 *   rank, checked).
 * sa_spp_prefill: q_local [2C, hq, 128], k_local / v_local [2C, hkv, 128]
 *   bf16, contiguous, device memory: this rank's two chunks, chunk r first.
 *   Each rank writes its K/V chunks into every rank's buffer over NVLink,
 *   waits (bounded) for the others', then computes its query rows' causal
 *   attention over the whole prefix on the tensor cores, and writes
 *   out_local [2C, hq, 128] in out_dtype (SA_BF16 or SA_F32).  S must be a
 *   multiple of 2 x world.  Asynchronous on the context's stream; every rank
 *   makes the same calls in the same order.  A rank that does not take part
 *   makes the others' waits expire after a few seconds (NaN in out_local,
 *   SA_ERR_TIMEOUT at their next synchronising call).  The object's buffers
 *   for the partial outputs grow on the first call with a larger S x hq
 *   (a device allocation after a stream synchronisation); later calls of the
 *   same shape allocate nothing.
 */
#define SA_SPP_HANDLE_BYTES 128
typedef struct sa_spp sa_spp;
int sa_spp_create(sa_ctx* ctx, int rank, int world, int max_seq, int hkv, int d, sa_spp** out);
int sa_spp_handle(sa_spp* sp, void* handle);
int sa_spp_connect(sa_spp* sp, const void* handles);
int sa_spp_connect_local(sa_spp* const* sps, int n);
int sa_spp_destroy(sa_spp* sp);
int sa_spp_prefill(sa_spp* sp, const void* q_local, const void* k_local, const void* v_local, int S, int hq,
                   int hkv, int d, float scale, void* out_local, int out_dtype, unsigned flags);

/*
 * fp32 attention of Sq query rows on CUDA cores (fp32 throughout, like the
 * reference's own operators):
 *   q   [Sq, hq, d]       token-major, token stride q_tok_stride (elements)
 *   k,v [hkv, Skv(+pad), d] head-major (one batch row of the reference's
 *                         [B, H, S, D] tensors), head stride kv_head_stride
 *   out [Sq, hq, d] fp32  token stride o_tok_stride
 * causal = 1: query i sees keys 0 .. min(q_pos0 + i, Skv - 1) -- the causal
 *   mask of create_causal_mask (qwen3_ops.cpp:240-259) for a query block at
 *   offset q_pos0, and self_attention_streaming_blockwise
 *   (tensor_cpp/src/ops.cpp:1383-1450) with q_pos0 = 0;
 * causal = 0: every query sees all Skv keys -- ops::self_attention without a
 *   mask (ops.cpp:514-641) and the decode of self_attention_streaming
 *   (ops.cpp:964-1017, with the scale on the scores).
 * Query head h reads KV head h / (hq / hkv) (repeat_kv, qwen3_ops.cpp:194-234,
 * without the copy).  Scores are scaled by `scale` before the softmax.
 * Requirements: d in {64, 128, 256}; hq/hkv in {1, 2, 4, 8} (also 16 for
 * causal rows inside the sequence at d = 128); strides multiples of 4
 * elements (kv_head_stride a multiple of d); device pointers 16-byte aligned
 * unless SA_HOST_PTRS.
 */
int sa_attn_prompt_f32(sa_ctx* ctx, const float* q, const float* k, const float* v, int Sq, int Skv,
                       int q_pos0, int causal, int d, int hq, int hkv, long long q_tok_stride,
                       long long kv_head_stride, float scale, float* out, long long o_tok_stride,
                       unsigned flags);

/*
 * One decode step over a device-resident KV cache (batch 1):
 *   k_cache, v_cache [hkv, max_seq, d]  device memory, element type `dtype`
 *   k_new, v_new     [hkv, d]           the new token's key / value
 *   q [hq, d] -> out [hq, d] fp32
 * Writes k_new / v_new at row `pos` of every head, then attends over rows
 * [0, pos] (pos + 1 rows).  Replaces, per layer, kv_cache->update() +
 * attention over the cache in qwen3_decoder_layer_with_cache
 * (tensor_cpp/src/qwen3_ops.cpp:849,876-885; kv_cache.h:94-130).
 * SA_ERR_FULL when pos >= max_seq (kv_cache.h:109-111).  With SA_HOST_PTRS,
 * q, k_new, v_new and out are host memory (the cache stays on the device).
 */
int sa_attn_decode_step(sa_ctx* ctx, int dtype, const void* q, const void* k_new,
                        const void* v_new, void* k_cache, void* v_cache, int max_seq, int pos,
                        int d, int hq, int hkv, int block, float scale, float* out,
                        unsigned flags);

/*
 * Allocation-free variant of sa_attn_decode.  It has no counterpart in the
 * reference; it exists for callers that cannot call cudaMalloc -- serving
 * runtimes that reserve nearly all device memory for their own pools at
 * start-up, and latency-critical loops that cannot afford cudaMalloc's
 * implicit device synchronisation.  Such callers cannot create an sa_ctx
 * either (its constructor allocates), so this call takes a plain stream.
 *
 * Same arguments and result as sa_attn_decode with device pointers (q, k, v
 * and out are the caller's device memory; `stream` is a cudaStream_t, NULL =
 * the legacy default stream; the GPU is the one holding `out`).  The call
 * never calls cudaMalloc, cudaFree or any allocating routine: its scratch
 * (per-split partial states and per-KV-head counters) lives in a file-scope
 * device array of SA_NOALLOC_SCRATCH_BYTES that every GPU which loads the
 * library holds until the process exits.
 *  - Shapes whose scratch (about hq * splits * (d + 2) * 4 bytes, splits
 *    ~ 2 * SMs / hkv) exceeds SA_NOALLOC_SCRATCH_BYTES are rejected with
 *    SA_ERR_ARG and a message naming the sizes.
 *  - The first call on a GPU looks up the array's device address
 *    (cudaGetSymbolAddress) with that GPU current and caches it for the life
 *    of the process; make that first call before any stream capture, and do
 *    not reset the device (cudaDeviceReset) between calls.
 *  - All calls on a GPU share the array, which keeps the last call's
 *    contents; each call clears the counters and the status word it needs.
 *    Calls whose executions overlap on the GPU (different streams, or host
 *    threads without ordering) race on the array and give wrong results.
 *  - Asynchronous: argument errors are returned; a device-side wait of the
 *    kernel that expired (a fault of the GPU, not of the arguments) is not
 *    reported by a return code but leaves NaN in `out`.
 */
#define SA_NOALLOC_SCRATCH_BYTES (2u << 20)
int sa_attn_decode_noalloc(void* stream, int dtype, const void* q, const void* k, const void* v,
                           long long kv_head_stride, int T, int d, int hq, int hkv, int block,
                           float scale, float* out);

/* ======================================================================== */
/* Qwen3 forward                                                             */
/* ======================================================================== */

typedef struct sa_qwen3 sa_qwen3;

/* Model shape (Qwen3-0.6B: vocab 151936, hidden 1024, 28 layers, 16/8 heads,
 * head_dim 128, intermediate 3072, eps 1e-6, theta 1e6) and KV-cache
 * capacity in tokens (the reference's KVCache max_seq_len, kv_cache.h:47-52). */
typedef struct {
    int vocab, hidden, n_layers, hq, hkv, head_dim, inter;
    float eps, theta;
    int max_seq;
} sa_qwen3_config;

/* Allocate a model (weights, fp32 KV cache of n_layers x hkv x max_seq x
 * head_dim, activation buffers) on the context's GPU.  Weights are uploaded
 * with sa_qwen3_set_embed / sa_qwen3_set_layer.  Requirements: head_dim 128,
 * hidden and inter multiples of 64, hq/hkv in {1, 2, 4}. */
int sa_qwen3_create(sa_ctx* ctx, const sa_qwen3_config* cfg, sa_qwen3** out);
int sa_qwen3_destroy(sa_qwen3* m);

/* Token embedding [vocab, hidden], final norm [hidden], lm_head [vocab,
 * hidden] (NULL or equal to the embedding = tied), host fp32, stored as bf16
 * (exact for bf16 checkpoints; qwen3_loader.cpp reads bf16). */
int sa_qwen3_set_embed(sa_qwen3* m, const float* embed, const float* final_norm, const float* lm_head);

/* One decoder layer's weights, host fp32, in the reference's shapes
 * (Qwen3LayerWeights, tensor_cpp/include/tensor_cpp/qwen3_ops.h:37-57):
 * norms [hidden]; q [hq*128, hidden]; k, v [hkv*128, hidden]; q_norm, k_norm
 * [128]; o [hidden, hq*128]; gate, up [inter, hidden]; down [hidden, inter]. */
int sa_qwen3_set_layer(sa_qwen3* m, int layer, const float* in_norm, const float* wq, const float* wk,
                       const float* wv, const float* q_norm, const float* k_norm, const float* wo,
                       const float* post_norm, const float* w_gate, const float* w_up,
                       const float* w_down);

/*
 * Qwen3 weights from a safetensors checkpoint (load_qwen3_weights,
 * tensor_cpp/src/qwen3_loader.cpp:140-297): the file is memory-mapped and
 * each tensor is uploaded from its stored bytes (BF16 as it is; F16 / F32
 * rounded to bf16), without the reference's widening to fp32.  Tensor names
 * are the Hugging Face Qwen3 ones (model.embed_tokens.weight,
 * model.layers.{i}.self_attn.q_proj.weight, ...); lm_head.weight may be
 * absent (tied to the embedding).  The configuration is inferred from the
 * shapes; eps / theta <= 0 select Qwen3's 1e-6 / 1e6.
 * sa_safetensors_inspect validates the file and reports the configuration
 * (max_seq 0) without touching a GPU; sa_qwen3_load_safetensors creates the
 * model on the context's GPU with room for max_seq cached tokens and uploads
 * the weights (blocking).  Malformed files, missing tensors and wrong shapes
 * are SA_ERR_ARG with the tensor named in the message.
 */
int sa_safetensors_inspect(const char* path, sa_qwen3_config* out);
int sa_qwen3_load_safetensors(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta,
                              sa_qwen3** out);

/* KVCache::reset (kv_cache.h:142-153): the cache length returns to 0. */
int sa_qwen3_reset(sa_qwen3* m);
/* KVCache::current_seq_len. */
int sa_qwen3_cache_len(sa_qwen3* m);

/*
 * Mirror of the host KVCache contents (kv_cache.h:60-70: one tensor per layer
 * of [batch, num_kv_heads, max_seq_len, head_dim], here batch 1).
 * sa_qwen3_read_kv copies rows 0..cache_len-1 of one layer's K and V cache
 * (fp32) into host arrays laid out [hkv][seq_stride][head_dim]
 * (seq_stride >= cache_len; KVCache uses its max_seq_len); blocking.
 * sa_qwen3_write_kv uploads rows 0..len-1 of one layer from the same layout
 * (len <= max_seq); blocking.  sa_qwen3_set_cache_len makes the first len
 * rows the live cache (KVCache::current_seq_len = len), so a cache filled
 * elsewhere (e.g. a CPU prefill) can be continued on the GPU.
 */
int sa_qwen3_read_kv(sa_qwen3* m, int layer, float* k_out, float* v_out, int seq_stride);
int sa_qwen3_write_kv(sa_qwen3* m, int layer, const float* k, const float* v, int len, int seq_stride);
int sa_qwen3_set_cache_len(sa_qwen3* m, int len);

/*
 * Forward S tokens.  use_cache = 0: qwen3_forward (qwen3_ops.cpp:537-614),
 * positions 0..S-1, the cache length is left unchanged.  use_cache = 1:
 * qwen3_forward_with_cache (:936-1014, STANDARD attention): positions start
 * at the cache length, K/V are appended and the length advances by S.
 * logits_mode 0: logits [S, vocab]; 1: last token only [vocab]; 2: none.
 * ids are checked against the vocabulary (SA_ERR_RANGE, ops.cpp:296);
 * SA_ERR_FULL when the cache cannot hold S more tokens (kv_cache.h:109-111).
 * With SA_HOST_PTRS ids/logits are host memory and the call is blocking.
 */
int sa_qwen3_forward(sa_qwen3* m, const int64_t* ids, int S, int use_cache, float* logits,
                     int logits_mode, unsigned flags);

/*
 * Greedy decode: forward the S-token prompt with the cache, then n_new times
 * take the argmax of the last logits (ops::argmax, ops.cpp:213-272; first
 * index of the maximum) as the next token and forward it.  Writes the n_new
 * generated tokens.  Token selection stays on the GPU; with SA_HOST_PTRS the
 * prompt/tokens are host memory.  The driver loop of benchmark_qwen3's decode
 * phase (benchmark_qwen3.cpp:406-520) with the argmax taken over the returned
 * logits.
 */
int sa_qwen3_generate(sa_qwen3* m, const int64_t* prompt, int S, int n_new, int64_t* out_tokens,
                      unsigned flags);

/*
 * Head-parallel Qwen3 over `world` GPUs (1..8), one model per GPU, usually
 * one process per GPU.  Replaces the reference's head-wise MPI model path
 * (qwen3_ops_mpi.cpp, ParallelStrategy HEADWISE, qwen3_ops_mpi.h:30-50) for
 * qwen3_forward / qwen3_forward_with_cache / greedy decode.
 *
 * Rank r keeps q heads [r*hq/world, (r+1)*hq/world), the KV heads, o_proj
 * columns and KV cache of those heads, gate/up rows and down_proj columns of
 * intermediate features [r*inter/world, ...), and the whole embedding and
 * lm_head.  Each layer's o_proj and down_proj give partial sums that every
 * rank sends to every rank's exchange buffer over NVLink (peer stores from
 * the projection kernels); the next normed projection adds them, in rank
 * order, so the residual stream is the same on every rank.  Greedy decode
 * splits the lm_head over the vocabulary and exchanges the ranks' argmax.
 *
 * sa_qwen3_create_tp: as sa_qwen3_create for rank `rank` of `world`
 *   (hkv divisible by world, inter by 64 * world).  Weights are set with
 *   the same full tensors on every rank (sa_qwen3_set_embed / _set_layer, or
 *   sa_qwen3_load_safetensors_tp); each rank keeps its share.
 * sa_qwen3_tp_handle: SA_TP_HANDLE_BYTES bytes naming this rank's exchange
 *   buffer (a CUDA IPC handle), to be passed to every rank.
 * sa_qwen3_tp_connect: the world handles in rank order (world *
 *   SA_TP_HANDLE_BYTES bytes); maps the other ranks' buffers.  Required
 *   before forward / generate.
 * Every rank then calls sa_qwen3_forward / sa_qwen3_generate with the same
 * arguments in the same order; logits and tokens come back on every rank.
 * Head-parallel forwards take at most min(max_seq, 8192) tokens per call.
 * A rank that stops taking part makes the others' waits give up after a few
 * seconds (SA_ERR_TIMEOUT at the next synchronising call).
 * sa_qwen3_read_kv / _write_kv address this rank's KV heads only.
 */
#define SA_TP_HANDLE_BYTES 64
int sa_qwen3_create_tp(sa_ctx* ctx, const sa_qwen3_config* cfg, int rank, int world, sa_qwen3** out);
int sa_qwen3_load_safetensors_tp(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta, int rank,
                                 int world, sa_qwen3** out);
int sa_qwen3_tp_handle(sa_qwen3* m, void* handle);
int sa_qwen3_tp_connect(sa_qwen3* m, const void* handles);

/*
 * Sequence-parallel Qwen3 over `world` GPUs (1..8), one model per GPU -- the
 * reference's SEQUENCE strategy (ParallelStrategy, qwen3_ops_mpi.h:30-50;
 * qwen3_forward_mpi_omp, qwen3_ops_mpi.cpp:498-642), whose outputs are wrong
 * there; here they equal the single-GPU forward's.
 *
 * Every rank holds the whole model and a whole KV cache.  A prompt of S >=
 * 2 * world tokens is split over the ranks by tokens, rank r taking tokens
 * [S*r/world, S*(r+1)/world): its projections and MLP run on its own tokens
 * at their global RoPE positions; after each layer's K/V cache append the
 * rank stores its new K/V rows into the same rows of every other rank's
 * cache over NVLink (CUDA IPC mappings) and publishes a flag, and every rank
 * waits for all ranks' rows before its causal attention; at the end the
 * final residual rows are gathered the same way, so every rank computes the
 * same logits / next token.  Shorter prompts and single-token decode steps
 * run whole on every rank (the caches are identical), so generate() gives the
 * same tokens on every rank without further exchanges.
 *
 * sa_qwen3_create_sp: as sa_qwen3_create for rank `rank` of `world`; weights
 *   are set with the same full tensors on every rank.
 * sa_qwen3_sp_handle: SA_QWEN3_SP_HANDLE_BYTES bytes naming this rank's row
 *   buffer and K/V caches (CUDA IPC handles) and its GPU, for every rank.
 * sa_qwen3_sp_connect: the world handles in rank order; maps the other ranks'
 *   buffers.  Ranks on one GPU are rejected (SA_ERR_ARG).  Required before
 *   forward / generate.
 * Every rank then calls sa_qwen3_forward / sa_qwen3_generate with the same
 * arguments in the same order; prompts of up to min(max_seq, 8192) tokens.
 * A rank that stops taking part makes the others' waits give up after a few
 * seconds (SA_ERR_TIMEOUT at the next synchronising call).
 */
#define SA_QWEN3_SP_HANDLE_BYTES 256
int sa_qwen3_create_sp(sa_ctx* ctx, const sa_qwen3_config* cfg, int rank, int world, sa_qwen3** out);
/* The same rank with its weights read from a safetensors checkpoint, as
 * sa_qwen3_load_safetensors. */
int sa_qwen3_load_safetensors_sp(sa_ctx* ctx, const char* path, int max_seq, float eps, float theta, int rank,
                                 int world, sa_qwen3** out);
int sa_qwen3_sp_handle(sa_qwen3* m, void* handle);
int sa_qwen3_sp_connect(sa_qwen3* m, const void* handles);

#ifdef __cplusplus
}
#endif
#endif /* SA_CUDA_H */
