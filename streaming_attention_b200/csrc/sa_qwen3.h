// sa_qwen3.h -- internal declarations shared by the Qwen3 translation units.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

// GEMM / GEMV epilogues
#define QW_EPI_STORE  0   // y = W x
#define QW_EPI_RESID  1   // y += W x          (residual stream)
#define QW_EPI_SWIGLU 2   // y_i = silu(g_i) * u_i over [gate(32); up(32)] row blocks
#define QW_EPI_QKV    3   // decode QKV projection + QK-norm + RoPE + KV-cache append (head_dim 128)
#define QW_EPI_XCHG   4   // partial sums sent to every rank's receive block (head-parallel)
#define QW_EPI_RESID_NORM 5   // prompt GEMM: C += acc, then the next GEMM's A operand hi/lo(g . C)
                              // and per-tile row sums of C^2 (its RMSNorm, deferred)
#define QW_EPI_QKV_ROWS   6   // prompt GEMM: QK-norm + RoPE + KV-cache append of whole heads

namespace sa {

// Operands of the QW_EPI_QKV epilogue: one token at RoPE position
// (pos_dev ? *pos_dev : pos0), written to cache row position + row_shift.
struct QkvEpi {
    int hq = 0, hkv = 0, max_seq = 0, pos0 = 0, row_shift = 0;
    const int* pos_dev = nullptr;
    const float *qn = nullptr, *kn = nullptr, *cos_t = nullptr, *sin_t = nullptr;
    float *q_out = nullptr, *kc = nullptr, *vc = nullptr;
    unsigned* cnt = nullptr;   // [hq + hkv] arrival counters, zero between launches
};

// Prompt GEMM (sa_gemm.cu): output tile width and the number of CTAs of a
// cluster that split K.
struct GemmPlan {
    int bn, splits;
};

// Optional epilogue operands of an unsplit prompt GEMM (gemm_launch).
//
// Deferred RMSNorm: RMSNorm(x) W^T = diag(1 / rms(x)) (g . x) W^T, so the
// producer of x (a QW_EPI_RESID_NORM GEMM) writes A = hi/lo(g . x) and, per
// output tile p, rowsq[p * M + r] = sum of x[r, :]^2 over the tile's columns;
// the consumer multiplies row r of its accumulator by
// 1 / sqrt(sum_p rowsq[p * M + r] / norm_k + eps) (parts added in order)
// before its own epilogue.  rowsq_in == nullptr: A is already normalised.
//
// QW_EPI_QKV_ROWS (tile width a multiple of 128, so tiles hold whole heads):
// token m at RoPE position pos0 + m; Q heads -> QK-norm + RoPE -> q_out
// (fp32 [M, hq, 128]) and/or q_bf (bf16, same layout); K heads -> QK-norm +
// RoPE -> K cache row (pos0 + m + row_shift) of kc and/or bf16 row pos0 + m
// of k_bf ([rows, hkv, 128]); V heads -> vc / v_bf likewise.
struct GemmEpi {
    const float* rowsq_in = nullptr;
    int rowsq_parts = 0;
    float norm_k = 0.f, eps = 0.f;
    const float* g = nullptr;      // RESID_NORM: gain of the next GEMM's RMSNorm [N]
    float* rowsq_out = nullptr;    // RESID_NORM: [N / bn][M]
    int hq = 0, hkv = 0, max_seq = 0, pos0 = 0, row_shift = 0;
    const float *qn = nullptr, *kn = nullptr, *cos_t = nullptr, *sin_t = nullptr;
    float *q_out = nullptr, *kc = nullptr, *vc = nullptr;
    __nv_bfloat16 *q_bf = nullptr, *k_bf = nullptr, *v_bf = nullptr;
};
// Occupancy queries of the GEMM variants, once per device; call before any
// stream capture.
void gemm_prepare(int device);
// Tile width and split count for C[M, N] = A[M, K] W^T; split plans (splits
// > 1) leave partial planes for the next kernel, so `split_ok` says whether
// the consumer of this output adds them.
GemmPlan gemm_plan(int device, int num_sms, int M, int N, int K, bool split_ok);
// plan.splits > 1: writes planes part[z][M][N] (z < splits) instead of
// applying `mode`.
int gemm_launch(cudaStream_t st, int* status, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo,
                long long lda, const __nv_bfloat16* w, int M, int N, int K, int mode, float* C,
                long long ldc, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo, long long ldo, GemmPlan plan,
                float* part, size_t part_floats, const GemmEpi* epi = nullptr);


// Causal attention of M prompt queries (q at q + m*q_stride, [hq, 128]) over
// rows [0, T0 + m) of each KV head of a head-major fp32 cache (head h at
// k / v + h * kv_head_stride; kv_rows = rows of 128 floats addressable from
// k); output fp32 (out) and/or bf16 hi/lo planes (out_hi/out_lo), row m at
// m*o_stride.  Defined in sa_prompt_attn.cu.
int prompt_attn_launch(cudaStream_t st, int* status, const float* q, long long q_stride, const float* k,
                       const float* v, long long kv_head_stride, long long kv_rows, int T0, int M, int d, int hq,
                       int hkv, float scale, float* out, long long o_stride, __nv_bfloat16* out_hi,
                       __nv_bfloat16* out_lo);
// element-wise / GEMV launchers (sa_qwen3_kernels.cu)
int launch_embedding(cudaStream_t st, const int64_t* ids, int M, const __nv_bfloat16* E, int V, int H, float* x,
                     int* status);
// RMSNorm of rows [0, M) of x to bf16 hi / lo terms; with splits > 0 the
// partial planes part[z][M][H] are first added to x (and x written back).
int launch_rmsnorm_hilo(cudaStream_t st, float* x, const float* w, int M, int H, float eps,
                        __nv_bfloat16* hi, __nv_bfloat16* lo, const float* part = nullptr, int splits = 0);
// x[M, H] += sum of the partial planes part[z][M][H], z < splits.
int launch_resid_add(cudaStream_t st, float* x, const float* part, int splits, int M, int H, int num_sms);
// SwiGLU of the gate/up partial planes part[z][M][2I] to bf16 hi / lo [M, ldo].
int launch_swiglu_hilo(cudaStream_t st, const float* part, int splits, int M, int I, __nv_bfloat16* hi,
                       __nv_bfloat16* lo, long long ldo, int num_sms);
int launch_rope_table(cudaStream_t st, int n_pos, int D, float theta, float* cos_t, float* sin_t);
int launch_qknorm_rope_append(cudaStream_t st, const float* qkv, int splits, int M, int hq, int hkv, const float* qn,
                              const float* kn, const float* cos_t, const float* sin_t, int pos0, const int* pos_dev,
                              int row_shift, float* q_out, float* kc, float* vc, int max_seq);
int launch_advance(cudaStream_t st, int* state, const int64_t* tok, int64_t* toks, int cap, int inc_len,
                   bool after_kernel);
size_t decode_dev_scratch_floats(int num_sms, int max_T, int d, int hq, int hkv, int* n_splits);
int decode_dev_launch(cudaStream_t st, int* status, int num_sms, const float* q, const float* k, const float* v,
                      long long kv_head_stride, const int* len_dev, int T_host, int max_T, int d, int hq, int hkv,
                      float scale, float* out, float* scratch, unsigned* counters);
int launch_gemv2(cudaStream_t st, int mode, bool norm, const __nv_bfloat16* W, int N_out, int K, const float* x,
                 const float* nw, float eps, float* y, unsigned long long* amax, const QkvEpi* qkv = nullptr);

// ---- head-parallel exchange (sa_qwen3_create_tp) ---------------------------
// Every rank owns one exchange buffer: flag words [2 slots][world], word
// areas [2 slots][world sources][ll_stride] (single-token exchanges), then
// receive blocks [2 slots][world sources][slot_floats] (prompt exchanges).  Exchange instance i
// (counted over the whole run, the same on every rank) uses slot i & 1; the
// source rank writes its partial sums into block [slot][source] of every
// rank (itself included) and then sets flag [slot][source] on every rank to
// i + 1.  A consumer waits until all `world` flags of its slot reach i + 1
// and adds the blocks in rank order, so every rank computes the same sums.
// Two slots suffice: a rank can only start instance i + 2 after every rank
// published instance i + 1, which each does after consuming instance i.
constexpr int TP_MAX = 8;
struct TpArgs {
    int rank = 0, world = 1;
    float* recv[TP_MAX] = {};       // receive blocks of every rank (own at [rank])
    unsigned* flags[TP_MAX] = {};   // flag words of every rank
    long long slot_floats = 0;      // floats per (slot, source) block
    const unsigned* seq = nullptr;  // instances completed before this segment (device)
    int k = 0;                      // this instance's index within the segment
    unsigned* cnt = nullptr;        // producer grid's arrival counter (zero between launches)
    int* status = nullptr;
    float* x_out = nullptr;         // consumer GEMV: residual + exchanged sums are written here
    int row = 0;                    // consumer / producer: row of the receive block
    int n_base = 0;                 // argmax: index of output 0 in the full vocabulary
    // Single-token exchanges use self-validating words instead of blocks and
    // flags: word = (epoch << 32) | value bits, stored with one 8-byte store,
    // so a reader that sees the epoch also sees the value.
    unsigned long long* ll[TP_MAX] = {};   // word areas [2 slots][world][ll_stride] of every rank
    int ll_stride = 0;
    int use_ll = 0;                 // consumer: the producer wrote words (single-token path)
};
int launch_gemv2_tp(cudaStream_t st, int mode, bool norm, const __nv_bfloat16* W, int N_out, int K,
                    const float* x, const float* nw, float eps, float* y, unsigned long long* amax,
                    const QkvEpi* qkv, const TpArgs& tp, bool consume);
// Copy rows [0, M) x H of `part` to every rank's receive block and publish.
int launch_tp_scatter(cudaStream_t st, const float* part, int M, int H, const TpArgs& tp, int grid);
// RMSNorm (as launch_rmsnorm_hilo) of rows r0.. of x after adding the exchanged sums
// (rows r0 + m of the receive blocks) into x in place.
int launch_rmsnorm_hilo_tp(cudaStream_t st, float* x, const float* w, int M, int H, float eps,
                           __nv_bfloat16* hi, __nv_bfloat16* lo, const TpArgs& tp);
// Greedy token over the ranks' vocabulary slices: max of the argmax keys,
// then *seq += seg (the segment's instances).
int launch_tp_amax_token(cudaStream_t st, unsigned long long* amax, int64_t* tok, const TpArgs& tp, int seg);
int launch_tp_seq_add(cudaStream_t st, unsigned* seq, int n);
// Sequence-parallel prompt: up to two regions of nblk blocks of blk_floats
// floats (stride floats apart) that this rank produced, copied to the same
// offsets (plus slot * slot_floats) in every other rank's copy of the region,
// then the instance published on every rank (the flags and sequence word of
// a TpArgs); and the matching bounded wait for every rank's publication.
struct SpCopy {
    int nreg = 0;
    const float* src[2] = {};
    float* dst[2][TP_MAX] = {};
    long long slot_floats = 0;
    int nblk = 0;
    long long blk_floats = 0;
    long long stride = 0;
};
int launch_sp_rows_scatter(cudaStream_t st, const SpCopy& c, const TpArgs& tp, int grid);
// Long prompts' attention on the tensor cores: q [M, QD] fp32 -> bf16 (same
// layout), and rows [0, T) of the fp32 head-major K/V cache view (head h at
// h * max_seq rows) -> bf16 token-major [T, hkv, 128] for K and V (M = 0,
// q = nullptr: K and V only, e.g. the cached prefix when the QKV GEMM's
// epilogue wrote the new rows); then the tcgen05 causal prefill
// (sa_prefill.cu), which writes the o_proj GEMM's bf16 hi/lo planes.
int launch_tc_pack(cudaStream_t st, const float* q, int M, int QD, const float* kc, const float* vc, int max_seq,
                   int hkv, int T, __nv_bfloat16* qb, __nv_bfloat16* kb, __nv_bfloat16* vb, int num_sms);
// A block of query rows against a block of keys for prefill_pieces_launch
// (sa_prefill.cu): queries q_row0 .. q_row0+Sq-1 of the Q tensor, keys
// kv_row0 .. kv_row0+Skv-1 of the K/V tensors, query i seeing key j of the
// block when j <= q_pos0 + i; output rows `out`, and with `lse` the rows'
// log2-domain log-sum-exp of the scaled scores ([Sq][hq] floats), so that
// pieces of one query block over disjoint key blocks can be merged.
constexpr int kPrefillMaxPieces = 32;   // pieces of one prefill_pieces_launch
struct PrefillPiece {
    int q_row0 = 0, kv_row0 = 0, Sq = 0, Skv = 0, q_pos0 = 0;
    void* out = nullptr;
    float* lse = nullptr;
};
int prefill_pieces_launch(cudaStream_t st, int* status, const void* q, int q_rows, long long q_tok, const void* k,
                          const void* v, int kv_rows, long long kv_tok, int hq, int hkv, float scale, int out_dtype,
                          long long o_tok, const PrefillPiece* pieces, int n, void* out_lo = nullptr);
// out_lo != nullptr (with out_dtype SA_BF16): the output as two bf16 planes,
// out = bf16(o) and out_lo = bf16(o - out), the next GEMM's A operand.
int prefill_launch(cudaStream_t st, int* status, const void* q, const void* k, const void* v, void* out,
                   int out_dtype, int Sq, int Skv, int q_pos0, int hq, int hkv, long long q_tok, long long kv_tok,
                   long long o_tok, float scale, void* out_lo = nullptr);
int launch_sp_wait(cudaStream_t st, const TpArgs& tp);

// Model allocation for rank `rank` of `world` (sa_qwen3.cu).
int qwen3_create_model(sa_ctx* ctx, const sa_qwen3_config* cfg, int rank, int world, sa_qwen3** out);
int launch_amax_to_token(cudaStream_t st, unsigned long long* amax, int64_t* tok);

// ---- single-launch decode step (sa_qwen3_mega.cu) ---------------------------
struct MegaLayer {
    const __nv_bfloat16 *wqkv, *wo, *wgu, *wd;
    const float *in_norm, *post_norm, *q_norm, *k_norm;
};
struct MegaParams {
    const MegaLayer* layers;   // device array [L]
    int L, H, I, hq, hkv, V, max_seq;
    float eps;
    const __nv_bfloat16* embed;
    const __nv_bfloat16* lm_head;
    const float* final_norm;
    float *kc, *vc;
    const float *cos_t, *sin_t;
    float *x, *qkv, *attn, *act;
    float* part;               // [hkv][grid / hkv][hq / hkv][130]
    unsigned* head_cnt;        // [hkv], zeroed
    unsigned long long* amax;  // zeroed
    unsigned* gbar;            // [4], zeroed before a run of launches
    int* state;
    int64_t* ids;
    int64_t* toks;
    int toks_cap;
    int* status;
};
bool mega_supported(const sa_qwen3_config& c, int num_sms);
int mega_grid(int device);   // CTAs of one launch (one per SM), 0 if the device cannot run it
int launch_decode_mega(cudaStream_t st, int grid, const MegaParams& q);

// A host weight array in one of the element types a checkpoint may hold.
enum : int { QW_SRC_F32 = 0, QW_SRC_BF16 = 1, QW_SRC_F16 = 2 };
struct QwSrc {
    const void* p;
    int type;   // QW_SRC_*
};
// Upload the embedding / final norm / lm_head (lm_head.p NULL = tied) and one
// layer's weights from host arrays of any QW_SRC type; bf16 arrays are copied
// to the device as they are, others are rounded to bf16 on the host.  Shapes
// as sa_qwen3_set_embed / sa_qwen3_set_layer.  Blocking.
int qwen3_upload_embed(sa_qwen3* m, QwSrc embed, QwSrc final_norm, QwSrc lm_head);
int qwen3_upload_layer(sa_qwen3* m, int layer, QwSrc in_norm, QwSrc wq, QwSrc wk, QwSrc wv, QwSrc q_norm,
                       QwSrc k_norm, QwSrc wo, QwSrc post_norm, QwSrc w_gate, QwSrc w_up, QwSrc w_down);

}  // namespace sa
