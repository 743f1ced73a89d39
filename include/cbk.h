/*
 * cbk.h -- C ABI of libcbk, the sm_100a kernels behind CacheBlend's
 * selective-KV-recompute path.
 *
 * All tensor arguments are DEVICE pointers on the current CUDA device; every
 * call is asynchronous on `stream` (a cudaStream_t / CUstream handle) and never
 * synchronises the host.  Nothing here allocates device memory: buffers,
 * descriptor tables and workspaces are owned by the caller.  Calls are
 * re-entrant (no mutable global state other than the per-thread error text).
 *
 * Return value: CBK_OK (0) or a negative CBK_ERR_* code; cbk_last_error()
 * returns a message for the most recent failure on the calling thread.
 * Errors that can only be seen on the device (an index outside the fused
 * sequence, a bounded wait that gave up) are OR-ed into the optional
 * `status` word (device int32, may be NULL) as CBK_STATUS_* bits; the kernel
 * skips the offending access instead of faulting.
 *
 * Element types: CBK_BF16 or CBK_F16 for every K/V/Q tensor of one call.
 * Layouts follow the reference's memory layout:
 *   - a chunk's cached K (pre-RoPE) and V for one layer: [len][kv_dim] row-major,
 *     kv_dim = n_kv_heads * head_dim (cacheblend/kv_store.py:7-9, one
 *     `(1, Lc, Hkv*D)` tensor per chunk per layer);
 *   - the fused cache of one layer: [S][n_kv_heads][head_dim] (token-major),
 *     which is the memory order of the reference's DynamicCache tensors
 *     (fusor.py:439-460 builds them as transposed views of `(1, S, Hkv*D)`);
 *   - selected queries: [n_sel][n_q_heads][head_dim]; attention output:
 *     [n_sel][n_q_heads * head_dim] (the o_proj input of fusor.py:471-474).
 */
#ifndef CBK_H_
#define CBK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CBK_ABI_VERSION 1

enum {
  CBK_OK = 0,
  CBK_ERR_INVALID = -1,      /* bad argument: NULL, size, stride or alignment */
  CBK_ERR_UNSUPPORTED = -2,  /* dtype / head_dim / GQA group not supported */
  CBK_ERR_CUDA = -3,         /* CUDA runtime or launch error */
  CBK_ERR_WORKSPACE = -4     /* caller workspace too small */
};

enum { CBK_BF16 = 0, CBK_F16 = 1 };

/* RoPE rounding modes for K/Q rotation.
 * CBK_ROPE_REF:  reproduce HF `apply_rotary_pos_emb` on 16-bit tensors: cos/sin
 *                rounded to the element type, each product rounded, the sum
 *                rounded (modeling_mistral.py rotate_half / apply_rotary_pos_emb,
 *                MistralRotaryEmbedding.forward casts cos/sin to x.dtype).
 * CBK_ROPE_FP32: rotate in fp32 with one final rounding (more accurate). */
enum { CBK_ROPE_REF = 0, CBK_ROPE_FP32 = 1 };
/* cbk_rope_scatter only, OR-ed into rope_mode: rope_table row j holds the
 * cos/sin of position idx[j] (a copy of the position-indexed table's rows at
 * the selection, made once per selection), so the kernel loads it without
 * waiting for idx[j]; table_rows must be >= n_sel. */
enum { CBK_ROPE_TABLE_BY_ROW = 16 };

/* Device status bits (OR-ed into *status). */
enum {
  CBK_STATUS_BAD_INDEX = 1,     /* a position / row index outside its buffer; access skipped */
  CBK_STATUS_TIMEOUT = 2,       /* a bounded wait inside a kernel gave up */
  CBK_STATUS_COUNT = 4          /* top-K count check failed */
};

/* One chunk's cached tensors for one layer (device pointers, row-major
 * [len][kv_dim], rows contiguous). */
typedef struct {
  const void* k;
  const void* v;
} cbk_chunk_src;

const char* cbk_last_error(void);
int cbk_abi_version(void);

/* RoPE table: table[p * half_dim + i] = (cos, sin)(inv_freq[i] * p) * attention_scaling,
 * fp32, for p in [0, n_pos).  inv_freq is the model's own buffer (device, fp32).
 * Replaces the per-call `rotary_emb(x, position_ids)` of fusor.py:285 and
 * rope.py:54 (MistralRotaryEmbedding.forward, angle = fp32(inv_freq) * fp32(pos)). */
int cbk_rope_table(const float* inv_freq, int half_dim, int64_t n_pos,
                   float attention_scaling, void* table /* float2[n_pos][half_dim] */,
                   void* stream);

/* (a)+(b) chunk-KV concatenation with RoPE shift, all layers in one launch.
 * For every layer l < n_layers and fused row t in [0, S): find chunk c with
 * chunk_start[c] <= t < chunk_start[c+1]; then
 *   k_out[l][t] = RoPE(srcs[l*n_chunks+c].k[t - chunk_start[c]], pos(t))
 *   v_out[l][t] = srcs[l*n_chunks+c].v[t - chunk_start[c]]
 * with pos(t) = positions ? positions[t] : t.  Output rows have kv_dim
 * elements; layer l starts at element l * out_layer_stride.
 * Replaces fusor.py:258-272 (zeros + per-chunk slice copies) together with the
 * cached-K rotation of fusor.py:439-447 (rope.py:33-64 applied to the concat). */
int cbk_assemble_kv(const cbk_chunk_src* srcs, const int64_t* chunk_start, int n_chunks,
                    int n_layers, int64_t S, int n_kv_heads, int head_dim, int dtype,
                    const void* rope_table, int64_t table_rows, const int64_t* positions,
                    int rope_mode, void* k_out, void* v_out, int64_t out_layer_stride,
                    int32_t* status, void* stream);

/* apply_rope_shift (rope.py:33-64) on plain rows: out[r] = RoPE(in[r], positions[r])
 * for r < n_rows, rows of n_heads*head_dim elements (in/out may alias). */
int cbk_rope_rows(const void* in, void* out, int64_t n_rows, int n_heads, int head_dim,
                  int dtype, const void* rope_table, int64_t table_rows,
                  const int64_t* positions, int rope_mode, int32_t* status, void* stream);

/* (b)+(d) fresh rows of one layer.  For j < n_sel, with src row
 * r = gather ? idx[j] : j and position p = idx[j]:
 *   q_out[j]      = RoPE(q_src[r], p)              [n_sel][n_q_heads*head_dim]
 *   k_cache[p]    = RoPE(k_src[r], p)              fused [S][kv_dim]
 *   v_cache[p]    = v_src[r]
 * Row strides are in elements.  With CBK_ROPE_TABLE_BY_ROW in rope_mode the
 * cos/sin of row j are rope_table row j instead of row p.  Replaces
 * fusor.py:355-361 + 370-376 (check
 * layer: mixed K, RoPE of Q and K, Q sliced to the selection) and
 * fusor.py:432-458 (sparse layers: RoPE of sparse Q/K, clone + index_put of K/V). */
int cbk_rope_scatter(const void* q_src, int64_t q_row_stride, const void* k_src,
                     int64_t k_row_stride, const void* v_src, int64_t v_row_stride,
                     int gather, const int64_t* idx, int64_t n_sel, int64_t S,
                     int n_q_heads, int n_kv_heads, int head_dim, int dtype,
                     const void* rope_table, int64_t table_rows, int rope_mode,
                     void* q_out, void* k_cache, void* v_cache, int32_t* status, void* stream);

/* (c) HKVD deviation (hkvd.py:23-55, kv_deviation):
 *   dev[t] = sum_f (K_new[t][f] - K_old[t][f])^2 in fp32, fixed order: each
 * 8-element vector's squares summed in element order, then a complete binary
 * tree of pairwise adds over the vectors (zero-padded to a power of two).  The
 * deviation of an aligned power-of-two slice of the features (one rank's KV
 * heads) is a node of that tree, so slices combined with the same tree give
 * these bits exactly.  K_new rows have stride new_row_stride elements; K_old
 * rows come from the chunk table (srcs[c].k, c < n_chunks, rows
 * chunk_start[c] .. chunk_start[c+1]).  feat % 8 == 0, feat < 2^27. */
int cbk_kv_deviation(const void* k_new, int64_t new_row_stride, const cbk_chunk_src* old_srcs,
                     const int64_t* chunk_start, int n_chunks, int64_t S, int64_t feat,
                     int dtype, float* dev, void* stream);

/* k selected count of select_top_k (hkvd.py:70-73): max(1, min(S, (int64)(S * ratio))). */
int64_t cbk_topk_count(int64_t S, double ratio);

/* (c) top-K select (hkvd.py:58-77) + optional force-include of S-1 (fusor.py:344-353).
 * idx[0..k) = the k largest dev values' indices, ascending.  Ties at the k-th
 * value are taken lowest index first.  With force_last != 0 and S-1 not
 * selected, the lowest-index selected element equal to the k-th value (the
 * reference's argmin pick) is dropped and S-1 appended.  One CTA, no workspace. */
int cbk_topk_select(const float* dev, int64_t S, int64_t k, int force_last, int64_t* idx,
                    int32_t* status, void* stream);

/* (c) deviation + select in one call.  `workspace` (device, >= cbk_hkvd_workspace_bytes(S))
 * receives dev[S] (readable afterwards as float[S]). */
size_t cbk_hkvd_workspace_bytes(int64_t S);
int cbk_hkvd_select(const void* k_new, int64_t new_row_stride, const cbk_chunk_src* old_srcs,
                    const int64_t* chunk_start, int n_chunks, int64_t S, int64_t feat, int dtype,
                    int64_t k, int force_last, int64_t* idx, void* workspace, size_t workspace_bytes,
                    int32_t* status, void* stream);

/* (c) deviation + select with no allocation at all: the deviation scores live in
 * a fixed device array owned by the library (cbk_hkvd_noalloc_max_tokens() fp32
 * entries, 1 MiB, kept on every GPU that loads the library until exit).  For
 * callers that cannot allocate device memory when they select (an engine that
 * has reserved the HBM for its own pools, or a step where cudaMalloc would
 * synchronise the device).  No counterpart in the reference.  Same arguments
 * and results as cbk_hkvd_select without the workspace; S above the maximum is
 * rejected (CBK_ERR_INVALID).  The first call on a device looks up the array's
 * address (make it before any stream capture) and keeps it for the process; a
 * device reset (cudaDeviceReset, or a reset of the primary context) reloads the
 * module and invalidates that address, so do not call this entry point on a
 * device after resetting it.  Calls that overlap on the GPU share the array and
 * race. */
int64_t cbk_hkvd_noalloc_max_tokens(void);
int cbk_hkvd_select_noalloc(const void* k_new, int64_t new_row_stride, const cbk_chunk_src* old_srcs,
                            const int64_t* chunk_start, int n_chunks, int64_t S, int64_t feat,
                            int dtype, int64_t k, int force_last, int64_t* idx, int32_t* status,
                            void* stream);

/* (e) partial-query attention on tcgen05 (fusor.py:381-399, 462-474):
 *   out[j][h] = softmax_t<=pos[j]( scale * q[j][h] . k[t][h/G] ) . v[t][h/G]
 * for j < n_sel, h < n_q_heads, G = n_q_heads / n_kv_heads, keys t in [0, pos[j]].
 * q: [n_sel][n_q_heads][head_dim]; k/v: [S][n_kv_heads][head_dim]; pos ascending
 * (int64), distinct, each in [0, S).  head_dim 64 or 128; G in {1,2,4,8,16};
 * S <= 262144.  fp32 accumulation in TMEM, fp32 online softmax, 16-bit P and
 * output.  The key range of long query tiles is split across CTAs; a plan
 * (computed on the device from pos) and the split partial results live in the
 * caller's `workspace` (>= cbk_partial_attn_workspace_bytes(...) bytes, which
 * depends on the current device's SM count).  With reuse_plan != 0 the plan
 * already in `workspace` is reused: the caller guarantees the same pos, n_sel
 * and head geometry as the call that built it (e.g. every sparse layer of one
 * blended prefill).  Three launches: plan (unless reused), attention, combine. */
size_t cbk_partial_attn_workspace_bytes(int64_t n_sel, int64_t S, int n_q_heads, int n_kv_heads,
                                        int head_dim);
int cbk_partial_attn(const void* q, const void* k, const void* v, const int64_t* pos,
                     int64_t n_sel, int64_t S, int n_q_heads, int n_kv_heads, int head_dim,
                     float scale, int dtype, void* out, void* workspace, size_t workspace_bytes,
                     int reuse_plan, int32_t* status, void* stream);

/* Decoder-layer row kernels around the recompute path.  They replace the HF
 * modules that fuse_selective runs between its projections (transformers
 * MistralRMSNorm/LlamaRMSNorm.forward, MistralMLP/LlamaMLP act_fn(gate) * up,
 * and the residual adds of MistralDecoderLayer.forward) with the same 16-bit
 * roundings, one HBM pass each.
 *
 * cbk_add_rmsnorm: for r < n_rows, with s = x[src] (src = rows ? rows[r] : r,
 * 0 <= src < x_rows) plus delta[r] when delta is not NULL (sum rounded to 16
 * bits, like torch's bf16 add):
 *   out[r] = weight * round16(s * rsqrt(mean(s^2) + eps))   (rounded to 16 bits)
 * and sum_out[r] = s when sum_out is not NULL (sum_out may equal x only when
 * rows is NULL).  cols % 8 == 0, cols <= 8192; 16-byte aligned pointers, row
 * strides (elements) multiples of 8.  An out-of-range rows[r] sets
 * CBK_STATUS_BAD_INDEX and leaves row r untouched.
 *
 * cbk_silu_mul: out[r][c] = round16(round16(g / (1 + exp(-g))) * up[r][c]),
 * g = gate[r][c] (torch's silu in fp32, then the 16-bit product). */
int cbk_add_rmsnorm(const void* x, int64_t x_stride, int64_t x_rows, const int64_t* rows,
                    const void* delta, int64_t delta_stride, void* sum_out, int64_t sum_stride,
                    const void* weight, float eps, int64_t n_rows, int cols, int dtype, void* out,
                    int64_t out_stride, int32_t* status, void* stream);
int cbk_silu_mul(const void* gate, int64_t gate_stride, const void* up, int64_t up_stride,
                 int64_t n_rows, int cols, int dtype, void* out, int64_t out_stride, void* stream);

/* One-row projection of a decode step (the HF q/k/v, o, gate/up, down and
 * lm_head Linear layers at one token, runners.py:106-152 via the model
 * forward): y[i] = round16(sum_j w[i][j] x[j]) for i < n, accumulated in fp32
 * (order differs from cuBLAS: results agree within fp32 rounding).  w: n rows
 * of k elements with row stride w_row_stride (elements, multiple of 8), k % 8
 * == 0, k <= 16384; 16-byte aligned pointers.  When gate and up are given
 * (both, instead of x), x[j] = round16(round16(silu(gate[j])) * up[j]) as in
 * cbk_silu_mul. */
int cbk_gemv(const void* w, int64_t w_row_stride, const void* x, const void* gate, const void* up,
             int64_t n, int k, int dtype, void* y, void* stream);

/* Attention of one query token at position *pos over cache rows 0..*pos (a
 * greedy decode step, runners.py:106-152 through the HF attention with
 * past_key_values): out[hq] = softmax(scale * q[hq] . K[j]) V[j] over j <= *pos
 * for each q head hq (G = n_q_heads / n_kv_heads in {1, 2, 4, 8} heads per KV head).
 * q, out: [n_q_heads][head_dim]; k_cache, v_cache: cap rows of kv_row_stride
 * elements (>= n_kv_heads * head_dim, multiple of 8), head h at h * head_dim.
 * *pos is read on the device (a captured graph stays valid as it advances); a
 * *pos outside [0, cap) sets CBK_STATUS_BAD_INDEX and leaves out untouched.
 * fp32 throughout, one rounding of the output.  head_dim 64 or 128.  The
 * workspace (cbk_decode_attn_workspace_bytes) holds the per-split partial
 * results between the two kernels of a call; it needs no initialisation, and
 * calls that overlap on the GPU must not share it. */
size_t cbk_decode_attn_workspace_bytes(int64_t cap, int n_q_heads, int n_kv_heads, int head_dim);
int cbk_decode_attn(const void* q, const void* k_cache, const void* v_cache, int64_t kv_row_stride,
                    const int64_t* pos, int64_t cap, int n_q_heads, int n_kv_heads, int head_dim, float scale,
                    int dtype, void* out, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Dense logits of the selected rows (fusor.py:483-491, the (1, S, vocab) zeros
 * plus index_copy_): dst[r] = src[j] for idx[j] == r, zero rows elsewhere, each
 * output byte written once.  idx: k int64 ascending distinct positions in
 * [0, S); rows of row_bytes (multiple of 16), 16-byte aligned, byte strides. */
int cbk_scatter_rows(const void* src, int64_t src_stride_bytes, const int64_t* idx, int64_t k, void* dst,
                     int64_t dst_stride_bytes, int64_t S, int64_t row_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CBK_H_ */
