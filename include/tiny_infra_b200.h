/*
 * tiny_infra_b200 -- C ABI of the B200 (sm_100a) kernels for the Tiny_Infra continuous-batching
 * decode/prefill hot path (Qwen2.5-0.5B architecture).
 *
 * Conventions
 *   - Plain device pointers, sizes and element strides; no framework types.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every entry point returns TI_OK (0) or a TI_ERR_* code; ti_last_error() gives the
 *     message of the last failure on the calling thread.  Launches are asynchronous: a kernel
 *     fault shows up in the next CUDA call on that stream.
 *   - Element types: TI_DTYPE_BF16 / TI_DTYPE_FP16 for activations and the KV pool.
 *   - Nothing here allocates device memory unless its comment says so; scratch space is a
 *     caller-provided `workspace` whose size a *_workspace_bytes() function returns.
 */
#ifndef TINY_INFRA_B200_H
#define TINY_INFRA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TI_DTYPE_BF16 0
#define TI_DTYPE_FP16 1
#define TI_DTYPE_FP32 2

#define TI_OK 0
#define TI_ERR_INVALID_ARGUMENT 1
#define TI_ERR_UNSUPPORTED 2
#define TI_ERR_CUDA 3
#define TI_ERR_WORKSPACE 4

/* Bits of the device status word (ti_device_status): a bounded wait inside a kernel gave up,
 * or a kernel rejected an input it cannot check on the host. */
#define TI_DEVERR_ATTN_WAIT 0x1u
#define TI_DEVERR_GEMM_WAIT 0x2u
#define TI_DEVERR_PREFILL_WAIT 0x4u
#define TI_DEVERR_ATTN_PLAN 0x8u   /* a planned attention call got a plan of another batch */
#define TI_DEVERR_BAD_INPUT 0x10u  /* a slot / position / block id outside the table or pool */

/* ---- library ---------------------------------------------------------------------------- */

/* Launch order.  Every kernel of this library is launched with programmatic dependent launch:
 * it may start while the previous kernel on the stream (if it is one of this library's) is
 * still running, and waits for it before touching its inputs -- except the weight operands
 * (ti_gemm's B, ti_gemm_qkv_rope's W, ti_rmsnorm's weight), which are fetched before that
 * wait.  They must therefore not be outputs of this library's kernels still in flight on the
 * same stream (weights written by other means, e.g. a copy, are fine).  The environment
 * variable TI_PDL=0 turns programmatic dependent launch off (plain stream order). */

/* Message of the last failed call on this thread ("" if none). */
const char* ti_last_error(void);
/* ABI version of this library. */
int ti_version(void);
/* Number of kernel launches this library has issued in this process (all threads). */
uint64_t ti_launch_count(void);
/* Read (and optionally clear) the device status word on the current device; synchronises
 * `stream`.  *bits receives the TI_DEVERR_* bits raised since the last clear. */
int ti_device_status(unsigned int* bits, int clear, void* stream);

/* ---- paged decode attention ----------------------------------------------------------
 * Replaces custom_paged_attn.launch_paged_attention (reference src/attention.cu:156-197,
 * binding src/attention_binding.cpp:3-13).
 *   out [batch, num_heads, head_dim] (row stride out_seq_stride elements, written in place)
 *   q   [batch, num_heads, head_dim] (row stride q_seq_stride elements)
 *   k_cache / v_cache: one layer of the pool, [num_blocks, num_kv_heads, block_size, head_dim]
 *   block_tables [*, max_blocks_per_seq] int32 (row stride bt_stride), -1 = unassigned;
 *   row_index [batch] int32 or NULL: block-table row of each sequence (NULL: row = sequence)
 *   context_lens [batch] int32.
 * Same semantics as the reference kernel: ctx 0 leaves the row untouched, reading stops at the
 * first negative entry, and a sequence with no readable token gets NaN.  Block ids >=
 * num_blocks are treated like -1.  head_dim 64 or 128, block_size 16, at most 16 query heads
 * per kv head.  head_dim 64 with batch <= 4096 runs a persistent kernel that splits the whole
 * batch's KV blocks evenly over the GPU's warps (split-K only where a sequence is cut);
 * otherwise one CTA per `partition_blocks` (1..16, 0 = 16) KV blocks.  A workspace of
 * ti_paged_attention_workspace_bytes() bytes is required.  Its first 64 KiB hold split-K
 * arrival counters (one per sequence and kv head, batch * num_kv_heads <= 16384): they must be
 * zero before the first call and every call leaves them zero; the rest is scratch.  Calls
 * that share a workspace must not overlap on the GPU. */
size_t ti_paged_attention_workspace_bytes(int batch, int num_heads, int num_kv_heads,
                                          int head_dim, int max_blocks_per_seq,
                                          int partition_blocks);
int ti_paged_attention_decode(void* out, int64_t out_seq_stride, const void* q,
                              int64_t q_seq_stride, const void* k_cache, const void* v_cache,
                              int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
                              const int32_t* row_index, const int32_t* context_lens, int batch,
                              int num_heads, int num_kv_heads, int head_dim, int block_size,
                              int max_blocks_per_seq, int dtype, int partition_blocks,
                              void* workspace, size_t workspace_bytes, void* stream);

/* ---- decode attention plan ------------------------------------------------------------------
 * No counterpart in the reference.  A decode step calls the attention once per layer with the
 * same batch (context_lens, block tables).  ti_paged_attention_plan resolves that batch once --
 * the split of all sequences' KV blocks over the GPU's attention consumers, each position's
 * pool row and valid-token count -- into a caller buffer of ti_paged_attention_plan_bytes(batch)
 * bytes (16-byte aligned).  ti_paged_attention_decode_planned computes exactly what
 * ti_paged_attention_decode does (default partitioning) but loads the plan instead of
 * rebuilding it.  The plan stays valid while context_lens and the block tables are unchanged; the calls
 * that read it must follow it on the same stream.  A plan of another batch raises
 * TI_DEVERR_ATTN_PLAN.  For shapes the planned kernel does not serve (head_dim != 64, an odd
 * number of kv heads, more than 8 query heads per kv head, batch > 4096, contexts too long for
 * the batch size) the plan is a zero header and the planned call behaves as the plain one. */
size_t ti_paged_attention_plan_bytes(int batch);
int ti_paged_attention_plan(const int32_t* block_tables, int64_t bt_stride,
                            const int32_t* row_index, const int32_t* context_lens, int batch,
                            int num_heads, int num_kv_heads, int head_dim, int max_blocks_per_seq,
                            int64_t num_blocks, void* plan, size_t plan_bytes, void* stream);
/* The plan with flags.  TI_ATTN_PLAN_AFTER_QKV: every attention call that reads the plan comes
 * right after ti_gemm_qkv_rope of the same `batch` rows (hidden size qkv_hidden, dtype), as in
 * a decode layer.  That GEMM holds some SMs when the attention grid launches, so the CTAs that
 * wait for them start a few microseconds late; the plan gives those CTAs fewer KV blocks (how
 * many fewer from the batch's KV bytes) so that all CTAs end together.  The output differs from
 * the unskewed plan's only by the float32 summation order of the split sequences. */
#define TI_ATTN_PLAN_AFTER_QKV 1
int ti_paged_attention_plan_ex(const int32_t* block_tables, int64_t bt_stride,
                               const int32_t* row_index, const int32_t* context_lens, int batch,
                               int num_heads, int num_kv_heads, int head_dim,
                               int max_blocks_per_seq, int64_t num_blocks, void* plan,
                               size_t plan_bytes, int flags, int qkv_hidden, int dtype,
                               void* stream);
int ti_paged_attention_decode_planned(void* out, int64_t out_seq_stride, const void* q,
                                      int64_t q_seq_stride, const void* k_cache,
                                      const void* v_cache, int64_t num_blocks,
                                      const int32_t* block_tables, int64_t bt_stride,
                                      const int32_t* row_index, const int32_t* context_lens,
                                      int batch, int num_heads, int num_kv_heads, int head_dim,
                                      int block_size, int max_blocks_per_seq, int dtype,
                                      void* workspace, size_t workspace_bytes, const void* plan,
                                      void* stream);
/* The same with flags.  TI_ATTN_EARLY_KV: the caller guarantees that the plan, and every KV
 * block of the batch except the last block of each sequence, were complete before the kernel
 * that precedes this call on the stream started (in a decode step: the plan is written before
 * layer 0 and only the new token's block changes); the kernel then loads the plan and starts
 * streaming those blocks while that kernel still runs (programmatic dependent launch), and
 * waits for it only before it reads q and the last blocks.  Results are identical to flags 0. */
#define TI_ATTN_EARLY_KV 1
int ti_paged_attention_decode_planned_ex(void* out, int64_t out_seq_stride, const void* q,
                                         int64_t q_seq_stride, const void* k_cache,
                                         const void* v_cache, int64_t num_blocks,
                                         const int32_t* block_tables, int64_t bt_stride,
                                         const int32_t* row_index, const int32_t* context_lens,
                                         int batch, int num_heads, int num_kv_heads, int head_dim,
                                         int block_size, int max_blocks_per_seq, int dtype,
                                         void* workspace, size_t workspace_bytes,
                                         const void* plan, int flags, void* stream);

/* ---- paged decode attention without caller scratch ---------------------------------------------
 * No counterpart in the reference.  Same computation and arguments as
 * ti_paged_attention_decode (default partitioning), but the split-K scratch is a static array
 * inside this library, so the caller allocates nothing.  Meant for callers that cannot call
 * cudaMalloc: a process whose device memory is already fully handed out (to the KV pool and a
 * caching allocator it does not own), or code running where a device allocation would
 * synchronise the device or is forbidden.  The array holds TI_NOALLOC_SCRATCH_BYTES (16 MiB) on
 * every GPU that loads the library, until the process exits; a batch whose scratch need
 * (ti_paged_attention_workspace_bytes) exceeds it is rejected with TI_ERR_WORKSPACE.  The first
 * call on each device looks the array's device address up (cudaGetSymbolAddress) and loads
 * the library's device code there: make that first call before any stream capture.  All calls
 * share the array; each clears its arrival counters on `stream` before launching, and calls
 * that overlap on the GPU race on the array.  A call that splits no sequence (head_dim 128 with
 * at most 16 blocks per sequence) uses no scratch and is never refused.  The looked-up address
 * belongs to the device's context: do not call this again after cudaDeviceReset of the device. */
#define TI_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int ti_paged_attention_decode_noalloc(void* out, int64_t out_seq_stride, const void* q,
                                      int64_t q_seq_stride, const void* k_cache,
                                      const void* v_cache, int64_t num_blocks,
                                      const int32_t* block_tables, int64_t bt_stride,
                                      const int32_t* row_index, const int32_t* context_lens,
                                      int batch, int num_heads, int num_kv_heads, int head_dim,
                                      int block_size, int max_blocks_per_seq, int dtype,
                                      void* stream);

/* ---- RoPE in place -------------------------------------------------------------------
 * Replaces custom_rope.apply_inplace (reference src/fused_rope.cu:84-128, binding
 * src/rope_binding.cpp:3-11): rotate-half RoPE on q [T, num_heads, head_dim] and
 * k [T, num_kv_heads, head_dim] (token strides q_tok_stride / k_tok_stride elements, heads
 * contiguous), tables cos/sin float32 [*, head_dim/2], positions pos [T] int32. */
int ti_rope_inplace(void* q, int64_t q_tok_stride, void* k, int64_t k_tok_stride,
                    const float* cos, const float* sin, const int32_t* pos, int num_tokens,
                    int num_heads, int num_kv_heads, int head_dim, int dtype, void* stream);

/* ---- RoPE fused with the KV-append write ---------------------------------------------
 * q/k/v of T new tokens, as laid out by the fused QKV projection: row t of `qkv` holds
 * [q (num_heads*head_dim) | k (num_kv_heads*head_dim) | v (num_kv_heads*head_dim)], row stride
 * qkv_stride elements.  Applies RoPE to q (in place) and k, then writes k and v into the pool at
 * slot_mapping[t] = physical_block * block_size + offset (reference
 * engine/cache_manager.py:95-99); slot_mapping < 0 skips the token's KV write. */
int ti_rope_kv_append(void* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                      const int64_t* slot_mapping, const float* cos, const float* sin,
                      const int32_t* pos, int num_tokens, int num_heads, int num_kv_heads,
                      int head_dim, int block_size, int dtype, void* stream);

/* ---- SwiGLU ----------------------------------------------------------------------------
 * Replaces custom_swiglu.forward (reference src/fused_swiglu.cu:56-93): out[t, i] =
 * silu(x[t, i]) * x[t, I + i] for x [T, 2I] (gate half first), out [T, I]; I % 8 == 0,
 * contiguous rows. */
int ti_swiglu(void* out, const void* x, int64_t num_tokens, int inter, int dtype, void* stream);

/* ---- RMSNorm ----------------------------------------------------------------------------
 * models/qwen_25.py:24-36.  out[t] = w * (x[t] * rsqrt(mean(x[t]^2) + eps)), x float32 or
 * the activation dtype (x_dtype), out and w in `dtype`.  The normalised row is rounded to
 * `dtype` before the weight multiply, as the reference does.  `weight` is read before the
 * kernel waits for the previous kernel on the stream (see "Launch order" above). */
int ti_rmsnorm(void* out, const void* x, int x_dtype, const void* weight, float eps,
               int num_tokens, int hidden, int dtype, void* stream);

/* Embedding gather: out[t] (float32 residual stream) = table[ids[t]] (dtype rows of `hidden`).
 * Token ids outside [0, vocab) produce a zero row and raise no error. */
int ti_embedding(float* out, const void* table, const int32_t* ids, int num_tokens, int hidden,
                 int64_t vocab, int dtype, void* stream);

/* ---- projections on tcgen05 tensor cores -----------------------------------------
 * Replaces the reference's nn.Linear calls (models/qwen_25.py:46-49,66-68,130,136-151,237-250)
 * with D[M, N] = A[M, K] . B[N, K]^T (A activations row-major, B an nn.Linear weight
 * [out_features, in_features], both `dtype`, fp32 accumulation in TMEM) and a fused epilogue:
 *   TI_EPI_STORE     out[M, N] (dtype, leading dim ldo) = D + bias (bias [N] or NULL)
 *   TI_EPI_SWIGLU    out[M, N/2] = silu(gate) * up (fused_swiglu.cu:39-50), where every group
 *                    of block_n weight rows holds block_n/2 gate rows followed by the matching
 *                    block_n/2 up rows
 *   TI_EPI_SWIGLU16  out[M, N/2] = silu(gate) * up with every 16 weight rows holding 8 gate rows
 *                    followed by the matching 8 up rows (N % 16 == 0); block_n and split_k are
 *                    ignored: the library picks the tile width (up to 256 rows: 80 or 144, so
 *                    that one wave of CTAs covers the GPU; above: 256)
 *   TI_EPI_RESIDUAL  out (float32 [M, N], ldo) += D
 *   TI_EPI_RESIDUAL_DET  the same, bit-reproducible: the K slices of a tile run on a
 *                    thread-block cluster (1, 2, 4 or 8 slices) and are summed in a fixed order
 *                    before the one add per element (parity runs; ~13 % slower decode steps)
 *   TI_EPI_ARGMAX    aux_val/aux_idx [M, N/block_n] = (max, first argmax) of each row within each
 *                    block_n column tile; `out` (dtype logits) is also written when not NULL
 * split_k is an upper bound on the split-K factor; it is lowered until the launch fits one wave
 * of the GPU and each K slice has at least two 64-wide K blocks.  RESIDUAL (up to 16 slices):
 * every slice adds its partial sums into `out` with atomic adds, so the order of the fp32
 * additions -- and the last bits of `out` -- can vary from run to run.  STORE / SWIGLU
 * (1, 2, 4 or 8 slices; block_n 64 or 128): the slices of a tile run on a thread-block cluster
 * and are summed in a fixed order through distributed shared memory (deterministic).  ARGMAX
 * and block_n 256 do not split.
 * Requirements: N % block_n == 0 (block_n 64, 128 or 256; 0 = 128), K % 64 == 0, 16-byte
 * aligned operands with leading dimensions multiple of 8 elements. */
#define TI_EPI_STORE 0
#define TI_EPI_SWIGLU 1
#define TI_EPI_RESIDUAL 2
#define TI_EPI_ARGMAX 3
#define TI_EPI_SWIGLU16 5
#define TI_EPI_RESIDUAL_DET 6
int ti_gemm(int epilogue, const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N,
            int K, void* out, int64_t ldo, const void* bias, float* aux_val, int32_t* aux_idx,
            int dtype, int block_n, int split_k, void* stream);

/* ---- weight-only INT8 lm_head (greedy decoding) --------------------------------------------
 * The reference names weight-only INT8/INT4 quantised projections as its next step
 * (README.md:156-157) and has no implementation; these two calls apply it to the tied lm_head
 * (models/qwen_25.py:237,250).
 * ti_quantize_rows_int8: per row r of w [rows, cols] (dtype, leading dim ldw):
 *   scale[r] = max_c |w[r, c]| / 127 (1 for an all-zero row), q[r, c] = rint(w[r, c] / scale[r])
 *   clamped to [-127, 127] (int8, leading dim ldq).  cols, ldw, ldq multiples of 8.
 * ti_lm_head_argmax_int8: logits[m, n] = scale[n] * sum_k A[m, k] q[n, k] (A: M <= 256 rows of
 *   dtype, fp32 accumulation of the exact products) reduced, like TI_EPI_ARGMAX with block_n 128,
 *   to aux_val / aux_idx [M, N / 128] = (max, first argmax) of each row in each 128-column tile
 *   (finish with ti_argmax_finish).  N % 128 == 0, K % 64 == 0, ldb (bytes) % 16 == 0, 16-byte
 *   aligned operands.  The int8 weights are half the bytes of bf16 ones. */
int ti_quantize_rows_int8(const void* w, int64_t ldw, int rows, int cols, int8_t* q, int64_t ldq,
                          float* scale, int dtype, void* stream);
int ti_lm_head_argmax_int8(const void* A, int64_t lda, const int8_t* Bq, int64_t ldb,
                           const float* scale, int M, int N, int K, float* aux_val,
                           int32_t* aux_idx, int dtype, void* stream);

/* ---- QKV projection fused with RoPE and the KV-append write ----------------------
 * [q | k | v] = A[M, hidden] . W^T + bias, W = the fused [(NH+2*KVH)*64, hidden] q/k/v weight
 * (models/qwen_25.py:46-48,66-68).  RoPE (src/fused_rope.cu:37-50, tables cos/sin float32
 * [*, 32], positions pos[M]) is applied to q and k on the fp32 accumulators, so each value is
 * rounded to `dtype` once; q goes to q_out [M, NH*64] (leading dim ldq), k and v go straight to
 * the pool at slot_mapping[m] (< 0: skipped) as engine/cache_manager.py:95-99 would place them.
 * head_dim must be 64. */
#define TI_EPI_QKV_ROPE 4
int ti_gemm_qkv_rope(const void* A, int64_t lda, const void* W, int64_t ldw, const void* bias,
                     int M, int hidden, int num_heads, int num_kv_heads, int head_dim,
                     void* q_out, int64_t ldq, void* k_cache, void* v_cache,
                     const int64_t* slot_mapping, const float* cos, const float* sin,
                     const int32_t* pos, int block_size, int dtype, void* stream);

/* ---- ragged causal prefill attention over the paged pool -----------------------------------
 * Replaces the prefill branch of Qwen2Attention.forward (reference models/qwen_25.py:89-104,
 * SDPA over the call's own tokens) with attention over the pool, so chunks of a prompt can be
 * prefilled separately and several sequences packed in one call.  Sequence i's new tokens are
 * query rows cu_seqlens[i] .. cu_seqlens[i+1]-1 of q/out ([rows, num_heads, head_dim], token
 * strides in elements) at positions start_pos[i] + j; their K/V must already be in the pool
 * (ti_rope_kv_append).  Each query attends causally to positions 0 .. its own.  Work is given
 * as query tiles of up to 16 tokens: tile t covers chunk tile_seq[t] from token tile_q0[t]. */
int ti_paged_prefill_attention(void* out, int64_t out_tok_stride, const void* q,
                               int64_t q_tok_stride, const void* k_cache, const void* v_cache,
                               int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
                               const int32_t* row_index, const int32_t* start_pos,
                               const int32_t* cu_seqlens, const int32_t* tile_seq,
                               const int32_t* tile_q0, int num_tiles, int num_heads,
                               int num_kv_heads, int head_dim, int block_size, int dtype,
                               void* stream);

/* ---- sampler: temperature / top-k / top-p / draw ----------------------------------------------
 * Replaces ContinuousBatcher._sample_next_token (engine/scheduler.py:104-156) for `rows` rows of
 * logits [rows, vocab] (leading dimension ld elements, dtype bf16 / fp16 / fp32).  Per row r:
 * x = logits[r] / temperatures[r] (temperature 0: the result is the first argmax);
 * cut_ks[r] > 0 keeps x >= the cut_ks[r]-th largest value (0: no cut); top_ps[r] < 1 keeps the
 * descending order up to and including the first token whose cumulative softmax probability
 * exceeds top_ps[r] (>= 1: no cut); the token is the first kept one in descending order (ties:
 * lower index first) whose cumulative probability exceeds uniforms[r] in [0, 1).
 * The reference's batch-level rules (top-k only in rows whose top_k equals the batch's largest
 * one, :119-130; top-p in every row once any row has p < 1, :133-134) are applied by the caller
 * when it fills cut_ks / top_ps.  out_tokens[r] receives the token; when slots / seq_len are not
 * NULL, seq_len[slots[r]] += seq_inc for slots[r] >= 0. */
int ti_sample(const void* logits, int64_t ld, int dtype, int rows, int vocab,
              const float* temperatures, const int32_t* cut_ks, const float* top_ps,
              const float* uniforms, int32_t* out_tokens, const int32_t* slots, int32_t* seq_len,
              int seq_inc, void* stream);

/* ---- decode-step packing on the device ---------------------------------------------
 * For rows r < rows: slot = slots[r] (-1 = padding row).  First writes this step's new block,
 * block_tables[slot][seq_len[slot] / block_size] = new_block[r] when new_block[r] >= 0 (the
 * host allocator decided it, FIFO order of engine/cache_manager.py:86-92), then sets
 * positions[r] = seq_len[slot] (models/qwen_25.py:218-222), slot_mapping[r] (pool slot of the
 * new token), ctx_lens[r] = seq_len[slot] + 1 (models/qwen_25.py:115) and hidden[r] (float32)
 * = embed[tokens[r]].  Padding rows get slot_mapping -1, ctx 0 and a zero hidden row.
 * block_tables has num_slots rows of max_blocks_per_seq entries (row stride bt_stride); the pool
 * has num_blocks blocks.  A slot >= num_slots or a position beyond the row's last block makes
 * the row padding, a new_block >= num_blocks is not written, a table entry >= num_blocks gets
 * no pool slot (-1); each raises TI_DEVERR_BAD_INPUT. */
int ti_decode_prepare(const int32_t* tokens, const int32_t* slots, const int32_t* new_block,
                      const int32_t* seq_len, int32_t* block_tables, int64_t bt_stride,
                      int num_slots, int max_blocks_per_seq, int64_t num_blocks,
                      int block_size, int32_t* positions, int64_t* slot_mapping,
                      int32_t* ctx_lens, float* hidden, const void* embed, int hidden_size,
                      int64_t vocab, int rows, int dtype, void* stream);

/* Greedy token per row from TI_EPI_ARGMAX partials (largest value, lowest index among equal
 * values; reference engine/scheduler.py:153 uses torch.argmax), written to out_tokens[rows].
 * If seq_len and slots are given, seq_len[slots[r]] += seq_inc for every slot >= 0
 * (engine/scheduler.py:266). */
int ti_argmax_finish(const float* part_val, const int32_t* part_idx, int ntiles, int rows,
                     int32_t* out_tokens, const int32_t* slots, int32_t* seq_len, int seq_inc,
                     void* stream);

/* Write K/V rows of num_tokens tokens into the pool at slot_mapping[t] (-1 = skip):
 * k/v element (t, h, d) at t*tok_stride + h*head_stride + d.  The write of
 * engine/cache_manager.py:95-99.  Slots at or beyond num_blocks * block_size (outside the pool
 * of num_blocks blocks) are not written and raise TI_DEVERR_BAD_INPUT. */
int ti_kv_scatter(void* k_cache, void* v_cache, const void* k, int64_t k_tok_stride,
                  int64_t k_head_stride, const void* v, int64_t v_tok_stride,
                  int64_t v_head_stride, const int64_t* slot_mapping, int num_tokens,
                  int64_t num_blocks, int num_kv_heads, int head_dim, int block_size, int dtype,
                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TINY_INFRA_B200_H */
