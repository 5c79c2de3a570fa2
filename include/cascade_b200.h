/*
 * cascade_b200.h - C ABI of libcascade_b200.so, the sm_100a kernels behind the
 * Llama-3.1-8B decode path of Cascade-LLM's `layer_streaming` package.
 *
 * Conventions for every entry point:
 *   - plain device pointers (BF16 data as `void*`, row-major, 16-byte aligned),
 *     element counts, and a `cudaStream_t` passed as `void* stream`;
 *   - nothing allocates: scratch workspaces and zero-initialised counters
 *     are caller-provided (the kernels leave the counters zero again);
 *   - the return value is 0 on success, else a nonzero cb_status code, and
 *     cb_last_error() describes the failure (thread-local);
 *   - kernels are enqueued asynchronously on `stream`; none synchronises the
 *     host, so calls can be captured into a CUDA graph;
 *   - each BF16 rounding point of the reference's PyTorch ops is reproduced
 *     (llama31.py: F.linear -> bf16, residual adds, SiLU, gate*up, RoPE).
 *
 * Reference file:line citations are paths inside the Cascade-LLM project.
 */
#ifndef CASCADE_B200_H
#define CASCADE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum cb_status { CB_OK = 0, CB_ERR_INVALID = 1, CB_ERR_CUDA = 2, CB_ERR_UNSUPPORTED = 3 };

/* Library version (major*10000 + minor*100 + patch). */
int cb_version(void);
/* Message of the last failure on this host thread ("" if none). */
const char* cb_last_error(void);
/* Enable (1) / disable (0) programmatic dependent launch between the
 * engine's kernels (default: enabled). Returns the previous setting. */
int cb_set_pdl(int enable);
/* Number of SMs of the current device (grid size of the streaming kernels). */
int cb_sm_count(void);
/* One-time per-device set-up of the kernels (shared-memory limits). Call it
 * with the device current before capturing engine calls into a CUDA graph;
 * entry points otherwise do it on first use. */
int cb_prepare(void);
/* Registers a caller-owned device int32 (zeroed) that kernels set to a
 * nonzero code when a bounded wait gives up or an index is out of range,
 * instead of hanging or faulting. NULL disables the reporting. One word per
 * process (one process per GPU). The host reads it between steps. */
int cb_set_error_word(int32_t* device_word);
/* Per-CTA launch timeline of the decode kernels, for profiling: launches
 * issued while a buffer is set append one record per CTA (u64 words: the
 * buffer's word 0 is the record count, to be zeroed by the caller, word 1 the
 * capacity in records; record r is the 8 words at 8 * (r + 1): launch tag
 * << 32 | CTA index, SM id, and %globaltimer ns at CTA start, after the
 * dependency wait, after the main loop, at the end). Launch tags count up
 * from 0 per cb_set_trace call, in issue order (a captured graph replays its
 * tags). NULL (the default) turns tracing off. */
int cb_set_trace(void* device_buffer);
/* Cross-kernel L2 staging of a decode layer's gate+up weights. No
 * counterpart in the reference (an HBM-residency scheduling hint of this
 * engine). The QKV, attention and o_proj launches of a layer are
 * latency-bound and leave HBM mostly idle, while the gate+up projection that
 * follows them streams 235 MB; launches of kind `kind` (0 QKV, 1 one-token
 * attention, 2 o_proj = cb_proj_residual with K = N = 4096) issued while a
 * target is set prefetch into L2 `take` units (row pairs) per gate+up CTA,
 * after the `skip` units that CTA loads before its dependency wait anyway.
 * `where` is the issue point (0 off; GEMV: 1 before the dependency wait,
 * 2 after it, 3 at the end; attention: 1 at the start, 2 after the last
 * K/V copy is issued, 3 after the sub-chunk loop, 4 after the merge);
 * `policy` 0 normal, 1 evict_last L2 priority. Default: the attention
 * kernel stages 10 row pairs per gate+up CTA after its sub-chunk loop
 * (kind 1: where 3, take 10, skip 4); QKV and o_proj stage nothing. */
int cb_set_l2_stage(int kind, int where, int take, int skip, int policy);
/* The gate+up slabs (gate rows, up rows: `units` rows of K bf16 each) that
 * launches issued from now on stage; w_gate NULL clears the target. A
 * captured graph keeps the target of its capture. The target is
 * process-wide: clear it before the slabs are freed (the executor sets it
 * for the launches of one step and clears it after them). */
int cb_set_l2_stage_target(const void* w_gate, const void* w_up, int units, int K);

/* ---------------------------------------------------------------- set-up */

/* Seeded N(0, std) BF16 initialiser: element i of the stream `key`
 * (key = cb_stream_key(seed, tensor_name)). Same bits as the CPU oracle.
 * Replaces the checkpoint load of layer_streaming/weight_store.py:109-171
 * for the random-init benchmark configurations. */
uint64_t cb_stream_key(uint64_t seed, const char* tensor_name);
int cb_fill_normal_bf16(void* out, int64_t n, int64_t offset, uint64_t key, double std_dev,
                        void* stream);
int cb_fill_bf16(void* out, int64_t n, float value, void* stream);

/* Device position counter of the request (int32): the first position of
 * the next step. cb_position_set copies an int64 device position (e.g.
 * position_ids[0, 0]) or, if src is NULL, `value`. cb_position_advance adds
 * `count` (after a step of `count` tokens). */
int cb_position_set(int32_t* position, const int64_t* src, int32_t value, void* stream);
int cb_position_advance(int32_t* position, int32_t count, void* stream);

/* ---------------------------------------------------------------- layers */

/* Row gather of token embeddings. Replaces F.embedding
 * (layer_streaming/llama31.py:144-148). ids: int64 [M] (device);
 * table: [vocab, hidden]; out: [M, hidden]. Out-of-range ids -> error word. */
int cb_embedding(const int64_t* ids, int M, const void* table, int64_t vocab, int hidden, void* out,
                 void* stream);

/* RMSNorm (layer_streaming/llama31.py:21-25): out = bf16(w * bf16(x * rsqrt(mean(x^2)+eps))).
 * x, out: [M, hidden]; w: [hidden]. */
int cb_rmsnorm(const void* x, const void* w, int M, int hidden, float eps, void* out, void* stream);

/* Fused input RMSNorm + Q/K/V projection + RoPE + KV-cache write for token
 * `token` of the step (position = *position + token). Replaces
 * llama31.py:173-179 (_start_attention), :238-245 (q/k/v F.linear) and the
 * RoPE + SimpleKVCache.append of :200-217. Any of wq/wk/wv may be NULL (the
 * `matrix` granularity streams them as separate units); present ones need
 * their output. x: hidden row [4096] of this token; norm_w: [4096] or NULL
 * (x already normalised); wq [4096,4096], wk/wv [1024,4096]; inv_freq: fp32
 * [64] (llama3-scaled); q_out: [4096] (this token's row); k_cache/v_cache:
 * this layer's [kv_heads, cache_len, 128]. q_heads / kv_heads: 32 / 8, or a
 * tensor-parallel rank's share (32/N, 8/N; the weights are that rank's rows). */
int cb_qkv_rope(const void* x, const void* norm_w, float eps, const void* wq, const void* wk,
                const void* wv, const float* inv_freq, const int32_t* position, int token,
                void* q_out, void* k_cache, void* v_cache, int64_t cache_len, int q_heads, int kv_heads,
                void* stream);

/* out = bf16(residual + bf16(x . W^T)) for one token row. Replaces the o_proj
 * (llama31.py:246-250) and down_proj (:272-280) F.linear + residual add.
 * K in {4096, 14336}; W: [N, K]; x: [K]; residual/out: [N] (may alias). */
int cb_proj_residual(const void* x, int K, const void* w, int N, const void* residual, void* out,
                     void* stream);
/* Tensor-parallel partial of the same projection: out[N] (fp32) = x . W^T
 * over this rank's columns (K = 4096/N or 14336/N), unrounded, to be summed
 * across ranks (all-reduce) and added with cb_residual_add_f32. Supported K:
 * 512, 1024, 1792, 2048, 3584, 4096, 7168, 14336. */
int cb_proj_partial(const void* x, int K, const void* w, int N, float* out, void* stream);
/* out = bf16(x + bf16(sum)): the residual add of llama31.py:249/279 after a
 * projection whose fp32 sum was all-reduced across ranks. x, out: [n] bf16. */
int cb_residual_add_f32(const void* x, const float* sum, int n, void* out, void* stream);

/* Post-attention RMSNorm + gate/up projection + SwiGLU for one token row:
 * out = bf16(bf16(silu(bf16(xn . Wg^T))) * bf16(xn . Wu^T)). Replaces
 * llama31.py:252-275 (the matrix_group `gate_up` unit). W_gate/W_up:
 * [rows, 4096]; out: [rows]. rows = 14336, or a tensor-parallel rank's
 * 14336/N (its rows of both matrices). */
int cb_gate_up_swiglu(const void* x, const void* norm_w, float eps, const void* w_gate,
                      const void* w_up, int rows, void* out, void* stream);
/* The same split in two for the `matrix` granularity (gate_proj and up_proj
 * are separate units, llama31.py:252-271): cb_gate_silu writes
 * bf16(silu(...)), cb_up_mul multiplies it by the up projection in place. */
int cb_gate_silu(const void* x, const void* norm_w, float eps, const void* w_gate, void* out,
                 void* stream);
int cb_up_mul(const void* x, const void* norm_w, float eps, const void* w_up, void* gate_act,
              void* stream);

/* Fused final RMSNorm + LM-head logits + exact top-k over `rows` vocabulary
 * rows (a 16,384-row chunk, a vocab shard, or the whole head). Replaces
 * llama31.py:325-339 and the per-chunk F.linear/.float()/topk of
 * layer_streaming/vocab.py:247-253. Logits are bf16-rounded then fp32, as
 * F.linear(...).float(). Indices are row_offset + row. Order: larger value
 * first, then smaller index. k <= 64 and k <= rows. logits (fp32 [rows]) may
 * be NULL. workspace: cb_lm_head_workspace_bytes(k) bytes of scratch (no
 * initialisation). ticket: one uint32, zeroed once by the caller, used by
 * the last CTA to finish the merge and reset to zero by it. */
int64_t cb_lm_head_workspace_bytes(int k);
int cb_lm_head_topk(const void* x, const void* norm_w, float eps, const void* w, int64_t rows,
                    int64_t row_offset, int k, float* logits, float* out_values,
                    int64_t* out_indices, void* workspace, unsigned int* ticket, void* stream);

/* Exact merge of two candidate sets (values fp32, indices int64) into the
 * top k (k <= 64). Replaces merge_topk (layer_streaming/vocab.py:11-32); also
 * merges the all-gathered per-rank candidates of a vocab-sharded head.
 * `a` may be NULL with na = 0. Output may alias neither input. */
int cb_topk_merge(const float* a_values, const int64_t* a_indices, int na, const float* b_values,
                  const int64_t* b_indices, int nb, int k, float* out_values, int64_t* out_indices,
                  void* stream);

/* GQA attention of M query tokens at positions *position .. *position+M-1
 * over the cache [0, *position + M) (causal within the step). Replaces
 * llama31.py:182-234 (_repeat_kv + scaled_dot_product_attention): scale
 * 1/sqrt(128), fp32 softmax, bf16 output [M, 4096]. Split-KV: `splits`
 * chunks per (token, kv head), combined by the last CTA of each group.
 * q: [M, 4*kv_heads, 128]; k_cache/v_cache: this layer's [kv_heads, cache_len, 128];
 * kv_heads = 8, or a tensor-parallel rank's 8/N.
 * chunk = positions per split (multiple of 64); splits*chunk must cover the
 * longest context of the step (the position lives on the device, so a launch
 * whose splits fall short records code 204 in the error word; the positions
 * beyond splits*chunk are then left out). chunk = 0: the kernel sizes the
 * chunks from the device position (the least multiple of 64, at least 128,
 * with which `splits` chunks cover the step), so one captured launch serves
 * every context length up to splits x chunk. workspace: cb_attention_workspace_bytes(M,
 * splits) bytes of scratch for the per-split partials (no initialisation).
 * tickets: M*kv_heads uint32 counters, zeroed once by the caller; each launch
 * leaves them zero. */
int64_t cb_attention_workspace_bytes(int M, int splits);
/* One-token launches with splits <= 16 merge a KV head's splits inside a
 * thread-block cluster through distributed shared memory (no use of the
 * workspace or the tickets; bit-identical outputs) when the device holds
 * such a cluster; cb_set_attention_cluster(0) selects the global-memory
 * merge for every launch. Returns the previous setting (default 1). */
int cb_set_attention_cluster(int enable);
/* Least positions per split when cb_attention sizes the splits on the device
 * (chunk = 0): a multiple of 64; 0 restores the default (128). Affects
 * launches issued from now on. Returns the previous value, or -1 (nothing
 * changed) for an invalid one. */
int cb_set_attention_min_chunk(int positions);
int cb_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                 const int32_t* position, int M, int kv_heads, int splits, int chunk, void* out,
                 void* workspace, unsigned int* tickets, void* stream);

/* One-token decode attention fused with the o_proj projection and its
 * residual add: out = bf16(residual + bf16(attn . W_o^T)), attn the GQA
 * attention of the token at *position over the cache [0, *position] (8 KV
 * heads, written to attn_out [4096] as well). Replaces llama31.py:182-250
 * (SDPA, o_proj F.linear, residual add) in one launch: the o_proj weights
 * stream into registers and shared memory while the attention runs, and the
 * projection finishes as soon as the 8 heads are merged. Bit-identical to
 * cb_attention (chunk 0) followed by cb_proj_residual. splits: 1 ..
 * cb_attention_oproj_max_splits() (16 fits a B200); chunks are sized on the
 * device. wo: [4096, 4096]; residual/out: [4096] (may alias). workspace:
 * cb_attention_workspace_bytes(1, splits) bytes; tickets: 10 uint32 zeroed
 * once by the caller (left zero by each launch). Error code 205: the
 * projection's wait for the attention gave up (2 s). */
int cb_attention_oproj_max_splits(void);
int cb_attention_oproj(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                       const int32_t* position, int splits, const void* wo, const void* residual, void* attn_out,
                       void* out, void* workspace, unsigned int* tickets, void* stream);

/* Allocation-free variant of cb_attention, for callers that cannot allocate
 * device memory (a host framework that owns the whole memory budget in its
 * own pool, or a latency-critical loop where cudaMalloc would synchronise the
 * device). No counterpart in the reference, which has no custom kernels.
 * The split-KV scratch is a fixed 4 MiB + 8 KiB static device array that
 * every GPU loading this library holds until exit, so the limits are
 * 1 <= M <= 256 and cb_attention_workspace_bytes(M, splits) <= 4 MiB
 * (e.g. one decode token with up to 252 splits); larger requests fail with
 * CB_ERR_INVALID. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture. Each call clears its ticket range with a
 * cudaMemsetAsync and calls no cudaMalloc/cudaFree. All calls share the
 * scratch, so calls that overlap on the GPU (different streams) race.
 * Arguments otherwise as cb_attention, for the full 8-KV-head layout only
 * (kv_heads = 8: the scratch and tickets are sized for it; a
 * tensor-parallel rank's 1, 2 or 4 KV heads need cb_attention). The array's
 * address is looked up once per device and kept for the life of the
 * process: it assumes the device's primary context is never reset
 * (cudaDeviceReset) while the library is loaded. */
int cb_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                         const int32_t* position, int M, int splits, int chunk, void* out,
                         void* stream);

/* ------------------------------------------------------------- prefill */

/* Prefill projections of an M-token chunk on the tcgen05 tensor cores
 * (BF16 in, FP32 accumulate in TMEM, bf16 out): the F.linear calls of
 * llama31.py:238-280 with M > 1. A / xn: [M, K] row-major activations; W:
 * [N, K] row-major weights; K a multiple of 128; all pointers 16-byte
 * aligned. Rounding points are those of the decode kernels.
 *   cb_gemm_bf16:        out[M, N] = bf16(A . W^T); N a multiple of 128
 *   cb_gemm_residual:    out = bf16(residual + bf16(A . W^T)) (out may be residual)
 *   cb_gemm_partial:     out[M, N] = A . W^T in fp32 (a tensor-parallel partial sum)
 *   cb_gemm_silu / cb_gemm_mul: the two halves of cb_gemm_swiglu for the `matrix`
 *                        granularity (gate and up in separate units): out =
 *                        bf16(silu(bf16(A . Wg^T))), then gate_act = bf16(gate_act *
 *                        bf16(A . Wu^T)) in place
 *   cb_gemm_swiglu:      out[M, rows] = bf16(silu(bf16(A . Wg^T)) * bf16(A . Wu^T)),
 *                        K = 4096, rows a multiple of 128 (14336 or a rank's share)
 *   cb_prefill_qkv_rope: q_out[M, 128*q_heads] = RoPE(xn . Wq^T); K/V of the M
 *                        positions *position .. *position+M-1 written into the
 *                        caches [kv_heads, cache_len, 128] (K after RoPE); any of
 *                        wq / wk / wv may be NULL (the `matrix` granularity) */
int cb_gemm_bf16(const void* a, int M, int K, const void* w, int N, void* out, void* stream);
/* Split-K for short chunks (M <= 64 with 128-wide output tiles, M <= 16 with
 * 256-wide ones; fewer output tiles than SMs, e.g. a
 * 6-token prompt: 32 down_proj tiles on 148 SMs): registers the fp32
 * workspace and the zeroed per-tile tickets that the prefill GEMMs above use
 * to split a tile's K range into 9 slices when K >= 8192 (the down
 * projection; the count depends on K only, so projections of equal K give
 * the same bits however they are grouped into launches; shorter K is not
 * split, measured slower); the last CTA of a tile (acquire-release ticket)
 * sums the slices' partials in slice order, runs the fused epilogue and
 * resets the ticket (the tile is summed into shared memory by all epilogue
 * threads at once). A launch splits only when the workspace holds tiles x
 * slices x M x (128 or 256) floats (9 MB covers every Llama-3.1-8B
 * projection at M = 16) and `ntickets` >= its tiles.
 * The registration is process-wide and outlives nothing: unregister (NULL)
 * before the workspace or the tickets are freed, or a later launch writes
 * into freed memory (the executor registers around each short prefill unit
 * and unregisters after it). Launches captured in a CUDA graph keep the
 * registration of their capture; concurrent launches on different streams
 * must not share a workspace.
 * NULL turns splitting off (the default). No counterpart in the reference,
 * which runs these projections through cuBLAS. cb_gemm_split_k returns the
 * slice count a launch of that shape would use (swiglu: N = FFN rows). */
int cb_set_gemm_workspace(void* workspace, int64_t bytes, unsigned int* tickets, int ntickets);
int cb_gemm_split_k(int M, int K, int N, int swiglu);
int cb_gemm_residual(const void* a, int M, int K, const void* w, int N, const void* residual, void* out,
                     void* stream);
int cb_gemm_partial(const void* a, int M, int K, const void* w, int N, float* out, void* stream);
int cb_gemm_silu(const void* a, int M, const void* w_gate, int rows, void* out, void* stream);
int cb_gemm_mul(const void* a, int M, const void* w_up, int rows, void* gate_act, void* stream);
int cb_gemm_swiglu(const void* a, int M, const void* w_gate, const void* w_up, int rows, void* out,
                   void* stream);
int cb_prefill_qkv_rope(const void* xn, int M, const void* wq, const void* wk, const void* wv, int q_heads,
                        int kv_heads, const float* inv_freq, const int32_t* position, void* q_out,
                        void* k_cache, void* v_cache, int64_t cache_len, void* stream);

/* Causal GQA attention of an M-token prefill chunk on the tensor cores: the
 * M tokens at *position .. *position+M-1 attend to the cache [0, *position +
 * t] (token t), scale 1/sqrt(128), fp32 softmax, bf16 out. q / out: [M,
 * 4*kv_heads, 128]; caches [kv_heads, cache_len, 128] (this step's K/V
 * already written). Replaces llama31.py:182-234 for multi-token steps. */
int cb_prefill_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                         const int32_t* position, int M, int kv_heads, void* out, void* stream);
/* Selects the kernel of cb_prefill_attention: 1 (default) tcgen05 MMAs with
 * S and O in TMEM and TMA-loaded Q/K/V tiles (128 query rows = 32 tokens x
 * the 4 query heads of a KV head per CTA, 128-position K/V tiles); 0 the
 * mma.sync kernel (16 tokens per CTA). Returns the previous setting. */
int cb_set_prefill_attention_tc(int enable);

/* ------------------------------------------------ int8 weights (optional) */

/* Low-precision weight transfer: int8 weight-only decode projections. No
 * counterpart in the reference, whose README lists INT8/INT4 weight transfer
 * as not supported (README.md:156); this reduced-precision mode is outside
 * the bf16 parity contract and is never the benchmark's headline value.
 * Row r of an [N, K] matrix is K int8 values q and an fp32 scale s_r, with
 * w ~= q * s_r:
 *   cb_quantize_rows_i8: s_r = max|w_r| / 127 (fp32 division), q =
 *       round-half-even(w / s_r) clamped to [-127, 127] (fp32 division); an
 *       all-zero row gets s_r = 0, q = 0. w: bf16 [rows, K], K a multiple of
 *       256; q: int8 [rows, K] (16-byte aligned); scale: fp32 [rows].
 * The projections below are the bf16 entry points of the same names with
 * each weight matrix replaced by (int8 matrix, its row scales): the row's
 * integer dot product with the bf16 activations is accumulated in fp32 and
 * multiplied by s_r, then the same fused prologue / epilogue runs. They
 * stream half the weight bytes. K: 4096 (14336 for down_proj). */
int cb_quantize_rows_i8(const void* w, int64_t rows, int K, void* q, float* scale, void* stream);
/* out = bf16(q * scale) row by row: the bf16 weights that the prefill GEMMs
 * use when a unit arrives in int8 (the streamed int8 transfer). q: int8
 * [rows, K] (16-byte aligned); out: bf16 [rows, K]; K a multiple of 8. */
int cb_dequantize_rows_i8(const void* q, const float* scale, int64_t rows, int K, void* out, void* stream);
int cb_qkv_rope_i8(const void* x, const void* norm_w, float eps, const void* wq, const float* sq,
                   const void* wk, const float* sk, const void* wv, const float* sv, const float* inv_freq,
                   const int32_t* position, int token, void* q_out, void* k_cache, void* v_cache,
                   int64_t cache_len, int q_heads, int kv_heads, void* stream);
int cb_proj_residual_i8(const void* x, int K, const void* w, const float* scale, int N, const void* residual,
                        void* out, void* stream);
int cb_gate_up_swiglu_i8(const void* x, const void* norm_w, float eps, const void* w_gate, const float* s_gate,
                         const void* w_up, const float* s_up, int rows, void* out, void* stream);
int cb_lm_head_topk_i8(const void* x, const void* norm_w, float eps, const void* w, const float* scale,
                       int64_t rows, int64_t row_offset, int k, float* logits, float* out_values,
                       int64_t* out_indices, void* workspace, unsigned int* ticket, void* stream);

/* ------------------------------------------------------ tensor parallelism */

/* Decode across N GPUs of one node (one process per GPU), an addition to the
 * reference (whose executor is single-GPU, llama31.py:82-352): each rank
 * holds query heads [32r/N, 32(r+1)/N), KV heads [8r/N, 8(r+1)/N), FFN rows
 * [14336r/N, ...), the matching columns of o_proj / down_proj, and vocabulary
 * rows [128256r/N, ...) of the LM head; the residual stream is replicated.
 *
 * Exchange buffer: cb_exchange_bytes() of device memory per rank, allocated
 * zeroed by cb_exchange_alloc and mapped into the other ranks' processes with
 * cb_ipc_handle (CB_IPC_HANDLE_BYTES opaque bytes, sent by any host channel)
 * and cb_ipc_open. `exchange` arguments are HOST arrays of `world` device
 * pointers: entry q is rank q's buffer as mapped in this process (entry
 * `rank` is this rank's own).
 *
 * Sequence numbers: each launch of a step has a `slot` (0 <= slot < slots,
 * slots even, the same on every rank); `epoch` is a device int32 step counter
 * that every rank advances by one after each step (cb_position_advance).
 * Ranks must issue the same launches in the same order. A peer that does not
 * arrive within the exchange wait limit (default 2 s) sets the error word
 * (120: projection, 121: LM head) and the launch completes with undefined
 * values instead of hanging. */
#define CB_IPC_HANDLE_BYTES 64
int64_t cb_exchange_bytes(void);
int cb_exchange_alloc(void** buffer_out);
int cb_exchange_free(void* buffer);
int cb_ipc_handle(const void* buffer, void* handle_out);
int cb_ipc_open(const void* handle, void** buffer_out);
int cb_ipc_close(void* buffer);
/* Sets the wall-clock limit of the exchange waits for launches issued from
 * now on (a captured CUDA graph keeps the limit it was captured with); 0
 * restores the 2 s default. Returns the previous limit. A short limit lets a
 * test make a wait run out on one GPU. */
uint64_t cb_set_exchange_wait_ns(uint64_t ns);

/* Row-parallel projection fused with its all-reduce and the residual add:
 * out = bf16(residual + bf16(sum over ranks q of x_q . W_q^T)), where x_q / W_q
 * are rank q's K columns (K = 4096/N for o_proj, 14336/N for down_proj) and
 * the fp32 partials are summed in rank order, so every rank gets the same
 * bits. Replaces F.linear + residual of llama31.py:246-250 / :276-280 under
 * tensor parallelism. N <= 4096; residual may equal out. */
int cb_proj_allreduce_residual(const void* x, int K, const void* w, int N, const void* residual, void* out,
                               void* const* exchange, int rank, int world, int slot, int slots,
                               const int32_t* epoch, void* stream);
/* Vocabulary-sharded cb_lm_head_topk: this rank's `rows` rows starting at
 * global row `row_offset`, its exact top-k, then the k candidates of every
 * rank gathered through the exchange buffers and merged: every rank gets the
 * global top-k (same tie rule). No full logits. */
int cb_lm_head_topk_allgather(const void* x, const void* norm_w, float eps, const void* w, int64_t rows,
                              int64_t row_offset, int k, float* out_values, int64_t* out_indices,
                              void* workspace, unsigned int* ticket, void* const* exchange, int rank,
                              int world, int slot, int slots, const int32_t* epoch, void* stream);

/* -------------------------------------------------------------- host I/O */

/* Host-only helpers of the weight stores (no CUDA calls; any host thread).
 * cb_host_copy: memcpy of `bytes` split over `threads` native threads (0 =
 * up to 16 hardware threads); replaces the single-threaded pageable ->
 * pinned staging copy (weight_store.py:252-261). cb_read_file_ranges: n
 * byte ranges of the file at `path` (offsets[i], sizes[i]) read with
 * parallel pread straight into host memory dsts[i] (the safetensors tensor
 * data -> packed arena path of weight_store.py:109-171). */
int cb_host_copy(void* dst, const void* src, int64_t bytes, int threads);
int cb_read_file_ranges(const char* path, int n, const int64_t* offsets, void* const* dsts, const int64_t* sizes,
                        int threads);
/* Embedding rows ids[0..n) of a row-major host table ([rows, row_bytes])
 * gathered into consecutive rows of host memory dst (the pinned staging rows
 * of the streamed-vocabulary embedding, vocab.py:100-131); ids outside
 * [0, rows) fail before any copy. */
int cb_host_gather_rows(void* dst, const void* table, int64_t rows, int64_t row_bytes, const int64_t* ids,
                        int64_t n);

/* ------------------------------------------------------ streamed weights */

/* Slot ring: the H2D pipeline of the streamed mode (DoubleBufferRuntime.run,
 * layer_streaming/runtime.py:137-268, and the LM-head chunks of
 * VocabStreamingRuntime.lm_head_topk, vocab.py:207-266). `slots` device
 * buffers of slot_bytes are filled from host spans on `copy_stream` while a
 * compute stream consumes them: span i lands in slot i % slots, and span
 * i + slots is copied once the compute stream has released span i.
 * staging (NULL, or `slots` pinned host buffers of staging_bytes): the
 * spans are pageable; a native stager thread copies each span into a
 * staging buffer (copy_threads threads; 0 = up to 16) once the DMA that last
 * read that buffer has finished, then starts its H2D copy.
 * Per pass: cb_ring_begin (orders both streams after the coordinator's
 * queued work and starts the first `slots` copies), then for each span i in
 * order cb_ring_acquire (compute stream waits for the copy; returns the
 * slot's device pointer) and cb_ring_release (after the span's compute work
 * was enqueued), then cb_ring_end (the coordinator waits for the last
 * release and the host for the coordinator). stats (8 doubles, may be NULL):
 * pass ms, sum of copy ms, sum of compute ms (the three with profile = 1),
 * host ms spent waiting for copies to be issued, staging copies, their ms
 * sum and max, bytes moved. cb_ring_abort ends a pass cut short. One pass at
 * a time per ring; calls from one host thread. */
int cb_ring_create(int slots, void* const* device_slots, int64_t slot_bytes, void* copy_stream,
                   void* const* staging, int64_t staging_bytes, int copy_threads, void** ring_out);
int cb_ring_destroy(void* ring);
int cb_ring_begin(void* ring, int spans, const void* const* sources, const int64_t* bytes, void* compute_stream,
                  void* coordinator_stream, int profile);
int cb_ring_acquire(void* ring, int span, void** device_ptr);
int cb_ring_release(void* ring, int span);
int cb_ring_end(void* ring, int last_span, double* stats);
int cb_ring_abort(void* ring);

/* ---------------------------------------------------------------- copies */

/* Host -> device copy of `bytes` on `stream` (cudaMemcpyAsync). The H2D leg
 * of DoubleBufferRuntime.run (layer_streaming/runtime.py:194-204) and of the
 * vocab chunks (layer_streaming/vocab.py:228-236). `src` must be pinned for
 * the copy to be asynchronous. */
int cb_memcpy_h2d_async(void* dst, const void* src, int64_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CASCADE_B200_H */
