// Weight-streaming decode GEMVs for sm_100a (BF16 in, fp32 accumulate).
//
// One kernel family computes every M=1 projection of the Llama-3.1-8B decode
// step (reference: layer_streaming/llama31.py:236-283 and the LM head at
// :330-339 / layer_streaming/vocab.py:247-253), each with its fused
// prologue/epilogue:
//
//   QKV      RMSNorm prologue, RoPE epilogue, K/V written into the cache
//   O, down  residual-add epilogue
//   gate+up  RMSNorm prologue, SwiGLU epilogue
//   LM head  final RMSNorm prologue, fp32 logits + per-CTA top-k, and a
//            last-CTA merge into the launch's exact top-k
//
// Design (HBM-bound: 0.5 FMA per weight byte):
//   * two CTAs of 8 warps per SM (grid = 2 x SM count), <= 128 registers;
//   * work is a list of "units"; a unit is a PAIR of weight rows (A, B) whose
//     outputs an epilogue needs together: rows d and d+64 of one head for
//     RoPE, gate row j and up row j for SwiGLU, rows j and j+N/2 otherwise.
//     Each CTA owns a contiguous range of units (row granularity);
//   * CTA-cooperative split-K: every warp streams its 1/8 of K for every unit
//     of the range straight into registers (128-bit ld.global.nc, a batch of
//     up to 16 loads in flight per lane), reduces with shuffles into shared
//     memory, and after ONE barrier the epilogues of all units run in
//     parallel, one thread per unit;
//   * the first batch of weight loads is issued BEFORE griddepcontrol.wait
//     (weights do not depend on the previous kernel), so with programmatic
//     dependent launch the next projection's weights are in flight while the
//     previous kernel drains; everything read from the previous kernel (the
//     activation slice, RMSNorm weights, the epilogue's residual / gate
//     values, RoPE frequency and position) is requested in one round trip
//     right after the wait.
#include <cuda_bf16.h>

#include <algorithm>
#include <initializer_list>
#include <utility>

#include "common.cuh"
#include "gemv_device.cuh"
#include "internal.h"
#include "cascade_b200.h"

// Two CTAs of 8 warps per SM, one batch of UB units in flight per warp.
#define CB_GEMV_CTAS_PER_SM 2
#define CB_GEMV_DEPTH 1

namespace cb {

// Every GEMV launch is two CTAs per SM (one full wave at <= 128 registers
// per thread); the LM-head candidate workspace is sized by the same grid.
static int gemv_grid() { return CB_GEMV_CTAS_PER_SM * sm_count(); }
static int lm_head_grid() { return gemv_grid(); }

// Stand-alone projection: prefetch the first weight batch, wait for the
// previous kernel (programmatic dependent launch), then run.
template <int K, bool W8 = false>
__global__ void __launch_bounds__(kThreads, CB_GEMV_CTAS_PER_SM) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t times[5];  // launch trace: start, after the wait, after the main loop, two extra points
  if (p.trace && threadIdx.x == 0) {
    times[0] = globaltimer_ns();
    times[3] = times[4] = 0;
  }
  GemvRegs<K, CB_GEMV_DEPTH, W8> r;
  gemv_prefetch<K, CB_GEMV_DEPTH, W8>(p, blockIdx.x, gridDim.x, r);
  if (p.stage.where == 1 && threadIdx.x < 32) l2_stage_issue(p.stage, blockIdx.x, gridDim.x, threadIdx.x, 32);
  grid_dep_wait();  // the activation row comes from the previous kernel
  if (threadIdx.x == 0) {
    if (p.trace) times[1] = globaltimer_ns();
    grid_dep_launch();
  }
  if (p.stage.where == 2 && threadIdx.x < 32) l2_stage_issue(p.stage, blockIdx.x, gridDim.x, threadIdx.x, 32);
  gemv_run<K, CB_GEMV_DEPTH, W8>(p, smem, blockIdx.x, gridDim.x, r, p.trace ? &times[2] : nullptr);
  if (p.stage.where == 3 && threadIdx.x < 32) l2_stage_issue(p.stage, blockIdx.x, gridDim.x, threadIdx.x, 32);
  if (p.trace && threadIdx.x == 0)
    trace_commit(p.trace, p.trace_tag, blockIdx.x, times[0], times[1], times[2], times[3], times[4]);
}

}  // namespace cb

// ====================================================================== host
namespace cb {

int32_t* error_word();

int finish_params(GemvParams& p) {
  p.total_units = 0;
  for (int i = 0; i < p.nseg; ++i) p.total_units += p.seg[i].units;
  p.err = error_word();
  p.trace = trace_buffer(&p.trace_tag);
  return kOk;
}

template <int K, bool W8 = false>
static int run_gemv(const char* what, GemvParams& p, cudaStream_t stream) {
  using S = GemvShape<K, CB_GEMV_DEPTH, W8>;
  int rc = configure_smem(what, gemv_kernel<K, W8>, kMaxSmem);
  if (rc != kOk) return rc;
  finish_params(p);
  if (p.total_units == 0) return kOk;
  const int grid = gemv_grid();
  const size_t per_cta = size_t((p.total_units + grid - 1) / grid);
  size_t smem = S::SMEM + per_cta * 2 * S::WK * sizeof(float);  // per-unit partials
  if (p.cand_values) {
    // EPI_TOPK: the CTA's logits, later reused as the last CTA's merge scratch
    // logits -> keys of this CTA's rows and the selection stage; the last CTA
    // reuses the region for the merge of all CTAs' candidates
    smem += std::max(per_cta * 2 * sizeof(float) + size_t(kThreads / 32) * kTopkMax * 8, kTopkScratchBytes);
  }
  if (smem > kMaxSmem) return fail(kErrInvalid, "%s: %zu units per CTA exceed shared memory", what, per_cta);
  return launch(what, gemv_kernel<K, W8>, dim3(grid), dim3(kThreads), smem, stream, p);
}

int gemv_grid_size() { return gemv_grid(); }

// Row lengths with a kernel instance: the model's 4096 and 14336, and their
// tensor-parallel shards (O: 4096/N, down: 14336/N for N = 2, 4, 8).
#define CB_GEMV_KS(X) X(512) X(1024) X(1792) X(2048) X(3584) X(4096) X(7168) X(14336)

static int run_gemv_any(const char* what, int K, GemvParams& p, cudaStream_t stream) {
  switch (K) {
#define CB_CASE(k) \
  case k:          \
    return run_gemv<k>(what, p, stream);
    CB_GEMV_KS(CB_CASE)
#undef CB_CASE
    default:
      return fail(kErrUnsupported, "%s: K=%d has no kernel (512, 1024, 1792, 2048, 3584, 4096, 7168, 14336)",
                  what, K);
  }
}

static bool gemv_k_supported(int K) {
  switch (K) {
#define CB_CASE(k) case k:
    CB_GEMV_KS(CB_CASE)
#undef CB_CASE
    return true;
    default:
      return false;
  }
}

int prepare_gemv() {
  int rc = kOk;
#define CB_CASE(k) \
  if (rc == kOk) rc = configure_smem("gemv", gemv_kernel<k>, kMaxSmem);
  CB_GEMV_KS(CB_CASE)
#undef CB_CASE
  if (rc == kOk) rc = configure_smem("gemv", gemv_kernel<4096, true>, kMaxSmem);
  if (rc == kOk) rc = configure_smem("gemv", gemv_kernel<14336, true>, kMaxSmem);
  return rc;
}

// wbytes: bytes per weight (2 bf16, 1 int8); scale: the int8 rows' scales
static Segment half_segment(const void* w, int N, int K, int mode, void* out, const void* aux, int wbytes = 2,
                            const float* scale = nullptr) {
  Segment s = {};
  s.a_base = static_cast<const uint16_t*>(w);
  s.b_base = reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(w) + int64_t(N / 2) * K * wbytes);
  s.a_scale = scale;
  s.b_scale = scale ? scale + N / 2 : nullptr;
  s.units = N / 2;
  s.group = N / 2;
  s.group_stride = 0;
  s.mode = mode;
  s.out = static_cast<uint16_t*>(out);
  s.aux = static_cast<const uint16_t*>(aux);
  s.head_stride = 0;
  s.b_offset = N / 2;
  s.pos_stride = 0;
  return s;
}

// rows (h*128 + d, h*128 + 64 + d) of `heads` heads of 128
static Segment head_segment(const void* w, int heads, int mode, void* out, int64_t head_stride,
                            int64_t pos_stride, int64_t pos_limit = 0, int wbytes = 2,
                            const float* scale = nullptr) {
  Segment s = {};
  s.a_base = static_cast<const uint16_t*>(w);
  s.b_base = reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(w) + int64_t(64) * 4096 * wbytes);
  s.a_scale = scale;
  s.b_scale = scale ? scale + 64 : nullptr;
  s.units = heads * 64;
  s.group = 64;
  s.group_stride = 128;
  s.mode = mode;
  s.out = static_cast<uint16_t*>(out);
  s.aux = nullptr;
  s.head_stride = head_stride;
  s.b_offset = 64;
  s.pos_stride = pos_stride;
  s.pos_limit = pos_limit;
  return s;
}

}  // namespace cb

using namespace cb;

namespace cb {

int build_qkv_params(GemvParams& p, const void* x, const void* norm_w, float eps, const void* wq,
                     const void* wk, const void* wv, const float* inv_freq, const int32_t* position,
                     int token, void* q_out, void* k_cache, void* v_cache, int64_t cache_len, int q_heads,
                     int kv_heads, int wbytes, const float* sq, const float* sk, const float* sv) {
  CB_REQUIRE(q_heads >= 1 && q_heads <= 32 && kv_heads >= 1 && kv_heads <= 8,
             "cb_qkv_rope: %d query / %d key-value heads (1..32 / 1..8)", q_heads, kv_heads);
  CB_REQUIRE(x && aligned16(x), "cb_qkv_rope: x must be a 16-byte aligned device pointer");
  CB_REQUIRE(!norm_w || aligned16(norm_w), "cb_qkv_rope: norm_w must be 16-byte aligned");
  CB_REQUIRE(inv_freq && position, "cb_qkv_rope: inv_freq and position are required");
  CB_REQUIRE(token >= 0, "cb_qkv_rope: token must be >= 0");
  p = GemvParams{};
  p.x = static_cast<const uint16_t*>(x);
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  p.inv_freq = inv_freq;
  p.pos = position;
  p.token = token;
  if (wq) {
    CB_REQUIRE(aligned16(wq) && q_out, "cb_qkv_rope: wq needs alignment and q_out");
    p.seg[p.nseg++] = head_segment(wq, q_heads, EPI_ROPE, q_out, 128, 0, 0, wbytes, sq);
  }
  if (wk || wv) CB_REQUIRE(cache_len > 0, "cb_qkv_rope: cache_len must be positive");
  if (wk) {
    CB_REQUIRE(aligned16(wk) && k_cache, "cb_qkv_rope: wk needs alignment and k_cache");
    p.seg[p.nseg++] = head_segment(wk, kv_heads, EPI_ROPE, k_cache, cache_len * 128, 128, cache_len, wbytes, sk);
  }
  if (wv) {
    CB_REQUIRE(aligned16(wv) && v_cache, "cb_qkv_rope: wv needs alignment and v_cache");
    p.seg[p.nseg++] = head_segment(wv, kv_heads, EPI_STORE, v_cache, cache_len * 128, 128, cache_len, wbytes, sv);
  }
  return finish_params(p);
}

int build_residual_params(GemvParams& p, const void* x, int K, const void* w, int N, const void* residual,
                          void* out, int wbytes, const float* scale) {
  CB_REQUIRE(x && w && residual && out, "cb_proj_residual: null pointer");
  CB_REQUIRE(aligned16(x) && aligned16(w), "cb_proj_residual: x and w must be 16-byte aligned");
  CB_REQUIRE(N > 0 && N % 2 == 0, "cb_proj_residual: N must be even and positive");
  CB_REQUIRE(gemv_k_supported(K), "cb_proj_residual: K=%d has no kernel", K);
  p = GemvParams{};
  p.x = static_cast<const uint16_t*>(x);
  p.seg[p.nseg++] = half_segment(w, N, K, EPI_RESIDUAL, out, residual, wbytes, scale);
  return finish_params(p);
}

int build_partial_params(GemvParams& p, const void* x, int K, const void* w, int N, float* out) {
  CB_REQUIRE(x && w && out, "cb_proj_partial: null pointer");
  CB_REQUIRE(aligned16(x) && aligned16(w), "cb_proj_partial: x and w must be 16-byte aligned");
  CB_REQUIRE(N > 0 && N % 2 == 0, "cb_proj_partial: N must be even and positive");
  CB_REQUIRE(gemv_k_supported(K), "cb_proj_partial: K=%d has no kernel", K);
  p = GemvParams{};
  p.x = static_cast<const uint16_t*>(x);
  Segment s = half_segment(w, N, K, EPI_PARTIAL, nullptr, nullptr);
  s.outf = out;
  p.seg[p.nseg++] = s;
  return finish_params(p);
}

int build_gate_up_params(GemvParams& p, const char* what, const void* x, const void* norm_w, float eps,
                         const void* w_gate, const void* w_up, int N, int mode, void* out, const void* aux,
                         int wbytes, const float* s_gate, const float* s_up) {
  CB_REQUIRE(x && out && aligned16(x), "%s: x/out invalid", what);
  CB_REQUIRE(N > 0 && N % 2 == 0, "%s: rows=%d must be even and positive", what, N);
  CB_REQUIRE(!norm_w || aligned16(norm_w), "%s: norm_w must be 16-byte aligned", what);
  p = GemvParams{};
  p.x = static_cast<const uint16_t*>(x);
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  if (mode == EPI_SWIGLU) {
    CB_REQUIRE(w_gate && w_up && aligned16(w_gate) && aligned16(w_up), "%s: weights invalid", what);
    Segment s = half_segment(w_gate, 2 * N, 4096, EPI_SWIGLU, out, nullptr, wbytes, s_gate);
    s.b_base = static_cast<const uint16_t*>(w_up);
    s.b_scale = s_up;
    s.b_offset = 0;
    p.seg[p.nseg++] = s;
  } else {
    const void* w = mode == EPI_SILU ? w_gate : w_up;
    CB_REQUIRE(w && aligned16(w), "%s: weight invalid", what);
    p.seg[p.nseg++] = half_segment(w, N, 4096, mode, out, aux, wbytes, mode == EPI_SILU ? s_gate : s_up);
  }
  return finish_params(p);
}

}  // namespace cb

extern "C" int cb_qkv_rope(const void* x, const void* norm_w, float eps, const void* wq,
                           const void* wk, const void* wv, const float* inv_freq,
                           const int32_t* position, int token, void* q_out, void* k_cache,
                           void* v_cache, int64_t cache_len, int q_heads, int kv_heads, void* stream) {
  GemvParams p;
  int rc = build_qkv_params(p, x, norm_w, eps, wq, wk, wv, inv_freq, position, token, q_out, k_cache, v_cache,
                            cache_len, q_heads, kv_heads, 2, nullptr, nullptr, nullptr);
  if (rc != kOk) return rc;
  p.stage = l2_stage_for(0);
  return run_gemv<4096>("cb_qkv_rope", p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_proj_residual(const void* x, int K, const void* w, int N, const void* residual,
                                void* out, void* stream) {
  GemvParams p;
  int rc = build_residual_params(p, x, K, w, N, residual, out, 2, nullptr);
  if (rc != kOk) return rc;
  if (K == 4096 && N == 4096) p.stage = l2_stage_for(2);  // o_proj
  return run_gemv_any("cb_proj_residual", K, p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_proj_partial(const void* x, int K, const void* w, int N, float* out, void* stream) {
  GemvParams p;
  int rc = build_partial_params(p, x, K, w, N, out);
  if (rc != kOk) return rc;
  return run_gemv_any("cb_proj_partial", K, p, static_cast<cudaStream_t>(stream));
}

static int gate_up_common(const char* what, const void* x, const void* norm_w, float eps,
                          const void* w_gate, const void* w_up, int rows, int mode, void* out,
                          const void* aux, void* stream) {
  GemvParams p;
  int rc = build_gate_up_params(p, what, x, norm_w, eps, w_gate, w_up, rows, mode, out, aux, 2, nullptr, nullptr);
  if (rc != kOk) return rc;
  return run_gemv<4096>(what, p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_gate_up_swiglu(const void* x, const void* norm_w, float eps, const void* w_gate,
                                 const void* w_up, int rows, void* out, void* stream) {
  return gate_up_common("cb_gate_up_swiglu", x, norm_w, eps, w_gate, w_up, rows, EPI_SWIGLU, out,
                        nullptr, stream);
}

extern "C" int cb_gate_silu(const void* x, const void* norm_w, float eps, const void* w_gate,
                            void* out, void* stream) {
  return gate_up_common("cb_gate_silu", x, norm_w, eps, w_gate, nullptr, 14336, EPI_SILU, out, nullptr,
                        stream);
}

extern "C" int cb_up_mul(const void* x, const void* norm_w, float eps, const void* w_up,
                         void* gate_act, void* stream) {
  return gate_up_common("cb_up_mul", x, norm_w, eps, nullptr, w_up, 14336, EPI_MUL, gate_act, gate_act,
                        stream);
}

// Tensor-parallel exchange arguments shared by the two exchange entry points.
static int set_exchange(GemvParams& p, const char* what, void* const* exchange, int rank, int world, int slot,
                        int slots, const int32_t* epoch) {
  CB_REQUIRE(exchange && epoch, "%s: exchange and epoch are required", what);
  CB_REQUIRE(world >= 1 && world <= kXchgMaxWorld && rank >= 0 && rank < world,
             "%s: rank %d of world %d (world 1..%d)", what, rank, world, kXchgMaxWorld);
  CB_REQUIRE(slots >= 2 && slots % 2 == 0 && slot >= 0 && slot < slots,
             "%s: slot %d of %d (slots even, >= 2)", what, slot, slots);
  for (int q = 0; q < world; ++q) {
    CB_REQUIRE(exchange[q] && aligned16(exchange[q]), "%s: exchange buffer of rank %d invalid", what, q);
    p.xchg[q] = static_cast<uint8_t*>(exchange[q]);
  }
  p.rank = rank;
  p.world = world;
  p.slot = slot;
  p.slots = slots;
  p.epoch = epoch;
  p.wait_ns = exchange_wait_ns();
  return kOk;
}

extern "C" int64_t cb_exchange_bytes(void) { return int64_t(kXchgBytes); }

extern "C" int cb_proj_allreduce_residual(const void* x, int K, const void* w, int N, const void* residual,
                                          void* out, void* const* exchange, int rank, int world, int slot,
                                          int slots, const int32_t* epoch, void* stream) {
  GemvParams p;
  int rc = build_residual_params(p, x, K, w, N, residual, out, 2, nullptr);
  if (rc != kOk) return rc;
  CB_REQUIRE(N <= kXchgWidth, "cb_proj_allreduce_residual: N=%d exceeds the exchange width %d", N, kXchgWidth);
  p.seg[0].mode = EPI_EXCHANGE;
  rc = set_exchange(p, "cb_proj_allreduce_residual", exchange, rank, world, slot, slots, epoch);
  if (rc != kOk) return rc;
  return run_gemv_any("cb_proj_allreduce_residual", K, p, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t cb_lm_head_workspace_bytes(int k) {
  // candidates: values [CTAs*k] fp32, then indices [CTAs*k] int64
  const int64_t n = int64_t(lm_head_grid()) * k;
  return ((n * 4 + 15) / 16) * 16 + n * 8;
}

static int build_lm_head_params(GemvParams& p, const void* x, const void* norm_w, float eps, const void* w,
                                int64_t rows, int64_t row_offset, int k, float* logits, float* out_values,
                                int64_t* out_indices, void* workspace, unsigned int* ticket, int wbytes = 2,
                                const float* scale = nullptr) {
  CB_REQUIRE(x && w && out_values && out_indices && workspace && ticket, "cb_lm_head_topk: null pointer");
  CB_REQUIRE(aligned16(x) && aligned16(w), "cb_lm_head_topk: x and w must be 16-byte aligned");
  CB_REQUIRE(!norm_w || aligned16(norm_w), "cb_lm_head_topk: norm_w must be 16-byte aligned");
  CB_REQUIRE(rows > 0 && rows % 2 == 0 && rows <= (int64_t(1) << 30),
             "cb_lm_head_topk: rows must be even, positive and < 2^30 (got %lld)", (long long)rows);
  CB_REQUIRE(k >= 1 && k <= kTopkMax && k <= rows, "cb_lm_head_topk: need 1 <= k <= min(64, rows)");
  CB_REQUIRE(row_offset >= 0 && row_offset + rows <= (int64_t(1) << 31),
             "cb_lm_head_topk: row ids must fit 31 bits (row_offset + rows <= 2^31)");
  p = GemvParams{};
  p.x = static_cast<const uint16_t*>(x);
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  Segment s = half_segment(w, int(rows), 4096, EPI_TOPK, nullptr, nullptr, wbytes, scale);
  p.seg[p.nseg++] = s;
  p.k = k;
  p.row_offset = row_offset;
  p.logits = logits;
  const int64_t n = int64_t(lm_head_grid()) * k;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.cand_values = reinterpret_cast<float*>(ws);
  p.cand_indices = reinterpret_cast<int64_t*>(ws + ((n * 4 + 15) / 16) * 16);
  p.ticket = ticket;
  p.out_values = out_values;
  p.out_indices = out_indices;
  return kOk;
}

extern "C" int cb_lm_head_topk(const void* x, const void* norm_w, float eps, const void* w,
                               int64_t rows, int64_t row_offset, int k, float* logits,
                               float* out_values, int64_t* out_indices, void* workspace,
                               unsigned int* ticket, void* stream) {
  GemvParams p;
  int rc = build_lm_head_params(p, x, norm_w, eps, w, rows, row_offset, k, logits, out_values, out_indices,
                                workspace, ticket);
  if (rc != kOk) return rc;
  return run_gemv<4096>("cb_lm_head_topk", p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_lm_head_topk_allgather(const void* x, const void* norm_w, float eps, const void* w,
                                         int64_t rows, int64_t row_offset, int k, float* out_values,
                                         int64_t* out_indices, void* workspace, unsigned int* ticket,
                                         void* const* exchange, int rank, int world, int slot, int slots,
                                         const int32_t* epoch, void* stream) {
  GemvParams p;
  int rc = build_lm_head_params(p, x, norm_w, eps, w, rows, row_offset, k, nullptr, out_values, out_indices,
                                workspace, ticket);
  if (rc != kOk) return rc;
  CB_REQUIRE(row_offset >= 0 && row_offset + rows <= (int64_t(1) << 31),
             "cb_lm_head_topk_allgather: global row ids must fit 31 bits");
  rc = set_exchange(p, "cb_lm_head_topk_allgather", exchange, rank, world, slot, slots, epoch);
  if (rc != kOk) return rc;
  return run_gemv<4096>("cb_lm_head_topk_allgather", p, static_cast<cudaStream_t>(stream));
}

// ============================================================================
// Int8 weight-only decode projections (low-precision weight transfer).
//
// Row r of a weight matrix is stored as K int8 values q and one fp32 scale
// s_r = max|w_r| / 127, w ~= q * s_r (symmetric, per output row). The GEMV
// streams half the bytes of the bf16 kernel and computes the row's dot
// product of the integers with the bf16 activations in fp32, times s_r, then
// applies the same fused prologue / epilogue as the bf16 kernel. No
// counterpart in the reference, whose README lists INT8/INT4 weight transfer
// as unsupported (README.md:156); these are this engine's optional
// reduced-precision mode, outside the bf16 parity contract.
// ============================================================================
namespace cb {

// One warp per row: the row's absolute maximum (bf16 values, exact in fp32),
// scale = max / 127 (fp32 division, round to nearest), q = round-half-even
// of w / scale (fp32 division) clamped to [-127, 127]; a zero row gets scale
// 0 and q = 0.
__global__ void __launch_bounds__(256) quantize_rows_i8_kernel(const uint16_t* __restrict__ w, int64_t rows, int K,
                                                               int8_t* __restrict__ q, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint16_t* src = w + row * K;
  float mx = 0.f;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + c);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fmaxf(fabsf(bf16lo(u[e])), fabsf(bf16hi(u[e]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  const float s = __fdiv_rn(mx, 127.0f);
  if (lane == 0) scale[row] = s;
  int8_t* dst = q + row * K;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + c);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = (e & 1) ? bf16hi(u[e >> 1]) : bf16lo(u[e >> 1]);
      int iq = 0;
      if (s > 0.f) iq = min(127, max(-127, __float2int_rn(__fdiv_rn(x, s))));
      packed[e >> 2] |= (uint32_t(iq) & 0xFFu) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(dst + c) = make_uint2(packed[0], packed[1]);
  }
}

}  // namespace cb

extern "C" int cb_quantize_rows_i8(const void* w, int64_t rows, int K, void* q, float* scale, void* stream) {
  if (!w || !q || !scale || !aligned16(w) || !aligned16(q))
    return fail(kErrInvalid, "cb_quantize_rows_i8: w and q must be 16-byte aligned device pointers");
  if (rows < 1 || K < 256 || K % 256) return fail(kErrInvalid, "cb_quantize_rows_i8: rows >= 1, K a multiple of 256");
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7FFFFFFF) return fail(kErrInvalid, "cb_quantize_rows_i8: too many rows");
  quantize_rows_i8_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), rows, K, static_cast<int8_t*>(q), scale);
  return check_launch("cb_quantize_rows_i8");
}

static bool scales_ok(std::initializer_list<std::pair<const void*, const float*>> pairs) {
  for (const auto& ws : pairs)
    if (ws.first && !ws.second) return false;
  return true;
}

extern "C" int cb_qkv_rope_i8(const void* x, const void* norm_w, float eps, const void* wq, const float* sq,
                              const void* wk, const float* sk, const void* wv, const float* sv,
                              const float* inv_freq, const int32_t* position, int token, void* q_out,
                              void* k_cache, void* v_cache, int64_t cache_len, int q_heads, int kv_heads,
                              void* stream) {
  if (!scales_ok({{wq, sq}, {wk, sk}, {wv, sv}})) return fail(kErrInvalid, "cb_qkv_rope_i8: a weight lacks its scales");
  GemvParams p;
  int rc = build_qkv_params(p, x, norm_w, eps, wq, wk, wv, inv_freq, position, token, q_out, k_cache, v_cache,
                            cache_len, q_heads, kv_heads, 1, sq, sk, sv);
  if (rc != kOk) return rc;
  p.stage = l2_stage_for(0);
  return run_gemv<4096, true>("cb_qkv_rope_i8", p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_proj_residual_i8(const void* x, int K, const void* w, const float* scale, int N,
                                   const void* residual, void* out, void* stream) {
  if (!scale) return fail(kErrInvalid, "cb_proj_residual_i8: scale is required");
  if (K != 4096 && K != 14336) return fail(kErrUnsupported, "cb_proj_residual_i8: K=%d (4096 or 14336)", K);
  GemvParams p;
  int rc = build_residual_params(p, x, K, w, N, residual, out, 1, scale);
  if (rc != kOk) return rc;
  if (K == 4096 && N == 4096) p.stage = l2_stage_for(2);
  return K == 4096 ? run_gemv<4096, true>("cb_proj_residual_i8", p, static_cast<cudaStream_t>(stream))
                   : run_gemv<14336, true>("cb_proj_residual_i8", p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_gate_up_swiglu_i8(const void* x, const void* norm_w, float eps, const void* w_gate,
                                    const float* s_gate, const void* w_up, const float* s_up, int rows, void* out,
                                    void* stream) {
  if (!s_gate || !s_up) return fail(kErrInvalid, "cb_gate_up_swiglu_i8: scales are required");
  GemvParams p;
  int rc = build_gate_up_params(p, "cb_gate_up_swiglu_i8", x, norm_w, eps, w_gate, w_up, rows, EPI_SWIGLU, out,
                                nullptr, 1, s_gate, s_up);
  if (rc != kOk) return rc;
  return run_gemv<4096, true>("cb_gate_up_swiglu_i8", p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_lm_head_topk_i8(const void* x, const void* norm_w, float eps, const void* w, const float* scale,
                                  int64_t rows, int64_t row_offset, int k, float* logits, float* out_values,
                                  int64_t* out_indices, void* workspace, unsigned int* ticket, void* stream) {
  if (!scale) return fail(kErrInvalid, "cb_lm_head_topk_i8: scale is required");
  GemvParams p;
  int rc = build_lm_head_params(p, x, norm_w, eps, w, rows, row_offset, k, logits, out_values, out_indices,
                                workspace, ticket, 1, scale);
  if (rc != kOk) return rc;
  return run_gemv<4096, true>("cb_lm_head_topk_i8", p, static_cast<cudaStream_t>(stream));
}

namespace cb {

// bf16(q * scale) of int8 rows (the weights that prefill GEMMs use when a
// unit arrives in int8): one thread per 8 weights.
__global__ void __launch_bounds__(256) dequantize_rows_i8_kernel(const int8_t* __restrict__ q,
                                                                 const float* __restrict__ scale, int64_t rows,
                                                                 int K, uint16_t* __restrict__ out) {
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= rows * K) return;
  const float s = __ldg(scale + i / K);
  const uint2 v = *reinterpret_cast<const uint2*>(q + i);
  const uint32_t w0 = v.x ^ 0x80808080u, w1 = v.y ^ 0x80808080u;
  const float f[8] = {i8_at<0>(w0), i8_at<1>(w0), i8_at<2>(w0), i8_at<3>(w0),
                      i8_at<0>(w1), i8_at<1>(w1), i8_at<2>(w1), i8_at<3>(w1)};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e] = uint32_t(f2bf(f[2 * e] * s)) | (uint32_t(f2bf(f[2 * e + 1] * s)) << 16);
  *reinterpret_cast<uint4*>(out + i) = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace cb

extern "C" int cb_dequantize_rows_i8(const void* q, const float* scale, int64_t rows, int K, void* out,
                                     void* stream) {
  if (!q || !scale || !out || !aligned16(q) || !aligned16(out))
    return fail(kErrInvalid, "cb_dequantize_rows_i8: q and out must be 16-byte aligned device pointers");
  if (rows < 1 || K < 8 || K % 8) return fail(kErrInvalid, "cb_dequantize_rows_i8: rows >= 1, K a multiple of 8");
  const int64_t threads = rows * K / 8;
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > 0x7FFFFFFF) return fail(kErrInvalid, "cb_dequantize_rows_i8: too many weights");
  dequantize_rows_i8_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const int8_t*>(q), scale, rows, K, static_cast<uint16_t*>(out));
  return check_launch("cb_dequantize_rows_i8");
}
