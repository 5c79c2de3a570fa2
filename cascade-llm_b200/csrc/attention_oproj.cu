// Decode attention fused with the o_proj projection and its residual add,
// for one token over the full 8-KV-head layout (sm_100a).
//
// Replaces, in one launch, llama31.py:182-234 (`_repeat_kv` + SDPA) and
// :246-250 (o_proj F.linear + residual) of the reference. The two kernels it
// replaces run back to back with a grid-wide dependency between them, so the
// o_proj weights (33.5 MB) only start streaming once attention has finished
// and its launch has drained. Here the CTAs of one grid take two roles:
//
//   attention CTAs (blockIdx < 8 * splits): the split-KV attention of
//     attention.cu, unchanged; the CTA that merges a KV head's splits also
//     counts the head as done (release at GPU scope);
//   o_proj CTAs (the rest, 2 per SM together with the attention CTAs): each
//     owns a contiguous range of row pairs (j, j + 2048) of W_o. Before the
//     attention is done it already holds its first 4 pairs in registers and
//     the next 6 in shared memory (one bulk copy per half), so the weights
//     stream while attention computes; once the 8 heads are counted
//     (acquire) it reads the attention output and finishes the projection,
//     loading the few pairs left after the wait.
//
// Every o_proj dot product is summed in the order of gemv_kernel<4096>
// (per lane two 8-element chunks, warp butterfly, then the 8 K-slices in
// order), so the result is bit-identical to cb_attention + cb_proj_residual.
// All CTAs of the grid are resident together (2 per SM, grid = 2 x SMs),
// so the o_proj CTAs' wait always ends; it is bounded anyway (error 205).
#include "attention_device.cuh"
#include "common.cuh"
#include "gemv_device.cuh"
#include "internal.h"
#include "cascade_b200.h"

namespace cb {

int32_t* error_word();

constexpr int kOpPairs = 2048;       // row pairs (j, j + 2048) of W_o
constexpr int kOpRegPairs = 4;       // pairs a warp holds in registers (one batch)
constexpr int kOpSmemPairs = 6;      // pairs staged in shared memory
constexpr int kOpMaxPairs = kOpRegPairs + kOpSmemPairs + kOpRegPairs;  // + one batch after the wait
constexpr int kOpWarps = 8;          // K slices of 512 (warp 8 issues the bulk copies)

struct OpSmem {
  static constexpr size_t W = 0;                                            // [2][6][4096] bf16
  static constexpr size_t BAR = W + size_t(2) * kOpSmemPairs * 4096 * 2;   // one mbarrier
  static constexpr size_t PART = BAR + 16;                                  // [14][2][8] fp32
  static constexpr size_t BYTES = PART + size_t(kOpMaxPairs) * 2 * kOpWarps * 4;
};

struct AttnOprojParams {
  AttnParams a;              // the attention; a.out receives the [4096] attention output
  const uint16_t* wo;        // [4096][4096]
  const uint16_t* residual;  // [4096]
  uint16_t* out;             // [4096], may alias residual
  unsigned int* counters;    // [0] KV heads merged, [1] o_proj CTAs past the wait; zero between launches
  int attn_ctas;             // 8 * splits
  uint64_t wait_ns;
  int* err;
  uint64_t* trace;
  uint32_t trace_tag;
};

// Dot products of one pair's K slice for this lane (two 8-element chunks).
__device__ __forceinline__ void op_dot(const uint4 (&wa)[2], const uint4 (&wb)[2], const uint4 (&x)[2], float& a,
                                       float& b) {
  a = dot8(wa[0], x[0], 0.f);
  b = dot8(wb[0], x[0], 0.f);
  a = dot8(wa[1], x[1], a);
  b = dot8(wb[1], x[1], b);
}

static __device__ void oproj_cta(const AttnOprojParams& p, int cta, int ncta, uint8_t* smem) {
  const uint64_t t0 = trace_now(p.trace);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int u0 = kOpPairs * cta / ncta, u1 = kOpPairs * (cta + 1) / ncta, pairs = u1 - u0;
  const int nreg = min(pairs, kOpRegPairs);
  const int nsm = min(pairs - nreg, kOpSmemPairs);
  const int ntail = pairs - nreg - nsm;  // <= kOpRegPairs (checked by the host)
  uint16_t* wsm = reinterpret_cast<uint16_t*>(smem + OpSmem::W);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OpSmem::BAR);
  float* part = reinterpret_cast<float*>(smem + OpSmem::PART);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == kOpWarps * 32 && nsm > 0) {
    // pairs [u0 + nreg, u0 + nreg + nsm): their A rows, then their B rows
    const uint32_t bytes = uint32_t(nsm) * 4096 * 2;
    mbar_arrive_expect_tx(bar, 2 * bytes);
    bulk_g2s(wsm, p.wo + int64_t(u0 + nreg) * 4096, bytes, bar);
    bulk_g2s(wsm + kOpSmemPairs * 4096, p.wo + int64_t(u0 + nreg + kOpPairs) * 4096, bytes, bar);
  }
  const int kbase = warp * 512 + lane * 8;  // this warp's K slice (warps 0..7)
  uint4 w[kOpRegPairs][2][2];
  if (warp < kOpWarps) {
#pragma unroll
    for (int i = 0; i < kOpRegPairs; ++i) {
      if (i < nreg) {
        const uint16_t* ra = p.wo + int64_t(u0 + i) * 4096 + kbase;
        const uint16_t* rb = ra + int64_t(kOpPairs) * 4096;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          w[i][0][c] = ld_stream(ra + c * 256);
          w[i][1][c] = ld_stream(rb + c * 256);
        }
      }
    }
  }

  // wait until the 8 KV heads of this launch are merged
  if (tid == 0) {
    const uint64_t began = globaltimer_ns();
    bool ok = false;
    // relaxed polls with a short back-off (one thread per CTA), then one
    // acquire fence: the attention's output stores are visible after it
    for (uint32_t i = 0; i < (kSpinLimit << 4); ++i) {
      if (ld_relaxed_gpu(p.counters) >= 8u) {
        ok = true;
        break;
      }
      __nanosleep(100);
      if ((i & 15u) == 15u && globaltimer_ns() - began > p.wait_ns) break;
    }
    fence_acq_rel_gpu();
    if (!ok && p.err) atomicExch(p.err, 205);
    // every o_proj CTA is past the wait once the last one counts itself:
    // that one returns both counters to zero for the next launch
    if (atomicAdd(p.counters + 1, 1u) == unsigned(ncta - 1)) {
      p.counters[0] = 0u;
      p.counters[1] = 0u;
    }
    grid_dep_launch();  // the next projection may start placing its CTAs
  }
  __syncthreads();
  const uint64_t t1 = trace_now(p.trace);

  // the attention output (this warp's K slice) and the epilogue's residuals
  uint4 x[2];
  if (warp < kOpWarps) {
    x[0] = ld_cg_u4(p.a.out + kbase);
    x[1] = ld_cg_u4(p.a.out + kbase + 256);
  }
  float res_a = 0.f, res_b = 0.f;
  if (tid < pairs) {
    res_a = bf16f(__ldcg(p.residual + u0 + tid));
    res_b = bf16f(__ldcg(p.residual + u0 + tid + kOpPairs));
  }
  if (warp < kOpWarps) {
    auto publish = [&](int i, float a, float b) {
      a = warp_sum(a);
      b = warp_sum(b);
      if (lane == 0) {
        part[(i * 2 + 0) * kOpWarps + warp] = a;
        part[(i * 2 + 1) * kOpWarps + warp] = b;
      }
    };
#pragma unroll
    for (int i = 0; i < kOpRegPairs; ++i) {
      if (i < nreg) {
        float a, b;
        op_dot(w[i][0], w[i][1], x, a, b);
        publish(i, a, b);
      }
    }
    // the pairs after the staged ones: reuse the registers, loads in flight
    // while the staged pairs are consumed
#pragma unroll
    for (int i = 0; i < kOpRegPairs; ++i) {
      if (i < ntail) {
        const uint16_t* ra = p.wo + int64_t(u0 + nreg + nsm + i) * 4096 + kbase;
        const uint16_t* rb = ra + int64_t(kOpPairs) * 4096;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          w[i][0][c] = ld_stream(ra + c * 256);
          w[i][1][c] = ld_stream(rb + c * 256);
        }
      }
    }
    if (nsm > 0) mbar_wait(bar, 0, p.err, 206);
    for (int i = 0; i < nsm; ++i) {
      const uint16_t* sa = wsm + i * 4096 + kbase;
      const uint16_t* sb = wsm + (kOpSmemPairs + i) * 4096 + kbase;
      const uint4 wa[2] = {*reinterpret_cast<const uint4*>(sa), *reinterpret_cast<const uint4*>(sa + 256)};
      const uint4 wb[2] = {*reinterpret_cast<const uint4*>(sb), *reinterpret_cast<const uint4*>(sb + 256)};
      float a, b;
      op_dot(wa, wb, x, a, b);
      publish(nreg + i, a, b);
    }
#pragma unroll
    for (int i = 0; i < kOpRegPairs; ++i) {
      if (i < ntail) {
        float a, b;
        op_dot(w[i][0], w[i][1], x, a, b);
        publish(nreg + nsm + i, a, b);
      }
    }
  }
  __syncthreads();
  const uint64_t t2 = trace_now(p.trace);
  for (int i = tid; i < pairs; i += kAttnThreads) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int q = 0; q < kOpWarps; ++q) {
      a += part[(i * 2 + 0) * kOpWarps + q];
      b += part[(i * 2 + 1) * kOpWarps + q];
    }
    // the residual was loaded by thread i (i < 288 always: pairs <= 14)
    p.out[u0 + i] = f2bf(res_a + rbf(a));
    p.out[u0 + i + kOpPairs] = f2bf(res_b + rbf(b));
  }
  if (tid == 0) trace_commit(p.trace, p.trace_tag, blockIdx.x, t0, t1, t2);
}

__global__ void __launch_bounds__(kAttnThreads, 2) attn_oproj_kernel(const __grid_constant__ AttnOprojParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x;
  if (b < p.attn_ctas) {
    attention_cta(p.a, b % p.a.splits, b / p.a.splits, 0, unsigned(b), smem);
    return;
  }
  oproj_cta(p, b - p.attn_ctas, int(gridDim.x) - p.attn_ctas, smem);
}

constexpr size_t kAttnOprojSmem = AttnSmem::BYTES > OpSmem::BYTES ? AttnSmem::BYTES : OpSmem::BYTES;

int prepare_attention_oproj() {
  return configure_smem("cb_attention_oproj", attn_oproj_kernel, kAttnOprojSmem);
}

}  // namespace cb

using namespace cb;

extern "C" int cb_attention_oproj_max_splits(void) {
  // the o_proj CTAs (grid 2 x SMs minus 8 per split) must hold <= 14 pairs each
  const int grid = 2 * sm_count();
  int splits = 0;
  while (8 * (splits + 1) < grid && (kOpPairs + grid - 8 * (splits + 1) - 1) / (grid - 8 * (splits + 1)) <= kOpMaxPairs)
    ++splits;
  return splits;
}

extern "C" int cb_attention_oproj(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                                  const int32_t* position, int splits, const void* wo, const void* residual,
                                  void* attn_out, void* out, void* workspace, unsigned int* tickets, void* stream) {
  CB_REQUIRE(q && k_cache && v_cache && position && wo && residual && attn_out && out && workspace && tickets,
             "cb_attention_oproj: null pointer");
  CB_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(wo) && aligned16(attn_out),
             "cb_attention_oproj: q, caches, wo and attn_out must be 16-byte aligned");
  CB_REQUIRE(cache_len >= 1, "cb_attention_oproj: cache_len must be positive");
  const int max_splits = cb_attention_oproj_max_splits();
  CB_REQUIRE(splits >= 1 && splits <= max_splits, "cb_attention_oproj: splits=%d (1..%d on this GPU)", splits,
             max_splits);
  int rc = configure_smem("cb_attention_oproj", attn_oproj_kernel, kAttnOprojSmem);
  if (rc != kOk) return rc;
  AttnOprojParams p = {};
  AttnParams& a = p.a;
  a.q = static_cast<const uint16_t*>(q);
  a.k_cache = static_cast<const uint16_t*>(k_cache);
  a.v_cache = static_cast<const uint16_t*>(v_cache);
  a.cache_len = cache_len;
  a.pos = position;
  a.M = 1;
  a.kv_heads = 8;
  a.splits = splits;
  a.chunk = 0;  // sized on the device from the position
  a.out = static_cast<uint16_t*>(attn_out);
  const int64_t rows = int64_t(8) * kGroup * splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.part_o = reinterpret_cast<float*>(ws);
  a.part_ml = reinterpret_cast<float*>(ws + rows * kHeadDim * 4);
  a.tickets = tickets;
  a.heads_done = tickets + 8;
  a.err = error_word();
  uint32_t tag = 0;
  uint64_t* trace = trace_buffer(&tag);
  a.trace = trace;
  a.trace_tag = tag;
  p.wo = static_cast<const uint16_t*>(wo);
  p.residual = static_cast<const uint16_t*>(residual);
  p.out = static_cast<uint16_t*>(out);
  p.counters = tickets + 8;
  p.attn_ctas = 8 * splits;
  p.wait_ns = 2000000000ull;
  p.err = a.err;
  p.trace = trace;
  p.trace_tag = tag;
  const int grid = 2 * sm_count();
  return launch("cb_attention_oproj", attn_oproj_kernel, dim3(grid), dim3(kAttnThreads), kAttnOprojSmem,
                static_cast<cudaStream_t>(stream), p);
}
