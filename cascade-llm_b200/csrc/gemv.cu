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
//   * one CTA per SM (grid = SM count), 8 consumer warps + 1 producer warp;
//   * work is a list of "units"; a unit is a PAIR of weight rows (A, B) whose
//     outputs an epilogue needs together: rows d and d+64 of one head for
//     RoPE, gate row j and up row j for SwiGLU, rows j and j+N/2 otherwise.
//     Units are split evenly over CTAs (row granularity, <=1.2% imbalance);
//   * the producer streams tiles of T units (2T contiguous-row slabs) with
//     cp.async.bulk into an NSTAGE-deep shared-memory ring, tracked by
//     mbarriers, with an L2 evict_first hint (weights are read once);
//   * the producer starts streaming BEFORE griddepcontrol.wait (weights do
//     not depend on the previous kernel), so with programmatic dependent
//     launch the next projection's weights are already in flight while the
//     previous kernel drains;
//   * consumers hold their slice of the activation vector in registers for
//     the whole kernel; each warp owns one row of a tile and 1/WPR of K, so
//     smem reads are 512 contiguous bytes per warp instruction (no bank
//     conflicts) and the reduction is one warp shuffle tree + WPR partials.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "cascade_b200.h"

namespace cb {

// Every GEMV launch is two CTAs per SM (one full wave at <= 128 registers
// per thread); the LM-head candidate workspace is sized by the same grid.
static int gemv_grid() { return 2 * sm_count(); }
static int lm_head_grid() { return gemv_grid(); }

enum EpiMode : int {
  EPI_STORE = 0,     // out[oA] = bf16(a), out[oB] = bf16(b)
  EPI_RESIDUAL = 1,  // out[o] = bf16(aux[o] + bf16(acc))
  EPI_ROPE = 2,      // RoPE on the (d, d+64) pair, store
  EPI_SILU = 3,      // out[o] = bf16(silu(bf16(acc)))
  EPI_MUL = 4,       // out[o] = bf16(aux[o] * bf16(acc))
  EPI_SWIGLU = 5,    // out[j] = bf16(bf16(silu(bf16(a))) * bf16(b))
  EPI_TOPK = 6,      // fp32 logits of bf16(acc) -> running top-k
};

constexpr int kThreads = 256;
constexpr int kTopkMax = 64;
constexpr size_t kMaxSmem = 227 * 1024;

struct Segment {
  const uint16_t* a_base;  // weight row base of slab A rows
  const uint16_t* b_base;  // weight row base of slab B rows
  int units;               // pair units in this segment
  int group;               // units per group; a tile never crosses a group
  int group_stride;        // weight rows between the starts of two groups
  int mode;                // EpiMode
  uint16_t* out;           // bf16 output base
  const uint16_t* aux;     // residual / silu(gate), same indexing as out
  int64_t head_stride;     // output elements between groups
  int64_t b_offset;        // output index of row B minus that of row A
  int64_t pos_stride;      // output elements per position (cache writes), 0 otherwise
  int64_t pos_limit;       // cache capacity in positions (cache writes)
};

struct GemvParams {
  Segment seg[3];
  int nseg;
  int total_units;
  const uint16_t* x;       // activation row [K] (this launch's token)
  const uint16_t* norm_w;  // RMSNorm weight [K] or null
  float eps;
  const float* inv_freq;   // [64] RoPE inverse frequencies
  const int32_t* pos;      // device position of token 0 of the step
  int token;               // token index within the step (position = *pos + token)
  // top-k (EPI_TOPK)
  int k;
  int64_t row_offset;
  float* logits;           // optional fp32 logits, indexed by local row
  float* cand_values;      // [gridDim.x * k]
  int64_t* cand_indices;
  unsigned int* ticket;    // zero-initialised, reset by the last CTA
  float* out_values;       // [k]
  int64_t* out_indices;
  int* err;
};

__device__ __forceinline__ int64_t unit_row(const Segment& s, int j) {
  return int64_t(j / s.group) * s.group_stride + (j % s.group);
}

__device__ __forceinline__ bool ranks_before(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

// Warp-cooperative exact top-k over n (value, index) pairs in shared memory.
__device__ void warp_select_rows_idx(const float* vals, const int64_t* idx, int n, int k, float* out_v,
                                     int64_t* out_i) {
  const int lane = threadIdx.x & 31;
  float pv = __int_as_float(0x7F800000);
  int64_t pi = -1;
  for (int r = 0; r < k; ++r) {
    float bv = -__int_as_float(0x7F800000);
    int64_t bi = INT64_MAX;
    for (int c = lane; c < n; c += 32) {
      const float v = vals[c];
      const int64_t i = idx[c];
      if (ranks_before(pv, pi, v, i) && ranks_before(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ranks_before(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_v[r] = bv;
      out_i[r] = bi;
    }
    pv = bv;
    pi = bi;
  }
}

// Warp-cooperative exact top-k over a CTA's logits in shared memory:
// entry i < na is row a0 + i, entry i >= na is row b0 + (i - na). Missing
// entries (n < k) are written as (-inf, INT64_MAX).
__device__ void warp_select_rows(const float* vals, int n, int na, int64_t a0, int64_t b0, int k,
                                 float* out_v, int64_t* out_i) {
  const int lane = threadIdx.x & 31;
  float pv = __int_as_float(0x7F800000);
  int64_t pi = -1;
  for (int r = 0; r < k; ++r) {
    float bv = -__int_as_float(0x7F800000);
    int64_t bi = INT64_MAX;
    for (int c = lane; c < n; c += 32) {
      const float v = vals[c];
      const int64_t i = c < na ? a0 + c : b0 + (c - na);
      if (ranks_before(pv, pi, v, i) && ranks_before(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ranks_before(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_v[r] = bv;
      out_i[r] = bi;
    }
    pv = bv;
    pi = bi;
  }
}

// Warp-cooperative exact top-k of n candidates; lane 0 writes the result.
// Round r selects the best candidate that ranks strictly after round r-1's.
__device__ void warp_select_topk(const float* vals, const int64_t* idx, int n, int k,
                                 float* out_v, int64_t* out_i) {
  const int lane = threadIdx.x & 31;
  float pv = __int_as_float(0x7F800000);  // +inf: everything ranks after it
  int64_t pi = -1;
  for (int r = 0; r < k; ++r) {
    float bv = -__int_as_float(0x7F800000);
    int64_t bi = INT64_MAX;
    bool have = false;
    for (int c = lane; c < n; c += 32) {
      // candidates were written by other CTAs: read through L2
      float v = __ldcg(vals + c);
      int64_t i = __ldcg(reinterpret_cast<const long long*>(idx) + c);
      if (ranks_before(pv, pi, v, i) && (!have || ranks_before(v, i, bv, bi))) {
        bv = v;
        bi = i;
        have = true;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ranks_before(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_v[r] = bv;
      out_i[r] = bi;
    }
    pv = bv;
    pi = bi;
  }
}

// Exact top-k of G sorted per-CTA candidate lists (k each, in global
// memory), by the whole CTA. The k-th best of the union is at least the
// largest per-list k-th value, so only candidates at or above that
// threshold can qualify: one parallel pass finds the threshold, a second
// copies the survivors to shared memory, and warp 0 selects among them.
// `scratch` must hold kMergeCap floats + kMergeCap int64s.
constexpr int kMergeCap = 1024;
__device__ void block_merge_topk(const float* vals, const int64_t* idx, int G, int k, float* out_v,
                                 int64_t* out_i, float* red, float* scratch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float thr = -__int_as_float(0x7F800000);
  for (int c = tid; c < G; c += blockDim.x) thr = fmaxf(thr, __ldcg(vals + size_t(c) * k + (k - 1)));
  thr = warp_max(thr);
  __syncthreads();
  if (lane == 0) red[warp] = thr;
  int* count = reinterpret_cast<int*>(red + 14);
  if (tid == 0) *count = 0;
  __syncthreads();
  thr = red[0];
  for (int q = 1; q < int(blockDim.x >> 5); ++q) thr = fmaxf(thr, red[q]);
  float* sv = scratch;
  int64_t* si = reinterpret_cast<int64_t*>(scratch + kMergeCap);
  const int n = G * k;
  for (int c = tid; c < n; c += blockDim.x) {
    const float v = __ldcg(vals + c);
    if (v >= thr) {
      const int slot = atomicAdd(count, 1);
      if (slot < kMergeCap) {
        sv[slot] = v;
        si[slot] = __ldcg(reinterpret_cast<const long long*>(idx) + c);
      }
    }
  }
  __syncthreads();
  const int kept = *count;
  if (warp == 0) {
    if (kept <= kMergeCap)
      warp_select_rows_idx(sv, si, kept, k, out_v, out_i);
    else  // pathological ties: fall back to scanning every candidate
      warp_select_topk(vals, idx, n, k, out_v, out_i);
  }
}


}  // namespace cb

namespace cb {

__device__ __forceinline__ uint4 normalize8(uint4 xu, uint4 wu, float inv) {
  const uint32_t in[4] = {xu.x, xu.y, xu.z, xu.w};
  const uint32_t wv[4] = {wu.x, wu.y, wu.z, wu.w};
  uint32_t out[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    // llama31.py:21-25: bf16(x * rsqrt(...)), then bf16(w * that)
    const float lo = rbf(bf16lo(wv[q]) * rbf(bf16lo(in[q]) * inv));
    const float hi = rbf(bf16hi(wv[q]) * rbf(bf16hi(in[q]) * inv));
    out[q] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// Loads of weights that are read exactly once: 128-bit, not cached in L1.
__device__ __forceinline__ uint4 ld_stream(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float silu_bf16(float g) {
  // torch's silu on a bf16 tensor: x / (1 + exp(-x)) in fp32, rounded
  return rbf(g / (1.0f + expf(-g)));
}

__device__ void gemv_epilogue(const GemvParams& p, const Segment& sg, int j, float a, float b,
                              int pos) {
  int64_t oa = int64_t(j / sg.group) * sg.head_stride + (j % sg.group);
  if (sg.pos_stride) {
    if (pos < 0 || pos >= sg.pos_limit) {  // never write outside the cache
      if (p.err) atomicExch(p.err, 103);
      return;
    }
    oa += int64_t(pos) * sg.pos_stride;
  }
  const int64_t ob = oa + sg.b_offset;
  switch (sg.mode) {
    case EPI_STORE:
      sg.out[oa] = f2bf(a);
      sg.out[ob] = f2bf(b);
      break;
    case EPI_RESIDUAL:
      sg.out[oa] = f2bf(bf16f(__ldcg(sg.aux + oa)) + rbf(a));
      sg.out[ob] = f2bf(bf16f(__ldcg(sg.aux + ob)) + rbf(b));
      break;
    case EPI_ROPE: {
      // transformers modeling_llama.py:124-168: cos/sin of (inv_freq * pos)
      // in fp32, cast to bf16; q*cos + rotate_half(q)*sin in bf16.
      const int d = j % sg.group;
      const float freq = __ldg(p.inv_freq + d) * float(pos);
      const float c = rbf(cosf(freq)), s = rbf(sinf(freq));
      const float qa = rbf(a), qb = rbf(b);
      sg.out[oa] = f2bf(rbf(qa * c) + rbf(-qb * s));
      sg.out[ob] = f2bf(rbf(qb * c) + rbf(qa * s));
      break;
    }
    case EPI_SILU:
      sg.out[oa] = f2bf(silu_bf16(rbf(a)));
      sg.out[ob] = f2bf(silu_bf16(rbf(b)));
      break;
    case EPI_MUL:
      sg.out[oa] = f2bf(bf16f(__ldcg(sg.aux + oa)) * rbf(a));
      sg.out[ob] = f2bf(bf16f(__ldcg(sg.aux + ob)) * rbf(b));
      break;
    case EPI_SWIGLU:
      sg.out[oa] = f2bf(silu_bf16(rbf(a)) * rbf(b));
      break;
    default:
      break;
  }
}

template <int K>
struct GemvShape {
  static constexpr int WARPS = kThreads / 32;
  static constexpr int KS = K / WARPS;          // K-slice of each warp
  static constexpr int CPL = KS / 256;          // 16-byte chunks per lane per row slice
  static constexpr int UB = (16 / (2 * CPL)) > 0 ? 16 / (2 * CPL) : 1;  // units per batch
  static constexpr size_t RED = 0;              // [16] fp32 (norm partials, flag)
  static constexpr size_t SMEM = RED + 16 * 4;  // + per-unit partials (+ logits), sized at launch
  static_assert(KS % 256 == 0, "each warp's K-slice must be whole 512-byte lane groups");
};

// CTA-cooperative split-K GEMV. A CTA owns a contiguous range of units (row
// pairs); each of its 8 warps streams its own 1/8 of K for EVERY unit of the
// range (UB units, i.e. 2*UB*CPL 128-bit loads per lane, in flight per
// batch), so all warps carry the same load and stream until the end. Per
// unit, each warp reduces its two partial dots with shuffles into shared
// memory; after ONE barrier the epilogues of all units run in parallel, one
// thread per unit. The activation slice of a warp stays in registers. The
// first batch of weight loads is issued before griddepcontrol.wait.
template <int K>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
  using S = GemvShape<K>;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + S::RED);
  float* part = reinterpret_cast<float*>(smem + S::SMEM);  // [units][2][WARPS]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x;
  const int u0 = int(int64_t(p.total_units) * blockIdx.x / G);
  const int u1 = int(int64_t(p.total_units) * (blockIdx.x + 1) / G);
  const int units = u1 - u0;
  float* lrow = part + size_t(units) * 2 * S::WARPS;  // EPI_TOPK: this CTA's logits
  const int kbase = warp * S::KS + lane * 8;            // first element of this lane

  auto locate = [&](int u, int& seg, int& j) {
    seg = 0;
    j = u;
    while (seg + 1 < p.nseg && j >= p.seg[seg].units) {
      j -= p.seg[seg].units;
      ++seg;
    }
  };
  auto row_ptrs = [&](int u, const uint16_t*& ra, const uint16_t*& rb) {
    int seg, j;
    locate(u, seg, j);
    const Segment& sg = p.seg[seg];
    const int64_t row = int64_t(j / sg.group) * sg.group_stride + (j % sg.group);
    ra = sg.a_base + row * K + kbase;
    rb = sg.b_base + row * K + kbase;
  };
  uint4 w[S::UB][2][S::CPL];
  auto load_batch = [&](int ub) {
#pragma unroll
    for (int i = 0; i < S::UB; ++i) {
      if (ub + i < u1) {
        const uint16_t *ra, *rb;
        row_ptrs(ub + i, ra, rb);
#pragma unroll
        for (int c = 0; c < S::CPL; ++c) {
          w[i][0][c] = ld_stream(ra + c * 256);
          w[i][1][c] = ld_stream(rb + c * 256);
        }
      }
    }
  };

  // weights do not depend on the previous kernel: start streaming now
  load_batch(u0);

  grid_dep_wait();  // the activation row comes from the previous kernel
  if (tid == 0) grid_dep_launch();
  float inv = 1.0f;
  if (p.norm_w) {
    float ss = 0.f;
    for (int c = tid; c < K / 8; c += kThreads) {
      const uint4 v = ld_cg_u4(p.x + c * 8);
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        ss = fmaf(bf16lo(w4[q]), bf16lo(w4[q]), ss);
        ss = fmaf(bf16hi(w4[q]), bf16hi(w4[q]), ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int q = 0; q < S::WARPS; ++q) tot += red[q];
    inv = rsqrtf(tot * (1.0f / K) + p.eps);
  }
  uint4 xr[S::CPL];
#pragma unroll
  for (int c = 0; c < S::CPL; ++c) {
    uint4 v = ld_cg_u4(p.x + kbase + c * 256);
    if (p.norm_w) v = normalize8(v, __ldg(reinterpret_cast<const uint4*>(p.norm_w + kbase + c * 256)), inv);
    xr[c] = v;
  }

  for (int ub = u0; ub < u1; ub += S::UB) {
    if (ub != u0) load_batch(ub);
#pragma unroll
    for (int i = 0; i < S::UB; ++i) {
      if (ub + i < u1) {
        float a = 0.f, b = 0.f;
#pragma unroll
        for (int c = 0; c < S::CPL; ++c) {
          a = dot8(w[i][0][c], xr[c], a);
          b = dot8(w[i][1][c], xr[c], b);
        }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
          part[((ub + i - u0) * 2 + 0) * S::WARPS + warp] = a;
          part[((ub + i - u0) * 2 + 1) * S::WARPS + warp] = b;
        }
      }
    }
  }
  __syncthreads();

  const int pos = p.pos ? __ldcg(p.pos) + p.token : 0;
  for (int i = tid; i < units; i += kThreads) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int q = 0; q < S::WARPS; ++q) {
      a += part[(i * 2 + 0) * S::WARPS + q];
      b += part[(i * 2 + 1) * S::WARPS + q];
    }
    int seg, j;
    locate(u0 + i, seg, j);
    const Segment& sg = p.seg[seg];
    if (sg.mode == EPI_TOPK) {
      const float la = rbf(a), lb = rbf(b);  // F.linear(...) is bf16, then .float()
      const int64_t row = int64_t(j / sg.group) * sg.group_stride + (j % sg.group);
      if (p.logits) {
        p.logits[row] = la;
        p.logits[row + sg.b_offset] = lb;
      }
      lrow[i] = la;
      lrow[units + i] = lb;
    } else {
      gemv_epilogue(p, sg, j, a, b, pos);
    }
  }

  if (p.cand_values == nullptr) return;
  // ---------------- LM head: this CTA's exact top-k, then the last CTA merges
  __syncthreads();
  if (warp == 0) {
    const int64_t half = p.seg[0].b_offset;
    warp_select_rows(lrow, 2 * units, units, p.row_offset + u0, p.row_offset + half + u0, p.k,
                     p.cand_values + size_t(blockIdx.x) * p.k, p.cand_indices + size_t(blockIdx.x) * p.k);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned int ticket = atomicAdd(p.ticket, 1u);
    red[15] = __int_as_float(ticket == unsigned(G - 1) ? 1 : 0);
  }
  __syncthreads();
  if (__float_as_int(red[15]) != 1) return;
  __threadfence();
  block_merge_topk(p.cand_values, p.cand_indices, G, p.k, p.out_values, p.out_indices, red,
                   reinterpret_cast<float*>(lrow));
  if (tid == 0) *p.ticket = 0u;
}

}  // namespace cb

// ====================================================================== host
namespace cb {

int32_t* error_word();

template <int K>
static int run_gemv(const char* what, GemvParams& p, cudaStream_t stream) {
  using S = GemvShape<K>;
  int rc = configure_smem(what, gemv_kernel<K>, kMaxSmem);
  if (rc != kOk) return rc;
  p.total_units = 0;
  for (int i = 0; i < p.nseg; ++i) p.total_units += p.seg[i].units;
  if (p.total_units == 0) return kOk;
  p.err = error_word();
  const int grid = gemv_grid();
  const size_t per_cta = size_t((p.total_units + grid - 1) / grid);
  size_t smem = S::SMEM + per_cta * 2 * S::WARPS * sizeof(float);  // per-unit partials
  if (p.cand_values) {
    // EPI_TOPK: the CTA's logits, later reused as the last CTA's merge scratch
    smem += std::max(per_cta * 2 * sizeof(float), size_t(kMergeCap) * (sizeof(float) + sizeof(int64_t)));
  }
  if (smem > kMaxSmem) return fail(kErrInvalid, "%s: %zu units per CTA exceed shared memory", what, per_cta);
  return launch(what, gemv_kernel<K>, dim3(grid), dim3(kThreads), smem, stream, p);
}

static Segment half_segment(const void* w, int N, int K, int mode, void* out, const void* aux) {
  Segment s = {};
  s.a_base = static_cast<const uint16_t*>(w);
  s.b_base = s.a_base + int64_t(N / 2) * K;
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
                            int64_t pos_stride, int64_t pos_limit = 0) {
  Segment s = {};
  s.a_base = static_cast<const uint16_t*>(w);
  s.b_base = s.a_base + int64_t(64) * 4096;
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

#define CB_REQUIRE(cond, ...) \
  do {                        \
    if (!(cond)) return fail(kErrInvalid, __VA_ARGS__); \
  } while (0)

extern "C" int cb_qkv_rope(const void* x, const void* norm_w, float eps, const void* wq,
                           const void* wk, const void* wv, const float* inv_freq,
                           const int32_t* position, int token, void* q_out, void* k_cache,
                           void* v_cache, int64_t cache_len, void* stream) {
  CB_REQUIRE(x && aligned16(x), "cb_qkv_rope: x must be a 16-byte aligned device pointer");
  CB_REQUIRE(!norm_w || aligned16(norm_w), "cb_qkv_rope: norm_w must be 16-byte aligned");
  CB_REQUIRE(inv_freq && position, "cb_qkv_rope: inv_freq and position are required");
  CB_REQUIRE(token >= 0, "cb_qkv_rope: token must be >= 0");
  GemvParams p = {};
  p.x = static_cast<const uint16_t*>(x);
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  p.inv_freq = inv_freq;
  p.pos = position;
  p.token = token;
  if (wq) {
    CB_REQUIRE(aligned16(wq) && q_out, "cb_qkv_rope: wq needs alignment and q_out");
    p.seg[p.nseg++] = head_segment(wq, 32, EPI_ROPE, q_out, 128, 0);
  }
  if (wk || wv) CB_REQUIRE(cache_len > 0, "cb_qkv_rope: cache_len must be positive");
  if (wk) {
    CB_REQUIRE(aligned16(wk) && k_cache, "cb_qkv_rope: wk needs alignment and k_cache");
    p.seg[p.nseg++] = head_segment(wk, 8, EPI_ROPE, k_cache, cache_len * 128, 128, cache_len);
  }
  if (wv) {
    CB_REQUIRE(aligned16(wv) && v_cache, "cb_qkv_rope: wv needs alignment and v_cache");
    p.seg[p.nseg++] = head_segment(wv, 8, EPI_STORE, v_cache, cache_len * 128, 128, cache_len);
  }
  return run_gemv<4096>("cb_qkv_rope", p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_proj_residual(const void* x, int K, const void* w, int N, const void* residual,
                                void* out, void* stream) {
  CB_REQUIRE(x && w && residual && out, "cb_proj_residual: null pointer");
  CB_REQUIRE(aligned16(x) && aligned16(w), "cb_proj_residual: x and w must be 16-byte aligned");
  CB_REQUIRE(N > 0 && N % 2 == 0, "cb_proj_residual: N must be even and positive");
  GemvParams p = {};
  p.x = static_cast<const uint16_t*>(x);
  p.seg[p.nseg++] = half_segment(w, N, K, EPI_RESIDUAL, out, residual);
  auto s = static_cast<cudaStream_t>(stream);
  if (K == 4096) return run_gemv<4096>("cb_proj_residual", p, s);
  if (K == 14336) return run_gemv<14336>("cb_proj_residual", p, s);
  return fail(kErrUnsupported, "cb_proj_residual: K=%d (supported: 4096, 14336)", K);
}

static int gate_up_common(const char* what, const void* x, const void* norm_w, float eps,
                          const void* w_gate, const void* w_up, int mode, void* out,
                          const void* aux, void* stream) {
  CB_REQUIRE(x && out && aligned16(x), "%s: x/out invalid", what);
  CB_REQUIRE(!norm_w || aligned16(norm_w), "%s: norm_w must be 16-byte aligned", what);
  GemvParams p = {};
  p.x = static_cast<const uint16_t*>(x);
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  const int N = 14336;
  if (mode == EPI_SWIGLU) {
    CB_REQUIRE(w_gate && w_up && aligned16(w_gate) && aligned16(w_up), "%s: weights invalid", what);
    Segment s = half_segment(w_gate, 2 * N, 4096, EPI_SWIGLU, out, nullptr);
    s.b_base = static_cast<const uint16_t*>(w_up);
    s.b_offset = 0;
    p.seg[p.nseg++] = s;
  } else {
    const void* w = mode == EPI_SILU ? w_gate : w_up;
    CB_REQUIRE(w && aligned16(w), "%s: weight invalid", what);
    p.seg[p.nseg++] = half_segment(w, N, 4096, mode, out, aux);
  }
  return run_gemv<4096>(what, p, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_gate_up_swiglu(const void* x, const void* norm_w, float eps, const void* w_gate,
                                 const void* w_up, void* out, void* stream) {
  return gate_up_common("cb_gate_up_swiglu", x, norm_w, eps, w_gate, w_up, EPI_SWIGLU, out,
                        nullptr, stream);
}

extern "C" int cb_gate_silu(const void* x, const void* norm_w, float eps, const void* w_gate,
                            void* out, void* stream) {
  return gate_up_common("cb_gate_silu", x, norm_w, eps, w_gate, nullptr, EPI_SILU, out, nullptr,
                        stream);
}

extern "C" int cb_up_mul(const void* x, const void* norm_w, float eps, const void* w_up,
                         void* gate_act, void* stream) {
  return gate_up_common("cb_up_mul", x, norm_w, eps, nullptr, w_up, EPI_MUL, gate_act, gate_act,
                        stream);
}

namespace cb {
int prepare_gemv() {
  int rc = configure_smem("gemv", gemv_kernel<4096>, kMaxSmem);
  if (rc == kOk) rc = configure_smem("gemv", gemv_kernel<14336>, kMaxSmem);
  return rc;
}
}  // namespace cb

extern "C" int64_t cb_lm_head_workspace_bytes(int k) {
  // candidates: values [CTAs*k] fp32, then indices [CTAs*k] int64
  const int64_t n = int64_t(lm_head_grid()) * k;
  return ((n * 4 + 15) / 16) * 16 + n * 8;
}

extern "C" int cb_lm_head_topk(const void* x, const void* norm_w, float eps, const void* w,
                               int64_t rows, int64_t row_offset, int k, float* logits,
                               float* out_values, int64_t* out_indices, void* workspace,
                               unsigned int* ticket, void* stream) {
  CB_REQUIRE(x && w && out_values && out_indices && workspace && ticket, "cb_lm_head_topk: null pointer");
  CB_REQUIRE(aligned16(x) && aligned16(w), "cb_lm_head_topk: x and w must be 16-byte aligned");
  CB_REQUIRE(!norm_w || aligned16(norm_w), "cb_lm_head_topk: norm_w must be 16-byte aligned");
  CB_REQUIRE(rows > 0 && rows % 2 == 0 && rows <= (int64_t(1) << 30),
             "cb_lm_head_topk: rows must be even, positive and < 2^30 (got %lld)", (long long)rows);
  CB_REQUIRE(k >= 1 && k <= kTopkMax && k <= rows, "cb_lm_head_topk: need 1 <= k <= min(64, rows)");
  GemvParams p = {};
  p.x = static_cast<const uint16_t*>(x);
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  Segment s = half_segment(w, int(rows), 4096, EPI_TOPK, nullptr, nullptr);
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
  return run_gemv<4096>("cb_lm_head_topk", p, static_cast<cudaStream_t>(stream));
}
