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

#include "common.cuh"
#include "internal.h"
#include "cascade_b200.h"

namespace cb {

enum EpiMode : int {
  EPI_STORE = 0,     // out[oA] = bf16(a), out[oB] = bf16(b)
  EPI_RESIDUAL = 1,  // out[o] = bf16(aux[o] + bf16(acc))
  EPI_ROPE = 2,      // RoPE on the (d, d+64) pair, store
  EPI_SILU = 3,      // out[o] = bf16(silu(bf16(acc)))
  EPI_MUL = 4,       // out[o] = bf16(aux[o] * bf16(acc))
  EPI_SWIGLU = 5,    // out[j] = bf16(bf16(silu(bf16(a))) * bf16(b))
  EPI_TOPK = 6,      // fp32 logits of bf16(acc) -> running top-k
};

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kTopkMax = 64;

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

// ---------------------------------------------------------------- tiles
// A CTA walks units [u0, u1) in tiles of <= T units that never cross a
// segment or group boundary; producer and consumers walk the same sequence.
struct TileWalker {
  int u, u1, seg, seg_start;
  __device__ void begin(const GemvParams& p, int first, int last) {
    u = first;
    u1 = last;
    seg = 0;
    seg_start = 0;
    while (seg < p.nseg && u >= seg_start + p.seg[seg].units) {
      seg_start += p.seg[seg].units;
      ++seg;
    }
  }
  // returns false when done; else segment index, local unit j0, count t
  template <int T>
  __device__ bool next(const GemvParams& p, int& s, int& j0, int& t) {
    if (u >= u1) return false;
    while (u >= seg_start + p.seg[seg].units) {
      seg_start += p.seg[seg].units;
      ++seg;
    }
    const Segment& sg = p.seg[seg];
    j0 = u - seg_start;
    int left_group = sg.group - (j0 % sg.group);
    int left_seg = sg.units - j0;
    int left_cta = u1 - u;
    t = min(T, min(left_group, min(left_seg, left_cta)));
    s = seg;
    u += t;
    return true;
  }
};

__device__ __forceinline__ int64_t unit_row(const Segment& s, int j) {
  return int64_t(j / s.group) * s.group_stride + (j % s.group);
}

__device__ __forceinline__ bool ranks_before(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

// Insert (v, i) into a sorted list of length *n (capacity k).
__device__ void topk_insert(float* vals, int64_t* idx, int& n, int k, float v, int64_t i) {
  if (n == k && !ranks_before(v, i, vals[k - 1], idx[k - 1])) return;
  int pos = n < k ? n : k - 1;
  while (pos > 0 && ranks_before(v, i, vals[pos - 1], idx[pos - 1])) {
    vals[pos] = vals[pos - 1];
    idx[pos] = idx[pos - 1];
    --pos;
  }
  vals[pos] = v;
  idx[pos] = i;
  if (n < k) ++n;
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

}  // namespace cb

namespace cb {

template <int K, int KT, int T, int NSTAGE, bool XS>
struct GemvCfg {
  static constexpr int R = 2 * T;                  // weight rows per tile
  static constexpr int WPR = kConsumerWarps / R;   // warps per row
  static constexpr int KSEG = KT / WPR;            // K elements per warp per K-tile
  static constexpr int KPL = KSEG / 256;           // uint4 (8 bf16) per lane per K-tile
  static constexpr int NKT = K / KT;               // K-tiles per row
  static constexpr int STAGE_ELEMS = R * KT;
  static constexpr size_t RING = size_t(NSTAGE) * STAGE_ELEMS * 2;
  static constexpr size_t BARS = RING;                               // full[NSTAGE], empty[NSTAGE]
  static constexpr size_t PART = BARS + 2 * NSTAGE * 8;              // [2][R][WPR] fp32
  static constexpr size_t RED = PART + 2 * R * WPR * 4;              // [8] fp32 + flag
  static constexpr size_t TOPV = (RED + 16 * 4 + 15) / 16 * 16;      // [kTopkMax] fp32
  static constexpr size_t TOPI = TOPV + kTopkMax * 4;                // [kTopkMax] int64
  static constexpr size_t XSM = TOPI + kTopkMax * 8;                 // [K] bf16 when XS
  static constexpr size_t SMEM = XSM + (XS ? size_t(K) * 2 : 0);
  static_assert(kConsumerWarps % R == 0, "rows per tile must divide the consumer warps");
  static_assert(KSEG % 256 == 0 && KPL >= 1, "K-tile must split into whole 512-byte warp reads");
  static_assert(K % KT == 0, "K-tiles must cover K");
  static_assert((KT * 2) % 16 == 0, "bulk copies move multiples of 16 bytes");
};

__device__ __forceinline__ uint4 normalize8(uint4 xu, uint4 wu, float inv) {
  uint32_t in[4] = {xu.x, xu.y, xu.z, xu.w};
  uint32_t wv[4] = {wu.x, wu.y, wu.z, wu.w};
  uint32_t out[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    // llama31.py:21-25: bf16(x * rsqrt(...)), then bf16(w * that)
    float lo = rbf(bf16lo(wv[q]) * rbf(bf16lo(in[q]) * inv));
    float hi = rbf(bf16hi(wv[q]) * rbf(bf16hi(in[q]) * inv));
    out[q] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
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

// Two CTAs of 288 threads x 112 registers fit one SM's 64K registers, so a
// kernel's CTAs can share an SM with the next kernel's early-launched ones.
template <int K, int KT, int T, int NSTAGE, bool XS>
__global__ void __maxnreg__(112)
    gemv_kernel(const __grid_constant__ GemvParams p) {
  using C = GemvCfg<K, KT, T, NSTAGE, XS>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint16_t* ring = reinterpret_cast<uint16_t*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BARS);
  uint64_t* empty = full + NSTAGE;
  float* partial = reinterpret_cast<float*>(smem + C::PART);
  float* red = reinterpret_cast<float*>(smem + C::RED);
  float* topv = reinterpret_cast<float*>(smem + C::TOPV);
  int64_t* topi = reinterpret_cast<int64_t*>(smem + C::TOPI);
  uint16_t* xsm = reinterpret_cast<uint16_t*>(smem + C::XSM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int u0 = int(int64_t(p.total_units) * blockIdx.x / G);
  const int u1 = int(int64_t(p.total_units) * (blockIdx.x + 1) / G);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer: weights only, so no grid-dependency wait
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      TileWalker w;
      w.begin(p, u0, u1);
      int s, j0, t, stage = 0;
      uint32_t phase = 0;
      while (w.next<T>(p, s, j0, t)) {
        const Segment& sg = p.seg[s];
        const int64_t row = unit_row(sg, j0);
        const uint16_t* a = sg.a_base + row * K;
        const uint16_t* b = sg.b_base + row * K;
        for (int kt = 0; kt < C::NKT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, 101)) return;
          uint16_t* dst = ring + size_t(stage) * C::STAGE_ELEMS;
          mbar_arrive_expect_tx(&full[stage], uint32_t(2 * t * KT * 2));
          if (KT == K) {
            bulk_g2s_stream(dst, a, uint32_t(t * K * 2), &full[stage], pol);
            bulk_g2s_stream(dst + T * KT, b, uint32_t(t * K * 2), &full[stage], pol);
          } else {
            for (int r = 0; r < t; ++r) {
              bulk_g2s_stream(dst + r * KT, a + r * K + kt * KT, KT * 2, &full[stage], pol);
              bulk_g2s_stream(dst + (T + r) * KT, b + r * K + kt * KT, KT * 2, &full[stage], pol);
            }
          }
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers
  const int ctid = threadIdx.x;
  grid_dep_wait();   // activations come from the previous kernel
  if (ctid == 0) grid_dep_launch();

  float inv = 1.0f;
  if (p.norm_w) {
    float ss = 0.f;
    for (int c = ctid; c < K / 8; c += kConsumers) {
      const uint4 u = ld_cg_u4(p.x + c * 8);
      const uint32_t v[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = bf16lo(v[q]), hi = bf16hi(v[q]);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    named_sync(1, kConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
    inv = rsqrtf(tot * (1.0f / K) + p.eps);
  }

  const int r = warp / C::WPR, part = warp % C::WPR;
  const int rr = r < T ? r : r - T;
  // activation slice of this warp: registers (XS=false) or the whole row in
  // shared memory (XS=true, for K=14336 where registers would spill)
  uint4 xf[XS ? 1 : C::NKT][XS ? 1 : C::KPL];
  if constexpr (XS) {
    for (int c = ctid; c < K / 8; c += kConsumers) {
      uint4 u = ld_cg_u4(p.x + c * 8);
      if (p.norm_w) u = normalize8(u, __ldg(reinterpret_cast<const uint4*>(p.norm_w + c * 8)), inv);
      reinterpret_cast<uint4*>(xsm)[c] = u;
    }
    named_sync(1, kConsumers);
  } else {
#pragma unroll
    for (int kt = 0; kt < C::NKT; ++kt)
#pragma unroll
      for (int i = 0; i < C::KPL; ++i) {
        const int k0 = kt * KT + part * C::KSEG + (lane + 32 * i) * 8;
        uint4 u = ld_cg_u4(p.x + k0);
        if (p.norm_w) u = normalize8(u, __ldg(reinterpret_cast<const uint4*>(p.norm_w + k0)), inv);
        xf[kt][i] = u;
      }
  }
  const int pos = p.pos ? __ldcg(p.pos) + p.token : 0;

  TileWalker w;
  w.begin(p, u0, u1);
  int s, j0, t, stage = 0, buf = 0, ntop = 0;
  uint32_t phase = 0;
  // A timed-out wait only records the error and stops further waiting: the
  // control flow (and so every named barrier) stays identical in all threads.
  bool failed = false;
  while (w.next<T>(p, s, j0, t)) {
    float acc = 0.f;
#pragma unroll
    for (int kt = 0; kt < C::NKT; ++kt) {
      if (!failed && !mbar_wait(&full[stage], phase, p.err, 102)) failed = true;
      if (rr < t) {
        const uint4* wrow = reinterpret_cast<const uint4*>(ring + size_t(stage) * C::STAGE_ELEMS +
                                                           r * KT + part * C::KSEG);
        if constexpr (XS) {
          const uint4* xrow = reinterpret_cast<const uint4*>(xsm + kt * KT + part * C::KSEG);
#pragma unroll
          for (int i = 0; i < C::KPL; ++i) acc = dot8(wrow[lane + 32 * i], xrow[lane + 32 * i], acc);
        } else {
#pragma unroll
          for (int i = 0; i < C::KPL; ++i) acc = dot8(wrow[lane + 32 * i], xf[kt][i], acc);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == NSTAGE) {
        stage = 0;
        phase ^= 1;
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) partial[(buf * C::R + r) * C::WPR + part] = acc;
    named_sync(1, kConsumers);
    const Segment& sg = p.seg[s];
    if (sg.mode == EPI_TOPK) {
      if (ctid == 0) {
        for (int u = 0; u < t; ++u) {
          float a = 0.f, b = 0.f;
#pragma unroll
          for (int q = 0; q < C::WPR; ++q) {
            a += partial[(buf * C::R + u) * C::WPR + q];
            b += partial[(buf * C::R + T + u) * C::WPR + q];
          }
          const int64_t oa = unit_row(sg, j0 + u), ob = oa + sg.b_offset;
          const float la = rbf(a), lb = rbf(b);  // F.linear(...) is bf16, then .float()
          if (p.logits) {
            p.logits[oa] = la;
            p.logits[ob] = lb;
          }
          topk_insert(topv, topi, ntop, p.k, la, p.row_offset + oa);
          topk_insert(topv, topi, ntop, p.k, lb, p.row_offset + ob);
        }
      }
    } else if (ctid < t) {
      float a = 0.f, b = 0.f;
#pragma unroll
      for (int q = 0; q < C::WPR; ++q) {
        a += partial[(buf * C::R + ctid) * C::WPR + q];
        b += partial[(buf * C::R + T + ctid) * C::WPR + q];
      }
      gemv_epilogue(p, sg, j0 + ctid, a, b, pos);
    }
    buf ^= 1;
  }

  if (p.cand_values == nullptr) return;
  // ---------------- LM head: publish this CTA's top-k, last CTA merges
  if (ctid == 0) {
    for (int i = 0; i < p.k; ++i) {
      const bool have = i < ntop;
      p.cand_values[size_t(blockIdx.x) * p.k + i] = have ? topv[i] : -__int_as_float(0x7F800000);
      p.cand_indices[size_t(blockIdx.x) * p.k + i] = have ? topi[i] : INT64_MAX;
    }
    __threadfence();
    const unsigned int ticket = atomicAdd(p.ticket, 1u);
    red[8] = __int_as_float(ticket == unsigned(G - 1) ? 1 : 0);
  }
  named_sync(1, kConsumers);
  if (__float_as_int(red[8]) == 1 && warp == 0) {
    __threadfence();
    warp_select_topk(p.cand_values, p.cand_indices, G * p.k, p.k, p.out_values, p.out_indices);
    if (lane == 0) *p.ticket = 0u;
  }
}

}  // namespace cb

// ====================================================================== host
namespace cb {

int32_t* error_word();

template <int K, int KT, int T, int NSTAGE, bool XS = false>
static int run_gemv(const char* what, GemvParams& p, cudaStream_t stream) {
  using C = GemvCfg<K, KT, T, NSTAGE, XS>;
  auto kernel = gemv_kernel<K, KT, T, NSTAGE, XS>;
  int rc = configure_smem(what, kernel, C::SMEM);
  if (rc != kOk) return rc;
  p.total_units = 0;
  for (int i = 0; i < p.nseg; ++i) p.total_units += p.seg[i].units;
  if (p.total_units == 0) return kOk;
  p.err = error_word();
  return launch(what, kernel, dim3(sm_count()), dim3(kThreads), C::SMEM, stream, p);
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
  return run_gemv<4096, 4096, 2, 3>("cb_qkv_rope", p, static_cast<cudaStream_t>(stream));
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
  if (K == 4096) return run_gemv<4096, 4096, 2, 3>("cb_proj_residual", p, s);
  if (K == 14336) return run_gemv<14336, 7168, 1, 3, true>("cb_proj_residual", p, s);
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
  return run_gemv<4096, 4096, 2, 3>(what, p, static_cast<cudaStream_t>(stream));
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
  int rc = configure_smem("gemv", gemv_kernel<4096, 4096, 2, 3, false>,
                          GemvCfg<4096, 4096, 2, 3, false>::SMEM);
  if (rc == kOk)
    rc = configure_smem("gemv", gemv_kernel<14336, 7168, 1, 3, true>,
                        GemvCfg<14336, 7168, 1, 3, true>::SMEM);
  return rc;
}
}  // namespace cb

extern "C" int64_t cb_lm_head_workspace_bytes(int k) {
  // candidates: values [SMs*k] fp32, then indices [SMs*k] int64
  const int64_t n = int64_t(sm_count()) * k;
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
  const int64_t n = int64_t(sm_count()) * k;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.cand_values = reinterpret_cast<float*>(ws);
  p.cand_indices = reinterpret_cast<int64_t*>(ws + ((n * 4 + 15) / 16) * 16);
  p.ticket = ticket;
  p.out_values = out_values;
  p.out_indices = out_indices;
  return run_gemv<4096, 4096, 2, 3>("cb_lm_head_topk", p, static_cast<cudaStream_t>(stream));
}
