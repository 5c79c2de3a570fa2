// Device-side building blocks of the weight-streaming GEMV (BF16 weights,
// fp32 accumulate) of the projection kernels (gemv.cu).
#pragma once

#include "common.cuh"

namespace cb {

enum EpiMode : int {
  EPI_STORE = 0,     // out[oA] = bf16(a), out[oB] = bf16(b)
  EPI_RESIDUAL = 1,  // out[o] = bf16(aux[o] + bf16(acc))
  EPI_ROPE = 2,      // RoPE on the (d, d+64) pair, store
  EPI_SILU = 3,      // out[o] = bf16(silu(bf16(acc)))
  EPI_MUL = 4,       // out[o] = bf16(aux[o] * bf16(acc))
  EPI_SWIGLU = 5,    // out[j] = bf16(bf16(silu(bf16(a))) * bf16(b))
  EPI_TOPK = 6,      // fp32 logits of bf16(acc) -> running top-k
  EPI_PARTIAL = 7,   // outf[o] = acc (fp32, unrounded: a tensor-parallel partial sum)
  EPI_EXCHANGE = 8,  // acc pushed to every rank; out[o] = bf16(aux[o] + bf16(sum over ranks))
};

constexpr int kThreads = 256;
constexpr int kTopkMax = 64;
constexpr size_t kMaxSmem = 226 * 1024;  // dynamic; the kernels also hold a little static shared memory

// Tensor-parallel exchange buffer of one rank (device memory that every rank
// maps; the same layout on all ranks). Every entry is a tagged 64-bit word
// {payload, sequence number of the exchange} (common.cuh). Two parities
// (slot & 1) alternate, so a rank can push the next exchange while a peer
// still reads the last one.
//   data   [2][kXchgMaxWorld][kXchgWidth]   fp32 projection partials, by source rank
//   cand_v [2][kXchgMaxWorld * kTopkMax]    top-k candidate values (fp32), rank-major, k per rank
//   cand_i [2][kXchgMaxWorld * kTopkMax]    their global row ids (uint32)
constexpr int kXchgMaxWorld = 8;
constexpr int kXchgWidth = 4096;
constexpr size_t kXchgData = 0;
constexpr size_t kXchgCandV = kXchgData + size_t(2) * kXchgMaxWorld * kXchgWidth * 8;
constexpr size_t kXchgCandI = kXchgCandV + size_t(2) * kXchgMaxWorld * 64 * 8;
constexpr size_t kXchgBytes = kXchgCandI + size_t(2) * kXchgMaxWorld * 64 * 8;
constexpr uint64_t kXchgWaitNs = 2000000000ull;  // default limit: a peer 2 s late is reported, not awaited

__device__ __forceinline__ uint64_t* xchg_data(uint8_t* base, int par, int rank) {
  return reinterpret_cast<uint64_t*>(base + kXchgData) + (par * kXchgMaxWorld + rank) * kXchgWidth;
}
__device__ __forceinline__ uint64_t* xchg_cand_v(uint8_t* base, int par) {
  return reinterpret_cast<uint64_t*>(base + kXchgCandV) + par * kXchgMaxWorld * 64;
}
__device__ __forceinline__ uint64_t* xchg_cand_i(uint8_t* base, int par) {
  return reinterpret_cast<uint64_t*>(base + kXchgCandI) + par * kXchgMaxWorld * 64;
}
__device__ __forceinline__ uint32_t xchg_seq(const int32_t* epoch, int slots, int slot) {
  return uint32_t(__ldcg(epoch)) * uint32_t(slots) + uint32_t(slot) + 1u;
}

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
  float* outf;             // fp32 output (EPI_PARTIAL)
  // int8 weights (W8 kernels): the bases above are byte addresses of rows of
  // K int8 values, and every row has an fp32 scale (weight = int8 x scale),
  // indexed like the weight rows
  const float* a_scale;
  const float* b_scale;
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
  // tensor-parallel exchange (EPI_EXCHANGE, and the LM head's candidate
  // gather when world > 0): exchange buffer of every rank, this rank's own at
  // [rank]; sequence number of this launch = epoch * slots + slot + 1
  uint8_t* xchg[kXchgMaxWorld];
  int rank, world;
  int slot, slots;
  const int32_t* epoch;    // device step counter, advanced once per step
  uint64_t wait_ns;        // how long a peer's word is awaited before the launch gives up
  uint64_t* trace;         // per-CTA timeline (cb_set_trace) or null
  uint32_t trace_tag;
  L2Stage stage;           // a later launch's weights staged into L2 (where: 1 start, 2 after the wait, 3 end)
};

__device__ __forceinline__ int64_t unit_row(const Segment& s, int j) {
  return int64_t(j / s.group) * s.group_stride + (j % s.group);
}

__device__ __forceinline__ bool ranks_before(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

// ------------------------------------------------------------ exact top-k
// Order: larger value first, then smaller row id (torch.topk leaves ties
// unspecified; this order is the engine's documented tie rule). Values are
// compared as order-preserving 32-bit keys; key 0 marks a removed or missing
// entry (no finite value or infinity maps to it). Row ids fit 31 bits (the
// host checks row_offset + rows <= 2^31).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// Warp-cooperative top-k of entries [lo, hi) of `keys` (shared memory) with
// distinct ids id_of(c): round r takes the largest key and, among equal
// keys, the smallest id (two warp reductions), removes it from `keys` and
// hands it to emit(r, key, id) in lane 0 (key 0 once the range is exhausted).
template <class IdOf, class Emit>
__device__ __forceinline__ void warp_topk(uint32_t* keys, IdOf id_of, int lo, int hi, int k, Emit emit) {
  const int lane = threadIdx.x & 31;
  for (int r = 0; r < k; ++r) {
    uint32_t bk = 0u, bi = 0xFFFFFFFFu;
    int bp = -1;
    for (int c = lo + lane; c < hi; c += 32) {
      const uint32_t kk = keys[c];
      if (kk == 0u || kk < bk) continue;
      const uint32_t ii = id_of(c);
      if (kk > bk || ii < bi) {
        bk = kk;
        bi = ii;
        bp = c;
      }
    }
    const uint32_t wk = __reduce_max_sync(0xFFFFFFFFu, bk);
    const uint32_t wi = __reduce_min_sync(0xFFFFFFFFu, bk == wk ? bi : 0xFFFFFFFFu);
    if (wk != 0u && bk == wk && bi == wi) keys[bp] = 0u;  // exactly one lane owns it
    if (lane == 0) emit(r, wk, wi);
    __syncwarp();
  }
}

// (key, id) as one word that ranks by plain unsigned comparison: larger key
// first, then smaller id. 0 is an empty entry (key 0).
__device__ __forceinline__ uint64_t rank_word(uint32_t key, uint32_t id) {
  return key ? (uint64_t(key) << 32) | uint32_t(~id) : 0ull;
}
__device__ __forceinline__ uint64_t max_word(uint64_t a, uint64_t b) { return a > b ? a : b; }

// Warp top-k of the rank words each lane holds in registers (at most NPL per
// lane, distinct ids). Round r: each lane's best word by a pairwise maximum
// tree (no dependent compare chain), the warp's by two 32-bit reductions
// (key, then the complemented id among lanes holding that key), then the one
// entry equal to the winner is cleared; emit(r, key, id) in lane 0 (key 0
// once every entry is taken). Branch-free: 3-9x fewer cycles than a
// per-entry compare-and-branch scan (0.6 us for 128 entries and k = 10).
template <int NPL, class Emit>
__device__ __forceinline__ void warp_select(uint64_t (&v)[NPL], int k, Emit emit) {
  const int lane = threadIdx.x & 31;
  for (int r = 0; r < k; ++r) {
    uint64_t m[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) m[j] = v[j];
#pragma unroll
    for (int s = 1; s < NPL; s *= 2)
#pragma unroll
      for (int j = 0; j + s < NPL; j += 2 * s) m[j] = max_word(m[j], m[j + s]);
    const uint32_t hk = uint32_t(m[0] >> 32);
    const uint32_t wk = __reduce_max_sync(0xFFFFFFFFu, hk);
    const uint32_t wl = __reduce_max_sync(0xFFFFFFFFu, hk == wk ? uint32_t(m[0]) : 0u);
    const uint64_t w = (uint64_t(wk) << 32) | wl;
#pragma unroll
    for (int j = 0; j < NPL; ++j) v[j] = v[j] == w ? 0ull : v[j];  // ids are distinct: one entry
    if (lane == 0) emit(r, wk, ~wl);
  }
}

// Register form of warp_topk for ranges of at most 32 * NPL entries.
template <int NPL, class IdOf, class Emit>
__device__ __forceinline__ void warp_topk_regs(const uint32_t* keys, IdOf id_of, int lo, int hi, int k, Emit emit) {
  const int lane = threadIdx.x & 31;
  uint64_t v[NPL];
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int c = lo + lane + 32 * j;
    v[j] = c < hi ? rank_word(keys[c], id_of(c)) : 0ull;
  }
  warp_select<NPL>(v, k, emit);
}

// Final stage of a block selection, run by warp 0: the k best of the 8k
// entries staged by the warps (keys [8][k], then ids [8][k]) to out_v / out_i
// (missing entries: -inf, INT64_MAX). Not inlined, so that the LM head's
// last-CTA merge runs the same instructions as every CTA's own top-k just
// before it instead of code that no warp of the SM has fetched yet.
static __device__ __noinline__ void stage_topk(uint32_t* stage, int k, float* out_v, int64_t* out_i) {
  constexpr int W = kThreads / 32;
  const uint32_t* ids = stage + W * k;
  auto to_out = [out_v, out_i](int r, uint32_t key, uint32_t id) {
    out_v[r] = key ? key_value(key) : -__int_as_float(0x7F800000);
    out_i[r] = key ? int64_t(id) : INT64_MAX;
  };
  auto stage_id = [ids](int c) { return ids[c]; };
  if (W * k <= 64)
    warp_topk_regs<2>(stage, stage_id, 0, W * k, k, to_out);
  else if (W * k <= 128)
    warp_topk_regs<4>(stage, stage_id, 0, W * k, k, to_out);
  else
    warp_topk(stage, stage_id, 0, W * k, k, to_out);
}

// Exact top-k of n entries (keys in shared memory, ids by id_of) by the whole
// CTA: each of the 8 warps selects the top-k of its eighth into `stage`
// (8k keys, then 8k ids), then warp 0 selects the k best of those and writes
// values / int64 ids to out_v / out_i (missing entries: -inf, INT64_MAX).
template <class IdOf>
static __device__ void block_topk(uint32_t* keys, IdOf id_of, int n, int k, uint32_t* stage, float* out_v,
                                  int64_t* out_i) {
  const int warp = threadIdx.x >> 5;
  constexpr int W = kThreads / 32;
  uint32_t* st_key = stage + warp * k;
  uint32_t* st_id = stage + W * k + warp * k;
  auto to_stage = [st_key, st_id](int r, uint32_t key, uint32_t id) {
    st_key[r] = key;
    st_id[r] = id;
  };
  const int lo = int(int64_t(n) * warp / W), hi = int(int64_t(n) * (warp + 1) / W);
  if (hi - lo <= 64)
    warp_topk_regs<2>(keys, id_of, lo, hi, k, to_stage);
  else if (hi - lo <= 128)
    warp_topk_regs<4>(keys, id_of, lo, hi, k, to_stage);
  else
    warp_topk(keys, id_of, lo, hi, k, to_stage);
  __syncthreads();
  if (warp == 0) stage_topk(stage, k, out_v, out_i);
}

// Reference selection over candidate lists in global memory by one warp,
// k rounds of a full scan: the fallback of block_merge_topk when more than
// kMergeCap candidates tie at the threshold.
static __device__ void warp_select_topk(const float* vals, const int64_t* idx, int n, int k,
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

// Exact top-k of G per-CTA candidate lists (k each, in global memory), by the
// whole CTA. Up to kMergeRegs candidates per thread (the LM head's 296 lists
// of 10), every candidate is loaded in one L2 round trip into registers and
// each warp selects the top-k of its share (warp_select), warp 0 the top-k of
// those. Larger sets: the k-th best of the union is at least the largest
// per-list k-th value, so only candidates at or above that threshold can
// qualify: one pass finds the threshold, a second copies the survivors (keys
// and ids) to shared memory, and block_topk selects among them. `scratch`
// holds kMergeCap keys, kMergeCap ids and the 8k-entry stage (12 KB).
// (Bf16 logits tie often, so the threshold pass kept 760-1000 of 2960
// candidates of the decode LM head, close to the kMergeCap above which the
// one-warp scan runs: 13 us per merge, against 7 us for the register path.)
constexpr int kMergeCap = 1024;
constexpr int kMergeRegs = 12;
constexpr size_t kTopkScratchBytes = size_t(kMergeCap) * 8 + size_t(kThreads / 32) * kTopkMax * 8;
static __device__ void block_merge_topk(const float* vals, const int64_t* idx, int G, int k, float* out_v,
                                 int64_t* out_i, float* red, uint32_t* scratch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (G * k <= kMergeRegs * kThreads) {
    // candidates were written by other CTAs: read through L2, every load
    // issued before the first is used (in-bounds indices, masked after), so
    // they share one round trip (a load-use per candidate measured 6.7 us)
    const int n = G * k;
    float x[kMergeRegs];
    long long ix[kMergeRegs];
#pragma unroll
    for (int j = 0; j < kMergeRegs; ++j) {
      const int c = min(tid + j * kThreads, n - 1);
      x[j] = __ldcg(vals + c);
      ix[j] = __ldcg(reinterpret_cast<const long long*>(idx) + c);
    }
    uint64_t v[kMergeRegs];
#pragma unroll
    for (int j = 0; j < kMergeRegs; ++j)
      v[j] = tid + j * kThreads < n && ix[j] != INT64_MAX ? rank_word(order_key(x[j]), uint32_t(ix[j])) : 0ull;
    uint32_t* st_key = scratch;  // [8][k] keys, then [8][k] ids
    uint32_t* st_id = scratch + (kThreads / 32) * k;
    warp_select<kMergeRegs>(v, k, [st_key, st_id, warp, k](int r, uint32_t key, uint32_t id) {
      st_key[warp * k + r] = key;
      st_id[warp * k + r] = id;
    });
    __syncthreads();
    if (warp == 0) stage_topk(scratch, k, out_v, out_i);
    return;
  }
  uint32_t thr = 0u;
  for (int c = tid; c < G; c += blockDim.x) thr = max(thr, order_key(__ldcg(vals + size_t(c) * k + (k - 1))));
  thr = __reduce_max_sync(0xFFFFFFFFu, thr);
  __syncthreads();
  uint32_t* wred = reinterpret_cast<uint32_t*>(red);
  if (lane == 0) wred[warp] = thr;
  int* count = reinterpret_cast<int*>(red + 14);
  if (tid == 0) *count = 0;
  __syncthreads();
  thr = wred[0];
  for (int q = 1; q < int(blockDim.x >> 5); ++q) thr = max(thr, wred[q]);
  uint32_t* keys = scratch;
  uint32_t* ids = scratch + kMergeCap;
  uint32_t* stage = scratch + 2 * kMergeCap;
  const int n = G * k;
  // eight candidates per thread in flight at a time (one L2 round trip per
  // group instead of one per candidate)
  constexpr int B = 8;
  for (int base = tid; base < n; base += B * int(blockDim.x)) {
    float v[B];
    long long ix[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int c = base + j * int(blockDim.x);
      v[j] = c < n ? __ldcg(vals + c) : -__int_as_float(0x7F800000);
      ix[j] = c < n ? __ldcg(reinterpret_cast<const long long*>(idx) + c) : INT64_MAX;
    }
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const uint32_t key = order_key(v[j]);
      if (key >= thr && ix[j] != INT64_MAX) {
        const int slot = atomicAdd(count, 1);
        if (slot < kMergeCap) {
          keys[slot] = key;
          ids[slot] = uint32_t(ix[j]);
        }
      }
    }
  }
  __syncthreads();
  const int kept = *count;
  if (kept <= kMergeCap) {
    block_topk(keys, [ids](int c) { return ids[c]; }, kept, k, stage, out_v, out_i);
  } else if (warp == 0) {  // pathological ties: scan every candidate
    warp_select_topk(vals, idx, n, k, out_v, out_i);
  }
}

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

// pre: aux_a / aux_b (the bf16 residual or gate values of rows A / B) and
// freq (the RoPE inverse frequency) were loaded earlier by this thread.
static __device__ void gemv_epilogue(const GemvParams& p, const Segment& sg, int j, float a, float b,
                              int pos, bool pre, float aux_a, float aux_b, float freq) {
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
      sg.out[oa] = f2bf((pre ? aux_a : bf16f(__ldcg(sg.aux + oa))) + rbf(a));
      sg.out[ob] = f2bf((pre ? aux_b : bf16f(__ldcg(sg.aux + ob))) + rbf(b));
      break;
    case EPI_ROPE: {
      // transformers modeling_llama.py:124-168: cos/sin of (inv_freq * pos)
      // in fp32, cast to bf16; q*cos + rotate_half(q)*sin in bf16.
      uint16_t ra, rb;
      rope_pair(a, b, pre ? freq : __ldg(p.inv_freq + j % sg.group), pos, ra, rb);
      sg.out[oa] = ra;
      sg.out[ob] = rb;
      break;
    }
    case EPI_SILU:
      sg.out[oa] = f2bf(silu_bf16(rbf(a)));
      sg.out[ob] = f2bf(silu_bf16(rbf(b)));
      break;
    case EPI_MUL:
      sg.out[oa] = f2bf((pre ? aux_a : bf16f(__ldcg(sg.aux + oa))) * rbf(a));
      sg.out[ob] = f2bf((pre ? aux_b : bf16f(__ldcg(sg.aux + ob))) * rbf(b));
      break;
    case EPI_SWIGLU:
      sg.out[oa] = f2bf(silu_bf16(rbf(a)) * rbf(b));
      break;
    case EPI_PARTIAL:
      sg.outf[oa] = a;
      sg.outf[ob] = b;
      break;
    case EPI_EXCHANGE: {
      // Push this rank's partials of rows oa / ob into every rank's buffer
      // (peer stores over NVLink), then sum every rank's partials of the same
      // rows in rank order, so all ranks compute the same bits, and add the
      // residual: x + F.linear(...) rounds the projection to bf16 once.
      const int par = p.slot & 1;
      const uint32_t seq = xchg_seq(p.epoch, p.slots, p.slot);
#pragma unroll
      for (int q = 0; q < kXchgMaxWorld; ++q) {
        if (q < p.world) {
          uint64_t* d = xchg_data(p.xchg[q], par, p.rank);
          st_tagged(d + oa, tag_word(__float_as_uint(a), seq));
          st_tagged(d + ob, tag_word(__float_as_uint(b), seq));
        }
      }
      float sa = 0.f, sb = 0.f;
      bool late = false;
#pragma unroll
      for (int q = 0; q < kXchgMaxWorld; ++q) {
        if (q < p.world) {
          const uint64_t* d = xchg_data(p.xchg[p.rank], par, q);
          sa += __uint_as_float(wait_tagged(d + oa, seq, p.wait_ns, &late));
          sb += __uint_as_float(wait_tagged(d + ob, seq, p.wait_ns, &late));
        }
      }
      if (late && p.err) atomicExch(p.err, 120);
      sg.out[oa] = f2bf((pre ? aux_a : bf16f(__ldcg(sg.aux + oa))) + rbf(sa));
      sg.out[ob] = f2bf((pre ? aux_b : bf16f(__ldcg(sg.aux + ob))) + rbf(sb));
      break;
    }
    default:
      break;
  }
}

// DEPTH scales the loads in flight per lane (units per batch); the kernels
// run DEPTH 1 at 2 CTAs per SM (16 warps, <= 128 registers), which measured
// faster than DEPTH 2 at 1 CTA per SM with the same bytes in flight. W8:
// int8 weights, 8-byte loads at the same element positions as the bf16
// kernel's 16-byte loads, twice the units per batch (the same bytes and
// registers in flight).
template <int K, int DEPTH = 1, bool W8 = false>
struct GemvShape {
  static constexpr int WARPS = kThreads / 32;
  static constexpr int GROUPS = K / 256;        // 512-byte lane groups per row
  // WK warps split K (the largest of 8, 4, 2, 1 dividing GROUPS); the CTA's
  // WARPS / WK warp rows work on different units at the same time. The int8
  // K = 4096 kernel splits K over 4 warps: a unit then carries twice the bytes
  // per lane, halving the per-unit addressing and reductions per byte
  // (gate+up 31.3 -> 29.3 us, measured)
  static constexpr int WK = (W8 && K == 4096) ? 4
                            : GROUPS % 8 == 0 ? 8 : GROUPS % 4 == 0 ? 4 : GROUPS % 2 == 0 ? 2 : 1;
  static constexpr int UL = WARPS / WK;          // units in flight side by side
  // K-part and unit lane of warp w (compile-time 0 lane when UL == 1)
  static __device__ __forceinline__ int kpart(unsigned w) { return UL == 1 ? int(w) : int(w % WK); }
  static __device__ __forceinline__ int ulane(unsigned w) { return UL == 1 ? 0 : int(w / WK); }
  static constexpr int KS = K / WK;              // K-slice of each warp
  static constexpr int CPL = KS / 256;           // 16-byte chunks per lane per row slice
  static constexpr int UB = (W8 ? 2 : 1) * DEPTH * ((16 / (2 * CPL)) > 0 ? 16 / (2 * CPL) : 1);  // units per warp per batch
  // long K-slices keep the activation slice in shared memory (7 chunks = 28
  // registers would otherwise crowd out the weight batch); one region per warp
  static constexpr bool XSMEM = CPL > 4;
  static constexpr size_t RED = 0;                                         // [16] fp32 (norm partials, flag)
  static constexpr size_t XS = RED + 16 * 4;                               // [WARPS][KS] bf16 when XSMEM
  static constexpr size_t SMEM = XS + (XSMEM ? size_t(WARPS) * KS * 2 : 0);  // + per-unit partials (+ logits)
  static_assert(K % 256 == 0 && KS % 256 == 0, "K must be whole 512-byte lane groups");
};

template <bool W8>
struct WeightChunk {
  using T = uint4;  // 8 bf16 weights
};
template <>
struct WeightChunk<true> {
  using T = uint2;  // 8 int8 weights
};

template <int K, int DEPTH = 1, bool W8 = false>
struct GemvRegs {
  typename WeightChunk<W8>::T w[GemvShape<K, DEPTH, W8>::UB][2][GemvShape<K, DEPTH, W8>::CPL];
};

__device__ __forceinline__ void gemv_locate(const GemvParams& p, int u, int& seg, int& j) {
  seg = 0;
  j = u;
  while (seg + 1 < p.nseg && j >= p.seg[seg].units) {
    j -= p.seg[seg].units;
    ++seg;
  }
}

// Weight rows of unit u for this lane: row A and row B of the pair (element
// kbase of each row: a bf16 address, or W8 the int8 byte address).
template <int K, int DEPTH = 1, bool W8 = false>
__device__ __forceinline__ void gemv_rows(const GemvParams& p, int u, const uint16_t*& ra,
                                          const uint16_t*& rb) {
  using S = GemvShape<K, DEPTH, W8>;
  int seg, j;
  gemv_locate(p, u, seg, j);
  const Segment& sg = p.seg[seg];
  const int64_t row = int64_t(j / sg.group) * sg.group_stride + (j % sg.group);
  const int kbase = S::kpart(threadIdx.x >> 5) * S::KS + (threadIdx.x & 31) * 8;
  if constexpr (W8) {
    ra = reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(sg.a_base) + row * K + kbase);
    rb = reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(sg.b_base) + row * K + kbase);
  } else {
    ra = sg.a_base + row * K + kbase;
    rb = sg.b_base + row * K + kbase;
  }
}

// Chunk c (elements c * 256 .. of the lane's row slice) of a weight row.
template <bool W8>
__device__ __forceinline__ typename WeightChunk<W8>::T ld_chunk(const uint16_t* row, int c) {
  if constexpr (W8)
    return ld_stream8(reinterpret_cast<const uint8_t*>(row) + c * 256);
  else
    return ld_stream(row + c * 256);
}

template <int K, int DEPTH = 1, bool W8 = false>
__device__ __forceinline__ void gemv_load_batch(const GemvParams& p, int ub, int u1, GemvRegs<K, DEPTH, W8>& r) {
  using S = GemvShape<K, DEPTH, W8>;
  const int ul = S::ulane(threadIdx.x >> 5);
#pragma unroll
  for (int i = 0; i < S::UB; ++i) {
    const int u = ub + i * S::UL + ul;
    if (u < u1) {
      const uint16_t *ra, *rb;
      gemv_rows<K, DEPTH, W8>(p, u, ra, rb);
#pragma unroll
      for (int c = 0; c < S::CPL; ++c) {
        r.w[i][0][c] = ld_chunk<W8>(ra, c);
        r.w[i][1][c] = ld_chunk<W8>(rb, c);
      }
    }
  }
}

// Half `half` (registers [half * UB/2, (half + 1) * UB/2)) of the batch whose
// first unit is ub.
template <int K, int DEPTH = 1, bool W8 = false>
__device__ __forceinline__ void gemv_load_half(const GemvParams& p, int ub, int u1, GemvRegs<K, DEPTH, W8>& r,
                                               int half) {
  using S = GemvShape<K, DEPTH, W8>;
  constexpr int H = S::UB / 2;
  const int ul = S::ulane(threadIdx.x >> 5);
#pragma unroll
  for (int i = 0; i < S::UB; ++i) {
    const int u = ub + i * S::UL + ul;
    if ((i >= half * H && i < (half + 1) * H) && u < u1) {
      const uint16_t *ra, *rb;
      gemv_rows<K, DEPTH, W8>(p, u, ra, rb);
#pragma unroll
      for (int c = 0; c < S::CPL; ++c) {
        r.w[i][0][c] = ld_chunk<W8>(ra, c);
        r.w[i][1][c] = ld_chunk<W8>(rb, c);
      }
    }
  }
}

__device__ __forceinline__ void gemv_cta_units(const GemvParams& p, int cta, int ncta, int& u0, int& u1) {
  u0 = int(int64_t(p.total_units) * cta / ncta);
  u1 = int(int64_t(p.total_units) * (cta + 1) / ncta);
}

// Issue the first batch of this CTA's weight loads. Weights never depend on
// earlier work, so this runs before the dependency wait / grid barrier.
template <int K, int DEPTH = 1, bool W8 = false>
__device__ __forceinline__ void gemv_prefetch(const GemvParams& p, int cta, int ncta, GemvRegs<K, DEPTH, W8>& r) {
  int u0, u1;
  gemv_cta_units(p, cta, ncta, u0, u1);
  gemv_load_batch<K, DEPTH, W8>(p, u0, u1, r);
}

// CTA-cooperative split-K GEMV over this CTA's contiguous range of units
// (row pairs). Each of the 8 warps streams its own 1/8 of K for EVERY unit
// of the range (UB units, 2*UB*CPL 128-bit loads per lane, in flight per
// batch), so all warps carry the same load until the end. Per unit each warp
// reduces its two partial dots with shuffles into shared memory; after ONE
// barrier the epilogues of all units run in parallel, one thread per unit.
// The activation slice of a warp stays in registers. `r` holds the first
// batch issued by gemv_prefetch. Requires the activation row to be complete.
template <int K, int DEPTH = 1, bool W8 = false>
static __device__ void gemv_run(const GemvParams& p, uint8_t* smem, int cta, int ncta, GemvRegs<K, DEPTH, W8>& r,
                                uint64_t* t_loop = nullptr) {
  using S = GemvShape<K, DEPTH, W8>;
  float* red = reinterpret_cast<float*>(smem + S::RED);
  float* part = reinterpret_cast<float*>(smem + S::SMEM);  // [units][2][WARPS]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  int u0, u1;
  gemv_cta_units(p, cta, ncta, u0, u1);
  const int units = u1 - u0;
  float* lrow = part + size_t(units) * 2 * S::WK;  // EPI_TOPK: this CTA's logits
  const int kp = S::kpart(warp), ul = S::ulane(warp);  // K-part and unit lane of this warp
  const int kbase = kp * S::KS + lane * 8;

  // this warp's activation slice: registers, or (XSMEM) its own region of
  // shared memory, written and read by the same warp only. In register form
  // the slice (and its RMSNorm weights) is loaded before the norm's
  // reduction, so both loads share one round trip.
  uint4 xr[S::XSMEM ? 1 : S::CPL];
  uint4 nw[S::XSMEM ? 1 : S::CPL];
  if constexpr (!S::XSMEM) {
#pragma unroll
    for (int c = 0; c < S::CPL; ++c) {
      xr[c] = ld_cg_u4(p.x + kbase + c * 256);
      if (p.norm_w) nw[c] = __ldg(reinterpret_cast<const uint4*>(p.norm_w + kbase + c * 256));
    }
  }
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
  // The epilogue operands of this thread's first unit (and the position) are
  // loaded here, in the same round trip as the activations, so the epilogue
  // after the main loop needs no further load.
  const int pos = p.pos ? __ldcg(p.pos) + p.token : 0;
  bool pre = false;
  float pre_a = 0.f, pre_b = 0.f, pre_f = 0.f;
  float sc_a = 1.f, sc_b = 1.f;  // W8: the row scales of this thread's first unit
  if (tid < units) {
    int seg, j;
    gemv_locate(p, u0 + tid, seg, j);
    const Segment& sg = p.seg[seg];
    if constexpr (W8) {
      sc_a = __ldg(sg.a_scale + unit_row(sg, j));
      sc_b = __ldg(sg.b_scale + unit_row(sg, j));
    }
    if (sg.mode == EPI_RESIDUAL || sg.mode == EPI_MUL || sg.mode == EPI_EXCHANGE) {
      const int64_t oa = int64_t(j / sg.group) * sg.head_stride + (j % sg.group);  // no position stride
      pre_a = bf16f(__ldcg(sg.aux + oa));
      pre_b = bf16f(__ldcg(sg.aux + oa + sg.b_offset));
      pre = true;
    } else if (sg.mode == EPI_ROPE) {
      pre_f = __ldg(p.inv_freq + j % sg.group);
      pre = true;
    }
  }
  uint4* xw = reinterpret_cast<uint4*>(smem + S::XS) + warp * (S::KS / 8) + lane;  // this warp's region
  if constexpr (S::XSMEM) {
#pragma unroll
    for (int c = 0; c < S::CPL; ++c) {
      uint4 v = ld_cg_u4(p.x + kbase + c * 256);
      if (p.norm_w) v = normalize8(v, __ldg(reinterpret_cast<const uint4*>(p.norm_w + kbase + c * 256)), inv);
      xw[c * 32] = v;
    }
    __syncwarp();
  } else if (p.norm_w) {
#pragma unroll
    for (int c = 0; c < S::CPL; ++c) xr[c] = normalize8(xr[c], nw[c], inv);
  }

  // dot products of one batch held in registers
  // dot products of registers [i0, i1) of the batch whose first unit is ub
  auto consume = [&](const GemvRegs<K, DEPTH, W8>& rr, int ub, int i0, int i1) {
#pragma unroll
    for (int i = 0; i < S::UB; ++i) {
      const int u = ub + i * S::UL + ul;
      if (i >= i0 && i < i1 && u < u1) {
        float a = 0.f, b = 0.f;
        if constexpr (W8) {
          uint64_t a2 = 0ull, b2 = 0ull;  // {even, odd} element sums
#pragma unroll
          for (int c = 0; c < S::CPL; ++c) {
            const uint4 xv = S::XSMEM ? xw[c * 32] : xr[S::XSMEM ? 0 : c];
            a2 = dot8_i8x2(rr.w[i][0][c], xv, a2);
            b2 = dot8_i8x2(rr.w[i][1][c], xv, b2);
          }
          a = f2sum(a2);
          b = f2sum(b2);
        } else {
#pragma unroll
          for (int c = 0; c < S::CPL; ++c) {
            const uint4 xv = S::XSMEM ? xw[c * 32] : xr[S::XSMEM ? 0 : c];
            a = dot8(rr.w[i][0][c], xv, a);
            b = dot8(rr.w[i][1][c], xv, b);
          }
        }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
          part[((u - u0) * 2 + 0) * S::WK + kp] = a;
          part[((u - u0) * 2 + 1) * S::WK + kp] = b;
        }
      }
    }
  };
  constexpr int STEP = S::UB * S::UL;  // units per batch of the CTA
  if constexpr (S::UB % 2 == 0) {
    // Two half-batches in flight: the registers of a batch are two halves,
    // and as soon as one half is consumed the loads of the half one batch
    // ahead go into it, so each lane keeps loads outstanding instead of
    // waiting for a whole batch after consuming the previous one.
    constexpr int H = S::UB / 2;
    for (int ub = u0; ub < u1; ub += STEP) {
      consume(r, ub, 0, H);
      if (ub + STEP < u1) gemv_load_half<K, DEPTH, W8>(p, ub + STEP, u1, r, 0);
      consume(r, ub, H, S::UB);
      if (ub + STEP < u1) gemv_load_half<K, DEPTH, W8>(p, ub + STEP, u1, r, 1);
    }
  } else {
    for (int ub = u0; ub < u1; ub += STEP) {
      if (ub != u0) gemv_load_batch<K, DEPTH, W8>(p, ub, u1, r);
      consume(r, ub, 0, S::UB);
    }
  }
  __syncthreads();
  if (t_loop && tid == 0) *t_loop = trace_now(p.trace);

  for (int i = tid; i < units; i += kThreads) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int q = 0; q < S::WK; ++q) {
      a += part[(i * 2 + 0) * S::WK + q];
      b += part[(i * 2 + 1) * S::WK + q];
    }
    int seg, j;
    gemv_locate(p, u0 + i, seg, j);
    const Segment& sg = p.seg[seg];
    if constexpr (W8) {  // int8 rows: dot of the integers times the row scale
      const int64_t row = unit_row(sg, j);
      a *= i == tid ? sc_a : __ldg(sg.a_scale + row);
      b *= i == tid ? sc_b : __ldg(sg.b_scale + row);
    }
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
      gemv_epilogue(p, sg, j, a, b, pos, pre && i == tid, pre_a, pre_b, pre_f);
    }
  }

  if (p.cand_values == nullptr) return;
  // ---------------- LM head: this CTA's exact top-k, then the last CTA merges
  __syncthreads();
  uint32_t* lkey = reinterpret_cast<uint32_t*>(lrow);  // the logits, as order keys in place
  for (int i = tid; i < 2 * units; i += kThreads) lkey[i] = order_key(lrow[i]);
  __syncthreads();
  {
    // entry i < units is row A of unit u0 + i, entry units + i its row B:
    // every B row (j + N/2) follows every A row, so entry order is id order
    const uint32_t a0 = uint32_t(p.row_offset + u0);
    const uint32_t b0 = uint32_t(p.row_offset + p.seg[0].b_offset + u0);
    const int na = units;
    block_topk(lkey, [a0, b0, na](int c) { return c < na ? a0 + uint32_t(c) : b0 + uint32_t(c - na); },
               2 * units, p.k, lkey + 2 * units, p.cand_values + size_t(cta) * p.k,
               p.cand_indices + size_t(cta) * p.k);
  }
  __syncthreads();
  if (tid == 0) {
    if (t_loop) t_loop[1] = trace_now(p.trace);
    // acq_rel: publishes this CTA's candidates (written before the barrier)
    // and, for the last CTA, orders its reads after everyone's
    const unsigned int ticket = atom_add_acq_rel_gpu(p.ticket, 1u);
    red[15] = __int_as_float(ticket == unsigned(ncta - 1) ? 1 : 0);
    if (t_loop) t_loop[2] = trace_now(p.trace);
  }
  __syncthreads();
  if (__float_as_int(red[15]) != 1) return;
  block_merge_topk(p.cand_values, p.cand_indices, ncta, p.k, p.out_values, p.out_indices, red,
                   reinterpret_cast<uint32_t*>(lrow));
  if (tid == 0) *p.ticket = 0u;
  if (!p.world) return;
  // ---------------- vocabulary-sharded LM head: push this rank's k
  // candidates (global row ids) into every rank's buffer, gather all ranks'
  // candidates into shared memory and select the global top-k.
  __syncthreads();  // this rank's top-k is in out_values / out_indices
  const int par = p.slot & 1;
  const int k = p.k;
  const uint32_t seq = xchg_seq(p.epoch, p.slots, p.slot);
  for (int e = tid; e < p.world * k; e += kThreads) {
    const int q = e / k, i = e % k;
    const float v = __ldcg(p.out_values + i);
    const uint32_t row = uint32_t(__ldcg(reinterpret_cast<const long long*>(p.out_indices) + i));
    st_tagged(xchg_cand_v(p.xchg[q], par) + p.rank * k + i, tag_word(__float_as_uint(v), seq));
    st_tagged(xchg_cand_i(p.xchg[q], par) + p.rank * k + i, tag_word(row, seq));
  }
  uint32_t* keys = reinterpret_cast<uint32_t*>(lrow);  // gathered keys, ids, then the stage
  uint32_t* ids = keys + kMergeCap;
  bool late = false;
  uint8_t* own = p.xchg[p.rank];
  for (int e = tid; e < p.world * k; e += kThreads) {
    keys[e] = order_key(__uint_as_float(wait_tagged(xchg_cand_v(own, par) + e, seq, p.wait_ns, &late)));
    ids[e] = wait_tagged(xchg_cand_i(own, par) + e, seq, p.wait_ns, &late);
  }
  if (late && p.err) atomicExch(p.err, 121);
  __syncthreads();  // also: every thread has read out_values / out_indices above before they are rewritten
  block_topk(keys, [ids](int c) { return ids[c]; }, p.world * k, k, keys + 2 * kMergeCap, p.out_values,
             p.out_indices);
}

// Host-side parameter builders (gemv.cu).
int finish_params(GemvParams& p);
int build_qkv_params(GemvParams& p, const void* x, const void* norm_w, float eps, const void* wq,
                     const void* wk, const void* wv, const float* inv_freq, const int32_t* position,
                     int token, void* q_out, void* k_cache, void* v_cache, int64_t cache_len, int q_heads,
                     int kv_heads, int wbytes = 2, const float* sq = nullptr, const float* sk = nullptr,
                     const float* sv = nullptr);
int build_residual_params(GemvParams& p, const void* x, int K, const void* w, int N, const void* residual,
                          void* out, int wbytes = 2, const float* scale = nullptr);
int build_gate_up_params(GemvParams& p, const char* what, const void* x, const void* norm_w, float eps,
                         const void* w_gate, const void* w_up, int N, int mode, void* out, const void* aux,
                         int wbytes = 2, const float* s_gate = nullptr, const float* s_up = nullptr);
int gemv_grid_size();

}  // namespace cb
