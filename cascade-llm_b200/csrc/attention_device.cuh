// Device-side building blocks of the split-KV GQA attention (flash-decoding)
// of attention.cu. Replaces
// layer_streaming/llama31.py:182-234 (`_repeat_kv` + SDPA): the 4 query heads
// of a KV head share one read of every K/V row.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace cb {

constexpr int kSub = 64;           // positions per sub-chunk
constexpr int kAttnWarps = 8;      // compute warps
constexpr int kAttnConsumers = kAttnWarps * 32;
constexpr int kHeadDim = 128;
constexpr int kGroup = 4;          // query heads per KV head
constexpr float kAttnScale = 0.08838834764831845f;  // 1/sqrt(128), SDPA's default

struct AttnParams {
  const uint16_t* q;         // [M][32][128]
  const uint16_t* k_cache;   // [8][cache_len][128]
  const uint16_t* v_cache;
  int64_t cache_len;
  const int32_t* pos;
  int M, splits, chunk;
  int kv_heads;              // KV heads of this rank (8 / tensor-parallel ranks)
  uint16_t* out;             // [M][kv_heads * 4 * 128]
  float* part_o;             // [M][kv_heads * 4][splits][128]
  float* part_ml;            // [M][kv_heads * 4][splits][2]
  unsigned int* tickets;     // [M][kv_heads]
  int* err;
  uint64_t* trace;           // per-CTA timeline (cb_set_trace) or null
  uint32_t trace_tag;
  unsigned int* heads_done;  // fused launches: count of merged (token, kv head) outputs, or null
  int min_chunk;             // least positions per split when chunk == 0 (0: kMinChunk)
  L2Stage stage;             // a later launch's weights staged into L2 (where: 1 start, 2 after the
                             // producer's last copy, 3 after the sub-chunk loop, 4 after the merge)
};

constexpr int kRowsPerWarp = kSub / kAttnWarps;  // 8 rows of a sub-chunk per warp
constexpr int kMergeBlock = 24;                    // splits merged per round trip

// Shared-memory scratch of the compute part: per-warp broadcast areas (p of
// the warp's 8 rows x 4 heads and alpha of 4 heads, each value stored twice
// as an f32x2 operand), per-warp softmax states and the merge staging. The
// cross-warp combine of o reuses the K ring.
struct AttnScratch {
  static constexpr size_t PW = 0;                                     // [8 warps][80] fp32
  static constexpr size_t WML = PW + kAttnWarps * 80 * 4;             // [8][4] m, [8][4] l
  static constexpr size_t MRG = WML + 2 * kAttnWarps * kGroup * 4;    // merge: w [4][24]; M, L, s [4]; flag
  static constexpr size_t BYTES = MRG + (kGroup * kMergeBlock + 3 * kGroup + 4) * 4;
};

// Positions per split: p.chunk, or (p.chunk == 0) sized on the device from
// the step's position: the least multiple of 64 positions, and at least
// kMinChunk, with which the launch's splits cover the longest context of the
// step. Short contexts leave the last splits empty rather than give every
// CTA a single sub-chunk (more partials to merge for the same bytes).
constexpr int64_t kMinChunk = 2 * kSub;
__device__ __forceinline__ int64_t attn_chunk(const AttnParams& p, int64_t pos0) {
  if (p.chunk > 0) return p.chunk;
  const int64_t longest = min(pos0 + p.M, p.cache_len);
  const int64_t per = (longest + p.splits - 1) / p.splits;
  return max(p.min_chunk > 0 ? int64_t(p.min_chunk) : kMinChunk, (per + kSub - 1) / kSub * kSub);
}

// Positions [start, stop) of split s for token m, and the sub-chunk count.
__device__ __forceinline__ int attn_range(const AttnParams& p, int s, int m, int64_t& pos0, int64_t& start,
                                          int64_t& stop) {
  pos0 = __ldcg(p.pos);
  int64_t visible = pos0 + m + 1;
  if (visible > p.cache_len) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, 201);
    visible = p.cache_len;
  }
  const int64_t chunk = attn_chunk(p, pos0);
  if (visible > int64_t(p.splits) * chunk && s == 0 && threadIdx.x == 0 && p.err)
    atomicExch(p.err, 204);  // too few splits for this position: the tail is left out
  start = int64_t(s) * chunk;
  stop = min(start + chunk, visible);
  return start < stop ? int((stop - start + kSub - 1) / kSub) : 0;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): each component is rounded as
// the scalar fma / mul would round it.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  return uint64_t(__float_as_uint(lo)) | (uint64_t(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// This lane's 4 dims of the 4 query heads of KV head g (token m), each value
// twice (qd[h][i] = {q, q}) to multiply two K rows at once.
__device__ __forceinline__ void attn_load_q(const AttnParams& p, int m, int g, uint64_t (&qd)[kGroup][4]) {
  const int lane = threadIdx.x & 31;
  const uint16_t* qrow = p.q + (int64_t(m) * p.kv_heads * kGroup + g * kGroup) * kHeadDim + 4 * lane;
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(qrow + h * kHeadDim));
    const float q4[4] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y)};
#pragma unroll
    for (int i = 0; i < 4; ++i) qd[h][i] = f2pack(q4[i], q4[i]);
  }
}

// Online softmax state of one warp: lane L tracks head L & 3 (m_run, l_run;
// the 8 lanes of a head hold the same values) and accumulates o[h][0..3] for
// dims 4L..4L+3 of all 4 heads, unnormalised, relative to m_run.
struct AttnWarpState {
  uint64_t o[kGroup][2];  // {dims 4L, 4L+1}, {4L+2, 4L+3} of each head
  float m_run, l_run;
};

__device__ __forceinline__ void attn_state_init(AttnWarpState& w) {
#pragma unroll
  for (int h = 0; h < kGroup; ++h) w.o[h][0] = w.o[h][1] = 0ull;
  w.m_run = -__int_as_float(0x7F800000);
  w.l_run = 0.f;
}

// Rows [8w, 8w + 8) of a sub-chunk (K and V rows in shared memory, `rows`
// valid) for warp w, with no synchronisation beyond the warp:
//   scores  each lane dots its 4 dims of the 4 heads with each of the 8 rows
//           (32 partial sums); a transposed butterfly (16+8+4+2+1 shuffles)
//           leaves lane L the full dot of row L >> 2, head L & 3;
//   softmax running max / sum per head over the 8 lanes of the head;
//   PV      p and the rescale factors go through the warp's 80-float area
//           (each stored twice); each lane accumulates its 4 dims of the 4
//           heads. Products and sums use f32x2 pairs (two K rows, or two
//           dims) in the same order as the scalar code.
__device__ __forceinline__ void attn_rows(const uint16_t* kst, const uint16_t* vst, int rows,
                                          const uint64_t (&qd)[kGroup][4], AttnWarpState& st, float* pw) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = warp * kRowsPerWarp;
  if (r0 >= rows) return;  // warp-uniform: no row of this warp in the sub-chunk
  float v[kRowsPerWarp * kGroup];
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; j += 2) {  // rows j, j + 1 as the two halves of each pair
    uint2 u = make_uint2(0u, 0u), w = make_uint2(0u, 0u);
    if (r0 + j < rows) u = *reinterpret_cast<const uint2*>(kst + (r0 + j) * kHeadDim + 4 * lane);
    if (r0 + j + 1 < rows) w = *reinterpret_cast<const uint2*>(kst + (r0 + j + 1) * kHeadDim + 4 * lane);
    const uint64_t k0 = f2pack(bf16lo(u.x), bf16lo(w.x)), k1 = f2pack(bf16hi(u.x), bf16hi(w.x));
    const uint64_t k2 = f2pack(bf16lo(u.y), bf16lo(w.y)), k3 = f2pack(bf16hi(u.y), bf16hi(w.y));
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      const uint64_t d = ffma2(qd[h][0], k0, ffma2(qd[h][1], k1, ffma2(qd[h][2], k2, fmul2(qd[h][3], k3))));
      v[j * kGroup + h] = f2lo(d);
      v[(j + 1) * kGroup + h] = f2hi(d);
    }
  }
  // level `half`: the lane whose bit `half` is set keeps the upper half of
  // its values and receives the partner's copy of it, the other the lower
#pragma unroll
  for (int half = 16; half >= 1; half >>= 1) {
    const bool hi = lane & half;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = hi ? v[i] : v[i + half];
      const float keep = hi ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, half);
    }
  }
  const float ninf = -__int_as_float(0x7F800000);
  const float s = r0 + (lane >> 2) < rows ? v[0] * kAttnScale : ninf;
  float mx = fmaxf(s, __shfl_xor_sync(0xFFFFFFFFu, s, 4));
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
  const float m_new = fmaxf(st.m_run, mx);  // finite: row r0 is valid
  const float p = expf(s - m_new);
  float ps = p + __shfl_xor_sync(0xFFFFFFFFu, p, 4);
  ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 8);
  ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 16);
  const float alpha = expf(st.m_run - m_new);  // 0 while m_run is -inf
  st.l_run = st.l_run * alpha + ps;
  st.m_run = m_new;
  // [row j][head h] at 2 (4j + h), alpha of head h at 64 + 2h, each twice
  *reinterpret_cast<float2*>(pw + 2 * lane) = make_float2(p, p);
  if (lane < kGroup) *reinterpret_cast<float2*>(pw + 64 + 2 * lane) = make_float2(alpha, alpha);
  __syncwarp();
  {
    const ulonglong2 a01 = *reinterpret_cast<const ulonglong2*>(pw + 64);
    const ulonglong2 a23 = *reinterpret_cast<const ulonglong2*>(pw + 68);
    const uint64_t a4[kGroup] = {a01.x, a01.y, a23.x, a23.y};
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      st.o[h][0] = fmul2(st.o[h][0], a4[h]);
      st.o[h][1] = fmul2(st.o[h][1], a4[h]);
    }
  }
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    if (r0 + j < rows) {  // warp-uniform; rows past the end may hold stale bytes
      const ulonglong2 p01 = *reinterpret_cast<const ulonglong2*>(pw + 8 * j);
      const ulonglong2 p23 = *reinterpret_cast<const ulonglong2*>(pw + 8 * j + 4);
      const uint2 u = *reinterpret_cast<const uint2*>(vst + (r0 + j) * kHeadDim + 4 * lane);
      const uint64_t v01 = f2pack(bf16lo(u.x), bf16hi(u.x)), v23 = f2pack(bf16lo(u.y), bf16hi(u.y));
      const uint64_t pp[kGroup] = {p01.x, p01.y, p23.x, p23.y};
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        st.o[h][0] = ffma2(pp[h], v01, st.o[h][0]);
        st.o[h][1] = ffma2(pp[h], v23, st.o[h][1]);
      }
    }
  }
  __syncwarp();  // pw is rewritten by the next batch
}

// Combine the 8 warps' states into this split's (m, l, o) per head, publish
// them, and let the last split of the (token, kv head) group to arrive
// (acquire-release ticket) merge all splits and write the bf16 output, then
// reset the ticket. pos0 = the step's first position (read at kernel start).
// `ring` (>= 16 KB of shared memory no longer read by any warp after
// the first barrier) stages the rescaled o of every warp.
template <class Sync>
static __device__ bool attn_publish(const AttnParams& p, int s, int g, int m, int64_t pos0,
                                    const AttnWarpState& st, uint8_t* scratch, float* ring, Sync sync) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const float ninf = -__int_as_float(0x7F800000);
  float* wm = reinterpret_cast<float*>(scratch + AttnScratch::WML);
  float* wl = wm + kAttnWarps * kGroup;
  if (lane < kGroup) {
    wm[warp * kGroup + lane] = st.m_run;
    wl[warp * kGroup + lane] = st.l_run;
  }
  sync();  // every warp is past its last row: the K ring is free
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    float mm = ninf;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, wm[w * kGroup + h]);
    const float mw = wm[warp * kGroup + h];
    const float f = mw == ninf ? 0.f : expf(mw - mm);
    *reinterpret_cast<float4*>(ring + (warp * kGroup + h) * kHeadDim + 4 * lane) =
        make_float4(f2lo(st.o[h][0]) * f, f2hi(st.o[h][0]) * f, f2lo(st.o[h][1]) * f, f2hi(st.o[h][1]) * f);
  }
  sync();
  for (int e = tid; e < kGroup * kHeadDim; e += kAttnConsumers) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) acc += ring[(w * kGroup + h) * kHeadDim + d];
    const int64_t row = (int64_t(m) * p.kv_heads * kGroup + g * kGroup + h) * p.splits + s;
    p.part_o[row * kHeadDim + d] = acc;
    if (d == 0) {
      float mm = ninf, ll = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, wm[w * kGroup + h]);
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = wm[w * kGroup + h];
        ll += mw == ninf ? 0.f : expf(mw - mm) * wl[w * kGroup + h];
      }
      *reinterpret_cast<float2*>(p.part_ml + row * 2) = make_float2(mm, ll);
    }
  }
  sync();
  float* mg = reinterpret_cast<float*>(scratch + AttnScratch::MRG);
  float* sm_w = mg;                               // [4][24] weights exp(m_s - M)
  float* st_M = sm_w + kGroup * kMergeBlock;      // [4] running maxima
  float* st_L = st_M + kGroup;                    // [4] running denominators
  float* st_s = st_L + kGroup;                    // [4] rescale of the previous blocks
  int* flag = reinterpret_cast<int*>(st_s + kGroup);
  if (tid == 0) {
    const unsigned int ticket = atom_add_acq_rel_gpu(&p.tickets[m * p.kv_heads + g], 1u);
    *flag = ticket == unsigned(p.splits - 1) ? 1 : 0;
  }
  sync();
  if (*flag == 0) return false;
  // Merge over the splits that hold keys for this token (a split that starts
  // past its last visible position has weight 0), kMergeBlock splits per
  // round trip: every (m, l) pair and every o value of the block is loaded
  // at once; thread t owns outputs t and t + 256 (head e / 128, dim e % 128).
  if (tid < kGroup) {
    st_M[tid] = ninf;
    st_L[tid] = 0.f;
  }
  const int64_t visible = min(pos0 + m + 1, p.cache_len);
  const int64_t chunk = attn_chunk(p, pos0);
  const int live = max(1, min(p.splits, int((visible + chunk - 1) / chunk)));
  const int64_t grp = int64_t(m) * p.kv_heads * kGroup + g * kGroup;  // first (token, head) row
  float acc[2] = {0.f, 0.f};
  const int h0 = tid / kHeadDim, h1 = (tid + kAttnConsumers) / kHeadDim, d0 = tid % kHeadDim;
  for (int base = 0; base < live; base += kMergeBlock) {
    const int nb = min(kMergeBlock, live - base);
    float ov[2][kMergeBlock];
#pragma unroll
    for (int j = 0; j < kMergeBlock; ++j) {
      if (j < nb) {
        ov[0][j] = __ldcg(p.part_o + ((grp + h0) * p.splits + base + j) * kHeadDim + d0);
        ov[1][j] = __ldcg(p.part_o + ((grp + h1) * p.splits + base + j) * kHeadDim + d0);
      }
    }
    // warp h, lane j: (m, l) of split base + j for head h, in flight with the o values
    float2 ml = make_float2(ninf, 0.f);
    if (warp < kGroup && lane < nb)
      ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + ((grp + warp) * p.splits + base + lane) * 2));
    sync();  // the previous block's weights have been used
    if (warp < kGroup) {  // warp h: new running max, weights, rescale of the previous blocks
      const float mold = st_M[warp], mnew = fmaxf(mold, warp_max(ml.x));
      const float w = ml.x == ninf ? 0.f : expf(ml.x - mnew);
      if (lane < nb) sm_w[warp * kMergeBlock + lane] = w;
      const float lsum = warp_sum(w * ml.y);
      if (lane == 0) {
        const float scale = mold == ninf ? 0.f : expf(mold - mnew);
        st_L[warp] = st_L[warp] * scale + lsum;
        st_M[warp] = mnew;
        st_s[warp] = scale;
      }
    }
    sync();
    float a = acc[0] * st_s[h0], b = acc[1] * st_s[h1];
#pragma unroll
    for (int j = 0; j < kMergeBlock; ++j) {
      if (j < nb) {
        a = fmaf(sm_w[h0 * kMergeBlock + j], ov[0][j], a);
        b = fmaf(sm_w[h1 * kMergeBlock + j], ov[1][j], b);
      }
    }
    acc[0] = a;
    acc[1] = b;
  }
  uint16_t* out = p.out + int64_t(m) * p.kv_heads * kGroup * kHeadDim + g * kGroup * kHeadDim;
  out[h0 * kHeadDim + d0] = f2bf(acc[0] / st_L[h0]);
  out[h1 * kHeadDim + d0] = f2bf(acc[1] / st_L[h1]);
  if (tid == 0) p.tickets[m * p.kv_heads + g] = 0u;
  if (p.heads_done) {
    // publish the (token, kv head)'s output to the CTAs that consume it in
    // this launch (release after the barrier covers every thread's stores)
    sync();
    if (tid == 0) red_add_release_gpu(p.heads_done, 1u);
  }
  return tid == 0;
}

constexpr int kAttnStages = 3;
__device__ __forceinline__ int attn_ncta() { return int(gridDim.x * gridDim.y * gridDim.z); }
constexpr int kAttnThreads = kAttnConsumers + 32;  // + one producer warp

struct AttnSmem {
  static constexpr size_t STAGE = size_t(kSub) * kHeadDim * 2;  // one of K or V
  static constexpr size_t K_OFF = 0;
  static constexpr size_t V_OFF = K_OFF + kAttnStages * STAGE;
  static constexpr size_t BAR_OFF = V_OFF + kAttnStages * STAGE;   // full, empty
  static constexpr size_t SCR_OFF = BAR_OFF + 2 * kAttnStages * 8;
  static constexpr size_t BYTES = SCR_OFF + AttnScratch::BYTES;
  static_assert(kAttnStages * STAGE >= size_t(kAttnWarps) * kGroup * kHeadDim * 4,
                "the K ring stages the cross-warp combine");
  static_assert(SCR_OFF % 16 == 0, "scratch alignment");
};

struct ConsumerSync {
  __device__ void operator()() const { named_sync(1, kAttnConsumers); }
};

// Splits of one (token, KV head) merged inside a thread-block cluster (one
// CTA per split, the cluster = the head's splits, at most 16): each CTA
// combines its warps into (m, l) per head and o[4][128] in its own shared
// memory; after a cluster barrier CTA r merges outputs [r * 512 / S, (r+1) *
// 512 / S) by reading every split's values through distributed shared
// memory, and a second barrier keeps each CTA's values alive until all have
// read them. No global partials, no ticket, no second kernel-wide round trip.
// The arithmetic is that of attn_publish's merge (same maxima, weights, warp
// sum of the denominators and fma order over the splits), so the outputs are
// bit-identical to the global-memory merge.
constexpr int kClusterMaxSplits = 16;
static __device__ void attn_publish_cluster(const AttnParams& p, int s, int g, int m, const AttnWarpState* st,
                                            uint8_t* scratch, float* ring) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const float ninf = -__int_as_float(0x7F800000);
  float* wm = reinterpret_cast<float*>(scratch + AttnScratch::WML);
  float* wl = wm + kAttnWarps * kGroup;
  // this split's combined values, published to the cluster: o [4][128], then (m, l) [4][2]
  float* cl_o = ring + kAttnWarps * kGroup * kHeadDim;
  float* cl_ml = cl_o + kGroup * kHeadDim;
  if (st) {  // the consumer warps (the producer warp passes null)
    if (lane < kGroup) {
      wm[warp * kGroup + lane] = st->m_run;
      wl[warp * kGroup + lane] = st->l_run;
    }
    named_sync(1, kAttnConsumers);
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      float mm = ninf;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, wm[w * kGroup + h]);
      const float mw = wm[warp * kGroup + h];
      const float f = mw == ninf ? 0.f : expf(mw - mm);
      *reinterpret_cast<float4*>(ring + (warp * kGroup + h) * kHeadDim + 4 * lane) =
          make_float4(f2lo(st->o[h][0]) * f, f2hi(st->o[h][0]) * f, f2lo(st->o[h][1]) * f, f2hi(st->o[h][1]) * f);
    }
    named_sync(1, kAttnConsumers);
    for (int e = tid; e < kGroup * kHeadDim; e += kAttnConsumers) {
      const int h = e / kHeadDim, d = e % kHeadDim;
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) acc += ring[(w * kGroup + h) * kHeadDim + d];
      cl_o[e] = acc;
      if (d == 0) {
        float mm = ninf, ll = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, wm[w * kGroup + h]);
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
          const float mw = wm[w * kGroup + h];
          ll += mw == ninf ? 0.f : expf(mw - mm) * wl[w * kGroup + h];
        }
        cl_ml[2 * h] = mm;
        cl_ml[2 * h + 1] = ll;
      }
    }
  }
  cluster.sync();  // every split's (m, l, o) is visible to the cluster
  const int S = p.splits;
  float* mg = reinterpret_cast<float*>(scratch + AttnScratch::MRG);
  float* sm_w = mg;                           // [4][16] weights exp(m_j - M)
  float* st_L = sm_w + kGroup * kClusterMaxSplits;  // [4] denominators
  if (warp < kGroup) {  // warp h: maximum, weights and denominator of head h over the splits
    float2 ml = make_float2(ninf, 0.f);
    if (lane < S) {
      const float* r = cluster.map_shared_rank(cl_ml, lane);
      ml = make_float2(r[2 * warp], r[2 * warp + 1]);
    }
    const float mnew = warp_max(ml.x);
    const float w = ml.x == ninf ? 0.f : expf(ml.x - mnew);
    if (lane < S) sm_w[warp * kClusterMaxSplits + lane] = w;
    const float lsum = warp_sum(w * ml.y);
    if (lane == 0) st_L[warp] = lsum;
  }
  __syncthreads();
  const int per = (kGroup * kHeadDim + S - 1) / S;
  for (int i = tid; i < per; i += int(blockDim.x)) {
    const int e = s * per + i;
    if (e >= kGroup * kHeadDim) break;
    const int h = e / kHeadDim;
    float a = 0.f;
    for (int j = 0; j < S; ++j) a = fmaf(sm_w[h * kClusterMaxSplits + j], cluster.map_shared_rank(cl_o, j)[e], a);
    p.out[int64_t(m) * p.kv_heads * kGroup * kHeadDim + g * kGroup * kHeadDim + e] = f2bf(a / st_L[h]);
  }
  cluster.sync();  // no CTA leaves while others read its shared memory
}

// One CTA of the split-KV attention, (split s, kv head g, token m): a
// producer warp streams its positions in 64-position sub-chunks through a
// 3-stage cp.async.bulk ring; rows of the history (< the step's first
// position) are fetched before griddepcontrol.wait, rows written by this
// step's QKV kernel after it. `cta` is the CTA's index in the launch trace.
// Returns true in thread 0 of the CTA that merged the (token, kv head).
template <bool kCluster = false>
static __device__ bool attention_cta(const AttnParams& p, int s, int g, int m, unsigned cta, uint8_t* smem) {
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem + AttnSmem::K_OFF);
  uint16_t* vs = reinterpret_cast<uint16_t*>(smem + AttnSmem::V_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + AttnSmem::BAR_OFF);
  uint64_t* empty = full + kAttnStages;
  uint8_t* scratch = smem + AttnSmem::SCR_OFF;

  const uint64_t t0 = trace_now(p.trace);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  if (p.stage.where == 1 && warp == 0) l2_stage_issue(p.stage, int(cta), attn_ncta(), lane, 32);
  int64_t pos0, start, stop;
  const int nsub = attn_range(p, s, m, pos0, start, stop);

  if (tid == 0) {
    for (int i = 0; i < kAttnStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kAttnWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kAttnWarps) {
    // ---------------- producer
    if (lane == 0) {
      bool waited = false;
      int stage = 0;
      uint32_t phase = 0;
      const uint16_t* kbase = p.k_cache + int64_t(g) * p.cache_len * kHeadDim;
      const uint16_t* vbase = p.v_cache + int64_t(g) * p.cache_len * kHeadDim;
      for (int i = 0; i < nsub; ++i) {
        const int64_t t0 = start + int64_t(i) * kSub;
        const int rows = int(min(int64_t(kSub), stop - t0));
        if (!waited && t0 + kSub > pos0) {  // touches rows written by this step
          grid_dep_wait();
          waited = true;
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, 202)) break;
        const uint32_t bytes = uint32_t(rows) * kHeadDim * 2;
        mbar_arrive_expect_tx(&full[stage], 2 * bytes);
        bulk_g2s(ks + size_t(stage) * kSub * kHeadDim, kbase + t0 * kHeadDim, bytes, &full[stage]);
        bulk_g2s(vs + size_t(stage) * kSub * kHeadDim, vbase + t0 * kHeadDim, bytes, &full[stage]);
        if (++stage == kAttnStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (p.stage.where == 2) l2_stage_issue(p.stage, int(cta), attn_ncta(), 0, 1);
    }
    if constexpr (!kCluster) return false;
    // cluster merge: the producer warp joins the cluster barriers
    __syncwarp();
    attn_publish_cluster(p, s, g, m, nullptr, scratch, reinterpret_cast<float*>(ks));
    return false;
  }

  // ---------------- consumers
  // q comes from the QKV kernel. No early griddepcontrol.launch_dependents:
  // the next kernel (o_proj) starts when this grid exits, since its CTAs
  // would otherwise stream weights during this kernel's latency-bound
  // publish/merge and slow it (decode step 3.37 -> 3.12 ms measured).
  grid_dep_wait();
  const uint64_t t1 = trace_now(p.trace);
  uint64_t qd[kGroup][4];
  attn_load_q(p, m, g, qd);
  AttnWarpState ws;
  attn_state_init(ws);
  float* pw = reinterpret_cast<float*>(scratch + AttnScratch::PW) + warp * 80;
  int stage = 0;
  uint32_t phase = 0;
  bool failed = false;  // a timed-out wait records the error; control flow is unchanged
  __shared__ uint64_t trace_sub[2];  // launch trace: first and last sub-chunk in shared memory
  if (tid == 0) trace_sub[0] = trace_sub[1] = 0;
  for (int i = 0; i < nsub; ++i) {
    const int64_t t0 = start + int64_t(i) * kSub;
    const int rows = int(min(int64_t(kSub), stop - t0));
    if (!failed && !mbar_wait(&full[stage], phase, p.err, 203)) failed = true;
    if (p.trace && tid == 0) {
      trace_sub[1] = globaltimer_ns();
      if (i == 0) trace_sub[0] = trace_sub[1];
    }
    attn_rows(ks + size_t(stage) * kSub * kHeadDim, vs + size_t(stage) * kSub * kHeadDim, rows, qd, ws, pw);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == kAttnStages) {
      stage = 0;
      phase ^= 1;
    }
  }
  const uint64_t t2 = trace_now(p.trace);
  if (p.stage.where == 3 && warp == 0) l2_stage_issue(p.stage, int(cta), attn_ncta(), lane, 32);
  bool merged;
  if constexpr (kCluster) {
    attn_publish_cluster(p, s, g, m, &ws, scratch, reinterpret_cast<float*>(ks));
    merged = false;
  } else {
    merged = attn_publish(p, s, g, m, pos0, ws, scratch, reinterpret_cast<float*>(ks), ConsumerSync());
  }
  if (p.stage.where == 4 && warp == 0) l2_stage_issue(p.stage, int(cta), attn_ncta(), lane, 32);
  if (tid == 0) trace_commit(p.trace, p.trace_tag, cta, t0, t1, t2, trace_sub[0], trace_sub[1]);
  return merged;
}

}  // namespace cb
