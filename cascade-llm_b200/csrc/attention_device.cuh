// Device-side building blocks of the split-KV GQA attention (flash-decoding),
// shared by the stand-alone attention kernel (attention.cu) and the
// persistent decode-step kernel (decode_step.cu). Replaces
// layer_streaming/llama31.py:182-234 (`_repeat_kv` + SDPA): the 4 query heads
// of a KV head share one read of every K/V row.
#pragma once

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
};

// Shared-memory scratch of the compute part: scores [2][4][64], softmax
// state (alpha [2][4], running max [4], running sum [4]) and a merge area.
struct AttnScratch {
  static constexpr size_t SC = 0;
  static constexpr size_t ST = SC + 2 * kGroup * kSub * 4;
  static constexpr size_t RED = ST + 16 * 4;
  static constexpr size_t RED_FLOATS = 4 * kGroup * kHeadDim > 2 * kGroup * 256 + 3 * kGroup
                                           ? 4 * kGroup * kHeadDim
                                           : 2 * kGroup * 256 + 3 * kGroup;
  static constexpr size_t BYTES = RED + RED_FLOATS * 4;
};

// Positions [start, stop) of split s for token m, and the sub-chunk count.
__device__ __forceinline__ int attn_range(const AttnParams& p, int s, int m, int64_t& pos0, int64_t& start,
                                          int64_t& stop) {
  pos0 = __ldcg(p.pos);
  int64_t visible = pos0 + m + 1;
  if (visible > p.cache_len) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, 201);
    visible = p.cache_len;
  }
  start = int64_t(s) * p.chunk;
  stop = min(start + int64_t(p.chunk), visible);
  return start < stop ? int((stop - start + kSub - 1) / kSub) : 0;
}

// This lane's 4 dims of the 4 query heads of KV head g (token m).
__device__ __forceinline__ void attn_load_q(const AttnParams& p, int m, int g, float (&q)[kGroup][4]) {
  const int lane = threadIdx.x & 31;
  const uint16_t* qrow = p.q + (int64_t(m) * p.kv_heads * kGroup + g * kGroup) * kHeadDim + 4 * lane;
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(qrow + h * kHeadDim));
    q[h][0] = bf16lo(u.x);
    q[h][1] = bf16hi(u.x);
    q[h][2] = bf16lo(u.y);
    q[h][3] = bf16hi(u.y);
  }
}

__device__ __forceinline__ void attn_reset(float* st) {
  if (threadIdx.x < kGroup) {
    st[8 + threadIdx.x] = -__int_as_float(0x7F800000);  // running max
    st[12 + threadIdx.x] = 0.f;                         // running sum
  }
}

// One sub-chunk (rows <= 64 positions of K and V in shared memory) of the
// online softmax: scores q.k (lanes split the 128 dims; a transposed shuffle
// tree leaves head (lane>>3)'s sum in 8 lanes), a running max/sum per head in
// fp32, then PV with 4 position groups x 64 dim pairs accumulating into
// o[head][2]. `sync` is the barrier over the 256 compute threads; `i` is the
// sub-chunk counter (selects the double-buffered score area).
template <class Sync>
__device__ __forceinline__ void attn_subchunk(const uint16_t* kst, const uint16_t* vst, int rows, int i,
                                              const float (&q)[kGroup][4], float (&o)[kGroup][2],
                                              uint8_t* scratch, Sync sync) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  float* scb = reinterpret_cast<float*>(scratch + AttnScratch::SC) + (i & 1) * kGroup * kSub;
  float* st = reinterpret_cast<float*>(scratch + AttnScratch::ST);
  float* alpha_s = st;
  float* m_run = st + 8;
  float* l_run = st + 12;
#pragma unroll 2
  for (int j = 0; j < 8; ++j) {
    const int t = warp * 8 + j;
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
    if (t < rows) {
      const uint2 u = *reinterpret_cast<const uint2*>(kst + t * kHeadDim + 4 * lane);
      const float k0 = bf16lo(u.x), k1 = bf16hi(u.x), k2 = bf16lo(u.y), k3 = bf16hi(u.y);
      d0 = fmaf(q[0][0], k0, fmaf(q[0][1], k1, fmaf(q[0][2], k2, q[0][3] * k3)));
      d1 = fmaf(q[1][0], k0, fmaf(q[1][1], k1, fmaf(q[1][2], k2, q[1][3] * k3)));
      d2 = fmaf(q[2][0], k0, fmaf(q[2][1], k1, fmaf(q[2][2], k2, q[2][3] * k3)));
      d3 = fmaf(q[3][0], k0, fmaf(q[3][1], k1, fmaf(q[3][2], k2, q[3][3] * k3)));
    }
    const bool up = lane & 16;
    float keep0 = up ? d2 : d0, keep1 = up ? d3 : d1;
    keep0 += __shfl_xor_sync(0xFFFFFFFFu, up ? d0 : d2, 16);
    keep1 += __shfl_xor_sync(0xFFFFFFFFu, up ? d1 : d3, 16);
    const bool b3 = lane & 8;
    float keep = b3 ? keep1 : keep0;
    keep += __shfl_xor_sync(0xFFFFFFFFu, b3 ? keep0 : keep1, 8);
    keep += __shfl_xor_sync(0xFFFFFFFFu, keep, 4);
    keep += __shfl_xor_sync(0xFFFFFFFFu, keep, 2);
    keep += __shfl_xor_sync(0xFFFFFFFFu, keep, 1);
    if ((lane & 7) == 0) scb[(lane >> 3) * kSub + t] = t < rows ? keep * kAttnScale : -__int_as_float(0x7F800000);
  }
  sync();
  if (warp < kGroup) {
    const float s0 = scb[warp * kSub + lane], s1 = scb[warp * kSub + 32 + lane];
    const float mx = warp_max(fmaxf(s0, s1));
    const float mold = m_run[warp];
    const float mnew = fmaxf(mold, mx);
    const float p0 = expf(s0 - mnew), p1 = expf(s1 - mnew);
    scb[warp * kSub + lane] = p0;
    scb[warp * kSub + 32 + lane] = p1;
    const float sum = warp_sum(p0 + p1);
    if (lane == 0) {
      const float a = expf(mold - mnew);
      alpha_s[(i & 1) * kGroup + warp] = a;
      l_run[warp] = l_run[warp] * a + sum;
      m_run[warp] = mnew;
    }
  }
  sync();
  const int pg = tid >> 6, dp = tid & 63;
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    const float a = alpha_s[(i & 1) * kGroup + h];
    o[h][0] *= a;
    o[h][1] *= a;
  }
  for (int t = pg; t < rows; t += 4) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(vst + t * kHeadDim + 2 * dp);
    const float v0 = bf16lo(u), v1 = bf16hi(u);
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      const float pr = scb[h * kSub + t];
      o[h][0] = fmaf(pr, v0, o[h][0]);
      o[h][1] = fmaf(pr, v1, o[h][1]);
    }
  }
}

// Publish this split's (m, l, o) for the 4 heads of KV head g (token m);
// the last split of the group to arrive (atomic ticket) merges all splits
// and writes the bf16 output, then resets the ticket.
template <class Sync>
static __device__ void attn_publish(const AttnParams& p, int s, int g, int m, const float (&o)[kGroup][2],
                             uint8_t* scratch, Sync sync) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int pg = tid >> 6, dp = tid & 63;
  float* st = reinterpret_cast<float*>(scratch + AttnScratch::ST);
  const float* m_run = st + 8;
  const float* l_run = st + 12;
  float* red = reinterpret_cast<float*>(scratch + AttnScratch::RED);
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    red[(pg * kGroup + h) * kHeadDim + 2 * dp] = o[h][0];
    red[(pg * kGroup + h) * kHeadDim + 2 * dp + 1] = o[h][1];
  }
  sync();
  for (int e = tid; e < kGroup * kHeadDim; e += kAttnConsumers) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    const float v = red[(0 * kGroup + h) * kHeadDim + d] + red[(1 * kGroup + h) * kHeadDim + d] +
                    red[(2 * kGroup + h) * kHeadDim + d] + red[(3 * kGroup + h) * kHeadDim + d];
    const int64_t row = (int64_t(m) * p.kv_heads * kGroup + g * kGroup + h) * p.splits + s;
    p.part_o[row * kHeadDim + d] = v;
    if (d == 0) {
      p.part_ml[row * 2] = m_run[h];
      p.part_ml[row * 2 + 1] = l_run[h];
    }
  }
  __threadfence();
  sync();
  if (tid == 0) {
    const unsigned int ticket = atomicAdd(&p.tickets[m * p.kv_heads + g], 1u);
    red[0] = __int_as_float(ticket == unsigned(p.splits - 1) ? 1 : 0);
  }
  sync();
  const bool last = __float_as_int(red[0]) == 1;
  sync();  // everyone has read the flag before the merge reuses red
  if (!last) return;
  __threadfence();
  // Merge: per-split (max, sum) of the 4 heads staged in blocks of 256 splits
  // (loads issued in parallel), then each thread reduces its 2 outputs over
  // the splits with independent, unrolled loads.
  float* st_m = red;                         // [4][256] split maxima
  float* st_w = red + kGroup * 256;          // [4][256] weights exp(m_s - M)
  float* st_l = red + 2 * kGroup * 256;      // [4] combined denominators
  float* st_M = st_l + kGroup;               // [4] combined maxima
  float* st_s = st_M + kGroup;               // [4] rescale factor of this block
  if (tid < kGroup) {
    st_M[tid] = -__int_as_float(0x7F800000);
    st_l[tid] = 0.f;
  }
  float acc[2] = {0.f, 0.f};
  const int e0 = tid, e1 = tid + kAttnConsumers;  // outputs (h, d) = e / 128, e % 128
  // splits that start past this token's last visible position hold no keys
  // (weight 0): only the first `live` take part
  const int64_t visible = min(int64_t(__ldcg(p.pos)) + m + 1, p.cache_len);
  const int live = max(1, min(p.splits, int((visible + p.chunk - 1) / p.chunk)));
  for (int base = 0; base < live; base += 256) {
    const int nb = min(256, live - base);
    sync();
    for (int i = tid; i < kGroup * nb; i += kAttnConsumers) {
      const int h = i / nb, j = i % nb;
      st_m[h * 256 + j] =
          __ldcg(p.part_ml + ((int64_t(m) * p.kv_heads * kGroup + g * kGroup + h) * p.splits + base + j) * 2);
    }
    sync();
    if (warp < kGroup) {  // warp h: new running max and rescale of the previous blocks
      float mx = -__int_as_float(0x7F800000);
      for (int j = lane; j < nb; j += 32) mx = fmaxf(mx, st_m[warp * 256 + j]);
      mx = warp_max(mx);
      const float mold = st_M[warp], mnew = fmaxf(mold, mx);
      float lsum = 0.f;
      for (int j = lane; j < nb; j += 32) {
        const float mj = st_m[warp * 256 + j];
        const float w = mj == -__int_as_float(0x7F800000) ? 0.f : expf(mj - mnew);
        st_w[warp * 256 + j] = w;
        lsum = fmaf(
            w, __ldcg(p.part_ml + ((int64_t(m) * p.kv_heads * kGroup + g * kGroup + warp) * p.splits + base + j) * 2 + 1),
            lsum);
      }
      lsum = warp_sum(lsum);
      if (lane == 0) {
        const float scale = mold == -__int_as_float(0x7F800000) ? 0.f : expf(mold - mnew);
        st_l[warp] = st_l[warp] * scale + lsum;
        st_M[warp] = mnew;
        st_s[warp] = scale;
      }
    }
    sync();
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int e = q ? e1 : e0;
      const int h = e / kHeadDim, d = e % kHeadDim;
      acc[q] *= st_s[h];
      const float* po = p.part_o + ((int64_t(m) * p.kv_heads * kGroup + g * kGroup + h) * p.splits + base) * kHeadDim + d;
      float sum = 0.f;
#pragma unroll 8
      for (int j = 0; j < nb; ++j) sum = fmaf(st_w[h * 256 + j], __ldcg(po + int64_t(j) * kHeadDim), sum);
      acc[q] += sum;
    }
  }
  sync();
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int e = q ? e1 : e0;
    const int h = e / kHeadDim, d = e % kHeadDim;
    p.out[int64_t(m) * p.kv_heads * kGroup * kHeadDim + (g * kGroup + h) * kHeadDim + d] = f2bf(acc[q] / st_l[h]);
  }
  if (tid == 0) p.tickets[m * p.kv_heads + g] = 0u;
}

}  // namespace cb
