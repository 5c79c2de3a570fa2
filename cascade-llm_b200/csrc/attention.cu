// Split-KV GQA attention (flash-decoding) for sm_100a.
//
// Replaces layer_streaming/llama31.py:182-234: `_repeat_kv` (a 4x copy of
// K/V) + F.scaled_dot_product_attention. Here the 4 query heads of a KV head
// share ONE read of every K/V row: a CTA owns (split s, kv head g, token m)
// and streams its positions [s*chunk, s*chunk + chunk) in 64-position
// sub-chunks through a 3-stage cp.async.bulk ring. Per sub-chunk:
//   scores  q.k for 4 heads (lanes split the 128 dims; a transposed shuffle
//           tree leaves one head's sum per 8 lanes), scaled by 1/sqrt(128);
//   softmax online (running max / sum per head, fp32);
//   PV      4 position groups x 64 dim pairs accumulate 4 heads each.
// Each CTA writes (m, l, o[128]) per head; the last CTA of a (token, kv head)
// group (atomic ticket) merges the splits and writes the bf16 output.
//
// Causality: token m of a step starting at position P0 sees [0, P0 + m].
// Rows of the history (< P0) are fetched before griddepcontrol.wait: they were
// written by earlier steps. Rows >= P0 were written by this step's QKV
// kernel and are fetched only after the wait.
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "cascade_b200.h"

namespace cb {

int32_t* error_word();

constexpr int kSub = 64;                 // positions per sub-chunk
constexpr int kAttnStages = 3;
constexpr int kAttnWarps = 8;
constexpr int kAttnConsumers = kAttnWarps * 32;
constexpr int kAttnThreads = kAttnConsumers + 32;
constexpr int kHeadDim = 128;
constexpr int kGroup = 4;                // query heads per KV head

struct AttnParams {
  const uint16_t* q;         // [M][32][128]
  const uint16_t* k_cache;   // [8][cache_len][128]
  const uint16_t* v_cache;
  int64_t cache_len;
  const int32_t* pos;
  int M, splits, chunk;
  uint16_t* out;             // [M][4096]
  float* part_o;             // [M][32][splits][128]
  float* part_ml;            // [M][32][splits][2]
  unsigned int* tickets;     // [M][8]
  int* err;
};

struct AttnSmem {
  static constexpr size_t STAGE = size_t(kSub) * kHeadDim * 2;  // one of K or V
  static constexpr size_t K_OFF = 0;
  static constexpr size_t V_OFF = K_OFF + kAttnStages * STAGE;
  static constexpr size_t BAR_OFF = V_OFF + kAttnStages * STAGE;         // full, empty
  static constexpr size_t SC_OFF = BAR_OFF + 2 * kAttnStages * 8;       // [2][4][64] fp32
  static constexpr size_t ST_OFF = SC_OFF + 2 * kGroup * kSub * 4;      // alpha[2][4], m[4], l[4]
  static constexpr size_t RED_OFF = ST_OFF + 16 * 4;                    // o merge / split merge
  static constexpr size_t RED_FLOATS = 4 * kGroup * kHeadDim > 2 * kGroup * 256 + 3 * kGroup
                                           ? 4 * kGroup * kHeadDim
                                           : 2 * kGroup * 256 + 3 * kGroup;
  static constexpr size_t BYTES = RED_OFF + RED_FLOATS * 4;
};

__global__ void __launch_bounds__(kAttnThreads, 2) attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem + AttnSmem::K_OFF);
  uint16_t* vs = reinterpret_cast<uint16_t*>(smem + AttnSmem::V_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + AttnSmem::BAR_OFF);
  uint64_t* empty = full + kAttnStages;
  float* sc = reinterpret_cast<float*>(smem + AttnSmem::SC_OFF);
  float* st = reinterpret_cast<float*>(smem + AttnSmem::ST_OFF);
  float* alpha_s = st;          // [2][4]
  float* m_run = st + 8;        // [4]
  float* l_run = st + 12;       // [4]
  float* red = reinterpret_cast<float*>(smem + AttnSmem::RED_OFF);

  const int s = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;

  // The position counter was written at the end of an earlier step.
  int64_t pos0 = __ldcg(p.pos);
  int64_t visible = pos0 + m + 1;
  if (visible > p.cache_len) {
    if (tid == 0 && p.err) atomicExch(p.err, 201);
    visible = p.cache_len;
  }
  const int64_t start = int64_t(s) * p.chunk;
  const int64_t stop = min(start + int64_t(p.chunk), visible);
  const int nsub = start < stop ? int((stop - start + kSub - 1) / kSub) : 0;

  if (tid == 0) {
    for (int i = 0; i < kAttnStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kAttnWarps);
    }
    fence_mbar_init();
  }
  if (tid < kGroup) {
    m_run[tid] = -__int_as_float(0x7F800000);
    l_run[tid] = 0.f;
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
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, 202)) return;
        const uint32_t bytes = uint32_t(rows) * kHeadDim * 2;
        mbar_arrive_expect_tx(&full[stage], 2 * bytes);
        bulk_g2s(ks + size_t(stage) * kSub * kHeadDim, kbase + t0 * kHeadDim, bytes, &full[stage]);
        bulk_g2s(vs + size_t(stage) * kSub * kHeadDim, vbase + t0 * kHeadDim, bytes, &full[stage]);
        if (++stage == kAttnStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;
  }

  // ---------------- consumers
  grid_dep_wait();  // q comes from the QKV kernel
  if (tid == 0) grid_dep_launch();
  const float scale = 0.08838834764831845f;  // 1/sqrt(128), SDPA's default
  float q[kGroup][4];
  {
    const uint16_t* qrow = p.q + (int64_t(m) * 32 + g * kGroup) * kHeadDim + 4 * lane;
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(qrow + h * kHeadDim));
      q[h][0] = bf16lo(u.x);
      q[h][1] = bf16hi(u.x);
      q[h][2] = bf16lo(u.y);
      q[h][3] = bf16hi(u.y);
    }
  }
  const int pg = tid >> 6, dp = tid & 63;
  float o[kGroup][2] = {};
  int stage = 0;
  uint32_t phase = 0;
  bool failed = false;  // a timed-out wait records the error; control flow is unchanged
  for (int i = 0; i < nsub; ++i) {
    const int64_t t0 = start + int64_t(i) * kSub;
    const int rows = int(min(int64_t(kSub), stop - t0));
    float* scb = sc + (i & 1) * kGroup * kSub;
    if (!failed && !mbar_wait(&full[stage], phase, p.err, 203)) failed = true;
    const uint16_t* kst = ks + size_t(stage) * kSub * kHeadDim;
    const uint16_t* vst = vs + size_t(stage) * kSub * kHeadDim;
    // scores: warp w handles positions 8w .. 8w+7
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
      // transposed reduction: afterwards lane l holds head (l >> 3)'s sum
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
      if ((lane & 7) == 0)
        scb[(lane >> 3) * kSub + t] = t < rows ? keep * scale : -__int_as_float(0x7F800000);
    }
    named_sync(1, kAttnConsumers);
    // online softmax: warp h < 4 owns head h
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
    named_sync(1, kAttnConsumers);
    // PV: position group pg takes t = pg, pg+4, ...; lane pair of dims 2dp, 2dp+1
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == kAttnStages) {
      stage = 0;
      phase ^= 1;
    }
  }

  // merge the 4 position groups, then publish this split's partial
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    red[(pg * kGroup + h) * kHeadDim + 2 * dp] = o[h][0];
    red[(pg * kGroup + h) * kHeadDim + 2 * dp + 1] = o[h][1];
  }
  named_sync(1, kAttnConsumers);
  for (int e = tid; e < kGroup * kHeadDim; e += kAttnConsumers) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    const float v = red[(0 * kGroup + h) * kHeadDim + d] + red[(1 * kGroup + h) * kHeadDim + d] +
                    red[(2 * kGroup + h) * kHeadDim + d] + red[(3 * kGroup + h) * kHeadDim + d];
    const int64_t row = (int64_t(m) * 32 + g * kGroup + h) * p.splits + s;
    p.part_o[row * kHeadDim + d] = v;
    if (d == 0) {
      p.part_ml[row * 2] = m_run[h];
      p.part_ml[row * 2 + 1] = l_run[h];
    }
  }
  __threadfence();
  named_sync(1, kAttnConsumers);
  if (tid == 0) {
    const unsigned int ticket = atomicAdd(&p.tickets[m * 8 + g], 1u);
    red[0] = __int_as_float(ticket == unsigned(p.splits - 1) ? 1 : 0);
  }
  named_sync(1, kAttnConsumers);
  if (__float_as_int(red[0]) != 1) return;
  __threadfence();
  // Last CTA of the group: merge the splits. The per-split (max, sum) pairs
  // of the 4 heads are staged in shared memory in blocks of 256 splits (all
  // loads issued in parallel), then each thread reduces its 2 outputs over
  // the splits with independent, unrolled loads.
  float* st_m = red;                         // [4][256] running maxima
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
  for (int base = 0; base < p.splits; base += 256) {
    const int nb = min(256, p.splits - base);
    named_sync(1, kAttnConsumers);
    for (int i = tid; i < kGroup * nb; i += kAttnConsumers) {
      const int h = i / nb, j = i % nb;
      st_m[h * 256 + j] = __ldcg(p.part_ml + ((int64_t(m) * 32 + g * kGroup + h) * p.splits + base + j) * 2);
    }
    named_sync(1, kAttnConsumers);
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
        lsum = fmaf(w, __ldcg(p.part_ml + ((int64_t(m) * 32 + g * kGroup + warp) * p.splits + base + j) * 2 + 1),
                    lsum);
      }
      lsum = warp_sum(lsum);
      if (lane == 0) {
        const float scale = mold == -__int_as_float(0x7F800000) ? 0.f : expf(mold - mnew);
        st_l[warp] = st_l[warp] * scale + lsum;
        st_M[warp] = mnew;
        st_s[warp] = scale;  // rescale of the earlier blocks
      }
    }
    named_sync(1, kAttnConsumers);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int e = q ? e1 : e0;
      const int h = e / kHeadDim, d = e % kHeadDim;
      acc[q] *= st_s[h];
      const float* po = p.part_o + ((int64_t(m) * 32 + g * kGroup + h) * p.splits + base) * kHeadDim + d;
      float sum = 0.f;
#pragma unroll 8
      for (int j = 0; j < nb; ++j) sum = fmaf(st_w[h * 256 + j], __ldcg(po + int64_t(j) * kHeadDim), sum);
      acc[q] += sum;
    }
  }
  named_sync(1, kAttnConsumers);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int e = q ? e1 : e0;
    const int h = e / kHeadDim, d = e % kHeadDim;
    p.out[int64_t(m) * 4096 + (g * kGroup + h) * kHeadDim + d] = f2bf(acc[q] / st_l[h]);
  }
  if (tid == 0) p.tickets[m * 8 + g] = 0u;
}

int prepare_attention() { return configure_smem("cb_attention", attention_kernel, AttnSmem::BYTES); }

}  // namespace cb

using namespace cb;

extern "C" int64_t cb_attention_workspace_bytes(int M, int splits) {
  if (M <= 0 || splits <= 0) return 0;
  const int64_t rows = int64_t(M) * 32 * splits;
  return rows * kHeadDim * 4 + rows * 2 * 4;
}

extern "C" int cb_attention(const void* q, const void* k_cache, const void* v_cache,
                            int64_t cache_len, const int32_t* position, int M, int splits, int chunk,
                            void* out, void* workspace, unsigned int* tickets, void* stream) {
  if (!q || !k_cache || !v_cache || !position || !out || !workspace || !tickets)
    return fail(kErrInvalid, "cb_attention: null pointer");
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(q))
    return fail(kErrInvalid, "cb_attention: q/k_cache/v_cache must be 16-byte aligned");
  if (M < 1 || M > 65535) return fail(kErrInvalid, "cb_attention: M=%d out of range", M);
  if (splits < 1 || splits > 65535) return fail(kErrInvalid, "cb_attention: splits=%d", splits);
  if (chunk < kSub || chunk % kSub) return fail(kErrInvalid, "cb_attention: chunk must be a multiple of 64");
  if (cache_len < 1) return fail(kErrInvalid, "cb_attention: cache_len must be positive");
  int rc = configure_smem("cb_attention", attention_kernel, AttnSmem::BYTES);
  if (rc != kOk) return rc;
  AttnParams p = {};
  p.q = static_cast<const uint16_t*>(q);
  p.k_cache = static_cast<const uint16_t*>(k_cache);
  p.v_cache = static_cast<const uint16_t*>(v_cache);
  p.cache_len = cache_len;
  p.pos = position;
  p.M = M;
  p.splits = splits;
  p.chunk = chunk;
  p.out = static_cast<uint16_t*>(out);
  const int64_t rows = int64_t(M) * 32 * splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float*>(ws + rows * kHeadDim * 4);
  p.tickets = tickets;
  p.err = error_word();
  return launch("cb_attention", attention_kernel, dim3(splits, 8, M), dim3(kAttnThreads),
                AttnSmem::BYTES, static_cast<cudaStream_t>(stream), p);
}

// ============================================================================
// Allocation-free variant of cb_attention.
//
// Some callers cannot call cudaMalloc: a host framework that owns the whole
// device-memory budget through its own pool and hands this library only the
// tensors of a call, or a caller in a latency-critical loop where an
// allocation would synchronise the device. For them the split-KV scratch
// (per-split partials and the last-CTA tickets) lives in a fixed
// file-scope device array instead of a caller workspace. Every GPU that
// loads this library holds these bytes until the process exits.
// ============================================================================
namespace cb {

constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;  // 4 MiB of partials
constexpr int kNoAllocMaxTokens = 256;                     // tickets for 256 tokens

struct NoAllocScratch {
  float partials[kNoAllocPartialBytes / sizeof(float)];
  unsigned int tickets[kNoAllocMaxTokens * 8];
};
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// Device address of g_noalloc_scratch per device ordinal. In host code the
// symbol's name is only a host-side stand-in, so the address is fetched with
// cudaGetSymbolAddress once per device, with that device current.
static std::mutex g_noalloc_lock;
static NoAllocScratch* g_noalloc_ptr[64] = {};

static int noalloc_scratch(NoAllocScratch** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_attention_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(kErrUnsupported, "cb_attention_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> guard(g_noalloc_lock);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(kErrCuda, "cb_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<NoAllocScratch*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return kOk;
}

}  // namespace cb

extern "C" int cb_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                    int64_t cache_len, const int32_t* position, int M, int splits,
                                    int chunk, void* out, void* stream) {
  if (M < 1 || M > kNoAllocMaxTokens)
    return fail(kErrInvalid, "cb_attention_noalloc: M=%d exceeds the fixed scratch (1..%d tokens)", M,
                kNoAllocMaxTokens);
  const int64_t need = cb_attention_workspace_bytes(M, splits);
  if (splits < 1 || need > int64_t(kNoAllocPartialBytes))
    return fail(kErrInvalid,
                "cb_attention_noalloc: M=%d x splits=%d needs %lld bytes of partials; the fixed scratch "
                "holds %lld",
                M, splits, (long long)need, (long long)kNoAllocPartialBytes);
  NoAllocScratch* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != kOk) return rc;
  // The tickets must start at zero; clear this call's range (a memset, not an
  // allocation) in case an earlier launch was cut short.
  cudaError_t e = cudaMemsetAsync(scratch->tickets, 0, size_t(M) * 8 * sizeof(unsigned int),
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(kErrCuda, "cb_attention_noalloc: clearing tickets: %s", cudaGetErrorString(e));
  return cb_attention(q, k_cache, v_cache, cache_len, position, M, splits, chunk, out, scratch->partials,
                      scratch->tickets, stream);
}
