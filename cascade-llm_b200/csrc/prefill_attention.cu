// Causal GQA attention of a prefill chunk on the tensor cores.
//
// Replaces llama31.py:182-234 (`_repeat_kv` + causal SDPA) for multi-token
// steps: M query tokens at positions *pos .. *pos+M-1 attend to the cache
// [0, *pos + t] (token t), scale 1/sqrt(128), fp32 softmax, bf16 output.
//
// A CTA owns 16 consecutive tokens and the 4 query heads of one KV head
// (warp w = query head 4g+w, a 16-row mma tile), so the 4 heads share every
// K/V tile read. K/V tiles of 64 positions stream through a 2-stage
// cp.async ring into XOR-swizzled shared memory. Per tile and warp:
// S = Q K^T with mma.sync m16n8k16 (bf16 in, fp32 accumulate; Q fragments
// stay in registers), the causal mask, an online softmax in registers, and
// O += P V with P taken straight from the S accumulators as A fragments
// (ldmatrix.trans gives the V fragments). The softmax follows the decode
// kernel: scores scaled in fp32, expf, running max/sum in fp32.
#include <cuda_runtime.h>

#include "cascade_b200.h"
#include "common.cuh"
#include "internal.h"

namespace cb {

int32_t* error_word();

namespace {

constexpr int kTok = 16;       // tokens per CTA (one mma row tile per head)
constexpr int kKV = 64;        // positions per K/V tile
constexpr int kDim = 128;
constexpr int kWarps = 4;      // the 4 query heads of a KV head
constexpr int kThreadsPA = kWarps * 32;
constexpr float kScale = 0.08838834764831845f;  // 1/sqrt(128)
constexpr int kTileBytes = kKV * kDim * 2;        // 16 KB
constexpr int kSmemPA = 2 * 2 * kTileBytes;       // K and V, 2 stages

struct PrefillAttnParams {
  const uint16_t* q;        // [M][kv_heads*4][128]
  const uint16_t* k_cache;  // [kv_heads][cache_len][128]
  const uint16_t* v_cache;
  int64_t cache_len;
  const int32_t* pos;
  int M, kv_heads;
  uint16_t* out;            // [M][kv_heads*4][128]
  int* err;
};

// byte offset of 16-byte chunk c (0..15) of row r in a swizzled [rows][256 B] tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return uint32_t(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
}

// Issue the cp.async copies of K/V tile `tile` (positions [tile*64, +64)) of
// KV head g into a stage (K at kbase, V at vbase, shared-window addresses;
// kptr/vptr the same as generic pointers). Rows past `limit` are written as
// zeros: their scores are masked, and a stale non-finite V value would turn
// the masked 0 * V into NaN.
__device__ __forceinline__ void load_tile(const PrefillAttnParams& p, int g, int tile, int limit, uint32_t kbase,
                                          uint32_t vbase, uint8_t* kptr, uint8_t* vptr) {
  const uint16_t* kg = p.k_cache + int64_t(g) * p.cache_len * kDim;
  const uint16_t* vg = p.v_cache + int64_t(g) * p.cache_len * kDim;
  for (int e = threadIdx.x; e < kKV * 16; e += kThreadsPA) {
    const int r = e >> 4, c = e & 15;
    const int64_t row = int64_t(tile) * kKV + r;
    if (row < limit) {
      cp_async16(kbase + swz(r, c), kg + row * kDim + c * 8);
      cp_async16(vbase + swz(r, c), vg + row * kDim + c * 8);
    } else {
      *reinterpret_cast<uint4*>(kptr + swz(r, c)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(vptr + swz(r, c)) = make_uint4(0, 0, 0, 0);
    }
  }
}

__global__ void __launch_bounds__(kThreadsPA) prefill_attention_kernel(const __grid_constant__ PrefillAttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.y;
  const int t0 = blockIdx.x * kTok;
  const int head = g * kWarps + warp;
  const int nheads = p.kv_heads * kWarps;
  grid_dep_wait();  // q and this step's K/V come from the QKV kernel
  if (threadIdx.x == 0) grid_dep_launch();
  const int64_t pos0 = __ldcg(p.pos);
  const int t_last = min(t0 + kTok, p.M) - 1;
  int64_t visible = pos0 + t_last + 1;  // keys the last token of the block sees
  if (visible > p.cache_len) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, 501);
    visible = p.cache_len;
  }
  const int limit = int(visible);
  const int ntiles = (limit + kKV - 1) / kKV;
  const uint32_t s0 = smem_u32(smem);
  auto kst = [&](int st) { return s0 + uint32_t(st * 2 * kTileBytes); };
  auto vst = [&](int st) { return s0 + uint32_t(st * 2 * kTileBytes + kTileBytes); };
  auto kpt = [&](int st) { return smem + st * 2 * kTileBytes; };
  auto vpt = [&](int st) { return smem + st * 2 * kTileBytes + kTileBytes; };

  load_tile(p, g, 0, limit, kst(0), vst(0), kpt(0), vpt(0));
  cp_async_commit();

  // Q fragments of this warp's head: rows = tokens t0 + (lane/4) and +8
  const int qr = lane >> 2, qc = (lane & 3) * 2;
  const int ta = min(t0 + qr, p.M - 1), tb = min(t0 + qr + 8, p.M - 1);
  const uint32_t* qa = reinterpret_cast<const uint32_t*>(p.q + (int64_t(ta) * nheads + head) * kDim);
  const uint32_t* qb = reinterpret_cast<const uint32_t*>(p.q + (int64_t(tb) * nheads + head) * kDim);
  uint32_t qf[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    qf[k][0] = __ldcg(qa + (16 * k + qc) / 2);
    qf[k][1] = __ldcg(qb + (16 * k + qc) / 2);
    qf[k][2] = __ldcg(qa + (16 * k + 8 + qc) / 2);
    qf[k][3] = __ldcg(qb + (16 * k + 8 + qc) / 2);
  }
  const int64_t pa = pos0 + min(t0 + qr, p.M - 1), pb = pos0 + min(t0 + qr + 8, p.M - 1);  // row positions

  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m_a = -__int_as_float(0x7F800000), m_b = m_a, l_a = 0.f, l_b = 0.f;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int st = tile & 1;
    if (tile + 1 < ntiles) load_tile(p, g, tile + 1, limit, kst(st ^ 1), vst(st ^ 1), kpt(st ^ 1), vpt(st ^ 1));
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int kv0 = tile * kKV;

    // ---- S = Q K^T (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {        // dims 16k .. 16k+15
#pragma unroll
      for (int j = 0; j < 8; j += 2) {   // positions 8j .. 8j+15
        // matrices: (pos 8j.., dims 16k..), (pos 8j.., dims 16k+8..), (pos 8j+8.., 16k..), (8j+8.., 16k+8..)
        const int r = 8 * j + (lane & 7) + ((lane >> 4) << 3);
        const int c = 2 * k + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kst(st) + swz(r, c), b0, b1, b2, b3);
        mma_bf16(s[j], qf[k][0], qf[k][1], qf[k][2], qf[k][3], b0, b1);
        mma_bf16(s[j + 1], qf[k][0], qf[k][1], qf[k][2], qf[k][3], b2, b3);
      }
    }
    // ---- scale, causal mask, online softmax (rows qr and qr+8)
    float mx_a = -__int_as_float(0x7F800000), mx_b = mx_a;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t key = kv0 + 8 * j + qc + e;
        s[j][e] = key <= pa ? s[j][e] * kScale : -__int_as_float(0x7F800000);
        s[j][2 + e] = key <= pb ? s[j][2 + e] * kScale : -__int_as_float(0x7F800000);
        mx_a = fmaxf(mx_a, s[j][e]);
        mx_b = fmaxf(mx_b, s[j][2 + e]);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xFFFFFFFFu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xFFFFFFFFu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xFFFFFFFFu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xFFFFFFFFu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);  // finite: key 0 is always visible
    const float al_a = expf(m_a - mn_a), al_b = expf(m_b - mn_b);
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[j][e] = expf(s[j][e] - mn_a);
        s[j][2 + e] = expf(s[j][2 + e] - mn_b);
        sum_a += s[j][e];
        sum_b += s[j][2 + e];
      }
    }
    l_a = l_a * al_a + sum_a;  // per-thread partial sums; reduced across the quad at the end
    l_b = l_b * al_b + sum_b;
    m_a = mn_a;
    m_b = mn_b;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= al_a;
      o[d][1] *= al_a;
      o[d][2] *= al_b;
      o[d][3] *= al_b;
    }
    // ---- O += P V (P from the S accumulators, bf16)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // positions 16kk .. 16kk+15
      const uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int d = 0; d < 16; d += 2) {  // dims 8d .. 8d+15
        // matrices: (pos 16kk.., dims 8d..), (pos 16kk+8.., 8d..), (16kk.., 8d+8..), (16kk+8.., 8d+8..)
        const int r = 16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = d + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vst(st) + swz(r, c), b0, b1, b2, b3);
        mma_bf16(o[d], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[d + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // everyone is done with this stage before it is refilled
  }
  cp_async_wait<0>();

  l_a += __shfl_xor_sync(0xFFFFFFFFu, l_a, 1);
  l_a += __shfl_xor_sync(0xFFFFFFFFu, l_a, 2);
  l_b += __shfl_xor_sync(0xFFFFFFFFu, l_b, 1);
  l_b += __shfl_xor_sync(0xFFFFFFFFu, l_b, 2);
  const float ia = 1.f / l_a, ib = 1.f / l_b;
  const int ra = t0 + qr, rb = t0 + qr + 8;
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    if (ra < p.M)
      *reinterpret_cast<uint32_t*>(p.out + (int64_t(ra) * nheads + head) * kDim + 8 * d + qc) =
          pack_bf16(o[d][0] * ia, o[d][1] * ia);
    if (rb < p.M)
      *reinterpret_cast<uint32_t*>(p.out + (int64_t(rb) * nheads + head) * kDim + 8 * d + qc) =
          pack_bf16(o[d][2] * ib, o[d][3] * ib);
  }
}

}  // namespace

int prepare_prefill_attention() { return configure_smem("cb_prefill_attention", prefill_attention_kernel, kSmemPA); }

}  // namespace cb

using namespace cb;

static bool g_prefill_tc = true;

extern "C" int cb_set_prefill_attention_tc(int enable) {
  const int previous = g_prefill_tc ? 1 : 0;
  g_prefill_tc = enable != 0;
  return previous;
}

extern "C" int cb_prefill_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                                    const int32_t* position, int M, int kv_heads, void* out, void* stream) {
  if (!q || !k_cache || !v_cache || !position || !out)
    return fail(kErrInvalid, "cb_prefill_attention: null pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(kErrInvalid, "cb_prefill_attention: pointers must be 16-byte aligned");
  if (M < 1 || kv_heads < 1 || kv_heads > 8 || cache_len < 1)
    return fail(kErrInvalid, "cb_prefill_attention: M=%d kv_heads=%d cache_len=%lld", M, kv_heads,
                (long long)cache_len);
  if (g_prefill_tc) {
    CB_REQUIRE(int64_t(kv_heads) * cache_len < (int64_t(1) << 31),
               "cb_prefill_attention: kv_heads x cache_len must be < 2^31");
    return run_prefill_attention_tc(q, k_cache, v_cache, cache_len, position, M, kv_heads, out,
                                    static_cast<cudaStream_t>(stream));
  }
  int rc = configure_smem("cb_prefill_attention", prefill_attention_kernel, kSmemPA);
  if (rc != kOk) return rc;
  PrefillAttnParams p = {};
  p.q = static_cast<const uint16_t*>(q);
  p.k_cache = static_cast<const uint16_t*>(k_cache);
  p.v_cache = static_cast<const uint16_t*>(v_cache);
  p.cache_len = cache_len;
  p.pos = position;
  p.M = M;
  p.kv_heads = kv_heads;
  p.out = static_cast<uint16_t*>(out);
  p.err = error_word();
  return launch("cb_prefill_attention", prefill_attention_kernel, dim3((M + kTok - 1) / kTok, kv_heads),
                dim3(kThreadsPA), kSmemPA, static_cast<cudaStream_t>(stream), p);
}
