// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05,
// TMEM accumulators, TMA tiles), sm_100a.
//
// Replaces llama31.py:182-234 (`_repeat_kv` + causal SDPA) for multi-token
// steps: M query tokens at positions *pos .. *pos+M-1 attend to the cache
// [0, *pos + t] (token t), scale 1/sqrt(128), fp32 softmax, bf16 output.
//
// A CTA owns 32 consecutive tokens and the 4 query heads of one KV head:
// 128 query rows (row r = token r/4, head r%4; the 4 heads of a token are
// adjacent in q, so one 3-D TMA box brings the whole tile) that share every
// K/V tile. Per 128-position K/V tile j:
//   S_j  = Q K_j^T   tcgen05.mma M=128 N=128 K=128 into a TMEM buffer (two
//                    buffers, so S_{j+1} is computed while S_j is softmaxed)
//   softmax          8 warps, two threads per TMEM lane (= row), each on
//                    half the columns: causal mask, running maximum (shared
//                    through shared memory), exp2, running sum; P_j (bf16)
//                    written to shared memory in the swizzled K-major layout
//                    of an MMA A operand
//   O   += P_j V_j   tcgen05.mma M=128 N=128 K=128 into the TMEM O; V is
//                    position-major in the cache, so it is the MN-major B
//                    operand (no transpose)
// Warp roles: 0 TMA producer (Q once, then K and V tiles through separate
// 2-stage rings: K_j is reloaded once S_{j-2} has read it, V_j once PV_{j-2}
// has), 1 MMA issuer (one thread), 2 TMEM allocation, 4-11 softmax and
// epilogue. The output is O / l per row.
//
// The running maximum is only moved (and O rescaled in TMEM) when a tile's
// maximum exceeds it by more than 2^8 in the exp2 domain: the probabilities
// of a tile are then at most 256, exact in fp32 and as precise in bf16 as
// any other value, and most tiles need no rescale. Cache rows at or past
// *pos + M were never written; their V rows are zeroed in shared memory so
// that a zero probability cannot meet a non-finite value.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "cascade_b200.h"
#include "common.cuh"
#include "gemm_device.cuh"
#include "internal.h"

namespace cb {

int32_t* error_word();

namespace {

constexpr int kTcTok = 32;                 // tokens per CTA (x 4 heads = 128 rows)
constexpr int kTcRows = 128;
constexpr int kTcKV = 128;                 // positions per K/V tile
constexpr int kTcPanel = 128 * 64 * 2;     // one 128-row x 128-byte swizzled panel (16 KB)
constexpr int kTcStages = 2;
constexpr int kTcThreads = 384;              // 12 warps: 8 of them softmax
constexpr uint32_t kTcTmemCols = 512;      // S buffers at 0 and 128, O at 256
constexpr float kTcScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
constexpr float kTcRescale = 8.0f;         // move the running maximum when it grows by more than this (log2)

struct TcSmem {
  static constexpr int Q = 0;                                   // 2 panels (dims 0-63, 64-127)
  static constexpr int K = Q + 2 * kTcPanel;                    // per stage 2 panels (dims)
  static constexpr int V = K + kTcStages * 2 * kTcPanel;        // per stage 2 panels (dims)
  static constexpr int P = V + kTcStages * 2 * kTcPanel;        // 2 buffers x 2 panels (positions 0-63, 64-127)
  static constexpr int BAR = P + 2 * 2 * kTcPanel;
  // q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_empty[2], p_full[2], pv_done[2], o_full
  static constexpr int NBAR = 18;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int XCHG = TMEM_SLOT + 16;                   // [2][128] fp32: row maxima / sums of the two halves
  static constexpr int BYTES = XCHG + 2 * 128 * 4 + 1024;       // + slack to align the tiles to 1024 B
};

struct TcParams {
  int M, kv_heads;
  int64_t cache_len;
  const int32_t* pos;
  uint16_t* out;  // [M][4 * kv_heads][128]
  int* err;
};

// MN-major operand with the 128-byte swizzle: 128-byte rows of 64 MN
// elements, 8 rows (K) per 1024-byte atom; `lbo` = bytes to the next 64 MN
// elements, `sbo` = bytes to the next 8 K rows.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Two floats rounded to nearest-even bf16 and packed (lo in the low half):
// one cvt instruction (the inputs are finite).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// 2^x on the special-function unit (denormal results flush to zero: a
// probability below 2^-126 of the row maximum contributes nothing anyway)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled panel
__device__ __forceinline__ uint32_t sw128(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

// position bound of the K/V tiles a CTA reads: the largest visible position + 1
__device__ __forceinline__ int64_t tc_span(const TcParams& p, int64_t pos0, int t0) {
  return pos0 + min(t0 + kTcTok, p.M);
}

__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                const __grid_constant__ CUtensorMap tv, const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;
  uint64_t* s_empty = bars + 11;
  uint64_t* p_full = bars + 13;
  uint64_t* pv_done = bars + 15;
  uint64_t* o_full = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::TMEM_SLOT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kTcTok, g = blockIdx.y;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 2 * kTcRows);  // both softmax halves of every row
      mbar_init(&p_full[i], 2 * kTcRows);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // q and this step's K/V rows come from the previous kernels
  if (threadIdx.x == 0) grid_dep_launch();
  const int64_t pos0 = __ldcg(p.pos);
  const int64_t span = min(tc_span(p, pos0, t0), p.cache_len);
  const int tiles = int((span + kTcKV - 1) / kTcKV);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTcPanel);
      tma_load_3d(smem + TcSmem::Q, &tq, 0, 4 * g, t0, q_full);
      tma_load_3d(smem + TcSmem::Q + kTcPanel, &tq, 64, 4 * g, t0, q_full);
      const int row0 = int(int64_t(g) * p.cache_len);
      for (int j = 0; j < tiles; ++j) {
        // K_j once S_{j-2} has read the stage, V_j once PV_{j-2} has
        const int s = j & 1;
        const int y = row0 + j * kTcKV;
        if (j >= 2) mbar_wait(&k_empty[s], ((j - 2) >> 1) & 1, p.err, 511);
        uint8_t* kd = smem + TcSmem::K + s * 2 * kTcPanel;
        mbar_arrive_expect_tx(&k_full[s], 2 * kTcPanel);
        tma_load_2d(kd, &tk, 0, y, &k_full[s]);
        tma_load_2d(kd + kTcPanel, &tk, 64, y, &k_full[s]);
        if (j >= 2) mbar_wait(&v_empty[s], ((j - 2) >> 1) & 1, p.err, 521);
        uint8_t* vd = smem + TcSmem::V + s * 2 * kTcPanel;
        mbar_arrive_expect_tx(&v_full[s], 2 * kTcPanel);
        tma_load_2d(vd, &tv, 0, y, &v_full[s]);
        tma_load_2d(vd + kTcPanel, &tv, 64, y, &v_full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kTcRows, kTcKV);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kTcRows, 128) | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(smem + TcSmem::Q);
      mbar_wait(q_full, 0, p.err, 512);
      auto issue_pv = [&](int j) {
        mbar_wait(&v_full[j & 1], (j >> 1) & 1, p.err, 522);
        mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.err, 513);
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + TcSmem::P + (j & 1) * 2 * kTcPanel);
        const uint32_t v_addr = smem_u32(smem + TcSmem::V + (j & 1) * 2 * kTcPanel);
#pragma unroll
        for (int k = 0; k < kTcKV / 16; ++k) {
          const uint64_t adesc = umma_desc_sw128(p_addr + (k >> 2) * kTcPanel + (k & 3) * 32);
          const uint64_t bdesc = umma_desc_sw128_mn(v_addr + k * 16 * 128, kTcPanel, 1024);
          umma_bf16(tmem + 256, adesc, bdesc, idesc_pv, (j | k) != 0);
        }
        umma_commit(&pv_done[j & 1]);
        umma_commit(&v_empty[j & 1]);
      };
      for (int j = 0; j < tiles; ++j) {
        const int s = j & 1;
        mbar_wait(&k_full[s], (j >> 1) & 1, p.err, 514);
        if (j >= 2) mbar_wait(&s_empty[s], ((j - 2) >> 1) & 1, p.err, 515);
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + TcSmem::K + s * 2 * kTcPanel);
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k) {  // K = the 128 head dims
          const uint32_t off = (k >> 2) * kTcPanel + (k & 3) * 32;
          umma_bf16(tmem + s * kTcKV, umma_desc_sw128(q_addr + off), umma_desc_sw128(k_addr + off), idesc_s, k != 0);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        if (j >= 1) issue_pv(j - 1);
      }
      issue_pv(tiles - 1);
      umma_commit(o_full);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue
    // two warps per TMEM lane quarter: warps 4-7 own columns 0-63 of their
    // 32 rows, warps 8-11 columns 64-127; the row maximum is exchanged
    // through shared memory, the row sums are combined at the end
    const int quarter = warp & 3, half = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;  // TMEM lane = query row
    const int t = r >> 2;
    // positions <= lim are visible to this row (rows past the chunk act as
    // its last token; their output is not stored)
    const int64_t lim = pos0 + min(t0 + t, p.M - 1);
    const uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16) + half * 64;
    const int64_t written = pos0 + p.M;  // cache rows at or past this were never written
    float* xchg = reinterpret_cast<float*>(smem + TcSmem::XCHG);  // [2 halves][128 rows]
    float m_used = -__int_as_float(0x7F800000), l = 0.f;
    float v[64];
    for (int j = 0; j < tiles; ++j) {
      const int s = j & 1;
      const int64_t base = int64_t(j) * kTcKV + half * 64;
      mbar_wait(&s_full[s], (j >> 1) & 1, p.err, 516);
      tc_fence_after();
      const uint32_t s_addr = lane_addr + s * kTcKV;
      tmem_ld32(s_addr, *reinterpret_cast<float(*)[32]>(v));
      tmem_ld32(s_addr + 32, *reinterpret_cast<float(*)[32]>(v + 32));
      tc_fence_before();
      mbar_arrive(&s_empty[s]);  // S is in registers: the next S_{j+2} may overwrite the buffer
      // scale to the log2 domain; mask positions past this row's limit (only
      // tiles at the end of the causal range have any)
      const int64_t rel = lim - base;  // column i is visible when i <= rel
      if (rel >= 63) {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] *= kTcScaleLog2;
      } else {
        const int cut = int(max(int64_t(-1), rel));
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = i <= cut ? v[i] * kTcScaleLog2 : -__int_as_float(0x7F800000);
      }
      float mx[4] = {v[0], v[1], v[2], v[3]};  // four independent chains
#pragma unroll
      for (int i = 4; i < 64; ++i) mx[i & 3] = fmaxf(mx[i & 3], v[i]);
      float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      xchg[half * kTcRows + r] = mt;
      named_sync(1, 8 * 32);
      mt = fmaxf(mt, xchg[(half ^ 1) * kTcRows + r]);
      named_sync(1, 8 * 32);  // both halves have read before the next tile writes
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_used = mt;
      } else if (mt > m_used + kTcRescale) {
        alpha = ex2_approx(m_used - mt);
        m_used = mt;
        rescale = true;
      }
      // O *= alpha once the previous tile's PV has landed in TMEM. TMEM loads
      // and stores are warp-wide, so the whole warp takes the branch when any
      // of its rows moved its maximum (alpha = 1 for the others).
      if (__any_sync(0xFFFFFFFFu, rescale)) {
        mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, 517);
        tc_fence_after();
        float o[32];
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(lane_addr + 256 + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(lane_addr + 256 + c * 32, o);
        }
        l *= alpha;
      }
      // the P buffer of tile j - 2 is free once its PV has completed
      if (j >= 2) mbar_wait(&pv_done[s], ((j - 2) >> 1) & 1, p.err, 518);
      // probabilities, their sum, and P (this half = one panel) in the swizzled A layout
      uint8_t* panel = smem + TcSmem::P + s * 2 * kTcPanel + half * kTcPanel;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // fp32 sums of the unrounded probabilities (P is bf16 in the MMA)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p0 = ex2_approx(v[8 * c + 2 * i] - m_used), p1 = ex2_approx(v[8 * c + 2 * i + 1] - m_used);
          ls[i] += p0 + p1;
          w[i] = pack_bf16x2(p0, p1);
        }
        *reinterpret_cast<uint4*>(panel + sw128(r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // V rows of never-written cache positions: zero (row r of this half's panel)
      if (int64_t(j) * kTcKV + kTcKV > written) {
        mbar_wait(&v_full[s], (j >> 1) & 1, p.err, 519);
        if (int64_t(j) * kTcKV + r >= written) {
          uint8_t* vt = smem + TcSmem::V + s * 2 * kTcPanel + half * kTcPanel;
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vt + sw128(r, c)) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();  // P (and zeroed V rows) are read by the MMA (async proxy)
      mbar_arrive(&p_full[s]);
    }
    // epilogue: O / l for the rows of this chunk's tokens (l = both halves' sums)
    xchg[half * kTcRows + r] = l;
    named_sync(1, 8 * 32);
    l += xchg[(half ^ 1) * kTcRows + r];
    mbar_wait(o_full, 0, p.err, 520);
    tc_fence_after();
    const bool live = t0 + t < p.M;
    const float inv = 1.0f / l;
    uint16_t* out = p.out + (int64_t(t0 + t) * 4 * p.kv_heads + 4 * g + (r & 3)) * 128 + half * 64;
    float o[32];
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      tmem_ld32(lane_addr + 256 + c * 32, o);
      if (!live) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(o[8 * q + 2 * i] * inv, o[8 * q + 2 * i + 1] * inv);
        *reinterpret_cast<uint4*>(out + c * 32 + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

}  // namespace

int prepare_prefill_attention_tc() {
  return configure_smem("cb_prefill_attention", prefill_attention_tc_kernel, TcSmem::BYTES);
}

// Tensor maps of one launch: q as [M][4 kv_heads][128] read in (64, 4, 32)
// boxes (dims, heads, tokens), the caches as [kv_heads * cache_len][128] read
// in (64, 128) boxes; 128-byte swizzle; out-of-range boxes read as zero.
int run_prefill_attention_tc(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                             const int32_t* position, int M, int kv_heads, void* out, cudaStream_t stream) {
  auto encode = tensor_map_encoder();
  if (!encode) return fail(kErrCuda, "cb_prefill_attention: cuTensorMapEncodeTiled unavailable");
  CUtensorMap tq, tk, tv;
  {
    cuuint64_t dims[3] = {128, cuuint64_t(4 * kv_heads), cuuint64_t(M)};
    cuuint64_t strides[2] = {256, cuuint64_t(4 * kv_heads) * 256};
    cuuint32_t box[3] = {64, 4, kTcTok};
    cuuint32_t elem[3] = {1, 1, 1};
    CUresult r = encode(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(kErrCuda, "cb_prefill_attention: q tensor map (%d)", int(r));
  }
  for (int i = 0; i < 2; ++i) {
    cuuint64_t dims[2] = {128, cuuint64_t(kv_heads) * cuuint64_t(cache_len)};
    cuuint64_t strides[1] = {256};
    cuuint32_t box[2] = {64, kTcKV};
    cuuint32_t elem[2] = {1, 1};
    CUresult r = encode(i == 0 ? &tk : &tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(i == 0 ? k_cache : v_cache), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(kErrCuda, "cb_prefill_attention: cache tensor map (%d)", int(r));
  }
  int rc = configure_smem("cb_prefill_attention", prefill_attention_tc_kernel, TcSmem::BYTES);
  if (rc != kOk) return rc;
  TcParams p = {};
  p.M = M;
  p.kv_heads = kv_heads;
  p.cache_len = cache_len;
  p.pos = position;
  p.out = static_cast<uint16_t*>(out);
  p.err = error_word();
  return launch("cb_prefill_attention", prefill_attention_tc_kernel, dim3((M + kTcTok - 1) / kTcTok, kv_heads),
                dim3(kTcThreads), TcSmem::BYTES, stream, tq, tk, tv, p);
}

}  // namespace cb
