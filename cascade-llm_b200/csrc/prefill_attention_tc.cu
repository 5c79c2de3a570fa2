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
// K/V tile. The K/V tiles (128 positions) alternate between two softmax warp
// groups: group h = j % 2 owns tile j.
//   S_j  = Q K_j^T   tcgen05.mma M=128 N=128 K=128 into group h's TMEM buffer
//   softmax          group h (4 warps, one thread per TMEM lane = query row,
//                    all 128 columns): causal mask, the group's own running
//                    maximum and sum, exp2; P_j (bf16 pairs) stored back over
//                    the first 64 columns of the thread's S_j
//   O_h += P_j V_j   tcgen05.mma M=128 N=128 K=128 with A = P read from TMEM
//                    and B = V from shared memory into the group's own
//                    accumulator; V is position-major in the cache, so it is
//                    the MN-major B operand (no transpose)
// The two groups never wait for each other inside the loop (no barrier, no
// exchanged maximum), so one group's exponentials overlap the other's loads,
// maxima and the tensor-core work of its tiles. The two partial softmaxes of a
// row are combined once at the end: O = (c0 O_0 + c1 O_1) / (c0 l_0 + c1 l_1),
// c_h = 2^(m_h - max(m_0, m_1)).
// Warp roles: 0 TMA producer of Q and the K tiles, 3 TMA producer of the V
// tiles (separate threads, so a K load never queues behind a V stage that is
// still being read), 1 MMA issuer (one thread), 2 TMEM allocation, 4-7 group
// 0, 8-11 group 1 (softmax and epilogue).
//
// TMEM columns: S (and P) of group 0 at 0, of group 1 at 128; O_0 at 256,
// O_1 at 384. S_{j+2} overwrites group h's buffer only after PV_j completed.
//
// A group's running maximum is only moved (and its O rescaled in TMEM) when a
// tile's maximum exceeds it by more than 2^8 in the exp2 domain: the
// probabilities of a tile are then at most 256, exact in fp32 and as precise
// in bf16 as any other value, and most tiles need no rescale. Cache rows at
// or past *pos + M were never written; their V rows are zeroed in shared
// memory so that a zero probability cannot meet a non-finite value.
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
constexpr int kTcKStages = 3;              // K ring depth
constexpr int kTcVStages = 3;              // V ring depth
constexpr int kTcThreads = 384;            // 12 warps: 8 of them softmax (two groups of 4)
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcO = 256;             // TMEM columns of O_0 (O_1 at kTcO + 128)
constexpr float kTcScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
constexpr float kTcRescale = 8.0f;         // move the running maximum when it grows by more than this (log2)

struct TcSmem {
  static constexpr int Q = 0;                                   // 2 panels (dims 0-63, 64-127)
  static constexpr int K = Q + 2 * kTcPanel;                    // per stage 2 panels (dims)
  static constexpr int V = K + kTcKStages * 2 * kTcPanel;       // per stage 2 panels (dims)
  static constexpr int BAR = V + kTcVStages * 2 * kTcPanel;
  // q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS], s_full[2], p_full[2], pv_done[2], o_full
  static constexpr int NBAR = 1 + 2 * kTcKStages + 2 * kTcVStages + 6 + 1;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int XCHG = TMEM_SLOT + 16;                   // [2 groups][128] fp32 (epilogue only)
  static constexpr int BYTES = XCHG + 2 * 128 * 4 + 1024;       // + slack to align the tiles to 1024 B
};
static_assert(TcSmem::BYTES <= 227 * 1024, "prefill attention shared memory");

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

// D[tmem] (+)= A[tmem] * B[smem] for one K=16 step: A is 128 lanes (rows) x
// 8 columns, each 32-bit column two bf16 of K (the lower one in the low half).
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 columns of this thread's TMEM lane without waiting; tmem_ld_wait()
// waits for every outstanding load and ties the registers to that wait so
// that no use of them is scheduled before it.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 32 words into 32 consecutive columns of this thread's TMEM lane, then wait
// until the stores are done.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 words into 16 consecutive columns of this thread's TMEM lane (no wait)
__device__ __forceinline__ void tmem_st16_async(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
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
  uint64_t* k_empty = k_full + kTcKStages;
  uint64_t* v_full = k_empty + kTcKStages;
  uint64_t* v_empty = v_full + kTcVStages;
  uint64_t* s_full = v_empty + kTcVStages;  // per group
  uint64_t* p_full = s_full + 2;            // per group
  uint64_t* pv_done = p_full + 2;           // per group: the group's latest PV completed
  uint64_t* o_full = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::TMEM_SLOT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kTcTok, g = blockIdx.y;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kTcKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kTcVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kTcRows);  // every thread (row) of the group
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
  const int row0 = int(int64_t(g) * p.cache_len);

  if (warp == 0) {
    // ------------------------------------------------------------ Q and K producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTcPanel);
      tma_load_3d(smem + TcSmem::Q, &tq, 0, 4 * g, t0, q_full);
      tma_load_3d(smem + TcSmem::Q + kTcPanel, &tq, 64, 4 * g, t0, q_full);
      for (int j = 0; j < tiles; ++j) {  // K_j once S_{j-KS} has read the stage
        const int s = j % kTcKStages;
        if (j >= kTcKStages) mbar_wait(&k_empty[s], ((j / kTcKStages) - 1) & 1, p.err, 511);
        uint8_t* kd = smem + TcSmem::K + s * 2 * kTcPanel;
        mbar_arrive_expect_tx(&k_full[s], 2 * kTcPanel);
        tma_load_2d(kd, &tk, 0, row0 + j * kTcKV, &k_full[s]);
        tma_load_2d(kd + kTcPanel, &tk, 64, row0 + j * kTcKV, &k_full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------ V producer
    if (lane == 0) {
      for (int j = 0; j < tiles; ++j) {  // V_j once PV_{j-VS} has read the stage
        const int s = j % kTcVStages;
        if (j >= kTcVStages) mbar_wait(&v_empty[s], ((j / kTcVStages) - 1) & 1, p.err, 521);
        uint8_t* vd = smem + TcSmem::V + s * 2 * kTcPanel;
        mbar_arrive_expect_tx(&v_full[s], 2 * kTcPanel);
        tma_load_2d(vd, &tv, 0, row0 + j * kTcKV, &v_full[s]);
        tma_load_2d(vd + kTcPanel, &tv, 64, row0 + j * kTcKV, &v_full[s]);
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
      auto issue_s = [&](int j) {
        const int sk = j % kTcKStages, h = j & 1;
        mbar_wait(&k_full[sk], (j / kTcKStages) & 1, p.err, 514);
        // PV_{j-2} has read P_{j-2} out of group h's buffer
        if (j >= 2) mbar_wait(&pv_done[h], ((j - 2) >> 1) & 1, p.err, 515);
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + TcSmem::K + sk * 2 * kTcPanel);
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k) {  // K = the 128 head dims
          const uint32_t off = (k >> 2) * kTcPanel + (k & 3) * 32;
          umma_bf16(tmem + h * kTcKV, umma_desc_sw128(q_addr + off), umma_desc_sw128(k_addr + off), idesc_s, k != 0);
        }
        umma_commit(&s_full[h]);
        umma_commit(&k_empty[sk]);
      };
      auto issue_pv = [&](int j) {
        const int sv = j % kTcVStages, h = j & 1;
        mbar_wait(&v_full[sv], (j / kTcVStages) & 1, p.err, 522);
        mbar_wait(&p_full[h], (j >> 1) & 1, p.err, 513);
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + TcSmem::V + sv * 2 * kTcPanel);
#pragma unroll
        for (int k = 0; k < kTcKV / 16; ++k) {
          const uint64_t bdesc = umma_desc_sw128_mn(v_addr + k * 16 * 128, kTcPanel, 1024);
          umma_bf16_tmem_a(tmem + kTcO + h * 128, tmem + h * kTcKV + k * 8, bdesc, idesc_pv, (j >= 2) || k != 0);
        }
        umma_commit(&pv_done[h]);
        umma_commit(&v_empty[sv]);
      };
      issue_s(0);
      if (tiles > 1) issue_s(1);
      for (int j = 0; j < tiles; ++j) {
        issue_pv(j);
        if (j + 2 < tiles) issue_s(j + 2);  // once PV_j has freed group h's buffer
      }
      umma_commit(o_full);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3, h = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;  // TMEM lane = query row
    const int t = r >> 2;
    // positions <= lim are visible to this row (rows past the chunk act as
    // its last token; their output is not stored)
    const int64_t lim = pos0 + min(t0 + t, p.M - 1);
    const uint32_t row_addr = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t s_addr = row_addr + h * kTcKV;
    const uint32_t o_addr = row_addr + kTcO + h * 128;
    const int64_t written = pos0 + p.M;  // cache rows at or past this were never written
    const float kNegInf = -__int_as_float(0x7F800000);
    float m_used = kNegInf, l = 0.f;
    for (int j = h; j < tiles; j += 2) {
      const int n = j >> 1;  // this group's tiles before j: the parity of its barriers
      mbar_wait(&s_full[h], n & 1, p.err, 516);
      tc_fence_after();
      uint32_t raw[4][32];  // S_j: the fp32 bits of this row's 128 columns
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_async(s_addr + 32 * c, raw[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_wait(raw[c]);
      auto v = [&](int i) { return __uint_as_float(raw[i >> 5][i & 31]); };
      // mask positions past this row's limit (only tiles at the end of the
      // causal range have any); column i is visible when i <= rel
      const int64_t rel = lim - int64_t(j) * kTcKV;
      if (rel < kTcKV - 1) {
        const int cut = int(max(int64_t(-1), rel));
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > cut) raw[i >> 5][i & 31] = __float_as_uint(kNegInf);
      }
      float mx[4] = {v(0), v(1), v(2), v(3)};  // four independent chains
#pragma unroll
      for (int i = 4; i < 128; ++i) mx[i & 3] = fmaxf(mx[i & 3], v(i));
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * kTcScaleLog2;
      bool rescale = false;
      float alpha = 1.f;
      if (j == h) {
        m_used = mt;  // -inf when every column of this first tile is masked
      } else if (mt > m_used + kTcRescale) {
        alpha = ex2_approx(m_used - mt);  // 0 when nothing was visible before
        m_used = mt;
        rescale = true;
      }
      // probabilities, their sum, and P (bf16 pairs) over the first 64
      // columns of S_j (already in registers); a fully masked row keeps the
      // reference 0 so that every probability is 2^-inf = 0
      const float neg_m = m_used == kNegInf ? 0.f : -m_used;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // fp32 sums of the unrounded probabilities (P is bf16 in the MMA)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(v(32 * c + 2 * i), kTcScaleLog2, neg_m));
          const float p1 = ex2_approx(fmaf(v(32 * c + 2 * i + 1), kTcScaleLog2, neg_m));
          ls[i & 3] += p0 + p1;
          pw[i] = pack_bf16x2(p0, p1);
        }
        tmem_st16_async(s_addr + 16 * c, pw);
      }
      tmem_st_wait();
      l = l * alpha + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
      // O_h *= alpha once the group's previous PV has landed in TMEM (it
      // completed before S_j was issued). TMEM loads and stores are
      // warp-wide, so the whole warp takes the branch when any of its rows
      // moved its maximum (alpha = 1 for the others).
      if (__any_sync(0xFFFFFFFFu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32_async(o_addr + c * 32, o);
          tmem_ld_wait(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_addr + c * 32, o);
        }
      }
      // V rows of never-written cache positions: zero (thread r takes row r,
      // both panels)
      if (int64_t(j) * kTcKV + kTcKV > written) {
        const int sv = j % kTcVStages;
        mbar_wait(&v_full[sv], (j / kTcVStages) & 1, p.err, 519);
        if (int64_t(j) * kTcKV + r >= written) {
          uint8_t* vt = smem + TcSmem::V + sv * 2 * kTcPanel;
#pragma unroll
          for (int c = 0; c < 16; ++c)
            *reinterpret_cast<uint4*>(vt + (c >> 3) * kTcPanel + sw128(r, c & 7)) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();  // the zeroed V rows are read by the MMA (async proxy)
      }
      tc_fence_before();  // P (and a rescaled O_h) before the MMA's PV_j
      mbar_arrive(&p_full[h]);
    }
    // epilogue: combine the groups' partial softmaxes of row r; group h
    // stores output dims 64h .. 64h+63. With a single tile, group 1 saw
    // nothing (m = -inf, l = 0, O_1 never written).
    float* xchg = reinterpret_cast<float*>(smem + TcSmem::XCHG);  // [2 groups][128 rows]
    xchg[h * kTcRows + r] = m_used;
    named_sync(1, 8 * 32);
    const float m_other = xchg[(h ^ 1) * kTcRows + r];
    const float m_all = fmaxf(m_used, m_other);  // finite: position 0 is visible to every row
    const float c_self = ex2_approx(m_used - m_all), c_other = ex2_approx(m_other - m_all);
    named_sync(1, 8 * 32);  // both maxima read before the sums overwrite them
    xchg[h * kTcRows + r] = l * c_self;
    named_sync(1, 8 * 32);
    const float inv = 1.0f / (l * c_self + xchg[(h ^ 1) * kTcRows + r]);
    const float c0 = (h == 0 ? c_self : c_other) * inv, c1 = (h == 0 ? c_other : c_self) * inv;
    mbar_wait(o_full, 0, p.err, 520);
    tc_fence_after();
    const bool live = t0 + t < p.M;
    const bool second = tiles > 1;
    uint16_t* out = p.out + (int64_t(t0 + t) * 4 * p.kv_heads + 4 * g + (r & 3)) * 128 + h * 64;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t o0[32], o1[32];
      tmem_ld32_async(row_addr + kTcO + h * 64 + c * 32, o0);
      if (second) tmem_ld32_async(row_addr + kTcO + 128 + h * 64 + c * 32, o1);
      tmem_ld_wait(o0);
      if (second) tmem_ld_wait(o1);
      if (!live) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int e = 8 * q + 2 * i;
          const float a0 = c0 * __uint_as_float(o0[e]), a1 = c0 * __uint_as_float(o0[e + 1]);
          w[i] = second ? pack_bf16x2(fmaf(c1, __uint_as_float(o1[e]), a0), fmaf(c1, __uint_as_float(o1[e + 1]), a1))
                        : pack_bf16x2(a0, a1);
        }
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
