// Prefill GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// A prefill chunk of M tokens turns every projection of the Llama block into
// a dense GEMM C[M, N] = A[M, K] . W[N, K]^T (reference: the F.linear calls
// of layer_streaming/llama31.py:238-280 with M > 1), the only place on the
// path that is tensor-core bound (M >~ 250 tokens at the B200 ridge point).
//
// Persistent: one CTA per SM walks the 128 x BN tiles of C (tile t, t + grid,
// ...; M tiles fastest, so the CTAs working at one time share a few weight
// tiles and the weights cross HBM about once):
//   warp 0        TMA producer: A (activations) and W (weights) K-blocks,
//                 128-byte swizzle, into a shared-memory ring (mbarriers
//                 full/empty per stage; each CTA loads its own tiles) that runs
//                 on across tile boundaries: 256-wide tiles take 64-wide K
//                 blocks in 4 stages, 128-wide tiles 128-wide K blocks (two
//                 64-column panels per operand) in 3 stages - a CTA spends a
//                 near-constant time per K block, so halving the blocks made
//                 o_proj 36.6 -> 28.6 us and down 94.3 -> 68.2 us at M = 512
//   warp 1        MMA issuer: one thread issues tcgen05.mma kind::f16
//                 (M=128, N=BN, K=16; BF16 in, FP32 accumulate in TMEM) and
//                 commits each stage back to the producer
//   warp 2        allocates / frees the TMEM columns of TWO accumulators
//   warps 4..7    epilogue: tcgen05.ld of their 32 TMEM lanes (= tile rows),
//                 the mode's fused epilogue, bf16 stores
// The accumulators alternate between tiles (acc_full / acc_empty mbarriers),
// so the epilogue of one tile runs while the tensor cores compute the next.
// Epilogues mirror the decode GEMV's rounding points: plain bf16 store,
// residual add, SwiGLU (gate and up rows of the same FFN index in one tile),
// and QKV with RoPE and the K/V cache write.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "cascade_b200.h"
#include "common.cuh"
#include "gemm_device.cuh"
#include "internal.h"

namespace cb {

int32_t* error_word();

enum GemmMode : int {
  GEMM_STORE = 0,     // out = bf16(acc)
  GEMM_RESIDUAL = 1,  // out = bf16(residual + bf16(acc))
  GEMM_SWIGLU = 2,    // out = bf16(silu(bf16(gate acc)) * bf16(up acc))
  GEMM_QKV_ROPE = 3,  // RoPE(q) -> out, RoPE(k) / v -> caches
  GEMM_PARTIAL = 4,   // outf = acc (fp32)
  GEMM_SILU = 5,      // out = bf16(silu(bf16(acc)))
  GEMM_MUL = 6,       // out = bf16(out * bf16(acc)), in place
};

constexpr int kBM = 128;
// split-K chunks: the reduced tile [M][BN] fp32 fits shared memory next to
// the ring (64 x 128 or 16 x 256 floats, 32 / 16 KB)
constexpr int split_max_tokens(int BN) { return BN == 128 ? 64 : 16; }
constexpr int kMaxSplit = 9;
constexpr int kBK = 64;  // columns of one 128-byte-swizzled panel (the TMA box width)
template <int BN> constexpr int panels_for() { return BN == 128 ? 2 : 1; }
template <int BN> constexpr int stages_for() { return BN == 128 ? 3 : 4; }
constexpr int kGemmThreads = 256;

struct GemmParams {
  int M, N, K;               // N: output columns (SwiGLU: FFN rows)
  int ntiles;                // tiles along N (the grid walks mtiles x ntiles)
  uint16_t* out;
  float* outf;               // GEMM_PARTIAL: fp32 output (a tensor-parallel partial sum)
  int64_t ld_out;            // output row stride (elements)
  const uint16_t* residual;  // GEMM_RESIDUAL, row stride ld_out (may equal out)
  // GEMM_QKV_ROPE: q rows [0, q_rows), k rows [q_rows, +k_rows), v rows after
  // (a section is empty when its matrix is not part of the launch)
  int q_rows, k_rows, v_rows;
  const float* inv_freq;
  const int32_t* pos;        // position of row 0 of A
  uint16_t* k_cache;         // [kv_heads][cache_len][128]
  uint16_t* v_cache;
  int64_t cache_len;
  int* err;
  // split-K (M <= 64 rows with 128-wide tiles, too few tiles for the SMs): the K blocks of a
  // tile are split over `ksplit` work items; each stores its fp32 partial
  // rows into `ws` [tile][ksplit][M][BN], and the last item of a tile to
  // finish (acq_rel ticket) sums them in slice order into shared memory and
  // runs the epilogue from there. ksplit == 1: no split.
  int ksplit;
  float* ws;
  unsigned int* tickets;     // [tiles], zero; reset by the reducing item
};

template <int BN>
struct GemmSmem {
  static constexpr int PANELS = panels_for<BN>();            // 64-column panels per K block
  static constexpr int BKB = PANELS * kBK;                     // K block
  static constexpr int A_PANEL = kBM * kBK * 2;
  static constexpr int B_PANEL = BN * kBK * 2;
  static constexpr int A_BYTES = PANELS * A_PANEL;
  static constexpr int B_BYTES = PANELS * B_PANEL;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int kStages = stages_for<BN>();
  static constexpr int BAR = kStages * STAGE;                 // full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int TMEM_SLOT = BAR + (2 * kStages + 4) * 8;
  static constexpr int RED = TMEM_SLOT + 16;                  // split-K: the reduced tile [M][BN] fp32
  static constexpr int BYTES = RED + split_max_tokens(BN) * BN * 4 + 1024;  // + slack to align the ring
  static_assert(BYTES <= 227 * 1024, "GEMM shared memory");
};

template <int BN, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap tb2,
                const __grid_constant__ GemmParams p) {
  using L = GemmSmem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* empty = full + L::kStages;
  uint64_t* acc_full = empty + L::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = p.K / L::BKB;
  const int mtiles = (p.M + kBM - 1) / kBM;
  const int tiles = mtiles * p.ntiles;
  const int S = p.ksplit;
  const int items = tiles * S;  // item w: tile w / S, K slice w % S

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4 * 32);  // every epilogue thread
    }
    fence_mbar_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // A comes from the previous kernel
  if (threadIdx.x == 0) grid_dep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;  // k-blocks issued so far (the ring position)
      for (int w = blockIdx.x; w < items; w += gridDim.x) {
        const int tile = w / S, ks = w % S;
        const int kb0 = ks * nk / S, kb1 = (ks + 1) * nk / S;
        const int m0 = (tile % mtiles) * kBM, nt = tile / mtiles;
        const CUtensorMap* mb = &tb0;
        int yb = 0;
        if (MODE == GEMM_QKV_ROPE) {
          const int n0 = nt * BN;
          if (n0 < p.q_rows) {
            yb = n0;
          } else if (n0 < p.q_rows + p.k_rows) {
            mb = &tb1;
            yb = n0 - p.q_rows;
          } else {
            mb = &tb2;
            yb = n0 - p.q_rows - p.k_rows;
          }
        } else if (MODE == GEMM_SWIGLU) {
          yb = nt * (BN / 2);
        } else {
          yb = nt * BN;
        }
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % L::kStages;
          const uint32_t ph = (it / L::kStages) & 1;
          mbar_wait(&empty[s], ph ^ 1, p.err, 401);
          uint8_t* a_dst = smem + s * L::STAGE;
          uint8_t* b_dst = a_dst + L::A_BYTES;
          mbar_arrive_expect_tx(&full[s], L::STAGE);
#pragma unroll
          for (int pnl = 0; pnl < L::PANELS; ++pnl) {
            const int x = kb * L::BKB + pnl * kBK;
            tma_load_2d(a_dst + pnl * L::A_PANEL, &ta, x, m0, &full[s]);
            if (MODE == GEMM_SWIGLU) {
              tma_load_2d(b_dst + pnl * L::B_PANEL, &tb0, x, yb, &full[s]);
              tma_load_2d(b_dst + pnl * L::B_PANEL + (BN / 2) * kBK * 2, &tb1, x, yb, &full[s]);
            } else {
              tma_load_2d(b_dst + pnl * L::B_PANEL, mb, x, yb, &full[s]);
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      int it = 0, i = 0;
      for (int w = blockIdx.x; w < items; w += gridDim.x, ++i) {
        const int ks = w % S;
        const int kb0 = ks * nk / S, kb1 = (ks + 1) * nk / S;
        const int a = i & 1;
        // accumulator a is free once the epilogue has read tile i - 2 out of it
        if (i >= 2) mbar_wait(&acc_empty[a], ((i >> 1) - 1) & 1, p.err, 404);
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % L::kStages;
          const uint32_t ph = (it / L::kStages) & 1;
          mbar_wait(&full[s], ph, p.err, 402);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::STAGE);
          const uint64_t adesc = umma_desc_sw128(a_addr);
          const uint64_t bdesc = umma_desc_sw128(a_addr + L::A_BYTES);
#pragma unroll
          for (int k = 0; k < L::BKB / 16; ++k) {  // +32 bytes per K step within a panel (16-byte units)
            const uint32_t pa = (k >> 2) * (L::A_PANEL >> 4) + 2 * (k & 3);
            const uint32_t pb = (k >> 2) * (L::B_PANEL >> 4) + 2 * (k & 3);
            umma_bf16(acc, adesc + pa, bdesc + pb, idesc, (kb != kb0) || (k != 0));
          }
          umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        umma_commit(&acc_full[a]);  // the tile's accumulator is complete
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    int i = 0;
    __shared__ int last_item;  // split-K: this CTA reduces the tile
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++i) {
      const int tile = w / S, ks = w % S;
      const int a = i & 1;
      mbar_wait(&acc_full[a], (i >> 1) & 1, p.err, 403);
      tc_fence_after();
      const int m0 = (tile % mtiles) * kBM, nt = tile / mtiles;
      const int row = (warp - 4) * 32 + lane;
      const int m = m0 + row;
      const bool live = m < p.M;
      const uint32_t taddr = tmem + a * BN + (uint32_t((warp & 3) * 32) << 16);
      float v[32];
      if (S > 1) {
        // this slice's partial rows -> ws; the accumulator is then free
        float* mine = p.ws + ((int64_t(tile) * S + ks) * p.M + m) * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(taddr + c * 32, v);
          if (!live) continue;
          float4* o = reinterpret_cast<float4*>(mine + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[a]);
        __threadfence();
        named_sync(1, 4 * 32);
        if (warp == 4 && lane == 0)
          last_item = atom_add_acq_rel_gpu(p.tickets + tile, 1u) == unsigned(S - 1) ? 1 : 0;
        named_sync(1, 4 * 32);
        const bool reduce = last_item != 0;
        named_sync(1, 4 * 32);  // every thread has read the flag before the next item rewrites it
        if (!reduce) continue;
        if (warp == 4 && lane == 0) p.tickets[tile] = 0u;
        // all 128 epilogue threads sum the slices of the whole tile into
        // shared memory, every slice's load of an output in flight at once
        // (the sum runs in slice order: the same bits as a per-row sum)
        float4* red4 = reinterpret_cast<float4*>(smem + L::RED);
        const float4* src = reinterpret_cast<const float4*>(p.ws + int64_t(tile) * S * p.M * BN);
        const int64_t slice4 = int64_t(p.M) * BN / 4;
        for (int o = int(threadIdx.x) - 128; o < p.M * BN / 4; o += 128) {
          float4 part[kMaxSplit];
#pragma unroll
          for (int q = 0; q < kMaxSplit; ++q)
            if (q < S) part[q] = __ldcg(src + q * slice4 + o);
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int q = 0; q < kMaxSplit; ++q) {
            if (q < S) {
              acc.x += part[q].x;
              acc.y += part[q].y;
              acc.z += part[q].z;
              acc.w += part[q].w;
            }
          }
          red4[o] = acc;
        }
        named_sync(1, 4 * 32);
      }
      // fp32 accumulator columns [col, col + 32) of this thread's row: from
      // TMEM, or (split-K) from the tile reduced into shared memory
      auto fetch = [&](int col, float (&dst)[32]) {
        if (S == 1) {
          tmem_ld32(taddr + col, dst);
          return;
        }
        const float4* r4 = reinterpret_cast<const float4*>(smem + L::RED) + (int64_t(live ? m : 0) * BN + col) / 4;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = r4[j];
          dst[4 * j] = f.x;
          dst[4 * j + 1] = f.y;
          dst[4 * j + 2] = f.z;
          dst[4 * j + 3] = f.w;
        }
      };
      if (MODE == GEMM_PARTIAL) {
        const int n0 = nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          fetch(c * 32, v);
          if (!live) continue;
          float4* o = reinterpret_cast<float4*>(p.outf + int64_t(m) * p.ld_out + n0 + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
      } else if (MODE == GEMM_STORE || MODE == GEMM_RESIDUAL || MODE == GEMM_SILU || MODE == GEMM_MUL) {
        const int n0 = nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          fetch(c * 32, v);
          if (!live) continue;
          uint16_t* o = p.out + int64_t(m) * p.ld_out + n0 + c * 32;
          const uint16_t* r = p.residual + int64_t(m) * p.ld_out + n0 + c * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
            uint4 rr = make_uint4(0, 0, 0, 0);
            if (MODE == GEMM_RESIDUAL) rr = ld_cg_u4(r + q * 8);
            if (MODE == GEMM_MUL) rr = ld_cg_u4(o + q * 8);
            const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float lo = v[q * 8 + 2 * e], hi = v[q * 8 + 2 * e + 1];
              if (MODE == GEMM_RESIDUAL) {  // x + F.linear(...): the projection rounds to bf16 first
                lo = bf16lo(rw[e]) + rbf(lo);
                hi = bf16hi(rw[e]) + rbf(hi);
              } else if (MODE == GEMM_SILU) {
                lo = silu_bf16(rbf(lo));
                hi = silu_bf16(rbf(hi));
              } else if (MODE == GEMM_MUL) {  // silu(gate) (already bf16) * bf16(up)
                lo = bf16lo(rw[e]) * rbf(lo);
                hi = bf16hi(rw[e]) * rbf(hi);
              }
              w[e] = uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
            }
            *reinterpret_cast<uint4*>(o + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else if (MODE == GEMM_SWIGLU) {
        const int n0 = nt * (BN / 2);
        float u[32];
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          fetch(c * 32, v);             // gate rows n0 + c*32 ..
          fetch(BN / 2 + c * 32, u);    // up rows, same FFN index
          if (!live) continue;
          uint16_t* o = p.out + int64_t(m) * p.ld_out + n0 + c * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = q * 8 + 2 * e;
              const float lo = silu_bf16(rbf(v[i])) * rbf(u[i]);
              const float hi = silu_bf16(rbf(v[i + 1])) * rbf(u[i + 1]);
              w[e] = uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
            }
            *reinterpret_cast<uint4*>(o + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else {  // GEMM_QKV_ROPE, BN == 128: one head per tile
        const int n0 = nt * BN;
        const int pos = __ldcg(p.pos) + m;
        const bool in_cache = pos >= 0 && pos < p.cache_len;
        if (live && n0 >= p.q_rows && !in_cache && p.err) atomicExch(p.err, 103);
        uint16_t* dst;
        if (n0 < p.q_rows) {
          dst = p.out + int64_t(m) * p.ld_out + n0;
        } else if (n0 < p.q_rows + p.k_rows) {
          dst = p.k_cache + ((int64_t(n0 - p.q_rows) / 128) * p.cache_len + pos) * 128;
        } else {
          dst = p.v_cache + ((int64_t(n0 - p.q_rows - p.k_rows) / 128) * p.cache_len + pos) * 128;
        }
        const bool store = live && (n0 < p.q_rows || in_cache);
        if (n0 >= p.q_rows + p.k_rows) {  // V: no rotation
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            fetch(c * 32, v);
            if (!store) continue;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = uint32_t(f2bf(v[q * 8 + 2 * e])) | (uint32_t(f2bf(v[q * 8 + 2 * e + 1])) << 16);
              *reinterpret_cast<uint4*>(dst + c * 32 + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        } else {  // Q or K: RoPE on the (d, d + 64) pairs of the head
          float u[32];
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            fetch(c * 32, v);
            fetch(64 + c * 32, u);
            if (!store) continue;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t wa[4], wb[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = q * 8 + 2 * e;
                const int d = c * 32 + i;
                uint16_t a0, b0, a1, b1;
                rope_pair(v[i], u[i], __ldg(p.inv_freq + d), pos, a0, b0);
                rope_pair(v[i + 1], u[i + 1], __ldg(p.inv_freq + d + 1), pos, a1, b1);
                wa[e] = uint32_t(a0) | (uint32_t(a1) << 16);
                wb[e] = uint32_t(b0) | (uint32_t(b1) << 16);
              }
              *reinterpret_cast<uint4*>(dst + c * 32 + q * 8) = make_uint4(wa[0], wa[1], wa[2], wa[3]);
              *reinterpret_cast<uint4*>(dst + 64 + c * 32 + q * 8) = make_uint4(wb[0], wb[1], wb[2], wb[3]);
            }
          }
        }
      }
      // the accumulator is read (tcgen05.wait::ld inside tmem_ld32): hand it back
      if (S == 1) {
        tc_fence_before();
        mbar_arrive(&acc_empty[a]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

}  // namespace cb

// ====================================================================== host
using namespace cb;

namespace cb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace cb

namespace {

// Row-major bf16 matrix [rows, inner] read in [box_rows, 64] tiles with the
// 128-byte swizzle; rows past the end read as zero.
int make_tile_map(CUtensorMap* map, const char* what, const void* base, int64_t rows, int64_t inner,
                  int box_rows) {
  auto encode = tensor_map_encoder();
  if (!encode) return fail(kErrCuda, "%s: cuTensorMapEncodeTiled unavailable", what);
  cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(inner) * 2};
  cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kErrCuda, "%s: cuTensorMapEncodeTiled failed (%d)", what, int(r));
  return kOk;
}

// Split-K workspace registered by cb_set_gemm_workspace (null: never split).
float* g_splitk_ws = nullptr;
int64_t g_splitk_bytes = 0;
unsigned int* g_splitk_tickets = nullptr;
int g_splitk_ntickets = 0;

// K slices per tile: 1, unless the chunk is short (M <= 64 with 128-wide
// tiles, M <= 16 with 256-wide ones: one M tile,
// fewer tiles than SMs) and K is long (>= 8192: the down projection's
// 14336, 9 slices, 32 tiles -> 288 work items). The count depends on K
// alone, so every projection with the same K sums the same fp32 slices in
// the same order. Measured at M = 6 (down 87 -> 40 us), and measured not to
// pay for K = 4096: a work item costs ~10 us of fixed overhead (partials,
// ticket, reduce), more than a fifth of a 4096-long tile streams (QKV 48 ->
// 74 us, gate+up 70 -> 87, o_proj 32.5 -> 32 with 5 slices). A workspace
// too small for the launch means no split.
int choose_ksplit(int M, int K, int tiles, int BN) {
  if (!g_splitk_ws || M > split_max_tokens(BN) || tiles >= sm_count() || tiles > g_splitk_ntickets) return 1;
  const int bk = BN == 128 ? 128 : 64;
  if (K / 64 < 128) return 1;
  const int S = kMaxSplit;
  if (K / bk / S < 4) return 1;
  if (int64_t(tiles) * S * M * BN * 4 > g_splitk_bytes) return 1;
  return S;
}

template <int BN, int MODE>
int run_gemm(const char* what, const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1,
             const CUtensorMap& tb2, GemmParams& p, int grid_x, cudaStream_t stream) {
  int rc = configure_smem(what, gemm_kernel<BN, MODE>, GemmSmem<BN>::BYTES);
  if (rc != kOk) return rc;
  p.err = error_word();
  p.ntiles = grid_x;
  // persistent: one CTA per SM (the shared-memory ring fills the SM), at most one per work item
  const int64_t tiles = int64_t((p.M + kBM - 1) / kBM) * grid_x;
  p.ksplit = choose_ksplit(p.M, p.K, int(tiles), BN);
  p.ws = p.ksplit > 1 ? g_splitk_ws : nullptr;
  p.tickets = p.ksplit > 1 ? g_splitk_tickets : nullptr;
  const int64_t items = tiles * p.ksplit;
  const dim3 grid(unsigned(items < sm_count() ? items : sm_count()));
  return launch(what, gemm_kernel<BN, MODE>, grid, dim3(kGemmThreads), GemmSmem<BN>::BYTES, stream, ta, tb0, tb1,
                tb2, p);
}

bool gemm_shape_ok(const void* a, int M, int K, const void* w) {
  return a && w && aligned16(a) && aligned16(w) && M >= 1 && M <= (1 << 20) && K >= 128 && K % 128 == 0;
}

}  // namespace

namespace cb {
int prepare_gemm() {
  int rc = configure_smem("gemm", gemm_kernel<256, GEMM_STORE>, GemmSmem<256>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<128, GEMM_STORE>, GemmSmem<128>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<256, GEMM_RESIDUAL>, GemmSmem<256>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<128, GEMM_RESIDUAL>, GemmSmem<128>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<256, GEMM_SWIGLU>, GemmSmem<256>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<128, GEMM_QKV_ROPE>, GemmSmem<128>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<256, GEMM_PARTIAL>, GemmSmem<256>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<128, GEMM_PARTIAL>, GemmSmem<128>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<256, GEMM_SILU>, GemmSmem<256>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<128, GEMM_SILU>, GemmSmem<128>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<256, GEMM_MUL>, GemmSmem<256>::BYTES);
  if (rc == kOk) rc = configure_smem("gemm", gemm_kernel<128, GEMM_MUL>, GemmSmem<128>::BYTES);
  if (rc == kOk && !tensor_map_encoder()) rc = fail(kErrCuda, "gemm: cuTensorMapEncodeTiled unavailable");
  return rc;
}
}  // namespace cb

static int gemm_linear(const char* what, int mode, const void* a, int M, int K, const void* w, int N,
                       const void* residual, void* out, void* stream) {
  if (!gemm_shape_ok(a, M, K, w) || !out || !aligned16(out))
    return fail(kErrInvalid, "%s: a/w/out must be 16-byte aligned device pointers, 1 <= M, K a multiple of 128",
                what);
  if (mode == GEMM_RESIDUAL && (!residual || !aligned16(residual)))
    return fail(kErrInvalid, "%s: residual must be a 16-byte aligned device pointer", what);
  if (N < 128 || N % 128) return fail(kErrInvalid, "%s: N=%d must be a positive multiple of 128", what, N);
  // 256-column tiles, unless they would leave SMs idle (one CTA per SM)
  const int mtiles = (M + kBM - 1) / kBM;
  const int bn = (N % 256 == 0 && int64_t(N / 256) * mtiles >= sm_count()) ? 256 : 128;
  CUtensorMap ta, tb;
  int rc = make_tile_map(&ta, what, a, M, K, kBM);
  if (rc == kOk) rc = make_tile_map(&tb, what, w, N, K, bn);
  if (rc != kOk) return rc;
  GemmParams p = {};
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = static_cast<uint16_t*>(out);
  p.outf = static_cast<float*>(out);
  p.ld_out = N;
  p.residual = static_cast<const uint16_t*>(residual);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mode == GEMM_PARTIAL)
    return bn == 256 ? run_gemm<256, GEMM_PARTIAL>(what, ta, tb, tb, tb, p, N / 256, s)
                     : run_gemm<128, GEMM_PARTIAL>(what, ta, tb, tb, tb, p, N / 128, s);
  if (mode == GEMM_SILU)
    return bn == 256 ? run_gemm<256, GEMM_SILU>(what, ta, tb, tb, tb, p, N / 256, s)
                     : run_gemm<128, GEMM_SILU>(what, ta, tb, tb, tb, p, N / 128, s);
  if (mode == GEMM_MUL)
    return bn == 256 ? run_gemm<256, GEMM_MUL>(what, ta, tb, tb, tb, p, N / 256, s)
                     : run_gemm<128, GEMM_MUL>(what, ta, tb, tb, tb, p, N / 128, s);
  if (mode == GEMM_STORE)
    return bn == 256 ? run_gemm<256, GEMM_STORE>(what, ta, tb, tb, tb, p, N / 256, s)
                     : run_gemm<128, GEMM_STORE>(what, ta, tb, tb, tb, p, N / 128, s);
  return bn == 256 ? run_gemm<256, GEMM_RESIDUAL>(what, ta, tb, tb, tb, p, N / 256, s)
                   : run_gemm<128, GEMM_RESIDUAL>(what, ta, tb, tb, tb, p, N / 128, s);
}

extern "C" int cb_set_gemm_workspace(void* workspace, int64_t bytes, unsigned int* tickets, int ntickets) {
  if (!workspace) {
    g_splitk_ws = nullptr;
    g_splitk_bytes = 0;
    g_splitk_tickets = nullptr;
    g_splitk_ntickets = 0;
    return kOk;
  }
  if (!aligned16(workspace) || bytes < 16 || !tickets || ntickets < 1)
    return fail(kErrInvalid, "cb_set_gemm_workspace: aligned workspace, bytes and tickets required");
  g_splitk_ws = static_cast<float*>(workspace);
  g_splitk_bytes = bytes;
  g_splitk_tickets = tickets;
  g_splitk_ntickets = ntickets;
  return kOk;
}

extern "C" int cb_gemm_split_k(int M, int K, int N, int swiglu) {
  const int mtiles = (M + kBM - 1) / kBM;
  const int bn = swiglu ? 256 : (N % 256 == 0 && int64_t(N / 256) * mtiles >= sm_count()) ? 256 : 128;
  const int ntiles = swiglu ? N / 128 : N / bn;
  return choose_ksplit(M, K, mtiles * ntiles, bn);
}

extern "C" int cb_gemm_bf16(const void* a, int M, int K, const void* w, int N, void* out, void* stream) {
  return gemm_linear("cb_gemm_bf16", GEMM_STORE, a, M, K, w, N, nullptr, out, stream);
}

extern "C" int cb_gemm_silu(const void* a, int M, const void* w_gate, int rows, void* out, void* stream) {
  return gemm_linear("cb_gemm_silu", GEMM_SILU, a, M, 4096, w_gate, rows, nullptr, out, stream);
}

extern "C" int cb_gemm_mul(const void* a, int M, const void* w_up, int rows, void* gate_act, void* stream) {
  return gemm_linear("cb_gemm_mul", GEMM_MUL, a, M, 4096, w_up, rows, nullptr, gate_act, stream);
}

extern "C" int cb_gemm_partial(const void* a, int M, int K, const void* w, int N, float* out, void* stream) {
  return gemm_linear("cb_gemm_partial", GEMM_PARTIAL, a, M, K, w, N, nullptr, out, stream);
}

extern "C" int cb_gemm_residual(const void* a, int M, int K, const void* w, int N, const void* residual, void* out,
                                void* stream) {
  return gemm_linear("cb_gemm_residual", GEMM_RESIDUAL, a, M, K, w, N, residual, out, stream);
}

extern "C" int cb_gemm_swiglu(const void* a, int M, const void* w_gate, const void* w_up, int rows, void* out,
                              void* stream) {
  const char* what = "cb_gemm_swiglu";
  if (!gemm_shape_ok(a, M, 4096, w_gate) || !w_up || !aligned16(w_up) || !out || !aligned16(out))
    return fail(kErrInvalid, "%s: a/w_gate/w_up/out must be 16-byte aligned device pointers", what);
  if (rows < 128 || rows % 128) return fail(kErrInvalid, "%s: rows=%d must be a multiple of 128", what, rows);
  CUtensorMap ta, tg, tu;
  int rc = make_tile_map(&ta, what, a, M, 4096, kBM);
  if (rc == kOk) rc = make_tile_map(&tg, what, w_gate, rows, 4096, 128);
  if (rc == kOk) rc = make_tile_map(&tu, what, w_up, rows, 4096, 128);
  if (rc != kOk) return rc;
  GemmParams p = {};
  p.M = M;
  p.N = rows;
  p.K = 4096;
  p.out = static_cast<uint16_t*>(out);
  p.ld_out = rows;
  return run_gemm<256, GEMM_SWIGLU>(what, ta, tg, tu, tu, p, rows / 128, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_prefill_qkv_rope(const void* xn, int M, const void* wq, const void* wk, const void* wv,
                                   int q_heads, int kv_heads, const float* inv_freq, const int32_t* position,
                                   void* q_out, void* k_cache, void* v_cache, int64_t cache_len, void* stream) {
  const char* what = "cb_prefill_qkv_rope";
  const void* any = wq ? wq : wk ? wk : wv;
  if (!gemm_shape_ok(xn, M, 4096, any) || (wq && !aligned16(wq)) || (wk && !aligned16(wk)) ||
      (wv && !aligned16(wv)))
    return fail(kErrInvalid, "%s: xn and the given weights must be 16-byte aligned device pointers", what);
  if (q_heads < 1 || q_heads > 32 || kv_heads < 1 || kv_heads > 8)
    return fail(kErrInvalid, "%s: %d query / %d key-value heads", what, q_heads, kv_heads);
  if (!inv_freq || !position) return fail(kErrInvalid, "%s: inv_freq and position are required", what);
  if (wq && (!q_out || !aligned16(q_out))) return fail(kErrInvalid, "%s: wq needs an aligned q_out", what);
  if ((wk && !k_cache) || (wv && !v_cache) || ((wk || wv) && cache_len < 1))
    return fail(kErrInvalid, "%s: wk / wv need their cache and cache_len", what);
  CUtensorMap ta, tq, tk, tv;
  int rc = make_tile_map(&ta, what, xn, M, 4096, kBM);
  if (rc == kOk) rc = make_tile_map(&tq, what, wq ? wq : any, int64_t(wq ? q_heads : kv_heads) * 128, 4096, 128);
  if (rc == kOk) rc = make_tile_map(&tk, what, wk ? wk : any, int64_t(wk || !wq ? kv_heads : q_heads) * 128, 4096, 128);
  if (rc == kOk) rc = make_tile_map(&tv, what, wv ? wv : any, int64_t(wv || !wq ? kv_heads : q_heads) * 128, 4096, 128);
  if (rc != kOk) return rc;
  GemmParams p = {};
  p.M = M;
  p.K = 4096;
  p.q_rows = wq ? q_heads * 128 : 0;
  p.k_rows = wk ? kv_heads * 128 : 0;
  p.v_rows = wv ? kv_heads * 128 : 0;
  p.N = p.q_rows + p.k_rows + p.v_rows;
  p.out = static_cast<uint16_t*>(q_out);
  p.ld_out = p.q_rows;
  p.inv_freq = inv_freq;
  p.pos = position;
  p.k_cache = static_cast<uint16_t*>(k_cache);
  p.v_cache = static_cast<uint16_t*>(v_cache);
  p.cache_len = cache_len;
  return run_gemm<128, GEMM_QKV_ROPE>(what, ta, tq, tk, tv, p, p.N / 128, static_cast<cudaStream_t>(stream));
}
