// Shared device helpers for the sm_100a kernels of the decode engine.
//
// Everything here is hand-written PTX or plain CUDA: BF16 bit conversions,
// mbarrier + cp.async.bulk (TMA bulk copy, global -> this CTA's shared memory)
// wrappers, and programmatic-dependent-launch controls (griddepcontrol).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cb {

// ---------------------------------------------------------------- bf16 bits
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16f(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }

// Round-to-nearest-even fp32 -> bf16 (inputs are finite in this engine;
// NaN is kept a NaN by forcing a mantissa bit).
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return uint16_t((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
// fp32 value of the bf16 rounding of f (one torch bf16 op result).
__device__ __forceinline__ float rbf(float f) { return bf16f(f2bf(f)); }

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait: every spin in this engine gives up after `limit` polls,
// records the failure in *err (if given) and returns false, so a lost
// arrival can never hang the GPU. try_wait itself suspends for a
// hardware-defined interval, so the bound is a wall-clock bound of roughly
// limit x (suspend time); 1<<22 polls is well above a second.
constexpr uint32_t kSpinLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicExch(err, code);
  return false;
}

// ------------------------------------------------- bulk copy (TMA, untiled)
// Global -> shared::cta copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned) that completes `bytes` transactions on `bar`. Every CTA
// fetches its own data into its own shared memory.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same, with an L2 eviction-priority hint: weights are streamed exactly once
// per token, so they are marked evict_first to keep L2 for activations.
__device__ __forceinline__ void bulk_g2s_stream(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                                uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
      "[%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Bulk prefetch of [src, src + bytes) into L2 (16-byte aligned, multiple of
// 16 bytes): no destination, no completion, no registers held.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_prefetch_l2_hint(const void* src, uint32_t bytes, uint64_t policy) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(policy)
               : "memory");
}

// ------------------------------------------- cross-kernel L2 staging
// A decode layer is a chain of five dependent kernels; three of them (QKV,
// attention, o_proj) are latency-bound and leave most of the HBM bandwidth
// idle, while the fourth (gate+up, 235 MB of weights) is bandwidth-bound.
// An L2Stage names a slice of that later launch's weights, which the earlier
// kernels prefetch into L2 while HBM would otherwise idle. The slabs are the
// consumer launch's two row-major weight matrices (gate rows, up rows), split
// into `units` row pairs over `ncta` CTAs exactly as the consumer splits them;
// consumer CTA c's units [u0 + skip, u0 + skip + take) of both slabs are
// staged (u0 = its first unit; skip = the units it loads before its
// dependency wait anyway). take == 0 or where == 0: nothing is staged.
struct L2Stage {
  const uint8_t* a;   // slab A (gate rows)
  const uint8_t* b;   // slab B (up rows)
  int64_t row_bytes;  // bytes per weight row
  int units, ncta, skip, take;
  int where;          // issue point inside the issuing kernel (kernel-specific; 0 = off)
  int policy;         // 0: normal L2 priority, 1: evict_last
};

// Issue the ranges of issuing CTA i of n, thread t of the nt issuing threads
// (two ranges, one per slab, per consumer CTA c = i, i + n, ...).
__device__ __forceinline__ void l2_stage_issue(const L2Stage& s, int i, int n, int t, int nt) {
  if (s.take <= 0 || s.where == 0) return;
  const unsigned per = (unsigned(s.ncta) + unsigned(n) - 1u) / unsigned(n);
  for (unsigned r = unsigned(t); r < 2u * per; r += unsigned(nt)) {
    const unsigned c = unsigned(i) + unsigned(n) * (r >> 1);
    if (c >= unsigned(s.ncta)) break;
    // units * ncta < 2^32 (checked on the host): 32-bit arithmetic
    const unsigned u0 = unsigned(s.units) * c / unsigned(s.ncta);
    const unsigned u1 = unsigned(s.units) * (c + 1u) / unsigned(s.ncta);
    const unsigned lo = min(u0 + unsigned(s.skip), u1), hi = min(lo + unsigned(s.take), u1);
    if (hi <= lo) continue;
    const uint8_t* src = ((r & 1u) ? s.b : s.a) + size_t(lo) * size_t(s.row_bytes);
    const uint32_t bytes = (hi - lo) * uint32_t(s.row_bytes);
    if (s.policy == 1)
      bulk_prefetch_l2_hint(src, bytes, policy_evict_last());
    else
      bulk_prefetch_l2(src, bytes);
  }
}

// Host side (misc.cu): the staging slice that a launch of `kind` (0 QKV,
// 1 attention, 2 o_proj) carries, from cb_set_l2_stage / _target.
L2Stage l2_stage_for(int kind);

// ------------------------------------------ programmatic dependent launch
// wait: block until every prerequisite grid has completed and its memory is
// visible. launch: allow the dependent grid to be scheduled. Both are no-ops
// for a kernel launched without the programmatic-serialization attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------- flags between GPUs (system scope)
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Tagged words: a 32-bit payload and the 32-bit sequence number of the
// exchange that wrote it, stored as ONE aligned 64-bit word. A 64-bit scalar
// access is single-copy atomic, so a reader that sees the expected tag sees
// that exchange's payload: no fence or separate flag is needed, and each
// reader waits for exactly the words it consumes.
__device__ __forceinline__ uint64_t tag_word(uint32_t payload, uint32_t tag) {
  return (uint64_t(tag) << 32) | payload;
}
__device__ __forceinline__ void st_tagged(uint64_t* p, uint64_t word) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(word) : "memory");
}
__device__ __forceinline__ uint64_t ld_tagged(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Wait until the word at p carries `tag`, for at most `limit_ns` of wall
// clock and kSpinLimit x 16 polls, whichever ends first; returns the payload
// and sets *timed_out on time-out (the payload is then undefined). Once
// *timed_out is set, later calls of the same thread only look once, so a
// missing peer costs one limit per thread, not one per awaited word.
__device__ __forceinline__ uint32_t wait_tagged(const uint64_t* p, uint32_t tag, uint64_t limit_ns,
                                                bool* timed_out) {
  uint64_t w = ld_tagged(p);
  if (uint32_t(w >> 32) == tag || *timed_out) return uint32_t(w);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (kSpinLimit << 4); ++i) {
    w = ld_tagged(p);
    if (uint32_t(w >> 32) == tag) return uint32_t(w);
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > limit_ns) break;
  }
  *timed_out = true;
  return uint32_t(w);
}

// ------------------------------------------------------- launch tracing
// Optional per-CTA timeline of the engine's kernels (cb_set_trace): buffer
// word 0 is the record cursor, word 1 the capacity in records; record r
// (8 words at 8 * (r + 1)) holds the launch tag << 32 | CTA index, the SM,
// and %globaltimer at CTA start, after the dependency wait, after the main
// loop and at the end, then two kernel-specific points (the LM head: its
// CTA's top-k selected, its ticket taken). A null buffer records nothing.
__device__ __forceinline__ uint32_t smid_u32() {
  uint32_t v;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(v));
  return v;
}
__device__ __forceinline__ uint64_t trace_now(const uint64_t* trace) { return trace ? globaltimer_ns() : 0; }
__device__ __forceinline__ void trace_commit(uint64_t* trace, uint32_t tag, uint32_t cta, uint64_t t0, uint64_t t1,
                                             uint64_t t2, uint64_t x0 = 0, uint64_t x1 = 0) {
  if (!trace) return;
  const uint64_t t3 = globaltimer_ns();
  const unsigned long long slot = atomicAdd(reinterpret_cast<unsigned long long*>(trace), 1ull);
  if (slot >= trace[1]) return;
  uint64_t* r = trace + 8 * (slot + 1);
  r[0] = (uint64_t(tag) << 32) | cta;
  r[1] = smid_u32();
  r[2] = t0;
  r[3] = t1;
  r[4] = t2;
  r[5] = t3;
  r[6] = x0;  // kernel-specific extra points (0: none)
  r[7] = x1;
}

// ------------------------------------------------------------ loads/stores
// Activations written by an earlier kernel are read through L2 only (.cg):
// with overlapping dependent launches no stale L1 line can be hit.
__device__ __forceinline__ uint4 ld_cg_u4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
// Ticket counter of a CTA group at GPU scope with acquire-release semantics:
// called by one thread after a barrier of its CTA, it publishes every write
// the CTA made before the barrier (release is cumulative over the barrier)
// and orders the CTA's later reads, after another barrier, behind the writes
// of the CTAs that took earlier tickets.
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Release-ordered increment of a counter at GPU scope (the other side polls
// it with ld_acquire_gpu). Called by one thread after a CTA barrier, it
// publishes every write the CTA made before the barrier.
__device__ __forceinline__ void red_add_release_gpu(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_relaxed_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Named barrier over `count` threads (multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// torch's silu on a bf16 tensor: x / (1 + exp(-x)) in fp32, rounded to bf16
__device__ __forceinline__ float silu_bf16(float g) { return rbf(g / (1.0f + expf(-g))); }

// RoPE of one (d, d+64) pair of a head at position `pos` (transformers
// modeling_llama.py:124-168): the projection outputs a, b are rounded to bf16,
// cos/sin of (inv_freq[d] * pos) in fp32 are cast to bf16, and
// q*cos + rotate_half(q)*sin is evaluated with a bf16 rounding after each op.
__device__ __forceinline__ void rope_pair(float a, float b, float inv_freq_d, int pos, uint16_t& out_a,
                                          uint16_t& out_b) {
  const float freq = inv_freq_d * float(pos);
  // one sincosf (a shared range reduction) instead of cosf + sinf: half the
  // trigonometric code in the epilogues, which measured QKV prefill GEMM
  // 173 -> 107 us at M = 2048 (the separate calls stalled instruction fetch)
  float sv, cv;
  sincosf(freq, &sv, &cv);
  const float c = rbf(cv), s = rbf(sv);
  const float qa = rbf(a), qb = rbf(b);
  out_a = f2bf(rbf(qa * c) + rbf(-qb * s));
  out_b = f2bf(rbf(qb * c) + rbf(qa * s));
}

// dot of 8 bf16 weights with 8 bf16 activations, accumulated in fp32
__device__ __forceinline__ float dot8(const uint4 w, const uint4 x, float acc) {
  acc = fmaf(bf16lo(w.x), bf16lo(x.x), acc);
  acc = fmaf(bf16hi(w.x), bf16hi(x.x), acc);
  acc = fmaf(bf16lo(w.y), bf16lo(x.y), acc);
  acc = fmaf(bf16hi(w.y), bf16hi(x.y), acc);
  acc = fmaf(bf16lo(w.z), bf16lo(x.z), acc);
  acc = fmaf(bf16hi(w.z), bf16hi(x.z), acc);
  acc = fmaf(bf16lo(w.w), bf16lo(x.w), acc);
  acc = fmaf(bf16hi(w.w), bf16hi(x.w), acc);
  return acc;
}

// ------------------------------------------------------------ int8 weights
// Exact fp32 value of signed byte b of w: byte b of (w ^ 0x80808080) is
// b + 128 in [0, 255]; one byte permute places it under the exponent of
// 2^23 (0x4B0000bb = 2^23 + b + 128), and subtracting 2^23 + 128 leaves b,
// exactly (every integer below 2^24 is a float). One PRMT and one FADD per
// weight instead of an integer-to-float conversion.
template <int B>
__device__ __forceinline__ float i8_at(uint32_t biased) {
  return __uint_as_float(__byte_perm(biased, 0x4B000000u, 0x7440u | B)) - 8388736.0f;
}

// Dot product of 8 int8 weights (two words) with 8 bf16 activations on packed
// fp32 pairs (sm_100 f32x2 arithmetic): each permuted byte pair becomes two
// exact integers with one add.rn.f32x2, and one fma.rn.f32x2 accumulates
// even and odd elements side by side into `acc` {even, odd} - 18
// instructions per 8 weights instead of 26 with scalar arithmetic.
__device__ __forceinline__ uint64_t i8_pair(uint32_t biased, int sel_lo, int sel_hi) {
  const uint32_t lo = __byte_perm(biased, 0x4B000000u, 0x7440u | sel_lo);
  const uint32_t hi = __byte_perm(biased, 0x4B000000u, 0x7440u | sel_hi);
  uint64_t p, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(p) : "r"(lo), "r"(hi));
  // 0xCB000080 = -8388736.0f (2^23 + 128) in both halves
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(p), "l"(0xCB000080CB000080ull));
  return d;
}
__device__ __forceinline__ uint64_t bf16_pair(uint32_t w) {
  uint64_t p;
  asm("mov.b64 %0, {%1, %2};" : "=l"(p) : "r"(w << 16), "r"(w & 0xFFFF0000u));
  return p;
}
__device__ __forceinline__ uint64_t dot8_i8x2(const uint2 w, const uint4 x, uint64_t acc) {
  const uint32_t w0 = w.x ^ 0x80808080u, w1 = w.y ^ 0x80808080u;
  auto fma2 = [](uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
  };
  acc = fma2(i8_pair(w0, 0, 1), bf16_pair(x.x), acc);
  acc = fma2(i8_pair(w0, 2, 3), bf16_pair(x.y), acc);
  acc = fma2(i8_pair(w1, 0, 1), bf16_pair(x.z), acc);
  acc = fma2(i8_pair(w1, 2, 3), bf16_pair(x.w), acc);
  return acc;
}
__device__ __forceinline__ float f2sum(uint64_t v) {
  return __uint_as_float(uint32_t(v)) + __uint_as_float(uint32_t(v >> 32));
}

// 8-byte streaming load (8 int8 weights), not cached in L1.
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

}  // namespace cb
