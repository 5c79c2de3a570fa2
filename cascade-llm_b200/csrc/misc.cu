// Small kernels and the C-ABI glue of libcascade_b200: error reporting, the
// programmatic-dependent-launch switch, seeded initialisation, embedding
// gather, stand-alone RMSNorm, top-k merge, the device position counter and
// the H2D copy used by the streamed runtime.
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "cascade_b200.h"

namespace cb {

static thread_local std::string g_last_error;
static bool g_pdl = true;
static std::atomic<uint64_t> g_exchange_wait_ns{2000000000ull};
static int32_t* g_error_word = nullptr;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(kErrCuda, "%s: %s", what, cudaGetErrorString(e));
  return kOk;
}

bool pdl_enabled() { return g_pdl; }
uint64_t exchange_wait_ns() { return g_exchange_wait_ns.load(); }

static uint64_t* g_trace = nullptr;
static std::atomic<uint32_t> g_trace_tag{0};
uint64_t* trace_buffer(uint32_t* tag) {
  if (g_trace && tag) *tag = g_trace_tag.fetch_add(1);
  return g_trace;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

int32_t* error_word() { return g_error_word; }

// Cross-kernel L2 staging (cb_set_l2_stage, cb_set_l2_stage_target): the
// issue point and size per issuing kernel kind, and the weights that
// launches issued while a target is set stage.
struct StageKnob {
  int where, take, skip, policy;
};
// Default: the attention kernel stages 10 row pairs per gate+up CTA after its
// sub-chunk loop (decode step at 2K context 3.053 -> 3.015 ms/token; every
// other issue point measured slower or no faster).
static StageKnob g_stage_knob[3] = {{0, 0, 0, 0}, {3, 10, 4, 0}, {0, 0, 0, 0}};
static L2Stage g_stage_target = {};

L2Stage l2_stage_for(int kind) {
  L2Stage s = g_stage_target;
  if (kind < 0 || kind > 2 || !s.a || g_stage_knob[kind].where == 0 || g_stage_knob[kind].take <= 0) {
    s = L2Stage{};
    return s;
  }
  s.where = g_stage_knob[kind].where;
  s.take = g_stage_knob[kind].take;
  s.skip = g_stage_knob[kind].skip;
  s.policy = g_stage_knob[kind].policy;
  return s;
}

int configure_smem_raw(const char* what, const void* kernel, size_t bytes) {
  static std::mutex lock;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(kErrCuda, "%s: no current device", what);
  std::lock_guard<std::mutex> guard(lock);
  if (done.count({kernel, dev})) return kOk;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e != cudaSuccess) return fail(kErrCuda, "%s: shared-memory attribute: %s", what, cudaGetErrorString(e));
  done.insert({kernel, dev});
  return kOk;
}

// ------------------------------------------------------------ seeded init
// Counter-based N(0, std) generator (same definition as the CPU oracle):
// key = splitmix64(seed ^ fnv1a64(name)); element i uses the uniforms of
// pair i>>1 in a double-precision Box-Muller transform, then fp32, then
// bf16 round-to-nearest-even.
__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ULL;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
  return x ^ (x >> 31);
}

__global__ void fill_normal_kernel(uint16_t* out, int64_t n, int64_t offset, uint64_t key,
                                   double std_dev) {
  for (int64_t j = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; j < n;
       j += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = offset + j;
    const uint64_t pr = uint64_t(i) >> 1;
    const uint64_t a = splitmix64(key + 2 * pr);
    const uint64_t b = splitmix64(key + 2 * pr + 1);
    const double u1 = __dmul_rn(double((a >> 11) + 1), 0x1.0p-53);
    const double u2 = __dmul_rn(double(b >> 11), 0x1.0p-53);
    const double r = sqrt(__dmul_rn(-2.0, log(u1)));
    const double t = __dmul_rn(6.283185307179586, u2);
    const double z = (i & 1) ? __dmul_rn(r, sin(t)) : __dmul_rn(r, cos(t));
    const float f = __double2float_rn(__dmul_rn(z, std_dev));
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);
    out[j] = uint16_t(u >> 16);
  }
}

__global__ void fill_value_kernel(uint16_t* out, int64_t n, uint16_t bits) {
  for (int64_t j = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; j < n;
       j += int64_t(gridDim.x) * blockDim.x)
    out[j] = bits;
}

// ------------------------------------------------------------ embedding
__global__ void embedding_kernel(const int64_t* ids, const uint16_t* table, int64_t vocab, int hidden,
                                 uint16_t* out, int* err) {
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_launch();
  const int m = blockIdx.x;
  int64_t id = __ldcg(reinterpret_cast<const long long*>(ids) + m);
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && err) atomicExch(err, 301);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + int64_t(m) * hidden);
  for (int c = threadIdx.x; c < hidden / 8; c += blockDim.x) dst[c] = __ldg(src + c);
}

// ------------------------------------------------------------ rmsnorm
__global__ void rmsnorm_kernel(const uint16_t* x, const uint16_t* w, int hidden, float eps,
                               uint16_t* out) {
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_launch();
  __shared__ float red[32];
  const int m = blockIdx.x;
  const uint16_t* row = x + int64_t(m) * hidden;
  float ss = 0.f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float v = bf16f(__ldcg(row + c));
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < int(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / float(hidden) + eps);
  for (int c = threadIdx.x; c < hidden; c += blockDim.x)
    out[int64_t(m) * hidden + c] = f2bf(bf16f(__ldg(w + c)) * rbf(bf16f(__ldcg(row + c)) * inv));
}

// ------------------------------------------------------------ top-k merge
__device__ __forceinline__ bool before(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

// One warp: k rounds, each picking the best candidate ranked after the last.
__global__ void topk_merge_kernel(const float* av, const int64_t* ai, int na, const float* bv,
                                  const int64_t* bi, int nb, int k, float* ov, int64_t* oi) {
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_launch();
  const int lane = threadIdx.x;
  const int n = na + nb;
  float pv = __int_as_float(0x7F800000);
  int64_t pi = -1;
  for (int r = 0; r < k; ++r) {
    float best_v = -__int_as_float(0x7F800000);
    int64_t best_i = INT64_MAX;
    bool have = false;
    for (int c = lane; c < n; c += 32) {
      const float v = c < na ? __ldcg(av + c) : __ldcg(bv + (c - na));
      const int64_t i = c < na ? __ldcg(reinterpret_cast<const long long*>(ai) + c)
                               : __ldcg(reinterpret_cast<const long long*>(bi) + (c - na));
      if (before(pv, pi, v, i) && (!have || before(v, i, best_v, best_i))) {
        best_v = v;
        best_i = i;
        have = true;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xFFFFFFFFu, best_v, o);
      const int64_t i2 = __shfl_xor_sync(0xFFFFFFFFu, best_i, o);
      if (before(v2, i2, best_v, best_i)) {
        best_v = v2;
        best_i = i2;
      }
    }
    if (lane == 0) {
      ov[r] = best_v;
      oi[r] = best_i;
    }
    pv = best_v;
    pi = best_i;
  }
}

// ------------------------------------------------------------ residual
// x + F.linear(...) when the projection's fp32 sum was assembled across
// tensor-parallel ranks: out = bf16(x + bf16(sum)).
__global__ void residual_add_kernel(const uint16_t* x, const float* sum, int n, uint16_t* out) {
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = f2bf(bf16f(__ldcg(x + i)) + rbf(__ldcg(sum + i)));
}

// ------------------------------------------------------------ position
__global__ void position_kernel(int32_t* pos, const int64_t* src, int32_t value, int32_t add) {
  grid_dep_wait();
  if (src)
    *pos = int32_t(__ldcg(reinterpret_cast<const long long*>(src)));
  else if (add)
    *pos = __ldcg(pos) + add;
  else
    *pos = value;
}

}  // namespace cb

using namespace cb;

extern "C" int cb_version(void) { return 100; }
extern "C" const char* cb_last_error(void) { return g_last_error.c_str(); }
extern "C" int cb_set_pdl(int enable) {
  const int prev = g_pdl ? 1 : 0;
  g_pdl = enable != 0;
  return prev;
}
extern "C" int cb_set_trace(void* device_buffer) {
  g_trace = static_cast<uint64_t*>(device_buffer);
  g_trace_tag = 0;
  return kOk;
}
extern "C" uint64_t cb_set_exchange_wait_ns(uint64_t ns) {
  return g_exchange_wait_ns.exchange(ns ? ns : 2000000000ull);
}
extern "C" int cb_sm_count(void) { return sm_count(); }
extern "C" int cb_set_l2_stage(int kind, int where, int take, int skip, int policy) {
  if (kind < 0 || kind > 2 || where < 0 || where > 4 || take < 0 || skip < 0 || policy < 0 || policy > 1)
    return fail(kErrInvalid, "cb_set_l2_stage: kind=%d where=%d take=%d skip=%d policy=%d", kind, where, take,
                skip, policy);
  g_stage_knob[kind] = StageKnob{where, take, skip, policy};
  return kOk;
}
extern "C" int cb_set_l2_stage_target(const void* w_a, const void* w_b, int units, int K) {
  if (!w_a) {
    g_stage_target = L2Stage{};
    return kOk;
  }
  if (!w_b || units < 1 || K < 8 || K % 8 || !aligned16(w_a) || !aligned16(w_b) ||
      int64_t(units) * (gemv_grid_size() + 1) >= (int64_t(1) << 32) || int64_t(units) * K * 2 >= (int64_t(1) << 32))
    return fail(kErrInvalid, "cb_set_l2_stage_target: bad slabs (units=%d, K=%d)", units, K);
  L2Stage s = {};
  s.a = static_cast<const uint8_t*>(w_a);
  s.b = static_cast<const uint8_t*>(w_b);
  s.row_bytes = int64_t(K) * 2;
  s.units = units;
  s.ncta = gemv_grid_size();
  g_stage_target = s;
  return kOk;
}
extern "C" int cb_prepare(void) {
  int rc = prepare_gemv();
  if (rc == kOk) rc = prepare_attention();
  if (rc == kOk) rc = prepare_attention_oproj();
  if (rc == kOk) rc = prepare_gemm();
  if (rc == kOk) rc = prepare_prefill_attention();
  if (rc == kOk) rc = prepare_prefill_attention_tc();
  return rc;
}
extern "C" int cb_set_error_word(int32_t* device_word) {
  g_error_word = device_word;
  return kOk;
}

extern "C" uint64_t cb_stream_key(uint64_t seed, const char* tensor_name) {
  uint64_t h = 0xCBF29CE484222325ULL;
  for (const char* s = tensor_name; s && *s; ++s) {
    h ^= uint8_t(*s);
    h *= 0x100000001B3ULL;
  }
  return splitmix64(seed ^ h);
}

static dim3 fill_grid(int64_t n) {
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 16;
  return dim3(unsigned(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap));
}

extern "C" int cb_fill_normal_bf16(void* out, int64_t n, int64_t offset, uint64_t key, double std_dev,
                                   void* stream) {
  if (!out || n < 0 || offset < 0) return fail(kErrInvalid, "cb_fill_normal_bf16: bad arguments");
  if (n == 0) return kOk;
  return launch("cb_fill_normal_bf16", fill_normal_kernel, fill_grid(n), dim3(256), 0,
                static_cast<cudaStream_t>(stream), static_cast<uint16_t*>(out), n, offset, key,
                std_dev);
}

extern "C" int cb_fill_bf16(void* out, int64_t n, float value, void* stream) {
  if (!out || n < 0) return fail(kErrInvalid, "cb_fill_bf16: bad arguments");
  if (n == 0) return kOk;
  uint32_t u;
  std::memcpy(&u, &value, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return launch("cb_fill_bf16", fill_value_kernel, fill_grid(n), dim3(256), 0,
                static_cast<cudaStream_t>(stream), static_cast<uint16_t*>(out), n,
                uint16_t(u >> 16));
}

extern "C" int cb_embedding(const int64_t* ids, int M, const void* table, int64_t vocab, int hidden,
                            void* out, void* stream) {
  if (!ids || !table || !out || M < 1 || M > 65535 || vocab < 1)
    return fail(kErrInvalid, "cb_embedding: bad arguments");
  if (hidden % 8 || !aligned16(table) || !aligned16(out))
    return fail(kErrInvalid, "cb_embedding: rows must be 16-byte aligned multiples of 8 elements");
  return launch("cb_embedding", embedding_kernel, dim3(M), dim3(256), 0,
                static_cast<cudaStream_t>(stream), ids, static_cast<const uint16_t*>(table), vocab,
                hidden, static_cast<uint16_t*>(out), error_word());
}

extern "C" int cb_rmsnorm(const void* x, const void* w, int M, int hidden, float eps, void* out,
                          void* stream) {
  if (!x || !w || !out || M < 1 || M > 65535 || hidden < 1)
    return fail(kErrInvalid, "cb_rmsnorm: bad arguments");
  return launch("cb_rmsnorm", rmsnorm_kernel, dim3(M), dim3(512), 0,
                static_cast<cudaStream_t>(stream), static_cast<const uint16_t*>(x),
                static_cast<const uint16_t*>(w), hidden, eps, static_cast<uint16_t*>(out));
}

extern "C" int cb_topk_merge(const float* a_values, const int64_t* a_indices, int na,
                             const float* b_values, const int64_t* b_indices, int nb, int k,
                             float* out_values, int64_t* out_indices, void* stream) {
  if (na < 0 || nb < 0 || (na && (!a_values || !a_indices)) || (nb && (!b_values || !b_indices)))
    return fail(kErrInvalid, "cb_topk_merge: bad candidate arrays");
  if (k < 1 || k > 64 || k > na + nb) return fail(kErrInvalid, "cb_topk_merge: need 1 <= k <= min(64, na+nb)");
  if (!out_values || !out_indices) return fail(kErrInvalid, "cb_topk_merge: null output");
  return launch("cb_topk_merge", topk_merge_kernel, dim3(1), dim3(32), 0,
                static_cast<cudaStream_t>(stream), a_values, a_indices, na, b_values, b_indices, nb,
                k, out_values, out_indices);
}

extern "C" int cb_residual_add_f32(const void* x, const float* sum, int n, void* out, void* stream) {
  if (!x || !sum || !out || n < 1) return fail(kErrInvalid, "cb_residual_add_f32: bad arguments");
  return launch("cb_residual_add_f32", residual_add_kernel, dim3((n + 255) / 256), dim3(256), 0,
                static_cast<cudaStream_t>(stream), static_cast<const uint16_t*>(x), sum, n,
                static_cast<uint16_t*>(out));
}

extern "C" int cb_position_set(int32_t* position, const int64_t* src, int32_t value, void* stream) {
  if (!position) return fail(kErrInvalid, "cb_position_set: null position");
  return launch("cb_position_set", position_kernel, dim3(1), dim3(1), 0,
                static_cast<cudaStream_t>(stream), position, src, value, int32_t(0));
}

extern "C" int cb_position_advance(int32_t* position, int32_t count, void* stream) {
  if (!position || count < 1) return fail(kErrInvalid, "cb_position_advance: bad arguments");
  return launch("cb_position_advance", position_kernel, dim3(1), dim3(1), 0,
                static_cast<cudaStream_t>(stream), position, static_cast<const int64_t*>(nullptr),
                int32_t(0), count);
}

extern "C" int cb_memcpy_h2d_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (!dst || !src || bytes < 0) return fail(kErrInvalid, "cb_memcpy_h2d_async: bad arguments");
  if (bytes == 0) return kOk;
  cudaError_t e = cudaMemcpyAsync(dst, src, size_t(bytes), cudaMemcpyHostToDevice,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(kErrCuda, "cb_memcpy_h2d_async: %s", cudaGetErrorString(e));
  return kOk;
}
