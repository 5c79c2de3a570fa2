// Split-KV GQA attention (flash-decoding) for sm_100a.
//
// Replaces layer_streaming/llama31.py:182-234: `_repeat_kv` (a 4x copy of
// K/V) + F.scaled_dot_product_attention. Here the 4 query heads of a KV head
// share ONE read of every K/V row: a CTA owns (split s, kv head g, token m)
// and streams its positions [s*chunk, s*chunk + chunk) in 64-position
// sub-chunks through a 3-stage cp.async.bulk ring. Each of the 8 compute
// warps owns 8 rows of every sub-chunk and runs its own online softmax over
// them (fp32; scores scaled by 1/sqrt(128)), with no barrier between warps
// until the end: then the warps' (m, l, o) are combined in shared memory,
// each CTA writes (m, l, o[128]) per head, and the last CTA of a (token, kv
// head) group (atomic ticket) merges the splits and writes the bf16 output.
//
// Causality: token m of a step starting at position P0 sees [0, P0 + m].
// Rows of the history (< P0) are fetched before griddepcontrol.wait: they were
// written by earlier steps. Rows >= P0 were written by this step's QKV
// kernel and are fetched only after the wait.
#include <mutex>

#include "attention_device.cuh"
#include "common.cuh"
#include "internal.h"
#include "cascade_b200.h"

namespace cb {

int32_t* error_word();

__global__ void __launch_bounds__(kAttnThreads, 2) attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  attention_cta(p, blockIdx.x, blockIdx.y, blockIdx.z, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                smem);
}

// The same attention with the splits of a (token, KV head) merged inside a
// thread-block cluster through distributed shared memory (M = 1, splits <=
// 16): no global partials and no last-CTA ticket. Bit-identical outputs.
__global__ void __launch_bounds__(kAttnThreads, 2) attention_cluster_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  attention_cta<true>(p, blockIdx.x, blockIdx.y, blockIdx.z,
                      (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x, smem);
}

static bool g_cluster_merge = true;
static int g_min_chunk = 0;  // 0: kMinChunk

// Launches attention_cluster_kernel; returns kErrUnsupported (nothing
// launched) when the device cannot hold a cluster of `splits` CTAs.
static int launch_cluster(const AttnParams& p, int splits, int kv_heads, cudaStream_t stream) {
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    if (cudaFuncSetAttribute(attention_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
            cudaSuccess ||
        cudaFuncSetAttribute(attention_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(AttnSmem::BYTES)) != cudaSuccess) {
      cudaGetLastError();
      return kErrUnsupported;
    }
    configured_device = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, kv_heads, 1);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = AttnSmem::BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int n = 1;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, attention_cluster_kernel, &cfg) != cudaSuccess || clusters < 1) {
    cudaGetLastError();
    return kErrUnsupported;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, attention_cluster_kernel, p);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_attention: cluster launch failed: %s", cudaGetErrorString(e));
  return check_launch("cb_attention");
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
                            int64_t cache_len, const int32_t* position, int M, int kv_heads, int splits,
                            int chunk, void* out, void* workspace, unsigned int* tickets, void* stream) {
  if (kv_heads < 1 || kv_heads > 8) return fail(kErrInvalid, "cb_attention: kv_heads=%d (1..8)", kv_heads);
  if (!q || !k_cache || !v_cache || !position || !out || !workspace || !tickets)
    return fail(kErrInvalid, "cb_attention: null pointer");
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(q))
    return fail(kErrInvalid, "cb_attention: q/k_cache/v_cache must be 16-byte aligned");
  if (M < 1 || M > 65535) return fail(kErrInvalid, "cb_attention: M=%d out of range", M);
  if (splits < 1 || splits > 65535) return fail(kErrInvalid, "cb_attention: splits=%d", splits);
  if (chunk < 0 || chunk % kSub) return fail(kErrInvalid, "cb_attention: chunk must be 0 or a multiple of 64");
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
  p.kv_heads = kv_heads;
  p.splits = splits;
  p.chunk = chunk;
  p.out = static_cast<uint16_t*>(out);
  const int64_t rows = int64_t(M) * kv_heads * kGroup * splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float*>(ws + rows * kHeadDim * 4);
  p.tickets = tickets;
  p.err = error_word();
  p.trace = trace_buffer(&p.trace_tag);
  if (M == 1) p.stage = l2_stage_for(1);
  p.min_chunk = g_min_chunk;
  if (g_cluster_merge && M == 1 && splits <= kClusterMaxSplits) {
    const int crc = launch_cluster(p, splits, kv_heads, static_cast<cudaStream_t>(stream));
    if (crc != kErrUnsupported) return crc;
  }
  return launch("cb_attention", attention_kernel, dim3(splits, kv_heads, M), dim3(kAttnThreads),
                AttnSmem::BYTES, static_cast<cudaStream_t>(stream), p);
}

extern "C" int cb_set_attention_min_chunk(int positions) {
  if (positions < 0 || positions % kSub) return -1;
  const int previous = g_min_chunk ? g_min_chunk : int(kMinChunk);
  g_min_chunk = positions;
  return previous;
}

extern "C" int cb_set_attention_cluster(int enable) {
  const int previous = g_cluster_merge ? 1 : 0;
  g_cluster_merge = enable != 0;
  return previous;
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
  return cb_attention(q, k_cache, v_cache, cache_len, position, M, 8, splits, chunk, out, scratch->partials,
                      scratch->tickets, stream);
}
