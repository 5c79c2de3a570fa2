// Host-side helpers shared by the .cu files of libcascade_b200 (not part of
// the C ABI): error recording and kernel launch with optional programmatic
// dependent launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

// Argument check of a C-ABI entry point: records the message and returns
// CB_ERR_INVALID before anything is launched.
#define CB_REQUIRE(cond, ...)                                 \
  do {                                                        \
    if (!(cond)) return ::cb::fail(::cb::kErrInvalid, __VA_ARGS__); \
  } while (0)

namespace cb {

// Error codes returned by every cb_* entry point.
enum Status : int {
  kOk = 0,
  kErrInvalid = 1,   // bad argument (shape, alignment, null pointer, range)
  kErrCuda = 2,      // a CUDA runtime call or launch failed
  kErrUnsupported = 3,
};

void set_error(const std::string& msg);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
bool pdl_enabled();
// Wall-clock limit of the tensor-parallel exchange waits (cb_set_exchange_wait_ns).
uint64_t exchange_wait_ns();
int sm_count();
// Grid of every GEMV launch (two CTAs per SM).
int gemv_grid_size();
// The launch-trace buffer set by cb_set_trace (null: tracing off) and, when
// set, the next launch tag.
uint64_t* trace_buffer(uint32_t* tag);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raise a kernel's dynamic shared-memory limit once per (kernel, device)
// (the attribute is per device context). Not a stream operation, so it is
// also safe while a stream is being captured; cb_prepare() does it up front.
int configure_smem_raw(const char* what, const void* kernel, size_t bytes);
template <typename... KArgs>
int configure_smem(const char* what, void (*kernel)(KArgs...), size_t bytes) {
  return configure_smem_raw(what, reinterpret_cast<const void*>(kernel), bytes);
}

int prepare_gemv();
int prepare_attention();
int prepare_attention_oproj();
int prepare_gemm();
int prepare_prefill_attention();
int prepare_prefill_attention_tc();
int run_prefill_attention_tc(const void* q, const void* k_cache, const void* v_cache, int64_t cache_len,
                             const int32_t* position, int M, int kv_heads, void* out, cudaStream_t stream);

// Launch `kernel<<<grid, block, smem, stream>>>(args...)` through
// cudaLaunchKernelEx, adding the programmatic-stream-serialization attribute
// when programmatic dependent launch is enabled: the kernel may then start
// while its predecessor drains and must call griddepcontrol.wait before it
// touches anything the predecessor writes.
template <typename... KArgs, typename... Args>
int launch(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(kErrCuda, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

}  // namespace cb
