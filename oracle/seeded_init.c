/*
 * TEST INFRASTRUCTURE ONLY (oracle). Nothing in the product links or loads
 * this file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg use it, as the checker.
 *
 * CPU restatement of the engine's seeded weight initialiser
 * (cascade-llm_b200/csrc/init_kernels.cu, `cb_fill_normal_bf16`). The
 * reference has no initialiser of its own: it loads a real checkpoint
 * (layer_streaming/weight_store.py:109-171). The random-init weights of the
 * benchmark configurations ("weights N(0,0.02), norm weights 1") are defined
 * by this counter-based generator so that a CPU process and a GPU produce
 * the same BF16 bits for every element, independently of thread count:
 *
 *   key      = splitmix64(seed ^ fnv1a64(tensor_name))
 *   pair p   = i >> 1
 *   a, b     = splitmix64(key + 2p), splitmix64(key + 2p + 1)
 *   u1       = ((a >> 11) + 1) * 2^-53          in (0, 1]
 *   u2       = (b >> 11) * 2^-53                in [0, 1)
 *   r        = sqrt(-2 ln u1),  t = 2*pi*u2      (double precision)
 *   z        = i even ? r cos t : r sin t       (Box-Muller)
 *   value    = bf16_rne((float)(z * std))
 *
 * The double-precision transcendental functions of glibc and of CUDA agree
 * to within one ulp, so a BF16 result can differ only when z*std lies within
 * ~1e-16 (relative) of a BF16 rounding boundary: about one element in 1e13.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ULL;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
  return x ^ (x >> 31);
}

uint64_t oracle_fnv1a64(const char* s) {
  uint64_t h = 0xCBF29CE484222325ULL;
  for (; *s; ++s) {
    h ^= (uint8_t)*s;
    h *= 0x100000001B3ULL;
  }
  return h;
}

uint64_t oracle_stream_key(uint64_t seed, const char* name) {
  return splitmix64(seed ^ oracle_fnv1a64(name));
}

static inline uint16_t bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline uint16_t normal_bf16(uint64_t key, int64_t i, double std_dev) {
  const uint64_t p = (uint64_t)i >> 1;
  const uint64_t a = splitmix64(key + 2 * p);
  const uint64_t b = splitmix64(key + 2 * p + 1);
  const double u1 = (double)((a >> 11) + 1) * 0x1.0p-53;
  const double u2 = (double)(b >> 11) * 0x1.0p-53;
  const double r = sqrt(-2.0 * log(u1));
  const double t = 6.283185307179586 * u2;
  const double z = (i & 1) ? r * sin(t) : r * cos(t);
  return bf16_rne((float)(z * std_dev));
}

/* Fills out[0..n) with elements [offset, offset + n) of the stream. Callers
 * parallelise by splitting [0, n) (ctypes releases the GIL). */
void oracle_fill_normal_bf16(uint16_t* out, int64_t n, int64_t offset,
                             uint64_t key, double std_dev) {
  for (int64_t j = 0; j < n; ++j) out[j] = normal_bf16(key, offset + j, std_dev);
}

/* Uniform integers in [0, bound): ((splitmix64(key + i) >> 32) * bound) >> 32. */
void oracle_uniform_ids(int64_t* out, int64_t n, uint64_t key, uint32_t bound) {
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t h = splitmix64(key + (uint64_t)i) >> 32;
    out[i] = (int64_t)((h * (uint64_t)bound) >> 32);
  }
}
