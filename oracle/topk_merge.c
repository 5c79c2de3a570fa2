/*
 * TEST INFRASTRUCTURE ONLY (oracle). Nothing in the product links or loads
 * this file.
 *
 * CPU restatement of the exact top-k used by the LM head
 * (layer_streaming/vocab.py:11-32 `merge_topk`, and the per-chunk
 * `torch.topk` at vocab.py:247-253 / llama31.py:335-339). The reference's
 * result is "the k largest logits"; torch.topk leaves the order of equal
 * values unspecified, so the oracle fixes it: larger value first, then
 * smaller vocabulary index first. The CUDA kernels use the same order, and
 * the parity tests compare positions only where the values differ.
 */
#include <stdint.h>

/* a ranks before b */
static inline int ranks_before(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

/*
 * Exact top-k of n candidates (values[], indices[]); writes k results
 * (k <= n) to out_values/out_indices in rank order. Insertion into a sorted
 * list of length k: O(n*k), which is all the merge step ever needs.
 */
void oracle_topk(const float* values, const int64_t* indices, int64_t n, int k,
                 float* out_values, int64_t* out_indices) {
  int have = 0;
  for (int64_t j = 0; j < n; ++j) {
    const float v = values[j];
    const int64_t id = indices ? indices[j] : j;
    if (have == k && !ranks_before(v, id, out_values[k - 1], out_indices[k - 1])) continue;
    int pos = have < k ? have : k - 1;
    while (pos > 0 && ranks_before(v, id, out_values[pos - 1], out_indices[pos - 1])) {
      out_values[pos] = out_values[pos - 1];
      out_indices[pos] = out_indices[pos - 1];
      --pos;
    }
    out_values[pos] = v;
    out_indices[pos] = id;
    if (have < k) ++have;
  }
}
