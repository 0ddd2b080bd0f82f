/*
 * Plain-C restatement of PaceServe's moe_align_block_size
 * (csrc/moe_align_block_size_kernels.cu:23-109, host :112-135).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernel, never shipped.
 *
 * Steps, as in the reference kernel:
 *   1. count the flat entries of each expert (:41-52);
 *   2. cumsum[e+1] = cumsum[e] + ceil(count[e] / block_size) * block_size,
 *      total = cumsum[E] (:65-75);
 *   3. expert_ids[b] = e for every block b in [cumsum[e], cumsum[e+1]) / bs (:83-86);
 *   4. sorted_token_ids[cumsum[e] + r] = i, r = rank of i among e's entries in
 *      ascending flat index (:95-108; the reference's per-thread contiguous
 *      shards visited in thread order give exactly this order).
 * Slots not written are left as the caller filled them (numel in PaceServe's
 * wrapper, fused_moe.py:191-195).  Entries outside [0, E) are skipped (the
 * reference would index out of its counter array).
 * Returns 0, or -1 for bad arguments / insufficient capacity.
 */
#include <stdint.h>
#include <stdlib.h>

int moe_align_block_size_ref(const int64_t* ids, int64_t numel, int num_experts, int block_size,
                             int32_t* sorted_ids, int64_t sorted_capacity, int32_t* expert_ids,
                             int64_t expert_capacity, int32_t* total_out) {
  if (numel < 0 || num_experts <= 0 || block_size <= 0) return -1;
  const int64_t need = numel + (int64_t)num_experts * (block_size - 1);
  if (sorted_capacity < need || expert_capacity < (need + block_size - 1) / block_size) return -1;
  int64_t* count = (int64_t*)calloc((size_t)num_experts, sizeof(int64_t));
  int64_t* cumsum = (int64_t*)calloc((size_t)num_experts + 1, sizeof(int64_t));
  if (!count || !cumsum) {
    free(count);
    free(cumsum);
    return -1;
  }
  for (int64_t i = 0; i < numel; ++i) {
    const int64_t e = ids[i];
    if (e >= 0 && e < num_experts) ++count[e];
  }
  for (int e = 0; e < num_experts; ++e)
    cumsum[e + 1] = cumsum[e] + (count[e] + block_size - 1) / block_size * block_size;
  *total_out = (int32_t)cumsum[num_experts];
  for (int e = 0; e < num_experts; ++e)
    for (int64_t p = cumsum[e]; p < cumsum[e + 1]; p += block_size)
      expert_ids[p / block_size] = e;
  /* count[] becomes the running rank of each expert */
  for (int e = 0; e < num_experts; ++e) count[e] = 0;
  for (int64_t i = 0; i < numel; ++i) {
    const int64_t e = ids[i];
    if (e < 0 || e >= num_experts) continue;
    sorted_ids[cumsum[e] + count[e]] = (int32_t)i;
    ++count[e];
  }
  free(count);
  free(cumsum);
  return 0;
}
