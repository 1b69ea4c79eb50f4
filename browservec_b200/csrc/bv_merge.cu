// bv_merge.cu -- the cross-shard merge of a row-sharded search.
//
// Every shard (one GPU) searched its own contiguous range of global rows and
// wrote, per query, its best F candidates by approximate score with their
// exact re-rank scores.  After the all-gather every rank holds all W shard
// records and this kernel rebuilds the single-store answer:
//   1. the global best F by approximate key (score desc, global row asc) --
//      the per-chunk partial merge of QuantIndex.search / mergePartials
//      (src/index/quant.ts:194-245, src/index/gpuTopk.ts:160-189);
//   2. among those F, the best k by exact key -- the re-rank's topK
//      (src/index.ts:583-594).
// A shard's local best F contains every one of its rows that is in the global
// best F under the same total order, so the result equals one GPU holding all
// rows.
//
// One CTA per query.  Step 1 ranks every entry by binary searches in the
// other shards' lists (each list is sorted by approximate key, as the search
// writes it); step 2 ranks the selected entries by counting, reading the keys
// as warp-wide broadcasts from shared memory.
#include <cstdint>

#include "bv_device.cuh"
#include "bv_internal.h"

namespace bv {

namespace {

constexpr int kMergeThreads = 256;
constexpr int kMaxWorld = 64;

// Entries of list `l` (length n, keys descending) greater than `key`.
__device__ __forceinline__ uint32_t count_greater(const uint64_t* l, uint32_t n, uint64_t key) {
  uint32_t lo = 0, hi = n;  // answer in [lo, hi]
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (l[mid] > key) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(kMergeThreads) merge_shards_kernel(
    const uint32_t* __restrict__ gathered, uint32_t world, uint32_t nq, uint32_t F, uint32_t k,
    uint32_t* __restrict__ out_rows, float* __restrict__ out_scores, uint32_t* __restrict__ out_counts) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* akey = reinterpret_cast<uint64_t*>(smem);           // world*F approximate keys
  uint64_t* sel = akey + static_cast<size_t>(world) * F;        // F exact keys, by approximate rank
  float* exact = reinterpret_cast<float*>(sel + F);             // world*F exact scores
  __shared__ uint32_t len[kMaxWorld];
  __shared__ uint32_t nsel;

  const uint32_t q = blockIdx.x;
  const size_t plane = static_cast<size_t>(nq) * F;
  const size_t rec = 3 * plane + nq;  // words per shard record
  const int t = threadIdx.x;

  if (t < static_cast<int>(world)) {
    const uint32_t c = gathered[static_cast<size_t>(t) * rec + 3 * plane + q];
    len[t] = c < F ? c : F;
  }
  __syncthreads();
  for (uint32_t i = t; i < world * F; i += kMergeThreads) {
    const uint32_t w = i / F, j = i - w * F;
    const uint32_t* r = gathered + static_cast<size_t>(w) * rec + static_cast<size_t>(q) * F;
    if (j < len[w]) {
      akey[i] = make_key(__uint_as_float(r[plane + j]), r[j]);
      exact[i] = __uint_as_float(r[2 * plane + j]);
    } else {
      akey[i] = 0ull;
    }
  }
  if (t == 0) {
    uint32_t tot = 0;
    for (uint32_t w = 0; w < world; ++w) tot += len[w];
    nsel = tot < F ? tot : F;
  }
  __syncthreads();

  // 1. global rank of every entry by approximate key; the best F are kept
  for (uint32_t i = t; i < world * F; i += kMergeThreads) {
    const uint32_t w = i / F, j = i - w * F;
    if (j >= len[w]) continue;
    const uint64_t key = akey[i];
    uint32_t rank = j;
    for (uint32_t v = 0; v < world && rank < F; ++v)
      if (v != w) rank += count_greater(akey + static_cast<size_t>(v) * F, len[v], key);
    if (rank < F) sel[rank] = make_key(exact[i], key_row(key));
  }
  __syncthreads();

  // 2. rank of every selected entry by exact key; the best k are written
  const uint32_t n = nsel;
  constexpr int kPer = 4;
  for (uint32_t base = 0; base < n; base += kPer * kMergeThreads) {
    uint64_t mine[kPer];
    uint32_t rank[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      const uint32_t s = base + static_cast<uint32_t>(e) * kMergeThreads + t;
      mine[e] = s < n ? sel[s] : ~0ull;
      rank[e] = 0;
    }
    for (uint32_t s = 0; s < n; ++s) {
      const uint64_t o = sel[s];
#pragma unroll
      for (int e = 0; e < kPer; ++e) rank[e] += o > mine[e] ? 1u : 0u;
    }
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      const uint32_t s = base + static_cast<uint32_t>(e) * kMergeThreads + t;
      if (s < n && rank[e] < k) {
        out_rows[static_cast<size_t>(q) * k + rank[e]] = key_row(mine[e]);
        out_scores[static_cast<size_t>(q) * k + rank[e]] = key_score(mine[e]);
      }
    }
  }
  if (t == 0) out_counts[q] = n < k ? n : k;
}

// One CTA per query: the best k of W lists of (row, exact score) pairs, each
// sorted by (score desc, row asc) with its own count, gathered in rank order
// as W records of [rows nq*k | scores nq*k | counts nq] u32 words.  An
// entry's rank is its index in its list plus, in every other list, the
// entries ahead of it (binary search over the keys staged in shared memory).
__global__ void __launch_bounds__(kMergeThreads) merge_topk_kernel(
    const uint32_t* __restrict__ gathered, uint32_t world, uint32_t nq, uint32_t k,
    uint32_t* __restrict__ out_rows, float* __restrict__ out_scores, uint32_t* __restrict__ out_counts) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* key = reinterpret_cast<uint64_t*>(smem);  // world*k keys
  __shared__ uint32_t len[kMaxWorld];
  const uint32_t q = blockIdx.x;
  const size_t plane = static_cast<size_t>(nq) * k;
  const size_t rec = 2 * plane + nq;
  const int t = threadIdx.x;
  if (t < static_cast<int>(world)) {
    const uint32_t c = gathered[static_cast<size_t>(t) * rec + 2 * plane + q];
    len[t] = c < k ? c : k;
  }
  __syncthreads();
  for (uint32_t i = t; i < world * k; i += kMergeThreads) {
    const uint32_t w = i / k, j = i - w * k;
    const uint32_t* r = gathered + static_cast<size_t>(w) * rec + static_cast<size_t>(q) * k;
    key[i] = j < len[w] ? make_key(__uint_as_float(r[plane + j]), r[j]) : 0ull;
  }
  __syncthreads();
  uint32_t total = 0;
  for (uint32_t w = 0; w < world; ++w) total += len[w];
  for (uint32_t i = t; i < world * k; i += kMergeThreads) {
    const uint32_t w = i / k, j = i - w * k;
    if (j >= len[w]) continue;
    const uint64_t kk = key[i];
    uint32_t rank = j;
    for (uint32_t v = 0; v < world && rank < k; ++v)
      if (v != w) rank += count_greater(key + static_cast<size_t>(v) * k, len[v], kk);
    if (rank < k) {
      out_rows[static_cast<size_t>(q) * k + rank] = key_row(kk);
      out_scores[static_cast<size_t>(q) * k + rank] = key_score(kk);
    }
  }
  if (t == 0) out_counts[q] = total < k ? total : k;
}

}  // namespace

cudaError_t launch_merge_topk(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t k,
                              uint32_t* out_rows, float* out_scores, uint32_t* out_counts, cudaStream_t stream) {
  static int opted[kMaxDevices] = {};
  const size_t smem = static_cast<size_t>(world) * k * 8;
  const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(merge_topk_kernel), smem, opted);
  if (e != cudaSuccess) return e;
  merge_topk_kernel<<<nq, kMergeThreads, smem, stream>>>(gathered, world, nq, k, out_rows, out_scores, out_counts);
  return cudaGetLastError();
}

size_t merge_smem_bytes(uint32_t world, uint32_t F) {
  return static_cast<size_t>(world) * F * 12 + static_cast<size_t>(F) * 8;
}

uint32_t merge_max_world() { return kMaxWorld; }

cudaError_t launch_merge_shards(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t F, uint32_t k,
                                uint32_t* out_rows, float* out_scores, uint32_t* out_counts,
                                cudaStream_t stream) {
  static int opted[kMaxDevices] = {};
  const size_t smem = merge_smem_bytes(world, F);
  const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(merge_shards_kernel), smem, opted);
  if (e != cudaSuccess) return e;
  merge_shards_kernel<<<nq, kMergeThreads, smem, stream>>>(gathered, world, nq, F, k, out_rows, out_scores,
                                                            out_counts);
  return cudaGetLastError();
}

}  // namespace bv
