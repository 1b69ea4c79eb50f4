// bv_tail.cu -- the per-query tail: merge the CTA candidate lists of a scan
// into the shard's best F (the device form of gpuTopk.ts:160-189), gather the
// F candidate rows of the fp32 originals, re-rank them with the exact f64 dot
// of store.ts:114-130 and write the best k (index.ts:583-594), all under the
// (score desc, row asc) order.
//
// One CTA, launched right after its scan with programmatic dependent launch:
// it lets the NEXT scan start at once (so the tail runs beside that scan on
// the one SM the scan grid leaves free) and waits for its own scan to finish
// before it reads the candidate lists.
#include <cstdint>

#include "bv_internal.h"
#include "bv_scan.cuh"
#include "bv_tail.cuh"

namespace bv {

// MINB CTAs per SM: 1 for the tail of a single query (latency), 2 for a
// batch's one CTA per query (two CTAs share an SM, so one's memory waits
// overlap the other's work).
template <int MINB>
__global__ void __launch_bounds__(kConsumerThreads, MINB) tail_kernel(const TailParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  // CTA b of a batched launch serves query b: its own partials, query and outputs
  const size_t b = blockIdx.x;
  const uint64_t* const partials = p.partials + b * p.partials_stride;
  const float* const query = p.query + b * p.dim;
  uint32_t* const out_rows = p.out_rows + b * p.k;
  float* const out_scores = p.out_scores + b * p.k;
  uint32_t* const out_count = p.out_count + b;
  uint32_t* const cand_rows = p.cand_rows ? p.cand_rows + b * p.F : nullptr;
  float* const cand_scores = p.cand_scores ? p.cand_scores + b * p.F : nullptr;
  uint32_t* const cand_count = p.cand_count ? p.cand_count + b : nullptr;
  float* const cand_exact = p.cand_exact ? p.cand_exact + b * p.F : nullptr;
  uint64_t* const trace = b == 0 ? p.trace : nullptr;
  const TailSmem lay = tail_smem_layout(p.dim, p.capc, p.rows_bytes);
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + lay.cand_off);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + lay.hist_off);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + lay.misc_off);
  float* q = reinterpret_cast<float*>(smem + lay.q_off);
  double* qd = reinterpret_cast<double*>(smem + lay.qd_off);
  float* rows_s = reinterpret_cast<float*>(smem + lay.rows_off);
  uint64_t* gbar = reinterpret_cast<uint64_t*>(smem + lay.bar_off);
  uint64_t* pbar = gbar + 1;  // the CTA lists staged into shared memory
  const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;

  pdl_trigger();  // the next query's scan may launch now
  if (trace && ctid == 0) trace[kTrTailEntry] = globaltimer();
  if (ctid == 0) {
    mbar_init(gbar, 1);
    mbar_init(pbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the normalized query (an input, ready before this kernel): gbar phase 0
  const uint32_t q_bulk =
      (reinterpret_cast<uintptr_t>(query) & 15u) == 0 ? (p.dim * 4u) & ~15u : 0u;
  if (ctid == 0) {
    mbar_arrive_expect_tx(gbar, p.rerank ? q_bulk : 0u);
    if (p.rerank && q_bulk) bulk_g2s(q, query, q_bulk, gbar);
  }
  pdl_wait();  // this query's scan has completed: the CTA lists are visible
  if (trace && ctid == 0) trace[kTrTailStart] = globaltimer();

  // ---------------------------------------------- merge of the CTA lists
  // Result: cand[0..Fp) = the shard's best keys, descending, zero padded;
  // nc = how many of the first F are real.
  uint32_t nc = 0;
  // The CTA lists come into shared memory in one wave of bulk copies (the row
  // staging area is free until the gather), so the merge reads no global
  // memory; lists that do not fit are merged from global memory.
  const uint32_t list_bytes = p.Fp * 8u;
  const bool staged = p.Fp <= 256u && static_cast<uint64_t>(p.G) * list_bytes <= p.rows_bytes &&
                      (reinterpret_cast<uintptr_t>(partials) & 15u) == 0;
  if (staged) {
    if (ctid == 0) mbar_arrive_expect_tx(pbar, p.G * list_bytes);
    named_bar_sync(kBarConsumers, kConsumerThreads);  // expect_tx precedes every copy
    for (uint32_t l = ctid; l < p.G; l += kConsumerThreads)
      bulk_g2s(reinterpret_cast<uint8_t*>(rows_s) + static_cast<size_t>(l) * list_bytes, partials + static_cast<size_t>(l) * p.Fp,
               list_bytes, pbar);
    mbar_wait_bounded(pbar, 0, p.err);
  }
  if (trace && ctid == 0) trace[kTrTailStaged] = globaltimer();
  if (p.Fp <= 256u) {
    bool selected = false;
    if (staged)
      selected = select_list_heads<true>(reinterpret_cast<const uint64_t*>(rows_s), p.G, p.F, p.Fp, cand, misc, ctid);
    if (!selected) {
      if (staged)
        merge_cta_lists_dispatch<true>(p.Fp, reinterpret_cast<const uint64_t*>(rows_s), p.G, cand, ctid);
      else
        merge_cta_lists_dispatch(p.Fp, partials, p.G, cand, ctid);
    }
    if (warp == 0) {
      uint32_t c = 0;
      for (uint32_t i = lane; i < p.Fp; i += 32) {
        if (i >= p.F) cand[i] = 0ull;
        c += __popc(__ballot_sync(0xffffffffu, i < p.F && cand[i] != 0ull));
      }
      if (lane == 0) misc[kMiscNc] = c;
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    nc = misc[kMiscNc];
  } else {
    // wide F: cand[0..nc) holds the running best F; the lists stream in by chunks
    const uint32_t total = p.G * p.Fp;
    constexpr uint32_t kChunkSlots = kMergeMax - 2;  // 2 slots per thread carry cand (F <= 1024)
    const uint32_t per_chunk = kChunkSlots * kConsumerThreads;
    for (uint32_t c0 = 0; c0 < total; c0 += per_chunk) {
      uint64_t v[kMergeMax];
      uint32_t cnt = 0;
#pragma unroll
      for (int i = 0; i < static_cast<int>(kChunkSlots); ++i) {
        const uint32_t idx = c0 + static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
        v[i] = idx < total ? __ldcg(partials + idx) : 0ull;
        cnt += v[i] != 0ull ? 1u : 0u;
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t idx = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
        v[kChunkSlots + i] = idx < nc ? cand[idx] : 0ull;
        cnt += v[kChunkSlots + i] != 0ull ? 1u : 0u;
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
      if (lane == 0) misc[kMiscRed + warp] = cnt;
      named_bar_sync(kBarConsumers, kConsumerThreads);
      uint32_t tot = 0;
#pragma unroll
      for (int i = 0; i < kConsumerWarps; ++i) tot += misc[kMiscRed + i];
      named_bar_sync(kBarConsumers, kConsumerThreads);
      nc = keep_best<kMergeMax>(v, tot, p.F, cand, hist, misc, ctid);
    }
    for (uint32_t i = nc + static_cast<uint32_t>(ctid); i < p.Fp; i += kConsumerThreads) cand[i] = 0ull;
    named_bar_sync(kBarConsumers, kConsumerThreads);
    // the candidates' order is output only through cand_rows or, without the
    // re-rank, as the result; the re-rank orders by its exact keys itself
    if (cand_rows || !p.rerank) cta_sort_desc(cand, p.Fp, ctid);
  }
  if (trace && ctid == 0) trace[kTrTailMerged] = globaltimer();
  if (cand_rows) {
    for (uint32_t i = ctid; i < nc; i += kConsumerThreads) {
      cand_rows[i] = map_row(p.rowmap, key_row(cand[i])) + p.row_base;
      cand_scores[i] = key_score(cand[i]);
    }
    if (ctid == 0) *cand_count = nc;
  }

  const uint32_t n = nc < p.k ? nc : p.k;
  if (p.rerank) {
    // Gather the candidate rows (row stride dim+4 floats, conflict-free for
    // the four-thread groups), then the exact f64 dot of Store.dotRow: in a
    // batch four threads per row, alone two rows a warp (dot_rows2_exact_warp).
    const uint32_t stride = p.dim + 4;
    mbar_wait_bounded(gbar, 0, p.err);
    for (uint32_t i = q_bulk / 4 + ctid; i < p.dim; i += kConsumerThreads) q[i] = query[i];
    const bool bulk = (p.dim % 4u) == 0u && (reinterpret_cast<uintptr_t>(p.originals) & 15u) == 0u;
    const uint32_t batch = p.rows_bytes / (stride * 4u);
    uint64_t* ex = cand + p.Fp;  // exact keys (cand has capc >= 2*Fp slots)
    uint32_t gph = 1;
    // Rows are gathered a batch at a time into the staging buffer; to keep
    // more bytes in flight than the buffer holds, warp 1 asks L2 for the rows
    // of the next two batches (bulk prefetch) while a batch is copied and dotted.
    auto prefetch = [&](uint32_t c0) {
      if (c0 >= nc) return;
      const uint32_t nb = nc - c0 < batch ? nc - c0 : batch;
      for (uint32_t c = lane; c < nb; c += 32)
        bulk_prefetch_l2(p.originals + static_cast<size_t>(map_row(p.rowmap, key_row(cand[c0 + c]))) * p.dim,
                         p.dim * 4u);
    };
    named_bar_sync(kBarConsumers, kConsumerThreads);
    // batches with wide F score with the warp form over the query widened
    // once to double (the products then convert only the row's elements)
    const bool wide = gridDim.x > 1 && p.F > 256u;
    if (wide) {
      for (uint32_t i = ctid; i < p.dim; i += kConsumerThreads) qd[i] = static_cast<double>(q[i]);
      named_bar_sync(kBarConsumers, kConsumerThreads);
    }
    if (bulk && warp == 1) prefetch(batch);
    for (uint32_t c0 = 0; c0 < nc; c0 += batch) {
      const uint32_t nb = nc - c0 < batch ? nc - c0 : batch;
      if (bulk && warp == 1) prefetch(c0 + 2u * batch);
      if (bulk) {
        if (warp == 0) {
          if (lane == 0) mbar_arrive_expect_tx(gbar, nb * p.dim * 4u);
          __syncwarp();
          for (uint32_t c = lane; c < nb; c += 32)
            bulk_g2s(rows_s + static_cast<size_t>(c) * stride,
                     p.originals + static_cast<size_t>(map_row(p.rowmap, key_row(cand[c0 + c]))) * p.dim,
                     p.dim * 4u, gbar);
        }
        mbar_wait_bounded(gbar, gph, p.err);
        gph ^= 1u;
        if (trace && ctid == 0) trace[kTrTailGathered] = globaltimer();
      } else {
        for (uint32_t c = 0; c < nb; ++c) {
          const float* src = p.originals + static_cast<size_t>(map_row(p.rowmap, key_row(cand[c0 + c]))) * p.dim;
          for (uint32_t i = ctid; i < p.dim; i += kConsumerThreads)
            rows_s[static_cast<size_t>(c) * stride + i] = src[i];
        }
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if (gridDim.x > 1 && p.F <= 256u) {
        // a batch (one CTA per query, many CTAs per SM) with few candidates a
        // query: four threads per row run Store.dotRow's four f64 lanes in
        // order, the fewest operations per element; the warp form below trades
        // operations for latency, which wins for wide F (config 4 tail 1.00 ->
        // 0.83 ms a step; config 3, F = 80: 0.84 vs 0.88 ms)
        const uint32_t vec = p.dim & ~3u;
        for (uint32_t cc = 0; cc < nb; cc += kConsumerThreads / 4) {
          const uint32_t c = cc + static_cast<uint32_t>(ctid) / 4u;
          const uint32_t j = static_cast<uint32_t>(ctid) & 3u;
          const bool act = c < nb;
          const float* xr = rows_s + static_cast<size_t>(act ? c : 0u) * stride;
          double a = 0.0;
          if (act) {
#pragma unroll 8
            for (uint32_t i = j; i < vec; i += 4)
              a = __fma_rn(static_cast<double>(xr[i]), static_cast<double>(q[i]), a);
          }
          const int gl = lane & ~3;
          const double a0 = __shfl_sync(0xffffffffu, a, gl + 0);
          const double a1 = __shfl_sync(0xffffffffu, a, gl + 1);
          const double a2 = __shfl_sync(0xffffffffu, a, gl + 2);
          const double a3 = __shfl_sync(0xffffffffu, a, gl + 3);
          if (act && j == 0) {
            double sacc = __dadd_rn(__dadd_rn(__dadd_rn(a0, a1), a2), a3);
            for (uint32_t i = vec; i < p.dim; ++i)
              sacc = __fma_rn(static_cast<double>(xr[i]), static_cast<double>(q[i]), sacc);
            ex[c0 + c] = make_key(__double2float_rn(sacc), key_row(cand[c0 + c]));
          }
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
        continue;
      }
      for (uint32_t c = static_cast<uint32_t>(warp); c < nb; c += 2u * kConsumerWarps) {  // two rows a warp
        const uint32_t c2 = c + kConsumerWarps;
        if (c2 < nb) {
          float sa, sb;
          if (wide)
            dot_rows2_exact_warp<false, double>(rows_s + static_cast<size_t>(c) * stride,
                                                rows_s + static_cast<size_t>(c2) * stride, qd, p.dim, lane, sa, sb);
          else
            dot_rows2_exact_warp<false>(rows_s + static_cast<size_t>(c) * stride,
                                        rows_s + static_cast<size_t>(c2) * stride, q, p.dim, lane, sa, sb);
          if (lane == 0) {
            ex[c0 + c] = make_key(sa, key_row(cand[c0 + c]));
            ex[c0 + c2] = make_key(sb, key_row(cand[c0 + c2]));
          }
        } else {
          const float sc = wide ? dot_row_exact_warp<false, double>(rows_s + static_cast<size_t>(c) * stride, qd,
                                                                    p.dim, lane)
                                : dot_row_exact_warp<false>(rows_s + static_cast<size_t>(c) * stride, q, p.dim, lane);
          if (lane == 0) ex[c0 + c] = make_key(sc, key_row(cand[c0 + c]));
        }
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
    }
    if (cand_exact)
      for (uint32_t i = ctid; i < nc; i += kConsumerThreads) cand_exact[i] = key_score(ex[i]);
    for (uint32_t i = nc + static_cast<uint32_t>(ctid); i < p.Fp; i += kConsumerThreads) ex[i] = 0ull;
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (trace && ctid == 0) trace[kTrTailDotted] = globaltimer();
    if (p.Fp <= 256u) {
      warp0_sort_dispatch(p.Fp, ex, ctid);
      if (warp == 0) {
        __syncwarp();
        for (uint32_t i = lane; i < n; i += 32) {
          out_rows[i] = map_row(p.rowmap, key_row(ex[i])) + p.row_base;
          out_scores[i] = key_score(ex[i]);
        }
      }
    } else if (n <= 256u && p.Fp <= 2u * kConsumerThreads) {
      // the best n exact keys (radix select), then one warp sorts those few
      uint64_t v2[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t u = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
        v2[i] = u < nc ? ex[u] : 0ull;
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      const uint32_t kept = keep_best<2>(v2, nc, n, ex, hist, misc, ctid);
      uint32_t np = 32;
      while (np < n) np <<= 1;
      for (uint32_t i = kept + static_cast<uint32_t>(ctid); i < np; i += kConsumerThreads) ex[i] = 0ull;
      named_bar_sync(kBarConsumers, kConsumerThreads);
      warp0_sort_dispatch(np, ex, ctid);
      if (warp == 0) {
        __syncwarp();
        for (uint32_t i = lane; i < n; i += 32) {
          out_rows[i] = map_row(p.rowmap, key_row(ex[i])) + p.row_base;
          out_scores[i] = key_score(ex[i]);
        }
      }
    } else {
      cta_sort_desc(ex, p.Fp, ctid);
      for (uint32_t i = ctid; i < n; i += kConsumerThreads) {
        out_rows[i] = map_row(p.rowmap, key_row(ex[i])) + p.row_base;
        out_scores[i] = key_score(ex[i]);
      }
    }
  } else {
    for (uint32_t i = ctid; i < n; i += kConsumerThreads) {
      out_rows[i] = map_row(p.rowmap, key_row(cand[i])) + p.row_base;
      out_scores[i] = key_score(cand[i]);
    }
  }
  if (ctid == 0) {
    *out_count = n;
    if (trace) trace[kTrTailDone] = globaltimer();
  }
}

cudaError_t launch_tail_grid(const TailParams& p, uint32_t nq, size_t smem, cudaStream_t stream) {
  static int opted[kMaxDevices] = {};
  const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(tail_kernel<2>), smem, opted);
  if (e != cudaSuccess) return e;
  tail_kernel<2><<<nq, kConsumerThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_tail(const TailParams& p, size_t smem, cudaStream_t stream) {
  static int opted[kMaxDevices] = {};
  const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(tail_kernel<1>), smem, opted);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kConsumerThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tail_kernel<1>, p);
}

}  // namespace bv
