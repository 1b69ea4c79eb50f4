// bv_filter.cu -- the metadata predicate of a filtered query on the GPU.
//
// compileFilter (src/store/filter.ts:18-68) builds an AND of per-field
// operator tests with strict JS equality; src/index.ts:372-395 runs it over
// every live record to build the score mask of a filtered query.  Here the
// store's metadata lives in device columns (type tag, f64 number, string
// dictionary code per row) and one thread evaluates one row; a warp ballot
// packs 32 rows into one mask word, so the mask is written coalesced.
#include <cstdint>

#include "../../include/browservec.h"
#include "bv_internal.h"

namespace bv {

struct FilterParams {
  bv_column cols[BV_FILTER_MAX_TERMS];
  bv_filter_term terms[BV_FILTER_MAX_TERMS];
  uint32_t nterms;
  uint64_t rows;
  const uint32_t* live;
  uint32_t* mask;
};

namespace {

// JS `row === v` for one metadata value (filter.ts:35-41).
__device__ __forceinline__ bool strict_eq(const bv_column& c, uint64_t r, uint32_t tag, const bv_value& v) {
  if (tag != v.tag) return false;
  switch (tag) {
    case BV_TAG_MISSING:
    case BV_TAG_NULL:
      return true;
    case BV_TAG_BOOL:
    case BV_TAG_NUMBER:
      return c.num[r] == v.num;  // IEEE: NaN never equals
    case BV_TAG_STRING:
      return v.code >= 0 && c.code[r] == v.code;
    default:
      return false;
  }
}

// Set.has (filter.ts:29-30) compares with SameValueZero: as ===, except that
// NaN matches NaN (+0 and -0 are already equal under ==).
__device__ __forceinline__ bool same_value_zero(const bv_column& c, uint64_t r, uint32_t tag, const bv_value& v) {
  if (tag == BV_TAG_NUMBER && v.tag == BV_TAG_NUMBER && v.num != v.num) {
    const double x = c.num[r];
    return x != x;
  }
  return strict_eq(c, r, tag, v);
}

__global__ void __launch_bounds__(256) filter_kernel(const __grid_constant__ FilterParams p) {
  const uint64_t r = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool ok = r < p.rows;
  if (ok) {
    for (uint32_t t = 0; t < p.nterms && ok; ++t) {
      const bv_filter_term& term = p.terms[t];
      const bv_column& c = p.cols[term.column];
      const uint32_t tag = c.tag[r];
      switch (term.op) {
        case BV_OP_EQ:
          ok = strict_eq(c, r, tag, term.vals[0]);
          break;
        case BV_OP_NE:  // filter.ts:43: matches records missing the field too
          ok = !strict_eq(c, r, tag, term.vals[0]);
          break;
        case BV_OP_IN: {
          bool any = false;
          for (uint32_t i = 0; i < term.nvals && !any; ++i) any = same_value_zero(c, r, tag, term.vals[i]);
          ok = any;
          break;
        }
        default: {  // range operators: numbers only (filter.ts:49-64)
          if (tag != BV_TAG_NUMBER) {
            ok = false;
            break;
          }
          const double x = c.num[r], a = term.vals[0].num;
          ok = term.op == BV_OP_GT ? x > a : (term.op == BV_OP_GTE ? x >= a : (term.op == BV_OP_LT ? x < a : x <= a));
        }
      }
    }
  }
  const uint32_t word = __ballot_sync(0xffffffffu, ok);
  if ((threadIdx.x & 31u) == 0 && r < p.rows) {
    const uint64_t w = r >> 5;
    p.mask[w] = p.live ? (word & p.live[w]) : word;
  }
}

}  // namespace

cudaError_t launch_filter(const bv_column* cols, uint32_t ncols, const bv_filter_term* terms, uint32_t nterms,
                          uint64_t rows, const uint32_t* live, uint32_t* mask, cudaStream_t s) {
  FilterParams p;
  for (uint32_t i = 0; i < ncols && i < BV_FILTER_MAX_TERMS; ++i) p.cols[i] = cols[i];
  for (uint32_t i = 0; i < nterms; ++i) p.terms[i] = terms[i];
  p.nterms = nterms;
  p.rows = rows;
  p.live = live;
  p.mask = mask;
  const uint64_t blocks = (rows + 255) / 256;
  if (blocks == 0) return cudaSuccess;
  if (blocks > 0x7FFFFFFFull) return cudaErrorInvalidValue;
  filter_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace bv
