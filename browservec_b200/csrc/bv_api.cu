// bv_api.cu -- the C ABI (include/browservec.h): index lifetime, corpus
// storage in HBM, the encoder and scan launches, and error reporting.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/browservec.h"
#include "bv_internal.h"
#include "bv_scan.cuh"
#include "bv_tail.cuh"
#include "bv_batch.cuh"

namespace {

thread_local std::string g_err;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return status;
}

constexpr const char* kLostMsg = "GPU device lost; re-create the store";  // quant.ts:183
constexpr uint32_t kRowAlign = 2048;      // capacity granularity (>= any scan tile)
// Per-query scratch of the single-query searches (the scan CTAs' candidate
// lists, tile counters) is a ring of kRing slots: consecutive queries never
// share one, so a scan never waits for an earlier query's tail; each wrap of
// the ring waits for all earlier work of the stream (an event), so a slot is
// reused only after the tail that read it has finished.
constexpr uint32_t kRing = 64;
constexpr size_t kRingMaxBytes = 256u << 20;
constexpr uint32_t kBatchMinQueries = 64;  // bv_search batches at least this many on the tensor cores
constexpr uint32_t kMaxFetch = 1024;      // fused single-query path: F <= 1024
constexpr uint32_t kMaxPadded = 4096;

bool is_sticky(cudaError_t e) {
  switch (e) {
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorHardwareStackError:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorInvalidAddressSpace:
    case cudaErrorInvalidPc:
    case cudaErrorECCUncorrectable:
    case cudaErrorLaunchTimeout:
    case cudaErrorUnknown:
      return true;
    default:
      return false;
  }
}

// prng.ts:5-14 (mulberry32) -- uint32 arithmetic.
uint32_t mulberry32_next(uint32_t* state) {
  uint32_t a = *state + 0x6d2b79f5u;
  *state = a;
  uint32_t t = (a ^ (a >> 15)) * (1u | a);
  t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;
  return t ^ (t >> 14);
}

uint32_t pad_to_pow2(uint32_t n) {  // rotator.ts:16-21
  uint32_t p = 4;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace

// Batched-search state kept between the phases of one search
// (bv_batch_select -> bv_batch_finish) and the optional device-time profile.
struct bv_batch_state {
  // plan of the last batched rounds (kept for bv_batch_finish)
  bool pending = false;
  uint32_t nq = 0, F = 0, Fp = 0, cap = 0, launches = 0, rounds = 0;
  bool empty = false;  // nothing to rank: outputs are zero counts
  // timing
  bool timing = false;
  std::vector<cudaEvent_t> ev;
  std::vector<std::pair<int, uint32_t>> marks;  // (phase, event index of its start); end = next event
  uint32_t used = 0;
  bv_batch_profile prof = {};
};

struct bv_index {
  int device = 0;
  uint32_t dim = 0, bits = 8, metric = 0, seed = 0, rounds = 2, scoring = 0, row_base = 0;
  uint32_t P = 0, R = 0;
  uint64_t rows = 0, cap_rows = 0;
  uint8_t* d_codes = nullptr;
  float* d_scales = nullptr;
  float* d_orig = nullptr;
  float* d_signs = nullptr;
  // scratch of the scan: per-CTA candidate lists, tile counters, error flags
  uint64_t* d_partials = nullptr;
  size_t partials_cap = 0;
  unsigned long long* d_tile_ctr = nullptr;  // kRing rotating dynamic-tile counters
  unsigned int* d_done = nullptr;            // kRing per-query finished-CTA counters
  size_t partials_slot = 0;                  // keys per query in the partials ring
  uint32_t ring = 0;                         // slots of the partials ring
  cudaEvent_t ev_ring = nullptr;             // all work before a ring wrap
  uint32_t epoch = 0;                        // scan launches so far
  uint32_t* d_err = nullptr;
  // staging for the host-pointer entry points
  float* d_q = nullptr;
  size_t q_cap = 0;
  uint32_t* d_mask = nullptr;
  size_t mask_cap = 0;
  uint32_t* d_rows = nullptr;
  size_t rows_cap = 0;
  uint32_t* d_out = nullptr;  // out rows | scores | counts | cand rows | cand scores | cand counts
  size_t out_cap = 0;
  void* h_pin = nullptr;
  size_t pin_cap = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  int num_sms = 148;
  int max_smem = 227 * 1024;
  int smem_per_sm = 228 * 1024;
  float last_ms = 0.0f;
  // TMA descriptor of the originals for the exact flat scan (re-encoded when
  // the buffer or the row count changes)
  alignas(64) unsigned char flat_map[128] = {};
  const float* flat_map_rows = nullptr;
  uint64_t flat_map_n = 0;
  uint32_t last_launches = 0;
  uint64_t* d_trace = nullptr;   // optional phase-timestamp buffer (caller-owned device memory)
  uint64_t trace_cap = 0;
  bool lost = false;
  // batched search: the codes as swizzled int8 MMA tiles (built lazily, for
  // rows [0, mma_rows)), per-row score factors, per-tile factor maxima
  // (positions: each appended block of rows in ascending score-factor order)
  int8_t* d_ctiles = nullptr;
  size_t ctiles_cap = 0;  // bytes
  float* d_posfac = nullptr;
  size_t posfac_cap = 0;
  uint32_t* d_posrow = nullptr;
  size_t posrow_cap = 0;
  float* d_tmax = nullptr;
  size_t tmax_cap = 0;
  uint64_t mma_rows = 0;
  // row-order sort scratch (factor keys, row ids, radix-sort temporary)
  float* d_sfac = nullptr;  // 2 x n
  size_t sfac_cap = 0;
  uint32_t* d_sids = nullptr;  // 2 x n
  size_t sids_cap = 0;
  uint8_t* d_stmp = nullptr;
  size_t stmp_cap = 0;
  // batched search scratch
  int8_t* d_qtiles = nullptr;
  size_t qtiles_cap = 0;
  float* d_qfac = nullptr;
  size_t qfac_cap = 0;
  uint64_t* d_thr = nullptr;
  size_t thr_cap = 0;
  uint32_t* d_bcnt = nullptr;  // candidate counts, then their backup
  size_t bcnt_cap = 0;
  uint64_t* d_bcand = nullptr;
  size_t bcand_cap = 0;
  uint32_t* d_scnt = nullptr;  // per query, per GEMM slice: candidates appended
  size_t scnt_cap = 0;
  uint32_t* d_overflow = nullptr;
  uint32_t last_rounds = 0;
  // filtered batches: the kept rows gathered into their own tiles
  uint32_t* d_cwoff = nullptr;  // per mask word: kept rows before it (within its scan block)
  size_t cwoff_cap = 0;
  uint32_t* d_cbsum = nullptr;  // per scan block, then the total
  size_t cbsum_cap = 0;
  uint32_t* d_cmap = nullptr;   // compacted row -> row
  size_t cmap_cap = 0;
  int8_t* d_cctiles = nullptr;
  size_t cctiles_cap = 0;
  float* d_cposfac = nullptr;
  size_t cposfac_cap = 0;
  uint32_t* d_cposrow = nullptr;
  size_t cposrow_cap = 0;
  float* d_ctmax = nullptr;
  size_t ctmax_cap = 0;
  uint32_t last_kept = 0;
  bv_batch_state* batch = nullptr;  // batched-search plan kept between phases, timing
  // candidate-list search: gathered codes, scales and their rows; rowmap is
  // set only while such a search enqueues its scans
  uint8_t* d_gcodes = nullptr;
  size_t gcodes_cap = 0;
  float* d_gscales = nullptr;
  size_t gscales_cap = 0;
  uint32_t* d_growmap = nullptr;
  size_t growmap_cap = 0;
  uint32_t* d_goffs = nullptr;  // per query: candidate offset, segment start
  size_t goffs_cap = 0;
  const uint32_t* rowmap = nullptr;
  // batched GEMM on CTA pairs (cta_group::2) for batches of two or more query
  // tiles, chosen with BV_GEMM_PAIR=1 in the environment; off by default: on
  // B200 it measured slower than the one-CTA GEMM (config 4 10.1 vs 9.2 ms)
  bool gemm_pair = false;
};

namespace {

int cuda_fail(bv_index* idx, cudaError_t e, const char* what) {
  if (is_sticky(e)) {
    if (idx) idx->lost = true;
    return fail(BV_ERR_DEVICE_LOST, "%s", kLostMsg);
  }
  if (e == cudaErrorMemoryAllocation) return fail(BV_ERR_NOMEM, "%s: out of device memory", what);
  return fail(BV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define BV_CUDA(idx, call, what)                  \
  do {                                            \
    cudaError_t e_ = (call);                      \
    if (e_ != cudaSuccess) return cuda_fail(idx, e_, what); \
  } while (0)

template <class T>
int grow(bv_index* idx, T** p, size_t* cap, size_t need, const char* what) {
  if (*cap >= need) return BV_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  size_t n = need < 64 ? 64 : need;
  BV_CUDA(idx, cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T)), what);
  *cap = n;
  return BV_OK;
}

int grow_pinned(bv_index* idx, size_t bytes) {
  if (idx->pin_cap >= bytes) return BV_OK;
  if (idx->h_pin) cudaFreeHost(idx->h_pin);
  idx->h_pin = nullptr;
  idx->pin_cap = 0;
  size_t n = bytes < 4096 ? 4096 : bytes;
  BV_CUDA(idx, cudaMallocHost(&idx->h_pin, n), "pinned staging");
  idx->pin_cap = n;
  return BV_OK;
}

int ensure_capacity(bv_index* idx, uint64_t need_rows) {
  if (need_rows <= idx->cap_rows) return BV_OK;
  uint64_t cap = idx->cap_rows * 2;
  if (cap < need_rows) cap = need_rows;
  cap = (cap + kRowAlign - 1) / kRowAlign * kRowAlign;
  uint8_t* codes = nullptr;
  float* scales = nullptr;
  float* orig = nullptr;
  BV_CUDA(idx, cudaMalloc(&codes, idx->R ? cap * idx->R : 16), "codes");
  cudaError_t e = cudaMalloc(&scales, cap * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&orig, cap * idx->dim * sizeof(float));
  if (e != cudaSuccess) {
    cudaFree(codes);
    cudaFree(scales);
    return cuda_fail(idx, e, "corpus");
  }
  BV_CUDA(idx, cudaMemsetAsync(codes, 0, cap * idx->R, idx->stream), "memset");
  BV_CUDA(idx, cudaMemsetAsync(scales, 0, cap * sizeof(float), idx->stream), "memset");
  if (idx->rows) {
    BV_CUDA(idx, cudaMemcpyAsync(codes, idx->d_codes, idx->rows * idx->R, cudaMemcpyDeviceToDevice,
                                 idx->stream), "copy");
    BV_CUDA(idx, cudaMemcpyAsync(scales, idx->d_scales, idx->rows * sizeof(float),
                                 cudaMemcpyDeviceToDevice, idx->stream), "copy");
    BV_CUDA(idx, cudaMemcpyAsync(orig, idx->d_orig, idx->rows * idx->dim * sizeof(float),
                                 cudaMemcpyDeviceToDevice, idx->stream), "copy");
  }
  BV_CUDA(idx, cudaStreamSynchronize(idx->stream), "grow");
  cudaFree(idx->d_codes);
  cudaFree(idx->d_scales);
  cudaFree(idx->d_orig);
  idx->d_codes = codes;
  idx->d_scales = scales;
  idx->d_orig = orig;
  idx->cap_rows = cap;
  return BV_OK;
}

struct Plan {
  bv::ScanShape sh;
  uint32_t tile_rows, tile_bytes, ntiles, stages, grid, F, Fp, capc, check_tiles;
  uint32_t slots;  // the largest grid a plan of this geometry launches (sizes the ring slots)
  size_t smem;
  bool fold;
};

// fold: the scan's last CTA finishes each query (no tail kernel), for the
// integer scorings with Fp <= 256; pl->fold says whether the plan does.
// alone: the query runs by itself (a synchronous call waits for it), so its
// grid takes every CTA slot instead of leaving room for the next query.
int plan_scan(bv_index* idx, uint32_t F, Plan* pl, bool fold = true, bool alone = false) {
  if (!bv::scan_shape(static_cast<int>(idx->bits), static_cast<int>(idx->scoring), idx->P, &pl->sh))
    return fail(BV_ERR_UNSUPPORTED, "padded dimension %u is outside the scan's range", idx->P);
  const uint32_t R = pl->sh.R;
  // ~32 KB tiles of at least one iteration's rows, at most 64 KB and 2048 rows
  uint32_t tr = 32768u / R;
  if (tr > 2048u) tr = 2048u;
  if (tr < pl->sh.rows_per_iter) tr = pl->sh.rows_per_iter;
  const uint32_t tr_max = 65536u / R > 0 ? 65536u / R : 1u;
  if (tr > tr_max) tr = tr_max;
  pl->tile_rows = tr;
  pl->tile_bytes = tr * R;
  pl->ntiles = static_cast<uint32_t>((idx->rows + tr - 1) / tr);
  pl->F = F;
  uint32_t fp = 32;
  while (fp < F) fp <<= 1;
  pl->Fp = fp;
  // candidate slots: room for 2*Fp plus a tile between checks, and for the
  // 16 warp lists of the register merge (Fp <= 256)
  uint32_t capc = 1024;
  while (capc < 2 * fp + tr || (fp <= 256 && capc < 16 * fp)) capc <<= 1;
  if (capc > static_cast<uint32_t>(bv::kSelMax * bv::kConsumerThreads))
    return fail(BV_ERR_UNSUPPORTED, "candidate buffer for fetch %u does not fit", F);
  pl->capc = capc;
  pl->check_tiles = (capc - 2 * fp) / tr;
  if (pl->check_tiles < 1) pl->check_tiles = 1;
  pl->fold = fold && fp <= 256;
  // Folded scans run two CTAs per SM (consecutive queries): each CTA then
  // keeps to half of the SM's shared memory.
  // A query alone runs one CTA per SM (below), so it may take an SM's whole
  // shared memory: a deeper ring, and room for all of its re-rank rows in the
  // finish.
  const uint32_t half = static_cast<uint32_t>(idx->smem_per_sm) / 2u - 1024u;
  const bool two = pl->fold && !alone;
  const uint32_t limit = two ? half : static_cast<uint32_t>(idx->max_smem);
  pl->stages = 0;
  for (uint32_t lim : {limit, static_cast<uint32_t>(idx->max_smem)}) {  // two CTAs per SM, else one
    for (uint32_t st = 4; st >= 2 && !pl->stages; --st) {
      bv::ScanSmem lay = bv::scan_smem_layout(pl->tile_bytes, tr, st, idx->P, idx->rounds, capc);
      if (lay.total <= lim) {
        pl->stages = st;
        pl->smem = lay.total;
      }
    }
    if (pl->stages) break;
  }
  if (!pl->stages) return fail(BV_ERR_UNSUPPORTED, "scan tile does not fit in shared memory");
  // Without folding two SMs stay free for the tail kernels (one query's merge
  // and re-rank can still run while the next query's finishes), so a
  // following scan finds a whole grid's worth of SMs.  With two CTAs per SM a
  // query takes a sixth of the CTA slots (num_sms / 3 CTAs), so six queries
  // stream at once.  The next query's kernel launches only once every CTA of
  // the one before it has started (programmatic dependent launch), and slots
  // that free before then stay empty; small grids start all their CTAs
  // quickly and keep that gap short, while each CTA's fixed prologue and
  // epilogue are spread over more tiles.  Measured on B200 (100k x 768 int8,
  // back-to-back queries): 98 CTAs 47.1k q/s, 74 50.4k, 59 53.4k, 49 55.6k,
  // 42 53.6k.
  const bool two_per_sm = pl->fold && pl->smem <= half;
  const uint32_t nsm = static_cast<uint32_t>(idx->num_sms);
  const uint32_t all = two_per_sm ? 2u * nsm : pl->fold ? nsm : (nsm > 2 ? nsm - 2u : 1u);
  // One CTA per SM (wide F with the tail kernel): back to back, a query takes
  // two sevenths of the SMs (measured when asym ran one CTA per SM, 100k x
  // 768 int8: 146 CTAs 27.0k q/s, 74 28.2k, 49 31.7k, 42 33.1k, 37 32.8k,
  // 29 28.1k).
  const uint32_t one_sm = nsm * 2u / 7u > 0 ? nsm * 2u / 7u : 1u;
  // A query alone takes one CTA per SM: twice the CTAs stream no faster and
  // leave twice the lists to its last CTA (measured, 100k x 768 int8, one
  // synchronous query per call: 296 CTAs 100 us a call, 222 97, 148 93, 100 105).
  const uint32_t sms = alone ? nsm : two_per_sm ? (nsm / 3u > 0 ? nsm / 3u : 1u) : (pl->fold ? all : one_sm);
  pl->grid = pl->ntiles < sms ? pl->ntiles : sms;
  pl->slots = pl->ntiles < all ? pl->ntiles : all;
  return BV_OK;
}

cudaError_t launch_scan(int bits, int mode, const bv::ScanShape& sh, const bv::ScanParams& p,
                        unsigned grid, size_t smem, cudaStream_t s) {
  if (bits == 8) return mode == 0 ? bv::launch_scan8_asym(sh, p, grid, smem, s)
                                  : bv::launch_scan8_int(sh, p, grid, smem, s);
  if (bits == 4) return mode == 0 ? bv::launch_scan4_asym(sh, p, grid, smem, s)
                                  : bv::launch_scan4_int(sh, p, grid, smem, s);
  if (mode == 0) return bv::launch_scan1_asym(sh, p, grid, smem, s);
  if (mode == 1) return bv::launch_scan1_int(sh, p, grid, smem, s);
  return bv::launch_scan1_hamming(sh, p, grid, smem, s);
}

// Validate a request; returns the effective F (0 on error, message set).
int check_args(bv_index* idx, const bv_search_args* a, uint32_t* F_out) {
  if (!idx || !a) return fail(BV_ERR_INVALID, "null index or args");
  if (idx->lost) return fail(BV_ERR_DEVICE_LOST, "%s", kLostMsg);
  if (a->nq && !a->queries) return fail(BV_ERR_INVALID, "queries is null");
  if (a->k == 0) return fail(BV_ERR_INVALID, "k must be >= 1");
  if (!a->out_rows || !a->out_scores || !a->out_counts)
    return fail(BV_ERR_INVALID, "output pointers are required");
  if (a->cand_exact && !(a->rerank && a->cand_rows && a->cand_scores && a->cand_counts))
    return fail(BV_ERR_INVALID, "cand_exact needs rerank and the cand_* outputs");
  uint32_t F = a->fetch ? a->fetch : a->k;
  if (F < a->k) F = a->k;
  if (F > kMaxFetch)
    return fail(BV_ERR_UNSUPPORTED, "fetch %u exceeds the single-query scan limit (%u)", F, kMaxFetch);
  if (a->mask) {
    const uint64_t words = (idx->rows + 31) / 32;
    if (a->mask_words < words)  // scoreMask.ts:68-70
      return fail(BV_ERR_INVALID, "mask has %llu words, need %llu for %llu rows",
                  static_cast<unsigned long long>(a->mask_words),
                  static_cast<unsigned long long>(words), static_cast<unsigned long long>(idx->rows));
  }
  *F_out = F;
  return BV_OK;
}

// Size the partials ring for `keys` candidate keys per query (keeping earlier
// slots is not needed: a resize happens between searches).
int ring_prepare(bv_index* idx, size_t keys) {
  uint32_t r = kRing;
  while (r > 2 && static_cast<size_t>(r) * keys * 8 > kRingMaxBytes) r >>= 1;
  // a ring with at least as many slots of at least this size serves as is
  // (searches over candidate lists of varying length would otherwise resize it)
  if (idx->partials_slot >= keys && idx->ring >= r && idx->ring && idx->d_partials) return BV_OK;
  if (idx->partials_slot != keys || idx->ring != r) {
    // a new geometry: earlier queries' slots must be out of use before reuse
    BV_CUDA(idx, cudaDeviceSynchronize(), "ring resize");
    idx->partials_slot = keys;
    idx->ring = r;
  }
  return grow(idx, &idx->d_partials, &idx->partials_cap, static_cast<size_t>(r) * keys, "scratch");
}

// The next query's slot; at a wrap the stream first waits for all its earlier
// work (every tail that read the slots being reused).
int ring_next(bv_index* idx, cudaStream_t s, uint32_t* epoch, uint32_t* slot) {
  *epoch = ++idx->epoch;
  *slot = *epoch % idx->ring;
  if (*slot == 0) {
    BV_CUDA(idx, cudaEventRecord(idx->ev_ring, s), "ring event");
    BV_CUDA(idx, cudaStreamWaitEvent(s, idx->ev_ring, 0), "ring wait");
  }
  return BV_OK;
}

// Exact fp32 index: per query the flat scan (CTA top lists, WASM-SIMD f32
// arithmetic) then the tail (merge into the top k; re-rank off).
int enqueue_flat(bv_index* idx, const bv_search_args* a, uint32_t F, cudaStream_t s, bool alone) {
  uint32_t Fp = 32;
  while (Fp < F) Fp <<= 1;
  if (Fp <= 256u && bv::flat_scan_supported(idx->d_orig, idx->dim)) {
    // TMA-fed scan, finished by its last CTA: one launch per query
    const uint32_t BR = bv::flat_scan_block_rows();
    uint32_t capc = 1024;
    while (capc < 2 * Fp + BR || capc < 16 * Fp) capc <<= 1;
    const uint32_t check_blocks = (capc - 2 * Fp) / BR;
    const uint32_t two = static_cast<uint32_t>(idx->smem_per_sm) / 2u - 1024u;
    uint32_t stages = 0, per_sm = 2;
    size_t smem = 0;
    for (uint32_t lim : {two, static_cast<uint32_t>(idx->max_smem)}) {
      for (uint32_t st = 6; st >= 2 && !stages; --st) {
        const bv::FlatSmem lay = bv::flat_smem_layout(idx->dim, st, capc);
        if (lay.total <= lim) {
          stages = st;
          smem = lay.total;
        }
      }
      if (stages) break;
      per_sm = 1;
    }
    if (stages && capc <= static_cast<uint32_t>(bv::kSelMax * bv::kConsumerThreads)) {
      if (idx->flat_map_rows != idx->d_orig || idx->flat_map_n != idx->rows) {
        cudaError_t e = bv::encode_flat_rows_map(idx->flat_map, idx->d_orig, idx->dim, idx->rows);
        if (e != cudaSuccess) return cuda_fail(idx, e, "flat scan tensor map");
        idx->flat_map_rows = idx->d_orig;
        idx->flat_map_n = idx->rows;
      }
      const uint32_t nblocks = static_cast<uint32_t>((idx->rows + BR - 1) / BR);
      const uint32_t nks = (idx->dim + 31u) / 32u;
      const uint32_t nsm = static_cast<uint32_t>(idx->num_sms);
      const uint32_t all = per_sm * nsm;
      const uint32_t want = alone && a->nq == 1 ? all : (per_sm == 2 ? (nsm / 3u > 0 ? nsm / 3u : 1u) : nsm);
      const uint32_t grid = nblocks < want ? nblocks : want;
      int rc = ring_prepare(idx, static_cast<size_t>(nblocks < all ? nblocks : all) * Fp);
      if (rc) return rc;
      bv::ScanParams p;
      memset(&p, 0, sizeof(p));
      p.mask = a->mask;
      p.nrows = idx->rows;
      p.dim = idx->dim;
      p.stages = stages;
      p.F = F;
      p.Fp = Fp;
      p.capc = capc;
      p.fold = 1;
      p.k = a->k;
      p.rerank = 0;
      p.originals = idx->d_orig;
      p.row_base = idx->row_base;
      p.err = idx->d_err;
      const bool tracing = idx->d_trace && idx->trace_cap >= (static_cast<uint64_t>(grid) + 1) * 8;
      p.trace = tracing ? idx->d_trace : nullptr;
      const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
      for (uint32_t q = 0; q < a->nq; ++q) {
        p.query = a->queries + static_cast<size_t>(q) * idx->dim;
        uint32_t slot = 0;
        if ((rc = ring_next(idx, s, &p.epoch, &slot))) return rc;
        p.tile_ctr = idx->d_tile_ctr + slot;
        p.done = idx->d_done + slot;
        p.partials = idx->d_partials + static_cast<size_t>(slot) * idx->partials_slot;
        p.out_rows = a->out_rows + static_cast<size_t>(q) * a->k;
        p.out_scores = a->out_scores + static_cast<size_t>(q) * a->k;
        p.out_count = a->out_counts + q;
        p.cand_rows = cand ? a->cand_rows + static_cast<size_t>(q) * F : nullptr;
        p.cand_scores = cand ? a->cand_scores + static_cast<size_t>(q) * F : nullptr;
        p.cand_count = cand ? a->cand_counts + q : nullptr;
        cudaError_t e = bv::launch_flat_scan(idx->flat_map, p, nblocks, nks, check_blocks, grid, smem, s);
        if (e != cudaSuccess) return cuda_fail(idx, e, "flat scan launch");
      }
      idx->last_launches = a->nq;
      return BV_OK;
    }
  }
  const uint32_t G = (static_cast<uint32_t>(idx->rows) + bv::flat_rows_per_cta() - 1) / bv::flat_rows_per_cta();
  int rc = ring_prepare(idx, static_cast<size_t>(G) * Fp);
  if (rc) return rc;
  bv::TailParams t;
  memset(&t, 0, sizeof(t));
  t.partials = idx->d_partials;
  t.G = G;
  t.F = F;
  t.Fp = Fp;
  t.capc = Fp <= 256 ? (16 * Fp > 1024 ? 16 * Fp : 1024) : (2 * Fp > 1024 ? 2 * Fp : 1024);
  t.k = a->k;
  t.rerank = 0;
  t.originals = idx->d_orig;
  t.dim = idx->dim;
  t.row_base = idx->row_base;
  t.err = idx->d_err;
  t.rows_bytes = 0;
  const size_t tail_smem = bv::tail_smem_layout(idx->dim, t.capc, 0).total;
  for (uint32_t q = 0; q < a->nq; ++q) {
    const float* query = a->queries + static_cast<size_t>(q) * idx->dim;
    uint32_t epoch = 0, slot = 0;
    if ((rc = ring_next(idx, s, &epoch, &slot))) return rc;
    uint64_t* part = idx->d_partials + static_cast<size_t>(slot) * idx->partials_slot;
    t.partials = part;
    cudaError_t e = bv::launch_flat(idx->d_orig, query, a->mask, static_cast<uint32_t>(idx->rows), idx->dim, Fp,
                                    part, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "flat launch");
    t.query = query;
    t.out_rows = a->out_rows + static_cast<size_t>(q) * a->k;
    t.out_scores = a->out_scores + static_cast<size_t>(q) * a->k;
    t.out_count = a->out_counts + q;
    const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
    t.cand_rows = cand ? a->cand_rows + static_cast<size_t>(q) * F : nullptr;
    t.cand_scores = cand ? a->cand_scores + static_cast<size_t>(q) * F : nullptr;
    t.cand_count = cand ? a->cand_counts + q : nullptr;
    e = bv::launch_tail(t, tail_smem, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "tail launch");
  }
  idx->last_launches = 2 * a->nq;
  return BV_OK;
}

// Enqueue every query of `a` (device pointers) on `s`: per query the scan
// kernel (CTA candidate lists into the query's ring slot) then the tail kernel
// (merge + exact re-rank + outputs), chained by programmatic dependent launch.
int enqueue_search(bv_index* idx, const bv_search_args* a, uint32_t F, cudaStream_t s, bool alone = false) {
  if (idx->bits == 0) return enqueue_flat(idx, a, F, s, alone);
  Plan pl;
  int rc = plan_scan(idx, F, &pl, true, alone && a->nq == 1);
  if (rc) return rc;
  rc = ring_prepare(idx, static_cast<size_t>(pl.slots) * pl.Fp);
  if (rc) return rc;
  bv::ScanParams p;
  memset(&p, 0, sizeof(p));
  p.codes = idx->d_codes;
  p.scales = idx->d_scales;
  p.signs = idx->d_signs;
  p.seed = idx->seed;
  p.sign_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(idx->P)));
  p.mask = a->mask;
  p.nrows = idx->rows;
  p.dim = idx->dim;
  p.P = idx->P;
  p.rounds = idx->rounds;
  p.R = pl.sh.R;
  p.tile_rows = pl.tile_rows;
  p.tile_bytes = pl.tile_bytes;
  p.ntiles = pl.ntiles;
  p.stages = pl.stages;
  p.F = pl.F;
  p.Fp = pl.Fp;
  p.capc = pl.capc;
  p.check_tiles = pl.check_tiles;
  p.partials = idx->d_partials;
  p.err = idx->d_err;
  p.rowmap = idx->rowmap;
  const bool tracing = idx->d_trace && idx->trace_cap >= (static_cast<uint64_t>(pl.grid) + 1) * 8;
  p.trace = tracing ? idx->d_trace : nullptr;

  bv::TailParams t;
  memset(&t, 0, sizeof(t));
  t.partials = idx->d_partials;
  t.G = pl.grid;
  t.F = pl.F;
  t.Fp = pl.Fp;
  t.capc = pl.capc;
  t.k = a->k;
  t.rerank = a->rerank ? 1 : 0;
  t.originals = idx->d_orig;
  t.dim = idx->dim;
  t.row_base = idx->row_base;
  t.err = idx->d_err;
  t.rowmap = idx->rowmap;
  t.trace = tracing ? idx->d_trace + static_cast<size_t>(pl.grid) * 8 : nullptr;
  // gathered-row staging: as many rows of stride dim+4 as fit beside the rest
  const uint32_t row_bytes = (idx->dim + 4) * 4;
  const uint32_t fixed = bv::tail_smem_layout(idx->dim, pl.capc, 0).total + 256;
  uint32_t rows_bytes = static_cast<uint32_t>(idx->max_smem) > fixed ? static_cast<uint32_t>(idx->max_smem) - fixed : 0;
  const uint32_t want = pl.F * row_bytes;
  if (rows_bytes > want) rows_bytes = want;
  rows_bytes = rows_bytes / row_bytes * row_bytes;
  if (rows_bytes < row_bytes) return fail(BV_ERR_UNSUPPORTED, "re-rank row does not fit in shared memory");
  t.rows_bytes = rows_bytes;
  const size_t tail_smem = bv::tail_smem_layout(idx->dim, pl.capc, rows_bytes).total;

  if (pl.fold) {
    // one launch per query: its last CTA merges, re-ranks and writes the results
    p.fold = 1;
    p.k = a->k;
    p.rerank = a->rerank ? 1 : 0;
    p.originals = idx->d_orig;
    p.row_base = idx->row_base;
    for (uint32_t q = 0; q < a->nq; ++q) {
      p.query = a->queries + static_cast<size_t>(q) * idx->dim;
      uint32_t slot = 0;
      if ((rc = ring_next(idx, s, &p.epoch, &slot))) return rc;
      p.tile_ctr = idx->d_tile_ctr + slot;
      p.done = idx->d_done + slot;
      p.partials = idx->d_partials + static_cast<size_t>(slot) * idx->partials_slot;
      p.out_rows = a->out_rows + static_cast<size_t>(q) * a->k;
      p.out_scores = a->out_scores + static_cast<size_t>(q) * a->k;
      p.out_count = a->out_counts + q;
      const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
      p.cand_rows = cand ? a->cand_rows + static_cast<size_t>(q) * F : nullptr;
      p.cand_scores = cand ? a->cand_scores + static_cast<size_t>(q) * F : nullptr;
      p.cand_count = cand ? a->cand_counts + q : nullptr;
      p.cand_exact = cand && a->cand_exact ? a->cand_exact + static_cast<size_t>(q) * F : nullptr;
      cudaError_t e = launch_scan(static_cast<int>(idx->bits), static_cast<int>(idx->scoring), pl.sh, p, pl.grid,
                                  pl.smem, s);
      if (e == cudaErrorNotSupported)
        return fail(BV_ERR_UNSUPPORTED, "no scan kernel for bits=%u scoring=%u P=%u", idx->bits, idx->scoring,
                    idx->P);
      if (e != cudaSuccess) return cuda_fail(idx, e, "scan launch");
    }
    idx->last_launches = a->nq;
    return BV_OK;
  }
  for (uint32_t q = 0; q < a->nq; ++q) {
    p.query = a->queries + static_cast<size_t>(q) * idx->dim;
    uint32_t slot = 0;
    if ((rc = ring_next(idx, s, &p.epoch, &slot))) return rc;
    p.tile_ctr = idx->d_tile_ctr + slot;
    p.partials = idx->d_partials + static_cast<size_t>(slot) * idx->partials_slot;
    t.partials = p.partials;
    cudaError_t e = launch_scan(static_cast<int>(idx->bits), static_cast<int>(idx->scoring), pl.sh,
                                p, pl.grid, pl.smem, s);
    if (e == cudaErrorNotSupported)
      return fail(BV_ERR_UNSUPPORTED, "no scan kernel for bits=%u scoring=%u P=%u", idx->bits,
                  idx->scoring, idx->P);
    if (e != cudaSuccess) return cuda_fail(idx, e, "scan launch");
    t.query = p.query;
    t.out_rows = a->out_rows + static_cast<size_t>(q) * a->k;
    t.out_scores = a->out_scores + static_cast<size_t>(q) * a->k;
    t.out_count = a->out_counts + q;
    const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
    t.cand_rows = cand ? a->cand_rows + static_cast<size_t>(q) * F : nullptr;
    t.cand_scores = cand ? a->cand_scores + static_cast<size_t>(q) * F : nullptr;
    t.cand_count = cand ? a->cand_counts + q : nullptr;
    t.cand_exact = cand && a->cand_exact ? a->cand_exact + static_cast<size_t>(q) * F : nullptr;
    e = bv::launch_tail(t, tail_smem, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "tail launch");
  }
  idx->last_launches = 2 * a->nq;
  return BV_OK;
}

// A set device error flag (a scan wait that ran out) becomes BV_ERR_TIMEOUT
// and is cleared with the query counters it may have left behind.
int report_err_flag(bv_index* idx, uint32_t flag) {
  if (flag) {
    cudaMemset(idx->d_err, 0, 4);
    cudaMemset(idx->d_done, 0, kRing * sizeof(unsigned int));  // a cut-short query may have left a count
    return fail(BV_ERR_TIMEOUT, "scan kernel wait ran out of budget (flag 0x%x)", flag);
  }
  return BV_OK;
}

int check_err_flag(bv_index* idx) {
  uint32_t flag = 0;
  BV_CUDA(idx, cudaMemcpy(&flag, idx->d_err, 4, cudaMemcpyDeviceToHost), "error flag");
  return report_err_flag(idx, flag);
}

}  // namespace

extern "C" {

const char* bv_last_error(void) { return g_err.c_str(); }

int bv_create(const bv_config* cfg, bv_index** out) {
  if (!cfg || !out) return fail(BV_ERR_INVALID, "null config or output");
  *out = nullptr;
  if (cfg->dim == 0) return fail(BV_ERR_INVALID, "dimension must be a positive integer, got 0");
  if (cfg->bits != 8 && cfg->bits != 4 && cfg->bits != 1 && cfg->bits != 0)
    return fail(BV_ERR_INVALID, "quantBits %u not supported (ships 0, 1, 4, 8)", cfg->bits);
  if (cfg->metric > BV_METRIC_DOT)  // index.ts:135-137
    return fail(BV_ERR_INVALID,
                "quantized mode supports metric cosine/dot only (l2 quantization is later work)");
  if (cfg->scoring > BV_SCORE_HAMMING) return fail(BV_ERR_INVALID, "unknown scoring mode %u", cfg->scoring);
  if (cfg->bits == 0 && cfg->scoring != BV_SCORE_ASYM)
    return fail(BV_ERR_INVALID, "the exact fp32 index (bits 0) has no quantized scoring");
  if (cfg->scoring == BV_SCORE_HAMMING && cfg->bits != 1)
    return fail(BV_ERR_INVALID, "hamming scoring needs 1-bit codes");
  const uint32_t P = pad_to_pow2(cfg->dim);
  if (P > kMaxPadded) return fail(BV_ERR_UNSUPPORTED, "dimension %u pads beyond %u", cfg->dim, kMaxPadded);
  if (cfg->bits == 4 && P % 8) return fail(BV_ERR_INVALID, "paddedDim must be a multiple of 8 for 4-bit");
  if (cfg->bits == 1 && P % 32)
    return fail(BV_ERR_INVALID, "paddedDim must be a multiple of 32 for 1-bit");
  bv_index* idx = new bv_index();
  idx->device = cfg->device;
  idx->dim = cfg->dim;
  idx->bits = cfg->bits;
  idx->metric = cfg->metric;
  idx->seed = cfg->seed;
  idx->rounds = cfg->rounds;
  idx->scoring = cfg->scoring;
  idx->row_base = cfg->row_base;
  idx->P = P;
  if (const char* gp = std::getenv("BV_GEMM_PAIR")) idx->gemm_pair = std::strcmp(gp, "1") == 0;
  idx->R = cfg->bits ? bv::code_row_bytes(static_cast<int>(cfg->bits), P) : 0;  // bits 0: originals only
  auto bail = [&](int rc) {
    bv_destroy(idx);
    return rc;
  };
  cudaError_t e = cudaSetDevice(cfg->device);
  if (e != cudaSuccess) return bail(cuda_fail(nullptr, e, "cudaSetDevice"));
  cudaDeviceGetAttribute(&idx->num_sms, cudaDevAttrMultiProcessorCount, cfg->device);
  cudaDeviceGetAttribute(&idx->max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, cfg->device);
  cudaDeviceGetAttribute(&idx->smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, cfg->device);
  if ((e = cudaStreamCreateWithFlags(&idx->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaEventCreate(&idx->ev0)) != cudaSuccess || (e = cudaEventCreate(&idx->ev1)) != cudaSuccess)
    return bail(cuda_fail(nullptr, e, "stream"));
  // rotator.ts:44-58: per round, signs from mulberry32((seed ^ 0x9e3779b9*(r+1)) >>> 0),
  // pre-scaled by f32(+-1 * (1/sqrt(P) in f64)).
  const size_t ns = static_cast<size_t>(P) * (cfg->rounds ? cfg->rounds : 1);
  float* hs = new float[ns];
  const double inv = 1.0 / std::sqrt(static_cast<double>(P));
  for (uint32_t r = 0; r < cfg->rounds; ++r) {
    uint32_t st = cfg->seed ^ (0x9e3779b9u * (r + 1u));
    for (uint32_t i = 0; i < P; ++i) {
      const double s = mulberry32_next(&st) < 0x80000000u ? -1.0 : 1.0;
      hs[static_cast<size_t>(r) * P + i] = static_cast<float>(s * inv);
    }
  }
  e = cudaMalloc(&idx->d_signs, ns * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(idx->d_signs, hs, ns * sizeof(float), cudaMemcpyHostToDevice);
  delete[] hs;
  if (e == cudaSuccess) e = cudaMalloc(&idx->d_tile_ctr, kRing * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&idx->d_done, kRing * sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(idx->d_done, 0, kRing * sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&idx->ev_ring, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMalloc(&idx->d_err, 16);
  if (e == cudaSuccess) e = cudaMemset(idx->d_tile_ctr, 0, kRing * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(idx->d_err, 0, 16);
  if (e != cudaSuccess) return bail(cuda_fail(nullptr, e, "index buffers"));
  *out = idx;
  return BV_OK;
}

int bv_destroy(bv_index* idx) {
  if (!idx) return BV_OK;
  if (idx->stream) cudaStreamSynchronize(idx->stream);
  cudaFree(idx->d_codes);
  cudaFree(idx->d_scales);
  cudaFree(idx->d_orig);
  cudaFree(idx->d_signs);
  cudaFree(idx->d_partials);
  cudaFree(idx->d_tile_ctr);
  cudaFree(idx->d_done);
  cudaFree(idx->d_err);
  cudaFree(idx->d_q);
  cudaFree(idx->d_mask);
  cudaFree(idx->d_rows);
  cudaFree(idx->d_out);
  cudaFree(idx->d_ctiles);
  cudaFree(idx->d_posfac);
  cudaFree(idx->d_posrow);
  cudaFree(idx->d_tmax);
  cudaFree(idx->d_sfac);
  cudaFree(idx->d_sids);
  cudaFree(idx->d_stmp);
  cudaFree(idx->d_qtiles);
  cudaFree(idx->d_qfac);
  cudaFree(idx->d_thr);
  cudaFree(idx->d_bcnt);
  cudaFree(idx->d_bcand);
  cudaFree(idx->d_scnt);
  cudaFree(idx->d_overflow);
  cudaFree(idx->d_cwoff);
  cudaFree(idx->d_cbsum);
  cudaFree(idx->d_cmap);
  cudaFree(idx->d_cctiles);
  cudaFree(idx->d_cposfac);
  cudaFree(idx->d_cposrow);
  cudaFree(idx->d_ctmax);
  cudaFree(idx->d_gcodes);
  cudaFree(idx->d_gscales);
  cudaFree(idx->d_growmap);
  cudaFree(idx->d_goffs);
  if (idx->h_pin) cudaFreeHost(idx->h_pin);
  if (idx->ev0) cudaEventDestroy(idx->ev0);
  if (idx->ev1) cudaEventDestroy(idx->ev1);
  if (idx->ev_ring) cudaEventDestroy(idx->ev_ring);
  if (idx->batch) {
    for (cudaEvent_t e : idx->batch->ev) cudaEventDestroy(e);
    delete idx->batch;
  }
  if (idx->stream) cudaStreamDestroy(idx->stream);
  delete idx;
  return BV_OK;
}

int bv_size(const bv_index* idx, uint64_t* rows) {
  if (!idx || !rows) return fail(BV_ERR_INVALID, "null argument");
  *rows = idx->rows;
  return BV_OK;
}

static int append_impl(bv_index* idx, const float* rows, uint64_t count, bool device, cudaStream_t s) {
  if (!idx) return fail(BV_ERR_INVALID, "null index");
  if (idx->lost) return fail(BV_ERR_DEVICE_LOST, "%s", kLostMsg);
  if (count == 0) return BV_OK;
  if (!rows) return fail(BV_ERR_INVALID, "rows is null");
  if (idx->rows + count > 0xFFFFFFFEull)
    return fail(BV_ERR_UNSUPPORTED, "a shard holds at most 2^32-2 rows");
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  if (s) BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
  int rc = ensure_capacity(idx, idx->rows + count);
  if (rc) return rc;
  float* dst = idx->d_orig + idx->rows * idx->dim;
  const size_t bytes = count * idx->dim * sizeof(float);
  BV_CUDA(idx, cudaMemcpyAsync(dst, rows, bytes, device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                               idx->stream), "append copy");
  if (idx->bits) {  // the exact fp32 index keeps the originals only
    cudaError_t e = bv::launch_encode(static_cast<int>(idx->bits), dst, count, idx->dim, idx->P, idx->d_signs,
                                      idx->rounds, idx->d_codes + idx->rows * idx->R,
                                      idx->d_scales + idx->rows, idx->R, idx->stream);
    if (e != cudaSuccess) return cuda_fail(idx, e, "encode");
  }
  BV_CUDA(idx, cudaStreamSynchronize(idx->stream), "encode");
  idx->rows += count;
  return BV_OK;
}

int bv_append(bv_index* idx, const float* rows, uint64_t count) {
  return append_impl(idx, rows, count, false, nullptr);
}

int bv_append_device(bv_index* idx, const float* rows_dev, uint64_t count, void* stream) {
  return append_impl(idx, rows_dev, count, true, static_cast<cudaStream_t>(stream));
}

int bv_search_async(bv_index* idx, const bv_search_args* a, void* stream) {
  uint32_t F = 0;
  int rc = check_args(idx, a, &F);
  if (rc) return rc;
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : idx->stream;
  if (idx->rows == 0 || a->nq == 0) {  // quant.ts:184: an empty index returns []
    if (a->nq) BV_CUDA(idx, cudaMemsetAsync(a->out_counts, 0, a->nq * 4, s), "memset");
    if (a->nq && a->cand_counts) BV_CUDA(idx, cudaMemsetAsync(a->cand_counts, 0, a->nq * 4, s), "memset");
    idx->last_launches = 0;
    return BV_OK;
  }
  return enqueue_search(idx, a, F, s);
}

int bv_search_async_n(bv_index* const* idx, const bv_search_args* args, uint32_t n, void* stream) {
  if (n && (!idx || !args)) return fail(BV_ERR_INVALID, "null index or args array");
  for (uint32_t i = 0; i < n; ++i) {
    const int rc = bv_search_async(idx[i], args + i, stream);
    if (rc) return rc;
  }
  return BV_OK;
}

int bv_search(bv_index* idx, const bv_search_args* a) {
  uint32_t F = 0;
  int rc = check_args(idx, a, &F);
  if (rc) return rc;
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  const uint32_t nq = a->nq;
  if (idx->rows == 0 || nq == 0) {
    for (uint32_t q = 0; q < nq; ++q) a->out_counts[q] = 0;
    if (a->cand_counts)
      for (uint32_t q = 0; q < nq; ++q) a->cand_counts[q] = 0;
    idx->last_launches = 0;
    return BV_OK;
  }
  const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
  const size_t qn = static_cast<size_t>(nq) * idx->dim;
  const size_t on = static_cast<size_t>(nq) * a->k;
  const size_t cn = cand ? static_cast<size_t>(nq) * F : 0;
  const size_t xn = cand && a->cand_exact ? cn : 0;
  // device staging: [rows on | scores on | counts nq | cand rows cn | cand scores cn | cand counts nq |
  //                  cand exact xn]
  const size_t out_words = 2 * on + nq + 2 * cn + (cand ? nq : 0) + xn;
  if ((rc = grow(idx, &idx->d_q, &idx->q_cap, qn, "query staging"))) return rc;
  if ((rc = grow(idx, &idx->d_out, &idx->out_cap, out_words, "output staging"))) return rc;
  const size_t mw = a->mask ? (idx->rows + 31) / 32 : 0;
  if (mw && (rc = grow(idx, &idx->d_mask, &idx->mask_cap, mw, "mask staging"))) return rc;
  const size_t pin_bytes = (qn > out_words ? qn : out_words) * 4;
  if ((rc = grow_pinned(idx, pin_bytes + 16))) return rc;  // + the error flag
  memcpy(idx->h_pin, a->queries, qn * 4);
  BV_CUDA(idx, cudaEventRecord(idx->ev0, idx->stream), "event");
  BV_CUDA(idx, cudaMemcpyAsync(idx->d_q, idx->h_pin, qn * 4, cudaMemcpyHostToDevice, idx->stream), "H2D");
  if (mw)
    BV_CUDA(idx, cudaMemcpyAsync(idx->d_mask, a->mask, mw * 4, cudaMemcpyHostToDevice, idx->stream), "H2D");
  bv_search_args d = *a;
  d.queries = idx->d_q;
  d.mask = mw ? idx->d_mask : nullptr;
  d.mask_words = mw;
  d.out_rows = idx->d_out;
  d.out_scores = reinterpret_cast<float*>(idx->d_out + on);
  d.out_counts = idx->d_out + 2 * on;
  d.cand_rows = cand ? idx->d_out + 2 * on + nq : nullptr;
  d.cand_scores = cand ? reinterpret_cast<float*>(idx->d_out + 2 * on + nq + cn) : nullptr;
  d.cand_counts = cand ? idx->d_out + 2 * on + nq + 2 * cn : nullptr;
  d.cand_exact = xn ? reinterpret_cast<float*>(idx->d_out + 2 * on + 2 * nq + 2 * cn) : nullptr;
  if (idx->scoring != BV_SCORE_ASYM && nq >= kBatchMinQueries) {
    // a batch on the tensor cores: the same results as the per-query scans
    if ((rc = bv_search_batch(idx, &d, idx->stream))) return rc;
  } else if ((rc = enqueue_search(idx, &d, F, idx->stream, true))) {
    return rc;
  }
  uint32_t* h_flag = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(idx->h_pin) + pin_bytes);
  BV_CUDA(idx, cudaMemcpyAsync(idx->h_pin, idx->d_out, out_words * 4, cudaMemcpyDeviceToHost, idx->stream),
          "D2H");
  BV_CUDA(idx, cudaMemcpyAsync(h_flag, idx->d_err, 4, cudaMemcpyDeviceToHost, idx->stream), "error flag");
  BV_CUDA(idx, cudaEventRecord(idx->ev1, idx->stream), "event");
  BV_CUDA(idx, cudaStreamSynchronize(idx->stream), "search");
  cudaEventElapsedTime(&idx->last_ms, idx->ev0, idx->ev1);
  if ((rc = report_err_flag(idx, *h_flag))) return rc;
  const uint32_t* h = static_cast<const uint32_t*>(idx->h_pin);
  memcpy(a->out_rows, h, on * 4);
  memcpy(a->out_scores, h + on, on * 4);
  memcpy(a->out_counts, h + 2 * on, nq * 4);
  if (cand) {
    memcpy(a->cand_rows, h + 2 * on + nq, cn * 4);
    memcpy(a->cand_scores, h + 2 * on + nq + cn, cn * 4);
    memcpy(a->cand_counts, h + 2 * on + nq + 2 * cn, nq * 4);
    if (xn) memcpy(a->cand_exact, h + 2 * on + 2 * nq + 2 * cn, xn * 4);
  }
  return BV_OK;
}

int bv_query_rows_exact(bv_index* idx, const float* query, const uint32_t* rows, uint32_t nrows,
                        uint32_t k, uint32_t* out_rows, float* out_scores, uint32_t* out_count) {
  if (!idx || !query || !out_rows || !out_scores || !out_count) return fail(BV_ERR_INVALID, "null argument");
  if (idx->lost) return fail(BV_ERR_DEVICE_LOST, "%s", kLostMsg);
  if (nrows > 4096) return fail(BV_ERR_INVALID, "exact row scan takes at most 4096 rows, got %u", nrows);
  if (nrows && !rows) return fail(BV_ERR_INVALID, "rows is null");
  for (uint32_t i = 0; i < nrows; ++i)
    if (rows[i] >= idx->rows) return fail(BV_ERR_INVALID, "row %u out of range (%llu rows)", rows[i],
                                          static_cast<unsigned long long>(idx->rows));
  if (nrows == 0 || k == 0) {
    *out_count = 0;
    return BV_OK;
  }
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  int rc;
  if ((rc = grow(idx, &idx->d_q, &idx->q_cap, idx->dim, "query staging"))) return rc;
  if ((rc = grow(idx, &idx->d_rows, &idx->rows_cap, nrows, "row staging"))) return rc;
  if ((rc = grow(idx, &idx->d_out, &idx->out_cap, 2 * static_cast<size_t>(k) + 1, "output staging"))) return rc;
  BV_CUDA(idx, cudaMemcpyAsync(idx->d_q, query, idx->dim * 4, cudaMemcpyHostToDevice, idx->stream), "H2D");
  BV_CUDA(idx, cudaMemcpyAsync(idx->d_rows, rows, nrows * 4, cudaMemcpyHostToDevice, idx->stream), "H2D");
  cudaError_t e = bv::launch_exact_rows(idx->d_orig, idx->dim, idx->d_q, idx->d_rows, nrows, k,
                                        idx->row_base, idx->d_out, reinterpret_cast<float*>(idx->d_out + k),
                                        idx->d_out + 2 * k, idx->stream);
  if (e != cudaSuccess) return cuda_fail(idx, e, "exact scan");
  uint32_t n = 0;
  BV_CUDA(idx, cudaMemcpyAsync(&n, idx->d_out + 2 * k, 4, cudaMemcpyDeviceToHost, idx->stream), "D2H");
  BV_CUDA(idx, cudaMemcpyAsync(out_rows, idx->d_out, k * 4, cudaMemcpyDeviceToHost, idx->stream), "D2H");
  BV_CUDA(idx, cudaMemcpyAsync(out_scores, idx->d_out + k, k * 4, cudaMemcpyDeviceToHost, idx->stream), "D2H");
  BV_CUDA(idx, cudaStreamSynchronize(idx->stream), "exact scan");
  *out_count = n;
  idx->last_launches = 1;
  return BV_OK;
}

int bv_export_codes(const bv_index* idx, uint64_t row0, uint64_t count, uint32_t* words, float* scales) {
  if (!idx) return fail(BV_ERR_INVALID, "null index");
  if (row0 + count > idx->rows) return fail(BV_ERR_INVALID, "rows out of range");
  bv_index* m = const_cast<bv_index*>(idx);
  BV_CUDA(m, cudaSetDevice(idx->device), "cudaSetDevice");
  if (words)
    BV_CUDA(m, cudaMemcpy(words, idx->d_codes + row0 * idx->R, count * idx->R, cudaMemcpyDeviceToHost), "D2H");
  if (scales)
    BV_CUDA(m, cudaMemcpy(scales, idx->d_scales + row0, count * 4, cudaMemcpyDeviceToHost), "D2H");
  return BV_OK;
}

int bv_export_originals(const bv_index* idx, uint64_t row0, uint64_t count, float* out) {
  if (!idx || (count && !out)) return fail(BV_ERR_INVALID, "null argument");
  if (row0 + count > idx->rows) return fail(BV_ERR_INVALID, "rows out of range");
  if (count == 0) return BV_OK;
  bv_index* m = const_cast<bv_index*>(idx);
  BV_CUDA(m, cudaSetDevice(idx->device), "cudaSetDevice");
  BV_CUDA(m, cudaStreamSynchronize(idx->stream), "sync");
  BV_CUDA(m, cudaMemcpy(out, idx->d_orig + row0 * idx->dim, count * idx->dim * sizeof(float), cudaMemcpyDeviceToHost),
          "D2H");
  return BV_OK;
}

int bv_get_stats(const bv_index* idx, bv_stats* out) {
  if (!idx || !out) return fail(BV_ERR_INVALID, "null argument");
  out->rows = idx->rows;
  out->dim = idx->dim;
  out->padded_dim = idx->P;
  out->bits = idx->bits;
  out->words_per_row = idx->R / 4;
  out->chunks = 1;
  out->last_query_gpu_ms = idx->last_ms;
  out->device_bytes = idx->cap_rows * (idx->R + 4 + static_cast<uint64_t>(idx->dim) * 4);
  return BV_OK;
}

int bv_set_phase_trace(bv_index* idx, uint64_t* trace_dev, uint64_t capacity) {
  if (!idx) return fail(BV_ERR_INVALID, "null index");
  idx->d_trace = trace_dev;
  idx->trace_cap = trace_dev ? capacity : 0;
  return BV_OK;
}

int bv_launches_last_search(const bv_index* idx, uint32_t* launches) {
  if (!idx || !launches) return fail(BV_ERR_INVALID, "null argument");
  *launches = idx->last_launches;
  return BV_OK;
}

}  // extern "C"

int bv_merge_shards(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t fetch, uint32_t k,
                    uint32_t* out_rows, float* out_scores, uint32_t* out_counts, void* stream) {
  if (!gathered || !out_rows || !out_scores || !out_counts) return fail(BV_ERR_INVALID, "null argument");
  if (world == 0 || world > bv::merge_max_world())
    return fail(BV_ERR_INVALID, "world %u outside [1, %u]", world, bv::merge_max_world());
  if (k == 0 || fetch < k) return fail(BV_ERR_INVALID, "need 1 <= k <= fetch (k=%u, fetch=%u)", k, fetch);
  if (fetch > kMaxFetch) return fail(BV_ERR_UNSUPPORTED, "fetch %u exceeds %u", fetch, kMaxFetch);
  if (nq == 0) return BV_OK;
  const cudaError_t e = bv::launch_merge_shards(gathered, world, nq, fetch, k, out_rows, out_scores, out_counts,
                                                static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue)
    return fail(BV_ERR_UNSUPPORTED, "merge of %u shards x %u candidates does not fit in shared memory", world,
                fetch);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "merge launch");
  return BV_OK;
}

int bv_merge_topk(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t k, uint32_t* out_rows,
                  float* out_scores, uint32_t* out_counts, void* stream) {
  if (nq && (!gathered || !out_rows || !out_scores || !out_counts)) return fail(BV_ERR_INVALID, "null argument");
  if (world == 0 || world > bv::merge_max_world())
    return fail(BV_ERR_INVALID, "world %u outside [1, %u]", world, bv::merge_max_world());
  if (k == 0 || k > kMaxFetch) return fail(BV_ERR_INVALID, "k %u outside [1, %u]", k, kMaxFetch);
  if (nq == 0) return BV_OK;
  const cudaError_t e = bv::launch_merge_topk(gathered, world, nq, k, out_rows, out_scores, out_counts,
                                              static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue)
    return fail(BV_ERR_UNSUPPORTED, "merge of %u shards x %u results does not fit in shared memory", world, k);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "merge launch");
  return BV_OK;
}

// ------------------------------------------------------- batched search
namespace {

// Grow a device buffer to `need` elements keeping its first `keep` elements.
template <class T>
int grow_keep(bv_index* idx, T** p, size_t* cap, size_t need, size_t keep, cudaStream_t s, const char* what) {
  if (*cap >= need) return BV_OK;
  size_t n = *cap ? *cap : 1;
  while (n < need) n *= 2;
  T* q = nullptr;
  cudaError_t e = cudaMalloc(&q, n * sizeof(T));
  if (e != cudaSuccess) return cuda_fail(idx, e, what);
  if (keep && *p) {
    e = cudaMemcpyAsync(q, *p, keep * sizeof(T), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
      cudaFree(q);
      return cuda_fail(idx, e, what);
    }
  }
  cudaFree(*p);
  *p = q;
  *cap = n;
  return BV_OK;
}

uint64_t gcd_u64(uint64_t a, uint64_t b) {
  while (b) {
    const uint64_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

// Inverse of g modulo K (gcd(g, K) = 1).
uint32_t inv_mod(uint32_t g, uint32_t K) {
  int64_t t = 0, nt = 1, r = K, nr = g;
  while (nr) {
    const int64_t q = r / nr;
    const int64_t a = t - q * nt;
    t = nt;
    nt = a;
    const int64_t b = r - q * nr;
    r = nr;
    nr = b;
  }
  return static_cast<uint32_t>(t < 0 ? t + K : t);
}

// Rows for positions [pos0, pos0 + n): `rows` (or row0 + i when null) in
// ascending order of their score factor, tiles scattered (scatter_tiles_kernel);
// the result is idx->d_sids + n.
int sort_rows_by_factor(bv_index* idx, const uint32_t* rows, uint32_t row0, uint32_t n, uint32_t pos0,
                        cudaStream_t s) {
  int rc;
  if ((rc = grow(idx, &idx->d_sfac, &idx->sfac_cap, 2 * static_cast<size_t>(n), "sort scratch"))) return rc;
  if ((rc = grow(idx, &idx->d_sids, &idx->sids_cap, 2 * static_cast<size_t>(n), "sort scratch"))) return rc;
  size_t tmp = 0;
  cudaError_t e = bv::launch_sort_rows(nullptr, &tmp, idx->d_sfac + n, idx->d_sfac, idx->d_sids + n, idx->d_sids,
                                       n, s);
  if (e != cudaSuccess) return cuda_fail(idx, e, "sort size");
  if ((rc = grow(idx, &idx->d_stmp, &idx->stmp_cap, tmp + 16, "sort scratch"))) return rc;
  e = bv::launch_factor(idx->bits, idx->d_scales, rows, row0, n, idx->d_sfac + n, idx->d_sids + n, s);
  if (e == cudaSuccess) {
    size_t cap = idx->stmp_cap;
    e = bv::launch_sort_rows(idx->d_stmp, &cap, idx->d_sfac + n, idx->d_sfac, idx->d_sids + n, idx->d_sids, n, s);
  }
  if (e == cudaSuccess) {
    const uint32_t head = static_cast<uint32_t>(
        std::min<uint64_t>(n, (bv::kBRowTile - pos0 % bv::kBRowTile) % bv::kBRowTile));
    const uint32_t K = (n - head) / bv::kBRowTile;
    uint32_t g = 1, ginv = 1;
    if (K > 1) {
      g = static_cast<uint32_t>(static_cast<double>(K) * 0.381966) | 1u;
      while (gcd_u64(g, K) != 1) ++g;
      ginv = inv_mod(g % K, K);
    }
    e = bv::launch_scatter_tiles(idx->d_sids, idx->d_sids + n, n, head, K > 1 ? K : 1, ginv, s);
  }
  if (e != cudaSuccess) return cuda_fail(idx, e, "sort");
  return BV_OK;
}

// Bring the MMA tiles up to date with the appended rows: the new block of
// rows, sorted by factor, fills positions [mma_rows, rows).
int ensure_mma(bv_index* idx, cudaStream_t s) {
  if (idx->mma_rows >= idx->rows) return BV_OK;
  const uint32_t KB = (idx->P + bv::kKBlock - 1) / bv::kKBlock;
  const size_t tiles = (idx->rows + bv::kBRowTile - 1) / bv::kBRowTile;
  const size_t kept_tiles = (idx->mma_rows + bv::kBRowTile - 1) / bv::kBRowTile;
  int rc;
  if ((rc = grow_keep(idx, &idx->d_ctiles, &idx->ctiles_cap, tiles * KB * bv::kBRowTileBytes,
                      kept_tiles * KB * bv::kBRowTileBytes, s, "batch tiles")))
    return rc;
  if ((rc = grow_keep(idx, &idx->d_posfac, &idx->posfac_cap, tiles * bv::kBRowTile, idx->mma_rows, s,
                      "batch factors")))
    return rc;
  if ((rc = grow_keep(idx, &idx->d_posrow, &idx->posrow_cap, tiles * bv::kBRowTile, idx->mma_rows, s,
                      "batch rows")))
    return rc;
  if ((rc = grow_keep(idx, &idx->d_tmax, &idx->tmax_cap, tiles, kept_tiles, s, "batch factors"))) return rc;
  const uint32_t n = static_cast<uint32_t>(idx->rows - idx->mma_rows);
  if ((rc = sort_rows_by_factor(idx, nullptr, static_cast<uint32_t>(idx->mma_rows), n,
                                static_cast<uint32_t>(idx->mma_rows), s)))
    return rc;
  bv::ExpandParams ep;
  ep.codes = idx->d_codes;
  ep.scales = idx->d_scales;
  ep.R = idx->R;
  ep.P = idx->P;
  ep.KB = KB;
  ep.bits = idx->bits;
  ep.rows = idx->d_sids + n;
  ep.pos0 = static_cast<uint32_t>(idx->mma_rows);
  ep.count = n;
  ep.total = static_cast<uint32_t>(idx->rows);
  ep.tiles = idx->d_ctiles;
  ep.posfac = idx->d_posfac;
  ep.posrow = idx->d_posrow;
  ep.tmax = idx->d_tmax;
  const cudaError_t e = bv::launch_expand(ep, s);
  if (e != cudaSuccess) return cuda_fail(idx, e, "batch expand");
  idx->mma_rows = idx->rows;
  return BV_OK;
}

}  // namespace

namespace {

// Device-time accounting of a batched search (bv_set_batch_timing): events
// recorded on the search stream around each phase's launches, summed once
// the search has synchronised.
enum BatchPhase : int { kPhPrep = 0, kPhGemm = 1, kPhSelect = 2, kPhTail = 3, kPhCompact = 4, kPhCount = 5 };

struct PhaseClock {
  bv_index* idx;
  cudaStream_t s;
  int open = -1;
  explicit PhaseClock(bv_index* i, cudaStream_t st) : idx(i), s(st) {}
  int begin(int ph);
  int end();
};

}  // namespace

namespace {

bv_batch_state* batch_state(bv_index* idx) {
  if (!idx->batch) idx->batch = new bv_batch_state();
  return idx->batch;
}

int PhaseClock::begin(int ph) {
  bv_batch_state* b = batch_state(idx);
  if (!b->timing) return BV_OK;
  if (b->used + 2 > b->ev.size()) {
    cudaEvent_t e;
    for (int i = 0; i < 2; ++i) {
      BV_CUDA(idx, cudaEventCreate(&e), "timing event");
      b->ev.push_back(e);
    }
  }
  BV_CUDA(idx, cudaEventRecord(b->ev[b->used], s), "timing event");
  b->marks.emplace_back(ph, b->used);
  b->used += 2;
  open = ph;
  return BV_OK;
}

int PhaseClock::end() {
  bv_batch_state* b = batch_state(idx);
  if (!b->timing || open < 0) return BV_OK;
  BV_CUDA(idx, cudaEventRecord(b->ev[b->marks.back().second + 1], s), "timing event");
  open = -1;
  return BV_OK;
}

// Fold the recorded phases into the profile (the stream has synchronised).
int fold_phases(bv_index* idx) {
  bv_batch_state* b = batch_state(idx);
  if (!b->timing) return BV_OK;
  for (const auto& m : b->marks) {
    float ms = 0.0f;
    BV_CUDA(idx, cudaEventElapsedTime(&ms, b->ev[m.second], b->ev[m.second + 1]), "timing");
    float* dst = m.first == kPhPrep ? &b->prof.prep_ms
                 : m.first == kPhGemm ? &b->prof.gemm_ms
                 : m.first == kPhSelect ? &b->prof.select_ms
                 : m.first == kPhTail ? &b->prof.tail_ms : &b->prof.compact_ms;
    *dst += ms;
    if (m.first == kPhGemm) ++b->prof.gemm_launches;
  }
  b->marks.clear();
  b->used = 0;
  return BV_OK;
}

// Prep + rounds of (GEMM, select) of a batched search: on return (stream
// synchronised) idx->d_bcand holds per query its best F keys (local rows;
// sorted descending for Fp <= 256, else unsorted), zero padded to Fp.
int batch_rounds(bv_index* idx, const bv_search_args* a, uint32_t F, cudaStream_t s) {
  int rc;
  bv_batch_state* bs = batch_state(idx);
  bs->pending = false;
  bs->empty = false;
  bs->prof = bv_batch_profile{};
  bs->marks.clear();
  bs->used = 0;
  PhaseClock clk(idx, s);
  const uint32_t nq = a->nq;
  if ((rc = ensure_mma(idx, s))) return rc;
  uint32_t Fp = 32;
  while (Fp < F) Fp <<= 1;
  const uint32_t cap = Fp * 16 > 4096 ? Fp * 16 : 4096;  // <= 16384 (F <= 1024)
  const uint32_t KB = (idx->P + bv::kKBlock - 1) / bv::kKBlock;
  const uint32_t nqt = (nq + bv::kBQTile - 1) / bv::kBQTile;
  bs->nq = nq;
  bs->F = F;
  bs->Fp = Fp;
  bs->cap = cap;
  // A mask that keeps at most half the rows: contract only the kept rows,
  // gathered into their own tiles (their order, hence the tie rule, is kept).
  bool compact = false;
  uint32_t kept = static_cast<uint32_t>(idx->rows);
  if (a->mask) {
    if ((rc = clk.begin(kPhCompact))) return rc;
    const uint64_t words = (idx->rows + 31) / 32;
    const uint64_t nb = (words + bv::compact_block_words() - 1) / bv::compact_block_words();
    if ((rc = grow(idx, &idx->d_cwoff, &idx->cwoff_cap, words, "filter scratch"))) return rc;
    if ((rc = grow(idx, &idx->d_cbsum, &idx->cbsum_cap, nb + 1, "filter scratch"))) return rc;
    cudaError_t e = bv::launch_mask_count(a->mask, idx->rows, idx->d_cwoff, idx->d_cbsum, idx->d_cbsum + nb, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "filter count");
    BV_CUDA(idx, cudaMemcpyAsync(&kept, idx->d_cbsum + nb, 4, cudaMemcpyDeviceToHost, s), "filter count");
    BV_CUDA(idx, cudaStreamSynchronize(s), "filter count");
    compact = static_cast<uint64_t>(kept) * 2 <= idx->rows;
    if (compact && kept > 0) {
      const size_t ct = (kept + bv::kBRowTile - 1) / bv::kBRowTile;
      if ((rc = grow(idx, &idx->d_cmap, &idx->cmap_cap, kept, "filter rows"))) return rc;
      if ((rc = grow(idx, &idx->d_cctiles, &idx->cctiles_cap, ct * KB * bv::kBRowTileBytes, "filter tiles")))
        return rc;
      if ((rc = grow(idx, &idx->d_cposfac, &idx->cposfac_cap, ct * bv::kBRowTile, "filter tiles"))) return rc;
      if ((rc = grow(idx, &idx->d_cposrow, &idx->cposrow_cap, ct * bv::kBRowTile, "filter tiles"))) return rc;
      if ((rc = grow(idx, &idx->d_ctmax, &idx->ctmax_cap, ct, "filter tiles"))) return rc;
      e = bv::launch_row_map(a->mask, idx->rows, idx->d_cwoff, idx->d_cbsum, idx->d_cmap, s);
      if (e != cudaSuccess) return cuda_fail(idx, e, "filter rows");
      if ((rc = sort_rows_by_factor(idx, idx->d_cmap, 0, kept, 0, s))) return rc;
      bv::ExpandParams ep;
      ep.codes = idx->d_codes;
      ep.scales = idx->d_scales;
      ep.R = idx->R;
      ep.P = idx->P;
      ep.KB = KB;
      ep.bits = idx->bits;
      ep.rows = idx->d_sids + kept;
      ep.pos0 = 0;
      ep.count = kept;
      ep.total = kept;
      ep.tiles = idx->d_cctiles;
      ep.posfac = idx->d_cposfac;
      ep.posrow = idx->d_cposrow;
      ep.tmax = idx->d_ctmax;
      e = bv::launch_expand(ep, s);
      if (e != cudaSuccess) return cuda_fail(idx, e, "filter compaction");
    }
    if ((rc = clk.end())) return rc;
  }
  idx->last_kept = kept;
  bs->prof.kept_rows = kept;
  bs->prof.nq = nq;
  if (a->mask && kept == 0) {  // nothing passes the filter
    BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
    bs->empty = true;
    bs->launches = 3;
    bs->rounds = 0;
    bs->pending = true;
    return fold_phases(idx);
  }
  const uint32_t npos = compact ? kept : static_cast<uint32_t>(idx->rows);
  const uint32_t T = static_cast<uint32_t>((static_cast<uint64_t>(npos) + bv::kBRowTile - 1) / bv::kBRowTile);
  bs->prof.gemm_macs = static_cast<double>(nq) * static_cast<double>(npos) * static_cast<double>(idx->P);
  // query tiles for an even count (the pair GEMM takes two at a time; an odd
  // last tile's partner holds no valid query)
  const uint32_t nqt_pad = (nqt + 1u) & ~1u;
  if ((rc = grow(idx, &idx->d_qtiles, &idx->qtiles_cap, static_cast<size_t>(nqt_pad) * KB * bv::kBQTileBytes,
                 "batch queries")))
    return rc;
  if ((rc = grow(idx, &idx->d_qfac, &idx->qfac_cap, nq, "batch queries"))) return rc;
  if ((rc = grow(idx, &idx->d_thr, &idx->thr_cap, nq, "batch thresholds"))) return rc;
  if ((rc = grow(idx, &idx->d_bcnt, &idx->bcnt_cap, 2 * static_cast<size_t>(nq), "batch counts"))) return rc;
  if ((rc = grow(idx, &idx->d_bcand, &idx->bcand_cap, static_cast<size_t>(nq) * cap, "batch candidates")))
    return rc;
  const uint32_t max_slices = static_cast<uint32_t>(idx->num_sms);
  if ((rc = grow(idx, &idx->d_scnt, &idx->scnt_cap, static_cast<size_t>(nq) * max_slices, "batch counts")))
    return rc;
  if (!idx->d_overflow) BV_CUDA(idx, cudaMalloc(&idx->d_overflow, 8), "batch flag");

  bv::PrepParams pp;
  pp.queries = a->queries;
  pp.signs = idx->d_signs;
  pp.nq = nq;
  pp.dim = idx->dim;
  pp.P = idx->P;
  pp.KB = KB;
  pp.rounds = idx->rounds;
  pp.hamming = idx->scoring == BV_SCORE_HAMMING && idx->bits == 1 ? 1 : 0;
  pp.qtiles = idx->d_qtiles;
  pp.qfac = idx->d_qfac;
  pp.thr = idx->d_thr;
  pp.cnt = idx->d_bcnt;

  bv::GemmParams g;
  g.ctiles = compact ? idx->d_cctiles : idx->d_ctiles;
  g.qtiles = idx->d_qtiles;
  g.posfac = compact ? idx->d_cposfac : idx->d_posfac;
  g.posrow = compact ? idx->d_cposrow : idx->d_posrow;
  g.tmax = compact ? idx->d_ctmax : idx->d_tmax;
  g.mask = compact ? nullptr : a->mask;
  g.npos = npos;
  g.nq = nq;
  g.KB = KB;
  g.nqt = nqt;
  g.thr = idx->d_thr;
  g.qfac = idx->d_qfac;
  g.cand = idx->d_bcand;
  g.cap = cap;
  g.Fp = Fp;
  g.scnt = idx->d_scnt;
  g.max_slices = max_slices;
  g.overflow = idx->d_overflow;
  g.err = idx->d_err;

  bv::SelectParams sp;
  sp.cand = idx->d_bcand;
  sp.cap = cap;
  sp.F = F;
  sp.Fp = Fp;
  sp.nq = nq;
  sp.cnt = idx->d_bcnt;
  sp.thr = idx->d_thr;
  sp.scnt = idx->d_scnt;
  sp.max_slices = max_slices;

  // Two or more query tiles: the CTA-pair GEMM (cta_group::2, 256 queries x
  // 256 rows per pair), its operands read by TMA tensor copies.
  const bool pair = nqt >= 2 && idx->gemm_pair;
  alignas(64) unsigned char amap[128], bmap[128];
  if (pair) {
    cudaError_t e = bv::encode_tile_rows_map(amap, idx->d_qtiles, static_cast<uint64_t>(nqt_pad) * KB * bv::kBQTile,
                                             bv::kBQTile);
    if (e == cudaSuccess)
      e = bv::encode_tile_rows_map(bmap, g.ctiles, static_cast<uint64_t>(T) * KB * bv::kBRowTile, bv::kBRowTile / 2);
    if (e != cudaSuccess) return cuda_fail(idx, e, "batch tensor maps");
  }
  uint32_t launches = 0;
  // A GEMM launch appends densely behind the kept keys (one slice, a global
  // counter per query) when `dense`, else each CTA into its own slice of the
  // queries it serves: CTA c of grid G serves query tiles qt = c (mod g),
  // g = gcd(nqt, G), as slice c / g of G / g, its counters in shared memory.
  // The first launch of a batch (nothing kept yet) appends from slot 0.
  auto gemm = [&](uint32_t rt0, uint32_t rt1, bool dense, bool first_launch) -> int {
    g.rt0 = rt0;
    g.rt1 = rt1;
    const uint64_t tiles = static_cast<uint64_t>(rt1 - rt0) * nqt;
    const uint32_t grid = static_cast<uint32_t>(tiles < static_cast<uint64_t>(idx->num_sms) ? tiles : idx->num_sms);
    g.sbase = first_launch ? 0u : Fp;
    // the first round writes every position's key at its own slot (no
    // threshold yet, so no filter and no append counters)
    g.direct = first_launch && rt0 == 0 && g.mask == nullptr && !pair &&
                       static_cast<uint64_t>(rt1 - rt0) * bv::kBRowTile <= cap ? 1u : 0u;
    g.slice_g = 0;
    g.slice_cap = cap - g.sbase;
    g.cnt_words = 0;
    if (!dense && !pair) {
      const uint32_t gg = static_cast<uint32_t>(gcd_u64(nqt, grid));
      const uint32_t nslices = grid / gg, words = (nqt / gg) * (bv::kBQTile / 2u);
      const uint32_t scap = (cap - Fp) / nslices;
      if (scap >= 64u && bv::batch_gemm_smem(words) <= static_cast<uint32_t>(idx->max_smem)) {
        g.slice_g = gg;
        g.slice_cap = scap;
        g.cnt_words = words;
      }
    }
    sp.nslices = g.slice_g ? grid / g.slice_g : 1u;
    sp.slice_cap = g.slice_cap;
    sp.sbase = g.sbase;
    int r;
    if ((r = clk.begin(kPhGemm))) return r;
    cudaError_t e;
    if (pair) {
      const uint64_t tiles2 = static_cast<uint64_t>(rt1 - rt0) * ((nqt + 1u) / 2u);
      const uint32_t max_pairs = static_cast<uint32_t>(idx->num_sms) / 2u;
      e = bv::launch_gemm_pair(g, amap, bmap, static_cast<uint32_t>(tiles2 < max_pairs ? tiles2 : max_pairs), s);
    } else {
      e = bv::launch_gemm(g, grid, s);
    }
    if (e != cudaSuccess) return cuda_fail(idx, e, "batch gemm");
    if ((r = clk.end())) return r;
    ++launches;
    return BV_OK;
  };
  auto select = [&]() -> int {
    int r;
    if ((r = clk.begin(kPhSelect))) return r;
    const cudaError_t e = bv::launch_select(sp, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "batch select");
    if ((r = clk.end())) return r;
    ++launches;
    return BV_OK;
  };
  auto prep = [&]() -> int {
    int r;
    if ((r = clk.begin(kPhPrep))) return r;
    const cudaError_t e = bv::launch_prep(pp, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "batch prep");
    if ((r = clk.end())) return r;
    ++launches;
    return BV_OK;
  };
  // Round sizes in row tiles: the first takes cap rows (every row is a
  // candidate, appended densely from slot 0); later ones take four times the rows already
  // seen, or fewer when that would expect more than (cap - F) / 2 rows to
  // beat the threshold of the rows seen.  Growth capped at 4 took config 5
  // from 436k to 553k q/s and config 3 from 1.02M to 1.11M (uncapped, about
  // 50x), when every row that beat the threshold cost the epilogue a global
  // atomic; it also keeps a CTA's slice well below its capacity.
  constexpr double kMaxGrow = 4.0;
  const uint32_t first = cap / bv::kBRowTile;
  auto next_size = [&](uint32_t seen_tiles) -> uint32_t {
    double grow = static_cast<double>(cap - F) / (2.0 * F);
    if (grow > kMaxGrow) grow = kMaxGrow;
    double m = static_cast<double>(seen_tiles) * grow;
    return m < 1.0 ? 1u : (m > 4.0e9 ? 0xFFFFFFFFu : static_cast<uint32_t>(m));
  };

  const size_t scnt_bytes = static_cast<size_t>(nq) * max_slices * 4;
  BV_CUDA(idx, cudaMemsetAsync(idx->d_overflow, 0, 4, s), "batch flag");
  BV_CUDA(idx, cudaMemsetAsync(idx->d_scnt, 0, scnt_bytes, s), "batch counts");
  if ((rc = prep())) return rc;
  uint32_t nrounds = 0;
  for (uint32_t rt = 0; rt < T;) {
    const uint32_t m = rt == 0 ? first : next_size(rt);
    const uint32_t rt1 = T - rt < m ? T : rt + m;
    if ((rc = gemm(rt, rt1, rt == 0, rt == 0)) || (rc = select())) return rc;
    ++nrounds;
    rt = rt1;
  }
  uint32_t flag = 0;
  BV_CUDA(idx, cudaMemcpyAsync(&flag, idx->d_overflow, 4, cudaMemcpyDeviceToHost, s), "batch flag");
  BV_CUDA(idx, cudaStreamSynchronize(s), "batch search");
  if (flag) {
    // A buffer overflowed (rows that arrive in increasing score order, for
    // instance): redo the batch round by round, halving a round that
    // overflows; a round of one tile (256 rows) cannot overflow (cap >= F + 256).
    // (the fallback appends densely: one slice of cap - Fp slots per query)
    BV_CUDA(idx, cudaMemsetAsync(idx->d_scnt, 0, scnt_bytes, s), "batch counts");
    if ((rc = prep())) return rc;
    uint32_t m = first;
    for (uint32_t rt = 0; rt < T;) {
      const uint32_t rt1 = T - rt < m ? T : rt + m;
      BV_CUDA(idx, cudaMemsetAsync(idx->d_overflow, 0, 4, s), "batch flag");
      if ((rc = gemm(rt, rt1, true, rt == 0))) return rc;
      BV_CUDA(idx, cudaMemcpyAsync(&flag, idx->d_overflow, 4, cudaMemcpyDeviceToHost, s), "batch flag");
      BV_CUDA(idx, cudaStreamSynchronize(s), "batch search");
      if (flag) {
        // the round's appends are discarded (the kept keys and the thresholds
        // are untouched by the GEMM) and the round is repeated smaller
        if (rt1 - rt == 1) return fail(BV_ERR_CUDA, "batch candidate buffer overflow on a single tile");
        BV_CUDA(idx, cudaMemsetAsync(idx->d_scnt, 0, scnt_bytes, s), "batch counts");
        m = (rt1 - rt) / 2;
        continue;
      }
      if ((rc = select())) return rc;
      ++nrounds;
      rt = rt1;
      m = m < 0x7FFFFFFFu ? 2 * m : m;
    }
    BV_CUDA(idx, cudaStreamSynchronize(s), "batch search");
  }
  if ((rc = check_err_flag(idx))) return rc;
  bs->launches = launches;
  bs->rounds = nrounds;
  bs->prof.rounds = nrounds;
  bs->pending = true;
  return fold_phases(idx);
}

// The re-rank tail of a batched search (after batch_rounds): one CTA per
// query re-ranks its best F exactly and writes the outputs.
int batch_tail(bv_index* idx, const bv_search_args* a, cudaStream_t s) {
  bv_batch_state* bs = batch_state(idx);
  const uint32_t nq = a->nq, F = bs->F, Fp = bs->Fp;
  PhaseClock clk(idx, s);
  int rc;
  if (bs->empty) {
    BV_CUDA(idx, cudaMemsetAsync(a->out_counts, 0, nq * 4, s), "memset");
    if (a->cand_counts) BV_CUDA(idx, cudaMemsetAsync(a->cand_counts, 0, nq * 4, s), "memset");
    BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
    idx->last_launches = bs->launches;
    idx->last_rounds = 0;
    bs->pending = false;
    return BV_OK;
  }
  bv::TailParams t;
  memset(&t, 0, sizeof(t));
  t.partials = idx->d_bcand;
  t.partials_stride = bs->cap;
  t.G = 1;
  t.F = F;
  t.Fp = Fp;
  t.capc = Fp <= 256 ? (16 * Fp > 1024 ? 16 * Fp : 1024) : (2 * Fp > 1024 ? 2 * Fp : 1024);
  t.k = a->k;
  t.rerank = a->rerank ? 1 : 0;
  t.query = a->queries;
  t.originals = idx->d_orig;
  t.dim = idx->dim;
  t.row_base = idx->row_base;
  t.err = idx->d_err;
  t.out_rows = a->out_rows;
  t.out_scores = a->out_scores;
  t.out_count = a->out_counts;
  const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
  t.cand_rows = cand ? a->cand_rows : nullptr;
  t.cand_scores = cand ? a->cand_scores : nullptr;
  t.cand_count = cand ? a->cand_counts : nullptr;
  t.cand_exact = cand ? a->cand_exact : nullptr;
  const uint32_t row_bytes = (idx->dim + 4) * 4;
  const uint32_t fixed = bv::tail_smem_layout(idx->dim, t.capc, 0).total + 256;
  // the batch's tail CTAs run two per SM: each stages rows in at most half
  // of the SM's shared memory (more batches of rows), when one row fits
  const uint32_t half = static_cast<uint32_t>(idx->smem_per_sm) / 2u - 1024u;
  const uint32_t lim = half >= fixed + row_bytes ? half : static_cast<uint32_t>(idx->max_smem);
  uint32_t rows_bytes = lim > fixed ? lim - fixed : 0;
  if (rows_bytes > F * row_bytes) rows_bytes = F * row_bytes;
  rows_bytes = rows_bytes / row_bytes * row_bytes;
  if (rows_bytes < row_bytes) return fail(BV_ERR_UNSUPPORTED, "re-rank row does not fit in shared memory");
  t.rows_bytes = rows_bytes;
  if ((rc = clk.begin(kPhTail))) return rc;
  const cudaError_t e = bv::launch_tail_grid(t, nq, bv::tail_smem_layout(idx->dim, t.capc, rows_bytes).total, s);
  if (e != cudaSuccess) return cuda_fail(idx, e, "batch tail");
  if ((rc = clk.end())) return rc;
  BV_CUDA(idx, cudaStreamSynchronize(s), "batch search");
  idx->last_launches = bs->launches + 1;
  idx->last_rounds = bs->rounds;
  bs->pending = false;
  if ((rc = fold_phases(idx))) return rc;
  return check_err_flag(idx);
}

int batch_check(bv_index* idx, const bv_search_args* a, uint32_t* F) {
  int rc = check_args(idx, a, F);
  if (rc) return rc;
  if (idx->scoring == BV_SCORE_ASYM || idx->bits == 0)
    return fail(BV_ERR_UNSUPPORTED, "the batched search scores with the integer modes (int, hamming), "
                                    "not asym");
  if (idx->rows >= 0x7FFFFF00ull) return fail(BV_ERR_UNSUPPORTED, "batched search takes < 2^31 rows per index");
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  return BV_OK;
}

}  // namespace

int bv_search_batch(bv_index* idx, const bv_search_args* a, void* stream) {
  uint32_t F = 0;
  int rc = batch_check(idx, a, &F);
  if (rc) return rc;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : idx->stream;
  const uint32_t nq = a->nq;
  if (idx->rows == 0 || nq == 0) {
    if (nq) BV_CUDA(idx, cudaMemsetAsync(a->out_counts, 0, nq * 4, s), "memset");
    if (nq && a->cand_counts) BV_CUDA(idx, cudaMemsetAsync(a->cand_counts, 0, nq * 4, s), "memset");
    BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
    idx->last_launches = 0;
    return BV_OK;
  }
  if ((rc = batch_rounds(idx, a, F, s))) return rc;
  return batch_tail(idx, a, s);
}

int bv_batch_select(bv_index* idx, const bv_search_args* a, uint64_t* keys_out, void* stream) {
  uint32_t F = 0;
  int rc = batch_check(idx, a, &F);
  if (rc) return rc;
  if (!keys_out && a->nq) return fail(BV_ERR_INVALID, "keys_out is null");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : idx->stream;
  const uint32_t nq = a->nq;
  bv_batch_state* bs = batch_state(idx);
  if (idx->rows == 0 || nq == 0) {
    if (nq) BV_CUDA(idx, cudaMemsetAsync(keys_out, 0, static_cast<size_t>(nq) * F * 8, s), "memset");
    BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
    bs->pending = true;
    bs->empty = true;
    bs->nq = nq;
    bs->F = F;
    bs->launches = 0;
    return BV_OK;
  }
  if ((rc = batch_rounds(idx, a, F, s))) return rc;
  if (bs->empty) {
    BV_CUDA(idx, cudaMemsetAsync(keys_out, 0, static_cast<size_t>(nq) * F * 8, s), "memset");
  } else {
    const cudaError_t e =
        bv::launch_export_keys(idx->d_bcand, bs->cap, idx->d_bcnt, nq, F, idx->row_base, keys_out, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "export keys");
  }
  return BV_OK;  // the keys are written in stream order (the rounds themselves synchronised)
}

int bv_batch_finish(bv_index* idx, const bv_search_args* a, const uint64_t* min_keys, void* stream) {
  uint32_t F = 0;
  int rc = batch_check(idx, a, &F);
  if (rc) return rc;
  bv_batch_state* bs = batch_state(idx);
  if (!bs->pending || bs->nq != a->nq || bs->F != F)
    return fail(BV_ERR_INVALID, "bv_batch_finish needs the same request right after bv_batch_select");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : idx->stream;
  const uint32_t nq = a->nq;
  if (idx->rows == 0 || nq == 0) {
    if (nq) BV_CUDA(idx, cudaMemsetAsync(a->out_counts, 0, nq * 4, s), "memset");
    if (nq && a->cand_counts) BV_CUDA(idx, cudaMemsetAsync(a->cand_counts, 0, nq * 4, s), "memset");
    BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
    bs->pending = false;
    idx->last_launches = 0;
    return BV_OK;
  }
  if (min_keys && !bs->empty) {
    const cudaError_t e = bv::launch_trim_keys(idx->d_bcand, bs->cap, bs->Fp, nq, idx->row_base, min_keys, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "trim keys");
  }
  return batch_tail(idx, a, s);
}

int bv_keys_threshold(const uint64_t* gathered, uint32_t world, uint32_t nq, uint32_t fetch, uint64_t* thr_out,
                      void* stream) {
  if ((nq && (!gathered || !thr_out)) || world == 0 || fetch == 0) return fail(BV_ERR_INVALID, "bad argument");
  if (static_cast<uint64_t>(world) * fetch > bv::keys_threshold_max())
    return fail(BV_ERR_UNSUPPORTED, "%u shards x %u candidates exceed the threshold kernel's %u keys", world, fetch,
                bv::keys_threshold_max());
  if (nq == 0) return BV_OK;
  const cudaError_t e = bv::launch_keys_threshold(gathered, world, nq, fetch, thr_out,
                                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "threshold launch");
  return BV_OK;
}

int bv_set_batch_timing(bv_index* idx, int enable) {
  if (!idx) return fail(BV_ERR_INVALID, "null index");
  batch_state(idx)->timing = enable != 0;
  return BV_OK;
}

int bv_last_batch_profile(bv_index* idx, bv_batch_profile* out) {
  if (!idx || !out) return fail(BV_ERR_INVALID, "null argument");
  *out = batch_state(idx)->prof;
  return BV_OK;
}

int bv_search_rows(bv_index* idx, const bv_search_args* a, const uint32_t* offsets, const uint32_t* cand_rows,
                   void* stream) {
  uint32_t F = 0;
  int rc = check_args(idx, a, &F);
  if (rc) return rc;
  if (idx->bits == 0) return fail(BV_ERR_UNSUPPORTED, "the candidate-list search scans quantized codes (bits 1, 4, 8)");
  if (a->mask) return fail(BV_ERR_UNSUPPORTED, "the candidate-list search takes no score mask");
  const uint32_t nq = a->nq;
  if (nq && !offsets) return fail(BV_ERR_INVALID, "offsets is null");
  uint32_t max_n = 0;
  for (uint32_t q = 0; q < nq; ++q) {
    if (offsets[q + 1] < offsets[q]) return fail(BV_ERR_INVALID, "offsets decrease at query %u", q);
    max_n = std::max(max_n, offsets[q + 1] - offsets[q]);
  }
  const uint64_t total = nq ? static_cast<uint64_t>(offsets[nq]) - offsets[0] : 0;
  if (total && !cand_rows) return fail(BV_ERR_INVALID, "cand_rows is null");
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : idx->stream;
  // Per query a segment of whole scan tiles (the scan reads whole tiles and
  // ignores the rows past its count), starting on a tile boundary.
  Plan pl0;
  const uint64_t saved_rows = idx->rows;
  idx->rows = 1;
  rc = plan_scan(idx, F, &pl0, true, false);
  idx->rows = saved_rows;
  if (rc) return rc;
  const uint32_t tr = pl0.tile_rows;
  std::vector<uint32_t> host(2 * static_cast<size_t>(nq) + 1);
  uint64_t seg = 0;
  for (uint32_t q = 0; q < nq; ++q) {
    host[nq + 1 + q] = static_cast<uint32_t>(seg);
    seg += (static_cast<uint64_t>(offsets[q + 1] - offsets[q]) + tr - 1) / tr * tr;
  }
  if (seg >= 0xFFFFFFFFull) return fail(BV_ERR_UNSUPPORTED, "candidate lists too long for one call");
  for (uint32_t q = 0; q <= nq; ++q) host[q] = offsets[q];
  if ((rc = grow(idx, &idx->d_gcodes, &idx->gcodes_cap, (seg + tr) * idx->R, "candidate codes"))) return rc;
  if ((rc = grow(idx, &idx->d_gscales, &idx->gscales_cap, seg + tr, "candidate scales"))) return rc;
  if ((rc = grow(idx, &idx->d_growmap, &idx->growmap_cap, seg + tr, "candidate rows"))) return rc;
  if ((rc = grow(idx, &idx->d_goffs, &idx->goffs_cap, host.size() + 1, "candidate offsets"))) return rc;
  uint32_t* bad = idx->d_err + 1;  // the gather's out-of-range flag
  BV_CUDA(idx, cudaMemcpyAsync(idx->d_goffs, host.data(), host.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
  BV_CUDA(idx, cudaMemsetAsync(bad, 0, 4, s), "flag");
  cudaError_t e = bv::launch_gather_rows(idx->d_codes, idx->d_scales, idx->R, idx->rows, cand_rows, idx->d_goffs,
                                         idx->d_goffs + nq + 1, nq, max_n, idx->d_gcodes, idx->d_gscales,
                                         idx->d_growmap, bad, s);
  if (e != cudaSuccess) return cuda_fail(idx, e, "candidate gather");
  // each query scans its segment as if it were the whole index
  uint8_t* const codes0 = idx->d_codes;
  float* const scales0 = idx->d_scales;
  const uint64_t rows0 = idx->rows;
  const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
  uint32_t launches = 0;
  for (uint32_t q = 0; q < nq && rc == BV_OK; ++q) {
    const uint32_t n = offsets[q + 1] - offsets[q];
    if (n == 0) {
      BV_CUDA(idx, cudaMemsetAsync(a->out_counts + q, 0, 4, s), "memset");
      if (cand) BV_CUDA(idx, cudaMemsetAsync(a->cand_counts + q, 0, 4, s), "memset");
      continue;
    }
    const uint32_t s0 = host[nq + 1 + q];
    idx->d_codes = idx->d_gcodes + static_cast<size_t>(s0) * idx->R;
    idx->d_scales = idx->d_gscales + s0;
    idx->rows = n;
    idx->rowmap = idx->d_growmap + s0;
    bv_search_args sub = *a;
    sub.queries = a->queries + static_cast<size_t>(q) * idx->dim;
    sub.nq = 1;
    sub.out_rows = a->out_rows + static_cast<size_t>(q) * a->k;
    sub.out_scores = a->out_scores + static_cast<size_t>(q) * a->k;
    sub.out_counts = a->out_counts + q;
    sub.cand_rows = cand ? a->cand_rows + static_cast<size_t>(q) * F : nullptr;
    sub.cand_scores = cand ? a->cand_scores + static_cast<size_t>(q) * F : nullptr;
    sub.cand_counts = cand ? a->cand_counts + q : nullptr;
    sub.cand_exact = cand && a->cand_exact ? a->cand_exact + static_cast<size_t>(q) * F : nullptr;
    rc = enqueue_search(idx, &sub, F, s, false);
    launches += idx->last_launches;
  }
  idx->d_codes = codes0;
  idx->d_scales = scales0;
  idx->rows = rows0;
  idx->rowmap = nullptr;
  if (rc) return rc;
  idx->last_launches = launches + 1;
  uint32_t flags[2] = {0, 0};
  BV_CUDA(idx, cudaStreamSynchronize(s), "candidate search");
  BV_CUDA(idx, cudaMemcpy(flags, idx->d_err, 8, cudaMemcpyDeviceToHost), "error flag");
  if (flags[1]) {
    BV_CUDA(idx, cudaMemset(bad, 0, 4), "flag");
    return fail(BV_ERR_INVALID, "a candidate row is outside the index (%llu rows)",
                static_cast<unsigned long long>(idx->rows));
  }
  return report_err_flag(idx, flags[0]);
}

int bv_check_wait_timeout(bv_index* idx, uint32_t polls) {
  if (!idx) return fail(BV_ERR_INVALID, "null index");
  if (idx->lost) return fail(BV_ERR_DEVICE_LOST, "%s", kLostMsg);
  if (polls == 0 || polls > bv::kWaitBudget)
    return fail(BV_ERR_INVALID, "polls must be in [1, %u], got %u", bv::kWaitBudget, polls);
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  const cudaError_t e = bv::launch_wait_probe(idx->d_err, polls, idx->stream);
  if (e != cudaSuccess) return cuda_fail(idx, e, "wait probe");
  BV_CUDA(idx, cudaStreamSynchronize(idx->stream), "wait probe");
  return check_err_flag(idx);
}

int bv_set_scoring(bv_index* idx, uint32_t scoring) {
  if (!idx) return fail(BV_ERR_INVALID, "null index");
  if (scoring > BV_SCORE_HAMMING) return fail(BV_ERR_INVALID, "unknown scoring mode %u", scoring);
  if (idx->bits == 0 && scoring != BV_SCORE_ASYM)
    return fail(BV_ERR_INVALID, "the exact fp32 index (bits 0) has no quantized scoring");
  if (scoring == BV_SCORE_HAMMING && idx->bits != 1) return fail(BV_ERR_INVALID, "hamming scoring needs 1-bit codes");
  if (idx->stream) BV_CUDA(idx, cudaStreamSynchronize(idx->stream), "sync");
  idx->scoring = scoring;
  return BV_OK;
}

int bv_filter_mask(const bv_column* cols, uint32_t ncols, const bv_filter_term* terms, uint32_t nterms,
                   uint64_t rows, const uint32_t* live, uint32_t* mask_out, void* stream) {
  if ((ncols && !cols) || (nterms && !terms) || !mask_out) return fail(BV_ERR_INVALID, "null argument");
  if (ncols > BV_FILTER_MAX_TERMS || nterms > BV_FILTER_MAX_TERMS)
    return fail(BV_ERR_UNSUPPORTED, "a filter takes at most %d columns and %d terms", BV_FILTER_MAX_TERMS,
                BV_FILTER_MAX_TERMS);
  for (uint32_t i = 0; i < nterms; ++i) {
    const bv_filter_term& t = terms[i];
    if (t.column >= ncols) return fail(BV_ERR_INVALID, "filter term %u: column %u out of range", i, t.column);
    if (t.op > BV_OP_LTE) return fail(BV_ERR_INVALID, "filter term %u: unknown operator %u", i, t.op);
    const uint32_t nv = t.op == BV_OP_IN ? t.nvals : 1u;
    if (nv > BV_FILTER_MAX_IN || (t.op != BV_OP_IN && t.nvals != 1))
      return fail(BV_ERR_INVALID, "filter term %u: %u values", i, t.nvals);
    const bv_column& c = cols[t.column];
    if (!c.tag) return fail(BV_ERR_INVALID, "filter term %u: column without tags", i);
    for (uint32_t v = 0; v < nv; ++v) {
      const uint32_t tag = t.vals[v].tag;
      if (tag > BV_TAG_STRING) return fail(BV_ERR_INVALID, "filter term %u: bad value tag %u", i, tag);
      if (t.op >= BV_OP_GT && tag != BV_TAG_NUMBER)
        return fail(BV_ERR_INVALID, "filter term %u: range operator expects a number", i);
      if ((tag == BV_TAG_NUMBER || tag == BV_TAG_BOOL) && !c.num)
        return fail(BV_ERR_INVALID, "filter term %u: column has no numbers", i);
      if (tag == BV_TAG_STRING && !c.code) return fail(BV_ERR_INVALID, "filter term %u: column has no strings", i);
    }
  }
  const cudaError_t e =
      bv::launch_filter(cols, ncols, terms, nterms, rows, live, mask_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "filter");
  return BV_OK;
}

// ------------------------------------------------------- no-alloc search
// bv_search_noalloc: the same scan + tail launches as bv_search_async, but all
// of their scratch lives in one fixed device array of this file instead of
// buffers the index allocates on demand.  For hosts that must not allocate
// device memory after start-up.
namespace {

constexpr uint32_t kNoAllocMaxCtas = 160;  // scan grid bound (one CTA per SM, minus one)
constexpr uint32_t kNoAllocMaxFp = 256;    // candidate slots per CTA: fetch <= 256
constexpr size_t kNoAllocKeys = static_cast<size_t>(kNoAllocMaxCtas) * kNoAllocMaxFp;
constexpr uint32_t kNoAllocSlots = 64;            // rotating tile counters (one per query in flight)
constexpr size_t kNoAllocCtr = kNoAllocKeys;
constexpr size_t kNoAllocErr = kNoAllocKeys + kNoAllocSlots;  // kernel error word
constexpr size_t kNoAllocWords = kNoAllocErr + 1;

struct NoAllocDevice {
  bool ready = false;
  unsigned long long* base = nullptr;  // device address of the scratch array
  uint32_t epoch = 0;                  // tile-counter epochs used on this device
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

}  // namespace

// 320 KB per device, loaded with the library and held until the process exits.
static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocWords];

extern "C" int bv_search_noalloc(bv_index* idx, const bv_search_args* a, void* stream) {
  uint32_t F = 0;
  int rc = check_args(idx, a, &F);
  if (rc) return rc;
  // the exact fp32 index (bits 0) has no codes for the quantized scan
  if (idx->bits == 0)
    return fail(BV_ERR_UNSUPPORTED, "bv_search_noalloc: serves quantized indexes only (bits 1, 4, 8), not bits 0");
  uint32_t fp = 32;
  while (fp < F) fp <<= 1;
  if (fp > kNoAllocMaxFp)
    return fail(BV_ERR_INVALID,
                "bv_search_noalloc: fetch %u is above its fixed scratch limit of %u candidates per query",
                F, kNoAllocMaxFp);
  if (idx->device < 0 || idx->device >= kNoAllocMaxDevices)
    return fail(BV_ERR_INVALID, "bv_search_noalloc: device ordinal %d out of range", idx->device);
  BV_CUDA(idx, cudaSetDevice(idx->device), "cudaSetDevice");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : idx->stream;

  // First call on a device: resolve the array's device address (host code only
  // sees a stand-in symbol).  Later calls reuse it.
  unsigned long long* base = nullptr;
  uint32_t epoch0 = 0;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocDevice& d = g_noalloc_dev[idx->device];
    if (!d.ready) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(idx, e, "bv_search_noalloc: scratch address");
      d.base = static_cast<unsigned long long*>(ptr);
      d.ready = true;
    }
    base = d.base;
    epoch0 = d.epoch;
    d.epoch += a->nq;
  }
  if (idx->rows == 0 || a->nq == 0) {
    if (a->nq) BV_CUDA(idx, cudaMemsetAsync(a->out_counts, 0, a->nq * 4, s), "memset");
    if (a->nq && a->cand_counts) BV_CUDA(idx, cudaMemsetAsync(a->cand_counts, 0, a->nq * 4, s), "memset");
    BV_CUDA(idx, cudaStreamSynchronize(s), "sync");
    idx->last_launches = 0;
    return BV_OK;
  }
  Plan pl;
  if ((rc = plan_scan(idx, F, &pl, false))) return rc;
  if (pl.grid > kNoAllocMaxCtas)
    return fail(BV_ERR_UNSUPPORTED, "bv_search_noalloc: scan grid %u above its scratch bound %u", pl.grid,
                kNoAllocMaxCtas);
  uint32_t* err = reinterpret_cast<uint32_t*>(base + kNoAllocErr);
  BV_CUDA(idx, cudaMemsetAsync(err, 0, sizeof(unsigned long long), s), "clear error word");

  bv::ScanParams p;
  memset(&p, 0, sizeof(p));
  p.codes = idx->d_codes;
  p.scales = idx->d_scales;
  p.signs = idx->d_signs;
  p.seed = idx->seed;
  p.sign_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(idx->P)));
  p.mask = a->mask;
  p.nrows = idx->rows;
  p.dim = idx->dim;
  p.P = idx->P;
  p.rounds = idx->rounds;
  p.R = pl.sh.R;
  p.tile_rows = pl.tile_rows;
  p.tile_bytes = pl.tile_bytes;
  p.ntiles = pl.ntiles;
  p.stages = pl.stages;
  p.F = pl.F;
  p.Fp = pl.Fp;
  p.capc = pl.capc;
  p.check_tiles = pl.check_tiles;
  p.partials = reinterpret_cast<uint64_t*>(base);
  p.err = err;
  p.serial = 1;  // one partials area for every query: each scan waits for the previous tail

  bv::TailParams t;
  memset(&t, 0, sizeof(t));
  t.partials = reinterpret_cast<const uint64_t*>(base);
  t.G = pl.grid;
  t.F = pl.F;
  t.Fp = pl.Fp;
  t.capc = pl.capc;
  t.k = a->k;
  t.rerank = a->rerank ? 1 : 0;
  t.originals = idx->d_orig;
  t.dim = idx->dim;
  t.row_base = idx->row_base;
  t.err = err;
  const uint32_t row_bytes = (idx->dim + 4) * 4;
  const uint32_t fixed = bv::tail_smem_layout(idx->dim, pl.capc, 0).total + 256;
  uint32_t rows_bytes =
      static_cast<uint32_t>(idx->max_smem) > fixed ? static_cast<uint32_t>(idx->max_smem) - fixed : 0;
  if (rows_bytes > pl.F * row_bytes) rows_bytes = pl.F * row_bytes;
  rows_bytes = rows_bytes / row_bytes * row_bytes;
  if (rows_bytes < row_bytes) return fail(BV_ERR_UNSUPPORTED, "re-rank row does not fit in shared memory");
  t.rows_bytes = rows_bytes;
  const size_t tail_smem = bv::tail_smem_layout(idx->dim, pl.capc, rows_bytes).total;

  for (uint32_t q = 0; q < a->nq; ++q) {
    // Each scan lets the next kernels launch at its start (programmatic
    // dependent launch), so on a small grid later queries' scans can run while
    // this one still takes tiles.  Queries q and q + kNoAllocSlots share a
    // counter: before reusing the slots, the stream waits for all earlier work.
    if (q && q % kNoAllocSlots == 0) {
      BV_CUDA(idx, cudaEventRecord(idx->ev_ring, s), "slot event");
      BV_CUDA(idx, cudaStreamWaitEvent(s, idx->ev_ring, 0), "slot wait");
    }
    p.query = a->queries + static_cast<size_t>(q) * idx->dim;
    p.epoch = epoch0 + q + 1;  // unique per device; the array starts zeroed (epoch 0)
    p.tile_ctr = base + kNoAllocCtr + (epoch0 + q) % kNoAllocSlots;
    cudaError_t e = launch_scan(static_cast<int>(idx->bits), static_cast<int>(idx->scoring), pl.sh, p,
                                pl.grid, pl.smem, s);
    if (e == cudaErrorNotSupported)
      return fail(BV_ERR_UNSUPPORTED, "no scan kernel for bits=%u scoring=%u P=%u", idx->bits, idx->scoring,
                  idx->P);
    if (e != cudaSuccess) return cuda_fail(idx, e, "scan launch");
    t.query = p.query;
    t.out_rows = a->out_rows + static_cast<size_t>(q) * a->k;
    t.out_scores = a->out_scores + static_cast<size_t>(q) * a->k;
    t.out_count = a->out_counts + q;
    const bool cand = a->cand_rows && a->cand_scores && a->cand_counts;
    t.cand_rows = cand ? a->cand_rows + static_cast<size_t>(q) * F : nullptr;
    t.cand_scores = cand ? a->cand_scores + static_cast<size_t>(q) * F : nullptr;
    t.cand_count = cand ? a->cand_counts + q : nullptr;
    t.cand_exact = cand && a->cand_exact ? a->cand_exact + static_cast<size_t>(q) * F : nullptr;
    e = bv::launch_tail(t, tail_smem, s);
    if (e != cudaSuccess) return cuda_fail(idx, e, "tail launch");
  }
  idx->last_launches = 2 * a->nq;
  BV_CUDA(idx, cudaStreamSynchronize(s), "bv_search_noalloc");
  uint32_t flag = 0;
  BV_CUDA(idx, cudaMemcpy(&flag, err, sizeof(flag), cudaMemcpyDeviceToHost), "error word");
  if (flag) return fail(BV_ERR_TIMEOUT, "scan kernel wait ran out of budget (flag 0x%x)", flag);
  return BV_OK;
}
