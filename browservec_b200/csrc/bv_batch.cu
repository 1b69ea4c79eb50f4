// bv_batch.cu -- kernels of the batched tensor-core search (see bv_batch.cuh).
//
//   expand_kernel  codes -> swizzled int8 row tiles + per-row score factor
//                  (the layout the MMA reads; built once per appended row)
//   prep_kernel    per query: rotation (rotator.ts:60-70), int8 codec
//                  (codec.ts:32-54) or signs, swizzled query tiles
//   gemm_kernel    persistent; warp-specialised: one producer warp (bulk
//                  copies), one MMA warp (tcgen05.mma kind::i8, accumulators
//                  double-buffered in TMEM), four epilogue warps (tcgen05.ld,
//                  threshold filter, candidate append)
//   select_kernel  per query: keep the best F candidates, sorted, and set the
//                  threshold for the next round
#include <cuda.h>

#include <climits>
#include <cstdint>

#include <cub/device/device_radix_sort.cuh>

#include "bv_batch.cuh"
#include "bv_device.cuh"
#include "bv_internal.h"
#include "bv_scan.cuh"

namespace bv {

namespace {

// ------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] x B[smem desc]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma this thread issued so far completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
// 128 consecutive 32-bit TMEM columns of this thread's lane (one load, so a
// tile's 256 columns take two loads and two waits).
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&v)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,"
      "%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,"
      "%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,"
      "%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,"
      "%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127"
      "}, [%128];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]),
        "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]),
        "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]),
        "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]),
        "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63]),
        "=r"(v[64]), "=r"(v[65]), "=r"(v[66]), "=r"(v[67]), "=r"(v[68]), "=r"(v[69]), "=r"(v[70]), "=r"(v[71]),
        "=r"(v[72]), "=r"(v[73]), "=r"(v[74]), "=r"(v[75]), "=r"(v[76]), "=r"(v[77]), "=r"(v[78]), "=r"(v[79]),
        "=r"(v[80]), "=r"(v[81]), "=r"(v[82]), "=r"(v[83]), "=r"(v[84]), "=r"(v[85]), "=r"(v[86]), "=r"(v[87]),
        "=r"(v[88]), "=r"(v[89]), "=r"(v[90]), "=r"(v[91]), "=r"(v[92]), "=r"(v[93]), "=r"(v[94]), "=r"(v[95]),
        "=r"(v[96]), "=r"(v[97]), "=r"(v[98]), "=r"(v[99]), "=r"(v[100]), "=r"(v[101]), "=r"(v[102]), "=r"(v[103]),
        "=r"(v[104]), "=r"(v[105]), "=r"(v[106]), "=r"(v[107]), "=r"(v[108]), "=r"(v[109]), "=r"(v[110]), "=r"(v[111]),
        "=r"(v[112]), "=r"(v[113]), "=r"(v[114]), "=r"(v[115]), "=r"(v[116]), "=r"(v[117]), "=r"(v[118]), "=r"(v[119]),
        "=r"(v[120]), "=r"(v[121]), "=r"(v[122]), "=r"(v[123]), "=r"(v[124]), "=r"(v[125]), "=r"(v[126]), "=r"(v[127])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait_regs128(uint32_t (&v)[128]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                 "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
                 "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31]),
                 "+r"(v[32]), "+r"(v[33]), "+r"(v[34]), "+r"(v[35]), "+r"(v[36]), "+r"(v[37]), "+r"(v[38]), "+r"(v[39]),
                 "+r"(v[40]), "+r"(v[41]), "+r"(v[42]), "+r"(v[43]), "+r"(v[44]), "+r"(v[45]), "+r"(v[46]), "+r"(v[47]),
                 "+r"(v[48]), "+r"(v[49]), "+r"(v[50]), "+r"(v[51]), "+r"(v[52]), "+r"(v[53]), "+r"(v[54]), "+r"(v[55]),
                 "+r"(v[56]), "+r"(v[57]), "+r"(v[58]), "+r"(v[59]), "+r"(v[60]), "+r"(v[61]), "+r"(v[62]), "+r"(v[63]),
                 "+r"(v[64]), "+r"(v[65]), "+r"(v[66]), "+r"(v[67]), "+r"(v[68]), "+r"(v[69]), "+r"(v[70]), "+r"(v[71]),
                 "+r"(v[72]), "+r"(v[73]), "+r"(v[74]), "+r"(v[75]), "+r"(v[76]), "+r"(v[77]), "+r"(v[78]), "+r"(v[79]),
                 "+r"(v[80]), "+r"(v[81]), "+r"(v[82]), "+r"(v[83]), "+r"(v[84]), "+r"(v[85]), "+r"(v[86]), "+r"(v[87]),
                 "+r"(v[88]), "+r"(v[89]), "+r"(v[90]), "+r"(v[91]), "+r"(v[92]), "+r"(v[93]), "+r"(v[94]), "+r"(v[95]),
                 "+r"(v[96]), "+r"(v[97]), "+r"(v[98]), "+r"(v[99]), "+r"(v[100]), "+r"(v[101]), "+r"(v[102]), "+r"(v[103]),
                 "+r"(v[104]), "+r"(v[105]), "+r"(v[106]), "+r"(v[107]), "+r"(v[108]), "+r"(v[109]), "+r"(v[110]), "+r"(v[111]),
                 "+r"(v[112]), "+r"(v[113]), "+r"(v[114]), "+r"(v[115]), "+r"(v[116]), "+r"(v[117]), "+r"(v[118]), "+r"(v[119]),
                 "+r"(v[120]), "+r"(v[121]), "+r"(v[122]), "+r"(v[123]), "+r"(v[124]), "+r"(v[125]), "+r"(v[126]), "+r"(v[127])
               :
               : "memory");
}

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), Blackwell descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
// Instruction descriptor: s32 accumulator, s8 x s8, both K-major, M=128, N=256.
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((kBRowTile >> 3) << 17) |
                              ((kBQTile >> 4) << 24);

// Epilogue: groups of four warps (one per TMEM lane quarter); group g drains
// the accumulator buffer g, so with two groups two tiles drain at once and
// each warp has two tiles' time to hide its latencies.
#ifndef BV_EPI_GROUPS
#define BV_EPI_GROUPS 2
#endif
#ifndef BV_GEMM_STAGES
#define BV_GEMM_STAGES 3
#endif
constexpr int kEpiGroups = BV_EPI_GROUPS;
constexpr int kEpiWarps = 4 * kEpiGroups;
constexpr int kProdWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1;
constexpr int kGemmThreads = (kEpiWarps + 2) * 32;
constexpr int kGemmStages = BV_GEMM_STAGES;
static_assert(kEpiGroups == 1 || kEpiGroups == 2, "one group per accumulator buffer at most");
constexpr uint32_t kStageBytes = kBQTileBytes + kBRowTileBytes;
constexpr uint32_t kTmemCols = 2 * kBRowTile;  // two accumulator buffers

constexpr uint32_t kSlotWords = 36;  // per epilogue thread: 32 accumulators, padded for STS.128

// The CTA-pair GEMM (cta_group::2): each CTA of a cluster of two holds 128
// queries (A) and half of a row tile (B, 128 rows) per stage, and the pair's
// MMA computes 256 queries x 256 rows; per CTA a stage is then 32 KB for the
// same MMA time as the single CTA's 48 KB, so the operands need two thirds of
// the shared-memory fill bandwidth.
#ifndef BV_PAIR_STAGES
#define BV_PAIR_STAGES 4
#endif
constexpr int kPairStages = BV_PAIR_STAGES;
constexpr uint32_t kBHalfBytes = kBRowTileBytes / 2;
constexpr uint32_t kPairStageBytes = kBQTileBytes + kBHalfBytes;
// Instruction descriptor of the pair: M = 256 (both CTAs' queries), N = 256.
constexpr uint32_t kIdescI8Pair = (2u << 4) | (1u << 7) | (1u << 10) | ((kBRowTile >> 3) << 17) |
                                  ((2u * kBQTile >> 4) << 24);

struct GemmSmem {
  uint32_t slots_off, rowfac_off, rowid_off, bars_off, cnt_off, total;
};
__host__ __device__ inline GemmSmem gemm_smem_layout(bool pair = false, uint32_t cnt_words = 0) {
  GemmSmem s;
  const int stages = pair ? kPairStages : kGemmStages;
  s.slots_off = stages * (pair ? kPairStageBytes : kStageBytes);
  s.rowfac_off = s.slots_off + kEpiWarps * 32 * kSlotWords * 4;  // per epilogue warp: the tile's factors
  s.rowid_off = s.rowfac_off + kEpiWarps * kBRowTile * 4;        // ... and the tile's rows
  s.bars_off = s.rowid_off + kEpiWarps * kBRowTile * 4;
  // full[S], empty[S], tfull[2], tempty[2], done, then the TMEM address word
  s.cnt_off = s.bars_off + (2 * stages + 5) * 8 + 16;
  // the slice counters (two 16-bit counters a word)
  s.total = s.cnt_off + cnt_words * 4;
  return s;
}

// ------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// The shared::cluster address of this CTA's `p` in the cluster's CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// 2-D tiled tensor load for a CTA pair: the box lands in this CTA's shared
// memory and its bytes complete on `cluster_bar` (the pair leader's barrier).
// No multicast: every CTA loads only its own operand halves.
__device__ __forceinline__ void tma_load_pair(void* dst, const CUtensorMap* map, uint32_t x, uint32_t y,
                                              uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[both CTAs' smem] x B[both CTAs' smem]^T.
__device__ __forceinline__ void mma_i8_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` in every CTA of `mask` once the pair's MMAs issued so far complete.
__device__ __forceinline__ void mma_commit_pair_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_addr(bar)),
      "h"(mask)
      : "memory");
}

}  // namespace

// ------------------------------------------------------------- expand
// Score factor of a row (the row half of the integer-mode score).
template <int BITS>
__device__ __forceinline__ float row_factor(float scale) {
  return BITS == 8 ? __fmul_rn(scale, kInv127) : (BITS == 4 ? __fmul_rn(scale, kInv7) : scale);
}

// Sort input for a block of rows: factor keys and row ids (rows[i] if given,
// else row0 + i).
template <int BITS>
__global__ void __launch_bounds__(256) factor_kernel(const float* scales, const uint32_t* rows, uint32_t row0,
                                                     uint32_t n, float* fac, uint32_t* ids) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t r = rows ? rows[i] : row0 + i;
  fac[i] = row_factor<BITS>(scales[r]);
  ids[i] = r;
}

// Tiles of one sorted block in a scattered order: after the `head` positions
// that complete an earlier block's last tile, the K full tiles of sorted rows
// are placed with tile t holding sorted chunk (t * ginv) mod K (a
// multiplicative permutation); a trailing partial tile stays last.  Every tile
// keeps rows of nearly equal factor, and any range of tiles -- one round of a
// batched search -- samples the whole range of factors.
__global__ void __launch_bounds__(256) scatter_tiles_kernel(const uint32_t* in, uint32_t* out, uint32_t count,
                                                            uint32_t head, uint32_t K, uint32_t ginv) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= count) return;
  uint32_t src = j;
  if (j >= head) {
    const uint32_t q = j - head, t = q / kBRowTile, off = q % kBRowTile;
    if (t < K) src = head + static_cast<uint32_t>(static_cast<uint64_t>(t) * ginv % K) * kBRowTile + off;
  }
  out[j] = in[src];
}

// One CTA per tile; eight threads per position, each writing one 16-byte
// chunk (16 int8 elements) of the position's row into the tile's K blocks:
// int8 codes copied 16 bytes at a time, int4 sign-extended, 1-bit as +-1,
// zero beyond P.  A warp covers four positions, so its loads read whole
// 128-byte rows and its stores write whole 128-byte tile rows.  Then the tile
// maximum of the factors of the positions in use.
template <int BITS>
__device__ __forceinline__ uint4 expand_chunk(const uint8_t* src, uint32_t e0, uint32_t P, uint32_t R) {
  // elements e0 .. e0+15 of the row at src (R bytes)
  if constexpr (BITS == 8) {
    if (e0 + 16u <= P && (R & 15u) == 0u) return *reinterpret_cast<const uint4*>(src + e0);
  }
  alignas(16) int8_t b[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t e = e0 + static_cast<uint32_t>(j);
    int v = 0;
    if (e < P) {
      if constexpr (BITS == 8) {
        v = static_cast<int8_t>(src[e]);
      } else if constexpr (BITS == 4) {
        const int n = (src[e >> 1] >> ((e & 1u) * 4u)) & 0xF;
        v = n > 7 ? n - 16 : n;
      } else {
        v = ((src[e >> 3] >> (e & 7u)) & 1u) ? 1 : -1;
      }
    }
    b[j] = static_cast<int8_t>(v);
  }
  return *reinterpret_cast<const uint4*>(b);
}

template <int BITS>
__global__ void __launch_bounds__(kBRowTile) expand_kernel(const ExpandParams p) {
  const uint32_t tile = p.pos0 / kBRowTile + blockIdx.x;
  const uint32_t c = threadIdx.x & 7u;  // 16-byte chunk of a 128-byte K block
  __shared__ float red[kBRowTile / 32];
  for (uint32_t tp = threadIdx.x >> 3; tp < kBRowTile; tp += kBRowTile / 8) {
    const uint32_t pos = tile * kBRowTile + tp;
    if (pos >= p.pos0 && pos < p.pos0 + p.count) {
      const uint32_t row = p.rows[pos - p.pos0];
      const uint8_t* src = p.codes + static_cast<size_t>(row) * p.R;
      if (c == 0) {
        p.posfac[pos] = row_factor<BITS>(p.scales[row]);
        p.posrow[pos] = row;
      }
      for (uint32_t kb = 0; kb < p.KB; ++kb) {
        int8_t* dst = p.tiles + (static_cast<size_t>(tile) * p.KB + kb) * kBRowTileBytes;
        *reinterpret_cast<uint4*>(dst + sw128_offset(tp, c * 16)) =
            expand_chunk<BITS>(src, kb * kKBlock + c * 16, p.P, p.R);
      }
    } else if (pos >= p.total) {
      // positions past the end are zeroed so the MMA reads defined values;
      // positions before pos0 were written by an earlier expansion
      if (c == 0) p.posfac[pos] = 0.0f;
      for (uint32_t kb = 0; kb < p.KB; ++kb) {
        int8_t* dst = p.tiles + (static_cast<size_t>(tile) * p.KB + kb) * kBRowTileBytes;
        *reinterpret_cast<uint4*>(dst + sw128_offset(tp, c * 16)) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  __syncthreads();
  const uint32_t pos = tile * kBRowTile + threadIdx.x;
  float m = pos < p.total ? p.posfac[pos] : 0.0f;
#pragma unroll
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < static_cast<int>(kBRowTile / 32); ++w) t = fmaxf(t, red[w]);
    p.tmax[tile] = t;
  }
}

// ------------------------------------------------------------- prep
// One CTA (kConsumerThreads) per query.
__global__ void __launch_bounds__(kConsumerThreads, 1) prep_kernel(const PrepParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* q = reinterpret_cast<float*>(smem);                  // P
  int8_t* qb = reinterpret_cast<int8_t*>(q + p.P);            // KB*128
  float* red = reinterpret_cast<float*>(qb + p.KB * kKBlock);  // 16
  const int ctid = threadIdx.x;
  const uint32_t qi = blockIdx.x;
  const float* src = p.queries + static_cast<size_t>(qi) * p.dim;
  for (uint32_t i = ctid; i < p.P; i += kConsumerThreads) q[i] = i < p.dim ? src[i] : 0.0f;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  rotate_query(q, p.signs, p.P, p.rounds, ctid);
  float qfac = 1.0f;
  if (p.hamming) {
    for (uint32_t i = ctid; i < p.KB * kKBlock; i += kConsumerThreads)
      qb[i] = i < p.P ? (q[i] >= 0.0f ? 1 : -1) : 0;
  } else {
    const float qscale = quantize_query8(q, qb, p.P, ctid, red);
    for (uint32_t i = p.P + ctid; i < p.KB * kKBlock; i += kConsumerThreads) qb[i] = 0;
    qfac = __fmul_rn(qscale, kInv127);
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t qt = qi / kBQTile, qr = qi % kBQTile;
  for (uint32_t c = ctid; c < p.KB * 8; c += kConsumerThreads) {
    const uint32_t kb = c / 8, cc = c % 8;
    int8_t* dst = p.qtiles + (static_cast<size_t>(qt) * p.KB + kb) * kBQTileBytes;
    *reinterpret_cast<uint4*>(dst + sw128_offset(qr, cc * 16)) =
        *reinterpret_cast<const uint4*>(qb + kb * kKBlock + cc * 16);
  }
  if (ctid == 0) {
    p.qfac[qi] = qfac;
    p.thr[qi] = 0ull;
    p.cnt[qi] = 0u;
  }
}

// ------------------------------------------------------------- gemm
// Epilogue warps of one CTA.  Group g drains accumulator buffer g for this
// CTA's tiles tc = g, g + 2, ... of the tile sequence t = first, first +
// stride, ...; tile t covers row tile rt0 + t / nqt and query tile t % nqt
// (kPair: query tile 2 * (t % nqt) + rank, this CTA's half of the pair's 256
// queries, and the buffer is released on the pair leader's barrier).
template <bool kPair, bool kDirect = false>
__device__ __forceinline__ void gemm_epilogue(const GemmParams& p, uint8_t* smem, const GemmSmem& lay,
                                              uint64_t* tfull, uint64_t* tempty, uint32_t tmem, uint32_t first,
                                              uint32_t stride, uint32_t ntiles, uint32_t nqt, uint32_t rank,
                                              uint32_t* cnt_s, int warp, int lane) {
  // ------------------------------------------------------ epilogue
  const uint32_t grp = static_cast<uint32_t>(warp) / 4u;
  const uint32_t lane_base = static_cast<uint32_t>(warp % 4) * 32u;
  float* rf_s = reinterpret_cast<float*>(smem + lay.rowfac_off) + warp * kBRowTile;
  uint32_t* rid_s = reinterpret_cast<uint32_t*>(smem + lay.rowid_off) + warp * kBRowTile;
  // this CTA's tiles in order are tc = 0, 1, 2, ...; group g takes tc = g mod groups
  uint32_t tc = grp;
  for (uint32_t t = first + grp * stride; t < ntiles; t += kEpiGroups * stride, tc += kEpiGroups) {
    const uint32_t rt = p.rt0 + t / nqt, qt = kPair ? 2u * (t % nqt) + rank : t % nqt;
    const uint32_t buf = tc & 1u, use = tc >> 1;
    const uint32_t qi = qt * kBQTile + lane_base + static_cast<uint32_t>(lane);
    const bool qvalid = qi < p.nq;
    // the tile's inputs are loaded before the accumulator wait, so their
    // latency hides behind the MMA
    const uint64_t thr = qvalid ? p.thr[qi] : 0ull;
    const float qf = qvalid ? p.qfac[qi] : 0.0f;
    const float tm = p.tmax[rt];
    float rf[kBRowTile / 32];
    uint32_t rid[kBRowTile / 32];
#pragma unroll
    for (int i = 0; i < static_cast<int>(kBRowTile / 32); ++i) {
      const uint32_t pos = rt * kBRowTile + static_cast<uint32_t>(lane + 32 * i);
      rf[i] = pos < p.npos ? p.posfac[pos] : 0.0f;
      rid[i] = pos < p.npos ? p.posrow[pos] : 0u;
    }
    const bool ready = mbar_wait_bounded(&tfull[buf], use & 1u, p.err);
    if (!__all_sync(0xffffffffu, ready)) break;  // tcgen05.ld below is warp-collective
    tc_fence_after();
#pragma unroll
    for (int i = 0; i < static_cast<int>(kBRowTile / 32); ++i) {
      rf_s[lane + 32 * i] = rf[i];
      rid_s[lane + 32 * i] = rid[i];
    }
    __syncwarp();
    int bound = INT_MIN;
    if (qvalid && thr != 0ull) {
      const float ts = key_score(thr);
      const float den = __fmul_rn(tm, qf);
      if (ts > 0.0f && den > 0.0f) {
        // score = ((f32(idot) * rowfac) * qfac) >= ts needs idot >= ts / (tmax * qfac)
        // up to five f32 roundings (three in the score, two here): a 2^-16
        // margin keeps the bound below every idot that can pass
        const float b = floorf(__fmul_rn(__fdiv_rn(ts, den), 1.0f - 0x1p-16f));
        bound = b >= 2147483520.0f ? INT_MAX : static_cast<int>(b);
      }
    }
    uint64_t* cq = p.cand + static_cast<size_t>(qvalid ? qi : 0) * p.cap;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + lay.slots_off) + threadIdx.x * kSlotWords;
    // Columns [c0, c0 + 32) of this lane's accumulator row, in registers:
    // prefilter, then exact scores of the hits only.
    auto chunk = [&](const uint32_t (&v)[32], uint32_t c0) {
      if constexpr (kDirect) {
        // first round: every position is a candidate, its key at its own slot
        if (!qvalid) return;
        const uint32_t pbase = rt * kBRowTile + c0;
        uint64_t* dst = cq + (pbase - p.rt0 * kBRowTile);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const uint64_t k0 = make_key(
              __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(v[j])), rf_s[c0 + j]), qf), rid_s[c0 + j]);
          const uint64_t k1 = make_key(
              __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(v[j + 1])), rf_s[c0 + j + 1]), qf),
              rid_s[c0 + j + 1]);
          if (pbase + j + 1 < p.npos) {
            *reinterpret_cast<ulonglong2*>(dst + j) = make_ulonglong2(k0, k1);
          } else if (pbase + j < p.npos) {
            dst[j] = k0;
          }
        }
        return;
      }
      // the common case is a chunk with no hit: one 3-input max tree decides it
      int mx[11];
#pragma unroll
      for (int i = 0; i < 10; ++i)
        mx[i] = __vimax3_s32(static_cast<int>(v[3 * i]), static_cast<int>(v[3 * i + 1]), static_cast<int>(v[3 * i + 2]));
      mx[10] = max(static_cast<int>(v[30]), static_cast<int>(v[31]));
      const int top = __vimax3_s32(__vimax3_s32(mx[0], mx[1], mx[2]), __vimax3_s32(mx[3], mx[4], mx[5]),
                                   __vimax3_s32(__vimax3_s32(mx[6], mx[7], mx[8]), mx[9], mx[10]));
      if (!qvalid || top < bound) return;
      const uint32_t pbase = rt * kBRowTile + c0;
      const uint32_t valid =
          pbase >= p.npos ? 0u : (p.npos - pbase >= 32u ? 0xFFFFFFFFu : ((1u << (p.npos - pbase)) - 1u));
      uint32_t m = 0;
#pragma unroll
      for (int j = 0; j < 32; ++j) m |= (static_cast<int>(v[j]) >= bound ? 1u : 0u) << j;
      m &= valid;
      if (m) {
        // this lane's 32 accumulators go to its own shared-memory slot, and
        // only the columns that passed the prefilter are scored exactly
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<uint4*>(slot)[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        uint32_t pass = 0;
        for (uint32_t mm = m; mm; mm &= mm - 1u) {
          const uint32_t j = __ffs(mm) - 1u;
          const uint32_t row = rid_s[c0 + j];
          if (p.mask && !((p.mask[row >> 5] >> (row & 31u)) & 1u)) continue;
          const float sc = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(slot[j])), rf_s[c0 + j]), qf);
          if (make_key(sc, row) > thr) pass |= 1u << j;
        }
        if (pass) {
          const uint32_t n = __popc(pass);
          uint32_t base, off;
          if (p.slice_g) {
            // this CTA's slice of the query: a 16-bit counter in shared memory
            const uint32_t jc = (qt / p.slice_g) * kBQTile + (qi % kBQTile), sh = (jc & 1u) * 16u;
            base = (atomicAdd(cnt_s + (jc >> 1), n << sh) >> sh) & 0xFFFFu;
            off = p.sbase + (blockIdx.x / p.slice_g) * p.slice_cap;
          } else {
            base = atomicAdd(p.scnt + qi, n);  // slice 0: the queries' counters are contiguous
            off = p.sbase;
          }
          if (base + n > p.slice_cap) atomicOr(p.overflow, 1u);
          uint32_t w = base;
          for (uint32_t mm = pass; mm; mm &= mm - 1u, ++w) {
            const uint32_t j = __ffs(mm) - 1u;
            const uint32_t row = rid_s[c0 + j];
            const float sc = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(slot[j])), rf_s[c0 + j]), qf);
            if (w < p.slice_cap) cq[off + w] = make_key(sc, row);
          }
        }
      }
    };
    // 128 columns per TMEM load: tcgen05.wait::ld waits for every load in
    // flight, so a few wide loads expose its latency fewer times than many
    // narrow ones
    const uint32_t taddr = tmem + (lane_base << 16) + buf * kBRowTile;
#pragma unroll 1
    for (uint32_t h = 0; h < kBRowTile; h += 128) {
      uint32_t v[128];
      tmem_ld128(taddr + h, v);
      tmem_ld_wait_regs128(v);
#pragma unroll
      for (uint32_t i = 0; i < 4; ++i) {
        chunk(*reinterpret_cast<const uint32_t(*)[32]>(&v[32 * i]), h + 32 * i);
        __syncwarp();
      }
    }
    if (kDirect && qvalid) {  // the tile's positions in use, counted for the select
      const uint32_t p0 = rt * kBRowTile;
      const uint32_t nv = p.npos <= p0 ? 0u : (p.npos - p0 < kBRowTile ? p.npos - p0 : kBRowTile);
      if (nv) atomicAdd(p.scnt + qi, nv);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if constexpr (kPair) mbar_arrive_remote(cluster_addr(&tempty[buf], 0));  // the pair leader's barrier
      else mbar_arrive(&tempty[buf]);
    }
  }
}

// kDirect: the first round's variant (GemmParams::direct), a separate
// instantiation so the filtering epilogue of the later rounds is unchanged.
template <bool kDirect>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base for the swizzled operand tiles
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const GemmSmem lay = gemm_smem_layout(false, p.slice_g ? p.cnt_words : 0u);
  uint32_t* cnt_s = reinterpret_cast<uint32_t*>(smem + lay.cnt_off);
  if (p.slice_g)
    for (uint32_t i = threadIdx.x; i < p.cnt_words; i += blockDim.x) cnt_s[i] = 0u;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.bars_off);
  uint64_t* empty = full + kGemmStages;
  uint64_t* tfull = empty + kGemmStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_word = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // the four warps of the group draining buffer b
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_word, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_word;

  const uint32_t ntiles = (p.rt1 - p.rt0) * p.nqt;
  const uint32_t KB = p.KB;

  if (warp == kProdWarp) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const uint32_t rt = p.rt0 + t / p.nqt, qt = t % p.nqt;
        for (uint32_t kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % kGemmStages, ph = (it / kGemmStages) & 1u;
          if (it >= kGemmStages && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.err)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + s * kStageBytes;
          uint8_t* b = a + kBQTileBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          bulk_g2s(a, p.qtiles + (static_cast<size_t>(qt) * KB + kb) * kBQTileBytes, kBQTileBytes, &full[s]);
          bulk_g2s(b, p.ctiles + (static_cast<size_t>(rt) * KB + kb) * kBRowTileBytes, kBRowTileBytes,
                   &full[s]);
        }
      }
      // copies still in flight land before the CTA may exit
      for (uint32_t j = it > kGemmStages ? it - kGemmStages : 0; j < it; ++j)
        mbar_wait_bounded(&full[j % kGemmStages], (j / kGemmStages) & 1u, p.err);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
        const uint32_t buf = tc & 1u, use = tc >> 1;
        if (use > 0 && !mbar_wait_bounded(&tempty[buf], (use - 1u) & 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBRowTile;
        for (uint32_t kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % kGemmStages, ph = (it / kGemmStages) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_addr(smem + s * kStageBytes);
          const uint64_t ad = sw128_desc(a), bd = sw128_desc(a + kBQTileBytes);
#pragma unroll
          for (uint32_t j = 0; j < kKBlock / 32; ++j)  // K = 32 bytes per instruction
            mma_i8(d, ad + 2u * j, bd + 2u * j, kIdescI8, (kb | j) != 0u ? 1u : 0u);
          mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) mma_commit(&tfull[buf]);
      }
      // every MMA issued has completed before TMEM is released
      mma_commit(done);
      mbar_wait_bounded(done, 0, p.err);
    }
  } else {
    gemm_epilogue<false, kDirect>(p, smem, lay, tfull, tempty, tmem, blockIdx.x, gridDim.x, ntiles, p.nqt, 0u, cnt_s, warp,
                         lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  } else if (p.slice_g && warp < kEpiWarps) {
    // publish this CTA's slice counts: every query of its query tiles, zeros
    // included (the select reads each slice's count)
    const uint32_t slice = blockIdx.x / p.slice_g, qt0 = blockIdx.x % p.slice_g;
    const uint32_t nlocal = p.nqt / p.slice_g;
    for (uint32_t e = threadIdx.x; e < nlocal * kBQTile; e += kEpiWarps * 32) {
      const uint32_t qi = (qt0 + (e / kBQTile) * p.slice_g) * kBQTile + e % kBQTile;
      if (qi < p.nq) p.scnt[static_cast<size_t>(slice) * p.nq + qi] = (cnt_s[e >> 1] >> ((e & 1u) * 16u)) & 0xFFFFu;
    }
  }
}


// The CTA-pair GEMM (cluster of two, tcgen05.mma.cta_group::2, M = 256
// queries x N = 256 rows x K = 32 per instruction).  Both CTAs run the same
// tile sequence.  Each CTA's producer loads its 128 queries and its 128 of the
// row tile's 256 rows by TMA tensor copies (no multicast) whose bytes complete
// on the leader's (rank 0) full barrier; the leader's MMA thread issues the
// pair's MMAs and multicasts its commits to both CTAs' empty / tfull barriers;
// each CTA's epilogue drains its own TMEM (its 128 queries x 256 rows) and
// frees the buffer on the leader's tempty barrier.  Every wait is bounded.
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ GemmParams p, const __grid_constant__ CUtensorMap amap,
                     const __grid_constant__ CUtensorMap bmap) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base (the same offset in both CTAs: the MMA reads the
  // peer's operands at this CTA's addresses)
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const GemmSmem lay = gemm_smem_layout(true);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.bars_off);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_word = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank(), pair = cluster_id(), npairs = cluster_count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx; both CTAs' bytes complete it
      mbar_init(&empty[s], 1);  // the leader's commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // the four warps draining buffer b, in each CTA
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(tmem_word, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers and TMEM of both CTAs are ready before any copy or remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_word;
  const uint32_t nqt2 = (p.nqt + 1u) / 2u;
  const uint32_t ntiles = (p.rt1 - p.rt0) * nqt2;
  const uint32_t KB = p.KB;

  if (warp == kProdWarp) {
    if (lane == 0) {
      const uint32_t lead_full = cluster_addr(&full[0], 0);  // full[s] of the leader: + 8 s
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t t = pair; t < ntiles && ok; t += npairs) {
        const uint32_t rt = p.rt0 + t / nqt2, qt = 2u * (t % nqt2) + rank;
        for (uint32_t kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % kPairStages, ph = (it / kPairStages) & 1u;
          if (it >= kPairStages && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.err)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + s * kPairStageBytes;
          uint8_t* b = a + kBQTileBytes;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2u * kPairStageBytes);
          const uint32_t fb = lead_full + 8u * s;
          tma_load_pair(a, &amap, 0u, (qt * KB + kb) * kBQTile, fb);
          tma_load_pair(b, &bmap, 0u, (rt * KB + kb) * kBRowTile + rank * (kBRowTile / 2u), fb);
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (rank == 0 && lane == 0) {
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (uint32_t t = pair; t < ntiles && ok; t += npairs, ++tc) {
        const uint32_t buf = tc & 1u, use = tc >> 1;
        if (use > 0 && !mbar_wait_bounded(&tempty[buf], (use - 1u) & 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBRowTile;
        for (uint32_t kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % kPairStages, ph = (it / kPairStages) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_addr(smem + s * kPairStageBytes);
          const uint64_t ad = sw128_desc(a), bd = sw128_desc(a + kBQTileBytes);
#pragma unroll
          for (uint32_t j = 0; j < kKBlock / 32; ++j)  // K = 32 bytes per instruction
            mma_i8_pair(d, ad + 2u * j, bd + 2u * j, kIdescI8Pair, (kb | j) != 0u ? 1u : 0u);
          mma_commit_pair_mc(&empty[s], 0x3);  // both CTAs' stage s is free once these MMAs have read it
        }
        if (ok) mma_commit_pair_mc(&tfull[buf], 0x3);
      }
      // every MMA issued has completed before either CTA's TMEM or stages go
      mma_commit_pair_mc(done, 0x1);
      mbar_wait_bounded(done, 0, p.err);
    }
  } else {
    gemm_epilogue<true>(p, smem, lay, tfull, tempty, tmem, pair, npairs, ntiles, nqt2, rank, nullptr, warp, lane);
  }
  tc_fence_before();
  cluster_sync_all();  // the pair's MMAs are complete and both epilogues have drained their TMEM
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------- select
// One CTA per query: the best F of the query's candidates, sorted descending
// into cand[0..Fp) (zero padded); thr = the F-th best key once F exist.
//
// select_run<K>: the selection with K key registers a thread, for at most
// K x 512 candidates.  The kernel sizes K to the candidates present (the
// kept list plus the round's hits, usually a few thousand), so the radix
// passes walk a few registers a thread rather than the buffer's capacity.
template <int MAXK>
__device__ __forceinline__ void select_run(const SelectParams& p, uint64_t* c, uint32_t* sc, uint32_t nk,
                                           uint32_t total, uint64_t* kept, uint32_t* hist, uint32_t* misc,
                                           const uint32_t* pre, int ctid, uint32_t qi);

template <int MAXK>
__global__ void __launch_bounds__(kConsumerThreads, 1) select_kernel(const SelectParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* kept = reinterpret_cast<uint64_t*>(smem);          // Fp
  uint32_t* hist = reinterpret_cast<uint32_t*>(kept + p.Fp);   // kSelBins
  uint32_t* misc = hist + kSelBins;                            // 128
  uint32_t* pre = misc + 128;                                  // nslices + 1: keys before each slice
  const int ctid = threadIdx.x;
  const uint32_t qi = blockIdx.x;
  uint64_t* c = p.cand + static_cast<size_t>(qi) * p.cap;
  uint32_t* sc = p.scnt + qi;  // slice s at sc[s * nq]
  const uint32_t nk = p.sbase == 0 ? 0u : (p.cnt[qi] < p.Fp ? p.cnt[qi] : p.Fp);  // the kept region
  if (ctid < 32) {  // one warp: the slices' counts (capped at their size) and their prefix
    uint32_t carry = 0;
    for (uint32_t s0 = 0; s0 < p.nslices; s0 += 32) {
      const uint32_t s = s0 + static_cast<uint32_t>(ctid);
      uint32_t m = s < p.nslices ? sc[static_cast<size_t>(s) * p.nq] : 0u;
      m = m < p.slice_cap ? m : p.slice_cap;
      uint32_t x = m;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
        if (ctid >= off) x += y;
      }
      if (s < p.nslices) pre[s] = carry + x - m;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (ctid == 0) pre[p.nslices] = carry;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t total = nk + pre[p.nslices];
  const uint32_t per = (total + kConsumerThreads - 1) / kConsumerThreads;  // uniform in the CTA
  if (MAXK > 4 && per <= 4) return select_run<(MAXK > 4 ? 4 : MAXK)>(p, c, sc, nk, total, kept, hist, misc, pre, ctid, qi);
  if (MAXK > 8 && per <= 8) return select_run<(MAXK > 8 ? 8 : MAXK)>(p, c, sc, nk, total, kept, hist, misc, pre, ctid, qi);
  if (MAXK > 16 && per <= 16) return select_run<(MAXK > 16 ? 16 : MAXK)>(p, c, sc, nk, total, kept, hist, misc, pre, ctid, qi);
  select_run<MAXK>(p, c, sc, nk, total, kept, hist, misc, pre, ctid, qi);
}

template <int MAXK>
__device__ __forceinline__ void select_run(const SelectParams& p, uint64_t* c, uint32_t* sc, uint32_t nk,
                                           uint32_t total, uint64_t* kept, uint32_t* hist, uint32_t* misc,
                                           const uint32_t* pre, int ctid, uint32_t qi) {
  // candidate u: the kept keys first, then slice by slice (the slice of a key
  // by binary search over the prefix)
  uint64_t v[MAXK];
#pragma unroll
  for (int i = 0; i < MAXK; ++i) {
    const uint32_t u = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
    uint64_t x = 0ull;
    if (u < nk) {
      x = c[u];
    } else if (u < total && p.nslices == 1u) {
      x = c[p.sbase + (u - nk)];
    } else if (u < total) {
      const uint32_t w = u - nk;
      uint32_t lo = 0, hi = p.nslices - 1u;  // the last slice with pre[s] <= w
      while (lo < hi) {
        const uint32_t mid = (lo + hi + 1u) >> 1;
        if (pre[mid] <= w) lo = mid;
        else hi = mid - 1u;
      }
      x = c[p.sbase + lo * p.slice_cap + (w - pre[lo])];
    }
    v[i] = x;
  }
  for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) kept[i] = 0ull;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  for (uint32_t s = ctid; s < p.nslices; s += kConsumerThreads) sc[static_cast<size_t>(s) * p.nq] = 0u;  // next GEMM starts empty
  const uint32_t n = keep_best<MAXK>(v, total, p.F, kept, hist, misc, ctid);
  if (p.Fp <= 256u) {  // one warp sorts the kept keys in registers, no block barriers
    warp0_sort_dispatch(p.Fp, kept, ctid);
    named_bar_sync(kBarConsumers, kConsumerThreads);
    for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) c[i] = kept[i];
    if (ctid == 0) {
      p.cnt[qi] = n;
      p.thr[qi] = n >= p.F ? kept[p.F - 1] : 0ull;
    }
    return;
  }
  // wide F: the kept keys stay unsorted (the re-rank tail selects and sorts
  // them itself); the F-th best key is the least kept key
  uint64_t mn = ~0ull;
  for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) {
    const uint64_t x = kept[i];
    c[i] = x;
    if (i < n && x < mn) mn = x;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const uint64_t o = __shfl_xor_sync(0xffffffffu, mn, off);
    mn = o < mn ? o : mn;
  }
  uint64_t* red = reinterpret_cast<uint64_t*>(misc + kMiscSel);
  if ((ctid & 31) == 0) red[ctid >> 5] = mn;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (ctid == 0) {
    for (int w = 1; w < kConsumerWarps; ++w) mn = red[w] < mn ? red[w] : mn;
    p.cnt[qi] = n;
    p.thr[qi] = n >= p.F ? mn : 0ull;
  }
}

// The rounds after the first: the same selection in chunks, with K key
// registers a thread of which two carry the best F so far (Fp <= 1024) from
// chunk to chunk, so any number of candidates fits and a thread needs few
// registers: two CTAs share an SM, and their barrier waits overlap.
template <int K>
__global__ void __launch_bounds__(kConsumerThreads, 2) select_lean_kernel(const SelectParams p) {
  constexpr int KC = 2;       // carried keys a thread (Fp <= KC x 512)
  constexpr int KN = K - KC;  // new keys a thread per chunk
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* kept = reinterpret_cast<uint64_t*>(smem);          // Fp
  uint32_t* hist = reinterpret_cast<uint32_t*>(kept + p.Fp);   // kSelBins
  uint32_t* misc = hist + kSelBins;                            // 128
  uint32_t* pre = misc + 128;                                  // nslices + 1
  const int ctid = threadIdx.x;
  const uint32_t qi = blockIdx.x;
  uint64_t* c = p.cand + static_cast<size_t>(qi) * p.cap;
  uint32_t* sc = p.scnt + qi;
  const uint32_t nk = p.sbase == 0 ? 0u : (p.cnt[qi] < p.Fp ? p.cnt[qi] : p.Fp);
  if (ctid < 32) {
    uint32_t carry = 0;
    for (uint32_t s0 = 0; s0 < p.nslices; s0 += 32) {
      const uint32_t s = s0 + static_cast<uint32_t>(ctid);
      uint32_t m = s < p.nslices ? sc[static_cast<size_t>(s) * p.nq] : 0u;
      m = m < p.slice_cap ? m : p.slice_cap;
      uint32_t x = m;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
        if (ctid >= off) x += y;
      }
      if (s < p.nslices) pre[s] = carry + x - m;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (ctid == 0) pre[p.nslices] = carry;
  }
  for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) kept[i] = 0ull;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t total = nk + pre[p.nslices];
  for (uint32_t s = ctid; s < p.nslices; s += kConsumerThreads) sc[static_cast<size_t>(s) * p.nq] = 0u;
  uint32_t n = 0;  // keys in kept (the best F of the chunks so far)
  for (uint32_t c0 = 0; c0 < total; c0 += KN * kConsumerThreads) {
    uint64_t v[K];
#pragma unroll
    for (int i = 0; i < KN; ++i) {
      const uint32_t u = c0 + static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
      uint64_t x = 0ull;
      if (u < nk) {
        x = c[u];
      } else if (u < total && p.nslices == 1u) {
        x = c[p.sbase + (u - nk)];
      } else if (u < total) {
        const uint32_t w = u - nk;
        uint32_t lo = 0, hi = p.nslices - 1u;  // the last slice with pre[s] <= w
        while (lo < hi) {
          const uint32_t mid = (lo + hi + 1u) >> 1;
          if (pre[mid] <= w) lo = mid;
          else hi = mid - 1u;
        }
        x = c[p.sbase + lo * p.slice_cap + (w - pre[lo])];
      }
      v[i] = x;
    }
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      const uint32_t u = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(j) * kConsumerThreads;
      v[KN + j] = u < n ? kept[u] : 0ull;
    }
    const uint32_t fresh = total - c0 < KN * kConsumerThreads ? total - c0 : KN * kConsumerThreads;
    named_bar_sync(kBarConsumers, kConsumerThreads);  // kept is read before keep_best rewrites it
    n = keep_best<K>(v, fresh + n, p.F, kept, hist, misc, ctid);
  }
  if (p.Fp <= 256u) {
    warp0_sort_dispatch(p.Fp, kept, ctid);
    named_bar_sync(kBarConsumers, kConsumerThreads);
    for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) c[i] = kept[i];
    if (ctid == 0) {
      p.cnt[qi] = n;
      p.thr[qi] = n >= p.F ? kept[p.F - 1] : 0ull;
    }
    return;
  }
  uint64_t mn = ~0ull;
  for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) {
    const uint64_t x = kept[i];
    c[i] = x;
    if (i < n && x < mn) mn = x;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const uint64_t o = __shfl_xor_sync(0xffffffffu, mn, off);
    mn = o < mn ? o : mn;
  }
  uint64_t* red = reinterpret_cast<uint64_t*>(misc + kMiscSel);
  if ((ctid & 31) == 0) red[ctid >> 5] = mn;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (ctid == 0) {
    for (int w = 1; w < kConsumerWarps; ++w) mn = red[w] < mn ? red[w] : mn;
    p.cnt[qi] = n;
    p.thr[qi] = n >= p.F ? mn : 0ull;
  }
}

// ------------------------------------------------------------- compaction
// A filtered batch contracts only the rows its mask keeps: the kept rows'
// tiles are gathered into a dense corpus (row c of it = the c-th kept row, in
// row order, so ordering by c is ordering by row) and the candidates' rows
// are mapped back before the re-rank.
constexpr uint32_t kScanWords = 1024;  // mask words per scan block

// Per block: exclusive prefix of the popcounts of its mask words, and the block total.
// Mask word w with the bits of rows past the end cleared.
__device__ __forceinline__ uint32_t mask_word(const uint32_t* mask, uint64_t w, uint64_t rows) {
  uint32_t m = mask[w];
  const uint64_t end = (w + 1) * 32u;
  if (end > rows) m &= (1u << static_cast<uint32_t>(rows - w * 32u)) - 1u;
  return m;
}

__global__ void __launch_bounds__(kScanWords) mask_scan_kernel(const uint32_t* mask, uint64_t rows, uint64_t words,
                                                               uint32_t* word_off, uint32_t* block_sum) {
  __shared__ uint32_t warp_tot[32];
  const uint64_t w = static_cast<uint64_t>(blockIdx.x) * kScanWords + threadIdx.x;
  const uint32_t c = w < words ? __popc(mask_word(mask, w, rows)) : 0u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t t = warp_tot[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, t, off);
      if (lane >= off) t += y;
    }
    warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  const uint32_t before = (warp ? warp_tot[warp - 1] : 0u) + x - c;
  if (w < words) word_off[w] = before;
  if (threadIdx.x == kScanWords - 1) block_sum[blockIdx.x] = warp_tot[31];
}

// Exclusive prefix of the block totals (one CTA, any count), and the grand total.
__global__ void __launch_bounds__(1024) block_scan_kernel(uint32_t* block_sum, uint32_t nblocks, uint32_t* total) {
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint32_t b0 = 0; b0 < nblocks; b0 += 1024) {
    const uint32_t b = b0 + threadIdx.x;
    const uint32_t c = b < nblocks ? block_sum[b] : 0u;
    uint32_t x = c;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      uint32_t t = warp_tot[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, t, off);
        if (lane >= off) t += y;
      }
      warp_tot[lane] = t;
    }
    __syncthreads();
    const uint32_t before = carry + (warp ? warp_tot[warp - 1] : 0u) + x - c;
    if (b < nblocks) block_sum[b] = before;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_tot[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

// map[c] = the c-th kept row.
__global__ void __launch_bounds__(256) row_map_kernel(const uint32_t* mask, uint64_t rows, uint64_t words,
                                                      const uint32_t* word_off, const uint32_t* block_sum,
                                                      uint32_t* map) {
  const uint64_t w = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w >= words) return;
  uint32_t m = mask_word(mask, w, rows);
  uint32_t o = word_off[w] + block_sum[w / kScanWords];
  while (m) {
    const uint32_t b = __ffs(m) - 1u;
    m &= m - 1u;
    map[o++] = static_cast<uint32_t>(w * 32u + b);
  }
}

// ------------------------------------------------------------- shards
// A key of local row r as a key of global row r + base (same score bits).
__device__ __forceinline__ uint64_t global_key(uint64_t key, uint32_t base) {
  const uint32_t row = ~static_cast<uint32_t>(key);
  return (key & 0xFFFFFFFF00000000ull) | static_cast<uint32_t>(~(row + base));
}

// keys[q*F + i] = the i-th kept key of query q as a global-row key (zero past
// the kept count).
__global__ void __launch_bounds__(256) export_keys_kernel(const uint64_t* cand, uint32_t cap, const uint32_t* cnt,
                                                          uint32_t nq, uint32_t F, uint32_t base, uint64_t* keys) {
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<uint64_t>(nq) * F) return;
  const uint32_t q = static_cast<uint32_t>(i / F), j = static_cast<uint32_t>(i % F);
  const uint32_t n = cnt[q] < F ? cnt[q] : F;
  const uint64_t x = j < n ? cand[static_cast<size_t>(q) * cap + j] : 0ull;
  keys[i] = x ? global_key(x, base) : 0ull;
}

// Drop (zero) the kept keys of query q below thr[q] (global-row keys); a
// descending list stays descending with its zeros at the end.
__global__ void __launch_bounds__(256) trim_keys_kernel(uint64_t* cand, uint32_t cap, uint32_t Fp, uint32_t nq,
                                                        uint32_t base, const uint64_t* thr) {
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<uint64_t>(nq) * Fp) return;
  const uint32_t q = static_cast<uint32_t>(i / Fp), j = static_cast<uint32_t>(i % Fp);
  uint64_t* c = cand + static_cast<size_t>(q) * cap + j;
  const uint64_t x = *c;
  if (x && global_key(x, base) < thr[q]) *c = 0ull;
}

// One CTA per query: among the W gathered key lists (W x nq x F, list w of
// query q at (w * nq + q) * F), a threshold with exactly min(F, total) keys at
// or above it.
template <int MAXK>
__global__ void __launch_bounds__(kConsumerThreads, 1) keys_threshold_kernel(const uint64_t* gathered, uint32_t world,
                                                                            uint32_t nq, uint32_t F, uint64_t* thr) {
  __shared__ uint32_t hist[kSelBins];
  __shared__ uint32_t sh[kSelScratch];
  __shared__ uint32_t red[kConsumerWarps];
  const int ctid = threadIdx.x;
  const uint32_t q = blockIdx.x, total_slots = world * F;
  uint64_t v[MAXK];
  uint32_t c = 0;
#pragma unroll
  for (int i = 0; i < MAXK; ++i) {
    const uint32_t idx = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
    uint64_t x = 0ull;
    if (idx < total_slots) {
      const uint32_t w = idx / F, j = idx - w * F;
      x = __ldcg(gathered + (static_cast<size_t>(w) * nq + q) * F + j);
    }
    v[i] = x;
    c += x ? 1u : 0u;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
  if ((ctid & 31) == 0) red[ctid >> 5] = c;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  uint32_t total = 0;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) total += red[w];
  const uint64_t t = block_select_threshold<MAXK, kConsumerThreads>(v, MAXK, F, total, hist, sh, ctid,
                                                                    kBarConsumers);
  if (ctid == 0) thr[q] = t;
}

// ------------------------------------------------------------- launchers
uint32_t batch_gemm_smem(uint32_t cnt_words) { return gemm_smem_layout(false, cnt_words).total + 1024; }

cudaError_t launch_mask_count(const uint32_t* mask, uint64_t rows, uint32_t* word_off, uint32_t* block_sum,
                              uint32_t* count, cudaStream_t s) {
  const uint64_t words = (rows + 31) / 32;
  const uint32_t nb = static_cast<uint32_t>((words + kScanWords - 1) / kScanWords);
  mask_scan_kernel<<<nb, kScanWords, 0, s>>>(mask, rows, words, word_off, block_sum);
  block_scan_kernel<<<1, 1024, 0, s>>>(block_sum, nb, count);
  return cudaGetLastError();
}

cudaError_t launch_row_map(const uint32_t* mask, uint64_t rows, const uint32_t* word_off, const uint32_t* block_sum,
                           uint32_t* map, cudaStream_t s) {
  const uint64_t words = (rows + 31) / 32;
  row_map_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, s>>>(mask, rows, words, word_off, block_sum,
                                                                            map);
  return cudaGetLastError();
}

uint32_t compact_block_words() { return kScanWords; }

cudaError_t launch_expand(const ExpandParams& p, cudaStream_t s) {
  if (p.count == 0) return cudaSuccess;
  const uint32_t t0 = p.pos0 / kBRowTile, t1 = (p.pos0 + p.count + kBRowTile - 1) / kBRowTile;
  const dim3 grid(t1 - t0);
  if (p.bits == 8) expand_kernel<8><<<grid, kBRowTile, 0, s>>>(p);
  else if (p.bits == 4) expand_kernel<4><<<grid, kBRowTile, 0, s>>>(p);
  else expand_kernel<1><<<grid, kBRowTile, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_factor(uint32_t bits, const float* scales, const uint32_t* rows, uint32_t row0, uint32_t n,
                          float* fac, uint32_t* ids, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const unsigned grid = (n + 255) / 256;
  if (bits == 8) factor_kernel<8><<<grid, 256, 0, s>>>(scales, rows, row0, n, fac, ids);
  else if (bits == 4) factor_kernel<4><<<grid, 256, 0, s>>>(scales, rows, row0, n, fac, ids);
  else factor_kernel<1><<<grid, 256, 0, s>>>(scales, rows, row0, n, fac, ids);
  return cudaGetLastError();
}

cudaError_t launch_scatter_tiles(const uint32_t* in, uint32_t* out, uint32_t count, uint32_t head, uint32_t K,
                                 uint32_t ginv, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  scatter_tiles_kernel<<<(count + 255) / 256, 256, 0, s>>>(in, out, count, head, K, ginv);
  return cudaGetLastError();
}

// Rows ordered by ascending factor (a radix sort of the factor keys carrying
// the row ids); tmp == nullptr only sizes the temporary storage.
cudaError_t launch_sort_rows(void* tmp, size_t* tmp_bytes, const float* fac_in, float* fac_out,
                             const uint32_t* ids_in, uint32_t* ids_out, uint32_t n, cudaStream_t s) {
  return cub::DeviceRadixSort::SortPairs(tmp, *tmp_bytes, fac_in, fac_out, ids_in, ids_out, static_cast<int>(n), 0,
                                         32, s);
}

cudaError_t launch_prep(const PrepParams& p, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(p.P) * 4 + p.KB * kKBlock + 64;
  static int opted[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(prep_kernel), smem, opted);
  if (e != cudaSuccess) return e;
  prep_kernel<<<p.nq, kConsumerThreads, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmParams& p, uint32_t grid, cudaStream_t s) {
  const size_t smem = batch_gemm_smem(p.slice_g ? p.cnt_words : 0u);
  static int opted[2][kMaxDevices] = {};
  auto kern = p.direct ? gemm_kernel<true> : gemm_kernel<false>;
  cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(kern), smem, opted[p.direct ? 1 : 0]);
  if (e != cudaSuccess) return e;
  kern<<<grid, kGemmThreads, smem, s>>>(p);
  return cudaGetLastError();
}

uint32_t batch_gemm_pair_smem() { return gemm_smem_layout(true).total + 1024; }

// The pair GEMM over `npairs` clusters of two CTAs; amap / bmap: tensor maps
// (encode_tile_rows_map) of the query tiles (128-row boxes) and the row tiles
// (128-row boxes, half a tile).
cudaError_t launch_gemm_pair(const GemmParams& p, const void* amap, const void* bmap, uint32_t npairs,
                             cudaStream_t s) {
  const size_t smem = batch_gemm_pair_smem();
  static int opted[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(gemm_pair_kernel), smem, opted);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2u * npairs);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_pair_kernel, p, *static_cast<const CUtensorMap*>(amap),
                            *static_cast<const CUtensorMap*>(bmap));
}

cudaError_t launch_select(const SelectParams& p, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(p.Fp) * 8 + kSelBins * 4 + 128 * 4 + (static_cast<size_t>(p.nslices) + 1) * 4;
  const uint32_t maxk = (p.cap + kConsumerThreads - 1) / kConsumerThreads;
  auto go = [&](auto kern) -> cudaError_t {
    static int opted[kMaxDevices] = {};
    cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(kern), smem, opted);
    if (e != cudaSuccess) return e;
    kern<<<p.nq, kConsumerThreads, smem, s>>>(p);
    return cudaGetLastError();
  };
  // the first round (every row a candidate) in one pass; later rounds of a
  // wide F (a kept list of up to 1,024 keys plus hits) in chunks, two CTAs an
  // SM (config 4 select 0.56 -> 0.47 ms a step; with F <= 256 the one-pass
  // kernel stays faster: config 3 1.38 vs 1.53 ms, config 5 0.62 vs 0.70)
  if (p.sbase != 0 && p.Fp > 256u && p.Fp <= 2u * kConsumerThreads) return go(select_lean_kernel<8>);
  if (maxk <= 8) return go(select_kernel<8>);
  if (maxk <= 16) return go(select_kernel<16>);
  if (maxk <= 32) return go(select_kernel<32>);
  return cudaErrorInvalidValue;
}

cudaError_t launch_export_keys(const uint64_t* cand, uint32_t cap, const uint32_t* cnt, uint32_t nq, uint32_t F,
                               uint32_t base, uint64_t* keys, cudaStream_t s) {
  const uint64_t n = static_cast<uint64_t>(nq) * F;
  if (n == 0) return cudaSuccess;
  export_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(cand, cap, cnt, nq, F, base, keys);
  return cudaGetLastError();
}

cudaError_t launch_trim_keys(uint64_t* cand, uint32_t cap, uint32_t Fp, uint32_t nq, uint32_t base,
                             const uint64_t* thr, cudaStream_t s) {
  const uint64_t n = static_cast<uint64_t>(nq) * Fp;
  if (n == 0) return cudaSuccess;
  trim_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(cand, cap, Fp, nq, base, thr);
  return cudaGetLastError();
}

uint32_t keys_threshold_max() { return 32u * kConsumerThreads; }

cudaError_t launch_keys_threshold(const uint64_t* gathered, uint32_t world, uint32_t nq, uint32_t F, uint64_t* thr,
                                  cudaStream_t s) {
  const uint32_t maxk = (world * F + kConsumerThreads - 1) / kConsumerThreads;
  if (maxk <= 8) keys_threshold_kernel<8><<<nq, kConsumerThreads, 0, s>>>(gathered, world, nq, F, thr);
  else if (maxk <= 16) keys_threshold_kernel<16><<<nq, kConsumerThreads, 0, s>>>(gathered, world, nq, F, thr);
  else if (maxk <= 32) keys_threshold_kernel<32><<<nq, kConsumerThreads, 0, s>>>(gathered, world, nq, F, thr);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace bv
