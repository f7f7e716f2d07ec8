// Grouped bf16 expert GEMM on the 5th-generation tensor cores (tcgen05).
//
// Problem: for every expert e, D[rows of e] = A[rows of e] . B[e]^T, where
// A [rows, K] holds the permuted token rows (expert-contiguous, ranges from
// expert_offsets) and B [E, Nb, K] the expert weights, both K-major bf16.
// This is the contraction of ref_grouped_gemm (tests/test_reference.py:228-254)
// and of the expert FFN flow in USAGE.md:40-57.
//
// Tiling.  A tile is 128 rows x 256 B-rows x all of K.  A work unit is one
// n-tile of one expert against: a pair of tiles (up to 256 rows: two MMAs
// that share every weight box, one TMEM accumulator each); one wide swapped
// tile of 129..192 rows (below); or one tile of at most 128 rows.  Every
// expert row passes through a weight stage once per n-tile, and no weight
// tile is filled into shared memory twice for one expert.  Units are (expert, n-tile, m-unit) in that
// nesting, m fastest, so the m-units that share one weight tile are taken by
// neighbouring CTAs at the same time and the weight tile is read from HBM
// once (later reads hit L2); the 16-28 n-tiles of one expert reuse its A rows
// from L2.  A persistent grid of one CTA per SM takes units from an atomic
// counter in caller scratch (or, with no scratch, with a static stride):
// CTAs that become free together take neighbouring units, so units that
// share a weight tile read each line within microseconds of each other and
// the later reads hit L2, where a static stride lets the CTAs drift apart
// until the line has been evicted.  At DeepSeek-V3 shape the kernel is bound
// by streaming the weights from HBM.
//
// One CTA = 10 warps:
//   warp 0      TMA producer: takes the next unit id, publishes it to the
//               other warps through a 4-entry shared-memory queue, then per
//               k-block loads one stage (two weight boxes [128 x 64] and the
//               A box [128 x 64], or two A boxes for a paired unit) into a
//               208 KB byte ring (128-byte swizzle), completing on the
//               stage's `full` mbarrier.  Single stages (48 KB) and paired
//               ones (64 KB) share the ring back to back.
//   warp 1      MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=16) per stage
//               and accumulator, into one of two TMEM accumulators (2 x 256
//               fp32 columns = all 512 columns), or both for a paired unit;
//               tcgen05.commit frees the stage and, after the last k-block,
//               signals each accumulator full.
//   warps 2-9   epilogue, two groups of four: tcgen05.ld 32 columns at a
//               time (warp w reads TMEM lanes 32*(w%4)..+31 = its 32 rows;
//               each group takes half of the columns), convert, store to
//               global, then release the accumulator; a single unit's
//               epilogue overlaps the next unit's main loop thanks to the
//               second accumulator (a paired unit waits for both).
// Swapped tiles (wide ones of 129..192 rows; small ones of at most
// kSwapMaxRows rows at decode sizes and with a gathered A) put the two
// weight boxes on the MMA's M side (2 x M=128) and the tile's r token rows
// on its N side (N = r rounded up to 16).  An M=128 tcgen05.mma costs about
// 71 cycles for any N <= 144 and runs at the dense rate only from N ~ 144 up
// (measured on B200), so the unit kinds are chosen by MMA count: at
// DeepSeek-V3 shape (about 128-150 rows per expert) a full tile plus a
// swapped tail of a few rows took 4 + 8 MMAs (~1110 cycles) per k-block,
// more than the weights take to arrive at the B200's clock under this load
// (1.5-1.6 GHz measured), while one wide tile takes 8 MMAs at N ~ 144 (~580
// cycles).  A wide tile's A rows arrive as one 128-row box and 16-row boxes
// (a second tensor map).  The epilogue of a swapped tile reads the transposed accumulator
// (TMEM lane = output column, TMEM column = token); a wide tile's occupies
// TMEM columns 0 .. 2N-1, both accumulators.  The same products are summed
// in the same k order either way.
// COMBINE mode (the expert-parallel down projection) ends each output row
// in the combine instead of D: row p becomes bf16(w[p] * bf16(acc)) stored at
// row dst_row[p] of rank dst_rank[p]'s combine buffer (peer memory over
// NVLink), and the last CTA publishes the combine epoch to every rank.  The
// per-element arithmetic is that of the plain GEMM followed by
// moe_unpermute_bf16_perslot.
// SWIGLU mode stacks 128 gate rows (rows n*128 of the expert) and the matching
// 128 up rows (rows I + n*128) as the two B boxes, so one N=256 MMA yields g
// and u for 128 output columns; the epilogue rounds both to bf16 and applies
// swiglu_f32, which makes the result bit-identical to the plain GEMM followed
// by the standalone fused_swiglu kernel.
//
// Every mbarrier wait is bounded (kWaitLimitNs).  A role whose wait expires
// records a device error, raises the CTA abort flag and leaves its loop; the
// producer then waits (bounded) for the loads it issued, the MMA warp for its
// outstanding MMAs, and warp 1 frees TMEM before the CTA exits.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "ep_peer.cuh"
#include "swiglu.cuh"

namespace lsek {

lsek_status ep_take_device_error(int32_t* code);  // ep.cu

// Device-side error word (see DeviceError in common.cuh).
__device__ int32_t g_device_error = 0;

__device__ __forceinline__ void report_device_error(int32_t code) {
  atomicCAS(&g_device_error, 0, code);
}

namespace gemm {

constexpr int kBM = 128;                       // UMMA M, rows per tile
constexpr int kBK = 64;                        // K per stage = one 128-byte swizzle row
constexpr int kBN = 256;                       // UMMA N
constexpr int kBoxRows = 128;                  // rows per TMA box
constexpr int kBoxBytes = kBoxRows * kBK * 2;  // 16 KB
constexpr int kTmemCols = 2 * kBN;             // two accumulators
constexpr int kEpiWarps = 8;                   // two groups of four, one warp per TMEM lane quarter each
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxExperts = 1024;
constexpr int kUnitQ = 4;                      // unit ids in flight between warps
constexpr int kSwapMaxRows = 64;               // tiles this small use swapped operands
constexpr int kA16Bytes = 16 * kBK * 2;        // one 16-row A box (2 KB)
constexpr int kWideMaxRows = 192;              // remainders of 129..192 rows run as wide tiles

// Pipeline geometry.  Each k-block of a unit is one stage: two 128-row
// weight boxes (adjacent, one N=256 MMA reads both) and the A rows of its
// tile (of both tiles for a paired unit).  A full tile's A rows are one
// 16 KB box; a swapped tile needs only its rows rounded up to 16, so its A
// part is that many 2 KB (16-row) boxes and its stage takes only the bytes
// it loads: 48 KB for a single full tile, 34-40 KB for a small expert's
// tile, 50-56 KB for the usual DeepSeek-V3 pair of a full tile and a few
// rows, 64 KB for two full tiles.  Stages lie back to back in a byte ring of
// RING_BYTES; a box that would cross the ring's end starts at its beginning
// instead (the skipped tail counts towards that stage), and every part of a
// stage starts on a 1024-byte boundary as the 128-byte swizzle needs.  Each
// stage has one full and one empty barrier (a ring of kRecs records).
// A_ROWS is the token rows of the tiled A box, MAX_E the largest expert
// count the unit table holds.
template <int RING_BYTES, int A_ROWS, int MAX_E>
struct Geom {
  static constexpr int kRingBytes = RING_BYTES;
  static constexpr int kARows = A_ROWS;
  static constexpr int kABytes = A_ROWS * kBK * 2;
  static constexpr int kMaxE = MAX_E;
  static constexpr int kRecs = 8;  // more than the stages that fit in the ring
  // Every tile has at most kARows rows, so every tile is a swapped small tile.
  static constexpr bool kSmallOnly = A_ROWS <= kSwapMaxRows;
  // Units may cover two m-tiles of an expert (M = 256 against one weight tile).
  static constexpr bool kPairs = !kSmallOnly;
  // The smallest stage: the weight boxes and one 16-row A box (or the tiled
  // A box of the decode geometry).
  static constexpr int kMinStageBytes = 2 * kBoxBytes + (kSmallOnly ? kABytes : 16 * kBK * 2);
  static_assert(kABytes % 1024 == 0 && RING_BYTES % 1024 == 0,
                "swizzled boxes start on 1024-byte boundaries");
  static_assert(RING_BYTES >= 2 * kBoxBytes + 2 * kABytes, "the largest stage fits the ring");
  static_assert(kRecs * kMinStageBytes > RING_BYTES, "a record is reused only after its stage left");
};
// Up to 256 experts (DeepSeek-V3 and smaller): the unit table takes 2 KB of
// shared memory and the ring the rest, 223 KB.  The ring is the kernel's
// main lever: at cfg1 it holds the weight bytes in flight while the MMA
// works through landed stages (a 176 KB ring measured 13 % slower than
// 208 KB).
using GeomFull = Geom<223 * 1024, 128, 256>;
// Up to 1024 experts: an 8 KB unit table and a 208 KB ring.
using GeomFullWide = Geom<13 * kBoxBytes, 128, kMaxExperts>;
// Decode (every expert has at most 32 rows): a 4 KB token box, six 36 KB
// stages in flight.
using GeomDecode = Geom<6 * (4096 + 2 * kBoxBytes), 32, 256>;
constexpr int kDecodeMaxRows = GeomDecode::kARows;

// M=128, N=256, A/B bf16 K-major, D fp32 (tcgen05 instruction descriptor:
// D format bits 4-5, A format bits 7-9, B format bits 10-12, N>>3 bits 17-22,
// M>>4 bits 24-28).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                            (static_cast<uint32_t>(kBN >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

struct Params {
  const int32_t* offsets;  // [E+1]
  int num_experts;
  int rows;                // rows of A and D
  int num_kb;              // ceil(K / kBK)
  int n_tiles;             // n-tiles per expert
  int b_rows;              // B rows per expert
  int b_tile_rows;         // first-box row step per n-tile
  int b_second;            // row offset of the second box
  __nv_bfloat16* D;
  int64_t ldd;
  int out_tile_cols;       // output columns per tile
  int n_out;               // output width
  float swiglu_limit;
  int32_t* counter;        // zeroed unit counter in device memory, or null (static stride)
  // Gathered A: row r of the (virtual) permuted A is row gather_idx[r] / gather_k
  // of the tensor behind tmap_a (the token rows), loaded with tile::gather4.
  const int32_t* gather_idx;
  int gather_k;
  // COMBINE mode
  const int32_t* dst_rank;  // [rows] rank whose combine buffer receives row p
  const int32_t* dst_row;   // [rows] row there
  const float* dst_w;       // [rows] routing weight
  PeerTable peers;          // every rank's domain buffer
  size_t back_offset;       // combine buffer offset inside a domain buffer
  int64_t back_rows;        // rows of each rank's combine buffer (larger dst_row: skipped)
  int world, me;
  uint32_t* done;           // zeroed local CTA counter
  uint32_t epoch;
};

enum GemmMode : int { kModePlain = 0, kModeSwiglu = 1, kModeCombine = 2 };

template <class G>
struct SmemT {
  uint8_t ring[G::kRingBytes];  // 1024-byte aligned (base is aligned)
  uint64_t full_bar[G::kRecs];
  uint64_t empty_bar[G::kRecs];
  uint64_t acc_full_bar[2];
  uint64_t acc_empty_bar[2];
  uint64_t mma_done_bar;
  uint64_t q_full[kUnitQ];
  uint64_t q_empty[kUnitQ];
  int32_t unit_q[kUnitQ];
  uint32_t span[G::kRecs];  // ring bytes of each outstanding stage (producer only)
  uint32_t tmem_base;
  int32_t abort;
  int32_t warp_tot[kThreads / 32];
  int32_t arow[kBM];  // gathered A: source row of each tile row (producer only)
  int32_t offs[G::kMaxE + 1];
  int32_t cum[G::kMaxE + 1];
};
template <class G>
constexpr size_t smem_bytes() {
  return sizeof(SmemT<G>) + 1024;
}
static_assert(smem_bytes<GeomFull>() <= 227 * 1024, "shared memory budget");
static_assert(smem_bytes<GeomFullWide>() <= 227 * 1024, "shared memory budget");
static_assert(smem_bytes<GeomDecode>() <= 227 * 1024, "shared memory budget");

// ---- PTX wrappers ----------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for phase `parity` of `bar`.  Gives up when another role has aborted
// (honor_abort) or after kWaitLimitNs, recording `code`.
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int32_t* abort,
                                       int32_t code, bool honor_abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (honor_abort && *abort) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      report_device_error(code);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// Four rows (row coordinates y0..y3, one 128-byte box row each) of a tensor
// whose map has a one-row box, stored back to back at `dst`.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int y0, int y1, int y2, int y3,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(y0), "r"(y1), "r"(y2),
      "r"(y3), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Shared-memory matrix descriptor: K-major tile of 128-byte rows with the
// 128-byte swizzle; 8-row groups 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

template <class S>
__device__ __forceinline__ int mtiles_of(const S& s, int e) {
  const int n = s.offs[e + 1] - s.offs[e];
  return n > 0 ? (n + kBM - 1) / kBM : 0;
}

// Units of one n-tile of expert e.  Without pairing: one per m-tile.  With
// pairing: one per 256-row block and one for the remaining rows (see
// decode_unit for how the last rows are cut).
template <class S>
__device__ __forceinline__ int munits_of(const S& s, int e, bool pairs) {
  if (!pairs) return mtiles_of(s, e);
  const int n = s.offs[e + 1] - s.offs[e];
  return n > 0 ? (n + 2 * kBM - 1) / (2 * kBM) : 0;
}

// Instruction descriptor of a swapped tile: M=128 weight rows, N=nn tokens.
__device__ __forceinline__ uint32_t swap_idesc(int nn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(nn >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

// A work unit: n-tile n of expert e against `rows` token rows starting at
// m-tile t0.  Three kinds (decode_unit cuts an expert's rows into them):
//   pair    tiles t0 and t0 + 1 (193..256 rows; the second may be partial)
//           against one weight stage, one TMEM accumulator each
//   wide    129..192 rows as one swapped tile: the two weight boxes on M and
//           all the rows on N (rounded up to 16), into TMEM columns
//           0 .. 2N-1, i.e. both accumulators.  An M=128 MMA costs about as
//           much at N=16 as at N=144 (measured ~71 cycles, the dense rate
//           only from N~144 up), so this takes 8 MMAs at N~144-192
//           (~580-770 cycles a k-block) where a full tile plus a swapped tail
//           took 4 + 8 (~1110) and a pair 8 at N=256 (~1024); above 192 rows
//           a pair costs no more and keeps the faster unswapped epilogue
//   single  at most 128 rows: one tile, swapped only where single_swapped
//           says so
struct Unit {
  int e, n, t0, rows;
  bool pair, wide;
};

// Maps a unit id to its unit: the largest e with cum[e] <= id is the
// (non-empty) expert that owns it; an expert's units are ordered
// (n-tile, m-unit) with the m-unit fastest.
template <class S>
__device__ __forceinline__ Unit decode_unit(const S& s, int num_experts, int id, bool pairs) {
  int lo = 0, hi = num_experts - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s.cum[mid] <= id) lo = mid;
    else hi = mid - 1;
  }
  Unit u;
  u.e = lo;
  const int local = id - s.cum[lo];
  const int mu = munits_of(s, lo, pairs);
  u.n = local / mu;
  const int m = local - u.n * mu;
  const int n = s.offs[lo + 1] - s.offs[lo];
  u.pair = u.wide = false;
  if (!pairs) {
    u.t0 = m;
    u.rows = min(n - m * kBM, kBM);
    return u;
  }
  // 256-row blocks run as pairs.  When at most 64 rows follow the last
  // block, its second half and those rows run as one wide tile instead
  // (128 + r rows): a full tile + a wide tile cost 4 + 8 MMAs at N >= 144 per
  // k-block, a pair plus a tile of r rows 8 + 4 at N = 256.
  const int nb = n / (2 * kBM), r = n - nb * 2 * kBM;
  const bool split = r > 0 && r <= kSwapMaxRows && nb >= 1;
  const int full_pairs = nb - (split ? 1 : 0);
  if (m < full_pairs) {
    u.t0 = 2 * m;
    u.pair = true;
    u.rows = 2 * kBM;
  } else if (split) {
    u.t0 = 2 * full_pairs + (m - full_pairs);
    u.wide = m > full_pairs;
    u.rows = u.wide ? kBM + r : kBM;
  } else {
    u.t0 = 2 * m;
    const int left = n - u.t0 * kBM;
    u.pair = left > kWideMaxRows;
    u.wide = !u.pair && left > kBM;
    u.rows = u.pair ? min(left, 2 * kBM) : left;
  }
  return u;
}

// Whether a single tile runs with swapped operands: in the decode geometry,
// and for a gathered A of at most kSwapMaxRows rows (a full tile would
// gather 128 rows per k-block).  A tiled single tile always runs unswapped:
// its four N=256 MMAs (~512 cycles a k-block) cost less than a swapped
// tile's eight (~570-780 cycles measured), whatever its row count.
template <class G>
__device__ __forceinline__ bool single_swapped(int rows, bool gathered) {
  return G::kSmallOnly || (gathered && rows <= kSwapMaxRows);
}

// A bytes of one single tile in a stage: a full tile's 128-row box, the
// tiled box of the decode geometry, or a swapped tile's rows rounded up to 16.
template <class G>
__device__ __forceinline__ uint32_t tile_a_bytes(int rows, bool gathered) {
  if (!single_swapped<G>(rows, gathered)) return static_cast<uint32_t>(kBM * kBK * 2);
  if (G::kSmallOnly && !gathered) return static_cast<uint32_t>(G::kABytes);
  return static_cast<uint32_t>(((rows + 15) & ~15) * kBK * 2);
}

// A bytes of a unit's stage: the first part (a0) and, for a pair, the second
// tile's (a1; 0 otherwise).  A wide unit's rows form one part.
template <class G>
__device__ __forceinline__ void unit_a_bytes(const Unit& u, bool gathered, uint32_t& a0,
                                             uint32_t& a1) {
  if (u.pair) {
    a0 = a1 = static_cast<uint32_t>(kBM * kBK * 2);
    return;
  }
  a1 = 0u;
  a0 = u.wide ? static_cast<uint32_t>(((u.rows + 15) & ~15) * kBK * 2)
              : tile_a_bytes<G>(u.rows, gathered);
}

// Position in the stage ring: stage j uses record j % kRecs (barrier parity
// (j / kRecs) & 1) and starts at byte `off` of the ring.  Producer and MMA
// issuer walk the same stage sequence and each keeps its own copy.
template <class G>
struct RingPos {
  uint32_t j = 0;    // stages so far
  uint32_t off = 0;  // ring offset of stage j
  __device__ __forceinline__ int rec() const { return static_cast<int>(j % G::kRecs); }
  __device__ __forceinline__ uint32_t parity() const { return (j / G::kRecs) & 1u; }
  __device__ __forceinline__ void advance(uint32_t span) {
    ++j;
    off += span;
    if (off >= static_cast<uint32_t>(G::kRingBytes)) off -= G::kRingBytes;
  }
  // Ring offsets of the current stage's parts: the weight boxes (b0, 32 KB),
  // the first tile's A rows (a0, a0_bytes) and, for a paired unit, the
  // second tile's (a1, a1_bytes; a1_bytes == 0 otherwise).  A part that
  // would cross the ring end starts at 0; when the weight boxes do not fit
  // before the end but the first A part does, that part goes first so the
  // tail is used.  Returns the stage's span: its bytes plus any skipped tail.
  __device__ __forceinline__ uint32_t layout(uint32_t a0_bytes, uint32_t a1_bytes, uint32_t& b0,
                                             uint32_t& a0, uint32_t& a1) const {
    constexpr uint32_t R = static_cast<uint32_t>(G::kRingBytes);
    uint32_t cur = off, span = 0;
    auto place = [&](uint32_t size) -> uint32_t {
      if (cur + size > R) {
        span += R - cur;
        cur = 0;
      }
      const uint32_t at = cur;
      cur += size;
      span += size;
      if (cur == R) cur = 0;
      return at;
    };
    if (off + 2u * kBoxBytes > R && off + a0_bytes <= R) {
      a0 = place(a0_bytes);
      b0 = place(2u * kBoxBytes);
    } else {
      b0 = place(2u * kBoxBytes);
      a0 = place(a0_bytes);
    }
    a1 = a1_bytes != 0u ? place(a1_bytes) : 0u;
    return span;
  }
};

template <int MODE, class G>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_a16, const __grid_constant__ Params p) {
  constexpr bool SWIGLU = MODE == kModeSwiglu;
  constexpr bool COMBINE = MODE == kModeCombine;
  using Smem = SmemT<G>;
  constexpr int kRecs = G::kRecs;
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = p.num_experts;
  // Pairing reads the second m-tile through the tiled A map, so a gathered A
  // keeps one m-tile per unit.
  const bool pairs = G::kPairs && p.gather_idx == nullptr;

  // ---- unit table: cum[e] = sum over e' < e of m-units(e') * n_tiles -------
  // Offsets are clamped to [0, rows]; an expert whose end precedes its start
  // has no tiles, so every stored row stays inside D.
  for (int i = tid; i <= E; i += kThreads) {
    int v = __ldg(p.offsets + i);
    v = v < 0 ? 0 : (v > p.rows ? p.rows : v);
    s.offs[i] = v;
  }
  if (tid == 0) s.abort = 0;
  __syncthreads();
  {
    const int per = (E + kThreads - 1) / kThreads;
    const int eb = tid * per;
    const int ee = min(E, eb + per);
    int local = 0;
    for (int e = eb; e < ee; ++e) local += munits_of(s, e, pairs) * p.n_tiles;
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) s.warp_tot[warp] = incl;
    __syncthreads();
    int run = incl - local;
    for (int w = 0; w < warp; ++w) run += s.warp_tot[w];
    for (int e = eb; e < ee; ++e) {
      s.cum[e] = run;
      run += munits_of(s, e, pairs) * p.n_tiles;
    }
    if (eb < E && ee == E) s.cum[E] = run;
  }

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < kRecs; ++i) {
      mbar_init(&s.full_bar[i], 1);
      mbar_init(&s.empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full_bar[i], 1);
      mbar_init(&s.acc_empty_bar[i], kEpiWarps);
    }
    mbar_init(&s.mma_done_bar, 1);
    for (int i = 0; i < kUnitQ; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1 + kEpiWarps);  // MMA lane + every epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a16)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = s.tmem_base;
  const int total = s.cum[E];
  volatile int32_t* abort = &s.abort;

  if (warp == 0) {
    // ===================== TMA producer =====================
    if (lane == 0) {
      // Weights: normal eviction, so the other m-units of an expert, which
      // read the same weight tile moments later, find it in L2 (an
      // evict-first hint made them re-read it from HBM: 4-9 % slower).
      const uint64_t pol_w = policy_evict_normal();
      const uint64_t pol_a = policy_evict_last();
      RingPos<G> pos;
      uint32_t j_free = 0;        // stages before this one have been released
      uint32_t held = 0;          // ring bytes of stages j_free .. pos.j - 1
      bool ok = true;
      int qslot = 0;
      uint32_t qphase = 0;
      // Reserves `span` bytes of ring for the next stage: releases the
      // oldest stages (waiting for the MMA to free them) until the stage and
      // its record are free, then arms its full barrier for `tx` bytes.
      // False on abort.
      auto reserve = [&](uint32_t span, uint32_t tx) -> bool {
        while (pos.j - j_free >= static_cast<uint32_t>(kRecs) ||
               held + span > static_cast<uint32_t>(G::kRingBytes)) {
          const int r = static_cast<int>(j_free % kRecs);
          if (!mbar_wait(&s.empty_bar[r], (j_free / kRecs) & 1u, abort, kDevErrGemmProducerWait,
                         true))
            return false;
          held -= s.span[r];
          ++j_free;
        }
        s.span[pos.rec()] = span;
        held += span;
        mbar_expect_tx(&s.full_bar[pos.rec()], tx);
        return true;
      };
      for (int i = 0; ok; ++i) {
        if (!mbar_wait(&s.q_empty[qslot], qphase ^ 1u, abort, kDevErrGemmProducerWait, true)) {
          ok = false;
          break;
        }
        int unit = p.counter ? atomicAdd(p.counter, 1) : blockIdx.x + i * static_cast<int>(gridDim.x);
        if (unit >= total) unit = -1;
        s.unit_q[qslot] = unit;
        mbar_arrive(&s.q_full[qslot]);
        if (++qslot == kUnitQ) {
          qslot = 0;
          qphase ^= 1u;
        }
        if (unit < 0) break;
        const Unit u = decode_unit(s, E, unit, pairs);
        const int row0 = s.offs[u.e] + u.t0 * kBM;
        const int brow = u.e * p.b_rows + u.n * p.b_tile_rows;
        // A swapped tile needs only its rows rounded up to 16: tiled A loads
        // a small tile's rows as that many 16-row boxes, and a wide unit's
        // as one 128-row box followed by 16-row boxes for the rest.
        const bool gathered = p.gather_idx != nullptr;
        uint32_t a0_bytes, a1_bytes;
        unit_a_bytes<G>(u, gathered, a0_bytes, a1_bytes);
        // A wide unit's rows: one 128-row box, then 16-row boxes.
        const int n16 = u.wide ? static_cast<int>((a0_bytes - kBM * kBK * 2) / kA16Bytes) : 0;
        // Gathered A: the MMA reads 128 rows (or, for a swapped small tile,
        // its rows rounded up to 16); rows past the expert repeat its first
        // row (their results are discarded).
        int nload = 0;
        if (p.gather_idx != nullptr) {
          const int valid = min(kBM, s.offs[u.e + 1] - row0);
          nload = (G::kSmallOnly || valid <= kSwapMaxRows) ? ((valid + 15) & ~15) : kBM;
          for (int r = 0; r < nload; ++r)
            s.arow[r] = __ldg(p.gather_idx + row0 + (r < valid ? r : 0)) / p.gather_k;
        }
        const uint32_t tx = a0_bytes + a1_bytes + 2u * kBoxBytes;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          uint32_t oa0, oa1, ob0;
          const uint32_t span = pos.layout(a0_bytes, a1_bytes, ob0, oa0, oa1);
          if (!reserve(span, tx)) {
            ok = false;
            break;
          }
          uint64_t* full = &s.full_bar[pos.rec()];
          uint8_t* a0 = s.ring + oa0;
          if (p.gather_idx != nullptr) {
            for (int r = 0; r < nload; r += 4)
              tma_gather4(a0 + r * kBK * 2, &tmap_a, full, kb * kBK, s.arow[r], s.arow[r + 1],
                          s.arow[r + 2], s.arow[r + 3], pol_a);
          } else {
            tma_load_2d(a0, &tmap_a, full, kb * kBK, row0, pol_a);
            for (int b = 0; b < n16; ++b)
              tma_load_2d(a0 + kBM * kBK * 2 + b * kA16Bytes, &tmap_a16, full, kb * kBK,
                          row0 + kBM + 16 * b, pol_a);
          }
          if (u.pair) tma_load_2d(s.ring + oa1, &tmap_a, full, kb * kBK, row0 + kBM, pol_a);
          tma_load_2d(s.ring + ob0, &tmap_b, full, kb * kBK, brow, pol_w);
          tma_load_2d(s.ring + ob0 + kBoxBytes, &tmap_b, full, kb * kBK, brow + p.b_second, pol_w);
          pos.advance(span);
        }
      }
      if (!ok) {  // let every issued load land before the CTA can exit
        for (uint32_t j = j_free; j < pos.j; ++j)
          mbar_wait(&s.full_bar[j % kRecs], (j / kRecs) & 1u, abort, kDevErrGemmProducerWait,
                    false);
      }
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    if (lane == 0) {
      RingPos<G> pos;
      uint32_t ac = 0;  // accumulators taken so far (slot ac & 1, lap parity (ac >> 1) & 1)
      bool ok = true;
      int qslot = 0;
      uint32_t qphase = 0;
      const uint32_t ring = smem_u32(s.ring);
      while (ok) {
        if (!mbar_wait(&s.q_full[qslot], qphase, abort, kDevErrGemmMmaWait, true)) break;
        const int unit = s.unit_q[qslot];
        mbar_arrive(&s.q_empty[qslot]);
        if (++qslot == kUnitQ) {
          qslot = 0;
          qphase ^= 1u;
        }
        if (unit < 0) break;
        const Unit u = decode_unit(s, E, unit, pairs);
        const bool two = u.pair || u.wide;  // the unit takes both accumulators
        const bool gathered = p.gather_idx != nullptr;
        const bool swapped = u.wide || (!u.pair && single_swapped<G>(u.rows, gathered));
        const int nn = (u.rows + 15) & ~15;
        const uint32_t sw_idesc = swap_idesc(nn);
        const int acc0 = static_cast<int>(ac & 1u);
        const int acc1 = static_cast<int>((ac + 1) & 1u);
        if (!mbar_wait(&s.acc_empty_bar[acc0], ((ac >> 1) & 1u) ^ 1u, abort, kDevErrGemmMmaWait,
                       true) ||
            (two && !mbar_wait(&s.acc_empty_bar[acc1], (((ac + 1) >> 1) & 1u) ^ 1u, abort,
                               kDevErrGemmMmaWait, true))) {
          ok = false;
          break;
        }
        ac += two ? 2u : 1u;
        tc_fence_after();
        // A wide tile spans TMEM columns 0 .. 2nn-1 (both accumulators).
        const uint32_t d0 = tmem_base + (u.wide ? 0u : static_cast<uint32_t>(acc0 * kBN));
        const uint32_t d1 = tmem_base + static_cast<uint32_t>(acc1 * kBN);
        uint32_t a0_bytes, a1_bytes;
        unit_a_bytes<G>(u, gathered, a0_bytes, a1_bytes);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          const int rec = pos.rec();
          if (!mbar_wait(&s.full_bar[rec], pos.parity(), abort, kDevErrGemmMmaWait, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t oa0, oa1, ob0;
          const uint32_t span = pos.layout(a0_bytes, a1_bytes, ob0, oa0, oa1);
          const uint32_t a0_addr = ring + oa0;
          const uint32_t a1_addr = ring + oa1;
          const uint32_t b0_addr = ring + ob0;
          const uint32_t b1_addr = b0_addr + kBoxBytes;
          if (swapped) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t tok = smem_desc_sw128(a0_addr + kk * 32);
              const uint32_t acc_in = (kb | kk) != 0 ? 1u : 0u;
              umma_bf16(d0, smem_desc_sw128(b0_addr + kk * 32), tok, sw_idesc, acc_in);
              umma_bf16(d0 + static_cast<uint32_t>(nn), smem_desc_sw128(b1_addr + kk * 32), tok,
                        sw_idesc, acc_in);
            }
          } else {
            // One N=256 MMA per K step against both (adjacent) weight boxes;
            // all K steps of one accumulator before the other's.
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_bf16(d0, smem_desc_sw128(a0_addr + kk * 32), smem_desc_sw128(b0_addr + kk * 32),
                        kIdesc, (kb | kk) != 0 ? 1u : 0u);
            if (u.pair) {
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                umma_bf16(d1, smem_desc_sw128(a1_addr + kk * 32),
                          smem_desc_sw128(b0_addr + kk * 32), kIdesc, (kb | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&s.empty_bar[rec]);
          pos.advance(span);
        }
        if (ok) {
          umma_commit(&s.acc_full_bar[acc0]);
          if (two) umma_commit(&s.acc_full_bar[acc1]);
        }
      }
      // Outstanding MMAs read shared memory and write TMEM: finish them first.
      umma_commit(&s.mma_done_bar);
      mbar_wait(&s.mma_done_bar, 0, abort, kDevErrGemmMmaWait, false);
    }
  } else {
    // ===================== epilogue (warps 2..9) =====================
    // Two groups of four warps split every accumulator's columns, so one
    // tile drains in half the time and a paired unit's two tiles in the
    // time of one.
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int grp = (warp - 2) >> 2;  // column half this warp drains
    int qslot = 0;
    uint32_t qphase = 0;
    uint32_t ac = 0;
    bool running = true;
    while (running) {
      if (!mbar_wait(&s.q_full[qslot], qphase, abort, kDevErrGemmEpilogueWait, true)) break;
      const int unit = s.unit_q[qslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.q_empty[qslot]);
      if (++qslot == kUnitQ) {
        qslot = 0;
        qphase ^= 1u;
      }
      if (unit < 0) break;
      const Unit u = decode_unit(s, E, unit, pairs);
      const int e = u.e;
      // A wide tile fills both accumulators: wait for the second one too.
      if (u.wide && !mbar_wait(&s.acc_full_bar[(ac + 1) & 1u], ((ac + 1) >> 1) & 1u, abort,
                               kDevErrGemmEpilogueWait, true))
        break;
      for (int ti = 0; ti < (u.pair ? 2 : 1); ++ti, ++ac) {
        const int acc = static_cast<int>(ac & 1u);
        if (!mbar_wait(&s.acc_full_bar[acc], (ac >> 1) & 1u, abort, kDevErrGemmEpilogueWait,
                       true)) {
          running = false;
          break;
        }
        tc_fence_after();
        const int m = u.t0 + ti;
        const int rows_here = u.pair ? min(kBM, u.rows - ti * kBM) : u.rows;
        const bool swapped = u.wide || (!u.pair && single_swapped<G>(rows_here, p.gather_idx != nullptr));
        const int row0 = s.offs[e] + m * kBM;
        const int r = row0 + q * 32 + lane;
        const bool valid = r < s.offs[e + 1];
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               (u.wide ? 0u : static_cast<uint32_t>(acc * kBN));
        const int col0 = u.n * p.out_tile_cols;
        const int cols_here = min(p.out_tile_cols, p.n_out - col0);
        __nv_bfloat16* drow = nullptr;
        float wrow = 1.0f;
        bool live = valid;
        if (COMBINE) {
          if (valid) {
            const int32_t rk = __ldg(p.dst_rank + r), dr = __ldg(p.dst_row + r);
            live = rk >= 0 && rk < p.world && dr >= 0 && dr < p.back_rows;
            if (live)
              drow = reinterpret_cast<__nv_bfloat16*>(p.peers.base[rk] + p.back_offset) +
                     static_cast<int64_t>(dr) * p.ldd + col0;
            wrow = __ldg(p.dst_w + r);
          }
        } else {
          drow = p.D + static_cast<int64_t>(valid ? r : 0) * p.ldd + col0;
        }
        if (swapped) {
          // Transposed accumulator: this thread's TMEM lane is weight row
          // w = 32q + lane of each box, columns [0, nn) hold box 0 for the
          // tile's tokens and [nn, 2nn) box 1.
          const int nn = (rows_here + 15) & ~15;
          const int w = q * 32 + lane;
          __nv_bfloat16* dcol = COMBINE ? nullptr : p.D + static_cast<int64_t>(row0) * p.ldd + col0;
#pragma unroll 1
          for (int t0 = grp * 16; t0 < nn; t0 += 32) {
            uint32_t v0[16], v1[16];
            tmem_ld16(tbase + t0, v0);
            tmem_ld16(tbase + nn + t0, v1);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int t = t0 + i;
              if (t >= rows_here) break;
              if (COMBINE) {
                const int pr = row0 + t;
                const int32_t rk = __ldg(p.dst_rank + pr), dr = __ldg(p.dst_row + pr);
                if (rk < 0 || rk >= p.world || dr < 0 || dr >= p.back_rows) continue;
                __nv_bfloat16* dst =
                    reinterpret_cast<__nv_bfloat16*>(p.peers.base[rk] + p.back_offset) +
                    static_cast<int64_t>(dr) * p.ldd + col0;
                const float wt = __ldg(p.dst_w + pr);
                if (w < cols_here)
                  dst[w] = __float2bfloat16_rn(__fmul_rn(wt, round_bf16(__uint_as_float(v0[i]))));
                if (kBoxRows + w < cols_here)
                  dst[kBoxRows + w] =
                      __float2bfloat16_rn(__fmul_rn(wt, round_bf16(__uint_as_float(v1[i]))));
                continue;
              }
              __nv_bfloat16* dst = dcol + static_cast<int64_t>(t) * p.ldd;
              if (SWIGLU) {
                if (w < cols_here)
                  dst[w] = __float2bfloat16_rn(swiglu_f32(round_bf16(__uint_as_float(v0[i])),
                                                          round_bf16(__uint_as_float(v1[i])),
                                                          p.swiglu_limit));
              } else {
                if (w < cols_here) dst[w] = __float2bfloat16_rn(__uint_as_float(v0[i]));
                if (kBoxRows + w < cols_here)
                  dst[kBoxRows + w] = __float2bfloat16_rn(__uint_as_float(v1[i]));
              }
            }
          }
        } else if (SWIGLU) {
#pragma unroll 1
          for (int c = grp * (kBoxRows / 2); c < (grp + 1) * (kBoxRows / 2); c += 32) {
            uint32_t g[32], u[32];
            tmem_ld32(tbase + c, g);
            tmem_ld32(tbase + kBoxRows + c, u);
            tmem_ld_wait();
            if (valid && c < cols_here) {
              uint32_t packed[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float h0 = swiglu_f32(round_bf16(__uint_as_float(g[2 * j])),
                                            round_bf16(__uint_as_float(u[2 * j])), p.swiglu_limit);
                const float h1 = swiglu_f32(round_bf16(__uint_as_float(g[2 * j + 1])),
                                            round_bf16(__uint_as_float(u[2 * j + 1])),
                                            p.swiglu_limit);
                packed[j] = pack_bf16x2(h0, h1);
              }
              uint4* dst = reinterpret_cast<uint4*>(drow + c);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                                    packed[4 * j + 3]);
            }
          }
        } else {
#pragma unroll 1
          for (int c = grp * (kBN / 2); c < (grp + 1) * (kBN / 2); c += 32) {
            uint32_t v[32];
            tmem_ld32(tbase + c, v);
            tmem_ld_wait();
            if (live && c < cols_here) {
              uint32_t packed[16];
              if (COMBINE) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  packed[j] = pack_bf16x2(__fmul_rn(wrow, round_bf16(__uint_as_float(v[2 * j]))),
                                          __fmul_rn(wrow, round_bf16(__uint_as_float(v[2 * j + 1]))));
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  packed[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
              }
              uint4* dst = reinterpret_cast<uint4*>(drow + c);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                                    packed[4 * j + 3]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.acc_empty_bar[acc]);
          if (u.wide) mbar_arrive(&s.acc_empty_bar[(ac + 1) & 1u]);
        }
        if (u.wide) ++ac;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
  if (COMBINE) grid_release_to_peers(p.peers, p.world, p.me, kCtrlCombineFlags, p.done, p.epoch);
}

// Publishes the combine epoch when a rank has no rows to multiply.
__global__ void combine_release_kernel(const __grid_constant__ Params p) {
  grid_release_to_peers(p.peers, p.world, p.me, kCtrlCombineFlags, p.done, p.epoch);
}

// ---- host side -----------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 map over a [outer, inner] row-major tensor, box [box_rows, kBK],
// 128-byte swizzle, zero fill out of bounds.
lsek_status make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint32_t box_rows = kBoxRows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(LSEK_ERR_CUDA, "grouped_gemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LSEK_ERR_CUDA, "grouped_gemm: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return LSEK_OK;
}

// Gathered A (gather_idx non-null): A is the [a_rows, K] token tensor and row r
// of the permuted A is A[gather_idx[r] / gather_k]; `rows` counts permuted rows.
struct Gather {
  const int32_t* idx = nullptr;
  int k = 1;
  int a_rows = 0;
};

template <int MODE, class G>
lsek_status launch_geom(void* D, const void* A, const void* B, const int32_t* offsets, int E,
                        int rows, int n_out, int b_rows, int K, float limit, int32_t* counter,
                        cudaStream_t st, const Params* combine, const Gather& gather) {
  constexpr bool SWIGLU = MODE == kModeSwiglu;
  static PerDeviceOnce attrs;
  const cudaError_t ae = once_per_device(attrs, [] {
    return cudaFuncSetAttribute(grouped_gemm_kernel<MODE, G>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem_bytes<G>()));
  });
  if (ae != cudaSuccess) return fail(LSEK_ERR_CUDA, "grouped_gemm: %s", cudaGetErrorString(ae));
  CUtensorMap ma, mb;
  lsek_status s =
      gather.idx != nullptr
          ? make_map(&ma, A, static_cast<uint64_t>(K), static_cast<uint64_t>(gather.a_rows), 1u)
          : make_map(&ma, A, static_cast<uint64_t>(K), static_cast<uint64_t>(rows),
                     static_cast<uint32_t>(G::kARows));
  if (s != LSEK_OK) return s;
  s = make_map(&mb, B, static_cast<uint64_t>(K), static_cast<uint64_t>(E) * b_rows);
  if (s != LSEK_OK) return s;
  // 16-row boxes for tiles that run with swapped operands (tiled A only).
  CUtensorMap ma16 = ma;
  if (gather.idx == nullptr && !G::kSmallOnly) {
    s = make_map(&ma16, A, static_cast<uint64_t>(K), static_cast<uint64_t>(rows), 16u);
    if (s != LSEK_OK) return s;
  }
  Params p;
  if (combine != nullptr) p = *combine;
  p.offsets = offsets;
  p.num_experts = E;
  p.rows = rows;
  p.num_kb = static_cast<int>(ceil_div(K, kBK));
  p.D = static_cast<__nv_bfloat16*>(D);
  p.ldd = n_out;
  p.n_out = n_out;
  p.b_rows = b_rows;
  p.swiglu_limit = limit;
  p.counter = counter;
  p.gather_idx = gather.idx;
  p.gather_k = gather.k;
  if (counter != nullptr) LSEK_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(int32_t), st));
  if (SWIGLU) {
    p.n_tiles = static_cast<int>(ceil_div(n_out, kBoxRows));
    p.b_tile_rows = kBoxRows;
    p.b_second = n_out;  // up rows start at I
    p.out_tile_cols = kBoxRows;
  } else {
    p.n_tiles = static_cast<int>(ceil_div(n_out, kBN));
    p.b_tile_rows = kBN;
    p.b_second = kBoxRows;
    p.out_tile_cols = kBN;
  }
  const int64_t max_units = (ceil_div(rows, kBM) + E) * static_cast<int64_t>(p.n_tiles);
  const int grid = static_cast<int>(max_units < num_sms() ? max_units : num_sms());
  if (MODE == kModeCombine) LSEK_CUDA_TRY(cudaMemsetAsync(p.done, 0, sizeof(uint32_t), st));
  grouped_gemm_kernel<MODE, G><<<grid, kThreads, smem_bytes<G>(), st>>>(ma, mb, ma16, p);
  return check_launch(SWIGLU ? "grouped_gemm_swiglu_bf16"
                             : (MODE == kModeCombine ? "ep_down_gemm_combine" : "grouped_gemm_bf16"));
}

// max_rows_per_expert: an upper bound on the rows of any expert (or -1 if
// unknown); at most kDecodeMaxRows selects the decode geometry.
template <int MODE>
lsek_status launch(void* D, const void* A, const void* B, const int32_t* offsets, int E, int rows,
                   int n_out, int b_rows, int K, float limit, int32_t* counter, cudaStream_t st,
                   const Params* combine = nullptr, int max_rows_per_expert = -1,
                   const Gather& gather = Gather()) {
  const int bound = rows <= kDecodeMaxRows ? rows : max_rows_per_expert;
  if (bound >= 0 && bound <= kDecodeMaxRows && E <= GeomDecode::kMaxE)
    return launch_geom<MODE, GeomDecode>(D, A, B, offsets, E, rows, n_out, b_rows, K, limit,
                                         counter, st, combine, gather);
  if (E <= GeomFull::kMaxE)
    return launch_geom<MODE, GeomFull>(D, A, B, offsets, E, rows, n_out, b_rows, K, limit,
                                       counter, st, combine, gather);
  return launch_geom<MODE, GeomFullWide>(D, A, B, offsets, E, rows, n_out, b_rows, K, limit,
                                         counter, st, combine, gather);
}

lsek_status validate(const char* name, const void* D, const void* A, const void* B,
                     const int32_t* offsets, int E, int rows, int n_out, int K) {
  LSEK_REQUIRE(E >= 1, "%s: num_experts must be >= 1", name);
  LSEK_REQUIRE(rows >= 0 && n_out >= 0 && K >= 0, "%s: sizes must be >= 0", name);
  if (E > kMaxExperts) return fail(LSEK_ERR_UNSUPPORTED, "%s: num_experts must be <= %d", name, kMaxExperts);
  LSEK_REQUIRE(K % 8 == 0, "%s: K must be a multiple of 8 (16-byte rows), got %d", name, K);
  LSEK_REQUIRE(n_out % 32 == 0, "%s: output width must be a multiple of 32, got %d", name, n_out);
  if (rows == 0 || n_out == 0) return LSEK_OK;  // nothing to compute (pointers may be NULL)
  LSEK_REQUIRE(K > 0, "%s: K must be > 0 when there are rows to compute", name);
  LSEK_REQUIRE(offsets != nullptr, "%s: expert_offsets is NULL", name);
  LSEK_REQUIRE(D && A && B, "%s: NULL tensor pointer", name);
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(B) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(D) % 16 == 0,
               "%s: A, B and D must be 16-byte aligned", name);
  return LSEK_OK;
}

}  // namespace gemm

// Used by the layer forward.  `counter` is one zero-able int32 of device
// scratch for dynamic unit scheduling, or null for the static stride;
// `max_rows_per_expert` an upper bound on any expert's rows, or -1.
lsek_status grouped_gemm_plain(void* D, const void* A, const void* B, const int32_t* offsets, int E,
                               int rows, int N, int K, int32_t* counter, cudaStream_t st,
                               int max_rows_per_expert) {
  if (rows == 0 || N == 0) return LSEK_OK;
  return gemm::launch<gemm::kModePlain>(D, A, B, offsets, E, rows, N, N, K, 0.0f, counter, st,
                                        nullptr, max_rows_per_expert);
}
lsek_status grouped_gemm_swiglu(void* H, const void* A, const void* Wgu, const int32_t* offsets,
                                int E, int rows, int I, int K, float limit, int32_t* counter,
                                cudaStream_t st, int max_rows_per_expert) {
  if (rows == 0 || I == 0) return LSEK_OK;
  return gemm::launch<gemm::kModeSwiglu>(H, A, Wgu, offsets, E, rows, I, 2 * I, K, limit, counter,
                                         st, nullptr, max_rows_per_expert);
}
// The same with the permute folded into the A load: permuted row r is
// hidden[permuted_idx[r] / topk] (hidden has num_tokens rows).
lsek_status grouped_gemm_swiglu_gather(void* H, const void* hidden, const void* Wgu,
                                       const int32_t* offsets, const int32_t* permuted_idx,
                                       int num_tokens, int topk, int E, int rows, int I, int K,
                                       float limit, int32_t* counter, cudaStream_t st,
                                       int max_rows_per_expert) {
  if (rows == 0 || I == 0) return LSEK_OK;
  gemm::Gather g;
  g.idx = permuted_idx;
  g.k = topk;
  g.a_rows = num_tokens;
  return gemm::launch<gemm::kModeSwiglu>(H, hidden, Wgu, offsets, E, rows, I, 2 * I, K, limit,
                                         counter, st, nullptr, max_rows_per_expert, g);
}

}  // namespace lsek

extern "C" lsek_status lsek_device_error(int32_t* code, void* stream) {
  using namespace lsek;
  LSEK_REQUIRE(code != nullptr, "lsek_device_error: code is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LSEK_CUDA_TRY(cudaStreamSynchronize(st));
  int32_t zero = 0;
  LSEK_CUDA_TRY(cudaMemcpyFromSymbol(code, g_device_error, sizeof(int32_t)));
  LSEK_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int32_t)));
  int32_t ep_code = 0;
  const lsek_status s = ep_take_device_error(&ep_code);
  if (s != LSEK_OK) return s;
  if (*code == 0) *code = ep_code;
  return LSEK_OK;
}

static int32_t* gemm_counter(void* workspace, size_t workspace_bytes) {
  return (workspace != nullptr && workspace_bytes >= sizeof(int32_t)) ? static_cast<int32_t*>(workspace)
                                                                      : nullptr;
}

extern "C" lsek_status lsek_grouped_gemm_bf16(void* D, const void* A, const void* B,
                                              const int32_t* expert_offsets, int32_t num_experts,
                                              int32_t rows, int32_t N, int32_t K, void* workspace,
                                              size_t workspace_bytes, void* stream) {
  using namespace lsek;
  lsek_status s = gemm::validate("grouped_gemm_bf16", D, A, B, expert_offsets, num_experts, rows, N, K);
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(static_cast<int64_t>(num_experts) * N < (1ll << 31),
               "grouped_gemm_bf16: num_experts * N must fit in int32");
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 4 == 0,
               "grouped_gemm_bf16: workspace must be 4-byte aligned");
  return grouped_gemm_plain(D, A, B, expert_offsets, num_experts, rows, N, K,
                            gemm_counter(workspace, workspace_bytes),
                            static_cast<cudaStream_t>(stream), -1);
}

extern "C" lsek_status lsek_grouped_gemm_swiglu_bf16(void* Hout, const void* A, const void* W_gu,
                                                     const int32_t* expert_offsets,
                                                     int32_t num_experts, int32_t rows, int32_t I,
                                                     int32_t K, float swiglu_limit, void* workspace,
                                                     size_t workspace_bytes, void* stream) {
  using namespace lsek;
  lsek_status s =
      gemm::validate("grouped_gemm_swiglu_bf16", Hout, A, W_gu, expert_offsets, num_experts, rows, I, K);
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(swiglu_limit >= 0.0f, "grouped_gemm_swiglu_bf16: swiglu_limit must be >= 0");
  LSEK_REQUIRE(static_cast<int64_t>(num_experts) * 2 * I < (1ll << 31),
               "grouped_gemm_swiglu_bf16: num_experts * 2I must fit in int32");
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 4 == 0,
               "grouped_gemm_swiglu_bf16: workspace must be 4-byte aligned");
  return grouped_gemm_swiglu(Hout, A, W_gu, expert_offsets, num_experts, rows, I, K, swiglu_limit,
                             gemm_counter(workspace, workspace_bytes),
                             static_cast<cudaStream_t>(stream), -1);
}

extern "C" lsek_status lsek_ep_down_gemm_combine(lsek_ep_domain* h, const void* hact,
                                                 const void* w_down, const int32_t* expert_offsets,
                                                 int32_t local_experts, int32_t rows, int32_t inter,
                                                 const int32_t* dst_rank, const int32_t* dst_row,
                                                 const float* dst_w, uint32_t epoch,
                                                 void* workspace, size_t workspace_bytes,
                                                 void* stream) {
  using namespace lsek;
  LSEK_REQUIRE(h != nullptr, "ep_down_gemm_combine: domain is NULL");
  const EpDomain& d = h->d;
  for (int g = 0; g < d.world; ++g)
    LSEK_REQUIRE(d.peer[g] != nullptr, "ep_down_gemm_combine: rank %d has not been imported", g);
  const int H = static_cast<int>(d.H);
  lsek_status s = gemm::validate("ep_down_gemm_combine", d.local, hact, w_down, expert_offsets,
                                 local_experts, rows, H, inter);
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(static_cast<int64_t>(local_experts) * H < (1ll << 31),
               "ep_down_gemm_combine: local_experts * hidden must fit in int32");
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 4 == 0,
               "ep_down_gemm_combine: workspace must be 4-byte aligned");
  gemm::Params cp{};
  cp.dst_rank = dst_rank;
  cp.dst_row = dst_row;
  cp.dst_w = dst_w;
  cp.peers = peer_table(d);
  cp.back_offset = d.lay.back;
  cp.back_rows = d.lay.cap_slots;
  cp.world = d.world;
  cp.me = d.rank;
  cp.done = reinterpret_cast<uint32_t*>(d.local + kCtrlGemmDone);
  cp.epoch = epoch;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0 || inter == 0) {
    LSEK_CUDA_TRY(cudaMemsetAsync(cp.done, 0, sizeof(uint32_t), st));
    gemm::combine_release_kernel<<<1, 32, 0, st>>>(cp);
    return check_launch("ep_down_gemm_combine(release)");
  }
  LSEK_REQUIRE(dst_rank && dst_row && dst_w, "ep_down_gemm_combine: NULL plan pointer");
  return gemm::launch<gemm::kModeCombine>(nullptr, hact, w_down, expert_offsets, local_experts,
                                          rows, H, H, inter, 0.0f,
                                          gemm_counter(workspace, workspace_bytes), st, &cp);
}
