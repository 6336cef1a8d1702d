// Device code of the sm_100a BF16 GEMM (included once, by gemm_sm100.cu, which holds the
// host side: planning, launch and the C ABI).
//
// The GEMM: C[m,n] = A[m,k] · B[k,n], all row-major, BF16 inputs, FP32 accumulation,
// BF16 (round-to-nearest-even) output.  This is the B200 replacement for the reference's
// kernel library src/kernels/bf16_gemm_v1.cu (dispatcher :2098-2180): one persistent,
// warp-specialised kernel family covers every shape on the tensor cores instead of the
// reference's hero-shape region split plus scalar fallback kernel (layouts TMA cannot describe
// reach it through padded copies made on the host side).
//
// Kernel structure (one CTA per SM, 384 threads, optionally a CTA pair per tile):
//   warp 0      TMA producer: per K block, one A box of tile_rows x 64 (K-major; 128 rows, or
//               fewer for short 1-CTA tiles and skinny A) and BN_CTA/64 boxes of
//               64x64 B (N-major) into a STAGES-deep 128-byte-swizzled shared-memory ring
//               (full/empty mbarriers).  Out-of-bounds rows, columns and K are zero-filled.
//               It also tells the epilogue when a K chunk's accumulator is complete: the
//               ring stage holding the chunk's last K block has been freed by the MMAs.
//   warp 1      allocates TMEM and, from one lane of the leader CTA, issues tcgen05.mma
//               (A K-major, B MN-major straight from the row-major B: no transpose pass).
//               With cta_group::2 the CTA pair computes a 256 x (2·BN_CTA) tile: each CTA
//               loads its own 128 A rows and its own BN_CTA-column half of B, so each SM
//               feeds half the B bytes it would for a 1-CTA tile of the same width.
//   warps 4..11 epilogue: two-level accumulation.  The MMA writes the partial product of
//               each K chunk (at most 1856 wide) into one of two TMEM buffers; the epilogue adds
//               it into FP32 registers (IEEE round-to-nearest adds) and releases the buffer, and
//               after the last chunk rounds to BF16 and stores the rows/columns inside C.
//
// Schedules (the unit functions below): whole tiles dealt round-robin to persistent clusters;
// K split into (tile, chunk) units whose FP32 partials a reduce kernel sums; or stream-K, whole
// tiles plus the leftover tiles' chunks spread over all clusters and finished from the pieces'
// FP32 results.  All three perform the same FP32 adds in the same order.
//
// Why two-level: the tensor core's FP32 accumulation over K = 7232 in one TMEM accumulator
// loses enough low bits that near-zero outputs miss the |err| <= 2^-7|ref| + 1e-2·sqrt(K)/K
// bound of this build (cuBLAS on the same part gives the same bits); summing chunk partials
// in FP32 keeps the worst element inside the bound.
//
// Determinism: every variant (1-CTA or CTA pair, any tile width) computes every output as
// the same sequence of K=16 MMAs per K chunk and the same FP32 chunk sum, so a column
// slab of C is bit-identical to the same columns of a full-width run (the N-shard contract).
//
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel records which wait gave
// up in a device watchdog word, drains in-flight copies and MMAs with bounded waits, frees
// TMEM and exits, so a lost arrival yields an error status rather than a hung GPU.

#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <type_traits>

#include "sm100_ptx.cuh"

namespace mo {
namespace {

constexpr int kRowsPerCta = 128;    // UMMA M per CTA (TMEM lanes)
constexpr int kBlockK = 64;         // one 128-byte swizzle atom of BF16 along K
constexpr int kUmmaK = 16;          // K of one kind::f16 tcgen05.mma
// Longest TMEM partial, in K blocks, for K <= 7424: 29 x 64 = 1856 K elements (the hero's 113
// K blocks become 4 chunks of 28-29).  Each switch of the MMA accumulator between the two
// TMEM chunk buffers costs about one K block of tensor time, so chunks are as long as the
// accuracy bound allows.  Measured: the worst element's error grows with the chunk length,
// and the bound's absolute term 1e-2/sqrt(K) shrinks with K, so the chunk shrinks as
// 1/sqrt(K) beyond the hero's K (chunk_blocks_for_k).  The worst element over the hero,
// M = 129, M = 1000 and long-K cases then uses 0.5-0.84 of the bound (2.7 with a single
// accumulator; 0.95 already with 3 chunks per hero tile).
constexpr int kMaxChunkKBlocks = 29;
constexpr int kNumEpilogueWarps = 8;
constexpr int kFirstEpilogueWarp = 4;  // warpgroup 0: producer, MMA, two idle warps
constexpr int kNumThreads = (kFirstEpilogueWarp + kNumEpilogueWarps) * 32;
// Register split (setmaxnreg): the block launches with 168 registers per thread
// (384 x 168 = 64512); warpgroup 0 drops to 72 and the two epilogue warpgroups rise to 216:
// 128 x 72 + 256 x 216 = 64512 <= 64512, inside the launch allocation, so the increase is
// always satisfied by what warpgroup 0 releases.
constexpr int kControlRegs = 72;
constexpr int kEpilogueRegs = 216;
static_assert(128 * kControlRegs + 256 * kEpilogueRegs <= kNumThreads * 168,
              "register split exceeds the launch allocation");
constexpr int kABoxBytes = kRowsPerCta * kBlockK * 2;  // 16 KiB
constexpr int kBChunkBytes = kBlockK * 64 * 2;          // 8 KiB: 64 K rows x 64 N columns
constexpr int kStoreBox = 32;                            // C store box: 32 rows x 32 columns
constexpr int kStoreBoxBytes = kStoreBox * kStoreBox * 2;  // 2 KiB, 64-byte swizzled rows

// Watchdog codes written to the device flag when a bounded wait expires.
enum : int {
  kWatchNone = 0,
  kWatchProducerEmpty = 1,
  kWatchMmaFull = 2,
  kWatchMmaChunkEmpty = 3,
  kWatchEpilogueChunkFull = 4,
  kWatchDrain = 5,
  kWatchSelfTest = 6,
  kWatchStreamK = 7,  // a stream-K arrival CAS loop, or a tail's wait for its tile's pieces, hit its bound
};

__device__ int g_watchdog_flag = 0;

// Stream-K arrival words: kSkRegions regions of kSkRegionWords words.  A file-scope device
// array is zero-filled when the module is loaded on a device, so no launch allocates, clears
// or synchronises for it; the host looks its address up once per device.
constexpr int kSkRegions = 16;
constexpr int kSkRegionWords = 1024;  // >= split tiles x CTAs per tile (<= 148 x 2)
__device__ unsigned int g_sk_counters[kSkRegions * kSkRegionWords];

// Scratch of mo_launch_bf16_gemm_v1_noalloc: the FP32 K-chunk partials of the split kernel
// (num_chunks x m x n floats).  A fixed 32 MiB that every GPU which loads this library keeps
// until the process exits; no call allocates it or frees it.
constexpr size_t kNoAllocScratchBytes = size_t{32} << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

struct GemmArgs {
  uint16_t* c;
  int m, n, k;
  int num_m_blocks, num_n_blocks, num_k_blocks;
  int num_tiles;
  int num_chunks;  // K chunks of the two-level accumulation (a function of k only)
  int num_units;   // work units: tiles, or (tile, chunk) pairs when split
  int split;       // 1: each unit is one K chunk of one tile, written as FP32 to `partials`
  int a_box_rows;  // rows per A TMA box: 128, or M rounded up to 8 when M < 128 (1-CTA only)
  // Rows of C per CTA: 128, or (1-CTA, M > 128) the least multiple of 32 that keeps the count
  // of row tiles, so a CTA loads no more A rows than its tile holds.  The MMA still computes
  // 128 rows; the rows past tile_rows are never stored.
  int tile_rows;
  int l2_prefetch_kb;  // > 0: the producer also prefetches B this many K blocks ahead into L2
  float* partials; // [num_chunks][m][n] FP32 chunk partials (split only)
  int num_clusters;   // persistent CTAs (or CTA pairs) in the grid
  // Stream-K schedule (sk = 1): the K chunks of the tiles [sk_tile0, num_tiles) left over
  // after `dp_per_cluster` whole tiles per cluster are dealt out as contiguous ranges over
  // `sk_clusters` clusters.  A tile whose chunks land on several clusters is finished by its
  // tail piece (the one holding the last chunk): the head piece publishes its running sum and
  // any middle piece its chunks in sk_ws, each counts itself in on sk_counters, and the tail
  // waits (bounded) for them and adds everything in chunk order.
  int sk;
  int dp_per_cluster;
  int sk_tile0;
  int sk_units;       // (num_tiles - sk_tile0) x num_chunks
  int sk_clusters;    // min(num_clusters, sk_units)
  float* sk_ws;       // [sk tile][cta][1 + num_chunks][128 x tile_n] FP32
  unsigned int* sk_counters;  // [sk tile][cta] arrival words: epoch << 8 | pieces counted
  unsigned int sk_epoch;      // this launch's tag (1 .. 2^24 - 1); other tags count as zero
  int group_m;
  int* watchdog;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void record_watchdog(const GemmArgs& a, int code) {
  if (a.watchdog != nullptr) atomicCAS(a.watchdog, 0, code);
}

// Stream-K arrival counters live in a per-device array the library keeps, tagged with the
// launch's epoch, so nothing has to clear them before a launch: a word carrying another
// launch's tag counts as zero.  Pieces of one tile count themselves in with a CAS.
__device__ __forceinline__ unsigned int sk_count_of(unsigned int word, unsigned int epoch) {
  return (word >> 8) == epoch ? (word & 0xFFu) : 0u;
}

// Counts one piece in; returns how many pieces were in before it (or 0xFFFFFFFF if the CAS
// loop hit its bound, recorded in the watchdog: then this piece does not finish the tile).
__device__ __forceinline__ unsigned int sk_arrive(unsigned int* ctr, unsigned int epoch,
                                                  const GemmArgs& a) {
  unsigned int old = *reinterpret_cast<volatile unsigned int*>(ctr);
  for (int i = 0; i < (1 << 20); ++i) {
    const unsigned int prior = sk_count_of(old, epoch);
    const unsigned int seen = atomicCAS(ctr, old, (epoch << 8) | (prior + 1u));
    if (seen == old) return prior;
    old = seen;
  }
  record_watchdog(a, kWatchStreamK);
  return 0xFFFFFFFFu;
}

// The schedule functions below also compile for the host, where mo_gemm_schedule lists a plan's
// work units with the same code the kernel runs.
__host__ __device__ constexpr int imin(int x, int y) { return x < y ? x : y; }
__host__ __device__ constexpr int imax(int x, int y) { return x > y ? x : y; }

// Grouped raster: tiles walk down `group_m` M-blocks, then step one N-block, so the tiles in
// flight at any moment share a compact band of A rows and B columns in L2.
__host__ __device__ __forceinline__ void tile_coords(int tile, const GemmArgs& a, int& mb, int& nb) {
  const int per_group = a.group_m * a.num_n_blocks;
  const int group = tile / per_group;
  const int first_m = group * a.group_m;
  const int gsz = imin(a.num_m_blocks - first_m, a.group_m);
  const int local = tile - group * per_group;
  mb = first_m + local % gsz;
  nb = local / gsz;
}

// K-chunk boundaries of the two-level accumulation: nkb K blocks split into nchunks nearly
// equal chunks.  A function of K alone, so every kernel variant sums the same partials.  The
// product c * nkb fits 32 unsigned bits whenever nkb < 2^16 (c <= nchunks <= nkb), which covers
// K up to 4 Mi; 64-bit division, a long software routine on the GPU, only runs beyond that.
__host__ __device__ __forceinline__ int chunk_begin(int c, int nkb, int nchunks) {
  if (c == 0) return 0;
  if (nkb < 65536) {
    return static_cast<int>((static_cast<unsigned int>(c) * static_cast<unsigned int>(nkb)) /
                            static_cast<unsigned int>(nchunks));
  }
  return static_cast<int>((static_cast<long long>(c) * nkb) / nchunks);
}

// (c * r0) mod nchunks with r0 = nkb mod nchunks: the remainder that steps the boundaries of
// the chunks after chunk c without a division (r0 < nchunks <= nkb, so 32 bits as above).
__host__ __device__ __forceinline__ int chunk_carry(int c, int r0, int nchunks) {
  if (c == 0) return 0;
  if (nchunks < 65536) {
    return static_cast<int>((static_cast<unsigned int>(c) * static_cast<unsigned int>(r0)) %
                            static_cast<unsigned int>(nchunks));
  }
  return static_cast<int>((static_cast<long long>(c) * r0) % nchunks);
}

// A work unit: one tile, all its K chunks; or (split) one K chunk of one tile.  Split units
// are ordered chunk-major, so the units in flight together share the A and B bands of one
// K chunk.
struct Unit {
  int mb, nb, ch_begin, ch_end;
  int sk_tile;  // stream-K tile index when this unit is one piece of a split tile, else -1
};

// Stream-K range of cluster c: units [lo, hi) of the stream-K region.  The host plans stream-K
// only while sk_units < 2^24, so (c + 1) * sk_units (c < 148 clusters) fits 32 unsigned bits.
__host__ __device__ __forceinline__ void sk_range(int c, const GemmArgs& a, int& lo, int& hi) {
  const unsigned int units = static_cast<unsigned int>(a.sk_units);
  const unsigned int clusters = static_cast<unsigned int>(a.sk_clusters);
  lo = static_cast<int>(static_cast<unsigned int>(c) * units / clusters);
  hi = static_cast<int>(static_cast<unsigned int>(c + 1) * units / clusters);
}

// Cluster whose stream-K range holds unit u (every range is non-empty: sk_units >= sk_clusters).
__host__ __device__ __forceinline__ int sk_owner(int u, const GemmArgs& a) {
  return static_cast<int>((static_cast<unsigned int>(u + 1) * static_cast<unsigned int>(a.sk_clusters) - 1u) /
                          static_cast<unsigned int>(a.sk_units));
}

__host__ __device__ __forceinline__ int num_units_of(int c, const GemmArgs& a) {
  if (!a.sk) return c < a.num_units ? (a.num_units - c + a.num_clusters - 1) / a.num_clusters : 0;
  int count = a.dp_per_cluster;
  if (c < a.sk_clusters) {
    int lo, hi;
    sk_range(c, a, lo, hi);
    if (hi > lo) count += (hi - 1) / a.num_chunks - lo / a.num_chunks + 1;
  }
  return count;
}

// Unit j of cluster c (the same sequence in the producer, MMA and epilogue roles).  With
// stream-K a cluster's pieces of split tiles run in decreasing tile order, and its whole tiles
// sit between the first pieces and a closing tail: a piece that starts a tile (its head) or lies
// inside one (a middle) runs first in its cluster, the cluster's whole tiles run next, and a piece
// that ends a tile (its tail, which finishes the tile from the others' published sums) runs last.
// The heads and middles thus publish early, while the other clusters are still busy with whole
// tiles, and a tail finds their sums ready without waiting or holding a TMEM buffer.  Every SM's
// link to L2 is nearly full with the TMA operand loads, so the pieces' FP32 sums cost MMA time
// wherever they move; this order moves one sum per two-piece tile (measured on the 8-GPU slab,
// instrumented: the tail's two chunk sums written and read back slowed the tail clusters' MMAs
// by 3.8 us).  unit_piece works out all of it but the tile's coordinates (the tile index, chunk
// range and stream-K tile, which is all the MMA issuer needs); unit_at adds the coordinates.
__host__ __device__ __forceinline__ int unit_piece(int c, int j, const GemmArgs& a, Unit& w) {
  w.sk_tile = -1;
  if (!a.sk) {
    const int u = c + j * a.num_clusters;
    if (a.split) {
      const int ch = u / a.num_tiles;
      w.ch_begin = ch;
      w.ch_end = ch + 1;
      return u - ch * a.num_tiles;
    }
    w.ch_begin = 0;
    w.ch_end = a.num_chunks;
    return u;
  }
  int tile = 0;
  const int q = a.num_chunks;
  int lo = 0, hi = 0;
  if (c < a.sk_clusters) sk_range(c, a, lo, hi);
  int npieces = 0;
  if (c < a.sk_clusters && hi > lo) npieces = (hi - 1) / q - lo / q + 1;
  // The last piece in decreasing tile order is that of tile lo / q: a tail when it starts inside
  // the tile and runs to its last chunk.
  const int first_tile = lo / q;
  const bool tail_last = npieces > 0 && lo % q != 0 && hi - first_tile * q >= q;
  const int lead = tail_last ? npieces - 1 : npieces;
  int piece;
  if (j < lead) {
    piece = j;
  } else if (j < lead + a.dp_per_cluster) {
    piece = -1;
    tile = c + (j - lead) * a.num_clusters;
    w.ch_begin = 0;
    w.ch_end = a.num_chunks;
  } else {
    piece = npieces - 1;
  }
  if (piece >= 0) {
    const int st = (hi - 1) / q - piece;
    w.ch_begin = imax(lo - st * q, 0);
    w.ch_end = imin(hi - st * q, q);
    tile = a.sk_tile0 + st;
    if (w.ch_begin != 0 || w.ch_end != q) w.sk_tile = st;  // a whole tile needs no fix-up
  }
  return tile;
}

__host__ __device__ __forceinline__ Unit unit_at(int c, int j, const GemmArgs& a) {
  Unit w;
  const int tile = unit_piece(c, j, a, w);
  tile_coords(tile, a, w.mb, w.nb);
  return w;
}

// Pieces a stream-K tile is split into, and the chunk where its head piece (chunk 0) ends.
__host__ __device__ __forceinline__ void sk_tile_pieces(int st, const GemmArgs& a, int& pieces, int& head_end) {
  const int q = a.num_chunks;
  const int first = sk_owner(st * q, a);
  pieces = sk_owner(st * q + q - 1, a) - first + 1;
  int lo, hi;
  sk_range(first, a, lo, hi);
  head_end = imin(hi - st * q, q);
}

// How the epilogue folds a drained TMEM chunk into its registers.
enum : int { kDrainAssign = 0, kDrainRunning = 1, kDrainAdd = 2 };
template <int M>
using DrainMode = std::integral_constant<int, M>;

constexpr int tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

// Compile-time geometry of one variant: CG = CTAs per tile (cta_group), BN_CTA = B columns
// each CTA stages per K block.
template <int CG, int BN_CTA, int STAGES>
struct Geometry {
  static constexpr int kTileM = kRowsPerCta * CG;
  static constexpr int kTileN = BN_CTA * CG;           // = UMMA N
  static constexpr int kBBytes = (BN_CTA / 64) * kBChunkBytes;
  static constexpr int kStageBytes = kABoxBytes + kBBytes;
  static constexpr int kTmemCols = tmem_cols_for(2 * kTileN);  // two chunk buffers
  static constexpr int kEpiCols = kTileN / 2;                    // columns per epilogue warp
  static constexpr int kStagingBytes = kNumEpilogueWarps * 2 * kStoreBoxBytes;  // C staging
  static constexpr int kBarrierBytes = (2 * STAGES + 5) * 8;
  static constexpr int kSmemBytes =
      STAGES * kStageBytes + kStagingBytes + kBarrierBytes + 16 + 1024;
  static_assert(BN_CTA % 64 == 0, "B is staged in 64-column swizzle atoms");
  static_assert(kTileN >= 64 && kTileN <= 256, "UMMA N range used here");
  static_assert(kEpiCols % 32 == 0, "epilogue reads TMEM 32 columns at a time");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ uint32_t bf16x2_rne(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int CG, int BN_CTA, int STAGES>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_bf16_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_c,
                           const __grid_constant__ GemmArgs args) {
  using G = Geometry<CG, BN_CTA, STAGES>;
  constexpr uint32_t kIdesc = ptx::idesc_bf16_f32(G::kTileM, G::kTileN, false, true);
  constexpr int kBChunks = BN_CTA / 64;

  // The kernel's first steps stall on cold constant-cache lines (the kernel parameters) one after
  // another.  Two otherwise idle warps fetch every line of the arguments and the three tensor
  // maps at entry, in parallel with the set-up below, so the producer's and the MMA issuer's
  // first reads hit (measured: the producer's first TMA issue came 0.7 us (one CTA) to 1.5 us
  // (stream-K pairs) after its set-up, most of it waiting on argument reads).
  {
    const int w = static_cast<int>(threadIdx.x) / 32;
    const int l = static_cast<int>(threadIdx.x) % 32;
    if (w == 2 && l < static_cast<int>(sizeof(GemmArgs) / 16)) {
      const uint4 v = reinterpret_cast<const uint4*>(&args)[l];
      asm volatile("" ::"r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
    } else if (w == 3 && l == 0) {
      ptx::tma_prefetch_desc(&tmap_a);
      ptx::tma_prefetch_desc(&tmap_b);
      ptx::tma_prefetch_desc(&tmap_c);
    }
  }
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled TMA destinations and UMMA operands must be 1024-byte aligned.  The
  // offset is the same in both CTAs of a pair (same kernel, same dynamic smem base).
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const uint32_t smem_base = ptx::smem_addr(smem);

  const uint32_t staging_base = smem_base + STAGES * G::kStageBytes;
  uint8_t* bar_area = smem + STAGES * G::kStageBytes + G::kStagingBytes;
  const uint32_t bar_base = ptx::smem_addr(bar_area);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto chunk_full_bar = [&](int i) { return bar_base + 8u * (2 * STAGES + i); };
  auto chunk_empty_bar = [&](int i) { return bar_base + 8u * (2 * STAGES + 2 + i); };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_area + G::kBarrierBytes);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = ptx::lane_id();
  const uint32_t cta_rank = (CG == 2) ? ptx::cluster_cta_rank() : 0u;
  const bool leader = cta_rank == 0;
  const int cluster = static_cast<int>(blockIdx.x) / CG;

  // The cluster's unit count and first unit (a chain of integer divisions, about a microsecond
  // on the stream-K schedule) are worked out by an idle warp while thread 0 initialises the
  // barriers and warp 1 allocates TMEM, so the producer's first TMA issue does not wait for them.
  __shared__ Unit s_unit0;
  __shared__ int s_my_units;
  if (warp == 3 && lane == 0) {
    const int units = num_units_of(cluster, args);
    s_my_units = units;
    if (units > 0) s_unit0 = unit_at(cluster, 0, args);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(chunk_full_bar(i), 1);
      ptx::mbar_init(chunk_empty_bar(i), kNumEpilogueWarps * CG);
    }
    ptx::mbar_init(drain_bar, 1);
    ptx::fence_barrier_init();
  }
  if (warp == 1) ptx::tmem_alloc<CG>(ptx::smem_addr(tmem_slot), G::kTmemCols);
  ptx::tc_fence_before_sync();
  __syncthreads();
  if constexpr (CG == 2) ptx::cluster_sync();  // peer barriers initialised before use
  ptx::tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int my_units = s_my_units;
  // Launched with programmatic stream serialization, the kernel may start while the previous
  // kernel in the stream drains; everything above touched only this CTA's shared memory and
  // TMEM.  From here on it reads A and B and writes C and workspaces, so it first waits for
  // the previous grid to complete and its memory to be visible.  (A no-op otherwise.)
  ptx::grid_dependency_wait();
  const uint64_t timeout = args.timeout_ns;
  const int nkb = args.num_k_blocks;
  const int nchunks = args.num_chunks;

  if (warp < kFirstEpilogueWarp) {
    ptx::setmaxnreg_dec<kControlRegs>();
    if (warp == 0) {
      // ---------------------------- TMA producer (both CTAs) ----------------------------
      if (lane == 0) {
        // A row bands are re-read by every N block of a raster group; keep them in L2.  B is
        // evict_first where each element is loaded at most twice and nothing prefetches it:
        // CTA-pair plans with one or two row bands.  Measured with a flush before each launch,
        // that took M = 129 from 42.7 to 37.2 us, M = 256 from 43.0 to 38.9 us and M = 300 from
        // 52.1 to 48.6 us (N = 7776, K = 7232); with more row bands it cost the square 8192^3
        // and the LLM projection 1.5-2 %.  The 1-CTA skinny plans, whose B is prefetched into L2
        // ahead of the loads, measured 5-6 % slower with it at M = 1 and 16, and keep
        // evict_normal.
        const uint64_t hint_a = ptx::policy_evict_last();
        const uint64_t hint_b = (CG == 2 && args.num_m_blocks <= 2) ? ptx::policy_evict_first()
                                                                    : ptx::policy_evict_normal();
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0;  // K blocks loaded, capped at STAGES (only the last STAGES matter)
        bool ok = true;
        const uint32_t stage_tx = static_cast<uint32_t>(args.a_box_rows) * 128u + G::kBBytes;
        // Chunk completions reach the epilogue through this thread, not through an extra
        // tcgen05.commit per chunk (a commit that frees no stage stalls the tensor pipe).  A
        // stage that holds the last K block of a chunk is marked (2 bits per stage: 1 + the
        // chunk's TMEM buffer); when the producer next sees that stage freed -- the MMAs that
        // read it, and all before them, complete -- it arrives on the chunk's full barrier.
        uint32_t chunk_ends = 0;
        uint32_t chunk_count = 0;
        const int q0 = nkb / nchunks;
        const int r0 = nkb - q0 * nchunks;
        // The next unit is worked out while this one's first loads are in flight, so the loads of
        // a new tile follow the last ones of the previous tile without a gap.
        for (int j = 0; j < my_units && ok; ++j) {
          const Unit w = j == 0 ? s_unit0 : unit_at(cluster, j, args);
          const int a_row = (w.mb * CG + static_cast<int>(cta_rank)) * args.tile_rows;
          const int b_col = w.nb * G::kTileN + BN_CTA * static_cast<int>(cta_rank);
          int kb = chunk_begin(w.ch_begin, nkb, nchunks);
          int rem = chunk_carry(w.ch_begin, r0, nchunks);
          const int kb_unit_end = args.l2_prefetch_kb > 0 ? chunk_begin(w.ch_end, nkb, nchunks) : 0;
          for (int ch = w.ch_begin; ch < w.ch_end && ok; ++ch, ++chunk_count) {
            rem += r0;
            const bool carry = rem >= nchunks;
            if (carry) rem -= nchunks;
            const int kb_hi = kb + q0 + (carry ? 1 : 0);
            for (; kb < kb_hi; ++kb) {
              // As in the issuer, the stage's addresses are ready before the empty-barrier wait, and
              // the chunk-end hand-off (not urgent) follows the loads, so a freed stage refills as
              // soon as the wait returns.  A CTA pair's bytes complete on the leader's full
              // barrier (lf); only the leader arms it.
              uint32_t sa = smem_base + stage * G::kStageBytes;
              uint32_t fb = full_bar(stage);
              int kx = kb * kBlockK;
              uint32_t lf = (CG == 2) ? ptx::map_to_cta(fb, 0) : fb;
              asm volatile("" : "+r"(sa), "+r"(fb), "+r"(kx), "+r"(lf));
              if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, timeout)) {
                record_watchdog(args, kWatchProducerEmpty);
                ok = false;
                break;
              }
              const uint32_t sb = sa + kABoxBytes;
              if constexpr (CG == 1) {
                ptx::mbar_arrive_expect_tx(fb, stage_tx);
                ptx::tma_load_2d(sa, &tmap_a, fb, kx, a_row, hint_a);
  #pragma unroll
                for (int c = 0; c < kBChunks; ++c) {
                  ptx::tma_load_2d(sb + c * kBChunkBytes, &tmap_b, fb, b_col + c * 64, kx, hint_b);
                }
              } else {
                if (leader) ptx::mbar_arrive_expect_tx(fb, 2 * stage_tx);
                ptx::tma_load_2d_pair(sa, &tmap_a, lf, kx, a_row, hint_a);
  #pragma unroll
                for (int c = 0; c < kBChunks; ++c) {
                  ptx::tma_load_2d_pair(sb + c * kBChunkBytes, &tmap_b, lf, b_col + c * 64, kx, hint_b);
                }
              }
              if (const uint32_t e = (chunk_ends >> (2 * stage)) & 3u) {
                ptx::mbar_arrive(chunk_full_bar(static_cast<int>(e - 1)));
                chunk_ends &= ~(3u << (2 * stage));
              }
              if (kb + args.l2_prefetch_kb < kb_unit_end) {
                // Skinny A: the kernel streams B from HBM and the ring alone cannot cover the
                // DRAM latency, so B is pulled into L2 a few K blocks ahead of its TMA load.
  #pragma unroll
                for (int c = 0; c < kBChunks; ++c) {
                  ptx::tma_prefetch_2d(&tmap_b, b_col + c * 64, (kb + args.l2_prefetch_kb) * kBlockK, hint_b);
                }
              }
              if (kb == kb_hi - 1) chunk_ends |= (1u + (chunk_count & 1u)) << (2 * stage);
              if (issued < STAGES) ++issued;
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
        }
        // Tail: wait, oldest first, for the MMAs of the last min(issued, STAGES) stages and
        // forward their chunk ends.  This also keeps the CTA from exiting while its stages may
        // still be written (a stage is freed only after its bytes landed and were read).
        const int outstanding = issued;
        int s_tail = stage;
        uint32_t ph_tail = phase;
        for (int i = 0; i < outstanding; ++i) {
          if (s_tail == 0) {
            s_tail = STAGES - 1;
            ph_tail ^= 1u;
          } else {
            --s_tail;
          }
        }
        for (int i = 0; i < outstanding; ++i) {
          if (!ptx::mbar_wait(empty_bar(s_tail), ph_tail, timeout)) {
            record_watchdog(args, kWatchDrain);
            break;
          }
          if (const uint32_t e = (chunk_ends >> (2 * s_tail)) & 3u) {
            ptx::mbar_arrive(chunk_full_bar(static_cast<int>(e - 1)));
            chunk_ends &= ~(3u << (2 * s_tail));
          }
          if (++s_tail == STAGES) {
            s_tail = 0;
            ph_tail ^= 1u;
          }
        }
      }
    } else if (warp == 1) {
      // ---------------------------- MMA issuer (leader CTA) ----------------------------
      if (lane == 0 && leader) {
        int stage = 0;
        uint32_t phase = 0;
        uint32_t chunk_count = 0;
        bool ok = true;
        // The tensor pipe keeps only a short queue, so nothing slow may sit between two K
        // blocks' MMAs.  Chunk boundaries floor(c * nkb / nchunks) therefore step without a
        // division: c * nkb = c * q0 * nchunks + c * r0, so each boundary advances by q0 plus
        // the carry of the remainder c * r0 mod nchunks (divisions remain only where a unit
        // starts mid-tile: K-split and stream-K pieces).
        const int q0 = nkb / nchunks;
        const int r0 = nkb - q0 * nchunks;
        // The issuer needs only each unit's chunk range (no tile coordinates, whose divisions would
        // sit between the MMAs of two units); whole-tile schedules need no division at all.
        for (int j = 0; j < my_units && ok; ++j) {
          Unit w;
          if (j == 0) {
            w = s_unit0;
          } else {
            unit_piece(cluster, j, args, w);
          }
          int kb_lo = chunk_begin(w.ch_begin, nkb, nchunks);
          int rem = chunk_carry(w.ch_begin, r0, nchunks);
          for (int ch = w.ch_begin; ch < w.ch_end && ok; ++ch, ++chunk_count) {
            const int buf = static_cast<int>(chunk_count & 1u);
            const uint32_t use_parity = (chunk_count >> 1) & 1u;
            if (!ptx::mbar_wait(chunk_empty_bar(buf), use_parity ^ 1u, timeout)) {
              record_watchdog(args, kWatchMmaChunkEmpty);
              ok = false;
              break;
            }
            ptx::tc_fence_after_sync();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * G::kTileN);
            rem += r0;
            const bool carry = rem >= nchunks;
            if (carry) rem -= nchunks;
            const int kb_hi = kb_lo + q0 + (carry ? 1 : 0);
            for (int kb = kb_lo; kb < kb_hi; ++kb) {
              // The stage's descriptors are built before its full-barrier wait (the empty asm pins
              // them there), so only the fence and the four MMAs sit between the data landing and
              // the tensor pipe starting on it.  The ring's round trip runs through this path once
              // per K block: building them after the wait measured 2 % slower on the hero.
              // A: K-major, +16 elements (32 bytes, 2 in the descriptor's address field) per K
              // step inside the swizzle atom.  B: MN-major, +16 K rows = two 8-row groups of
              // 1024 bytes (128 in the address field) per K step.
              const uint32_t sa = smem_base + stage * G::kStageBytes;
              uint64_t a_desc0 = ptx::smem_desc_sw128(sa, 16, 1024);
              uint64_t b_desc0 = ptx::smem_desc_sw128(sa + kABoxBytes, kBChunkBytes, 1024);
              uint32_t acc0 = kb != kb_lo ? 1u : 0u;
              asm volatile("" : "+l"(a_desc0), "+l"(b_desc0), "+r"(acc0));
              if (!ptx::mbar_wait(full_bar(stage), phase, timeout)) {
                record_watchdog(args, kWatchMmaFull);
                ok = false;
                break;
              }
              ptx::tc_fence_after_sync();
  #pragma unroll
              for (int step = 0; step < kBlockK / kUmmaK; ++step) {
                ptx::mma_bf16<CG>(d_tmem, a_desc0 + 2u * step, b_desc0 + 128u * step, kIdesc, step != 0 ? 1u : acc0);
              }
              if constexpr (CG == 1) {
                ptx::mma_commit<1>(empty_bar(stage));
              } else {
                ptx::mma_commit_pair(empty_bar(stage), 0x3);
              }
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
            }
            if (!ok) break;
            kb_lo = kb_hi;
          }
        }
        // Every MMA this thread issued must be complete before TMEM is freed.
        ptx::mma_commit<CG>(drain_bar);
        if (!ptx::mbar_wait(drain_bar, 0, timeout)) record_watchdog(args, kWatchDrain);
      }
    }
  } else {
    ptx::setmaxnreg_inc<kEpilogueRegs>();
    // ---------------------------- Epilogue (warps 4..11, both CTAs) ----------------------------
    const int quarter = warp & 3;                 // TMEM lanes 32*quarter .. +31
    const int half = (warp - kFirstEpilogueWarp) >> 2;  // column half of the tile
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(half * G::kEpiCols);
    // Two 32x32 staging boxes per warp for the TMA stores of C (64-byte swizzled rows).
    const uint32_t staging =
        staging_base + static_cast<uint32_t>((warp - kFirstEpilogueWarp) * 2 * kStoreBoxBytes);
    const uint32_t row_swizzle = (lane >> 1) & 3u;
    uint32_t chunk_count = 0, box_count = 0;
    bool ok = true;
    const int row_local = quarter * 32 + static_cast<int>(lane);  // row of this CTA's 128
    const int col_local = half * G::kEpiCols;                     // first column in the tile

    // Stream-K workspace of this thread: slot 0 = head running sum, slot 1 + c = chunk c.  The
    // piece that writes a slot and the piece that reads it back map threads to (row, columns)
    // identically, so a slot is laid out thread-major: float4 v of epilogue thread t sits at
    // v * 256 + t, and every warp-wide access covers 512 contiguous bytes.
    const int epi_thread = (warp - kFirstEpilogueWarp) * 32 + static_cast<int>(lane);
    auto sk_slot = [&](int st, int slot) {
      const size_t tile_floats = static_cast<size_t>(kRowsPerCta) * G::kTileN;
      return reinterpret_cast<float4*>(
                 args.sk_ws +
                 ((static_cast<size_t>(st) * CG + cta_rank) * (args.num_chunks + 1) + slot) * tile_floats) +
             epi_thread;
    };
    constexpr int kSlotStride = kNumEpilogueWarps * 32;  // float4s between a thread's vectors

    // After a timed-out wait a warp drains nothing more, but it still walks its units to
    // meet the other epilogue warps at the next stream-K piece barrier, where all of them
    // learn of the failure and stop together.
    for (int j = 0; j < my_units; ++j) {
      const Unit w = unit_at(cluster, j, args);
      const int mb = w.mb, nb = w.nb;
      const bool piece = w.sk_tile >= 0;           // one piece of a stream-K split tile
      if (!ok && !piece) continue;
      const bool running = !piece || w.ch_begin == 0;  // sums its chunks (else stores each alone)
      // A thread whose row lies below C skips the pieces' workspace traffic: its sums are
      // never stored (the TMA store clips them), so skinny tiles move only their real rows.
      const bool row_in_c = row_local < args.tile_rows &&
                            (mb * CG + static_cast<int>(cta_rank)) * args.tile_rows + row_local < args.m;
      float acc[G::kEpiCols];
      const int unit_chunks = w.ch_end - w.ch_begin;
      // Drains chunk i of this unit from TMEM into acc (assigned or added, by the mode).
      auto drain = [&](int i, auto sum_chunks) -> bool {
        const int buf = static_cast<int>(chunk_count & 1u);
        const uint32_t use_parity = (chunk_count >> 1) & 1u;
        ++chunk_count;
        if (!ptx::mbar_wait(chunk_full_bar(buf), use_parity, timeout)) {
          record_watchdog(args, kWatchEpilogueChunkFull);
          return false;
        }
        ptx::tc_fence_after_sync();
        const uint32_t taddr = lane_base + static_cast<uint32_t>(buf * G::kTileN);
        // kDrainAssign: every chunk replaces acc; kDrainRunning: chunk 0 replaces, later chunks add;
        // kDrainAdd: every chunk adds (a tail piece, onto the tile's earlier sum).
        constexpr int kMode = decltype(sum_chunks)::value;
        const bool first = kMode == kDrainAssign || (kMode == kDrainRunning && i == 0);
        // Two 32-column TMEM loads in flight per wait.
        constexpr int kLoads = G::kEpiCols / 32;
        constexpr int kPerWait = kLoads >= 2 ? 2 : 1;
#pragma unroll
        for (int jj = 0; jj < kLoads; jj += kPerWait) {
          uint32_t r[kPerWait][32];
#pragma unroll
          for (int u = 0; u < kPerWait; ++u) ptx::tmem_ld_32x32b_x32(taddr + (jj + u) * 32, r[u]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < kPerWait; ++u) {
#pragma unroll
            for (int ii = 0; ii < 32; ++ii) {
              const float v = __uint_as_float(r[u][ii]);
              float& a = acc[(jj + u) * 32 + ii];
              a = first ? v : __fadd_rn(a, v);
            }
          }
        }
        ptx::tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1) {
            ptx::mbar_arrive(chunk_empty_bar(buf));
          } else {
            ptx::mbar_arrive_cluster(chunk_empty_bar(buf), 0);
          }
        }
        return true;
      };
      // Roles of a stream-K piece: the head (from chunk 0) sums its chunks and publishes the
      // running sum; a middle piece publishes each chunk apart; the tail (to the last chunk)
      // finishes the tile.
      const bool is_head = piece && w.ch_begin == 0;
      const bool is_tail = piece && !is_head && w.ch_end == args.num_chunks;
      if (!ok) {
        // reach the piece barrier below without draining
      } else if (running) {
        // Zero-based so the compiler peels the first (assigning) iteration.
        for (int i = 0; i < unit_chunks; ++i) {
          if (!drain(i, DrainMode<kDrainRunning>{})) {
            ok = false;
            break;
          }
        }
      } else if (is_tail) {
        // The tail first waits for the tile's earlier pieces (below), then drains its chunks.
      } else {
        for (int i = 0; i < unit_chunks; ++i) {
          if (!drain(i, DrainMode<kDrainAssign>{})) {
            ok = false;
            break;
          }
          // A middle piece keeps each chunk's partial apart, so the tail can add them in chunk
          // order after the head's running sum.
          if (row_in_c) {
            float4* dst = sk_slot(w.sk_tile, 1 + w.ch_begin + i);
#pragma unroll
            for (int v = 0; v < G::kEpiCols / 4; ++v) {
              dst[v * kSlotStride] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
            }
          }
        }
      }
      if (!ok && !piece) continue;
      if (args.split) {
        // One K chunk's FP32 partial: each thread writes its row's columns (16-byte stores;
        // n % 8 == 0 keeps every 4-column group wholly inside or outside C).
        const int row = (mb * CG + static_cast<int>(cta_rank)) * args.tile_rows + row_local;
        const int col_base = nb * G::kTileN + col_local;
        if (row_in_c) {
          float* prow = args.partials +
                        (static_cast<size_t>(w.ch_begin) * args.m + row) * static_cast<size_t>(args.n);
#pragma unroll
          for (int v = 0; v < G::kEpiCols / 4; ++v) {
            const int col = col_base + 4 * v;
            if (col < args.n) {
              *reinterpret_cast<float4*>(prow + col) =
                  make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
            }
          }
        }
        continue;
      }
      if (piece) {
        // ---- one piece of a stream-K split tile ----
        // Every epilogue warp meets here, so a failed wait stops all of them at the same unit.
        if (ptx::named_barrier_or(1, kNumEpilogueWarps * 32, !ok)) {
          ok = false;
          break;
        }
        int pieces, head_end;
        sk_tile_pieces(w.sk_tile, args, pieces, head_end);
        unsigned int* counter = &args.sk_counters[w.sk_tile * CG + cta_rank];
        const bool leader = warp == kFirstEpilogueWarp && lane == 0;
        if (!is_tail) {
          // Head or middle: publish (the CTA's stores, then one release) and count in.  These
          // pieces never wait, and each runs first in its cluster (unit_at).
          if (is_head && row_in_c) {
            float4* dst = sk_slot(w.sk_tile, 0);
#pragma unroll
            for (int v = 0; v < G::kEpiCols / 4; ++v) {
              dst[v * kSlotStride] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
            }
          }
          ptx::named_barrier_sync(1, kNumEpilogueWarps * 32);
          if (leader) {
            ptx::fence_acq_rel_gpu();
            sk_arrive(counter, args.sk_epoch, args);
          }
          continue;
        }
        // Tail: wait (bounded) until the head and every middle piece have counted in, then
        // finish the tile: acc starts as the head's running sum plus the middle chunks, and this
        // piece's chunks are added to it from TMEM -- the same FP32 adds in the same order as the
        // unsplit epilogue.  Waiting before the first drain keeps only one 128-column sum live;
        // the tail runs after its cluster's whole tiles and the others began with the kernel, so
        // their sums are normally in long before.
        bool all_in = false;
        if (leader) {
          const uint64_t t0 = ptx::global_timer_ns();
          while (true) {
            if (sk_count_of(ptx::ld_acquire_gpu(counter), args.sk_epoch) ==
                static_cast<unsigned int>(pieces - 1)) {
              all_in = true;
              break;
            }
            if (ptx::global_timer_ns() - t0 >= args.timeout_ns) {
              record_watchdog(args, kWatchStreamK);
              break;
            }
            __nanosleep(64);
          }
        }
        if (!ptx::named_barrier_or(1, kNumEpilogueWarps * 32, all_in)) {
          ok = false;
          break;
        }
        const float4* head = sk_slot(w.sk_tile, 0);
#pragma unroll
        for (int v0 = 0; v0 < G::kEpiCols / 4; v0 += 2) {
          float4 t[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) t[u] = row_in_c ? __ldcg(head + (v0 + u) * kSlotStride) : make_float4(0.f, 0.f, 0.f, 0.f);
          for (int ch = head_end; ch < w.ch_begin && row_in_c; ++ch) {
            const float4* mid = sk_slot(w.sk_tile, 1 + ch);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float4 m = __ldcg(mid + (v0 + u) * kSlotStride);
              t[u] = make_float4(__fadd_rn(t[u].x, m.x), __fadd_rn(t[u].y, m.y), __fadd_rn(t[u].z, m.z),
                                 __fadd_rn(t[u].w, m.w));
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int v = v0 + u;
            acc[4 * v] = t[u].x;
            acc[4 * v + 1] = t[u].y;
            acc[4 * v + 2] = t[u].z;
            acc[4 * v + 3] = t[u].w;
          }
        }
        for (int i = 0; i < unit_chunks; ++i) {
          if (!drain(i, DrainMode<kDrainAdd>{})) {
            ok = false;
            break;
          }
        }
        if (!ok) continue;
      }  // stream-K piece
      // Round to BF16 and store through shared memory: each thread owns one row of the warp's
      // 32 rows; each 32x32 box goes out as one TMA store (clipped at the C edges).
      const int row0 = (mb * CG + static_cast<int>(cta_rank)) * args.tile_rows + quarter * 32;
      const bool quarter_in_tile = quarter * 32 < args.tile_rows;
      const int col_base = nb * G::kTileN + col_local;
#pragma unroll
      for (int p = 0; p < G::kEpiCols / kStoreBox; ++p, ++box_count) {
        const uint32_t box = staging + (box_count & 1u) * kStoreBoxBytes;
        // The store issued from this buffer two boxes ago must have finished reading it.
        if (lane == 0) ptx::tma_store_wait_read<1>();
        __syncwarp();
        const uint32_t row_addr = box + lane * 64u;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float* v = &acc[p * kStoreBox + c * 8];
          ptx::st_shared_v4(row_addr + ((static_cast<uint32_t>(c) ^ row_swizzle) << 4),
                            bf16x2_rne(v[0], v[1]), bf16x2_rne(v[2], v[3]),
                            bf16x2_rne(v[4], v[5]), bf16x2_rne(v[6], v[7]));
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int col = col_base + p * kStoreBox;
          if (quarter_in_tile && row0 < args.m && col < args.n) ptx::tma_store_2d(&tmap_c, box, col, row0);
          ptx::tma_store_commit();  // one group per box, empty when the box is outside C
        }
      }
    }
    if (lane == 0) ptx::tma_store_wait_all<0>();  // C writes complete before the CTA exits
  }

  ptx::tc_fence_before_sync();
  __syncthreads();
  if constexpr (CG == 2) ptx::cluster_sync();  // no CTA leaves while its peer may signal it
  if (warp == 1) {
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc<CG>(tmem_base, G::kTmemCols);
  }
}

// Column re-layout after an all-gather: block i of `gathered` is a row-major [m, w_i] slab;
// C is row-major [m, sum w_i].  HBM-bound copy, 16-byte vectors when every width is a
// multiple of 8.
constexpr int kMaxShards = 64;
struct UnshardArgs {
  const uint16_t* gathered;
  uint16_t* c;
  int g, m, n;
  long long block_elems;
  int begin[kMaxShards + 1];
};

__global__ void unshard_columns_kernel(const UnshardArgs a, bool vec8) {
  const long long total = static_cast<long long>(a.m) * a.n;
  const int step = vec8 ? 8 : 1;
  const long long units = total / step;
  for (long long u = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = u * step;
    const int row = static_cast<int>(e / a.n);
    const int col = static_cast<int>(e - static_cast<long long>(row) * a.n);
    int s = 0;
    while (col >= a.begin[s + 1]) ++s;
    const int w = a.begin[s + 1] - a.begin[s];
    const uint16_t* src = a.gathered + s * a.block_elems + static_cast<long long>(row) * w +
                          (col - a.begin[s]);
    if (vec8) {
      *reinterpret_cast<uint4*>(a.c + e) = *reinterpret_cast<const uint4*>(src);
    } else {
      a.c[e] = *src;
    }
  }
}

// Waits on an mbarrier that nothing ever completes, with a short limit, and records the
// expiry in the watchdog flag: exercises the bounded-wait path without a fault or a hang.
__global__ void selftest_wait_timeout_kernel(int* watchdog, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_addr(&bar), 1);
    ptx::fence_barrier_init();
    if (!ptx::mbar_wait(ptx::smem_addr(&bar), 0, timeout_ns)) {
      if (watchdog != nullptr) atomicCAS(watchdog, 0, kWatchSelfTest);
    }
  }
}

}  // namespace
}  // namespace mo
