// Host side of the sm_100a BF16 GEMM, the B200 replacement for the reference's kernel
// library src/kernels/bf16_gemm_v1.cu (dispatcher :2098-2180): kernel variants and the cost
// model that picks one, the schedules (whole tiles, K split, stream-K), workspaces, launch,
// padded copies for layouts TMA cannot describe, the host-buffer pipeline, the reference's C++
// ABI and the C ABI of include/mo_gemm.h.  The kernel itself is in gemm_kernel.cuh.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <mutex>
#include <vector>
#include <type_traits>

#include "../../include/kernel_api.h"
#include "../../include/mo_gemm.h"
#include "gemm_kernel.cuh"

namespace mo {
namespace {

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// 2-D BF16 tensor map over a row-major [rows, cols] matrix, box [box_rows, box_cols],
// 128-byte swizzle, zero fill out of bounds.
bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                  uint32_t box_rows, uint32_t box_cols,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Kernel variants compiled into the library.
enum Variant : int {
  kVarPair256 = 0,  // CTA pair, 256 x 256 tile
  kVar1x256 = 1,    // one CTA, 128 x 256 tile
  kVar1x128 = 2,    // one CTA, 128 x 128 tile
  kVar1x64 = 3,     // one CTA, 128 x 64 tile
  kVarPair128 = 4,  // CTA pair, 256 x 128 tile (short rows: skinny M just over 128)
  kNumVariants = 5
};

struct VariantInfo {
  int cta_group;
  int block_n_cta;
  int stages;
  int smem;
  double mma_efficiency;  // fraction of tensor peak the tile shape sustains (measured)
};

constexpr VariantInfo kVariants[kNumVariants] = {
    {2, 128, 6, Geometry<2, 128, 6>::kSmemBytes, 0.92},
    {1, 256, 4, Geometry<1, 256, 4>::kSmemBytes, 0.70},
    {1, 128, 6, Geometry<1, 128, 6>::kSmemBytes, 0.62},
    {1, 64, 8, Geometry<1, 64, 8>::kSmemBytes, 0.50},
    {2, 64, 8, Geometry<2, 64, 8>::kSmemBytes, 0.60},
};

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int cc_major = 0;
  int* watchdog = nullptr;
  std::array<bool, kNumVariants> attr_done{};
  std::array<int, kNumVariants> max_units{};  // co-resident tiles (CTAs or CTA pairs)
  float* noalloc_scratch = nullptr;           // device address of g_noalloc_scratch
  cudaMemPool_t pool = nullptr;               // workspaces (split partials, stream-K pieces)
  // Streams of the host-buffer entry point (created on first use): uploads, GEMMs, downloads.
  cudaStream_t h2d = nullptr, compute = nullptr, d2h = nullptr;
  // Stream-K arrival counters: the device address of g_sk_counters (kSkRegions regions of
  // kSkRegionWords words, zero-filled at module load).  A region belongs to one stream at a
  // time, so launches that use it run in stream order and never overlap; each launch tags its
  // words with the region's next epoch.  Handing a region to another stream makes that stream
  // wait for the previous owner's work.
  unsigned int* sk_counters = nullptr;
  std::array<cudaStream_t, 16> sk_owner{};
  std::array<bool, 16> sk_owned{};
  std::array<unsigned int, 16> sk_epoch{};
  // Each region's stream-K workspace (the pieces' FP32 sums), from the pool, kept with the
  // region between launches (it moves between streams with the region) and grown when a
  // launch needs more: a launch in steady state queues no allocation or free around its kernel
  // (measured: the pool's allocate and free around each launch added 1.4 us to the 8-GPU slab).
  std::array<void*, 16> sk_ws{};
  std::array<size_t, 16> sk_ws_bytes{};
  int sk_next_victim = 0;
  cudaEvent_t sk_handoff = nullptr;
};
constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
DeviceState g_dev[kMaxDevices];

int device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MO_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceState& st = g_dev[dev];
  if (!st.ready) {
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return MO_ERR_DEVICE;
    st.sm_count = prop.multiProcessorCount;
    st.cc_major = prop.major;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_watchdog_flag) != cudaSuccess) return MO_ERR_DEVICE;
    st.watchdog = static_cast<int*>(p);
    // The stream-K arrival words and the event that hands a region to another stream are set
    // up here, once per device, so that no launch allocates or clears anything for them.
    if (cudaGetSymbolAddress(&p, g_sk_counters) != cudaSuccess ||
        cudaEventCreateWithFlags(&st.sk_handoff, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return MO_ERR_DEVICE;
    }
    st.sk_counters = static_cast<unsigned int*>(p);
    for (int v = 0; v < kNumVariants; ++v) {
      st.max_units[v] = st.sm_count / kVariants[v].cta_group;
    }
    st.ready = true;
  }
  *out = &st;
  return MO_OK;
}

// The library's own stream-ordered pool for per-call workspaces.  It keeps what it has
// mapped across synchronisations (release threshold: never), so a call after a
// cudaStreamSynchronize reuses memory instead of mapping it again; mo_release_workspace
// returns it.  Created on the first call that needs a workspace on this device.
int workspace_pool(DeviceState* st, cudaMemPool_t* out) {
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (st->pool == nullptr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MO_ERR_DEVICE;
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      cudaGetLastError();
      return MO_ERR_DEVICE;
    }
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    st->pool = pool;
  }
  *out = st->pool;
  return MO_OK;
}

// Stream-ordered workspace from the library's pool; nullptr when it cannot be had.
void* workspace_alloc(DeviceState* st, size_t bytes, cudaStream_t stream) {
  cudaMemPool_t pool = nullptr;
  if (workspace_pool(st, &pool) != MO_OK) return nullptr;
  void* p = nullptr;
  if (cudaMallocFromPoolAsync(&p, bytes, pool, stream) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

// Gives a launch on `stream` its stream-K counter region and epoch: the stream's own region,
// or a free one, or (round robin) one taken over from another stream after a wait for that
// stream's work.  The words are a device array set up with the device (device_state).  The
// region's workspace of at least `ws_bytes` comes with it (allocated, stream-ordered, only when
// the region has none that large yet).  Returns false when no region or workspace can be had
// without blocking the host; the caller then plans without stream-K (same bits).
bool acquire_sk_region(DeviceState* st, cudaStream_t stream, size_t ws_bytes,
                       unsigned int** counters, unsigned int* epoch, void** ws) {
  cudaMemPool_t pool = nullptr;
  if (workspace_pool(st, &pool) != MO_OK) return false;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (st->sk_counters == nullptr || st->sk_handoff == nullptr) return false;
  int region = -1;
  for (int r = 0; r < kSkRegions && region < 0; ++r) {
    if (st->sk_owned[r] && st->sk_owner[r] == stream) region = r;
  }
  for (int r = 0; r < kSkRegions && region < 0; ++r) {
    if (!st->sk_owned[r]) region = r;
  }
  if (region < 0) {
    region = st->sk_next_victim;
    st->sk_next_victim = (st->sk_next_victim + 1) % kSkRegions;
    // Everything queued so far on the previous owner (its last launch on this region
    // included) comes before this stream's use.
    if (cudaEventRecord(st->sk_handoff, st->sk_owner[region]) != cudaSuccess ||
        cudaStreamWaitEvent(stream, st->sk_handoff, 0) != cudaSuccess) {
      // The region stays with its owner; this launch runs without stream-K.
      cudaGetLastError();
      return false;
    }
  }
  st->sk_owned[region] = true;
  st->sk_owner[region] = stream;
  unsigned int* base = st->sk_counters + static_cast<size_t>(region) * kSkRegionWords;
  // Epochs 1 .. 2^24 - 1 (a word's top 24 bits); 0 is the zeroed state.  When a region's
  // epochs wrap it is zeroed on the stream, so no word from 2^24 launches ago can match.
  unsigned int& e = st->sk_epoch[region];
  const bool wrap = e >= 0xFFFFFFu;
  e = wrap ? 1u : e + 1u;
  if (wrap && cudaMemsetAsync(base, 0, sizeof(unsigned int) * kSkRegionWords, stream) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (st->sk_ws_bytes[region] < ws_bytes) {
    // The old buffer is freed on this stream, after every launch that used it: its own earlier
    // launches are ahead in the stream, and another owner's work was waited for above.
    if (st->sk_ws[region] != nullptr) cudaFreeAsync(st->sk_ws[region], stream);
    st->sk_ws[region] = nullptr;
    st->sk_ws_bytes[region] = 0;
    void* fresh = nullptr;
    if (cudaMallocFromPoolAsync(&fresh, ws_bytes, pool, stream) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    st->sk_ws[region] = fresh;
    st->sk_ws_bytes[region] = ws_bytes;
  }
  *counters = base;
  *epoch = e;
  *ws = st->sk_ws[region];
  return true;
}

constexpr double kStreamKFixupChunks = 1.25;  // fix-up cost of a split tile, in chunk-times
constexpr double kStreamKFixupSeconds = 2.0e-6;  // publish, counter and prefetch latency
constexpr double kSmFlopsPerSec = 2.25e15 / 148.0;  // dense BF16 per SM (nominal)
constexpr double kSmFeedBytesPerSec = 110e9;        // L2 -> one SM, sustained TMA
constexpr double kL2BytesPerSec = 24e12;            // L2 -> all SMs
constexpr double kHbmBytesPerSec = 3.5e12;           // effective, after the 256 MiB L2 flush
constexpr double kLoadLatencySeconds = 2.0e-6;      // TMA load round trip under load (measured)
constexpr double kLaunchSeconds = 4.0e-6;           // an extra dependent kernel launch

int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// Chunk length (K blocks) of the two-level accumulation for a given K: 29 up to K = 7424,
// then 29 x sqrt(7424 / K), at least 2.  Depends on K alone, so every kernel variant and every
// N shard of one problem uses the same chunks.
int chunk_blocks_for_k(int k) {
  if (k <= 7424) return kMaxChunkKBlocks;
  const int b = static_cast<int>(std::floor(kMaxChunkKBlocks * std::sqrt(7424.0 / k)));
  return std::max(2, std::min(kMaxChunkKBlocks, b));
}

// A stream-K plan: `dp` whole tiles per cluster, then the K chunks of the tiles left over
// (tiles % clusters of them) dealt out as contiguous ranges over as few clusters as keep the
// busiest at `per` chunks (fewer pieces per split tile, so less to write, read back and sum).
struct SkPlan {
  int dp = 0, sk_tile0 = 0, units = 0, per = 0, clusters = 0;
};

// Plans stream-K for `tiles` tiles on `clusters` clusters; false when nothing is left over, K has
// a single chunk, or (need_wave) there is no whole wave before the leftover: without one every
// tile would be split and pay the fix-up (measured: slower than whole tiles on an M = 256
// problem), so the model asks for one; a forced stream-K (MO_GEMM_STREAMK=1) also runs without.
bool plan_stream_k(int tiles, int clusters, int nchunks, bool need_wave, SkPlan* out) {
  if (nchunks < 2 || clusters <= 0 || (need_wave && tiles < clusters)) return false;
  const int rem = tiles % clusters;
  if (rem == 0) return false;
  const long long units = static_cast<long long>(rem) * nchunks;
  if (units >= (1ll << 24)) return false;
  SkPlan p;
  p.dp = tiles / clusters;
  p.sk_tile0 = p.dp * clusters;
  p.units = static_cast<int>(units);
  p.per = static_cast<int>((units + clusters - 1) / clusters);
  p.clusters = static_cast<int>((units + p.per - 1) / p.per);
  *out = p;
  return true;
}

// Work schedules: whole tiles; K split into (tile, chunk) units plus an ordered reduce;
// whole-tile waves then stream-K pieces of the leftover tiles.
enum Schedule { kWholeTiles = 0, kSplitK = 1, kStreamK = 2 };

struct Estimate {
  double seconds;
  int tiles;
  int units;    // work units (tiles, or tile x chunk when split)
  int running;  // units running at once
};

// Rows of C per CTA tile.  A tile of a problem taller than one CTA's 128 rows holds, per CTA, the
// least multiple of 32 rows that keeps the number of row tiles, so no CTA loads the A rows of the
// next tile: 1-CTA tiles at M = 129 hold 96 and 33 rows, not 128 and 1 (the busier CTAs load 28 KB
// per K block instead of 32), and a CTA pair at M = 129 holds 2 x 96 rows in one row band instead
// of 2 x 128.  At most 128 rows a 1-CTA tile is one tile whose A box is trimmed instead.
int tile_rows_for(int m, int cta_group) {
  if (cta_group == 1 && m <= kRowsPerCta) return kRowsPerCta;
  const int tiles = ceil_div(m, kRowsPerCta * cta_group);
  for (int h = 32; h < kRowsPerCta; h += 32) {
    if (ceil_div(m, h * cta_group) == tiles) return h;
  }
  return kRowsPerCta;
}

// Rows per A TMA box: the tile's rows, or M rounded up to 8 below 128 rows (1-CTA).
int a_box_rows_for(int m, int cta_group) {
  return (cta_group == 1 && m < kRowsPerCta) ? std::max(8, (m + 7) / 8 * 8)
                                             : tile_rows_for(m, cta_group);
}

// Analytic cost model.  A unit's time is the slower of its tensor-core time (scaled by the
// sustained efficiency of the tile shape) and its operand feed, where one SM's feed is bounded
// by the bytes its pipeline keeps in flight over the load latency; units run in waves of
// `running`.  The result is the slowest of that, the aggregate L2 feed and the compulsory HBM
// traffic, plus, when split, the partials' round trip and the reduce launch.
Estimate estimate(int m, int n, int k, int num_units, const VariantInfo& v, Schedule sched) {
  const bool split = sched == kSplitK;
  const int tile_m = tile_rows_for(m, v.cta_group) * v.cta_group;
  const int tile_n = v.block_n_cta * v.cta_group;
  const long long tiles = static_cast<long long>(ceil_div(m, tile_m)) * ceil_div(n, tile_n);
  const int nkb = ceil_div(k, kBlockK);
  const int nchunks = ceil_div(nkb, chunk_blocks_for_k(k));
  const long long units = split ? tiles * nchunks : tiles;
  const double kp_unit = static_cast<double>(nkb) * kBlockK / (split ? nchunks : 1);
  const long long waves = (units + num_units - 1) / num_units;
  const int a_rows = a_box_rows_for(m, v.cta_group);
  const double sm_flops = 2.0 * kRowsPerCta * tile_n * kp_unit;             // per SM per unit
  // Bytes the TMA unit moves into one SM per unit, zero-filled out-of-bounds rows included.
  const double sm_bytes = (a_rows + v.block_n_cta) * kp_unit * 2.0;
  const double in_flight = v.stages * (a_rows + v.block_n_cta) * kBlockK * 2.0;
  const double feed_bw = std::min(kSmFeedBytesPerSec, in_flight / kLoadLatencySeconds);
  const double t_unit = std::max(sm_flops / (kSmFlopsPerSec * v.mma_efficiency), sm_bytes / feed_bw);
  const double t_l2 = units * v.cta_group * sm_bytes / kL2BytesPerSec;
  double t_hbm = 2.0 * (static_cast<double>(m) * k + static_cast<double>(k) * n +
                        static_cast<double>(m) * n) /
                 kHbmBytesPerSec;
  double t_reduce = 0.0;
  if (split) {
    const double mn = static_cast<double>(m) * n;
    t_hbm += nchunks * 4.0 * mn / kHbmBytesPerSec;                       // partial writes
    t_reduce = (nchunks * 4.0 + 2.0) * mn / kHbmBytesPerSec + kLaunchSeconds;
  }
  double t_compute = waves * t_unit;
  if (sched == kStreamK) {
    // Whole-tile waves, then the busiest cluster's chunks of the leftover tiles, then the
    // fix-up: the pieces' FP32 results written, read back and summed (in proportion to the
    // tile rows inside C), plus the publish and prefetch latency.
    SkPlan sk;
    plan_stream_k(static_cast<int>(std::min<long long>(tiles, INT32_MAX)), num_units, nchunks, false, &sk);
    const double t_chunk = t_unit / nchunks;
    const double rows_in_c = std::min(1.0, static_cast<double>(m) / tile_m);
    t_compute = static_cast<double>(tiles / num_units) * t_unit + sk.per * t_chunk +
                kStreamKFixupChunks * t_chunk * rows_in_c + kStreamKFixupSeconds;
  }
  Estimate e;
  e.seconds = std::max(std::max(t_compute, t_l2), t_hbm) + t_reduce;
  e.tiles = static_cast<int>(std::min<long long>(tiles, INT32_MAX));
  e.units = static_cast<int>(std::min<long long>(units, INT32_MAX));
  e.running = static_cast<int>(std::min<long long>(units, num_units));
  return e;
}

struct Choice {
  int var;
  bool split;
  bool stream_k;
};

// split_mode / streamk_mode: -1 = the model decides, 0 = never, 1 = whenever the shape allows
// (K split: K has more than one chunk; stream-K: a partial last wave and no forced split).
Choice select_variant(int m, int n, int k, int num_sms, int forced_tile_n, int split_mode,
                      int forced_variant = -1, int streamk_mode = -1) {
  Choice best{-1, false, false};
  double best_t = std::numeric_limits<double>::infinity();
  // Skinny A (one band of 256-row pair tiles, fewer tiles than clusters, at most 4 K chunks and at
  // least 2 per cluster): stream-K over every cluster without a whole wave first.  The model puts
  // these shapes at the HBM term whatever the plan, so it cannot rank them; measured with a
  // flush before each launch, the spread plan beat the model's whole-tile pick by 8-14 % at
  // M = 129-256 with N = 5120-8192, K = 7232 (M = 129, N = 7776: 46.0 -> 42.2 us), was level at
  // N = 12288-16384, K = 2048-7232, and lost with 256 x 128 pair tiles (M = 512, N = 2048:
  // +9 %) or with more chunks (K = 16384: +24 %).  Such a plan, within 3 % of the model's best,
  // is taken.
  Choice spread{-1, false, true};
  double spread_t = std::numeric_limits<double>::infinity();
  const int nchunks = ceil_div(ceil_div(k, kBlockK), chunk_blocks_for_k(k));
  const bool multi_chunk = nchunks > 1;
  for (int sc = kWholeTiles; sc <= kStreamK; ++sc) {
    const Schedule sched = static_cast<Schedule>(sc);
    if (sched == kSplitK && (!multi_chunk || split_mode == 0)) continue;
    if (sched != kSplitK && split_mode == 1 && multi_chunk) continue;
    if (sched == kStreamK && (streamk_mode == 0 || split_mode == 1)) continue;
    for (int v = 0; v < kNumVariants; ++v) {
      const VariantInfo& vi = kVariants[v];
      const int tile_n = vi.block_n_cta * vi.cta_group;
      if (forced_tile_n > 0 && tile_n != forced_tile_n) continue;
      if (forced_variant >= 0 && v != forced_variant) continue;
      // A CTA pair only pays off when A has more rows than one CTA holds.
      if (forced_variant < 0 && vi.cta_group == 2 && m <= kRowsPerCta) continue;
      const int clusters = num_sms / vi.cta_group;
      const long long tiles = static_cast<long long>(ceil_div(m, kRowsPerCta * vi.cta_group)) *
                              ceil_div(n, tile_n);
      const bool skinny_spread = vi.cta_group == 2 && vi.block_n_cta == 128 && nchunks <= 4 &&
                                 tiles < clusters && tiles * nchunks > clusters;
      SkPlan sk_probe;
      const bool sk_possible = plan_stream_k(static_cast<int>(std::min<long long>(tiles, INT32_MAX)),
                                             clusters, nchunks, streamk_mode != 1 && !skinny_spread,
                                             &sk_probe);
      if (sched == kStreamK && !sk_possible) continue;
      if (sched == kWholeTiles && streamk_mode == 1 && sk_possible && split_mode != 1) continue;
      const double t = estimate(m, n, k, clusters, vi, sched).seconds;
      if (sched == kStreamK && skinny_spread && t < spread_t) {
        spread_t = t;
        spread.var = v;
      }
      if (best.var < 0 || t < best_t * 0.97) {  // earlier (larger, unsplit) choices win near-ties
        best_t = t;
        best = {v, sched == kSplitK, sched == kStreamK};
      }
    }
  }
  if (best.var < 0) best = {kVarPair256, false, false};
  if (spread.var >= 0 && !best.stream_k && spread_t <= best_t * 1.03) best = spread;
  return best;
}

void fill_plan(int m, int n, int k, int num_units, Choice c, mo_gemm_plan* out) {
  const VariantInfo& v = kVariants[c.var];
  const Estimate e = estimate(m, n, k, num_units, v, c.split ? kSplitK : kWholeTiles);
  out->block_m = tile_rows_for(m, v.cta_group) * v.cta_group;
  out->block_n = v.block_n_cta * v.cta_group;
  out->block_k = kBlockK;
  out->stages = v.stages;
  out->cta_group = v.cta_group;
  out->num_tiles = e.tiles;
  out->grid = e.running * v.cta_group;
  out->smem_bytes = v.smem;
  out->num_chunks = ceil_div(ceil_div(k, kBlockK), chunk_blocks_for_k(k));
  out->split = c.split ? 1 : 0;
  out->stream_k = 0;
  SkPlan sk;
  if (c.stream_k && plan_stream_k(out->num_tiles, num_units, out->num_chunks, false, &sk)) {
    out->stream_k = 1;
    out->grid = num_units * v.cta_group;
  }
}



// MO_GEMM_VARIANT: forces the kernel variant ("pair256", "1x256", "1x128", "1x64" or "pair128"); unset or
// empty lets the cost model choose.  Every variant computes the same bits, so this is a tuning
// and testing knob only.  Returns the variant index, -1 (unset) or -2 (invalid).
int parse_variant_override() {
  const char* raw = std::getenv("MO_GEMM_VARIANT");
  if (raw == nullptr || raw[0] == '\0') return -1;
  static const char* const kNames[kNumVariants] = {"pair256", "1x256", "1x128", "1x64", "pair128"};
  for (int v = 0; v < kNumVariants; ++v) {
    if (std::strcmp(raw, kNames[v]) == 0) return v;
  }
  std::fprintf(stderr, "Unsupported MO_GEMM_VARIANT value '%s'; expected pair256, 1x256, 1x128, 1x64 or pair128.\n",
               raw);
  return -2;
}

// MO_GEMM_STREAMK: "0" never uses the stream-K schedule, "1" uses it whenever the last wave of
// tiles is partial; unset or empty lets the library decide.  Same bits either way.
int parse_streamk_override() {
  const char* raw = std::getenv("MO_GEMM_STREAMK");
  if (raw == nullptr || raw[0] == '\0') return -1;
  if (raw[0] == '0' && raw[1] == '\0') return 0;
  if (raw[0] == '1' && raw[1] == '\0') return 1;
  std::fprintf(stderr, "Unsupported MO_GEMM_STREAMK value '%s'; expected 0 or 1.\n", raw);
  return -2;
}

// MO_GEMM_SPLIT: "0" never splits K across CTAs, "1" always does when K has more than one
// accumulation chunk; unset or empty lets the cost model decide.  Split and unsplit runs give
// identical bits (the same chunk partials summed in the same order), so this only moves time.
int parse_split_override() {
  const char* raw = std::getenv("MO_GEMM_SPLIT");
  if (raw == nullptr || raw[0] == '\0') return -1;
  if (raw[0] == '0' && raw[1] == '\0') return 0;
  if (raw[0] == '1' && raw[1] == '\0') return 1;
  std::fprintf(stderr, "Unsupported MO_GEMM_SPLIT value '%s'; expected 0 or 1.\n", raw);
  return -2;
}

constexpr int kHeroM = 6464, kHeroN = 7776, kHeroK = 7232;

// MATMUL_FIXED_MAIN_TILE_N: the reference's tile override for the hero shape
// (src/kernels/bf16_gemm_v1.cu:159, :1194-1269).  The reference accepts the widths its sweep
// tool iterates (scripts/sweep_fixed_main_tiles.py:20): 32, 64, 96, 128, 160, 192, 256, 320,
// 384 and 480.  This kernel family has tiles 64, 128 and 256 wide (256 = the CTA pair or the
// 1-CTA 256 variant), so each reference width runs the widest of them that is no wider than it
// (32 runs 64, the narrowest): 32, 64, 96 -> 64; 128, 160, 192 -> 128; 256, 320, 384, 480 ->
// 256.  A width that is mapped is named once per process on stderr.  Every width gives the same
// bits.  Unset or empty means the analytic choice; any other value is an error, as in the
// reference.  Returns 0 (no override), the tile width to run, or -1 (invalid).
int tile_width_for_reference_width(int w) {
  switch (w) {
    case 32: case 64: case 96: return 64;
    case 128: case 160: case 192: return 128;
    case 256: case 320: case 384: case 480: return 256;
    default: return -1;
  }
}

int parse_tile_override() {
  const char* raw = std::getenv("MATMUL_FIXED_MAIN_TILE_N");
  if (raw == nullptr || raw[0] == '\0') return 0;
  char* end = nullptr;
  const long v = std::strtol(raw, &end, 10);
  const int width = (end == raw || *end != '\0' || v <= 0 || v > 480)
                        ? -1 : tile_width_for_reference_width(static_cast<int>(v));
  if (width < 0) {
    std::fprintf(stderr,
                 "Unsupported MATMUL_FIXED_MAIN_TILE_N value '%s'; expected one of 32, 64, 96, 128, "
                 "160, 192, 256, 320, 384, 480.\n",
                 raw);
    return -1;
  }
  if (width != v) {
    static std::mutex note_mutex;
    static bool noted[481] = {};
    std::lock_guard<std::mutex> lock(note_mutex);
    if (!noted[v]) {
      noted[v] = true;
      std::fprintf(stderr, "MATMUL_FIXED_MAIN_TILE_N=%ld runs the %d-column tile of the sm_100a kernel.\n", v,
                   width);
    }
  }
  return width;
}

template <int CG, int BN_CTA, int STAGES>
int init_variant(DeviceState* st, int var) {
  using G = Geometry<CG, BN_CTA, STAGES>;
  auto kernel = gemm_bf16_sm100_kernel<CG, BN_CTA, STAGES>;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (st->attr_done[var]) return MO_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           G::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return MO_ERR_LAUNCH;
  }
  if constexpr (CG == 2) {
    // Co-resident CTA pairs on this device: the persistent grid is exactly this many, since
    // the work-unit schedule assumes every cluster of the grid runs.
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (st->sm_count / 2), 1, 1);
    cfg.blockDim = dim3(kNumThreads, 1, 1);
    cfg.dynamicSmemBytes = G::kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess && clusters > 0) {
      st->max_units[var] = std::min(st->max_units[var], clusters);
    }
    cudaGetLastError();
  }
  st->attr_done[var] = true;
  return MO_OK;
}

// Launches num_clusters persistent clusters; prepare_gemm sized them from the co-resident
// count found by init_variant.
template <int CG, int BN_CTA, int STAGES>
int launch_variant(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                   const GemmArgs& args, cudaStream_t stream) {
  using G = Geometry<CG, BN_CTA, STAGES>;
  auto kernel = gemm_bf16_sm100_kernel<CG, BN_CTA, STAGES>;
  const int grid = args.num_clusters * CG;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  cfg.stream = stream;
  int num_attrs = 0;
  if constexpr (CG == 2) {
    attr[num_attrs].id = cudaLaunchAttributeClusterDimension;
    attr[num_attrs].val.clusterDim.x = 2;
    attr[num_attrs].val.clusterDim.y = 1;
    attr[num_attrs].val.clusterDim.z = 1;
    ++num_attrs;
  }
  // Programmatic dependent launch: when the previous work in the stream is a kernel, this one
  // may be launched and set up (barriers, TMEM) while that kernel drains; the kernel waits for
  // it (griddepcontrol.wait) before touching global memory.  Measured on back-to-back calls:
  // 1000^3 12.6 -> 10.0 us, M = 16 27.0 -> 24.2 us, the 8-GPU slab 76.9 -> 74.7 us.
  attr[num_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[num_attrs].val.programmaticStreamSerializationAllowed = 1;
  ++num_attrs;
  cfg.attrs = attr;
  cfg.numAttrs = num_attrs;
  if (cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, args) != cudaSuccess) {
    cudaGetLastError();
    return MO_ERR_LAUNCH;
  }
  return cudaGetLastError() == cudaSuccess ? MO_OK : MO_ERR_LAUNCH;
}

constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;  // 2 s per wait

// Everything a launch needs, decided on the host: plan, tensor maps and kernel arguments.
struct Prepared {
  Choice choice{};
  mo_gemm_plan plan{};
  CUtensorMap ta{}, tb{}, tc{};
  GemmArgs args{};
  DeviceState* st = nullptr;
  size_t workspace_bytes = 0;  // FP32 chunk partials when split, else 0
  size_t sk_bytes = 0;         // stream-K workspace (piece slots), else 0
};

// Kernel arguments of a plan, all but the C pointer and the watchdog word: tile counts, chunks,
// the stream-K schedule (when the plan asks for it and it fits; else plan->stream_k is cleared)
// and the workspace sizes.  `clusters` is the co-resident cluster count.  Needs no device, so
// mo_gemm_schedule can list a plan's work units on the host.
void fill_args(int m, int n, int k, int clusters, mo_gemm_plan* plan, GemmArgs* out,
               size_t* workspace_bytes, size_t* sk_bytes) {
  GemmArgs& args = *out;
  args = GemmArgs{};
  args.m = m;
  args.n = n;
  args.k = k;
  args.num_m_blocks = ceil_div(m, plan->block_m);
  args.num_n_blocks = ceil_div(n, plan->block_n);
  args.num_k_blocks = ceil_div(k, kBlockK);
  args.num_tiles = plan->num_tiles;
  args.num_chunks = plan->num_chunks;
  args.split = plan->split;
  args.num_units = args.split ? args.num_tiles * args.num_chunks : args.num_tiles;
  args.a_box_rows = a_box_rows_for(m, plan->cta_group);
  args.tile_rows = tile_rows_for(m, plan->cta_group);
  // With A trimmed below 128 rows the kernel is an HBM stream of B; measured on M = 1 and 16
  // (N = 7776, K = 7232): 8 K blocks ahead takes 40 us to 32 us; on L2-resident shapes it only
  // adds traffic, so it stays off there.
  args.l2_prefetch_kb = (plan->cta_group == 1 && m < kRowsPerCta) ? 8 : 0;
  // Raster group height.  Pairs use 8 M-blocks, except on narrow N (at most 8 pair columns,
  // the N-sharded slabs of a 7776-wide GEMM on 4 and 8 GPUs), where 4 measured 2 us faster on
  // 6464x976x7232 (69.7 against 71.7 us) and 1 us on 6464x1952x7232; on the full 6464x7776x7232
  // 4 is 1.5-3 % slower than 8.
  args.group_m = plan->cta_group == 2 ? (args.num_n_blocks <= 8 ? 4 : 8) : 16;
  args.timeout_ns = kDefaultTimeoutNs;
  *sk_bytes = 0;
  *workspace_bytes =
      args.split ? static_cast<size_t>(args.num_chunks) * m * static_cast<size_t>(n) * sizeof(float) : 0;
  args.num_clusters = plan->grid / plan->cta_group;
  SkPlan sk;
  bool use_sk = plan->stream_k && plan_stream_k(args.num_tiles, clusters, args.num_chunks, false, &sk);
  if (use_sk && (args.num_tiles % clusters) * plan->cta_group > kSkRegionWords) use_sk = false;
  if (!use_sk) plan->stream_k = 0;
  if (use_sk) {
    args.sk = 1;
    args.num_clusters = clusters;
    args.dp_per_cluster = sk.dp;
    args.sk_tile0 = sk.sk_tile0;
    const int sk_tiles = args.num_tiles - args.sk_tile0;
    args.sk_units = sk.units;
    args.sk_clusters = sk.clusters;
    plan->grid = clusters * plan->cta_group;
    const size_t slot = static_cast<size_t>(kRowsPerCta) * plan->block_n * sizeof(float);
    *sk_bytes = static_cast<size_t>(sk_tiles) * plan->cta_group * (args.num_chunks + 1) * slot;
  }
}

// split_mode: -1 = cost model (after MO_GEMM_SPLIT), 0 = never split, 1 = split if possible.
int prepare_gemm(const uint16_t* a, const uint16_t* b, uint16_t* c, int m, int n, int k,
                 int split_mode, Prepared* p, int streamk_mode = -1) {
  if (a == nullptr || b == nullptr || c == nullptr) return MO_ERR_NULL_POINTER;
  if (m <= 0 || n <= 0 || k <= 0) return MO_ERR_BAD_DIMS;
  // TMA needs 16-byte aligned bases and 16-byte multiple row strides.
  if ((k % 8) != 0 || (n % 8) != 0) return MO_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(c)) & 15u) {
    return MO_ERR_UNSUPPORTED;
  }
  int forced = 0;
  if (m == kHeroM && n == kHeroN && k == kHeroK) {
    forced = parse_tile_override();
    if (forced < 0) return MO_ERR_BAD_ARGUMENT;
  }
  if (split_mode == -1) {
    split_mode = parse_split_override();
    if (split_mode == -2) return MO_ERR_BAD_ARGUMENT;
  }
  const int forced_variant = parse_variant_override();
  if (forced_variant == -2) return MO_ERR_BAD_ARGUMENT;
  if (streamk_mode == -1) {
    streamk_mode = parse_streamk_override();
    if (streamk_mode == -2) return MO_ERR_BAD_ARGUMENT;
  }
  const int rc = device_state(&p->st);
  if (rc != MO_OK) return rc;
  if (p->st->cc_major != 10) return MO_ERR_DEVICE;

  p->choice = select_variant(m, n, k, p->st->sm_count, forced, split_mode, forced_variant, streamk_mode);
  int irc;
  switch (p->choice.var) {
    case kVarPair256: irc = init_variant<2, 128, 6>(p->st, p->choice.var); break;
    case kVar1x256: irc = init_variant<1, 256, 4>(p->st, p->choice.var); break;
    case kVar1x128: irc = init_variant<1, 128, 6>(p->st, p->choice.var); break;
    case kVarPair128: irc = init_variant<2, 64, 8>(p->st, p->choice.var); break;
    default: irc = init_variant<1, 64, 8>(p->st, p->choice.var); break;
  }
  if (irc != MO_OK) return irc;
  fill_plan(m, n, k, p->st->max_units[p->choice.var], p->choice, &p->plan);
  const int a_rows = a_box_rows_for(m, p->plan.cta_group);
  if (!make_tmap_2d(&p->ta, a, m, k, a_rows, kBlockK)) return MO_ERR_LAUNCH;
  if (!make_tmap_2d(&p->tb, b, k, n, kBlockK, 64)) return MO_ERR_LAUNCH;
  if (!make_tmap_2d(&p->tc, c, m, n, kStoreBox, kStoreBox, CU_TENSOR_MAP_SWIZZLE_64B)) {
    return MO_ERR_LAUNCH;
  }
  fill_args(m, n, k, p->st->max_units[p->choice.var], &p->plan, &p->args, &p->workspace_bytes,
            &p->sk_bytes);
  p->args.c = c;
  p->args.watchdog = p->st->watchdog;
  return MO_OK;
}

// FP32 chunk partials -> BF16 C: acc = p0, then acc = acc + p_c in chunk order, then RNE,
// exactly the unsplit kernel's epilogue arithmetic.  mn is a multiple of 4 (n % 8 == 0).
__global__ void reduce_chunks_kernel(const float* __restrict__ partials, uint16_t* __restrict__ c,
                                     long long mn, int nchunks) {
  const long long groups = mn / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < groups;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(partials)[i];
    for (int ch = 1; ch < nchunks; ++ch) {
      const float4 v = reinterpret_cast<const float4*>(partials + ch * mn)[i];
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    reinterpret_cast<uint2*>(c)[i] = make_uint2(bf16x2_rne(acc.x, acc.y), bf16x2_rne(acc.z, acc.w));
  }
}

// dst[r][c] = src[r * src_pitch + c] inside the rows x cols source, 0 in the rest of the
// drows x dcols destination (row pitch dcols).  Copies matrices into and out of the padded
// buffers of launch_padded; HBM-bound, 2-byte accesses (the source may sit at any even address).
__global__ void pad_copy_kernel(const uint16_t* __restrict__ src, int rows, int cols,
                                long long src_pitch, uint16_t* __restrict__ dst, int drows,
                                int dcols) {
  const long long total = static_cast<long long>(drows) * dcols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / dcols);
    const int c = static_cast<int>(i - static_cast<long long>(r) * dcols);
    dst[i] = (r < rows && c < cols) ? src[r * src_pitch + c] : static_cast<uint16_t>(0);
  }
}

int pad_copy(const uint16_t* src, int rows, int cols, long long src_pitch, uint16_t* dst,
             int drows, int dcols, int sm_count, cudaStream_t stream) {
  const long long total = static_cast<long long>(drows) * dcols;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 8LL * sm_count));
  pad_copy_kernel<<<blocks, 256, 0, stream>>>(src, rows, cols, src_pitch, dst, drows, dcols);
  return cudaGetLastError() == cudaSuccess ? MO_OK : MO_ERR_LAUNCH;
}

// Launches the prepared GEMM; when split, `workspace` holds workspace_bytes of device memory
// and a reduce kernel follows on the same stream.
int run_prepared(Prepared& p, float* workspace, cudaStream_t stream) {
  if (p.args.split) {
    if (workspace == nullptr) return MO_ERR_NULL_POINTER;
    p.args.partials = workspace;
  }
  int rc;
  switch (p.choice.var) {
    case kVarPair256: rc = launch_variant<2, 128, 6>(p.ta, p.tb, p.tc, p.args, stream); break;
    case kVar1x256: rc = launch_variant<1, 256, 4>(p.ta, p.tb, p.tc, p.args, stream); break;
    case kVar1x128: rc = launch_variant<1, 128, 6>(p.ta, p.tb, p.tc, p.args, stream); break;
    case kVarPair128: rc = launch_variant<2, 64, 8>(p.ta, p.tb, p.tc, p.args, stream); break;
    default: rc = launch_variant<1, 64, 8>(p.ta, p.tb, p.tc, p.args, stream); break;
  }
  if (rc != MO_OK || !p.args.split) return rc;
  const long long mn = static_cast<long long>(p.args.m) * p.args.n;
  const int blocks = static_cast<int>(std::min<long long>((mn / 4 + 255) / 256, 4LL * p.st->sm_count));
  reduce_chunks_kernel<<<blocks, 256, 0, stream>>>(workspace, p.args.c, mn, p.args.num_chunks);
  return cudaGetLastError() == cudaSuccess ? MO_OK : MO_ERR_LAUNCH;
}

// Device address of g_noalloc_scratch on the current device.  In host code the array's name
// only stands for the symbol, so the address comes from cudaGetSymbolAddress, looked up once
// per device (with that device current) and cached in its DeviceState.
int noalloc_scratch(DeviceState* st, float** out) {
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (st->noalloc_scratch == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return MO_ERR_DEVICE;
    }
    st->noalloc_scratch = static_cast<float*>(p);
  }
  *out = st->noalloc_scratch;
  return MO_OK;
}

int launch_padded(const uint16_t* a, const uint16_t* b, uint16_t* c, int m, int n, int k,
                  cudaStream_t stream);

int launch_gemm(const uint16_t* a, const uint16_t* b, uint16_t* c, int m, int n, int k,
                cudaStream_t stream) {
  if (a == nullptr || b == nullptr || c == nullptr) return MO_ERR_NULL_POINTER;
  if (m <= 0 || n <= 0 || k <= 0) return MO_ERR_BAD_DIMS;
  // TMA needs 16-byte aligned bases and row strides that are multiples of 16 bytes.
  if ((k % 8) != 0 || (n % 8) != 0 ||
      ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
        reinterpret_cast<uintptr_t>(c)) & 15u) != 0) {
    return launch_padded(a, b, c, m, n, k, stream);
  }
  // A launch captured into a CUDA graph replays with the arguments it was captured with, so it
  // cannot use the device's epoch-tagged stream-K arrival words: every replay would reuse one
  // epoch and count the previous replay's arrivals.  A captured launch gets arrival words of its
  // own instead, taken from the pool with its workspace and zeroed on the stream before the
  // kernel (both recorded into the graph), and counts them with epoch 1.
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
    cudaGetLastError();
    capture = cudaStreamCaptureStatusNone;
  }
  const bool captured = capture != cudaStreamCaptureStatusNone;
  Prepared p;
  int rc = prepare_gemm(a, b, c, m, n, k, -1, &p);
  if (rc != MO_OK) return rc;
  float* ws = nullptr;
  if (p.workspace_bytes > 0) {
    // Stream-ordered workspace for the chunk partials, freed on the same stream after the
    // reduce.  If it cannot be had, the unsplit kernel computes the same bits without it.
    ws = static_cast<float*>(workspace_alloc(p.st, p.workspace_bytes, stream));
    if (ws == nullptr) {
      rc = prepare_gemm(a, b, c, m, n, k, 0, &p);
      if (rc != MO_OK) return rc;
    }
  }
  char* sk = nullptr;        // a captured launch's own stream-K workspace, freed after it
  bool have_sk = false;
  if (p.sk_bytes > 0) {
    // Stream-K workspace (the pieces' FP32 results) and arrival words: the region's kept
    // workspace and epoch-tagged words, or under capture the launch's own workspace and zeroed
    // words from the pool.  Without either the plain schedule computes the same bits.
    if (captured) {
      const size_t own_words = sizeof(unsigned int) * kSkRegionWords;
      sk = static_cast<char*>(workspace_alloc(p.st, p.sk_bytes + own_words, stream));
      if (sk != nullptr) {
        unsigned int* words = reinterpret_cast<unsigned int*>(sk + p.sk_bytes);
        have_sk = cudaMemsetAsync(words, 0, own_words, stream) == cudaSuccess;
        p.args.sk_counters = words;
        p.args.sk_epoch = 1;
        p.args.sk_ws = reinterpret_cast<float*>(sk);
        if (!have_sk) {
          cudaGetLastError();
          cudaFreeAsync(sk, stream);
          sk = nullptr;
        }
      }
    } else {
      void* kept = nullptr;
      have_sk = acquire_sk_region(p.st, stream, p.sk_bytes, &p.args.sk_counters, &p.args.sk_epoch, &kept);
      p.args.sk_ws = static_cast<float*>(kept);
    }
    if (!have_sk) {
      rc = prepare_gemm(a, b, c, m, n, k, 0, &p, 0);
      if (rc != MO_OK) return rc;
    }
  }
  rc = run_prepared(p, ws, stream);
  if (ws != nullptr && cudaFreeAsync(ws, stream) != cudaSuccess && rc == MO_OK) rc = MO_ERR_LAUNCH;
  if (sk != nullptr && cudaFreeAsync(sk, stream) != cudaSuccess && rc == MO_OK) rc = MO_ERR_LAUNCH;
  return rc;
}

// Layouts TMA cannot describe -- k or n not a multiple of 8, or a pointer off a 16-byte
// boundary -- still run on the tensor cores: A and B are copied into aligned buffers with k and n
// rounded up to multiples of 8 (zeros in the padding), the GEMM runs on those, and C is copied
// back without its padding columns.  The padded K columns are zeros inside the last K block,
// like the zeros TMA fills in out of bounds, so they add nothing to any sum.  The reference takes
// its scalar fallback kernel for these layouts (src/kernels/bf16_gemm_v1.cu:2173-2177).  The
// buffers come from the library's pool, stream-ordered like the other workspaces.
int launch_padded(const uint16_t* a, const uint16_t* b, uint16_t* c, int m, int n, int k,
                  cudaStream_t stream) {
  // A uint16_t array at an odd address is not a BF16 matrix.
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(c)) & 1u) {
    return MO_ERR_UNSUPPORTED;
  }
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc != MO_OK) return rc;
  if (st->cc_major != 10) return MO_ERR_DEVICE;
  const int k8 = (k + 7) / 8 * 8;
  const int n8 = (n + 7) / 8 * 8;
  auto up256 = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t a_bytes = up256(static_cast<size_t>(m) * k8 * 2);
  const size_t b_bytes = up256(static_cast<size_t>(k8) * n8 * 2);
  const size_t c_bytes = up256(static_cast<size_t>(m) * n8 * 2);
  char* dev = static_cast<char*>(workspace_alloc(st, a_bytes + b_bytes + c_bytes, stream));
  if (dev == nullptr) return MO_ERR_NO_MEMORY;
  uint16_t* a_p = reinterpret_cast<uint16_t*>(dev);
  uint16_t* b_p = reinterpret_cast<uint16_t*>(dev + a_bytes);
  uint16_t* c_p = reinterpret_cast<uint16_t*>(dev + a_bytes + b_bytes);
  rc = pad_copy(a, m, k, k, a_p, m, k8, st->sm_count, stream);
  if (rc == MO_OK) rc = pad_copy(b, k, n, n, b_p, k8, n8, st->sm_count, stream);
  if (rc == MO_OK) rc = launch_gemm(a_p, b_p, c_p, m, n8, k8, stream);
  if (rc == MO_OK) rc = pad_copy(c_p, m, n, n8, c, m, n, st->sm_count, stream);
  if (cudaFreeAsync(dev, stream) != cudaSuccess && rc == MO_OK) rc = MO_ERR_LAUNCH;
  return rc;
}

// Host-buffer GEMM.  A goes up first (every column slab of C needs all of it); then B goes up
// in column slabs (2-D copies into contiguous slab buffers), each slab's GEMM starts as soon as
// its columns have landed, and each slab of C comes back (a 2-D copy into the row-major host C)
// while later slabs compute.  Uploads, GEMMs and downloads run on three streams of their own,
// so both PCIe directions and the tensor cores work at once, and the first slab of C starts
// down after A plus one B slab instead of after all of B.  The caller's stream waits for the
// last download.  The slab GEMMs sum exactly what the whole GEMM sums (chunks depend on K
// alone), so C is bit-identical to mo_launch_bf16_gemm_v1 on device copies of A and B.
// `a_on_device`: A is already resident on the device (for example gathered from the other
// ranks over NVLink); only B and C cross PCIe then.
int gemm_from_host(const uint16_t* a_h, const uint16_t* b_h, uint16_t* c_h, int m, int n, int k,
                   int slabs, cudaStream_t stream, bool a_on_device = false) {
  if (a_h == nullptr || b_h == nullptr || c_h == nullptr) return MO_ERR_NULL_POINTER;
  if (a_on_device && (reinterpret_cast<uintptr_t>(a_h) & 15u)) return MO_ERR_UNSUPPORTED;
  if (m <= 0 || n <= 0 || k <= 0) return MO_ERR_BAD_DIMS;
  if (slabs < 0) return MO_ERR_BAD_ARGUMENT;
  if ((k % 8) != 0 || (n % 8) != 0) return MO_ERR_UNSUPPORTED;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc != MO_OK) return rc;
  if (st->cc_major != 10) return MO_ERR_DEVICE;
  {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    for (cudaStream_t* sp : {&st->h2d, &st->compute, &st->d2h}) {
      if (*sp == nullptr && cudaStreamCreateWithFlags(sp, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        *sp = nullptr;
        return MO_ERR_DEVICE;
      }
    }
  }
  // Column slabs of a multiple of 16 columns (TMA row pitch).  Measured on the hero shape
  // (PCIe 55 GB/s up and 57 GB/s down alone, 45 and 38 GB/s when both run): 1 slab 6.0 ms, 4 slabs
  // 4.66 ms, 8 slabs 4.55 ms, 16 slabs 4.70 ms; narrower slabs make the 2-D copies and the
  // slab GEMMs less efficient.  8 is within ~10 % of the PCIe floor.
  if (slabs == 0) slabs = 8;
  const int w = std::max(16, ceil_div(ceil_div(n, slabs), 16) * 16);
  const int ns = ceil_div(n, w);
  const size_t a_bytes = static_cast<size_t>(m) * k * 2;
  const size_t b_bytes = static_cast<size_t>(k) * n * 2;
  const size_t c_bytes = static_cast<size_t>(m) * n * 2;
  auto up256 = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t a_room = a_on_device ? 0 : up256(a_bytes);
  char* dev = static_cast<char*>(workspace_alloc(st, a_room + up256(b_bytes) + c_bytes, stream));
  if (dev == nullptr) return MO_ERR_NO_MEMORY;
  const uint16_t* a_d = a_on_device ? a_h : reinterpret_cast<uint16_t*>(dev);
  uint16_t* b_d = reinterpret_cast<uint16_t*>(dev + a_room);  // slab j at k * j0
  uint16_t* c_d = reinterpret_cast<uint16_t*>(dev + a_room + up256(b_bytes));  // m * j0

  std::vector<cudaEvent_t> ev(3 + 2 * static_cast<size_t>(ns), nullptr);
  for (cudaEvent_t& e : ev) {
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      for (cudaEvent_t& x : ev) if (x != nullptr) cudaEventDestroy(x);
      cudaFreeAsync(dev, stream);
      return MO_ERR_LAUNCH;
    }
  }
  cudaEvent_t ev_start = ev[0], ev_a = ev[1], ev_done = ev[2];
  // The compute stream also waits for ev_start, so a device-resident A written on the caller's
  // stream is complete before the first slab GEMM reads it.
  bool ok = cudaEventRecord(ev_start, stream) == cudaSuccess &&
            cudaStreamWaitEvent(st->h2d, ev_start, 0) == cudaSuccess &&
            cudaStreamWaitEvent(st->compute, ev_start, 0) == cudaSuccess &&
            (a_on_device || cudaMemcpyAsync(const_cast<uint16_t*>(a_d), a_h, a_bytes, cudaMemcpyHostToDevice,
                                            st->h2d) == cudaSuccess) &&
            cudaEventRecord(ev_a, st->h2d) == cudaSuccess &&
            cudaStreamWaitEvent(st->compute, ev_a, 0) == cudaSuccess;
  for (int j = 0; ok && j < ns; ++j) {
    const int j0 = j * w;
    const int wj = std::min(w, n - j0);
    uint16_t* b_slab = b_d + static_cast<size_t>(k) * j0;
    uint16_t* c_slab = c_d + static_cast<size_t>(m) * j0;
    cudaEvent_t ev_b = ev[3 + 2 * j], ev_c = ev[4 + 2 * j];
    ok = cudaMemcpy2DAsync(b_slab, static_cast<size_t>(wj) * 2, b_h + j0, static_cast<size_t>(n) * 2,
                           static_cast<size_t>(wj) * 2, k, cudaMemcpyHostToDevice, st->h2d) == cudaSuccess &&
         cudaEventRecord(ev_b, st->h2d) == cudaSuccess &&
         cudaStreamWaitEvent(st->compute, ev_b, 0) == cudaSuccess;
    if (!ok) break;
    rc = launch_gemm(a_d, b_slab, c_slab, m, wj, k, st->compute);
    if (rc != MO_OK) break;
    ok = cudaEventRecord(ev_c, st->compute) == cudaSuccess &&
         cudaStreamWaitEvent(st->d2h, ev_c, 0) == cudaSuccess &&
         cudaMemcpy2DAsync(c_h + j0, static_cast<size_t>(n) * 2, c_slab, static_cast<size_t>(wj) * 2,
                           static_cast<size_t>(wj) * 2, m, cudaMemcpyDeviceToHost, st->d2h) == cudaSuccess;
  }
  // Join on the caller's stream even after a failure, so the buffers are freed only once
  // nothing queued on the three streams can still touch them.
  const bool joined = cudaEventRecord(ev_done, st->d2h) == cudaSuccess &&
                      cudaStreamWaitEvent(stream, ev_done, 0) == cudaSuccess;
  bool ok2 = true;
  if (joined) {
    cudaEvent_t ev_h = nullptr, ev_k = nullptr;
    // The h2d and compute streams' last work precedes ev_done through the slab events; after a
    // failure part-way, wait for them explicitly too.
    if (cudaEventCreateWithFlags(&ev_h, cudaEventDisableTiming) == cudaSuccess &&
        cudaEventCreateWithFlags(&ev_k, cudaEventDisableTiming) == cudaSuccess) {
      ok2 = cudaEventRecord(ev_h, st->h2d) == cudaSuccess && cudaStreamWaitEvent(stream, ev_h, 0) == cudaSuccess &&
            cudaEventRecord(ev_k, st->compute) == cudaSuccess && cudaStreamWaitEvent(stream, ev_k, 0) == cudaSuccess;
    } else {
      ok2 = false;
    }
    if (ev_h != nullptr) cudaEventDestroy(ev_h);
    if (ev_k != nullptr) cudaEventDestroy(ev_k);
  }
  if (!(joined && ok2)) {
    cudaStreamSynchronize(st->h2d);
    cudaStreamSynchronize(st->compute);
    cudaStreamSynchronize(st->d2h);
  }
  cudaFreeAsync(dev, stream);
  for (cudaEvent_t& e : ev) cudaEventDestroy(e);
  if (rc != MO_OK) return rc;
  if (!ok || !joined || !ok2) {
    cudaGetLastError();
    return MO_ERR_LAUNCH;
  }
  return MO_OK;
}

}  // namespace
}  // namespace mo

// ---------------------------------------------------------------------------------------
// C++ ABI (reference include/kernel_api.h:10-17)
// ---------------------------------------------------------------------------------------
namespace matmul_optimizer {
bool launch_bf16_gemm_v1(const std::uint16_t* a_bf16, const std::uint16_t* b_bf16,
                         std::uint16_t* c_bf16, int m, int n, int k, cudaStream_t stream) {
  return mo::launch_gemm(a_bf16, b_bf16, c_bf16, m, n, k, stream) == MO_OK;
}
}  // namespace matmul_optimizer

// ---------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------
extern "C" {

const char* mo_error_string(int code) {
  switch (code) {
    case MO_OK: return "ok";
    case MO_ERR_NULL_POINTER: return "null pointer argument";
    case MO_ERR_BAD_DIMS: return "non-positive or overflowing dimension";
    case MO_ERR_UNSUPPORTED: return "unsupported layout (a pointer at an odd address; or, for the no-allocation and host-buffer calls, k or n not a multiple of 8 or a pointer off a 16-byte boundary)";
    case MO_ERR_LAUNCH: return "CUDA launch or runtime call failed";
    case MO_ERR_DEVICE: return "no usable sm_100 device";
    case MO_ERR_BAD_ARGUMENT: return "invalid argument";
    case MO_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
    case MO_ERR_NO_MEMORY: return "device memory for the call's buffers could not be had";
    case MO_ERR_SCRATCH_LIMIT:
      return "problem needs more than the 32 MiB fixed scratch of mo_launch_bf16_gemm_v1_noalloc "
             "(K chunks x m x n x 4 bytes)";
    default: return "unknown error";
  }
}

int mo_version(void) { return 100; }

int mo_launch_bf16_gemm_v1(const uint16_t* a_bf16, const uint16_t* b_bf16, uint16_t* c_bf16,
                           int m, int n, int k, void* stream) {
  return mo::launch_gemm(a_bf16, b_bf16, c_bf16, m, n, k, static_cast<cudaStream_t>(stream));
}

int mo_gemm_from_host(const uint16_t* a_host, const uint16_t* b_host, uint16_t* c_host, int m, int n,
                      int k, int slabs, void* stream) {
  return mo::gemm_from_host(a_host, b_host, c_host, m, n, k, slabs, static_cast<cudaStream_t>(stream));
}

int mo_gemm_b_from_host(const uint16_t* a_dev, const uint16_t* b_host, uint16_t* c_host, int m, int n,
                        int k, int slabs, void* stream) {
  return mo::gemm_from_host(a_dev, b_host, c_host, m, n, k, slabs, static_cast<cudaStream_t>(stream), true);
}

int mo_launch_bf16_gemm_v1_noalloc(const uint16_t* a_bf16, const uint16_t* b_bf16,
                                   uint16_t* c_bf16, int m, int n, int k, void* stream) {
  // The K-split kernel with its chunk partials in g_noalloc_scratch instead of a stream-ordered
  // allocation.  K with a single chunk has nothing to split and runs the unsplit kernel, which
  // needs no scratch.
  mo::Prepared p;
  int rc = mo::prepare_gemm(a_bf16, b_bf16, c_bf16, m, n, k, 1, &p, 0);
  if (rc != MO_OK) return rc;
  if (p.workspace_bytes > mo::kNoAllocScratchBytes) return MO_ERR_SCRATCH_LIMIT;
  float* scratch = nullptr;
  if (p.workspace_bytes > 0) {
    rc = mo::noalloc_scratch(p.st, &scratch);
    if (rc != MO_OK) return rc;
  }
  return mo::run_prepared(p, scratch, static_cast<cudaStream_t>(stream));
}

namespace mo {
namespace {
// The plan and kernel arguments a launch of this shape would get on a device with `num_sms` SMs,
// after the MO_GEMM_* and MATMUL_FIXED_MAIN_TILE_N overrides; no device needed.
int plan_on_host(int m, int n, int k, int num_sms, mo_gemm_plan* plan, GemmArgs* args) {
  if (m <= 0 || n <= 0 || k <= 0) return MO_ERR_BAD_DIMS;
  if (num_sms <= 0) return MO_ERR_BAD_ARGUMENT;
  int forced = 0;
  if (m == kHeroM && n == kHeroN && k == kHeroK) {
    forced = parse_tile_override();
    if (forced < 0) return MO_ERR_BAD_ARGUMENT;
  }
  const int split_mode = parse_split_override();
  const int forced_variant = parse_variant_override();
  const int streamk_mode = parse_streamk_override();
  if (split_mode == -2 || forced_variant == -2 || streamk_mode == -2) return MO_ERR_BAD_ARGUMENT;
  const Choice c = select_variant(m, n, k, num_sms, forced, split_mode, forced_variant, streamk_mode);
  const int clusters = num_sms / kVariants[c.var].cta_group;
  *plan = mo_gemm_plan{};
  fill_plan(m, n, k, clusters, c, plan);
  size_t ws = 0, sk = 0;
  fill_args(m, n, k, clusters, plan, args, &ws, &sk);
  return MO_OK;
}
}  // namespace
}  // namespace mo

int mo_gemm_select_plan(int m, int n, int k, int num_sms, mo_gemm_plan* out) {
  if (out == nullptr) return MO_ERR_NULL_POINTER;
  mo::GemmArgs args{};
  return mo::plan_on_host(m, n, k, num_sms, out, &args);
}

int mo_gemm_schedule(int m, int n, int k, int num_sms, int* units, int cap, int* count) {
  if (count == nullptr || (units == nullptr && cap > 0)) return MO_ERR_NULL_POINTER;
  if (cap < 0) return MO_ERR_BAD_ARGUMENT;
  mo_gemm_plan plan{};
  mo::GemmArgs args{};
  const int rc = mo::plan_on_host(m, n, k, num_sms, &plan, &args);
  if (rc != MO_OK) return rc;
  long long total = 0;
  for (int cl = 0; cl < args.num_clusters; ++cl) {
    const int nu = mo::num_units_of(cl, args);
    for (int j = 0; j < nu; ++j, ++total) {
      if (total >= cap) continue;
      const mo::Unit w = mo::unit_at(cl, j, args);
      int* u = units + 7 * total;
      u[0] = cl;
      u[1] = j;
      u[2] = w.mb;
      u[3] = w.nb;
      u[4] = w.ch_begin;
      u[5] = w.ch_end;
      u[6] = w.sk_tile;
    }
  }
  *count = static_cast<int>(std::min<long long>(total, INT32_MAX));
  return MO_OK;
}

int mo_shard_partition(int n, int g, int* slab_begin, int* slab_n) {
  if (slab_begin == nullptr || slab_n == nullptr) return MO_ERR_NULL_POINTER;
  if (n <= 0) return MO_ERR_BAD_DIMS;
  if (g <= 0 || g > mo::kMaxShards) return MO_ERR_BAD_ARGUMENT;
  const int w = ((n + g - 1) / g + 15) / 16 * 16;
  for (int i = 0; i < g; ++i) {
    const long long begin = static_cast<long long>(i) * w;
    slab_begin[i] = static_cast<int>(std::min<long long>(begin, n));
    slab_n[i] = static_cast<int>(std::max<long long>(0, std::min<long long>(w, n - begin)));
  }
  return MO_OK;
}

int mo_gemm_nshard(int g, const int* devices, const uint16_t* const* a,
                   const uint16_t* const* b_slabs, uint16_t* const* c_slabs, int m, int k,
                   const int* slab_n, void* const* streams) {
  if (devices == nullptr || a == nullptr || b_slabs == nullptr || c_slabs == nullptr ||
      slab_n == nullptr || streams == nullptr) {
    return MO_ERR_NULL_POINTER;
  }
  if (g <= 0 || g > mo::kMaxShards) return MO_ERR_BAD_ARGUMENT;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return MO_ERR_DEVICE;
  int rc = MO_OK;
  for (int i = 0; i < g && rc == MO_OK; ++i) {
    if (slab_n[i] == 0) continue;  // an empty trailing slab has no work
    if (cudaSetDevice(devices[i]) != cudaSuccess) {
      rc = MO_ERR_DEVICE;
      break;
    }
    rc = mo::launch_gemm(a[i], b_slabs[i], c_slabs[i], m, slab_n[i], k,
                         static_cast<cudaStream_t>(streams[i]));
  }
  cudaSetDevice(prev);
  return rc;
}

int mo_unshard_columns(const uint16_t* gathered, uint16_t* c, int g, int m, const int* slab_n,
                       int64_t block_elems, void* stream) {
  if (gathered == nullptr || c == nullptr || slab_n == nullptr) return MO_ERR_NULL_POINTER;
  if (g <= 0 || g > mo::kMaxShards || m <= 0) return MO_ERR_BAD_ARGUMENT;
  mo::UnshardArgs args{};
  args.gathered = gathered;
  args.c = c;
  args.g = g;
  args.m = m;
  args.block_elems = block_elems;
  bool vec8 = ((reinterpret_cast<uintptr_t>(gathered) | reinterpret_cast<uintptr_t>(c)) & 15u) == 0 &&
              (block_elems % 8) == 0;
  int total = 0;
  for (int i = 0; i < g; ++i) {
    if (slab_n[i] < 0) return MO_ERR_BAD_ARGUMENT;
    if (static_cast<long long>(m) * slab_n[i] > block_elems) return MO_ERR_BAD_ARGUMENT;
    args.begin[i] = total;
    total += slab_n[i];
    if (slab_n[i] % 8) vec8 = false;
  }
  args.begin[g] = total;
  for (int i = g + 1; i <= mo::kMaxShards; ++i) args.begin[i] = std::numeric_limits<int>::max();
  if (total <= 0) return MO_ERR_BAD_DIMS;
  args.n = total;
  mo::DeviceState* st = nullptr;
  const int rc = mo::device_state(&st);
  if (rc != MO_OK) return rc;
  const long long units = static_cast<long long>(m) * total / (vec8 ? 8 : 1);
  const int blocks = static_cast<int>(std::min<long long>((units + 255) / 256, 8LL * st->sm_count));
  mo::unshard_columns_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(args, vec8);
  return cudaGetLastError() == cudaSuccess ? MO_OK : MO_ERR_LAUNCH;
}

int mo_read_device_watchdog(int clear, int* flag_out) {
  mo::DeviceState* st = nullptr;
  const int rc = mo::device_state(&st);
  if (rc != MO_OK) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return MO_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpy(&v, st->watchdog, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    return MO_ERR_LAUNCH;
  }
  if (clear) {
    const int zero = 0;
    if (cudaMemcpy(st->watchdog, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
      return MO_ERR_LAUNCH;
    }
  }
  if (flag_out) *flag_out = v;
  return MO_OK;
}

int mo_release_workspace(int64_t* held_before) {
  mo::DeviceState* st = nullptr;
  const int rc = mo::device_state(&st);
  if (rc != MO_OK) return rc;
  std::lock_guard<std::mutex> lock(mo::g_dev_mutex);
  uint64_t held = 0;
  // The stream-K regions' kept workspaces go back to the pool first.  Their owner streams may
  // be gone, so the device is synchronised and they are freed on the legacy stream.
  bool any_kept = false;
  for (void* w : st->sk_ws) any_kept = any_kept || w != nullptr;
  if (any_kept) {
    if (cudaDeviceSynchronize() != cudaSuccess) {
      cudaGetLastError();
      return MO_ERR_DEVICE;
    }
    for (int r = 0; r < mo::kSkRegions; ++r) {
      if (st->sk_ws[r] != nullptr) cudaFreeAsync(st->sk_ws[r], nullptr);
      st->sk_ws[r] = nullptr;
      st->sk_ws_bytes[r] = 0;
    }
    if (cudaStreamSynchronize(nullptr) != cudaSuccess) {
      cudaGetLastError();
      return MO_ERR_DEVICE;
    }
  }
  if (st->pool != nullptr) {
    if (cudaMemPoolGetAttribute(st->pool, cudaMemPoolAttrReservedMemCurrent, &held) != cudaSuccess ||
        cudaMemPoolTrimTo(st->pool, 0) != cudaSuccess) {
      cudaGetLastError();
      return MO_ERR_DEVICE;
    }
  }
  if (held_before) *held_before = static_cast<int64_t>(held);
  return MO_OK;
}

int mo_selftest_wait_timeout(int timeout_us, void* stream) {
  if (timeout_us <= 0 || timeout_us > 10000000) return MO_ERR_BAD_ARGUMENT;
  mo::DeviceState* st = nullptr;
  const int rc = mo::device_state(&st);
  if (rc != MO_OK) return rc;
  mo::selftest_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      st->watchdog, static_cast<unsigned long long>(timeout_us) * 1000ull);
  return cudaGetLastError() == cudaSuccess ? MO_OK : MO_ERR_LAUNCH;
}

}  // extern "C"
