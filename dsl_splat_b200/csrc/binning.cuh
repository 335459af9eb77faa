// Tile binning and sorting: the B200 replacement for splatting/binning.py:
// 116-217 (duplicate + bin_and_sort), primitives/tiling.py:39-100 (scan,
// radix sort, identify_ranges) and Warp's array_scan / radix_sort_pairs.
//
// The reference emits one (tile<<32 | float_bits(depth), id) pair per
// Gaussian-tile overlap in Gaussian order and radix-sorts the 64-bit keys
// stably, so within a tile entries are ordered by (depth bits, Gaussian
// index).  This file produces the identical order with less traffic:
//
//   1. bin_prepare: per Gaussian, depth key (culled -> 0xFFFFFFFF), packed
//      tile rectangle, +-1 corners into a 2D difference grid over tiles and
//      the four 8-bit digit histograms of the depth keys.
//   2. four stable onesweep passes sort (depth bits, index) over N.
//   3. exclusive scan of tile counts in depth order -> pair offsets, M.
//   4. tile_counts: 2D prefix of the difference grid -> per-tile counts ->
//      ranges (T,2) and the digit histograms of the tile ids.
//   5. a stable onesweep pass keyed on tile bits 0-7 whose loader generates
//      the pairs directly from the depth-ordered Gaussians (no pair buffer
//      is written before sorting), then one pass per further 8 tile bits.
//
// A stable sort by tile of a sequence already ordered by (depth, index) is
// exactly the reference order.  Every pass uses decoupled look-back with a
// bounded spin: on expiry it records kDeviceTimeout in g_splat_device_error
// and finishes without waiting further.
#pragma once
#include "splat_common.cuh"
#include "tile_modes.cuh"

namespace splat {

constexpr int kSortBlock = 256;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortBlock * kSortItems;  // elements per onesweep block
constexpr int kSortWarps = kSortBlock / 32;
constexpr int kRadix = 256;
constexpr uint32_t kFlagAggregate = 1u << 30;
constexpr uint32_t kFlagInclusive = 2u << 30;
constexpr uint32_t kValueMask = (1u << 30) - 1u;
constexpr uint32_t kSpinLimit = 1u << 22;


__device__ int g_splat_device_error;

SPLAT_DEV void record_device_error(int code) { atomicCAS(&g_splat_device_error, 0, code); }

// Status word formats of the decoupled look-backs: a 2-bit flag (0 = not
// yet published, aggregate, inclusive) over the value.
struct Status32 {
  using Word = uint32_t;
  static constexpr Word kAggregate = kFlagAggregate, kInclusive = kFlagInclusive;
  static constexpr Word kMask = kValueMask;
  static SPLAT_DEV Word load(const Word* p) { return ld_relaxed(p); }
};
struct Status64 {
  using Word = unsigned long long;
  static constexpr Word kAggregate = 1ull << 62, kInclusive = 2ull << 62;
  static constexpr Word kMask = (1ull << 62) - 1ull;
  static SPLAT_DEV Word load(const Word* p) { return ld_relaxed64(p); }
};

// Exclusive prefix of tile `tile` from its predecessors' status words
// (status[t * stride] for tile t): kWindow predecessors are read at once
// with independent loads, then consumed nearest first, adding aggregates up
// to the first inclusive value; an unpublished word stops the window and it
// is read again after a short sleep.  Tile 0 is always inclusive, so the
// walk ends; a wait longer than kSpinLimit records kDeviceTimeout.
template <class S, int kWindow>
SPLAT_DEV typename S::Word lookback(const typename S::Word* status, int64_t tile, size_t stride,
                                    uint32_t spin_limit = kSpinLimit) {
  using Word = typename S::Word;
  Word excl = 0;
  uint32_t spins = 0;
  int64_t t = tile - 1;
  while (t >= 0) {
    Word w[kWindow];
#pragma unroll
    for (int k = 0; k < kWindow; ++k) w[k] = t - k >= 0 ? S::load(status + (t - k) * stride) : 0;
    Word add = 0;
    int consumed = 0, state = 0;  // 0 continue, 1 inclusive reached, 2 unpublished
#pragma unroll
    for (int k = 0; k < kWindow; ++k) {
      if (state == 0) {
        if (t - k < 0) {
          state = 1;
        } else {
          const Word flag = w[k] & ~S::kMask;
          if (flag == 0) {
            state = 2;
          } else {
            add += w[k] & S::kMask;
            consumed = k + 1;
            if (flag == S::kInclusive) state = 1;
          }
        }
      }
    }
    excl += add;
    if (state == 1) break;
    if (state == 2) {
      if (++spins > spin_limit) {
        record_device_error(kDeviceTimeout);
        break;
      }
      __nanosleep(32);
    }
    t -= consumed;
  }
  return excl;
}

// The same walk by a whole warp (all 32 lanes call; every lane returns the
// prefix): lane l reads the status of tile t - l, so one round covers 32
// predecessors, nearest first up to the first inclusive or unpublished one.
// Positions before tile 0 read as inclusive zero.
template <class S>
SPLAT_DEV typename S::Word warp_lookback(const typename S::Word* status, int64_t tile,
                                         size_t stride, uint32_t spin_limit = kSpinLimit) {
  using Word = typename S::Word;
  const int lane = threadIdx.x & 31;
  Word excl = 0;
  uint32_t spins = 0;
  int64_t t = tile - 1;
  while (t >= 0) {
    const int64_t mine = t - lane;
    const Word w = mine >= 0 ? S::load(status + mine * stride) : S::kInclusive;
    const Word flag = w & ~S::kMask;
    const uint32_t incl = __ballot_sync(0xffffffffu, flag == S::kInclusive);
    const uint32_t stop_mask = incl | __ballot_sync(0xffffffffu, flag == 0);
    const int stop = stop_mask ? __ffs(stop_mask) - 1 : 32;
    const bool done = stop < 32 && ((incl >> stop) & 1u);
    const int consumed = done ? stop + 1 : stop;  // lanes summed in this step of the walk
    Word v = lane < consumed ? (w & S::kMask) : Word(0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    excl += v;
    if (done) break;
    if (stop < 32) {
      if (++spins > spin_limit) {
        if (lane == 0) record_device_error(kDeviceTimeout);
        break;
      }
      __nanosleep(32);
    }
    t -= consumed;
  }
  return excl;
}

// One thread walks the look-back of tile 1 over `status` (two words the
// caller zeroed, i.e. never published) with a short spin limit: the wait
// runs out, kDeviceTimeout is recorded and the thread returns.  This is how
// the tests check that an expired wait ends and is reported, without
// faulting or hanging anything.
__global__ void lookback_expiry_kernel(const uint32_t* __restrict__ status, uint32_t spin_limit,
                                       uint32_t* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *out = lookback<Status32, 1>(status, 1, 1, spin_limit);
}

// ---- phase 1: per-Gaussian preparation ---------------------------------
// diff == nullptr selects the chunked path (no difference grid; the pair
// total is the sum of rectangle areas).
__global__ void __launch_bounds__(256)
    bin_prepare_kernel(int n, const float* __restrict__ centers, const float* __restrict__ conics,
                       const int* __restrict__ radii, const int* __restrict__ tiles,
                       const float* __restrict__ depths, int gx, int gy, int tile_mode,
                       uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
                       uint2* __restrict__ rects, int* __restrict__ diff,
                       uint32_t* __restrict__ hist, unsigned long long* __restrict__ total) {
  __shared__ uint32_t s_hist[4 * kRadix];
  for (int k = threadIdx.x; k < 4 * kRadix; k += blockDim.x) s_hist[k] = 0;
  __syncthreads();
  const int stride = gridDim.x * blockDim.x;
  unsigned long long pairs = 0;
  const uint32_t lt = lanemask_lt();
  // Every lane of a warp runs the same number of iterations (lanes past n
  // are predicated off) so the warp-aggregated histogram updates can use
  // full-warp collectives: depth keys share few top-byte values, and 32
  // lanes incrementing one shared counter would serialise.
  const int n_round = (n + 31) & ~31;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_round; i += stride) {
    const bool valid = i < n;
    const int radius = valid ? radii[i] : 0;
    uint32_t key = kCulledKey;
    if (valid) {
      uint2 rect = make_uint2(0u, 0u);
      if (radius > 0) {
        key = __float_as_uint(depths[i]);
        const float2 c = reinterpret_cast<const float2*>(centers)[i];
        // the tile rectangle of the mode (snugbox: the clipped box; accutile:
        // the box bounding its strips)
        TileVisit tv;
        if (tile_mode == kTileRadius) {
          tv.e.bounds = tile_bounds(c.x, c.y, radius, gx, gy);
          tv.strips = false;
        } else {
          tv = tile_visit(tile_mode, c.x, c.y, reinterpret_cast<const float4*>(conics)[i], radius,
                          gx, gy);
        }
        int4 b = tv.e.bounds;
        if (b.z <= b.x || b.w <= b.y) b = make_int4(0, 0, 0, 0);  // no tiles
        rect = make_uint2(static_cast<uint32_t>(b.x) | (static_cast<uint32_t>(b.y) << 16),
                          static_cast<uint32_t>(b.z) | (static_cast<uint32_t>(b.w) << 16));
        if (diff) {  // onesweep path: per-tile counts from a global difference grid
          const int row = gx + 1;
          if (tv.strips) {  // accutile: one 1-wide rectangle per strip
            walk_strips(tv, [&](int r, int2 span) {
              const int x0 = tv.is_y ? span.x : r, x1 = tv.is_y ? span.y : r + 1;
              const int y0 = tv.is_y ? r : span.x, y1 = tv.is_y ? r + 1 : span.y;
              atomicAdd(diff + y0 * row + x0, 1);
              atomicAdd(diff + y0 * row + x1, -1);
              atomicAdd(diff + y1 * row + x0, -1);
              atomicAdd(diff + y1 * row + x1, 1);
            });
          } else if (b.z > b.x && b.w > b.y) {
            atomicAdd(diff + b.y * row + b.x, 1);
            atomicAdd(diff + b.y * row + b.z, -1);
            atomicAdd(diff + b.w * row + b.x, -1);
            atomicAdd(diff + b.w * row + b.z, 1);
          }
          pairs += static_cast<unsigned long long>(max(tiles[i], 0));
        } else {  // chunked path: pairs are the rectangle areas it scatters
          pairs += static_cast<unsigned long long>(max(b.z - b.x, 0)) *
                   static_cast<unsigned long long>(max(b.w - b.y, 0));
        }
      }
      keys[i] = key;
      vals[i] = static_cast<uint32_t>(i);
      rects[i] = rect;
    }
    // the two low digits of visible rows are spread over all 256 values
    // (lanes rarely collide); culled rows (all digits 255) are counted once
    // per warp, and the two high digits, which take few values, are
    // aggregated per warp
    const bool culled = valid && key == kCulledKey;
#pragma unroll
    for (int p = 0; p < 2; ++p)
      if (valid && !culled) atomicAdd(&s_hist[p * kRadix + ((key >> (8 * p)) & 255u)], 1u);
    const uint32_t culled_lanes = __popc(__ballot_sync(0xffffffffu, culled));
    if ((threadIdx.x & 31) == 0 && culled_lanes) {
      atomicAdd(&s_hist[0 * kRadix + 255], culled_lanes);
      atomicAdd(&s_hist[1 * kRadix + 255], culled_lanes);
    }
#pragma unroll
    for (int p = 2; p < 4; ++p) {
      const uint32_t d = valid ? ((key >> (8 * p)) & 255u) : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      if (valid && (peers & lt) == 0u) atomicAdd(&s_hist[p * kRadix + d], __popc(peers));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pairs += __shfl_xor_sync(0xffffffffu, pairs, o);
  if ((threadIdx.x & 31) == 0 && pairs) atomicAdd(total, pairs);
  __syncthreads();
  for (int k = threadIdx.x; k < 4 * kRadix; k += blockDim.x)
    if (s_hist[k]) atomicAdd(hist + k, s_hist[k]);
}

// Block-wide exclusive scan of one value per thread (blockDim.x <= 1024).
SPLAT_DEV uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < warps ? s_warp[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < warps) s_warp[lane] = w;
  }
  __syncthreads();
  const uint32_t before = (warp > 0 ? s_warp[warp - 1] : 0u) + x - v;
  if (total) *total = s_warp[warps - 1];
  __syncthreads();
  return before;
}

// ---- generic onesweep pass ---------------------------------------------

struct KeyValueLoader {
  const uint32_t* keys;
  const uint32_t* vals;
  struct Shared {};
  SPLAT_DEV void prepare(uint32_t, uint32_t, Shared&) {}
  SPLAT_DEV void load(uint32_t idx, const Shared&, uint32_t& key, uint32_t& val) const {
    key = keys[idx];
    val = vals[idx];
  }
};

// Largest j in [lo, hi) with offsets[j] <= target, given offsets[lo] <=
// target < offsets[hi]: a block-wide 256-ary search (all threads call).
SPLAT_DEV uint32_t block_upper_search(const uint32_t* __restrict__ offsets, uint32_t lo,
                                      uint32_t hi, uint32_t target) {
  while (hi - lo > 1) {
    const uint32_t span = hi - lo;
    const uint32_t step = (span + kSortBlock - 1) / kSortBlock;
    const uint32_t j = lo + threadIdx.x * step;
    const bool pred = j < hi && offsets[j] <= target;
    const uint32_t count = static_cast<uint32_t>(__syncthreads_count(pred));
    const uint32_t new_lo = lo + (count - 1) * step;
    const uint32_t cand = lo + count * step;
    hi = cand < hi ? cand : hi;
    lo = new_lo;
  }
  return lo;
}

// Generates the (tile id, Gaussian id) pairs of depth-ordered Gaussians:
// pair p belongs to the Gaussian j with offsets[j] <= p < offsets[j+1] and
// is its (p - offsets[j])-th tile in row-major rectangle order.
struct EmitLoader {
  const uint32_t* offsets;  // exclusive, length nsorted + 1
  const uint32_t* order;    // depth-ordered Gaussian ids
  const uint2* rects;
  uint32_t nsorted;
  int gx;
  struct Shared {
    uint32_t j0;
    uint32_t count;
    uint32_t off[kSortTile + 1];
  };
  SPLAT_DEV void prepare(uint32_t base, uint32_t end, Shared& s) {
    const uint32_t j0 = block_upper_search(offsets, 0u, nsorted, base);
    const uint32_t j1 = block_upper_search(offsets, j0, nsorted, end - 1);
    uint32_t cnt = j1 - j0 + 1;
    if (cnt > static_cast<uint32_t>(kSortTile)) {  // impossible for consistent offsets
      if (threadIdx.x == 0) record_device_error(kInconsistentInput);
      cnt = kSortTile;
    }
    for (uint32_t k = threadIdx.x; k <= cnt; k += blockDim.x) s.off[k] = offsets[j0 + k];
    if (threadIdx.x == 0) {
      s.j0 = j0;
      s.count = cnt;
    }
    __syncthreads();
  }
  SPLAT_DEV void load(uint32_t idx, const Shared& s, uint32_t& key, uint32_t& val) const {
    uint32_t lo = 0, hi = s.count;  // off[lo] <= idx < off[hi]
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (s.off[mid] <= idx) lo = mid; else hi = mid;
    }
    const uint32_t g = order[s.j0 + lo];
    const uint32_t local = idx - s.off[lo];
    const uint2 r = rects[g];
    const uint32_t x0 = r.x & 0xFFFFu, y0 = r.x >> 16, x1 = r.y & 0xFFFFu;
    const uint32_t w = x1 > x0 ? x1 - x0 : 1u;
    const uint32_t dy = local / w;
    key = (y0 + dy) * static_cast<uint32_t>(gx) + x0 + (local - dy * w);
    val = g;
  }
};

// THREADS >= 256: the first 256 threads own one digit each in the look-back;
// larger blocks shorten the look-back chain at the cost of fewer blocks.
// ITEMS keys per thread: fewer make more, shorter tiles (more blocks in
// flight and a shorter ranking loop per block, a longer look-back chain).
// SCAN_HIST: digit_offsets holds this pass's 256-bin key histogram, whose
// exclusive prefix every block forms itself (no separate offsets launch).
template <class Loader, bool WRITE_KEYS, int THREADS = kSortBlock, int ITEMS = kSortItems,
          bool SCAN_HIST = false>
__global__ void __launch_bounds__(THREADS)
    onesweep_kernel(Loader ld, uint32_t n, int shift, const uint32_t* __restrict__ digit_offsets,
                    uint32_t* __restrict__ status, uint32_t* __restrict__ counter,
                    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out) {
  constexpr int kWarps = THREADS / 32;
  constexpr uint32_t kTile = static_cast<uint32_t>(THREADS) * ITEMS;
  static_assert(THREADS >= kRadix && THREADS % 32 == 0, "one thread per digit");
  // Staged output: the tile's keys and values are first placed in digit
  // order in shared memory, then written out by consecutive threads, so a
  // digit's run in the output is written with contiguous stores (direct
  // stores put every lane of a warp in a different 32-byte sector).  Taken
  // when the two staging arrays fit beside the loader's shared state.
  constexpr bool kStage = 8 * kTile + sizeof(typename Loader::Shared) <= 40 * 1024;
  constexpr uint32_t kStaged = kStage ? kTile : 1u;
  __shared__ uint32_t s_hist[kWarps][kRadix];
  __shared__ uint32_t s_base[kRadix];
  __shared__ uint32_t s_start[kStage ? kRadix : 1];
  __shared__ uint32_t s_key[kStaged], s_val[kStaged];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_tile;
  __shared__ typename Loader::Shared s_ld;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_tile = atomicAdd(counter, 1u);
  for (int k = threadIdx.x; k < kWarps * kRadix; k += THREADS) (&s_hist[0][0])[k] = 0u;
  __syncthreads();
  const uint32_t tile = s_tile;
  const uint32_t base = tile * kTile;
  const uint32_t end = min(base + kTile, n);
  ld.prepare(base, end, s_ld);

  uint32_t keys[ITEMS], vals[ITEMS], rank[ITEMS];
  const uint32_t lt = lanemask_lt();
  uint32_t digit_first = 0u;  // SCAN_HIST: output position of this thread's digit
  if constexpr (SCAN_HIST)
    digit_first = block_exclusive_scan(
        threadIdx.x < kRadix ? __ldg(digit_offsets + threadIdx.x) : 0u, s_warp, nullptr);
  // every load of the thread is issued before the ranking (whose warp
  // barriers would otherwise wait out one load latency per item)
#pragma unroll
  for (int r = 0; r < ITEMS; ++r) {
    const uint32_t idx = base + warp * (32 * ITEMS) + r * 32 + lane;
    keys[r] = 0u;
    vals[r] = 0u;
    if (idx < end) ld.load(idx, s_ld, keys[r], vals[r]);
  }
#pragma unroll
  for (int r = 0; r < ITEMS; ++r) {
    const uint32_t idx = base + warp * (32 * ITEMS) + r * 32 + lane;
    const bool valid = idx < end;
    const uint32_t key = keys[r];
    const uint32_t d = valid ? ((key >> shift) & 255u) : 256u;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    uint32_t before = 0u;
    if (valid) before = s_hist[warp][d];
    __syncwarp();
    if (valid && (peers & lt) == 0u) s_hist[warp][d] = before + __popc(peers);
    __syncwarp();
    rank[r] = valid ? before + __popc(peers & lt) : 0xFFFFFFFFu;
  }
  __syncthreads();

  // per digit: the warps' exclusive offsets, the tile's count, published
  // as this tile's aggregate (tile 0: inclusive) before anything else
  uint32_t total = 0u;
  uint32_t* mine = status + static_cast<size_t>(tile) * kRadix + threadIdx.x;
  if (threadIdx.x < kRadix) {
    const int d = threadIdx.x;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t c = s_hist[w][d];
      s_hist[w][d] = total;
      total += c;
    }
    st_relaxed(mine, (tile == 0 ? kFlagInclusive : kFlagAggregate) | total);
  }
  if constexpr (kStage) {
    // digit-ordered positions inside the tile, filled while predecessors
    // publish
    const uint32_t start = block_exclusive_scan(threadIdx.x < kRadix ? total : 0u, s_warp, nullptr);
    if (threadIdx.x < kRadix) s_start[threadIdx.x] = start;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
      if (rank[r] == 0xFFFFFFFFu) continue;
      const uint32_t d = (keys[r] >> shift) & 255u;
      const uint32_t local = s_start[d] + s_hist[warp][d] + rank[r];
      s_key[local] = keys[r];
      s_val[local] = vals[r];
    }
  }
  if (threadIdx.x < kRadix) {
    const int d = threadIdx.x;
    uint32_t excl = 0u;
    if (tile != 0) {
      excl = lookback<Status32, 8>(status + d, static_cast<int64_t>(tile), kRadix);
      st_relaxed(mine, kFlagInclusive | (excl + total));
    }
    // output position of the digit's first key, less its tile-local start
    // when staged
    s_base[d] = (SCAN_HIST ? digit_first : digit_offsets[d]) + excl - (kStage ? s_start[d] : 0u);
  }
  __syncthreads();

  if constexpr (kStage) {
    const uint32_t count = end > base ? end - base : 0u;
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
      const uint32_t i = r * THREADS + threadIdx.x;
      if (i >= count) break;
      const uint32_t key = s_key[i];
      const uint32_t pos = s_base[(key >> shift) & 255u] + i;
      if (pos >= n) {  // only reachable with inconsistent histograms
        record_device_error(kInconsistentInput);
        continue;
      }
      if (WRITE_KEYS) keys_out[pos] = key;
      vals_out[pos] = s_val[i];
    }
  } else {
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
      if (rank[r] == 0xFFFFFFFFu) continue;
      const uint32_t d = (keys[r] >> shift) & 255u;
      const uint32_t pos = s_base[d] + s_hist[warp][d] + rank[r];
      if (pos >= n) {  // only reachable with inconsistent histograms
        record_device_error(kInconsistentInput);
        continue;
      }
      if (WRITE_KEYS) keys_out[pos] = keys[r];
      vals_out[pos] = vals[r];
    }
  }
}

// ---- scans --------------------------------------------------------------
// values[gather ? gather[i] : i] summed in blocks of kSortTile.

SPLAT_DEV uint32_t scan_value(const int* __restrict__ values, const uint32_t* __restrict__ gather,
                              uint32_t i, uint32_t bias) {
  const uint32_t src = gather ? gather[i] : i;
  const int v = values[src];
  return (v > 0 ? static_cast<uint32_t>(v) : 0u) + bias;
}

__global__ void __launch_bounds__(kSortBlock)
    scan_block_sums_kernel(const int* __restrict__ values, const uint32_t* __restrict__ gather,
                           uint32_t n, uint32_t* __restrict__ block_sums, uint32_t bias = 0u) {
  __shared__ uint32_t s_warp[32];
  const uint32_t base = blockIdx.x * kSortTile;
  uint32_t sum = 0u;
  for (int k = 0; k < kSortItems; ++k) {
    const uint32_t i = base + k * kSortBlock + threadIdx.x;
    if (i < n) sum += scan_value(values, gather, i, bias);
  }
  uint32_t total;
  block_exclusive_scan(sum, s_warp, &total);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// One block: exclusive scan of block_sums in place; total -> *total.
__global__ void scan_block_prefix_kernel(uint32_t* __restrict__ block_sums, uint32_t nblocks,
                                         uint32_t* __restrict__ total) {
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_carry;
  if (threadIdx.x == 0) s_carry = 0u;
  __syncthreads();
  for (uint32_t base = 0; base < nblocks; base += blockDim.x) {
    const uint32_t i = base + threadIdx.x;
    const uint32_t v = i < nblocks ? block_sums[i] : 0u;
    uint32_t chunk;
    const uint32_t before = block_exclusive_scan(v, s_warp, &chunk);
    if (i < nblocks) block_sums[i] = s_carry + before;
    __syncthreads();
    if (threadIdx.x == 0) s_carry += chunk;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = s_carry;
}

// ---- count scan (splat_scan_counts*): 64-bit total ----------------------------
// The offsets are int32 (as the reference's array_scan output), so a count
// total above INT32_MAX cannot be represented; the total itself is formed in
// 64 bits so that it never wraps, and exceeding INT32_MAX is reported.

SPLAT_DEV unsigned long long block_sum_u64(unsigned long long v, unsigned long long* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  if (lane == 0) s_warp[warp] = v;
  __syncthreads();
  unsigned long long sum = 0ull;
  for (int w = 0; w < warps; ++w) sum += s_warp[w];
  __syncthreads();
  return sum;
}

// Per block of kSortTile counts: the sum in 64 bits, stored saturated at
// 0xFFFFFFFF (a block sum that large already puts the total past INT32_MAX).
__global__ void __launch_bounds__(kSortBlock)
    scan_count_block_sums_kernel(const int* __restrict__ values, uint32_t n,
                                 uint32_t* __restrict__ block_sums) {
  __shared__ unsigned long long s_warp[32];
  const uint32_t base = blockIdx.x * kSortTile;
  unsigned long long sum = 0ull;
  for (int k = 0; k < kSortItems; ++k) {
    const uint32_t i = base + k * kSortBlock + threadIdx.x;
    if (i < n) sum += static_cast<unsigned long long>(scan_value(values, nullptr, i, 0u));
  }
  const unsigned long long total = block_sum_u64(sum, s_warp);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total > 0xFFFFFFFFull ? 0xFFFFFFFFu
                                                                        : static_cast<uint32_t>(total);
}

// One block: exclusive scan of the block sums in place (exact whenever the
// total fits int32) and their 64-bit sum into *total (may be null).  A total
// above INT32_MAX records kTooLarge in the device error word: the offsets of
// that call are not valid.
__global__ void scan_count_prefix_kernel(uint32_t* __restrict__ block_sums, uint32_t nblocks,
                                         long long* __restrict__ total) {
  __shared__ uint32_t s_warp[32];
  __shared__ unsigned long long s_warp64[32];
  __shared__ uint32_t s_carry;
  if (threadIdx.x == 0) s_carry = 0u;
  __syncthreads();
  unsigned long long mine = 0ull;
  for (uint32_t base = 0; base < nblocks; base += blockDim.x) {
    const uint32_t i = base + threadIdx.x;
    const uint32_t v = i < nblocks ? block_sums[i] : 0u;
    mine += v;
    uint32_t chunk;
    const uint32_t before = block_exclusive_scan(v, s_warp, &chunk);
    if (i < nblocks) block_sums[i] = s_carry + before;
    __syncthreads();
    if (threadIdx.x == 0) s_carry += chunk;
    __syncthreads();
  }
  const unsigned long long sum = block_sum_u64(mine, s_warp64);
  if (threadIdx.x == 0) {
    if (total) *total = static_cast<long long>(sum);
    if (sum > 0x7FFFFFFFull) record_device_error(kTooLarge);
  }
}

// out[i] = exclusive (or inclusive) prefix; when exclusive, out[n] = total.
__global__ void __launch_bounds__(kSortBlock)
    scan_apply_kernel(const int* __restrict__ values, const uint32_t* __restrict__ gather,
                      uint32_t n, const uint32_t* __restrict__ block_prefix, int inclusive,
                      uint32_t* __restrict__ out, uint32_t bias = 0u) {
  __shared__ uint32_t s_val[kSortTile];
  __shared__ uint32_t s_warp[32];
  const uint32_t base = blockIdx.x * kSortTile;
  for (int k = 0; k < kSortItems; ++k) {
    const int j = k * kSortBlock + threadIdx.x;
    const uint32_t i = base + j;
    s_val[j] = i < n ? scan_value(values, gather, i, bias) : 0u;
  }
  __syncthreads();
  uint32_t local[kSortItems];
  uint32_t sum = 0u;
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    local[k] = s_val[threadIdx.x * kSortItems + k];
    sum += local[k];
  }
  uint32_t run = block_exclusive_scan(sum, s_warp, nullptr) + block_prefix[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    const uint32_t v = local[k];
    s_val[threadIdx.x * kSortItems + k] = inclusive ? run + v : run;
    run += v;
  }
  __syncthreads();
  for (int k = 0; k < kSortItems; ++k) {
    const int j = k * kSortBlock + threadIdx.x;
    const uint32_t i = base + j;
    if (i < n) out[i] = s_val[j];
  }
  if (!inclusive && blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
    // the last element's exclusive prefix plus its value
    const uint32_t last = n - 1;
    if (last >= base) out[n] = s_val[last - base] + scan_value(values, gather, last, bias);
  }
}

// The chunked path's work prefix and chunk bounds in one pass (replacing a
// block-sum / block-prefix / apply scan and a binary-search kernel).
// offsets[i] = sum over j < i of (max(values[order[j]], 0) + bias) in depth
// order, offsets[n] = the total; bounds[k] = the first i in [0, n] with
// offsets[i] >= floor(W k / chunks) and bounds[chunks] = n, where
// W = *pair_total + bias * n is bin_prepare's total, known before the scan.
// Each tile finds the few bounds whose targets fall inside its prefix range
// by binary search over its exclusive prefixes in shared memory.  Decoupled
// look-back over
// kSortTile-element tiles taken in ticket order; 64-bit status words
// (2-bit flag, 62-bit inclusive/aggregate value).
__global__ void __launch_bounds__(kSortBlock)
    work_scan_kernel(const int* __restrict__ values, const uint32_t* __restrict__ order,
                     uint32_t n, uint32_t bias, const unsigned long long* __restrict__ pair_total,
                     unsigned chunks, unsigned long long* __restrict__ status,
                     uint32_t* __restrict__ counter, uint32_t* __restrict__ offsets,
                     uint32_t* __restrict__ bounds) {
  __shared__ uint32_t s_val[kSortTile];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_tile, s_excl;
  if (threadIdx.x == 0) s_tile = atomicAdd(counter, 1u);
  __syncthreads();
  const uint32_t tile = s_tile;
  const uint32_t base = tile * kSortTile;
  for (int k = 0; k < kSortItems; ++k) {
    const int j = k * kSortBlock + threadIdx.x;
    const uint32_t i = base + j;
    s_val[j] = i < n ? scan_value(values, order, i, bias) : 0u;
  }
  __syncthreads();
  uint32_t local[kSortItems];
  uint32_t sum = 0u;
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    local[k] = s_val[threadIdx.x * kSortItems + k];
    sum += local[k];
  }
  uint32_t tile_total;
  uint32_t run = block_exclusive_scan(sum, s_warp, &tile_total);
  if (threadIdx.x < 32) {
    unsigned long long* mine = status + tile;
    unsigned long long excl = 0ull;
    if (tile == 0) {
      if (threadIdx.x == 0) st_relaxed64(mine, Status64::kInclusive | tile_total);
    } else {
      if (threadIdx.x == 0) st_relaxed64(mine, Status64::kAggregate | tile_total);
      excl = warp_lookback<Status64>(status, static_cast<int64_t>(tile), 1);
      if (threadIdx.x == 0) st_relaxed64(mine, Status64::kInclusive | (excl + tile_total));
    }
    if (threadIdx.x == 0) s_excl = static_cast<uint32_t>(excl);
  }
  __syncthreads();
  run += s_excl;
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    s_val[threadIdx.x * kSortItems + k] = run;
    run += local[k];
  }
  __syncthreads();
  const unsigned long long W = *pair_total + static_cast<unsigned long long>(bias) * n;
  // number of k in [0, chunks) whose target floor(W k / chunks) is <= w
  auto below = [&](uint32_t w) -> uint32_t {
    if (W == 0ull) return chunks;
    const unsigned long long c =
        ((static_cast<unsigned long long>(w) + 1ull) * chunks + W - 1ull) / W;
    return static_cast<uint32_t>(c < chunks ? c : chunks);
  };
  const uint32_t cnt = min(static_cast<uint32_t>(kSortTile), n - base);
  const bool last = base + cnt == n;
  for (int k = 0; k < kSortItems; ++k) {  // coalesced
    const uint32_t j = k * kSortBlock + threadIdx.x;
    if (j < cnt) offsets[base + j] = s_val[j];
  }
  // this tile owns the bounds whose target lies in (e_0, e_end] (e: the
  // exclusive prefixes, e_end the tile's inclusive total): bound k is
  // base + (the first j in [1, cnt] with e_j >= target, e_cnt = e_end); tile
  // 0 also writes those at or below 0, the last tile every bound left and
  // bounds[chunks] = n.  Each bound is written once, complete and monotone
  // whatever the totals.
  const uint32_t e0 = s_val[0], e_end = s_excl + tile_total;
  const uint32_t k_lo = below(e0), k_hi = last ? chunks : below(e_end);
  if (tile == 0)
    for (uint32_t c = threadIdx.x; c < k_lo; c += blockDim.x) bounds[c] = 0u;
  for (uint32_t c = k_lo + threadIdx.x; c < k_hi; c += blockDim.x) {
    const unsigned long long target = W * c / chunks;
    uint32_t lo = 1, hi = cnt;  // first j in [1, cnt] with e_j >= target
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (s_val[mid] >= target) hi = mid; else lo = mid + 1;
    }
    bounds[c] = base + lo;
  }
  if (last && threadIdx.x == 0) {
    bounds[chunks] = n;
    offsets[n] = e_end;
  }
}

// ---- accutile emission --------------------------------------------------
// Pairs of the depth-ordered Gaussians in emission order (the strip walk of
// intersections.py:155-218), written at their depth-order offsets; stable
// passes on the tile id then give the reference order.  One thread per
// Gaussian.
__global__ void __launch_bounds__(256)
    emit_strips_kernel(uint32_t n, const uint32_t* __restrict__ order,
                       const uint32_t* __restrict__ offsets, const float* __restrict__ centers,
                       const float* __restrict__ conics, const int* __restrict__ radii,
                       int gx, int gy, uint32_t m, uint32_t* __restrict__ keys,
                       uint32_t* __restrict__ vals) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t g = order[i];
  const int radius = radii[g];
  if (radius <= 0) return;
  const float2 c = reinterpret_cast<const float2*>(centers)[g];
  const TileVisit tv = tile_visit(kTileAccutile, c.x, c.y,
                                  reinterpret_cast<const float4*>(conics)[g], radius, gx, gy);
  uint32_t pos = offsets[i];
  const uint32_t end = offsets[i + 1];
  walk_strips(tv, [&](int r, int2 span) {
    for (int col = span.x; col < span.y; ++col) {
      if (pos >= end || pos >= m) {  // counts disagree with the projection's
        record_device_error(kInconsistentInput);
        return;
      }
      keys[pos] = static_cast<uint32_t>(tv.is_y ? r * gx + col : col * gx + r);
      vals[pos] = g;
      ++pos;
    }
  });
}

// ---- chunked stable scatter ----------------------------------------------
// The depth-ordered Gaussians are cut into K chunks of about equal work
// (tiles + kChunkGaussianCost per Gaussian, from a prefix scan in depth
// order).  cnt[k][t] = pairs of chunk k in tile t; an exclusive prefix over
// k plus the tile's range start gives every chunk its first write position
// per tile, so all chunks scatter independently.  Inside a chunk the
// Gaussians are placed in depth order (tile_scatter_kernel).  The result is
// the depth order within every tile, i.e. the reference's stable sort of
// 64-bit keys.

constexpr uint32_t kChunkGaussianCost = 8;  // per-Gaussian scatter overhead, in pairs

SPLAT_DEV void unpack_rect(uint2 r, uint32_t& x0, uint32_t& y0, uint32_t& x1, uint32_t& y1) {
  x0 = r.x & 0xFFFFu;
  y0 = r.x >> 16;
  x1 = r.y & 0xFFFFu;
  y1 = r.y >> 16;
}

SPLAT_DEV uint32_t rect_area(uint2 r) {
  uint32_t x0, y0, x1, y1;
  unpack_rect(r, x0, y0, x1, y1);
  return (x1 > x0 && y1 > y0) ? (x1 - x0) * (y1 - y0) : 0u;
}

// cnt[k * T + t] for chunk k = blockIdx.x, from a difference grid of the
// chunk's rectangles in shared memory ((gx+1)*(gy+1) ints); also gathers
// the rectangles into depth order for the scatter.
__global__ void __launch_bounds__(256)
    chunk_counts_kernel(const uint32_t* __restrict__ order, const uint32_t* __restrict__ bounds,
                        const uint2* __restrict__ rects, int gx, int gy,
                        uint2* __restrict__ sorted_rects, uint32_t* __restrict__ cnt) {
  extern __shared__ int s_diff[];
  const int row = gx + 1, cells = row * (gy + 1);
  for (int c = threadIdx.x; c < cells; c += blockDim.x) s_diff[c] = 0;
  __syncthreads();
  const uint32_t begin = bounds[blockIdx.x], end = bounds[blockIdx.x + 1];
  for (uint32_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const uint2 r = rects[order[i]];
    sorted_rects[i] = r;
    uint32_t x0, y0, x1, y1;
    unpack_rect(r, x0, y0, x1, y1);
    if (x1 > x0 && y1 > y0) {
      atomicAdd(s_diff + y0 * row + x0, 1);
      atomicAdd(s_diff + y0 * row + x1, -1);
      atomicAdd(s_diff + y1 * row + x0, -1);
      atomicAdd(s_diff + y1 * row + x1, 1);
    }
  }
  __syncthreads();
  for (int y = threadIdx.x; y <= gy; y += blockDim.x) {
    int acc = 0;
    for (int x = 0; x <= gx; ++x) acc = (s_diff[y * row + x] += acc);
  }
  __syncthreads();
  for (int x = threadIdx.x; x <= gx; x += blockDim.x) {
    int acc = 0;
    for (int y = 0; y <= gy; ++y) acc = (s_diff[y * row + x] += acc);
  }
  __syncthreads();
  const int T = gx * gy;
  uint32_t* out = cnt + static_cast<size_t>(blockIdx.x) * T;
  for (int t = threadIdx.x; t < T; t += blockDim.x)
    out[t] = static_cast<uint32_t>(s_diff[(t / gx) * row + (t % gx)]);
}

// In place: cnt[k][t] -> sum of cnt[k'][t] over k' < k; totals[t] = the sum
// over all chunks.  Block: 32 tiles x 32 chunk segments (one warp each).
__global__ void __launch_bounds__(1024)
    chunk_prefix_kernel(uint32_t* __restrict__ cnt, int chunks, int T,
                        uint32_t* __restrict__ totals) {
  constexpr int kSegments = 32;
  __shared__ uint32_t s_seg[kSegments][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int t = blockIdx.x * 32 + lane;
  const int per = (chunks + kSegments - 1) / kSegments;
  const int k0 = min(seg * per, chunks), k1 = min(k0 + per, chunks);
  // kBatch independent loads in flight per step (a segment is tens of chunks)
  constexpr int kBatch = 8;
  uint32_t sum = 0u;
  if (t < T) {
    int k = k0;
    for (; k + kBatch <= k1; k += kBatch) {
      uint32_t v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) v[j] = cnt[static_cast<size_t>(k + j) * T + t];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) sum += v[j];
    }
    for (; k < k1; ++k) sum += cnt[static_cast<size_t>(k) * T + t];
  }
  s_seg[seg][lane] = sum;
  __syncthreads();
  uint32_t run = 0u;
  for (int q = 0; q < seg; ++q) run += s_seg[q][lane];
  if (t < T) {
    int k = k0;
    for (; k + kBatch <= k1; k += kBatch) {
      uint32_t v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) v[j] = cnt[static_cast<size_t>(k + j) * T + t];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        cnt[static_cast<size_t>(k + j) * T + t] = run;
        run += v[j];
      }
    }
    for (; k < k1; ++k) {
      uint32_t* c = cnt + static_cast<size_t>(k) * T + t;
      const uint32_t v = *c;
      *c = run;
      run += v;
    }
    if (seg == kSegments - 1) totals[t] = run;
  }
}

// One block: ranges from per-tile totals (empty tiles get [0, 0), as
// identify_ranges leaves them), the first position of every tile, and the
// pair total.  Each round stages kPer * 1024 totals in shared memory with
// coalesced loads, scans them (thread t owns kPer consecutive tiles), and
// writes the results back through shared memory with coalesced stores (a
// single block storing thread-major runs would touch a new 32-byte sector
// with every lane).
__global__ void __launch_bounds__(1024)
    tile_ranges_kernel(const uint32_t* __restrict__ totals, int T, int* __restrict__ ranges,
                       uint32_t* __restrict__ starts, uint32_t* __restrict__ total) {
  constexpr int kPer = 8;
  constexpr int kRound = 1024 * kPer;
  // row t of s_v at t + t / 32: thread-major reads of kPer words stay off
  // one bank
  __shared__ uint32_t s_v[kRound + kRound / 32];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_carry;
  auto slot = [](int k) { return k + (k >> 5); };
  if (threadIdx.x == 0) s_carry = 0u;
  for (int base = 0; base < T; base += kRound) {
    const int count = min(kRound, T - base);
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int k = r * 1024 + threadIdx.x;
      s_v[slot(k)] = k < count ? totals[base + k] : 0u;
    }
    __syncthreads();
    uint32_t v[kPer];
    uint32_t sum = 0u;
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      v[r] = s_v[slot(threadIdx.x * kPer + r)];
      sum += v[r];
    }
    uint32_t round_total;
    uint32_t run = block_exclusive_scan(sum, s_warp, &round_total) + s_carry;
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      s_v[slot(threadIdx.x * kPer + r)] = run;  // exclusive start of the tile
      run += v[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int k = r * 1024 + threadIdx.x;
      if (k < count) {
        const uint32_t first = s_v[slot(k)];
        const uint32_t n = totals[base + k];
        starts[base + k] = first;
        reinterpret_cast<int2*>(ranges)[base + k] =
            n ? make_int2(static_cast<int>(first), static_cast<int>(first + n)) : make_int2(0, 0);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) s_carry += round_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = s_carry;
}

// Scatter of chunk k = blockIdx.x: 8 warps, warp w places the chunk's pairs
// in tile rows y with y % 8 == w (interleaved rows keep the warps' loads
// even), so no two warps touch one tile and the block needs no barrier (a
// warp fills next[] for its own rows).  Dynamic shared memory: next[T], the
// next write position of every tile.  A warp walks the chunk's members
// 32 at a time in depth order; the pairs of those members in its rows
// (row-major inside each member's rectangle) are laid out over the lanes by
// a warp prefix scan, 32 per step.  Pairs of one step that share a tile
// come from distinct members in lane (= depth) order: each takes next[t]
// plus the number of lower peer lanes, and the highest peer advances
// next[t] by the peer count.
constexpr int kScatterWarps = 8;

__global__ void __launch_bounds__(32 * kScatterWarps)
    tile_scatter_kernel(const uint32_t* __restrict__ order, const uint32_t* __restrict__ bounds,
                        const uint2* __restrict__ sorted_rects, int gx, int gy,
                        const uint32_t* __restrict__ prefix, const uint32_t* __restrict__ starts,
                        uint32_t m, const uint32_t* __restrict__ pair_total,
                        uint32_t* __restrict__ ids) {
  // ids holds m entries; m may be a capacity above or below the true pair
  // count: positions past m are skipped (the caller re-emits when m was too
  // small) and only positions past the true count are an error
  const uint32_t total = __ldg(pair_total);
  extern __shared__ __align__(16) uint32_t s_next[];  // [T]
  const int T = gx * gy;
  const uint32_t* base = prefix + static_cast<size_t>(blockIdx.x) * T;
  const uint32_t begin = bounds[blockIdx.x], end = bounds[blockIdx.x + 1];
  const uint32_t lane = threadIdx.x & 31, band = threadIdx.x >> 5;
  // each warp fills next[] for its own rows only (no block barrier: a warp
  // starts placing pairs as soon as its rows are ready)
  for (int y = static_cast<int>(band); y < gy; y += kScatterWarps) {
#pragma unroll 4
    for (int x = static_cast<int>(lane); x < gx; x += 32) {
      const int t = y * gx + x;
      s_next[t] = starts[t] + base[t];
    }
  }
  __syncwarp();
  const uint32_t lt = lanemask_lt();
  // per warp, the window's Gaussians as (id, x0 | first row << 16, width,
  // 1/width bits): one shared-memory load per pair instead of a shuffle per
  // field
  __shared__ uint4 s_member[kScatterWarps][32];
  uint4* member = s_member[band];
  // member loads run one window ahead
  uint32_t next_g = 0u;
  uint2 next_r = make_uint2(0u, 0u);
  if (begin + lane < end) {
    next_g = __ldg(order + begin + lane);
    next_r = __ldg(sorted_rects + begin + lane);
  }
  for (uint32_t m0 = begin; m0 < end; m0 += 32) {
    const uint32_t g = next_g;
    const uint2 r = next_r;
    const uint32_t ahead = m0 + 32 + lane;
    next_g = 0u;
    next_r = make_uint2(0u, 0u);
    if (ahead < end) {
      next_g = __ldg(order + ahead);
      next_r = __ldg(sorted_rects + ahead);
    }
    // an empty rectangle (also the padding lanes past end) has no pairs
    uint32_t x0, y0, x1, y1, width = 0u, count = 0u;
    unpack_rect(r, x0, y0, x1, y1);
    // first row of the band at or below y0, and the band's rows in [y0, y1)
    const uint32_t fy = y0 + ((band - y0) & (kScatterWarps - 1));
    if (x1 > x0 && fy < y1) {
      width = x1 - x0;
      count = ((y1 - 1u - fy) / kScatterWarps + 1u) * width;
    }
    uint32_t incl = count;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= static_cast<uint32_t>(o)) incl += v;
    }
    const uint32_t P = __shfl_sync(0xffffffffu, incl, 31);
    if (P == 0u) continue;  // warp-uniform
    const float inv_w = width ? 1.0f / static_cast<float>(width) : 0.0f;
    __syncwarp();  // the previous window's readers are done with member[]
    member[lane] = make_uint4(g, x0 | (fy << 16), width, __float_as_uint(inv_w));
    __syncwarp();
    for (uint32_t o = 0; o < P; o += 32) {
      const uint32_t p = o + lane;
      // member j: the number of lanes whose inclusive prefix is <= p; before:
      // the largest such prefix (the index of the member's first pair)
      uint32_t j = 0u, before = 0u;
#pragma unroll
      for (uint32_t step = 16; step > 0; step >>= 1) {
        const uint32_t v = __shfl_sync(0xffffffffu, incl, j + step - 1u);
        if (v <= p) {
          j += step;
          before = v;
        }
      }
      const uint4 d = member[j];
      const uint32_t local = p - before;
      const uint32_t w = d.z;
      const float inv = __uint_as_float(d.w);
      const uint32_t mx0 = d.y & 0xFFFFu;
      const uint32_t mfy = d.y >> 16;
      const uint32_t mg = d.x;
      // local < 2^24: the float quotient is within one of the integer one
      uint32_t q = static_cast<uint32_t>(static_cast<float>(local) * inv);
      if (q * w > local)
        --q;
      else if ((q + 1u) * w <= local)
        ++q;
      const bool active = p < P;
      const uint32_t tile = active ? (mfy + kScatterWarps * q) * static_cast<uint32_t>(gx) +
                                         mx0 + (local - q * w)
                                   : 0xFFFFFFFFu;
      const uint32_t peers = __match_any_sync(0xffffffffu, tile);
      if (active) {
        const uint32_t pos = s_next[tile] + __popc(peers & lt);
        if (pos < m)
          ids[pos] = mg;
        else if (pos >= total)
          record_device_error(kInconsistentInput);
      }
      __syncwarp();
      if (active && (peers >> lane) == 1u) s_next[tile] += __popc(peers);
      __syncwarp();
    }
  }
}

// ---- tile counts, ranges and tile-id digit offsets (one block) ----------
__global__ void __launch_bounds__(1024)
    tile_counts_kernel(int* __restrict__ diff, int gx, int gy, int passes,
                       int* __restrict__ ranges, uint32_t* __restrict__ digit_offsets,
                       uint32_t* __restrict__ total) {
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_hist[3 * kRadix];
  __shared__ uint32_t s_carry;
  const int row = gx + 1;
  // 2D inclusive prefix of the difference grid: rows, then columns.
  for (int y = threadIdx.x; y <= gy; y += blockDim.x) {
    int acc = 0;
    for (int x = 0; x <= gx; ++x) {
      acc += diff[y * row + x];
      diff[y * row + x] = acc;
    }
  }
  __syncthreads();
  for (int x = threadIdx.x; x <= gx; x += blockDim.x) {
    int acc = 0;
    for (int y = 0; y <= gy; ++y) {
      acc += diff[y * row + x];
      diff[y * row + x] = acc;
    }
  }
  for (int k = threadIdx.x; k < 3 * kRadix; k += blockDim.x) s_hist[k] = 0u;
  if (threadIdx.x == 0) s_carry = 0u;
  __syncthreads();
  const int T = gx * gy;
  for (int base = 0; base < T; base += blockDim.x) {
    const int t = base + threadIdx.x;
    uint32_t c = 0u;
    if (t < T) c = static_cast<uint32_t>(max(diff[(t / gx) * row + (t % gx)], 0));
    uint32_t chunk;
    const uint32_t before = block_exclusive_scan(c, s_warp, &chunk) + s_carry;
    if (t < T) {
      ranges[2 * t] = c ? static_cast<int>(before) : 0;
      ranges[2 * t + 1] = c ? static_cast<int>(before + c) : 0;
      for (int p = 0; p < passes; ++p)
        if (c) atomicAdd(&s_hist[p * kRadix + ((static_cast<uint32_t>(t) >> (8 * p)) & 255u)], c);
    }
    __syncthreads();
    if (threadIdx.x == 0) s_carry += chunk;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = s_carry;
  __syncthreads();
  // exclusive scans of the tile-id digit histograms (first 256 threads)
  for (int p = 0; p < passes; ++p) {
    const uint32_t v = threadIdx.x < kRadix ? s_hist[p * kRadix + threadIdx.x] : 0u;
    const uint32_t before = block_exclusive_scan(v, s_warp, nullptr);
    if (threadIdx.x < kRadix) digit_offsets[p * kRadix + threadIdx.x] = before;
  }
}

}  // namespace splat
