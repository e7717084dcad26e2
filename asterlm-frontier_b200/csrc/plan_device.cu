// Device-side schedule for a ragged, paged decode batch (asterq_plan_batch) and the in-place
// append of a step's new tokens to the hot windows (asterq_batch_append).
//
// The host planner (Python, asterq.plan.build_plan) walks every sequence's chunks and cuts the
// batch into one contiguous share of equal estimated time per worker CTA.  In a decode loop
// every sequence grows by q_len tokens per step, so the schedule changes every step; this
// kernel rebuilds it on the GPU from page tables and lengths that live on the GPU, so the
// host's per-step planning cost is one launch (and a whole step can be recorded as a graph).
//
// Same tables and the same time model as the host planner (one B200 SM: a full cold tile
// 3.1 us, a full hot tile 2.1 us, a fixed 5 us per work item).  The cut: the concatenated
// units (16-row query blocks with the tiles they can see) have estimated time C; worker
// boundary k sits at k * ceil(C / W).  A boundary inside a unit becomes a cut at the first
// tile starting at or after it, kept when it is at least half the minimum piece time away from
// the unit's ends and from the previous boundary's cut (so no piece is a sliver, while cuts a
// worker share apart survive the snap to tile starts).  Pieces of a cut unit
// write partial records; the decode kernel merges a unit of at most 16 pieces itself (in the
// CTA that writes the last one), more go to the combine launch.
//
// One CTA of 1024 threads.  Every stage is a loop over an index space (sequences x pages,
// tiles, units, boundaries, items) strided over the threads, with block-wide prefix sums
// between stages over arrays in the caller's scratch buffer (the segment offsets also in
// shared memory while the tile table is written, up to 40K segments).
#include "asterq_internal.h"

namespace asterq {
namespace plan {

constexpr int kThreads = 1024;
constexpr int kColdTile = 128;
constexpr int kHotTile = 32;
constexpr int kRows = 16;
constexpr int kMaxQLen = 2048;
constexpr int kFusedMaxParts = 16;
constexpr long long kColdFixed = 1200, kColdFull = 1890;  // ns: fixed + per full tile (scaled by tokens)
constexpr long long kHotFixed = 800, kHotFull = 1285;
constexpr long long kItemNs = 5000;
constexpr long long kColdTileNs = kColdFixed + kColdFull;

struct Scratch {
  long long* tile_cost;  // [cap_tiles + 1] per-tile time, then its exclusive prefix
  long long* seg;        // [n_segs + 1] tiles per segment (cold page / hot window / new tokens), then offsets
  long long* seq_units;  // [n_seqs + 1]
  long long* unit_cost;  // [cap_units + 1]
  long long* unit_t;     // [cap_units + 1] first tile | (end of visible tiles << 32)
  long long* unit_np;    // [cap_units + 1] pieces, then item offsets
  long long* unit_ns;    // [cap_units + 1] partial-record slots, then offsets
  long long* unit_sep;   // [cap_units + 1] combine-launch jobs (0/1), then offsets
  long long* unit_fus;   // [cap_units + 1] fused jobs (0/1), then offsets
  long long* kept;       // [n_workers + 1] kept cut at boundary k (0/1), then its rank
  int* cand_tile;        // [n_workers] cut tile of boundary k, or -1
  int* cand_unit;        // [n_workers]
  int* kept_list;        // [n_workers] boundary of the r-th kept cut
  int* item_worker;      // [cap_items]
};

__host__ __device__ inline long long n_segments(int n_seqs, int max_cold_pages) {
  return (long long)n_seqs * (max_cold_pages + 2);
}

__host__ __device__ inline Scratch scratch_of(void* base, long long n_segs, int n_seqs, int cap_tiles, int cap_units,
                                              int n_workers) {
  long long* p = reinterpret_cast<long long*>(base);
  Scratch s;
  s.tile_cost = p;
  p += cap_tiles + 1;
  s.seg = p;
  p += n_segs + 1;
  s.seq_units = p;
  p += n_seqs + 1;
  long long** per_unit[] = {&s.unit_cost, &s.unit_t, &s.unit_np, &s.unit_ns, &s.unit_sep, &s.unit_fus};
  for (long long** q : per_unit) {
    *q = p;
    p += cap_units + 1;
  }
  s.kept = p;
  p += n_workers + 1;
  int* ip = reinterpret_cast<int*>(p);
  s.cand_tile = ip;
  ip += n_workers;
  s.cand_unit = ip;
  ip += n_workers;
  s.kept_list = ip;
  ip += n_workers;
  s.item_worker = ip;
  return s;
}

inline int64_t scratch_bytes(long long n_segs, int n_seqs, int cap_tiles, int cap_units, int cap_items, int n_workers) {
  const int64_t words = (int64_t)cap_tiles + 1 + n_segs + 1 + n_seqs + 1 + 6LL * ((int64_t)cap_units + 1) + n_workers + 1;
  return 8 * words + 4LL * (3LL * n_workers + cap_items);
}

// Exclusive prefix sum of a[0 .. n) in place over the whole block; returns the total.  Warp w
// owns one contiguous chunk, read 32 consecutive elements at a time (coalesced): the chunk
// sums are scanned by the first warp (two block barriers in all), then every warp scans its
// chunk 32 elements at a time with shuffles, carrying the running sum.
constexpr int kWarps = kThreads / 32;
static_assert(kWarps == 32, "the chunk totals are scanned by one warp");
__device__ long long block_scan(long long* a, long long n, long long* sm) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const long long per_warp = ((n + kWarps - 1) / kWarps + 31) / 32 * 32;
  const long long lo = min(n, wid * per_warp), hi = min(n, lo + per_warp);
  long long sum = 0;
  for (long long i = lo + lane; i < hi; i += 32) sum += a[i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) sm[wid] = sum;
  __syncthreads();
  if (wid == 0) {
    long long x = sm[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    sm[lane] = x;  // inclusive chunk sums
  }
  __syncthreads();
  long long run = (wid > 0) ? sm[wid - 1] : 0;
  const long long total = sm[kWarps - 1];
  for (long long base = lo; base < hi; base += 32) {
    const long long i = base + lane;
    const long long v = (i < hi) ? a[i] : 0;
    long long x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (i < hi) a[i] = run + x - v;
    run += __shfl_sync(0xffffffffu, x, 31);
  }
  __syncthreads();  // every thread has read `total` before `sm` is reused
  return total;
}

// largest i in [0, n) with off[i] <= x (off nondecreasing, off[0] <= x)
__device__ int upper_index(const long long* off, int n, long long x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// smallest i in [lo, hi) with pc[i] >= y, or hi
__device__ int lower_tile(const long long* pc, int lo, int hi, long long y) {
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (pc[mid] >= y) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

// a full cold tile costs the same whatever its token count: a 64-token int8 tile holds as many
// code bytes and MMAs as a 128-token INT4 tile
__device__ __forceinline__ long long cold_cost(int n, int ct) { return kColdFixed + (kColdFull * n) / ct; }
__host__ __device__ inline int cold_tile_of(const asterq_batch_desc& d) {
  return d.cold_tile_tokens == 64 ? 64 : kColdTile;
}
__device__ __forceinline__ long long hot_cost(int n) { return kHotFixed + (kHotFull * n) / kHotTile; }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }

__device__ void fail_all(const asterq_plan_buffers& b, int n_workers) {
  if (threadIdx.x == 0) {
    for (int k = 0; k < 8; ++k) b.counts[k] = 0;
    b.counts[5] = 1;
  }
  for (int w = threadIdx.x; w <= n_workers; w += kThreads) b.workers[w] = 0;
}

// segment offsets staged in shared memory for the per-tile pass (int32), when they fit
constexpr long long kSegSharedMax = 40 * 1024;

__host__ __device__ inline bool segs_in_shared(long long n_segs) { return n_segs + 1 <= kSegSharedMax; }

__global__ void __launch_bounds__(kThreads) plan_kernel(const asterq_batch_desc d, const asterq_plan_buffers b) {
  __shared__ long long sm[kThreads];
  extern __shared__ int seg_sh[];  // [n_segs + 1] when segs_in_shared(n_segs)
  const int tid = threadIdx.x;
  const int B = d.n_seqs, H = d.n_heads, W = d.n_workers, P = d.page_tokens, MC = d.max_cold_pages;
  const int seg_w = MC + 2;  // segments per sequence: MC cold pages, the hot window, the new tokens
  const long long n_segs = n_segments(B, MC);
  const Scratch s = scratch_of(b.scratch, n_segs, B, b.cap_tiles, b.cap_units, W);
  const int hot_tiles_per_page = (P + kHotTile - 1) / kHotTile;
  const int CT = cold_tile_of(d);  // tokens of a cold tile

  auto q_len = [&](int q) { return min(d.q_len[q], kMaxQLen); };  // <= 0: an inactive sequence slot

  // 1. tiles per segment, 16-row units per sequence (four segments per thread and pass, their
  //    loads in flight together)
  // (32-bit indices throughout: segment and tile counts are bounded by the int32 capacities,
  // and 64-bit division is a long software routine)
  const int n_segs32 = (int)n_segs;
  for (int g0 = tid; g0 < n_segs32; g0 += 4 * kThreads) {
    int ql[4], nc[4], x[4], qq[4], kk[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int g = min(g0 + u * kThreads, n_segs32 - 1);
      qq[u] = g / seg_w;
      kk[u] = g - qq[u] * seg_w;
      ql[u] = __ldg(d.q_len + qq[u]);
      nc[u] = __ldg(d.n_cold_pages + qq[u]);
      x[u] = (kk[u] < MC) ? __ldg(d.cold_page_tokens + (long long)qq[u] * MC + kk[u])
                          : (kk[u] == MC ? __ldg(d.hot_tokens + qq[u]) : 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int g = g0 + u * kThreads;
      if (g >= n_segs32) break;
      const int k = kk[u];
      const int qlen = min(ql[u], kMaxQLen);
      long long n = 0;
      if (qlen > 0) {
        if (k < MC) {
          if (k < clampi(nc[u], 0, MC)) n = (clampi(x[u], 0, P) + CT - 1) / CT;
        } else if (k == MC) {
          const int h = clampi(x[u], 0, d.max_hot_pages * P);
          n = (long long)(h / P) * hot_tiles_per_page + ((h % P) + kHotTile - 1) / kHotTile;
        } else {
          n = (qlen + kHotTile - 1) / kHotTile;
        }
      }
      s.seg[g] = n;
    }
  }
  for (int q = tid; q < B; q += kThreads)
    s.seq_units[q] = q_len(q) > 0 ? ((long long)q_len(q) * H + kRows - 1) / kRows : 0;
  __syncthreads();
  const long long n_tiles = block_scan(s.seg, n_segs, sm);
  const long long n_units = block_scan(s.seq_units, B, sm);
  if (n_tiles > b.cap_tiles || n_units > b.cap_units) {
    fail_all(b, W);
    return;
  }
  if (tid == 0) {
    s.seg[n_segs] = n_tiles;
    s.seq_units[B] = n_units;
  }
  __syncthreads();

  // 2. the tile table and the tiles' estimated times, one thread per tile (a segment can hold
  //    a whole hot window of tiles, too many for one thread): tile t lies in the last segment
  //    whose offset is <= t, found by binary search over the offsets (in shared memory when
  //    they fit; empty segments share their successor's offset and never win the search)
  const bool sh = segs_in_shared(n_segs);
  if (sh)
    for (long long g = tid; g <= n_segs; g += kThreads) seg_sh[g] = (int)s.seg[g];
  __syncthreads();
  // four tiles per thread and pass: their searches, then all their loads, then the stores, so
  // the loads of the four are in flight together
  constexpr int kU = 4;
  const int n_tiles32 = (int)n_tiles;
  for (int t0 = tid; t0 < n_tiles32; t0 += kU * kThreads) {
    int g[kU], i[kU], kk[kU];
    const int* src1[kU];
    const int* src2[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = t0 + u * kThreads;
      g[u] = 0;
      if (t < n_tiles32) {
        int lo = 0, hi = n_segs32 - 1;
        if (sh) {
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (seg_sh[mid] <= t) lo = mid;
            else hi = mid - 1;
          }
        } else {
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s.seg[mid] <= t) lo = mid;
            else hi = mid - 1;
          }
        }
        g[u] = lo;
      }
      i[u] = t - (sh ? seg_sh[g[u]] : (int)s.seg[g[u]]);
      const int q = g[u] / seg_w, k = g[u] - q * seg_w;
      kk[u] = k;
      if (k < MC) {  // page id, tokens in the page
        src1[u] = d.cold_pages + (long long)q * MC + k;
        src2[u] = d.cold_page_tokens + (long long)q * MC + k;
      } else if (k == MC) {  // page id, hot tokens
        src1[u] = d.hot_pages + (long long)q * d.max_hot_pages + i[u] / hot_tiles_per_page;
        src2[u] = d.hot_tokens + q;
      } else {  // first row of the new tokens, their number
        src1[u] = d.q_start + q;
        src2[u] = d.q_len + q;
      }
    }
    int v1[kU], v2[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const bool live = t0 + u * kThreads < n_tiles32;
      v1[u] = live ? __ldg(src1[u]) : 0;
      v2[u] = live ? __ldg(src2[u]) : 0;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = t0 + u * kThreads;
      if (t >= n_tiles32) break;
      const int k = kk[u];
      int4 tile;
      if (k < MC) {
        const int tok = clampi(v2[u], 0, P), off = i[u] * CT;
        tile = make_int4(ASTERQ_TILE_COLD, v1[u], off, min(CT, tok - off));
        s.tile_cost[t] = cold_cost(tile.w, CT);
      } else if (k == MC) {
        const int h = clampi(v2[u], 0, d.max_hot_pages * P), page = i[u] / hot_tiles_per_page;
        const int off = (i[u] - page * hot_tiles_per_page) * kHotTile;
        tile = make_int4(ASTERQ_TILE_HOT, v1[u], off, min(kHotTile, min(P, h - page * P) - off));
        s.tile_cost[t] = hot_cost(tile.w);
      } else {
        const int off = i[u] * kHotTile;
        tile = make_int4(ASTERQ_TILE_NEW, v1[u], off, min(kHotTile, min(v2[u], kMaxQLen) - off));
        s.tile_cost[t] = hot_cost(tile.w);
      }
      *reinterpret_cast<int4*>(b.tiles + 4 * t) = tile;
    }
  }
  __syncthreads();
  const long long tile_total = block_scan(s.tile_cost, n_tiles, sm);
  if (tid == 0) s.tile_cost[n_tiles] = tile_total;
  __syncthreads();
  const long long* pc = s.tile_cost;

  // 3. units: query rows, visible tiles (new-token tiles wholly after the block's last token
  //    are fully masked, latent_attention.py:151-153, and dropped), estimated time
  for (long long u = tid; u < n_units; u += kThreads) {
    const int q = upper_index(s.seq_units, B, u);
    const int rb = (int)(u - s.seq_units[q]);
    const int rows = q_len(q) * H;
    const long long t0 = s.seg[(long long)q * seg_w];
    const long long t_new = s.seg[(long long)q * seg_w + MC + 1];
    const int last_token = (min(rows, kRows * (rb + 1)) - 1) / H;
    const long long t1 = t_new + last_token / kHotTile + 1;
    s.unit_cost[u] = pc[t1] - pc[t0] + kItemNs;
    s.unit_t[u] = t0 | (t1 << 32);
    b.units[2 * u] = d.q_start[q] * H + kRows * rb;
    b.units[2 * u + 1] = min(kRows, rows - kRows * rb);
  }
  __syncthreads();
  const long long total = block_scan(s.unit_cost, n_units, sm);
  if (tid == 0) s.unit_cost[n_units] = total;
  __syncthreads();
  const long long* uoff = s.unit_cost;
  const long long wd = max(1LL, (total + W - 1) / W);
  const long long min_gap = max(kColdTileNs, min(4 * kColdTileNs, total / W)) / 2;

  // 4. candidate cuts, one per worker boundary k = 1 .. W-1 at time k * wd
  for (int k = tid; k < W; k += kThreads) {
    int ct = -1, cu = -1;
    const long long x = (long long)k * wd;
    if (k > 0 && x < total) {
      const int u = upper_index(uoff, (int)n_units, x);
      const int t0 = (int)(s.unit_t[u] & 0xffffffffLL), t1 = (int)(s.unit_t[u] >> 32);
      const long long y = x - (uoff[u] + kItemNs) + pc[t0];  // the item's fixed time comes first
      if (y > pc[t0]) {
        const int lo = lower_tile(pc, t0 + 1, t1, y);
        if (lo < t1) {
          ct = lo;
          cu = u;
        }
      }
    }
    s.cand_tile[k] = ct;
    s.cand_unit[k] = cu;
  }
  __syncthreads();
  for (int k = tid; k < W; k += kThreads) {
    long long keep = 0;
    const int ct = s.cand_tile[k], u = s.cand_unit[k];
    if (ct >= 0) {
      const int t0 = (int)(s.unit_t[u] & 0xffffffffLL), t1 = (int)(s.unit_t[u] >> 32);
      keep = pc[ct] - pc[t0] >= min_gap && pc[t1] - pc[ct] >= min_gap;
      if (keep && k > 1 && s.cand_unit[k - 1] == u && s.cand_tile[k - 1] >= 0)
        keep = pc[ct] - pc[s.cand_tile[k - 1]] >= min_gap;
    }
    s.kept[k] = keep;
  }
  __syncthreads();
  const long long n_cuts = block_scan(s.kept, W, sm);
  if (tid == 0) s.kept[W] = n_cuts;
  __syncthreads();
  for (int k = tid; k < W; k += kThreads)
    if (s.kept[k + 1] > s.kept[k]) s.kept_list[s.kept[k]] = k;

  // 5. pieces per unit (boundaries k in [ceil(ub / wd), ceil(ue / wd)) fall inside unit u)
  auto boundary_range = [&](long long u, int& kb, int& ke) {
    kb = (int)min((long long)W, (uoff[u] + wd - 1) / wd);
    ke = (int)min((long long)W, (uoff[u + 1] + wd - 1) / wd);
  };
  for (long long u = tid; u < n_units; u += kThreads) {
    int kb, ke;
    boundary_range(u, kb, ke);
    const long long np = 1 + s.kept[ke] - s.kept[kb];
    s.unit_np[u] = np;
    s.unit_ns[u] = np > 1 ? np : 0;
    s.unit_sep[u] = np > kFusedMaxParts;
    s.unit_fus[u] = np > 1 && np <= kFusedMaxParts;
  }
  __syncthreads();
  const long long n_items = block_scan(s.unit_np, n_units, sm);
  const long long n_slots = block_scan(s.unit_ns, n_units, sm);
  const long long n_sep = block_scan(s.unit_sep, n_units, sm);
  const long long n_fus = block_scan(s.unit_fus, n_units, sm);
  if (n_items > b.cap_items) {
    fail_all(b, W);
    return;
  }
  if (tid == 0) s.unit_np[n_units] = n_items;
  __syncthreads();

  // 6. work items, in unit order (which is also worker order): the first piece of every unit,
  //    then the piece after every kept cut
  auto emit = [&](long long u, long long idx, int a, int e, int piece, long long np) {
    const int q = upper_index(s.seq_units, B, u);
    const int rb = (int)(u - s.seq_units[q]);
    const int slot = np > 1 ? (int)(s.unit_ns[u] + piece) : -1;
    int* it = b.items + 8 * idx;
    *reinterpret_cast<int4*>(it) = make_int4((int)u, rb, a, e);
    *reinterpret_cast<int4*>(it + 4) = make_int4(slot, b.units[2 * u], b.units[2 * u + 1], q_len(q));
    const int t0 = (int)(s.unit_t[u] & 0xffffffffLL);
    // A later piece starts at its cut, a worker boundary.  A unit's first piece goes to the
    // worker whose share holds the middle of its time span: when the boundary just after the
    // unit's start made no cut (the piece would have been a sliver), the piece runs on to the
    // next cut, a whole share further on, and belongs to the later worker; when that boundary
    // did cut a short first piece, the piece lies before it and belongs to the earlier one.
    long long at;
    if (a == t0) {
      const long long end = (e < (int)(s.unit_t[u] >> 32)) ? uoff[u] + kItemNs + pc[e] - pc[t0] : uoff[u + 1];
      at = (uoff[u] + end) / 2;
    } else {
      at = uoff[u] + kItemNs + pc[a] - pc[t0];
    }
    s.item_worker[idx] = (int)min((long long)W - 1, at / wd);
  };
  for (long long u = tid; u < n_units; u += kThreads) {
    int kb, ke;
    boundary_range(u, kb, ke);
    const int t0 = (int)(s.unit_t[u] & 0xffffffffLL), t1 = (int)(s.unit_t[u] >> 32);
    const long long np = s.unit_np[u + 1] - s.unit_np[u];
    const int e = np > 1 ? s.cand_tile[s.kept_list[s.kept[kb]]] : t1;
    emit(u, s.unit_np[u], t0, e, 0, np);
    if (np > 1) {
      const int slot0 = (int)s.unit_ns[u];
      const bool fused = np <= kFusedMaxParts;
      const long long job = fused ? n_sep + s.unit_fus[u] : s.unit_sep[u];
      *reinterpret_cast<int4*>(b.combine + 4 * job) =
          make_int4(slot0, slot0 + (int)np, b.units[2 * u], b.units[2 * u + 1]);
      b.unit_jobs[u] = fused ? (int)job : -1;
    } else {
      b.unit_jobs[u] = -1;
    }
  }
  for (int k = tid; k < W; k += kThreads) {
    if (s.kept[k + 1] == s.kept[k]) continue;
    const int u = s.cand_unit[k];
    int kb, ke;
    boundary_range(u, kb, ke);
    const long long r = s.kept[k];
    const int t1 = (int)(s.unit_t[u] >> 32);
    const int e = (r + 1 < s.kept[ke]) ? s.cand_tile[s.kept_list[r + 1]] : t1;
    const long long np = s.unit_np[u + 1] - s.unit_np[u];
    const int piece = 1 + (int)(r - s.kept[kb]);
    emit(u, s.unit_np[u] + piece, s.cand_tile[k], e, piece, np);
  }
  __syncthreads();

  // 7. workers[w] = first item of worker w (items are in nondecreasing worker order)
  if (n_items == 0)
    for (int w = tid; w <= W; w += kThreads) b.workers[w] = 0;
  for (long long i = tid; i < n_items; i += kThreads) {
    const int wi = s.item_worker[i], wp = (i > 0) ? s.item_worker[i - 1] : -1;
    for (int w = wp + 1; w <= wi; ++w) b.workers[w] = (int)i;
    if (i == n_items - 1)
      for (int w = wi + 1; w <= W; ++w) b.workers[w] = (int)n_items;
  }
  __syncthreads();

  // 8. a worker whose last item is a piece of a cut unit runs it first, so that the unit's
  //    pieces all end early and its merge does not trail the kernel
  for (int w = tid; w < W; w += kThreads) {
    const int i0 = b.workers[w], i1 = b.workers[w + 1];
    if (i1 - i0 < 2 || b.items[8 * (i1 - 1) + 4] < 0) continue;
    const int f = i0 + (b.items[8 * i0 + 4] >= 0 ? 1 : 0);  // after a leading piece, if any
    if (f >= i1 - 1) continue;
    const int4 lo = *reinterpret_cast<const int4*>(b.items + 8 * (i1 - 1));
    const int4 hi = *reinterpret_cast<const int4*>(b.items + 8 * (i1 - 1) + 4);
    for (int i = i1 - 1; i > f; --i) {
      *reinterpret_cast<int4*>(b.items + 8 * i) = *reinterpret_cast<const int4*>(b.items + 8 * (i - 1));
      *reinterpret_cast<int4*>(b.items + 8 * i + 4) = *reinterpret_cast<const int4*>(b.items + 8 * (i - 1) + 4);
    }
    *reinterpret_cast<int4*>(b.items + 8 * f) = lo;
    *reinterpret_cast<int4*>(b.items + 8 * f + 4) = hi;
  }
  if (tid == 0) {
    b.counts[0] = (int)n_tiles;
    b.counts[1] = (int)n_units;
    b.counts[2] = (int)n_items;
    b.counts[3] = (int)n_slots;
    b.counts[4] = (int)(n_sep + n_fus);
    b.counts[5] = 0;
    b.counts[6] = (int)n_sep;
    b.counts[7] = 0;
  }
}

// One CTA per sequence: copy its q_len new tokens (rows q_start ..) into its hot window at
// positions hot_tokens .., then advance hot_tokens.  A position whose page is missing
// (beyond max_hot_pages, or a page id outside the pool) or rows beyond total_q fail the whole
// sequence: nothing is written, hot_tokens stays, *status = 1.
__global__ void __launch_bounds__(128) append_kernel(const asterq_batch_desc d, int* __restrict__ hot_tokens,
                                                    const uint4* __restrict__ new_latent,
                                                    const uint4* __restrict__ new_rope, uint4* __restrict__ hot_latent,
                                                    uint4* __restrict__ hot_rope, long long total_q,
                                                    long long n_pool_pages, int* __restrict__ status) {
  constexpr int kLatVec = 512 * 2 / 16, kRopeVec = 64 * 2 / 16, kVec = kLatVec + kRopeVec;
  __shared__ int ok;
  const int q = blockIdx.x, tid = threadIdx.x, P = d.page_tokens;
  const int ql = min(d.q_len[q], kMaxQLen);
  if (ql <= 0) return;
  const int h = hot_tokens[q];
  if (tid == 0) {
    int good = h >= 0 && (long long)h + ql <= (long long)d.max_hot_pages * P && d.q_start[q] >= 0 &&
               (long long)d.q_start[q] + ql <= total_q;
    for (int pg = good ? h / P : 0; good && pg <= (h + ql - 1) / P; ++pg) {
      const int id = d.hot_pages[(long long)q * d.max_hot_pages + pg];
      good = id >= 0 && id < n_pool_pages;
    }
    ok = good;
    if (!good && status) atomicExch(status, 1);
  }
  __syncthreads();
  if (!ok) return;
  const long long row0 = d.q_start[q];
  for (int v = tid; v < ql * kVec; v += blockDim.x) {
    const int t = v / kVec, c = v % kVec, pos = h + t;
    const long long dst = (long long)d.hot_pages[(long long)q * d.max_hot_pages + pos / P] * P + pos % P;
    if (c < kLatVec) hot_latent[dst * kLatVec + c] = new_latent[(row0 + t) * kLatVec + c];
    else hot_rope[dst * kRopeVec + (c - kLatVec)] = new_rope[(row0 + t) * kRopeVec + (c - kLatVec)];
  }
  __syncthreads();
  if (tid == 0) hot_tokens[q] = h + ql;
}

}  // namespace plan
}  // namespace asterq

using namespace asterq;

namespace {

int check_desc(const asterq_batch_desc* d, const char* who) {
  if (!d) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "%s: null descriptor", who);
  if (d->n_seqs < 0 || d->n_heads <= 0 || d->n_workers <= 0 || d->max_cold_pages < 0 || d->max_hot_pages < 0)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "%s: bad sizes", who);
  if (d->page_tokens <= 0 || d->page_tokens % 16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "%s: page_tokens %d must be a positive multiple of 16", who,
                     d->page_tokens);
  if (d->cold_tile_tokens != 0 && d->cold_tile_tokens != 64 && d->cold_tile_tokens != 128)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "%s: cold_tile_tokens %d must be 0, 64 or 128", who,
                     d->cold_tile_tokens);
  if (d->n_seqs > 0 && (!d->n_cold_pages || !d->cold_page_tokens || !d->hot_tokens || !d->q_len || !d->q_start ||
                        (d->max_cold_pages > 0 && !d->cold_pages) || (d->max_hot_pages > 0 && !d->hot_pages)))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "%s: null sequence table", who);
  return ASTERQ_OK;
}

}  // namespace

extern "C" int64_t asterq_plan_scratch_bytes(const asterq_batch_desc* d, int32_t cap_tiles, int32_t cap_units,
                                             int32_t cap_items) {
  if (!d || d->n_seqs < 0 || d->max_cold_pages < 0 || d->n_workers <= 0 || cap_tiles < 0 || cap_units < 0 ||
      cap_items < 0)
    return 0;
  return plan::scratch_bytes(plan::n_segments(d->n_seqs, d->max_cold_pages), d->n_seqs, cap_tiles, cap_units,
                             cap_items, d->n_workers);
}

extern "C" int asterq_plan_batch(const asterq_batch_desc* d, const asterq_plan_buffers* b, void* stream) {
  clear_error();
  int st = check_desc(d, "plan_batch");
  if (st != ASTERQ_OK) return st;
  if (!b) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "plan_batch: null plan buffers");
  if (b->cap_tiles < 0 || b->cap_units < 0 || b->cap_items < 0)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "plan_batch: negative capacity");
  if (!b->tiles || !b->units || !b->items || !b->combine || !b->unit_jobs || !b->workers || !b->counts || !b->scratch)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "plan_batch: null plan buffer");
  const void* aligned[] = {b->tiles, b->items, b->combine, b->units, b->scratch};
  for (const void* ptr : aligned)
    if (reinterpret_cast<uintptr_t>(ptr) & 15)
      return set_error(ASTERQ_ERR_MISALIGNED, "plan_batch: tables and scratch must be 16-byte aligned");
  const long long n_segs = plan::n_segments(d->n_seqs, d->max_cold_pages);
  const size_t smem = plan::segs_in_shared(n_segs) ? (size_t)(n_segs + 1) * sizeof(int) : 0;
  static int configured_device = -1;  // the opt-in above 48 KB is per device
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev != configured_device) {
    cudaError_t e = cudaFuncSetAttribute(plan::plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(plan::kSegSharedMax * sizeof(int)));
    if (e != cudaSuccess)
      return set_error(ASTERQ_ERR_CUDA, "plan_batch: shared memory opt-in: %s", cudaGetErrorString(e));
    configured_device = dev;
  }
  plan::plan_kernel<<<1, plan::kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(*d, *b);
  return check_launch("plan_batch");
}

extern "C" int asterq_batch_append(const asterq_batch_desc* d, int32_t* hot_tokens, const void* new_latent,
                                   const void* new_rope, int64_t total_q, void* hot_latent, void* hot_rope,
                                   int64_t n_hot_pool_pages, int32_t* status, void* stream) {
  clear_error();
  int st = check_desc(d, "batch_append");
  if (st != ASTERQ_OK) return st;
  if (d->n_seqs == 0) return ASTERQ_OK;
  if (!hot_tokens || !new_latent || !new_rope || !hot_latent || !hot_rope || n_hot_pool_pages < 0 || total_q < 0)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "batch_append: null pointer or bad size");
  const void* aligned[] = {new_latent, new_rope, hot_latent, hot_rope};
  for (const void* ptr : aligned)
    if (reinterpret_cast<uintptr_t>(ptr) & 15)
      return set_error(ASTERQ_ERR_MISALIGNED, "batch_append: token arrays and pools must be 16-byte aligned");
  plan::append_kernel<<<d->n_seqs, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      *d, hot_tokens, static_cast<const uint4*>(new_latent), static_cast<const uint4*>(new_rope),
      static_cast<uint4*>(hot_latent), static_cast<uint4*>(hot_rope), total_q, n_hot_pool_pages, status);
  return check_launch("batch_append");
}
