// Device-side step metadata and work lists, so that a whole decode (or
// verify) step can be replayed from a CUDA graph with no host planning and no
// host-to-device copies.
//
// The reference builds the step on the host every step: CudaModel::prepare
// (src/cuda_model.cpp:131-142) walks every sequence's tokens to form slots,
// positions, qo/kv indptr, the concatenated block tables and the last-page
// fill (padding entries of a graph bucket get slot -1, the dummy page and
// last = rows, :138), and prepare_plan (src/flashinfer_attention.cu:29-34)
// plans on the host and copies four pageable vectors to the device. Here one
// kernel does both from device-resident state:
//
//  mode 1 (fe_step_prepare_device): from block tables, per-sequence start
//         positions and a fixed row count per sequence (the graph entry's
//         shape), it writes slots / positions (int64, the store kernel's
//         input) and the qo / kv / last / pages arrays;
//  mode 0 (fe_attn_plan_prepare_device): the caller's device qo / kv /
//         pages / last (the layout of fe_attn_plan_prepare).
//
// Then it validates the step like the host planner (fe_attn_plan.cpp) and
// writes the packed work lists in place:
//  - the decode list (sequences with at most 16 packed query rows) is the
//    host planner's exact-cut list: the units' key-tile ranges are laid end
//    to end and cut into equal contiguous pieces, one per CTA. Every cut is a
//    function of prefix sums, so the device list is the host's item for item
//    (the same split points, hence bit-identical outputs);
//  - the row lists (prefill / verify units, never split: head_dim 256 plans
//    too, where the host planner may split them) sort the units by
//    cost, longest first (a bitonic sort in shared memory, up to
//    kMaxRowUnits units), and deal them to the CTAs in a snake order (0, 1,
//    ..., n-1, n-1, ..., 0, ...), which needs only each unit's rank instead
//    of the host's sequential least-loaded choice. Each item is computed whole
//    by one CTA either way, so outputs do not depend on the assignment.
// The plan is graph-mode: both attention kernels run at full width and CTAs
// without work exit. Invalid metadata or exceeded capacity empties the plan
// (every list has zero items) and raises FE_DEVERR_PLAN.
//
// One CTA of 1024 threads: every step is a block-wide scan, a per-sequence
// loop or a per-unit loop, with no atomics and no inter-CTA synchronisation.
#include "fe_attn_plan.h"
#include "fe_common.cuh"
#include "fe_plan_device.h"

namespace fe {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kMaxRowUnits = 8192;  // sort keys in shared memory (64 KiB)

__device__ __forceinline__ int64_t align16_dev(int64_t n) { return (n + 15) & ~int64_t(15); }
__device__ __forceinline__ int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Exclusive block-wide prefix sum of one value per thread; `total` receives
// the sum over the block. Every thread of the block must call it.
__device__ int64_t block_scan_excl(int64_t v, int64_t* wsum, int64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t s = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    wsum[lane] = s;  // inclusive over warps
  }
  __syncthreads();
  const int64_t before = warp > 0 ? wsum[warp - 1] : 0;
  total = wsum[kPlanWarps - 1];
  __syncthreads();  // wsum is reused by the next call
  return before + x - v;
}

// Exclusive prefix sum over n values (value(i)), written through write(i, ex);
// returns the total. Index i is handled by thread i % 1024, so a later loop
// over the same indices reads back what this thread wrote.
template <typename F, typename W>
__device__ int64_t scan_range(int n, F value, W write, int64_t* wsum) {
  int64_t carry = 0;
  for (int base = 0; base < n; base += kPlanThreads) {
    const int i = base + threadIdx.x;
    const int64_t v = i < n ? value(i) : 0;
    int64_t tot;
    const int64_t ex = block_scan_excl(v, wsum, tot);
    if (i < n) write(i, carry + ex);
    carry += tot;
  }
  return carry;
}

// First item of CTA c when `n` items of rank 0..n-1 are dealt in snake order
// to `grid` CTAs: rank r goes to round q = r / grid, position m = r % grid,
// CTA m in even rounds and grid-1-m in odd ones.
__device__ __forceinline__ int snake_off(int c, int n, int grid) {
  const int Q = n / grid, R = n % grid;
  return c * Q + ((Q & 1) == 0 ? min(c, R) : max(0, c - (grid - R)));
}

// Sort n (<= kMaxRowUnits) keys ascending in shared memory.
__device__ void bitonic_sort(uint64_t* keys, int n) {
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int i = n + threadIdx.x; i < n2; i += kPlanThreads) keys[i] = ~uint64_t(0);
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += kPlanThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = keys[i], y = keys[ixj];
          if ((x > y) == ((i & k) == 0)) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

__global__ void __launch_bounds__(kPlanThreads, 1) plan_device_kernel(const DevPlanArgs a) {
  extern __shared__ uint64_t sort_keys[];  // [kMaxRowUnits]
  __shared__ int64_t wsum[32];
  __shared__ int64_t sh[16];
  int bad = 0;  // this thread's verdict; combined over the block by __syncthreads_or
  const int tid = threadIdx.x;
  const int B = a.batch;
  const int page = a.page;
  MetaHeader* hdr = reinterpret_cast<MetaHeader*>(a.meta);
  const int64_t seqs_off = sizeof(MetaHeader);
  const int64_t pages_off = align16_dev(seqs_off + int64_t(sizeof(SeqInfo)) * B);
  int32_t* pages_out = reinterpret_cast<int32_t*>(a.meta + pages_off);
  if (B < 0 || B > a.max_batch || a.rows < 0) goto fail;  // uniform over the block

  {
    const int32_t* qo = a.qo;
    const int32_t* kv = a.kv;
    const int32_t* last = a.last;
    const int32_t* pages_in = a.pages;
    if (a.mode == 1) {
      // ---- step build (CudaModel::prepare): page counts, fill, slots ----
      const int rps = a.rows_per_seq;
      const int64_t total_pages = scan_range(
          B,
          [&](int b) -> int64_t {
            const int st = a.starts[b];
            if (st < 0) return 1;  // padding entry: the dummy page
            const int64_t n = cdiv(int64_t(st) + rps, page);
            if (n > a.stride || n > a.max_pages) bad = 1;  // the table must cover the context
            return n;
          },
          [&](int b, int64_t ex) { a.s_kv[b] = static_cast<int32_t>(ex); }, wsum);
      if (total_pages > int64_t(a.max_batch) * a.max_pages) bad = 1;
      if (__syncthreads_or(bad)) goto fail;
      for (int b = tid; b <= B; b += kPlanThreads) {
        a.s_qo[b] = b * rps;
        if (b == B) {
          a.s_kv[B] = static_cast<int32_t>(total_pages);
        } else {
          const int st = a.starts[b];
          a.s_last[b] = st < 0 ? rps : static_cast<int32_t>((int64_t(st) + rps - 1) % page + 1);
        }
      }
      __syncthreads();
      // block-table rows -> concatenated pages (one warp per sequence; four
      // independent loads per lane in flight before their stores)
      for (int b = tid >> 5; b < B; b += kPlanWarps) {
        const int st = a.starts[b];
        const int p0 = a.s_kv[b];
        const int n = a.s_kv[b + 1] - p0;
        const int32_t* row = a.tables + int64_t(b) * a.stride;
        for (int i0 = tid & 31; i0 < n; i0 += 128) {
          int32_t v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = i0 + 32 * u;
            v[u] = i < n ? (st < 0 ? a.num_blocks : __ldg(row + i)) : 0;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (i0 + 32 * u < n) pages_out[p0 + i0 + 32 * u] = v[u];
        }
      }
      // slot and position of every row (padding rows: slot -1, position j)
      for (int r = tid; r < B * rps; r += kPlanThreads) {
        const int b = r / rps, j = r % rps;
        const int st = a.starts[b];
        int64_t pos = j, slot = -1;
        if (st >= 0) {
          pos = int64_t(st) + j;
          const int32_t blk = a.tables[int64_t(b) * a.stride + pos / page];
          slot = int64_t(blk) * page + pos % page;
        }
        a.positions[r] = pos;
        a.slots[r] = slot;
      }
      __syncthreads();
      qo = a.s_qo;
      kv = a.s_kv;
      last = a.s_last;
      pages_in = pages_out;
    }

    // ---- validation (the host planner's checks) --------------------------
    if (tid == 0 && B > 0) {
      if (qo[0] != 0 || kv[0] != 0 || qo[B] != a.rows || kv[B] < 0 ||
          int64_t(kv[B]) > int64_t(a.max_batch) * a.max_pages)
        bad = 1;
    }
    if (tid == 0 && B == 0 && a.rows != 0) bad = 1;
    if (__syncthreads_or(bad)) goto fail;
    for (int b = tid; b < B; b += kPlanThreads) {
      const int q0 = qo[b], q1 = qo[b + 1], p0 = kv[b], p1 = kv[b + 1], ln = last[b];
      if (q1 < q0 || p1 <= p0 || ln < 1 || ln > page || p1 - p0 > a.max_pages) {
        bad = 1;
      } else if (int64_t(p1 - p0 - 1) * page + ln < q1 - q0) {
        bad = 1;  // fewer keys than query rows
      }
    }
    if (__syncthreads_or(bad)) goto fail;
    const int total_pages = B > 0 ? kv[B] : 0;
    for (int i0 = tid; i0 < total_pages; i0 += 4 * kPlanThreads) {
      int32_t pid[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kPlanThreads;
        pid[u] = i < total_pages ? pages_in[i] : 0;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kPlanThreads;
        if (i >= total_pages) continue;
        if (pid[u] < 0 || pid[u] > a.num_blocks) bad = 1;
        if (a.mode == 0) pages_out[i] = pid[u];
      }
    }
    if (__syncthreads_or(bad)) goto fail;

    // ---- sequences and work units ----------------------------------------
    const int G = a.hq / a.hkv, H = a.dec_heads;
    SeqInfo* seqs = reinterpret_cast<SeqInfo*>(a.meta + seqs_off);
    int32_t* c_row = a.s_cnt;                           // row-unit offsets
    int32_t* c_item = a.s_cnt + (a.max_batch + 1);      // decode-item offsets
    int32_t* c_grp = a.s_cnt + 2 * (a.max_batch + 1);   // split-group offsets
    int64_t* p_tiles = a.s_pref;                        // decode-tile offsets
    int64_t* p_part = a.s_pref + (a.max_batch + 1);     // split-record float offsets
    auto seq_len = [&](int b) -> int { return (kv[b + 1] - kv[b] - 1) * page + last[b]; };
    auto seq_rb = [&](int b) -> int {
      return int(cdiv(int64_t(qo[b + 1] - qo[b]) * G, kRowBlock));
    };
    auto n_dec = [&](int b) -> int {
      const int q = qo[b + 1] - qo[b];
      return (q > 0 && seq_rb(b) == 1) ? a.hkv / H : 0;
    };
    auto n_row = [&](int b) -> int {
      const int rb = seq_rb(b);
      return rb > 1 ? int(cdiv(rb, 8)) * a.hkv : 0;
    };
    for (int b = tid; b < B; b += kPlanThreads)
      seqs[b] = SeqInfo{qo[b], qo[b + 1] - qo[b], seq_len(b), kv[b]};
    const int64_t NR = scan_range(
        B, [&](int b) -> int64_t { return n_row(b); },
        [&](int b, int64_t ex) { c_row[b] = int(ex); }, wsum);
    const int64_t T = scan_range(
        B, [&](int b) -> int64_t { return int64_t(n_dec(b)) * cdiv(seq_len(b), kTileTokens); },
        [&](int b, int64_t ex) { p_tiles[b] = ex; }, wsum);
    // decode cut: ncta CTAs of `per` tiles (at least 8 tiles per CTA), as
    // build_cut_view
    int64_t per = 1, ncta = 0;
    if (T > 0) {
      ncta = T / 8 < 1 ? 1 : T / 8;
      if (ncta > a.dec_grid_cap) ncta = a.dec_grid_cap;
      per = cdiv(T, ncta);
      ncta = cdiv(T, per);
    }
    // CTA blocks of `per` tiles that the range [U0, U0 + tiles) touches
    auto pieces = [&](int64_t U0, int64_t tiles) -> int64_t {
      return (U0 + tiles - 1) / per - U0 / per + 1;
    };
    const int64_t NI = scan_range(
        B,
        [&](int b) -> int64_t {
          const int64_t tiles = cdiv(seq_len(b), kTileTokens);
          int64_t s = 0;
          for (int g = 0; g < n_dec(b); ++g) s += pieces(p_tiles[b] + g * tiles, tiles);
          return s;
        },
        [&](int b, int64_t ex) { c_item[b] = int(ex); }, wsum);
    const int64_t NG = scan_range(
        B,
        [&](int b) -> int64_t {
          const int64_t tiles = cdiv(seq_len(b), kTileTokens);
          int64_t s = 0;
          for (int g = 0; g < n_dec(b); ++g) s += pieces(p_tiles[b] + g * tiles, tiles) > 1;
          return s;
        },
        [&](int b, int64_t ex) { c_grp[b] = int(ex); }, wsum);
    const int64_t PF = scan_range(
        B,
        [&](int b) -> int64_t {
          const int64_t tiles = cdiv(seq_len(b), kTileTokens);
          const int rec = partial_rec_floats(H * (qo[b + 1] - qo[b]) * G, a.dim);
          int64_t s = 0;
          for (int g = 0; g < n_dec(b); ++g) {
            const int64_t pc = pieces(p_tiles[b] + g * tiles, tiles);
            if (pc > 1) s += rec * pc;
          }
          return s;
        },
        [&](int b, int64_t ex) { p_part[b] = ex; }, wsum);
    if (tid == 0) {
      if (NI > a.max_items || NR > a.max_items || NR > kMaxRowUnits || NG > a.max_groups ||
          PF > a.partial_capacity || PF > int64_t(INT32_MAX))
        bad = 1;
      // layout: header | seqs | pages | per list: cta_off, items, groups
      const int grid_row = NR > 0 ? a.grid_cap : 0;
      const int grid_dec = T > 0 ? a.dec_grid_cap : 0;
      int64_t off = align16_dev(pages_off + 4 * int64_t(total_pages));
      for (int c = 0; c < 3; ++c) {
        const int grid = c < 2 ? grid_row : grid_dec;
        const int64_t n = c < 2 ? NR : NI;
        sh[c] = off;  // cta_off
        off = align16_dev(off + 4 * int64_t(grid > 0 ? grid + 1 : 0));
        sh[3 + c] = off;  // items
        off += int64_t(sizeof(WorkItem)) * n;
        sh[6 + c] = off;  // groups
        off += c == 2 ? int64_t(sizeof(SplitGroup)) * NG : 0;
      }
      sh[9] = off;
      if (off > a.meta_cap || off > int64_t(INT32_MAX)) bad = 1;
    }
    if (__syncthreads_or(bad)) goto fail;

    // ---- decode list: the exact cut ---------------------------------------
    {
      int32_t* cta = reinterpret_cast<int32_t*>(a.meta + sh[2]);
      WorkItem* items = reinterpret_cast<WorkItem*>(a.meta + sh[5]);
      SplitGroup* groups = reinterpret_cast<SplitGroup*>(a.meta + sh[8]);
      for (int b = tid; b < B; b += kPlanThreads) {
        const int nd = n_dec(b);
        if (nd == 0) continue;
        const int P = (qo[b + 1] - qo[b]) * G;
        const int64_t tiles = cdiv(seq_len(b), kTileTokens);
        const int rec = partial_rec_floats(H * P, a.dim);
        int idx = c_item[b], gid = c_grp[b];
        int64_t part = p_part[b];
        for (int g = 0; g < nd; ++g) {
          const int64_t U0 = p_tiles[b] + g * tiles;
          const int64_t pc = pieces(U0, tiles);
          const int64_t c0 = U0 / per;
          const bool split = pc > 1;
          for (int64_t s = 0; s < pc; ++s) {
            const int64_t c = c0 + s;
            const int64_t lo = max(U0, c * per), hi = min(U0 + tiles, (c + 1) * per);
            WorkItem it;
            it.seq = b;
            it.kvh = static_cast<int16_t>(g * H);
            it.key_mode = 1;
            it.rb0 = 0;
            it.nrb = 1;
            it.kt0 = static_cast<int32_t>(lo - U0);
            it.kt1 = static_cast<int32_t>(hi - U0);
            it.part = split ? static_cast<int32_t>(part + s * rec) : -1;
            it.group = split ? gid : -1;
            items[idx] = it;
            if (lo == c * per) cta[c] = idx;  // the first item of CTA c
            ++idx;
          }
          if (split) {
            groups[gid] = SplitGroup{static_cast<int32_t>(pc), static_cast<int32_t>(part), rec,
                                     H * P, b, g * H, 0, 0};
            ++gid;
            part += rec * pc;
          }
        }
      }
      // graph mode launches every CTA: the ones past the cut get empty lists
      if (T > 0)
        for (int c = int(ncta) + tid; c <= a.dec_grid_cap; c += kPlanThreads) cta[c] = int(NI);
      for (int i = tid; i < NG; i += kPlanThreads) a.counters[i] = 0;
    }

    // ---- row lists: sort by cost, snake deal -------------------------------
    if (NR > 0) {
      const int grid = a.grid_cap;
      auto unit_of = [&](int u, int& b, int& h, int& rb0, int& nrb, int& tiles_full,
                         int& tiles_causal) {
        // the last b with c_row[b] <= u (sequences without row units share
        // their successor's offset)
        int lo = 0, hi = B;
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (c_row[mid] <= u) lo = mid; else hi = mid;
        }
        b = lo;
        const int k = u - c_row[b];
        const int qrows = qo[b + 1] - qo[b], P = qrows * G, RB = seq_rb(b), len = seq_len(b);
        h = k % a.hkv;
        rb0 = (k / a.hkv) * 8;
        nrb = min(8, RB - rb0);
        const int last_row = min(P, (rb0 + nrb) * kRowBlock) - 1;
        const int64_t limit = int64_t(len) - qrows + last_row / G + 1;  // bottom-right causal
        tiles_full = int(cdiv(len, kTileTokens));
        tiles_causal = int(cdiv(limit, kTileTokens));
      };
      for (int v = 0; v < 2; ++v) {
        // key: cost descending, then unit index (the host planner's stable order)
        for (int u = tid; u < NR; u += kPlanThreads) {
          int b, h, rb0, nrb, tf, tc;
          unit_of(u, b, h, rb0, nrb, tf, tc);
          const int64_t cost = int64_t(v == 0 ? tf : tc) * nrb + 4;
          sort_keys[u] = (uint64_t(0x7fffffff - cost) << 32) | uint32_t(u);
        }
        bitonic_sort(sort_keys, int(NR));
        WorkItem* items = reinterpret_cast<WorkItem*>(a.meta + sh[3 + v]);
        for (int r = tid; r < NR; r += kPlanThreads) {
          const int u = int(sort_keys[r] & 0xffffffffu);
          int b, h, rb0, nrb, tf, tc;
          unit_of(u, b, h, rb0, nrb, tf, tc);
          WorkItem it;
          it.seq = b;
          it.kvh = static_cast<int16_t>(h);
          it.key_mode = 0;
          it.rb0 = rb0;
          it.nrb = nrb;
          it.kt0 = 0;
          it.kt1 = v == 0 ? tf : tc;
          it.part = -1;
          it.group = -1;
          const int q = r / grid, m = r % grid;
          const int c = (q & 1) ? grid - 1 - m : m;
          items[snake_off(c, int(NR), grid) + q] = it;
        }
        int32_t* cta = reinterpret_cast<int32_t*>(a.meta + sh[v]);
        for (int c = tid; c <= grid; c += kPlanThreads) cta[c] = snake_off(c, int(NR), grid);
        __syncthreads();  // the keys are rewritten for the next list
      }
    }

    // ---- header ------------------------------------------------------------
    __syncthreads();
    if (tid == 0) {
      MetaHeader h{};
      const int grid_row = NR > 0 ? a.grid_cap : 0;
      for (int c = 0; c < 3; ++c) {
        h.n_items[c] = static_cast<int32_t>(c < 2 ? NR : NI);
        h.n_groups[c] = static_cast<int32_t>(c < 2 ? 0 : NG);
        h.grid[c] = c < 2 ? grid_row : (T > 0 ? a.dec_grid_cap : 0);
        h.cta_off_off[c] = static_cast<int32_t>(sh[c]);
        h.items_off[c] = static_cast<int32_t>(sh[3 + c]);
        h.groups_off[c] = static_cast<int32_t>(sh[6 + c]);
      }
      h.batch = B;
      h.rows = a.rows;
      h.seqs_off = static_cast<int32_t>(seqs_off);
      h.pages_off = static_cast<int32_t>(pages_off);
      h.total_bytes = static_cast<int32_t>(sh[9]);
      h.chunk_tiles = T > 0 ? static_cast<int32_t>(per) : (1 << 29);
      h.dec_heads = H;
      *hdr = h;
    }
    // the lists are complete before this grid ends, for kernels that a
    // programmatic launch lets start as soon as it has
    __threadfence();
    return;
  }

fail:
  if (tid == 0) {
    MetaHeader h{};  // no items, no CTAs: the attention kernels return at once
    h.batch = B;
    h.rows = a.rows;
    h.seqs_off = static_cast<int32_t>(sizeof(MetaHeader));
    h.pages_off = static_cast<int32_t>(sizeof(MetaHeader));
    h.total_bytes = static_cast<int32_t>(sizeof(MetaHeader));
    *hdr = h;
    raise_device_error(a.err, FE_DEVERR_PLAN);
  }
  __threadfence();
}

}  // namespace

size_t plan_device_scratch_bytes(int max_batch) {
  const size_t nb = size_t(max_batch) + 1;
  return 8 * 2 * nb + 4 * 3 * nb + 4 * 3 * nb + 6 * 16;
}

void plan_device_bind_scratch(DevPlanArgs& a, void* base) {
  const size_t nb = size_t(a.max_batch) + 1;
  uint8_t* p = static_cast<uint8_t*>(base);
  auto take = [&](size_t bytes) {
    uint8_t* q = p;
    p += (bytes + 15) & ~size_t(15);
    return q;
  };
  a.s_pref = reinterpret_cast<int64_t*>(take(8 * 2 * nb));
  a.s_qo = reinterpret_cast<int32_t*>(take(4 * nb));
  a.s_kv = reinterpret_cast<int32_t*>(take(4 * nb));
  a.s_last = reinterpret_cast<int32_t*>(take(4 * nb));
  a.s_cnt = reinterpret_cast<int32_t*>(take(4 * 3 * nb));
}

int plan_device_launch(const DevPlanArgs& a, cudaStream_t stream) {
  // A plain launch (no programmatic serialization): the planner starts only
  // after every earlier kernel of the stream has completed, since the
  // previous step's attention still reads the lists it rewrites.
  static const cudaError_t attr = cudaFuncSetAttribute(
      plan_device_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
      int(sizeof(uint64_t) * kMaxRowUnits));
  FE_CUDA_TRY(attr);
  plan_device_kernel<<<1, kPlanThreads, sizeof(uint64_t) * kMaxRowUnits, stream>>>(a);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

}  // namespace fe
