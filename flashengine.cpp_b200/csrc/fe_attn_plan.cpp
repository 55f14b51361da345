// Host work planner for the paged-attention kernel (see fe_attn_plan.h).
#include "fe_attn_plan.h"

#include <algorithm>
#include <cstring>
#include <functional>
#include <queue>
#include <utility>

#include "fe_kv.h"

namespace fe {
namespace {

struct Unit {
  int seq, kvh, key_mode, rb0, nrb, tiles, rows;
};

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

inline size_t align16(size_t n) { return (n + 15) & ~size_t(15); }

struct View {
  std::vector<int32_t> cta_off;
  std::vector<WorkItem> items;
  std::vector<SplitGroup> groups;
  int grid = 0, chunk = 0, decode_items = 0, prefill_items = 0, split_units = 0;
  int64_t partial_floats = 0;
};

// Split every unit's key range into balanced chunks and assign the items to
// CTAs, longest first onto the least-loaded CTA.
int build_view(const PlanConfig& cfg, const std::vector<Unit>& units, int grid_cap_in,
               int items_per_cta, int min_chunk, bool fixed_grid, View& v, std::string& err) {
  int64_t total_tiles = 0;
  for (const auto& u : units) total_tiles += u.tiles;
  const int grid_cap = std::max(1, grid_cap_in);
  int chunk = std::max<int>(min_chunk, ceil_div(total_tiles, int64_t(grid_cap) * items_per_cta));
  for (int attempt = 0; attempt < 32; ++attempt) {
    v.items.clear();
    v.groups.clear();
    v.decode_items = v.prefill_items = v.split_units = 0;
    v.partial_floats = 0;
    bool over = false;
    for (const auto& u : units) {
      const int nsplit = std::max(1, ceil_div(u.tiles, chunk));
      const int base = u.tiles / nsplit, extra = u.tiles % nsplit;
      int group = -1, part0 = -1;
      const int rec = partial_rec_floats(u.rows, cfg.dim);
      if (nsplit > 1) {
        group = static_cast<int>(v.groups.size());
        part0 = static_cast<int>(v.partial_floats);
        // key-mode records hold all of the sequence's rows; row-mode ones
        // hold the unit's rows of one KV head from packed row rb0*16
        const bool rows_rec = u.key_mode != 1;
        v.groups.push_back(SplitGroup{nsplit, part0, rec, u.rows, u.seq, u.kvh,
                                      rows_rec ? u.rb0 * kRowBlock : 0, rows_rec ? u.rows : 0});
        v.partial_floats += int64_t(rec) * nsplit;
        ++v.split_units;
      }
      int kt = 0;
      for (int s = 0; s < nsplit; ++s) {
        const int n = base + (s < extra ? 1 : 0);
        WorkItem it;
        it.seq = u.seq;
        it.kvh = static_cast<int16_t>(u.kvh);
        it.key_mode = static_cast<int16_t>(u.key_mode);
        it.rb0 = u.rb0;
        it.nrb = u.nrb;
        it.kt0 = kt;
        it.kt1 = kt + n;
        it.part = nsplit > 1 ? part0 + s * rec : -1;
        it.group = group;
        kt += n;
        v.items.push_back(it);
        (u.key_mode == 1 ? v.decode_items : v.prefill_items)++;
      }
    }
    if (static_cast<int>(v.items.size()) > cfg.max_items || v.partial_floats > cfg.partial_capacity ||
        static_cast<int>(v.groups.size()) > cfg.max_groups ||
        v.partial_floats > int64_t(INT32_MAX)) {
      over = true;
    }
    if (!over) break;
    if (attempt == 31) {
      err = "attention work exceeds the plan's item / split-workspace capacity";
      return FE_ERR_CAPACITY;
    }
    chunk *= 2;
  }
  v.chunk = chunk;

  const int n = static_cast<int>(v.items.size());
  v.grid = n == 0 ? 0 : (fixed_grid ? grid_cap : std::min(grid_cap, n));
  // Cost model: key tiles times row blocks computed, plus a fixed per-item
  // overhead (Q load, epilogue) worth a few tiles.
  std::vector<std::pair<int64_t, int>> order(n);
  for (int i = 0; i < n; ++i) {
    const auto& it = v.items[i];
    const int64_t tiles = it.kt1 - it.kt0;
    const int64_t cost = (it.key_mode == 1 ? tiles : tiles * it.nrb) + 4;
    order[i] = {cost, i};
  }
  std::stable_sort(order.begin(), order.end(),
                   [](const auto& a, const auto& b) { return a.first > b.first; });
  std::vector<std::vector<int>> per_cta(std::max(1, v.grid));
  using Load = std::pair<int64_t, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < v.grid; ++c) heap.push({0, c});
  for (const auto& [cost, idx] : order) {
    auto [load, c] = heap.top();
    heap.pop();
    per_cta[c].push_back(idx);
    heap.push({load + cost, c});
  }
  std::vector<WorkItem> sorted;
  sorted.reserve(n);
  v.cta_off.assign(v.grid + 1, 0);
  for (int c = 0; c < v.grid; ++c) {
    v.cta_off[c] = static_cast<int32_t>(sorted.size());
    for (int idx : per_cta[c]) sorted.push_back(v.items[idx]);
  }
  v.cta_off[v.grid] = static_cast<int32_t>(sorted.size());
  v.items.swap(sorted);
  return FE_OK;
}

// Decode lists (and head_dim 256 row lists) cost in proportion to key
// tiles, so they are balanced exactly: the units' tile ranges are laid end to
// end and cut into `grid` equal contiguous pieces, one per CTA. A unit cut
// into several pieces becomes a split unit (its pieces write partial records,
// merged by a separate kernel). Every CTA streams the same number of tiles, to
// within one.
int build_cut_view(const PlanConfig& cfg, const std::vector<Unit>& units, int grid_cap_in,
                   int min_tiles_per_cta, bool fixed_grid, View& v, std::string& err) {
  v = View{};
  int64_t total = 0;
  for (const auto& u : units) total += u.tiles;
  if (total == 0) {
    v.grid = 0;
    return FE_OK;
  }
  const int grid_cap = std::max(1, grid_cap_in);
  int n = static_cast<int>(std::min<int64_t>(grid_cap, std::max<int64_t>(1, total / min_tiles_per_cta)));
  const int64_t per = (total + n - 1) / n;
  n = static_cast<int>((total + per - 1) / per);
  // pass 1: pieces per unit
  std::vector<int> pieces(units.size(), 0);
  {
    int64_t room = per;
    for (size_t i = 0; i < units.size(); ++i) {
      int64_t left = units[i].tiles;
      while (left > 0) {
        const int64_t take = std::min(left, room);
        ++pieces[i];
        left -= take;
        room -= take;
        if (room == 0) room = per;
      }
    }
  }
  // pass 2: emit items CTA by CTA
  std::vector<int> group_of(units.size(), -1), part0_of(units.size(), -1), next_split(units.size(), 0);
  for (size_t i = 0; i < units.size(); ++i) {
    if (pieces[i] > 1) {
      const Unit& u = units[i];
      const int rec = partial_rec_floats(u.rows, cfg.dim);
      group_of[i] = static_cast<int>(v.groups.size());
      part0_of[i] = static_cast<int>(v.partial_floats);
      // key-mode records hold all of the sequence's rows; row-mode ones the
      // unit's rows of one KV head from packed row rb0*16
      const bool rows_rec = u.key_mode != 1;
      v.groups.push_back(SplitGroup{pieces[i], part0_of[i], rec, u.rows, u.seq, u.kvh,
                                    rows_rec ? u.rb0 * kRowBlock : 0, rows_rec ? u.rows : 0});
      v.partial_floats += int64_t(rec) * pieces[i];
      ++v.split_units;
    }
  }
  v.cta_off.clear();
  int64_t room = per;
  int cta = 0;
  v.cta_off.push_back(0);
  for (size_t i = 0; i < units.size(); ++i) {
    const Unit& u = units[i];
    int kt = 0;
    while (kt < u.tiles) {
      const int take = static_cast<int>(std::min<int64_t>(u.tiles - kt, room));
      WorkItem it;
      it.seq = u.seq;
      it.kvh = static_cast<int16_t>(u.kvh);
      it.key_mode = static_cast<int16_t>(u.key_mode);
      it.rb0 = u.rb0;
      it.nrb = u.nrb;
      it.kt0 = kt;
      it.kt1 = kt + take;
      const int s = next_split[i]++;
      it.group = group_of[i];
      it.part = group_of[i] >= 0 ? part0_of[i] + s * partial_rec_floats(u.rows, cfg.dim) : -1;
      v.items.push_back(it);
      (u.key_mode ? v.decode_items : v.prefill_items)++;
      kt += take;
      room -= take;
      if (room == 0) {
        room = per;
        ++cta;
        v.cta_off.push_back(static_cast<int32_t>(v.items.size()));
      }
    }
  }
  if (static_cast<int>(v.cta_off.size()) == cta + 1 && v.cta_off.back() != static_cast<int32_t>(v.items.size())) {
    ++cta;
    v.cta_off.push_back(static_cast<int32_t>(v.items.size()));
  }
  v.grid = static_cast<int>(v.cta_off.size()) - 1;
  v.chunk = static_cast<int>(per);
  if (static_cast<int>(v.items.size()) > cfg.max_items || v.partial_floats > cfg.partial_capacity ||
      static_cast<int>(v.groups.size()) > cfg.max_groups) {
    err = "attention work exceeds the plan's item / split-workspace capacity";
    return FE_ERR_CAPACITY;
  }
  if (fixed_grid && v.grid < grid_cap) {
    // graph mode launches grid_cap CTAs; the extra ones get empty lists
    while (static_cast<int>(v.cta_off.size()) < grid_cap + 1)
      v.cta_off.push_back(static_cast<int32_t>(v.items.size()));
    v.grid = grid_cap;
  }
  return FE_OK;
}

}  // namespace

int concurrent_decode_ctas(const PlanConfig& cfg, int sms, double dec_bytes, double row_pieces,
                           double max_row_pieces) {
  if (!cfg.concurrent || sms < 2 || dec_bytes <= 0 || row_pieces <= 0) return 0;
  const double b_sm = double(cfg.dec_sm_gbs) * 1e3;  // bytes per microsecond
  const double b_hbm = double(cfg.hbm_gbs) * 1e3;
  const double c = cfg.row_piece_us;
  auto t_dec = [&](int d) { return dec_bytes / std::min(d * b_sm, b_hbm) + cfg.dec_fixed_us; };
  auto t_row = [&](int r) { return std::max(row_pieces * c / r, max_row_pieces * c); };
  // one after the other: both at full width, plus the second kernel's ramp
  const double serial = t_dec(sms) + t_row(sms) + 4.0;
  int best = 0;
  double best_t = serial;
  for (int d = 1; d < sms; ++d) {
    const double t = std::max(t_dec(d), t_row(sms - d));
    if (t < best_t) {
      best_t = t;
      best = d;
    }
  }
  // side by side only when it is clearly faster (the model is coarse)
  return best_t < 0.92 * serial ? best : 0;
}

int build_plan(const PlanConfig& cfg, const int32_t* qo, const int32_t* kv, const int32_t* pages,
               const int32_t* last, int batch, int rows, bool fixed_grid, PlanResult& out,
               std::string& err) {
  out = PlanResult{};
  if (batch < 0 || rows < 0) {
    err = "batch and rows must be non-negative";
    return FE_ERR_INVALID_ARGUMENT;
  }
  if (batch > 0 && (!qo || !kv || !last)) {
    err = "qo, kv and last must be non-null";
    return FE_ERR_INVALID_ARGUMENT;
  }
  // Capacity check of the reference's CUDA plan (src/flashinfer_attention.cu:30).
  if (batch > cfg.max_batch || (batch > 0 && int64_t(kv[batch]) > int64_t(cfg.max_batch) * cfg.max_pages)) {
    err = "attention metadata exceeds plan capacity";
    return FE_ERR_CAPACITY;
  }
  if (batch > 0 && (qo[0] != 0 || kv[0] != 0)) {
    err = "qo[0] and kv[0] must be 0";
    return FE_ERR_INVALID_ARGUMENT;
  }
  if ((batch == 0 && rows != 0) || (batch > 0 && qo[batch] != rows)) {
    err = "qo[batch] must equal rows";
    return FE_ERR_INVALID_ARGUMENT;
  }
  const int G = cfg.hq / cfg.hkv;
  const int total_pages = batch > 0 ? kv[batch] : 0;
  if (total_pages > 0 && !pages) {
    err = "pages must be non-null";
    return FE_ERR_INVALID_ARGUMENT;
  }
  std::vector<SeqInfo> seqs(batch);
  std::vector<Unit> key_units, row_units_causal, row_units_full;
  int64_t kv_tokens = 0;
  for (int b = 0; b < batch; ++b) {
    const int q0 = qo[b], q1 = qo[b + 1];
    const int p0 = kv[b], p1 = kv[b + 1];
    if (q1 < q0 || p1 <= p0) {
      err = "qo must be non-decreasing and every sequence must own at least one page (b=" +
            std::to_string(b) + ")";
      return FE_ERR_INVALID_ARGUMENT;
    }
    if (last[b] < 1 || last[b] > cfg.page) {
      err = "last[b] must be in [1, page] (b=" + std::to_string(b) + ")";
      return FE_ERR_INVALID_ARGUMENT;
    }
    if (p1 - p0 > cfg.max_pages) {
      err = "sequence uses more pages than max_pages (b=" + std::to_string(b) + ")";
      return FE_ERR_CAPACITY;
    }
    const int64_t length = int64_t(p1 - p0 - 1) * cfg.page + last[b];
    const int qrows = q1 - q0;
    // Context check of the reference ATen path (src/portable_gpu_ops.cpp:30).
    if (length < qrows) {
      err = "sequence has fewer keys than query rows (b=" + std::to_string(b) + ")";
      return FE_ERR_CONTEXT;
    }
    for (int i = p0; i < p1; ++i)
      if (pages[i] < 0 || pages[i] > cfg.num_blocks) {
        err = "page id out of range [0, num_blocks] at pages[" + std::to_string(i) + "]";
        return FE_ERR_INVALID_ARGUMENT;
      }
    seqs[b] = SeqInfo{q0, qrows, static_cast<int32_t>(length), p0};
    kv_tokens += length;
    if (qrows == 0) continue;
    const int P = qrows * G;
    const int RB = ceil_div(P, kRowBlock);
    const int tiles_full = ceil_div(length, kTileTokens);
    if (RB == 1) {
      const int H = cfg.dec_heads;
      for (int h = 0; h < cfg.hkv; h += H)
        key_units.push_back(Unit{b, h, 1, 0, 1, tiles_full, H * P});
    } else {
      const int grp = cfg.row_group_blocks;
      for (int rb0 = 0; rb0 < RB; rb0 += grp) {
        const int nrb = std::min(grp, RB - rb0);
        const int last_row = std::min(P, (rb0 + nrb) * kRowBlock) - 1;
        const int rows_valid = last_row + 1 - rb0 * kRowBlock;
        const int64_t i_max = last_row / G;
        const int64_t limit = length - qrows + i_max + 1;  // bottom-right causal
        const int tiles_causal = ceil_div(limit, kTileTokens);
        for (int h = 0; h < cfg.hkv; ++h) {
          row_units_full.push_back(Unit{b, h, 0, rb0, nrb, tiles_full, rows_valid});
          row_units_causal.push_back(Unit{b, h, 0, rb0, nrb, tiles_causal, rows_valid});
        }
      }
    }
  }

  // Mixed steps outside graph mode may run the two kernels side by side:
  // dec_ctas decode CTAs and the rest of the SMs for the row kernel.
  int row_cap = cfg.grid_cap, dec_cap = cfg.dec_grid_cap;
  if (!fixed_grid && !key_units.empty() && !row_units_causal.empty()) {
    double dec_bytes = 0, pieces = 0, max_pieces = 0;
    for (const auto& u : key_units)
      dec_bytes += double(u.tiles) * kTileTokens * cfg.dec_heads * cfg.dim * 4.0;
    for (const auto* list : {&row_units_full, &row_units_causal}) {
      double total = 0;
      for (const auto& u : *list) {
        total += u.tiles;
        max_pieces = std::max(max_pieces, double(u.tiles));
      }
      pieces = std::max(pieces, total);
    }
    const int sms = cfg.dec_grid_cap;
    const int d = concurrent_decode_ctas(cfg, sms, dec_bytes, pieces, max_pieces);
    if (d > 0) {
      dec_cap = d;
      row_cap = std::max(1, (sms - d) * std::max(1, cfg.grid_cap / sms));
      out.concurrent = true;
    }
  }
  // List 0: row work, non-causal; 1: row work, causal (identical key ranges
  // when there is no row work); 2: decode work.
  View views[3];
  {
    int rc;
    if (cfg.dim == kWideHeadDim) {
      // head_dim 256 row lists are cut exactly like the decode list: the
      // tcgen05 kernel's time per key tile hardly depends on how many of an
      // item's 128 rows are valid, so equal tile counts per CTA balance it,
      // at the price of up to one split unit per CTA boundary (pieces of at
      // least kWideMinChunk tiles per CTA)
      rc = build_cut_view(cfg, row_units_full, row_cap, kWideMinChunk, fixed_grid, views[0], err);
      if (rc != FE_OK) return rc;
      rc = build_cut_view(cfg, row_units_causal, row_cap, kWideMinChunk, fixed_grid, views[1],
                          err);
    } else {
      // head_dim 128 keeps whole items (cfg.row_split), longest first onto
      // the least-loaded CTA
      const int row_min_chunk = cfg.row_split ? 16 : (1 << 29);
      rc = build_view(cfg, row_units_full, row_cap, 4, row_min_chunk, fixed_grid, views[0], err);
      if (rc != FE_OK) return rc;
      rc = build_view(cfg, row_units_causal, row_cap, 4, row_min_chunk, fixed_grid, views[1], err);
    }
    if (rc != FE_OK) return rc;
    rc = build_cut_view(cfg, key_units, dec_cap, 8, fixed_grid, views[2], err);
    if (rc != FE_OK) return rc;
  }
  // Both kernels of one run share the split workspace and counters: offset
  // the decode list's records and groups past the larger row list's.
  const int64_t row_floats = std::max(views[0].partial_floats, views[1].partial_floats);
  const int row_groups = static_cast<int>(std::max(views[0].groups.size(), views[1].groups.size()));
  for (auto& it : views[2].items) {
    if (it.group >= 0) {
      it.group += row_groups;
      it.part += static_cast<int32_t>(row_floats);
    }
  }
  {
    std::vector<SplitGroup> shifted(row_groups);
    for (auto gi : views[2].groups) {
      gi.part0 += static_cast<int32_t>(row_floats);
      shifted.push_back(gi);
    }
    views[2].groups.swap(shifted);
  }
  if (row_floats + views[2].partial_floats > cfg.partial_capacity ||
      row_floats + views[2].partial_floats > int64_t(INT32_MAX) ||
      static_cast<int>(views[2].groups.size()) > cfg.max_groups) {
    err = "attention work exceeds the plan's split-workspace capacity";
    return FE_ERR_CAPACITY;
  }

  // Pack: header | per list: cta_off, items, groups | seqs | pages.
  size_t off = align16(sizeof(MetaHeader));
  size_t cta_off_off[3], items_off[3], groups_off[3];
  for (int c = 0; c < 3; ++c) {
    const View& v = views[c];
    cta_off_off[c] = off;
    off = align16(off + sizeof(int32_t) * v.cta_off.size());
    items_off[c] = off;
    off = align16(off + sizeof(WorkItem) * v.items.size());
    groups_off[c] = off;
    off = align16(off + sizeof(SplitGroup) * v.groups.size());
  }
  const size_t seqs_off = off;
  off = align16(off + sizeof(SeqInfo) * seqs.size());
  const size_t pages_off = off;
  off = align16(off + sizeof(int32_t) * total_pages);
  if (off > size_t(INT32_MAX)) {
    err = "metadata too large";
    return FE_ERR_CAPACITY;
  }
  out.meta.assign(off, 0);
  uint8_t* m = out.meta.data();
  for (int c = 0; c < 3; ++c) {
    const View& v = views[c];
    if (!v.cta_off.empty())
      std::memcpy(m + cta_off_off[c], v.cta_off.data(), sizeof(int32_t) * v.cta_off.size());
    if (!v.items.empty())
      std::memcpy(m + items_off[c], v.items.data(), sizeof(WorkItem) * v.items.size());
    if (!v.groups.empty())
      std::memcpy(m + groups_off[c], v.groups.data(), sizeof(SplitGroup) * v.groups.size());
  }
  if (!seqs.empty()) std::memcpy(m + seqs_off, seqs.data(), sizeof(SeqInfo) * seqs.size());
  if (total_pages) std::memcpy(m + pages_off, pages, sizeof(int32_t) * total_pages);

  MetaHeader h{};
  for (int c = 0; c < 3; ++c) {
    const View& v = views[c];
    h.n_items[c] = static_cast<int32_t>(v.items.size());
    h.n_groups[c] = static_cast<int32_t>(v.groups.size());
    h.grid[c] = v.grid;
    h.cta_off_off[c] = static_cast<int32_t>(cta_off_off[c]);
    h.items_off[c] = static_cast<int32_t>(items_off[c]);
    h.groups_off[c] = static_cast<int32_t>(groups_off[c]);
  }
  h.batch = batch;
  h.rows = rows;
  h.seqs_off = static_cast<int32_t>(seqs_off);
  h.pages_off = static_cast<int32_t>(pages_off);
  h.total_bytes = static_cast<int32_t>(off);
  h.chunk_tiles = views[2].items.empty() ? views[1].chunk : views[2].chunk;
  h.dec_heads = cfg.dec_heads;
  std::memcpy(m, &h, sizeof(h));

  out.n_items = static_cast<int>(views[1].items.size() + views[2].items.size());
  out.n_groups = static_cast<int>(views[2].groups.size());
  out.decode_items = static_cast<int>(views[2].items.size());
  out.prefill_items = static_cast<int>(views[1].items.size());
  out.split_units = views[1].split_units + views[2].split_units;
  out.chunk_tiles = h.chunk_tiles;
  for (int c = 0; c < 3; ++c) out.grid[c] = views[c].grid;
  out.kv_tokens = kv_tokens;
  out.partial_floats = row_floats + views[2].partial_floats;
  for (int c = 0; c < 3; ++c)
    for (const auto& gi : views[c].groups)
      if (gi.nsplit > 1) out.split_rows[c] = std::max(out.split_rows[c], gi.rows);
  return FE_OK;
}

}  // namespace fe
