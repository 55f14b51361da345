// Host-side work planner for the paged-attention kernel, and the device
// metadata layout it produces. Pure C++ (no CUDA calls), so the planner runs
// and is tested without a GPU.
//
// Replaces the role of FlashInfer's PrefillPlan in the reference
// (src/flashinfer_attention.cu:29-34), with two differences: work over long
// contexts is split across CTAs (split-K; the reference disables split-KV,
// :31) and the per-CTA work lists are balanced on the host (longest item
// first onto the least-loaded CTA), so the kernel needs no atomics to fetch
// work and a captured CUDA graph stays valid for any later layout.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace fe {

constexpr int kHeadDim = 128;
constexpr int kWideHeadDim = 256;  // the hybrid / DFlash models' full-attention head dim
constexpr int kWideMinChunk = 16;  // fewest key tiles in a split piece of a head_dim 256 row item
constexpr int kTileTokens = 16;   // key tokens per tile (one TMA box per K/V half)
constexpr int kRowBlock = 16;     // packed query rows per mma row block

struct SeqInfo {  // 16 bytes
  int32_t q_row0;    // first query row (qo[b])
  int32_t qrows;     // query rows
  int32_t length;    // keys
  int32_t page_off;  // kv[b]: first entry of this sequence in pages[]
};

// One CTA-sized unit of work: packed query rows [rb0*16, (rb0+nrb)*16) of
// sequence `seq` against KV head `kvh`, keys in tiles [kt0, kt1).
//   key_mode = 1: a single row block; the consumer warps split the key tiles
//                 (decode and short verify) and their results are merged in
//                 shared memory.
//   key_mode = 0: up to eight row blocks (one 128-row tcgen05 tile), each
//                 over all key tiles of the item (prefill / long verify);
//                 for head_dim 256 the key range may be split across CTAs
//                 (a piece of [kt0, kt1) writes a partial record).
// A packed row p is query row p / G of the sequence, query head kvh*G + p % G.
struct WorkItem {  // 32 bytes
  int32_t seq;
  int16_t kvh;
  int16_t key_mode;
  int32_t rb0;
  int32_t nrb;
  int32_t kt0, kt1;
  int32_t part;   // float offset of this item's partial record, -1 if unsplit
  int32_t group;  // split group id, -1 if unsplit
};

struct SplitGroup {  // 32 bytes
  int32_t nsplit;      // 0 for the placeholder entries that keep row and decode ids apart
  int32_t part0;       // float offset of split 0's record; split s at part0 + s*rec_floats
  int32_t rec_floats;  // rows*(dim+2) rounded up to a multiple of 4
  int32_t rows;        // valid packed rows in each record
  int32_t seq, kvh;    // the unit's sequence and first KV head (where merged rows go)
  // record row r is packed row row0 + r % rph of KV head kvh + r / rph, with
  // rph = rows_per_head, or the sequence's packed rows (qrows x G) when 0
  int32_t row0, rows_per_head;
};

// Byte offsets are from the start of the metadata buffer. Index [c] of the
// per-list arrays selects a work list: 0 = row-mode work for the non-causal
// mask, 1 = row-mode work for the causal mask (the key range of a row block
// depends on the mask), 2 = decode work (key mode, mask-independent ranges;
// served by the decode kernel with H heads per item).
struct MetaHeader {  // 128 bytes
  int32_t n_items[3], n_groups[3], grid[3], cta_off_off[3], items_off[3], groups_off[3];
  int32_t batch, rows, seqs_off, pages_off, total_bytes, chunk_tiles, dec_heads;
  int32_t pad[7];
};
static_assert(sizeof(MetaHeader) == 128, "MetaHeader layout");

struct PlanConfig {
  int hq, hkv, dim, page, max_batch, max_pages, num_blocks;
  int grid_cap;               // persistent CTAs of the row kernel (SMs x CTAs per SM)
  int dec_grid_cap;           // persistent CTAs of the decode kernel (one per SM)
  int dec_heads;              // KV heads per decode item: gcd(hkv, 8)
  int row_group_blocks;       // 16-row blocks per row-mode item (8 = one 128-row tcgen05 tile)
  bool row_split;             // row-mode key ranges may be split across CTAs
  int max_items;              // work-item capacity
  int64_t partial_capacity;   // floats in the split-K workspace
  int max_groups;             // split-counter capacity
  // Mixed steps (decode rows and multi-row sequences) outside graph mode
  // run the two kernels side by side on disjoint SMs when the cost model
  // below predicts a gain: the decode list takes dec_fixed_us plus its bytes
  // at dec_sm_gbs per decode SM, at most hbm_gbs in all; the row list takes
  // row_piece_us per 16-key piece of a 128-row item on one SM.
  bool concurrent;
  float dec_sm_gbs, hbm_gbs, dec_fixed_us, row_piece_us;
};

struct PlanResult {
  std::vector<uint8_t> meta;  // packed device metadata (header first)
  int n_items = 0, n_groups = 0, decode_items = 0, prefill_items = 0, split_units = 0;
  int chunk_tiles = 0;
  int grid[3] = {0, 0, 0};    // CTAs per work list (0 = nothing to launch)
  int split_rows[3] = {0, 0, 0};  // most rows in one split unit's records, per list
  int64_t kv_tokens = 0, partial_floats = 0;
  bool concurrent = false;  // decode and row kernels run side by side (grids sum to the SMs)
};

// The SM split of a mixed step: CTAs of the decode kernel when both kernels
// should run side by side, 0 to run them one after the other at full width.
// `sms` persistent decode CTAs fit the GPU; dec_bytes are the decode list's
// K/V bytes, row_pieces the row list's 16-key pieces (summed over items),
// max_row_pieces those of its longest item (never split across CTAs).
int concurrent_decode_ctas(const PlanConfig& cfg, int sms, double dec_bytes, double row_pieces,
                           double max_row_pieces);

// Validates the step metadata (same checks as the reference plus range
// checks on page ids) and builds the work list. Returns an fe_status; on
// failure `err` holds the reason.
int build_plan(const PlanConfig& cfg, const int32_t* qo, const int32_t* kv, const int32_t* pages,
               const int32_t* last, int batch, int rows, bool fixed_grid, PlanResult& out,
               std::string& err);

#ifdef __CUDACC__
#define FE_HOST_DEVICE __host__ __device__
#else
#define FE_HOST_DEVICE
#endif

// Floats of one split record of `rows` rows: O[rows][dim], m[rows], l[rows],
// padded to a multiple of 4 (16-byte aligned records).
FE_HOST_DEVICE inline int partial_rec_floats(int rows, int dim = kHeadDim) {
  return ((rows * (dim + 2)) + 3) & ~3;
}

}  // namespace fe
