// Paged GQA attention for sm_100a: the plan object, its host planner hand-off
// and the launch of the two kernels that serve one fe_attn_run call.
//
// Reference behaviour: Cambridgebit/FlashEngine.cpp src/flashinfer_attention.cu:22-44
// (create_plan / prepare_plan / attention over NHD pages, scale 1/sqrt(128),
// causal or no mask) with the arithmetic oracle src/portable_gpu_ops.cpp:27-44.
//
//  * fe_attn_plan_prepare: the host planner (fe_attn_plan.cpp) cuts every
//    (sequence, KV head, query-row group) into key-range work items and
//    balances them over the CTAs of each kernel; the metadata block is copied
//    from pinned memory into a fixed device buffer (graph-replayable).
//  * fe_attn_run: decode items (one query row per sequence) go to the
//    split-K decode kernel (fe_decode.cu); multi-row items (chunked prefill,
//    speculative verify) go to the tcgen05/TMEM kernel (fe_prefill_tc.cu).
//    Tensor maps of the K and V pools are encoded once per pool address.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "fe_attn_common.cuh"
#include "fe_plan_device.h"

namespace fe {

int decode_launch(int dtype, int dim, int heads, const CUtensorMap& kmap, const CUtensorMap& vmap,
                  bool per_head_tma, const void* args, int grid, cudaStream_t stream);
int decode_merge_launch(int dtype, int dim, int list, const void* args, int grid, int grid_rows,
                        cudaStream_t stream, bool pdl);
int prefill_tc_launch(int dtype, int dim, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const CUtensorMap& qmap, const void* args, int grid, cudaStream_t stream);

namespace {

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_nd(CUtensorMap* map, const void* pool, int dtype, int rank, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return fail(FE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map,
                  dtype == FE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  rank, const_cast<void*>(pool), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FE_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return FE_OK;
}

int encode_3d(CUtensorMap* map, const void* pool, int dtype, const cuuint64_t dims[3],
              const cuuint64_t strides[2], const cuuint32_t box[3]) {
  return encode_nd(map, pool, dtype, 3, dims, strides, box);
}

// tcgen05 row kernel: pool viewed as [cache_slots/8][hkv*dim/64][8][64]
// (slot groups of 8, 64-dim boxes, slots within the group, 64 elements);
// box = 2 groups x dim/64 boxes x 8 slots x 64 elements, so one TMA copies a
// 16-token piece of one KV head and lays it out as [group][box][8 rows of
// 128 B]: 1 KiB swizzle atoms, the boxes 1 KiB apart, 8-key groups dim*16 B
// apart.
int encode_tc_map(CUtensorMap* map, const void* pool, int dtype, int hkv, int dim,
                  int64_t cache_slots) {
  const cuuint64_t boxes = cuuint64_t(dim / 64);
  const cuuint64_t dims[4] = {64, 8, cuuint64_t(hkv) * boxes, cuuint64_t(cache_slots / 8)};
  const cuuint64_t strides[3] = {cuuint64_t(hkv) * dim * 2, 128, cuuint64_t(hkv) * dim * 2 * 8};
  const cuuint32_t box[4] = {64, 8, cuuint32_t(boxes), 2};
  return encode_nd(map, pool, dtype, 4, dims, strides, box);
}

// tcgen05 row kernel, queries: q [rows][hq][dim] with box (128/G rows) x
// (G heads) x 64 elements: one box is a 64-dim slice of a 128-row packed Q
// tile (packed row p = query row p / G, head p % G of the KV head's group),
// landing in packed-row order.
int encode_q_map(CUtensorMap* map, const void* q, int dtype, int hq, int dim, int rows, int G) {
  const cuuint64_t dims[3] = {cuuint64_t(dim), cuuint64_t(hq), cuuint64_t(rows)};
  const cuuint64_t strides[2] = {cuuint64_t(dim) * 2, cuuint64_t(hq) * dim * 2};
  const cuuint32_t box[3] = {64, cuuint32_t(G), cuuint32_t(128 / G)};
  return encode_nd(map, q, dtype, 3, dims, strides, box);
}

// Per-box fallback of the decode kernel: pool viewed as
// [cache_slots][hkv*dim/64][64] (64-element rows of 128 B: head-halves for
// head_dim 128); box = 16 slots x 1 row x 64 elements.
int encode_pool_map(CUtensorMap* map, const void* pool, int dtype, int hkv, int dim,
                    int64_t cache_slots) {
  const cuuint64_t dims[3] = {64, cuuint64_t(hkv) * (dim / 64), cuuint64_t(cache_slots)};
  const cuuint64_t strides[2] = {128, cuuint64_t(hkv) * dim * 2};
  const cuuint32_t box[3] = {64, 1, kTileTokens};
  return encode_3d(map, pool, dtype, dims, strides, box);
}

// Decode kernel: the same memory walked slots-first, [hkv*dim/64][cache_slots]
// [64]; box = H*dim/64 rows x 16 slots x 64 elements, so one TMA copies a
// 16-token tile of H heads (a contiguous 16 x H x 2*dim-byte block of the
// page) and lays it out 64 dims at a time, 16 swizzled rows each.
int encode_decode_map(CUtensorMap* map, const void* pool, int dtype, int hkv, int dim, int heads,
                      int64_t cache_slots) {
  const cuuint64_t dims[3] = {64, cuuint64_t(cache_slots), cuuint64_t(hkv) * (dim / 64)};
  const cuuint64_t strides[2] = {cuuint64_t(hkv) * dim * 2, 128};
  const cuuint32_t box[3] = {64, kTileTokens, cuuint32_t(heads * (dim / 64))};
  return encode_3d(map, pool, dtype, dims, strides, box);
}

}  // namespace
}  // namespace fe

using namespace fe;

struct fe_attn_plan {
  PlanConfig cfg{};
  int dtype = 0;
  bool host_only = false;
  int device = -1;
  // device workspaces
  uint8_t* d_meta = nullptr;
  size_t meta_cap = 0;
  float* d_partials = nullptr;
  int32_t* d_counters = nullptr;
  void* d_plan_scratch = nullptr;  // device-side planner (fe_plan_device.cu)
  // pinned staging, double-buffered
  uint8_t* h_meta[2] = {nullptr, nullptr};
  cudaEvent_t h_ev[2] = {nullptr, nullptr};
  bool h_used[2] = {false, false};
  int h_idx = 0;
  // last prepare
  bool prepared = false, fixed_grid = false;
  bool device_planned = false;  // the last prepare built the lists on the device
  bool graph_shape_set = false;
  int graph_batch = 0, graph_rows = 0;
  PlanResult last;
  int grid_view[3] = {0, 0, 0};
  // cached tensor maps (row kernel, decode kernel)
  CUtensorMap kmap, vmap, kmap_dec, vmap_dec, kmap_tc, vmap_tc;
  const void* kmap_ptr = nullptr;
  const void* vmap_ptr = nullptr;
  bool per_head_tma = false;  // decode falls back to per-head-half boxes
  // mixed steps run the row kernel on this stream beside the decode kernel
  // (fork and join through the two events, so a capture follows them too)
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
};

namespace {

size_t meta_capacity(const PlanConfig& c) {
  size_t per_view = sizeof(int32_t) * (std::max(c.grid_cap, c.dec_grid_cap) + 1) +
                    sizeof(WorkItem) * c.max_items + sizeof(SplitGroup) * c.max_groups + 64;
  return sizeof(MetaHeader) + 3 * per_view + sizeof(SeqInfo) * c.max_batch +
         sizeof(int32_t) * size_t(c.max_batch) * c.max_pages + 256;
}

int check_shape(int hq, int hkv, int dim, int page, int max_batch, int max_pages, int dtype,
                int num_blocks) {
  if (dtype != FE_DTYPE_F16 && dtype != FE_DTYPE_BF16)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: bad dtype");
  if (dim != kHeadDim && dim != kWideHeadDim)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: head_dim must be 128 or 256");
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0 || hq / hkv > kRowBlock)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: need hq % hkv == 0 and hq/hkv <= 16");
  if (hkv * 2 > 256 * 1024)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: hkv too large");
  if (page <= 0 || page % kTileTokens != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: page must be a multiple of 16");
  if (max_batch <= 0 || max_pages <= 0 || num_blocks <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: sizes must be positive");
  if (int64_t(num_blocks + 1) * page >= INT32_MAX)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: (num_blocks+1)*page overflows");
  if (int64_t(max_batch) * max_pages >= INT32_MAX / 4)
    return fail(FE_ERR_CAPACITY, "fe_attn_plan_create: max_batch*max_pages too large");
  return FE_OK;
}

int gcd8(int hkv) {
  int h = 8;
  while (hkv % h) h >>= 1;
  return h;
}

PlanConfig make_config(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                       int num_blocks, int grid_cap, int dec_grid_cap) {
  PlanConfig c{};
  c.hq = hq;
  c.hkv = hkv;
  c.dim = dim;
  c.page = page;
  c.max_batch = max_batch;
  c.max_pages = max_pages;
  c.num_blocks = num_blocks;
  c.grid_cap = grid_cap;
  c.dec_grid_cap = dec_grid_cap;
  // KV heads per decode item: one 16-token tile of them is one TMA box; for
  // head_dim 256 (8 KiB per head and tile) at most two
  c.dec_heads = dim == kWideHeadDim ? (hkv % 2 == 0 ? 2 : 1) : gcd8(hkv);
  c.row_group_blocks = 8;  // 128 packed rows per tcgen05 work item
  c.row_split = false;      // the tcgen05 kernel walks an item's whole key range
  int64_t items = int64_t(max_batch) * hkv * 64;
  if (items < 8192) items = 8192;
  if (items > (1 << 20)) items = 1 << 20;
  c.max_items = static_cast<int>(items);
  c.max_groups = c.max_items;
  c.partial_capacity = int64_t(16) << 20;  // 64 MiB of floats
  // side-by-side mixed steps, fitted to B200 timings of these kernels on a
  // C3 step: the decode kernel moves ~100 GB/s per SM on part of the GPU
  // (90 while the tcgen05 kernel runs beside it) after ~10 us of fill and
  // merge, and reaches ~5.8 TB/s at full width on mid-size launches; the
  // tcgen05 kernel takes ~0.2 us per 16-key piece of a 128-row item per SM
  // (twice that at head_dim 256)
  c.concurrent = true;
  c.dec_sm_gbs = 90.f;
  c.hbm_gbs = 5800.f;
  c.dec_fixed_us = 10.f;
  c.row_piece_us = dim == kWideHeadDim ? 0.4f : 0.2f;
  return c;
}

void destroy(fe_attn_plan* p) {
  if (!p) return;
  if (!p->host_only) {
    for (int i = 0; i < 2; ++i) {
      if (p->h_ev[i]) cudaEventSynchronize(p->h_ev[i]);
      if (p->h_ev[i]) cudaEventDestroy(p->h_ev[i]);
      if (p->h_meta[i]) cudaFreeHost(p->h_meta[i]);
    }
    if (p->d_meta) cudaFree(p->d_meta);
    if (p->d_partials) cudaFree(p->d_partials);
    if (p->d_counters) cudaFree(p->d_counters);
    if (p->d_plan_scratch) cudaFree(p->d_plan_scratch);
    if (p->side) {
      cudaStreamSynchronize(p->side);
      cudaStreamDestroy(p->side);
    }
    if (p->fork_ev) cudaEventDestroy(p->fork_ev);
    if (p->join_ev) cudaEventDestroy(p->join_ev);
  }
  delete p;
}

}  // namespace

extern "C" {

int fe_attn_plan_create(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                        int dtype, int num_blocks, fe_attn_plan** plan_out) {
  if (!plan_out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: plan_out is null");
  *plan_out = nullptr;
  int rc = check_shape(hq, hkv, dim, page, max_batch, max_pages, dtype, num_blocks);
  if (rc != FE_OK) return rc;
  int dev = 0;
  FE_CUDA_TRY(cudaGetDevice(&dev));
  int major = 0, sms = 0;
  FE_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  FE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  if (major != 10)
    return fail(FE_ERR_NO_DEVICE, "fe_attn_plan_create: needs an sm_100 (B200) device");
  auto* p = new (std::nothrow) fe_attn_plan();
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: out of host memory");
  p->cfg = make_config(hq, hkv, dim, page, max_batch, max_pages, num_blocks, sms, sms);
  p->dtype = dtype;
  p->device = dev;
  p->meta_cap = meta_capacity(p->cfg);
  cudaError_t e = cudaMalloc(&p->d_meta, p->meta_cap);
  if (e == cudaSuccess) e = cudaMalloc(&p->d_partials, sizeof(float) * p->cfg.partial_capacity);
  if (e == cudaSuccess) e = cudaMalloc(&p->d_counters, sizeof(int32_t) * p->cfg.max_groups);
  if (e == cudaSuccess) e = cudaMemset(p->d_counters, 0, sizeof(int32_t) * p->cfg.max_groups);
  if (e == cudaSuccess) e = cudaMemset(p->d_meta, 0, sizeof(MetaHeader));
  if (e == cudaSuccess) e = cudaMalloc(&p->d_plan_scratch, plan_device_scratch_bytes(max_batch));
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    e = cudaMallocHost(&p->h_meta[i], p->meta_cap);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->h_ev[i], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->fork_ev, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->join_ev, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    destroy(p);
    return cuda_fail(e, "fe_attn_plan_create: workspace allocation");
  }
  *plan_out = p;
  return FE_OK;
}

// Test hook: a plan with no device state, for exercising the planner on a
// host without a GPU. fe_attn_plan_prepare() then only builds the work list.
int fe_attn_plan_create_host(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                             int dtype, int num_blocks, int grid_cap, fe_attn_plan** plan_out) {
  if (!plan_out) return fail(FE_ERR_INVALID_ARGUMENT, "plan_out is null");
  *plan_out = nullptr;
  int rc = check_shape(hq, hkv, dim, page, max_batch, max_pages, dtype, num_blocks);
  if (rc != FE_OK) return rc;
  if (grid_cap <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "grid_cap must be positive");
  auto* p = new (std::nothrow) fe_attn_plan();
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "out of host memory");
  p->cfg = make_config(hq, hkv, dim, page, max_batch, max_pages, num_blocks, grid_cap,
                       std::max(1, grid_cap / 2));
  p->dtype = dtype;
  p->host_only = true;
  p->meta_cap = meta_capacity(p->cfg);
  *plan_out = p;
  return FE_OK;
}

int fe_attn_plan_destroy(fe_attn_plan* plan) {
  destroy(plan);
  return FE_OK;
}

int fe_attn_plan_prepare(fe_attn_plan* p, const int32_t* qo, const int32_t* kv,
                         const int32_t* pages, const int32_t* last, int batch, int rows, int graph,
                         void* stream) {
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_prepare: plan is null");
  if (graph && p->graph_shape_set && (p->graph_batch != batch || p->graph_rows != rows))
    return fail(FE_ERR_INVALID_ARGUMENT,
                "fe_attn_plan_prepare: graph plan batch/rows changed since capture");
  std::string err;
  PlanResult res;
  int rc = build_plan(p->cfg, qo, kv, pages, last, batch, rows, graph != 0, res, err);
  if (rc != FE_OK) return fail(rc, "fe_attn_plan_prepare: " + err);
  if (res.meta.size() > p->meta_cap)
    return fail(FE_ERR_CAPACITY, "fe_attn_plan_prepare: metadata exceeds workspace");
  if (!p->host_only) {
    auto s = static_cast<cudaStream_t>(stream);
    const int i = p->h_idx;
    if (p->h_used[i]) FE_CUDA_TRY(cudaEventSynchronize(p->h_ev[i]));
    std::memcpy(p->h_meta[i], res.meta.data(), res.meta.size());
    FE_CUDA_TRY(cudaMemcpyAsync(p->d_meta, p->h_meta[i], res.meta.size(), cudaMemcpyHostToDevice, s));
    FE_CUDA_TRY(cudaEventRecord(p->h_ev[i], s));
    p->h_used[i] = true;
    p->h_idx ^= 1;
    if (res.n_groups > 0)
      FE_CUDA_TRY(cudaMemsetAsync(p->d_counters, 0, sizeof(int32_t) * res.n_groups, s));
  }
  for (int c = 0; c < 3; ++c) p->grid_view[c] = res.grid[c];
  p->last = std::move(res);
  p->prepared = true;
  p->device_planned = false;
  p->fixed_grid = graph != 0;
  if (graph) {
    p->graph_shape_set = true;
    p->graph_batch = batch;
    p->graph_rows = rows;
  }
  return FE_OK;
}

}  // extern "C"

namespace {

// Shared tail of the two device-side prepares: launch the planner, then
// record on the host only what the launches need (graph-mode grids, the
// step's batch and rows; the item counts stay on the device).
int prepare_on_device(fe_attn_plan* p, DevPlanArgs& a, int batch, int rows, void* stream,
                      const char* what) {
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, std::string(what) + ": plan is null");
  if (p->host_only) return fail(FE_ERR_INVALID_ARGUMENT, std::string(what) + ": host-only plan");
  if (batch < 0 || rows < 0)
    return fail(FE_ERR_INVALID_ARGUMENT,
                std::string(what) + ": batch and rows must be non-negative");
  if (batch > p->cfg.max_batch)
    return fail(FE_ERR_CAPACITY, std::string(what) + ": batch exceeds the plan's max_batch");
  if (p->graph_shape_set && (p->graph_batch != batch || p->graph_rows != rows))
    return fail(FE_ERR_INVALID_ARGUMENT,
                std::string(what) + ": graph plan batch/rows changed since capture");
  const PlanConfig& c = p->cfg;
  a.batch = batch;
  a.rows = rows;
  a.hq = c.hq;
  a.hkv = c.hkv;
  a.dim = c.dim;
  a.page = c.page;
  a.max_batch = c.max_batch;
  a.max_pages = c.max_pages;
  a.num_blocks = c.num_blocks;
  a.dec_heads = c.dec_heads;
  a.grid_cap = c.grid_cap;
  a.dec_grid_cap = c.dec_grid_cap;
  a.max_items = c.max_items;
  a.max_groups = c.max_groups;
  a.partial_capacity = c.partial_capacity;
  a.meta_cap = static_cast<int64_t>(p->meta_cap);
  a.meta = p->d_meta;
  a.counters = p->d_counters;
  a.err = device_error_word();
  plan_device_bind_scratch(a, p->d_plan_scratch);
  int rc = plan_device_launch(a, static_cast<cudaStream_t>(stream));
  if (rc != FE_OK) return rc;
  PlanResult res;
  res.meta.assign(sizeof(MetaHeader), 0);
  MetaHeader h{};
  h.batch = batch;
  h.rows = rows;
  std::memcpy(res.meta.data(), &h, sizeof(h));
  res.n_items = res.decode_items = res.prefill_items = res.split_units = -1;
  res.chunk_tiles = -1;
  res.kv_tokens = -1;
  p->last = std::move(res);
  p->grid_view[0] = p->grid_view[1] = c.grid_cap;
  p->grid_view[2] = c.dec_grid_cap;
  p->prepared = true;
  p->device_planned = true;
  p->fixed_grid = true;
  p->graph_shape_set = true;
  p->graph_batch = batch;
  p->graph_rows = rows;
  return FE_OK;
}

}  // namespace

extern "C" {

int fe_attn_plan_prepare_device(fe_attn_plan* p, const int32_t* qo, const int32_t* kv,
                                const int32_t* pages, const int32_t* last, int batch, int rows,
                                void* stream) {
  if (batch > 0 && (!qo || !kv || !pages || !last))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_prepare_device: null metadata pointer");
  DevPlanArgs a{};
  a.mode = 0;
  a.qo = qo;
  a.kv = kv;
  a.pages = pages;
  a.last = last;
  return prepare_on_device(p, a, batch, rows, stream, "fe_attn_plan_prepare_device");
}

int fe_step_prepare_device(fe_attn_plan* p, const int32_t* block_tables, int table_stride,
                           const int32_t* starts, int batch, int rows_per_seq, int64_t* slots,
                           int64_t* positions, void* stream) {
  if (rows_per_seq < 1 || table_stride < 1)
    return fail(FE_ERR_INVALID_ARGUMENT,
                "fe_step_prepare_device: rows_per_seq and table_stride must be positive");
  if (batch > 0 && (!block_tables || !starts || !slots || !positions))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_step_prepare_device: null pointer");
  if (int64_t(batch) * rows_per_seq > INT32_MAX / 2)
    return fail(FE_ERR_CAPACITY, "fe_step_prepare_device: batch * rows_per_seq too large");
  DevPlanArgs a{};
  a.mode = 1;
  a.tables = block_tables;
  a.stride = table_stride;
  a.starts = starts;
  a.rows_per_seq = rows_per_seq;
  a.slots = slots;
  a.positions = positions;
  return prepare_on_device(p, a, batch, batch * rows_per_seq, stream, "fe_step_prepare_device");
}

// Test hook: copy the plan's device metadata (the lists the kernels read)
// into host memory `dst`, at most `cap` bytes; synchronises `stream`.
int fe_attn_plan_debug_device_meta(const fe_attn_plan* p, void* dst, int64_t cap, void* stream) {
  if (!p || !dst) return fail(FE_ERR_INVALID_ARGUMENT, "null pointer");
  if (p->host_only) return fail(FE_ERR_INVALID_ARGUMENT, "host-only plan");
  const size_t n = static_cast<size_t>(std::min<int64_t>(cap, static_cast<int64_t>(p->meta_cap)));
  auto s = static_cast<cudaStream_t>(stream);
  FE_CUDA_TRY(cudaMemcpyAsync(dst, p->d_meta, n, cudaMemcpyDeviceToHost, s));
  FE_CUDA_TRY(cudaStreamSynchronize(s));
  return FE_OK;
}

int fe_attn_run(fe_attn_plan* p, const void* q, const void* k_pool, const void* v_pool, void* out,
                int causal, void* stream) {
  return fe_attn_run_lists(p, q, k_pool, v_pool, out, causal, FE_ATTN_LISTS_ALL, stream);
}

int fe_attn_run_lists(fe_attn_plan* p, const void* q, const void* k_pool, const void* v_pool,
                      void* out, int causal, int lists, void* stream) {
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: plan is null");
  if (p->host_only) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: host-only plan");
  if (!p->prepared) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: plan not prepared");
  const int view = causal ? 1 : 0;
  // A plan prepared for graph capture launches both kernels at full width
  // every time (CTAs without work exit at once), so the captured launches
  // stay valid for any later metadata.
  const int grid_rows =
      (lists & FE_ATTN_LISTS_ROWS) ? (p->fixed_grid ? p->cfg.grid_cap : p->grid_view[view]) : 0;
  const int grid_dec =
      (lists & FE_ATTN_LISTS_DECODE) ? (p->fixed_grid ? p->cfg.dec_grid_cap : p->grid_view[2]) : 0;
  if (grid_rows == 0 && grid_dec == 0) return FE_OK;
  if (!q || !k_pool || !v_pool || !out)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: null pointer");
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: buffers must be 16-byte aligned");
  const int64_t cache_slots = int64_t(p->cfg.num_blocks + 1) * p->cfg.page;
  const int H = p->cfg.dec_heads;
  const int dim = p->cfg.dim;
  const bool wide = dim == kWideHeadDim;
  if (k_pool != p->kmap_ptr) {
    int rc = encode_pool_map(&p->kmap, k_pool, p->dtype, p->cfg.hkv, dim, cache_slots);
    if (rc != FE_OK) return rc;
    if (encode_decode_map(&p->kmap_dec, k_pool, p->dtype, p->cfg.hkv, dim, H, cache_slots) !=
        FE_OK)
      p->per_head_tma = true;
    rc = encode_tc_map(&p->kmap_tc, k_pool, p->dtype, p->cfg.hkv, dim, cache_slots);
    if (rc != FE_OK) return rc;
    p->kmap_ptr = k_pool;
  }
  if (v_pool != p->vmap_ptr) {
    int rc = encode_pool_map(&p->vmap, v_pool, p->dtype, p->cfg.hkv, dim, cache_slots);
    if (rc != FE_OK) return rc;
    if (encode_decode_map(&p->vmap_dec, v_pool, p->dtype, p->cfg.hkv, dim, H, cache_slots) !=
        FE_OK)
      p->per_head_tma = true;
    rc = encode_tc_map(&p->vmap_tc, v_pool, p->dtype, p->cfg.hkv, dim, cache_slots);
    if (rc != FE_OK) return rc;
    p->vmap_ptr = v_pool;
  }
  MetaHeader h;
  std::memcpy(&h, p->last.meta.data(), sizeof(h));
  // split units of the decode list are merged by a second, dependent kernel
  int grid_merge = 0;
  if (grid_dec > 0) grid_merge = p->fixed_grid ? p->cfg.dec_grid_cap : h.n_groups[2];
  // Merge CTAs per split unit: one warp per record row, 32 rows per CTA. The
  // host plan knows its units' rows; a graph plan (fixed launch geometry) or
  // a device-built plan takes the bound: H heads x 16 packed rows for the
  // decode list, 128 rows for a row list.
  auto merge_y = [&](int list) {
    const int bound = list == 2 ? p->cfg.dec_heads * kRowBlock : 128;
    const int rows = (p->fixed_grid || p->device_planned) ? bound : p->last.split_rows[list];
    return std::max(1, (rows + 31) / 32);
  };
  // the row kernel's Q tiles come from a tensor map over this call's q
  // (the prepared step's query rows, which a graph plan keeps fixed)
  CUtensorMap qmap;
  std::memset(&qmap, 0, sizeof(qmap));  // unused when G does not divide 128
  int q_map_rows = 0;
  if (grid_rows > 0 && 128 % (p->cfg.hq / p->cfg.hkv) == 0 && h.rows > 0) {
    int rc = encode_q_map(&qmap, q, p->dtype, p->cfg.hq, dim, h.rows, p->cfg.hq / p->cfg.hkv);
    if (rc != FE_OK) return rc;
    q_map_rows = h.rows;
  }
  // split pieces of the row list (head_dim 256 steps with few row items)
  // are merged by the merge kernel over that list
  const int grid_row_merge =
      !wide || grid_rows == 0 ? 0 : (p->fixed_grid ? p->cfg.grid_cap : h.n_groups[view]);
  const float scale_log2 = 1.4426950408889634f / sqrtf(float(dim));
  auto s = static_cast<cudaStream_t>(stream);
  const int G = p->cfg.hq / p->cfg.hkv;
  const CUtensorMap& kd = p->per_head_tma ? p->kmap : p->kmap_dec;
  const CUtensorMap& vd = p->per_head_tma ? p->vmap : p->vmap_dec;
  // A mixed step planned side by side (the two lists' grids sum to the SMs)
  // forks: the row kernel runs on the plan's side stream while the decode
  // kernel and its merge run on `stream`, which then waits for the side.
  // They read the same q and pools and write disjoint output rows and split
  // records.
  const bool fork = grid_dec > 0 && grid_rows > 0 && !p->fixed_grid && p->last.concurrent;
  cudaStream_t rs = s;
  if (fork) {
    FE_CUDA_TRY(cudaEventRecord(p->fork_ev, s));
    FE_CUDA_TRY(cudaStreamWaitEvent(p->side, p->fork_ev, 0));
    rs = p->side;
  }
  auto launch_all = [&](const auto& a) -> int {
    // Side by side, a merge waits for its kernel's grid to complete before
    // it takes an SM (a programmatic dependent would sit on SMs the other
    // kernel needs while it waits).
    if (grid_rows > 0 && fork) {
      int rc = prefill_tc_launch(p->dtype, dim, p->kmap_tc, p->vmap_tc, qmap, &a, grid_rows, rs);
      if (rc == FE_OK)
        rc = decode_merge_launch(p->dtype, dim, view, &a, grid_row_merge, merge_y(view), rs,
                                 false);
      if (rc != FE_OK) return rc;
    }
    if (grid_dec > 0) {
      int rc = decode_launch(p->dtype, dim, H, kd, vd, p->per_head_tma, &a, grid_dec, s);
      if (rc == FE_OK)
        rc = decode_merge_launch(p->dtype, dim, 2, &a, grid_merge, merge_y(2), s, !fork);
      if (rc != FE_OK) return rc;
    }
    if (grid_rows > 0 && !fork) {
      int rc = prefill_tc_launch(p->dtype, dim, p->kmap_tc, p->vmap_tc, qmap, &a, grid_rows, s);
      if (rc == FE_OK)
        rc = decode_merge_launch(p->dtype, dim, view, &a, grid_row_merge, merge_y(view), s, true);
      return rc;
    }
    return FE_OK;
  };
  int rc;
  if (p->dtype == FE_DTYPE_BF16) {
    AttnArgs<__nv_bfloat16> a{p->d_meta, static_cast<const __nv_bfloat16*>(q),
                              static_cast<__nv_bfloat16*>(out), p->d_partials, p->d_counters,
                              device_error_word(), p->cfg.hq, G, p->cfg.page, view, scale_log2,
                              q_map_rows};
    rc = launch_all(a);
  } else {
    AttnArgs<__half> a{p->d_meta, static_cast<const __half*>(q), static_cast<__half*>(out),
                       p->d_partials, p->d_counters, device_error_word(), p->cfg.hq, G,
                       p->cfg.page, view, scale_log2, q_map_rows};
    rc = launch_all(a);
  }
  if (fork) {
    // join even after a failed launch, so `stream` never runs ahead of the side
    cudaError_t e1 = cudaEventRecord(p->join_ev, p->side);
    cudaError_t e2 = cudaStreamWaitEvent(s, p->join_ev, 0);
    if (rc == FE_OK && e1 != cudaSuccess) return cuda_fail(e1, "fe_attn_run: join record");
    if (rc == FE_OK && e2 != cudaSuccess) return cuda_fail(e2, "fe_attn_run: join wait");
  }
  if (rc != FE_OK) return rc;
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

int fe_attn_plan_get_info(const fe_attn_plan* p, fe_attn_plan_info* info) {
  if (!p || !info) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_get_info: null pointer");
  std::memset(info, 0, sizeof(*info));
  if (!p->prepared) return FE_OK;
  MetaHeader h;
  std::memcpy(&h, p->last.meta.data(), sizeof(h));
  // after a device-side prepare the counts stay on the device: they read -1
  info->batch = h.batch;
  info->rows = h.rows;
  info->decode_items = p->last.decode_items;
  info->prefill_items = p->last.prefill_items;
  info->split_sequences = p->last.split_units;
  info->chunk_tiles = p->last.chunk_tiles;
  info->grid_ctas = p->fixed_grid ? p->cfg.grid_cap + p->cfg.dec_grid_cap
                                  : p->last.grid[1] + p->last.grid[2];
  info->kv_tokens = p->last.kv_tokens;
  return FE_OK;
}

// Test hook: copy the packed metadata of the last prepare into `dst`
// (returns its size in *bytes; copies at most `cap` bytes).
int fe_attn_plan_debug_meta(const fe_attn_plan* p, void* dst, int64_t cap, int64_t* bytes) {
  if (!p || !bytes) return fail(FE_ERR_INVALID_ARGUMENT, "null pointer");
  *bytes = static_cast<int64_t>(p->last.meta.size());
  if (dst && cap > 0)
    std::memcpy(dst, p->last.meta.data(),
                static_cast<size_t>(std::min<int64_t>(cap, *bytes)));
  return FE_OK;
}

}  // extern "C"
