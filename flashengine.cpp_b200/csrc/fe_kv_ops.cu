// KV pool data-movement kernels: append (scatter through the slot mapping),
// block copy / copy-on-write, page clearing, and sequence gather. All are
// HBM-bound byte moves done with 16-byte vector loads/stores; nothing here
// computes, so results are bit-exact copies by construction.
//
// Reference: Cambridgebit/FlashEngine.cpp src/cuda_kernels.cu:24 (store_kernel,
// one 2-byte element per thread) and :34 (its launcher); the ATen variant
// src/portable_gpu_ops.cpp:54.
#include <cstring>
#include <mutex>
#include <string>

#include "fe_common.cuh"

namespace fe {

namespace {
thread_local std::string t_error;
__device__ unsigned int g_device_errors = 0;
}  // namespace

unsigned int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  static unsigned int* cache[64] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_errors) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<unsigned int*>(p);
  }
  return cache[dev];
}

void set_error(const std::string& msg) { t_error = msg; }

int fail(int status, const std::string& msg) {
  t_error = msg;
  return status;
}

int cuda_fail(cudaError_t rc, const char* what) {
  t_error = std::string(what) + ": " + cudaGetErrorName(rc) + " (" + cudaGetErrorString(rc) + ")";
  return FE_ERR_CUDA;
}

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // 16-byte chunks in flight per thread

// ---------------------------------------------------------------------------
// append: one warp per (row, K|V) unit, units strided over the grid's warps.
// The row's slot is read once; the lanes move the row's 16-byte chunks,
// kUnroll per lane in flight, all loads before any store.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) append_kernel(const uint4* __restrict__ k,
                                                          const uint4* __restrict__ v,
                                                          uint4* __restrict__ kc,
                                                          uint4* __restrict__ vc,
                                                          const int64_t* __restrict__ slots,
                                                          int rows, int chunks_per_row,
                                                          int64_t cache_slots) {
  pdl_trigger();
  pdl_wait();  // k, v come from, and the pools are read by, earlier kernels
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  for (int w = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); w < 2 * rows; w += warps) {
    const int row = w >> 1;
    const bool is_v = w & 1;
    const int64_t slot = __ldg(slots + row);
    if (slot < 0) continue;  // graph padding rows, as the reference store skips them
    if (slot >= cache_slots) {
      if (lane == 0 && !is_v) raise_device_error(&g_device_errors, FE_DEVERR_SLOT_RANGE);
      continue;
    }
    const uint4* src = (is_v ? v : k) + static_cast<int64_t>(row) * chunks_per_row;
    uint4* dst = (is_v ? vc : kc) + slot * chunks_per_row;
    for (int c0 = 0; c0 < chunks_per_row; c0 += 32 * kUnroll) {
      uint4 val[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < chunks_per_row) val[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < chunks_per_row) dst[c] = val[u];
      }
    }
  }
}

struct PoolTable {
  void* k[FE_MAX_LAYERS];
  void* v[FE_MAX_LAYERS];
};

// ---------------------------------------------------------------------------
// copy_blocks: blockIdx.y = copy index, blockIdx.z = layer * 2 + (K|V).
// Each copy is one contiguous byte range (pages are page-major), so a CTA
// streams ntok*width*2 bytes with 16-byte vectors.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) copy_blocks_kernel(
    const __grid_constant__ PoolTable pools, const int32_t* __restrict__ src,
    const int32_t* __restrict__ dst, const int32_t* __restrict__ ntok, int page,
    int chunks_per_row, int num_pages_total) {
  const int c = blockIdx.y;
  const int layer = blockIdx.z >> 1;
  const bool is_v = blockIdx.z & 1;
  const int s = __ldg(src + c), d = __ldg(dst + c), n = __ldg(ntok + c);
  if (s < 0 || s >= num_pages_total || d < 0 || d >= num_pages_total) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_device_error(&g_device_errors, FE_DEVERR_PAGE_RANGE);
    return;
  }
  if (n < 0 || n > page) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_device_error(&g_device_errors, FE_DEVERR_NTOK_RANGE);
    return;
  }
  uint4* pool = static_cast<uint4*>(is_v ? pools.v[layer] : pools.k[layer]);
  const int64_t page_chunks = static_cast<int64_t>(page) * chunks_per_row;
  const uint4* from = pool + s * page_chunks;
  uint4* to = pool + d * page_chunks;
  const int total = n * chunks_per_row;
  const int stride = gridDim.x * blockDim.x;
  for (int base = blockIdx.x * blockDim.x + threadIdx.x; base < total; base += stride * kUnroll) {
    uint4 val[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = base + u * stride;
      if (i < total) val[u] = from[i];
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = base + u * stride;
      if (i < total) to[i] = val[u];
    }
  }
}

struct PoolList {
  void* p[2 * FE_MAX_LAYERS];
};

__global__ void __launch_bounds__(kThreads) clear_pages_kernel(const __grid_constant__ PoolList pools,
                                                               const int32_t* __restrict__ pages,
                                                               int page_chunks,
                                                               int num_pages_total) {
  const int p = __ldg(pages + blockIdx.y);
  if (p < 0 || p >= num_pages_total) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_device_error(&g_device_errors, FE_DEVERR_PAGE_RANGE);
    return;
  }
  uint4* pool = static_cast<uint4*>(pools.p[blockIdx.z]);
  uint4* to = pool + static_cast<int64_t>(p) * page_chunks;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < page_chunks; i += gridDim.x * blockDim.x)
    to[i] = zero;
}

// gather: blockIdx.y = sequence; one warp per token row, the warps of the
// grid's x dimension striding over the sequence's tokens. The row's slot is
// computed once per warp; the lanes move its 16-byte chunks, kUnroll per lane
// in flight, all loads before any store.
__global__ void __launch_bounds__(kThreads) gather_kernel(const uint4* __restrict__ pool,
                                                          uint4* __restrict__ out,
                                                          const int32_t* __restrict__ kv,
                                                          const int32_t* __restrict__ pages,
                                                          const int32_t* __restrict__ last,
                                                          const int32_t* __restrict__ row_offset,
                                                          int page, int chunks_per_row) {
  const int b = blockIdx.y;
  const int p0 = __ldg(kv + b), p1 = __ldg(kv + b + 1);
  const int len = (p1 - p0 - 1) * page + __ldg(last + b);
  const int64_t orow = __ldg(row_offset + b);
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  for (int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); t < len; t += warps) {
    const int64_t slot = static_cast<int64_t>(__ldg(pages + p0 + t / page)) * page + t % page;
    const uint4* src = pool + slot * chunks_per_row;
    uint4* dst = out + (orow + t) * chunks_per_row;
    for (int c0 = 0; c0 < chunks_per_row; c0 += 32 * kUnroll) {
      uint4 val[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < chunks_per_row) val[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < chunks_per_row) dst[c] = val[u];
      }
    }
  }
}

int sm_count() {
  static int cached = 0;
  if (!cached) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      return 148;
    cached = n;
  }
  return cached;
}


}  // namespace
}  // namespace fe

using namespace fe;

extern "C" {

const char* fe_status_string(int status) {
  switch (status) {
    case FE_OK: return "ok";
    case FE_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FE_ERR_CAPACITY: return "capacity exceeded";
    case FE_ERR_CONTEXT: return "context out of bounds";
    case FE_ERR_CUDA: return "CUDA error";
    case FE_ERR_UNSUPPORTED: return "unsupported configuration";
    case FE_ERR_DEVICE: return "device-side error";
    case FE_ERR_NO_DEVICE: return "no usable device";
    default: return "unknown status";
  }
}

const char* fe_last_error(void) { return t_error.c_str(); }

int fe_abi_version(void) { return FE_KV_ABI_VERSION; }

int fe_device_errors(void* stream, uint32_t* bits_out) {
  if (!bits_out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_device_errors: bits_out is null");
  auto s = static_cast<cudaStream_t>(stream);
  unsigned int host = 0, zero = 0;
  FE_CUDA_TRY(cudaMemcpyFromSymbolAsync(&host, g_device_errors, sizeof(host), 0,
                                        cudaMemcpyDeviceToHost, s));
  FE_CUDA_TRY(cudaMemcpyToSymbolAsync(g_device_errors, &zero, sizeof(zero), 0,
                                      cudaMemcpyHostToDevice, s));
  FE_CUDA_TRY(cudaStreamSynchronize(s));
  *bits_out = host;
  return FE_OK;
}

int fe_kv_append(const void* k, const void* v, void* k_pool, void* v_pool, const int64_t* slots,
                 int rows, int width, int dtype, int cache_slots, void* stream) {
  if (!valid_dtype(dtype)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_append: bad dtype");
  if (rows < 0 || width <= 0 || cache_slots <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_append: rows/width/cache_slots out of range");
  if (width % 8 != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_kv_append: width must be a multiple of 8 elements");
  if (rows == 0) return FE_OK;
  if (!k || !v || !k_pool || !v_pool || !slots)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_append: null pointer");
  if (!aligned16(k) || !aligned16(v) || !aligned16(k_pool) || !aligned16(v_pool))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_append: buffers must be 16-byte aligned");
  const int chunks = width / 8;
  if (rows > INT32_MAX / 2) return fail(FE_ERR_CAPACITY, "fe_kv_append: too many rows");
  // one warp per (row, K|V)
  int64_t blocks = (static_cast<int64_t>(rows) * 2 + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  FE_CUDA_TRY(launch_pdl(append_kernel, dim3(static_cast<int>(blocks)), dim3(kThreads), 0,
                         static_cast<cudaStream_t>(stream), static_cast<const uint4*>(k),
                         static_cast<const uint4*>(v), static_cast<uint4*>(k_pool),
                         static_cast<uint4*>(v_pool), slots, rows, chunks,
                         static_cast<int64_t>(cache_slots)));
  return FE_OK;
}

int fe_kv_copy_blocks(void* const* k_pools, void* const* v_pools, int num_layers,
                      const int32_t* src, const int32_t* dst, const int32_t* ntok, int num_copies,
                      int page, int width, int num_pages_total, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_copy_blocks: bad dtype");
  if (num_layers < 0 || num_layers > FE_MAX_LAYERS)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_copy_blocks: num_layers out of range");
  if (num_copies < 0 || page <= 0 || width <= 0 || num_pages_total <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_copy_blocks: bad sizes");
  if (width % 8 != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_kv_copy_blocks: width must be a multiple of 8 elements");
  if (num_copies == 0 || num_layers == 0) return FE_OK;
  if (num_copies > 65535)
    return fail(FE_ERR_CAPACITY, "fe_kv_copy_blocks: at most 65535 copies per call");
  if (!k_pools || !v_pools || !src || !dst || !ntok)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_copy_blocks: null pointer");
  PoolTable t;
  std::memset(&t, 0, sizeof(t));
  for (int l = 0; l < num_layers; ++l) {
    if (!k_pools[l] || !v_pools[l] || !aligned16(k_pools[l]) || !aligned16(v_pools[l]))
      return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_copy_blocks: pool pointers must be non-null "
                                           "and 16-byte aligned");
    t.k[l] = k_pools[l];
    t.v[l] = v_pools[l];
  }
  const int chunks = width / 8;
  const int per_copy = page * chunks;
  int bx = (per_copy + kThreads * kUnroll - 1) / (kThreads * kUnroll);
  if (bx < 1) bx = 1;
  dim3 grid(bx, num_copies, num_layers * 2);
  copy_blocks_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      t, src, dst, ntok, page, chunks, num_pages_total);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

int fe_kv_clear_pages(void* const* pools, int num_pools, const int32_t* pages, int num_pages,
                      int page, int width, int num_pages_total, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_clear_pages: bad dtype");
  if (num_pools < 0 || num_pools > 2 * FE_MAX_LAYERS || num_pages < 0 || page <= 0 || width <= 0 ||
      num_pages_total <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_clear_pages: bad sizes");
  if (width % 8 != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_kv_clear_pages: width must be a multiple of 8 elements");
  if (num_pools == 0 || num_pages == 0) return FE_OK;
  if (num_pages > 65535)
    return fail(FE_ERR_CAPACITY, "fe_kv_clear_pages: at most 65535 pages per call");
  if (!pools || !pages) return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_clear_pages: null pointer");
  PoolList t;
  std::memset(&t, 0, sizeof(t));
  for (int i = 0; i < num_pools; ++i) {
    if (!pools[i] || !aligned16(pools[i]))
      return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_clear_pages: pool pointers must be non-null "
                                           "and 16-byte aligned");
    t.p[i] = pools[i];
  }
  const int page_chunks = page * (width / 8);
  int bx = (page_chunks + kThreads - 1) / kThreads;
  dim3 grid(bx, num_pages, num_pools);
  clear_pages_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      t, pages, page_chunks, num_pages_total);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

int fe_kv_gather(const void* pool, void* out, const int32_t* kv, const int32_t* pages,
                 const int32_t* last, const int32_t* row_offset, int batch, int max_len, int page,
                 int width, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_gather: bad dtype");
  if (batch < 0 || max_len < 0 || page <= 0 || width <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_gather: bad sizes");
  if (width % 8 != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_kv_gather: width must be a multiple of 8 elements");
  if (batch == 0 || max_len == 0) return FE_OK;
  if (batch > 65535) return fail(FE_ERR_CAPACITY, "fe_kv_gather: at most 65535 sequences");
  if (!pool || !out || !kv || !pages || !last || !row_offset)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_gather: null pointer");
  if (!aligned16(pool) || !aligned16(out))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_gather: buffers must be 16-byte aligned");
  const int chunks = width / 8;
  // one warp per token row of the longest sequence, at most 1024 CTAs per
  // sequence (the warps stride over longer ones)
  int64_t bx = (static_cast<int64_t>(max_len) + kThreads / 32 - 1) / (kThreads / 32);
  if (bx > 1024) bx = 1024;
  dim3 grid(static_cast<unsigned>(bx), batch);
  gather_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(pool), static_cast<uint4*>(out), kv, pages, last, row_offset, page,
      chunks);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

}  // extern "C"
