// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// Builds the reference's own ATen attention/store path
// (FlashEngine.cpp src/portable_gpu_ops.cpp, the `-DFE_REFERENCE_OPS=ON`
// backend) for the CPU, straight from the reference source tree, unmodified.
// Only tests, smoke() and bench.py's CPU baseline / reference arm load the
// resulting oracle/_ref/libfe_ref_aten.so.
//
// Two retargetings make that file run on a host without a GPU; both are done
// here, from outside the reference source:
//  1. `kCUDA` is macro-renamed to `kCPU` for the body of the reference file
//     only (the ATen headers are included first, so their own declarations
//     are untouched). Tensors the reference creates "on the device" are
//     therefore CPU tensors.
//  2. On the CPU `.to(at::kCPU)` is a no-op, so the reference's `upload()`
//     helper (portable_gpu_ops.cpp:16) would return a tensor aliasing a local
//     std::vector that dies when prepare_plan returns. The overload of
//     at::from_blob below is an exact match for `int64_t*` (the original
//     takes `void*`) and is therefore picked for that one call; it returns an
//     owning copy. Every other from_blob call in the file passes `void*`,
//     `uint8_t*` or `float*` and still aliases the caller's memory, which is
//     what the pool views need.
#include <ATen/ATen.h>
#include <ATen/Parallel.h>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>

namespace at {
inline Tensor from_blob(int64_t* data, IntArrayRef sizes, const TensorOptions& options) {
  return at::from_blob(static_cast<void*>(data), sizes, options).clone();
}
}  // namespace at

#define kCUDA kCPU
#include "../src/portable_gpu_ops.cpp"
#undef kCUDA

// ---------------------------------------------------------------------------
// extern "C" surface for ctypes. Every function returns 0 on success and 1
// when the reference threw; the message is kept for fe_ref_last_error().
// ---------------------------------------------------------------------------
namespace {
thread_local std::string g_error;
template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  } catch (...) {
    g_error = "unknown exception";
    return 1;
  }
}
}  // namespace

extern "C" {
const char* fe_ref_last_error() { return g_error.c_str(); }

void fe_ref_set_threads(int n) { at::set_num_threads(n); }
int fe_ref_get_threads() { return at::get_num_threads(); }

int fe_ref_create_plan(int hq, int hkv, int dim, int page, int max_batch, int max_pages, int bf16,
                       int blocks, void** out) {
  return guarded([&] {
    *out = fe::cuda::create_plan(hq, hkv, dim, page, max_batch, max_pages, bf16 != 0, blocks);
  });
}

void fe_ref_destroy_plan(void* plan) {
  fe::cuda::destroy_plan(static_cast<fe::cuda::AttentionPlan*>(plan));
}

int fe_ref_prepare_plan(void* plan, const int32_t* qo, const int32_t* kv, const int32_t* pages,
                        const int32_t* last, int batch, int rows, int graph) {
  return guarded([&] {
    fe::cuda::prepare_plan(static_cast<fe::cuda::AttentionPlan*>(plan), qo, kv, pages, last, batch,
                           rows, graph != 0, nullptr);
  });
}

int fe_ref_attention(void* plan, void* q, void* k, void* v, void* out, int causal) {
  return guarded([&] {
    fe::cuda::attention(static_cast<fe::cuda::AttentionPlan*>(plan), q, k, v, out, causal != 0,
                        nullptr);
  });
}

int fe_ref_store(const void* k, const void* v, void* kc, void* vc, const int64_t* slots, int rows,
                 int width, int bf16, int cache_slots) {
  return guarded([&] {
    fe::cuda::store(k, v, kc, vc, slots, rows, width, bf16 != 0, nullptr, cache_slots);
  });
}
}
