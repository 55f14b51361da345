// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// Builds the reference's own CUDA attention path (FlashEngine.cpp
// src/flashinfer_attention.cu: create_plan / prepare_plan / attention over
// FlashInfer's FA2 paged prefill kernel, split-KV disabled) for sm_100a,
// straight from the reference source tree, unmodified, with the FlashInfer
// headers installed in this image (0.6.11.post2; the reference pins 0.6.14,
// dependencies.lock.json:10). It is the reference's GPU comparator: GPU tests
// check its output against the oracle and this repository's kernels, and
// bench.py's reference arm times it on the same inputs as this repository's
// decode and verify launches.
//
// The reference file throws std::runtime_error on errors; the extern "C"
// surface below catches every exception and returns 1, keeping the message
// for fe_ref_fi_last_error(). The library is linked with -Bsymbolic so these
// wrappers always call the reference's fe::cuda functions, never the shim's
// functions of the same name.
#include "../src/flashinfer_attention.cu"

#include <exception>
#include <string>

namespace {
thread_local std::string g_fi_error;
template <class F>
int fi_guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_fi_error = e.what();
    return 1;
  } catch (...) {
    g_fi_error = "unknown exception";
    return 1;
  }
}
}  // namespace

extern "C" {
const char* fe_ref_fi_last_error() { return g_fi_error.c_str(); }

int fe_ref_fi_create_plan(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                          int bf16, int blocks, void** out) {
  return fi_guarded([&] {
    *out = fe::cuda::create_plan(hq, hkv, dim, page, max_batch, max_pages, bf16 != 0, blocks);
  });
}

void fe_ref_fi_destroy_plan(void* plan) {
  fe::cuda::destroy_plan(static_cast<fe::cuda::AttentionPlan*>(plan));
}

int fe_ref_fi_prepare_plan(void* plan, const int32_t* qo, const int32_t* kv, const int32_t* pages,
                           const int32_t* last, int batch, int rows, int graph, void* stream) {
  return fi_guarded([&] {
    fe::cuda::prepare_plan(static_cast<fe::cuda::AttentionPlan*>(plan), qo, kv, pages, last, batch,
                           rows, graph != 0, stream);
  });
}

int fe_ref_fi_attention(void* plan, void* q, void* k, void* v, void* out, int causal,
                        void* stream) {
  return fi_guarded([&] {
    fe::cuda::attention(static_cast<fe::cuda::AttentionPlan*>(plan), q, k, v, out, causal != 0,
                        stream);
  });
}
}
