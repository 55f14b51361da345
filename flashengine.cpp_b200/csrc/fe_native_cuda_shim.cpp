// fe::cuda shim over the fe_kv.h C ABI: the reference's operator signatures
// (Cambridgebit/FlashEngine.cpp include/fe/native_cuda.hpp:6-14) with its
// error behaviour (std::runtime_error from a failed status, as check() at
// src/cuda_kernels.cu:10 / src/flashinfer_attention.cu:13).
#include "fe_native_cuda.hpp"

#include <stdexcept>
#include <string>

#include "fe_kv.h"

namespace fe::cuda {
namespace {
void check(int status, const char* what) {
  if (status != FE_OK)
    throw std::runtime_error(std::string(what) + ": " + fe_status_string(status) + ": " +
                             fe_last_error());
}
}  // namespace

struct AttentionPlan {
  fe_attn_plan* plan = nullptr;
};

AttentionPlan* create_plan(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                           bool bf16, int blocks) {
  fe_attn_plan* raw = nullptr;
  check(fe_attn_plan_create(hq, hkv, dim, page, max_batch, max_pages,
                            bf16 ? FE_DTYPE_BF16 : FE_DTYPE_F16, blocks, &raw),
        "create_plan");
  auto* p = new AttentionPlan();
  p->plan = raw;
  return p;
}

void destroy_plan(AttentionPlan* plan) {
  if (!plan) return;
  fe_attn_plan_destroy(plan->plan);
  delete plan;
}

void prepare_plan(AttentionPlan* plan, const int32_t* qo, const int32_t* kv, const int32_t* pages,
                  const int32_t* last, int batch, int rows, bool graph, void* stream) {
  if (!plan) throw std::runtime_error("prepare_plan: null plan");
  check(fe_attn_plan_prepare(plan->plan, qo, kv, pages, last, batch, rows, graph ? 1 : 0, stream),
        "prepare_plan");
}

void attention(AttentionPlan* plan, void* q, void* k, void* v, void* output, bool causal,
               void* stream) {
  if (!plan) throw std::runtime_error("attention: null plan");
  check(fe_attn_run(plan->plan, q, k, v, output, causal ? 1 : 0, stream), "attention");
}

void store(const void* k, const void* v, void* kc, void* vc, const int64_t* slots, int rows,
           int width, bool bf16, void* stream, int cache_slots) {
  check(fe_kv_append(k, v, kc, vc, slots, rows, width, bf16 ? FE_DTYPE_BF16 : FE_DTYPE_F16,
                     cache_slots, stream),
        "store");
}

void rope(void* q, void* k, const int64_t* pos, const float* cache, int rows, int hq, int hkv,
          int dim, bool bf16, void* stream, int max_positions) {
  check(fe_rope(q, k, pos, cache, rows, hq, hkv, dim, dim, max_positions,
                bf16 ? FE_DTYPE_BF16 : FE_DTYPE_F16, stream),
        "rope");
}

void accept(const int64_t* draft, const int64_t* verify, int64_t* committed, int batch, int k,
            void* stream) {
  check(fe_accept(draft, verify, committed, batch, k, stream), "accept");
}

void rope_store(void* q, void* k, const void* v, void* kc, void* vc, const int64_t* slots,
                const int64_t* pos, const float* cache, int rows, int hq, int hkv, int dim,
                bool bf16, void* stream, int max_positions, int cache_slots, int rotary_dim) {
  check(fe_rope_append(q, k, v, k, kc, vc, slots, pos, cache, rows, hq, hkv, dim,
                       rotary_dim <= 0 ? dim : rotary_dim, max_positions,
                       bf16 ? FE_DTYPE_BF16 : FE_DTYPE_F16, cache_slots, stream),
        "rope_store");
}

void copy_blocks(void* const* k_pools, void* const* v_pools, int layers, const int32_t* src,
                 const int32_t* dst, const int32_t* ntok, int num_copies, int page, int width,
                 int blocks, bool bf16, void* stream) {
  check(fe_kv_copy_blocks(k_pools, v_pools, layers, src, dst, ntok, num_copies, page, width,
                          blocks + 1, bf16 ? FE_DTYPE_BF16 : FE_DTYPE_F16, stream),
        "copy_blocks");
}

void clear_pages(void* const* pools, int num_pools, const int32_t* pages, int num_pages, int page,
                 int width, int blocks, bool bf16, void* stream) {
  check(fe_kv_clear_pages(pools, num_pools, pages, num_pages, page, width, blocks + 1,
                          bf16 ? FE_DTYPE_BF16 : FE_DTYPE_F16, stream),
        "clear_pages");
}
}  // namespace fe::cuda
