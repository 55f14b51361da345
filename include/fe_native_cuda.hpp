// fe_native_cuda.hpp — C++ operator boundary for FlashEngine.cpp's CUDA
// DeviceModel, implemented over the fe_kv.h C ABI (libfe_native_cuda_b200.so).
//
// The KV / attention declarations keep the exact signatures of the
// reference's namespace fe::cuda (Cambridgebit/FlashEngine.cpp
// include/fe/native_cuda.hpp:6-10,13-15), so src/cuda_model.cpp compiles
// unchanged against this library in place of src/flashinfer_attention.cu and
// the rope(), store() and accept() of src/cuda_kernels.cu. Errors surface as std::runtime_error,
// as check() does in the reference (src/cuda_kernels.cu:10,
// src/flashinfer_attention.cu:13). No LibTorch types.
//
// rope_store, copy_blocks and clear_pages are additions with no reference
// counterpart.
#pragma once
#include <cstddef>
#include <cstdint>

namespace fe::cuda {
struct AttentionPlan;
// include/fe/native_cuda.hpp:7
AttentionPlan* create_plan(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                           bool bf16, int blocks);
// include/fe/native_cuda.hpp:8
void destroy_plan(AttentionPlan* plan);
// include/fe/native_cuda.hpp:9 — qo/kv/pages/last are HOST pointers.
void prepare_plan(AttentionPlan* plan, const int32_t* qo, const int32_t* kv, const int32_t* pages,
                  const int32_t* last, int batch, int rows, bool graph, void* stream);
// include/fe/native_cuda.hpp:10 — device pointers.
void attention(AttentionPlan* plan, void* q, void* k, void* v, void* output, bool causal,
               void* stream);
// include/fe/native_cuda.hpp:13 — q [rows, hq, dim] and k [rows, hkv, dim]
// rotated in place with the fp32 cache [max_positions, dim]; pos is a device
// int64 array. Bit-identical to the reference kernel.
void rope(void* q, void* k, const int64_t* pos, const float* cache, int rows, int hq, int hkv,
          int dim, bool bf16, void* stream, int max_positions);
// include/fe/native_cuda.hpp:14 — slots is a device int64 array.
void store(const void* k, const void* v, void* kc, void* vc, const int64_t* slots, int rows,
           int width, bool bf16, void* stream, int cache_slots);
// include/fe/native_cuda.hpp:15 — draft [batch, k], verify [batch, k+1],
// committed [batch, k+2], all device int64.
void accept(const int64_t* draft, const int64_t* verify, int64_t* committed, int batch, int k,
            void* stream);

// rope() followed by store() in one launch: q rotated in place, rotated keys
// written back to k and, with v, to the pools through `slots` (no reference
// counterpart; same results as the two calls).
// rotary_dim <= 0 rotates all dims (the cache is [max_positions, dim]);
// 0 < rotary_dim < dim rotates the leading rotary_dim dims with a
// [max_positions, rotary_dim] cache (Qwen3.5 partial rotary).
void rope_store(void* q, void* k, const void* v, void* kc, void* vc, const int64_t* slots,
                const int64_t* pos, const float* cache, int rows, int hq, int hkv, int dim,
                bool bf16, void* stream, int max_positions, int cache_slots, int rotary_dim = 0);

// Block copy / copy-on-write across layers (no reference counterpart):
// k_pools/v_pools are host arrays of per-layer device pool pointers,
// src/dst/ntok are device int32 arrays of num_copies entries.
void copy_blocks(void* const* k_pools, void* const* v_pools, int layers, const int32_t* src,
                 const int32_t* dst, const int32_t* ntok, int num_copies, int page, int width,
                 int blocks, bool bf16, void* stream);
// Zero whole pages (e.g. the graph-padding page `blocks`) of every pool.
void clear_pages(void* const* pools, int num_pools, const int32_t* pages, int num_pages, int page,
                 int width, int blocks, bool bf16, void* stream);
}  // namespace fe::cuda
