// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// Builds the reference's own CUDA kernels for the paged-KV neighbours of the
// hot path (FlashEngine.cpp src/cuda_kernels.cu: rope, store, accept) for
// sm_100a, straight from the reference source tree, unmodified, and exposes
// them with C linkage so the GPU tests can run them beside this repository's
// kernels on the same device buffers. Only tests load the resulting
// oracle/_ref/libfe_ref_cuda.so.
#include <cstdint>
#include <exception>

#include "../src/cuda_kernels.cu"

extern "C" {

int ref_cuda_rope(void* q, void* k, const int64_t* pos, const float* cache, int rows, int hq,
                  int hkv, int dim, int bf16, void* stream, int max_positions) {
  try {
    fe::cuda::rope(q, k, pos, cache, rows, hq, hkv, dim, bf16 != 0, stream, max_positions);
  } catch (const std::exception&) {
    return 1;
  }
  return 0;
}

int ref_cuda_store(const void* k, const void* v, void* kc, void* vc, const int64_t* slots,
                   int rows, int width, int bf16, void* stream, int cache_slots) {
  try {
    fe::cuda::store(k, v, kc, vc, slots, rows, width, bf16 != 0, stream, cache_slots);
  } catch (const std::exception&) {
    return 1;
  }
  return 0;
}

int ref_cuda_accept(const int64_t* draft, const int64_t* verify, int64_t* out, int batch, int k,
                    void* stream) {
  try {
    fe::cuda::accept(draft, verify, out, batch, k, stream);
  } catch (const std::exception&) {
    return 1;
  }
  return 0;
}

}  // extern "C"
