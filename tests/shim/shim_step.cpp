// TEST INFRASTRUCTURE — drives one attention layer-step through the C++ shim
// (libfe_native_cuda_b200.so, include/fe_native_cuda.hpp) with the call
// sequence of the reference's CUDA DeviceModel (Cambridgebit/FlashEngine.cpp
// src/cuda_model.cpp:94-96 and :118-140): create_plan, prepare_plan with host
// metadata, rope, store, attention, then accept (:184), destroy_plan. Then
// checks the shim's error behaviour: invalid calls must throw
// std::runtime_error, as check() does in the reference (src/cuda_kernels.cu:10).
//
//   shim_step <dir>
// <dir>/dims.txt holds "hq hkv dim page batch rows max_pages blocks bf16
// max_positions kdraft"; the inputs are raw little-endian arrays in <dir>
// (kpool, vpool, knew, vnew, q: uint16; slots, pos, draft, verify: int64;
// qo, kv, pages, last: int32; cache: float32). Outputs are written beside
// them: kpool.out, vpool.out, q.out, knew.out, attn.out, accept.out.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "fe_native_cuda.hpp"

namespace {
std::string g_dir;

std::vector<char> read_file(const std::string& name) {
  std::ifstream f(g_dir + "/" + name, std::ios::binary);
  if (!f) throw std::runtime_error("missing input " + name);
  return std::vector<char>(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
}

void write_file(const std::string& name, const std::vector<char>& data) {
  std::ofstream f(g_dir + "/" + name, std::ios::binary);
  f.write(data.data(), static_cast<std::streamsize>(data.size()));
}

void cu(cudaError_t rc, const char* what) {
  if (rc != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(rc));
}

struct Dev {
  void* p = nullptr;
  size_t n = 0;
  explicit Dev(const std::vector<char>& h) : n(h.size()) {
    cu(cudaMalloc(&p, n ? n : 16), "cudaMalloc");
    if (n) cu(cudaMemcpy(p, h.data(), n, cudaMemcpyHostToDevice), "H2D");
  }
  explicit Dev(size_t bytes) : n(bytes) { cu(cudaMalloc(&p, n ? n : 16), "cudaMalloc"); }
  ~Dev() { cudaFree(p); }
  std::vector<char> host() const {
    std::vector<char> h(n);
    if (n) cu(cudaMemcpy(h.data(), p, n, cudaMemcpyDeviceToHost), "D2H");
    return h;
  }
  template <class T>
  T* as() const { return static_cast<T*>(p); }
};

template <class F>
bool throws_runtime_error(F&& f) {
  try {
    f();
  } catch (const std::runtime_error&) {
    return true;
  }
  return false;
}
}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: shim_step <dir>\n");
    return 2;
  }
  g_dir = argv[1];
  try {
    int hq, hkv, dim, page, batch, rows, max_pages, blocks, bf16, max_positions, kdraft;
    {
      std::ifstream f(g_dir + "/dims.txt");
      if (!(f >> hq >> hkv >> dim >> page >> batch >> rows >> max_pages >> blocks >> bf16 >>
            max_positions >> kdraft))
        throw std::runtime_error("bad dims.txt");
    }
    const int width = hkv * dim;
    const int cache_slots = (blocks + 1) * page;
    auto qo = read_file("qo"), kv = read_file("kv"), pages = read_file("pages"),
         last = read_file("last");
    Dev kc(read_file("kpool")), vc(read_file("vpool")), k(read_file("knew")),
        v(read_file("vnew")), q(read_file("q")), slots(read_file("slots")), pos(read_file("pos")),
        cache(read_file("cache")), draft(read_file("draft")), verify(read_file("verify"));
    Dev out(q.n), committed(size_t(batch) * (kdraft + 2) * sizeof(int64_t));
    cu(cudaMemset(committed.p, 0xff, committed.n), "memset");
    cudaStream_t stream;
    cu(cudaStreamCreate(&stream), "stream");
    void* s = stream;

    fe::cuda::AttentionPlan* plan =
        fe::cuda::create_plan(hq, hkv, dim, page, batch, max_pages, bf16 != 0, blocks);
    fe::cuda::prepare_plan(plan, reinterpret_cast<const int32_t*>(qo.data()),
                           reinterpret_cast<const int32_t*>(kv.data()),
                           reinterpret_cast<const int32_t*>(pages.data()),
                           reinterpret_cast<const int32_t*>(last.data()), batch, rows, false, s);
    fe::cuda::rope(q.p, k.p, pos.as<int64_t>(), cache.as<float>(), rows, hq, hkv, dim, bf16 != 0,
                   s, max_positions);
    fe::cuda::store(k.p, v.p, kc.p, vc.p, slots.as<int64_t>(), rows, width, bf16 != 0, s,
                    cache_slots);
    fe::cuda::attention(plan, q.p, kc.p, vc.p, out.p, true, s);
    fe::cuda::accept(draft.as<int64_t>(), verify.as<int64_t>(), committed.as<int64_t>(), batch,
                     kdraft, s);
    cu(cudaStreamSynchronize(stream), "sync");

    write_file("kpool.out", kc.host());
    write_file("vpool.out", vc.host());
    write_file("q.out", q.host());
    write_file("knew.out", k.host());
    write_file("attn.out", out.host());
    write_file("accept.out", committed.host());

    // Error behaviour: each of these must surface as std::runtime_error.
    std::vector<int32_t> big_qo(batch + 2), big_kv(batch + 2, 0), big_last(batch + 1, 1);
    for (int b = 0; b <= batch + 1; ++b) big_qo[b] = b;
    for (int b = 0; b <= batch + 1; ++b) big_kv[b] = b;
    std::vector<int32_t> some_pages(batch + 1, 0);
    const bool e_capacity = throws_runtime_error([&] {
      fe::cuda::prepare_plan(plan, big_qo.data(), big_kv.data(), some_pages.data(),
                             big_last.data(), batch + 1, batch + 1, false, s);
    });
    const int32_t ctx_qo[2] = {0, 5}, ctx_kv[2] = {0, 1}, ctx_pages[1] = {0}, ctx_last[1] = {3};
    const bool e_context = throws_runtime_error([&] {
      fe::cuda::prepare_plan(plan, ctx_qo, ctx_kv, ctx_pages, ctx_last, 1, 5, false, s);
    });
    const int32_t bad_pages[1] = {blocks + 1}, one_last[1] = {1}, one_qo[2] = {0, 1};
    const bool e_page = throws_runtime_error([&] {
      fe::cuda::prepare_plan(plan, one_qo, ctx_kv, bad_pages, one_last, 1, 1, false, s);
    });
    const bool e_dim = throws_runtime_error(
        [&] { fe::cuda::destroy_plan(fe::cuda::create_plan(hq, hkv, 64, page, 1, 4, true, 8)); });
    const bool e_width = throws_runtime_error([&] {
      fe::cuda::store(k.p, v.p, kc.p, vc.p, slots.as<int64_t>(), rows, width - 4, bf16 != 0, s,
                      cache_slots);
    });
    const bool e_null = throws_runtime_error(
        [&] { fe::cuda::attention(nullptr, q.p, kc.p, vc.p, out.p, true, s); });
    fe::cuda::destroy_plan(plan);
    cu(cudaStreamDestroy(stream), "stream destroy");
    std::printf("errors capacity=%d context=%d page=%d dim=%d width=%d null_plan=%d\n", e_capacity,
                e_context, e_page, e_dim, e_width, e_null);
    std::printf("shim_step ok\n");
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "shim_step failed: %s\n", e.what());
    return 1;
  }
}
