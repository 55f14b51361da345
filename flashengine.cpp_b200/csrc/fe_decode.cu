// Paged decode attention for sm_100a: sequences whose query rows x GQA group
// fit one 16-row block (decode, short speculative verify).
//
// Reference behaviour: Cambridgebit/FlashEngine.cpp src/flashinfer_attention.cu:35-44
// (FlashInfer paged kernel, qo_len 1 per request for decode; split-KV
// disabled) with the arithmetic of src/portable_gpu_ops.cpp:39-44.
//
// B200 design: HBM-bound, so the kernel is built around contiguous reads.
//  * One persistent CTA per SM: 8 consumer warps + 1 producer warp.
//  * A work item is (sequence, group of H = gcd(hkv, 8) KV heads, range of
//    16-token key tiles). A key tile of all H heads is one contiguous
//    16 x H x 256-byte block of the page for K and one for V; the producer
//    fetches each with a single TMA box (a tensor map that walks slots
//    before heads, so each head's 16 rows land contiguously and swizzled)
//    into a 3-8 stage ring (64 KiB stages for H = 8).
//  * Consumer warp w serves head w % H; when H < 8, the 8/H warps of a head
//    take alternate tiles and merge in shared memory. Tile math: KeyState
//    (S^T = K Q^T and O^T = V^T P^T on mma.m16n8k16, fp32 accumulation).
//  * Split-K across CTAs: partial records + last-arriving CTA merges
//    (atomic ticket, no waiting), counter re-armed for graph replay.
//  * Bounded waits as in fe_attn.cu; a CTA that gives up records
//    FE_DEVERR_TIMEOUT and drains its own copies before exiting.
#include <mutex>
#include <string>

#include "fe_attn_common.cuh"

namespace fe {

int decode_launch(int dtype, int heads, const CUtensorMap& kmap, const CUtensorMap& vmap,
                  bool per_head_tma, const void* args, int grid, cudaStream_t stream);
int decode_smem_bytes(int heads);

namespace {

constexpr int kDecWarps = 8;
constexpr int kDecThreads = (kDecWarps + 1) * 32;

template <int H>
struct DecCfg {
  static constexpr int kWh = kDecWarps / H;  // warps per head
  static constexpr int kKBytes = 2 * H * kHalfBytes;
  static constexpr int kStageBytes = 2 * kKBytes;
  static constexpr int kStages = H == 8 ? 3 : (H == 4 ? 4 : 8);
  static constexpr int kCombBytes = kWh > 1 ? kDecWarps * kRowBlock * kCombStride * 4 : 0;
  static constexpr int kBarOff = kStages * kStageBytes + kCombBytes;
  static constexpr int kSmem = 1024 + kBarOff + 2 * kStages * 8 + 16;
};

template <typename T>
__device__ __forceinline__ T to_elem(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 to_elem<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half to_elem<__half>(float x) {
  return __float2half_rn(x);
}

template <typename T, int H, int NT>
__device__ __forceinline__ void decode_item(const AttnArgs<T>& a, const WorkItem& wi,
                                            const SeqInfo& si, const SplitGroup* groups,
                                            uint8_t* stages, uint64_t* full, uint64_t* empty,
                                            volatile int* flags, float* comb, int w, int lane,
                                            uint32_t& g, bool& aborted) {
  using C = DecCfg<H>;
  const int hh = w % H, sub = w / H;
  const int G = a.G;
  const int P = si.qrows * G;
  const int head0 = (wi.kvh + hh) * G;
  const bool causal = a.view == 1;
  KeyState<T, NT> ks;
  ks.init(a.q, a.hq, si.q_row0, si.qrows, si.length, head0, G, causal, lane);

  const int ntiles = wi.kt1 - wi.kt0;
  for (int jt = sub; jt < ntiles; jt += C::kWh) {
    const uint32_t gg = g + jt;
    const int s = gg % C::kStages;
    if (aborted || flags[0] || !wait_bounded(&full[s], (gg / C::kStages) & 1u, flags)) {
      aborted = true;
      break;
    }
    const uint32_t base = smem_u32(stages + s * C::kStageBytes);
    TileAddr t;
    t.k0 = base + (2 * hh) * kHalfBytes;
    t.k1 = t.k0 + kHalfBytes;
    t.v0 = t.k0 + C::kKBytes;
    t.v1 = t.v0 + kHalfBytes;
    ks.tile(t, (wi.kt0 + jt) * kTileTokens, si.length, a.scale_log2, lane);
    __syncwarp();
    if (lane == 0) mbar_arrive_cnt(&empty[s], C::kWh);
  }
  g += ntiles;
  ks.reduce_l();

  const int tid = threadIdx.x;
  const int r8 = lane >> 2, cq = lane & 3;
  const int R = H * P;  // merged rows of the item: head-major, then packed row
  if constexpr (C::kWh == 1) {
    // One warp per head: write straight from the fragments.
    if (wi.group < 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int p = nt * 8 + 2 * cq + e;
          if (p < P && !aborted) {
            const float inv = 1.f / ks.l[nt][e];
            T* dst = a.out +
                     (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + head0 + p % G) * kHeadDim;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              dst[16 * mt + r8] = to_elem<T>(ks.o[nt][mt][e] * inv);
              dst[16 * mt + r8 + 8] = to_elem<T>(ks.o[nt][mt][2 + e] * inv);
            }
          }
        }
    } else {
      float* rec = a.partials + wi.part;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int p = nt * 8 + 2 * cq + e;
          if (p < P) {
            float* row = rec + (hh * P + p) * kHeadDim;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              row[16 * mt + r8] = ks.o[nt][mt][e];
              row[16 * mt + r8 + 8] = ks.o[nt][mt][2 + e];
            }
            if (r8 == 0) {
              rec[R * kHeadDim + hh * P + p] = ks.m[nt][e];
              rec[R * (kHeadDim + 1) + hh * P + p] = ks.l[nt][e];
            }
          }
        }
    }
  } else {
    // Several warps per head: merge their states through shared memory.
    ks.stash(comb + w * kRowBlock * kCombStride, lane);
    named_barrier_sync(1, kDecWarps * 32);
    const int d4 = (tid & 31) * 4;
    for (int r = tid >> 5; r < R; r += kDecWarps) {
      const int rh = r / P, p = r % P;
      float M = -INFINITY;
#pragma unroll
      for (int sw = 0; sw < C::kWh; ++sw)
        M = fmaxf(M, comb[((sw * H + rh) * kRowBlock + p) * kCombStride + kHeadDim]);
      const float basev = M == -INFINITY ? 0.f : M;
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sw = 0; sw < C::kWh; ++sw) {
        const float* row = comb + ((sw * H + rh) * kRowBlock + p) * kCombStride;
        const float sc = fast_exp2(row[kHeadDim] - basev);
        L = fmaf(row[kHeadDim + 1], sc, L);
        const float4 x = *reinterpret_cast<const float4*>(row + d4);
        acc.x = fmaf(x.x, sc, acc.x);
        acc.y = fmaf(x.y, sc, acc.y);
        acc.z = fmaf(x.z, sc, acc.z);
        acc.w = fmaf(x.w, sc, acc.w);
      }
      if (wi.group < 0) {
        const float inv = 1.f / L;
        T* dst = a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + (wi.kvh + rh) * G +
                          p % G) * kHeadDim + d4;
        store4<T>(dst, acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      } else {
        float* rec = a.partials + wi.part;
        *reinterpret_cast<float4*>(rec + r * kHeadDim + d4) = acc;
        if ((tid & 31) == 0) {
          rec[R * kHeadDim + r] = M;
          rec[R * (kHeadDim + 1) + r] = L;
        }
      }
    }
    named_barrier_sync(1, kDecWarps * 32);
  }

  if (wi.group >= 0) {
    __threadfence();
    named_barrier_sync(1, kDecWarps * 32);
    if (tid == 0) {
      const int prev = atomicAdd(a.counters + wi.group, 1);
      flags[1] = prev == groups[wi.group].nsplit - 1 ? 1 : 0;
    }
    named_barrier_sync(1, kDecWarps * 32);
    if (flags[1]) {
      __threadfence();
      const SplitGroup gi = groups[wi.group];
      merge_partials<T>(a.partials, gi, tid, kDecWarps * 32, [&](int r) {
        const int rh = r / P, p = r % P;
        return a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + (wi.kvh + rh) * G +
                        p % G) * kHeadDim;
      });
      if (tid == 0) a.counters[wi.group] = 0;
    }
    named_barrier_sync(1, kDecWarps * 32);
  }
}

template <typename T, int H>
__global__ void __launch_bounds__(kDecThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const AttnArgs<T> a,
                        int per_head_tma) {
  using C = DecCfg<H>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* comb = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + C::kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MetaHeader* hdr = reinterpret_cast<const MetaHeader*>(a.meta);
  constexpr int kView = 2;  // decode work list
  if (static_cast<int>(blockIdx.x) >= hdr->grid[kView]) return;
  const int32_t* cta_off = reinterpret_cast<const int32_t*>(a.meta + hdr->cta_off_off[kView]);
  const WorkItem* items = reinterpret_cast<const WorkItem*>(a.meta + hdr->items_off[kView]);
  const SplitGroup* groups = reinterpret_cast<const SplitGroup*>(a.meta + hdr->groups_off[kView]);
  const SeqInfo* seqs = reinterpret_cast<const SeqInfo*>(a.meta + hdr->seqs_off);
  const int32_t* pages = reinterpret_cast<const int32_t*>(a.meta + hdr->pages_off);
  const int it0 = cta_off[blockIdx.x], it1 = cta_off[blockIdx.x + 1];
  if (it0 >= it1) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    uint32_t g = 0;
    bool ok = true;
    for (int it = it0; it < it1 && ok; ++it) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int hh0 = w.kvh * 2;
      for (int j0 = w.kt0; j0 < w.kt1 && ok; j0 += 32) {
        const int n = min(32, w.kt1 - j0);
        int slot0 = 0;
        if (lane < n) {
          const int t0 = (j0 + lane) * kTileTokens;
          const int pid = __ldg(pages + si.page_off + t0 / a.page);
          slot0 = pid * a.page + (t0 % a.page);
        }
        for (int jj = 0; jj < n; ++jj) {
          const int s0 = __shfl_sync(0xffffffffu, slot0, jj);
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1u;
          int good = 1;
          if (lane == 0) {
            if (flags[0] || !wait_bounded(&empty[s], ph ^ 1u, flags)) {
              good = 0;
            } else {
              mbar_arrive_expect_tx(&full[s], C::kStageBytes);
              uint8_t* st = stages + s * C::kStageBytes;
              if (!per_head_tma) {
                tma_load_3d(st, &kmap, &full[s], 0, s0, hh0);
                tma_load_3d(st + C::kKBytes, &vmap, &full[s], 0, s0, hh0);
              } else {
                for (int x = 0; x < 2 * H; ++x) {
                  tma_load_3d(st + x * kHalfBytes, &kmap, &full[s], 0, hh0 + x, s0);
                  tma_load_3d(st + C::kKBytes + x * kHalfBytes, &vmap, &full[s], 0, hh0 + x, s0);
                }
              }
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          ++g;
        }
      }
    }
    if (!ok && lane == 0) {
      raise_device_error(a.err, FE_DEVERR_TIMEOUT);
      flags[0] = 1;
      const uint32_t pending = g < C::kStages ? g : C::kStages;
      for (uint32_t k = 1; k <= pending; ++k) {
        const uint32_t gg = g - k;
        volatile int never = 0;
        (void)wait_bounded(&full[gg % C::kStages], (gg / C::kStages) & 1u, &never);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  uint32_t g = 0;
  bool aborted = false;
  for (int it = it0; it < it1; ++it) {
    const WorkItem wi = items[it];
    const SeqInfo si = seqs[wi.seq];
    if (si.qrows * a.G <= 8)
      decode_item<T, H, 1>(a, wi, si, groups, stages, full, empty, flags, comb, warp, lane, g,
                           aborted);
    else
      decode_item<T, H, 2>(a, wi, si, groups, stages, full, empty, flags, comb, warp, lane, g,
                           aborted);
  }
  if (aborted && lane == 0) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
}

template <typename T, int H>
int launch_t(const CUtensorMap& kmap, const CUtensorMap& vmap, bool per_head_tma,
             const AttnArgs<T>& args, int grid, cudaStream_t stream) {
  using C = DecCfg<H>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(paged_decode_kernel<T, H>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "paged_decode_kernel attribute");
  paged_decode_kernel<T, H><<<grid, kDecThreads, C::kSmem, stream>>>(kmap, vmap, args,
                                                                     per_head_tma ? 1 : 0);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

}  // namespace

int decode_smem_bytes(int heads) {
  switch (heads) {
    case 8: return DecCfg<8>::kSmem;
    case 4: return DecCfg<4>::kSmem;
    case 2: return DecCfg<2>::kSmem;
    default: return DecCfg<1>::kSmem;
  }
}

int decode_launch(int dtype, int heads, const CUtensorMap& kmap, const CUtensorMap& vmap,
                  bool per_head_tma, const void* args, int grid, cudaStream_t stream) {
  if (dtype == FE_DTYPE_BF16) {
    const auto& a = *static_cast<const AttnArgs<__nv_bfloat16>*>(args);
    switch (heads) {
      case 8: return launch_t<__nv_bfloat16, 8>(kmap, vmap, per_head_tma, a, grid, stream);
      case 4: return launch_t<__nv_bfloat16, 4>(kmap, vmap, per_head_tma, a, grid, stream);
      case 2: return launch_t<__nv_bfloat16, 2>(kmap, vmap, per_head_tma, a, grid, stream);
      default: return launch_t<__nv_bfloat16, 1>(kmap, vmap, per_head_tma, a, grid, stream);
    }
  }
  const auto& a = *static_cast<const AttnArgs<__half>*>(args);
  switch (heads) {
    case 8: return launch_t<__half, 8>(kmap, vmap, per_head_tma, a, grid, stream);
    case 4: return launch_t<__half, 4>(kmap, vmap, per_head_tma, a, grid, stream);
    case 2: return launch_t<__half, 2>(kmap, vmap, per_head_tma, a, grid, stream);
    default: return launch_t<__half, 1>(kmap, vmap, per_head_tma, a, grid, stream);
  }
}

}  // namespace fe
