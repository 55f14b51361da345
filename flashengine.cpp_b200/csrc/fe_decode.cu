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
//  * Split-K across CTAs: the pieces of a split unit write partial (O, m, l)
//    records; decode_merge_kernel, launched as a programmatic dependent of
//    this kernel, merges every split unit once the whole grid has finished,
//    so no streaming CTA carries merge work into the tail. (The allocation-free
//    entry point keeps the in-kernel merge: the last piece to arrive merges,
//    atomic ticket, counter re-armed for graph replay.)
//  * Bounded waits as in fe_attn.cu; a CTA that gives up records
//    FE_DEVERR_TIMEOUT and drains its own copies before exiting.
#include <mutex>
#include <string>

#include "fe_attn_common.cuh"

namespace fe {

int decode_launch(int dtype, int dim, int heads, const CUtensorMap& kmap, const CUtensorMap& vmap,
                  bool per_head_tma, const void* args, int grid, cudaStream_t stream);
int decode_merge_launch(int dtype, int dim, int list, const void* args, int grid, int grid_rows,
                        cudaStream_t stream, bool pdl);

namespace {

constexpr int kDecWarps = 8;
constexpr int kDecThreads = (kDecWarps + 1) * 32;

// H KV heads of D dims per item. head_dim 128: the 8/H warps of a head merge
// through kDecWarps 16-row slots. head_dim 256 (H <= 2): a tile is 8 KiB per
// head for K and for V, so stages hold 1-2 heads; warps are grouped per (head,
// 8-column half) and merge pairwise in log2 rounds through kDecWarps/2 slots
// of 8 rows.
//
// The warps sharing a head take tiles j, j + w, j + 2w, ... (w warps); the
// stage count is a multiple of w, so the tile that last used a warp's stage is
// that warp's own earlier tile: a warp never waits on a stage's full barrier
// while the phase before the one it wants is still pending (the parity test
// would pass a phase early). Items end with a merge barrier of all consumer
// warps, so this holds across items too.
template <int H, int D = kHeadDim>
struct DecCfg {
  static constexpr int kQ = D / 64;          // 64-dim boxes per head
  static constexpr int kWh = kDecWarps / H;  // warps per head (most per group)
  static constexpr int kKBytes = kQ * H * kHalfBytes;
  static constexpr int kStageBytes = 2 * kKBytes;
  static constexpr int kStages = D == kHeadDim ? (H == 8 ? 3 : (H == 4 ? 4 : 8)) : (H == 2 ? 4 : 8);
  static_assert(kStages % kWh == 0 || kWh == 1, "stage count must be a multiple of the warps per head");
  static constexpr int kCombBytes =
      D == kHeadDim ? (kWh > 1 ? kDecWarps * kRowBlock * kCombStride * 4 : 0)
                    : (kDecWarps / 2) * 8 * (D + 4) * 4;
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

template <typename T, int H, int NT, bool kInlineMerge>
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
    t.k = base + (2 * hh) * kHalfBytes;
    t.v = t.k + C::kKBytes;
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

  if (kInlineMerge && wi.group >= 0) {
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

// head_dim 256: warp w serves group w % (H*C) = (head hh, column half ch),
// C = 2 when the item has more than 8 packed rows; the kWh = 8/(H*C) warps of
// a group take alternate tiles, then fold their states pairwise (round `step`:
// warps step..2*step-1 of the group stash, warps 0..step-1 absorb), so the
// group's first warp ends with the item's whole key range.
template <typename T, int H>
__device__ __forceinline__ void decode_item_d256(const AttnArgs<T>& a, const WorkItem& wi,
                                                 const SeqInfo& si, uint8_t* stages,
                                                 uint64_t* full, uint64_t* empty,
                                                 volatile int* flags, float* comb, int w, int lane,
                                                 uint32_t& g, bool& aborted) {
  constexpr int D = kWideHeadDim;
  using C = DecCfg<H, D>;
  const int G = a.G;
  const int P = si.qrows * G;
  const int halves = P > 8 ? 2 : 1;
  const int groups = H * halves;
  const int kwh = kDecWarps / groups;
  const int grp = w % groups, sub = w / groups;
  const int hh = grp % H, ch = grp / H;
  const int head0 = (wi.kvh + hh) * G;
  const bool causal = a.view == 1;
  KeyState<T, 1, D> ks;
  ks.init(a.q, a.hq, si.q_row0, si.qrows, si.length, head0, G, causal, lane, ch * 8);

  const int ntiles = wi.kt1 - wi.kt0;
  for (int jt = sub; jt < ntiles; jt += kwh) {
    const uint32_t gg = g + jt;
    const int s = gg % C::kStages;
    if (aborted || flags[0] || !wait_bounded(&full[s], (gg / C::kStages) & 1u, flags)) {
      aborted = true;
      break;
    }
    const uint32_t base = smem_u32(stages + s * C::kStageBytes);
    TileAddr t;
    t.k = base + (C::kQ * hh) * kHalfBytes;
    t.v = t.k + C::kKBytes;
    ks.tile(t, (wi.kt0 + jt) * kTileTokens, si.length, a.scale_log2, lane);
    __syncwarp();
    if (lane == 0) mbar_arrive_cnt(&empty[s], kwh);
  }
  g += ntiles;
  ks.reduce_l();

  constexpr int kSlot = 8 * (D + 4);  // floats per stash slot (8 columns)
  for (int step = kwh >> 1; step >= 1; step >>= 1) {
    if (sub >= step && sub < 2 * step) ks.stash(comb + ((sub - step) * groups + grp) * kSlot, lane);
    named_barrier_sync(1, kDecWarps * 32);
    if (sub < step) ks.absorb(comb + (sub * groups + grp) * kSlot, lane);
    named_barrier_sync(1, kDecWarps * 32);
  }
  if (sub != 0 || aborted) return;

  const int r8 = lane >> 2, cq = lane & 3;
  const int R = H * P;  // rows of the item's record: head-major, then packed row
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int p = ch * 8 + 2 * cq + e;
    if (p >= P) continue;
    if (wi.group < 0) {
      const float inv = 1.f / ks.l[0][e];
      T* dst = a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + head0 + p % G) * D;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        dst[16 * mt + r8] = to_elem<T>(ks.o[0][mt][e] * inv);
        dst[16 * mt + r8 + 8] = to_elem<T>(ks.o[0][mt][2 + e] * inv);
      }
    } else {
      float* rec = a.partials + wi.part;
      float* row = rec + (hh * P + p) * D;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        row[16 * mt + r8] = ks.o[0][mt][e];
        row[16 * mt + r8 + 8] = ks.o[0][mt][2 + e];
      }
      if (r8 == 0) {
        rec[R * D + hh * P + p] = ks.m[0][e];
        rec[R * (D + 1) + hh * P + p] = ks.l[0][e];
      }
    }
  }
}

template <typename T, int H, int D>
__global__ void __launch_bounds__(kDecThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const AttnArgs<T> a,
                        int per_head_tma) {
  using C = DecCfg<H, D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* comb = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + C::kStages);

  // the merge kernel may be scheduled now; it waits for this grid's completion
  pdl_trigger();
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
    // Slots of 32 tiles are fetched per batch (one per lane); the next batch
    // is requested before the current one is consumed.
    auto tile_slot = [&](const WorkItem& w, const SeqInfo& si, int j) -> int {
      if (j >= w.kt1) return 0;
      const int t0 = j * kTileTokens;
      return __ldg(pages + si.page_off + t0 / a.page) * a.page + (t0 % a.page);
    };
    // The work list and page ids are the plan's metadata, copied in by the
    // prepare before the previous kernel started: the first item's page ids
    // are fetched before waiting for that kernel, which owns the pools
    // (a no-op wait when launched without programmatic serialization).
    const int first_slot = tile_slot(items[it0], seqs[items[it0].seq], items[it0].kt0 + lane);
    pdl_wait();
    uint32_t g = 0;
    bool ok = true;
    for (int it = it0; it < it1 && ok; ++it) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int hh0 = w.kvh * C::kQ;  // first 64-dim box of the item's heads
      int nxt = it == it0 ? first_slot : tile_slot(w, si, w.kt0 + lane);
      for (int j0 = w.kt0; j0 < w.kt1 && ok; j0 += 32) {
        const int n = min(32, w.kt1 - j0);
        const int slot0 = nxt;
        nxt = tile_slot(w, si, j0 + 32 + lane);
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
                for (int x = 0; x < C::kQ * H; ++x) {
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
  // q and the split workspace belong to earlier kernels until here
  pdl_wait();
  uint32_t g = 0;
  bool aborted = false;
  for (int it = it0; it < it1; ++it) {
    const WorkItem wi = items[it];
    const SeqInfo si = seqs[wi.seq];
    if constexpr (D != kHeadDim)
      decode_item_d256<T, H>(a, wi, si, stages, full, empty, flags, comb, warp, lane, g, aborted);
    else if (si.qrows * a.G <= 8)
      decode_item<T, H, 1, false>(a, wi, si, groups, stages, full, empty, flags, comb, warp, lane,
                                  g, aborted);
    else
      decode_item<T, H, 2, false>(a, wi, si, groups, stages, full, empty, flags, comb, warp, lane,
                                  g, aborted);
  }
  if (aborted && lane == 0) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
}

template <typename T, int H, int D = kHeadDim>
int launch_t(const CUtensorMap& kmap, const CUtensorMap& vmap, bool per_head_tma,
             const AttnArgs<T>& args, int grid, cudaStream_t stream) {
  using C = DecCfg<H, D>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(paged_decode_kernel<T, H, D>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "paged_decode_kernel attribute");
  FE_CUDA_TRY(launch_pdl(paged_decode_kernel<T, H, D>, dim3(grid), dim3(kDecThreads), C::kSmem,
                         stream, kmap, vmap, args, per_head_tma ? 1 : 0));
  return FE_OK;
}

// Merge the partial records of every split unit of a work list (the decode
// list, or a head_dim 256 row list): gridDim.x CTAs stride over the units
// (fewer than units under graph replay, where the grid is fixed and the unit
// count comes from the metadata), gridDim.y CTAs share a unit's rows, one
// warp per merged row, so all rows of a unit are in flight at once. A row's
// loads are issued together (the split records' O vectors four at a time, m
// and l one split per lane), so a row costs about one L2 round trip.
// Launched with programmatic stream serialization after the kernel that
// wrote the records: its CTAs become resident on the SMs that grid's early
// finishers free and start when that grid has completed.
constexpr int kMergeThreads = 1024;

// Records of a D-dim split unit: O[rows][D] unnormalised, then m[rows], l[rows].
template <typename T, int D>
__device__ __forceinline__ void merge_row_warp(const float* partials, const SplitGroup& gi, int r,
                                               int lane, T* out_row) {
  constexpr int kV = D / 128;  // float4 vectors per lane
  const int ns = gi.nsplit;
  float4 acc[kV];
#pragma unroll
  for (int v = 0; v < kV; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
  // head_dim 256 with two splits (the usual case there): both splits' O
  // vectors are loaded together with the (m, l) pairs, one L2 round trip for
  // the row, then weighted in the order of the general path below (same
  // arithmetic, same bits). Measured +2% on a head_dim 256 decode step; for
  // head_dim 128 the same preload (up to four splits) measured 0.5% slower,
  // so there the general path runs.
  constexpr int kPre = 2;  // also the register budget of 1024-thread CTAs
  if (D != kHeadDim && ns <= kPre) {
    float m = -INFINITY, l = 0.f;
    if (lane < ns) {
      const float* rec = partials + gi.part0 + static_cast<int64_t>(lane) * gi.rec_floats;
      m = __ldcg(rec + gi.rows * D + r);
      l = __ldcg(rec + gi.rows * (D + 1) + r);
    }
    float4 x[kPre][kV];
#pragma unroll
    for (int j = 0; j < kPre; ++j)
      if (j < ns) {
        const float* rec = partials + gi.part0 + static_cast<int64_t>(j) * gi.rec_floats;
#pragma unroll
        for (int v = 0; v < kV; ++v)
          x[j][v] = __ldcg(reinterpret_cast<const float4*>(rec + r * D + v * 128 + lane * 4));
      }
    float mc = m;
#pragma unroll
    for (int o = 16; o; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
    const float base = mc == -INFINITY ? 0.f : mc;
    const float sc = lane < ns ? fast_exp2(m - base) : 0.f;
    float lw = l * sc;
#pragma unroll
    for (int o = 16; o; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
#pragma unroll
    for (int j = 0; j < kPre; ++j)
      if (j < ns) {
        const float w = __shfl_sync(0xffffffffu, sc, j);
#pragma unroll
        for (int v = 0; v < kV; ++v) {
          acc[v].x = fmaf(x[j][v].x, w, acc[v].x);
          acc[v].y = fmaf(x[j][v].y, w, acc[v].y);
          acc[v].z = fmaf(x[j][v].z, w, acc[v].z);
          acc[v].w = fmaf(x[j][v].w, w, acc[v].w);
        }
      }
    const float inv = 1.f / lw;
#pragma unroll
    for (int v = 0; v < kV; ++v)
      store4<T>(out_row + v * 128 + lane * 4, acc[v].x * inv, acc[v].y * inv, acc[v].z * inv,
                acc[v].w * inv);
    return;
  }
  float M = -INFINITY, L = 0.f;
  for (int s0 = 0; s0 < ns; s0 += 32) {
    // this chunk's maxima and sums: split s0 + lane per lane
    const int sl = s0 + lane;
    float m = -INFINITY, l = 0.f;
    if (sl < ns) {
      const float* rec = partials + gi.part0 + static_cast<int64_t>(sl) * gi.rec_floats;
      m = __ldcg(rec + gi.rows * D + r);
      l = __ldcg(rec + gi.rows * (D + 1) + r);
    }
    float mc = m;
#pragma unroll
    for (int o = 16; o; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
    const float M_new = fmaxf(M, mc);
    const float base = M_new == -INFINITY ? 0.f : M_new;
    // rescale what the earlier chunks accumulated
    const float resc = M == -INFINITY ? 0.f : fast_exp2(M - base);
#pragma unroll
    for (int v = 0; v < kV; ++v) {
      acc[v].x *= resc;
      acc[v].y *= resc;
      acc[v].z *= resc;
      acc[v].w *= resc;
    }
    L *= resc;
    M = M_new;
    const float sc = sl < ns ? fast_exp2(m - base) : 0.f;
    float lw = l * sc;
#pragma unroll
    for (int o = 16; o; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    L += lw;
    const int n = min(32, ns - s0);
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
      const float* rec = partials + gi.part0 + static_cast<int64_t>(s0 + j) * gi.rec_floats;
      const float w = __shfl_sync(0xffffffffu, sc, j);
#pragma unroll
      for (int v = 0; v < kV; ++v) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(rec + r * D + v * 128 + lane * 4));
        acc[v].x = fmaf(x.x, w, acc[v].x);
        acc[v].y = fmaf(x.y, w, acc[v].y);
        acc[v].z = fmaf(x.z, w, acc[v].z);
        acc[v].w = fmaf(x.w, w, acc[v].w);
      }
    }
  }
  const float inv = 1.f / L;
#pragma unroll
  for (int v = 0; v < kV; ++v)
    store4<T>(out_row + v * 128 + lane * 4, acc[v].x * inv, acc[v].y * inv, acc[v].z * inv,
              acc[v].w * inv);
}

template <typename T, int D>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_kernel(const AttnArgs<T> a,
                                                                     int list) {
  pdl_trigger();
  // The plan's metadata was complete before the kernel ahead of this one
  // started (the kernel that wrote the records read it from its first
  // instruction on), so the CTA's first unit is read before the wait; only
  // the records need that kernel's completion.
  const MetaHeader* hdr = reinterpret_cast<const MetaHeader*>(a.meta);
  const int n = hdr->n_groups[list];
  const SplitGroup* groups = reinterpret_cast<const SplitGroup*>(a.meta + hdr->groups_off[list]);
  const SeqInfo* seqs = reinterpret_cast<const SeqInfo*>(a.meta + hdr->seqs_off);
  SplitGroup first{};
  SeqInfo first_seq{};
  if (static_cast<int>(blockIdx.x) < n) {
    first = groups[blockIdx.x];
    if (first.nsplit >= 2) first_seq = seqs[first.seq];
  }
  pdl_wait();
  const int G = a.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int gidx = blockIdx.x; gidx < n; gidx += gridDim.x) {
    const bool head = gidx == static_cast<int>(blockIdx.x);
    const SplitGroup gi = head ? first : groups[gidx];
    if (gi.nsplit < 2) continue;  // placeholder ids of the row lists
    const SeqInfo si = head ? first_seq : seqs[gi.seq];
    const int rph = gi.rows_per_head > 0 ? gi.rows_per_head : si.qrows * G;
    for (int r = warp + blockIdx.y * (kMergeThreads / 32); r < gi.rows;
         r += gridDim.y * (kMergeThreads / 32)) {
      const int rh = r / rph, p = gi.row0 + r % rph;
      T* dst = a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + (gi.kvh + rh) * G +
                        p % G) * D;
      merge_row_warp<T, D>(a.partials, gi, r, lane, dst);
    }
  }
}

template <typename T>
int launch_merge_t(const AttnArgs<T>& args, int dim, int list, dim3 grid, cudaStream_t stream,
                   bool pdl) {
  auto kernel = dim == kWideHeadDim ? decode_merge_kernel<T, kWideHeadDim>
                                    : decode_merge_kernel<T, kHeadDim>;
  if (pdl) {
    FE_CUDA_TRY(launch_pdl(kernel, grid, dim3(kMergeThreads), 0, stream, args, list));
  } else {
    kernel<<<grid, kMergeThreads, 0, stream>>>(args, list);
    FE_CUDA_TRY(cudaGetLastError());
  }
  return FE_OK;
}

}  // namespace

// grid: CTAs over the list's split units (strided); grid_rows: CTAs per
// unit, each taking 32 of its record rows (one per warp), strided. With
// `pdl` the merge is a programmatic dependent of the kernel before it (its
// CTAs become resident on SMs that grid frees and wait for its completion);
// without, it starts once that grid has completed, so it takes no SM from a
// kernel running beside the decode kernel.
int decode_merge_launch(int dtype, int dim, int list, const void* args, int grid, int grid_rows,
                        cudaStream_t stream, bool pdl) {
  if (grid <= 0) return FE_OK;
  const dim3 g(grid, grid_rows > 0 ? grid_rows : 1);
  if (dtype == FE_DTYPE_BF16)
    return launch_merge_t(*static_cast<const AttnArgs<__nv_bfloat16>*>(args), dim, list, g,
                          stream, pdl);
  return launch_merge_t(*static_cast<const AttnArgs<__half>*>(args), dim, list, g, stream, pdl);
}

int decode_launch(int dtype, int dim, int heads, const CUtensorMap& kmap, const CUtensorMap& vmap,
                  bool per_head_tma, const void* args, int grid, cudaStream_t stream) {
  if (dtype == FE_DTYPE_BF16) {
    const auto& a = *static_cast<const AttnArgs<__nv_bfloat16>*>(args);
    if (dim == kWideHeadDim)
      return heads == 2
                 ? launch_t<__nv_bfloat16, 2, kWideHeadDim>(kmap, vmap, per_head_tma, a, grid, stream)
                 : launch_t<__nv_bfloat16, 1, kWideHeadDim>(kmap, vmap, per_head_tma, a, grid, stream);
    switch (heads) {
      case 8: return launch_t<__nv_bfloat16, 8>(kmap, vmap, per_head_tma, a, grid, stream);
      case 4: return launch_t<__nv_bfloat16, 4>(kmap, vmap, per_head_tma, a, grid, stream);
      case 2: return launch_t<__nv_bfloat16, 2>(kmap, vmap, per_head_tma, a, grid, stream);
      default: return launch_t<__nv_bfloat16, 1>(kmap, vmap, per_head_tma, a, grid, stream);
    }
  }
  const auto& a = *static_cast<const AttnArgs<__half>*>(args);
  if (dim == kWideHeadDim)
    return heads == 2 ? launch_t<__half, 2, kWideHeadDim>(kmap, vmap, per_head_tma, a, grid, stream)
                      : launch_t<__half, 1, kWideHeadDim>(kmap, vmap, per_head_tma, a, grid, stream);
  switch (heads) {
    case 8: return launch_t<__half, 8>(kmap, vmap, per_head_tma, a, grid, stream);
    case 4: return launch_t<__half, 4>(kmap, vmap, per_head_tma, a, grid, stream);
    case 2: return launch_t<__half, 2>(kmap, vmap, per_head_tma, a, grid, stream);
    default: return launch_t<__half, 1>(kmap, vmap, per_head_tma, a, grid, stream);
  }
}

}  // namespace fe

// ===========================================================================
// Allocation-free decode entry point (fe_paged_decode_noalloc, fe_kv.h).
//
// For callers that cannot allocate device memory where they run attention:
// hosts that hand all of HBM to their own pool allocator at start-up (as a
// KV-cache engine sized by a memory-utilisation fraction does), so that a
// later cudaMalloc fails, and hot loops in which an allocation, which may
// synchronise the device, is not allowed. The plan-based entry points
// allocate their work lists and split-K workspace in fe_attn_plan_create;
// this one needs neither: its work split is computed on the device from the
// caller's metadata, and its split-K scratch is the file-scope array below.
// head_dim 128 only: q and out are [batch, hq, 128].
//
// When batch x KV-head groups is so large that even two split records per
// unit would not fit the array, every unit runs unsplit (one CTA per unit,
// no records): the results are the same, long contexts just get less
// parallelism.
//
// The array is fixed at kNoAllocScratchBytes (16 MiB of fp32 split records +
// 64 KiB of split counters) and exists on every GPU that loads this library
// until the process exits. Every call shares it and it keeps the last call's
// contents: the counters are cleared by each call (cudaMemsetAsync, no
// allocation) and every record is written before it is read, so sequential
// calls are safe, but calls that overlap on the GPU (other streams, other
// host threads) race on it.
// ===========================================================================
namespace fe {
namespace {

constexpr size_t kNoAllocPartialBytes = size_t(16) << 20;
constexpr int kNoAllocCounters = 16384;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocPartialBytes + sizeof(int32_t) * size_t(kNoAllocCounters);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

template <typename T, int H>
__global__ void __launch_bounds__(kDecThreads, 1)
    paged_decode_noalloc_kernel(const __grid_constant__ CUtensorMap kmap,
                                const __grid_constant__ CUtensorMap vmap, const AttnArgs<T> a0,
                                const int32_t* __restrict__ kv, const int32_t* __restrict__ pages,
                                const int32_t* __restrict__ last, int groups_per_seq, int nsplit,
                                int max_pages, int num_blocks, int rec_floats, int per_head_tma) {
  using C = DecCfg<H>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ SplitGroup sg;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* comb = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + C::kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, grp = blockIdx.y, s = blockIdx.x;
  // the metadata, q, the pools and the split scratch belong to earlier
  // kernels until here (a no-op when launched without programmatic
  // serialization, as fe_paged_decode_noalloc launches it)
  pdl_wait();
  const int p0 = __ldg(kv + b), p1 = __ldg(kv + b + 1), ln = __ldg(last + b);
  if (p1 <= p0 || p1 - p0 > max_pages || ln < 1 || ln > a0.page) {
    if (threadIdx.x == 0 && s == 0 && grp == 0) raise_device_error(a0.err, FE_DEVERR_PAGE_RANGE);
    return;
  }
  const int length = (p1 - p0 - 1) * a0.page + ln;
  const int tiles = (length + kTileTokens - 1) / kTileTokens;
  const int unit = b * groups_per_seq + grp;
  WorkItem wi;
  wi.seq = b;
  wi.kvh = static_cast<int16_t>(grp * H);
  wi.key_mode = 1;
  wi.rb0 = 0;
  wi.nrb = 1;
  wi.kt0 = static_cast<int>(int64_t(tiles) * s / nsplit);
  wi.kt1 = static_cast<int>(int64_t(tiles) * (s + 1) / nsplit);
  wi.part = nsplit > 1 ? (unit * nsplit + s) * rec_floats : -1;
  wi.group = nsplit > 1 ? 0 : -1;  // counters below are offset to this unit
  SeqInfo si;
  si.q_row0 = b;
  si.qrows = 1;
  si.length = length;
  si.page_off = p0;
  AttnArgs<T> a = a0;
  a.counters = a0.counters + unit;

  if (threadIdx.x == 0) {
    sg.nsplit = nsplit;
    sg.part0 = unit * nsplit * rec_floats;
    sg.rec_floats = rec_floats;
    sg.rows = H * a0.G;
    for (int st = 0; st < C::kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kDecWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecWarps) {
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    uint32_t g = 0;
    bool ok = true;
    const int hh0 = wi.kvh * 2;
    for (int j0 = wi.kt0; j0 < wi.kt1 && ok; j0 += 32) {
      const int n = min(32, wi.kt1 - j0);
      int slot0 = 0;
      if (lane < n) {
        const int t0 = (j0 + lane) * kTileTokens;
        int pid = __ldg(pages + p0 + t0 / a.page);
        if (pid < 0 || pid > num_blocks) {
          raise_device_error(a.err, FE_DEVERR_PAGE_RANGE);
          pid = num_blocks;  // read the padding page instead
        }
        slot0 = pid * a.page + (t0 % a.page);
      }
      for (int jj = 0; jj < n; ++jj) {
        const int s0 = __shfl_sync(0xffffffffu, slot0, jj);
        const int st = g % C::kStages;
        const uint32_t ph = (g / C::kStages) & 1u;
        int good = 1;
        if (lane == 0) {
          if (flags[0] || !wait_bounded(&empty[st], ph ^ 1u, flags)) {
            good = 0;
          } else {
            mbar_arrive_expect_tx(&full[st], C::kStageBytes);
            uint8_t* dst = stages + st * C::kStageBytes;
            if (!per_head_tma) {
              tma_load_3d(dst, &kmap, &full[st], 0, s0, hh0);
              tma_load_3d(dst + C::kKBytes, &vmap, &full[st], 0, s0, hh0);
            } else {
              for (int x = 0; x < 2 * H; ++x) {
                tma_load_3d(dst + x * kHalfBytes, &kmap, &full[st], 0, hh0 + x, s0);
                tma_load_3d(dst + C::kKBytes + x * kHalfBytes, &vmap, &full[st], 0, hh0 + x, s0);
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

  uint32_t g = 0;
  bool aborted = false;
  if (a.G <= 8)
    decode_item<T, H, 1, true>(a, wi, si, &sg, stages, full, empty, flags, comb, warp, lane, g,
                               aborted);
  else
    decode_item<T, H, 2, true>(a, wi, si, &sg, stages, full, empty, flags, comb, warp, lane, g,
                               aborted);
  if (aborted && lane == 0) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
}

using NoAllocEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                     const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                     const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Per-device set-up of the allocation-free path: the device address of the
// scratch array (the host-side symbol is only a stand-in) and the kernels'
// shared-memory attribute. Done by the first call on each device.
struct NoAllocDevice {
  unsigned char* scratch = nullptr;
  bool attr_set[2][4] = {};
  int sms = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

template <typename T, int H>
int noalloc_launch(NoAllocDevice& d, int ti, const CUtensorMap& km, const CUtensorMap& vm,
                   const AttnArgs<T>& a, const int32_t* kv, const int32_t* pages,
                   const int32_t* last, int batch, int groups, int nsplit, int max_pages,
                   int num_blocks, int rec, bool per_head, cudaStream_t stream) {
  using C = DecCfg<H>;
  const int hi = H == 8 ? 3 : H == 4 ? 2 : H == 2 ? 1 : 0;
  if (!d.attr_set[ti][hi]) {
    FE_CUDA_TRY(cudaFuncSetAttribute(paged_decode_noalloc_kernel<T, H>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    d.attr_set[ti][hi] = true;
  }
  dim3 grid(nsplit, groups, batch);
  paged_decode_noalloc_kernel<T, H><<<grid, kDecThreads, C::kSmem, stream>>>(
      km, vm, a, kv, pages, last, groups, nsplit, max_pages, num_blocks, rec, per_head ? 1 : 0);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

template <typename T>
int noalloc_dispatch(NoAllocDevice& d, int ti, int H, const CUtensorMap& km,
                     const CUtensorMap& vm, const AttnArgs<T>& a, const int32_t* kv,
                     const int32_t* pages, const int32_t* last, int batch, int groups, int nsplit,
                     int max_pages, int num_blocks, int rec, bool per_head, cudaStream_t s) {
  switch (H) {
    case 8: return noalloc_launch<T, 8>(d, ti, km, vm, a, kv, pages, last, batch, groups, nsplit,
                                        max_pages, num_blocks, rec, per_head, s);
    case 4: return noalloc_launch<T, 4>(d, ti, km, vm, a, kv, pages, last, batch, groups, nsplit,
                                        max_pages, num_blocks, rec, per_head, s);
    case 2: return noalloc_launch<T, 2>(d, ti, km, vm, a, kv, pages, last, batch, groups, nsplit,
                                        max_pages, num_blocks, rec, per_head, s);
    default: return noalloc_launch<T, 1>(d, ti, km, vm, a, kv, pages, last, batch, groups, nsplit,
                                         max_pages, num_blocks, rec, per_head, s);
  }
}

}  // namespace
}  // namespace fe

extern "C" int fe_paged_decode_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                       void* out, const int32_t* kv, const int32_t* pages,
                                       const int32_t* last, int batch, int hq, int hkv, int page,
                                       int num_blocks, int max_pages, int dtype, void* stream) {
  using namespace fe;
  if (dtype != FE_DTYPE_F16 && dtype != FE_DTYPE_BF16)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_paged_decode_noalloc: bad dtype");
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0 || hq / hkv > kRowBlock)
    return fail(FE_ERR_UNSUPPORTED, "fe_paged_decode_noalloc: need hq % hkv == 0, hq/hkv <= 16");
  if (page <= 0 || page % kTileTokens != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_paged_decode_noalloc: page must be a multiple of 16");
  if (batch < 0 || num_blocks <= 0 || max_pages <= 0 || batch > 65535 ||
      int64_t(num_blocks + 1) * page >= INT32_MAX)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_paged_decode_noalloc: bad sizes");
  if (batch == 0) return FE_OK;
  if (!q || !k_pool || !v_pool || !out || !kv || !pages || !last)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_paged_decode_noalloc: null pointer");
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_paged_decode_noalloc: buffers must be 16-byte aligned");
  const int G = hq / hkv;
  int H = 8;
  while (hkv % H) H >>= 1;
  const int groups = hkv / H;
  const int units = batch * groups;
  const int rec = partial_rec_floats(H * G);
  const size_t unit_bytes = sizeof(float) * size_t(rec);
  // One split counter per unit. When the units' split records would not fit
  // the scratch even twice over, every unit runs unsplit (nsplit = 1 below),
  // which needs neither records nor counters.
  if (units > kNoAllocCounters)
    return fail(FE_ERR_CAPACITY, "fe_paged_decode_noalloc: batch x KV-head groups exceeds " +
                                     std::to_string(kNoAllocCounters));

  int dev = 0;
  FE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FE_ERR_NO_DEVICE, "fe_paged_decode_noalloc: device id");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.scratch) {
    int major = 0;
    FE_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10)
      return fail(FE_ERR_NO_DEVICE, "fe_paged_decode_noalloc: needs an sm_100 (B200) device");
    FE_CUDA_TRY(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    void* p = nullptr;
    FE_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    d.scratch = static_cast<unsigned char*>(p);
  }
  float* partials = reinterpret_cast<float*>(d.scratch);
  int32_t* counters = reinterpret_cast<int32_t*>(d.scratch + kNoAllocPartialBytes);

  // Splits per (sequence, head group): enough CTAs for about two per SM,
  // at least 8 key tiles each, and no more records than the scratch holds.
  const int64_t max_tiles = (int64_t(max_pages) * page + kTileTokens - 1) / kTileTokens;
  int nsplit = static_cast<int>((2 * int64_t(d.sms) + units - 1) / units);
  nsplit = static_cast<int>(std::min<int64_t>(nsplit, std::max<int64_t>(1, max_tiles / 8)));
  nsplit = static_cast<int>(std::min<size_t>(nsplit, kNoAllocPartialBytes / (size_t(units) * unit_bytes)));
  if (nsplit > 65535) nsplit = 65535;
  if (nsplit < 1) nsplit = 1;

  auto s = static_cast<cudaStream_t>(stream);
  if (nsplit > 1) FE_CUDA_TRY(cudaMemsetAsync(counters, 0, sizeof(int32_t) * units, s));

  // Tensor maps (host-side encoding only).
  static NoAllocEncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) !=
            cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
      return fail(FE_ERR_CUDA, "fe_paged_decode_noalloc: cuTensorMapEncodeTiled unavailable");
    encode = reinterpret_cast<NoAllocEncodeFn>(fn);
  }
  const cuuint64_t cache_slots = cuuint64_t(num_blocks + 1) * page;
  const CUtensorMapDataType et =
      dtype == FE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap km, vm;
  bool per_head = false;
  {
    const cuuint64_t dims[3] = {64, cache_slots, cuuint64_t(hkv) * 2};
    const cuuint64_t strides[2] = {cuuint64_t(hkv) * 256, 128};
    const cuuint32_t box[3] = {64, kTileTokens, cuuint32_t(2 * H)};
    CUresult r1 = encode(&km, et, 3, const_cast<void*>(k_pool), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = encode(&vm, et, 3, const_cast<void*>(v_pool), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    per_head = r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS;
  }
  if (per_head) {
    const cuuint64_t dims[3] = {64, cuuint64_t(hkv) * 2, cache_slots};
    const cuuint64_t strides[2] = {128, cuuint64_t(hkv) * 256};
    const cuuint32_t box[3] = {64, 1, kTileTokens};
    if (encode(&km, et, 3, const_cast<void*>(k_pool), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        encode(&vm, et, 3, const_cast<void*>(v_pool), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(FE_ERR_CUDA, "fe_paged_decode_noalloc: tensor map encoding failed");
  }

  const float scale_log2 = 1.4426950408889634f / sqrtf(float(kHeadDim));
  if (dtype == FE_DTYPE_BF16) {
    AttnArgs<__nv_bfloat16> a{nullptr, static_cast<const __nv_bfloat16*>(q),
                              static_cast<__nv_bfloat16*>(out), partials, counters,
                              device_error_word(), hq, G, page, 1, scale_log2};
    return noalloc_dispatch<__nv_bfloat16>(d, 1, H, km, vm, a, kv, pages, last, batch, groups,
                                           nsplit, max_pages, num_blocks, rec, per_head, s);
  }
  AttnArgs<__half> a{nullptr, static_cast<const __half*>(q), static_cast<__half*>(out), partials,
                     counters, device_error_word(), hq, G, page, 1, scale_log2};
  return noalloc_dispatch<__half>(d, 0, H, km, vm, a, kv, pages, last, batch, groups, nsplit,
                                  max_pages, num_blocks, rec, per_head, s);
}
