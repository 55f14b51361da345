// Paged chunked-prefill / speculative-verify attention on the 5th-generation
// tensor cores (tcgen05, TMEM) for sm_100a.
//
// Reference behaviour: Cambridgebit/FlashEngine.cpp src/flashinfer_attention.cu:35-44
// (multi-row requests of the FlashInfer paged prefill kernel; causal = the
// bottom-right mask, or none for DFlash block verify) with the arithmetic of
// src/portable_gpu_ops.cpp:39-44.
//
// One persistent CTA per SM, six warps:
//  warp 0   producer: gathers each 64-key tile (four 16-token page pieces) of
//           one KV head with TMA into a 3-stage ring (K and V, 2 x 16 KiB).
//  warp 1   MMA issuer (one thread) and TMEM owner:
//             S  = Q K^T  (M = 128 packed rows, N = 64 keys, K = 128 dims)
//                         into one of two TMEM S buffers;
//             O += P V    (M = 128, N = 128 dims, K = 64 keys) into TMEM,
//                         P as a 16-bit high part plus its residual (two MMAs)
//                         so P keeps ~16 significant bits.
//  warps 2-5  softmax + epilogue, one thread per packed row (TMEM lane): read S
//           from TMEM, mask, base-2 online softmax with a lazy rescale (O in
//           TMEM is rescaled only when the row max grows by more than 2^8),
//           write P (128-byte swizzled, K-major) for the next MMA, and at the
//           end read O, divide by l and store the 16-bit output.
// Packed row p of a work item is query row p / G, head kvh*G + p % G.
// All cross-warp hand-offs are mbarriers; every wait is bounded.
#include <mutex>

#include "fe_attn_common.cuh"
#include "fe_tcgen05.cuh"

namespace fe {

int prefill_tc_launch(int dtype, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const void* args, int grid, cudaStream_t stream);
int prefill_tc_smem_bytes();

namespace {

constexpr int kTcM = 128;               // packed rows per work item
constexpr int kTcN = 64;                // keys per tile
constexpr int kTcStages = 3;
constexpr int kTcThreads = 6 * 32;
constexpr int kQHalf = kTcM * 128;      // 16 KiB: 128 rows x 64 dims
constexpr int kKVHalf = kTcN * 128;     // 8 KiB: 64 keys x 64 dims
constexpr int kKVStage = 4 * kKVHalf;   // K lo, K hi, V lo, V hi
constexpr int kPMat = kTcM * 128;       // 16 KiB: 128 rows x 64 keys
constexpr int kPBuf = 2 * kPMat;        // high part + residual
constexpr int kOffQ = 0;
constexpr int kOffKV = 2 * kQHalf;
constexpr int kOffP = kOffKV + kTcStages * kKVStage;
constexpr int kOffBar = kOffP + 2 * kPBuf;
constexpr int kNumBars = 2 + 2 * kTcStages + 8;
constexpr int kTcSmem = 1024 + kOffBar + kNumBars * 8 + 32;
constexpr uint32_t kTmemCols = 256;     // S0 [0,64) S1 [64,128) O [128,256)
constexpr float kRescaleThreshold = 8.f;

template <typename T>
struct Fmt;
template <>
struct Fmt<__half> {
  static constexpr int v = 0;
};
template <>
struct Fmt<__nv_bfloat16> {
  static constexpr int v = 1;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* flags,
                                              bool& aborted) {
  if (aborted) return false;
  if (flags[0] || !wait_bounded(bar, parity, flags)) aborted = true;
  return !aborted;
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const AttnArgs<T> a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* o_free = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + kTcStages;
  uint64_t* s_full = kv_empty + kTcStages;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MetaHeader* hdr = reinterpret_cast<const MetaHeader*>(a.meta);
  const int view = a.view;
  if (static_cast<int>(blockIdx.x) >= hdr->grid[view]) return;
  const int32_t* cta_off = reinterpret_cast<const int32_t*>(a.meta + hdr->cta_off_off[view]);
  const WorkItem* items = reinterpret_cast<const WorkItem*>(a.meta + hdr->items_off[view]);
  const SeqInfo* seqs = reinterpret_cast<const SeqInfo*>(a.meta + hdr->seqs_off);
  const int32_t* pages = reinterpret_cast<const int32_t*>(a.meta + hdr->pages_off);
  const int it0 = cta_off[blockIdx.x], it1 = cta_off[blockIdx.x + 1];
  if (it0 >= it1) return;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 128);
    mbar_init(o_free, 128);
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 128);
      mbar_init(&p_full[b], 128);
      mbar_init(&o_done[b], 1);
    }
    flags[0] = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    uint32_t g = 0;
    for (int it = it0; it < it1 && !aborted; ++it) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int h2 = w.kvh * 2;
      const int n16 = w.kt1 - w.kt0;
      const int ntiles = (n16 + 3) / 4;
      for (int j = 0; j < ntiles && !aborted; ++j, ++g) {
        const int t16 = w.kt0 + 4 * j;
        const int pieces = min(4, w.kt1 - t16);
        int slot0 = 0;
        if (lane < pieces) {
          const int t0 = (t16 + lane) * kTileTokens;
          slot0 = __ldg(pages + si.page_off + t0 / a.page) * a.page + (t0 % a.page);
        }
        const int st = g % kTcStages;
        int good = 1;
        if (lane == 0) {
          if (!wait_or_abort(&kv_empty[st], ((g / kTcStages) & 1u) ^ 1u, flags, aborted)) {
            good = 0;
          } else {
            mbar_arrive_expect_tx(&kv_full[st], pieces * 4 * kHalfBytes);
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          aborted = true;
          break;
        }
        uint8_t* stage = smem + kOffKV + st * kKVStage;
        for (int u = 0; u < pieces; ++u) {
          const int s0 = __shfl_sync(0xffffffffu, slot0, u);
          if (lane == 0) {
            tma_load_3d(stage + u * kHalfBytes, &kmap, &kv_full[st], 0, h2, s0);
            tma_load_3d(stage + kKVHalf + u * kHalfBytes, &kmap, &kv_full[st], 0, h2 + 1, s0);
            tma_load_3d(stage + 2 * kKVHalf + u * kHalfBytes, &vmap, &kv_full[st], 0, h2, s0);
            tma_load_3d(stage + 3 * kKVHalf + u * kHalfBytes, &vmap, &kv_full[st], 0, h2 + 1, s0);
          }
        }
      }
    }
    if (aborted && lane == 0) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16(Fmt<T>::v, false, false, kTcM, kTcN);
      constexpr uint32_t idesc_o = tc::idesc_f16(Fmt<T>::v, false, true, kTcM, kHeadDim);
      const uint32_t q_base = smem_u32(smem + kOffQ);
      uint32_t g = 0;
      int unit = 0;
      auto issue_pv = [&](uint32_t jp, bool first_in_unit) {
        const int pb = jp & 1;
        if (!wait_or_abort(&p_full[pb], (jp >> 1) & 1u, flags, aborted)) return;
        tc::fence_after_sync();
        const int st = jp % kTcStages;
        const uint32_t v_base = smem_u32(smem + kOffKV + st * kKVStage + 2 * kKVHalf);
        const uint32_t p_base = smem_u32(smem + kOffP + pb * kPBuf);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
#pragma unroll
          for (int kk = 0; kk < kTcN / 16; ++kk) {
            const uint64_t ad = tc::smem_desc_sw128(p_base + part * kPMat + kk * 32, 16, 1024);
            const uint64_t bd = tc::smem_desc_sw128(v_base + kk * 2048, kKVHalf, 1024);
            tc::mma_f16(tmem + 128, ad, bd, idesc_o, (first_in_unit && part == 0 && kk == 0) ? 0u : 1u);
          }
        }
        tc::commit(&o_done[pb]);
        tc::commit(&kv_empty[st]);
      };
      for (int it = it0; it < it1 && !aborted; ++it, ++unit) {
        const WorkItem w = items[it];
        const int ntiles = (w.kt1 - w.kt0 + 3) / 4;
        if (!wait_or_abort(q_full, unit & 1, flags, aborted)) break;
        bool o_ready = unit == 0;
        for (int j = 0; j < ntiles && !aborted; ++j) {
          const uint32_t jg = g + j;
          const int st = jg % kTcStages;
          const int sb = jg & 1;
          if (!wait_or_abort(&kv_full[st], (jg / kTcStages) & 1u, flags, aborted)) break;
          if (!wait_or_abort(&s_free[sb], ((jg >> 1) & 1u) ^ 1u, flags, aborted)) break;
          tc::fence_after_sync();
          const uint32_t k_base = smem_u32(smem + kOffKV + st * kKVStage);
#pragma unroll
          for (int kk = 0; kk < kHeadDim / 16; ++kk) {
            const int half = kk >> 2, ko = (kk & 3) * 32;
            const uint64_t ad = tc::smem_desc_sw128(q_base + half * kQHalf + ko, 16, 1024);
            const uint64_t bd = tc::smem_desc_sw128(k_base + half * kKVHalf + ko, 16, 1024);
            tc::mma_f16(tmem + sb * kTcN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          tc::commit(&s_full[sb]);
          if (j > 0) {
            if (!o_ready) {
              if (!wait_or_abort(o_free, (unit - 1) & 1, flags, aborted)) break;
              tc::fence_after_sync();
              o_ready = true;
            }
            issue_pv(jg - 1, j == 1);
          }
        }
        if (aborted) break;
        if (!o_ready) {
          if (!wait_or_abort(o_free, (unit - 1) & 1, flags, aborted)) break;
          tc::fence_after_sync();
        }
        issue_pv(g + ntiles - 1, ntiles == 1);
        g += ntiles;
      }
      if (aborted) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------ softmax / epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // packed row = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const int G = a.G;
    const bool causal = view == 1;
    uint32_t g = 0;
    for (int it = it0; it < it1 && !aborted; ++it) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int ntiles = (w.kt1 - w.kt0 + 3) / 4;
      const int P = si.qrows * G;
      const int p = w.rb0 * kRowBlock + r;
      const bool row_valid = p < P;
      // Q row -> swizzled K-major shared tile (zeros for padding rows)
      {
        const uint4* src = row_valid
                               ? reinterpret_cast<const uint4*>(
                                     a.q + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq +
                                            w.kvh * G + p % G) * kHeadDim)
                               : nullptr;
        uint8_t* qrow = smem + kOffQ + r * 128;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const uint4 v = src ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
          const int half = c >> 3, cc = c & 7;
          *reinterpret_cast<uint4*>(qrow + half * kQHalf + ((cc ^ (r & 7)) << 4)) = v;
        }
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(q_full);

      const int lim = (causal && row_valid) ? si.length - si.qrows + p / G + 1 : si.length;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < ntiles; ++j) {
        const uint32_t jg = g + j;
        const int sb = jg & 1;
        wait_or_abort(&s_full[sb], (jg >> 1) & 1u, flags, aborted);
        if (__any_sync(0xffffffffu, aborted)) {  // tcgen05.ld below needs the whole warp
          aborted = true;
          break;
        }
        tc::fence_after_sync();
        float s[kTcN];
        {
          uint32_t raw[32];
          tc::ld_32x32b_x32(lane_addr + sb * kTcN, raw);
          tc::wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) s[c] = __uint_as_float(raw[c]);
          tc::ld_32x32b_x32(lane_addr + sb * kTcN + 32, raw);
          tc::wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) s[32 + c] = __uint_as_float(raw[c]);
        }
        tc::fence_before_sync();
        mbar_arrive(&s_free[sb]);

        const int tbase = (w.kt0 + 4 * j) * kTileTokens;
        float mx = -INFINITY;
        if (tbase + kTcN > lim) {
#pragma unroll
          for (int c = 0; c < kTcN; ++c)
            if (tbase + c >= lim) s[c] = -INFINITY;
        }
#pragma unroll
        for (int c = 0; c < kTcN; ++c) mx = fmaxf(mx, s[c]);
        const float m_new = fmaxf(m_used, mx * a.scale_log2);
        if (j == 0) {
          m_used = m_new == -INFINITY ? 0.f : m_new;
        } else if (__any_sync(0xffffffffu, m_new > m_used + kRescaleThreshold)) {
          // O holds P_0..P_{j-1} V scaled by 2^-m_used: wait for the last PV,
          // then move every row of this warp to its current max in TMEM (the
          // TMEM accesses are warp-wide, so the decision is too).
          const uint32_t jp = jg - 1;
          wait_or_abort(&o_done[jp & 1], (jp >> 1) & 1u, flags, aborted);
          if (__any_sync(0xffffffffu, aborted)) {
            aborted = true;
            break;
          }
          tc::fence_after_sync();
          const float alpha = fast_exp2(m_used - m_new);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t raw[32];
            tc::ld_32x32b_x32(lane_addr + 128 + c4 * 32, raw);
            tc::wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) raw[c] = __float_as_uint(__uint_as_float(raw[c]) * alpha);
            tc::st_32x32b_x32(lane_addr + 128 + c4 * 32, raw);
          }
          tc::wait_st();
          l *= alpha;
          m_used = m_new;
        }
        // P for this tile; buffer jg&1 was last read by PV_{jg-2}
        // buffer jg&1 was last read by PV_{jg-2}: phase (jg>>1)-1 of o_done[jg&1]
        wait_or_abort(&o_done[jg & 1], ((jg >> 1) & 1u) ^ 1u, flags, aborted);
        if (__any_sync(0xffffffffu, aborted)) {
          aborted = true;
          break;
        }
        uint8_t* prow = smem + kOffP + (jg & 1) * kPBuf + r * 128;
#pragma unroll
        for (int c8 = 0; c8 < kTcN / 8; ++c8) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = fast_exp2(fmaf(s[c8 * 8 + 2 * e], a.scale_log2, -m_used));
            const float p1 = fast_exp2(fmaf(s[c8 * 8 + 2 * e + 1], a.scale_log2, -m_used));
            l += p0 + p1;
            hi[e] = pack2<T>(p0, p1);
            const float2 f = unpack2<T>(hi[e]);
            lo[e] = pack2<T>(p0 - f.x, p1 - f.y);
          }
          const int off = (c8 ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(prow + kPMat + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        // V rows past the sequence end: zero them (the pool may hold NaN there;
        // pieces past the last page are not loaded at all)
        const int valid = min(si.length - tbase, (w.kt1 - w.kt0 - 4 * j) * kTileTokens);
        if (valid < kTcN) {
          const int st = jg % kTcStages;
          if (!wait_or_abort(&kv_full[st], (jg / kTcStages) & 1u, flags, aborted)) break;
          uint8_t* vb = smem + kOffKV + st * kKVStage + 2 * kKVHalf;
          for (int i = r; i < 2 * (kTcN - valid) * 8; i += 128) {
            const int half = i / ((kTcN - valid) * 8);
            const int rem = i % ((kTcN - valid) * 8);
            const int row = valid + rem / 8, ch = rem % 8;
            *reinterpret_cast<uint4*>(vb + half * kKVHalf + row * 128 + (ch << 4)) =
                make_uint4(0, 0, 0, 0);
          }
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        mbar_arrive(&p_full[jg & 1]);
      }
      if (aborted) break;
      g += ntiles;
      // epilogue: wait for the last PV of the item, read O, normalise, store
      const uint32_t jl = g - 1;
      wait_or_abort(&o_done[jl & 1], (jl >> 1) & 1u, flags, aborted);
      if (__any_sync(0xffffffffu, aborted)) {
        aborted = true;
        break;
      }
      tc::fence_after_sync();
      const float inv = 1.f / l;
      T* dst = row_valid ? a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + w.kvh * G +
                                    p % G) * kHeadDim
                         : nullptr;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t raw[32];
        tc::ld_32x32b_x32(lane_addr + 128 + c4 * 32, raw);
        tc::wait_ld();
        if (dst) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            pk.x = pack2<T>(__uint_as_float(raw[8 * v + 0]) * inv, __uint_as_float(raw[8 * v + 1]) * inv);
            pk.y = pack2<T>(__uint_as_float(raw[8 * v + 2]) * inv, __uint_as_float(raw[8 * v + 3]) * inv);
            pk.z = pack2<T>(__uint_as_float(raw[8 * v + 4]) * inv, __uint_as_float(raw[8 * v + 5]) * inv);
            pk.w = pack2<T>(__uint_as_float(raw[8 * v + 6]) * inv, __uint_as_float(raw[8 * v + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c4 * 32 + 8 * v) = pk;
          }
        }
      }
      tc::fence_before_sync();
      mbar_arrive(o_free);
    }
    if (aborted && lane == 0) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T>
int launch_t(const CUtensorMap& kmap, const CUtensorMap& vmap, const AttnArgs<T>& args, int grid,
             cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(paged_prefill_tc_kernel<T>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "paged_prefill_tc_kernel attribute");
  paged_prefill_tc_kernel<T><<<grid, kTcThreads, kTcSmem, stream>>>(kmap, vmap, args);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

}  // namespace

int prefill_tc_smem_bytes() { return kTcSmem; }

int prefill_tc_launch(int dtype, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const void* args, int grid, cudaStream_t stream) {
  if (dtype == FE_DTYPE_BF16)
    return launch_t<__nv_bfloat16>(kmap, vmap,
                                   *static_cast<const AttnArgs<__nv_bfloat16>*>(args), grid, stream);
  return launch_t<__half>(kmap, vmap, *static_cast<const AttnArgs<__half>*>(args), grid, stream);
}

}  // namespace fe
