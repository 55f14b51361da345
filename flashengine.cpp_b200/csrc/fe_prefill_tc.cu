// Paged chunked-prefill / speculative-verify attention on the 5th-generation
// tensor cores (tcgen05, TMEM) for sm_100a.
//
// Reference behaviour: Cambridgebit/FlashEngine.cpp src/flashinfer_attention.cu:35-44
// (multi-row requests of the FlashInfer paged prefill kernel; causal = the
// bottom-right mask, or none for DFlash block verify) with the arithmetic of
// src/portable_gpu_ops.cpp:39-44.
//
// One persistent CTA per SM, twelve warps (three warpgroups). A work item is
// 128 packed query rows (row p = query row p / G, head kvh*G + p % G) of one
// sequence and KV head against a range of keys, processed in 64-key tiles.
//  warps 8/11 producers of K / of V: gather each key tile (four 16-token
//             page pieces, one 4 KiB TMA box each) into a 6-stage ring (16
//             KiB of K + 16 KiB of V per stage); the page ids of the next 32
//             pieces are fetched ahead by the warp's lanes.
//  warp 9     S issuer (one thread) and TMEM owner (512 columns):
//               S_j  = Q K_j^T  (M = 128, N = 64, K = 128, both operands in
//                      shared memory) into one of four TMEM S slots (two per
//                      softmax group), as soon as the slot's P was consumed;
//  warp 10    PV issuer (one thread):
//               O_g += P_j V_j  (M = 128, N = 128, K = 64) with P read from
//                      TMEM, where the softmax wrote it over its own S slot:
//                      a 16-bit high part and its 16-bit residual (two MMAs
//                      per 16 keys), keeping ~16 bits of every weight.
//  warps 0-3  softmax group 0 (even tiles) and warps 4-7 group 1 (odd tiles):
//             one thread per packed row (TMEM lane). Each group keeps its own
//             base-2 online softmax with a lazy rescale (its O is rescaled in
//             TMEM only when the row max grows by more than 2^8); the two
//             groups alternate so one group's exponentials overlap the other
//             group's MMAs, and two S slots per group let a group start its
//             next tile before the tensor core has consumed its last P. At the
//             end group 0 merges both (O, m, l) states, divides and stores
//             the 16-bit output.
// All hand-offs are mbarriers; every wait is bounded.
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
constexpr int kTcStages = 6;
constexpr int kTcThreads = 12 * 32;     // 3 warpgroups: softmax 0, softmax 1, producer/MMA
constexpr int kProducerWarp = 8, kMmaWarp = 9, kPvWarp = 10, kVProducerWarp = 11;
constexpr int kQHalf = kTcM * 128;      // 16 KiB: 128 rows x 64 dims
// A stage holds the K tile then the V tile, each as four 4 KiB pieces laid
// out [8-key group][head-half][8 rows x 128 B] (swizzled 1 KiB atoms): the
// 8-key groups of one head-half are 2 KiB apart, the two halves 1 KiB apart.
constexpr int kPieceBytes = kTileTokens * 256;  // 16 keys x 128 dims x 2 B
constexpr int kKVTile = 4 * kPieceBytes;        // 16 KiB: 64 keys x 128 dims
constexpr int kKVStage = 2 * kKVTile;           // K tile, V tile
constexpr int kOffQ = 0;
constexpr int kOffKV = 2 * kQHalf;
constexpr int kOffX = kOffKV + kTcStages * kKVStage;    // group-1 (m, l) exchange
constexpr int kXBytes = kTcM * 2 * 4;                   // 128 rows x (m, l)
constexpr int kOffBar = kOffX + kXBytes;
// q_full, o_free, g1_done, k_full[6], v_full[6], kv_empty[6], s_full[2][2],
// s_free[2][2], p_full[2][2], mma_drain
constexpr int kNumBars = 3 + 3 * kTcStages + 4 + 4 + 4 + 1;
constexpr int kTcSmem = 1024 + kOffBar + kNumBars * 8 + 32;
// TMEM columns: S/P slot (g, s) at g*128 + s*64 (64 fp32 S columns, later P
// high part in the first 32 and residual in the last 32); O_g at 256 + g*128.
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.f;
static_assert(kTcSmem <= 232448, "shared memory budget");

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

// 16-bit high part of a weight pair, back in fp32.
template <typename T>
__device__ __forceinline__ float2 hi_as_float(uint32_t h);
template <>
__device__ __forceinline__ float2 hi_as_float<__nv_bfloat16>(uint32_t h) {
  return make_float2(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 hi_as_float<__half>(uint32_t h) {
  return unpack2<__half>(h);
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* flags,
                                              bool& aborted) {
  if (aborted) return false;
  if (flags[0] || !wait_bounded(bar, parity, flags)) aborted = true;
  return !aborted;
}

// Warp-uniform wait (the tcgen05.ld / st that follow need the whole warp).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* flags,
                                          bool& aborted) {
  wait_or_abort(bar, parity, flags, aborted);
  if (__any_sync(0xffffffffu, aborted)) aborted = true;
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
  uint64_t* g1_done = bars + 2;
  uint64_t* k_full = bars + 3;
  uint64_t* v_full = k_full + kTcStages;
  uint64_t* kv_empty = v_full + kTcStages;
  uint64_t* s_full = kv_empty + kTcStages;  // [group*2 + slot]: S written
  // s_free completes when the PV that read the slot's P has completed, and
  // with it every MMA issued before (a commit tracks all earlier MMAs).
  uint64_t* s_free = s_full + 4;            // [group*2 + slot]: P consumed
  uint64_t* p_full = s_free + 4;            // [group*2 + slot]: P written
  uint64_t* mma_drain = p_full + 4;         // every MMA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 2);
  float* xchg = reinterpret_cast<float*>(smem + kOffX);  // [row][m, l] of group 1

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
    mbar_init(g1_done, 128);
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 1);
      mbar_init(&p_full[b], 4);  // one arrival per softmax warp
    }
    mbar_init(mma_drain, 2);  // one commit per issuing thread
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;
  // Registers are allocated per warpgroup, so the kernel runs three full
  // warpgroups (168 registers each thread); warp 11 only waits at the final
  // barrier.

  if (warp == kProducerWarp || warp == kVProducerWarp) {
    // ---------------------------------------------------------- producers
    const bool is_v = warp == kVProducerWarp;
    const CUtensorMap* map = is_v ? &vmap : &kmap;
    uint64_t* full = is_v ? v_full : k_full;
    uint8_t* region = smem + kOffKV + (is_v ? kKVTile : 0);
    if (lane == 0) prefetch_tensormap(map);
    uint32_t g = 0;
    for (int it = it0; it < it1 && !aborted; ++it) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int h2 = w.kvh * 2;
      const int ntiles = (w.kt1 - w.kt0 + 3) / 4;
      const int npieces = w.kt1 - w.kt0;
      // Slot of 16-token piece `i` of the item; lanes fetch 32 pieces (8
      // tiles) at a time and the next 32 are requested before they are needed.
      auto piece_slot = [&](int i) -> int {
        if (i >= npieces) return 0;
        const int t0 = (w.kt0 + i) * kTileTokens;
        return __ldg(pages + si.page_off + t0 / a.page) * a.page + (t0 % a.page);
      };
      int cur = piece_slot(lane), nxt = piece_slot(32 + lane);
      for (int j = 0; j < ntiles && !aborted; ++j, ++g) {
        const int pb = (4 * j) & 31;
        if (j > 0 && pb == 0) {
          cur = nxt;
          nxt = piece_slot(4 * j + 32 + lane);
        }
        const int pieces = min(4, npieces - 4 * j);
        const int st = g % kTcStages;
        int sl[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) sl[u] = __shfl_sync(0xffffffffu, cur, (pb + u) & 31);
        int good = 1;
        if (lane == 0) {
          if (!wait_or_abort(&kv_empty[st], ((g / kTcStages) & 1u) ^ 1u, flags, aborted)) {
            good = 0;
          } else {
            mbar_arrive_expect_tx(&full[st], pieces * kPieceBytes);
            uint8_t* dst = region + st * kKVStage;
            // piece start slots are multiples of 16: coordinates (0, 0,
            // head-half pair, slot / 8)
            for (int u = 0; u < pieces; ++u)
              tma_load_4d(dst + u * kPieceBytes, map, &full[st], 0, 0, h2, sl[u] >> 3);
          }
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) {
          aborted = true;
          break;
        }
      }
    }
    if (lane == 0) {
      if (aborted) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
      // The last load into each stage has landed before the CTA may exit
      // (consumed stages return at once; bounded for an aborted run).
      for (uint32_t t = g > kTcStages ? g - kTcStages : 0; t < g; ++t)
        wait_bounded(&full[t % kTcStages], (t / kTcStages) & 1u, flags + 1);
    }
  } else if (warp == kMmaWarp || warp == kPvWarp) {
    // ------------------------------------------- MMA issuers (S and PV streams)
    // Two threads issue into the same tensor pipe so that a PV whose P is
    // ready never waits behind an S issue (an issue blocks while the pipe's
    // queue is full) and S runs ahead as far as its slots allow.
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16(Fmt<T>::v, false, false, kTcM, kTcN);
      constexpr uint32_t idesc_o = tc::idesc_f16(Fmt<T>::v, false, true, kTcM, kHeadDim);
      // Descriptors of stage 0 / the Q tile; the 14-bit start-address field
      // (address >> 4) is advanced by plain addition (shared addresses stay
      // below 256 KiB, so it never carries out of the field).
      // K: K-major, 8-key groups 2 KiB apart, dims 64..127 at +1 KiB.
      // V: MN-major, 64-dim halves 1 KiB apart (leading), 8-key groups 2 KiB
      // apart (stride), 16 keys per 4 KiB.
      const uint64_t q_desc = tc::smem_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
      const uint64_t k_desc0 = tc::smem_desc_sw128(smem_u32(smem + kOffKV), 16, 2048);
      const uint64_t v_desc0 = tc::smem_desc_sw128(smem_u32(smem + kOffKV + kKVTile), 1024, 2048);
      const bool s_stream = warp == kMmaWarp;
      uint32_t tbase = 0;      // global index of the item's first tile
      uint32_t n[2] = {0, 0};  // tiles issued per softmax group (S slot and phase)
      int unit = 0;
      for (int it = it0; it < it1 && !aborted; ++it, ++unit) {
        const WorkItem w = items[it];
        const int ntiles = (w.kt1 - w.kt0 + 3) / 4;
        if (s_stream) {
          // S_t = Q K_t^T into the group's next slot once the PV that read
          // the slot's P has completed.
          if (!wait_or_abort(q_full, unit & 1, flags, aborted)) break;
          for (int t = 0; t < ntiles && !aborted; ++t) {
            const int gi = t & 1;
            const int slot = n[gi] & 1;
            const uint32_t tg = tbase + t;
            const int st = tg % kTcStages;
            if (!wait_or_abort(&s_free[gi * 2 + slot], ((n[gi] >> 1) & 1u) ^ 1u, flags, aborted))
              break;
            if (!wait_or_abort(&k_full[st], (tg / kTcStages) & 1u, flags, aborted)) break;
            tc::fence_after_sync();
            const uint64_t k_desc = k_desc0 + uint64_t((st * kKVStage) >> 4);
            const uint32_t d = tmem + gi * 128 + slot * kTcN;
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 16; ++kk) {
              const int half = kk >> 2, ko = (kk & 3) * 32;
              tc::mma_f16(d, q_desc + uint64_t((half * kQHalf + ko) >> 4),
                          k_desc + uint64_t((half * 1024 + ko) >> 4), idesc_s,
                          kk > 0 ? 1u : 0u);
            }
            tc::commit(&s_full[gi * 2 + slot]);
            ++n[gi];
          }
        } else {
          // O_g += P_t V_t as soon as the group has written P_t.
          for (int j = 0; j < ntiles && !aborted; ++j) {
            const int gi = j & 1;
            const int slot = n[gi] & 1;
            if (j == 0 && unit > 0) {
              // both O accumulators are free once group 0 merged the last item
              if (!wait_or_abort(o_free, (unit - 1) & 1, flags, aborted)) break;
              tc::fence_after_sync();
            }
            if (!wait_or_abort(&p_full[gi * 2 + slot], (n[gi] >> 1) & 1u, flags, aborted)) break;
            const uint32_t tg = tbase + j;
            const int st = tg % kTcStages;
            if (!wait_or_abort(&v_full[st], (tg / kTcStages) & 1u, flags, aborted)) break;
            tc::fence_after_sync();
            const uint64_t v_desc = v_desc0 + uint64_t((st * kKVStage) >> 4);
            const uint32_t p_col = tmem + gi * 128 + slot * kTcN;
            const uint32_t d = tmem + 256 + gi * 128;
#pragma unroll
            for (int part = 0; part < 2; ++part) {
#pragma unroll
              for (int kk = 0; kk < kTcN / 16; ++kk) {
                const bool first = j < 2 && part == 0 && kk == 0;
                tc::mma_f16_ts(d, p_col + part * 32 + kk * 8,
                               v_desc + uint64_t((kk * kPieceBytes) >> 4), idesc_o,
                               first ? 0u : 1u);
              }
            }
            // this PV and every earlier one complete -> slot reusable, stage free
            tc::commit(&s_free[gi * 2 + slot]);
            tc::commit(&kv_empty[st]);
            ++n[gi];
          }
        }
        tbase += ntiles;
      }
      if (aborted) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
      // TMEM is released only after every MMA issued here has completed.
      tc::commit(mma_drain);
      wait_bounded(mma_drain, 0, flags + 1);
    }
  } else if (warp < 8) {
    // ------------------------------------------------ softmax groups / epilogue
    const int gi = warp >= 4 ? 1 : 0;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // packed row = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const uint32_t s_col = gi * 128, o_col = 256 + gi * 128;
    const int G = a.G;
    const bool causal = view == 1;
    uint32_t tbase = 0;
    uint32_t nt = 0;  // tiles this group has processed (global): S slot and phase
    int unit = 0;
    for (int it = it0; it < it1 && !aborted; ++it, ++unit) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int ntiles = (w.kt1 - w.kt0 + 3) / 4;
      const int P = si.qrows * G;
      const int p = w.rb0 * kRowBlock + r;
      const bool row_valid = p < P;
      if (gi == 0) {
        // Q row -> swizzled K-major shared tile (zeros for padding rows); the
        // previous item's MMAs have all completed (its merge waited for them)
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
        tc::fence_proxy_async_smem();
        mbar_arrive(q_full);
      } else if (unit > 0) {
        // stay within one item of group 0 (exchange slots, o_free phases)
        if (!wait_warp(o_free, (unit - 1) & 1, flags, aborted)) break;
      }

      const int lim = (causal && row_valid) ? si.length - si.qrows + p / G + 1 : si.length;
      float m_used = -INFINITY, l = 0.f;
      bool first = true;
      for (int j = gi; j < ntiles; j += 2, ++nt) {
        const uint32_t tg = tbase + j;
        const int slot = nt & 1;
        const uint32_t slot_addr = lane_addr + s_col + slot * kTcN;
        if (!wait_warp(&s_full[gi * 2 + slot], (nt >> 1) & 1u, flags, aborted)) break;
        tc::fence_after_sync();
        // S row: 64 fp32 columns straight into registers
        float s[kTcN];
        tc::ld_32x32b_x32(slot_addr, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tc::ld_32x32b_x32(slot_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        tc::wait_ld();

        const int tkey = (w.kt0 + 4 * j) * kTileTokens;
        if (tkey + kTcN > lim) {
#pragma unroll
          for (int c = 0; c < kTcN; ++c)
            if (tkey + c >= lim) s[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = s[e];
#pragma unroll
        for (int c = 8; c < kTcN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_new = fmaxf(m_used, mx * a.scale_log2);
        if (first) {
          m_used = m_new == -INFINITY ? 0.f : m_new;
        } else if (__any_sync(0xffffffffu, m_new > m_used + kRescaleThreshold)) {
          // O_g holds this group's earlier tiles of the item: wait for the
          // last PV into it (tile nt - 1; the one before it completed before
          // S of tile nt was issued), then rescale it in TMEM.
          if (!wait_warp(&s_free[gi * 2 + ((nt - 1) & 1)], ((nt - 1) >> 1) & 1u, flags, aborted))
            break;
          tc::fence_after_sync();
          const float alpha = fast_exp2(m_used - m_new);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float ov[32];
            tc::ld_32x32b_x32(lane_addr + o_col + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
            tc::wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] *= alpha;
            tc::st_32x32b_x32(lane_addr + o_col + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
          }
          l *= alpha;
          m_used = m_new;
        }
        first = false;
        // P = exp2(S * scale - m): high 16-bit part over S columns [0, 32),
        // residual over [32, 64) (S is already in registers).
        float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 32 keys -> 16 high + 16 residual columns
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = fast_exp2(fmaf(s[32 * h + 2 * e], a.scale_log2, -m_used));
            const float p1 = fast_exp2(fmaf(s[32 * h + 2 * e + 1], a.scale_log2, -m_used));
            l8[(2 * e) & 7] += p0;
            l8[(2 * e + 1) & 7] += p1;
            hi[e] = pack2<T>(p0, p1);
            const float2 f = hi_as_float<T>(hi[e]);
            lo[e] = pack2<T>(p0 - f.x, p1 - f.y);
          }
          tc::st_32x32b_x16(slot_addr + 16 * h, hi);
          tc::st_32x32b_x16(slot_addr + 32 + 16 * h, lo);
        }
        l += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
        // V rows past the sequence end or past the loaded pieces are zeroed
        // (the pool may hold NaN there; unloaded rows hold an older tile)
        const int valid = min(si.length - tkey, (w.kt1 - w.kt0 - 4 * j) * kTileTokens);
        if (valid < kTcN) {
          const int st = tg % kTcStages;
          if (!wait_warp(&v_full[st], (tg / kTcStages) & 1u, flags, aborted)) break;
          uint8_t* vb = smem + kOffKV + st * kKVStage + kKVTile;
          const int n = (kTcN - valid) * 8;  // 16-byte chunks per head-half
          for (int i = r; i < 2 * n; i += 128) {
            const int half = i / n, rem = i % n;
            const int row = valid + rem / 8, ch = rem % 8;
            *reinterpret_cast<uint4*>(vb + (row >> 3) * 2048 + half * 1024 + (row & 7) * 128 +
                                      (ch << 4)) = make_uint4(0, 0, 0, 0);
          }
          tc::fence_proxy_async_smem();
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[gi * 2 + slot]);
      }
      if (aborted) break;
      tbase += ntiles;
      const bool had = ntiles > gi;  // this group processed at least one tile
      // Group 1 rewrites its slot only after waiting o_free for this item,
      // i.e. after group 0 has read it.
      float* xrow = xchg + r * 2;
      // Wait for the group's last PV (tile nt - 1) through its slot: the
      // PV before it completed before that tile's S was issued, so the
      // slot's barrier is at most one phase short of it.
      if (had && !wait_warp(&s_free[gi * 2 + ((nt - 1) & 1)], ((nt - 1) >> 1) & 1u, flags, aborted))
        break;
      if (gi == 1) {
        xrow[0] = m_used;
        xrow[1] = l;
        tc::fence_before_sync();
        mbar_arrive(g1_done);
        continue;
      }
      // group 0: merge both groups' states and write the output
      if (!wait_warp(g1_done, unit & 1, flags, aborted)) break;
      tc::fence_after_sync();
      const bool had1 = ntiles > 1;
      const float m1 = had1 ? xrow[0] : -INFINITY, l1 = had1 ? xrow[1] : 0.f;
      const float M = fmaxf(m_used, m1);
      const float a0 = fast_exp2(m_used - M), a1 = had1 ? fast_exp2(m1 - M) : 0.f;
      const float inv = 1.f / (l * a0 + l1 * a1);
      T* dst = row_valid ? a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + w.kvh * G +
                                    p % G) * kHeadDim
                         : nullptr;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        float o0[32], o1[32];
        tc::ld_32x32b_x32(lane_addr + 256 + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&o0[0]));
        if (had1)
          tc::ld_32x32b_x32(lane_addr + 384 + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&o1[0]));
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) o0[c] = (o0[c] * a0 + (had1 ? o1[c] * a1 : 0.f)) * inv;
        if (dst) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            pk.x = pack2<T>(o0[8 * v + 0], o0[8 * v + 1]);
            pk.y = pack2<T>(o0[8 * v + 2], o0[8 * v + 3]);
            pk.z = pack2<T>(o0[8 * v + 4], o0[8 * v + 5]);
            pk.w = pack2<T>(o0[8 * v + 6], o0[8 * v + 7]);
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
  if (warp == kMmaWarp) {
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
