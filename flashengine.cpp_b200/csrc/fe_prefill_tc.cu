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
// sequence and KV head against a range of keys, processed in 128-key tiles.
//  warps 8/11 producers of K / of V: gather each key tile (eight 16-token
//             page pieces, one 4 KiB TMA box each) into a 3-stage K ring and a
//             2-stage V ring (32 KiB per stage; 2 K and 3 V stages at head_dim
//             256); a K stage is released when its S MMA completed, a V stage
//             when its PV did. The page ids of the
//             next 32 pieces are fetched ahead by the warp's lanes. The K
//             producer also loads each item's Q tile with two TMA boxes (query
//             rows x GQA heads x 64 dims, which lands in packed-row order) into
//             one of two Q buffers, as soon as the item two back has released
//             it, so S of the next item starts while the current one finishes.
//  warp 9     S issuer (one thread) and TMEM owner (512 columns):
//               S_t = Q K_t^T (M = 128, N = 128, K = 128, both operands in
//                     shared memory) into one of three 128-column TMEM slots,
//                     as soon as the slot's P was consumed;
//  warp 10    PV issuer (one thread):
//               O += P_t V_t (M = 128, N = 128, K = 128) once both softmax
//                    groups wrote their half of P_t over the slot in TMEM: a
//                    16-bit high part and its 16-bit residual (two MMAs per 16
//                    keys), keeping ~16 bits of every weight.
//  warps 0-7  softmax: one thread per packed row (TMEM lane); warps q and q+4
//             share rows 32q..32q+31, group 0 (warps 0-3) exponentiates keys
//             0-63 of every tile and group 1 (warps 4-7) keys 64-127. The two
//             warps of a row trade their half-row maxima through shared
//             memory, so both keep the same base-2 online-softmax state and
//             one O accumulator serves both;
//             the rescale is lazy (O is rescaled in TMEM, each group its 64
//             dims, only when the row max grows by more than 2^8). Three slots
//             let the softmax run two tiles ahead of the tensor core's
//             consumption of P. At the end each group divides its 64 dims by
//             the summed row weights and stores them in 16 bits.
// All hand-offs are mbarriers; every wait is bounded.
//
// head_dim 256 (hybrid and DFlash draft models, which the reference serves
// through ATen with any head_dim) instantiates the same kernel with 64-key
// tiles, one 64 KiB Q buffer, S slots of 64 TMEM columns and O (256 fp32
// columns) at column 256; each softmax group then owns 32 keys of a tile and
// 128 of O's dims. Its items may be pieces of a key range split across CTAs
// (few 128-row items, as DFlash draft blocks give): a piece stores its
// unnormalised O with the row's (m, l) into a partial record, and
// decode_merge_kernel combines them.
#include <mutex>

#include "fe_attn_common.cuh"
#include "fe_tcgen05.cuh"

namespace fe {

int prefill_tc_launch(int dtype, int dim, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const CUtensorMap& qmap, const void* args, int grid, cudaStream_t stream);

namespace {

// Per head dim D (128, or 256 for the hybrid / DFlash models' full-attention
// layers). Both use the same shared-memory budget: 64 KiB of Q (two 128-dim
// tiles, or one 256-dim tile) and five 32 KiB K / V stages (128 keys of 128
// dims, or 64 keys of 256 dims). A K stage is refilled only when the S that
// read it has completed, and a V stage when its P·V has, so the rings'
// depths bound how far the loads run ahead. S of a tile is issued about two
// tiles before its P·V, so K tiles are needed earlier than V tiles: head_dim
// 128 runs 3 K + 2 V stages (S no longer waits on its K tile: C4 and C3's
// prefill rows ~1.3% faster than with 2 K + 3 V); at head_dim 256 2 K + 3 V
// and 3 K + 2 V measured the same.
constexpr int kSlotsTc = 3;
constexpr int kKVStagesTc = 5;  // K + V stages
constexpr int kTcThreads = 12 * 32;  // 3 warpgroups: softmax 0, softmax 1, producers/MMA
constexpr int kProducerWarp = 8, kMmaWarp = 9, kPvWarp = 10, kVProducerWarp = 11;
// q_full[2], q_empty[2], o_free, l_done, k_full[K], k_empty[K], v_full[V],
// v_empty[V] (K + V = 5 stages), s_full[3], s_free[3], p_full[3][2],
// mma_drain, xmax[2][4]
constexpr int kNumBarsTc =
    4 + 2 + 2 * kKVStagesTc + kSlotsTc + kSlotsTc + 2 * kSlotsTc + 1 + 8;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.f;

template <int D>
struct TcCfg {
  static constexpr int kM = 128;                        // packed rows per work item
  static constexpr int kN = D == kHeadDim ? 128 : 64;   // keys per tile (S MMA N)
  static constexpr int kHalfN = kN / 2;                 // keys per softmax group and tile
  static constexpr int kPiecesPerTile = kN / kTileTokens;
  static constexpr int kBoxes = D / 64;                 // 64-dim boxes per row
  static constexpr int kQBox = kM * 128;                // 16 KiB: 128 rows x 64 dims
  static constexpr int kQBytes = kBoxes * kQBox;        // one Q tile
  static constexpr int kQBufs = D == kHeadDim ? 2 : 1;
  // A K (or V) stage holds one tile as 16-token pieces laid out
  // [8-key group][64-dim box][8 rows x 128 B] (swizzled 1 KiB atoms): the
  // 8-key groups of one box are kGroupBytes apart, the boxes 1 KiB apart.
  static constexpr int kPieceBytes = kTileTokens * D * 2;
  static constexpr int kGroupBytes = 8 * D * 2;
  static constexpr int kKVTile = kPiecesPerTile * kPieceBytes;  // 32 KiB
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kQBufs * kQBytes;
  static constexpr int kKStages = D == kHeadDim ? 3 : 2;
  static constexpr int kVStages = kKVStagesTc - kKStages;
  static constexpr int kOffV = kOffK + kKStages * kKVTile;
  static constexpr int kOffX = kOffV + kVStages * kKVTile;   // half-row maxima
  static constexpr int kXBytes = 2 * 2 * kM * 4;               // [tile parity][group][128 rows]
  static constexpr int kOffBar = kOffX + kXBytes;
  static constexpr int kSmem = kOffBar + kNumBarsTc * 8 + 32;
  // TMEM columns: slot s at s*kN (S fp32; group g's half [g*kN/2, (g+1)*kN/2)
  // is later overwritten by its P: high part in its first kN/4 columns,
  // residual in the last kN/4); O (D fp32 columns) at kOCol.
  static constexpr uint32_t kOCol = D == kHeadDim ? kSlotsTc * kN : 256;
  static constexpr int kGroupDims = D / 2;  // O dims each softmax group rescales / stores
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(kSlotsTc * kN <= int(kOCol) && kOCol + D <= 512, "TMEM budget");
  static_assert(32 % kPiecesPerTile == 0, "page-id prefetch assumes whole tiles per 32 pieces");
  static_assert(kHalfN % 32 == 0, "softmax loads S in 32-column chunks");
};

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

// The abort flag is read only once a wait has to spin (the slow path), so a
// completed phase costs one try_wait.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* flags,
                                              bool& aborted) {
  if (aborted) return false;
  if (!wait_bounded_short(bar, parity, flags)) aborted = true;
  return !aborted;
}

// Warp-uniform wait (the tcgen05.ld / st that follow need the whole warp).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* flags,
                                          bool& aborted) {
  wait_or_abort(bar, parity, flags, aborted);
  if (__any_sync(0xffffffffu, aborted)) aborted = true;
  return !aborted;
}

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap,
                            const __grid_constant__ CUtensorMap qmap, const AttnArgs<T> a) {
  using C = TcCfg<D>;
  constexpr int kTcM = C::kM, kTcN = C::kN, kHalfN = C::kHalfN;
  constexpr int kPiecesPerTile = C::kPiecesPerTile;
  constexpr int kSlots = kSlotsTc, kKStages = C::kKStages, kVStages = C::kVStages;
  constexpr uint32_t kOCol = C::kOCol;
  constexpr bool kSplits = D != kHeadDim;  // the planner splits head_dim 256 row items only
  // declared 16-byte aligned so that the 1 KiB check below is not folded away
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars + 0;   // [buffer]: Q tile landed
  uint64_t* q_empty = bars + 2;  // [buffer]: both groups done with the item
  uint64_t* o_free = bars + 4;
  uint64_t* l_done = bars + 5;
  uint64_t* k_full = bars + 6;
  uint64_t* k_empty = k_full + kKStages;
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* s_full = v_empty + kVStages;    // [slot]: S written
  // s_free[slot] completes when the PV that read the slot's P has completed,
  // and with it every MMA the PV thread issued before.
  uint64_t* s_free = s_full + kSlots;
  uint64_t* p_full = s_free + kSlots;       // [slot*2 + group]: P written
  uint64_t* mma_drain = p_full + 2 * kSlots;  // every MMA issued has completed
  uint64_t* xmax_bar = mma_drain + 1;         // [tile parity*4 + quad]: maxima written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBarsTc);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 2);
  float* xmax = reinterpret_cast<float*>(smem + C::kOffX);  // [parity][group][row]
  // Row weight sums at the end of an item go to the item's Q buffer (dead by
  // then, [group][row]); the buffer is released for the item kQBufs ahead
  // only after both groups have read them.

  pdl_trigger();
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
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) raise_device_error(a.err, FE_DEVERR_SMEM_ALIGN);
    return;
  }

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 8);  // one arrival per softmax warp
    }
    mbar_init(o_free, 256);
    mbar_init(l_done, 256);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 1);
    }
    for (int b = 0; b < 2 * kSlots; ++b) mbar_init(&p_full[b], 4);  // one arrival per warp
    mbar_init(mma_drain, 2);  // one commit per issuing thread
    for (int b = 0; b < 8; ++b) mbar_init(&xmax_bar[b], 64);  // both warps of a quad
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
  // q and the pools belong to earlier kernels until here (a no-op when
  // launched without programmatic serialization)
  pdl_wait();
  // Registers are allocated per warpgroup, so the kernel runs three full
  // warpgroups (168 registers each thread).

  if (warp == kProducerWarp || warp == kVProducerWarp) {
    // ---------------------------------------------------------- producers
    const bool is_v = warp == kVProducerWarp;
    const CUtensorMap* map = is_v ? &vmap : &kmap;
    uint64_t* full = is_v ? v_full : k_full;
    uint64_t* empty = is_v ? v_empty : k_empty;
    const int stages = is_v ? kVStages : kKStages;
    uint8_t* region = smem + (is_v ? C::kOffV : C::kOffK);
    // Q tiles by TMA when a tile is whole query rows (G divides 128) inside
    // the rows the Q map covers, else by the warp's lanes
    const bool q_tma = (kTcM % a.G) == 0 && a.q_map_rows > 0;
    if (lane == 0) {
      prefetch_tensormap(map);
      if (!is_v && q_tma) prefetch_tensormap(&qmap);
    }
    uint32_t g = 0;
    int unit = 0;
    for (int it = it0; it < it1 && !aborted; ++it, ++unit) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int hbox = w.kvh * C::kBoxes;  // the KV head's first 64-dim box
      if (!is_v) {
        // the item's Q tile: packed row p = query row p / G, head kvh*G + p % G,
        // i.e. 128/G query rows x G heads x 64 dims per box (rows past the
        // sequence are other sequences' q or zero fill; their output is
        // never stored)
        const int b = unit % C::kQBufs;
        uint8_t* dst = smem + C::kOffQ + b * C::kQBytes;
        const int G = a.G, P = si.qrows * G;
        const bool tma_item =
            q_tma && si.q_row0 + (min(P, w.rb0 * kRowBlock + kTcM) - 1) / G < a.q_map_rows;
        int good = 1;
        if (lane == 0) {
          if (!wait_or_abort(&q_empty[b], ((unit / C::kQBufs) & 1u) ^ 1u, flags, aborted)) {
            good = 0;
          } else if (tma_item) {
            mbar_arrive_expect_tx(&q_full[b], C::kQBytes);
            const int row0 = si.q_row0 + (w.rb0 * kRowBlock) / a.G;
#pragma unroll
            for (int x = 0; x < C::kBoxes; ++x)
              tma_load_3d(dst + x * C::kQBox, &qmap, &q_full[b], 64 * x, w.kvh * a.G, row0);
          }
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) {
          aborted = true;
          break;
        }
        if (!tma_item) {
          // copy with the lanes into the swizzled K-major tile (zeros past the
          // sequence), then publish
          constexpr int kChunks = D / 8;  // 16-byte chunks per row
          for (int i = lane; i < kTcM * kChunks; i += 32) {
            const int r = i / kChunks, c = i % kChunks;
            const int pr = w.rb0 * kRowBlock + r;
            uint4 val = make_uint4(0, 0, 0, 0);
            if (pr < P)
              val = __ldg(reinterpret_cast<const uint4*>(
                            a.q + (static_cast<int64_t>(si.q_row0 + pr / G) * a.hq + w.kvh * G +
                                   pr % G) * D) + c);
            const int box = c >> 3, cc = c & 7;
            *reinterpret_cast<uint4*>(dst + box * C::kQBox + r * 128 + ((cc ^ (r & 7)) << 4)) =
                val;
          }
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&q_full[b]);
        }
      }
      const int npieces = w.kt1 - w.kt0;
      const int ntiles = (npieces + kPiecesPerTile - 1) / kPiecesPerTile;
      // Slot of 16-token piece `i` of the item; lanes fetch 32 pieces at a
      // time and the next 32 are requested before they are needed.
      auto piece_slot = [&](int i) -> int {
        if (i >= npieces) return 0;
        const int t0 = (w.kt0 + i) * kTileTokens;
        return __ldg(pages + si.page_off + t0 / a.page) * a.page + (t0 % a.page);
      };
      int cur = piece_slot(lane), nxt = piece_slot(32 + lane);
      for (int j = 0; j < ntiles && !aborted; ++j, ++g) {
        const int pb = (kPiecesPerTile * j) & 31;
        if (j > 0 && pb == 0) {
          cur = nxt;
          nxt = piece_slot(kPiecesPerTile * j + 32 + lane);
        }
        const int pieces = min(kPiecesPerTile, npieces - kPiecesPerTile * j);
        const int st = g % stages;
        int sl[kPiecesPerTile];
#pragma unroll
        for (int u = 0; u < kPiecesPerTile; ++u) sl[u] = __shfl_sync(0xffffffffu, cur, pb + u);
        int good = 1;
        if (lane == 0) {
          if (!wait_or_abort(&empty[st], ((g / stages) & 1u) ^ 1u, flags, aborted)) {
            good = 0;
          } else {
            mbar_arrive_expect_tx(&full[st], pieces * C::kPieceBytes);
            uint8_t* dst = region + st * C::kKVTile;
            // piece start slots are multiples of 16: coordinates (0, 0,
            // first box of the head, slot / 8)
#pragma unroll
            for (int u = 0; u < kPiecesPerTile; ++u)
              if (u < pieces)
                tma_load_4d(dst + u * C::kPieceBytes, map, &full[st], 0, 0, hbox, sl[u] >> 3);
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
      for (uint32_t t = g > uint32_t(stages) ? g - stages : 0; t < g; ++t)
        wait_bounded_short(&full[t % stages], (t / stages) & 1u, flags + 1);
      if (!is_v && unit > 0) {  // and the last Q tiles
        for (int u = unit > C::kQBufs ? unit - C::kQBufs : 0; u < unit; ++u)
          wait_bounded_short(&q_full[u % C::kQBufs], (u / C::kQBufs) & 1u, flags + 1);
      }
    }
  } else if (warp == kMmaWarp || warp == kPvWarp) {
    // ------------------------------------------- MMA issuers (S and PV streams)
    // Two threads issue into the same tensor pipe so that a PV whose P is
    // ready never waits behind an S issue (an issue blocks while the pipe's
    // queue is full) and S runs ahead as far as its slots allow.
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16(Fmt<T>::v, false, false, kTcM, kTcN);
      constexpr uint32_t idesc_o = tc::idesc_f16(Fmt<T>::v, false, true, kTcM, D);
      // Descriptors of stage 0 / the Q tile; the 14-bit start-address field
      // (address >> 4) is advanced by plain addition (shared addresses stay
      // below 256 KiB, so it never carries out of the field).
      // K: K-major, 8-key groups kGroupBytes apart, each next 64 dims at +1 KiB.
      // V: MN-major, 64-dim boxes 1 KiB apart (leading), 8-key groups
      // kGroupBytes apart (stride), 16 keys per piece.
      const uint64_t q_desc0 = tc::smem_desc_sw128(smem_u32(smem + C::kOffQ), 16, 1024);
      const uint64_t k_desc0 = tc::smem_desc_sw128(smem_u32(smem + C::kOffK), 16, C::kGroupBytes);
      const uint64_t v_desc0 =
          tc::smem_desc_sw128(smem_u32(smem + C::kOffV), 1024, C::kGroupBytes);
      const bool s_stream = warp == kMmaWarp;
      uint32_t tbase = 0;  // global index of the item's first tile
      uint32_t n = 0;      // tiles issued (slot and phase)
      int unit = 0;
      for (int it = it0; it < it1 && !aborted; ++it, ++unit) {
        const WorkItem w = items[it];
        const int ntiles = (w.kt1 - w.kt0 + kPiecesPerTile - 1) / kPiecesPerTile;
        if (s_stream) {
          // S_t = Q K_t^T into the next slot once both PVs that read the
          // slot's P have completed.
          const int qb = unit % C::kQBufs;
          if (!wait_or_abort(&q_full[qb], (unit / C::kQBufs) & 1u, flags, aborted)) break;
          const uint64_t q_desc = q_desc0 + uint64_t((qb * C::kQBytes) >> 4);
          for (int t = 0; t < ntiles && !aborted; ++t, ++n) {
            const int slot = n % kSlots;
            const uint32_t tg = tbase + t;
            const int st = tg % kKStages;
            if (!wait_or_abort(&s_free[slot], ((n / kSlots) & 1u) ^ 1u, flags, aborted)) break;
            if (!wait_or_abort(&k_full[st], (tg / kKStages) & 1u, flags, aborted)) break;
            tc::fence_after_sync();
            const uint64_t k_desc = k_desc0 + uint64_t((st * C::kKVTile) >> 4);
            const uint32_t d = tmem + slot * kTcN;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int box = kk >> 2, ko = (kk & 3) * 32;
              tc::mma_f16(d, q_desc + uint64_t((box * C::kQBox + ko) >> 4),
                          k_desc + uint64_t((box * 1024 + ko) >> 4), idesc_s, kk > 0 ? 1u : 0u);
            }
            tc::commit(&s_full[slot]);
            tc::commit(&k_empty[st]);  // S (and every earlier S) done -> K stage free
          }
        } else {
          // O += P_t V_t once both groups have written their half of P_t
          // (and finished any rescale of O that tile needed).
          for (int j = 0; j < ntiles && !aborted; ++j, ++n) {
            const int slot = n % kSlots;
            const uint32_t tg = tbase + j;
            const int st = tg % kVStages;
            if (j == 0 && unit > 0) {
              // O is free once both groups stored the last item's output
              if (!wait_or_abort(o_free, (unit - 1) & 1, flags, aborted)) break;
            }
            if (!wait_or_abort(&v_full[st], (tg / kVStages) & 1u, flags, aborted)) break;
            if (!wait_or_abort(&p_full[slot * 2], (n / kSlots) & 1u, flags, aborted)) break;
            if (!wait_or_abort(&p_full[slot * 2 + 1], (n / kSlots) & 1u, flags, aborted)) break;
            tc::fence_after_sync();
            const uint64_t v_desc = v_desc0 + uint64_t((st * C::kKVTile) >> 4);
            const uint32_t d = tmem + kOCol;
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
              const uint32_t p_col = tmem + slot * kTcN + gi * kHalfN;
              const uint64_t vg =
                  v_desc + uint64_t((gi * (kPiecesPerTile / 2) * C::kPieceBytes) >> 4);
#pragma unroll
              for (int part = 0; part < 2; ++part) {
#pragma unroll
                for (int kk = 0; kk < kHalfN / 16; ++kk) {
                  const bool first = j == 0 && gi == 0 && part == 0 && kk == 0;
                  tc::mma_f16_ts(d, p_col + part * (kHalfN / 2) + kk * 8,
                                 vg + uint64_t((kk * C::kPieceBytes) >> 4), idesc_o,
                                 first ? 0u : 1u);
                }
              }
            }
            // the tile's PV (and every earlier MMA of this thread) complete ->
            // the slot is reusable and the V stage is free
            tc::commit(&s_free[slot]);
            tc::commit(&v_empty[st]);
          }
        }
        tbase += ntiles;
      }
      if (aborted) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
      // TMEM is released only after every MMA issued here has completed.
      tc::commit(mma_drain);
      wait_bounded_short(mma_drain, 0, flags + 1);
    }
  } else if (warp < 8) {
    // ------------------------------------------------ softmax groups / epilogue
    constexpr int kGD = C::kGroupDims;
    const int gi = warp >= 4 ? 1 : 0;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // packed row = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const uint32_t o_dims = lane_addr + kOCol + gi * kGD;  // this group's O dims
    const int G = a.G;
    const bool causal = view == 1;
    uint32_t tbase = 0;
    uint32_t nt = 0;  // tiles processed (global): slot and phase
    int unit = 0;
    for (int it = it0; it < it1 && !aborted; ++it, ++unit) {
      const WorkItem w = items[it];
      const SeqInfo si = seqs[w.seq];
      const int npieces = w.kt1 - w.kt0;
      const int ntiles = (npieces + kPiecesPerTile - 1) / kPiecesPerTile;
      const int P = si.qrows * G;
      const int p = w.rb0 * kRowBlock + r;
      const bool row_valid = p < P;
      // keys this row sees in this item: the mask's, cut at the end of the
      // item's pieces (a split item covers part of the range; head_dim 128
      // items are never split)
      int lim = (causal && row_valid) ? si.length - si.qrows + p / G + 1 : si.length;
      if constexpr (kSplits) lim = min(lim, w.kt1 * kTileTokens);
      // m_used stays -inf until the first unmasked key (its weights are 0)
      float m_used = -INFINITY, l = 0.f;
      bool first = true;
      for (int j = 0; j < ntiles; ++j, ++nt) {
        const uint32_t tg = tbase + j;
        const int slot = nt % kSlots;
        const uint32_t slot_addr = lane_addr + slot * kTcN;
        const uint32_t half_addr = slot_addr + gi * kHalfN;
        if (!wait_warp(&s_full[slot], (nt / kSlots) & 1u, flags, aborted)) break;
        tc::fence_after_sync();
        // this group's S columns straight into registers
        const int key0 = (w.kt0 + kPiecesPerTile * j) * kTileTokens;
        const int tkey = key0 + gi * kHalfN;
        float s[kHalfN];
#pragma unroll
        for (int c = 0; c < kHalfN; c += 32)
          tc::ld_32x32b_x32(half_addr + c, *reinterpret_cast<uint32_t(*)[32]>(&s[c]));
        tc::wait_ld();
        if (tkey + kHalfN > lim) {
#pragma unroll
          for (int c = 0; c < kHalfN; ++c)
            if (tkey + c >= lim) s[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = fmax3(s[e], s[8 + e], s[16 + e]);
#pragma unroll
        for (int c = 24; c < kHalfN - 8; c += 16)
#pragma unroll
          for (int e = 0; e < 8; ++e) mx8[e] = fmax3(mx8[e], s[c + e], s[c + 8 + e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = fmaxf(mx8[e], s[kHalfN - 8 + e]);
        float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]),
                         fmax3(fmax3(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7]));
        {
          // trade half-row maxima with the other warp of these rows; the
          // buffer of tile parity b is rewritten only after the partner
          // passed the exchange of the tile in between
          const int b = nt & 1;
          float* xm = xmax + b * 2 * kTcM;
          xm[gi * kTcM + r] = mx;
          mbar_arrive(&xmax_bar[b * 4 + quad]);
          if (!wait_warp(&xmax_bar[b * 4 + quad], (nt >> 1) & 1u, flags, aborted)) break;
          mx = fmaxf(mx, xm[(gi ^ 1) * kTcM + r]);
        }
        const float m_new = fmaxf(m_used, mx * a.scale_log2);
        // true for a row's first finite max too (m_used = -inf); both groups
        // see the same maxima and take the same decisions
        const bool grow = m_new > m_used + kRescaleThreshold;
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? fast_exp2(m_used - m_new) : 1.f;
          if (!first) {
            // O holds the item's earlier tiles: wait for the last PV into it
            // (tile nt - 1; every earlier one completed before S of tile
            // nt - 1 was issued), then rescale this group's O dims in TMEM.
            if (!wait_warp(&s_free[(nt - 1) % kSlots], ((nt - 1) / kSlots) & 1u, flags, aborted))
              break;
            tc::fence_after_sync();
#pragma unroll
            for (int c2 = 0; c2 < kGD / 32; ++c2) {
              float ov[32];
              tc::ld_32x32b_x32(o_dims + c2 * 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
              tc::wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) ov[c] *= alpha;
              tc::st_32x32b_x32(o_dims + c2 * 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
            }
          }
          l *= alpha;
          if (grow) m_used = m_new;
        }
        first = false;
        const float m_sub = m_used == -INFINITY ? 0.f : m_used;
        // P = exp2(S * scale - m): high 16-bit part over the half's first
        // kHalfN/2 columns, residual over the last kHalfN/2 (S is already in
        // registers).
        float2 l4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
        const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
        const float2 nm2 = make_float2(-m_sub, -m_sub);
#pragma unroll
        for (int h = 0; h < kHalfN / 32; ++h) {  // 32 keys -> 16 high + 16 residual columns
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float2 x = fma2(make_float2(s[32 * h + 2 * e], s[32 * h + 2 * e + 1]), sc2, nm2);
            const float2 pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
            l4[e & 3] = add2(l4[e & 3], pp);
            hi[e] = pack2<T>(pp.x, pp.y);
            const float2 res = sub2(pp, hi_as_float<T>(hi[e]));
            lo[e] = pack2<T>(res.x, res.y);
          }
          tc::st_32x32b_x16(half_addr + 16 * h, hi);
          tc::st_32x32b_x16(half_addr + kHalfN / 2 + 16 * h, lo);
        }
        l += ((l4[0].x + l4[0].y) + (l4[1].x + l4[1].y)) + ((l4[2].x + l4[2].y) + (l4[3].x + l4[3].y));
        // V rows of this half past the sequence end or past the loaded pieces
        // are zeroed (the pool may hold NaN there; unloaded rows hold an
        // older tile)
        const int valid = min(si.length - tkey,
                              (npieces - kPiecesPerTile * j) * kTileTokens - gi * kHalfN);
        if (valid < kHalfN) {
          const int st = tg % kVStages;
          if constexpr (kVStages < kSlots) {
            // The softmax runs up to kSlots tiles ahead of P·V, further than
            // the V ring is deep: until the stage's previous tile (tg -
            // kVStages) has been consumed, its v_full phase is still open and
            // a parity wait for this tile's phase would return at once (the
            // phase before has the same parity). Wait for that P·V first.
            if (tg >= uint32_t(kVStages) &&
                !wait_warp(&s_free[(tg - kVStages) % kSlots], ((tg - kVStages) / kSlots) & 1u,
                           flags, aborted))
              break;
          }
          if (!wait_warp(&v_full[st], (tg / kVStages) & 1u, flags, aborted)) break;
          uint8_t* vb = smem + C::kOffV + st * C::kKVTile;
          const int r0 = max(valid, 0);
          const int nch = (kHalfN - r0) * 8;  // 16-byte chunks per 64-dim box
          for (int i = r; i < C::kBoxes * nch; i += 128) {
            const int box = i / nch, rem = i % nch;
            const int row = gi * kHalfN + r0 + rem / 8, ch = rem % 8;
            *reinterpret_cast<uint4*>(vb + (row >> 3) * C::kGroupBytes + box * 1024 +
                                      (row & 7) * 128 + (ch << 4)) = make_uint4(0, 0, 0, 0);
          }
          tc::fence_proxy_async_smem();
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[slot * 2 + gi]);
      }
      if (aborted) break;
      tbase += ntiles;
      // Wait for the item's last PV (tile nt - 1) through its slot: every PV
      // before it completed before that tile's S was issued, so the slot's
      // barrier is at most one phase short of it.
      if (ntiles > 0 &&
          !wait_warp(&s_free[(nt - 1) % kSlots], ((nt - 1) / kSlots) & 1u, flags, aborted))
        break;
      // Row weight sums of both groups (same max) -> divide and store this
      // group's O dims, or write them unnormalised into the item's split
      // record with the row's (m, l).
      const int qb = unit % C::kQBufs;
      float* xsum = reinterpret_cast<float*>(smem + C::kOffQ + qb * C::kQBytes);
      xsum[gi * kTcM + r] = l;
      mbar_arrive(l_done);
      if (!wait_warp(l_done, unit & 1, flags, aborted)) break;
      tc::fence_after_sync();
      const float lsum = l + xsum[(gi ^ 1) * kTcM + r];
      const float inv = 1.f / lsum;
      // the Q buffer (and these sums) may now take the next item
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[qb]);
      const bool split = kSplits && w.part >= 0;
      const int rows_rec = min(P, w.rb0 * kRowBlock + kTcM) - w.rb0 * kRowBlock;
      float* rec = split ? a.partials + w.part : nullptr;
      T* dst = row_valid && !split
                   ? a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + w.kvh * G + p % G) *
                                 D + gi * kGD
                   : nullptr;
      if (split && row_valid && gi == 0) {
        rec[rows_rec * D + r] = m_used;
        rec[rows_rec * (D + 1) + r] = lsum;
      }
#pragma unroll
      for (int c2 = 0; c2 < kGD / 32; ++c2) {
        float o[32];
        tc::ld_32x32b_x32(o_dims + c2 * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
        tc::wait_ld();
        if (dst) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            pk.x = pack2<T>(o[8 * v + 0] * inv, o[8 * v + 1] * inv);
            pk.y = pack2<T>(o[8 * v + 2] * inv, o[8 * v + 3] * inv);
            pk.z = pack2<T>(o[8 * v + 4] * inv, o[8 * v + 5] * inv);
            pk.w = pack2<T>(o[8 * v + 6] * inv, o[8 * v + 7] * inv);
            *reinterpret_cast<uint4*>(dst + c2 * 32 + 8 * v) = pk;
          }
        } else if (split && row_valid) {
          float* row = rec + r * D + gi * kGD + c2 * 32;
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<float4*>(row + 4 * v) =
                make_float4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
        }
      }
      // O and this item's sums have been read: the next item may reuse them
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

template <typename T, int D>
int launch_t(const CUtensorMap& kmap, const CUtensorMap& vmap, const CUtensorMap& qmap,
             const AttnArgs<T>& args, int grid, cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(paged_prefill_tc_kernel<T, D>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<D>::kSmem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "paged_prefill_tc_kernel attribute");
  FE_CUDA_TRY(launch_pdl(paged_prefill_tc_kernel<T, D>, dim3(grid), dim3(kTcThreads),
                         TcCfg<D>::kSmem, stream, kmap, vmap, qmap, args));
  return FE_OK;
}

template <typename T>
int launch_dim(int dim, const CUtensorMap& kmap, const CUtensorMap& vmap, const CUtensorMap& qmap,
               const void* args, int grid, cudaStream_t stream) {
  const auto& a = *static_cast<const AttnArgs<T>*>(args);
  if (dim == kWideHeadDim) return launch_t<T, kWideHeadDim>(kmap, vmap, qmap, a, grid, stream);
  return launch_t<T, kHeadDim>(kmap, vmap, qmap, a, grid, stream);
}

}  // namespace

int prefill_tc_launch(int dtype, int dim, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const CUtensorMap& qmap, const void* args, int grid, cudaStream_t stream) {
  if (dtype == FE_DTYPE_BF16)
    return launch_dim<__nv_bfloat16>(dim, kmap, vmap, qmap, args, grid, stream);
  return launch_dim<__half>(dim, kmap, vmap, qmap, args, grid, stream);
}

}  // namespace fe
