// Paged GQA attention for sm_100a: one persistent kernel serves decode
// (one query row per sequence), speculative verify and chunked prefill.
//
// Reference behaviour: Cambridgebit/FlashEngine.cpp src/flashinfer_attention.cu:35-44
// (FlashInfer FA2 paged kernel, NHD pages, scale 1/sqrt(128), causal or no
// mask) and its arithmetic oracle src/portable_gpu_ops.cpp:39-44 (fp32
// softmax(q k^T / sqrt(d)) v with the bottom-right causal mask of :31).
//
// Design (B200):
//  * Work: the host planner (fe_attn_plan.cpp) cuts every (sequence, KV
//    head, query-row group) into key-range items of whole 16-token tiles and
//    hands each CTA a balanced list. Grid = SMs x resident CTAs.
//  * Data movement: one producer warp streams K and V tiles (16 tokens x 128
//    dims of one KV head, two 2 KiB TMA boxes each) from the paged pool into
//    an 8-stage shared-memory ring with cp.async.bulk.tensor, completion on
//    mbarriers; page ids are fetched 32 tiles at a time, one per lane.
//  * Math: four consumer warps. Query rows are packed (query row, head of
//    the GQA group) into 16-row blocks so one K/V tile serves the whole
//    group. S = Q K^T and O += P V run on mma.m16n8k16 with fp32
//    accumulation; P is split into a 16-bit high part and a 16-bit residual
//    so P V keeps ~16 significant bits (fp32-softmax accuracy). Online softmax
//    in base 2 with quad shuffles.
//      key mode  (one row block, e.g. decode): warps take alternate key tiles
//                 and merge (m, l, O) in shared memory.
//      row mode  (prefill / long verify): each warp owns a row block and
//                 walks every key tile of the item.
//  * Split-K: items of a split unit write (O, m, l) partial records; the last
//    CTA to finish (atomic ticket, no waiting) merges them and writes the
//    output, then re-arms the counter, so a replayed CUDA graph needs no reset.
//  * Every mbarrier wait is bounded (2 s of %globaltimer); on expiry the CTA
//    records FE_DEVERR_TIMEOUT, drains its own in-flight copies (bounded)
//    and returns.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "fe_attn_common.cuh"

namespace fe {

int decode_launch(int dtype, int heads, const CUtensorMap& kmap, const CUtensorMap& vmap,
                  bool per_head_tma, const void* args, int grid, cudaStream_t stream);
int prefill_tc_launch(int dtype, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const void* args, int grid, cudaStream_t stream);

namespace {

constexpr int kStages = 8;
constexpr int kStageBytes = 4 * kHalfBytes;  // K lo, K hi, V lo, V hi of one head
constexpr int kThreadsAttn = (kConsumerWarps + 1) * 32;
constexpr int kCombBytes = kConsumerWarps * kRowBlock * kCombStride * 4;
constexpr int kBarBytes = 2 * kStages * 8 + 16;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kCombBytes + kBarBytes;

struct ConsumerCtx {
  uint8_t* stages;
  uint64_t* full;
  uint64_t* empty;
  volatile int* flags;
  float* comb;
  int w, lane;
  bool causal;
};

// Wait for a tile's full barrier; false once the CTA has given up.
__device__ __forceinline__ bool acquire_tile(const ConsumerCtx& cx, uint32_t gg, bool& aborted) {
  if (aborted) return false;
  const int s = gg % kStages;
  if (cx.flags[0] || !wait_bounded(&cx.full[s], (gg / kStages) & 1u, cx.flags)) aborted = true;
  return !aborted;
}

// Row mode: warp w owns packed-row block rb0 + w (if any) and walks every key
// tile of the item. S = Q K^T with the rows on the mma M side. Each active
// warp releases a stage with one arrival; warp 0 also arrives for the
// warps that have no block, so every stage still completes with four.
template <typename T>
__device__ __forceinline__ void row_item(const AttnArgs<T>& a, const WorkItem& wi,
                                         const SeqInfo& si, const ConsumerCtx& cx, uint32_t& g,
                                         bool& aborted) {
  const int lane = cx.lane, w = cx.w;
  const int ntiles = wi.kt1 - wi.kt0;
  if (w >= wi.nrb) {
    g += ntiles;
    return;
  }
  const int r_lo = lane >> 2, cq = lane & 3, mi = lane >> 3, li = lane & 7;
  const int G = a.G;
  const int P = si.qrows * G;
  const int my_rb = wi.rb0 + w;
  const int p_lo = my_rb * kRowBlock + r_lo, p_hi = p_lo + 8;
  const uint32_t arrivals = w == 0 ? 1u + kConsumerWarps - wi.nrb : 1u;

  uint32_t qa[8][4];
  {
    const T* q_lo = nullptr;
    const T* q_hi = nullptr;
    if (p_lo < P)
      q_lo = a.q + (static_cast<int64_t>(si.q_row0 + p_lo / G) * a.hq + wi.kvh * G + p_lo % G) *
                       kHeadDim;
    if (p_hi < P)
      q_hi = a.q + (static_cast<int64_t>(si.q_row0 + p_hi / G) * a.hq + wi.kvh * G + p_hi % G) *
                       kHeadDim;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int col = kk * 16 + 2 * cq;
      qa[kk][0] = q_lo ? ldg32(q_lo + col) : 0u;
      qa[kk][1] = q_hi ? ldg32(q_hi + col) : 0u;
      qa[kk][2] = q_lo ? ldg32(q_lo + col + 8) : 0u;
      qa[kk][3] = q_hi ? ldg32(q_hi + col + 8) : 0u;
    }
  }
  const int lim_lo = (cx.causal && p_lo < P) ? si.length - si.qrows + p_lo / G + 1 : si.length;
  const int lim_hi = (cx.causal && p_hi < P) ? si.length - si.qrows + p_hi / G + 1 : si.length;
  const int lim_min = min(lim_lo, lim_hi);

  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int dn = 0; dn < 16; ++dn) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;

  for (int jt = 0; jt < ntiles; ++jt) {
    const uint32_t gg = g + jt;
    if (!acquire_tile(cx, gg, aborted)) break;
    const int s = gg % kStages;
    const uint32_t kb0 = smem_u32(cx.stages + s * kStageBytes);
    const uint32_t kb1 = kb0 + kHalfBytes, vb0 = kb0 + 2 * kHalfBytes, vb1 = kb0 + 3 * kHalfBytes;
    const int tbase = (wi.kt0 + jt) * kTileTokens;

    // ---- S = Q K^T (16 packed rows x 16 tokens)
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int sp = 0; sp < 2; ++sp) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int tok = nt * 8 + li;
          const int c = sp * 4 + mi;
          const uint32_t addr = (h ? kb1 : kb0) + tok * 128 + ((c ^ li) << 4);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(addr, b0, b1, b2, b3);
          const int kk = h * 4 + sp * 2;
          mma_16816<T>(sc[nt], qa[kk], b0, b1);
          mma_16816<T>(sc[nt], qa[kk + 1], b2, b3);
        }
      }
    }
    if (tbase + kTileTokens > lim_min) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = tbase + nt * 8 + 2 * cq + e;
          if (t >= lim_lo) sc[nt][e] = -INFINITY;
          if (t >= lim_hi) sc[nt][2 + e] = -INFINITY;
        }
    }
    float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m_r[0], mx0 * a.scale_log2);
    const float mn1 = fmaxf(m_r[1], mx1 * a.scale_log2);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = fast_exp2(m_r[0] - base0), al1 = fast_exp2(m_r[1] - base1);
    m_r[0] = mn0;
    m_r[1] = mn1;
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      p[nt][0] = fast_exp2(fmaf(sc[nt][0], a.scale_log2, -base0));
      p[nt][1] = fast_exp2(fmaf(sc[nt][1], a.scale_log2, -base0));
      p[nt][2] = fast_exp2(fmaf(sc[nt][2], a.scale_log2, -base1));
      p[nt][3] = fast_exp2(fmaf(sc[nt][3], a.scale_log2, -base1));
    }
    l_r[0] = l_r[0] * al0 + (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
    l_r[1] = l_r[1] * al1 + (p[0][2] + p[0][3]) + (p[1][2] + p[1][3]);
#pragma unroll
    for (int dn = 0; dn < 16; ++dn) {
      o[dn][0] *= al0;
      o[dn][1] *= al0;
      o[dn][2] *= al1;
      o[dn][3] *= al1;
    }
    uint32_t phi[4], plo[4];
    {
      const float pv[4][2] = {{p[0][0], p[0][1]}, {p[0][2], p[0][3]},
                              {p[1][0], p[1][1]}, {p[1][2], p[1][3]}};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        phi[r] = pack2<T>(pv[r][0], pv[r][1]);
        const float2 f = unpack2<T>(phi[r]);
        plo[r] = pack2<T>(pv[r][0] - f.x, pv[r][1] - f.y);
      }
    }
    uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
    if (tbase + kTileTokens > si.length) {
      const int ta = tbase + 2 * cq;
      vm0 = (ta < si.length ? 0x0000ffffu : 0u) | (ta + 1 < si.length ? 0xffff0000u : 0u);
      vm1 = (ta + 8 < si.length ? 0x0000ffffu : 0u) | (ta + 9 < si.length ? 0xffff0000u : 0u);
    }
#pragma unroll
    for (int qd = 0; qd < 8; ++qd) {
      const int tok = (mi & 1) * 8 + li;
      const int c = 2 * qd + (mi >> 1);
      const uint32_t addr = ((c >> 3) ? vb1 : vb0) + tok * 128 + (((c & 7) ^ li) << 4);
      uint32_t r0, r1, r2, r3;
      ldmatrix_x4_trans(addr, r0, r1, r2, r3);
      r0 &= vm0;
      r1 &= vm1;
      r2 &= vm0;
      r3 &= vm1;
      mma_16816<T>(o[2 * qd], phi, r0, r1);
      mma_16816<T>(o[2 * qd], plo, r0, r1);
      mma_16816<T>(o[2 * qd + 1], phi, r2, r3);
      mma_16816<T>(o[2 * qd + 1], plo, r2, r3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_cnt(&cx.empty[s], arrivals);
  }
  g += ntiles;

  l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 1);
  l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 2);
  l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 1);
  l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 2);
  float* cw = cx.comb + w * kRowBlock * kCombStride;
#pragma unroll
  for (int dn = 0; dn < 16; ++dn) {
    *reinterpret_cast<float2*>(cw + r_lo * kCombStride + dn * 8 + 2 * cq) =
        make_float2(o[dn][0], o[dn][1]);
    *reinterpret_cast<float2*>(cw + (r_lo + 8) * kCombStride + dn * 8 + 2 * cq) =
        make_float2(o[dn][2], o[dn][3]);
  }
  if (cq == 0) {
    cw[r_lo * kCombStride + kHeadDim] = m_r[0];
    cw[r_lo * kCombStride + kHeadDim + 1] = l_r[0];
    cw[(r_lo + 8) * kCombStride + kHeadDim] = m_r[1];
    cw[(r_lo + 8) * kCombStride + kHeadDim + 1] = l_r[1];
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreadsAttn, 2)
    paged_attn_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const AttnArgs<T> a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* comb = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kCombBytes);
  uint64_t* empty = full + kStages;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MetaHeader* hdr = reinterpret_cast<const MetaHeader*>(a.meta);
  const int view = a.view;
  if (static_cast<int>(blockIdx.x) >= hdr->grid[view]) return;
  const int32_t* cta_off = reinterpret_cast<const int32_t*>(a.meta + hdr->cta_off_off[view]);
  const WorkItem* items = reinterpret_cast<const WorkItem*>(a.meta + hdr->items_off[view]);
  const SplitGroup* groups = reinterpret_cast<const SplitGroup*>(a.meta + hdr->groups_off[view]);
  const SeqInfo* seqs = reinterpret_cast<const SeqInfo*>(a.meta + hdr->seqs_off);
  const int32_t* pages = reinterpret_cast<const int32_t*>(a.meta + hdr->pages_off);
  const int it0 = cta_off[blockIdx.x], it1 = cta_off[blockIdx.x + 1];
  if (it0 >= it1) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
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
      const int h2 = w.kvh * 2;
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
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          int good = 1;
          if (lane == 0) {
            if (flags[0] || !wait_bounded(&empty[s], ph ^ 1u, flags)) {
              good = 0;
            } else {
              mbar_arrive_expect_tx(&full[s], kStageBytes);
              uint8_t* st = stages + s * kStageBytes;
              tma_load_3d(st, &kmap, &full[s], 0, h2, s0);
              tma_load_3d(st + kHalfBytes, &kmap, &full[s], 0, h2 + 1, s0);
              tma_load_3d(st + 2 * kHalfBytes, &vmap, &full[s], 0, h2, s0);
              tma_load_3d(st + 3 * kHalfBytes, &vmap, &full[s], 0, h2 + 1, s0);
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
      // Drain: wait (bounded) for the copies this CTA issued into its own
      // shared memory before the CTA exits.
      const uint32_t pending = g < kStages ? g : kStages;
      for (uint32_t k = 1; k <= pending; ++k) {
        const uint32_t gg = g - k;
        volatile int never = 0;
        (void)wait_bounded(&full[gg % kStages], (gg / kStages) & 1u, &never);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int tid = threadIdx.x;  // 0..127
  const int G = a.G;
  ConsumerCtx cx{stages, full, empty, flags, comb, warp, lane, view == 1};
  uint32_t g = 0;
  bool aborted = false;

  for (int it = it0; it < it1; ++it) {
    const WorkItem wi = items[it];
    const SeqInfo si = seqs[wi.seq];
    const int P = si.qrows * G;
    row_item<T>(a, wi, si, cx, g, aborted);
    named_barrier_sync(1, kConsumerWarps * 32);

    const int nrows = min(wi.nrb * kRowBlock, P - wi.rb0 * kRowBlock);
    const int d4 = (tid & 31) * 4;
    for (int r = tid >> 5; r < nrows; r += kConsumerWarps) {
      const float* row = comb + r * kCombStride;  // warp r/16, row r%16: contiguous
      const float M = row[kHeadDim], L = row[kHeadDim + 1];
      const float4 acc = *reinterpret_cast<const float4*>(row + d4);
      const int pr = wi.rb0 * kRowBlock + r;
      if (wi.group < 0) {
        const float inv = 1.f / L;
        T* dst = a.out + (static_cast<int64_t>(si.q_row0 + pr / G) * a.hq + wi.kvh * G + pr % G) *
                             kHeadDim + d4;
        store4<T>(dst, acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      } else {
        float* rec = a.partials + wi.part;
        *reinterpret_cast<float4*>(rec + r * kHeadDim + d4) = acc;
        if ((tid & 31) == 0) {
          rec[nrows * kHeadDim + r] = M;
          rec[nrows * (kHeadDim + 1) + r] = L;
        }
      }
    }

    if (wi.group >= 0) {
      __threadfence();
      named_barrier_sync(1, kConsumerWarps * 32);
      if (tid == 0) {
        const int nsplit = groups[wi.group].nsplit;
        const int prev = atomicAdd(a.counters + wi.group, 1);
        flags[1] = prev == nsplit - 1 ? 1 : 0;
      }
      named_barrier_sync(1, kConsumerWarps * 32);
      if (flags[1]) {
        __threadfence();
        const SplitGroup gi = groups[wi.group];
        merge_partials<T>(a.partials, gi, tid, kConsumerWarps * 32, [&](int r) {
          const int pr = wi.rb0 * kRowBlock + r;
          return a.out +
                 (static_cast<int64_t>(si.q_row0 + pr / G) * a.hq + wi.kvh * G + pr % G) * kHeadDim;
        });
        if (tid == 0) a.counters[wi.group] = 0;
      }
    }
    named_barrier_sync(1, kConsumerWarps * 32);
  }
  if (aborted && lane == 0) raise_device_error(a.err, FE_DEVERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_nd(CUtensorMap* map, const void* pool, int dtype, int rank, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return fail(FE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map,
                  dtype == FE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  rank, const_cast<void*>(pool), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FE_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return FE_OK;
}

int encode_3d(CUtensorMap* map, const void* pool, int dtype, const cuuint64_t dims[3],
              const cuuint64_t strides[2], const cuuint32_t box[3]) {
  return encode_nd(map, pool, dtype, 3, dims, strides, box);
}

// tcgen05 row kernel: pool viewed as [cache_slots/8][hkv*2][8][64] (slot
// groups of 8, head-halves, slots within the group, 64 elements); box =
// 2 groups x 2 head-halves x 8 slots x 64 elements, so one TMA copies both
// halves of a 16-token piece of one KV head and lays it out as
// [group][half][8 rows of 128 B]: 1 KiB swizzle atoms, 8-key groups 2 KiB
// apart, the two head-halves 1 KiB apart.
int encode_tc_map(CUtensorMap* map, const void* pool, int dtype, int hkv, int64_t cache_slots) {
  const cuuint64_t dims[4] = {64, 8, cuuint64_t(hkv) * 2, cuuint64_t(cache_slots / 8)};
  const cuuint64_t strides[3] = {cuuint64_t(hkv) * 256, 128, cuuint64_t(hkv) * 256 * 8};
  const cuuint32_t box[4] = {64, 8, 2, 2};
  return encode_nd(map, pool, dtype, 4, dims, strides, box);
}

// Row kernel: pool viewed as [cache_slots][hkv*2][64] (64-element head-half
// rows of 128 B); box = 16 slots x 1 head-half x 64 elements.
int encode_pool_map(CUtensorMap* map, const void* pool, int dtype, int hkv, int64_t cache_slots) {
  const cuuint64_t dims[3] = {64, cuuint64_t(hkv) * 2, cuuint64_t(cache_slots)};
  const cuuint64_t strides[2] = {128, cuuint64_t(hkv) * 256};
  const cuuint32_t box[3] = {64, 1, kTileTokens};
  return encode_3d(map, pool, dtype, dims, strides, box);
}

// Decode kernel: the same memory walked slots-first, [hkv*2][cache_slots][64];
// box = 2H head-halves x 16 slots x 64 elements, so one TMA copies a 16-token
// tile of H heads (a contiguous 16 x H x 256 B block of the page) and lays it
// out head-half by head-half, 16 swizzled rows each.
int encode_decode_map(CUtensorMap* map, const void* pool, int dtype, int hkv, int heads,
                      int64_t cache_slots) {
  const cuuint64_t dims[3] = {64, cuuint64_t(cache_slots), cuuint64_t(hkv) * 2};
  const cuuint64_t strides[2] = {cuuint64_t(hkv) * 256, 128};
  const cuuint32_t box[3] = {64, kTileTokens, cuuint32_t(2 * heads)};
  return encode_3d(map, pool, dtype, dims, strides, box);
}

template <typename T>
int kernel_setup(int* ctas_per_sm) {
  static int cached = -1;
  static cudaError_t err = cudaSuccess;
  static std::once_flag once;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(paged_attn_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kSmemBytes);
    if (err == cudaSuccess) {
      int n = 0;
      err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, paged_attn_kernel<T>, kThreadsAttn,
                                                          kSmemBytes);
      cached = n;
    }
  });
  if (err != cudaSuccess) return cuda_fail(err, "paged_attn_kernel setup");
  *ctas_per_sm = cached > 0 ? cached : 1;
  return FE_OK;
}

}  // namespace
}  // namespace fe

using namespace fe;

struct fe_attn_plan {
  PlanConfig cfg{};
  int dtype = 0;
  bool host_only = false;
  int device = -1;
  // device workspaces
  uint8_t* d_meta = nullptr;
  size_t meta_cap = 0;
  float* d_partials = nullptr;
  int32_t* d_counters = nullptr;
  // pinned staging, double-buffered
  uint8_t* h_meta[2] = {nullptr, nullptr};
  cudaEvent_t h_ev[2] = {nullptr, nullptr};
  bool h_used[2] = {false, false};
  int h_idx = 0;
  // last prepare
  bool prepared = false, fixed_grid = false;
  bool graph_shape_set = false;
  int graph_batch = 0, graph_rows = 0;
  PlanResult last;
  int grid_view[3] = {0, 0, 0};
  // cached tensor maps (row kernel, decode kernel)
  CUtensorMap kmap, vmap, kmap_dec, vmap_dec, kmap_tc, vmap_tc;
  const void* kmap_ptr = nullptr;
  const void* vmap_ptr = nullptr;
  bool per_head_tma = false;  // decode falls back to per-head-half boxes
  bool row_tc = true;         // row-mode work on the tcgen05 kernel
};

namespace {

size_t meta_capacity(const PlanConfig& c) {
  size_t per_view = sizeof(int32_t) * (std::max(c.grid_cap, c.dec_grid_cap) + 1) +
                    sizeof(WorkItem) * c.max_items + sizeof(SplitGroup) * c.max_groups + 64;
  return sizeof(MetaHeader) + 3 * per_view + sizeof(SeqInfo) * c.max_batch +
         sizeof(int32_t) * size_t(c.max_batch) * c.max_pages + 256;
}

int check_shape(int hq, int hkv, int dim, int page, int max_batch, int max_pages, int dtype,
                int num_blocks) {
  if (dtype != FE_DTYPE_F16 && dtype != FE_DTYPE_BF16)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: bad dtype");
  if (dim != kHeadDim)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: head_dim must be 128");
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0 || hq / hkv > kRowBlock)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: need hq % hkv == 0 and hq/hkv <= 16");
  if (hkv * 2 > 256 * 1024)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: hkv too large");
  if (page <= 0 || page % kTileTokens != 0)
    return fail(FE_ERR_UNSUPPORTED, "fe_attn_plan_create: page must be a multiple of 16");
  if (max_batch <= 0 || max_pages <= 0 || num_blocks <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: sizes must be positive");
  if (int64_t(num_blocks + 1) * page >= INT32_MAX)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: (num_blocks+1)*page overflows");
  if (int64_t(max_batch) * max_pages >= INT32_MAX / 4)
    return fail(FE_ERR_CAPACITY, "fe_attn_plan_create: max_batch*max_pages too large");
  return FE_OK;
}

int gcd8(int hkv) {
  int h = 8;
  while (hkv % h) h >>= 1;
  return h;
}

// Row-mode engine: tcgen05 (default) or the mma.sync kernel (FE_ROW_ENGINE=mma).
bool row_engine_tc() {
  const char* e = getenv("FE_ROW_ENGINE");
  return !(e && std::string(e) == "mma");
}

PlanConfig make_config(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                       int num_blocks, int grid_cap, int dec_grid_cap) {
  PlanConfig c{};
  c.hq = hq;
  c.hkv = hkv;
  c.dim = dim;
  c.page = page;
  c.max_batch = max_batch;
  c.max_pages = max_pages;
  c.num_blocks = num_blocks;
  c.grid_cap = grid_cap;
  c.dec_grid_cap = dec_grid_cap;
  c.dec_heads = gcd8(hkv);
  c.row_group_blocks = row_engine_tc() ? 8 : kConsumerWarps;
  c.row_split = !row_engine_tc();
  int64_t items = int64_t(max_batch) * hkv * 64;
  if (items < 8192) items = 8192;
  if (items > (1 << 20)) items = 1 << 20;
  c.max_items = static_cast<int>(items);
  c.max_groups = c.max_items;
  c.partial_capacity = int64_t(16) << 20;  // 64 MiB of floats
  return c;
}

void destroy(fe_attn_plan* p) {
  if (!p) return;
  if (!p->host_only) {
    for (int i = 0; i < 2; ++i) {
      if (p->h_ev[i]) cudaEventSynchronize(p->h_ev[i]);
      if (p->h_ev[i]) cudaEventDestroy(p->h_ev[i]);
      if (p->h_meta[i]) cudaFreeHost(p->h_meta[i]);
    }
    if (p->d_meta) cudaFree(p->d_meta);
    if (p->d_partials) cudaFree(p->d_partials);
    if (p->d_counters) cudaFree(p->d_counters);
  }
  delete p;
}

}  // namespace

extern "C" {

int fe_attn_plan_create(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                        int dtype, int num_blocks, fe_attn_plan** plan_out) {
  if (!plan_out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: plan_out is null");
  *plan_out = nullptr;
  int rc = check_shape(hq, hkv, dim, page, max_batch, max_pages, dtype, num_blocks);
  if (rc != FE_OK) return rc;
  int dev = 0;
  FE_CUDA_TRY(cudaGetDevice(&dev));
  int major = 0, sms = 0;
  FE_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  FE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  if (major != 10)
    return fail(FE_ERR_NO_DEVICE, "fe_attn_plan_create: needs an sm_100 (B200) device");
  int per_sm = 1;
  rc = dtype == FE_DTYPE_BF16 ? kernel_setup<__nv_bfloat16>(&per_sm) : kernel_setup<__half>(&per_sm);
  if (rc != FE_OK) return rc;
  auto* p = new (std::nothrow) fe_attn_plan();
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_create: out of host memory");
  p->row_tc = row_engine_tc();
  p->cfg = make_config(hq, hkv, dim, page, max_batch, max_pages, num_blocks,
                       p->row_tc ? sms : sms * per_sm, sms);
  p->dtype = dtype;
  p->device = dev;
  p->meta_cap = meta_capacity(p->cfg);
  cudaError_t e = cudaMalloc(&p->d_meta, p->meta_cap);
  if (e == cudaSuccess) e = cudaMalloc(&p->d_partials, sizeof(float) * p->cfg.partial_capacity);
  if (e == cudaSuccess) e = cudaMalloc(&p->d_counters, sizeof(int32_t) * p->cfg.max_groups);
  if (e == cudaSuccess) e = cudaMemset(p->d_counters, 0, sizeof(int32_t) * p->cfg.max_groups);
  if (e == cudaSuccess) e = cudaMemset(p->d_meta, 0, sizeof(MetaHeader));
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    e = cudaMallocHost(&p->h_meta[i], p->meta_cap);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->h_ev[i], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    destroy(p);
    return cuda_fail(e, "fe_attn_plan_create: workspace allocation");
  }
  *plan_out = p;
  return FE_OK;
}

// Test hook: a plan with no device state, for exercising the planner on a
// host without a GPU. fe_attn_plan_prepare() then only builds the work list.
int fe_attn_plan_create_host(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                             int dtype, int num_blocks, int grid_cap, fe_attn_plan** plan_out) {
  if (!plan_out) return fail(FE_ERR_INVALID_ARGUMENT, "plan_out is null");
  *plan_out = nullptr;
  int rc = check_shape(hq, hkv, dim, page, max_batch, max_pages, dtype, num_blocks);
  if (rc != FE_OK) return rc;
  if (grid_cap <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "grid_cap must be positive");
  auto* p = new (std::nothrow) fe_attn_plan();
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "out of host memory");
  p->cfg = make_config(hq, hkv, dim, page, max_batch, max_pages, num_blocks, grid_cap,
                       std::max(1, grid_cap / 2));
  p->dtype = dtype;
  p->host_only = true;
  p->meta_cap = meta_capacity(p->cfg);
  *plan_out = p;
  return FE_OK;
}

int fe_attn_plan_destroy(fe_attn_plan* plan) {
  destroy(plan);
  return FE_OK;
}

int fe_attn_plan_prepare(fe_attn_plan* p, const int32_t* qo, const int32_t* kv,
                         const int32_t* pages, const int32_t* last, int batch, int rows, int graph,
                         void* stream) {
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_prepare: plan is null");
  if (graph && p->graph_shape_set && (p->graph_batch != batch || p->graph_rows != rows))
    return fail(FE_ERR_INVALID_ARGUMENT,
                "fe_attn_plan_prepare: graph plan batch/rows changed since capture");
  std::string err;
  PlanResult res;
  int rc = build_plan(p->cfg, qo, kv, pages, last, batch, rows, graph != 0, res, err);
  if (rc != FE_OK) return fail(rc, "fe_attn_plan_prepare: " + err);
  if (res.meta.size() > p->meta_cap)
    return fail(FE_ERR_CAPACITY, "fe_attn_plan_prepare: metadata exceeds workspace");
  if (!p->host_only) {
    auto s = static_cast<cudaStream_t>(stream);
    const int i = p->h_idx;
    if (p->h_used[i]) FE_CUDA_TRY(cudaEventSynchronize(p->h_ev[i]));
    std::memcpy(p->h_meta[i], res.meta.data(), res.meta.size());
    FE_CUDA_TRY(cudaMemcpyAsync(p->d_meta, p->h_meta[i], res.meta.size(), cudaMemcpyHostToDevice, s));
    FE_CUDA_TRY(cudaEventRecord(p->h_ev[i], s));
    p->h_used[i] = true;
    p->h_idx ^= 1;
    if (res.n_groups > 0)
      FE_CUDA_TRY(cudaMemsetAsync(p->d_counters, 0, sizeof(int32_t) * res.n_groups, s));
  }
  for (int c = 0; c < 3; ++c) p->grid_view[c] = res.grid[c];
  p->last = std::move(res);
  p->prepared = true;
  p->fixed_grid = graph != 0;
  if (graph) {
    p->graph_shape_set = true;
    p->graph_batch = batch;
    p->graph_rows = rows;
  }
  return FE_OK;
}

int fe_attn_run(fe_attn_plan* p, const void* q, const void* k_pool, const void* v_pool, void* out,
                int causal, void* stream) {
  if (!p) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: plan is null");
  if (p->host_only) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: host-only plan");
  if (!p->prepared) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: plan not prepared");
  const int view = causal ? 1 : 0;
  // A plan prepared for graph capture launches both kernels at full width
  // every time (CTAs without work exit at once), so the captured launches
  // stay valid for any later metadata.
  const int grid_rows = p->fixed_grid ? p->cfg.grid_cap : p->grid_view[view];
  const int grid_dec = p->fixed_grid ? p->cfg.dec_grid_cap : p->grid_view[2];
  if (grid_rows == 0 && grid_dec == 0) return FE_OK;
  if (!q || !k_pool || !v_pool || !out)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: null pointer");
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_run: buffers must be 16-byte aligned");
  const int64_t cache_slots = int64_t(p->cfg.num_blocks + 1) * p->cfg.page;
  const int H = p->cfg.dec_heads;
  if (k_pool != p->kmap_ptr) {
    int rc = encode_pool_map(&p->kmap, k_pool, p->dtype, p->cfg.hkv, cache_slots);
    if (rc != FE_OK) return rc;
    if (encode_decode_map(&p->kmap_dec, k_pool, p->dtype, p->cfg.hkv, H, cache_slots) != FE_OK)
      p->per_head_tma = true;
    rc = encode_tc_map(&p->kmap_tc, k_pool, p->dtype, p->cfg.hkv, cache_slots);
    if (rc != FE_OK) return rc;
    p->kmap_ptr = k_pool;
  }
  if (v_pool != p->vmap_ptr) {
    int rc = encode_pool_map(&p->vmap, v_pool, p->dtype, p->cfg.hkv, cache_slots);
    if (rc != FE_OK) return rc;
    if (encode_decode_map(&p->vmap_dec, v_pool, p->dtype, p->cfg.hkv, H, cache_slots) != FE_OK)
      p->per_head_tma = true;
    rc = encode_tc_map(&p->vmap_tc, v_pool, p->dtype, p->cfg.hkv, cache_slots);
    if (rc != FE_OK) return rc;
    p->vmap_ptr = v_pool;
  }
  const float scale_log2 = 1.4426950408889634f / sqrtf(float(p->cfg.dim));
  auto s = static_cast<cudaStream_t>(stream);
  const int G = p->cfg.hq / p->cfg.hkv;
  const CUtensorMap& kd = p->per_head_tma ? p->kmap : p->kmap_dec;
  const CUtensorMap& vd = p->per_head_tma ? p->vmap : p->vmap_dec;
  if (p->dtype == FE_DTYPE_BF16) {
    AttnArgs<__nv_bfloat16> a{p->d_meta, static_cast<const __nv_bfloat16*>(q),
                              static_cast<__nv_bfloat16*>(out), p->d_partials, p->d_counters,
                              device_error_word(), p->cfg.hq, G, p->cfg.page, view, scale_log2};
    if (grid_dec > 0) {
      int rc = decode_launch(p->dtype, H, kd, vd, p->per_head_tma, &a, grid_dec, s);
      if (rc != FE_OK) return rc;
    }
    if (grid_rows > 0) {
      if (p->row_tc) {
        int rc = prefill_tc_launch(p->dtype, p->kmap_tc, p->vmap_tc, &a, grid_rows, s);
        if (rc != FE_OK) return rc;
      } else {
        paged_attn_kernel<__nv_bfloat16><<<grid_rows, kThreadsAttn, kSmemBytes, s>>>(p->kmap,
                                                                                    p->vmap, a);
      }
    }
  } else {
    AttnArgs<__half> a{p->d_meta, static_cast<const __half*>(q), static_cast<__half*>(out),
                       p->d_partials, p->d_counters, device_error_word(), p->cfg.hq, G,
                       p->cfg.page, view, scale_log2};
    if (grid_dec > 0) {
      int rc = decode_launch(p->dtype, H, kd, vd, p->per_head_tma, &a, grid_dec, s);
      if (rc != FE_OK) return rc;
    }
    if (grid_rows > 0) {
      if (p->row_tc) {
        int rc = prefill_tc_launch(p->dtype, p->kmap_tc, p->vmap_tc, &a, grid_rows, s);
        if (rc != FE_OK) return rc;
      } else {
        paged_attn_kernel<__half><<<grid_rows, kThreadsAttn, kSmemBytes, s>>>(p->kmap, p->vmap, a);
      }
    }
  }
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

int fe_attn_plan_get_info(const fe_attn_plan* p, fe_attn_plan_info* info) {
  if (!p || !info) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attn_plan_get_info: null pointer");
  std::memset(info, 0, sizeof(*info));
  if (!p->prepared) return FE_OK;
  MetaHeader h;
  std::memcpy(&h, p->last.meta.data(), sizeof(h));
  info->batch = h.batch;
  info->rows = h.rows;
  info->decode_items = p->last.decode_items;
  info->prefill_items = p->last.prefill_items;
  info->split_sequences = p->last.split_units;
  info->chunk_tiles = p->last.chunk_tiles;
  info->grid_ctas = p->fixed_grid ? p->cfg.grid_cap + p->cfg.dec_grid_cap
                                  : p->last.grid[1] + p->last.grid[2];
  info->kv_tokens = p->last.kv_tokens;
  return FE_OK;
}

// Test hook: copy the packed metadata of the last prepare into `dst`
// (returns its size in *bytes; copies at most `cap` bytes).
int fe_attn_plan_debug_meta(const fe_attn_plan* p, void* dst, int64_t cap, int64_t* bytes) {
  if (!p || !bytes) return fail(FE_ERR_INVALID_ARGUMENT, "null pointer");
  *bytes = static_cast<int64_t>(p->last.meta.size());
  if (dst && cap > 0)
    std::memcpy(dst, p->last.meta.data(),
                static_cast<size_t>(std::min<int64_t>(cap, *bytes)));
  return FE_OK;
}

}  // extern "C"
