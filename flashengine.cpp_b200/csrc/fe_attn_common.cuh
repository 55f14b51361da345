// Device code shared by the two paged-attention kernels (fe_decode.cu for
// one-row-block sequences, fe_attn.cu for multi-block prefill / verify):
// launch arguments, the bounded mbarrier wait, and the key-mode tile math.
//
// Shared-memory tile layout (both kernels): a key tile is 16 consecutive
// tokens of one page. For one KV head it is stored as D/64 boxes of 16 rows x
// 128 bytes (dims 0-63, 64-127, ...; "head-halves" for head_dim 128), written
// by TMA with the 128-byte swizzle: 16-byte chunk c of row r sits at chunk
// c ^ (r & 7).
#pragma once

#include "fe_attn_plan.h"
#include "fe_common.cuh"

namespace fe {

constexpr int kHalfBytes = kTileTokens * 128;  // one 64-dim box: 16 rows x 128 B
constexpr int kCombStride = kHeadDim + 4;      // merge rows: O[128], m, l, pad
constexpr uint64_t kWaitLimitNs = 2000000000ull;

template <typename T>
struct AttnArgs {
  const uint8_t* meta;
  const T* q;
  T* out;
  float* partials;
  int32_t* counters;
  unsigned int* err;
  int hq, G, page, view;
  float scale_log2;
  int q_map_rows;  // query rows the row kernel's Q tensor map covers (0: none)
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded mbarrier wait. Returns false when the phase did not complete
// within kWaitLimitNs, or when another warp of the CTA already gave up
// (abort flag), so that every warp of the CTA winds down together.
__device__ __noinline__ inline bool wait_bounded_slow(uint64_t* bar, uint32_t parity,
                                                      volatile int* abort_flag) {
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_bounded_slow(bar, parity, abort_flag);
}

// The same bound with short try_waits (no suspend hint): for pipelines whose
// hand-offs each have one or a few waiters on the critical path.
__device__ __noinline__ inline bool wait_bounded_short_slow(uint64_t* bar, uint32_t parity,
                                                            volatile int* abort_flag) {
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_short(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bounded_short(uint64_t* bar, uint32_t parity,
                                                   volatile int* abort_flag) {
  if (mbar_try_wait_short(bar, parity)) return true;
  return wait_bounded_short_slow(bar, parity, abort_flag);
}

template <typename T>
__device__ __forceinline__ void store4(T* dst, float a, float b, float c, float d) {
  uint2 v;
  v.x = pack2<T>(a, b);
  v.y = pack2<T>(c, d);
  *reinterpret_cast<uint2*>(dst) = v;
}

__device__ __forceinline__ uint32_t ldg32(const void* p) {
  return __ldg(reinterpret_cast<const uint32_t*>(p));
}

// Shared-memory addresses of one KV head's slice of a staged tile: the
// head's 64-dim boxes of K (and of V) follow one another, kHalfBytes apart.
struct TileAddr {
  uint32_t k, v;
};

// ---------------------------------------------------------------------------
// Key mode: one row block of P <= 16 packed rows (packed row p = query row
// p / G, head p % G of the GQA group) against a KV head of D dims. The key
// tile sits on the mma M side: S^T = K Q^T (16 tokens x 8*NT columns), so a
// GQA group of 8 fills the N dimension; O^T = V^T P^T accumulates D dims x
// 8*NT columns. The state covers packed rows col0 .. col0 + 8*NT - 1.
// P^T is split into a 16-bit high part and its residual (two mma), keeping
// ~16 significant bits of the fp32 softmax weights.
// ---------------------------------------------------------------------------
template <typename T, int NT, int D = kHeadDim>
struct KeyState {
  static constexpr int kMT = D / 16;  // k-steps of S^T, m-tiles of O^T
  uint32_t qb[NT][kMT][2];  // Q^T as B fragments: column lane/4 (+8 nt)
  int lim[NT][2];           // visible-key limit of this lane's columns
  int lim_min;
  float m[NT][2], l[NT][2];
  float o[NT][kMT][4];

  __device__ __forceinline__ void init(const T* q, int hq, int q_row0, int qrows, int length,
                                       int head0, int G, bool causal, int lane, int col0 = 0) {
    const int r8 = lane >> 2, cq = lane & 3;
    const int P = qrows * G;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int p = col0 + nt * 8 + r8;
      const T* qp = p < P ? q + (static_cast<int64_t>(q_row0 + p / G) * hq + head0 + p % G) * D
                          : nullptr;
#pragma unroll
      for (int kk = 0; kk < kMT; ++kk) {
        qb[nt][kk][0] = qp ? ldg32(qp + kk * 16 + 2 * cq) : 0u;
        qb[nt][kk][1] = qp ? ldg32(qp + kk * 16 + 8 + 2 * cq) : 0u;
      }
    }
    lim_min = length;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int p = col0 + nt * 8 + 2 * cq + e;
        lim[nt][e] = (causal && p < P) ? length - qrows + p / G + 1 : length;
        lim_min = min(lim_min, lim[nt][e]);
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)
        o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    }
  }

  // One 16-token tile starting at token `tbase` of a sequence of `length` keys.
  __device__ __forceinline__ void tile(const TileAddr& t, int tbase, int length, float scale_log2,
                                       int lane) {
    const int r8 = lane >> 2, cq = lane & 3, mi = lane >> 3, li = lane & 7;
    // ---- S^T = K Q^T
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kMT; ++kk) {
      const int tok = li + ((mi & 1) << 3);
      const int c = 2 * kk + (mi >> 1);  // 16-byte chunk of the row (8 per 64-dim box)
      const uint32_t addr = t.k + (c >> 3) * kHalfBytes + tok * 128 + (((c & 7) ^ li) << 4);
      uint32_t af[4];
      ldmatrix_x4(addr, af[0], af[1], af[2], af[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816<T>(sc[nt], af, qb[nt][kk][0], qb[nt][kk][1]);
    }
    // ---- mask keys past each column's limit (causal) or the sequence end
    if (tbase + kTileTokens > lim_min) {
      const int t0 = tbase + r8, t1 = t0 + 8;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (t0 >= lim[nt][e]) sc[nt][e] = -INFINITY;
          if (t1 >= lim[nt][e]) sc[nt][2 + e] = -INFINITY;
        }
    }
    // ---- online softmax per column; the 8 lanes sharing lane%4 hold a column
    float al[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float mx = fmaxf(sc[nt][e], sc[nt][2 + e]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[nt][e], mx * scale_log2);
        const float base = mn == -INFINITY ? 0.f : mn;
        al[nt][e] = fast_exp2(m[nt][e] - base);
        m[nt][e] = mn;
        const float p0 = fast_exp2(fmaf(sc[nt][e], scale_log2, -base));
        const float p1 = fast_exp2(fmaf(sc[nt][2 + e], scale_log2, -base));
        sc[nt][e] = p0;
        sc[nt][2 + e] = p1;
        l[nt][e] = fmaf(l[nt][e], al[nt][e], p0 + p1);
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt) {
        o[nt][mt][0] *= al[nt][0];
        o[nt][mt][1] *= al[nt][1];
        o[nt][mt][2] *= al[nt][0];
        o[nt][mt][3] *= al[nt][1];
      }
    // ---- P^T as B fragments (high part + residual), transposed with movmatrix
    uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t x = pack2<T>(sc[nt][2 * h], sc[nt][2 * h + 1]);
        const float2 f = unpack2<T>(x);
        const uint32_t y = pack2<T>(sc[nt][2 * h] - f.x, sc[nt][2 * h + 1] - f.y);
        bh[nt][h] = movmatrix_trans(x);
        bl[nt][h] = movmatrix_trans(y);
      }
    // ---- V rows past the sequence end are zeroed in the fragments (the
    // pool may hold anything there; 0 * NaN would poison O)
    uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
    if (tbase + kTileTokens > length) {
      const int ta = tbase + 2 * cq;
      vm0 = (ta < length ? 0x0000ffffu : 0u) | (ta + 1 < length ? 0xffff0000u : 0u);
      vm1 = (ta + 8 < length ? 0x0000ffffu : 0u) | (ta + 9 < length ? 0xffff0000u : 0u);
    }
    // ---- O^T += V^T P^T (16 dims per m-tile)
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt) {
      const int tok = li + ((mi >> 1) << 3);
      const int c = 2 * mt + (mi & 1);
      const uint32_t addr = t.v + (c >> 3) * kHalfBytes + tok * 128 + (((c & 7) ^ li) << 4);
      uint32_t va[4];
      ldmatrix_x4_trans(addr, va[0], va[1], va[2], va[3]);
      va[0] &= vm0;
      va[1] &= vm0;
      va[2] &= vm1;
      va[3] &= vm1;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816<T>(o[nt][mt], va, bh[nt][0], bh[nt][1]);
        mma_16816<T>(o[nt][mt], va, bl[nt][0], bl[nt][1]);
      }
    }
  }

  // Sum each column's l over the 8 lanes that share it.
  __device__ __forceinline__ void reduce_l() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], 4);
        l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], 8);
        l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], 16);
      }
  }

  // Stash (O, m, l) of every column into merge rows `rows` (D + 4 floats
  // apart; row = column index).
  __device__ __forceinline__ void stash(float* rows, int lane) const {
    const int r8 = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float* row = rows + (nt * 8 + 2 * cq + e) * (D + 4);
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt) {
          row[16 * mt + r8] = o[nt][mt][e];
          row[16 * mt + r8 + 8] = o[nt][mt][2 + e];
        }
        if (r8 == 0) {
          row[D] = m[nt][e];
          row[D + 1] = l[nt][e];
        }
      }
  }

  // Fold a state stashed by another warp over a disjoint key range (same
  // columns, same lane layout) into this one: O, m and l of the union.
  __device__ __forceinline__ void absorb(const float* rows, int lane) {
    const int r8 = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float* row = rows + (nt * 8 + 2 * cq + e) * (D + 4);
        const float mo = row[D], lo = row[D + 1];
        const float mn = fmaxf(m[nt][e], mo);
        const float base = mn == -INFINITY ? 0.f : mn;
        const float as = fast_exp2(m[nt][e] - base), ao = fast_exp2(mo - base);
        m[nt][e] = mn;
        l[nt][e] = l[nt][e] * as + lo * ao;
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt) {
          o[nt][mt][e] = o[nt][mt][e] * as + row[16 * mt + r8] * ao;
          o[nt][mt][2 + e] = o[nt][mt][2 + e] * as + row[16 * mt + r8 + 8] * ao;
        }
      }
  }
};

// Merge `nsplit` partial records (O unnormalised, m, l for `rows` rows) of a
// split unit into the final 16-bit output. `out_row(r)` gives the output
// pointer of merged row r. Threads `tid` of `nthreads` share the rows.
template <typename T, typename OutRow>
__device__ __forceinline__ void merge_partials(const float* partials, const SplitGroup& gi, int tid,
                                               int nthreads, OutRow out_row) {
  const int d4 = (tid & 31) * 4;
  for (int r = tid >> 5; r < gi.rows; r += nthreads >> 5) {
    float M = -INFINITY;
    for (int sidx = 0; sidx < gi.nsplit; ++sidx) {
      const float* rec = partials + gi.part0 + sidx * gi.rec_floats;
      M = fmaxf(M, __ldcg(rec + gi.rows * kHeadDim + r));
    }
    const float base = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sidx = 0; sidx < gi.nsplit; ++sidx) {
      const float* rec = partials + gi.part0 + sidx * gi.rec_floats;
      const float sc = fast_exp2(__ldcg(rec + gi.rows * kHeadDim + r) - base);
      L = fmaf(__ldcg(rec + gi.rows * (kHeadDim + 1) + r), sc, L);
      const float4 x = __ldcg(reinterpret_cast<const float4*>(rec + r * kHeadDim + d4));
      acc.x = fmaf(x.x, sc, acc.x);
      acc.y = fmaf(x.y, sc, acc.y);
      acc.z = fmaf(x.z, sc, acc.z);
      acc.w = fmaf(x.w, sc, acc.w);
    }
    const float inv = 1.f / L;
    store4<T>(out_row(r) + d4, acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
}

}  // namespace fe
