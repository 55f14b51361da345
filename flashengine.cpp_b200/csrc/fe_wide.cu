// Paged attention for head_dim 256: the full-attention layers of Qwen3.5-style
// hybrid models (src/hybrid_model.cpp:41-50) and DFlash drafts of such models
// (src/block_draft.cpp:24-30), whose reference path is an ATen gather over
// max_model_len slots of a flat [slots, hkv, dim] pool with any head_dim. The
// reference's CUDA build stops at head_dim 128 (src/cuda_model.cpp:35); this
// kernel serves the same plan / attention calls when the plan is created with
// dim = 256, for decode rows, verify / draft blocks and prefill chunks alike,
// with the bottom-right causal or the full mask.
//
// Design: one CTA of 4 warps per work item = 64 packed query rows (row p =
// query row p / G, head kvh*G + p % G) of one (sequence, KV head) against the
// item's key range: all keys the mask shows the item's rows, or, when the
// planner splits an item whose rows are too few to fill the GPU, one piece of
// that range (the piece writes an unnormalised (O, m, l) record, merged by
// decode_merge_kernel). Q is staged once in shared memory; K and V tiles of 32 keys (16 KiB each) are
// gathered through the page table with 16-byte cp.async (positions past the
// key limit read as zeros) into a 2-stage ring; rows of 512 bytes are stored
// with the 16-byte chunk index XOR-swizzled by the row, so ldmatrix reads are
// conflict free. Each warp owns 16 rows: S = Q K^T and O += P V on
// mma.m16n8k16 with fp32 accumulation, an exact online softmax in base 2 (O
// rescaled every tile), and P entering the PV product as a 16-bit high part
// plus its 16-bit residual (two MMAs), which keeps ~16 bits of each fp32 weight
// like the 128-dim kernels. Each CTA walks its own item list (cta_off), laid
// out by the host planner longest first onto the least-loaded CTA.
#include "fe_attn_common.cuh"

namespace fe {

int wide_launch(int dtype, const void* args, const void* k_pool, const void* v_pool, int hkv,
                int grid, cudaStream_t stream);

namespace {

constexpr int kWD = 256;                       // head dim
constexpr int kWRows = 64;                     // packed rows per item (16 per warp)
constexpr int kWKeys = 32;                     // keys per tile
constexpr int kWThreads = 128;
constexpr int kWRowBytes = kWD * 2;            // 512 B per row of Q, K or V
constexpr int kWChunks = kWRowBytes / 16;      // 16-byte chunks per row
constexpr int kWQBytes = kWRows * kWRowBytes;  // 32 KiB
constexpr int kWTileBytes = kWKeys * kWRowBytes;  // 16 KiB
constexpr int kWSmem = kWQBytes + 2 * 2 * kWTileBytes;  // Q + 2 stages of (K, V): 96 KiB

// Byte offset of 16-byte chunk `c` of row `r` (chunk index XOR row mod 8).
__device__ __forceinline__ uint32_t wswz(int r, int c) {
  return uint32_t(r * kWRowBytes + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
__device__ __forceinline__ float2 hi_back(uint32_t h) {
  return unpack2<T>(h);
}

template <typename T>
__global__ void __launch_bounds__(kWThreads) paged_wide_kernel(const AttnArgs<T> a,
                                                               const T* __restrict__ kpool,
                                                               const T* __restrict__ vpool,
                                                               int hkv) {
  extern __shared__ __align__(128) uint8_t wsmem[];
  pdl_trigger();
  pdl_wait();
  const MetaHeader* hdr = reinterpret_cast<const MetaHeader*>(a.meta);
  const int view = a.view;
  if (static_cast<int>(blockIdx.x) >= hdr->grid[view]) return;
  const int32_t* cta_off = reinterpret_cast<const int32_t*>(a.meta + hdr->cta_off_off[view]);
  const WorkItem* items = reinterpret_cast<const WorkItem*>(a.meta + hdr->items_off[view]);
  const SeqInfo* seqs = reinterpret_cast<const SeqInfo*>(a.meta + hdr->seqs_off);
  const int32_t* pages = reinterpret_cast<const int32_t*>(a.meta + hdr->pages_off);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.G, page = a.page;
  const bool causal = view == 1;
  const uint32_t q_s = smem_u32(wsmem);
  const uint32_t kv_s = q_s + kWQBytes;  // stage s: K at kv_s + s*2*tile, V after it

  const int it_end = cta_off[blockIdx.x + 1];
  for (int it = cta_off[blockIdx.x]; it < it_end; ++it) {
    const WorkItem w = items[it];
    const SeqInfo si = seqs[w.seq];
    const int len = si.length, qrows = si.qrows, P = qrows * G;
    const int p0 = w.rb0 * kRowBlock;  // first packed row of the item
    const int p_last = min(P, p0 + kWRows) - 1;
    const int lim_block = causal ? len - qrows + p_last / G + 1 : len;
    // this item's keys: [key0, key_end), the piece of the mask's range
    const int key0 = w.kt0 * kTileTokens;
    const int key_end = min(lim_block, w.kt1 * kTileTokens);
    const int ntiles = key_end > key0 ? (key_end - key0 + kWKeys - 1) / kWKeys : 0;

    auto load_tile = [&](int j) {
      const int st = j & 1;
      const int t0 = key0 + j * kWKeys;
      const uint32_t kb = kv_s + st * 2 * kWTileBytes, vb = kb + kWTileBytes;
      for (int i = tid; i < kWKeys * kWChunks; i += kWThreads) {
        const int key = i / kWChunks, c = i % kWChunks;
        const int t = t0 + key;
        const bool ok = t < key_end;
        int64_t off = 0;
        if (ok) {
          const int64_t slot = int64_t(__ldg(pages + si.page_off + t / page)) * page + t % page;
          off = (slot * hkv + w.kvh) * kWD + c * 8;
        }
        cp_async16(kb + wswz(key, c), kpool + off, ok);
        cp_async16(vb + wswz(key, c), vpool + off, ok);
      }
    };

    // Q rows (zeros past the sequence) with the first K/V tile, then the second
    for (int i = tid; i < kWRows * kWChunks; i += kWThreads) {
      const int r = i / kWChunks, c = i % kWChunks;
      const int p = p0 + r;
      const bool ok = p < P;
      const T* src = a.q;
      if (ok)
        src = a.q + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + w.kvh * G + p % G) * kWD +
              c * 8;
      cp_async16(q_s + wswz(r, c), src, ok);
    }
    if (ntiles > 0) load_tile(0);
    cp_async_commit();
    if (ntiles > 1) load_tile(1);
    cp_async_commit();

    // this thread's two rows of the warp's 16: g and g + 8 (mma C layout)
    const int g = lane >> 2, tq = lane & 3;
    int lim[2];
    bool valid[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int p = p0 + warp * 16 + g + 8 * e;
      valid[e] = p < P;
      lim[e] = min((causal && valid[e]) ? len - qrows + p / G + 1 : len, key_end);
    }
    float o[kWD / 8][4];
#pragma unroll
    for (int d = 0; d < kWD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

    for (int j = 0; j < ntiles; ++j) {
      if (j + 1 < ntiles) cp_async_wait<1>(); else cp_async_wait<0>();
      __syncthreads();
      const uint32_t kb = kv_s + (j & 1) * 2 * kWTileBytes, vb = kb + kWTileBytes;
      // S = Q K^T for this warp's 16 rows and the tile's 32 keys
      float s[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll 4
      for (int kk = 0; kk < kWD / 16; ++kk) {
        uint32_t qa[4];
        ldmatrix_x4(q_s + wswz(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), qa[0], qa[1], qa[2],
                    qa[3]);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kb + wswz(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)),
                      b0, b1, b2, b3);
          mma_16816<T>(s[2 * np], qa, b0, b1);
          mma_16816<T>(s[2 * np + 1], qa, b2, b3);
        }
      }
      // mask, online softmax (base 2), P
      const int t0 = key0 + j * kWKeys;
      float alpha[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float mx = -INFINITY;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int key = t0 + n * 8 + 2 * tq + c;
            float x = s[n][2 * e + c] * a.scale_log2;
            if (key >= lim[e]) x = -INFINITY;
            s[n][2 * e + c] = x;
            mx = fmaxf(mx, x);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m[e], mx);
        const float base = m_new == -INFINITY ? 0.f : m_new;
        alpha[e] = m[e] == -INFINITY ? 0.f : fast_exp2(m[e] - base);
        m[e] = m_new;
        float sum = 0.f;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float p = fast_exp2(s[n][2 * e + c] - base);
            s[n][2 * e + c] = p;
            sum += p;
          }
        l[e] = l[e] * alpha[e] + sum;
      }
#pragma unroll
      for (int d = 0; d < kWD / 8; ++d) {
        o[d][0] *= alpha[0];
        o[d][1] *= alpha[0];
        o[d][2] *= alpha[1];
        o[d][3] *= alpha[1];
      }
      // O += P V, P as a 16-bit high part and its residual
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        uint32_t ph[4], pl[4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float x0 = s[2 * k2 + h][2 * e], x1 = s[2 * k2 + h][2 * e + 1];
            const uint32_t hi = pack2<T>(x0, x1);
            const float2 hb = hi_back<T>(hi);
            ph[2 * h + e] = hi;
            pl[2 * h + e] = pack2<T>(x0 - hb.x, x1 - hb.y);
          }
#pragma unroll
        for (int dp = 0; dp < kWD / 16; ++dp) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vb + wswz(k2 * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                      dp * 2 + (lane >> 4)),
                            b0, b1, b2, b3);
          mma_16816<T>(o[2 * dp], ph, b0, b1);
          mma_16816<T>(o[2 * dp + 1], ph, b2, b3);
          mma_16816<T>(o[2 * dp], pl, b0, b1);
          mma_16816<T>(o[2 * dp + 1], pl, b2, b3);
        }
      }
      __syncthreads();  // the stage is read by every warp before it is refilled
      if (j + 2 < ntiles) load_tile(j + 2);
      cp_async_commit();
    }
    cp_async_wait<0>();

    // divide by the row sums (over the quad's columns) and store, or write
    // this piece's record: O[r][256] unnormalised, then m[r], l[r] (r = row
    // within the item; rows = the item's valid rows)
    const int rows = p_last + 1 - p0;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float sum = l[e];
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (!valid[e]) continue;
      const int r = warp * 16 + g + 8 * e;
      const int p = p0 + r;
      if (w.part < 0) {
        const float inv = 1.f / sum;
        T* dst =
            a.out + (static_cast<int64_t>(si.q_row0 + p / G) * a.hq + w.kvh * G + p % G) * kWD;
#pragma unroll
        for (int d = 0; d < kWD / 8; ++d)
          *reinterpret_cast<uint32_t*>(dst + d * 8 + 2 * tq) =
              pack2<T>(o[d][2 * e] * inv, o[d][2 * e + 1] * inv);
      } else {
        float* rec = a.partials + w.part;
        float* row = rec + r * kWD;
#pragma unroll
        for (int d = 0; d < kWD / 8; ++d)
          *reinterpret_cast<float2*>(row + d * 8 + 2 * tq) = make_float2(o[d][2 * e], o[d][2 * e + 1]);
        if (tq == 0) {
          rec[rows * kWD + r] = m[e];
          rec[rows * (kWD + 1) + r] = sum;
        }
      }
    }
    __syncthreads();  // Q and the ring are reused by the next item
  }
}

template <typename T>
int launch_t(const AttnArgs<T>& args, const T* kpool, const T* vpool, int hkv, int grid,
             cudaStream_t stream) {
  static const cudaError_t attr = cudaFuncSetAttribute(
      paged_wide_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWSmem);
  FE_CUDA_TRY(attr);
  FE_CUDA_TRY(launch_pdl(paged_wide_kernel<T>, dim3(grid), dim3(kWThreads), kWSmem, stream, args,
                         kpool, vpool, hkv));
  return FE_OK;
}

}  // namespace

int wide_launch(int dtype, const void* args, const void* k_pool, const void* v_pool, int hkv,
                int grid, cudaStream_t stream) {
  if (grid <= 0) return FE_OK;
  if (dtype == FE_DTYPE_BF16)
    return launch_t(*static_cast<const AttnArgs<__nv_bfloat16>*>(args),
                    static_cast<const __nv_bfloat16*>(k_pool),
                    static_cast<const __nv_bfloat16*>(v_pool), hkv, grid, stream);
  return launch_t(*static_cast<const AttnArgs<__half>*>(args), static_cast<const __half*>(k_pool),
                  static_cast<const __half*>(v_pool), hkv, grid, stream);
}

}  // namespace fe
