// Neighbours of the paged-KV hot path: rotary embedding (alone and fused with
// the K/V append) and greedy speculative acceptance.
//
// Reference: Cambridgebit/FlashEngine.cpp src/cuda_kernels.cu:19-23 (rope_kernel:
// per pair (j, j + dim/2) of a head, a' = a*c - b*s and b' = b*c + a*s with
// every product and sum rounded separately in fp32, c/s read from an fp32 cache
// [positions][dim] holding cos in the first and sin in the second half, result
// rounded to the 16-bit type), :24 (store_kernel), :25 (accept_kernel) and their
// launchers :33, :34, :35. The arithmetic below keeps those roundings (IEEE
// round-to-nearest multiply / add intrinsics, no contraction into FMA), so the
// results are bit-identical to the reference kernels.
//
// B200 shape of the work: both are tiny, launch-bound ops on a decode step
// (C2: 64 rows x 48 heads x 256 B). The fused kernel reads q, k and v once and
// writes q', the pool rows of k' and v (and optionally k') in one launch, where
// the reference runs rope (read/write q and k) and then store (read k and v).
// The usual shapes run rope_vec_kernel (16-byte accesses, eight rotation
// pairs per thread); others run rope_kernel, where one thread owns two
// adjacent pairs (4-byte loads and stores).
#include "fe_common.cuh"

namespace fe {
namespace {

constexpr int kRopeThreads = 256;

template <typename T>
struct Pair2;
template <>
struct Pair2<__half> {
  using V = __half2;
  static __device__ __forceinline__ float2 to_float(V x) { return __half22float2(x); }
  static __device__ __forceinline__ V from_float(float a, float b) {
    return __halves2half2(__float2half_rn(a), __float2half_rn(b));
  }
};
template <>
struct Pair2<__nv_bfloat16> {
  using V = __nv_bfloat162;
  static __device__ __forceinline__ float2 to_float(V x) { return __bfloat1622float2(x); }
  static __device__ __forceinline__ V from_float(float a, float b) {
    return __halves2bfloat162(__float2bfloat16_rn(a), __float2bfloat16_rn(b));
  }
};

// Rotate the pairs (j, j+r) and (j+1, j+r+1) of one head in registers (r =
// half the rotary dims), given cos c and sin s of both.
template <typename T>
__device__ __forceinline__ void rotate(typename Pair2<T>::V& lo, typename Pair2<T>::V& hi,
                                       float2 c, float2 s) {
  const float2 a = Pair2<T>::to_float(lo), b = Pair2<T>::to_float(hi);
  lo = Pair2<T>::from_float(__fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, s.x)),
                            __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, s.y)));
  hi = Pair2<T>::from_float(__fadd_rn(__fmul_rn(b.x, c.x), __fmul_rn(a.x, s.x)),
                            __fadd_rn(__fmul_rn(b.y, c.y), __fmul_rn(a.y, s.y)));
}

// Thread -> (row, head, jp) with jp in [0, dim/4). k and k_out may be the
// same buffer (in-place RoPE). With rot = rotary_dim: threads jp < rot/4 own
// the rotation pairs (2jp, 2jp+1) <-> (rot/2 + 2jp, rot/2 + 2jp + 1); threads
// jp >= rot/4 own four unrotated dims starting at rot + 4(jp - rot/4) (the
// partial-rotary heads of Qwen3.5, src/hybrid_model.cpp:44). Heads [0, hq) are
// query heads, rotated in place in q. Heads [hq, hq + hkv) are key heads:
// rotated, then written to k_out (if given) and, when kc is given, to the pool
// row of the row's slot together with the value head (slot < 0: skipped, as
// the reference store does; slot >= cache_slots: skipped and flagged).
template <typename T>
__global__ void __launch_bounds__(kRopeThreads)
    rope_kernel(T* __restrict__ q, const T* k, const T* __restrict__ v, T* k_out,
                T* __restrict__ kc, T* __restrict__ vc,
                const int64_t* __restrict__ slots, const int64_t* __restrict__ pos,
                const float* __restrict__ cache, int rows, int hq, int hkv, int dim, int rot,
                int max_positions, int64_t cache_slots, unsigned int* err) {
  using V = typename Pair2<T>::V;
  pdl_trigger();
  pdl_wait();  // q, k, v come from, and the pools are read by, earlier kernels
  const int per_head = dim / 4;
  const int heads = hq + hkv;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * heads * per_head) return;
  const int jp = static_cast<int>(idx % per_head);
  const int head = static_cast<int>((idx / per_head) % heads);
  const int row = static_cast<int>(idx / (static_cast<int64_t>(per_head) * heads));
  const int64_t p = pos[row];
  if (p < 0 || p >= max_positions) {
    if (jp == 0 && head == 0) raise_device_error(err, FE_DEVERR_POS_RANGE);
    return;
  }
  const bool rotating = jp < rot / 4;
  // element offsets (in pairs of elements) of this thread's two pairs
  const int i0 = rotating ? jp : (rot + 4 * (jp - rot / 4)) / 2;
  const int i1 = rotating ? (rot / 2 + 2 * jp) / 2 : i0 + 1;
  float2 c = make_float2(0.f, 0.f), s = c;
  if (rotating) {
    const float* cs = cache + p * rot;
    c = *reinterpret_cast<const float2*>(cs + 2 * jp);
    s = *reinterpret_cast<const float2*>(cs + rot / 2 + 2 * jp);
  }
  if (head < hq) {
    if (!rotating) return;  // q's unrotated dims stay as they are
    V* base = reinterpret_cast<V*>(q + (static_cast<int64_t>(row) * hq + head) * dim);
    V lo = base[i0], hi = base[i1];
    rotate<T>(lo, hi, c, s);
    base[i0] = lo;
    base[i1] = hi;
    return;
  }
  const int h = head - hq;
  const int64_t off = (static_cast<int64_t>(row) * hkv + h) * dim;
  const V* kb = reinterpret_cast<const V*>(k + off);
  V lo = kb[i0], hi = kb[i1];
  if (rotating) rotate<T>(lo, hi, c, s);
  if (k_out && (rotating || k_out != k)) {
    V* ko = reinterpret_cast<V*>(k_out + off);
    ko[i0] = lo;
    ko[i1] = hi;
  }
  if (!kc) return;
  const int64_t slot = slots[row];
  if (slot < 0) return;
  if (slot >= cache_slots) {
    if (jp == 0 && h == 0) raise_device_error(err, FE_DEVERR_SLOT_RANGE);
    return;
  }
  const int64_t dst = (slot * hkv + h) * dim;
  V* kd = reinterpret_cast<V*>(kc + dst);
  kd[i0] = lo;
  kd[i1] = hi;
  const V* vb = reinterpret_cast<const V*>(v + off);
  V* vd = reinterpret_cast<V*>(vc + dst);
  vd[i0] = vb[i0];
  vd[i1] = vb[i1];
}

// 16-byte form of rope_kernel, for rotary_dim a multiple of 16, dim a
// multiple of 8 and 16-byte aligned buffers (every model shape the path
// serves): block (x, y) covers units of rows y, y + gridDim.y, ...; a unit is
// (head, u) with u < rot/16 owning the eight rotation pairs 8u..8u+7 <->
// r+8u..r+8u+7 (r = rot/2), two 16-byte chunks of the head, or u >= rot/16
// owning the unrotated 8-element chunk rot + 8(u - rot/16). Same roundings as
// rope_kernel (the rotate() above), so the same bits; 32-bit indexing.
template <typename T>
__global__ void __launch_bounds__(kRopeThreads)
    rope_vec_kernel(T* __restrict__ q, const T* k, const T* __restrict__ v, T* k_out,
                    T* __restrict__ kc, T* __restrict__ vc, const int64_t* __restrict__ slots,
                    const int64_t* __restrict__ pos, const float* __restrict__ cache, int rows,
                    int hq, int hkv, int dim, int rot, int max_positions, int64_t cache_slots,
                    unsigned int* err) {
  using V = typename Pair2<T>::V;
  union Chunk {
    uint4 u;
    V v[4];
  };
  pdl_trigger();
  pdl_wait();  // q, k, v come from, and the pools are read by, earlier kernels
  const int rot_units = rot / 16;
  const int per_head = rot_units + (dim - rot) / 8;
  const int heads = hq + hkv;
  const int unit = blockIdx.x * blockDim.x + threadIdx.x;
  if (unit >= heads * per_head) return;
  const int head = unit / per_head, u = unit - head * per_head;
  const bool rotating = u < rot_units;
  const int r = rot / 2;
  const int e0 = rotating ? 8 * u : rot + 8 * (u - rot_units);  // first element of the chunk
  const int e1 = e0 + r;                                        // its partner (rotating)
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    // every load that does not depend on the position first (the chunk, its
    // partner, the value chunk and the slot), then the position and its
    // cos / sin: one dependent round trip per row instead of three
    const bool is_q = head < hq;
    const bool idle = is_q && !rotating;  // q's unrotated dims stay as they are
    const int h = head - hq;
    T* qbase = q + (static_cast<int64_t>(row) * hq + head) * dim;
    const int64_t off = (static_cast<int64_t>(row) * hkv + h) * dim;
    const T* src = is_q ? qbase : k + off;
    Chunk lo, hi, vlo, vhi;
    if (!idle) lo.u = *reinterpret_cast<const uint4*>(src + e0);
    if (rotating) hi.u = *reinterpret_cast<const uint4*>(src + e1);
    int64_t slot = -1;
    if (!is_q && kc) {
      slot = slots[row];
      vlo.u = *reinterpret_cast<const uint4*>(v + off + e0);
      if (rotating) vhi.u = *reinterpret_cast<const uint4*>(v + off + e1);
    }
    const int64_t p = pos[row];
    if (p < 0 || p >= max_positions) {
      if (unit == 0) raise_device_error(err, FE_DEVERR_POS_RANGE);
      continue;
    }
    if (idle) continue;
    if (rotating) {
      const float4* cp = reinterpret_cast<const float4*>(cache + p * rot + 8 * u);
      const float4* sp = reinterpret_cast<const float4*>(cache + p * rot + r + 8 * u);
      const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
      const float2 c[4] = {make_float2(c0.x, c0.y), make_float2(c0.z, c0.w),
                           make_float2(c1.x, c1.y), make_float2(c1.z, c1.w)};
      const float2 sn[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w),
                            make_float2(s1.x, s1.y), make_float2(s1.z, s1.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) rotate<T>(lo.v[i], hi.v[i], c[i], sn[i]);
    }
    if (is_q) {
      *reinterpret_cast<uint4*>(qbase + e0) = lo.u;
      *reinterpret_cast<uint4*>(qbase + e1) = hi.u;
      continue;
    }
    if (k_out && (rotating || k_out != k)) {
      *reinterpret_cast<uint4*>(k_out + off + e0) = lo.u;
      if (rotating) *reinterpret_cast<uint4*>(k_out + off + e1) = hi.u;
    }
    if (!kc || slot < 0) continue;
    if (slot >= cache_slots) {
      if (u == 0 && h == 0) raise_device_error(err, FE_DEVERR_SLOT_RANGE);
      continue;
    }
    const int64_t dst = (slot * hkv + h) * dim;
    *reinterpret_cast<uint4*>(kc + dst + e0) = lo.u;
    *reinterpret_cast<uint4*>(vc + dst + e0) = vlo.u;
    if (rotating) {
      *reinterpret_cast<uint4*>(kc + dst + e1) = hi.u;
      *reinterpret_cast<uint4*>(vc + dst + e1) = vhi.u;
    }
  }
}

// One thread per batch row: accept drafts while they equal the verifier's
// argmax, then take the verifier's token; out row b (stride k + 2) holds the
// committed tokens and, at k + 1, their count. Other entries are untouched.
__global__ void accept_kernel(const int64_t* __restrict__ draft,
                              const int64_t* __restrict__ verify, int64_t* __restrict__ out,
                              int batch, int k) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int64_t* d = draft + static_cast<int64_t>(b) * k;
  const int64_t* ver = verify + static_cast<int64_t>(b) * (k + 1);
  int64_t* o = out + static_cast<int64_t>(b) * (k + 2);
  int m = 0;
  while (m < k && d[m] == ver[m]) {
    o[m] = d[m];
    ++m;
  }
  o[m] = ver[m];
  o[k + 1] = m + 1;
}

template <typename T>
int launch_rope(void* q, const void* k, const void* v, void* k_out, void* kc, void* vc,
                const int64_t* slots, const int64_t* pos, const float* cache, int rows, int hq,
                int hkv, int dim, int rot, int max_positions, int64_t cache_slots,
                cudaStream_t stream) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (rot % 16 == 0 && dim % 8 == 0 && a16(q) && a16(k) && a16(v) && a16(k_out) && a16(kc) &&
      a16(vc) && a16(cache)) {
    const int64_t units = static_cast<int64_t>(hq + hkv) * (rot / 16 + (dim - rot) / 8);
    if (units <= INT32_MAX / 2) {
      // one row's units over as few blocks as 256 threads allow, evenly sized
      const int nb = static_cast<int>((units + kRopeThreads - 1) / kRopeThreads);
      const int bt = static_cast<int>(((units + nb - 1) / nb + 31) / 32 * 32);
      const dim3 grid(nb, rows < 65535 ? rows : 65535);
      FE_CUDA_TRY(launch_pdl(rope_vec_kernel<T>, grid, dim3(bt), 0, stream, static_cast<T*>(q),
                             static_cast<const T*>(k), static_cast<const T*>(v),
                             static_cast<T*>(k_out), static_cast<T*>(kc), static_cast<T*>(vc),
                             slots, pos, cache, rows, hq, hkv, dim, rot, max_positions,
                             cache_slots, device_error_word()));
      return FE_OK;
    }
  }
  const int64_t threads = static_cast<int64_t>(rows) * (hq + hkv) * (dim / 4);
  const int64_t blocks = (threads + kRopeThreads - 1) / kRopeThreads;
  if (blocks > INT32_MAX) return fail(FE_ERR_CAPACITY, "rope: too many rows");
  FE_CUDA_TRY(launch_pdl(rope_kernel<T>, dim3(static_cast<int>(blocks)), dim3(kRopeThreads), 0,
                         stream, static_cast<T*>(q), static_cast<const T*>(k),
                         static_cast<const T*>(v), static_cast<T*>(k_out), static_cast<T*>(kc),
                         static_cast<T*>(vc), slots, pos, cache, rows, hq, hkv, dim, rot,
                         max_positions, cache_slots, device_error_word()));
  return FE_OK;
}

int check_rope(const char* what, const void* q, const void* k, const int64_t* pos,
               const float* cache, int rows, int hq, int hkv, int dim, int rot, int max_positions,
               int dtype) {
  if (!valid_dtype(dtype)) return fail(FE_ERR_INVALID_ARGUMENT, std::string(what) + ": bad dtype");
  if (rows < 0 || hq < 0 || hkv <= 0 || dim <= 0 || max_positions <= 0)
    return fail(FE_ERR_INVALID_ARGUMENT, std::string(what) + ": sizes out of range");
  if (dim % 4 != 0 || rot < 0 || rot > dim || rot % 4 != 0)
    return fail(FE_ERR_UNSUPPORTED,
                std::string(what) + ": dim and rotary_dim must be multiples of 4, rotary_dim <= dim");
  if (rows > 0 && (!k || !pos || !cache || (hq > 0 && !q)))
    return fail(FE_ERR_INVALID_ARGUMENT, std::string(what) + ": null pointer");
  auto a4 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; };
  auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  if ((q && !a4(q)) || (k && !a4(k)) || (cache && !a8(cache)))
    return fail(FE_ERR_INVALID_ARGUMENT,
                std::string(what) + ": q/k must be 4-byte and the cache 8-byte aligned");
  return FE_OK;
}

}  // namespace
}  // namespace fe

using namespace fe;

extern "C" {

int fe_rope(void* q, void* k, const int64_t* pos, const float* cache, int rows, int hq, int hkv,
            int dim, int rotary_dim, int max_positions, int dtype, void* stream) {
  int rc = check_rope("fe_rope", q, k, pos, cache, rows, hq, hkv, dim, rotary_dim, max_positions,
                      dtype);
  if (rc != FE_OK || rows == 0) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  if (dtype == FE_DTYPE_BF16)
    return launch_rope<__nv_bfloat16>(q, k, nullptr, k, nullptr, nullptr, nullptr, pos, cache,
                                      rows, hq, hkv, dim, rotary_dim, max_positions, 0, s);
  return launch_rope<__half>(q, k, nullptr, k, nullptr, nullptr, nullptr, pos, cache, rows, hq,
                             hkv, dim, rotary_dim, max_positions, 0, s);
}

int fe_rope_append(void* q, const void* k, const void* v, void* k_out, void* k_pool,
                   void* v_pool, const int64_t* slots, const int64_t* pos, const float* cache,
                   int rows, int hq, int hkv, int dim, int rotary_dim, int max_positions,
                   int dtype, int64_t cache_slots, void* stream) {
  int rc = check_rope("fe_rope_append", q, k, pos, cache, rows, hq, hkv, dim, rotary_dim,
                      max_positions, dtype);
  if (rc != FE_OK || rows == 0) return rc;
  if (cache_slots <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rope_append: cache_slots <= 0");
  if (!v || !k_pool || !v_pool || !slots)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_rope_append: null pointer");
  auto a4 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; };
  if (!a4(v) || !a4(k_pool) || !a4(v_pool) || (k_out && !a4(k_out)))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_rope_append: buffers must be 4-byte aligned");
  auto s = static_cast<cudaStream_t>(stream);
  if (dtype == FE_DTYPE_BF16)
    return launch_rope<__nv_bfloat16>(q, k, v, k_out, k_pool, v_pool, slots, pos, cache, rows, hq,
                                      hkv, dim, rotary_dim, max_positions, cache_slots, s);
  return launch_rope<__half>(q, k, v, k_out, k_pool, v_pool, slots, pos, cache, rows, hq, hkv,
                             dim, rotary_dim, max_positions, cache_slots, s);
}

int fe_accept(const int64_t* draft, const int64_t* verify, int64_t* out, int batch, int k,
              void* stream) {
  if (batch < 0 || k < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_accept: batch/k < 0");
  if (batch == 0) return FE_OK;
  if ((k > 0 && !draft) || !verify || !out)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_accept: null pointer");
  const int threads = 128;
  accept_kernel<<<(batch + threads - 1) / threads, threads, 0,
                  static_cast<cudaStream_t>(stream)>>>(draft, verify, out, batch, k);
  FE_CUDA_TRY(cudaGetLastError());
  return FE_OK;
}

}  // extern "C"
